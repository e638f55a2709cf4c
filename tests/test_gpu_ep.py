"""Expert parallelism on the GPU: the device steps of open_rknpu2_lm_infer_b200.ep.

One GPU plays every rank: the EP forward with one rank, and two ranks each
owning half of the experts with the all-to-all done by hand, must reproduce
the single-device layer (moe_b200_forward_device) bit for bit, and the CPU
restatement of the reference layer within 1e-2 rel / 1e-3 abs.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.ep import DeviceOps, ep_forward
from open_rknpu2_lm_infer_b200.moe import Backend

pytestmark = pytest.mark.gpu

SPEC = S.small_spec("c2", experts=32)
T = 96


class LocalDist:
    @staticmethod
    def all_to_all_single(out, inp, out_splits=None, in_splits=None, group=None):
        out.copy_(inp)


def _single(torch, layer, x, res):
    be = Backend(max_rows=T)
    moe = be.load_moe(layer.gate, layer.down, SPEC.top)
    router = be.router(layer.router, SPEC.top, layer.bias)
    out = torch.empty_like(x)
    moe.forward_device(router, T, x.data_ptr(), res.data_ptr(), out.data_ptr(),
                       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    moe.status()
    r = out.cpu().numpy()
    moe.close(); router.close(); be.close()
    return r


def _rank(world, g, layer, rows):
    P = SPEC.experts // world
    be = Backend(max_rows=world * rows)
    moe = be.load_moe(layer.gate[g * P:(g + 1) * P], layer.down[g * P:(g + 1) * P], SPEC.top)
    router = be.router(layer.router, SPEC.top, layer.bias)
    return be, moe, router, DeviceOps(be, moe, router, world, rows)


def test_ep_one_rank_matches_single_device(cuda, oracle):
    torch = cuda
    layer = S.make_layer(SPEC, seed=5)
    x = torch.from_numpy(S.make_input(SPEC, T, seed=6)).cuda()
    res = torch.from_numpy(S.make_input(SPEC, T, seed=7, stream=5)).cuda()
    ref = _single(torch, layer, x, res)
    be, moe, router, ops = _rank(1, 0, layer, T)
    out, plan = ep_forward(ops, LocalDist, None, x, res)
    torch.cuda.synchronize()
    ops.status()
    assert plan.n_send == plan.n_recv == T * SPEC.top
    assert np.array_equal(out.cpu().numpy(), ref)
    assert_close(out.cpu().numpy(), oracle.OracleLayer(layer).forward(x.cpu().numpy(), res.cpu().numpy()),
                 what="EP one rank vs restatement")
    ops.close(); moe.close(); router.close(); be.close()


def test_ep_two_ranks_by_hand_match_single_device(cuda, oracle):
    torch = cuda
    world = 2
    layer = S.make_layer(SPEC, seed=5)
    xs = [torch.from_numpy(S.make_input(SPEC, T, seed=10 + g)).cuda() for g in range(world)]
    rs = [torch.from_numpy(S.make_input(SPEC, T, seed=20 + g, stream=5)).cuda() for g in range(world)]
    refs = [_single(torch, layer, xs[g], rs[g]) for g in range(world)]
    ranks = [_rank(world, g, layer, T) for g in range(world)]
    ops = [r[3] for r in ranks]
    routed = [ops[g].route(xs[g]) for g in range(world)]
    packed = [ops[g].pack(xs[g], *routed[g]) for g in range(world)]
    counts = [p[3].cpu().numpy() for p in packed]
    assert all(c.sum() == T * SPEC.top for c in counts)
    starts = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    # the exchange by hand: rank b receives from ranks 0..G-1 in order
    ys = []
    for b in range(world):
        q = torch.cat([packed[a][0][starts[a][b]:starts[a][b + 1]] for a in range(world)])
        sc = torch.cat([packed[a][1][starts[a][b]:starts[a][b + 1]] for a in range(world)])
        ex = torch.cat([packed[a][2][starts[a][b]:starts[a][b + 1]] for a in range(world)])
        assert int(ex.max()) < SPEC.experts // world
        ys.append(ops[b].expert_rows(q.contiguous(), sc.contiguous(), ex.contiguous()).clone())
    recv = [[int(counts[a][b]) for a in range(world)] for b in range(world)]
    for a in range(world):
        parts = []
        for b in range(world):
            off = sum(recv[b][:a])
            parts.append(ys[b][off:off + recv[b][a]])
        y_back = torch.cat(parts).contiguous()
        out = ops[a].combine(y_back, packed[a][4], routed[a][1], rs[a])
        torch.cuda.synchronize()
        ops[a].status()
        assert np.array_equal(out.cpu().numpy(), refs[a]), f"rank {a} differs"
        assert_close(out.cpu().numpy(),
                     oracle.OracleLayer(layer).forward(xs[a].cpu().numpy(), rs[a].cpu().numpy()),
                     what=f"EP rank {a} vs restatement")
    for be, moe, router, op in ranks:
        op.close(); moe.close(); router.close(); be.close()


def test_ep_pack_groups_by_destination(cuda):
    torch = cuda
    world = 4
    layer = S.make_layer(SPEC, seed=5)
    x = torch.from_numpy(S.make_input(SPEC, T, seed=31)).cuda()
    be, moe, router, ops = _rank(world, 0, layer, T)
    ids, routes = ops.route(x)
    send_q, send_s, send_e, counts, pos = ops.pack(x, ids, routes)
    torch.cuda.synchronize()
    ids_n, pos_n = ids.cpu().numpy().reshape(-1), pos.cpu().numpy()
    P = SPEC.experts // world
    dest = ids_n // P
    order = np.argsort(dest, kind="stable")  # every assignment is kept (no pruning)
    assert np.array_equal(pos_n[order], np.arange(T * SPEC.top))
    assert np.array_equal(counts.cpu().numpy(), np.bincount(dest, minlength=world))
    assert np.array_equal(send_e.cpu().numpy()[:T * SPEC.top], (ids_n % P)[order])
    # each packed row is its token's A8 row (the single-device quantiser)
    q_tok = send_q.cpu().numpy()[pos_n, :SPEC.hidden].reshape(T, SPEC.top, -1)
    assert all(np.array_equal(q_tok[:, 0], q_tok[:, r]) for r in range(SPEC.top))
    ops.close(); moe.close(); router.close(); be.close()
