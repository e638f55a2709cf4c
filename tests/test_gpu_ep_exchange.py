"""The device-initiated expert-parallel exchange (moe_b200_ep_exchange_*).

One rank (one GPU): the whole path -- route, pack, peer-memory exchange (here
into the rank's own region), expert rows, return, combine -- reproduces the
single-device layer bit for bit, also when the step is captured in a CUDA
graph and replayed. Two ranks on two GPUs (skipped with fewer GPUs): each
rank owns half of the experts and its output equals the single-device layer
bit for bit. Waits across ranks are bounded; the two ranks run on two GPUs,
never as concurrent launches on one.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import synthetic as S

pytestmark = pytest.mark.gpu

SPEC = S.small_spec("c2", experts=32)
T = 64


def _single(torch, layer, x, res, device=0):
    from open_rknpu2_lm_infer_b200.moe import Backend
    be = Backend(device=device, max_rows=T)
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


def _rank_setup(world, g, layer):
    from open_rknpu2_lm_infer_b200.ep import DeviceOps
    from open_rknpu2_lm_infer_b200.moe import Backend
    P = SPEC.experts // world
    be = Backend(device=g, max_rows=world * T)
    moe = be.load_moe(layer.gate[g * P:(g + 1) * P], layer.down[g * P:(g + 1) * P], SPEC.top)
    router = be.router(layer.router, SPEC.top, layer.bias)
    return be, moe, router, DeviceOps(be, moe, router, world, T)


def test_exchange_one_rank_matches_single_device_and_replays(cuda, oracle):
    torch = cuda
    from open_rknpu2_lm_infer_b200.ep import DeviceExchange, ep_forward_device
    layer = S.make_layer(SPEC, seed=5)
    x = torch.from_numpy(S.make_input(SPEC, T, seed=6)).cuda()
    res = torch.from_numpy(S.make_input(SPEC, T, seed=7, stream=5)).cuda()
    ref = _single(torch, layer, x, res)
    # the single-device layer itself against the CPU restatement
    from conftest import assert_close
    assert_close(ref, oracle.OracleLayer(layer).forward(x.cpu().numpy(), res.cpu().numpy()),
                 what="single-device layer vs restatement")
    be, moe, router, ops = _rank_setup(1, 0, layer)
    ex = DeviceExchange(ops, None)
    from open_rknpu2_lm_infer_b200 import _lib as L
    from open_rknpu2_lm_infer_b200.moe import MoeError
    with pytest.raises(MoeError) as e:  # no profiled step yet
        ex.profile_read()
    assert e.value.code == L.ERR_INVALID
    ex.profile(True)
    for _ in range(2):  # the step counter advances; results repeat
        out = ep_forward_device(ops, ex, x, res)
        torch.cuda.synchronize()
        ex.status(); ops.status()
        assert np.array_equal(out.cpu().numpy(), ref)
    stages = ex.profile_read()  # the stage timings of the last profiled step
    assert set(stages) == set(ex.STAGES)
    assert all(v >= 0.0 for v in stages.values()) and stages["expert_rows_us"] > 0.0
    ex.profile(False)
    # the same step captured once and replayed
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out_g = ep_forward_device(ops, ex, x, res)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        out_g.zero_()
        g.replay()
        torch.cuda.synchronize()
        ex.status()
        assert np.array_equal(out_g.cpu().numpy(), ref)
    del g
    ex.close(); ops.close(); moe.close(); router.close(); be.close()


def test_exchange_wait_gives_up_and_the_exchange_recovers(cuda, oracle):
    """A wait that nothing completes ends with an error, not a hang: the
    exchange's row wait on a step that no source dispatches gives up after its
    limit (~2 s) and the status reports MOE_B200_ERR_DEVICE_TIMEOUT; the
    context and the exchange stay usable and the next layer step is exact."""
    torch = cuda
    from open_rknpu2_lm_infer_b200 import _lib as L
    from open_rknpu2_lm_infer_b200.ep import DeviceExchange, ep_forward_device
    from open_rknpu2_lm_infer_b200.moe import MoeError
    layer = S.make_layer(SPEC, seed=5)
    x = torch.from_numpy(S.make_input(SPEC, T, seed=6)).cuda()
    res = torch.from_numpy(S.make_input(SPEC, T, seed=7, stream=5)).cuda()
    ref = _single(torch, layer, x, res)
    # the single-device layer itself against the CPU restatement
    from conftest import assert_close
    assert_close(ref, oracle.OracleLayer(layer).forward(x.cpu().numpy(), res.cpu().numpy()),
                 what="single-device layer vs restatement")
    be, moe, router, ops = _rank_setup(1, 0, layer)
    ex = DeviceExchange(ops, None)
    ex.probe_timeout()
    with pytest.raises(MoeError) as e:
        ex.status()
    assert e.value.code == L.ERR_DEVICE_TIMEOUT
    ex.status()  # cleared
    out = ep_forward_device(ops, ex, x, res)
    torch.cuda.synchronize()
    ex.status(); ops.status()
    assert np.array_equal(out.cpu().numpy(), ref)
    ex.close(); ops.close(); moe.close(); router.close(); be.close()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _two_rank_main(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from open_rknpu2_lm_infer_b200.ep import DeviceExchange, ep_forward_device
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        layer = S.make_layer(SPEC, seed=5)
        x = torch.from_numpy(S.make_input(SPEC, T, seed=10 + rank)).cuda()
        res = torch.from_numpy(S.make_input(SPEC, T, seed=20 + rank, stream=5)).cuda()
        ref = _single(torch, layer, x, res, device=rank)
        be, moe, router, ops = _rank_setup(world, rank, layer)
        ex = DeviceExchange(ops, dist)
        dist.barrier()
        outs = []
        for _ in range(3):
            out = ep_forward_device(ops, ex, x, res)
            outs.append(out.clone())
        torch.cuda.synchronize()
        ex.status(); ops.status()
        same = all(np.array_equal(o.cpu().numpy(), ref) for o in outs)
        # and the CPU restatement of the reference layer on this rank's tokens
        from oracle import oracle as O
        want = O.OracleLayer(layer).forward(x.cpu().numpy(), res.cpu().numpy())
        got = outs[-1].cpu().numpy().astype(np.float64)
        close = bool(np.all(np.abs(got - want) <= 1e-3 + 1e-2 * np.abs(want)))
        np.save(os.path.join(outdir, f"ok{rank}.npy"), np.array([same and close]))
        dist.barrier()  # every rank done with its peers' memory before unmapping
        ex.close(); ops.close(); moe.close(); router.close(); be.close()
    finally:
        dist.destroy_process_group()


def test_exchange_two_ranks_match_single_device(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_two_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        assert bool(np.load(tmp_path / f"ok{r}.npy")[0]), f"rank {r} differs"
