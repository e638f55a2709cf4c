"""Expert-parallel exchange logic on CPU ranks (gloo, world size 2).

The device steps of open_rknpu2_lm_infer_b200.ep (route, pack, expert rows,
combine) are stood in for by numpy code over the CPU restatement (oracle/);
the exchange itself -- counts, row and metadata all-to-alls, the y rows back,
the combine by send slot -- is the module's own ep_forward. Each rank's
output must equal the same computation with every expert on one rank bit for
bit, and the oracle's single-device layer within the output tolerance.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.ep import ep_forward, owner_of

SPEC = S.LayerSpec("ep_small", 256, 128, 8, 2)
TOKENS = 24
SEED = 77


class NumpyOps:
    """The EP device steps restated on the CPU (oracle primitives)."""

    def __init__(self, layer, rank, world):
        from oracle import oracle as O
        self.O = O
        self.layer = layer
        self.rank, self.world = rank, world
        self.E, self.k = SPEC.experts, SPEC.top
        self.per_rank = self.E // world
        self.H, self.I = SPEC.hidden, SPEC.inter

    def route(self, x):
        O = self.O
        logits = O.router_logits(x.numpy(), self.layer.router, self.layer.bias)
        ids, w = O.routes(logits, self.k)
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def pack(self, x, ids, routes):
        O = self.O
        q, s = O.quantize(x.numpy())
        ids_n, w = ids.numpy().reshape(-1), routes.numpy().reshape(-1)
        kept = np.flatnonzero(w > 0)
        dest = owner_of(ids_n[kept], self.per_rank)
        order = kept[np.argsort(dest, kind="stable")]  # by destination, assignment order within
        n = len(order)
        send_q = torch.from_numpy(q[order // self.k].copy())
        send_scale = torch.from_numpy(s[order // self.k].astype(np.float32))
        send_expert = torch.from_numpy((ids_n[order] % self.per_rank).astype(np.int32))
        counts = torch.from_numpy(np.bincount(owner_of(ids_n[order], self.per_rank),
                                              minlength=self.world).astype(np.int32))
        pos = np.full(ids_n.size, -1, np.int32)
        pos[order] = np.arange(n, dtype=np.int32)
        return send_q, send_scale, send_expert, counts, torch.from_numpy(pos)

    def empty_rows(self, n):
        return torch.empty((n, self.H), dtype=torch.int8)

    def empty_y(self, n):
        return torch.empty((n, self.H), dtype=torch.float32)

    def expert_rows(self, q, scale, expert):
        O = self.O
        q, scale, expert = q.numpy(), scale.numpy(), expert.numpy()
        y = np.zeros((q.shape[0], self.H), np.float32)
        for le in np.unique(expert):
            rows = np.flatnonzero(expert == le)
            e = self.rank * self.per_rank + int(le)
            gu = O.gemm_dequant(q[rows], scale[rows], self.layer.gate[e])
            qm, sm = O.quantize(O.swiglu(gu, self.I))
            y[rows] = O.gemm_dequant(qm, sm, self.layer.down[e])
        return torch.from_numpy(y)

    def combine(self, y_back, pos, routes, residual):
        # the single-device combine: fma over ranks ascending, weights > 0, then residual
        y, pos, w = y_back.numpy(), pos.numpy().reshape(-1, self.k), routes.numpy()
        out = np.zeros((w.shape[0], self.H), np.float32)
        for t in range(w.shape[0]):
            acc = np.zeros(self.H, np.float64)
            for r in range(self.k):
                if w[t, r] > 0:
                    acc = (y[pos[t, r]].astype(np.float64) * np.float64(w[t, r]) + acc).astype(
                        np.float32).astype(np.float64)
            out[t] = acc.astype(np.float32)
        if residual is not None:
            out = (residual.numpy() + out).astype(np.float32)
        return torch.from_numpy(out)


class LocalDist:
    """torch.distributed stand-in for one rank holding every expert."""

    @staticmethod
    def all_to_all_single(out, inp, out_splits=None, in_splits=None, group=None):
        out.copy_(inp)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = S.make_layer(SPEC, seed=SEED)
        x = torch.from_numpy(S.make_input(SPEC, TOKENS, seed=SEED + rank, stream=4))
        res = torch.from_numpy(S.make_input(SPEC, TOKENS, seed=SEED + rank, stream=5))
        out, plan = ep_forward(NumpyOps(layer, rank, world), dist, None, x, res)
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(outdir, f"plan{rank}.npy"), np.array([plan.send, plan.recv]))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def oracle_built():
    from oracle import oracle as O
    O.build()
    return O


def test_ep_two_ranks_match_one_rank(tmp_path, oracle_built):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    layer = S.make_layer(SPEC, seed=SEED)
    sends = []
    for rank in range(world):
        x = torch.from_numpy(S.make_input(SPEC, TOKENS, seed=SEED + rank, stream=4))
        res = torch.from_numpy(S.make_input(SPEC, TOKENS, seed=SEED + rank, stream=5))
        ref, _ = ep_forward(NumpyOps(layer, 0, 1), LocalDist, None, x, res)
        got = np.load(tmp_path / f"out{rank}.npy")
        assert np.array_equal(got, ref.numpy()), f"rank {rank}: EP output differs from one rank"
        # the oracle's single-device layer (its own combine), within the output tolerance
        full = oracle_built.OracleLayer(layer).forward(x.numpy(), res.numpy())
        np.testing.assert_allclose(got, full, rtol=1e-5, atol=1e-6)
        sends.append(np.load(tmp_path / f"plan{rank}.npy"))
    # what rank a sent to rank b is what rank b received from rank a
    for a in range(world):
        for b in range(world):
            assert sends[a][0][b] == sends[b][1][a]
    assert sum(int(sends[r][0].sum()) for r in range(world)) == world * TOKENS * SPEC.top


def _failing_rank_main(rank, world, port, outdir):
    """Rank 1 leaves before the layer (a host-side failure: it never joins the
    exchange); rank 0 runs the layer and must get an error from its first
    collective within the process group's short timeout, not hang."""
    import time
    from datetime import timedelta
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    if rank == 1:
        dist.destroy_process_group()
        return
    layer = S.make_layer(SPEC, seed=SEED)
    x = torch.from_numpy(S.make_input(SPEC, TOKENS, seed=SEED, stream=4))
    t0 = time.monotonic()
    status = "completed"
    try:
        ep_forward(NumpyOps(layer, rank, world), dist, None, x, None)
    except Exception as e:  # the collective's error surfaces on the host
        status = f"error: {type(e).__name__}"
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(f"{status}\n{time.monotonic() - t0:.1f}\n")


def test_a_rank_that_never_joins_makes_the_others_fail_not_hang(tmp_path, oracle_built):
    import torch.multiprocessing as mp
    mp.start_processes(_failing_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    status, seconds = (tmp_path / "rank0.txt").read_text().split("\n")[:2]
    assert status.startswith("error"), status
    assert float(seconds) < 60.0


def test_owner_of_partitions_experts():
    ids = np.arange(128)
    own = owner_of(ids, 16)
    assert own.min() == 0 and own.max() == 7
    assert all(np.count_nonzero(own == g) == 16 for g in range(8))
