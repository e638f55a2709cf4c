"""Parity of the sm_100a path (through the C ABI) against the CPU restatement.

Bit-exact: router logits, expert ids, permutation, offsets, quantised
activations and scales, every INT32 accumulator (per group for group-32
weights; the down GEMM fed with the GPU's own middle codes). Floating-point
outputs: |gpu - ref| <= 1e-3 + 1e-2 * |ref| elementwise.
"""
import numpy as np
import pytest

from conftest import ATOL, RTOL, assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError

pytestmark = pytest.mark.gpu


class _CAI:
    """Zero-copy view of a library-owned device buffer for torch."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


def dev_view(torch, moe, name, shape, dtype):
    ptr, nbytes = moe.buffer(name)
    typestr = {np.int32: "<i4", np.float32: "<f4", np.int8: "|i1", np.uint32: "<u4"}[dtype]
    assert int(np.prod(shape)) * np.dtype(dtype).itemsize <= nbytes
    return torch.as_tensor(_CAI(ptr, shape, typestr), device="cuda").cpu().numpy()


_LAYERS = {}


def layer_for(spec, seed=3):
    key = (spec, seed)
    if key not in _LAYERS:
        _LAYERS[key] = S.make_layer(spec, seed=seed)
    return _LAYERS[key]


def build(layer, max_rows, shared_mode=None, order=0, min_weight=0.0, exact=True):
    be = Backend(device=0, max_rows=max_rows)
    spec = layer.spec
    if layer.shared is not None:
        moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared, shared_mode)
    else:
        moe = be.load_moe(layer.gate, layer.down, spec.top, exact=exact)
    router = be.router(layer.router, spec.top, layer.bias, order, min_weight)
    return be, moe, router


SPECS = {
    "c1": S.CONFIGS["c1"],
    "c2_e32": S.small_spec("c2", experts=32),
    "c2": S.CONFIGS["c2"],
    "c3_e32": S.small_spec("c3", experts=32),
    "w4pc": S.small_spec("c1", routed="w4pc"),
    "w8pc": S.small_spec("c1", routed="w8pc"),
    "joint": S.small_spec("c1", routed="w4pc", shared_inter=512),
}

# group-32 banks run both GEMMs on exact int32 group sums; "_rounded": the
# opt-in down projection on the fp16 tensor cores
CASES = [("c1", 32), ("c1", 1), ("c2_e32", 1), ("c2_e32", 37), ("c2_e32", 300),
         ("c3_e32", 64), ("w4pc", 48), ("w8pc", 48), ("joint", 40), ("c2", 512),
         ("c2_e32_rounded", 37), ("c2_rounded", 512), ("c1_rounded", 32),
         # 4 rows per expert: 16-token tiles
         ("c2", 64), ("c2_rounded", 64),
         # small batches of a bank with a shared expert: the routed GEMVs with
         # the shared FFN beside them on the side stream
         ("c3_e32", 1), ("c3_e32", 3), ("c3_e32", 4),
         # small batches of a per-channel int8 bank: the routed split-K GEMVs
         ("w8pc", 1), ("w8pc", 3), ("w8pc", 4),
         # just above the small batches (8 tokens): the tensor-core paths
         ("c2_e32", 8), ("c3_e32", 8), ("w8pc", 8)]


@pytest.mark.parametrize("name,T", CASES)
def test_forward_matches_oracle(cuda, oracle, name, T):
    exact = not name.endswith("_rounded")
    spec = SPECS[name.removesuffix("_rounded")]
    layer = layer_for(spec)
    x = S.make_input(spec, T, seed=11)
    res = S.make_input(spec, T, seed=12, stream=5)
    be, moe, router = build(layer, max_rows=max(T, 8), exact=exact)
    out, ids, routes = moe.forward(router, x, res)
    ref, d = oracle.OracleLayer(layer).forward(x, res, dump=True)
    assert np.array_equal(ids, d["ids"]), "expert ids differ"
    assert_close(routes, d["weights"], rtol=1e-5, atol=1e-7, what="routing weights")
    assert_close(out, ref, what=f"{name} T={T} output")
    moe.close(); router.close(); be.close()


@pytest.mark.parametrize("order", [L.ROUTER_NEON16, L.ROUTER_SEQUENTIAL])
@pytest.mark.parametrize("name,T", [("c1", 5), ("c2", 70), ("c3_e32", 33), ("c2", 2048)])
def test_router_logits_and_ids_bit_exact(cuda, oracle, name, T, order):
    torch = cuda
    spec = SPECS[name]
    layer = layer_for(spec)
    x = S.make_input(spec, T, seed=21)
    be, moe, router = build(layer, max_rows=T, order=order)
    dx = torch.from_numpy(x).cuda()
    logits = torch.empty((T, spec.experts), device="cuda", dtype=torch.float32)
    ids = torch.empty((T, spec.top), device="cuda", dtype=torch.int32)
    w = torch.empty((T, spec.top), device="cuda", dtype=torch.float32)
    moe.route_device(router, T, dx.data_ptr(), logits.data_ptr(), ids.data_ptr(), w.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    moe.status()
    ref_l = oracle.router_logits(x, layer.router, layer.bias, order)
    ref_ids, ref_w = oracle.routes(ref_l, spec.top)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), ref_l.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert_close(w.cpu().numpy(), ref_w, rtol=1e-5, atol=1e-7, what="routing weights")
    moe.close(); router.close(); be.close()


def test_router_ties_and_bias(cuda, oracle):
    torch = cuda
    spec = S.small_spec("c1", experts=16, top=4)
    layer = layer_for(spec)
    # duplicated router rows produce exactly tied logits: lower id must win
    layer.router[5] = layer.router[9]
    layer.router[2] = layer.router[9]
    layer.bias = np.linspace(0.5, -0.5, 16).astype(np.float32)
    layer.bias[5] = layer.bias[2] = layer.bias[9] = 3.0
    x = S.make_input(spec, 16, seed=5)
    be, moe, router = build(layer, max_rows=16)
    out, ids, routes = moe.forward(router, x)
    ref_l = oracle.router_logits(x, layer.router, layer.bias)
    ref_ids, _ = oracle.routes(ref_l, 4)
    assert np.array_equal(ids, ref_ids)
    assert (ids[:, :3] == np.array([2, 5, 9])).all()
    moe.close(); router.close(); be.close()
    _LAYERS.pop((spec, 3))


@pytest.mark.parametrize("name,T", [("c1", 32), ("c2_e32", 200), ("w4pc", 48), ("w8pc", 20),
                                    ("c2", 64)])
def test_dispatch_and_accumulators_bit_exact(cuda, oracle, name, T):
    torch = cuda
    spec = SPECS[name]
    layer = layer_for(spec)
    x = S.make_input(spec, T, seed=31)
    be, moe, router = build(layer, max_rows=T)
    out, ids, routes = moe.forward(router, x)
    ref, d = oracle.OracleLayer(layer).run(x, ids, routes, dump=True)
    H, I, E, k = spec.hidden, spec.inter, spec.experts, spec.top
    A = len(d["perm"])
    assert np.array_equal(dev_view(torch, moe, "offsets", (E + 1,), np.int32), d["offsets"])
    assert np.array_equal(dev_view(torch, moe, "perm", (A,), np.int32), d["perm"])
    pos = dev_view(torch, moe, "pos", (T * k,), np.int32)
    inv = np.full(T * k, -1, np.int32)
    inv[d["perm"]] = np.arange(A)
    assert np.array_equal(pos, inv)
    Kh = (H + 127) // 128 * 128
    qx = dev_view(torch, moe, "q_x", (T, Kh), np.int8)[:, :H]
    assert np.array_equal(qx, d["qx"])
    assert np.array_equal(dev_view(torch, moe, "s_x", (T,), np.float32).view(np.uint32),
                          d["sx"].view(np.uint32))
    a_perm = dev_view(torch, moe, "a_perm", (A, Kh), np.int8)[:, :H]
    assert np.array_equal(a_perm, d["qx"][d["perm"] // k])

    # gate/up INT32 accumulators (per group for group-32) vs the restatement
    G = (Kh // 32) if layer.gate[0].group else 1
    acc = torch.zeros(A * G * 2 * I, dtype=torch.int32, device="cuda")
    moe.debug_accumulators(0, acc.data_ptr(), acc.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    moe.status()
    acc = acc.cpu().numpy().reshape(A, G, 2 * I) if G > 1 else acc.cpu().numpy().reshape(A, 2 * I)
    off = d["offsets"]
    for e in range(E):
        rows = slice(off[e], off[e + 1])
        if off[e] == off[e + 1]:
            continue
        ref_acc = oracle.gemm_acc(d["qx"][d["perm"][rows] // k], layer.gate[e])
        got = acc[rows][:, : H // 32] if G > 1 else acc[rows]
        assert np.array_equal(got, ref_acc), f"gate/up accumulators differ for expert {e}"

    # middle (fp tolerance) and the down accumulators fed with the GPU's own codes
    Ki = (I + 127) // 128 * 128
    mid = oracle.swiglu(dev_view(torch, moe, "gate_up", (A, 2 * I), np.float32), I)
    assert_close(mid, d["middle"], what="SwiGLU middle")
    qm = dev_view(torch, moe, "q_m", (A, Ki), np.int8)[:, :I]
    flips = np.abs(qm.astype(np.int32) - d["qm"].astype(np.int32))
    assert flips.max() <= 1 and (flips > 0).mean() < 1e-3, "middle codes differ beyond rounding"
    G2 = (Ki // 32) if layer.down[0].group else 1
    acc2 = torch.zeros(A * G2 * H, dtype=torch.int32, device="cuda")
    moe.debug_accumulators(1, acc2.data_ptr(), acc2.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    acc2 = acc2.cpu().numpy().reshape(A, G2, H) if G2 > 1 else acc2.cpu().numpy().reshape(A, H)
    for e in range(E):
        rows = slice(off[e], off[e + 1])
        if off[e] == off[e + 1]:
            continue
        ref_acc = oracle.gemm_acc(qm[rows], layer.down[e])
        got = acc2[rows][:, : I // 32] if G2 > 1 else acc2[rows]
        assert np.array_equal(got, ref_acc), f"down accumulators differ for expert {e}"
    assert_close(out, ref, what="output")
    moe.close(); router.close(); be.close()


def test_run_f32_reference_contract(cuda, oracle):
    """Moe::run with caller-supplied routing: duplicates, zero and pruned routes."""
    spec = SPECS["c1"]
    layer = layer_for(spec)
    T = 24
    x = S.make_input(spec, T, seed=41)
    x[3] = 0.0                                  # all-zero row -> scale 1
    rng = np.random.default_rng(9)
    ids = rng.integers(0, spec.experts, size=(T, spec.top)).astype(np.int32)
    ids[5] = [7, 7]                             # duplicate expert for one token
    routes = rng.random((T, spec.top)).astype(np.float32)
    routes[6, 1] = 0.0                          # skipped route
    routes[7] = [0.0, 0.0]                      # token with no routes
    be, moe, router = build(layer, max_rows=T)
    out = np.empty((T, spec.hidden), np.float32)
    t = moe.run_profiled(x, ids, routes, out, T)
    assert t["total_us"] > 0 and t["gate_us"] > 0
    ref = oracle.OracleLayer(layer).run(x, ids, routes)
    assert_close(out, ref, what="run output")
    assert (out[7] == 0).all()
    moe.close(); router.close(); be.close()


def test_run_device_matches_host_api(cuda):
    torch = cuda
    spec = SPECS["c2_e32"]
    layer = layer_for(spec)
    T = 64
    x = S.make_input(spec, T, seed=51)
    be, moe, router = build(layer, max_rows=T)
    out, ids, routes = moe.forward(router, x)
    dx, dout = torch.from_numpy(x).cuda(), torch.empty((T, spec.hidden), device="cuda")
    did, dr = torch.from_numpy(ids).cuda(), torch.from_numpy(routes).cuda()
    s = torch.cuda.current_stream().cuda_stream
    moe.run_device(dx.data_ptr(), did.data_ptr(), dr.data_ptr(), dout.data_ptr(), T, s)
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy(), out)
    dout2 = torch.empty_like(dout)
    moe.forward_device(router, T, dx.data_ptr(), None, dout2.data_ptr(), s)
    torch.cuda.synchronize()
    assert np.array_equal(dout2.cpu().numpy(), out)
    moe.close(); router.close(); be.close()


def test_pruning_min_weight(cuda, oracle):
    spec = S.small_spec("c1", top=4)
    layer = layer_for(spec)
    x = S.make_input(spec, 32, seed=61)
    be, moe, router = build(layer, max_rows=32, min_weight=0.2)
    out, ids, routes = moe.forward(router, x)
    ol = oracle.OracleLayer(layer, min_weight=0.2)
    ref, d = ol.forward(x, dump=True)
    assert np.array_equal(ids, d["ids"])
    assert np.array_equal(routes == 0, d["weights"] == 0)
    assert (routes == 0).any()
    assert_close(out, ref, what="pruned output")
    moe.close(); router.close(); be.close()


def test_invalid_inputs_are_rejected(cuda):
    spec = SPECS["c1"]
    layer = layer_for(spec)
    be, moe, router = build(layer, max_rows=8)
    x = S.make_input(spec, 8, seed=71)
    out = np.empty((8, spec.hidden), np.float32)
    ids = np.zeros((8, 2), np.int32)
    routes = np.full((8, 2), 0.5, np.float32)
    bad = ids.copy(); bad[2, 1] = spec.experts
    with pytest.raises(MoeError) as e:
        moe.run(x, bad, routes, out, 8)
    assert e.value.code == L.ERR_BAD_EXPERT
    neg = routes.copy(); neg[1, 0] = -1.0
    with pytest.raises(MoeError) as e:
        moe.run(x, ids, neg, out, 8)
    assert e.value.code == L.ERR_BAD_ROUTE
    big = np.zeros((9, spec.hidden), np.float32)
    with pytest.raises(MoeError) as e:
        moe.run(big, np.zeros((9, 2), np.int32), np.ones((9, 2), np.float32),
                np.empty_like(big), 9)
    assert e.value.code == L.ERR_CAPACITY
    with pytest.raises(ValueError):
        moe.run(x, ids[:4], routes, out, 8)
    # the device path flags an out-of-range id through the status word
    import torch
    dx, dout = torch.from_numpy(x).cuda(), torch.empty((8, spec.hidden), device="cuda")
    d_ids, d_w = torch.from_numpy(bad).cuda(), torch.from_numpy(routes).cuda()  # kept alive
    moe.run_device(dx.data_ptr(), d_ids.data_ptr(), d_w.data_ptr(), dout.data_ptr(), 8,
                   torch.cuda.current_stream().cuda_stream)
    with pytest.raises(MoeError) as e:
        moe.status()
    assert e.value.code == L.ERR_BAD_EXPERT
    moe.status()  # cleared
    # zero rows is a no-op
    moe.run(x[:0], ids[:0], routes[:0], out[:0], 0)
    moe.close(); router.close(); be.close()


def test_allocation_failure_is_reported(cuda, tmp_path):
    """Host-side allocation-failure injection (the reference's workspace fault
    shim, tests/board/workspace_fault_ioctl.c): the N-th device allocation fails."""
    import subprocess
    import sys
    import textwrap
    code = textwrap.dedent("""
        import sys
        sys.path.insert(0, %r)
        from open_rknpu2_lm_infer_b200 import synthetic as S
        from open_rknpu2_lm_infer_b200.moe import Backend, MoeError
        layer = S.make_layer(S.small_spec("c1", experts=4), seed=1)
        be = Backend(max_rows=4)
        try:
            be.load_moe(layer.gate, layer.down, 2)
        except MoeError as e:
            print("CODE", e.code)
        else:
            print("NOERROR")
    """ % str(__import__("pathlib").Path(__file__).resolve().parents[1]))
    import os
    env = dict(os.environ, MOE_B200_FAIL_ALLOC_AFTER="2")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=300)
    assert f"CODE {L.ERR_NOMEM}" in r.stdout, r.stdout + r.stderr


def test_exact_group_format_reaches_the_library(cuda, oracle):
    """The exact and the fp16 down projection give different roundings of the
    same layer: outputs close, not identical."""
    spec = SPECS["c2_e32"]
    layer = layer_for(spec)
    x = S.make_input(spec, 64, seed=41)
    outs = []
    for exact in (False, True):
        be, moe, router = build(layer, max_rows=64, exact=exact)
        outs.append(moe.forward(router, x)[0])
        moe.close(); router.close(); be.close()
    assert not np.array_equal(outs[0], outs[1])
    assert_close(outs[0], outs[1], what="fp16 vs exact down projection")


@pytest.mark.parametrize("name,T", [("c2_e32", 1), ("c2_e32", 37), ("c1", 32), ("w8pc", 2),
                                    ("c3_e32", 2)])
def test_graph_replay_matches_forward(cuda, oracle, name, T):
    """A captured forward (moe_b200_graph_*) replays the same layer bit for bit,
    and reads its input buffer afresh on every replay."""
    torch = cuda
    spec = SPECS[name]
    layer = layer_for(spec)
    be, moe, router = build(layer, max_rows=max(T, 8))
    s = torch.cuda.current_stream().cuda_stream
    x = torch.from_numpy(S.make_input(spec, T, seed=51)).cuda()
    res = torch.from_numpy(S.make_input(spec, T, seed=52, stream=5)).cuda()
    out_g = torch.empty_like(x)
    g = moe.graph(router, T, x.data_ptr(), res.data_ptr(), out_g.data_ptr())
    for seed in (51, 53):
        x.copy_(torch.from_numpy(S.make_input(spec, T, seed=seed)))
        ref = torch.empty_like(x)
        moe.forward_device(router, T, x.data_ptr(), res.data_ptr(), ref.data_ptr(), s)
        g.launch(s)
        torch.cuda.synchronize()
        moe.status()
        assert torch.equal(out_g, ref), f"replay differs (input seed {seed})"
    g.close(); moe.close(); router.close(); be.close()


@pytest.mark.parametrize("name,T,with_res", [("c1", 1, True), ("c3_e32", 1, True),
                                             ("w8pc", 3, True), ("c2_e32", 37, False),
                                             ("joint", 40, True), ("c2", 512, True)])
def test_host_call_graph_matches_eager(cuda, oracle, name, T, with_res):
    """Host-buffer calls on page-locked buffers run as a captured graph of the
    copies and the layer (replayed while the buffers stay the same): bit for
    bit the eager call on pageable buffers, reading the inputs afresh on every
    call and counting the same kernels."""
    torch = cuda
    spec = SPECS[name]
    layer = layer_for(spec)
    be, moe, router = build(layer, max_rows=max(T, 8))
    lib = L.load()

    def pinned(shape, dt):
        return torch.empty(shape, dtype=dt, pin_memory=True).numpy()

    H, k = spec.hidden, spec.top
    xp, rp, op = (pinned((T, H), torch.float32) for _ in range(3))
    ip, wp = pinned((T, k), torch.int32), pinned((T, k), torch.float32)
    seeds = (61, 62, 61)
    eager = {}
    for seed in set(seeds):
        x = S.make_input(spec, T, seed=seed)
        res = S.make_input(spec, T, seed=seed + 100, stream=5) if with_res else None
        n0 = lib.moe_b200_workspace_launches(moe.workspace)
        eager[seed] = moe.forward(router, x, res) + (
            lib.moe_b200_workspace_launches(moe.workspace) - n0,)
    for seed in seeds:
        xp[...] = S.make_input(spec, T, seed=seed)
        if with_res:
            rp[...] = S.make_input(spec, T, seed=seed + 100, stream=5)
        n0 = lib.moe_b200_workspace_launches(moe.workspace)
        moe.forward(router, xp, rp if with_res else None, out=op, ids=ip, routes=wp)
        launched = lib.moe_b200_workspace_launches(moe.workspace) - n0
        out, ids, routes, n_eager = eager[seed]
        assert np.array_equal(op, out), f"{name} T={T}: graph call differs (seed {seed})"
        assert np.array_equal(ip, ids) and np.array_equal(wp, routes)
        assert launched == n_eager > 0
    ref = oracle.OracleLayer(layer).forward(
        xp, rp if with_res else None)
    assert_close(op, ref, what=f"{name} T={T} graph call")
    moe.close(); router.close(); be.close()


def test_host_call_graph_follows_the_bank_and_router(cuda):
    """The captured host-call graph is keyed on the bank and router objects
    (a creation serial, not only the address) and on the buffers: a new
    router, or a bank freed and created again, on the same page-locked
    buffers gives what an eager call gives, never a replay of the old graph."""
    torch = cuda
    spec = SPECS["c2_e32"]
    T = 37
    l1, l2 = layer_for(spec, seed=3), layer_for(spec, seed=4)
    be = Backend(device=0, max_rows=T)

    def pinned(shape, dt):
        return torch.empty(shape, dtype=dt, pin_memory=True).numpy()

    xp, op = pinned((T, spec.hidden), torch.float32), pinned((T, spec.hidden), torch.float32)
    ip, wp = pinned((T, spec.top), torch.int32), pinned((T, spec.top), torch.float32)
    x = S.make_input(spec, T, seed=81)
    xp[...] = x
    for round_ in range(2):
        moe = be.load_moe(l1.gate, l1.down, spec.top)
        for lay in (l1, l2, l1):
            router = be.router(lay.router, spec.top, lay.bias)
            ref, ids, routes = moe.forward(router, x)  # pageable: eager
            moe.forward(router, xp, out=op, ids=ip, routes=wp)
            assert np.array_equal(op, ref), f"round {round_}: stale graph replayed"
            assert np.array_equal(ip, ids) and np.array_equal(wp, routes)
            router.close()
        moe.close()  # the next bank may reuse this one's address
    be.close()
