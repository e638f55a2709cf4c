"""Routing rules beyond softmax top-k, on the GPU through the C ABI.

Ling's grouped sigmoid routing (src/model/ling3tiny/moe.rs:146-223) with its
TF32 router (src/npu/tf32.rs:142-170), and the Qwen3.5 shared-expert sigmoid
gate (src/model/qwen35/moe.rs:334-347), against the CPU restatement.

Bars: the reference's own KATs for the routing function (ids exact, weights
equal up to the exp rounding: the GPU's f32 exp is the correctly rounded one,
glibc's expf differs by an ulp on about 1 in 13,000 arguments); TF32 logits
within 5e-5 of the f64 sum of the narrowed products (the reference's bound,
src/npu/tf32.rs:212-224); the gate logit bit-exact in the router's order;
layer outputs within 1e-3 + 1e-2 * |ref|.
"""
import numpy as np
import pytest

from conftest import assert_close
from kat_vectors import (LING_BIAS_CASE, LING_GEOMETRIES, LING_SCALE, LING_STEPS,
                         ling_sorted_oracle, ling_step)
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError

pytestmark = pytest.mark.gpu

KAT_H = 256


def _route_logits(torch, be, moe, logits, bias, groups, top_groups, top):
    """Runs the grouped router on rows whose logits are exactly `logits`:
    x = one-hot rows, router column t = logits of row t (exact products and sums)."""
    T, E = logits.shape
    w = np.zeros((E, KAT_H), np.float32)
    w[:, :T] = logits.T
    x = np.eye(T, KAT_H, dtype=np.float32)
    router = be.router(w, top, None, L.ROUTER_SEQUENTIAL, rule=L.ROUTE_GROUPED_SIGMOID,
                       groups=groups, top_groups=top_groups, routing_scale=LING_SCALE,
                       expert_bias=bias)
    dx = torch.from_numpy(x).cuda()
    dl = torch.empty((T, E), device="cuda", dtype=torch.float32)
    ids = torch.empty((T, top), device="cuda", dtype=torch.int32)
    rw = torch.empty((T, top), device="cuda", dtype=torch.float32)
    moe.route_device(router, T, dx.data_ptr(), dl.data_ptr(), ids.data_ptr(), rw.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    moe.status()
    router.close()
    assert np.array_equal(dl.cpu().numpy(), logits)
    return ids.cpu().numpy(), rw.cpu().numpy()


def _kat_bank(experts, top):
    spec = S.small_spec("c1", hidden=KAT_H, inter=256, experts=experts, top=top, routed="w4pc")
    layer = S.make_layer(spec, seed=1)
    be = Backend(device=0, max_rows=16)
    return be, be.load_moe(layer.gate, layer.down, top)


def test_ling_selection_kat_on_gpu(cuda, oracle):
    """src/model/ling3tiny/moe.rs:404-474, every geometry and step."""
    torch = cuda
    for experts, groups, top_groups, top in LING_GEOMETRIES:
        be, moe = _kat_bank(experts, top)
        for step in range(LING_STEPS):
            logits, bias = ling_step(experts, step)
            ids, w = _route_logits(torch, be, moe, logits[None, :], bias, groups, top_groups, top)
            ref_ids, ref_w = ling_sorted_oracle(logits, bias, groups, top_groups, top,
                                                LING_SCALE, oracle.sigmoid)
            assert ids[0].tolist() == ref_ids.tolist(), (experts, step)
            assert_close(w[0], ref_w, rtol=1e-6, atol=0, what=f"weights E={experts} step={step}")
        moe.close(); be.close()


def test_ling_group_bias_kat_on_gpu(cuda, oracle):
    """src/model/ling3tiny/moe.rs:475-492."""
    torch = cuda
    K = LING_BIAS_CASE
    experts, groups, top_groups, top = K["geometry"]
    be, moe = _kat_bank(experts, top)
    ids, w = _route_logits(torch, be, moe, K["logits"][None, :], K["bias"], groups, top_groups,
                           top)
    assert ids[0].tolist() == K["ids"]
    total = sum(oracle.sigmoid(v) for v in K["weight_logits"])
    for got, v in zip(w[0], K["weight_logits"]):
        assert abs(got - oracle.sigmoid(v) / total * 2.5) < 1e-6
    assert abs(float(w[0].sum()) - 2.5) < 1e-6
    moe.close(); be.close()


def test_grouped_router_rejects_invalid_geometry(cuda):
    be, moe = _kat_bank(8, 4)
    w = np.zeros((8, KAT_H), np.float32)
    bias = np.zeros(8, np.float32)
    for groups, top_groups in [(3, 1), (8, 1), (4, 5), (4, 1)]:  # (4, 1): top 4 > 1 * 2
        with pytest.raises((ValueError, MoeError)):
            be.router(w, 4, rule=L.ROUTE_GROUPED_SIGMOID, groups=groups, top_groups=top_groups,
                      routing_scale=2.5, expert_bias=bias)
    with pytest.raises((ValueError, MoeError)):  # the selection bias is required
        be.router(w, 4, rule=L.ROUTE_GROUPED_SIGMOID, groups=4, top_groups=2, routing_scale=2.5)
    moe.close(); be.close()


@pytest.mark.parametrize("rows", [1, 17, 128, 3, 1])
def test_tf32_router_matches_truncating_oracle(cuda, oracle, rows):
    """src/npu/tf32.rs:190-245 (resident_router_matches_truncating_oracle_across_batches)."""
    torch = cuda
    k, n = 1536, 128
    i = np.arange(k * n)
    wv = ((i * 13 % 71).astype(np.float32) - 35.0) * np.float32(0.001)
    # half::bf16::from_f32 rounds to nearest even
    u = wv.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    weights = u.view(np.float32).reshape(n, k)
    x = ((np.arange(rows * k) * 7 % 83).astype(np.float32) - 41.0) * np.float32(0.01317)
    x = x.reshape(rows, k).astype(np.float32)
    spec = S.small_spec("c1", hidden=k, inter=256, experts=n, top=8, routed="w4pc")
    layer = S.make_layer(spec, seed=2)
    be = Backend(device=0, max_rows=128)
    moe = be.load_moe(layer.gate, layer.down, 8)
    dx = torch.from_numpy(x).cuda()
    ids = torch.empty((rows, 8), device="cuda", dtype=torch.int32)
    rw = torch.empty((rows, 8), device="cuda", dtype=torch.float32)
    outs = []
    for wmat in (np.zeros_like(weights), weights, weights):
        router = be.router(wmat, 8, None, L.ROUTER_TF32)
        dl = torch.empty((rows, n), device="cuda", dtype=torch.float32)
        moe.route_device(router, rows, dx.data_ptr(), dl.data_ptr(), ids.data_ptr(),
                         rw.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        moe.status()
        outs.append(dl.cpu().numpy())
        router.close()
    assert (outs[0] == 0).all()
    tr = lambda a: (a.view(np.uint32) & ~np.uint32(0x1FFF)).view(np.float32).astype(np.float64)
    expected = tr(x) @ tr(weights).T
    assert np.abs(outs[1].astype(np.float64) - expected).max() < 5e-5
    assert (outs[1].view(np.uint32) & 0x1FFF).any(), "FP32 output was narrowed"
    assert np.array_equal(outs[1], outs[2])  # repeatable
    moe.close(); be.close()


LING_SPECS = {"ling_e32": S.small_spec("ling", experts=32), "ling": S.CONFIGS["ling"]}


@pytest.mark.parametrize("name,T", [("ling_e32", 1), ("ling_e32", 45), ("ling", 1),
                                    ("ling", 512)])
def test_ling_layer_matches_oracle(cuda, oracle, name, T):
    torch = cuda
    spec = LING_SPECS[name]
    layer = S.make_layer(spec, seed=4)
    x = S.make_input(spec, T, seed=41)
    res = S.make_input(spec, T, seed=42, stream=5)
    be = Backend(device=0, max_rows=max(T, 8))
    moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared)
    router = be.router_for(layer)
    out, ids, routes = moe.forward(router, x, res)
    # logits: TF32 within the reference's bound of the truncated f64 dot
    ptr, nbytes = moe.buffer("logits")
    assert nbytes >= T * spec.experts * 4
    gl = torch.as_tensor(_CAI(ptr, (T, spec.experts)), device="cuda").cpu().numpy()
    ref_l = oracle.router_logits(x, layer.router, None, oracle.ROUTER_TF32)
    assert np.abs(gl.astype(np.float64) - ref_l).max() < 5e-5
    # routing of the GPU's logits: ids exact, weights to the exp rounding
    r_ids, r_w = oracle.ling_routes(gl, layer.expert_bias, spec.groups, spec.top_groups,
                                    spec.top, spec.routing_scale)
    assert np.array_equal(ids, r_ids), "expert ids differ"
    assert_close(routes, r_w, rtol=1e-6, atol=0, what="routing weights")
    # the layer on those routes (joint shared expert, ungated)
    ref = oracle.OracleLayer(layer).run(x, ids, routes) + res
    assert_close(out, ref, what=f"{name} T={T} output")
    moe.close(); router.close(); be.close()


class _CAI:
    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4",
                                         "data": (ptr, False), "version": 3}


GATE_SPECS = {"q35g_e32": S.small_spec("q35g", experts=32), "q35g": S.CONFIGS["q35g"]}


@pytest.mark.parametrize("name,T", [("q35g_e32", 1), ("q35g_e32", 4), ("q35g_e32", 40),
                                    ("q35g", 512)])
def test_shared_gate_layer_matches_oracle(cuda, oracle, name, T):
    torch = cuda
    spec = GATE_SPECS[name]
    layer = S.make_layer(spec, seed=6)
    x = S.make_input(spec, T, seed=61)
    res = S.make_input(spec, T, seed=62, stream=5)
    be = Backend(device=0, max_rows=max(T, 8))
    moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared,
                                  L.SHARED_DENSE)
    router = be.router_for(layer)
    assert router.logit_columns == spec.experts + 1
    out, ids, routes = moe.forward(router, x, res)
    ptr, nbytes = moe.buffer("logits")
    assert nbytes >= T * (spec.experts + 1) * 4
    gl = torch.as_tensor(_CAI(ptr, (T, spec.experts + 1)), device="cuda").cpu().numpy()
    ol = oracle.OracleLayer(layer, shared_mode=oracle.SHARED_DENSE)
    ref, d = ol.forward(x, res, dump=True)
    # expert logits and the gate logit: bit-exact in the router's order
    assert np.array_equal(gl[:, :spec.experts].view(np.uint32), d["logits"].view(np.uint32))
    ref_gate = oracle.router_logits(x, layer.shared_gate[None, :])[:, 0]
    assert np.array_equal(gl[:, spec.experts].view(np.uint32), ref_gate.view(np.uint32))
    assert np.array_equal(ids, d["ids"]), "expert ids differ"
    assert_close(out, ref, what=f"{name} T={T} output")
    # the gate is live (scales well inside (0, 1)) and the oracle merges it as
    # projected + scale * shared
    scale = d["shared_scale"]
    assert ((scale > 0.05) & (scale < 0.95)).mean() > 0.5
    assert_close(d["routed"] + scale[:, None] * d["shared"] + res, ref, rtol=1e-6, atol=1e-6,
                 what="oracle gate merge")
    moe.close(); router.close(); be.close()


def test_shared_gate_graph_replay_matches_forward(cuda):
    torch = cuda
    spec = GATE_SPECS["q35g_e32"]
    layer = S.make_layer(spec, seed=6)
    T = 24
    x = S.make_input(spec, T, seed=63)
    res = S.make_input(spec, T, seed=64, stream=5)
    be = Backend(device=0, max_rows=T)
    moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared,
                                  L.SHARED_DENSE)
    router = be.router_for(layer)
    ref, _, _ = moe.forward(router, x, res)
    dx, dr = torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda()
    dout = torch.empty_like(dx)
    g = moe.graph(router, T, dx.data_ptr(), dr.data_ptr(), dout.data_ptr())
    g.launch(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    moe.status()
    assert np.array_equal(dout.cpu().numpy(), ref)
    g.close(); moe.close(); router.close(); be.close()
