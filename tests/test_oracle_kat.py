"""Pins the CPU restatement against the reference's own known-answer tests.

Each test names the reference test it ports (happyme531/open_rknpu2_lm_infer).
The reference has no golden vectors for the expert GEMM stages (they lived in
the un-vendored native submodule); those stages are pinned by the committed
fixtures in tests/golden/ and by the exact-arithmetic checks below.
"""
from fractions import Fraction

import numpy as np
import pytest

from oracle import oracle as O


# ---- routes(): src/model/qwen35/moe.rs:355-364 -------------------------------
def test_routing_is_normalized_over_selected_experts():
    ids, w = O.routes(np.array([-100.0, 1.0, 3.0, 2.0], np.float32), 2)
    assert ids.tolist() == [[2, 3]]
    assert abs(w[0, 0] - 1.0 / (1.0 + np.exp(-1.0))) < 1e-6
    assert abs(w.sum() - 1.0) < 1e-6
    with pytest.raises(ValueError):
        O.routes(np.zeros((1, 1), np.float32), 0)
    with pytest.raises(ValueError):
        O.routes(np.zeros((1, 1), np.float32), 2)


def test_routes_ties_prefer_lower_id_and_total_order():
    # equal logits: lower id first (sort_unstable_by(...).then(a.cmp(&b)))
    ids, _ = O.routes(np.array([1.0, 5.0, 5.0, 5.0, 0.0], np.float32), 3)
    assert ids.tolist() == [[1, 2, 3]]
    # total_cmp: +0 ranks above -0
    ids, _ = O.routes(np.array([-0.0, 0.0, -1.0], np.float32), 1)
    assert ids.tolist() == [[1]]
    assert O.total_key(0.0) > O.total_key(-0.0) > O.total_key(-1e-30)


# ---- Ling grouped routing: src/model/ling3tiny/moe.rs:404-493 ----------------
def test_ling_selection_matches_sorted_oracle_with_ties():
    from kat_vectors import (LING_GEOMETRIES, LING_SCALE, LING_STEPS, ling_sorted_oracle,
                             ling_step)
    for experts, groups, top_groups, top in LING_GEOMETRIES:
        for step in range(LING_STEPS):
            logits, bias = ling_step(experts, step)
            ref_ids, ref_w = ling_sorted_oracle(logits, bias, groups, top_groups, top,
                                                LING_SCALE, O.sigmoid)
            ids, w = O.ling_routes(logits, bias, groups, top_groups, top, LING_SCALE)
            assert ids[0].tolist() == ref_ids.tolist(), (experts, step)
            assert np.array_equal(w[0], ref_w), (experts, step)  # assert_eq! on f32


def test_ling_group_bias_selects_but_weights_use_original_sigmoid():
    from kat_vectors import LING_BIAS_CASE as K, LING_SCALE
    experts, groups, top_groups, top = K["geometry"]
    ids, w = O.ling_routes(K["logits"], K["bias"], groups, top_groups, top, LING_SCALE)
    assert ids[0].tolist() == K["ids"]
    total = sum(O.sigmoid(v) for v in K["weight_logits"])
    for got, v in zip(w[0], K["weight_logits"]):
        assert abs(got - O.sigmoid(v) / total * 2.5) < 1e-6
    assert abs(float(w[0].sum()) - 2.5) < 1e-6


def test_ling_geometry_is_validated():
    z = np.zeros((1, 8), np.float32)
    for g, tg, k in [(3, 1, 1), (8, 1, 1), (4, 5, 1), (4, 2, 5), (4, 2, 0)]:
        with pytest.raises(ValueError):
            O.ling_routes(z, np.zeros(8, np.float32), g, tg, k, 2.5)


def test_sigmoid_branches():
    # x >= 0: 1 / (1 + exp(-x)); x < 0: e / (1 + e) with e = exp(x)
    for x in (0.0, 0.5, 3.5, 20.0, 100.0):
        assert O.sigmoid(x) == np.float32(1.0) / (np.float32(1.0) + np.exp(np.float32(-x)))
    assert O.sigmoid(-100.0) > 0.0 and O.sigmoid(-1000.0) == 0.0
    assert O.sigmoid(0.0) == 0.5


def test_tf32_router_is_the_truncated_f64_dot():
    # src/npu/tf32.rs:190-224: both operands lose their low 13 mantissa bits
    k, n, rows = 1536, 128, 3
    i = np.arange(k * n)
    w = ((i * 13 % 71).astype(np.float32) - 35.0) * np.float32(0.001)
    w = (w.view(np.uint32) + 0x7FFF + ((w.view(np.uint32) >> 16) & 1)).astype(np.uint32)
    w = (w & 0xFFFF0000).view(np.float32).reshape(n, k)  # bf16-rounded weights, [N][K]
    x = (((np.arange(rows * k) * 7 % 83).astype(np.float32) - 41.0) * np.float32(0.01317))
    x = x.reshape(rows, k)
    got = O.router_logits(x, w, order=O.ROUTER_TF32)
    tr = lambda a: (a.view(np.uint32) & ~np.uint32(0x1FFF)).view(np.float32).astype(np.float64)
    expected = tr(x) @ tr(w).T
    assert np.abs(got.astype(np.float64) - expected).max() < 5e-5
    assert (got.view(np.uint32) & 0x1FFF).any()  # FP32 output, not narrowed
    assert not O.router_logits(x, np.zeros_like(w), order=O.ROUTER_TF32).any()


# ---- pruning::apply: src/model/experts/pruning.rs:64-84 --------------------
def test_threshold_keeps_boundary_and_best_without_renormalizing():
    # logits whose softmax weights are ~[0.5, 0.25, 0.125, 0.125]
    logits = np.log(np.array([0.5, 0.25, 0.125, 0.125], np.float64)).astype(np.float32)
    _, w0 = O.routes(logits, 4, 0.0)
    _, w = O.routes(logits, 4, 0.2)
    assert w[0, 0] == w0[0, 0] and w[0, 1] == w0[0, 1]  # no renormalisation
    assert w[0, 2] == 0.0 and w[0, 3] == 0.0
    _, w = O.routes(logits, 4, 1.0)
    assert w[0, 0] == w0[0, 0] and (w[0, 1:] == 0).all()  # the best route always stays
    # the boundary itself is kept: minimum == weight -> kept (`< minimum` drops)
    _, w = O.routes(logits, 4, float(w0[0, 1]))
    assert w[0, 1] == w0[0, 1]


# ---- SwiGLU: src/model/cpu.rs:481-518 (tolerance close(), :370-377) ----------
@pytest.mark.parametrize("rows,width", [(1, 128), (1, 9728), (3, 513), (4, 9728)])
def test_swiglu_matches_scalar_for_decode_and_prefill(rows, width):
    i = np.arange(rows * 2 * width, dtype=np.float32)
    gu = (np.sin(i * np.float32(0.019)) * np.float32(90.0)).astype(np.float32).reshape(rows, 2 * width)
    y = O.swiglu(gu, width)
    g, u = gu[:, :width], gu[:, width:]
    expected = (g / (np.float32(1.0) + np.exp(-g))) * u
    tol = np.float32(3e-7)
    assert np.all(np.abs(y - expected) <= tol * (1 + np.abs(expected)))


# ---- router order: src/model/cpu.rs:96-153, batch test :322-369 --------------
def _round_f32(fr: Fraction) -> np.float32:
    """Correctly rounded (nearest-even) float32 of an exact rational."""
    if fr == 0:
        return np.float32(0.0)
    f = np.float32(float(fr))
    cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
    best = min(cands, key=lambda c: (abs(Fraction(float(c)) - fr),
                                     int(np.array(c, np.float32).view(np.uint32)) & 1))
    return np.float32(best)


def _fma(a, b, c):
    return _round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _add(a, b):
    return _round_f32(Fraction(float(a)) + Fraction(float(b)))


def _neon16_dot_exact(w, x):
    """The aarch64 F32 dense_dot (src/model/cpu.rs:127-151) in exact arithmetic."""
    H = len(x)
    lanes = [np.float32(0.0)] * 16
    i = 0
    while i + 16 <= H:
        for j in range(16):
            lanes[j] = _fma(w[i + j], x[i + j], lanes[j])
        i += 16
    v = [_add(_add(lanes[j], lanes[4 + j]), _add(lanes[8 + j], lanes[12 + j])) for j in range(4)]
    s = _add(_add(v[0], v[1]), _add(v[2], v[3]))
    while i < H:
        s = _add(s, _round_f32(Fraction(float(w[i])) * Fraction(float(x[i]))))
        i += 1
    return s


def _seq_dot_exact(w, x):
    s = np.float32(0.0)
    for i in range(len(x)):
        s = _add(s, _round_f32(Fraction(float(w[i])) * Fraction(float(x[i]))))
    return s


def _pattern(n, k, rows):
    i = np.arange(n * k)
    w = (((i * 37 % 509).astype(np.float32) - 254.0) * np.float32(0.00791)).astype(np.float32)
    j = np.arange(rows * k)
    x = (((j * 53 % 487).astype(np.float32) - 243.0) * np.float32(0.019)).astype(np.float32)
    return w.reshape(n, k), x.reshape(rows, k)


@pytest.mark.parametrize("order", [O.ROUTER_NEON16, O.ROUTER_SEQUENTIAL])
def test_batched_router_preserves_row_order_and_exact_dots(order):
    for n, k in [(7, 19), (256, 2048)]:
        w, x = _pattern(n, k, 16)
        batched = O.router_logits(x, w, order=order)
        for r in (0, 7, 15):
            single = O.router_logits(x[r:r + 1], w, order=order)
            assert np.array_equal(batched[r].view(np.uint32), single[0].view(np.uint32))
    # exact-arithmetic restatement of the accumulation order on a few dots
    ref = _neon16_dot_exact if order == O.ROUTER_NEON16 else _seq_dot_exact
    for n, k in [(7, 19), (4, 300)]:
        w, x = _pattern(n, k, 2)
        got = O.router_logits(x, w, order=order)
        for r in range(2):
            for e in range(n):
                assert got[r, e].view(np.uint32) == ref(w[e], x[r]).view(np.uint32), (n, k, r, e)


# ---- quantisation rules ------------------------------------------------------
def test_moe_quantisation_rounds_half_even_and_zero_row_scale_one():
    # s = 127/127 = 1 -> q = rne(x): 0.5 -> 0, 1.5 -> 2, 2.5 -> 2
    x = np.array([[127.0, 0.5, 1.5, 2.5, -0.5, -1.5]], np.float32)
    q, s = O.quantize(x, O.QUANT_MOE)
    assert s[0] == 1.0 and q[0].tolist() == [127, 0, 2, 2, 0, -2]
    q, s = O.quantize(np.zeros((1, 8), np.float32), O.QUANT_MOE)
    assert s[0] == 1.0 and not q.any()


def test_dense_quantisation_rounds_half_away():
    x = np.array([[127.0, 0.5, 1.5, 2.5, -0.5, -2.5]], np.float32)
    q, s = O.quantize(x, O.QUANT_DENSE)
    assert s[0] == 1.0 and q[0].tolist() == [127, 1, 2, 3, -1, -3]


def test_group_accumulators_are_exact_integer_dots():
    rng = np.random.default_rng(7)
    q = rng.integers(-127, 128, size=(5, 64), dtype=np.int8)
    codes = rng.integers(-8, 8, size=(64, 24), dtype=np.int8)

    class M:
        bits, k, n, group = 4, 64, 24, 32
        scales = np.ones((2, 24), np.float16)
    M.codes = codes
    acc = O.gemm_acc(q, M)
    ref = np.einsum("rgk,gkn->rgn", q.reshape(5, 2, 32).astype(np.int64),
                    codes.reshape(2, 32, 24).astype(np.int64))
    assert np.array_equal(acc, ref)


def test_half_conversion_round_trips():
    for v in (0.0, 1.0, -2.5, 6.1e-5, 3.0e-7, 65504.0, 0.0123):
        h = O.lib().oracle_float_to_half(v)
        assert h == int(np.array(v, np.float16).view(np.uint16))
        assert O.lib().oracle_half_to_float(h) == float(np.float16(v))


# ---- shared-expert gate merge: src/model/qwen35/moe.rs:334-347 --------------
def test_shared_gate_merge_is_projected_plus_scaled_shared():
    from open_rknpu2_lm_infer_b200 import synthetic as S
    spec = S.small_spec("q35g", hidden=256, inter=64, experts=8, top=2, shared_inter=64)
    layer = S.make_layer(spec, seed=9)
    x = S.make_input(spec, 6, seed=1)
    res = S.make_input(spec, 6, seed=2, stream=5)
    ol = O.OracleLayer(layer, shared_mode=O.SHARED_DENSE)
    out, d = ol.forward(x, res, dump=True)
    g = O.router_logits(x, layer.shared_gate[None, :])[:, 0]
    one = np.float32(1.0)
    # the reference's scale: 1 / (1 + exp(-gate)) in f32 (glibc expf via the oracle)
    scale = np.array([one / (one + np.float32(np.exp(np.float64(-v)))) for v in g], np.float32)
    assert np.allclose(d["shared_scale"], scale, rtol=1e-6, atol=0)
    merged = (d["routed"] + (d["shared_scale"][:, None] * d["shared"]).astype(np.float32))
    assert np.array_equal(out, (res + merged.astype(np.float32)).astype(np.float32))


def test_ling_layer_routes_through_grouped_rule():
    from open_rknpu2_lm_infer_b200 import synthetic as S
    spec = S.small_spec("ling", hidden=256, inter=64, experts=16, top=4, groups=4, top_groups=2,
                        shared_inter=64)
    layer = S.make_layer(spec, seed=3)
    x = S.make_input(spec, 5, seed=4)
    out, d = O.OracleLayer(layer).forward(x, None, dump=True)
    logits = O.router_logits(x, layer.router, None, O.ROUTER_TF32)
    assert np.array_equal(d["logits"], logits)
    ids, w = O.ling_routes(logits, layer.expert_bias, 4, 2, 4, 2.5)
    assert np.array_equal(d["ids"], ids) and np.array_equal(d["weights"], w)
    assert np.allclose(w.sum(axis=1), 2.5, rtol=1e-6)
    # the chosen experts lie in at most top_groups groups
    assert all(len(set((row // 4).tolist())) <= 2 for row in ids)


def test_rms_norm_is_the_sequential_reference_sum():
    """The restatement's RMSNorm against a scalar loop written from
    src/ops/norm.rs:96-104: iterator sum of x*x (each product rounded, added in
    column order from -0.0), scale = recip(sqrt(sum / width + eps)), y = (x *
    scale) * w, w -> 1 + w when zero-centred; an all-zero row gives 0."""
    from oracle import oracle as O
    rng = np.random.default_rng(7)
    for rows, width, zc in ((3, 37, False), (4, 64, True)):
        x = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
        x[1] = 0.0
        w = (1 + rng.standard_normal(width) * 0.02).astype(np.float32)
        eps = np.float32(1e-6)
        ref = np.empty_like(x)
        for r in range(rows):
            s = np.float32(-0.0)
            for i in range(width):
                s = np.float32(s + np.float32(x[r, i] * x[r, i]))
            scale = np.float32(1.0) / np.sqrt(np.float32(s / np.float32(width) + eps))
            for i in range(width):
                wv = np.float32(1.0 + w[i]) if zc else w[i]
                ref[r, i] = np.float32(np.float32(x[r, i] * scale) * wv)
        got = O.rms_norm(x, w, float(eps), zc)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert not got[1].any()
