"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py).

CPU: the restatement still reproduces every stored stage bit for bit.
GPU: the C-ABI path matches the stored ids / permutation exactly and the
stored output within tolerance.
"""
from pathlib import Path

import numpy as np
import pytest

from conftest import assert_close
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, QuantMatrix

GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load_fixture(name):
    f = np.load(GOLDEN / f"{name}.npz")
    H, I, E, k, Is, T, fmt = (int(v) for v in f["meta"])
    routed = ["w4g32", "w4pc", "w8pc"][fmt]
    spec = S.LayerSpec(name, H, I, E, k, routed=routed, shared_inter=Is)

    def qm(prefix, kk, n):
        codes, scales = f[f"{prefix}_codes"], f[f"{prefix}_scales"]
        bits = 8 if routed == "w8pc" or prefix.startswith("s") else 4
        group = 32 if scales.dtype == np.float16 else 0
        return QuantMatrix(bits, kk, n, codes, scales, group)

    gate = [qm(f"gate{e}", H, 2 * I) for e in range(E)]
    down = [qm(f"down{e}", I, H) for e in range(E)]
    shared = (qm("sgate", H, 2 * Is), qm("sdown", Is, H)) if Is else None
    layer = S.Layer(spec, f["router"], f["bias"] if "bias" in f else None, gate, down, shared)
    refs = {k[4:]: f[k] for k in f.files if k.startswith("ref_")}
    return layer, f["x"], f["residual"], f["out"], refs


def test_fixtures_present():
    assert {"tiny_w4g32", "tiny_w8_shared"} <= set(NAMES)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_reproduces_golden(oracle, name):
    layer, x, res, out, refs = load_fixture(name)
    got, d = oracle.OracleLayer(layer).forward(x, res, dump=True)
    assert np.array_equal(got.view(np.uint32), out.view(np.uint32))
    for k, v in refs.items():
        a = d[k]
        if a.dtype == np.float32:
            assert np.array_equal(a.view(np.uint32), v.view(np.uint32)), k
        else:
            assert np.array_equal(a, v), k


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_gpu_matches_golden(cuda, name):
    layer, x, res, out, refs = load_fixture(name)
    spec = layer.spec
    be = Backend(max_rows=x.shape[0])
    if layer.shared is not None:
        moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared)
    else:
        moe = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    got, ids, routes = moe.forward(router, x, res)
    assert np.array_equal(ids, refs["ids"])
    assert_close(routes, refs["weights"], rtol=1e-5, atol=1e-7, what="weights")
    assert_close(got, out, what="output")
    moe.close(); router.close(); be.close()
