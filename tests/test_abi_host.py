"""CPU-only checks of the boundary and the host-side mirror (no GPU compute).

- the C-ABI library loads and exports every entry point include/moe_b200.h declares
- pure-host entry points (config_init, strerror, version) behave
- QuantMatrix validation and the pack-quantized unpack known-answer test
  (src/model/checkpoint.rs:750-780)
- Backend validation errors raise before any device call (src/npu/moe.rs:101-117)
"""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, QuantMatrix

HEADER = Path(__file__).resolve().parents[1] / "include" / "moe_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(moe_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    bound = {s[0] for s in L.SIGNATURES}
    assert set(names) == bound, "ctypes signatures out of sync with the header"


def test_host_only_entry_points():
    lib = L.load()
    cfg = L.Config()
    lib.moe_b200_config_init(C.byref(cfg), 2048, 768, 128, 0, 8, 512)
    assert (cfg.weights.hidden, cfg.weights.intermediate, cfg.weights.routed_experts,
            cfg.weights.shared_expert, cfg.top, cfg.max_rows) == (2048, 768, 128, 0, 8, 512)
    assert b"sm_100a" in lib.moe_b200_version()
    assert L.strerror(0) == "success"
    for code in range(-10, 0):
        assert L.strerror(code) != "unknown error"
    assert L.strerror(-99) == "unknown error"
    assert lib.moe_b200_weights_device_bytes(None) == 0
    assert lib.moe_b200_max_rows(None) == 0


def test_pack_quantized_unpack_known_answer():
    # c4_fixture: q.weight_packed I32 [2,1] = [0x87654321, 0xfedcba98], scales [0.25, 0.5]
    packed = np.array([[0x87654321], [0xFEDCBA98]], dtype=np.uint32).view(np.int32)
    m = QuantMatrix.from_pack_quantized(packed, np.array([[0.25], [0.5]], np.float32), 4, 2, 8)
    assert m.codes.reshape(-1).tolist() == [-7, 0, -6, 1, -5, 2, -4, 3, -3, 4, -2, 5, -1, 6, 0, 7]
    assert m.scales.tolist() == [0.25, 0.5]
    m.validate()
    with pytest.raises(ValueError):
        QuantMatrix.from_pack_quantized(packed, np.array([[0.25], [0.0]], np.float32), 4, 2, 8)


def test_quant_matrix_validation():
    ok = QuantMatrix(4, 4, 2, np.zeros(8, np.int8), np.ones(2, np.float32))
    ok.validate()
    for bad in (QuantMatrix(3, 4, 2, np.zeros(8, np.int8), np.ones(2, np.float32)),
                QuantMatrix(4, 4, 2, np.zeros(7, np.int8), np.ones(2, np.float32)),
                QuantMatrix(4, 4, 2, np.zeros(8, np.int8), np.ones(3, np.float32)),
                QuantMatrix(4, 4, 2, np.full(8, 9, np.int8), np.ones(2, np.float32)),
                QuantMatrix(4, 64, 2, np.zeros(128, np.int8), np.ones((3, 2), np.float16), 32)):
        with pytest.raises(ValueError):
            bad.validate()


def test_backend_validates_before_device_calls():
    layer = S.make_layer(S.small_spec("c1", experts=4, hidden=64, inter=32), seed=0)
    be = Backend(max_rows=4)
    with pytest.raises(ValueError, match="invalid expert bank"):
        be.load_moe([], [], 2)
    with pytest.raises(ValueError, match="invalid expert bank"):
        be.load_moe(layer.gate, layer.down[:3], 2)
    with pytest.raises(ValueError, match="incompatible expert matrices"):
        be.load_moe(layer.gate, [layer.gate[0]] * 4, 2)
    w8 = S.make_layer(S.small_spec("c1", experts=4, hidden=64, inter=32, routed="w8pc"), seed=0)
    with pytest.raises(ValueError, match="one weight format"):
        be.load_moe(layer.gate[:2] + w8.gate[2:], layer.down, 2)
    with pytest.raises(ValueError, match="joint MoE requires"):
        shared = S.quantize_pc(np.ones((64, 2 * 48), np.float32), 8), \
            S.quantize_pc(np.ones((48, 64), np.float32), 8)
        be.load_moe_with_shared(layer.gate, layer.down, 2, shared, mode=L.SHARED_JOINT)
    with pytest.raises(ValueError):
        be.router(layer.router, 2, min_weight=1.5)


def test_synthetic_quantisation_ranges_and_determinism():
    spec = S.small_spec("c1", experts=2, hidden=64, inter=32)
    a, b = S.make_layer(spec, seed=5), S.make_layer(spec, seed=5)
    assert np.array_equal(a.gate[1].codes, b.gate[1].codes)
    g = a.gate[0]
    assert g.group == 32 and g.scales.dtype == np.float16 and g.scales.shape == (2, 64)
    assert g.codes.min() >= -8 and g.codes.max() <= 7
    w8 = S.quantize_pc(np.linspace(-1, 1, 64 * 8, dtype=np.float32).reshape(64, 8), 8)
    assert w8.codes.min() >= -127 and w8.codes.max() <= 127
    c3 = S.make_layer(S.small_spec("c3", experts=8, hidden=64, inter=32, shared_inter=64), seed=1)
    assert c3.bias is not None and c3.bias.max() == np.float32(2.0)
