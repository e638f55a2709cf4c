"""Checkpoint ingest (open_rknpu2_lm_infer_b200.checkpoint) on CPU.

Ports the reference's own tests of src/model/checkpoint.rs:606-735
(source_stamps_follow_loaded_files_and_invalidate_changed_sources,
c4_metadata_uses_existing_packed_weight_math) and adds round trips of
synthetic expert banks through both storage forms, plus the loader's
rejections (checkpoint.rs:284-530).
"""
import json
import os

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import checkpoint as CK
from open_rknpu2_lm_infer_b200 import synthetic as S

CT = {"quantization_config": {"quant_method": "compressed-tensors",
                              "quantization_status": "compressed", "config_groups": {}}}


def _write(path, obj):
    path.write_bytes(json.dumps(obj).encode())


def test_source_stamps_follow_loaded_files(tmp_path):
    _write(tmp_path / "config.json", CT)
    CK.write_safetensors(tmp_path / "model.safetensors",
                         {"a": np.array([1.0], np.float32), "b": np.array([2.0], np.float32)})
    loader = CK.QuantLoader.open(tmp_path, CT)
    assert loader.store.contains("a") and loader.store.contains("b")
    assert [s[0] for s in loader.source_stamps()] == ["config.json", "model.safetensors"]
    single = loader.source_stamps()
    (tmp_path / "config.json").write_bytes(b'{"changed":true}')
    os.utime(tmp_path / "config.json", ns=(1, 1))
    assert loader.source_stamps() != single
    # an index over a renamed shard; an unrelated manifest is not a dependency
    (tmp_path / "part.safetensors").write_bytes((tmp_path / "model.safetensors").read_bytes())
    _write(tmp_path / "model.safetensors.index.json",
           {"weight_map": {"a": "part.safetensors", "b": "part.safetensors"}})
    (tmp_path / "bitwidth_manifest.json").write_bytes(b"{}")
    indexed = CK.QuantLoader.open(tmp_path, CT)
    assert indexed.store.contains("a") and indexed.store.contains("b")
    stamps = indexed.source_stamps()
    assert [s[0] for s in stamps] == ["config.json", "model.safetensors.index.json",
                                      "part.safetensors"]
    (tmp_path / "model.safetensors.index.json").write_bytes(b"changed")
    os.utime(tmp_path / "model.safetensors.index.json", ns=(2, 2))
    assert indexed.source_stamps() != stamps
    assert float(indexed.store.get("b").floats()[0]) == 2.0


def _c4_fixture(d):
    CK.write_safetensors(d / "model.safetensors", {
        "q.weight_packed": np.array([[0x87654321], [0xFEDCBA98]], np.uint32).view(np.int32),
        "q.weight_scale": np.array([[0.25], [0.5]], np.float32),
        "q.weight_shape": np.array([2, 8], np.int64),
        "q.input_scale": np.ones(8, np.float32),
        "fp.weight": np.full((2, 8), 0.25, np.float32),
    })
    (d / "bitwidth_manifest.json").write_bytes(
        b'{"format":"minicpmv47-c4-packed-v1","linear_bits":{"q":4}}')
    (d / "config.json").write_bytes(b'{"c4_quantization":{"format":"minicpmv47-c4-packed-v1"}}')


def test_c4_metadata_uses_existing_packed_weight_math(tmp_path):
    _c4_fixture(tmp_path)
    c4 = CK.QuantLoader.open(tmp_path, {"c4_quantization": {"format": CK.C4_FORMAT}})
    old = CK.QuantLoader.new(CK.TensorStore.open(tmp_path), {"quantization_config": {
        "quant_method": "compressed-tensors", "quantization_status": "compressed",
        "format": "pack-quantized",
        "config_groups": {"g": {"targets": ["q"],
                                "weights": {"num_bits": 4, "type": "int", "strategy": "channel",
                                            "symmetric": True},
                                "input_activations": {"num_bits": 8, "type": "int",
                                                      "strategy": "token", "symmetric": True,
                                                      "dynamic": True}}}}})
    actual = c4.load("q", 2, 8)
    assert [s[0] for s in c4.source_stamps()] == ["bitwidth_manifest.json", "config.json",
                                                   "model.safetensors"]
    baseline = old.load("q", 2, 8)
    assert actual.codes.reshape(-1).tolist() == [-7, 0, -6, 1, -5, 2, -4, 3, -3, 4, -2, 5, -1,
                                                 6, 0, 7]
    assert np.array_equal(actual.codes, baseline.codes)
    assert actual.scales.tolist() == [0.25, 0.5]
    row = c4.store.get("q.weight_packed").at(1)
    assert row.shape == (1,)
    assert row.data() == (0xFEDCBA98).to_bytes(4, "little")
    assert c4.quantized("q") and not c4.quantized("fp")
    with pytest.raises(CK.CheckpointError):
        c4.bits("fp")


def test_c4_rejects_non_unit_input_scale(tmp_path):
    _c4_fixture(tmp_path)
    t = CK.TensorStore.open(tmp_path).tensors
    arrays = {n: v.array() for n, v in t.items()}
    arrays["q.input_scale"] = np.full(8, 0.5, np.float32)
    CK.write_safetensors(tmp_path / "model.safetensors", arrays)
    with pytest.raises(CK.CheckpointError, match="input_scale"):
        CK.QuantLoader.open(tmp_path, {"c4_quantization": {"format": CK.C4_FORMAT}})


@pytest.mark.parametrize("routed,fmt", [("w4pc", "pack-quantized"), ("w8pc", "pack-quantized"),
                                        ("w8pc", "int-quantized")])
def test_expert_bank_round_trip(tmp_path, routed, fmt):
    spec = S.small_spec("c1", hidden=256, inter=128, experts=4, top=2, routed=routed)
    layer = S.make_layer(spec, seed=7)
    bits = 4 if routed == "w4pc" else 8
    H, I = spec.hidden, spec.inter
    tensors = {}
    prefix = "model.layers.3.mlp.experts"
    for e in range(spec.experts):
        g = layer.gate[e]
        codes = np.asarray(g.codes).reshape(H, 2 * I)
        sc = np.asarray(g.scales, np.float32)
        from open_rknpu2_lm_infer_b200.moe import QuantMatrix
        gate = QuantMatrix(bits, H, I, np.ascontiguousarray(codes[:, :I]), sc[:I])
        up = QuantMatrix(bits, H, I, np.ascontiguousarray(codes[:, I:]), sc[I:])
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.gate_proj", gate, fmt))
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.up_proj", up, fmt))
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.down_proj", layer.down[e], fmt))
    # two shards behind an index
    names = sorted(tensors)
    half = len(names) // 2
    CK.write_safetensors(tmp_path / "a.safetensors", {n: tensors[n] for n in names[:half]})
    CK.write_safetensors(tmp_path / "b.safetensors", {n: tensors[n] for n in names[half:]})
    _write(tmp_path / "model.safetensors.index.json",
           {"weight_map": {n: ("a" if i < half else "b") + ".safetensors"
                           for i, n in enumerate(names)}})
    cfg = CK.compressed_tensors_config(bits, targets=(r"re:.*experts\.\d+\.(gate|up|down)_proj",),
                                       fmt=fmt)
    loader = CK.QuantLoader.open(tmp_path, cfg)
    gates, downs = loader.experts(prefix, spec.experts, H, I)
    for e in range(spec.experts):
        for got, ref in ((gates[e], layer.gate[e]), (downs[e], layer.down[e])):
            got.validate()
            assert (got.bits, got.k, got.n) == (ref.bits, ref.k, ref.n)
            assert np.array_equal(got.codes.reshape(-1), np.asarray(ref.codes).reshape(-1))
            assert np.array_equal(got.scales, np.asarray(ref.scales, np.float32))


def test_c4_expert_tensors_round_trip(tmp_path):
    spec = S.small_spec("c1", hidden=256, inter=128, experts=3, top=2, routed="w4pc")
    layer = S.make_layer(spec, seed=8)
    H, I, E = spec.hidden, spec.inter, spec.experts
    mod = "model.layers.0.mlp.experts"
    t = {
        f"{mod}.gate_up_proj_packed": np.stack([CK.pack_codes(np.asarray(g.codes).reshape(H, 2 * I), 4)
                                                for g in layer.gate]),
        f"{mod}.gate_up_proj_scale": np.stack([np.asarray(g.scales, np.float32).reshape(-1, 1)
                                               for g in layer.gate]),
        f"{mod}.down_proj_packed": np.stack([CK.pack_codes(np.asarray(d.codes).reshape(I, H), 4)
                                             for d in layer.down]),
        f"{mod}.down_proj_scale": np.stack([np.asarray(d.scales, np.float32).reshape(-1, 1)
                                            for d in layer.down]),
    }
    CK.write_safetensors(tmp_path / "model.safetensors", t)
    (tmp_path / "bitwidth_manifest.json").write_bytes(
        json.dumps({"format": CK.C4_FORMAT, "linear_bits": {}}).encode())
    loader = CK.QuantLoader.open(tmp_path, {"c4_quantization": {"format": CK.C4_FORMAT}})
    gates, downs = loader.experts(mod, E, H, I)
    for e in range(E):
        assert np.array_equal(gates[e].codes.reshape(-1), np.asarray(layer.gate[e].codes).reshape(-1))
        assert np.array_equal(downs[e].scales, np.asarray(layer.down[e].scales, np.float32))


def test_pack_codes_inverts_unpack_for_ragged_k():
    rng = np.random.default_rng(3)
    for bits, lo, hi in ((4, -8, 8), (8, -128, 128)):
        for k in (1, 7, 9, 64, 67):
            codes = rng.integers(lo, hi, size=(k, 5)).astype(np.int8)
            words = CK.pack_codes(codes, bits)
            t = CK.Tensor(words.view(np.uint8).reshape(-1), "I32", words.shape)
            assert np.array_equal(CK.unpack_codes(t, bits, 5, k), codes)


def _one_linear(tmp_path, extra=None, scheme_patch=None, scale=None, quant_patch=None):
    from open_rknpu2_lm_infer_b200.moe import QuantMatrix
    m = QuantMatrix(4, 16, 2, np.arange(32, dtype=np.int8).reshape(16, 2) % 8,
                    np.array([0.5, 0.25], np.float32))
    t = CK.linear_tensors("q", m)
    if scale is not None:
        t["q.weight_scale"] = scale
    t.update(extra or {})
    CK.write_safetensors(tmp_path / "model.safetensors", t)
    cfg = CK.compressed_tensors_config(4, targets=("q",))
    g = cfg["quantization_config"]["config_groups"]["group_0"]
    for k, v in (scheme_patch or {}).items():
        g["weights"][k] = v
    cfg["quantization_config"].update(quant_patch or {})
    return CK.QuantLoader.open(tmp_path, cfg)


@pytest.mark.parametrize("case", ["ok", "bias", "g_idx", "zero_point", "zero_point_ok",
                                  "nonpositive_scale", "group_size", "actorder", "asymmetric",
                                  "ignored", "no_scheme", "shape", "sparsity", "kv_cache"])
def test_loader_rejections(tmp_path, case):
    kw = {}
    if case == "bias":
        kw["extra"] = {"q.bias": np.zeros(2, np.float32)}
    elif case == "g_idx":
        kw["extra"] = {"q.weight_g_idx": np.zeros(16, np.int32)}
    elif case == "zero_point":
        kw["extra"] = {"q.weight_zero_point": np.array([[0], [1]], np.int32)}
    elif case == "zero_point_ok":
        kw["extra"] = {"q.weight_zero_point": np.zeros((2, 1), np.int32)}
    elif case == "nonpositive_scale":
        kw["scale"] = np.array([[0.5], [0.0]], np.float32)
    elif case == "group_size":
        kw["scheme_patch"] = {"group_size": 32}
    elif case == "actorder":
        kw["scheme_patch"] = {"actorder": "group"}
    elif case == "asymmetric":
        kw["scheme_patch"] = {"symmetric": False}
    elif case == "ignored":
        kw["quant_patch"] = {"ignore": ["re:q"]}
    elif case == "shape":
        kw["extra"] = {"q.weight_shape": np.array([2, 17], np.int64)}
    elif case == "sparsity":
        kw["quant_patch"] = {"sparsity_config": {"format": "dense"}}
    elif case == "kv_cache":
        kw["quant_patch"] = {"kv_cache_scheme": {"num_bits": 8}}
    if case in ("sparsity", "kv_cache"):
        with pytest.raises(CK.CheckpointError):
            _one_linear(tmp_path, **kw)
        return
    loader = _one_linear(tmp_path, **kw)
    module = "r" if case == "no_scheme" else "q"
    if case in ("ok", "zero_point_ok"):
        m = loader.load("q", 2, 16)
        m.validate()
        assert m.scales.tolist() == [0.5, 0.25]
        return
    with pytest.raises(CK.CheckpointError):
        loader.load(module, 2, 16)


def test_store_rejections(tmp_path):
    # tensor listed in the index under another shard
    CK.write_safetensors(tmp_path / "s1.safetensors", {"a": np.zeros(1, np.float32)})
    _write(tmp_path / "model.safetensors.index.json", {"weight_map": {"a": "s2.safetensors"}})
    with pytest.raises(CK.CheckpointError):
        CK.TensorStore.open(tmp_path)
    _write(tmp_path / "model.safetensors.index.json", {"weight_map": {"a": "../s1.safetensors"}})
    with pytest.raises(CK.CheckpointError, match="plain filenames"):
        CK.TensorStore.open(tmp_path)
    _write(tmp_path / "model.safetensors.index.json",
           {"weight_map": {"a": "s1.safetensors", "b": "s1.safetensors"}})
    with pytest.raises(CK.CheckpointError, match="missing"):
        CK.TensorStore.open(tmp_path)
    (tmp_path / "model.safetensors.index.json").unlink()
    # unsupported dtype
    header = json.dumps({"u": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}}).encode()
    header += b" " * (-len(header) % 8)
    (tmp_path / "model.safetensors").write_bytes(
        len(header).to_bytes(8, "little") + header + b"\x00")
    with pytest.raises(CK.CheckpointError, match="dtype"):
        CK.TensorStore.open(tmp_path)


def test_bf16_and_f16_floats(tmp_path):
    v = np.array([1.5, -2.25, 3.0e-3], np.float32)
    bf = (v.view(np.uint32) >> 16).astype(np.uint16)
    CK.write_safetensors(tmp_path / "model.safetensors",
                         {"b": bf, "h": v.astype(np.float16), "f": v}, bf16=("b",))
    st = CK.TensorStore.open(tmp_path)
    assert st.get("b").dtype == "BF16"
    assert np.array_equal(st.get("b").floats(), (bf.astype(np.uint32) << 16).view(np.float32))
    assert np.array_equal(st.get("h").floats(), v.astype(np.float16).astype(np.float32))
    assert np.array_equal(st.get("f").floats(), v)
    with pytest.raises(CK.CheckpointError):
        st.get("missing")


def test_scheme_target_matching():
    assert CK.matches("Linear", "anything")
    assert CK.matches("model.q", "model.q")
    assert CK.matches(r"re:.*\.q_proj", "model.layers.0.q_proj")
    assert not CK.matches(r"re:q", "model.q")  # whole-name match
    assert not CK.matches("q", "model.q")
