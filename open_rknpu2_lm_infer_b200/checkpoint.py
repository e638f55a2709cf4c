"""Checkpoint ingest for the MoE bank: safetensors shards, compressed-tensors
W4/W8 per-channel layers and the C4 per-expert packed tensors, unpacked into
the reference's QuantMatrix layout (codes int8 [k][n], f32 scales [n]).

Restates src/model/checkpoint.rs (happyme531/open_rknpu2_lm_infer):
  Tensor / TensorStore           :18-230  (safetensors shards, index, dtypes, slices)
  QuantLoader::open / new        :284-384 (C4 manifest, compressed-tensors checks)
  matches / symmetric            :242-264 (scheme targets, per-channel W + per-token A8)
  QuantLoader::expert            :362-393 (gate|up concatenated per expert; C4 [E][n][cols])
  QuantLoader::bits / load       :420-530 (pack-quantized, int-quantized W8, zero points)
  unpack_codes / concatenate     :551-605

The safetensors container (an 8-byte little-endian header length, a JSON
header of {name: {dtype, shape, data_offsets}}, then the raw bytes) is read
with numpy memory maps; no safetensors package is needed. `write_safetensors`
and `pack_codes` are the inverse operations, for fixtures and tests.
"""
from __future__ import annotations

import json
import os
import re
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .moe import QuantMatrix

_DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2),
           "I8": (np.int8, 1), "I32": (np.int32, 4), "I64": (np.int64, 8)}
_FLOATING = ("F32", "F16", "BF16")
C4_FORMAT = "minicpmv47-c4-packed-v1"


class CheckpointError(ValueError):
    pass


def _ensure(cond, msg):
    if not cond:
        raise CheckpointError(msg)


@dataclass
class Tensor:
    """One tensor of a mapped shard (checkpoint.rs:18-116): raw bytes + dtype + shape."""
    raw: np.ndarray          # uint8 view of the tensor's bytes
    dtype: str
    shape: tuple

    def at(self, index: int) -> "Tensor":
        """The index-th slice along the first axis (checkpoint.rs:27-39)."""
        _ensure(len(self.shape) > 0 and 0 <= index < self.shape[0], "tensor slice out of range")
        step = self.raw.size // self.shape[0]
        return Tensor(self.raw[index * step:(index + 1) * step], self.dtype, self.shape[1:])

    def data(self) -> bytes:
        return self.raw.tobytes()

    def require_shape(self, shape, name: str) -> None:
        _ensure(tuple(self.shape) == tuple(shape),
                f"unexpected shape: {name}: {list(self.shape)}, expected {list(shape)}")

    def floating(self) -> bool:
        return self.dtype in _FLOATING

    def array(self) -> np.ndarray:
        """Typed view (BF16 as its uint16 bits)."""
        dt, _ = _DTYPES[self.dtype]
        return self.raw.view(dt).reshape(self.shape)

    def floats(self) -> np.ndarray:
        """f32 values, finite (checkpoint.rs:79-89)."""
        _ensure(self.floating(), "expected floating tensor")
        a = self.array()
        if self.dtype == "BF16":
            v = (a.astype(np.uint32) << 16).view(np.float32)
        else:
            v = a.astype(np.float32)
        v = np.ascontiguousarray(v).reshape(-1)
        _ensure(bool(np.isfinite(v).all()), "nonfinite model tensor")
        return v

    def integers(self) -> np.ndarray:
        _ensure(self.dtype in ("I8", "I32", "I64"), "expected integer tensor")
        return self.array().astype(np.int64).reshape(-1)


def _read_shard(path: Path):
    """(header dict, uint8 memmap of the data section) of one safetensors file."""
    _ensure(path.is_file(), f"cannot open shard {path}")
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    _ensure(mm.size >= 8, f"invalid safetensors shard {path}")
    (n,) = struct.unpack("<Q", bytes(mm[:8]))
    _ensure(8 + n <= mm.size, f"invalid safetensors shard {path}")
    try:
        header = json.loads(bytes(mm[8:8 + n]).decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise CheckpointError(f"invalid safetensors shard {path}") from e
    return header, mm[8 + n:]


class TensorStore:
    """Shards of one checkpoint directory (checkpoint.rs:118-230):
    model.safetensors.index.json (plain shard filenames, every indexed tensor
    present in its named shard) or a single model.safetensors."""

    def __init__(self):
        self.tensors: dict[str, Tensor] = {}
        self.files: list[Path] = []

    @classmethod
    def open(cls, directory) -> "TensorStore":
        directory = Path(directory)
        store = cls()
        index_path = directory / "model.safetensors.index.json"
        if index_path.exists():
            index = json.loads(index_path.read_bytes())
            weights = index.get("weight_map")
            _ensure(isinstance(weights, dict), "missing safetensors weight_map")
            shards = set()
            for value in weights.values():
                _ensure(isinstance(value, str), "invalid shard filename")
                p = Path(value)
                _ensure(len(p.parts) == 1 and p.parts[0] not in ("", ".", ".."),
                        "shard index requires plain filenames")
                shards.add(value)
            store.files.append(index_path)
            for shard in sorted(shards):
                store._add_file(directory / shard, weights)
            _ensure(len(store.tensors) == len(weights), "index has missing tensors")
        else:
            store._add_file(directory / "model.safetensors", None)
        return store

    def _add_file(self, path: Path, index: dict | None) -> None:
        header, data = _read_shard(path)
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            if index is not None:
                _ensure(index.get(name) == path.name, f"tensor/index mismatch: {name}")
            dtype = meta.get("dtype")
            _ensure(dtype in _DTYPES, f"unsupported safetensors dtype: {dtype}")
            shape = tuple(int(s) for s in meta["shape"])
            start, end = (int(o) for o in meta["data_offsets"])
            size = _DTYPES[dtype][1] * int(np.prod(shape, dtype=np.int64))
            _ensure(0 <= start <= end <= data.size and end - start == size,
                    f"invalid safetensors shard {path}")
            _ensure(name not in self.tensors, f"duplicate tensor: {name}")
            self.tensors[name] = Tensor(data[start:end], dtype, shape)
        self.files.append(path)

    def get(self, name: str) -> Tensor:
        t = self.tensors.get(name)
        _ensure(t is not None, f"missing tensor: {name}")
        return t

    def contains(self, name: str) -> bool:
        return name in self.tensors


def source_stamps(files) -> list[tuple[str, int, int]]:
    """(file name, bytes, mtime ns) of the files a loader consumed, sorted by
    name (SourceStamp, checkpoint.rs:124-129, 317-345): what an expert cache
    keys its validity on."""
    out = []
    for p in files:
        st = os.stat(p)
        out.append((Path(p).name, st.st_size, st.st_mtime_ns))
    return sorted(out)


def matches(target: str, module: str) -> bool:
    """Scheme target match (checkpoint.rs:242-250): "Linear", the exact module
    name, or "re:<pattern>" matching the whole name."""
    if target == "Linear" or target == module:
        return True
    if target.startswith("re:"):
        return re.fullmatch(f"(?:{target[3:]})", module) is not None
    return False


def _symmetric(q: dict, bits: int, strategy: str, dynamic: bool) -> None:
    """checkpoint.rs:251-264: symmetric int, the given strategy, no group
    scales, no activation order; `dynamic` absent means static."""
    q = q if isinstance(q, dict) else {}
    ok = (q.get("num_bits") == bits and q.get("type") == "int" and
          q.get("strategy") == strategy and q.get("symmetric") is True and
          (q["dynamic"] is dynamic if "dynamic" in q else not dynamic) and
          q.get("group_size") is None and q.get("actorder") is None)
    _ensure(ok, "expected symmetric static channel W4/W8 and dynamic token A8; "
                "unsupported group scales/actorder")


def unpack_codes(packed: Tensor, bits: int, n: int, k: int) -> np.ndarray:
    """Offset-binary codes packed little-end-first into I32 words [n][ceil(k /
    (32/bits))] -> int8 codes [k][n] (checkpoint.rs:551-564)."""
    factor = 32 // bits
    cols = -(-k // factor)
    packed.require_shape((n, cols), "packed weight")
    _ensure(packed.dtype == "I32", "packed weight must be I32")
    words = packed.array().view(np.uint32)
    ki = np.arange(k)
    vals = (words[:, ki // factor] >> ((ki % factor) * bits).astype(np.uint32)) & ((1 << bits) - 1)
    codes = (vals.astype(np.int32) - (1 << (bits - 1))).astype(np.int8)
    return np.ascontiguousarray(codes.T)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """The inverse of unpack_codes: codes [k][n] -> I32 words [n][cols]."""
    k, n = codes.shape
    factor = 32 // bits
    cols = -(-k // factor)
    off = (codes.astype(np.int32) + (1 << (bits - 1))).astype(np.uint32).T  # [n][k]
    pad = np.zeros((n, cols * factor), np.uint32)
    pad[:, :k] = off
    pad = pad.reshape(n, cols, factor)
    shifts = (np.arange(factor, dtype=np.uint32) * bits)
    words = np.bitwise_or.reduce(pad << shifts, axis=2).astype(np.uint32)
    return words.view(np.int32)


def concatenate(matrices: list[QuantMatrix]) -> QuantMatrix:
    """Fused projection (checkpoint.rs:573-605): columns of each matrix side
    by side (gate then up), same bits and K."""
    _ensure(len(matrices) > 0, "empty fused projection")
    if len(matrices) == 1:
        return matrices[0]
    bits, k = matrices[0].bits, matrices[0].k
    _ensure(all(m.bits == bits and m.k == k for m in matrices),
            "fused projections require identical bit widths and K")
    codes = np.concatenate([np.asarray(m.codes).reshape(k, m.n) for m in matrices], axis=1)
    scales = np.concatenate([np.asarray(m.scales, np.float32).reshape(-1) for m in matrices])
    return QuantMatrix(bits, k, codes.shape[1], np.ascontiguousarray(codes), scales)


class QuantLoader:
    """QuantLoader (checkpoint.rs:234-530)."""

    def __init__(self, store: TensorStore, quant, c4: dict | None, metadata_files):
        self.store = store
        self.quant = quant
        self.c4 = c4
        self.metadata_files = list(metadata_files)

    @classmethod
    def open(cls, directory, config: dict) -> "QuantLoader":
        directory = Path(directory)
        store = TensorStore.open(directory)
        if (config.get("c4_quantization") or {}).get("format") == C4_FORMAT:
            manifest = json.loads((directory / "bitwidth_manifest.json").read_bytes())
            _ensure(manifest.get("format") == C4_FORMAT, "C4 manifest format mismatch")
            bits = manifest.get("linear_bits")
            _ensure(isinstance(bits, dict), "C4 manifest format mismatch")
            bits = {str(k): int(v) for k, v in bits.items()}
            _ensure(all(b in (4, 8) for b in bits.values()), "unsupported C4 weight precision")
            for name, t in store.tensors.items():
                if name.endswith(".input_scale"):
                    _ensure(bool((t.floats() == 1.0).all()),
                            f"non-unit input_scale is unsupported: {name}")
            return cls(store, None, bits,
                       [directory / "config.json", directory / "bitwidth_manifest.json"])
        loader = cls.new(store, config)
        loader.metadata_files.append(directory / "config.json")
        return loader

    @classmethod
    def new(cls, store: TensorStore, config: dict) -> "QuantLoader":
        quant = config.get("quantization_config") or {}
        _ensure(quant.get("quant_method") == "compressed-tensors" and
                quant.get("quantization_status") == "compressed",
                "expected a compressed-tensors compressed checkpoint")
        for key in ("sparsity_config", "transform_config"):
            v = quant.get(key)
            _ensure(v is None or v == {}, f"unsupported compressed-tensors {key}")
        _ensure(quant.get("kv_cache_scheme") is None,
                "quantized KV cache schemes are unsupported")
        _ensure(isinstance(quant.get("config_groups"), dict),
                "missing quantization config_groups")
        return cls(store, quant, None, [])

    def is_c4(self) -> bool:
        return self.c4 is not None

    def source_stamps(self):
        return source_stamps(list(self.store.files) + self.metadata_files)

    def quantized(self, module: str) -> bool:
        if self.c4 is not None:
            return module in self.c4
        if self.store.contains(f"{module}.weight_packed"):
            return True
        t = self.store.tensors.get(f"{module}.weight")
        return t is not None and not t.floating()

    def _scheme(self, module: str) -> dict:
        for target in self.quant.get("ignore") or []:
            _ensure(isinstance(target, str), "invalid ignore target")
            _ensure(not matches(target, module),
                    f"required projection excluded from quantization: {module}")
        found = None
        for value in self.quant["config_groups"].values():
            targets = value.get("targets") if isinstance(value, dict) else None
            _ensure(isinstance(targets, list), "missing quantization targets")
            for target in targets:
                _ensure(isinstance(target, str), "invalid quantization target")
                if matches(target, module):
                    _ensure(found is None or found == value,
                            f"ambiguous quantization scheme: {module}")
                    found = value
        _ensure(found is not None, f"no quantization scheme for {module}")
        return found

    def bits(self, module: str) -> int:
        if self.c4 is not None:
            _ensure(module in self.c4, f"unquantized C4 module: {module}")
            return self.c4[module]
        s = self._scheme(module)
        bits = (s.get("weights") or {}).get("num_bits")
        _ensure(isinstance(bits, int), "missing weight bits")
        _ensure(bits in (4, 8), "only W4A8 and W8A8 are supported")
        _symmetric(s.get("weights"), bits, "channel", False)
        _symmetric(s.get("input_activations"), 8, "token", True)
        _ensure(s.get("output_activations") is None,
                f"quantized linear output is unsupported: {module}")
        return bits

    def load(self, module: str, n: int, k: int) -> QuantMatrix:
        """One W4/W8 per-channel linear [n][k] as a QuantMatrix (checkpoint.rs:451-530)."""
        _ensure(n > 0 and k > 0, "invalid linear dimensions")
        bits = self.bits(module)
        _ensure(not self.store.contains(f"{module}.bias"), f"linear bias is unsupported: {module}")
        _ensure(not self.store.contains(f"{module}.weight_g_idx"),
                f"weight_g_idx/actorder unsupported: {module}")
        scale = self.store.get(f"{module}.weight_scale")
        scale.require_shape((n, 1), "weight_scale")
        scales = scale.floats()
        _ensure(bool((scales > 0).all()), f"nonpositive scale: {module}")
        if self.store.contains(f"{module}.weight_zero_point"):
            zero = self.store.get(f"{module}.weight_zero_point")
            _ensure(bool((zero.integers() == 0).all()), f"nonzero weight zero point: {module}")
        if self.is_c4():
            fmt = "pack-quantized"
        else:
            # the scheme's "format" key wins when present, even as null
            scheme = self._scheme(module)
            fv = scheme["format"] if "format" in scheme else self.quant.get("format")
            fmt = fv if isinstance(fv, str) else ""
        if fmt == "pack-quantized":
            packed = self.store.get(f"{module}.weight_packed")
            shape = self.store.get(f"{module}.weight_shape")
            shape.require_shape((2,), "weight_shape")
            sv = shape.integers()
            _ensure(int(sv[0]) == n and int(sv[1]) == k, f"weight_shape mismatch: {module}")
            codes = unpack_codes(packed, bits, n, k)
        elif fmt == "int-quantized" and bits == 8:
            w = self.store.get(f"{module}.weight")
            w.require_shape((n, k), "weight")
            _ensure(w.dtype == "I8", "W8 weight must be signed I8")
            codes = np.ascontiguousarray(w.array().T)
        else:
            raise CheckpointError(f"unsupported compressed-tensors storage: {fmt}")
        return QuantMatrix(bits, k, n, codes, scales.astype(np.float32))

    def expert(self, module: str, expert: int, h: int, f: int) -> tuple[QuantMatrix, QuantMatrix]:
        """One routed expert as (gate|up [h][2f], down [f][h]) (checkpoint.rs:362-393).
        compressed-tensors: {module}.{e}.{gate,up,down}_proj; C4: W4 tensors
        {module}.gate_up_proj_packed / _scale and down_proj_packed / _scale with
        a leading expert axis."""
        if not self.is_c4():
            name = f"{module}.{expert}"
            return (concatenate([self.load(f"{name}.gate_proj", f, h),
                                 self.load(f"{name}.up_proj", f, h)]),
                    self.load(f"{name}.down_proj", h, f))

        def matrix(name, n, k):
            packed = self.store.get(f"{module}.{name}_packed").at(expert)
            scale = self.store.get(f"{module}.{name}_scale").at(expert)
            scale.require_shape((n, 1), "weight scale")
            scales = scale.floats()
            _ensure(bool((scales > 0).all()), "nonpositive weight scale")
            return QuantMatrix(4, k, n, unpack_codes(packed, 4, n, k), scales.astype(np.float32))

        return matrix("gate_up_proj", 2 * f, h), matrix("down_proj", h, f)

    def experts(self, module: str, count: int, h: int, f: int):
        """Every routed expert of a layer: ([gate|up], [down])."""
        pairs = [self.expert(module, e, h, f) for e in range(count)]
        return [p[0] for p in pairs], [p[1] for p in pairs]


# ---- writing (fixtures and tests) -------------------------------------------------

def _dtype_name(a: np.ndarray, bf16: bool) -> str:
    if bf16:
        return "BF16"
    return {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int8): "I8",
            np.dtype(np.int32): "I32", np.dtype(np.int64): "I64"}[a.dtype]


def write_safetensors(path, tensors: dict, bf16: tuple = ()) -> None:
    """Writes a safetensors file; names listed in `bf16` hold uint16 bf16 bits."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": _dtype_name(a, name in bf16), "shape": list(a.shape),
                        "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)


def compressed_tensors_config(bits: int, targets=("Linear",), fmt="pack-quantized") -> dict:
    """A compressed-tensors quantization_config of the accepted kind."""
    return {"quantization_config": {
        "quant_method": "compressed-tensors", "quantization_status": "compressed",
        "format": fmt,
        "config_groups": {"group_0": {
            "targets": list(targets),
            "weights": {"num_bits": bits, "type": "int", "strategy": "channel",
                        "symmetric": True, "dynamic": False},
            "input_activations": {"num_bits": 8, "type": "int", "strategy": "token",
                                  "symmetric": True, "dynamic": True}}}}}


def linear_tensors(module: str, m: QuantMatrix, fmt: str = "pack-quantized") -> dict:
    """The compressed-tensors tensors of one per-channel linear ([n][k] storage)."""
    out = {f"{module}.weight_scale": np.asarray(m.scales, np.float32).reshape(m.n, 1)}
    codes = np.asarray(m.codes).reshape(m.k, m.n)
    if fmt == "pack-quantized":
        out[f"{module}.weight_packed"] = pack_codes(codes, m.bits)
        out[f"{module}.weight_shape"] = np.array([m.n, m.k], np.int64)
    else:
        out[f"{module}.weight"] = np.ascontiguousarray(codes.T).astype(np.int8)
    return out
