"""Host-side mirror of the reference's MoE operator surface, over the C ABI.

Mirrors happyme531/open_rknpu2_lm_infer src/npu.rs (QuantMatrix, Backend) and
src/npu/moe.rs (Backend::load_moe*, Moe::run / run_profiled / max_rows):
same names, argument meaning and error behaviour (validation errors raise
ValueError like the reference's `ensure!`, native errors raise MoeError with
the library's strerror text like `check()`).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from ._lib import MoeError, check

__all__ = ["QuantMatrix", "Backend", "Moe", "Router", "Graph", "MoeError"]


@dataclass
class QuantMatrix:
    """QuantMatrix (src/npu.rs:135-157): codes int8 [k][n], f32 scales [n].

    `group` extends the reference format: with group > 0 the scales are fp16
    [k // group][n] (one per group of `group` consecutive k per channel).
    """
    bits: int
    k: int
    n: int
    codes: np.ndarray
    scales: np.ndarray
    group: int = 0

    def validate(self) -> None:
        """QuantMatrix::validate (src/npu.rs:142-157)."""
        if self.bits not in (4, 8):
            raise ValueError("linear weights must use 4 or 8 bits")
        if not (0 < self.k <= 2**31 - 1 and 0 < self.n <= 2**31 - 1):
            raise ValueError("invalid linear dimensions")
        codes = np.asarray(self.codes)
        if codes.dtype != np.int8 or codes.size != self.k * self.n:
            raise ValueError("linear weight shape mismatch")
        if self.group:
            if self.bits != 4 or self.group != 32 or self.k % 32:
                raise ValueError("group scales require W4 with group size 32")
            if np.asarray(self.scales).shape != (self.k // 32, self.n):
                raise ValueError("linear weight shape mismatch")
        elif np.asarray(self.scales).size != self.n:
            raise ValueError("linear weight shape mismatch")
        lo, hi = (-8, 7) if self.bits == 4 else (-128, 127)
        if codes.size and (codes.min() < lo or codes.max() > hi):
            raise ValueError("weight codes out of range for the bit width")

    @staticmethod
    def from_pack_quantized(packed: np.ndarray, scale: np.ndarray, bits: int, n: int,
                            k: int) -> "QuantMatrix":
        """compressed-tensors pack-quantized unpack (src/model/checkpoint.rs:537-571):
        packed I32 [n][ceil(k / (32/bits))], offset-binary codes (value + 2^(bits-1)),
        scale [n][1] positive; result codes are K-major [k][n]."""
        factor = 32 // bits
        cols = -(-k // factor)
        packed = np.asarray(packed)
        if packed.shape != (n, cols):
            raise ValueError("packed weight shape mismatch")
        scale = np.asarray(scale, dtype=np.float32)
        if scale.shape != (n, 1):
            raise ValueError("weight scale shape mismatch")
        if not np.all(scale > 0):
            raise ValueError("nonpositive weight scale")
        words = packed.astype(np.uint32)
        ki = np.arange(k)
        nib = (words[:, ki // factor] >> ((ki % factor) * bits).astype(np.uint32)) & ((1 << bits) - 1)
        codes = (nib.astype(np.int32) - (1 << (bits - 1))).astype(np.int8)  # [n][k]
        return QuantMatrix(bits, k, n, np.ascontiguousarray(codes.T), scale.reshape(n).copy())


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _format_of(m: QuantMatrix) -> int:
    if m.group:
        return L.W4_G32_FP16
    return L.W4_PER_CHANNEL if m.bits == 4 else L.W8_PER_CHANNEL


@dataclass
class _Handle:
    raw: int
    free: object

    def close(self):
        if self.raw:
            self.free(self.raw)
            self.raw = 0


class Backend:
    """The reference's `npu::Backend` (src/npu.rs) reduced to the MoE surface.

    Workspaces are shared by every bank of the same geometry key
    (src/npu/moe.rs:198-212)."""

    def __init__(self, device: int = 0, max_rows: int = 128):
        self.lib = L.load()
        self.device = device
        self.chunk = max_rows
        self._work: dict[tuple, _Handle] = {}
        self.weight_bytes = 0

    # ---- bank construction (src/npu/moe.rs:70-220) --------------------------
    def load_moe(self, gate: list[QuantMatrix], down: list[QuantMatrix], top: int,
                 exact: bool = True) -> "Moe":
        """exact=False: group-32 banks run the down GEMM on the fp16 tensor
        cores (MOE_B200_W4_G32_FP16_ROUNDED_DOWN: w * s rounded to fp16, no
        int32 down accumulators) instead of exact int32 group sums."""
        return self._load(gate, down, top, None, None, exact)

    def load_moe_with_shared(self, gate, down, top, shared: tuple[QuantMatrix, QuantMatrix],
                             mode: int | None = None) -> "Moe":
        return self._load(gate, down, top, shared, mode)

    def load_moe_full_k(self, gate, down, top) -> "Moe":
        # the full-K variant is the default schedule here
        return self._load(gate, down, top, None, None)

    def _load(self, gate, down, top, shared, mode, exact=True) -> "Moe":
        if not gate or len(gate) != len(down):
            raise ValueError("invalid expert bank")
        for m in [*gate, *down]:
            m.validate()
        fmts = {_format_of(m) for m in [*gate, *down]}
        if len(fmts) != 1:
            raise ValueError("grouped MoE requires one weight format for all routed experts")
        h, f, e = gate[0].k, gate[0].n // 2, len(gate)
        if not (all(g.k == h and g.n == 2 * f for g in gate)
                and all(d.k == f and d.n == h for d in down)):
            raise ValueError("incompatible expert matrices")
        shared_inter = 0
        if shared is not None:
            g, d = shared
            g.validate()
            d.validate()
            if g.group or d.group or g.bits != d.bits:
                raise ValueError("shared expert must use per-channel weights of one width")
            if not (g.k == h and g.n % 2 == 0 and d.k == g.n // 2 and d.n == h):
                raise ValueError("incompatible shared expert matrices")
            shared_inter = g.n // 2
            if mode is None:
                # joint bank when it fits (src/model/ling3tiny/moe.rs:240-246)
                mode = L.SHARED_JOINT if (shared_inter == f and g.bits == 8) else L.SHARED_DENSE
            if mode == L.SHARED_JOINT and (g.bits != 8 or shared_inter != f):
                raise ValueError(
                    "joint MoE requires a shared W8 expert with the routed intermediate width")
        cfg = self._config(h, f, e, shared is not None, top, shared_inter)
        keep = []  # host arrays referenced by the expert table during the call

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a

        def expert(g: QuantMatrix, d: QuantMatrix) -> L.Expert:
            ex = L.Expert()
            ex.gate_up = _ptr(arr(g.codes, np.int8))
            ex.down = _ptr(arr(d.codes, np.int8))
            if g.group:
                ex.gate_up_group_scales = _ptr(arr(np.asarray(g.scales, np.float16).view(np.uint16), np.uint16))
                ex.down_group_scales = _ptr(arr(np.asarray(d.scales, np.float16).view(np.uint16), np.uint16))
            else:
                ex.gate_up_scales = _ptr(arr(g.scales, np.float32))
                ex.down_scales = _ptr(arr(d.scales, np.float32))
            return ex

        table = (L.Expert * (e + (1 if shared is not None else 0)))()
        for i in range(e):
            table[i] = expert(gate[i], down[i])
        routed = fmts.pop()
        if not exact and routed == L.W4_G32_FP16:
            routed = L.W4_G32_FP16_ROUNDED_DOWN
        fmt = L.Format(routed, L.W8_PER_CHANNEL, L.SHARED_DENSE if mode is None else mode)
        if shared is not None:
            table[e] = expert(*shared)
            fmt.shared_format = L.W8_PER_CHANNEL if shared[0].bits == 8 else L.W4_PER_CHANNEL
        raw = self.lib.moe_b200_weights_create(C.byref(cfg), table, C.byref(fmt))
        if not raw:
            raise MoeError("cannot allocate packed MoE expert bank", L.ERR_NOMEM)
        weights = _Handle(raw, self.lib.moe_b200_weights_free)
        key = (h, f, e, top, shared is not None, shared_inter)
        if key not in self._work:
            ws = self.lib.moe_b200_workspace_create(C.byref(cfg))
            if not ws:
                weights.close()
                raise MoeError("cannot allocate grouped MoE workspace", L.ERR_NOMEM)
            self._work[key] = _Handle(ws, self.lib.moe_b200_workspace_free)
        self.weight_bytes += self.lib.moe_b200_weights_device_bytes(raw)
        return Moe(self, weights, key, cfg, routed)

    def moe_packed(self, h: int, f: int, slots: int, top: int,
                   fmt: int = L.W4_PER_CHANNEL) -> "Moe":
        """An empty bank of `slots` expert slots to import blobs into
        (Backend::moe_packed / moe_slots, src/npu/moe.rs:145-175)."""
        if not (h > 0 and f > 0 and 0 < top <= slots):
            raise ValueError("invalid MoE slot bank geometry")
        cfg = self._config(h, f, slots, False, top, 0)
        raw = self.lib.moe_b200_slots_create(C.byref(cfg), fmt)
        if not raw:
            raise MoeError("cannot allocate expert slot bank", L.ERR_NOMEM)
        weights = _Handle(raw, self.lib.moe_b200_weights_free)
        key = (h, f, slots, top, False, 0)
        if key not in self._work:
            ws = self.lib.moe_b200_workspace_create(C.byref(cfg))
            if not ws:
                weights.close()
                raise MoeError("cannot allocate grouped MoE workspace", L.ERR_NOMEM)
            self._work[key] = _Handle(ws, self.lib.moe_b200_workspace_free)
        self.weight_bytes += self.lib.moe_b200_weights_device_bytes(raw)
        return Moe(self, weights, key, cfg, fmt)

    def _config(self, h, f, e, shared, top, shared_inter) -> L.Config:
        cfg = L.Config()
        self.lib.moe_b200_config_init(C.byref(cfg), h, f, e, int(shared), top, self.chunk)
        cfg.weights.shared_intermediate = shared_inter
        cfg.device = self.device
        return cfg

    def router(self, weight: np.ndarray, top: int, bias: np.ndarray | None = None,
               order: int = L.ROUTER_NEON16, min_weight: float = 0.0, *,
               rule: int = L.ROUTE_SOFTMAX, groups: int = 1, top_groups: int = 1,
               routing_scale: float = 1.0, expert_bias: np.ndarray | None = None,
               shared_gate: np.ndarray | None = None) -> "Router":
        """Router over weight [experts][hidden] f32: Qwen's softmax top-k
        (src/model/qwen35/moe.rs:215-241), or with rule=ROUTE_GROUPED_SIGMOID
        Ling's grouped sigmoid routing (src/model/ling3tiny/moe.rs:146-223).
        shared_gate [hidden] gates the shared expert by sigmoid(gate . x)
        (src/model/qwen35/moe.rs:334-347)."""
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        e, h = weight.shape
        if not (np.isfinite(min_weight) and 0.0 <= min_weight <= 1.0):
            raise ValueError("expert minimum weight must be finite and between 0 and 1")
        if not (0 < top <= e):
            raise ValueError("invalid router top-k")
        if rule == L.ROUTE_GROUPED_SIGMOID:
            if not (groups > 0 and e % groups == 0 and e // groups >= 2 and
                    0 < top_groups <= groups and top <= top_groups * (e // groups) and
                    routing_scale > 0):
                raise ValueError("invalid Ling layer/router dimensions")
            if expert_bias is None:
                raise ValueError("grouped sigmoid routing needs the expert bias")
        cfg = self._config(h, 32, e, False, top, 0)
        keep = []

        def arr(a, n):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=np.float32)
            if a.size != n:
                raise ValueError("router vector has the wrong length")
            keep.append(a)
            return _ptr(a)

        opt = L.RouterOptions()
        self.lib.moe_b200_router_options_init(C.byref(opt))
        opt.order, opt.rule, opt.min_weight = order, rule, min_weight
        opt.bias = arr(bias, e)
        opt.groups, opt.top_groups, opt.routing_scale = groups, top_groups, routing_scale
        opt.expert_bias = arr(expert_bias, e)
        opt.shared_gate = arr(shared_gate, h)
        raw = self.lib.moe_b200_router_create_ex(C.byref(cfg), _ptr(weight), C.byref(opt))
        if not raw:
            raise MoeError("cannot create router", L.ERR_INVALID)
        return Router(_Handle(raw, self.lib.moe_b200_router_free), h, e, top,
                      shared_gate is not None)

    def router_for(self, layer, **kw) -> "Router":
        """The router a synthetic.Layer specifies (rule, order, biases, gate)."""
        spec = layer.spec
        return self.router(layer.router, spec.top, layer.bias, spec.router_order,
                           spec.min_weight, rule=spec.route_rule, groups=spec.groups,
                           top_groups=spec.top_groups, routing_scale=spec.routing_scale,
                           expert_bias=layer.expert_bias, shared_gate=layer.shared_gate, **kw)

    def close(self):
        for w in self._work.values():
            w.close()
        self._work.clear()


@dataclass
class Router:
    handle: _Handle
    hidden: int
    experts: int
    top: int
    gated: bool = False   # logits carry the shared-gate column (experts + 1 wide)

    @property
    def logit_columns(self) -> int:
        return self.experts + (1 if self.gated else 0)

    @property
    def raw(self):
        return self.handle.raw

    def close(self):
        self.handle.close()


@dataclass
class ImportBank:
    """A staging bank (npu::ImportBank): slots filled off the critical path,
    then swapped into a live bank with Moe.promote."""
    owner: "Backend"
    weights: "_Handle"
    slots: int

    def import_(self, slot: int, data) -> None:
        if not 0 <= slot < self.slots:
            raise ValueError("staging slot out of range")
        mv = memoryview(data).cast("B")
        buf = (C.c_uint8 * len(mv)).from_buffer_copy(mv)
        check(self.owner.lib.moe_b200_import_expert(self.weights.raw, slot, buf, len(mv)),
              "import staged expert")

    def weight_bytes(self) -> int:
        return self.owner.lib.moe_b200_weights_device_bytes(self.weights.raw)

    def close(self):
        self.weights.close()


class Moe:
    """npu::Moe (src/npu/moe.rs:10-14, 242-388)."""

    def __init__(self, owner: Backend, weights: _Handle, key: tuple, cfg: L.Config,
                 fmt: int = L.W4_PER_CHANNEL):
        self.owner = owner
        self.weights = weights
        self.key = key
        self.cfg = cfg
        self.fmt = fmt  # routed MOE_B200_W* format

    @property
    def workspace(self) -> int:
        return self.owner._work[self.key].raw

    @property
    def hidden(self) -> int:
        return self.key[0]

    @property
    def top(self) -> int:
        return self.key[3]

    def max_rows(self) -> int:
        return self.owner.lib.moe_b200_max_rows(self.workspace)

    # ---- slot bank (src/npu/moe.rs:243-320) ----
    @staticmethod
    def blob_version() -> int:
        return L.load().moe_b200_blob_version()

    def blob_bytes(self) -> int:
        return self.owner.lib.moe_b200_expert_blob_bytes(self.weights.raw)

    def export(self, expert: int) -> bytes:
        """The packed device image of one expert (Moe::export)."""
        if not 0 <= expert < self.key[2]:
            raise ValueError("expert index out of range")
        buf = (C.c_uint8 * self.blob_bytes())()
        check(self.owner.lib.moe_b200_export_expert(self.weights.raw, expert, buf, len(buf)),
              "export packed expert")
        return bytes(buf)

    def import_(self, slot: int, data) -> None:
        """Loads a blob into a slot (Moe::import)."""
        if not 0 <= slot < self.key[2]:
            raise ValueError("expert slot out of range")
        mv = memoryview(data).cast("B")
        buf = (C.c_uint8 * len(mv)).from_buffer_copy(mv) if mv.readonly else \
            (C.c_uint8 * len(mv)).from_buffer(mv)
        check(self.owner.lib.moe_b200_import_expert(self.weights.raw, slot, buf, len(mv)),
              "import packed expert")

    def import_device(self, slot: int, ptr: int, nbytes: int, stream: int = 0) -> None:
        """Stream-ordered import from host memory at `ptr` (page-locked for overlap)."""
        check(self.owner.lib.moe_b200_import_expert_async(self.weights.raw, slot, ptr, nbytes,
                                                          stream), "import packed expert")

    def import_bank(self, slots: int) -> "ImportBank":
        """A staging bank of the same geometry and format (Moe::import_bank)."""
        cfg = self.owner._config(self.key[0], self.key[1], slots, False, min(self.key[3], slots), 0)
        raw = self.owner.lib.moe_b200_slots_create(C.byref(cfg), self.fmt)
        if not raw:
            raise MoeError("cannot allocate expert staging bank", L.ERR_NOMEM)
        self.owner.weight_bytes += self.owner.lib.moe_b200_weights_device_bytes(raw)
        return ImportBank(self.owner, _Handle(raw, self.owner.lib.moe_b200_weights_free), slots)

    def promote(self, slot: int, bank: "ImportBank", staged: int, stream: int = 0) -> None:
        """Exchanges this bank's slot with a staged expert (Moe::promote)."""
        check(self.owner.lib.moe_b200_swap_slots(self.weights.raw, slot, bank.weights.raw, staged,
                                                 stream), "promote staged expert")

    def weight_bytes(self) -> int:
        return self.owner.lib.moe_b200_weights_device_bytes(self.weights.raw)

    def _shapes(self, inp, ids, routes, output, rows):
        h, top = self.hidden, self.top
        if not (inp.size == rows * h and output.size == rows * h and ids.size == rows * top
                and routes.size == ids.size):
            raise ValueError("grouped MoE input shape mismatch")

    def run(self, input: np.ndarray, ids: np.ndarray, routes: np.ndarray, output: np.ndarray,
            rows: int) -> None:
        """Moe::run (src/npu/moe.rs:324-333): host buffers, synchronous; output
        receives the weighted routed combine (+ shared expert)."""
        self._execute(input, ids, routes, output, rows, None)

    def run_profiled(self, input, ids, routes, output, rows) -> dict:
        """Moe::run_profiled (src/npu/moe.rs:334-352): same call, stage timings."""
        t = L.Timings()
        self._execute(input, ids, routes, output, rows, t)
        return t.as_dict()

    def _execute(self, inp, ids, routes, output, rows, timing):
        self._shapes(inp, ids, routes, output, rows)
        if output.dtype != np.float32 or not output.flags.c_contiguous:
            raise ValueError("output must be a contiguous float32 array")
        inp = np.ascontiguousarray(inp, dtype=np.float32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        routes = np.ascontiguousarray(routes, dtype=np.float32)
        rc = self.owner.lib.moe_b200_run_f32(self.workspace, self.weights.raw, rows, _ptr(inp),
                                             _ptr(ids), _ptr(routes), _ptr(output),
                                             None if timing is None else C.byref(timing))
        check(rc, "grouped routed FFN")

    def run_device(self, d_input: int, d_ids: int, d_routes: int, d_output: int, rows: int,
                   stream: int = 0) -> None:
        """Device pointers, asynchronous on `stream` (a cudaStream_t handle)."""
        rc = self.owner.lib.moe_b200_run_device(self.workspace, self.weights.raw, rows, d_input,
                                                d_ids, d_routes, d_output, stream)
        check(rc, "grouped routed FFN")

    def forward(self, router: Router, input: np.ndarray, residual: np.ndarray | None = None,
                timings: bool = False, out: np.ndarray | None = None,
                ids: np.ndarray | None = None, routes: np.ndarray | None = None):
        """Router-inclusive layer on host buffers: returns (output, ids, routes[, timings]).
        output = residual + (routed + shared) (src/model/qwen35/decoder.rs:215-217).
        out / ids / routes may be caller-owned (e.g. page-locked) arrays."""
        inp = np.ascontiguousarray(input, dtype=np.float32)
        rows = inp.size // self.hidden
        if inp.size != rows * self.hidden:
            raise ValueError("grouped MoE input shape mismatch")
        res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        if res is not None and res.size != inp.size:
            raise ValueError("residual shape mismatch")

        def own(a, shape, dt):
            if a is None:
                return np.empty(shape, dt)
            if a.dtype != dt or a.size != shape[0] * shape[1] or not a.flags.c_contiguous:
                raise ValueError("output buffer shape mismatch")
            return a
        out = own(out, (rows, self.hidden), np.float32)
        ids = own(ids, (rows, self.top), np.int32)
        routes = own(routes, (rows, self.top), np.float32)
        t = L.Timings() if timings else None
        rc = self.owner.lib.moe_b200_forward_f32(
            self.workspace, self.weights.raw, router.raw, rows, _ptr(inp), _ptr(res), _ptr(out),
            _ptr(ids), _ptr(routes), None if t is None else C.byref(t))
        check(rc, "MoE forward")
        return (out, ids, routes, t.as_dict()) if timings else (out, ids, routes)

    def forward_device(self, router: Router, rows: int, d_input: int, d_residual: int | None,
                       d_output: int, stream: int = 0) -> None:
        rc = self.owner.lib.moe_b200_forward_device(self.workspace, self.weights.raw, router.raw,
                                                    rows, d_input, d_residual, d_output, stream)
        check(rc, "MoE forward")

    def route_device(self, router: Router, rows: int, d_input: int, d_logits: int | None,
                     d_ids: int, d_routes: int, stream: int = 0) -> None:
        rc = self.owner.lib.moe_b200_route_device(self.workspace, router.raw, rows, d_input,
                                                  d_logits, d_ids, d_routes, stream)
        check(rc, "MoE router")

    def graph(self, router: Router, rows: int, d_input: int, d_residual: int | None,
              d_output: int) -> "Graph":
        """Captures forward_device over these device buffers into a CUDA graph."""
        raw = self.owner.lib.moe_b200_graph_create(self.workspace, self.weights.raw, router.raw,
                                                   rows, d_input, d_residual, d_output)
        if not raw:
            raise MoeError("cannot capture the MoE forward into a CUDA graph", L.ERR_CUDA)
        return Graph(_Handle(raw, self.owner.lib.moe_b200_graph_free), self.owner.lib)

    def status(self) -> None:
        check(self.owner.lib.moe_b200_workspace_status(self.workspace), "device status")

    def buffer(self, name: str) -> tuple[int, int]:
        p, n = C.c_void_p(), C.c_uint64()
        check(self.owner.lib.moe_b200_workspace_buffer(self.workspace, name.encode(), C.byref(p),
                                                       C.byref(n)), f"workspace buffer {name}")
        return p.value, n.value

    def debug_accumulators(self, which: int, d_acc: int, capacity: int, stream: int = 0) -> None:
        check(self.owner.lib.moe_b200_debug_accumulators(self.workspace, self.weights.raw, which,
                                                         d_acc, capacity, stream),
              "accumulator dump")

    def close(self):
        self.weights.close()


class Graph:
    """A captured router-inclusive forward (moe_b200_graph_*): one launch per replay."""

    def __init__(self, handle: _Handle, lib):
        self.handle = handle
        self.lib = lib

    def launch(self, stream: int = 0) -> None:
        check(self.lib.moe_b200_graph_launch(self.handle.raw, stream), "graph replay")

    def close(self):
        self.handle.close()
