"""ctypes wrapper of the CPU restatement (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; it is the checker and the reported CPU baseline, never the
product path. The C sources cite the reference file:line of every stage.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmoe_oracle.so"

ROUTER_NEON16, ROUTER_SEQUENTIAL, ROUTER_TF32 = 0, 1, 2
ROUTE_SOFTMAX, ROUTE_GROUPED_SIGMOID = 0, 1
QUANT_MOE, QUANT_DENSE = 0, 1
SHARED_JOINT, SHARED_DENSE = 0, 1


class QMat(C.Structure):
    _fields_ = [("bits", C.c_int), ("k", C.c_int), ("n", C.c_int), ("group", C.c_int),
                ("codes", C.c_void_p), ("scales", C.c_void_p), ("gscales", C.c_void_p)]


class LayerS(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("experts", C.c_int), ("top", C.c_int),
                ("shared_inter", C.c_int), ("shared_mode", C.c_int), ("router_order", C.c_int),
                ("min_weight", C.c_float), ("router", C.c_void_p), ("router_bias", C.c_void_p),
                ("gate_up", C.POINTER(QMat)), ("down", C.POINTER(QMat)),
                ("shared_gate_up", C.POINTER(QMat)), ("shared_down", C.POINTER(QMat)),
                ("route_rule", C.c_int), ("groups", C.c_int), ("top_groups", C.c_int),
                ("routing_scale", C.c_float), ("expert_bias", C.c_void_p),
                ("shared_gate", C.c_void_p)]


class Dump(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "logits", "ids", "weights", "perm", "offsets", "qx", "sx", "middle", "qm", "sm", "y",
        "routed", "shared")] + [("n_assign", C.c_int32), ("shared_scale", C.c_void_p)]


_lib = None


def build() -> Path:
    """Compiles the restatement with oracle/Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.oracle_total_key.restype = C.c_int32
        L.oracle_total_key.argtypes = [C.c_float]
        L.oracle_router_logits.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, P]
        L.oracle_routes.restype = C.c_int
        L.oracle_routes.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_float, P, P]
        L.oracle_ling_routes.restype = C.c_int
        L.oracle_ling_routes.argtypes = [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, P, P]
        L.oracle_sigmoid.restype = C.c_float
        L.oracle_sigmoid.argtypes = [C.c_float]
        L.oracle_permute.restype = C.c_int
        L.oracle_permute.argtypes = [P, P, C.c_int, C.c_int, C.c_int, P, P]
        L.oracle_quantize.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P]
        L.oracle_gemm_acc.argtypes = [P, C.c_int, C.POINTER(QMat), P]
        L.oracle_gemm_dequant.argtypes = [P, P, C.c_int, C.POINTER(QMat), P]
        L.oracle_swiglu.argtypes = [P, C.c_int, C.c_int, P]
        L.oracle_rms_norm.argtypes = [P, P, C.c_int, C.c_int, C.c_float, C.c_int, P]
        L.oracle_moe_run.restype = C.c_int
        L.oracle_moe_run.argtypes = [C.POINTER(LayerS), C.c_int, P, P, P, P, C.POINTER(Dump)]
        L.oracle_moe_forward.restype = C.c_int
        L.oracle_moe_forward.argtypes = [C.POINTER(LayerS), C.c_int, P, P, P, C.POINTER(Dump)]
        L.oracle_half_to_float.restype = C.c_float
        L.oracle_half_to_float.argtypes = [C.c_uint16]
        L.oracle_float_to_half.restype = C.c_uint16
        L.oracle_float_to_half.argtypes = [C.c_float]
        L.oracle_threads.restype = C.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def total_key(v: float) -> int:
    return lib().oracle_total_key(v)


def router_logits(x, router, bias=None, order=ROUTER_NEON16):
    x, router = _c(x, np.float32), _c(router, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    T, H = x.shape
    E = router.shape[0]
    out = np.empty((T, E), np.float32)
    lib().oracle_router_logits(_p(x), _p(router), _p(b), T, H, E, order, _p(out))
    return out


def routes(logits, k, min_weight=0.0):
    logits = _c(np.atleast_2d(logits), np.float32)
    T, E = logits.shape
    ids = np.empty((T, max(k, 1)), np.int32)
    w = np.empty((T, max(k, 1)), np.float32)
    rc = lib().oracle_routes(_p(logits), T, E, k, min_weight, _p(ids), _p(w))
    if rc != 0:
        raise ValueError("invalid router top-k")
    return ids, w


def ling_routes(logits, bias, groups, top_groups, k, routing_scale):
    """Ling's grouped sigmoid routing (src/model/ling3tiny/moe.rs:146-223)."""
    logits = _c(np.atleast_2d(logits), np.float32)
    bias = _c(bias, np.float32)
    T, E = logits.shape
    ids = np.empty((T, max(k, 1)), np.int32)
    w = np.empty((T, max(k, 1)), np.float32)
    rc = lib().oracle_ling_routes(_p(logits), _p(bias), T, E, groups, top_groups, k,
                                  routing_scale, _p(ids), _p(w))
    if rc != 0:
        raise ValueError("invalid grouped routing geometry")
    return ids, w


def sigmoid(x: float) -> float:
    return lib().oracle_sigmoid(x)


def permute(ids, weights, E):
    ids, weights = _c(ids, np.int32), _c(weights, np.float32)
    T, k = ids.shape
    perm = np.empty(T * k, np.int32)
    off = np.empty(E + 1, np.int32)
    n = lib().oracle_permute(_p(ids), _p(weights), T, k, E, _p(perm), _p(off))
    if n < 0:
        raise ValueError("expert id out of range")
    return perm[:n], off


def quantize(x, rule=QUANT_MOE):
    x = _c(np.atleast_2d(x), np.float32)
    R, Ccols = x.shape
    q = np.empty((R, Ccols), np.int8)
    s = np.empty(R, np.float32)
    lib().oracle_quantize(_p(x), R, Ccols, rule, _p(q), _p(s))
    return q, s


class _Mat:
    """Keeps a QuantMatrix's arrays alive next to its ctypes view."""

    def __init__(self, m):
        self.codes = _c(m.codes, np.int8)
        self.group = int(getattr(m, "group", 0) or 0)
        if self.group:
            self.sc = _c(np.asarray(m.scales, np.float16).view(np.uint16), np.uint16)
            self.s = QMat(m.bits, m.k, m.n, self.group, _p(self.codes), None, _p(self.sc))
        else:
            self.sc = _c(m.scales, np.float32)
            self.s = QMat(m.bits, m.k, m.n, 0, _p(self.codes), _p(self.sc), None)


def gemm_acc(q, m):
    """Integer accumulators: per-channel [rows][n]; grouped [rows][k/group][n]."""
    q = _c(np.atleast_2d(q), np.int8)
    mm = _Mat(m)
    G = m.k // mm.group if mm.group else 1
    acc = np.empty((q.shape[0], G, m.n), np.int32)
    lib().oracle_gemm_acc(_p(q), q.shape[0], C.byref(mm.s), _p(acc))
    return acc if mm.group else acc[:, 0, :]


def gemm_dequant(q, s, m):
    q, s = _c(np.atleast_2d(q), np.int8), _c(s, np.float32)
    mm = _Mat(m)
    out = np.empty((q.shape[0], m.n), np.float32)
    lib().oracle_gemm_dequant(_p(q), _p(s), q.shape[0], C.byref(mm.s), _p(out))
    return out


def swiglu(gu, width):
    gu = _c(np.atleast_2d(gu), np.float32)
    out = np.empty((gu.shape[0], width), np.float32)
    lib().oracle_swiglu(_p(gu), gu.shape[0], width, _p(out))
    return out


def rms_norm(x, weight, eps=1e-6, zero_centered=False):
    x, weight = _c(np.atleast_2d(x), np.float32), _c(weight, np.float32)
    out = np.empty_like(x)
    lib().oracle_rms_norm(_p(x), _p(weight), x.shape[0], x.shape[1], eps, int(zero_centered), _p(out))
    return out


class OracleLayer:
    """One MoE layer (a synthetic.Layer or anything with router / bias / gate /
    down / shared / spec) in the restatement's C structures."""

    def __init__(self, layer, shared_mode=None, router_order=None, min_weight=None):
        spec = layer.spec
        self.H, self.I, self.E, self.k = spec.hidden, spec.inter, spec.experts, spec.top
        self.router = _c(layer.router, np.float32)
        self.bias = None if layer.bias is None else _c(layer.bias, np.float32)
        self.gm = [_Mat(m) for m in layer.gate]
        self.dm = [_Mat(m) for m in layer.down]
        self.gate_arr = (QMat * self.E)(*[m.s for m in self.gm])
        self.down_arr = (QMat * self.E)(*[m.s for m in self.dm])
        self.s = LayerS()
        s = self.s
        s.hidden, s.inter, s.experts, s.top = self.H, self.I, self.E, self.k
        s.router_order = spec.router_order if router_order is None else router_order
        s.min_weight = spec.min_weight if min_weight is None else min_weight
        s.router, s.router_bias = _p(self.router), _p(self.bias)
        s.gate_up, s.down = self.gate_arr, self.down_arr
        self.Is = 0
        if layer.shared is not None:
            g, d = layer.shared
            self.sg, self.sd = _Mat(g), _Mat(d)
            self.Is = g.n // 2
            s.shared_inter = self.Is
            if shared_mode is None:
                shared_mode = SHARED_JOINT if (self.Is == self.I and g.bits == 8) else SHARED_DENSE
            s.shared_mode = shared_mode
            s.shared_gate_up = C.pointer(self.sg.s)
            s.shared_down = C.pointer(self.sd.s)
        s.route_rule = getattr(spec, "route_rule", ROUTE_SOFTMAX)
        s.groups = getattr(spec, "groups", 1)
        s.top_groups = getattr(spec, "top_groups", 1)
        s.routing_scale = getattr(spec, "routing_scale", 1.0)
        eb, sgate = getattr(layer, "expert_bias", None), getattr(layer, "shared_gate", None)
        self.expert_bias = None if eb is None else _c(eb, np.float32)
        self.shared_gate = None if sgate is None else _c(sgate, np.float32)
        s.expert_bias, s.shared_gate = _p(self.expert_bias), _p(self.shared_gate)

    def _dump(self, T, A, want):
        if not want:
            return None, None
        H, I, E, k = self.H, self.I, self.E, self.k
        bufs = dict(logits=np.empty((T, E), np.float32), ids=np.empty((T, k), np.int32),
                    weights=np.empty((T, k), np.float32), perm=np.empty(A, np.int32),
                    offsets=np.empty(E + 1, np.int32), qx=np.empty((T, H), np.int8),
                    sx=np.empty(T, np.float32), middle=np.empty((A, I), np.float32),
                    qm=np.empty((A, I), np.int8), sm=np.empty(A, np.float32),
                    y=np.empty((A, H), np.float32), routed=np.empty((T, H), np.float32),
                    shared=np.empty((T, H), np.float32), shared_scale=np.empty(T, np.float32))
        d = Dump(**{n: _p(a) for n, a in bufs.items()})
        return d, bufs

    def forward(self, x, residual=None, dump=False):
        x = _c(x, np.float32)
        T = x.shape[0]
        res = None if residual is None else _c(residual, np.float32)
        out = np.empty((T, self.H), np.float32)
        d, bufs = self._dump(T, T * self.k, dump)
        rc = lib().oracle_moe_forward(C.byref(self.s), T, _p(x), _p(res), _p(out),
                                      None if d is None else C.byref(d))
        if rc != 0:
            raise ValueError("oracle forward failed")
        if dump:
            A = d.n_assign
            for n in ("perm", "middle", "qm", "sm", "y"):
                bufs[n] = bufs[n][:A]
            return out, bufs
        return out

    def run(self, x, ids, weights, dump=False):
        x = _c(x, np.float32)
        ids, weights = _c(ids, np.int32), _c(weights, np.float32)
        T = x.shape[0]
        out = np.empty((T, self.H), np.float32)
        d, bufs = self._dump(T, T * self.k, dump)
        rc = lib().oracle_moe_run(C.byref(self.s), T, _p(x), _p(ids), _p(weights), _p(out),
                                  None if d is None else C.byref(d))
        if rc != 0:
            raise ValueError("expert id out of range")
        if dump:
            A = d.n_assign
            for n in ("perm", "middle", "qm", "sm", "y"):
                bufs[n] = bufs[n][:A]
            return out, bufs
        return out


def threads() -> int:
    return lib().oracle_threads()
