"""ctypes binding of libmoe_b200.so (declarations in include/moe_b200.h).

The library is built in-tree (python -m open_rknpu2_lm_infer_b200.build).
Loading fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmoe_b200.so"

# error codes
OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_NOMEM = -3
ERR_CUDA = -4
ERR_CAPACITY = -5
ERR_DEVICE_TIMEOUT = -6
ERR_BAD_EXPERT = -7
ERR_NONFINITE = -8
ERR_BAD_ROUTE = -9
ERR_NO_DEVICE = -10
ERR_NOALLOC_LIMIT = -11
NOALLOC_MAX_LOGITS = 1 << 20

W4_PER_CHANNEL = 0
W4_G32_FP16 = 1
W8_PER_CHANNEL = 2
W4_G32_FP16_EXACT = 3
W4_G32_FP16_ROUNDED_DOWN = 4
ROUTER_NEON16 = 0
ROUTER_SEQUENTIAL = 1
ROUTER_TF32 = 2
ROUTE_SOFTMAX = 0
ROUTE_GROUPED_SIGMOID = 1
EP_HANDLE_BYTES = 64
SHARED_JOINT = 0
SHARED_DENSE = 1


class WeightConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("intermediate", C.c_int32),
                ("routed_experts", C.c_int32), ("shared_expert", C.c_int32),
                ("shared_intermediate", C.c_int32)]


class Config(C.Structure):
    _fields_ = [("weights", WeightConfig), ("top", C.c_int32), ("max_rows", C.c_int32),
                ("device", C.c_int32), ("npu_cores", C.c_int32), ("cpu_threads", C.c_int32)]


class Expert(C.Structure):
    _fields_ = [("gate_up", C.c_void_p), ("gate_up_scales", C.c_void_p),
                ("down", C.c_void_p), ("down_scales", C.c_void_p),
                ("gate_up_group_scales", C.c_void_p), ("down_group_scales", C.c_void_p)]


class Format(C.Structure):
    _fields_ = [("routed_format", C.c_int32), ("shared_format", C.c_int32),
                ("shared_mode", C.c_int32)]


class RouterOptions(C.Structure):
    _fields_ = [("order", C.c_int32), ("rule", C.c_int32), ("min_weight", C.c_float),
                ("bias", C.c_void_p), ("groups", C.c_int32), ("top_groups", C.c_int32),
                ("routing_scale", C.c_float), ("expert_bias", C.c_void_p),
                ("shared_gate", C.c_void_p)]


class Timings(C.Structure):
    _fields_ = [(n, C.c_double) for n in (
        "input_us", "schedule_us", "build_us", "sync_us", "gather_us", "gate_us",
        "middle_npu_us", "middle_cpu_us", "down_us", "combine_us", "lut_load_us", "total_us")] + [
        ("gather_tasks", C.c_int64), ("middle_tasks", C.c_int64), ("gemm_tasks", C.c_int64),
        ("router_us", C.c_double)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


# (name, restype, argtypes) of every exported entry point of the header
SIGNATURES = [
    ("moe_b200_config_init", None,
     [C.POINTER(Config), C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    ("moe_b200_weights_create", C.c_void_p,
     [C.POINTER(Config), C.POINTER(Expert), C.POINTER(Format)]),
    ("moe_b200_weights_free", None, [C.c_void_p]),
    ("moe_b200_weights_device_bytes", C.c_uint64, [C.c_void_p]),
    ("moe_b200_blob_version", C.c_uint32, []),
    ("moe_b200_slots_create", C.c_void_p, [C.POINTER(Config), C.c_int32]),
    ("moe_b200_expert_blob_bytes", C.c_uint64, [C.c_void_p]),
    ("moe_b200_export_expert", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_uint64]),
    ("moe_b200_import_expert", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_uint64]),
    ("moe_b200_import_expert_async", C.c_int,
     [C.c_void_p, C.c_int32, C.c_void_p, C.c_uint64, C.c_void_p]),
    ("moe_b200_swap_slots", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p]),
    ("moe_b200_workspace_create", C.c_void_p, [C.POINTER(Config)]),
    ("moe_b200_workspace_free", None, [C.c_void_p]),
    ("moe_b200_workspace_device_bytes", C.c_uint64, [C.c_void_p]),
    ("moe_b200_max_rows", C.c_int32, [C.c_void_p]),
    ("moe_b200_run_f32", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.POINTER(Timings)]),
    ("moe_b200_run_device", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_router_create", C.c_void_p,
     [C.POINTER(Config), C.c_void_p, C.c_void_p, C.c_int32, C.c_float]),
    ("moe_b200_router_free", None, [C.c_void_p]),
    ("moe_b200_router_options_init", None, [C.POINTER(RouterOptions)]),
    ("moe_b200_router_create_ex", C.c_void_p,
     [C.POINTER(Config), C.c_void_p, C.POINTER(RouterOptions)]),
    ("moe_b200_forward_f32", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p, C.c_void_p, C.POINTER(Timings)]),
    ("moe_b200_forward_device", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_route_device", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_workspace_status", C.c_int, [C.c_void_p]),
    ("moe_b200_workspace_buffer", C.c_int,
     [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_uint64)]),
    ("moe_b200_debug_accumulators", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_uint64, C.c_void_p]),
    ("moe_b200_workspace_profile", C.c_int, [C.c_void_p, C.c_int32]),
    ("moe_b200_workspace_profile_read", C.c_int, [C.c_void_p, C.c_int32, C.POINTER(Timings)]),
    ("moe_b200_workspace_launches", C.c_int64, [C.c_void_p]),
    ("moe_b200_workspace_row_bytes", C.c_int64, [C.c_void_p]),
    ("moe_b200_ep_exchange_create", C.c_void_p,
     [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int64, C.c_int32]),
    ("moe_b200_ep_exchange_handle", C.c_int, [C.c_void_p, C.c_void_p]),
    ("moe_b200_ep_exchange_connect", C.c_int, [C.c_void_p, C.c_void_p]),
    ("moe_b200_ep_exchange_step", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_ep_exchange_y_back", C.c_void_p, [C.c_void_p]),
    ("moe_b200_ep_exchange_status", C.c_int, [C.c_void_p]),
    ("moe_b200_ep_exchange_probe_timeout", C.c_int, [C.c_void_p, C.c_void_p]),
    ("moe_b200_ep_exchange_profile", C.c_int, [C.c_void_p, C.c_int32]),
    ("moe_b200_ep_exchange_profile_read", C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    ("moe_b200_ep_exchange_free", None, [C.c_void_p]),
    ("moe_b200_graph_create", C.c_void_p,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("moe_b200_graph_launch", C.c_int, [C.c_void_p, C.c_void_p]),
    ("moe_b200_graph_free", None, [C.c_void_p]),
    ("moe_b200_ep_pack", C.c_int,
     [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32,
      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("moe_b200_ep_expert_rows", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_ep_combine", C.c_int,
     [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("moe_b200_rms_norm", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_float, C.c_int32, C.c_void_p, C.c_void_p]),
    ("moe_b200_route_noalloc", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
      C.c_float, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("moe_b200_strerror", C.c_char_p, [C.c_int]),
    ("moe_b200_version", C.c_char_p, []),
]

_lib = None


def load() -> C.CDLL:
    """Loads the in-tree library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m open_rknpu2_lm_infer_b200.build`"
                " (there is no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().moe_b200_strerror(code).decode()


class MoeError(RuntimeError):
    """A non-zero moe_b200 return code (the reference's `check()`, src/npu.rs:187-193)."""

    def __init__(self, what: str, code: int):
        super().__init__(f"{what}: {strerror(code)} ({code})")
        self.code = code


def check(code: int, what: str) -> None:
    if code != OK:
        raise MoeError(what, code)
