"""Tensor-core rate probe (tcgen05), the measured int8 peak of the roofline.

    python -m open_rknpu2_lm_infer_b200.mma_peak [--iters N]

Runs csrc/mma_peak.cu (libmoe_b200_peak.so) on the current GPU: one CTA per
SM, each issuing M=128 x N x K MMAs back to back (kind::i8 K=32, kind::f16
K=16; the A operand from shared or tensor memory; 1..3 issuing threads per
CTA) and prints one JSON object with cycles per MMA and ops/s for every case,
the dense int8 and fp16 peaks (the best N=256 rates), and the result of the
fp16 exactness check (integer-valued operands summed exactly in fp32). It is
a measurement tool: the MoE operator does not use this library.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
from pathlib import Path

LIB = Path(__file__).resolve().parent / "libmoe_b200_peak.so"
_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise RuntimeError(f"{LIB.name} is missing: run python -m open_rknpu2_lm_infer_b200.build")
        L = C.CDLL(str(LIB))
        L.mma_peak_rate.restype = C.c_int
        L.mma_peak_rate.argtypes = [C.c_int] * 10 + [C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.mma_peak_wake.restype = C.c_double
        L.mma_peak_wake.argtypes = [C.c_int, C.c_int, C.c_int]
        L.mma_peak_tmem_bw.restype = C.c_double
        L.mma_peak_tmem_bw.argtypes = [C.c_int] * 6
        L.mma_peak_exact.restype = C.c_int
        L.mma_peak_exact.argtypes = [C.c_int, C.c_uint, C.POINTER(C.c_float)]
        _lib = L
    return _lib


def rate(kind: int, n: int, ts: bool, issuers: int, iters: int, grid: int, rot: int = 1,
         gap: int = 0, waits: int = 0, variant: int = 0) -> dict:
    """One case: kind 0 = int8 (K=32), 1 = fp16 (K=16); rot accumulators
    used in turn (1: each MMA depends on the previous one); after each MMA
    the issuing thread spins `gap` cycles and waits `waits` times on an
    mbarrier phase that is already complete. variant: 0 the bare issue loop,
    1 with the spin, 2 with plain try_waits, 3 with bounded waits."""
    cyc, ms = C.c_double(), C.c_double()
    mode = variant << 2
    rc = load().mma_peak_rate(kind, n, int(ts), issuers, rot, gap, waits, mode, iters, grid,
                              C.byref(cyc), C.byref(ms))
    if rc != 0:
        raise RuntimeError(f"mma_peak_rate failed ({rc})")
    k = 32 if kind == 0 else 16
    ops = grid * issuers * iters * 2.0 * 128 * n * k
    return {"kind": "i8" if kind == 0 else "f16", "n": n, "a_operand": "tmem" if ts else "smem",
            "issuers": issuers, "rot": rot, "gap": gap, "waits": waits,
            "variant": variant,
            "cycles_per_mma": cyc.value, "ms": ms.value,
            "tops": ops / (ms.value * 1e-3) / 1e12}


def int8_peak_tops(iters: int = 20000) -> float:
    """Dense int8 tensor-core rate of this GPU (M=128, N=256, K=32 MMAs, one
    issuer per SM, A and B in shared memory), in TOPS."""
    import torch
    grid = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return rate(0, 256, False, 1, iters, grid)["tops"]


def exact_check() -> dict:
    out = {}
    for pattern, name in ((0, "random"), (1, "extreme"), (2, "mixed")):
        s = (C.c_float * 8)()
        rc = load().mma_peak_exact(pattern, 12345 + pattern, s)
        out[name] = {"mismatches": rc, "sample_got_want": list(s)}
    return out


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=8192)
    ap.add_argument("--quick", action="store_true", help="peaks and the issue-loop cases only")
    args = ap.parse_args()
    torch.cuda.init()
    props = torch.cuda.get_device_properties(0)
    grid = props.multi_processor_count
    cases = []
    for kind in (0, 1):
        for ts in (False, True):
            for n in (16, 32, 64, 128, 256) if not args.quick else (256,):
                cases.append(rate(kind, n, ts, 1, args.iters, grid))
                if n <= 64:
                    cases.append(rate(kind, n, ts, 1, args.iters, grid, rot=4))
            for n in (32, 64) if not args.quick else ():
                for iss in (2, 3):
                    cases.append(rate(kind, n, ts, iss, args.iters, grid, rot=2))
    # what the issuing loop costs (int8, A in tensor memory, N = 32): the bare
    # loop; plain try_waits; the bounded wait inline; an inline try_wait with
    # the spin out of line; commits every 1 / 4 MMAs; four unrolled MMAs then
    # one wait (+ one commit)
    n, ts, rot = 32, True, 2
    for v, w, g in ((0, 0, 0), (2, 1, 0), (3, 1, 0), (4, 0, 0), (4, 1, 0), (4, 2, 0),
                    (5, 0, 1), (5, 0, 4), (6, 0, 0), (6, 1, 0), (6, 2, 0)):
        cases.append(rate(0, n, ts, 1, args.iters // 4, grid, rot=rot, waits=w, gap=g,
                          variant=v))
    wake = {name: {d: load().mma_peak_wake(m, 64, d) for d in (0, 2000, 20000)}
            for m, name in ((0, "try_wait_hint_1ms"), (1, "try_wait"), (2, "test_wait_spin"))}
    tmem = {}
    for mode, mname in ((0, "ld"), (1, "st")):
        for cols in (8, 32):
            for batch in (1, 4):
                for w in (4, 8, 16):
                    tmem[f"{mname}_x{cols}_b{batch}_w{w}"] = load().mma_peak_tmem_bw(
                        mode, cols, batch, w, 2000, grid)
    peak_i8 = max(c["tops"] for c in cases if c["kind"] == "i8" and c["n"] == 256)
    peak_f16 = max(c["tops"] for c in cases if c["kind"] == "f16" and c["n"] == 256)
    print(json.dumps({"gpu": props.name, "sms": grid, "iters": args.iters,
                      "int8_dense_tops": peak_i8, "fp16_dense_tflops": peak_f16,
                      "exact_f16_integer_sums": exact_check(), "wake_cycles_by_delay": wake,
                      "tmem_bytes_per_cycle": tmem,
                      "cases": cases}))


if __name__ == "__main__":
    main()
