"""Benchmark of the B200 MoE layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the Qwen3-30B-A3B-shaped W4A8 MoE layer
(H=2048, 128 experts, top-8, I=768, int4 group-32 fp16 scales, per-token int8
activations), 512 prefill tokens per GPU, seeded synthetic data. One step =
one router-inclusive layer forward (router + top-k, dispatch, gate/up GEMM +
SwiGLU, requant, down GEMM, combine + residual) on inputs resident in HBM.
`e2e` times the same layer through the public host-pointer API with the
input/residual copied from pinned host memory and the output read back.
Decode (T=1) and 4096-token prefill are reported under "extra"; `--suite`
adds the other BASELINE configurations (3, 4 and 5) under "suite".

With N > 1 (torchrun) the layer runs expert parallel: rank g owns experts
[g*E/N, (g+1)*E/N) and routes its own 512 tokens; rows travel to the expert
owners and back by the GPUs' own stores into peer memory over NVLink
(moe_b200_ep_exchange_*, no host synchronisation, one CUDA-graph replay per
step; weak scaling); the time is the max over ranks. With --suite it also
measures the config-4 stack expert parallel.
`--impl reference` times the CPU restatement of the reference path (the
oracle, all host threads) on the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W4A8 MoE-layer tokens/s"
CONFIG = "c2"
TOKENS = 512
SEED = 1234
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
INT8_DATASHEET_TOPS = 4500.0  # B200 datasheet dense int8, for context only


def int8_peak():
    """Dense int8 tensor-core rate measured on this GPU by the tcgen05 probe
    (open_rknpu2_lm_infer_b200/mma_peak.py: M=128 x N=256 x K=32 MMAs back to
    back on every SM), in TOPS; the datasheet figure if the probe is missing."""
    try:
        from open_rknpu2_lm_infer_b200 import mma_peak
        return mma_peak.int8_peak_tops(), "measured (tcgen05 kind::i8 probe, this GPU)"
    except Exception as e:  # the probe library is built with the package
        return INT8_DATASHEET_TOPS, f"datasheet ({type(e).__name__})"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (read-only queries)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [s for s in sm if s > 0.5 * (max(sm) if sm else 1)]
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- traffic
def measured_traffic(key: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get(key)
        if isinstance(v, dict):
            return v.get("bytes_per_launch")
        return v
    return None


def layer_bytes(spec, T, U, A):
    """Algorithmic HBM bytes of one layer call, the formula of the hot-path
    plan: the int4 codes + fp16 group scales of the U experts hit, the f32
    router, x in, residual in, out."""
    H, I = spec.hidden, spec.inter
    w = 3 * H * I // 2 + 3 * H * I // 32 * 2          # int4 codes + fp16 group scales
    return U * w + spec.experts * H * 4 + 3 * T * H * 4


def layer_bytes_with_intermediates(spec, T, U, A):
    """The same plus the intermediates this design writes and reads back: the
    permuted int8 activation rows, the f32 gate | up rows (written by the
    gate/up GEMM, read by the SwiGLU + requantisation), the int8 middle codes,
    the f32 expert rows y (written by the down GEMM, read by the combine)."""
    H, I = spec.hidden, spec.inter
    return (layer_bytes(spec, T, U, A) + A * H * 2 + A * 2 * I * 4 * 2 + A * I * 2 +
            A * H * 4 * 2)


def gate_up_bytes(spec, U, A):
    """Algorithmic bytes of one gate/up GEMM launch: int4 codes + fp16 scales of
    the experts hit, the permuted int8 activation rows read, the f32 gate | up
    rows written."""
    H, I = spec.hidden, spec.inter
    return U * (2 * I * H // 2 + 2 * I * H // 32 * 2) + A * H + A * 2 * I * 4


def gate_up_ops(spec, A):
    """int8 tensor-core ops of one gate/up launch (2 per multiply-add)."""
    return 2 * A * 2 * spec.inter * spec.hidden


# ---------------------------------------------------------------- ours
def setup_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_ours(args):
    import torch
    import torch.distributed as dist
    from open_rknpu2_lm_infer_b200 import synthetic as S
    from open_rknpu2_lm_infer_b200.moe import Backend

    world, rank, local = setup_dist()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    spec = S.CONFIGS[CONFIG]
    T = args.tokens
    layer = S.make_layer(spec, seed=SEED)
    max_rows = max(T, 4096 if args.extra else T)
    be = Backend(device=local, max_rows=max_rows)
    moe = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    lib, wsp = be.lib, moe.workspace

    def inputs(t, stream_id):
        return torch.from_numpy(S.make_input(spec, t, seed=SEED + rank, stream=stream_id)).cuda()

    x, res = inputs(T, 4), inputs(T, 5)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step(t=T, xx=None, rr=None, oo=None):
        moe.forward_device(router, t, (xx if xx is not None else x).data_ptr(),
                           (rr if rr is not None else res).data_ptr(),
                           (oo if oo is not None else out).data_ptr(), sp)

    # the timed step: one replay of the captured layer (moe_b200_graph_*)
    graph = moe.graph(router, T, x.data_ptr(), res.data_ptr(), out.data_ptr())
    for _ in range(args.warmup):
        graph.launch(sp)
    torch.cuda.synchronize()
    moe.status()

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    launches0 = lib.moe_b200_workspace_launches(wsp)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        graph.launch(sp)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = lib.moe_b200_workspace_launches(wsp) - launches0
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    moe.status()
    graph.close()

    # per-stage device times: the same step launched kernel by kernel with
    # events between the stages (the profiling ring), after the timed region
    from open_rknpu2_lm_infer_b200 import _lib as L
    lib.moe_b200_workspace_profile(wsp, 1)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    stages = []
    for i in range(args.steps):
        tm = L.Timings()
        if lib.moe_b200_workspace_profile_read(wsp, i, tm) == 0:
            stages.append(tm.as_dict())
    lib.moe_b200_workspace_profile(wsp, 0)
    stage_avg = {k: statistics.mean(s[k] for s in stages) for k in stages[0]} if stages else {}

    # routing statistics of the last call: experts hit, kept assignments
    torch.cuda.synchronize()
    U, A = routing_stats(moe, spec, T)

    pk, pk_kind = peaks()
    hbm_peak = pk["hbm_gbs"]
    gu_bytes = gate_up_bytes(spec, U, A)
    gate_us = stage_avg.get("gate_us", float("nan"))
    achieved = gu_bytes / (gate_us * 1e-6) / 1e9 if gate_us == gate_us and gate_us > 0 else None
    traffic = measured_traffic(f"{CONFIG}_T{T}_gate_up")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": (achieved / hbm_peak) if achieved else None, "traffic": traffic,
                "kernel": "grouped_gemm_kernel<W4G32, GateUp, 32> (gate/up, exact int32 "
                          "group sums, f32 gate | up rows out)",
                "algorithmic_bytes_per_launch": gu_bytes, "kernel_us": gate_us,
                "peak_kind": f"{pk_kind} (hbm_gbs, STREAM-style copy)"}

    # ---------------------------------------------------------------- e2e
    e2e = run_e2e(args, moe, router, spec, T, rank, world)

    value = world * T / (ms * 1e-3)
    lbytes = layer_bytes(spec, T, U, A)
    ops = 2 * A * 3 * spec.hidden * spec.inter
    i8_peak, i8_kind = int8_peak()
    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: seeded activations ~N(0,1); weights ~N(0,0.02) quantised to int4 "
                "group-32 with fp16 scales",
        "config": {"workload": f"{CONFIG}: Qwen3-30B-A3B-shaped W4A8 MoE layer, {T}-token prefill "
                               "per GPU, router-inclusive forward with residual",
                   "hidden": spec.hidden, "experts": spec.experts, "top_k": spec.top,
                   "intermediate": spec.inter,
                   "weights": "int4 g32 fp16 scales (MOE_B200_W4_G32_FP16): exact int32 group "
                              "sums in both GEMMs, int8 activations",
                   "tokens_per_gpu": T, "global_batch": T * world, "seq_len": T,
                   "parallelism": f"replica x{world}" if world > 1 else "single GPU",
                   "l2": "no flush: the expert weights read per step (~330 MB) exceed the "
                         "126 MB L2",
                   "timing": "CUDA events around CUDA-graph replays of the layer"},
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk,
        "stage_us": stage_avg,
        "layer": {"experts_hit": U, "assignments": A,
                  "algorithmic_bytes": lbytes,
                  "hbm_frac_layer": lbytes / (ms * 1e-3) / 1e9 / hbm_peak,
                  "bytes_with_intermediates": layer_bytes_with_intermediates(spec, T, U, A),
                  "int8_tops": ops / (ms * 1e-3) / 1e12,
                  "int8_peak_tops": i8_peak, "int8_peak_kind": i8_kind,
                  "int8_frac": ops / (ms * 1e-3) / 1e12 / i8_peak},
    }
    if args.extra and world == 1:
        result["extra"] = run_extra(args, moe, router, spec, lib, wsp, hbm_peak, i8_peak, i8_kind)
    if args.suite and world == 1:
        result["suite"] = run_suite(args, hbm_peak)
    if rank == 0 and world == 1 and args.cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(layer, spec, T, budget_s=args.cpu_seconds)
    moe.close()
    router.close()
    be.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_ep(args):
    """N > 1: the expert-parallel layer (open_rknpu2_lm_infer_b200.ep). Rank g
    owns experts [g*E/N, (g+1)*E/N) and routes its own 512 tokens; rows travel
    to the expert owners and back through the device-initiated exchange (peer
    stores over NVLink). Weak scaling: the tokens per GPU are fixed; the time
    is the max over ranks."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from open_rknpu2_lm_infer_b200 import _lib as L
    from open_rknpu2_lm_infer_b200 import synthetic as S
    from open_rknpu2_lm_infer_b200.ep import DeviceExchange, DeviceOps, ep_forward_device
    from open_rknpu2_lm_infer_b200.moe import Backend

    world, rank, local = setup_dist()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    spec = S.CONFIGS[CONFIG]
    T = args.tokens
    P = spec.experts // world
    layer = S.make_layer(spec, seed=SEED)
    be = Backend(device=local, max_rows=world * T)
    moe = be.load_moe(layer.gate[rank * P:(rank + 1) * P], layer.down[rank * P:(rank + 1) * P],
                      spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    ops = DeviceOps(be, moe, router, world, T)
    lib = be.lib
    x = torch.from_numpy(S.make_input(spec, T, seed=SEED + rank, stream=4)).cuda()
    res = torch.from_numpy(S.make_input(spec, T, seed=SEED + rank, stream=5)).cuda()
    stream = torch.cuda.current_stream()
    # the exchange runs on the GPUs themselves (peer memory, no host
    # synchronisation), so one layer step is captured once and replayed
    ex = DeviceExchange(ops, dist)
    dist.barrier()

    def eager():
        return ep_forward_device(ops, ex, x, res)

    for _ in range(args.warmup):
        eager()
    torch.cuda.synchronize()
    ex.status()
    ops.status()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            out_g = eager()
    stream.wait_stream(side)

    def step():
        graph.replay()
        return out_g, None

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    ex.status()
    dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    # kernels per step: count one eager step's launches
    l0 = lib.moe_b200_workspace_launches(ops.ws) + lib.moe_b200_workspace_launches(moe.workspace)
    eager()
    torch.cuda.synchronize()
    per_step = (lib.moe_b200_workspace_launches(ops.ws) +
                lib.moe_b200_workspace_launches(moe.workspace) - l0)
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    launches = per_step * args.steps
    ms = e0.elapsed_time(e1) / args.steps
    ex.status()
    # rows sent / received per step (outside the timed region)
    recv_counts = torch.empty_like(ops.counts)
    dist.all_to_all_single(recv_counts, ops.counts.clone())
    sent = int(ops.counts.sum().item()) * args.steps
    recv = int(recv_counts.sum().item()) * args.steps
    # stage times of eager steps with the profiling ring on
    lib.moe_b200_workspace_profile(moe.workspace, 1)
    for _ in range(args.steps):
        eager()
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    stages = []
    for i in range(args.steps):
        tm = L.Timings()
        if lib.moe_b200_workspace_profile_read(moe.workspace, i, tm) == 0:
            stages.append(tm.as_dict())
    lib.moe_b200_workspace_profile(moe.workspace, 0)
    gate_us = statistics.mean(s_["gate_us"] for s_ in stages) if stages else float("nan")
    ep_stages = ep_stage_breakdown(args, ops, ex, x, res, stream, world)
    rows_here = recv // max(args.steps, 1)
    # the experts of this rank hit by its received rows: all of them at this size
    U = P
    gu_bytes = gate_up_bytes(spec, U, rows_here)
    pk, pk_kind = peaks()
    hbm_peak = pk["hbm_gbs"]
    achieved = gu_bytes / (gate_us * 1e-6) / 1e9 if gate_us == gate_us and gate_us > 0 else None

    # e2e: pinned host input/residual copied in and the output read back per step
    xh = torch.empty((T, spec.hidden), dtype=torch.float32, pin_memory=True)
    rh = torch.empty_like(xh, pin_memory=True)
    oh = torch.empty_like(xh, pin_memory=True)
    xh.copy_(x.cpu())
    rh.copy_(res.cpu())
    dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        x.copy_(xh, non_blocking=True)
        res.copy_(rh, non_blocking=True)
        out, _ = step()
        oh.copy_(out, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    t = torch.tensor([e2e_ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    ops.status()
    row_bytes = ops.row_bytes
    result = {
        "metric": METRIC, "value": world * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: seeded activations ~N(0,1); weights ~N(0,0.02) quantised to int4 "
                "group-32 with fp16 scales",
        "config": {"workload": f"{CONFIG}: Qwen3-30B-A3B-shaped W4A8 MoE layer, {T}-token prefill "
                               "per GPU, router-inclusive forward with residual, expert parallel",
                   "hidden": spec.hidden, "experts": spec.experts, "top_k": spec.top,
                   "intermediate": spec.inter, "weights": "int4 g32 fp16 scales",
                   "tokens_per_gpu": T, "global_batch": T * world, "seq_len": T,
                   "parallelism": f"ep{world} ({P} experts per GPU, dispatch and combine by "
                                  "peer-memory stores over NVLink)",
                   "timing": "CUDA events around CUDA-graph replays of the layer step, max over ranks",
                   "l2": "no flush: the expert weights read per step exceed the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": (achieved / hbm_peak) if achieved else None, "traffic": None,
                     "kernel": "grouped_gemm_kernel<W4G32, GateUp> (gate/up of the received rows, rank 0)",
                     "algorithmic_bytes_per_launch": gu_bytes, "kernel_us": gate_us,
                     "peak_kind": f"{pk_kind} (hbm_gbs, STREAM-style copy)"},
        "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * T * spec.hidden * 4,
                "d2h_bytes_per_step": T * spec.hidden * 4, "ms_per_step": e2e_ms,
                "api": "ep_forward_device over moe_b200_ep_* and moe_b200_ep_exchange_* "
                       "(graph replay, pinned host buffers)"},
        "gpu_launches": int(launches),
        "clocks": clk,
        "ep_stages_us": ep_stages,
        "exchange": {"rows_sent_per_step_rank0": sent // max(args.steps, 1),
                     "rows_received_per_step_rank0": rows_here,
                     "dispatch_bytes_per_row": row_bytes + 8,
                     "transport": "peer stores over NVLink (CUDA IPC mappings), step flags",
                     "combine_bytes_per_row": spec.hidden * 4},
    }
    del graph
    torch.cuda.synchronize()
    if args.suite:
        result["suite"] = {"c4_stack": run_ep_stack(args, world, rank, local, stream)}
    dist.barrier()  # every rank done with its peers' memory before unmapping
    ex.close()
    ops.close()
    moe.close()
    router.close()
    be.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def ep_stage_breakdown(args, ops, ex, x, res, stream, world):
    """Per-stage device times of eager EP layer steps (CUDA events on the
    layer's stream): route, pack, the exchange's five stages (dispatch, rows
    wait, expert rows, return, return wait), combine. Mean over the profiled
    steps on each rank, then the max and min over ranks of each stage."""
    import torch
    import torch.distributed as dist
    names = ["route_us", "pack_us", *ex.STAGES, "combine_us"]
    per = []
    ex.profile(True)
    for _ in range(max(args.steps, 1)):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(stream)
        ids, routes = ops.route(x)
        ev[1].record(stream)
        send_q, send_scale, send_expert, counts, pos = ops.pack(x, ids, routes)
        ev[2].record(stream)
        y_back = ex.step(send_q, send_scale, send_expert, counts, ops.moe)
        ev[3].record(stream)
        ops.combine(y_back, pos, routes, res)
        ev4 = torch.cuda.Event(enable_timing=True)
        ev4.record(stream)
        torch.cuda.synchronize()
        xs = ex.profile_read()
        per.append([1000 * ev[0].elapsed_time(ev[1]), 1000 * ev[1].elapsed_time(ev[2]),
                    *(xs[k] for k in ex.STAGES), 1000 * ev[3].elapsed_time(ev4)])
    ex.profile(False)
    mean = torch.tensor([statistics.mean(col) for col in zip(*per)], device="cuda")
    hi, lo = mean.clone(), mean.clone()
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    return {"max_over_ranks": dict(zip(names, hi.tolist())),
            "min_over_ranks": dict(zip(names, lo.tolist())),
            "steps": max(args.steps, 1), "n_ranks": world,
            "timing": "eager steps, CUDA events on the layer stream"}


def routing_stats(moe, spec, T):
    """(distinct experts hit, kept assignments) of the last routed call, from
    the workspace's ids and routing weights (valid for every execution path)."""
    ids = np.empty((T, spec.top), np.int32)
    w = np.empty((T, spec.top), np.float32)
    cudart_copy(ids, moe.buffer("ids")[0])
    cudart_copy(w, moe.buffer("routes")[0])
    kept = w > 0
    return int(np.unique(ids[kept]).size), int(kept.sum())


def cudart_copy(dst: np.ndarray, src_ptr: int):
    import torch

    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": dst.shape, "typestr": dst.dtype.str,
                                             "data": (src_ptr, False), "version": 3}
    dst[...] = torch.as_tensor(_CAI(), device="cuda").cpu().numpy()


def run_e2e(args, moe, router, spec, T, rank, world):
    """Public host API (moe_b200_forward_f32): pinned input/residual -> device,
    layer, output + routing -> host, all inside the timed call. Time per call =
    the host wall clock around the call (validation, the ctypes call, the
    copies, the layer and the synchronising return), max over ranks; the
    library's own CUDA-event time of the same calls is reported beside it."""
    import torch
    from open_rknpu2_lm_infer_b200 import synthetic as S
    xh = torch.empty((T, spec.hidden), dtype=torch.float32, pin_memory=True)
    rh = torch.empty_like(xh, pin_memory=True)
    xh.numpy()[...] = S.make_input(spec, T, seed=SEED + rank, stream=4)
    rh.numpy()[...] = S.make_input(spec, T, seed=SEED + rank, stream=5)
    x, r = xh.numpy(), rh.numpy()
    # page-locked outputs too: the copies back run at full PCIe rate
    oh = torch.empty_like(xh, pin_memory=True).numpy()
    ih = torch.empty((T, spec.top), dtype=torch.int32, pin_memory=True).numpy()
    wh = torch.empty((T, spec.top), dtype=torch.float32, pin_memory=True).numpy()
    for _ in range(args.warmup):
        moe.forward(router, x, r, out=oh, ids=ih, routes=wh)
    ev_times = []
    for _ in range(args.steps):
        *_, tm = moe.forward(router, x, r, timings=True, out=oh, ids=ih, routes=wh)
        ev_times.append(tm["total_us"])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        moe.forward(router, x, r, out=oh, ids=ih, routes=wh)
    mean_us = (time.perf_counter() - t0) / args.steps * 1e6
    ev_us = statistics.mean(ev_times)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([mean_us, ev_us], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mean_us, ev_us = float(t[0].item()), float(t[1].item())
    h2d = 2 * T * spec.hidden * 4
    d2h = T * spec.hidden * 4 + 2 * T * spec.top * 4
    return {"value": world * T / (mean_us * 1e-6), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": mean_us / 1000.0,
            "timing": "host wall clock (time.perf_counter) around each moe_b200_forward_f32 call",
            "device_event_ms_per_step": ev_us / 1000.0,
            "device_event_timing": "library CUDA events of eager calls (stage timings asked for)",
            "api": "moe_b200_forward_f32 (pinned host buffers: the call replays the "
                   "workspace's captured graph of its copies and layer)"}


def run_extra(args, moe, router, spec, lib, wsp, hbm_peak, i8_peak, i8_kind):
    import torch
    from open_rknpu2_lm_infer_b200 import _lib as L
    from open_rknpu2_lm_infer_b200 import synthetic as S
    out = {}
    for name, T in (("decode_t1", 1), ("prefill_t4096", 4096)):
        x = torch.from_numpy(S.make_input(spec, T, seed=SEED, stream=4)).cuda()
        res = torch.from_numpy(S.make_input(spec, T, seed=SEED, stream=5)).cuda()
        o = torch.empty_like(x)
        sp = torch.cuda.current_stream().cuda_stream
        call = lambda: moe.forward_device(router, T, x.data_ptr(), res.data_ptr(), o.data_ptr(), sp)
        g = moe.graph(router, T, x.data_ptr(), res.data_ptr(), o.data_ptr())
        for _ in range(max(3, args.warmup)):
            g.launch(sp)
        steps = max(3, min(args.steps, 20))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.launch(sp)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        g.close()
        lib.moe_b200_workspace_profile(wsp, 1)
        for _ in range(steps):
            call()
        torch.cuda.synchronize()
        st = []
        for i in range(steps):
            tm = L.Timings()
            if lib.moe_b200_workspace_profile_read(wsp, i, tm) == 0:
                st.append(tm.as_dict())
        lib.moe_b200_workspace_profile(wsp, 0)
        avg = {k: statistics.mean(s[k] for s in st) for k in st[0]} if st else {}
        U, A = routing_stats(moe, spec, T)
        lb = layer_bytes(spec, T, U, A)
        ops = 2 * A * 3 * spec.hidden * spec.inter
        gb = gate_up_bytes(spec, U, A)
        gu_us = avg.get("gate_us")
        out[name] = {"tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3),
                     "experts_hit": U, "hbm_frac_layer": lb / (ms * 1e-3) / 1e9 / hbm_peak,
                     "int8_tops": ops / (ms * 1e-3) / 1e12,
                     "int8_frac": ops / (ms * 1e-3) / 1e12 / i8_peak,
                     "gate_up_us": gu_us, "down_us": avg.get("down_us"),
                     "gate_up_gbs": gb / (gu_us * 1e-6) / 1e9 if avg else None,
                     "stage_us": avg}
        if name == "prefill_t4096" and gu_us:
            # the prefill-sized gate/up GEMM against the tensor-core roofline
            a = gate_up_ops(spec, A) / (gu_us * 1e-6) / 1e12
            out[name]["roofline"] = {
                "bound": "tensor", "achieved": a, "peak": i8_peak, "unit": "TOPS",
                "frac": a / i8_peak, "peak_kind": i8_kind,
                "kernel": "grouped_gemm_kernel<W4G32, GateUp, 32> (gate/up, 4096 tokens)",
                "ops_per_launch": gate_up_ops(spec, A), "kernel_us": gu_us,
                "traffic": measured_traffic(f"{CONFIG}_T4096_gate_up")}
    return out


def spec_bytes(spec, T, U):
    """Algorithmic HBM bytes of one layer call, any config: the weights of the
    U routed experts hit (int4 g32: codes + fp16 group scales; int8
    per-channel: codes + f32 scales), the shared expert (int8 per-channel),
    the f32 router, and x in, residual in, out."""
    H, I, Is = spec.hidden, spec.inter, spec.shared_inter
    if spec.routed == "w8pc":
        per_expert = 3 * H * I + 4 * (2 * I + H)
    elif spec.routed == "w4pc":
        per_expert = 3 * H * I // 2 + 4 * (2 * I + H)
    else:
        per_expert = 3 * H * I // 2 + 3 * H * I // 32 * 2
    shared = 3 * H * Is + 4 * (2 * Is + H) if Is else 0
    return U * per_expert + shared + spec.experts * H * 4 + 3 * T * H * 4


def run_suite(args, hbm_peak):
    """The other BASELINE configurations, one GPU, CUDA-graph replays timed with
    CUDA events (stack: eager launches): config 3 (routed W4 g32 + shared W8
    expert, Zipf-skewed router) at 498 and 2110 tokens; config 5 (the config-3
    layer with W4 g32 or W8 per-channel routed experts) at 1..256 tokens;
    config 4 (48 layers of config 2, RMSNorm before each, residual after) at
    4096 tokens, its 48 layers cycling over 4 distinct seeded banks (each bank,
    ~340 MB, is far above the 126 MB L2, so every layer streams its weights
    from HBM as 48 distinct banks would)."""
    import torch
    from open_rknpu2_lm_infer_b200 import synthetic as S
    from open_rknpu2_lm_infer_b200.moe import Backend
    from open_rknpu2_lm_infer_b200.stack import MoeStack
    sp = torch.cuda.current_stream().cuda_stream
    steps = max(3, min(args.steps, 20))
    out = {}

    def timed(fn, n):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def layer_case(name, tokens):
        spec = S.CONFIGS[name]
        layer = S.make_layer(spec, seed=SEED)
        be = Backend(max_rows=max(tokens))
        if layer.shared is not None:
            moe = be.load_moe_with_shared(layer.gate, layer.down, spec.top, layer.shared)
        else:
            moe = be.load_moe(layer.gate, layer.down, spec.top)
        router = be.router(layer.router, spec.top, layer.bias)
        res = {}
        for T in tokens:
            x = torch.from_numpy(S.make_input(spec, T, seed=SEED, stream=4)).cuda()
            r = torch.from_numpy(S.make_input(spec, T, seed=SEED, stream=5)).cuda()
            o = torch.empty_like(x)
            g = moe.graph(router, T, x.data_ptr(), r.data_ptr(), o.data_ptr())
            for _ in range(3):
                g.launch(sp)
            ms = timed(lambda: g.launch(sp), steps)
            g.close()
            moe.status()
            U, A = routing_stats(moe, spec, T)
            b = spec_bytes(spec, T, U)
            res[f"t{T}"] = {"tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3),
                            "experts_hit": U, "algorithmic_bytes": b,
                            "hbm_gbs": b / (ms * 1e-3) / 1e9,
                            "hbm_frac": b / (ms * 1e-3) / 1e9 / hbm_peak}
        moe.close(); router.close(); be.close()
        return res

    out["c3"] = layer_case("c3", (498, 2110))
    out["c5_w4"] = layer_case("c5_w4", (1, 8, 32, 128, 256))
    out["c5_w8"] = layer_case("c5_w8", (1, 8, 32, 128, 256))

    # config 4: the 48-layer stack at 4096 tokens
    spec, T, n_layers, n_banks = S.CONFIGS["c2"], 4096, 48, 4
    be = Backend(max_rows=T)
    banks = []
    for i in range(n_banks):
        lay = S.make_layer(spec, seed=SEED + 100 + i)
        banks.append((be.load_moe(lay.gate, lay.down, spec.top),
                      be.router(lay.router, spec.top, lay.bias)))
        del lay
    rng = np.random.default_rng(SEED)
    norms = [(1 + rng.standard_normal(spec.hidden) * 0.02).astype(np.float32)
             for _ in range(n_layers)]
    stack = MoeStack([banks[i % n_banks] for i in range(n_layers)], norms, eps=1e-6)
    h = torch.from_numpy(S.make_input(spec, T, seed=SEED, stream=4)).cuda()
    o = torch.empty_like(h)
    stack.forward_tensor(h, out=o)
    ms = timed(lambda: stack.forward_tensor(h, out=o), 3)
    for moe, _ in banks:
        moe.status()
    out["c4_stack"] = {"layers": n_layers, "tokens": T, "distinct_banks": n_banks,
                       "ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3),
                       "ms_per_layer": ms / n_layers, "n_gpus": 1}
    for moe, r in banks:
        moe.close(); r.close()
    be.close()
    return out


def run_ep_stack(args, world, rank, local, stream):
    """Config 4 expert parallel: 48 layers of config 2, RMSNorm before each and
    the residual after, 4096 tokens split over the ranks (4096 / N each); rank
    g holds experts [g E/N, (g+1) E/N) of every layer. The 48 layers cycle over
    4 distinct seeded banks (each ~340 MB whole, far above the L2, so every
    layer streams its weights from HBM as 48 distinct banks would). One
    exchange (sized for the stack's rows) shared by the layers; the stack is
    timed eagerly and as one captured CUDA graph; CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    from open_rknpu2_lm_infer_b200 import synthetic as S
    from open_rknpu2_lm_infer_b200.ep import DeviceExchange, DeviceOps, ep_forward_device
    from open_rknpu2_lm_infer_b200.moe import Backend
    spec, T_all, n_layers, n_banks = S.CONFIGS["c2"], 4096, 48, 4
    T = T_all // world
    P = spec.experts // world
    be = Backend(device=local, max_rows=world * T)
    banks = []
    for i in range(n_banks):
        lay = S.make_layer(spec, seed=SEED + 100 + i)
        moe = be.load_moe(lay.gate[rank * P:(rank + 1) * P], lay.down[rank * P:(rank + 1) * P],
                          spec.top)
        router = be.router(lay.router, spec.top, lay.bias)
        banks.append((moe, router, DeviceOps(be, moe, router, world, T)))
        del lay
    ex = DeviceExchange(banks[0][2], dist)
    rng = np.random.default_rng(SEED)
    norms = [torch.from_numpy((1 + rng.standard_normal(spec.hidden) * 0.02).astype(np.float32)).cuda()
             for _ in range(n_layers)]
    h0 = torch.from_numpy(S.make_input(spec, T, seed=SEED + rank, stream=4)).cuda()
    xn = torch.empty_like(h0)
    lib = be.lib
    sp = stream.cuda_stream

    def stack():
        h = h0
        for l in range(n_layers):
            moe, router, ops = banks[l % n_banks]
            rc = lib.moe_b200_rms_norm(h.data_ptr(), norms[l].data_ptr(), T, spec.hidden, 1e-6, 0,
                                       xn.data_ptr(), sp)
            if rc:
                raise RuntimeError(f"RMSNorm failed ({rc})")
            h = ep_forward_device(ops, ex, xn, h)
        return h

    stack()
    torch.cuda.synchronize()
    ex.status()
    dist.barrier()

    def timed(fn, n=3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / n], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    eager_ms = timed(stack)
    # the whole 48-layer stack captured once (the exchange's step counter
    # lives on the device, so replays stay in lockstep across the ranks)
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            stack()
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    ms = timed(graph.replay)
    del graph
    torch.cuda.synchronize()
    ex.status()
    for moe, router, ops in banks:
        ops.status()
    dist.barrier()  # every rank done with its peers' memory before unmapping
    ex.close()
    for moe, router, ops in banks:
        ops.close(); moe.close(); router.close()
    be.close()
    return {"layers": n_layers, "tokens": T_all, "tokens_per_gpu": T, "distinct_banks": n_banks,
            "ms_per_step": ms, "tokens_per_s": T_all / (ms * 1e-3), "ms_per_layer": ms / n_layers,
            "eager_ms_per_step": eager_ms, "timing": "CUDA-graph replays of the whole stack, "
            "CUDA events, max over ranks",
            "n_gpus": world, "parallelism": f"ep{world}"}


# ---------------------------------------------------------------- CPU side
def cpu_baseline(layer, spec, T, budget_s=10.0):
    """The CPU restatement (oracle/, all host threads) on a bounded sample of
    the same workload: repeated full forwards of the T-token layer."""
    from oracle import oracle as O
    from open_rknpu2_lm_infer_b200 import synthetic as S
    ol = O.OracleLayer(layer)
    x = S.make_input(spec, T, seed=SEED, stream=4)
    res = S.make_input(spec, T, seed=SEED, stream=5)
    ol.forward(x[:8], res[:8])  # warm-up (thread pool, page-in)
    reps, t0 = 0, time.perf_counter()
    while True:
        ol.forward(x, res)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    return {"value": reps * T / el, "unit": "tokens/s", "cores": O.threads(), "kind": "port",
            "sample": f"{reps} forwards of the {T}-token {CONFIG} layer ({el:.1f} s), "
                      "CPU restatement of the reference MoE path, OpenMP"}


def run_reference(args):
    """--impl reference: the reference path's CPU implementation (restated in
    oracle/, since the reference's Rust/NPU code cannot run here) on the host
    cores, same workload; rank 0 only."""
    world, rank, _ = setup_dist()
    if rank != 0:
        return
    from oracle import oracle as O
    from open_rknpu2_lm_infer_b200 import synthetic as S
    spec = S.CONFIGS[CONFIG]
    T = args.tokens
    layer = S.make_layer(spec, seed=SEED)
    ol = O.OracleLayer(layer)
    x = S.make_input(spec, T, seed=SEED, stream=4)
    res = S.make_input(spec, T, seed=SEED, stream=5)
    # bounded sample per step: tokens of the same layer, sized from a probe
    t0 = time.perf_counter()
    ol.forward(x[:64], res[:64])
    per_tok = (time.perf_counter() - t0) / 64
    budget = 150.0 / max(1, args.steps + args.warmup)  # whole run within a few minutes
    ts = int(max(16, min(T, budget / max(per_tok, 1e-9))))
    for _ in range(args.warmup):
        ol.forward(x[:ts], res[:ts])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ol.forward(x[:ts], res[:ts])
        times.append(time.perf_counter() - t0)
    ms = statistics.mean(times) * 1e3
    value = ts / (ms * 1e-3)
    sample = f"{ts} of the {T} tokens per step, CPU restatement of the reference MoE path"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (same seeded layer as the GPU arm)",
        "config": {"workload": f"{CONFIG}: Qwen3-30B-A3B-shaped W4A8 MoE layer, {T}-token prefill",
                   "hidden": spec.hidden, "experts": spec.experts, "top_k": spec.top,
                   "intermediate": spec.inter, "tokens_per_gpu": T, "seq_len": T,
                   "global_batch": T},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": O.threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--no-extra", dest="extra", action="store_false")
    ap.add_argument("--suite", action="store_true",
                    help="also measure BASELINE configs 3, 4 (48-layer stack) and 5 (one GPU)")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_ep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
