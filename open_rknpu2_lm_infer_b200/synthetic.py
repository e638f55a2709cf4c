"""Seeded synthetic MoE layers with the shapes of the benchmark configurations.

No checkpoints or datasets are available offline, so every tensor is drawn
from a seeded generator (one independent numpy stream per tensor):
activations ~ N(0, 1), router and expert weights ~ N(0, 0.02) before
quantisation. Weights use the reference's QuantMatrix layout (codes [k][n]).

Configurations (shapes only; token counts are parameters):
  c1  H=1024 E=16  k=2 I=512  W4 group-32 fp16, no shared expert (T=32)
  c2  H=2048 E=128 k=8 I=768  W4 group-32 fp16 (Qwen3-30B-A3B shape; T=1/512/4096)
  c3  H=2048 E=256 k=8 I=512  W4 group-32 + shared W8 per-channel I_s=2048,
      router logits + seeded Zipf(s=1.1) per-expert bias (T=498/2110)
  c5  the c3 layer with routed W4 group-32 ("c5_w4") or W8 per-channel ("c5_w8")
  ling  H=1536 E=128 k=8 I=512 W4 per-channel + joint shared W8 I_s=512, TF32
        router, grouped sigmoid routing (8 groups, top 4, scale 2.5) with a
        seeded N(0, 0.1) expert bias (the Ling 2.5 mini shapes)
  q35g  the c3 layer with a dense shared expert I_s=512 behind a sigmoid gate
        (the Qwen3.5 MoE shared-expert arrangement)
"""
from __future__ import annotations

import concurrent.futures as cf
from dataclasses import dataclass, replace

import numpy as np

from .moe import QuantMatrix

ROUTER_NEON16, ROUTER_TF32 = 0, 2
ROUTE_SOFTMAX, ROUTE_GROUPED_SIGMOID = 0, 1


@dataclass(frozen=True)
class LayerSpec:
    name: str
    hidden: int
    inter: int
    experts: int
    top: int
    routed: str = "w4g32"          # "w4g32" | "w4pc" | "w8pc"
    shared_inter: int = 0
    shared_bits: int = 8
    zipf_s: float = 0.0            # router bias exponent, 0 = no bias
    zipf_scale: float = 2.0        # bias of the rank-1 expert, in logit units
    router_order: int = ROUTER_NEON16
    min_weight: float = 0.0
    route_rule: int = ROUTE_SOFTMAX
    groups: int = 1
    top_groups: int = 1
    routing_scale: float = 1.0
    expert_bias_std: float = 0.0   # grouped sigmoid: selection bias ~ N(0, std)
    shared_gate: bool = False      # sigmoid-gated shared expert


CONFIGS: dict[str, LayerSpec] = {
    "c1": LayerSpec("c1", 1024, 512, 16, 2),
    "c2": LayerSpec("c2", 2048, 768, 128, 8),
    "c3": LayerSpec("c3", 2048, 512, 256, 8, shared_inter=2048, zipf_s=1.1),
    "c5_w4": LayerSpec("c5_w4", 2048, 512, 256, 8, shared_inter=2048, zipf_s=1.1),
    "c5_w8": LayerSpec("c5_w8", 2048, 512, 256, 8, routed="w8pc", shared_inter=2048, zipf_s=1.1),
    "ling": LayerSpec("ling", 1536, 512, 128, 8, routed="w4pc", shared_inter=512,
                      router_order=ROUTER_TF32, route_rule=ROUTE_GROUPED_SIGMOID, groups=8,
                      top_groups=4, routing_scale=2.5, expert_bias_std=0.1),
    "q35g": LayerSpec("q35g", 2048, 512, 256, 8, shared_inter=512, zipf_s=1.1,
                      shared_gate=True),
}

TOKENS = {"c1": (32,), "c2": (1, 512, 4096), "c3": (498, 2110),
          "c5_w4": (1, 8, 32, 128, 256), "c5_w8": (1, 8, 32, 128, 256), "ling": (1, 512),
          "q35g": (1, 512)}

# tensor ids of the per-tensor streams
_ROUTER, _BIAS, _PERM, _X, _RES, _NORM = 1, 2, 3, 4, 5, 6
_GATE, _DOWN, _SGATE, _SDOWN = 100, 200, 300, 400
_EBIAS, _SHGATE = 7, 8


def rng(seed: int, tensor: int, index: int = 0) -> np.random.Generator:
    return np.random.default_rng([seed, tensor, index])


def quantize_g32(w: np.ndarray) -> QuantMatrix:
    """Symmetric int4, group 32 along k, fp16 scales: s = maxabs_g/7 (fp16),
    q = clamp(rne(w/s), -8, 7)."""
    k, n = w.shape
    g = w.reshape(k // 32, 32, n)
    s16 = (np.abs(g).max(axis=1) / np.float32(7.0)).astype(np.float16)
    s = s16.astype(np.float32)
    safe = np.where(s > 0, s, np.float32(1.0))
    q = np.clip(np.rint(g / safe[:, None, :]), -8, 7).astype(np.int8).reshape(k, n)
    return QuantMatrix(4, k, n, q, s16, group=32)


def quantize_pc(w: np.ndarray, bits: int) -> QuantMatrix:
    """Symmetric per-output-channel: s = maxabs_n / qmax, q = clamp(rne(w/s))."""
    k, n = w.shape
    qmax = 7 if bits == 4 else 127
    s = (np.abs(w).max(axis=0) / np.float32(qmax)).astype(np.float32)
    safe = np.where(s > 0, s, np.float32(1.0))
    lo = -8 if bits == 4 else -127
    q = np.clip(np.rint(w / safe[None, :]), lo, qmax).astype(np.int8)
    return QuantMatrix(bits, k, n, q, s)


def _quant(w: np.ndarray, fmt: str) -> QuantMatrix:
    if fmt == "w4g32":
        return quantize_g32(w)
    return quantize_pc(w, 4 if fmt == "w4pc" else 8)


@dataclass
class Layer:
    spec: LayerSpec
    router: np.ndarray            # [E][H] f32
    bias: np.ndarray | None       # [E] f32
    gate: list[QuantMatrix]       # [E] k=H, n=2I (gate columns first)
    down: list[QuantMatrix]       # [E] k=I, n=H
    shared: tuple[QuantMatrix, QuantMatrix] | None
    expert_bias: np.ndarray | None = None   # [E] f32 selection bias (grouped sigmoid)
    shared_gate: np.ndarray | None = None   # [H] f32 shared-expert gate row


def _expert(spec: LayerSpec, seed: int, e: int) -> tuple[QuantMatrix, QuantMatrix]:
    H, I = spec.hidden, spec.inter
    wg = rng(seed, _GATE, e).standard_normal((H, 2 * I), dtype=np.float32) * np.float32(0.02)
    wd = rng(seed, _DOWN, e).standard_normal((I, H), dtype=np.float32) * np.float32(0.02)
    return _quant(wg, spec.routed), _quant(wd, spec.routed)


def make_layer(spec: LayerSpec | str, seed: int = 0, threads: int = 8) -> Layer:
    spec = CONFIGS[spec] if isinstance(spec, str) else spec
    H, E = spec.hidden, spec.experts
    router = rng(seed, _ROUTER).standard_normal((E, H), dtype=np.float32) * np.float32(0.02)
    bias = None
    if spec.zipf_s > 0:
        order = rng(seed, _PERM).permutation(E)          # expert -> rank (0-based)
        ranks = np.empty(E, np.int64)
        ranks[order] = np.arange(E)
        bias = (spec.zipf_scale * (ranks + 1.0) ** (-spec.zipf_s)).astype(np.float32)
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        pairs = list(ex.map(lambda e: _expert(spec, seed, e), range(E)))
    shared = None
    if spec.shared_inter:
        Is = spec.shared_inter
        wg = rng(seed, _SGATE).standard_normal((H, 2 * Is), dtype=np.float32) * np.float32(0.02)
        wd = rng(seed, _SDOWN).standard_normal((Is, H), dtype=np.float32) * np.float32(0.02)
        shared = (quantize_pc(wg, spec.shared_bits), quantize_pc(wd, spec.shared_bits))
    expert_bias = None
    if spec.route_rule == ROUTE_GROUPED_SIGMOID:
        expert_bias = (rng(seed, _EBIAS).standard_normal(E, dtype=np.float32)
                       * np.float32(spec.expert_bias_std))
    shared_gate = None
    if spec.shared_gate:
        shared_gate = rng(seed, _SHGATE).standard_normal(H, dtype=np.float32) * np.float32(0.02)
    return Layer(spec, router, bias, [p[0] for p in pairs], [p[1] for p in pairs], shared,
                 expert_bias, shared_gate)


def make_input(spec: LayerSpec | str, tokens: int, seed: int = 0, stream: int = _X) -> np.ndarray:
    spec = CONFIGS[spec] if isinstance(spec, str) else spec
    return rng(seed, stream, tokens).standard_normal((tokens, spec.hidden), dtype=np.float32)


def small_spec(name: str, **kw) -> LayerSpec:
    """A reduced copy of a configuration for fast parity cases."""
    return replace(CONFIGS[name], **kw)
