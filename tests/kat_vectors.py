"""Known-answer inputs ported from the reference's own tests (shared by the
oracle KATs and the GPU parity tests).

Ling grouped routing: src/model/ling3tiny/moe.rs:404-493
(selection_matches_sorted_oracle_with_ties_and_reused_scratch and
group_bias_selects_experts_but_weights_use_original_sigmoid). The official
Ling config fixes routing_scale = 2.5 (src/model/ling3tiny/config.rs:160-163).
"""
from __future__ import annotations

import numpy as np

LING_SCALE = 2.5
# (experts, groups, top_groups, top) of the selection KAT
LING_GEOMETRIES = [(128, 8, 4, 8), (8, 4, 4, 1), (8, 4, 2, 4)]
LING_STEPS = 100


def ling_step(experts: int, step: int) -> tuple[np.ndarray, np.ndarray]:
    """Logits and bias of one step: zeros every 10th step, else the formulas
    ((i*17 + step*31) % 29) * 0.25 - 3.5 and ((i*13 + step*7) % 11) * 0.125 - 0.625."""
    i = np.arange(experts)
    if step % 10 == 0:
        return np.zeros(experts, np.float32), np.zeros(experts, np.float32)
    logits = (((i * 17 + step * 31) % 29).astype(np.float32) * np.float32(0.25)
              - np.float32(3.5)).astype(np.float32)
    bias = (((i * 13 + step * 7) % 11).astype(np.float32) * np.float32(0.125)
            - np.float32(0.625)).astype(np.float32)
    return logits, bias


LING_BIAS_CASE = dict(
    geometry=(8, 4, 2, 3),
    logits=np.array([3.0, 2.0, -2.0, -1.0, 0.0, 0.5, 4.0, 3.5], np.float32),
    bias=np.array([0.0, 0.0, 3.0, 3.0, 4.0, 4.0, 0.0, 0.0], np.float32),
    ids=[5, 4, 3],
    weight_logits=[0.5, 0.0, -1.0],
)


def total_key(v: np.ndarray) -> np.ndarray:
    """Rust f32::total_cmp as a signed integer key."""
    b = np.asarray(v, np.float32).view(np.int32).astype(np.int64)
    return b ^ ((b >> 31) & 0x7FFFFFFF)


def ling_sorted_oracle(logits, bias, groups, top_groups, top, scale, sigmoid):
    """The reference test's own sorted computation (moe.rs:433-466), with the
    sigmoid given (the reference's, restated)."""
    experts = logits.size
    scores = np.array([sigmoid(float(x)) for x in logits], np.float32)
    selected = (scores + bias).astype(np.float32)
    width = experts // groups
    gscores = []
    for g in range(groups):
        v = selected[g * width:(g + 1) * width]
        order = sorted(range(width), key=lambda j: -total_key(v[j]))
        gscores.append(np.float32(v[order[0]] + v[order[1]]))
    gk = total_key(np.array(gscores, np.float32))
    chosen_groups = sorted(range(groups), key=lambda g: (-gk[g], g))[:top_groups]
    sk = total_key(selected)
    cand = [e for e in range(experts) if e // width in chosen_groups]
    ref = sorted(cand, key=lambda e: (-sk[e], e))[:top]
    s = np.float32(0.0)
    for e in ref:
        s = np.float32(s + scores[e])
    s = np.float32(s + np.float32(1e-20))
    w = [np.float32(np.float32(scores[e] / s if top > 1 else scores[e]) * np.float32(scale))
         for e in ref]
    return np.array(ref, np.int32), np.array(w, np.float32)
