"""Generates the committed golden fixtures from the CPU restatement.

Run from the repository root:  python tests/golden/make_golden.py
Each fixture stores the seeded inputs and quantised weights of a tiny layer and
every stage output of the restatement (router logits, ids, weights,
permutation, offsets, quantised activations, SwiGLU middle, middle codes,
per-assignment down outputs, final output). tests/test_golden.py checks that
the restatement still reproduces them bit for bit, and the GPU tests check the
C-ABI path against them.
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402
from open_rknpu2_lm_infer_b200 import synthetic as S  # noqa: E402

FIXTURES = {
    # name: (spec, tokens)
    "tiny_w4g32": (S.small_spec("c1", hidden=128, inter=64, experts=8, top=2), 16),
    "tiny_w8_shared": (S.small_spec("c3", hidden=128, inter=64, experts=8, top=2, routed="w8pc",
                                    shared_inter=128), 12),
}


def save(name, spec, T):
    layer = S.make_layer(spec, seed=2024)
    x = S.make_input(spec, T, seed=2024)
    res = S.make_input(spec, T, seed=2024, stream=5)
    out, d = O.OracleLayer(layer).forward(x, res, dump=True)
    arrays = dict(x=x, residual=res, router=layer.router, out=out)
    if layer.bias is not None:
        arrays["bias"] = layer.bias
    for i, (g, dn) in enumerate(zip(layer.gate, layer.down)):
        arrays[f"gate{i}_codes"], arrays[f"gate{i}_scales"] = g.codes, g.scales
        arrays[f"down{i}_codes"], arrays[f"down{i}_scales"] = dn.codes, dn.scales
    if layer.shared is not None:
        arrays["sgate_codes"], arrays["sgate_scales"] = layer.shared[0].codes, layer.shared[0].scales
        arrays["sdown_codes"], arrays["sdown_scales"] = layer.shared[1].codes, layer.shared[1].scales
    for k in ("logits", "ids", "weights", "perm", "offsets", "qx", "sx", "middle", "qm", "sm", "y"):
        arrays[f"ref_{k}"] = d[k]
    meta = np.array([spec.hidden, spec.inter, spec.experts, spec.top, spec.shared_inter, T,
                     {"w4g32": 0, "w4pc": 1, "w8pc": 2}[spec.routed]], np.int64)
    arrays["meta"] = meta
    path = Path(__file__).resolve().parent / f"{name}.npz"
    np.savez_compressed(path, **arrays)
    print(path, path.stat().st_size, "bytes")


if __name__ == "__main__":
    for name, (spec, T) in FIXTURES.items():
        save(name, spec, T)
