"""The algorithmic-bytes formula behind bench.py's HBM roofline figures,
checked against the worked examples of the measurement plan (per layer call,
uniform routing, residual fused): c2 at 1 token 22.30 MB (8 experts hit),
c5 with int4 group-32 routed experts at 1 token 28.9 MB (8 experts + the int8
shared expert), c5 with int8 routed experts at 256 tokens ~829 MB (all 256
experts hit; the plan's 827.1 MB leaves the fused residual out)."""
import importlib.util
from pathlib import Path

import pytest

from open_rknpu2_lm_infer_b200 import synthetic as S

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("name,T,U,mb,tol", [("c2", 1, 8, 22.30, 0.01), ("c5_w4", 1, 8, 28.9, 0.05),
                                             ("c5_w8", 256, 256, 829.5, 0.5)])
def test_layer_bytes_match_the_plan(name, T, U, mb, tol):
    b = _bench().spec_bytes(S.CONFIGS[name], T, U)
    assert abs(b / 1e6 - mb) <= tol, b / 1e6


def test_residual_is_the_only_difference_from_the_plan_at_256_tokens():
    spec = S.CONFIGS["c5_w8"]
    b = _bench().spec_bytes(spec, 256, 256)
    assert abs((b - 256 * spec.hidden * 4) / 1e6 - 827.4) <= 0.3
