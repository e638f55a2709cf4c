"""MoeStack's argument checks (open_rknpu2_lm_infer_b200/stack.py), which run
before any device work: one RMSNorm weight per layer, one hidden size, a
finite positive epsilon (src/ops/norm.rs:88-95), weights of the hidden size."""
from types import SimpleNamespace

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200.stack import MoeStack


def _layer(hidden):
    return (SimpleNamespace(hidden=hidden, owner=SimpleNamespace(lib=None)), None)


def test_stack_rejects_mismatched_arguments():
    w = np.ones(64, np.float32)
    with pytest.raises(ValueError, match="one RMSNorm weight per layer"):
        MoeStack([_layer(64), _layer(64)], [w])
    with pytest.raises(ValueError, match="one RMSNorm weight per layer"):
        MoeStack([], [])
    with pytest.raises(ValueError, match="hidden size"):
        MoeStack([_layer(64), _layer(32)], [w, w])
    for eps in (0.0, -1e-6, float("inf"), float("nan")):
        with pytest.raises(ValueError, match="epsilon"):
            MoeStack([_layer(64)], [w], eps=eps)
    with pytest.raises(ValueError, match="weight shape"):
        MoeStack([_layer(64)], [np.ones(63, np.float32)])
