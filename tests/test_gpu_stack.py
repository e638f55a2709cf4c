"""The layer stack's pre-norm (csrc/norm.cu) and a short stack of MoE layers.

RMSNorm is bit-exact with the restatement (src/ops/norm.rs:81-106: the squares
summed in column order, then the correctly rounded divide, square root and
products). The stack, x = RMSNorm(h), h = h + MoE(x) per layer
(src/model/qwen35/decoder.rs:180-217), matches the restatement's stack within
1e-2 rel / 1e-3 abs.
"""
import numpy as np
import pytest

from conftest import assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError
from open_rknpu2_lm_infer_b200.stack import MoeStack

pytestmark = pytest.mark.gpu


def _lib():
    return L.load()


@pytest.mark.parametrize("rows,width,zc", [(1, 64, 0), (5, 1000, 1), (33, 2048, 0), (70, 1536, 1)])
def test_rms_norm_bit_exact(cuda, oracle, rows, width, zc):
    torch = cuda
    rng = np.random.default_rng(rows * 7 + width)
    x = (rng.standard_normal((rows, width)) * rng.uniform(0.1, 30, (rows, 1))).astype(np.float32)
    if rows > 2:
        x[2] = 0.0  # zero row: scale 1/sqrt(eps), output 0
    w = (rng.standard_normal(width) * 0.1 + (0 if zc else 1)).astype(np.float32)
    ref = oracle.rms_norm(x, w, 1e-6, bool(zc))
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.empty_like(dx)
    s = torch.cuda.current_stream().cuda_stream
    assert _lib().moe_b200_rms_norm(dx.data_ptr(), dw.data_ptr(), rows, width, 1e-6, zc,
                                    out.data_ptr(), s) == 0
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # in place
    assert _lib().moe_b200_rms_norm(dx.data_ptr(), dw.data_ptr(), rows, width, 1e-6, zc,
                                    dx.data_ptr(), s) == 0
    assert np.array_equal(dx.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_rms_norm_rejects_what_the_reference_rejects(cuda):
    torch = cuda
    d = torch.zeros(4, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    for width, eps in ((0, 1e-6), (64, 0.0), (64, -1.0), (64, float("inf")), (64, float("nan"))):
        assert _lib().moe_b200_rms_norm(d.data_ptr(), w.data_ptr(), 4, width, eps, 0,
                                        d.data_ptr(), 0) == L.ERR_INVALID
    assert _lib().moe_b200_rms_norm(d.data_ptr(), w.data_ptr(), 0, 64, 1e-6, 0, d.data_ptr(), 0) == 0


def test_stack_matches_the_restatement(cuda, oracle):
    torch = cuda
    spec = S.small_spec("c2", experts=32)
    n_layers, T = 3, 37
    be = Backend(device=0, max_rows=64)
    layers, olayers, norms = [], [], []
    rng = np.random.default_rng(5)
    for i in range(n_layers):
        lay = S.make_layer(spec, seed=80 + i)
        layers.append((be.load_moe(lay.gate, lay.down, spec.top, exact=True),
                       be.router(lay.router, spec.top, lay.bias)))
        olayers.append(oracle.OracleLayer(lay))
        norms.append((1 + rng.standard_normal(spec.hidden) * 0.02).astype(np.float32))
    stack = MoeStack(layers, norms, eps=1e-6)
    h = S.make_input(spec, T, seed=90)
    got = stack.forward(h)
    ref = h
    for ol, w in zip(olayers, norms):
        ref = ol.forward(oracle.rms_norm(ref, w, 1e-6), ref)
    assert_close(got, ref, what="3-layer stack")
    # the device entry leaves its input alone and fills `out`
    dh = torch.from_numpy(h).cuda()
    out = torch.empty_like(dh)
    stack.forward_tensor(dh, out=out)
    torch.cuda.synchronize()
    assert np.array_equal(dh.cpu().numpy(), h)
    assert np.array_equal(out.cpu().numpy(), got)
    with pytest.raises(ValueError):
        MoeStack(layers, norms[:2])
    with pytest.raises(ValueError):
        MoeStack(layers, [np.ones(7, np.float32)] * n_layers)
    for moe, r in layers:
        moe.close(); r.close()
    be.close()
