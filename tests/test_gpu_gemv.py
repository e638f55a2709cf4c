"""The small-batch (decode) path of group-32 banks (csrc/gemv.cu).

Up to four tokens per call run as grouped GEMVs on exact int32 group sums, so
each token's output must equal, bit for bit, the same token's output from the
exact tensor-core path (MOE_B200_W4_G32_FP16_EXACT at five tokens, where the
tensor-core path runs): tokens are computed independently of each other. The
stages are checked against the restatement: requantised middle codes from the
GPU's own middle values, and expert rows from the GPU's own middle codes, bit
for bit.
"""
import numpy as np
import pytest

from conftest import assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError

pytestmark = pytest.mark.gpu

SPECS = {"c2_e32": S.small_spec("c2", experts=32), "c2": S.CONFIGS["c2"],
         "c1": S.CONFIGS["c1"]}


class _CAI:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


def _view(torch, moe, name, shape, typestr):
    ptr, nbytes = moe.buffer(name)
    return torch.as_tensor(_CAI(ptr, shape, typestr), device="cuda").cpu().numpy()


@pytest.mark.parametrize("name", ["c2_e32", "c2", "c1"])
def test_small_batches_equal_the_exact_tensor_core_path(cuda, name):
    spec = SPECS[name]
    layer = S.make_layer(spec, seed=61)
    x = S.make_input(spec, 5, seed=62)
    res = S.make_input(spec, 5, seed=63, stream=5)
    be = Backend(device=0, max_rows=8)
    exact = be.load_moe(layer.gate, layer.down, spec.top, exact=True)
    fast = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    ref, ids5, _ = exact.forward(router, x, res)  # 5 tokens: tensor-core path
    for T in (1, 2, 4):
        for moe in (exact, fast):
            out, ids, _ = moe.forward(router, x[:T], res[:T])
            assert np.array_equal(ids, ids5[:T])
            assert np.array_equal(out, ref[:T]), f"T={T}"
    exact.close(); fast.close(); router.close(); be.close()


def test_small_batch_stages_are_the_restatement(cuda, oracle):
    torch = cuda
    spec = SPECS["c2_e32"]
    layer = S.make_layer(spec, seed=64)
    T, k, H, I = 3, spec.top, spec.hidden, spec.inter
    x = S.make_input(spec, T, seed=65)
    be = Backend(device=0, max_rows=8)
    moe = be.load_moe(layer.gate, layer.down, k)
    router = be.router(layer.router, k, layer.bias)
    out, ids, routes = moe.forward(router, x)
    torch.cuda.synchronize()
    middle = _view(torch, moe, "gate_up", (T * k, I), "<f4")
    Ki = moe.buffer("q_m")[1] // (8 * k)  # row stride of the code buffer (max_rows 8)
    q_m = _view(torch, moe, "q_m", (T * k, Ki), "|i1")[:, :I]
    s_m = _view(torch, moe, "s_m", (T * k,), "<f4")
    y = _view(torch, moe, "y", (T * k, H), "<f4")
    # requantisation of the GPU's middle values, bit for bit
    q_ref, s_ref = oracle.quantize(middle)
    assert np.array_equal(q_m, q_ref) and np.array_equal(s_m, s_ref)
    # middle values: the restatement's SwiGLU of the exact gate/up (expf may differ by an ulp)
    qx, sx = oracle.quantize(x)
    for a in range(T * k):
        e = int(ids.reshape(-1)[a])
        gu = oracle.gemm_dequant(qx[a // k][None, :], sx[a // k:a // k + 1], layer.gate[e])
        assert_close(middle[a], oracle.swiglu(gu, I)[0], rtol=1e-5, atol=1e-6, what="middle")
        # expert rows from the GPU's own middle codes, bit for bit
        y_ref = oracle.gemm_dequant(q_m[a][None, :], s_m[a:a + 1], layer.down[e])[0]
        assert np.array_equal(y[a], y_ref), f"assignment {a}"
    ref = oracle.OracleLayer(layer).forward(x)
    assert_close(out, ref, what="small-batch output")
    moe.close(); router.close(); be.close()


def test_small_batch_pruning_and_bad_routes(cuda, oracle):
    torch = cuda
    spec = SPECS["c2_e32"]
    layer = S.make_layer(spec, seed=66)
    T = 3
    x = S.make_input(spec, T, seed=67)
    be = Backend(device=0, max_rows=8)
    moe = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias, min_weight=0.12)
    out, ids, routes = moe.forward(router, x)
    assert (routes == 0).any(), "the threshold should prune some routes"
    ref = oracle.OracleLayer(layer, min_weight=0.12).forward(x)
    assert_close(out, ref, what="pruned small-batch output")
    # the device path flags a negative route and an out-of-range id
    dx = torch.from_numpy(x).cuda()
    dout = torch.empty_like(dx)
    bad_w = routes.copy(); bad_w[1, 2] = -0.5
    d_ids, d_w = torch.from_numpy(ids).cuda(), torch.from_numpy(bad_w).cuda()  # kept alive
    moe.run_device(dx.data_ptr(), d_ids.data_ptr(), d_w.data_ptr(), dout.data_ptr(), T,
                   torch.cuda.current_stream().cuda_stream)
    with pytest.raises(MoeError) as e:
        moe.status()
    assert e.value.code == L.ERR_BAD_ROUTE
    bad_id = ids.copy(); bad_id[0, 0] = spec.experts + 3
    w1 = np.where(routes > 0, routes, 0.1).astype(np.float32)
    d_ids, d_w = torch.from_numpy(bad_id).cuda(), torch.from_numpy(w1).cuda()
    moe.run_device(dx.data_ptr(), d_ids.data_ptr(), d_w.data_ptr(), dout.data_ptr(), T,
                   torch.cuda.current_stream().cuda_stream)
    with pytest.raises(MoeError) as e:
        moe.status()
    assert e.value.code == L.ERR_BAD_EXPERT
    # and the path recovers: the next call is clean and correct
    out2, _, _ = moe.forward(router, x)
    moe.status()
    assert np.array_equal(out2, out)
    moe.close(); router.close(); be.close()
