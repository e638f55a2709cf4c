"""The no-allocation router entry point (moe_b200_route_noalloc).

Callers that cannot call cudaMalloc (an engine whose own memory pool owns the
device, or a hot path that must not risk an allocation) use this entry point
instead of moe_b200_route_device, which needs a workspace. It must give the
same routing: this test calls it through the C ABI twice in a row, with
different inputs and sizes, and compares each result with the workspace
entry point's on the same inputs, within the tolerance of the other parity
tests. It lives in its own file so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import ATOL, RTOL, assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend

pytestmark = pytest.mark.gpu


def test_noalloc_router_matches_workspace_router(cuda):
    torch = cuda
    spec = S.small_spec("c3", experts=64, inter=64, shared_inter=0)
    layer = S.make_layer(spec, seed=77)
    be = Backend(device=0, max_rows=512)
    moe = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    lib = L.load()
    d_router = torch.from_numpy(layer.router).cuda()
    d_bias = torch.from_numpy(layer.bias).cuda()
    stream = torch.cuda.current_stream().cuda_stream

    for call, T in enumerate((300, 40)):  # two calls in a row, different sizes
        x = torch.from_numpy(S.make_input(spec, T, seed=100 + call)).cuda()
        ids_ref = torch.empty((T, spec.top), dtype=torch.int32, device="cuda")
        w_ref = torch.empty((T, spec.top), dtype=torch.float32, device="cuda")
        moe.route_device(router, T, x.data_ptr(), None, ids_ref.data_ptr(), w_ref.data_ptr(),
                         stream)
        ids = torch.full((T, spec.top), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, spec.top), -1.0, dtype=torch.float32, device="cuda")
        rc = lib.moe_b200_route_noalloc(x.data_ptr(), d_router.data_ptr(), d_bias.data_ptr(), T,
                                        spec.hidden, spec.experts, spec.top, L.ROUTER_NEON16,
                                        C.c_float(0.0), ids.data_ptr(), w.data_ptr(), stream)
        assert rc == L.OK, L.strerror(rc)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy()), f"call {call}: ids differ"
        assert_close(w.cpu().numpy(), w_ref.cpu().numpy(), rtol=RTOL, atol=ATOL,
                     what=f"call {call} routing weights")

    # a request beyond the fixed scratch is rejected before anything is launched
    rows = L.NOALLOC_MAX_LOGITS // spec.experts + 1
    rc = lib.moe_b200_route_noalloc(x.data_ptr(), d_router.data_ptr(), None, rows, spec.hidden,
                                    spec.experts, spec.top, L.ROUTER_NEON16, C.c_float(0.0),
                                    ids.data_ptr(), w.data_ptr(), stream)
    assert rc == L.ERR_NOALLOC_LIMIT
    assert "scratch" in L.strerror(rc)
    moe.close()
    router.close()
    be.close()
