"""The no-allocation router entry point (moe_b200_route_noalloc).

Callers that cannot call cudaMalloc (an engine whose own memory pool owns the
device, or a hot path that must not risk an allocation) use this entry point
instead of moe_b200_route_device, which needs a workspace. It must give the
same routing: this test calls it through the C ABI on several calls in a row,
with different inputs and sizes, and compares each result with the workspace
entry point's on the same inputs (ids exactly, weights within the tolerance of
the other parity tests) and with the CPU restatement of the reference's
router (logits in the same dot order, then routes()). The sizes cover both
router paths: fewer than 16 rows (the decode router, whose last CTA per token
routes it and resets the tile counter kept in the fixed scratch) and 16 or
more (the tile router and a routing kernel), in the NEON16 and the x86
sequential dot order. Device memory in use must not change across the calls.
It lives in its own file so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import ATOL, RTOL, assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend

pytestmark = pytest.mark.gpu

# (rows, dot order): two calls in a row of each router path, then the decode
# path at its largest size and the sequential order on both sides of 16 rows
CASES = [(300, L.ROUTER_NEON16), (40, L.ROUTER_NEON16), (1, L.ROUTER_NEON16),
         (5, L.ROUTER_NEON16), (15, L.ROUTER_NEON16), (7, L.ROUTER_SEQUENTIAL),
         (300, L.ROUTER_SEQUENTIAL)]


def _noalloc(lib, x, router, bias, T, spec, order, ids, w, stream, hidden=None):
    return lib.moe_b200_route_noalloc(
        x, router, bias, T, spec.hidden if hidden is None else hidden, spec.experts, spec.top,
        order, C.c_float(0.0), ids, w, stream)


def test_noalloc_router_matches_workspace_router_and_oracle(cuda, oracle):
    torch = cuda
    spec = S.small_spec("c3", experts=64, inter=64, shared_inter=0)
    layer = S.make_layer(spec, seed=77)
    be = Backend(device=0, max_rows=512)
    moe = be.load_moe(layer.gate, layer.down, spec.top)
    routers = {o: be.router(layer.router, spec.top, layer.bias, order=o)
               for o in (L.ROUTER_NEON16, L.ROUTER_SEQUENTIAL)}
    lib = L.load()
    d_router = torch.from_numpy(layer.router).cuda()
    d_bias = torch.from_numpy(layer.bias).cuda()
    stream = torch.cuda.current_stream().cuda_stream

    for call, (T, order) in enumerate(CASES):
        xh = S.make_input(spec, T, seed=100 + call)
        x = torch.from_numpy(xh).cuda()
        ids_ref = torch.empty((T, spec.top), dtype=torch.int32, device="cuda")
        w_ref = torch.empty((T, spec.top), dtype=torch.float32, device="cuda")
        moe.route_device(routers[order], T, x.data_ptr(), None, ids_ref.data_ptr(),
                         w_ref.data_ptr(), stream)
        ids = torch.full((T, spec.top), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, spec.top), -1.0, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        # the first call loads the library's module with its fixed scratch;
        # after it, a call must leave the device memory in use unchanged
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(lib, x.data_ptr(), d_router.data_ptr(), d_bias.data_ptr(), T, spec, order,
                      ids.data_ptr(), w.data_ptr(), stream)
        assert rc == L.OK, L.strerror(rc)
        torch.cuda.synchronize()
        if call > 0:
            assert torch.cuda.mem_get_info()[0] == free_before, f"call {call}: device memory changed"
        got_ids, got_w = ids.cpu().numpy(), w.cpu().numpy()
        assert np.array_equal(got_ids, ids_ref.cpu().numpy()), f"call {call}: ids differ"
        assert_close(got_w, w_ref.cpu().numpy(), rtol=RTOL, atol=ATOL,
                     what=f"call {call} routing weights")
        # the CPU restatement: logits in the same dot order, then routes()
        logits = oracle.router_logits(xh, layer.router, layer.bias, order=order)
        o_ids, o_w = oracle.routes(logits, spec.top)
        assert np.array_equal(got_ids, o_ids), f"call {call}: ids differ from the restatement"
        assert_close(got_w, o_w, rtol=RTOL, atol=ATOL, what=f"call {call} weights vs restatement")

    # rejected before anything is launched (the outputs stay untouched)
    ids.fill_(-7)
    # beyond the fixed scratch
    rows = L.NOALLOC_MAX_LOGITS // spec.experts + 1
    rc = _noalloc(lib, x.data_ptr(), d_router.data_ptr(), None, rows, spec,
                  L.ROUTER_NEON16, ids.data_ptr(), w.data_ptr(), stream)
    assert rc == L.ERR_NOALLOC_LIMIT
    assert "scratch" in L.strerror(rc)
    # a hidden width the 16-byte row loads cannot take
    rc = _noalloc(lib, x.data_ptr(), d_router.data_ptr(), None, 4, spec, L.ROUTER_NEON16,
                  ids.data_ptr(), w.data_ptr(), stream, hidden=spec.hidden - 4)
    assert rc == L.ERR_UNSUPPORTED
    # a small batch whose router rows do not fit shared memory
    rc = _noalloc(lib, x.data_ptr(), d_router.data_ptr(), None, 4, spec, L.ROUTER_NEON16,
                  ids.data_ptr(), w.data_ptr(), stream, hidden=5696)
    assert rc == L.ERR_UNSUPPORTED
    # input and router rows must start on 16 bytes (a row slice 4 bytes in)
    rc = _noalloc(lib, x.data_ptr() + 4, d_router.data_ptr(), None, 4, spec, L.ROUTER_NEON16,
                  ids.data_ptr(), w.data_ptr(), stream)
    assert rc == L.ERR_INVALID
    rc = _noalloc(lib, x.data_ptr(), d_router.data_ptr() + 4, None, 4, spec, L.ROUTER_NEON16,
                  ids.data_ptr(), w.data_ptr(), stream)
    assert rc == L.ERR_INVALID
    torch.cuda.synchronize()
    assert bool((ids == -7).all()), "a rejected call wrote its outputs"
    moe.close()
    for r in routers.values():
        r.close()
    be.close()
