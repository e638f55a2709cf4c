"""The fused small-batch layer (csrc/gemv.cu, decode_layer_kernel): at one
token on a group-32 bank, moe_b200_forward_device runs router, routing, both
GEMVs and the combine as one cooperative launch (from two tokens on, the
router kernels and the two GEMV kernels, measured faster there). Either way it
must give, bit for bit, the ids, routing weights and outputs of the unfused
path (the router kernels, moe_b200_route_device, then the two GEMV kernels,
moe_b200_run_device), for every router rule the fused launch serves: NEON16
and TF32 dot orders, softmax top-k with and without pruning, Ling's grouped
sigmoid routing.
"""
import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError

pytestmark = pytest.mark.gpu

SPEC = S.small_spec("c2", experts=32)

ROUTERS = {
    "neon16": {},
    "tf32": {"order": L.ROUTER_TF32},
    "pruned": {"min_weight": 0.12},
    "grouped": {"rule": L.ROUTE_GROUPED_SIGMOID, "groups": 8, "top_groups": 4,
                "routing_scale": 2.5},
}


@pytest.mark.parametrize("name", list(ROUTERS))
@pytest.mark.parametrize("T", [1, 3, 4])
def test_fused_layer_equals_router_plus_gemvs(cuda, name, T):
    torch = cuda
    layer = S.make_layer(SPEC, seed=71)
    kw = dict(ROUTERS[name])
    if kw.get("rule") == L.ROUTE_GROUPED_SIGMOID:
        kw["expert_bias"] = np.random.default_rng(3).normal(0, 0.1, SPEC.experts).astype(np.float32)
        bias = None
    else:
        bias = layer.bias
    be = Backend(device=0, max_rows=8)
    moe = be.load_moe(layer.gate, layer.down, SPEC.top)
    router = be.router(layer.router, SPEC.top, bias, **kw)
    x = torch.from_numpy(S.make_input(SPEC, T, seed=72)).cuda()
    s = torch.cuda.current_stream().cuda_stream
    lib, ws = be.lib, moe.workspace

    out_f = torch.empty_like(x)
    n0 = lib.moe_b200_workspace_launches(ws)
    moe.forward_device(router, T, x.data_ptr(), None, out_f.data_ptr(), s)
    launches = lib.moe_b200_workspace_launches(ws) - n0
    torch.cuda.synchronize()
    moe.status()
    ids_f = torch.empty((T, SPEC.top), dtype=torch.int32, device="cuda")
    w_f = torch.empty((T, SPEC.top), dtype=torch.float32, device="cuda")
    for buf, name_ in ((ids_f, "ids"), (w_f, "routes")):
        ptr, _ = moe.buffer(name_)
        src = torch.as_tensor(_View(ptr, (T, SPEC.top), "<i4" if name_ == "ids" else "<f4"),
                              device="cuda")
        buf.copy_(src)
    if T == 1:
        assert launches == 1, "the one-token layer should be one launch"
    else:
        assert launches > 1, "from two tokens on, the router and the GEMV kernels"

    ids_u = torch.empty_like(ids_f)
    w_u = torch.empty_like(w_f)
    out_u = torch.empty_like(x)
    moe.route_device(router, T, x.data_ptr(), None, ids_u.data_ptr(), w_u.data_ptr(), s)
    moe.run_device(x.data_ptr(), ids_u.data_ptr(), w_u.data_ptr(), out_u.data_ptr(), T, s)
    torch.cuda.synchronize()
    moe.status()
    assert torch.equal(ids_f, ids_u)
    assert torch.equal(w_f.view(torch.int32), w_u.view(torch.int32))
    assert torch.equal(out_f.view(torch.int32), out_u.view(torch.int32))
    if name == "pruned":
        assert (w_u == 0).any(), "the threshold should prune some routes"
    # a second call reuses the grid barrier and the row-max scratch
    out_2 = torch.empty_like(x)
    moe.forward_device(router, T, x.data_ptr(), None, out_2.data_ptr(), s)
    torch.cuda.synchronize()
    moe.status()
    assert torch.equal(out_2.view(torch.int32), out_f.view(torch.int32))
    moe.close(); router.close(); be.close()


class _View:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


@pytest.mark.parametrize("T", [1, 4, 40])
def test_non_finite_activations_are_flagged_and_the_next_call_is_clean(cuda, T):
    """A NaN or infinite activation makes the router logits non-finite: the
    call reports MOE_B200_ERR_NONFINITE (the fused small-batch layer at one
    token, the router kernels and the GEMVs at 4, the tile router and pipeline
    at 40 tokens), and the next clean call runs
    normally with the same result as before."""
    layer = S.make_layer(SPEC, seed=73)
    be = Backend(device=0, max_rows=64)
    moe = be.load_moe(layer.gate, layer.down, SPEC.top)
    router = be.router(layer.router, SPEC.top, layer.bias)
    x = S.make_input(SPEC, T, seed=74)
    ref, _, _ = moe.forward(router, x)
    for bad in (np.nan, np.inf):
        xb = x.copy()
        xb[T - 1, 5] = bad
        with pytest.raises(MoeError) as e:
            moe.forward(router, xb)
        assert e.value.code == L.ERR_NONFINITE
        out, _, _ = moe.forward(router, x)
        assert np.array_equal(out.view(np.int32), ref.view(np.int32))
    moe.close(); router.close(); be.close()
