"""Expert slot bank and paging on the GPU (moe_b200_slots_create,
moe_b200_export_expert / import_expert / swap_slots; experts.Pager).

A bank assembled slot by slot from exported blobs, in a permuted slot order,
must compute the resident layer bit for bit once the expert ids are mapped to
their slots; so must the pager, with a window smaller than the demand. Both
are also checked against the CPU restatement of the reference layer (within
1e-2 rel / 1e-3 abs)."""
import numpy as np
import pytest

from conftest import assert_close
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.experts import Geometry, Pager, Store, Writer
from open_rknpu2_lm_infer_b200.moe import Backend, MoeError

pytestmark = pytest.mark.gpu

FORMATS = {"w4g32": L.W4_G32_FP16, "w4pc": L.W4_PER_CHANNEL, "w8pc": L.W8_PER_CHANNEL}


@pytest.mark.parametrize("routed", ["w4g32", "w4pc", "w8pc"])
def test_slot_bank_from_blobs_matches_resident_bank(cuda, oracle, routed):
    spec = S.small_spec("c2", experts=16, routed=routed)
    layer = S.make_layer(spec, seed=21)
    T = 33
    x = S.make_input(spec, T, seed=22)
    be = Backend(device=0, max_rows=T)
    moe = be.load_moe(layer.gate, layer.down, spec.top)
    router = be.router(layer.router, spec.top, layer.bias)
    ref, ids, routes = moe.forward(router, x)

    def run(bank, slot_ids):
        out = np.empty_like(x)
        bank.run(x, np.ascontiguousarray(slot_ids, np.int32), routes, out, T)
        return out

    assert np.array_equal(run(moe, ids), ref)
    blobs = [moe.export(e) for e in range(spec.experts)]
    assert all(len(b) == moe.blob_bytes() for b in blobs)
    assert moe.blob_version() == L.load().moe_b200_blob_version() == 1
    perm = np.random.default_rng(3).permutation(spec.experts)  # expert e -> slot perm[e]
    slots = be.moe_packed(spec.hidden, spec.inter, spec.experts, spec.top, FORMATS[routed])
    for e in range(spec.experts):
        slots.import_(int(perm[e]), blobs[e])
    got = run(slots, perm[ids])
    assert np.array_equal(got, ref)
    # the restatement with the same routing, on the original expert ids
    assert_close(got, oracle.OracleLayer(layer).run(x, ids, routes), what=f"{routed} slot bank")
    # blobs round-trip through the slot bank unchanged
    assert slots.export(int(perm[5])) == blobs[5]
    # a staging bank: promote swaps a staged expert into a live slot
    staging = slots.import_bank(2)
    staging.import_(1, blobs[3])
    slots.promote(int(perm[3]), staging, 1)  # the same expert: output unchanged
    assert np.array_equal(run(slots, perm[ids]), ref)
    slots.promote(int(perm[3]), staging, 1)
    slots.promote(int(perm[3]), staging, 1)
    assert slots.export(int(perm[3])) == blobs[3]
    # the blob header pins format and geometry
    bad = bytearray(blobs[0])
    bad[12] ^= 1
    with pytest.raises(MoeError):
        slots.import_(0, bytes(bad))
    with pytest.raises(MoeError):
        slots.import_(0, blobs[0][:-16])
    staging.close(); slots.close(); moe.close(); router.close(); be.close()


@pytest.mark.parametrize("slots_n,T", [(16, 1), (8, 40), (8, 1)])
def test_pager_matches_resident_layer(cuda, oracle, tmp_path, slots_n, T):
    torch = cuda
    spec = S.small_spec("c2", experts=32)
    layer = S.make_layer(spec, seed=31)
    be = Backend(device=0, max_rows=T * spec.top)
    # exact group sums in both GEMMs: the resident small-batch path and the
    # pager's expert rows then compute the same values whatever the row count
    moe = be.load_moe(layer.gate, layer.down, spec.top, exact=True)
    router = be.router(layer.router, spec.top, layer.bias)
    g = Geometry(native_version=moe.blob_version(), layers=1, experts=spec.experts,
                 hidden=spec.hidden, intermediate=spec.inter, down_bits=4)
    w = Writer(tmp_path, g, [], moe.blob_bytes())
    for e in range(spec.experts):
        w.write(0, e, moe.export(e))
    w.finish()
    store = Store(tmp_path, g, [])
    pager = Pager(be, store, 0, slots_n, spec.top, L.W4_G32_FP16_EXACT, max_rows=T)
    for step in range(3):
        x = S.make_input(spec, T, seed=40 + step)
        res = S.make_input(spec, T, seed=50 + step, stream=5)
        ref, ids, routes = moe.forward(router, x, res)
        out = pager.run(torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                        torch.from_numpy(routes).cuda(), torch.from_numpy(res).cuda())
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ref), f"step {step}"
        assert_close(out.cpu().numpy(), oracle.OracleLayer(layer).forward(x, res),
                     what=f"pager step {step} vs restatement")
    st = pager.stats
    assert st.calls == 3 and st.imports >= min(slots_n, st.unique_demand // 3)
    if slots_n < spec.experts and T > 1:
        assert st.groups > st.calls  # the demand exceeded the window
    pager.close(); store.close(); moe.close(); router.close(); be.close()
