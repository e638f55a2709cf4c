"""A bank ingested from a compressed-tensors checkpoint runs bit-identically
to the same bank built from the matrices directly (GPU, through the C ABI)."""
import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import checkpoint as CK
from open_rknpu2_lm_infer_b200 import synthetic as S
from open_rknpu2_lm_infer_b200.moe import Backend, QuantMatrix

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("routed", ["w4pc", "w8pc"])
def test_checkpoint_bank_matches_direct_bank(cuda, oracle, tmp_path, routed):
    spec = S.small_spec("c2", experts=16, routed=routed)
    layer = S.make_layer(spec, seed=12)
    H, I, bits = spec.hidden, spec.inter, 4 if routed == "w4pc" else 8
    prefix = "model.layers.0.mlp.experts"
    tensors = {}
    for e in range(spec.experts):
        codes = np.asarray(layer.gate[e].codes).reshape(H, 2 * I)
        sc = np.asarray(layer.gate[e].scales, np.float32)
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.gate_proj",
                                         QuantMatrix(bits, H, I, codes[:, :I].copy(), sc[:I])))
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.up_proj",
                                         QuantMatrix(bits, H, I, codes[:, I:].copy(), sc[I:])))
        tensors.update(CK.linear_tensors(f"{prefix}.{e}.down_proj", layer.down[e]))
    CK.write_safetensors(tmp_path / "model.safetensors", tensors)
    loader = CK.QuantLoader.open(tmp_path, CK.compressed_tensors_config(bits))
    gates, downs = loader.experts(prefix, spec.experts, H, I)
    T = 40
    x = S.make_input(spec, T, seed=13)
    outs = []
    for g, d in ((layer.gate, layer.down), (gates, downs)):
        be = Backend(device=0, max_rows=T)
        moe = be.load_moe(g, d, spec.top)
        router = be.router(layer.router, spec.top, layer.bias)
        out, ids, routes = moe.forward(router, x)
        outs.append(out)
        moe.close(); router.close(); be.close()
    assert np.array_equal(outs[0], outs[1])
    ref = oracle.OracleLayer(layer).forward(x)
    np.testing.assert_allclose(outs[1], ref, rtol=1e-2, atol=1e-3)
