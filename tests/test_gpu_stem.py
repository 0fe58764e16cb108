"""Conv stem on the device (vox_cuda_conv_stem_*) against the reference's
stream_conv_stem (golden tests/golden/stem.npz): chunks of 2, 150, 37, 1,
200, 64 and 5 mel frames, so the stride-2 residual, the conv0 tail and the
reference's tail after a one-frame chunk are all exercised.  Operands are
fp16 on the tensor cores (two convolutions: K = 384 and 3840)."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
import voxcuda as V
from conftest import load_golden, unpack

pytestmark = pytest.mark.gpu

STEM_TOL = 2e-3   # two fp16-operand tensor-core GEMMs with GELU (contract: 5e-3 per GEMM)


@pytest.fixture(scope="module", autouse=True)
def cuda():
    V.init()
    yield


def test_conv_stem_matches_reference():
    g = load_golden("stem")
    w = B.ConvStemWeights(seed=G.DEC_SEED)
    st = V.ConvStem(w.w0, w.b0, w.w1, w.b1, max_mel=512)
    rels = []
    for i, mel in enumerate(G.stem_chunks()):
        y = st.step(mel)
        assert y.shape[0] == int(g[f"chunk{i}_rows"])
        assert np.isfinite(y).all()
        if y.size:
            idx, val, _, _ = unpack(g, f"chunk{i}")
            rels.append(B.rel_l2(y.reshape(-1)[idx], val))
    print("conv stem rel-L2 per chunk:", rels)
    assert max(rels) < STEM_TOL, rels
    # a new stream starts from zero history again
    st.reset()
    y0 = st.step(G.stem_chunks()[0])
    idx, val, _, _ = unpack(g, "chunk0")
    assert B.rel_l2(y0.reshape(-1)[idx], val) < STEM_TOL
    st.free()


def test_conv_stem_capacity_error():
    w = B.ConvStemWeights(seed=1)
    st = V.ConvStem(w.w0, w.b0, w.w1, w.b1, max_mel=64)
    with pytest.raises(V.VoxCudaError):
        st.step(np.zeros((65, B.MEL_BINS), np.float32))
    st.free()
