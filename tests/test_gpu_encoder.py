"""Encoder chunk (tcgen05 GEMMs + windowed fp16 flash attention + fp16 ring)
and adapter against the reference's golden vectors and the oracle.

The GEMMs round activations (and the bf16 weights, exactly) to fp16 and
attention runs on fp16 inputs; over 32 residual layers the encoder output
stays within ENC_TOL of the fp32 reference."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
import voxcuda as V
from conftest import load_golden, unpack

pytestmark = pytest.mark.gpu

ENC_TOL = 2e-3       # 32-layer encoder output rel-L2 vs the fp32 reference (measured ~4.4e-4)
ADAPTER_TOL = 1e-2   # adapter (2 tensor-core GEMMs) on identical inputs


@pytest.fixture(scope="module", autouse=True)
def cuda():
    V.init()
    yield


def make_gpu_encoder(ew):
    layers = [tuple(ew.layer_w[i]) + tuple(ew.layer_b[i]) + tuple(ew.layer_n[i])
              for i in range(ew.n_layers)]
    return V.Encoder(layers, ew.norm, ew.adapter0, ew.adapter1)


@pytest.fixture(scope="module")
def enc_w():
    return B.EncoderWeights(seed=G.DEC_SEED)


@pytest.fixture(scope="module")
def gpu_enc(enc_w):
    e = make_gpu_encoder(enc_w)
    yield e
    e.free()


def sampled_rel(arr, g, prefix):
    idx, val, _, size = unpack(g, prefix)
    flat = np.asarray(arr, np.float32).reshape(-1)
    assert flat.size == size
    return B.rel_l2(flat[idx], val)


def test_encoder_chunks_match_reference(gpu_enc):
    """Chunks of 100, 37, 700, 100 rows: the last two cross the 750-row window
    (the reference compacts its cache before the fourth)."""
    g = load_golden("encoder")
    st = gpu_enc.state(max_chunk=1024)
    rels = []
    for i, x in enumerate(G.enc_chunks()):
        y = st.step(x)
        assert np.isfinite(y).all()
        rels.append(sampled_rel(y, g, f"chunk{i}"))
    print("encoder chunk rel-L2 vs reference:", rels)
    assert max(rels) < ENC_TOL, rels
    assert st.position == sum(G.ENC_CHUNKS)
    st.free()


def test_encoder_benchmark_chunks_match_reference(gpu_enc):
    """The benchmarked chunk sizes with the bench's
    max_chunk of 1500: a 750-row history, then 500 rows and 1500 rows, each
    attending a full 750-row window (golden encoder_big.npz from the
    reference's vox_encoder_forward_incremental)."""
    g = load_golden("encoder_big")
    st = gpu_enc.state(max_chunk=1500)
    rels = []
    for i, x in enumerate(G.enc_big_chunks()):
        y = st.step(x)
        assert np.isfinite(y).all()
        flat = y.reshape(-1)
        assert flat.size == int(g[f"chunk{i}_size"])
        rels.append(B.rel_l2(flat[G.sample_idx(flat.size)], g[f"chunk{i}_val"]))
    print("encoder 750/500/1500-row chunks rel-L2 vs reference:", rels)
    assert max(rels) < ENC_TOL, rels
    assert st.position == sum(G.ENC_BIG_CHUNKS)
    st.free()


@pytest.mark.parametrize("pair", ["0", "1"])
def test_encoder_epilogue_paths_agree(pair, monkeypatch):
    """The TMA-store epilogue (staged tiles, TMA reduce-add for the residual)
    and the direct-store epilogue compute the same values in the same order:
    outputs agree bit for bit, also across the ring's wrap and ragged tails."""
    monkeypatch.setenv("VOX_CUDA_TC_PAIR", pair)
    ew = B.EncoderWeights(seed=7, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    outs = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("VOX_CUDA_TC_TMA_OUT", mode)
        st = e.state(max_chunk=256)
        ys = []
        for i, n in enumerate([64, 200, 3, 250, 130, 250, 256, 77]):   # wraps the 1006-slot ring
            ys.append(st.step(B.normal_f32((n, B.ENC_DIM), 950 + i)))
        outs[mode] = ys
        st.free()
    e.free()
    for a, b in zip(outs["1"], outs["0"]):
        assert np.isfinite(a).all()
        assert np.array_equal(a, b)


def test_encoder_attention_kernels_agree(monkeypatch):
    """The tcgen05 attention (S and P.V in TMEM, fp16 P) and the mma.sync
    flash attention on the same chunks, across the window and the ring's
    wrap: the same math with different roundings of P and of exp."""
    ew = B.EncoderWeights(seed=9, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    outs = {}
    for mode in ("tc", "mma"):
        monkeypatch.setenv("VOX_CUDA_ENC_ATTN", mode)
        st = e.state(max_chunk=256)
        ys = []
        for i, n in enumerate([64, 200, 3, 250, 130, 250, 256, 77, 129]):
            ys.append(st.step(B.normal_f32((n, B.ENC_DIM), 990 + i)))
        outs[mode] = ys
        st.free()
    e.free()
    for i, (a, b) in enumerate(zip(outs["tc"], outs["mma"])):
        assert np.isfinite(a).all()
        assert B.rel_l2(a, b) < 2e-3, (i, B.rel_l2(a, b))


def test_encoder_split_k_matches_unsplit(monkeypatch):
    """Small chunks run their GEMMs split along K: by default the slices of a
    tile are one thread-block cluster summed through distributed shared
    memory in rank order (one or two row tiles here: 100, 3, 256, 64 rows);
    with VOX_CUDA_TC_CLUSTER=-1 through the global workspace (fp32 partials
    summed in a fixed slice order by the last slice to finish).  Against the
    same chunks with split-K off (VOX_CUDA_TC_KSPLIT=1) only the fp32
    summation grouping differs; a second run of the default is bit-identical."""
    ew = B.EncoderWeights(seed=10, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    outs = {}
    for mode, ks, cl in (("cluster", "", ""), ("workspace", "", "-1"), ("off", "1", ""), ("again", "", "")):
        monkeypatch.setenv("VOX_CUDA_TC_KSPLIT", ks)
        monkeypatch.setenv("VOX_CUDA_TC_CLUSTER", cl)
        st = e.state(max_chunk=256)
        outs[mode] = [st.step(B.normal_f32((n, B.ENC_DIM), 1010 + i)) for i, n in enumerate([100, 3, 256, 64])]
        st.free()
    e.free()
    for i in range(4):
        a = outs["cluster"][i]
        assert np.isfinite(a).all()
        assert np.array_equal(a, outs["again"][i]), i
        for other in ("workspace", "off"):
            assert B.rel_l2(a, outs[other][i]) < 2e-3, (i, other, B.rel_l2(a, outs[other][i]))


def test_folded_norm_matches_separate_norm_pass_and_oracle(monkeypatch):
    """The RMSNorms folded into the GEMMs (the residual epilogues write
    fp16(x * w) and per-chunk sums of squares, the consumers scale their rows
    by 1 / rms) against the separate normalisation pass
    (VOX_CUDA_ENC_FOLD_NORM=0) and the oracle: ragged chunks, the single-state
    path and the batched one."""
    ew = B.EncoderWeights(seed=16, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sizes = [100, 37, 256, 3]
    xs = [B.normal_f32((n, B.ENC_DIM), 1160 + i) for i, n in enumerate(sizes)]
    outs = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("VOX_CUDA_ENC_FOLD_NORM", mode)
        st = e.state(max_chunk=256)
        outs[mode] = [st.step(x) for x in xs]
        st.free()
    o = B.OracleEncoder(ew, kv_max=2400)
    ref = [o.step(x) for x in xs]
    for i in range(len(sizes)):
        assert np.isfinite(outs["1"][i]).all()
        assert B.rel_l2(outs["1"][i], outs["0"][i]) < 2e-3, (i, B.rel_l2(outs["1"][i], outs["0"][i]))
        assert B.rel_l2(outs["1"][i], ref[i]) < 5e-3, (i, B.rel_l2(outs["1"][i], ref[i]))
    e.free()


def test_folded_norm_tma_residual_path_is_bit_identical(monkeypatch):
    """Where a residual GEMM's stage ring is free (the CTA's last tile, or the
    reduction of a cluster split), the folded norm's producer loads its
    residual tiles and stores the updated rows by TMA: the same arithmetic as
    the direct loads and stores (VOX_CUDA_TC_FOLD_TMA=0), so bit-identical.
    The fold is forced up to 1500 rows; chunks of one row tile (cluster
    split), several row tiles, 1500 rows (one tile per CTA) and 1500 rows
    with 64-wide tiles (two tiles on some CTAs: the first by direct stores,
    the last through TMA); the 1500-row chunk also against the oracle."""
    ew = B.EncoderWeights(seed=18, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sizes = [100, 37, 700, 1500]
    xs = [B.normal_f32((n, B.ENC_DIM), 1180 + i) for i, n in enumerate(sizes)]
    monkeypatch.setenv("VOX_CUDA_ENC_FOLD_MAX_ROWS", "1500")
    outs = {}
    for bn in ("", "64"):
        monkeypatch.setenv("VOX_CUDA_TC_BN", bn)
        for mode in ("0", ""):
            monkeypatch.setenv("VOX_CUDA_TC_FOLD_TMA", mode)
            st = e.state(max_chunk=1500)
            outs[(bn, mode)] = [st.step(x) for x in xs]
            st.free()
    e.free()
    for bn in ("", "64"):
        for i in range(len(sizes)):
            a, b = outs[(bn, "")][i], outs[(bn, "0")][i]
            assert np.isfinite(a).all()
            assert np.array_equal(a, b), (bn, sizes[i])
    o = B.OracleEncoder(ew, kv_max=2400)
    ref = [o.step(x) for x in xs]
    assert B.rel_l2(outs[("", "")][3], ref[3]) < 5e-3, B.rel_l2(outs[("", "")][3], ref[3])


def test_encoder_attention_key_split_matches_unsplit(monkeypatch):
    """Chunks of few row tiles split each tile's key blocks over several CTAs:
    by default the CTAs of one thread-block cluster whose partials are merged
    through distributed shared memory ("cluster"; at most 2 of them with
    VOX_CUDA_ENC_ATTN_CLUSTER=2), or (VOX_CUDA_ENC_ATTN_KSPLIT=4) unnormalised
    partials in a workspace merged by the last CTA ("workspace").  Against
    the unsplit kernel ("off"), from position 0 (splits with no key block)
    through window-crossing and ragged chunks, and against the oracle."""
    ew = B.EncoderWeights(seed=17, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sizes = [100, 37, 256, 3, 100, 64]
    xs = [B.normal_f32((n, B.ENC_DIM), 1170 + i) for i, n in enumerate(sizes)]
    outs = {}
    modes = {"off": ("1", "-1"), "workspace": ("4", "-1"), "cluster": ("", ""), "cluster2": ("", "2")}
    for mode, (ks, cl) in modes.items():
        monkeypatch.setenv("VOX_CUDA_ENC_ATTN_KSPLIT", ks)
        monkeypatch.setenv("VOX_CUDA_ENC_ATTN_CLUSTER", cl)
        st = e.state(max_chunk=256)
        outs[mode] = [st.step(x) for x in xs]
        st.free()
    o = B.OracleEncoder(ew, kv_max=2400)
    for i, x in enumerate(xs):
        ref = o.step(x)
        for mode in ("workspace", "cluster", "cluster2"):
            a = outs[mode][i]
            assert np.isfinite(a).all(), (i, mode)
            assert B.rel_l2(a, outs["off"][i]) < 1e-3, (i, mode, B.rel_l2(a, outs["off"][i]))
            assert B.rel_l2(a, ref) < 5e-3, (i, mode, B.rel_l2(a, ref))
    e.free()


def test_encoder_attention_softmax_split_matches(monkeypatch):
    """The attention's softmax as one warp per TMEM lane quarter (all 64 key
    columns) or two (32 each, block maxima and row sums exchanged through
    shared memory): chunk sizes that take either launch shape by default, both
    forced, against each other and the oracle."""
    ew = B.EncoderWeights(seed=18, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sizes = [100, 37, 256, 3, 700]
    xs = [B.normal_f32((n, B.ENC_DIM), 1180 + i) for i, n in enumerate(sizes)]
    outs = {}
    for nh in ("1", "2"):
        monkeypatch.setenv("VOX_CUDA_ENC_ATTN_NH", nh)
        st = e.state(max_chunk=700)
        outs[nh] = [st.step(x) for x in xs]
        st.free()
    o = B.OracleEncoder(ew, kv_max=2400)
    for i, x in enumerate(xs):
        ref = o.step(x)
        assert np.isfinite(outs["2"][i]).all()
        assert B.rel_l2(outs["2"][i], outs["1"][i]) < 1e-4, (i, B.rel_l2(outs["2"][i], outs["1"][i]))
        assert B.rel_l2(outs["2"][i], ref) < 5e-3, (i, B.rel_l2(outs["2"][i], ref))
    e.free()


def test_encoder_tile_widths_agree(monkeypatch):
    """The tensor-core GEMM's tile width (64 / 128 / 192 / 256 columns, picked
    by a rounds x tile-cost model) changes which CTA computes an output
    element, not how: each element sums its K blocks in the same order.
    500- and 800-row chunks, where the model picks 192 for q|k|v (and at
    500 for w1|w3), against forced widths: bit-identical.  Split-K is held
    off: a forced width can change whether wo / w2 split, which regroups
    their fp32 sums (equally accurate, not bit-identical)."""
    ew = B.EncoderWeights(seed=15, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sizes = [500, 800]
    outs = {}
    monkeypatch.setenv("VOX_CUDA_TC_KSPLIT", "1")
    for bn in ("", "256", "128"):
        monkeypatch.setenv("VOX_CUDA_TC_BN", bn)
        st = e.state(max_chunk=800)
        outs[bn] = [st.step(B.normal_f32((n, B.ENC_DIM), 1110 + i)) for i, n in enumerate(sizes)]
        st.free()
    e.free()
    for i in range(len(sizes)):
        assert np.isfinite(outs[""][i]).all()
        assert np.array_equal(outs[""][i], outs["256"][i]), i
        assert np.array_equal(outs[""][i], outs["128"][i]), i


def test_encoder_async_steps_match_sync_steps():
    """vox_cuda_encoder_step_dev enqueues without waiting: chunks issued back
    to back (positions travel by value) equal the synchronous host-pointer
    steps."""
    import torch
    ew = B.EncoderWeights(seed=11, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    chunks = [B.normal_f32((n, B.ENC_DIM), 1030 + i) for i, n in enumerate([100, 37, 256, 90])]
    sa = e.state(max_chunk=256)
    ref = [sa.step(x) for x in chunks]
    sb = e.state(max_chunk=256)
    stream = torch.cuda.Stream()
    devs = [torch.from_numpy(x).cuda() for x in chunks]
    torch.cuda.synchronize()
    for d in devs:
        sb.step_dev(d.data_ptr(), d.shape[0], stream.cuda_stream)
    stream.synchronize()
    for d, r in zip(devs, ref):
        assert np.array_equal(d.cpu().numpy(), r)
    assert sb.position == sa.position == sum(x.shape[0] for x in chunks)
    sa.free()
    sb.free()
    e.free()


def test_encoder_host_rope_table_matches_device_table():
    """vox_cuda_encoder_full_step with the host's RoPE table (the reference
    API passes rope_freqs) and with the table computed on the device.  The two
    tables differ in the last ulp of some angles, which moves a few fp16 / bf16
    roundings downstream (~5e-4 rel-L2); a wrongly laid out table is O(1) off."""
    ew = B.EncoderWeights(seed=8, n_layers=2, distinct=2, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    sa, sb = e.state(max_chunk=256), e.state(max_chunk=256)
    pos = 0
    for i, n in enumerate([100, 256, 37, 250, 200]):
        x = B.normal_f32((n, B.ENC_DIM), 970 + i)
        ya = sa.step(x, rope=B.rope_freqs(np.arange(pos, pos + n), B.ENC_HEAD_DIM))
        yb = sb.step(x)
        pos += n
        assert B.rel_l2(ya, yb) < 2e-3, (i, B.rel_l2(ya, yb))
    sa.free()
    sb.free()
    e.free()


def test_encoder_matches_oracle_small_model():
    ew = B.EncoderWeights(seed=5, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    st = e.state(max_chunk=256)
    o = B.OracleEncoder(ew, kv_max=2400)
    for i, n in enumerate([64, 200, 3, 250, 130]):   # crosses the window, ragged sizes
        x = B.normal_f32((n, B.ENC_DIM), 900 + i)
        yo = o.step(x)
        yg = st.step(x)
        assert B.rel_l2(yg, yo) < 5e-3, (i, B.rel_l2(yg, yo))
    st.free()
    e.free()


def test_adapter_matches_oracle(gpu_enc, enc_w):
    o = B.OracleEncoder(enc_w, kv_max=2400)
    chunks = G.enc_chunks()
    enc = np.concatenate([o.step(chunks[0]), o.step(chunks[1])], axis=0)[:136]
    want = o.adapter(enc)
    st = gpu_enc.state(max_chunk=256)
    got = st.adapter(enc)
    assert B.rel_l2(got, want) < ADAPTER_TOL
    g = load_golden("encoder")
    assert sampled_rel(got, g, "adapter136") < ADAPTER_TOL
    st.free()


def test_encoder_rejects_oversized_chunk(gpu_enc):
    st = gpu_enc.state(max_chunk=64)
    with pytest.raises(V.VoxCudaError):
        st.step(np.zeros((65, B.ENC_DIM), np.float32))
    st.free()


def test_encoder_batched_launch_matches_per_state_steps():
    """vox_cuda_encoder_step_batch_dev: four states' chunks (100, 37, 256 and
    90 rows, two rounds, the second state starting from position 300) as
    one launch per round against each state stepping alone.  The GEMMs see
    another M (tiling and split-K choices differ), so the fp16 operands may
    round differently: the encoder tolerance applies."""
    import torch
    ew = B.EncoderWeights(seed=12, n_layers=3, distinct=3, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    lens = [100, 37, 256, 90]
    alone = [e.state(max_chunk=256) for _ in lens]
    batch = [e.state(max_chunk=256) for _ in lens]
    alone[1].set_position(300)
    batch[1].set_position(300)
    stream = torch.cuda.Stream()
    for rnd in range(2):
        xs = [B.normal_f32((n, B.ENC_DIM), 1100 + 10 * rnd + i) for i, n in enumerate(lens)]
        want = [st.step(x) for st, x in zip(alone, xs)]
        devs = [torch.from_numpy(x).cuda() for x in xs]
        torch.cuda.synchronize()
        V.encoder_step_batch_dev(batch, [d.data_ptr() for d in devs], lens, stream.cuda_stream)
        stream.synchronize()
        for i, (d, w) in enumerate(zip(devs, want)):
            got = d.cpu().numpy()
            assert np.isfinite(got).all()
            assert B.rel_l2(got, w) < ENC_TOL, (rnd, i, B.rel_l2(got, w))
    for a, b in zip(alone, batch):
        assert a.position == b.position
    # a state freed and replaced (possibly at the same address) must not reuse
    # the launch captured with the old one
    batch[1].free()
    alone[1].free()
    batch[1], alone[1] = e.state(max_chunk=256), e.state(max_chunk=256)
    xs = [B.normal_f32((n, B.ENC_DIM), 1200 + i) for i, n in enumerate(lens)]
    want = [st.step(x) for st, x in zip(alone, xs)]
    devs = [torch.from_numpy(x).cuda() for x in xs]
    torch.cuda.synchronize()
    V.encoder_step_batch_dev(batch, [d.data_ptr() for d in devs], lens, stream.cuda_stream)
    stream.synchronize()
    for i, (d, w) in enumerate(zip(devs, want)):
        assert B.rel_l2(d.cpu().numpy(), w) < ENC_TOL, (i, B.rel_l2(d.cpu().numpy(), w))
    for a, b in zip(alone, batch):
        a.free()
        b.free()
    e.free()


def test_encoder_ring_wraps_match_oracle():
    """Chunks of 1..64 rows until the positions pass twice the ring's
    capacity (max_chunk 64: 896 slots), so the fp16 ring wraps twice, q|k|v
    rows land across the wrap and attention key blocks follow it; against
    the oracle's compacting cache (the reference's keep-the-last-750 rule)."""
    ew = B.EncoderWeights(seed=21, n_layers=1, distinct=1, norm_noise=0.1)
    e = make_gpu_encoder(ew)
    st = e.state(max_chunk=64)
    o = B.OracleEncoder(ew, kv_max=1024)
    rng = np.random.default_rng(3)
    pos, i = 0, 0
    while pos < 2 * 896 + 100:
        n = int(rng.integers(1, 65))
        x = B.normal_f32((n, B.ENC_DIM), 1300 + i)
        yo, yg = o.step(x), st.step(x)
        assert B.rel_l2(yg, yo) < 5e-3, (i, pos, n, B.rel_l2(yg, yo))
        pos += n
        i += 1
    assert st.position == pos
    st.free()
    e.free()


def test_adapter_dev_matches_host_adapter(gpu_enc):
    """vox_cuda_adapter_forward_dev (device rows in and out, asynchronous)
    gives the host entry point's rows bit for bit."""
    import torch
    st = gpu_enc.state(max_chunk=256)
    enc = B.normal_f32((200, B.ENC_DIM), 1600, 1.0)
    want = st.adapter(enc)
    d_in = torch.from_numpy(enc).cuda()
    d_out = torch.empty((50, B.DEC_DIM), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    st.adapter_dev(d_in.data_ptr(), 200, d_out.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), want)
    st.free()


def _to_bf16_bits(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _heavy_tailed(ew, seed, scale=1.0, w13_gain=1.0):
    """Replace every weight matrix of `ew` in place by Student-t (3 degrees of
    freedom) values with the same 0.02 scale: heavy tails, as real checkpoints
    have; w1 / w3 (and the adapter's first matrix) optionally amplified."""
    rng = np.random.default_rng(seed)
    for ws, _, _ in ew.sets:
        for j, w in enumerate(ws):
            gain = w13_gain if j in (4, 6) else 1.0
            t = rng.standard_t(3, size=w.shape).astype(np.float32) * (0.02 / np.sqrt(3.0)) * scale * gain
            w[...] = _to_bf16_bits(t)


def test_heavy_tailed_weights_match_oracle_without_saturation():
    """Heavy-tailed weights (Student-t, df 3) and inputs at scale 1e3: the
    fp16 operands stay in range (no saturations counted) and the encoder
    stays within its parity bound against the fp32 oracle."""
    ew = B.EncoderWeights(seed=11, n_layers=3, distinct=3, norm_noise=0.1)
    _heavy_tailed(ew, 1800)
    e = make_gpu_encoder(ew)
    st = e.state(max_chunk=256)
    o = B.OracleEncoder(ew, kv_max=1024)
    V.fp16_saturations(reset=True)
    for i, n in enumerate((100, 37, 160)):
        x = B.normal_f32((n, B.ENC_DIM), 1810 + i, 1000.0)
        y = st.step(x)
        want = o.step(x)
        assert np.isfinite(y).all()
        assert B.rel_l2(y, want) < ENC_TOL, (i, B.rel_l2(y, want))
    assert V.fp16_saturations() == 0
    st.free()
    e.free()


def test_fp16_overflow_is_clamped_and_counted():
    """w1 / w3 amplified so that silu(gate) * up exceeds fp16's range: the
    values are clamped to +-65504 (no inf or NaN reaches the residual
    stream) and counted by vox_cuda_fp16_saturations."""
    ew = B.EncoderWeights(seed=12, n_layers=2, distinct=2)
    _heavy_tailed(ew, 1900, w13_gain=400.0)
    e = make_gpu_encoder(ew)
    st = e.state(max_chunk=128)
    V.fp16_saturations(reset=True)
    y = st.step(B.normal_f32((64, B.ENC_DIM), 1901, 1.0))
    n = V.fp16_saturations(reset=True)
    assert n > 0
    assert np.isfinite(y).all()
    assert V.fp16_saturations() == 0   # the reset took
    st.free()
    e.free()
