"""The C restatement (oracle/vo_oracle.c) against golden vectors produced by
the reference's own CPU path (tests/golden/gen_golden.py).  CPU only."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
from conftest import load_golden, unpack


def sampled_rel(arr, g, prefix):
    idx, val, _, size = unpack(g, prefix)
    flat = np.asarray(arr, np.float32).reshape(-1)
    assert flat.size == size
    return B.rel_l2(flat[idx], val)


@pytest.mark.parametrize("case", G.LINEAR_CASES, ids=[c[0] for c in G.LINEAR_CASES])
def test_linear_matches_reference(case):
    g = load_golden("linear")
    name, M, K, N, bias, path, seed = case
    x, W, b = G.linear_inputs(M, K, N, bias, seed)
    assert str(g[name + "_xsum"]) == str(G.checksum(x)), "input generator changed"
    assert str(g[name + "_wsum"]) == str(G.checksum(W)), "input generator changed"
    y = B.linear(x, W, b)
    assert sampled_rel(y, g, name) < 1e-5


def test_rope_matches_reference():
    g = load_golden("rope")
    pos = g["pos"]
    for hd in (128, 64):
        f = B.rope_freqs(pos, hd)
        ref = g[f"freqs{hd}"]
        # Identical formula; the reference is built with -ffast-math, whose powf
        # may differ by 1 ulp (2^-23 relative) from glibc's, so the angle error
        # grows with the position: |d angle| <= pos * freq * 2^-23, freq <= 1.
        bound = 1e-6 + 2.0 * 2.0**-23 * pos.astype(np.float64)
        assert np.all(np.abs(f - ref).max(axis=1) <= bound)
    x = B.normal_f32((len(pos), 32 * 128), 31)
    # apply_rope with the reference's own table is exact arithmetic
    assert np.array_equal(B.apply_rope(x, g["freqs128"], 32, 128), g["apply128"])
    x = B.normal_f32((len(pos), 32 * 64), 32)
    assert np.array_equal(B.apply_rope(x, g["freqs64"], 32, 64), g["apply64"])


@pytest.mark.parametrize("case", G.ATTN_DECODE, ids=[c[0] for c in G.ATTN_DECODE])
def test_decode_attention_matches_reference(case):
    g = load_golden("attention")
    name, L, slot, seed = case
    q, k, v = G.attn_decode_inputs(L, seed)
    if slot >= 0:
        k, v = G.ring_to_logical(k, slot), G.ring_to_logical(v, slot)
    o = B.causal_attention(q, k, v, 1, L, 32, 8, 128, 8192, L - 1)
    assert sampled_rel(o, g, name) < 1e-5


@pytest.mark.parametrize("case", G.ATTN_PREFILL, ids=[c[0] for c in G.ATTN_PREFILL])
def test_prefill_attention_matches_reference(case):
    g = load_golden("attention")
    name, sq, cache, h, kvh, hd, win, seed = case
    q, k, v = G.attn_prefill_inputs(sq, cache, h, kvh, hd, seed)
    o = B.causal_attention(q, k, v, sq, cache + sq, h, kvh, hd, win, cache)
    assert sampled_rel(o, g, name) < 1e-5


def test_fill_alts_matches_reference():
    g = load_golden("alts")
    for i, (seed, std, n_alt, cut) in enumerate(G.ALT_CASES):
        lg = B.normal_f32(B.VOCAB, seed, std)
        best = int(np.argmax(lg))
        assert best == int(g[f"case{i}_best"])
        assert B.fill_alts(lg, best, n_alt, cut) == g[f"case{i}_ids"].tolist()


@pytest.fixture(scope="module")
def dec_weights():
    return B.DecoderWeights(seed=G.DEC_SEED)


def test_decoder_prefill_and_steps_match_reference(dec_weights):
    g = load_golden("decoder")
    o = B.OracleDecoder(dec_weights, 8192 + 38 + 1024)
    o.prefill(G.dec_embeds(G.PROMPT, 7001))
    assert list(o.state) == [int(g["state_prefill"][0]), int(g["state_prefill"][2])]
    assert sampled_rel(o.k[25, :G.PROMPT], g, "prefill_k25") < 1e-5
    assert sampled_rel(o.v[0, :G.PROMPT], g, "prefill_v0") < 1e-5
    steps = G.dec_embeds(G.DEC_STEPS, 7002)
    for s in range(G.DEC_STEPS):
        tok, lg = o.step(steps[s])
        assert sampled_rel(lg, g, f"step{s}_logits") < 1e-4
        assert tok == int(g[f"step{s}_token"])


def test_decoder_compaction_matches_reference(dec_weights):
    g = load_golden("decoder")
    o = B.OracleDecoder(dec_weights, G.COMPACT_MAX)
    kf, vf = G.compact_kv_fill(7100)
    o.k[...] = kf
    o.v[...] = vf
    del kf, vf
    o.kv.len, o.kv.pos_offset = G.COMPACT_MAX, G.COMPACT_OFFSET
    steps = G.dec_embeds(2, 7003)
    for s in range(2):
        tok, lg = o.step(steps[s])
        st = g[f"compact{s}_state"]
        assert (o.kv.len, o.kv.pos_offset) == (int(st[0]), int(st[2]))
        assert sampled_rel(lg, g, f"compact{s}_logits") < 1e-4
        assert tok == int(g[f"compact{s}_token"])


def test_encoder_chunks_and_adapter_match_reference():
    g = load_golden("encoder")
    ew = B.EncoderWeights(seed=G.DEC_SEED)
    o = B.OracleEncoder(ew, kv_max=2400)
    outs = []
    for i, x in enumerate(G.enc_chunks()):
        y = o.step(x)
        outs.append(y)
        st = g[f"chunk{i}_state"]
        assert (o.kv.len, o.kv.pos_offset) == (int(st[3]), int(st[5]))
        assert sampled_rel(y, g, f"chunk{i}") < 1e-4
    a = o.adapter(np.concatenate(outs[:2], axis=0)[:136])
    assert sampled_rel(a, g, "adapter136") < 1e-4


def _gelu(v):
    # tanh GELU (vox_gelu, voxtral_kernels.c:376-384)
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


def _stem_restated(w, chunks):
    """The conv stem chunk by chunk (stream_conv_stem, voxtral.c:487-665),
    restated as causal convs over the mel stream with two pieces of state:
    the last two mel frames (after a one-frame chunk the older of the two is
    zero: the reference rebuilds its tail as [0, frame], voxtral.c:519-524,
    551-556) and the conv0 outputs by global frame index.  Chunk i yields
    conv1 rows floor(T_i / 2) .. floor(T_{i+1} / 2) - 1."""
    w0, w1 = w.w0.astype(np.float64), w.w1.astype(np.float64)
    hist = np.zeros((2, w0.shape[1]))
    c0 = {}
    t, outs = 0, []
    for mel in chunks:
        n = mel.shape[0]
        ext = np.concatenate([hist, mel.astype(np.float64)], axis=0)   # frames t-2 .. t+n-1
        for r in range(n):
            win = ext[r:r + 3]
            c0[t + r] = _gelu(w.b0 + np.einsum("oik,ki->o", w0, win))
        u0, u1 = t // 2, (t + n) // 2
        rows = []
        for u in range(u0, u1):
            win = np.stack([c0[i] if i >= 0 else np.zeros(w1.shape[1]) for i in (2 * u - 1, 2 * u, 2 * u + 1)])
            rows.append(_gelu(w.b1 + np.einsum("oik,ki->o", w1, win)))
        outs.append(np.array(rows).reshape(-1, w1.shape[0]))
        hist = ext[-2:].copy() if n >= 2 else np.stack([np.zeros(w0.shape[1]), ext[-1]])
        t += n
    return outs


def test_conv_stem_matches_reference_golden():
    g = load_golden("stem")
    w = B.ConvStemWeights(seed=G.DEC_SEED)
    outs = _stem_restated(w, G.stem_chunks())
    for i, y in enumerate(outs):
        assert int(g[f"chunk{i}_rows"]) == y.shape[0]
        if y.size:
            idx, val, _, _ = unpack(g, f"chunk{i}")
            assert B.rel_l2(y.reshape(-1)[idx], val) < 1e-5, i


# log-mel: fp32 sums of 400 (DFT) and 201 (filters) terms in another order than
# the reference's vectorised -ffast-math loops; the weakest bands (highest mel
# bins of pink noise) carry the largest relative error after log10.
MEL_MAX_ABS = 1e-3
MEL_REL = 1e-4


def mel_stream_rows(tag):
    """The restated streaming context over the golden's feed schedule."""
    import mel as M
    x = G.mel_audio()
    feeds, pad, zeros, right = ((G.mel_feeds(G.MEL_FEEDS_A), G.MEL_PAD_A, G.MEL_RIGHT_A, 0) if tag == "a"
                                else (G.mel_feeds(G.MEL_FEEDS_B), 0, 0, G.MEL_RIGHT_B))
    m = M.StreamingMel(pad)
    rows, off = [], 0
    for f in feeds:
        rows.append(m.feed(x[off:off + f]))
        off += f
    while zeros > 0:
        c = min(zeros, 4096)
        rows.append(m.feed(np.zeros(c, np.float32)))
        zeros -= c
    rows.append(m.finish(right))
    return rows


@pytest.mark.parametrize("tag", ["a", "b"])
def test_streaming_mel_matches_reference_golden(tag):
    g = load_golden("mel")
    assert str(g["audio_sum"]) == str(G.checksum(G.mel_audio())), "audio generator changed"
    rows = mel_stream_rows(tag)
    assert [r.shape[0] for r in rows] == g[f"{tag}_counts"].tolist()
    mel = np.concatenate(rows, axis=0)
    idx, val, _, size = unpack(g, f"{tag}_mel")
    assert mel.size == size
    assert np.abs(mel.reshape(-1)[idx] - val).max() < MEL_MAX_ABS
    assert B.rel_l2(mel.reshape(-1)[idx], val) < MEL_REL


@pytest.mark.parametrize("n", G.MEL_ONESHOT)
def test_oneshot_mel_matches_reference_golden(n):
    import mel as M
    g = load_golden("mel")
    m = M.mel_spectrogram(G.mel_audio()[:n])
    frames = int(g[f"oneshot{n}_frames"])
    if frames == 0:
        assert m is None
        return
    idx, val, _, size = unpack(g, f"oneshot{n}")
    assert m.size == size
    assert np.abs(m.reshape(-1)[idx] - val).max() < MEL_MAX_ABS
    assert B.rel_l2(m.reshape(-1)[idx], val) < MEL_REL
