"""Generate the golden vectors in tests/golden/ from the reference itself.

Runs the reference's own CPU path (oracle/_ref/libvoxref.so, compiled from the
unmodified reference sources by oracle/Makefile) on seeded synthetic inputs
and stores its outputs.  Inputs are not stored: they are regenerated from the
recorded seeds with the oracle's counter-based generator, and a checksum of
each input is stored so that a change of generator is caught.

Outputs up to 32768 values are stored whole; larger ones as a fixed sample of
32768 positions plus their L2 norm.

    python tests/golden/gen_golden.py        # needs oracle/_ref (reference tree present)
"""
from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import bind as B  # noqa: E402

SAMPLE = 32768


def sample_idx(n, seed=12345):
    if n <= SAMPLE:
        return np.arange(n, dtype=np.int64)
    rng = np.random.default_rng(seed + n)
    return np.sort(rng.choice(n, SAMPLE, replace=False)).astype(np.int64)


def pack(prefix, arr, out):
    flat = np.asarray(arr, np.float32).reshape(-1)
    idx = sample_idx(flat.size)
    out[prefix + "_idx"] = idx
    out[prefix + "_val"] = flat[idx]
    out[prefix + "_norm"] = np.float64(np.linalg.norm(flat.astype(np.float64)))
    out[prefix + "_size"] = np.int64(flat.size)


def pack_vals(prefix, arr, out, n_sample=SAMPLE):
    """Like pack, without the indices: the sample positions are
    sample_idx(size) (or all values when size <= n_sample), recomputed by the
    reader, which keeps files with many outputs of one size small."""
    flat = np.asarray(arr, np.float32).reshape(-1)
    idx = sample_idx(flat.size) if n_sample == SAMPLE else sample_n(flat.size, n_sample)
    out[prefix + "_val"] = flat[idx]
    out[prefix + "_norm"] = np.float64(np.linalg.norm(flat.astype(np.float64)))
    out[prefix + "_size"] = np.int64(flat.size)


def sample_n(n, k, seed=4242):
    if n <= k:
        return np.arange(n, dtype=np.int64)
    rng = np.random.default_rng(seed + n + k)
    return np.sort(rng.choice(n, k, replace=False)).astype(np.int64)


def checksum(a):
    return np.array(hashlib.sha1(np.ascontiguousarray(a).tobytes()).hexdigest()[:16])


# (name, M, K, N, bias, path, seed)
LINEAR_CASES = [
    ("gemv_wq", 1, 3072, 4096, False, "linear", 11),
    ("gemv_wk", 1, 3072, 1024, False, "linear", 12),
    ("gemv_wo", 1, 4096, 3072, False, "linear", 13),
    ("gemv_w1", 1, 3072, 9216, False, "linear", 14),
    ("gemv_w2", 1, 9216, 3072, False, "linear", 15),
    ("gemv_lmhead_slice", 1, 3072, 8192, False, "matmul_t", 16),
    ("gemv_bias", 1, 1280, 2048, True, "linear", 17),
    ("linear_m5_bias", 5, 1280, 2048, True, "linear", 18),
    ("linear_m38_wq", 38, 3072, 4096, False, "linear", 19),
    ("linear_m100_w2_bias", 100, 5120, 1280, True, "linear", 20),
    ("linear_m8_wo", 8, 4096, 3072, False, "linear", 21),
]


def linear_inputs(M, K, N, bias, seed):
    x = B.normal_f32((M, K), seed * 10 + 1)
    W = B.normal_bf16((N, K), seed * 10 + 2)
    b = B.normal_f32(N, seed * 10 + 3, 0.02) if bias else None
    return x, W, b


def gen_linear():
    out = {}
    for name, M, K, N, bias, path, seed in LINEAR_CASES:
        x, W, b = linear_inputs(M, K, N, bias, seed)
        y = B.ref_linear(x, W, b, path=path)
        pack(name, y, out)
        out[name + "_xsum"] = checksum(x)
        out[name + "_wsum"] = checksum(W)
    np.savez_compressed(os.path.join(HERE, "linear.npz"), **out)


ROPE_POS = [0, 1, 2, 38, 750, 1000, 5000, 8191, 8192, 20000, 100000, 1234567]


def gen_rope():
    out = {"pos": np.array(ROPE_POS, np.int32)}
    for hd in (128, 64):
        out[f"freqs{hd}"] = B.ref_rope_freqs(out["pos"], hd)
    x = B.normal_f32((len(ROPE_POS), 32 * 128), 31)
    out["apply128"] = B.ref_apply_rope(x, out["freqs128"], 32, 128)
    x = B.normal_f32((len(ROPE_POS), 32 * 64), 32)
    out["apply64"] = B.ref_apply_rope(x, out["freqs64"], 32, 64)
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)


# decode attention: (name, L, ring_write_slot or -1, seed)
ATTN_DECODE = [("dec_L512", 512, -1, 41), ("dec_L2048", 2048, -1, 42),
               ("dec_L8192", 8192, -1, 43), ("dec_ring5000", 8192, 5000, 44),
               ("dec_L1", 1, -1, 45), ("dec_L777", 777, -1, 46)]


def attn_decode_inputs(L, seed):
    q = B.normal_f32((1, B.Q_DIM), seed * 10 + 1)
    k = B.normal_f32((L, B.KV_DIM), seed * 10 + 2)
    v = B.normal_f32((L, B.KV_DIM), seed * 10 + 3)
    return q, k, v


def ring_to_logical(buf, write_slot):
    """A full ring whose newest row sits at write_slot, in logical order."""
    return np.ascontiguousarray(np.roll(buf, -(write_slot + 1), axis=0))


# prefill-style attention: (name, seq_q, cache_len, n_heads, n_kv, head_dim, window, seed)
ATTN_PREFILL = [("enc_q100_c200", 100, 200, 32, 32, 64, 750, 51),
                ("enc_q37_c750", 37, 750, 32, 32, 64, 750, 52),
                ("dec_prefill_q38", 38, 0, 32, 8, 128, 8192, 53)]


def attn_prefill_inputs(seq_q, cache, h, kvh, hd, seed):
    q = B.normal_f32((seq_q, h * hd), seed * 10 + 1)
    k = B.normal_f32((cache + seq_q, kvh * hd), seed * 10 + 2)
    v = B.normal_f32((cache + seq_q, kvh * hd), seed * 10 + 3)
    return q, k, v


def gen_attention():
    out = {}
    for name, L, slot, seed in ATTN_DECODE:
        q, k, v = attn_decode_inputs(L, seed)
        if slot >= 0:
            k, v = ring_to_logical(k, slot), ring_to_logical(v, slot)
        o = B.ref_attention(q, k, v, 1, L, 32, 8, 128, 8192, L - 1)
        pack(name, o, out)
    for name, sq, cache, h, kvh, hd, win, seed in ATTN_PREFILL:
        q, k, v = attn_prefill_inputs(sq, cache, h, kvh, hd, seed)
        o = B.ref_attention(q, k, v, sq, cache + sq, h, kvh, hd, win, cache)
        pack(name, o, out)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


DEC_SEED = 0
PROMPT = 38
DEC_STEPS = 4
COMPACT_MAX, COMPACT_OFFSET = 8200, 3000


def dec_embeds(n, seed):
    return B.normal_f32((n, B.DEC_DIM), seed, 1.0)


def compact_kv_fill(seed):
    k = B.normal_f32((B.DEC_LAYERS, COMPACT_MAX, B.KV_DIM), seed, 1.0)
    v = B.normal_f32((B.DEC_LAYERS, COMPACT_MAX, B.KV_DIM), seed + 1, 1.0)
    return k, v


def top(logits, n=16):
    idx = np.argsort(-logits, kind="stable")[:n]
    return idx.astype(np.int32), logits[idx]


def gen_decoder(w):
    out = {}
    ref = B.RefCtx(dec=w)
    prompt = dec_embeds(PROMPT, 7001)
    ref.decoder_prefill(prompt)
    st = ref.state()
    k, v = ref.dec_kv()
    pack("prefill_k25", k[25, :PROMPT], out)
    pack("prefill_v0", v[0, :PROMPT], out)
    steps = dec_embeds(DEC_STEPS, 7002)
    for s in range(DEC_STEPS):
        tok, lg = ref.decoder_forward(steps[s])
        pack(f"step{s}_logits", lg, out)
        out[f"step{s}_token"] = np.int32(tok)
        out[f"step{s}_top_idx"], out[f"step{s}_top_val"] = top(lg)
    out["state_after"] = np.array(ref.state(), np.int32)
    out["state_prefill"] = np.array(st, np.int32)
    # the reference's own RoPE tables for these positions (its -ffast-math
    # powf can differ from other builds by an ulp; a caller passes them on)
    out["prefill_rope"] = B.ref_rope_freqs(np.arange(PROMPT), 128)
    out["step_rope"] = B.ref_rope_freqs(np.arange(PROMPT, PROMPT + DEC_STEPS), 128)
    out["compact_rope"] = B.ref_rope_freqs(
        np.arange(COMPACT_OFFSET + 8200, COMPACT_OFFSET + 8202), 128)
    ref.free()

    # compaction: a full cache (len == max) at logical offset COMPACT_OFFSET
    ref = B.RefCtx(dec=w)
    assert B.ref_lib().voxref_decoder_kv_preallocate(ref.ctx, COMPACT_MAX) == 0
    k, v = ref.dec_kv()
    kf, vf = compact_kv_fill(7100)
    k[...] = kf
    v[...] = vf
    del kf, vf
    B.ref_lib().voxref_set_dec_kv_state(ref.ctx, COMPACT_MAX, COMPACT_OFFSET)
    steps = dec_embeds(2, 7003)
    for s in range(2):
        tok, lg = ref.decoder_forward(steps[s])
        pack(f"compact{s}_logits", lg, out)
        out[f"compact{s}_token"] = np.int32(tok)
        out[f"compact{s}_state"] = np.array(ref.state(), np.int32)
    ref.free()
    np.savez_compressed(os.path.join(HERE, "decoder.npz"), **out)


# The benchmarked batched step: 8 streams sharing one decoder, with cached
# histories of 39 + 100 i positions (streams 0..6) and one full cache of
# 8200 rows at logical offset 3000 (stream 7), which the reference compacts
# before its first step and which wraps the device ring (8192 + 1024 slots).
# Each stream is its own reference context (vox_decoder_forward,
# voxtral_decoder.c:401-516); the histories are seeded random K / V rows.
BATCH_N = 8
BATCH_STEPS = 3
BATCH_LOGIT_SAMPLE = 8192


def batch_history(i):
    """(rows, logical offset) of stream i's cached history."""
    if i < BATCH_N - 1:
        return 39 + 100 * i, 0
    return COMPACT_MAX, COMPACT_OFFSET


def batch_kv(i):
    rows, _ = batch_history(i)
    k = B.normal_f32((B.DEC_LAYERS, rows, B.KV_DIM), 7300 + 2 * i, 1.0)
    v = B.normal_f32((B.DEC_LAYERS, rows, B.KV_DIM), 7301 + 2 * i, 1.0)
    return k, v


def batch_embeds(step):
    return B.normal_f32((BATCH_N, B.DEC_DIM), 7400 + step, 1.0)


def gen_batch8(w):
    out = {}
    rope = np.zeros((BATCH_STEPS, BATCH_N, 128), np.float32)
    for i in range(BATCH_N):
        rows, off = batch_history(i)
        ref = B.RefCtx(dec=w)
        assert B.ref_lib().voxref_decoder_kv_preallocate(ref.ctx, rows if off else rows + 8) == 0
        k, v = ref.dec_kv()
        kf, vf = batch_kv(i)
        k[:, :rows] = kf
        v[:, :rows] = vf
        del kf, vf, k, v
        B.ref_lib().voxref_set_dec_kv_state(ref.ctx, rows, off)
        for s_ in range(BATCH_STEPS):
            rope[s_, i] = B.ref_rope_freqs([off + rows + s_], 128)[0]
            tok, lg = ref.decoder_forward(batch_embeds(s_)[i])
            pack_vals(f"s{i}_step{s_}", lg, out, BATCH_LOGIT_SAMPLE)
            out[f"s{i}_step{s_}_token"] = np.int32(tok)
            srt = np.sort(lg)
            out[f"s{i}_step{s_}_margin"] = np.float32(srt[-1] - srt[-2])
        out[f"s{i}_state"] = np.array(ref.state(), np.int32)
        ref.free()
    out["rope"] = rope
    np.savez_compressed(os.path.join(HERE, "batch8.npz"), **out)


# The benchmarked encoder chunk sizes: a 750-row
# history, then 500 and 1500 rows, run on the device with max_chunk = 1500
# as the bench runs them (vox_encoder_forward_incremental,
# voxtral_encoder.c:452-636).
ENC_BIG_CHUNKS = [750, 500, 1500]


def enc_big_chunks(seed=8501):
    return [B.normal_f32((n, B.ENC_DIM), seed + i, 1.0) for i, n in enumerate(ENC_BIG_CHUNKS)]


def gen_encoder_big(ew):
    out = {}
    ref = B.RefCtx(enc=ew)
    for i, x in enumerate(enc_big_chunks()):
        y = ref.encoder_incremental(x)
        pack_vals(f"chunk{i}", y, out)
        out[f"chunk{i}_state"] = np.array(ref.state(), np.int32)
        del y
    ref.free()
    np.savez_compressed(os.path.join(HERE, "encoder_big.npz"), **out)


ENC_CHUNKS = [100, 37, 700, 100]


def enc_chunks(seed=8001):
    return [B.normal_f32((n, B.ENC_DIM), seed + i, 1.0) for i, n in enumerate(ENC_CHUNKS)]


def gen_encoder(ew):
    out = {}
    ref = B.RefCtx(enc=ew)
    outs = []
    for i, x in enumerate(enc_chunks()):
        y = ref.encoder_incremental(x)
        outs.append(y)
        pack(f"chunk{i}", y, out)
        out[f"chunk{i}_state"] = np.array(ref.state(), np.int32)
    enc = np.concatenate(outs[:2], axis=0)[:136]
    a = ref.adapter(enc)
    pack("adapter136", a, out)
    ref.free()
    np.savez_compressed(os.path.join(HERE, "encoder.npz"), **out)


# End-to-end chain (configs[3] in small): post-conv-stem chunks -> encoder ->
# adapter -> decoder inputs adapter_out[i] + tok_embed(id) (voxtral.c:346)
# -> prompt [BOS] + [STREAMING_PAD] * (32 + 6 delay tokens) prefilled as
# 38 rows + one step (voxtral.c:839-867), then teacher-forced steps on the
# reference's own tokens (voxtral.c:898-906).
CHAIN_CHUNKS = [120, 80]
CHAIN_PROMPT = 1 + 32 + 6
CHAIN_STEPS = 9
TOKEN_BOS, TOKEN_PAD = 1, 32


def chain_chunks(seed=8101):
    return [B.normal_f32((n, B.ENC_DIM), seed + i, 1.0) for i, n in enumerate(CHAIN_CHUNKS)]


def chain_embed(w, adapter_row, token):
    return adapter_row + B.bf16_to_f32(w.tok_emb[token])


def gen_chain(w, ew):
    out = {}
    ref = B.RefCtx(dec=w, enc=ew)
    enc = np.concatenate([ref.encoder_incremental(x) for x in chain_chunks()], axis=0)
    ad = ref.adapter(enc)
    pack("adapter", ad, out)
    prompt = np.stack([chain_embed(w, ad[i], TOKEN_BOS if i == 0 else TOKEN_PAD)
                       for i in range(CHAIN_PROMPT)])
    ref.decoder_prefill(prompt[:CHAIN_PROMPT - 1])
    inputs = []
    tok, lg = ref.decoder_forward(prompt[CHAIN_PROMPT - 1])
    for g in range(CHAIN_STEPS):
        if g > 0:
            inputs.append(tok)
            tok, lg = ref.decoder_forward(chain_embed(w, ad[CHAIN_PROMPT - 1 + g], tok))
        pack(f"step{g}_logits", lg, out)
        out[f"step{g}_token"] = np.int32(tok)
        srt = np.sort(lg)
        out[f"step{g}_margin"] = np.float32(srt[-1] - srt[-2])
        out[f"step{g}_top_idx"], out[f"step{g}_top_val"] = top(lg)
    out["teacher_tokens"] = np.array(inputs, np.int32)   # the token fed at steps 1..
    ref.free()
    np.savez_compressed(os.path.join(HERE, "chain.npz"), **out)


# Conv stem (stream_conv_stem, voxtral.c:487-665): mel chunks of odd and even
# lengths, one frame, and a first chunk shorter than the kernel.
STEM_CHUNKS = [2, 150, 37, 1, 200, 64, 5]


def stem_chunks(seed=8201):
    return [B.normal_f32((n, B.MEL_BINS), seed + i, 1.0) for i, n in enumerate(STEM_CHUNKS)]


def gen_stem():
    out = {}
    w = B.ConvStemWeights(seed=DEC_SEED)
    ref = B.RefStem(w)
    for i, mel in enumerate(stem_chunks()):
        y = ref.step(mel)
        out[f"chunk{i}_rows"] = np.int32(y.shape[0])
        if y.size:
            pack(f"chunk{i}", y, out)
    ref.free()
    np.savez_compressed(os.path.join(HERE, "stem.npz"), **out)


# Log-mel front end (voxtral_audio.c).  Streaming: the stream path's left
# pad of 32 tokens of silence (voxtral.c:936) with feeds of 1, 159, 160, 161,
# 400 ... samples, the stream finish's zero feeds in 4096-sample pieces then
# vox_mel_finish(0) (voxtral.c:985-1003); and a context without left pad
# finished with right_pad > 0.  One-shot: the whole clip and clips of 150
# (rejected), 399, 500 and 561 samples.
MEL_AUDIO = 24000
MEL_FEEDS_A = [1, 159, 160, 161, 400, 3200, 7, 12000]
MEL_PAD_A = 40960
MEL_RIGHT_A = 1280 * 9 + 1000      # zeros fed before finish(0)
MEL_FEEDS_B = [399, 1, 5000]
MEL_RIGHT_B = 1000                 # finish(1000)
MEL_ONESHOT = [MEL_AUDIO, 150, 399, 500, 561]


def mel_audio(seed=8301):
    return B.synthetic_audio(MEL_AUDIO, seed)


def mel_feeds(feeds):
    return feeds + [MEL_AUDIO - sum(feeds)]


def gen_mel():
    out = {}
    x = mel_audio()
    out["audio_sum"] = checksum(x)
    for tag, pad, feeds, zeros, right in (("a", MEL_PAD_A, mel_feeds(MEL_FEEDS_A), MEL_RIGHT_A, 0),
                                          ("b", 0, mel_feeds(MEL_FEEDS_B), 0, MEL_RIGHT_B)):
        ref = B.RefMel(pad)
        off, rows = 0, []
        for f in feeds:
            rows.append(ref.feed(x[off:off + f]))
            off += f
        z = zeros
        while z > 0:
            c = min(z, 4096)
            rows.append(ref.feed(np.zeros(c, np.float32)))
            z -= c
        rows.append(ref.finish(right))
        out[f"{tag}_counts"] = np.array([r.shape[0] for r in rows], np.int32)
        pack(f"{tag}_mel", np.concatenate(rows, axis=0), out)
        ref.free()
    for n in MEL_ONESHOT:
        m = B.ref_mel_spectrogram(x[:n])
        out[f"oneshot{n}_frames"] = np.int32(0 if m is None else m.shape[0])
        if m is not None:
            pack(f"oneshot{n}", m, out)
    np.savez_compressed(os.path.join(HERE, "mel.npz"), **out)


# Audio front end end to end: samples -> incremental log-mel -> conv stem ->
# encoder -> adapter, chunked as the stream path chunks it
# (stream_run_encoder, voxtral.c:668-690): the first conv-stem call once 312
# mel frames are pending, later ones at 200; vox_stream_finish feeds the
# right pad as zeros (align to 1280 + (delay 6 + 1 + 10) tokens), finishes
# the mel and runs the rest (voxtral.c:979-1007).
FRONT_SAMPLES = 48000
FRONT_FEED = 8000
FRONT_LEFT_PAD = 32 * 1280
FRONT_DELAY = 6


def front_right_pad(n_samples):
    align = (1280 - n_samples % 1280) % 1280
    return align + (FRONT_DELAY + 1 + 10) * 1280


def front_stem_chunks(feed_frames, finish_frames):
    """Mel frames per conv-stem call for the given frames per feed."""
    chunks, pending, first = [], 0, True
    for n in feed_frames:
        pending += n
        if pending >= (312 if first else 200):
            chunks.append(pending)
            pending, first = 0, False
    pending += finish_frames
    if pending > 0:
        chunks.append(pending)
    return chunks


def front_audio(seed=8401):
    return B.synthetic_audio(FRONT_SAMPLES, seed)


def gen_front(ew):
    out = {}
    x = front_audio()
    out["audio_sum"] = checksum(x)
    mel = B.RefMel(FRONT_LEFT_PAD)
    rows = [mel.feed(x[o:o + FRONT_FEED]) for o in range(0, FRONT_SAMPLES, FRONT_FEED)]
    z = front_right_pad(FRONT_SAMPLES)
    tail = []
    while z > 0:
        c = min(z, 4096)
        tail.append(mel.feed(np.zeros(c, np.float32)))
        z -= c
    tail.append(mel.finish(0))
    mel.free()
    feed_frames = [r.shape[0] for r in rows]
    fin = sum(t.shape[0] for t in tail)
    chunks = front_stem_chunks(feed_frames, fin)
    out["stem_chunks"] = np.array(chunks, np.int32)
    all_mel = np.concatenate(rows + tail, axis=0)
    assert all_mel.shape[0] == sum(chunks)
    stem = B.RefStem(B.ConvStemWeights(seed=DEC_SEED))
    ref = B.RefCtx(enc=ew)
    enc, off = [], 0
    for i, n in enumerate(chunks):
        conv = stem.step(all_mel[off:off + n])
        off += n
        out[f"stem{i}_rows"] = np.int32(conv.shape[0])
        if conv.shape[0]:
            enc.append(ref.encoder_incremental(conv))
    enc = np.concatenate(enc, axis=0)
    pack("encoder", enc, out)
    usable = enc.shape[0] // 4 * 4
    pack("adapter", ref.adapter(enc[:usable]), out)
    stem.free()
    ref.free()
    np.savez_compressed(os.path.join(HERE, "front.npz"), **out)


# configs[3] at full length: 60 s of seeded synthetic 16 kHz audio fed in
# 2.0 s pieces through the stream path's front end (incremental log-mel with
# the 32-token left pad, conv stem at 312 then 200 pending mel frames, the
# encoder per stem chunk, the adapter over whole groups of 4 rows,
# voxtral.c:668-774), the 39-token prompt prefilled as 38 rows plus one step
# (voxtral.c:836-891), then greedy steps on the reference's own tokens
# (voxtral.c:893-921) to 750 generated tokens.  Every step's token and top-1
# margin is kept; the logits of a fixed set of steps are sampled.
E2E_SAMPLES = 60 * 16000
E2E_FEED = 32000
E2E_TOKENS = 750
E2E_LOGIT_STEPS = [0, 1, 2, 3, 10, 50, 100, 200, 300, 400, 500, 600, 700, 749]
E2E_LOGIT_SAMPLE = 8192


def e2e_audio(seed=8601):
    return B.synthetic_audio(E2E_SAMPLES, seed)


def e2e_mel_schedule(mel_feed, mel_finish):
    """Drive a mel context (host or device) the way the stream path does:
    (per-feed frame counts, tail frame count, list of mel frame arrays)."""
    x = e2e_audio()
    rows = [mel_feed(x[o:o + E2E_FEED]) for o in range(0, E2E_SAMPLES, E2E_FEED)]
    z = front_right_pad(E2E_SAMPLES)
    tail = []
    while z > 0:
        c = min(z, 4096)
        tail.append(mel_feed(np.zeros(c, np.float32)))
        z -= c
    tail.append(mel_finish())
    return [r.shape[0] for r in rows], sum(t.shape[0] for t in tail), rows + tail


def gen_e2e(w, ew):
    out = {}
    t0 = time.time()
    mel = B.RefMel(FRONT_LEFT_PAD)
    feed_frames, fin, parts = e2e_mel_schedule(mel.feed, lambda: mel.finish(0))
    mel.free()
    chunks = front_stem_chunks(feed_frames, fin)
    out["stem_chunks"] = np.array(chunks, np.int32)
    all_mel = np.concatenate(parts, axis=0)
    assert all_mel.shape[0] == sum(chunks)
    stem = B.RefStem(B.ConvStemWeights(seed=DEC_SEED))
    ref = B.RefCtx(dec=w, enc=ew)
    enc, off = [], 0
    for n in chunks:
        conv = stem.step(all_mel[off:off + n])
        off += n
        if conv.shape[0]:
            enc.append(ref.encoder_incremental(conv))
    stem.free()
    enc = np.concatenate(enc, axis=0)
    out["encoder_rows"] = np.int32(enc.shape[0])
    usable = enc.shape[0] // 4 * 4
    ad = ref.adapter(enc[:usable])
    del enc
    pack_vals("adapter", ad, out)
    print("e2e front end", ad.shape, time.time() - t0, flush=True)
    assert ad.shape[0] >= CHAIN_PROMPT - 1 + E2E_TOKENS
    prompt = np.stack([chain_embed(w, ad[i], TOKEN_BOS if i == 0 else TOKEN_PAD)
                       for i in range(CHAIN_PROMPT)])
    ref.decoder_prefill(prompt[:CHAIN_PROMPT - 1])
    toks = np.zeros(E2E_TOKENS, np.int32)
    margins = np.zeros(E2E_TOKENS, np.float32)
    tok, lg = ref.decoder_forward(prompt[CHAIN_PROMPT - 1])
    for g in range(E2E_TOKENS):
        if g > 0:
            tok, lg = ref.decoder_forward(chain_embed(w, ad[CHAIN_PROMPT - 1 + g], tok))
        toks[g] = tok
        srt = np.partition(lg, -2)[-2:]
        margins[g] = np.float32(abs(srt[1] - srt[0]))
        if g in E2E_LOGIT_STEPS:
            pack_vals(f"step{g}_logits", lg, out, E2E_LOGIT_SAMPLE)
        if g % 50 == 0:
            print("e2e step", g, time.time() - t0, flush=True)
    out["tokens"] = toks
    out["margins"] = margins
    out["state_after"] = np.array(ref.state(), np.int32)
    ref.free()
    np.savez_compressed(os.path.join(HERE, "e2e60.npz"), **out)


ALT_CASES = [(61, 3.0, 4, 0.999), (62, 0.5, 4, 0.5), (63, 8.0, 3, 0.99), (64, 1.0, 2, 0.9),
             (65, 0.01, 4, 0.999)]


def gen_alts():
    out = {}
    for i, (seed, std, n_alt, cut) in enumerate(ALT_CASES):
        lg = B.normal_f32(B.VOCAB, seed, std)
        best = int(np.argmax(lg))
        ids = B.ref_fill_alts(lg, best, n_alt, cut)
        out[f"case{i}_ids"] = np.array(ids, np.int32)
        out[f"case{i}_best"] = np.int32(best)
    np.savez_compressed(os.path.join(HERE, "alts.npz"), **out)


def main():
    assert B.ref_available(), "build oracle/_ref first (make -C oracle ref)"
    t = time.time()
    if sys.argv[1:] == ["front"]:   # only the audio front end chain
        gen_front(B.EncoderWeights(seed=DEC_SEED))
        print("front", time.time() - t)
        return
    if sys.argv[1:] == ["mel"]:   # only the log-mel front end
        gen_mel()
        print("mel", time.time() - t)
        return
    if sys.argv[1:] == ["stem"]:   # only the conv stem
        gen_stem()
        print("stem", time.time() - t)
        return
    if sys.argv[1:] == ["e2e60"]:   # only configs[3] at full length (~15 min)
        gen_e2e(B.DecoderWeights(seed=DEC_SEED), B.EncoderWeights(seed=DEC_SEED))
        print("e2e60", time.time() - t)
        return
    if sys.argv[1:] == ["batch8"]:   # only the 8-stream batched step
        gen_batch8(B.DecoderWeights(seed=DEC_SEED))
        print("batch8", time.time() - t)
        return
    if sys.argv[1:] == ["encoder_big"]:   # only the 500 / 1500-row encoder chunks
        gen_encoder_big(B.EncoderWeights(seed=DEC_SEED))
        print("encoder_big", time.time() - t)
        return
    if sys.argv[1:] == ["chain"]:   # only the end-to-end chain
        gen_chain(B.DecoderWeights(seed=DEC_SEED), B.EncoderWeights(seed=DEC_SEED))
        print("chain", time.time() - t)
        return
    gen_linear(); print("linear", time.time() - t)
    gen_rope(); print("rope", time.time() - t)
    gen_attention(); print("attention", time.time() - t)
    gen_alts(); print("alts", time.time() - t)
    gen_stem(); print("stem", time.time() - t)
    gen_mel(); print("mel", time.time() - t)
    w = B.DecoderWeights(seed=DEC_SEED)
    gen_decoder(w); print("decoder", time.time() - t)
    gen_batch8(w); print("batch8", time.time() - t)
    del w
    ew = B.EncoderWeights(seed=DEC_SEED)
    gen_encoder(ew); print("encoder", time.time() - t)
    gen_encoder_big(ew); print("encoder_big", time.time() - t)
    gen_chain(B.DecoderWeights(seed=DEC_SEED), ew); print("chain", time.time() - t)
    gen_front(ew); print("front", time.time() - t)
    gen_e2e(B.DecoderWeights(seed=DEC_SEED), ew); print("e2e60", time.time() - t)


if __name__ == "__main__":
    main()
