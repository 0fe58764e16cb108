"""BASELINE configs[3] at full length against the reference's own CPU path:
60 s of seeded synthetic 16 kHz audio -> incremental log-mel (2.0 s feeds,
the stream path's 32-token left pad and finishing right pad) -> conv stem on
the stream path's schedule -> 32-layer encoder (its ring wraps many times
over ~3150 rows) -> adapter -> the 39-token prompt prefilled as 38 rows plus
one step -> 749 more greedy steps, teacher-forced on the reference's tokens
(voxtral.c:668-774, 836-921).  Golden: tests/golden/e2e60.npz
(gen_golden.py gen_e2e).

Contract (north_star): teacher-forced logits within 1e-2 relative L2, greedy
token ids bit-exact wherever the reference's top-1 margin exceeds 1e-3."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
import voxcuda as V
from conftest import load_golden

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2      # contract: teacher-forced logits rel-L2
ADAPTER_TOL = 2e-3    # log-mel + fp16 stem + 32 fp16-operand encoder layers + adapter
MARGIN = 1e-3         # contract: ids exact where the reference's top-1 margin exceeds this


@pytest.fixture(scope="module", autouse=True)
def cuda():
    V.init()
    yield


def gpu_front_end(x_unused=None):
    """Samples -> adapter rows through the library's host entry points."""
    ew = B.EncoderWeights(seed=G.DEC_SEED)
    enc = V.Encoder([tuple(ew.layer_w[i]) + tuple(ew.layer_b[i]) + tuple(ew.layer_n[i])
                     for i in range(ew.n_layers)], ew.norm, ew.adapter0, ew.adapter1)
    cw = B.ConvStemWeights(seed=G.DEC_SEED)
    mel = V.Mel(G.FRONT_LEFT_PAD, G.E2E_FEED)
    feed_frames, fin, parts = G.e2e_mel_schedule(mel.feed, lambda: mel.finish(0))
    mel.free()
    chunks = G.front_stem_chunks(feed_frames, fin)
    all_mel = np.concatenate(parts, axis=0)
    stem = V.ConvStem(cw.w0, cw.b0, cw.w1, cw.b1, max_mel=max(chunks))
    st_rows = max(chunks) // 2 + 2
    st = enc.state(max_chunk=st_rows)
    outs, off = [], 0
    for n in chunks:
        conv = stem.step(all_mel[off:off + n])
        off += n
        if conv.shape[0]:
            outs.append(st.step(conv))
    enc_out = np.concatenate(outs, axis=0)
    usable = enc_out.shape[0] // 4 * 4
    piece = st_rows // 4 * 4    # the adapter's rows per call fit the state's workspace
    ad = np.concatenate([st.adapter(enc_out[r:min(r + piece, usable)]) for r in range(0, usable, piece)], axis=0)
    st.free()
    stem.free()
    enc.free()
    return chunks, enc_out.shape[0], ad


def test_60s_audio_to_750_tokens_matches_reference():
    g = load_golden("e2e60")
    chunks, enc_rows, ad = gpu_front_end()
    assert chunks == g["stem_chunks"].tolist()
    assert enc_rows == int(g["encoder_rows"])
    flat = ad.reshape(-1)
    assert flat.size == int(g["adapter_size"])
    rel_ad = B.rel_l2(flat[G.sample_idx(flat.size)], g["adapter_val"])

    w = B.DecoderWeights(seed=G.DEC_SEED)
    dec = V.Decoder(w.tok_emb, w.norm, [tuple(w.layer_w[i]) + tuple(w.layer_n[i]) for i in range(w.n_layers)],
                    ada_scale=w.ada_scale, vocab=w.vocab)
    ds = dec.state()
    P = G.CHAIN_PROMPT
    prompt = np.stack([G.chain_embed(w, ad[i], G.TOKEN_BOS if i == 0 else G.TOKEN_PAD) for i in range(P)])
    ds.prefill(prompt[:P - 1])
    ref_toks, margins = g["tokens"], g["margins"]
    rels, mism, checked = {}, [], 0
    for s in range(G.E2E_TOKENS):
        embed = prompt[P - 1] if s == 0 else G.chain_embed(w, ad[P - 1 + s], int(ref_toks[s - 1]))
        want_lg = s in G.E2E_LOGIT_STEPS
        tok, lg = ds.step(embed, want_logits=want_lg)
        if want_lg:
            idx = G.sample_n(lg.size, G.E2E_LOGIT_SAMPLE)
            rels[s] = B.rel_l2(lg[idx], g[f"step{s}_logits_val"])
        if float(margins[s]) > MARGIN:
            checked += 1
            if tok != int(ref_toks[s]):
                mism.append((s, tok, int(ref_toks[s]), float(margins[s])))
    assert ds.position == P - 1 + G.E2E_TOKENS
    ds.free()
    dec.free()
    print(f"e2e60: adapter rel-L2 {rel_ad:.2e}; logits rel-L2 {rels}; "
          f"{checked} of {G.E2E_TOKENS} steps above the margin, mismatches {mism}")
    assert rel_ad < ADAPTER_TOL
    assert max(rels.values()) < LOGIT_TOL, rels
    assert not mism, mism
