"""The audio front end end to end on the device: 16 kHz samples -> incremental
log-mel -> conv stem -> 32-layer encoder -> adapter, chunked as the
reference's stream path chunks it (stream_run_encoder, voxtral.c:668-690;
vox_stream_finish, :979-1007), against the reference's own mel, stem,
encoder and adapter on the same schedule (golden tests/golden/front.npz,
gen_golden.py gen_front).

Then the same chain through the device-resident entry points (mel_feed_dev
-> conv_stem_step_dev -> encoder_step_dev, one CUDA stream, no host waits):
bit-identical to the host entry points."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
import voxcuda as V
from conftest import load_golden, unpack

pytestmark = pytest.mark.gpu

# log-mel (~3e-5) -> two fp16 conv GEMMs (~4e-4) -> 32 encoder layers of fp16
# tensor-core GEMMs (~5e-4 alone); the chain test's adapter bound applies
ENC_TOL = 2e-3
ADAPTER_TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def cuda():
    V.init()
    yield


@pytest.fixture(scope="module")
def front():
    ew = B.EncoderWeights(seed=G.DEC_SEED)
    enc = V.Encoder([tuple(ew.layer_w[i]) + tuple(ew.layer_b[i]) + tuple(ew.layer_n[i])
                     for i in range(ew.n_layers)], ew.norm, ew.adapter0, ew.adapter1)
    cw = B.ConvStemWeights(seed=G.DEC_SEED)
    yield enc, cw
    enc.free()


def host_chain(enc, cw, x):
    """The host entry points: mel rows per feed, stem calls on the stream
    path's schedule, encoder rows."""
    mel = V.Mel(G.FRONT_LEFT_PAD, G.FRONT_FEED)
    rows = [mel.feed(x[o:o + G.FRONT_FEED]) for o in range(0, x.size, G.FRONT_FEED)]
    z, tail = G.front_right_pad(x.size), []
    while z > 0:
        c = min(z, 4096)
        tail.append(mel.feed(np.zeros(c, np.float32)))
        z -= c
    tail.append(mel.finish(0))
    mel.free()
    chunks = G.front_stem_chunks([r.shape[0] for r in rows], sum(t.shape[0] for t in tail))
    all_mel = np.concatenate(rows + tail, axis=0)
    stem = V.ConvStem(cw.w0, cw.b0, cw.w1, cw.b1, max_mel=512)
    st = enc.state(max_chunk=512)   # the adapter runs over all rows at once
    conv_rows, outs, off = [], [], 0
    for n in chunks:
        conv = stem.step(all_mel[off:off + n])
        off += n
        conv_rows.append(conv.shape[0])
        if conv.shape[0]:
            outs.append(st.step(conv))
    out = np.concatenate(outs, axis=0)
    usable = out.shape[0] // 4 * 4
    ad = st.adapter(out[:usable])
    st.free()
    stem.free()
    return chunks, conv_rows, out, ad


def test_audio_to_adapter_matches_reference(front):
    enc, cw = front
    g = load_golden("front")
    x = G.front_audio()
    assert str(g["audio_sum"]) == str(G.checksum(x)), "audio generator changed"
    chunks, conv_rows, out, ad = host_chain(enc, cw, x)
    assert chunks == g["stem_chunks"].tolist()
    assert conv_rows == [int(g[f"stem{i}_rows"]) for i in range(len(chunks))]
    idx, val, _, size = unpack(g, "encoder")
    assert out.size == size
    rel_enc = B.rel_l2(out.reshape(-1)[idx], val)
    idx, val, _, size = unpack(g, "adapter")
    assert ad.size == size
    rel_ad = B.rel_l2(ad.reshape(-1)[idx], val)
    print("front: encoder rel-L2", rel_enc, "adapter rel-L2", rel_ad)
    assert rel_enc < ENC_TOL
    assert rel_ad < ADAPTER_TOL


def test_device_resident_front_matches_host_entry_points(front):
    import torch
    enc, cw = front
    x = G.front_audio()
    chunks, conv_rows, want, _ = host_chain(enc, cw, x)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    xd = torch.from_numpy(x).cuda()
    zeros = torch.zeros(4096, dtype=torch.float32, device="cuda")
    mel = V.Mel(G.FRONT_LEFT_PAD, G.FRONT_FEED)
    mel_buf = torch.empty((2048, 128), dtype=torch.float32, device="cuda")
    n_mel = 0
    torch.cuda.synchronize()
    for o in range(0, x.size, G.FRONT_FEED):
        n_mel += mel.feed_dev(xd.data_ptr() + 4 * o, G.FRONT_FEED, mel_buf[n_mel].data_ptr(),
                              mel_buf.shape[0] - n_mel, sp)
    z = G.front_right_pad(x.size)
    while z > 0:
        c = min(z, 4096)
        n_mel += mel.feed_dev(zeros.data_ptr(), c, mel_buf[n_mel].data_ptr(), mel_buf.shape[0] - n_mel, sp)
        z -= c
    n_mel += mel.finish_dev(0, mel_buf[n_mel].data_ptr(), mel_buf.shape[0] - n_mel, sp)
    assert n_mel == sum(chunks)
    stem = V.ConvStem(cw.w0, cw.b0, cw.w1, cw.b1, max_mel=512)
    st = enc.state(max_chunk=256)
    enc_buf = torch.empty((sum(conv_rows), 1280), dtype=torch.float32, device="cuda")
    off, row = 0, 0
    for n, r in zip(chunks, conv_rows):
        got = stem.step_dev(mel_buf[off].data_ptr(), n, enc_buf[row].data_ptr(), sp)
        assert got == r
        off += n
        if r:
            st.step_dev(enc_buf[row].data_ptr(), r, sp)   # in place: stem rows -> encoder rows
        row += r
    stream.synchronize()
    assert np.array_equal(enc_buf.cpu().numpy(), want)
    st.free()
    stem.free()
    mel.free()
