"""The `make cuda` build of the reference's own C host (integration/Makefile:
the reference's sources with the USE_CUDA hooks of integration/apply_cuda.py,
linked to libvoxtral_cuda.so) against the unpatched `make blas` build.

The patched host is driven through its own entry points - vox_decoder_prefill,
vox_decoder_forward, vox_encoder_forward_incremental, vox_adapter_forward and
vox_set_delay - on a context over seeded synthetic weights (oracle/ref_shim.c).
The expected outputs are the golden vectors the unpatched build produced
(tests/golden/decoder.npz, encoder.npz) or, for vox_set_delay, the unpatched
build run here on the same inputs.  The host's cache bookkeeping
(kv_cache_len, enc_kv_cache_len, enc_kv_pos_offset) must come out as the CPU
path leaves it."""
import numpy as np
import pytest

import bind as B
import gen_golden as G
from conftest import load_golden, unpack

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2     # contract: teacher-forced logits rel-L2 (the decode path reaches ~1e-5)
ENC_TOL = 2e-3       # 32 fp16-operand tensor-core encoder layers (measured ~4.4e-4)
MARGIN = 1e-3


@pytest.fixture(scope="module")
def host():
    assert B.host_cuda_available(), "integration/_build/libvoxhost_cuda.so missing (make -C integration)"
    lib = B.host_cuda_lib()
    assert lib.vox_cuda_init() == 1, lib.vox_cuda_last_error()
    return lib


def rel(arr, g, prefix):
    idx, val, _, size = unpack(g, prefix)
    flat = np.asarray(arr, np.float32).reshape(-1)
    assert flat.size == size
    return B.rel_l2(flat[idx], val)


def attached(host, **weights):
    ctx = B.RefCtx(lib=host, **weights)
    assert host.vox_cuda_host_attach(ctx.ctx) == 0, host.vox_cuda_last_error()
    return ctx


def release(host, ctx, free_ada=0):
    host.vox_cuda_host_detach(ctx.ctx)
    host.voxref_ctx_free(ctx.ctx, free_ada)
    ctx.ctx = None


@pytest.fixture(scope="module")
def dec_w():
    return B.DecoderWeights(seed=G.DEC_SEED)


def test_make_cuda_decoder_matches_blas_build(host, dec_w):
    g = load_golden("decoder")
    ctx = attached(host, dec=dec_w)
    ctx.decoder_prefill(G.dec_embeds(G.PROMPT, 7001))
    st = ctx.state()
    assert (st[0], st[2]) == (int(g["state_prefill"][0]), int(g["state_prefill"][2]))
    steps = G.dec_embeds(G.DEC_STEPS, 7002)
    for s in range(G.DEC_STEPS):
        tok, lg = ctx.decoder_forward(steps[s])
        r = rel(lg, g, f"step{s}_logits")
        assert r < LOGIT_TOL * 1e-2, (s, r)
        want = int(g[f"step{s}_token"])
        if tok != want:
            top = g[f"step{s}_top_val"]
            assert top[0] - top[1] <= MARGIN, (s, tok, want)
    st = ctx.state()
    assert (st[0], st[2]) == (int(g["state_after"][0]), int(g["state_after"][2]))
    release(host, ctx)


def test_make_cuda_encoder_and_adapter_match_blas_build(host):
    g = load_golden("encoder")
    ew = B.EncoderWeights(seed=G.DEC_SEED)
    ctx = attached(host, enc=ew)
    outs = []
    for i, x in enumerate(G.enc_chunks()):
        y = ctx.encoder_incremental(x)
        outs.append(y)
        assert rel(y, g, f"chunk{i}") < ENC_TOL, i
        st, want = ctx.state(), g[f"chunk{i}_state"]
        # enc_kv_cache_len and enc_kv_pos_offset as the CPU path leaves them
        assert (st[3], st[5]) == (int(want[3]), int(want[5])), (i, st, want.tolist())
    enc = np.concatenate(outs[:2], axis=0)[:136]
    assert rel(ctx.adapter(enc), g, "adapter136") < 1e-2
    release(host, ctx)


def seeded_ada_mlp(lib, ctx, keep):
    for layer in range(B.DEC_LAYERS):
        down = B.normal_f32((32, B.DEC_DIM), 9100 + 2 * layer, 0.02)
        up = B.normal_f32((B.DEC_DIM, 32), 9101 + 2 * layer, 0.02)
        keep += [down, up]
        lib.voxref_set_ada_mlp(ctx.ctx, layer, B.fptr(down), B.fptr(up))


def run_prompt(ctx, lib, rows, step):
    lib.voxref_set_dec_kv_state(ctx.ctx, 0, 0)   # a new stream (voxtral.c:857-858)
    ctx.decoder_prefill(rows)
    return ctx.decoder_forward(step)


def test_make_cuda_set_delay_rewrites_the_device_ada_scale(host, dec_w):
    """vox_set_delay (voxtral.c:1344-1350) recomputes the time conditioning;
    the patched build passes it to the device without re-uploading weights.
    Logits before and after a delay change match the unpatched build's."""
    import copy
    ref_lib = B.ref_lib()
    keep = []
    w = copy.copy(dec_w)
    w.ada_scale = None    # each context computes (and owns) its own
    cpu = B.RefCtx(dec=w)
    gpu = B.RefCtx(dec=w, lib=host)
    for lib, ctx in ((ref_lib, cpu), (host, gpu)):
        seeded_ada_mlp(lib, ctx, keep)
        lib.voxref_time_conditioning(ctx.ctx, 6)     # the default delay of vox_load
    assert host.vox_cuda_host_attach(gpu.ctx) == 0, host.vox_cuda_last_error()
    rows = B.normal_f32((5, B.DEC_DIM), 9201, 1.0)
    step = B.normal_f32(B.DEC_DIM, 9202, 1.0)
    logits = {}
    for delay_ms in (480, 1200):
        for lib, ctx, tag in ((ref_lib, cpu, "cpu"), (host, gpu, "gpu")):
            lib.vox_set_delay(ctx.ctx, delay_ms)
            logits[(tag, delay_ms)] = run_prompt(ctx, lib, rows, step)
    for d in (480, 1200):
        (t_c, l_c), (t_g, l_g) = logits[("cpu", d)], logits[("gpu", d)]
        assert B.rel_l2(l_g, l_c) < LOGIT_TOL * 1e-2, (d, B.rel_l2(l_g, l_c))
        assert t_g == t_c or np.sort(l_c)[-1] - np.sort(l_c)[-2] <= MARGIN
    # the delay changes the output at all
    assert B.rel_l2(logits[("cpu", 480)][1], logits[("cpu", 1200)][1]) > 1e-3
    release(host, gpu, free_ada=1)
    ref_lib.voxref_ctx_free(cpu.ctx, 1)
    cpu.ctx = None
