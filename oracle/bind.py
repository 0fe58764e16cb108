"""ctypes bindings for the test oracles.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg / ``--impl reference`` arm of bench.py may import this
module.  It wraps

* ``oracle/liboracle.so`` - vo_oracle.c, the C restatement of the reference's
  hot path (always built by ``__graft_entry__.build()``), and
* ``oracle/_ref/libvoxref.so`` - the reference's own CPU path compiled from its
  sources (present only where the reference tree was available at build time).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO_V3 = os.path.join(HERE, "_ref", "libvoxref.so")
REF_SO_V4 = os.path.join(HERE, "_ref", "libvoxref_v4.so")


def _host_has_avx512():
    """True where /proc/cpuinfo lists the x86-64-v4 extensions."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    fl = set(line.split(":", 1)[1].split())
                    return {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= fl
    except OSError:
        pass
    return False


# The reference's own Makefile builds with -march=native; the build here
# matching this host's CPU stands in for it (x86-64-v4 with AVX-512, else v3).
REF_SO = REF_SO_V4 if (_host_has_avx512() and os.path.exists(REF_SO_V4)) else REF_SO_V3
REF_MARCH = "x86-64-v4" if REF_SO == REF_SO_V4 else "x86-64-v3"

DEC_DIM, DEC_LAYERS, DEC_HEADS, DEC_KV_HEADS, DEC_HEAD_DIM = 3072, 26, 32, 8, 128
DEC_HIDDEN, DEC_WINDOW, VOCAB = 9216, 8192, 131072
Q_DIM, KV_DIM = DEC_HEADS * DEC_HEAD_DIM, DEC_KV_HEADS * DEC_HEAD_DIM
ENC_DIM, ENC_LAYERS, ENC_HEADS, ENC_HEAD_DIM, ENC_HIDDEN, ENC_WINDOW = 1280, 32, 32, 64, 5120, 750
ENC_QKV = ENC_HEADS * ENC_HEAD_DIM
ROPE_THETA = 1.0e6

_fp = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)
_ip = C.POINTER(C.c_int)


def fptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def u16ptr(a):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def iptr(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


_oracle = None
_ref = None


def oracle_lib():
    global _oracle
    if _oracle is None:
        lib = C.CDLL(ORACLE_SO)
        lib.vo_fill_normal_f32.argtypes = [_fp, C.c_size_t, C.c_uint64, C.c_float, C.c_float]
        lib.vo_fill_normal_bf16.argtypes = [_u16p, C.c_size_t, C.c_uint64, C.c_float]
        lib.vo_linear_bf16.argtypes = [_fp, _fp, _u16p, _fp, C.c_int, C.c_int, C.c_int]
        lib.vo_rms_norm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_float]
        lib.vo_silu.argtypes = [_fp, C.c_size_t]
        lib.vo_gelu.argtypes = [_fp, C.c_size_t]
        lib.vo_rope_freqs.argtypes = [_fp, _ip, C.c_int, C.c_int, C.c_float]
        lib.vo_apply_rope.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int]
        lib.vo_causal_attention.argtypes = [_fp, _fp, _fp, _fp] + [C.c_int] * 5 + [
            C.c_float, C.c_int, C.c_int]
        lib.vo_argmax.argtypes = [_fp, C.c_int]
        lib.vo_argmax.restype = C.c_int
        lib.vo_fill_alts.argtypes = [_fp, C.c_int, C.c_int, C.c_int, C.c_float, _ip]
        lib.vo_fill_alts.restype = C.c_int
        lib.vo_decoder_step.argtypes = [C.c_void_p, C.c_void_p, _fp, _fp]
        lib.vo_decoder_step.restype = C.c_int
        lib.vo_decoder_prefill.argtypes = [C.c_void_p, C.c_void_p, _fp, C.c_int]
        lib.vo_decoder_prefill.restype = C.c_int
        lib.vo_encoder_step.argtypes = [C.c_void_p, C.c_void_p, _fp, C.c_int]
        lib.vo_encoder_step.restype = C.c_int
        lib.vo_adapter.argtypes = [_u16p, _u16p, _fp, C.c_int, _fp]
        lib.vo_adapter.restype = C.c_int
        _oracle = lib
    return _oracle


def ref_available():
    return os.path.exists(REF_SO)


HOST_CUDA_SO = os.path.join(HERE, "..", "integration", "_build", "libvoxhost_cuda.so")
_host_cuda = None


def host_cuda_available():
    return os.path.exists(HOST_CUDA_SO)


def host_cuda_lib():
    """The reference host built as `make cuda` (integration/Makefile): its own
    sources with the USE_CUDA hooks, linked to libvoxtral_cuda.so, plus the
    ref_shim.c test entry points.  Same functions as ref_lib(), and
    vox_cuda_init / vox_cuda_host_attach / vox_cuda_host_detach / vox_set_delay."""
    global _host_cuda
    if _host_cuda is None:
        lib = _setup_ref(C.CDLL(HOST_CUDA_SO))
        lib.vox_cuda_init.restype = C.c_int
        lib.vox_cuda_last_error.restype = C.c_char_p
        lib.vox_cuda_host_attach.argtypes = [C.c_void_p]
        lib.vox_cuda_host_attach.restype = C.c_int
        lib.vox_cuda_host_detach.argtypes = [C.c_void_p]
        _host_cuda = lib
    return _host_cuda


def ref_lib():
    global _ref
    if _ref is None:
        _ref = _setup_ref(C.CDLL(REF_SO))
    return _ref


def _setup_ref(lib):
    if True:
        lib.vox_linear_nobias_bf16.argtypes = [_fp, _fp, _u16p, C.c_int, C.c_int, C.c_int]
        lib.vox_linear_bf16.argtypes = [_fp, _fp, _u16p, _fp, C.c_int, C.c_int, C.c_int]
        lib.vox_matmul_t_bf16.argtypes = [_fp, _fp, _u16p, C.c_int, C.c_int, C.c_int]
        lib.vox_rms_norm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_float]
        lib.vox_silu.argtypes = [_fp, C.c_int]
        lib.vox_gelu.argtypes = [_fp, C.c_int]
        lib.vox_compute_rope_freqs.argtypes = [_fp, _ip, C.c_int, C.c_int, C.c_float]
        lib.vox_apply_rope.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int]
        lib.vox_causal_attention.argtypes = [_fp, _fp, _fp, _fp] + [C.c_int] * 5 + [
            C.c_float, C.c_int, C.c_int]
        lib.voxref_ctx_new.restype = C.c_void_p
        lib.voxref_set_decoder.argtypes = [C.c_void_p, _u16p, _fp, C.c_void_p, C.c_void_p, _fp]
        lib.voxref_set_encoder.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, _fp]
        lib.voxref_set_adapter.argtypes = [C.c_void_p, _u16p, _u16p]
        lib.voxref_set_ada_mlp.argtypes = [C.c_void_p, C.c_int, _fp, _fp]
        lib.voxref_time_conditioning.argtypes = [C.c_void_p, C.c_int]
        lib.voxref_time_conditioning.restype = _fp
        lib.vox_set_delay.argtypes = [C.c_void_p, C.c_int]
        lib.voxref_decoder_forward.argtypes = [C.c_void_p, _fp, _fp]
        lib.voxref_decoder_forward.restype = C.c_int
        lib.voxref_decoder_prefill.argtypes = [C.c_void_p, _fp, C.c_int]
        lib.voxref_decoder_kv_preallocate.argtypes = [C.c_void_p, C.c_int]
        lib.voxref_encoder_kv_preallocate.argtypes = [C.c_void_p, C.c_int]
        lib.voxref_encoder_incremental.argtypes = [C.c_void_p, _fp, C.c_int, _fp]
        lib.voxref_encoder_incremental.restype = C.c_int
        lib.voxref_adapter.argtypes = [C.c_void_p, _fp, C.c_int, _fp]
        lib.voxref_adapter.restype = C.c_int
        lib.voxref_get_state.argtypes = [C.c_void_p, _ip]
        lib.voxref_set_dec_kv_state.argtypes = [C.c_void_p, C.c_int, C.c_int]
        lib.voxref_set_enc_kv_state.argtypes = [C.c_void_p, C.c_int, C.c_int]
        for n in ("voxref_dec_kv_k", "voxref_dec_kv_v", "voxref_enc_kv_k", "voxref_enc_kv_v"):
            getattr(lib, n).argtypes = [C.c_void_p]
            getattr(lib, n).restype = _fp
        lib.voxref_ctx_free.argtypes = [C.c_void_p, C.c_int]
        lib.voxref_fill_alts.argtypes = [_fp, C.c_int, C.c_int, C.c_float, _ip]
        lib.voxref_fill_alts.restype = C.c_int
        lib.voxref_decode_threads.argtypes = [C.c_void_p, C.c_int, C.c_int, _fp, _fp, _ip]
        lib.voxref_decode_threads.restype = C.c_double
        # incremental log-mel (voxtral_audio.h:40-63) and the one-shot form (:33)
        lib.vox_mel_ctx_init.argtypes = [C.c_int]
        lib.vox_mel_ctx_init.restype = C.c_void_p
        lib.vox_mel_feed.argtypes = [C.c_void_p, _fp, C.c_int]
        lib.vox_mel_feed.restype = C.c_int
        lib.vox_mel_finish.argtypes = [C.c_void_p, C.c_int]
        lib.vox_mel_finish.restype = C.c_int
        lib.vox_mel_data.argtypes = [C.c_void_p, _ip]
        lib.vox_mel_data.restype = _fp
        lib.vox_mel_free.argtypes = [C.c_void_p]
        lib.vox_mel_spectrogram.argtypes = [_fp, C.c_int, _ip]
        lib.vox_mel_spectrogram.restype = _fp
        lib.free.argtypes = [C.c_void_p]
        lib.voxref_set_conv.argtypes = [C.c_void_p, _fp, _fp, _fp, _fp]
        lib.voxref_stem_new.argtypes = [C.c_void_p]
        lib.voxref_stem_new.restype = C.c_void_p
        lib.voxref_stem_step.argtypes = [C.c_void_p, _fp, C.c_int, _fp]
        lib.voxref_stem_step.restype = C.c_int
        lib.voxref_stem_free.argtypes = [C.c_void_p]
    return lib


# ---------------------------------------------------------------------------
# seeded synthetic data
# ---------------------------------------------------------------------------

def normal_f32(shape, seed, std=1.0, mean=0.0):
    a = np.empty(shape, dtype=np.float32)
    oracle_lib().vo_fill_normal_f32(fptr(a.reshape(-1)), a.size, seed, mean, std)
    return a


def normal_bf16(shape, seed, std=0.02):
    a = np.empty(shape, dtype=np.uint16)
    oracle_lib().vo_fill_normal_bf16(u16ptr(a.reshape(-1)), a.size, seed, std)
    return a


def bf16_to_f32(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64).reshape(-1)
    b = np.asarray(b, dtype=np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ---------------------------------------------------------------------------
# oracle kernels
# ---------------------------------------------------------------------------

def linear(x, W, b=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0] if x.ndim == 2 else 1
    N, K = W.shape
    y = np.empty((M, N), dtype=np.float32)
    oracle_lib().vo_linear_bf16(fptr(y), fptr(x), u16ptr(W), fptr(b), M, K, N)
    return y


def rms_norm(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    M = x.shape[0] if x.ndim == 2 else 1
    oracle_lib().vo_rms_norm(fptr(out), fptr(x), fptr(w), M, x.shape[-1], eps)
    return out


def rope_freqs(positions, head_dim):
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    f = np.empty((pos.size, head_dim), dtype=np.float32)
    oracle_lib().vo_rope_freqs(fptr(f), iptr(pos), pos.size, head_dim, ROPE_THETA)
    return f


def apply_rope(x, freqs, heads, head_dim):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    oracle_lib().vo_apply_rope(fptr(x), fptr(freqs), freqs.shape[0], heads, head_dim)
    return x


def causal_attention(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, window, q_offset):
    out = np.empty((seq_q, n_heads * head_dim), dtype=np.float32)
    oracle_lib().vo_causal_attention(fptr(out), fptr(Q), fptr(K), fptr(V), seq_q, seq_k,
                                     n_heads, n_kv_heads, head_dim,
                                     np.float32(1.0) / np.sqrt(np.float32(head_dim)),
                                     window, q_offset)
    return out


def fill_alts(logits, best, n_alt, cutoff):
    ids = np.full(4, -1, dtype=np.int32)
    n = oracle_lib().vo_fill_alts(fptr(np.ascontiguousarray(logits, dtype=np.float32)),
                                  logits.size, best, n_alt, cutoff, iptr(ids))
    return ids[:n].tolist()


# ---------------------------------------------------------------------------
# synthetic decoder / encoder weights (reference layout, bf16 row-major)
# ---------------------------------------------------------------------------

MEL_BINS = 128


class ConvStemWeights:
    """The encoder's conv stem (voxtral.h:84-88): conv0 [1280, 128, 3] and
    conv1 [1280, 1280, 3] fp32 with fp32 biases, seeded."""

    def __init__(self, seed=0, std=0.02):
        s = seed * 1000 + 60000
        self.w0 = normal_f32((ENC_DIM, MEL_BINS, 3), s + 1, std)
        self.b0 = normal_f32(ENC_DIM, s + 2, std)
        self.w1 = normal_f32((ENC_DIM, ENC_DIM, 3), s + 3, std)
        self.b1 = normal_f32(ENC_DIM, s + 4, std)


class RefStem:
    """The reference's stateful conv stem (stream_conv_stem) over a bare stream."""

    def __init__(self, w: ConvStemWeights):
        lib = ref_lib()
        self.lib, self.w = lib, w
        self.ctx = lib.voxref_ctx_new()
        lib.voxref_set_conv(self.ctx, fptr(w.w0), fptr(w.b0), fptr(w.w1), fptr(w.b1))
        self.st = lib.voxref_stem_new(self.ctx)

    def step(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        out = np.empty((mel.shape[0] // 2 + 2, ENC_DIM), np.float32)
        n = self.lib.voxref_stem_step(self.st, fptr(mel), mel.shape[0], fptr(out))
        return out[:n].copy()

    def free(self):
        if self.st:
            self.lib.voxref_stem_free(self.st)
            self.lib.voxref_ctx_free(self.ctx, 0)
            self.st = None


SAMPLE_RATE = 16000
HOP = 160
RAW_AUDIO_PER_TOKEN = 1280     # samples per decoder token (voxtral.h, 80 ms)


def synthetic_audio(n, seed, level_db=-20.0):
    """Seeded test audio in [-1, 1]: pink-ish noise (a one-pole low-pass of
    white noise) plus tone bursts of 200-3000 Hz, scaled to `level_db` dBFS
    RMS.  Stands in for the reference's sample WAVs (not part of the tree)."""
    rng = np.random.default_rng(seed)
    white = rng.standard_normal(n).astype(np.float64)
    pink = np.empty(n)
    acc = 0.0
    for i in range(n):          # small n only (tests)
        acc = 0.97 * acc + white[i]
        pink[i] = acc
    t = np.arange(n) / SAMPLE_RATE
    tones = np.zeros(n)
    for _ in range(max(1, n // 8000)):
        f = rng.uniform(200.0, 3000.0)
        a0 = int(rng.integers(0, max(1, n - 1)))
        ln = int(rng.integers(800, 6400))
        sl = slice(a0, min(n, a0 + ln))
        tones[sl] += np.sin(2 * np.pi * f * t[sl]) * 3.0
    x = pink / (np.std(pink) + 1e-12) + tones
    x *= 10 ** (level_db / 20.0) / (np.sqrt(np.mean(x * x)) + 1e-12)
    return np.clip(x, -1.0, 1.0).astype(np.float32)


class RefMel:
    """The reference's incremental log-mel context (vox_mel_ctx_t,
    voxtral_audio.c:392-612)."""

    def __init__(self, left_pad_samples):
        self.lib = ref_lib()
        self.ctx = self.lib.vox_mel_ctx_init(left_pad_samples)
        assert self.ctx
        self.seen = 0

    def _new_frames(self):
        n = np.zeros(1, np.int32)
        p = self.lib.vox_mel_data(self.ctx, iptr(n))
        total = int(n[0])
        if total <= self.seen:
            self.seen = total
            return np.zeros((0, MEL_BINS), np.float32)
        arr = np.ctypeslib.as_array(p, shape=(total * MEL_BINS,)).reshape(total, MEL_BINS)
        out = arr[self.seen:total].copy()
        self.seen = total
        return out

    def feed(self, samples):
        samples = np.ascontiguousarray(samples, np.float32)
        self.lib.vox_mel_feed(self.ctx, fptr(samples), samples.size)
        return self._new_frames()

    def finish(self, right_pad_samples=0):
        self.lib.vox_mel_finish(self.ctx, right_pad_samples)
        return self._new_frames()

    def free(self):
        if self.ctx:
            self.lib.vox_mel_free(self.ctx)
            self.ctx = None


def ref_mel_spectrogram(samples):
    """The reference's one-shot vox_mel_spectrogram (voxtral_audio.c:290-395):
    [frames, 128], or None where it rejects the input as too short."""
    lib = ref_lib()
    samples = np.ascontiguousarray(samples, np.float32)
    n = np.zeros(1, np.int32)
    p = lib.vox_mel_spectrogram(fptr(samples), samples.size, iptr(n))
    if not p:
        return None
    out = np.ctypeslib.as_array(p, shape=(int(n[0]) * MEL_BINS,)).reshape(-1, MEL_BINS).copy()
    lib.free(C.cast(p, C.c_void_p))
    return out


class DecoderWeights:
    """Decoder weights: `distinct` independent layer sets cycled over
    `n_layers` layers (aliasing keeps host memory small for parity runs; the
    reference reads them exactly as it would read 26 distinct layers)."""

    def __init__(self, seed=0, n_layers=DEC_LAYERS, distinct=2, vocab=VOCAB, ada=True,
                 norm_noise=0.0):
        self.n_layers, self.vocab = n_layers, vocab
        s = seed * 1000
        self.sets = []
        for d in range(distinct):
            b = s + 100 * (d + 1)
            ws = [normal_bf16((Q_DIM, DEC_DIM), b + 1), normal_bf16((KV_DIM, DEC_DIM), b + 2),
                  normal_bf16((KV_DIM, DEC_DIM), b + 3), normal_bf16((DEC_DIM, Q_DIM), b + 4),
                  normal_bf16((DEC_HIDDEN, DEC_DIM), b + 5), normal_bf16((DEC_DIM, DEC_HIDDEN), b + 6),
                  normal_bf16((DEC_HIDDEN, DEC_DIM), b + 7)]
            if norm_noise:
                ns = [normal_f32(DEC_DIM, b + 8, norm_noise, 1.0), normal_f32(DEC_DIM, b + 9, norm_noise, 1.0)]
            else:
                ns = [np.ones(DEC_DIM, np.float32), np.ones(DEC_DIM, np.float32)]
            self.sets.append((ws, ns))
        self.tok_emb = normal_bf16((vocab, DEC_DIM), s + 7)
        self.norm = np.ones(DEC_DIM, np.float32)
        self.ada_scale = normal_f32((n_layers, DEC_DIM), s + 9, 0.1) if ada else None
        self.layer_w = [self.sets[i % distinct][0] for i in range(n_layers)]
        self.layer_n = [self.sets[i % distinct][1] for i in range(n_layers)]

    def pointer_arrays(self):
        lw = (C.c_void_p * (7 * self.n_layers))()
        ln = (C.c_void_p * (2 * self.n_layers))()
        for i in range(self.n_layers):
            for j in range(7):
                lw[7 * i + j] = self.layer_w[i][j].ctypes.data
            for j in range(2):
                ln[2 * i + j] = self.layer_n[i][j].ctypes.data
        return lw, ln


class EncoderWeights:
    def __init__(self, seed=0, n_layers=ENC_LAYERS, distinct=2, norm_noise=0.0):
        self.n_layers = n_layers
        s = seed * 1000 + 50000
        self.sets = []
        for d in range(distinct):
            b = s + 100 * (d + 1)
            ws = [normal_bf16((ENC_QKV, ENC_DIM), b + 1), normal_bf16((ENC_QKV, ENC_DIM), b + 2),
                  normal_bf16((ENC_QKV, ENC_DIM), b + 3), normal_bf16((ENC_DIM, ENC_QKV), b + 4),
                  normal_bf16((ENC_HIDDEN, ENC_DIM), b + 5), normal_bf16((ENC_DIM, ENC_HIDDEN), b + 6),
                  normal_bf16((ENC_HIDDEN, ENC_DIM), b + 7)]
            bs = [normal_f32(ENC_QKV, b + 8, 0.02), normal_f32(ENC_QKV, b + 9, 0.02),
                  normal_f32(ENC_DIM, b + 10, 0.02), normal_f32(ENC_DIM, b + 11, 0.02)]
            if norm_noise:
                ns = [normal_f32(ENC_DIM, b + 12, norm_noise, 1.0), normal_f32(ENC_DIM, b + 13, norm_noise, 1.0)]
            else:
                ns = [np.ones(ENC_DIM, np.float32), np.ones(ENC_DIM, np.float32)]
            self.sets.append((ws, bs, ns))
        self.norm = np.ones(ENC_DIM, np.float32)
        self.layer_w = [self.sets[i % distinct][0] for i in range(n_layers)]
        self.layer_b = [self.sets[i % distinct][1] for i in range(n_layers)]
        self.layer_n = [self.sets[i % distinct][2] for i in range(n_layers)]
        self.adapter0 = normal_bf16((DEC_DIM, 4 * ENC_DIM), s + 20)
        self.adapter1 = normal_bf16((DEC_DIM, DEC_DIM), s + 21)

    def pointer_arrays(self):
        lw = (C.c_void_p * (7 * self.n_layers))()
        lb = (C.c_void_p * (4 * self.n_layers))()
        ln = (C.c_void_p * (2 * self.n_layers))()
        for i in range(self.n_layers):
            for j in range(7):
                lw[7 * i + j] = self.layer_w[i][j].ctypes.data
            for j in range(4):
                lb[4 * i + j] = self.layer_b[i][j].ctypes.data
            for j in range(2):
                ln[2 * i + j] = self.layer_n[i][j].ctypes.data
        return lw, lb, ln


# ---------------------------------------------------------------------------
# oracle decoder / encoder drivers
# ---------------------------------------------------------------------------

class _DecModel(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("vocab", C.c_int), ("tok_emb", C.c_void_p),
                ("norm", C.c_void_p), ("ada_scale", C.c_void_p), ("lw", C.c_void_p),
                ("ln", C.c_void_p)]


class _DecKV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("max", C.c_int), ("len", C.c_int),
                ("pos_offset", C.c_int)]


class OracleDecoder:
    """vo_decoder_step / vo_decoder_prefill over a caller-owned linear cache
    with the reference's compaction semantics."""

    def __init__(self, w: DecoderWeights, kv_max):
        self.w = w
        self.lw, self.ln = w.pointer_arrays()
        self.m = _DecModel(w.n_layers, w.vocab, w.tok_emb.ctypes.data, w.norm.ctypes.data,
                           w.ada_scale.ctypes.data if w.ada_scale is not None else None,
                           C.cast(self.lw, C.c_void_p), C.cast(self.ln, C.c_void_p))
        self.k = np.zeros((w.n_layers, kv_max, KV_DIM), np.float32)
        self.v = np.zeros((w.n_layers, kv_max, KV_DIM), np.float32)
        self.kv = _DecKV(self.k.ctypes.data, self.v.ctypes.data, kv_max, 0, 0)

    def step(self, embed):
        logits = np.empty(self.w.vocab, np.float32)
        tok = oracle_lib().vo_decoder_step(C.byref(self.m), C.byref(self.kv),
                                           fptr(np.ascontiguousarray(embed, np.float32)), fptr(logits))
        assert tok >= 0, "oracle KV cache too small"
        return tok, logits

    def prefill(self, embeds):
        embeds = np.ascontiguousarray(embeds, np.float32)
        r = oracle_lib().vo_decoder_prefill(C.byref(self.m), C.byref(self.kv), fptr(embeds),
                                            embeds.shape[0])
        assert r == 0

    @property
    def state(self):
        return self.kv.len, self.kv.pos_offset


class _EncModel(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("lw", C.c_void_p), ("lb", C.c_void_p),
                ("ln", C.c_void_p), ("norm", C.c_void_p)]


class _EncKV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("max", C.c_int), ("len", C.c_int),
                ("pos_offset", C.c_int)]


class OracleEncoder:
    def __init__(self, w: EncoderWeights, kv_max=2400):
        self.w = w
        self.lw, self.lb, self.ln = w.pointer_arrays()
        self.m = _EncModel(w.n_layers, C.cast(self.lw, C.c_void_p), C.cast(self.lb, C.c_void_p),
                           C.cast(self.ln, C.c_void_p), w.norm.ctypes.data)
        self.k = np.zeros((w.n_layers, kv_max, ENC_QKV), np.float32)
        self.v = np.zeros((w.n_layers, kv_max, ENC_QKV), np.float32)
        self.kv = _EncKV(self.k.ctypes.data, self.v.ctypes.data, kv_max, 0, 0)

    def step(self, x):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        r = oracle_lib().vo_encoder_step(C.byref(self.m), C.byref(self.kv), fptr(x), x.shape[0])
        assert r == x.shape[0]
        return x

    def adapter(self, enc):
        enc = np.ascontiguousarray(enc, np.float32)
        out = np.empty((enc.shape[0] // 4, DEC_DIM), np.float32)
        oracle_lib().vo_adapter(u16ptr(self.w.adapter0), u16ptr(self.w.adapter1), fptr(enc),
                                enc.shape[0], fptr(out))
        return out


# ---------------------------------------------------------------------------
# the compiled reference (oracle/_ref/libvoxref.so)
# ---------------------------------------------------------------------------

class RefCtx:
    """A reference vox_ctx_t over caller-owned synthetic weights."""

    def __init__(self, dec: DecoderWeights | None = None, enc: EncoderWeights | None = None, lib=None):
        assert dec is None or (dec.n_layers == DEC_LAYERS and dec.vocab == VOCAB)
        assert enc is None or enc.n_layers == ENC_LAYERS
        lib = lib or ref_lib()
        self.lib = lib
        self.ctx = lib.voxref_ctx_new()
        self.dec, self.enc = dec, enc
        self._keep = []
        if dec is not None:
            lw, ln = dec.pointer_arrays()
            self._keep += [lw, ln]
            lib.voxref_set_decoder(self.ctx, u16ptr(dec.tok_emb), fptr(dec.norm), lw, ln,
                                   fptr(dec.ada_scale) if dec.ada_scale is not None else None)
        if enc is not None:
            lw, lb, ln = enc.pointer_arrays()
            self._keep += [lw, lb, ln]
            lib.voxref_set_encoder(self.ctx, lw, lb, ln, fptr(enc.norm))
            lib.voxref_set_adapter(self.ctx, u16ptr(enc.adapter0), u16ptr(enc.adapter1))

    def decoder_forward(self, embed):
        logits = np.empty(VOCAB, np.float32)
        tok = self.lib.voxref_decoder_forward(self.ctx, fptr(np.ascontiguousarray(embed, np.float32)),
                                              fptr(logits))
        return tok, logits

    def decoder_prefill(self, embeds):
        embeds = np.ascontiguousarray(embeds, np.float32)
        self.lib.voxref_decoder_prefill(self.ctx, fptr(embeds), embeds.shape[0])

    def encoder_incremental(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        n = self.lib.voxref_encoder_incremental(self.ctx, fptr(x), x.shape[0], fptr(out))
        assert n == x.shape[0]
        return out

    def adapter(self, enc):
        enc = np.ascontiguousarray(enc, np.float32)
        out = np.empty((enc.shape[0] // 4, DEC_DIM), np.float32)
        n = self.lib.voxref_adapter(self.ctx, fptr(enc), enc.shape[0], fptr(out))
        assert n == enc.shape[0] // 4
        return out

    def state(self):
        s = np.zeros(6, np.int32)
        self.lib.voxref_get_state(self.ctx, iptr(s))
        return s.tolist()

    def dec_kv(self):
        """(k, v) numpy views of the reference's decoder cache [26, max, 1024]."""
        _, mx, *_ = self.state()
        n = DEC_LAYERS * mx * KV_DIM
        k = np.ctypeslib.as_array(self.lib.voxref_dec_kv_k(self.ctx), shape=(n,))
        v = np.ctypeslib.as_array(self.lib.voxref_dec_kv_v(self.ctx), shape=(n,))
        return k.reshape(DEC_LAYERS, mx, KV_DIM), v.reshape(DEC_LAYERS, mx, KV_DIM)

    def enc_kv(self):
        st = self.state()
        mx = st[4]
        n = ENC_LAYERS * mx * ENC_QKV
        k = np.ctypeslib.as_array(self.lib.voxref_enc_kv_k(self.ctx), shape=(n,))
        v = np.ctypeslib.as_array(self.lib.voxref_enc_kv_v(self.ctx), shape=(n,))
        return k.reshape(ENC_LAYERS, mx, ENC_QKV), v.reshape(ENC_LAYERS, mx, ENC_QKV)

    def free(self):
        if self.ctx:
            self.lib.voxref_ctx_free(self.ctx, 0)
            self.ctx = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def ref_linear(x, W, b=None, path="linear"):
    """The reference's vox_linear_bf16 / vox_linear_nobias_bf16 /
    vox_matmul_t_bf16 on x [M, K], W [N, K]."""
    lib = ref_lib()
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0] if x.ndim == 2 else 1
    N, K = W.shape
    y = np.empty((M, N), np.float32)
    if path == "matmul_t":
        lib.vox_matmul_t_bf16(fptr(y), fptr(x), u16ptr(W), M, K, N)
    elif b is None:
        lib.vox_linear_nobias_bf16(fptr(y), fptr(x), u16ptr(W), M, K, N)
    else:
        lib.vox_linear_bf16(fptr(y), fptr(x), u16ptr(W), fptr(b), M, K, N)
    return y


def ref_rope_freqs(positions, head_dim):
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    f = np.empty((pos.size, head_dim), dtype=np.float32)
    ref_lib().vox_compute_rope_freqs(fptr(f), iptr(pos), pos.size, head_dim, np.float32(ROPE_THETA))
    return f


def ref_apply_rope(x, freqs, heads, head_dim):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    ref_lib().vox_apply_rope(fptr(x), fptr(freqs), freqs.shape[0], heads, head_dim)
    return x


def ref_attention(Q, K, V, seq_q, seq_k, n_heads, n_kv_heads, head_dim, window, q_offset):
    out = np.empty((seq_q, n_heads * head_dim), dtype=np.float32)
    ref_lib().vox_causal_attention(fptr(out), fptr(Q), fptr(K), fptr(V), seq_q, seq_k, n_heads,
                                   n_kv_heads, head_dim,
                                   np.float32(1.0) / np.sqrt(np.float32(head_dim)), window, q_offset)
    return out


def ref_fill_alts(logits, best, n_alt, cutoff):
    lg = np.array(logits, dtype=np.float32, copy=True)
    ids = np.full(4, -1, dtype=np.int32)
    n = ref_lib().voxref_fill_alts(fptr(lg), best, n_alt, cutoff, iptr(ids))
    return ids[:n].tolist()
