"""ctypes binding of libvoxtral_cuda.so (include/voxtral_cuda.h).

This is how Python callers (tests, bench.py) reach the C ABI; the C host of
voxtral.c links the same library directly.  Device buffers handed to the
`_dev` entry points are plain integers (device addresses); nothing here
depends on PyTorch.  The library must be built (``make -C voxtral.c_b200``):
loading fails loudly otherwise - there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvoxtral_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "voxtral_cuda.h")

DEC_DIM, Q_DIM, KV_DIM, DEC_HIDDEN = 3072, 4096, 1024, 9216
MAX_LAYERS = 26
PROF_PHASES = ("qkv", "attn", "wo", "w13", "w2", "lm_head")
ENC_PROF_PHASES = ("norm", "qkv", "attn", "wo", "w13", "w2")

OK, ERR_UNAVAILABLE, ERR_ARG, ERR_OOM, ERR_CUDA, ERR_CAPACITY = 0, -1, -2, -3, -4, -5

_fp = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)
_ip = C.POINTER(C.c_int)


class VoxCudaError(RuntimeError):
    pass


def header_symbols():
    """Every function name declared in include/voxtral_cuda.h."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vox_cuda_\w+)\s*\(", src)))


class _LayerW(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3",
                                          "attention_norm", "ffn_norm")]


class _DecW(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("vocab", C.c_int), ("weights_on_device", C.c_int),
                ("tok_embeddings", C.c_void_p), ("norm", C.c_void_p), ("ada_scale", C.c_void_p),
                ("layers", _LayerW * MAX_LAYERS)]


class _EncLayerW(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "wq_bias",
                                          "wv_bias", "wo_bias", "w2_bias", "attention_norm",
                                          "ffn_norm")]


class _EncW(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("weights_on_device", C.c_int), ("norm", C.c_void_p),
                ("adapter0", C.c_void_p), ("adapter1", C.c_void_p), ("layers", _EncLayerW * 32)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise VoxCudaError(f"{LIB_PATH} is not built (run __graft_entry__.build())")
    L = C.CDLL(LIB_PATH)
    sig = {
        "vox_cuda_init": ([], C.c_int),
        "vox_cuda_available": ([], C.c_int),
        "vox_cuda_shutdown": ([], None),
        "vox_cuda_set_device": ([C.c_int], C.c_int),
        "vox_cuda_last_error": ([], C.c_char_p),
        "vox_cuda_memory_used": ([], C.c_size_t),
        "vox_cuda_sgemm_bf16": ([C.c_int, C.c_int, C.c_int, _fp, _u16p, _fp, _fp], C.c_int),
        "vox_cuda_warmup_bf16": ([_u16p, C.c_int, C.c_int], C.c_int),
        "vox_cuda_weight_cache_clear": ([], None),
        "vox_cuda_linear_bf16_dev": ([C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_gemm_bf16_dev": ([C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_decoder_create": ([C.c_void_p], C.c_void_p),
        "vox_cuda_decoder_free": ([C.c_void_p], None),
        "vox_cuda_dec_state_create": ([C.c_void_p, C.c_int], C.c_void_p),
        "vox_cuda_dec_state_free": ([C.c_void_p], None),
        "vox_cuda_dec_state_reset": ([C.c_void_p], C.c_int),
        "vox_cuda_dec_state_position": ([C.c_void_p], C.c_int),
        "vox_cuda_dec_state_set_position": ([C.c_void_p, C.c_int], C.c_int),
        "vox_cuda_dec_state_load_kv": ([C.c_void_p, C.c_int, C.c_int, C.c_int, _fp, _fp], C.c_int),
        "vox_cuda_dec_state_read_kv": ([C.c_void_p, C.c_int, C.c_int, C.c_int, _fp, _fp], C.c_int),
        "vox_cuda_decoder_full_step": ([C.c_void_p, _fp, _fp, _fp], C.c_int),
        "vox_cuda_decoder_fill_alts": ([C.c_void_p, C.c_int, C.c_float, _ip], C.c_int),
        "vox_cuda_decoder_prefill_step": ([C.c_void_p, _fp, C.c_int, _fp], C.c_int),
        "vox_cuda_decoder_prefill_batch": ([C.c_void_p, C.c_int, _fp, _ip, _fp], C.c_int),
        "vox_cuda_decoder_step_batch": ([C.c_void_p, C.c_int, _fp, _ip], C.c_int),
        "vox_cuda_decoder_step_batch_ex": ([C.c_void_p, C.c_int, _fp, _fp, _ip, _fp], C.c_int),
        "vox_cuda_decoder_set_ada_scale": ([C.c_void_p, _fp], C.c_int),
        "vox_cuda_decoder_step_batch_tokens_dev": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.c_void_p], C.c_int),
        "vox_cuda_decoder_embed_dev": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p],
                                       C.c_int),
        "vox_cuda_adapter_forward_dev": ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_fp16_saturations": ([C.c_void_p, C.c_int], C.c_int),
        "vox_cuda_decoder_step_batch_dev": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                             C.c_void_p], C.c_int),
        "vox_cuda_decoder_profile_batch": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, _fp],
                                           C.c_int),
        "vox_cuda_decoder_profile_sequence": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                               _fp], C.c_int),
        "vox_cuda_encoder_step_batch_dev": ([C.c_void_p, C.c_int, C.c_void_p, _ip, C.c_void_p], C.c_int),
        "vox_cuda_encoder_create": ([C.c_void_p], C.c_void_p),
        "vox_cuda_encoder_free": ([C.c_void_p], None),
        "vox_cuda_enc_state_create": ([C.c_void_p, C.c_int], C.c_void_p),
        "vox_cuda_enc_state_free": ([C.c_void_p], None),
        "vox_cuda_enc_state_reset": ([C.c_void_p], C.c_int),
        "vox_cuda_enc_state_position": ([C.c_void_p], C.c_int),
        "vox_cuda_encoder_full_step": ([C.c_void_p, _fp, C.c_int, _fp], C.c_int),
        "vox_cuda_encoder_step_dev": ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p], C.c_int),
        "vox_cuda_enc_state_set_position": ([C.c_void_p, C.c_int], C.c_int),
        "vox_cuda_encoder_profile": ([C.c_void_p, C.c_void_p, C.c_int, C.c_int, _fp], C.c_int),
        "vox_cuda_adapter_forward": ([C.c_void_p, _fp, C.c_int, _fp], C.c_int),
        "vox_cuda_conv_stem_create": ([_fp, _fp, _fp, _fp, C.c_int], C.c_void_p),
        "vox_cuda_conv_stem_free": ([C.c_void_p], None),
        "vox_cuda_conv_stem_reset": ([C.c_void_p], C.c_int),
        "vox_cuda_conv_stem_step": ([C.c_void_p, _fp, C.c_int, _fp], C.c_int),
        "vox_cuda_conv_stem_step_dev": ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_selftest_wait_timeout": ([C.c_int], C.c_int),
        "vox_cuda_mel_create": ([C.c_int, C.c_int], C.c_void_p),
        "vox_cuda_mel_free": ([C.c_void_p], None),
        "vox_cuda_mel_frames": ([C.c_void_p], C.c_int),
        "vox_cuda_mel_frames_for": ([C.c_void_p, C.c_int], C.c_int),
        "vox_cuda_mel_feed": ([C.c_void_p, _fp, C.c_int, _fp, C.c_int], C.c_int),
        "vox_cuda_mel_feed_dev": ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p],
                                  C.c_int),
        "vox_cuda_mel_finish": ([C.c_void_p, C.c_int, _fp, C.c_int], C.c_int),
        "vox_cuda_mel_finish_dev": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p], C.c_int),
        "vox_cuda_mel_spectrogram": ([_fp, C.c_int, _fp, C.c_int], C.c_int),
        "vox_cuda_attention_decode_dev": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                           C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_attention_decode_noalloc": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                               C.c_int, C.c_void_p, C.c_void_p], C.c_int),
        "vox_cuda_rope_dev": ([C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p],
                              C.c_int),
        "vox_cuda_fill_normal_bf16_dev": ([C.c_void_p, C.c_size_t, C.c_uint64, C.c_float,
                                           C.c_void_p], C.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def last_error():
    return lib().vox_cuda_last_error().decode(errors="replace")


def check(rc, what=""):
    if rc < 0:
        raise VoxCudaError(f"{what}: rc={rc}: {last_error()}")
    return rc


def init(device=None):
    L = lib()
    if device is not None:
        check(L.vox_cuda_set_device(device), "set_device")
    if L.vox_cuda_init() != 1:
        raise VoxCudaError("vox_cuda_init failed: " + last_error())


def _f(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _u16(a):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def sgemm_bf16(x, W, bias=None):
    """C = x W^T (+ bias) through vox_cuda_sgemm_bf16 (host arrays)."""
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0] if x.ndim == 2 else 1
    N, K = W.shape
    y = np.empty((M, N), np.float32)
    check(lib().vox_cuda_sgemm_bf16(M, N, K, _f(x), _u16(W), _f(bias), _f(y)), "sgemm_bf16")
    return y


class Decoder:
    """Resident decoder weights.  `layers` is a list of n_layers tuples
    (wq, wk, wv, wo, w1, w2, w3, attention_norm, ffn_norm); arrays are host
    numpy arrays, or device addresses (ints) with on_device=True."""

    def __init__(self, tok_emb, norm, layers, ada_scale=None, vocab=131072, on_device=False):
        def addr(a):
            if a is None:
                return None
            return int(a) if on_device else a.ctypes.data
        d = _DecW()
        d.n_layers = len(layers)
        d.vocab = vocab
        d.weights_on_device = 1 if on_device else 0
        d.tok_embeddings = addr(tok_emb)
        d.norm = addr(norm)
        d.ada_scale = addr(ada_scale)
        for i, lw in enumerate(layers):
            for name, a in zip(("wq", "wk", "wv", "wo", "w1", "w2", "w3", "attention_norm",
                                "ffn_norm"), lw):
                setattr(d.layers[i], name, addr(a))
        self.vocab = vocab
        self.n_layers = len(layers)
        self.h = lib().vox_cuda_decoder_create(C.byref(d))
        if not self.h:
            raise VoxCudaError("decoder_create: " + last_error())

    def state(self, kv_cap=8192 + 1024):
        return DecState(self, kv_cap)

    def set_ada_scale(self, ada_scale):
        ada = None if ada_scale is None else np.ascontiguousarray(ada_scale, np.float32)
        check(lib().vox_cuda_decoder_set_ada_scale(self.h, _f(ada)), "set_ada_scale")

    def free(self):
        if self.h:
            lib().vox_cuda_decoder_free(self.h)
            self.h = None


class DecState:
    def __init__(self, dec: Decoder, kv_cap):
        self.dec = dec
        self.kv_cap = kv_cap
        self.h = lib().vox_cuda_dec_state_create(dec.h, kv_cap)
        if not self.h:
            raise VoxCudaError("dec_state_create: " + last_error())

    @property
    def position(self):
        return lib().vox_cuda_dec_state_position(self.h)

    def set_position(self, pos):
        check(lib().vox_cuda_dec_state_set_position(self.h, pos), "set_position")

    def reset(self):
        check(lib().vox_cuda_dec_state_reset(self.h), "reset")

    def step(self, embed, rope=None, want_logits=True):
        embed = np.ascontiguousarray(embed, np.float32).reshape(-1)
        logits = np.empty(self.dec.vocab, np.float32) if want_logits else None
        rope = None if rope is None else np.ascontiguousarray(rope, np.float32).reshape(-1)
        tok = check(lib().vox_cuda_decoder_full_step(self.h, _f(embed), _f(rope), _f(logits)),
                    "full_step")
        return tok, logits

    def prefill(self, x, rope=None):
        x = np.ascontiguousarray(x, np.float32)
        rope = None if rope is None else np.ascontiguousarray(rope, np.float32)
        check(lib().vox_cuda_decoder_prefill_step(self.h, _f(x), x.shape[0], _f(rope)), "prefill")

    def fill_alts(self, n_alt, cutoff):
        ids = np.full(4, -1, np.int32)
        n = check(lib().vox_cuda_decoder_fill_alts(self.h, n_alt, cutoff, ids.ctypes.data_as(_ip)),
                  "fill_alts")
        return ids[:n].tolist()

    def load_kv(self, layer, first_pos, k_rows, v_rows):
        k_rows = np.ascontiguousarray(k_rows, np.float32)
        v_rows = np.ascontiguousarray(v_rows, np.float32)
        check(lib().vox_cuda_dec_state_load_kv(self.h, layer, first_pos, k_rows.shape[0],
                                               _f(k_rows), _f(v_rows)), "load_kv")

    def read_kv(self, layer, first_pos, n_rows):
        k = np.empty((n_rows, KV_DIM), np.float32)
        v = np.empty((n_rows, KV_DIM), np.float32)
        check(lib().vox_cuda_dec_state_read_kv(self.h, layer, first_pos, n_rows, _f(k), _f(v)),
              "read_kv")
        return k, v

    def free(self):
        if self.h:
            lib().vox_cuda_dec_state_free(self.h)
            self.h = None


def step_batch(states, embeds):
    embeds = np.ascontiguousarray(embeds, np.float32)
    n = len(states)
    arr = (C.c_void_p * n)(*[s.h for s in states])
    toks = np.empty(n, np.int32)
    check(lib().vox_cuda_decoder_step_batch(arr, n, _f(embeds), toks.ctypes.data_as(_ip)),
          "step_batch")
    return toks.tolist()


def step_batch_ex(states, embeds, rope=None, want_logits=True):
    """Batched step returning (tokens, logits [n, vocab] or None); rope:
    [n, 128] tables (cos, sin pairs) or None to derive them."""
    embeds = np.ascontiguousarray(embeds, np.float32)
    n = len(states)
    toks = np.empty(n, np.int32)
    logits = np.empty((n, states[0].dec.vocab), np.float32) if want_logits else None
    rope = None if rope is None else np.ascontiguousarray(rope, np.float32).reshape(n, -1)
    check(lib().vox_cuda_decoder_step_batch_ex(states_array(states), n, _f(embeds), _f(rope),
                                               toks.ctypes.data_as(_ip), _f(logits)), "step_batch_ex")
    return toks.tolist(), logits


def states_array(states):
    return (C.c_void_p * len(states))(*[s.h for s in states])


def attention_decode_dev(q, k_ring, v_ring, kv_cap, pos, out, stream=None):
    """Stand-alone decode attention on device addresses."""
    check(lib().vox_cuda_attention_decode_dev(q, k_ring, v_ring, kv_cap, pos, out, stream),
          "attention_decode_dev")


def prefill_batch(states, rows, rope=None):
    """Prefill several states in shared launches: rows[i] is state i's
    [n_i, 3072] block (n_i may be 0)."""
    lens = np.array([np.asarray(r).shape[0] for r in rows], np.int32)
    x = np.ascontiguousarray(np.concatenate([np.asarray(r, np.float32).reshape(-1, 3072) for r in rows], axis=0))
    rp = None if rope is None else np.ascontiguousarray(rope, np.float32)
    check(lib().vox_cuda_decoder_prefill_batch(states_array(states), len(states), _f(x), lens.ctypes.data_as(_ip),
                                               _f(rp) if rp is not None else None), "prefill_batch")


def step_batch_dev(states, embeds_dev, tokens_dev, stream=None):
    """Batched step with device embeddings / tokens (device addresses)."""
    arr = states_array(states)
    check(lib().vox_cuda_decoder_step_batch_dev(arr, len(states), embeds_dev, tokens_dev, stream),
          "step_batch_dev")


def step_batch_tokens_dev(states, row_ptrs, prev_tokens_dev, tokens_dev, stream=None):
    """Token-embedding batched step: row_ptrs is a list of n device addresses
    (each stream's [3072] adapter row); prev_tokens_dev / tokens_dev int32
    device addresses."""
    rows = (C.c_void_p * len(states))(*row_ptrs)
    check(lib().vox_cuda_decoder_step_batch_tokens_dev(states_array(states), len(states), rows,
                                                       prev_tokens_dev, tokens_dev, stream),
          "step_batch_tokens_dev")


def fp16_saturations(reset=False):
    """fp16 values clamped (or NaN) by the encoder path on this device."""
    n = C.c_ulonglong(0)
    check(lib().vox_cuda_fp16_saturations(C.byref(n), 1 if reset else 0), "fp16_saturations")
    return n.value


def embed_dev(dec, n, rows_dev, tokens_dev, out_dev, stream=None):
    check(lib().vox_cuda_decoder_embed_dev(dec.h, n, rows_dev, tokens_dev, out_dev, stream), "embed_dev")


def profile_batch(states, embeds_dev, iters=3):
    """Mean ms per step of each phase (PROF_PHASES) of the batched step."""
    ms = np.zeros(len(PROF_PHASES), np.float32)
    check(lib().vox_cuda_decoder_profile_batch(states_array(states), len(states), embeds_dev, iters,
                                               _f(ms)), "profile_batch")
    return dict(zip(PROF_PHASES, ms.tolist()))


def profile_sequence(states, embeds_dev, phase, iters=5):
    """Steady-state ms per launch of one phase's kernel (PROF_PHASES name),
    its per-layer launches replayed back to back in a graph."""
    ms = np.zeros(1, np.float32)
    check(lib().vox_cuda_decoder_profile_sequence(states_array(states), len(states), embeds_dev,
                                                  PROF_PHASES.index(phase), iters, _f(ms)),
          "profile_sequence")
    return float(ms[0])


def encoder_step_batch_dev(states, x_devs, lens, stream=None):
    """One launch over several encoder states' chunks (device addresses x_devs,
    rows lens), in place."""
    n = len(states)
    xs = (C.c_void_p * n)(*x_devs)
    ln = np.ascontiguousarray(lens, np.int32)
    check(lib().vox_cuda_encoder_step_batch_dev(states_array(states), n, xs, ln.ctypes.data_as(_ip), stream),
          "encoder_step_batch_dev")


class Encoder:
    """Resident encoder + adapter weights.  `layers`: n tuples of
    (wq, wk, wv, wo, w1, w2, w3, wq_bias, wv_bias, wo_bias, w2_bias,
    attention_norm, ffn_norm); host numpy arrays, or device addresses with
    on_device=True."""

    def __init__(self, layers, norm, adapter0, adapter1, on_device=False):
        def addr(a):
            return int(a) if on_device else a.ctypes.data
        d = _EncW()
        d.n_layers = len(layers)
        d.weights_on_device = 1 if on_device else 0
        d.norm = addr(norm)
        d.adapter0 = addr(adapter0)
        d.adapter1 = addr(adapter1)
        names = ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "wq_bias", "wv_bias", "wo_bias", "w2_bias",
                 "attention_norm", "ffn_norm")
        for i, lw in enumerate(layers):
            for name, a in zip(names, lw):
                setattr(d.layers[i], name, addr(a))
        self.h = lib().vox_cuda_encoder_create(C.byref(d))
        if not self.h:
            raise VoxCudaError("encoder_create: " + last_error())

    def state(self, max_chunk=1500):
        return EncState(self, max_chunk)

    def free(self):
        if self.h:
            lib().vox_cuda_encoder_free(self.h)
            self.h = None


class EncState:
    def __init__(self, enc, max_chunk):
        self.enc = enc
        self.h = lib().vox_cuda_enc_state_create(enc.h, max_chunk)
        if not self.h:
            raise VoxCudaError("enc_state_create: " + last_error())

    @property
    def position(self):
        return lib().vox_cuda_enc_state_position(self.h)

    def step(self, x, rope=None):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        rope = None if rope is None else np.ascontiguousarray(rope, np.float32)
        check(lib().vox_cuda_encoder_full_step(self.h, _f(x), x.shape[0], _f(rope)), "encoder_full_step")
        return x

    def adapter(self, enc):
        enc = np.ascontiguousarray(enc, np.float32)
        out = np.empty((enc.shape[0] // 4, DEC_DIM), np.float32)
        check(lib().vox_cuda_adapter_forward(self.h, _f(enc), enc.shape[0], _f(out)), "adapter_forward")
        return out

    def reset(self):
        check(lib().vox_cuda_enc_state_reset(self.h), "enc_state_reset")

    def set_position(self, pos):
        check(lib().vox_cuda_enc_state_set_position(self.h, pos), "enc_state_set_position")

    def adapter_dev(self, enc_dev, n, out_dev, stream=None):
        check(lib().vox_cuda_adapter_forward_dev(self.h, enc_dev, n, out_dev, stream), "adapter_forward_dev")

    def step_dev(self, x_dev, n, stream=None):
        check(lib().vox_cuda_encoder_step_dev(self.h, x_dev, n, stream), "encoder_step_dev")

    def profile(self, x_dev, n, iters=3):
        ms = np.zeros(len(ENC_PROF_PHASES), np.float32)
        check(lib().vox_cuda_encoder_profile(self.h, x_dev, n, iters, _f(ms)), "encoder_profile")
        return dict(zip(ENC_PROF_PHASES, ms.tolist()))

    def free(self):
        if self.h:
            lib().vox_cuda_enc_state_free(self.h)
            self.h = None


class ConvStem:
    """The encoder's conv stem with its streaming state
    (vox_cuda_conv_stem_*): mel chunks [n, 128] -> post-conv rows [*, 1280]."""

    def __init__(self, w0, b0, w1, b1, max_mel=3000):
        self._keep = [np.ascontiguousarray(a, np.float32) for a in (w0, b0, w1, b1)]
        self.h = lib().vox_cuda_conv_stem_create(*[_f(a) for a in self._keep], max_mel)
        if not self.h:
            raise VoxCudaError("conv_stem_create: " + last_error())

    def step(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        out = np.empty((mel.shape[0] // 2 + 1, 1280), np.float32)
        n = check(lib().vox_cuda_conv_stem_step(self.h, _f(mel), mel.shape[0], _f(out)), "conv_stem_step")
        return out[:n]

    def step_dev(self, mel_dev, n_new, out_dev, stream=None):
        """Device addresses; returns the rows written to out_dev."""
        return check(lib().vox_cuda_conv_stem_step_dev(self.h, mel_dev, n_new, out_dev, stream),
                     "conv_stem_step_dev")

    def reset(self):
        check(lib().vox_cuda_conv_stem_reset(self.h), "conv_stem_reset")

    def free(self):
        if self.h:
            lib().vox_cuda_conv_stem_free(self.h)
            self.h = None


MEL_BINS = 128


class Mel:
    """Incremental log-mel context on the device (vox_cuda_mel_*): the
    reference's vox_mel_ctx_init / vox_mel_feed / vox_mel_finish."""

    def __init__(self, left_pad_samples=0, max_feed_samples=32000):
        self.h = lib().vox_cuda_mel_create(left_pad_samples, max_feed_samples)
        if not self.h:
            raise VoxCudaError("mel_create: " + last_error())

    @property
    def frames(self):
        return lib().vox_cuda_mel_frames(self.h)

    def frames_for(self, n_samples):
        return lib().vox_cuda_mel_frames_for(self.h, n_samples)

    def feed(self, samples):
        samples = np.ascontiguousarray(samples, np.float32)
        cap = max(self.frames_for(samples.size), 1)
        out = np.empty((cap, MEL_BINS), np.float32)
        n = check(lib().vox_cuda_mel_feed(self.h, _f(samples), samples.size, _f(out), cap), "mel_feed")
        return out[:n]

    def feed_dev(self, samples_dev, n_samples, mel_dev, max_frames, stream=None):
        return check(lib().vox_cuda_mel_feed_dev(self.h, samples_dev, n_samples, mel_dev, max_frames, stream),
                     "mel_feed_dev")

    def finish(self, right_pad_samples=0):
        cap = max(self.frames_for(right_pad_samples + 200), 1)
        out = np.empty((cap, MEL_BINS), np.float32)
        n = check(lib().vox_cuda_mel_finish(self.h, right_pad_samples, _f(out), cap), "mel_finish")
        return out[:n]

    def finish_dev(self, right_pad_samples, mel_dev, max_frames, stream=None):
        return check(lib().vox_cuda_mel_finish_dev(self.h, right_pad_samples, mel_dev, max_frames, stream),
                     "mel_finish_dev")

    def free(self):
        if self.h:
            lib().vox_cuda_mel_free(self.h)
            self.h = None


def mel_spectrogram(samples):
    """One-shot log-mel (vox_cuda_mel_spectrogram): [n // 160, 128]."""
    samples = np.ascontiguousarray(samples, np.float32)
    cap = max(samples.size // 160, 1)
    out = np.empty((cap, MEL_BINS), np.float32)
    n = check(lib().vox_cuda_mel_spectrogram(_f(samples), samples.size, _f(out), cap), "mel_spectrogram")
    return out[:n]
