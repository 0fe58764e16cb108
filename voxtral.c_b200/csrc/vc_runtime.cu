// vc_runtime.cu - the C ABI of voxtral_cuda.h, part 1: per-device contexts,
// lifecycle, error reporting, the pointer-keyed weight cache and matmul entry
// points, and the kernel-level entries (decode attention, RoPE, the wait
// self-test, synthetic fills).  The decoder, encoder and front-end entry
// points live in vc_rt_decoder.cu, vc_rt_encoder.cu and vc_rt_front.cu.
#include "vc_runtime.h"

#include <stdarg.h>

#include <array>

using namespace vc;
using namespace vc::rt;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

static thread_local char t_err[512] = "";

namespace vc {
void set_last_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}
}  // namespace vc

// ---------------------------------------------------------------------------
// per-device context
// ---------------------------------------------------------------------------

namespace {

DevCtx g_dev[kMaxDevices];
std::mutex g_init_mu;
thread_local int t_device = -1;

}  // namespace

namespace vc {
namespace rt {

int current_device() {
    if (t_device >= 0) return t_device;
    const char *e = getenv("VOX_CUDA_DEVICE");
    return e ? atoi(e) : 0;
}

DevCtx *ctx_for(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    DevCtx *c = &g_dev[dev];
    return c->ready ? c : nullptr;
}

DevCtx *cur_ctx() {
    DevCtx *c = ctx_for(current_device());
    if (!c) set_error("vox_cuda_init has not succeeded on device %d", current_device());
    return c;
}

cudaError_t dev_alloc(DevCtx *c, void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(c->mu);
        c->bytes += bytes;
    }
    return e;
}

void dev_free(DevCtx *c, void *p, size_t bytes) {
    if (!p) return;
    cudaFree(p);
    std::lock_guard<std::mutex> lk(c->mu);
    c->bytes -= bytes;
}

// Host RoPE table for one logical position, the same formula as
// vox_compute_rope_freqs (voxtral_kernels.c:488-500).  The frequencies of the
// decoder's head size are computed once (the same expression, so the same
// values): the synchronous steps build these tables on the host before every
// launch, and the powf calls were most of that time.
void host_rope_table(int pos, int head_dim, float *cs) {
    static const std::array<float, kHeadDim / 2> freq = [] {
        std::array<float, kHeadDim / 2> f{};
        for (int d = 0; d < kHeadDim / 2; d++) f[d] = 1.0f / powf(kRopeTheta, (float)(2 * d) / (float)kHeadDim);
        return f;
    }();
    const float p = (float)pos;
    for (int d = 0; d < head_dim / 2; d++) {
        const float f = head_dim == kHeadDim ? freq[d] : 1.0f / powf(kRopeTheta, (float)(2 * d) / (float)head_dim);
        const float a = p * f;
        cs[2 * d] = cosf(a);
        cs[2 * d + 1] = sinf(a);
    }
}

}  // namespace rt
}  // namespace vc

// ---------------------------------------------------------------------------
// lifecycle
// ---------------------------------------------------------------------------

extern "C" int vox_cuda_set_device(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n || device >= kMaxDevices) {
        set_error("vox_cuda_set_device: no device %d", device);
        return VOX_CUDA_ERR_ARG;
    }
    t_device = device;
    VC_TRY(cudaSetDevice(device));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_init(void) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("vox_cuda_init: bad device %d", dev);
        return 0;
    }
    std::lock_guard<std::mutex> lk(g_init_mu);
    DevCtx *c = &g_dev[dev];
    if (c->ready) {
        cudaSetDevice(dev);
        return 1;
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || dev >= n) {
        set_error("vox_cuda_init: no CUDA device %d", dev);
        return 0;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major != 10) {
        set_error("vox_cuda_init: device %d is not an sm_100 (Blackwell) GPU", dev);
        return 0;
    }
    if (cudaSetDevice(dev) != cudaSuccess) {
        set_error("vox_cuda_init: cudaSetDevice(%d) failed", dev);
        return 0;
    }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_error("vox_cuda_init: stream creation failed");
        return 0;
    }
    c->device = dev;
    c->ready = true;
    t_device = dev;
    return 1;
}

extern "C" int vox_cuda_available(void) {
    return ctx_for(current_device()) != nullptr ? 1 : 0;
}

extern "C" const char *vox_cuda_last_error(void) { return t_err; }

extern "C" size_t vox_cuda_memory_used(void) {
    DevCtx *c = ctx_for(current_device());
    if (!c) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    return c->bytes;
}

static void release_scratch(DevCtx *c) {
    cudaFree(c->sx);
    cudaFree(c->sy);
    cudaFree(c->sb);
    cudaFree(c->attn_slot);
    cudaFree(c->attn_part_o);
    cudaFree(c->attn_part_ml);
    cudaFree(c->attn_counters);
    cudaFree(c->rope_tab);
    cudaFree(c->lin_xfrag);
    cudaFree(c->lin_err);
    if (c->lin_done) cudaEventDestroy(c->lin_done);
    if (c->attn_done) cudaEventDestroy(c->attn_done);
    c->attn_done = nullptr;
    c->lin_xfrag = nullptr;
    c->lin_xfrag_bytes = 0;
    c->lin_err = nullptr;
    c->lin_done = nullptr;
    c->sx = c->sy = c->sb = nullptr;
    c->sx_n = c->sy_n = c->sb_n = 0;
    c->attn_slot = nullptr;
    c->attn_part_o = c->attn_part_ml = c->rope_tab = nullptr;
    c->attn_counters = nullptr;
}

extern "C" void vox_cuda_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    for (int d = 0; d < kMaxDevices; d++) {
        DevCtx *c = &g_dev[d];
        if (!c->ready) continue;
        cudaSetDevice(d);
        cudaStreamSynchronize(c->stream);
        for (auto &kv : c->wcache) cudaFree(kv.second.dev);
        c->wcache.clear();
        for (auto &kv : c->wcache_rm) cudaFree(kv.second.dev);
        c->wcache_rm.clear();
        cudaFree(c->sa16);
        c->sa16 = nullptr;
        c->sa16_n = 0;
        cudaFree(c->stage);
        c->stage = nullptr;
        c->stage_bytes = 0;
        if (c->up_ring) cudaFreeHost(c->up_ring);
        c->up_ring = nullptr;
        release_scratch(c);
        cudaStreamDestroy(c->stream);
        c->stream = nullptr;
        c->bytes = 0;
        c->ready = false;
    }
}

// ---------------------------------------------------------------------------
// (1) matmul entry points
// ---------------------------------------------------------------------------

static int check_linear_args(int M, int N, int K, const void *A, const void *B, const void *C) {
    if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) {
        set_error("linear: bad arguments (M=%d N=%d K=%d)", M, N, K);
        return VOX_CUDA_ERR_ARG;
    }
    return VOX_CUDA_OK;
}


// y[M,N] = x[M,K] W^T (+b), all device pointers, W fragment-tiled; rows of x
// in chunks of 8 (each chunk: activations -> B fragments, then the GEMV).
// Caller holds c->mu; the scratch is ordered across streams by c->lin_done.
static int enqueue_linear(DevCtx *c, int M, int N, int K, const float *x, const uint16_t *W,
                          const float *b, float *y, cudaStream_t st) {
    const size_t xb = xfrag_bytes(K);
    if (c->lin_xfrag_bytes < xb) {
        if (c->lin_xfrag) {
            cudaFree(c->lin_xfrag);
            c->bytes -= c->lin_xfrag_bytes;
        }
        c->lin_xfrag = nullptr;
        c->lin_xfrag_bytes = 0;
        if (cudaMalloc(&c->lin_xfrag, xb) != cudaSuccess) {
            set_error("linear: scratch cudaMalloc(%zu) failed", xb);
            return VOX_CUDA_ERR_OOM;
        }
        VC_TRY(cudaMemset(c->lin_xfrag, 0, xb));
        c->lin_xfrag_bytes = xb;
        c->bytes += xb;
    }
    if (!c->lin_err) {
        if (cudaMalloc(&c->lin_err, sizeof(unsigned)) != cudaSuccess) {
            set_error("linear: scratch cudaMalloc failed");
            return VOX_CUDA_ERR_OOM;
        }
        VC_TRY(cudaMemset(c->lin_err, 0, sizeof(unsigned)));
        VC_TRY(cudaEventCreateWithFlags(&c->lin_done, cudaEventDisableTiming));
        VC_TRY(cudaEventRecord(c->lin_done, st));
    }
    VC_TRY(cudaStreamWaitEvent(st, c->lin_done, 0));
    for (int m0 = 0; m0 < M; m0 += kMaxBatch) {
        const int mm = (M - m0 < kMaxBatch) ? (M - m0) : kMaxBatch;
        VC_TRY(launch_prep_xfrag(x + (size_t)m0 * K, mm, K, K, nullptr, c->lin_xfrag, nullptr, st, false));
        GemvParams p = {};
        p.W = W;
        p.N = N;
        p.K = K;
        p.Kp = round_up(K, 16);
        p.xfrag = c->lin_xfrag;
        p.y = y + (size_t)m0 * N;
        p.ldy = N;
        p.bias = b;
        p.err = c->lin_err;
        VC_TRY(launch_gemv(mm, EPI_STORE, p, st, false));
    }
    VC_TRY(cudaEventRecord(c->lin_done, st));
    return VOX_CUDA_OK;
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

static const uint16_t *cached_weight(DevCtx *c, const uint16_t *src, int N, int K, bool on_host,
                                     int *rc);

extern "C" int vox_cuda_linear_bf16_dev(int M, int N, int K, const float *A, const uint16_t *B_bf16,
                                        const float *bias, float *C, void *stream) {
    int rc = check_linear_args(M, N, K, A, B_bf16, C);
    if (rc) return rc;

    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const uint16_t *W = cached_weight(c, B_bf16, N, K, false, &rc);
    if (!W) return rc;
    std::lock_guard<std::mutex> lk(c->mu);
    return enqueue_linear(c, M, N, K, A, W, bias, C, st);
}

// The fragment-tiled device copy of a caller's [N, K] bf16 weight, made on
// first use and kept, keyed by the caller's pointer (host: the mmap'd tensor;
// device: the caller's buffer).  Like the Metal backend's pointer-keyed cache,
// it assumes the weight memory is not rewritten while cached;
// vox_cuda_weight_cache_clear() drops every copy.
static const uint16_t *cached_weight(DevCtx *c, const uint16_t *src, int N, int K, bool on_host,
                                     int *rc) {
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->wcache.find(src);
    if (it != c->wcache.end()) {
        if (it->second.N == N && it->second.K == K) return it->second.dev;
        cudaFree(it->second.dev);
        c->bytes -= it->second.bytes;
        c->wcache.erase(it);
    }
    const int Np = round_up(N, kGemvRowAlign), Kp = round_up(K, 16);
    const size_t bytes = (size_t)Np * Kp * 2;
    uint16_t *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) {
        set_error("weight cache: cudaMalloc(%zu) failed", bytes);
        *rc = VOX_CUDA_ERR_OOM;
        return nullptr;
    }
    const uint16_t *rowmajor = src;
    const size_t raw = (size_t)N * K * 2;
    if (on_host) {
        if (c->stage_bytes < raw) {
            cudaFree(c->stage);
            c->bytes -= c->stage_bytes;
            c->stage = nullptr;
            c->stage_bytes = 0;
            if (cudaMalloc(&c->stage, raw) != cudaSuccess) {
                cudaFree(d);
                set_error("weight cache: staging cudaMalloc(%zu) failed", raw);
                *rc = VOX_CUDA_ERR_OOM;
                return nullptr;
            }
            c->stage_bytes = raw;
            c->bytes += raw;
        }
        if (cudaMemcpyAsync(c->stage, src, raw, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            cudaFree(d);
            set_error("weight cache: upload failed");
            *rc = VOX_CUDA_ERR_CUDA;
            return nullptr;
        }
        rowmajor = c->stage;
    }
    if (launch_tile_weights(d, rowmajor, N, K, Np, Kp, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) {
        cudaFree(d);
        set_error("weight cache: tiling failed");
        *rc = VOX_CUDA_ERR_CUDA;
        return nullptr;
    }
    c->wcache[src] = DevCtx::CachedW{d, N, K, bytes};
    c->bytes += bytes;
    return d;
}

extern "C" void vox_cuda_weight_cache_clear(void) {
    DevCtx *c = ctx_for(current_device());
    if (!c) return;
    cudaStreamSynchronize(c->stream);
    std::lock_guard<std::mutex> lk(c->mu);
    for (auto &kv : c->wcache) {
        cudaFree(kv.second.dev);
        c->bytes -= kv.second.bytes;
    }
    c->wcache.clear();
    for (auto &kv : c->wcache_rm) {
        cudaFree(kv.second.dev);
        c->bytes -= kv.second.bytes;
    }
    c->wcache_rm.clear();
}

// Row-major device copy of a host [N, K] weight for the tensor-core GEMM
// (same keying and staleness rules as cached_weight).  Caller holds c->mu.
static const uint16_t *cached_weight_rm(DevCtx *c, const uint16_t *host, int N, int K, int *rc) {
    auto it = c->wcache_rm.find(host);
    if (it != c->wcache_rm.end()) {
        if (it->second.N == N && it->second.K == K) return it->second.dev;
        cudaFree(it->second.dev);
        c->bytes -= it->second.bytes;
        c->wcache_rm.erase(it);
    }
    const size_t bytes = (size_t)N * K * 2;
    uint16_t *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) {
        set_error("weight cache: cudaMalloc(%zu) failed", bytes);
        *rc = VOX_CUDA_ERR_OOM;
        return nullptr;
    }
    if (cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        set_error("weight cache: upload failed");
        *rc = VOX_CUDA_ERR_CUDA;
        return nullptr;
    }
    c->wcache_rm[host] = DevCtx::CachedW{d, N, K, bytes};
    c->bytes += bytes;
    return d;
}

extern "C" int vox_cuda_warmup_bf16(const uint16_t *B_bf16, int N, int K) {
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    if (!B_bf16 || N <= 0 || K <= 0) {
        set_error("warmup: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    int rc = VOX_CUDA_OK;
    return cached_weight(c, B_bf16, N, K, true, &rc) ? VOX_CUDA_OK : rc;
}

extern "C" int vox_cuda_sgemm_bf16(int M, int N, int K, const float *A, const uint16_t *B_bf16,
                                   const float *bias, float *C) {
    int rc = check_linear_args(M, N, K, A, B_bf16, C);
    if (rc) return rc;
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    const bool tensor_core = M > kMaxBatch && K % 8 == 0;
    const uint16_t *W = nullptr;
    if (!tensor_core) {
        W = cached_weight(c, B_bf16, N, K, true, &rc);
        if (!W) return rc;
    }
    std::lock_guard<std::mutex> lk(c->mu);  // one user of the host-path scratch at a time
    if (tensor_core) {
        W = cached_weight_rm(c, B_bf16, N, K, &rc);
        if (!W) return rc;
    }
    // (dev_alloc takes the same mutex: allocate through grow_locked below)
    auto grow_locked = [&](float **p, size_t *cap, size_t n) -> int {
        if (*cap >= n) return VOX_CUDA_OK;
        if (*p) {
            cudaFree(*p);
            c->bytes -= *cap * sizeof(float);
        }
        *p = nullptr;
        *cap = 0;
        if (cudaMalloc((void **)p, n * sizeof(float)) != cudaSuccess) {
            set_error("scratch: cudaMalloc(%zu) failed", n * 4);
            return VOX_CUDA_ERR_OOM;
        }
        c->bytes += n * sizeof(float);
        *cap = n;
        return VOX_CUDA_OK;
    };
    if ((rc = grow_locked(&c->sx, &c->sx_n, (size_t)M * K))) return rc;
    if ((rc = grow_locked(&c->sy, &c->sy_n, (size_t)M * N))) return rc;
    if (bias && (rc = grow_locked(&c->sb, &c->sb_n, (size_t)N))) return rc;
    VC_TRY(cudaMemcpyAsync(c->sx, A, (size_t)M * K * 4, cudaMemcpyHostToDevice, c->stream));
    if (bias) VC_TRY(cudaMemcpyAsync(c->sb, bias, (size_t)N * 4, cudaMemcpyHostToDevice, c->stream));
    if (tensor_core) {
        // activations rounded to bf16 for the tensor cores (contract: <= 5e-3
        // relative L2 per tensor-core GEMM); fp32 accumulation and output
        if (c->sa16_n < (size_t)M * K) {
            cudaFree(c->sa16);
            c->bytes -= c->sa16_n * 2;
            c->sa16 = nullptr;
            c->sa16_n = 0;
            if (cudaMalloc(&c->sa16, (size_t)M * K * 2) != cudaSuccess) {
                set_error("scratch: cudaMalloc(%zu) failed", (size_t)M * K * 2);
                return VOX_CUDA_ERR_OOM;
            }
            c->sa16_n = (size_t)M * K;
            c->bytes += c->sa16_n * 2;
        }
        if (!c->lin_err) {
            if (cudaMalloc(&c->lin_err, sizeof(unsigned)) != cudaSuccess) return VOX_CUDA_ERR_OOM;
            VC_TRY(cudaMemset(c->lin_err, 0, sizeof(unsigned)));
            VC_TRY(cudaEventCreateWithFlags(&c->lin_done, cudaEventDisableTiming));
            VC_TRY(cudaEventRecord(c->lin_done, c->stream));
        }
        VC_TRY(launch_rows_to_bf16(c->sx, M, K, K, nullptr, c->sa16, c->stream, false));
        TcGemmParams tp = {};
        tp.M = M;
        tp.N = N;
        tp.K = K;
        tp.out = c->sy;
        tp.ldo = N;
        tp.bias = bias ? c->sb : nullptr;
        tp.err = c->lin_err;
        VC_TRY(launch_tc_gemm(TC_STORE, tp, c->sa16, W, c->stream, false));
    } else {
        rc = enqueue_linear(c, M, N, K, c->sx, W, bias ? c->sb : nullptr, c->sy, c->stream);
        if (rc) return rc;
    }
    VC_TRY(cudaMemcpyAsync(C, c->sy, (size_t)M * N * 4, cudaMemcpyDeviceToHost, c->stream));
    unsigned err = 0;
    VC_TRY(cudaMemcpyAsync(&err, c->lin_err, sizeof(err), cudaMemcpyDeviceToHost, c->stream));
    VC_TRY(cudaStreamSynchronize(c->stream));
    if (err) {
        cudaMemset(c->lin_err, 0, sizeof(unsigned));
        set_error("sgemm_bf16: a device-side wait timed out");
        return VOX_CUDA_ERR_CUDA;
    }
    return VOX_CUDA_OK;
}

// ---------------------------------------------------------------------------
// kernel-level entries
// ---------------------------------------------------------------------------

static int ensure_attn_scratch(DevCtx *c) {
    if (c->attn_slot) return VOX_CUDA_OK;
    const size_t np = (size_t)kDecHeads * kAttnSplits;
    if (cudaMalloc(&c->attn_slot, sizeof(StreamSlot)) != cudaSuccess ||
        cudaMalloc(&c->attn_part_o, np * kHeadDim * 4) != cudaSuccess ||
        cudaMalloc(&c->attn_part_ml, np * 2 * 4) != cudaSuccess ||
        cudaMalloc(&c->attn_counters, kDecKvHeads * 4) != cudaSuccess ||
        cudaMalloc(&c->rope_tab, 512 * 4) != cudaSuccess) {
        set_error("attention scratch allocation failed");
        return VOX_CUDA_ERR_OOM;
    }
    c->bytes += sizeof(StreamSlot) + np * kHeadDim * 4 + np * 8 + kDecKvHeads * 4 + 2048;
    VC_TRY(cudaMemset(c->attn_counters, 0, kDecKvHeads * 4));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_attention_decode_dev(const float *q, const float *k_ring,
                                             const float *v_ring, int kv_cap, int pos, float *out,
                                             void *stream) {
    if (!q || !k_ring || !v_ring || !out || kv_cap <= 0 || pos < 0) {
        set_error("attention_decode: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (!aligned16(q) || !aligned16(k_ring) || !aligned16(v_ring) || !aligned16(out)) {
        set_error("attention_decode: q, k_ring, v_ring and out must be 16-byte aligned");
        return VOX_CUDA_ERR_ARG;
    }
    const int n_keys = (pos + 1 < kDecWindow) ? pos + 1 : kDecWindow;
    if (n_keys > kv_cap) {
        set_error("attention_decode: ring of %d positions cannot hold %d keys", kv_cap, n_keys);
        return VOX_CUDA_ERR_CAPACITY;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    std::lock_guard<std::mutex> lk(c->mu);
    int rc = ensure_attn_scratch(c);
    if (rc) return rc;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    StreamSlot h = {const_cast<float *>(k_ring), const_cast<float *>(v_ring), kv_cap, pos,
                    pos % kv_cap, n_keys, pos};
    // the scratch is shared: a call on another stream waits for the last one
    if (!c->attn_done) VC_TRY(cudaEventCreateWithFlags(&c->attn_done, cudaEventDisableTiming));
    else VC_TRY(cudaStreamWaitEvent(st, c->attn_done, 0));
    // the slot descriptor travels by value in the launch's parameters, so
    // back-to-back calls neither race on it nor wait on the host
    AttnParams p = {};
    p.q = q;
    p.slots = c->attn_slot;
    p.slot1 = h;
    p.slot_inline = 1;
    p.layer = 0;
    p.out = out;
    p.part_o = c->attn_part_o;
    p.part_ml = c->attn_part_ml;
    p.counters = c->attn_counters;
    p.S = kAttnSplits;
    p.deep_hint = n_keys;
    VC_TRY(launch_attn_decode(1, p, st, false));
    VC_TRY(cudaEventRecord(c->attn_done, st));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_rope_dev(float *x, int n_heads, int head_dim, int pos,
                                 const float *rope_freqs, void *stream) {
    if (!x || n_heads <= 0 || head_dim <= 0 || head_dim > 512 || (head_dim & 1) || pos < 0) {
        set_error("rope: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (rope_freqs) {
        VC_TRY(launch_rope(x, n_heads, head_dim, rope_freqs, st));
        return VOX_CUDA_OK;
    }
    std::lock_guard<std::mutex> lk(c->mu);
    int rc = ensure_attn_scratch(c);
    if (rc) return rc;
    float tab[512];
    host_rope_table(pos, head_dim, tab);
    VC_TRY(cudaMemcpyAsync(c->rope_tab, tab, head_dim * 4, cudaMemcpyHostToDevice, st));
    VC_TRY(launch_rope(x, n_heads, head_dim, c->rope_tab, st));
    VC_TRY(cudaStreamSynchronize(st));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_selftest_wait_timeout(int wait_ms) {
    if (wait_ms <= 0 || wait_ms > 10000) {
        set_error("selftest_wait_timeout: wait_ms must be 1..10000");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    unsigned *err = nullptr;
    unsigned h = 0;
    if (dev_alloc(c, (void **)&err, sizeof(unsigned)) != cudaSuccess) {
        set_error("selftest_wait_timeout: allocation failed");
        return VOX_CUDA_ERR_OOM;
    }
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(unsigned), c->stream);
    if (e == cudaSuccess) e = launch_stuck_wait(err, (unsigned long long)wait_ms * 1000000ull, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    dev_free(c, err, sizeof(unsigned));
    if (e != cudaSuccess) {
        set_error("selftest_wait_timeout: %s", cudaGetErrorString(e));
        return VOX_CUDA_ERR_CUDA;
    }
    if (h) {   // the expected outcome, reported as every kernel's timeout is
        set_error("selftest: a device-side wait timed out after %d ms (results discarded)", wait_ms);
        return VOX_CUDA_ERR_CUDA;
    }
    set_error("selftest_wait_timeout: the wait did not time out");
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_fill_normal_bf16_dev(uint16_t *dst, size_t n, uint64_t seed, float std,
                                             void *stream) {
    if (!dst) {
        set_error("fill_normal: NULL destination");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    VC_TRY(launch_fill_normal_bf16(dst, n, seed, std, st));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_gemm_bf16_dev(int M, int N, int K, const uint16_t *A_bf16, const uint16_t *W_bf16,
                                      const float *bias, float *C, void *stream) {
    if (M <= 0 || N <= 0 || K <= 0 || K % 8 != 0 || !A_bf16 || !W_bf16 || !C) {
        set_error("gemm_bf16_dev: bad arguments (M=%d N=%d K=%d; K must be a multiple of 8)", M, N, K);
        return VOX_CUDA_ERR_ARG;
    }
    if (!aligned16(A_bf16) || !aligned16(W_bf16)) {
        set_error("gemm_bf16_dev: A and W must be 16-byte aligned");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->lin_err) {
        if (cudaMalloc(&c->lin_err, sizeof(unsigned)) != cudaSuccess) return VOX_CUDA_ERR_OOM;
        VC_TRY(cudaMemset(c->lin_err, 0, sizeof(unsigned)));
        VC_TRY(cudaEventCreateWithFlags(&c->lin_done, cudaEventDisableTiming));
        VC_TRY(cudaEventRecord(c->lin_done, st));
    }
    TcGemmParams tp = {};
    tp.M = M;
    tp.N = N;
    tp.K = K;
    tp.out = C;
    tp.ldo = N;
    tp.bias = bias;
    tp.err = c->lin_err;
    VC_TRY(launch_tc_gemm(TC_STORE, tp, A_bf16, W_bf16, st, false));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_fp16_saturations(unsigned long long *count, int reset) {
    if (!count) {
        set_error("fp16_saturations: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    // the counters are written by kernels that may still be queued
    VC_TRY(cudaDeviceSynchronize());
    *count = f16_saturations_gemm(reset != 0);
    return VOX_CUDA_OK;
}
