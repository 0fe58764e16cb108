// vc_runtime.cu - the C ABI of voxtral_cuda.h: device contexts, the
// pointer-keyed weight cache, the resident decoder (fused weight layout), the
// per-stream KV ring, and the decode / prefill / batched steps (enqueued as
// one CUDA graph of programmatic-dependent launches per step shape).
#include "voxtral_cuda.h"

#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <unordered_map>
#include <thread>
#include <vector>

using namespace vc;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

static thread_local char t_err[512] = "";

static void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

namespace vc {
void set_last_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}
}  // namespace vc

#define VC_TRY(call)                                                                  \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                      \
            return VOX_CUDA_ERR_CUDA;                                                 \
        }                                                                             \
    } while (0)

#define VC_TRY_NULL(call)                                                             \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                      __LINE__);                                                      \
            return nullptr;                                                           \
        }                                                                             \
    } while (0)

// ---------------------------------------------------------------------------
// per-device context
// ---------------------------------------------------------------------------

namespace {

constexpr int kMaxDevices = 16;

struct DevCtx {
    int device = -1;
    bool ready = false;
    cudaStream_t stream = nullptr;
    std::mutex mu;                  // guards the cache and the scratch below
    size_t bytes = 0;               // device bytes held by the library
    struct CachedW {
        uint16_t *dev;      // fragment-tiled copy
        int N, K;
        size_t bytes;
    };
    std::unordered_map<const void *, CachedW> wcache;  // caller's weight ptr -> tiled copy
    std::unordered_map<const void *, CachedW> wcache_rm;  // ... -> row-major copy (tensor-core GEMM)
    uint16_t *sa16 = nullptr;                           // bf16 activations of the M > 8 path
    size_t sa16_n = 0;
    uint16_t *stage = nullptr;                          // row-major upload staging
    size_t stage_bytes = 0;
    // scratch for the host-pointer matmul entry and the kernel-level entries
    float *sx = nullptr, *sy = nullptr, *sb = nullptr;
    size_t sx_n = 0, sy_n = 0, sb_n = 0;
    uint32_t *lin_xfrag = nullptr;   // B-fragment scratch of the matmul entries
    size_t lin_xfrag_bytes = 0;
    unsigned *lin_err = nullptr;     // bounded-wait error word of the matmul entries
    cudaEvent_t lin_done = nullptr;  // orders scratch reuse across caller streams
    char *up_ring = nullptr;         // pinned weight-upload ring (Uploader), kept across creates
    std::mutex up_mu;                // one upload at a time uses it
    StreamSlot *attn_slot = nullptr;
    float *attn_part_o = nullptr, *attn_part_ml = nullptr, *rope_tab = nullptr;
    unsigned *attn_counters = nullptr;
    cudaEvent_t attn_done = nullptr;   // orders the attention scratch across caller streams
};

DevCtx g_dev[kMaxDevices];
std::mutex g_init_mu;
thread_local int t_device = -1;

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

// Host -> device weight upload through a ring of pinned chunks: host threads
// copy (or gather, for row-interleaved layouts) each chunk into a pinned slot
// while the copy engine drains the previous slots, so the upload runs at the
// pinned-DMA rate instead of the driver's pageable path (measured 33 vs
// 11 GB/s).  Registering the caller's pages instead was slower for a
// one-time upload (pinning costs about as much as the copy), and so is
// pinning the ring itself: it is allocated once per device and kept.
// Device sources are copied directly.
class Uploader {
  public:
    Uploader(cudaStream_t st, bool host, DevCtx *c) : st_(st), host_(host), c_(c) {}
    Uploader(const Uploader &) = delete;
    Uploader &operator=(const Uploader &) = delete;
    ~Uploader() {
        if (ring_) cudaStreamSynchronize(st_);   // the ring is free for the next upload
        for (auto &e : ev_)
            if (e) cudaEventDestroy(e);
    }
    cudaError_t copy(void *dst, const void *src, size_t bytes) { return copy2d(dst, bytes, src, bytes, bytes, 1); }
    // rows of `width` bytes, source rows spitch apart, destination rows dpitch apart
    cudaError_t copy2d(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows) {
        if (!host_)
            return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDeviceToDevice, st_);
        if (!ring_) {
            lock_ = std::unique_lock<std::mutex>(c_->up_mu);
            if (!c_->up_ring && cudaHostAlloc((void **)&c_->up_ring, kSlots * kChunk, cudaHostAllocDefault) !=
                                    cudaSuccess) {
                c_->up_ring = nullptr;
                host_ = false;   // no pinned ring: the driver's pageable path
                cudaGetLastError();
            }
            ring_ = c_->up_ring;
            for (auto &e : ev_)
                if (host_ && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
                    return cudaErrorMemoryAllocation;
        }
        if (!host_) return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyHostToDevice, st_);
        if (rows == 1 || (spitch == width && dpitch == width)) {   // contiguous: chunks of bytes
            const size_t total = width * rows;
            for (size_t off = 0; off < total; off += kChunk) {
                const size_t n = std::min(kChunk, total - off);
                char *slot = nullptr;
                cudaError_t e = take(&slot);
                if (e != cudaSuccess) return e;
                par_copy(slot, (const char *)src + off, n);
                e = cudaMemcpyAsync((char *)dst + off, slot, n, cudaMemcpyHostToDevice, st_);
                if (e != cudaSuccess || (e = cudaEventRecord(ev_[cur_], st_)) != cudaSuccess) return e;
            }
            return cudaSuccess;
        }
        const size_t per = std::max<size_t>(1, kChunk / width);   // rows per chunk
        for (size_t r0 = 0; r0 < rows; r0 += per) {
            const size_t nr = std::min(per, rows - r0);
            char *slot = nullptr;
            cudaError_t e = take(&slot);
            if (e != cudaSuccess) return e;
            par_gather(slot, (const char *)src + r0 * spitch, spitch, width, nr);
            e = cudaMemcpy2DAsync((char *)dst + r0 * dpitch, dpitch, slot, width, width, nr, cudaMemcpyHostToDevice,
                                  st_);
            if (e != cudaSuccess || (e = cudaEventRecord(ev_[cur_], st_)) != cudaSuccess) return e;
        }
        return cudaSuccess;
    }

  private:
    static constexpr size_t kChunk = (size_t)16 << 20;
    static constexpr int kSlots = 4;
    // the next slot, once the copy that last read it has finished
    cudaError_t take(char **slot) {
        cur_ = next_++ % kSlots;
        if (used_[cur_]) {
            cudaError_t e = cudaEventSynchronize(ev_[cur_]);
            if (e != cudaSuccess) return e;
        }
        used_[cur_] = true;
        *slot = ring_ + (size_t)cur_ * kChunk;
        return cudaSuccess;
    }
    static int n_threads() {
        const unsigned h = std::thread::hardware_concurrency();
        return (int)std::max(1u, std::min(8u, h ? h : 1u));
    }
    static void par_copy(char *dst, const char *src, size_t n) {
        const int T = n >= ((size_t)4 << 20) ? n_threads() : 1;
        if (T == 1) {
            memcpy(dst, src, n);
            return;
        }
        std::vector<std::thread> ts;
        const size_t per = (n + T - 1) / T;
        for (int t = 0; t < T; t++) {
            const size_t a = std::min(n, per * t), b = std::min(n, a + per);
            if (a < b) ts.emplace_back([=] { memcpy(dst + a, src + a, b - a); });
        }
        for (auto &t : ts) t.join();
    }
    static void par_gather(char *dst, const char *src, size_t spitch, size_t width, size_t rows) {
        const int T = rows * width >= ((size_t)4 << 20) ? n_threads() : 1;
        auto run = [=](size_t r0, size_t r1) {
            for (size_t r = r0; r < r1; r++) memcpy(dst + r * width, src + r * spitch, width);
        };
        if (T == 1) {
            run(0, rows);
            return;
        }
        std::vector<std::thread> ts;
        const size_t per = (rows + T - 1) / T;
        for (int t = 0; t < T; t++) {
            const size_t a = std::min(rows, per * t), b = std::min(rows, a + per);
            if (a < b) ts.emplace_back(run, a, b);
        }
        for (auto &t : ts) t.join();
    }
    cudaStream_t st_;
    bool host_;
    DevCtx *c_;
    std::unique_lock<std::mutex> lock_;   // held while this upload uses the ring
    char *ring_ = nullptr;
    cudaEvent_t ev_[kSlots] = {};
    bool used_[kSlots] = {};
    int next_ = 0, cur_ = 0;
};

// Host RoPE table for one logical position, the same formula as
// vox_compute_rope_freqs (voxtral_kernels.c:488-500).
void host_rope_table(int pos, int head_dim, float *cs) {
    const float p = (float)pos;
    for (int d = 0; d < head_dim / 2; d++) {
        const float f = 1.0f / powf(kRopeTheta, (float)(2 * d) / (float)head_dim);
        const float a = p * f;
        cs[2 * d] = cosf(a);
        cs[2 * d + 1] = sinf(a);
    }
}

}  // namespace

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

static int round_up(int v, int a) { return (v + a - 1) / a * a; }

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
    // the slot descriptor travels by value into a stream-ordered write, so
    // back-to-back calls neither race on it nor wait on the host
    VC_TRY(launch_set_slot(c->attn_slot, h, st));
    AttnParams p = {};
    p.q = q;
    p.slots = c->attn_slot;
    p.layer = 0;
    p.out = out;
    p.part_o = c->attn_part_o;
    p.part_ml = c->attn_part_ml;
    p.counters = c->attn_counters;
    p.S = kAttnSplits;
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

// ---------------------------------------------------------------------------
// decoder
// ---------------------------------------------------------------------------

namespace {

struct DecLayer {
    // fused, fragment-tiled device copies: wq|wk|wv [6144, 3072],
    // wo [3072, 4096], w1/w3 row-interleaved [18432, 3072], w2 [3072, 9216]
    const uint16_t *qkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr;
    // the same fused matrices row-major (bf16, as stored), the tcgen05
    // prefill's TMA-fed W operands; NULL when the tensor-core prefill is off
    const uint16_t *qkv_rm = nullptr, *wo_rm = nullptr, *w13_rm = nullptr, *w2_rm = nullptr;
    // RMSNorm weights as folded into the activation fragments:
    // g_attn = attention_norm, g_ffn = ffn_norm * (1 + ada_scale)
    const float *g_attn = nullptr, *g_ffn = nullptr;
};

// Device workspace for one step shape (n rows).  The host staging block is
// pinned; its layout mirrors the device block it is copied to.
struct StepWork {
    int n = 0;
    int vocab = 0;
    // device
    char *dblock = nullptr;            // [slots | rope | embeds] uploaded per step
    size_t dblock_bytes = 0;
    StreamSlot *slots = nullptr;
    float *rope = nullptr;             // [n][128]
    float *x = nullptr;                // [n][3072] residual stream
    float *q = nullptr, *att = nullptr;  // [n][4096]
    float *h = nullptr;                // [n][9216]
    float *logits = nullptr;           // [n][vocab]
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned *counters = nullptr;      // attention [n][8] + argmax [1]
    ArgmaxPartial *amax = nullptr;
    int *tokens = nullptr;             // [n]
    int *alt_ids = nullptr;            // [4]
    float *ss_attn = nullptr;          // [n][48] sums of x^2 per row block, after w2 (next QKV norm)
    float *ss_ffn = nullptr;           // [n][48] after wo (the FFN norm)
    uint32_t *xf_attn = nullptr;       // B fragments of x * g_attn (QKV / LM head input)
    uint32_t *xf_ffn = nullptr;        // B fragments of x * g_ffn (w1|w3 input)
    uint32_t *xf_att = nullptr;        // B fragments of the attention output (wo input)
    uint32_t *xf_h = nullptr;          // B fragments of silu(g) * u (w2 input)
    unsigned *err = nullptr;           // follows tokens: bounded-wait error word
    size_t bytes = 0;
    // host (pinned)
    char *hblock = nullptr;
    int *h_tokens = nullptr;
    // asynchronous steps (step_batch_dev): the host block's upload and the
    // error word's copy back, each behind an event
    cudaEvent_t staged = nullptr;
    cudaEvent_t err_ev = nullptr;
    bool staged_pending = false;
    bool err_pending = false;
    // graphs: [0] layers only (prefill), [1] layers + LM head
    cudaGraphExec_t graph[2] = {nullptr, nullptr};
};

// Device workspace of the tensor-core prefill (shared by the decoder's
// states, serialised by the decoder's mutex): up to `cap` rows per launch
// sequence.  Split activations (xn, att16, h16) are in the hilo_row layout:
// per 64 rows their bf16 hi rows, then their bf16 lo rows (2 x cap rows).
struct PrefillTc {
    int cap = 0;                 // rows
    int splits = 0;              // attention key splits the partial buffers hold
    char *block = nullptr;
    size_t bytes = 0;
    float *part = nullptr;       // attention partials (grown with `splits`)
    size_t part_bytes = 0;
    // the head, uploaded per call: slots, RoPE tables, input rows
    StreamSlot *slots = nullptr; // [cap]
    float *rope = nullptr;       // [cap][128]
    float *x = nullptr;          // [cap][3072] fp32 residual stream
    size_t head_bytes = 0;       // bytes before x
    float *q = nullptr;          // [cap][4096] fp32 (RoPE applied)
    uint16_t *xn = nullptr;      // [2 cap][3072] bf16 hi / lo
    uint16_t *att16 = nullptr;   // [2 cap][4096]
    uint16_t *h16 = nullptr;     // [2 cap][9216]
    unsigned *counters = nullptr;  // [cap][8]
    float *split = nullptr;      // split-K partials [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    unsigned *err = nullptr;
    char *hblock = nullptr;      // pinned mirror of the head
    unsigned *h_err = nullptr;   // pinned
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (rows, splits) -> layers
};

}  // namespace

struct vox_cuda_decoder {
    int device = 0;
    int n_layers = 0;
    int vocab = 0;
    DecLayer L[kDecLayersMax];
    const uint16_t *tok_emb = nullptr;
    const float *norm = nullptr;
    std::vector<std::pair<void *, size_t>> owned;
    StepWork *batch_work[kMaxBatch + 1] = {};
    std::mutex mu;   // serialises batched steps (they share batch_work)
    bool pdl = true;
    cudaEvent_t tail = nullptr;   // the end of the last asynchronous step
    bool tail_set = false;
    bool tc_prefill = false;      // row-major weights kept: prefill on the tensor cores
    PrefillTc *pf = nullptr;
};

struct vox_cuda_dec_state {
    vox_cuda_decoder *dec = nullptr;
    int cap = 0;
    int pos = 0;                       // logical position of the next row
    float *k_ring = nullptr, *v_ring = nullptr;
    size_t ring_bytes = 0;
    StepWork *work = nullptr;          // single-stream workspace (n = 1)
    StepWork *prefill_work = nullptr;  // n = 8 workspace for prefill chunks
    int last_token = -1;
    bool have_logits = false;
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

void free_work(DevCtx *c, StepWork *w) {
    if (!w) return;
    for (auto &g : w->graph)
        if (g) cudaGraphExecDestroy(g);
    if (w->staged) cudaEventDestroy(w->staged);
    if (w->err_ev) cudaEventDestroy(w->err_ev);
    if (w->dblock) cudaFree(w->dblock);
    if (w->hblock) cudaFreeHost(w->hblock);
    if (c) {
        std::lock_guard<std::mutex> lk(c->mu);
        c->bytes -= w->bytes;
    }
    delete w;
}

StepWork *make_work(DevCtx *c, int n, int vocab) {
    StepWork *w = new StepWork();
    w->n = n;
    w->vocab = vocab;
    const size_t S = kAttnSplits;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_slots = take(sizeof(StreamSlot) * n);
    const size_t o_rope = take(sizeof(float) * n * kHeadDim);
    const size_t o_x = take(sizeof(float) * n * kDecDim);
    w->dblock_bytes = o_x + sizeof(float) * n * kDecDim;   // the uploaded prefix
    const size_t o_q = take(sizeof(float) * n * kQDim);
    const size_t o_att = take(sizeof(float) * n * kQDim);
    const size_t o_h = take(sizeof(float) * n * kDecHidden);
    const size_t o_logits = take(sizeof(float) * n * (size_t)vocab);
    const size_t o_po = take(sizeof(float) * n * kDecHeads * S * kHeadDim);
    const size_t o_pml = take(sizeof(float) * n * kDecHeads * S * 2);
    const size_t o_cnt = take(sizeof(unsigned) * (n * kDecKvHeads + 1));
    const size_t grid = (size_t)gemv_grid(n, EPI_LOGITS, vocab);
    const size_t o_amax = take(sizeof(ArgmaxPartial) * grid * n);
    const size_t o_tok = take(sizeof(int) * (n + 1));   // tokens then the error word
    const size_t o_alt = take(sizeof(int) * 4);
    const size_t n_ss = (size_t)n * gemv_row_blocks(kDecDim);
    const size_t o_ssa = take(sizeof(float) * n_ss);
    const size_t o_ssf = take(sizeof(float) * n_ss);
    const size_t o_frag0 = off;
    const size_t o_xfa = take(xfrag_bytes(kDecDim));
    const size_t o_xff = take(xfrag_bytes(kDecDim));
    const size_t o_xft = take(xfrag_bytes(kQDim));
    const size_t o_xfh = take(xfrag_bytes(kDecHidden));
    const size_t frag_bytes = off - o_frag0;
    if (dev_alloc(c, (void **)&w->dblock, off) != cudaSuccess) {
        set_error("decoder workspace: cudaMalloc(%zu) failed", off);
        delete w;
        return nullptr;
    }
    w->bytes = off;
    char *b = w->dblock;
    w->slots = (StreamSlot *)(b + o_slots);
    w->rope = (float *)(b + o_rope);
    w->x = (float *)(b + o_x);
    w->q = (float *)(b + o_q);
    w->att = (float *)(b + o_att);
    w->h = (float *)(b + o_h);
    w->logits = (float *)(b + o_logits);
    w->part_o = (float *)(b + o_po);
    w->part_ml = (float *)(b + o_pml);
    w->counters = (unsigned *)(b + o_cnt);
    w->amax = (ArgmaxPartial *)(b + o_amax);
    w->tokens = (int *)(b + o_tok);
    w->alt_ids = (int *)(b + o_alt);
    w->ss_attn = (float *)(b + o_ssa);
    w->ss_ffn = (float *)(b + o_ssf);
    w->xf_attn = (uint32_t *)(b + o_xfa);
    w->xf_ffn = (uint32_t *)(b + o_xff);
    w->xf_att = (uint32_t *)(b + o_xft);
    w->xf_h = (uint32_t *)(b + o_xfh);
    w->err = (unsigned *)(w->tokens + n);
    // fragments of streams >= n are never written and must read as zeros
    if (cudaMemset(b + o_frag0, 0, frag_bytes) != cudaSuccess ||
        cudaMemset(w->tokens, 0, sizeof(int) * (n + 1)) != cudaSuccess ||
        cudaMemset(w->counters, 0, sizeof(unsigned) * (n * kDecKvHeads + 1)) != cudaSuccess ||
        cudaHostAlloc((void **)&w->hblock, align_up(w->dblock_bytes, 16) + sizeof(int) * (n + 1), cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->staged, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->err_ev, cudaEventDisableTiming) != cudaSuccess) {
        set_error("decoder workspace: staging allocation failed");
        free_work(c, w);
        return nullptr;
    }
    w->h_tokens = (int *)(w->hblock + align_up(w->dblock_bytes, 16));
    w->h_tokens[n] = 0;
    return w;
}

// host-side views of the staging block
StreamSlot *h_slots(StepWork *w) { return (StreamSlot *)w->hblock; }
float *h_rope(StepWork *w) { return (float *)(w->hblock + ((char *)w->rope - w->dblock)); }
float *h_x(StepWork *w) { return (float *)(w->hblock + ((char *)w->x - w->dblock)); }

// The kernel sequence of one step over w->n rows: the embeddings' norm
// statistics and fragments, the decoder layers, then the LM head + argmax
// when with_head.  Each producer writes its consumer's activation fragments.
// evs (profiling only): 2 events per launch, recorded around it.
// only (profiling only): >= 0 enqueues that phase's launches alone
// (VOX_CUDA_PROF_*), one per layer, back to back.
int enqueue_layers(vox_cuda_decoder *d, StepWork *w, bool with_head, cudaStream_t st,
                   cudaEvent_t *evs = nullptr, int only = -1) {
    const int n = w->n;
    const bool pdl = d->pdl && evs == nullptr;
    const int ss_parts = gemv_row_blocks(kDecDim);
    int ei = 0;
#define VC_EV_BEGIN() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
#define VC_EV_END() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
#define VC_PHASE(ph) if (only < 0 || only == (ph))
    if (only < 0) {
        VC_EV_BEGIN();
        VC_TRY(launch_prep_xfrag(w->x, n, kDecDim, kDecDim, d->L[0].g_attn, w->xf_attn, w->ss_attn, st, pdl));
        VC_EV_END();
    }
    for (int l = 0; l < d->n_layers && only != VOX_CUDA_PROF_LM_HEAD; l++) {
        const DecLayer &L = d->L[l];
        GemvParams p = {};
        // q|k|v = rms_norm(x) Wqkv^T, RoPE, ring write
        p.W = L.qkv;
        p.N = kQkvRows;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_attn;
        p.ss_in = w->ss_attn;
        p.ss_parts = ss_parts;
        p.y = w->q;
        p.ldy = kQDim;
        p.slots = w->slots;
        p.rope = w->rope;
        p.layer = l;
        p.err = w->err;
        VC_PHASE(VOX_CUDA_PROF_QKV) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_QKV, p, st, pdl));
            VC_EV_END();
        }
        // attention over the ring -> wo's fragments
        AttnParams a = {};
        a.q = w->q;
        a.slots = w->slots;
        a.layer = l;
        a.out = nullptr;
        a.xfrag_out = w->xf_att;
        a.part_o = w->part_o;
        a.part_ml = w->part_ml;
        a.counters = w->counters;
        a.S = kAttnSplits;
        VC_PHASE(VOX_CUDA_PROF_ATTN) {
            VC_EV_BEGIN();
            VC_TRY(launch_attn_decode(n, a, st, pdl));
            VC_EV_END();
        }
        // x += att Wo^T; fragments of x * g_ffn and sums of x^2 for the FFN norm
        p = GemvParams{};
        p.W = L.wo;
        p.N = kDecDim;
        p.K = p.Kp = kQDim;
        p.xfrag = w->xf_att;
        p.y = w->x;
        p.ldy = kDecDim;
        p.ss_out = w->ss_ffn;
        p.xfrag_out = w->xf_ffn;
        p.g_next = L.g_ffn;
        p.err = w->err;
        VC_PHASE(VOX_CUDA_PROF_WO) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_ADD, p, st, pdl));
            VC_EV_END();
        }
        // h = silu(xn W1^T) * (xn W3^T), xn = rms_norm(x) * (1 + ada)
        p = GemvParams{};
        p.W = L.w13;
        p.N = 2 * kDecHidden;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_ffn;
        p.ss_in = w->ss_ffn;
        p.ss_parts = ss_parts;
        p.xfrag_out = w->xf_h;
        p.err = w->err;
        VC_PHASE(VOX_CUDA_PROF_W13) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_SWIGLU, p, st, pdl));
            VC_EV_END();
        }
        // x += h W2^T; fragments for the next norm (next layer's, or the final)
        p = GemvParams{};
        p.W = L.w2;
        p.N = kDecDim;
        p.K = p.Kp = kDecHidden;
        p.xfrag = w->xf_h;
        p.y = w->x;
        p.ldy = kDecDim;
        p.ss_out = w->ss_attn;
        p.xfrag_out = w->xf_attn;
        p.g_next = (l + 1 < d->n_layers) ? d->L[l + 1].g_attn : d->norm;
        p.err = w->err;
        VC_PHASE(VOX_CUDA_PROF_W2) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_ADD, p, st, pdl));
            VC_EV_END();
        }
    }
    if (with_head && (only < 0 || only == VOX_CUDA_PROF_LM_HEAD)) {
        GemvParams p = {};
        p.W = d->tok_emb;
        p.N = d->vocab;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_attn;
        p.ss_in = w->ss_attn;
        p.ss_parts = ss_parts;
        p.y = w->logits;
        p.ldy = d->vocab;
        p.partials = w->amax;
        p.counter = w->counters + n * kDecKvHeads;
        p.tokens = w->tokens;
        p.err = w->err;
        VC_EV_BEGIN();
        VC_TRY(launch_gemv(n, EPI_LOGITS, p, st, pdl));
        VC_EV_END();
    }
#undef VC_EV_BEGIN
#undef VC_EV_END
#undef VC_PHASE
    return VOX_CUDA_OK;
}

// The error word copied back after the tokens: a device-side bounded wait
// expired during the step.
int check_step_error(StepWork *w, cudaStream_t st) {
    if (w->h_tokens[w->n] == 0) return VOX_CUDA_OK;
    w->h_tokens[w->n] = 0;
    cudaMemsetAsync(w->err, 0, sizeof(unsigned), st);
    set_error("decoder step: a device-side wait timed out (results discarded)");
    return VOX_CUDA_ERR_CUDA;
}

// Upload the staged step inputs, run the (captured) kernel sequence, fetch
// the tokens.
int run_step(vox_cuda_decoder *d, DevCtx *c, StepWork *w, bool with_head, cudaStream_t st,
             bool sync) {
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, w->dblock_bytes, cudaMemcpyHostToDevice, st));
    cudaGraphExec_t &g = w->graph[with_head ? 1 : 0];
    if (!g) {
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_layers(d, w, with_head, st);
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        VC_TRY(e);
        e = cudaGraphInstantiate(&g, graph, 0);
        cudaGraphDestroy(graph);
        VC_TRY(e);
    }
    VC_TRY(cudaGraphLaunch(g, st));
    // tokens and the error word in one copy
    VC_TRY(cudaMemcpyAsync(w->h_tokens, w->tokens, sizeof(int) * (w->n + 1), cudaMemcpyDeviceToHost, st));
    if (sync) {
        VC_TRY(cudaStreamSynchronize(st));
        int rc = check_step_error(w, st);
        if (rc) return rc;
    }
    (void)c;
    return VOX_CUDA_OK;
}

void fill_slot(vox_cuda_dec_state *s, int pos, StreamSlot *slot) {
    slot->k_ring = s->k_ring;
    slot->v_ring = s->v_ring;
    slot->cap = s->cap;
    slot->pos = pos;
    slot->slot = pos % s->cap;
    slot->n_keys = (pos + 1 < kDecWindow) ? pos + 1 : kDecWindow;
    slot->fresh = pos;   // a launch with more rows of this sequence lowers it
}

// Rows first..last are written in one launch: the ring must hold, at once,
// the window of the first row and every later row of the launch.
int check_capacity(const vox_cuda_dec_state *s, int first, int last) {
    const int oldest = (first - kDecWindow + 1 > 0) ? first - kDecWindow + 1 : 0;
    const int span = last - oldest + 1;
    if (span > s->cap) {
        set_error("KV ring of %d positions cannot hold %d positions (%d..%d)", s->cap, span,
                  oldest, last);
        return VOX_CUDA_ERR_CAPACITY;
    }
    return VOX_CUDA_OK;
}

// ---- tensor-core prefill -------------------------------------------------

constexpr int kPrefillRows = 128;   // rows per launch sequence (one M tile)

void free_prefill(DevCtx *c, PrefillTc *f) {
    if (!f) return;
    for (auto &kv : f->graphs) cudaGraphExecDestroy(kv.second);
    if (c) {
        dev_free(c, f->block, f->block ? f->bytes : 0);
        dev_free(c, f->part, f->part ? f->part_bytes : 0);
    }
    if (f->hblock) cudaFreeHost(f->hblock);
    if (f->h_err) cudaFreeHost(f->h_err);
    delete f;
}

PrefillTc *make_prefill(DevCtx *c, int cap) {
    PrefillTc *f = new PrefillTc();
    f->cap = cap;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t C = (size_t)cap;
    const size_t o_slots = take(sizeof(StreamSlot) * C), o_rope = take(4 * C * kHeadDim);
    const size_t o_x = take(4 * C * kDecDim);
    f->head_bytes = o_x;   // + the rows of x actually used
    const size_t o_q = take(4 * C * kQDim);
    const size_t o_xn = take(2 * 2 * C * kDecDim), o_att16 = take(2 * 2 * C * kQDim);
    const size_t o_h16 = take(2 * 2 * C * kDecHidden), o_cnt = take(4 * C * kDecKvHeads);
    const size_t o_split = take(4 * kEncSplitFloats), o_scnt = take(4 * kTcSplitCounters), o_err = take(4);
    f->bytes = off;
    if (dev_alloc(c, (void **)&f->block, f->bytes) != cudaSuccess ||
        cudaMemset(f->block, 0, f->bytes) != cudaSuccess ||
        cudaHostAlloc((void **)&f->hblock, o_x + 4 * C * kDecDim, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&f->h_err, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess) {
        set_error("prefill workspace: allocation of %zu bytes failed", f->bytes);
        free_prefill(c, f);
        return nullptr;
    }
    char *b = f->block;
    f->slots = (StreamSlot *)(b + o_slots);
    f->rope = (float *)(b + o_rope);
    f->x = (float *)(b + o_x);
    f->q = (float *)(b + o_q);
    f->xn = (uint16_t *)(b + o_xn);
    f->att16 = (uint16_t *)(b + o_att16);
    f->h16 = (uint16_t *)(b + o_h16);
    f->counters = (unsigned *)(b + o_cnt);
    f->split = (float *)(b + o_split);
    f->split_cnt = (unsigned *)(b + o_scnt);
    f->err = (unsigned *)(b + o_err);
    *f->h_err = 0;
    return f;
}

// Grow the attention partials to `splits` key splits per (row, head).
int prefill_reserve_splits(DevCtx *c, PrefillTc *f, int splits) {
    if (splits <= f->splits) return VOX_CUDA_OK;
    const size_t bytes = (size_t)f->cap * kDecHeads * splits * (kHeadDim + 2) * 4;
    float *np = nullptr;
    if (dev_alloc(c, (void **)&np, bytes) != cudaSuccess) {
        set_error("prefill workspace: attention partials (%zu bytes) failed", bytes);
        return VOX_CUDA_ERR_OOM;
    }
    VC_TRY(cudaStreamSynchronize(c->stream));
    dev_free(c, f->part, f->part ? f->part_bytes : 0);
    for (auto &kv : f->graphs) cudaGraphExecDestroy(kv.second);   // they hold the old pointers
    f->graphs.clear();
    f->part = np;
    f->part_bytes = bytes;
    f->splits = splits;
    return VOX_CUDA_OK;
}

// The layers of one prefill launch sequence over M rows (their slots, RoPE
// tables and inputs already in f): per layer RMSNorm -> hi / lo rows,
// q|k|v GEMM (RoPE, ring writes), attention over each row's ring, wo GEMM +
// residual, FFN RMSNorm * (1 + ada), w1|w3 GEMM + SwiGLU, w2 GEMM + residual
// (vox_decoder_prefill, voxtral_decoder.c:233-373).  bf16 tensor-core
// operands: the weights as stored, the activations as hi + lo pairs.
int enqueue_prefill(vox_cuda_decoder *d, PrefillTc *f, int M, int S, cudaStream_t st) {
    const bool pdl = d->pdl;
    float *part_o = f->part;
    float *part_ml = f->part + (size_t)f->cap * kDecHeads * S * kHeadDim;
    auto gemm = [&](int M_, int N, int K) {
        TcGemmParams p = {};
        p.M = M_;
        p.N = N;
        p.K = K;
        p.hilo = 1;
        p.err = f->err;
        p.ws = f->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = f->split_cnt;
        return p;
    };
    for (int l = 0; l < d->n_layers; l++) {
        const DecLayer &L = d->L[l];
        VC_TRY(launch_rows_hilo(f->x, M, kDecDim, kDecDim, L.g_attn, f->xn, st, pdl));
        TcGemmParams p = gemm(M, kQkvRows, kDecDim);
        p.q32 = f->q;
        p.slots = f->slots;
        p.layer = l;
        p.rope_rows = f->rope;
        VC_TRY(launch_tc_gemm(TC_QKV_DEC, p, f->xn, L.qkv_rm, st, pdl));
        AttnParams a = {};
        a.q = f->q;
        a.slots = f->slots;
        a.layer = l;
        a.out_hilo = f->att16;   // straight into the wo GEMM's split operand
        a.part_o = part_o;
        a.part_ml = part_ml;
        a.counters = f->counters;
        a.S = S;
        VC_TRY(launch_attn_decode(M, a, st, pdl));
        p = gemm(M, kDecDim, kQDim);
        p.out = f->x;
        p.ldo = kDecDim;
        VC_TRY(launch_tc_gemm(TC_RESID, p, f->att16, L.wo_rm, st, pdl));
        VC_TRY(launch_rows_hilo(f->x, M, kDecDim, kDecDim, L.g_ffn, f->xn, st, pdl));
        p = gemm(M, 2 * kDecHidden, kDecDim);
        p.out_bf16 = f->h16;
        p.ldo_bf16 = kDecHidden;
        p.out_hilo = 1;
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, f->xn, L.w13_rm, st, pdl));
        p = gemm(M, kDecDim, kDecHidden);
        p.out = f->x;
        p.ldo = kDecDim;
        VC_TRY(launch_tc_gemm(TC_RESID, p, f->h16, L.w2_rm, st, pdl));
    }
    return VOX_CUDA_OK;
}

// Rows of one or more states (state i contributes n_rows[i] consecutive
// rows from its current position), in launch sequences of <= kPrefillRows
// rows; x: host [sum n_rows][3072]; rope: host [sum n_rows][64][2] or NULL.
// Caller holds d->mu.
int prefill_tc_rows(vox_cuda_decoder *d, DevCtx *c, vox_cuda_dec_state *const *states, const int *n_rows,
                    int n_states, const float *x, const float *rope) {
    if (!d->pf && !(d->pf = make_prefill(c, kPrefillRows))) return VOX_CUDA_ERR_OOM;
    PrefillTc *f = d->pf;
    cudaStream_t st = c->stream;
    StreamSlot *h_slots = (StreamSlot *)f->hblock;
    float *h_rope = (float *)(f->hblock + ((char *)f->rope - f->block));
    float *h_x = (float *)(f->hblock + ((char *)f->x - f->block));
    int si = 0, done_in_state = 0;   // next row: state si, its row done_in_state
    size_t row_in = 0;               // next row of x / rope
    while (si < n_states) {
        // gather up to kPrefillRows rows
        int M = 0, max_keys = 1;
        while (si < n_states && M < f->cap) {
            const int take = std::min(n_rows[si] - done_in_state, f->cap - M);
            vox_cuda_dec_state *s = states[si];
            for (int r = 0; r < take; r++) {
                const int pos = s->pos + done_in_state + r;
                fill_slot(s, pos, h_slots + M + r);
                h_slots[M + r].fresh = s->pos + done_in_state;   // this launch's first row of the state
                max_keys = std::max(max_keys, h_slots[M + r].n_keys);
                if (rope) memcpy(h_rope + (size_t)(M + r) * kHeadDim, rope + (row_in + r) * kHeadDim, kHeadDim * 4);
                else host_rope_table(pos, kHeadDim, h_rope + (size_t)(M + r) * kHeadDim);
            }
            memcpy(h_x + (size_t)M * kDecDim, x + row_in * kDecDim, (size_t)take * kDecDim * 4);
            M += take;
            row_in += take;
            done_in_state += take;
            if (done_in_state == n_rows[si]) {
                si++;
                done_in_state = 0;
            }
        }
        const int S = (max_keys + 63) / 64;
        int rc = prefill_reserve_splits(c, f, S);
        if (rc) return rc;
        VC_TRY(cudaMemcpyAsync(f->block, f->hblock, f->head_bytes + (size_t)M * kDecDim * 4, cudaMemcpyHostToDevice,
                               st));
        cudaGraphExec_t &g = f->graphs[std::make_pair(M, S)];
        if (!g) {
            cudaGraph_t graph = nullptr;
            VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            rc = enqueue_prefill(d, f, M, S, st);
            cudaError_t e = cudaStreamEndCapture(st, &graph);
            if (rc) {
                if (graph) cudaGraphDestroy(graph);
                f->graphs.erase(std::make_pair(M, S));
                return rc;
            }
            VC_TRY(e);
            e = cudaGraphInstantiate(&g, graph, 0);
            cudaGraphDestroy(graph);
            VC_TRY(e);
        }
        VC_TRY(cudaGraphLaunch(g, st));
        VC_TRY(cudaMemcpyAsync(f->h_err, f->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaStreamSynchronize(st));   // the host block is reused by the next sequence
        if (*f->h_err) {
            *f->h_err = 0;
            cudaMemset(f->err, 0, sizeof(unsigned));
            set_error("decoder prefill: a device-side wait timed out (results discarded)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" vox_cuda_decoder *vox_cuda_decoder_create(const vox_cuda_dec_weights *w) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (!w || w->n_layers <= 0 || w->n_layers > kDecLayersMax || w->vocab <= 0 ||
        !w->tok_embeddings || !w->norm) {
        set_error("decoder_create: bad weight descriptor");
        return nullptr;
    }
    for (int l = 0; l < w->n_layers; l++) {
        const vox_cuda_dec_layer_weights &L = w->layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.w1 || !L.w2 || !L.w3 || !L.attention_norm ||
            !L.ffn_norm) {
            set_error("decoder_create: layer %d has a NULL weight", l);
            return nullptr;
        }
    }
    vox_cuda_decoder *d = new vox_cuda_decoder();
    d->device = c->device;
    d->n_layers = w->n_layers;
    d->vocab = w->vocab;
    const char *pdl_env = getenv("VOX_CUDA_PDL");
    d->pdl = !(pdl_env && pdl_env[0] == '0');
    const cudaMemcpyKind kind = w->weights_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaStream_t st = c->stream;
    auto alloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        if (dev_alloc(c, &p, bytes) != cudaSuccess) return nullptr;
        d->owned.push_back({p, bytes});
        return p;
    };
    const size_t D = kDecDim;
    Uploader up(st, !w->weights_on_device, c);   // host weights: pinned, pipelined
    // row-major staging for one fused matrix (the largest is the LM head)
    const size_t stage_elems = std::max((size_t)w->vocab, (size_t)2 * kDecHidden) * D;
    uint16_t *stage = nullptr;
    if (cudaMalloc(&stage, stage_elems * 2) != cudaSuccess) {
        set_error("decoder_create: staging allocation (%zu bytes) failed", stage_elems * 2);
        delete d;
        return nullptr;
    }
    bool ok = true;
    bool reported = false;   // the first failure's message is kept
    auto chk = [&](cudaError_t e, const char *what) {
        if (e == cudaSuccess) return;
        if (!reported) set_error("decoder_create: %s: %s", what, cudaGetErrorString(e));
        reported = true;
        ok = false;
    };
    // Fused matrix from row-major pieces: [rows_i x K] blocks stacked (or
    // row-interleaved when interleave), then tiled for the GEMV.
    // VOX_CUDA_DEC_TC_PREFILL = 0 drops the row-major copies (6 GB at 4B):
    // the prefill then runs through the decode-step kernels
    const char *tcp_env = getenv("VOX_CUDA_DEC_TC_PREFILL");
    d->tc_prefill = !(tcp_env && tcp_env[0] == '0');
    auto fuse = [&](const uint16_t *const *parts, const int *rows, int n_parts, int K, bool interleave,
                    const uint16_t **rm = nullptr) -> uint16_t * {
        int N = 0;
        for (int i = 0; i < n_parts; i++) N += rows[i];
        uint16_t *dst = (uint16_t *)alloc((size_t)round_up(N, kGemvRowAlign) * round_up(K, 16) * 2);
        if (!dst) return nullptr;
        if (interleave) {  // row 2i = parts[0][i], row 2i+1 = parts[1][i]
            for (int i = 0; i < n_parts && ok; i++)
                chk(up.copy2d(stage + (size_t)i * K, (size_t)n_parts * K * 2, parts[i], (size_t)K * 2,
                              (size_t)K * 2, rows[i]),
                    "interleaved weight copy");
        } else {
            size_t off = 0;
            for (int i = 0; i < n_parts && ok; i++) {
                chk(up.copy(stage + off, parts[i], (size_t)rows[i] * K * 2), "weight copy");
                off += (size_t)rows[i] * K;
            }
        }
        chk(launch_tile_weights(dst, stage, N, K, round_up(N, kGemvRowAlign), round_up(K, 16), st), "tiling");
        if (rm && ok) {   // the row-major fused matrix as staged
            uint16_t *r = (uint16_t *)alloc((size_t)N * K * 2);
            if (!r) chk(cudaErrorMemoryAllocation, "row-major copy allocation");
            else chk(cudaMemcpyAsync(r, stage, (size_t)N * K * 2, cudaMemcpyDeviceToDevice, st), "row-major copy");
            *rm = r;
        }
        chk(cudaStreamSynchronize(st), "upload");   // the stage is reused next
        return ok ? dst : nullptr;
    };
    for (int l = 0; l < w->n_layers && ok; l++) {
        const vox_cuda_dec_layer_weights &L = w->layers[l];
        DecLayer &o = d->L[l];
        // layers that alias an earlier layer's tensors share its device copies
        for (int j = 0; j < l; j++) {
            const vox_cuda_dec_layer_weights &J = w->layers[j];
            if (J.wq == L.wq && J.wk == L.wk && J.wv == L.wv && J.wo == L.wo && J.w1 == L.w1 &&
                J.w2 == L.w2 && J.w3 == L.w3) {
                o.qkv = d->L[j].qkv;
                o.wo = d->L[j].wo;
                o.w13 = d->L[j].w13;
                o.w2 = d->L[j].w2;
                o.qkv_rm = d->L[j].qkv_rm;
                o.wo_rm = d->L[j].wo_rm;
                o.w13_rm = d->L[j].w13_rm;
                o.w2_rm = d->L[j].w2_rm;
                break;
            }
        }
        if (!o.qkv) {
            const uint16_t *qkv_parts[3] = {L.wq, L.wk, L.wv};
            const int qkv_rows[3] = {kQDim, kKvDim, kKvDim};
            const uint16_t *wo_parts[1] = {L.wo};
            const int wo_rows[1] = {kDecDim};
            const uint16_t *w13_parts[2] = {L.w1, L.w3};
            const int w13_rows[2] = {kDecHidden, kDecHidden};
            const uint16_t *w2_parts[1] = {L.w2};
            const int w2_rows[1] = {kDecDim};
            const bool rm = d->tc_prefill;
            o.qkv = fuse(qkv_parts, qkv_rows, 3, kDecDim, false, rm ? &o.qkv_rm : nullptr);
            o.wo = ok ? fuse(wo_parts, wo_rows, 1, kQDim, false, rm ? &o.wo_rm : nullptr) : nullptr;
            o.w13 = ok ? fuse(w13_parts, w13_rows, 2, kDecDim, true, rm ? &o.w13_rm : nullptr) : nullptr;
            o.w2 = ok ? fuse(w2_parts, w2_rows, 1, kDecHidden, false, rm ? &o.w2_rm : nullptr) : nullptr;
            ok &= o.qkv && o.wo && o.w13 && o.w2;
            if (!ok) break;
        }
        // g_attn = attention_norm; g_ffn = ffn_norm * (1 + ada_scale[l])
        // (voxtral_decoder.c:466, 488-492), folded into the activation fragments
        std::vector<float> ha(D), hf(D), hada(D, 0.0f);
        // host vectors are read on the host (a host-to-host cudaMemcpy may take
        // a DMA path when the source page is registered)
        auto fetch = [&](float *dst, const float *src) {
            if (w->weights_on_device) chk(cudaMemcpy(dst, src, D * 4, cudaMemcpyDeviceToHost), "norm fetch");
            else memcpy(dst, src, D * 4);
        };
        fetch(ha.data(), L.attention_norm);
        fetch(hf.data(), L.ffn_norm);
        if (w->ada_scale) fetch(hada.data(), w->ada_scale + (size_t)l * D);
        for (size_t i = 0; i < D; i++) hf[i] = hf[i] * (1.0f + hada[i]);
        float *g = (float *)alloc(2 * D * 4);
        if (!g || !ok) {
            ok = false;
            break;
        }
        ok &= cudaMemcpy(g, ha.data(), D * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        ok &= cudaMemcpy(g + D, hf.data(), D * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        o.g_attn = g;
        o.g_ffn = g + D;
    }
    if (ok) {
        const uint16_t *emb_parts[1] = {w->tok_embeddings};
        const int emb_rows[1] = {w->vocab};
        d->tok_emb = fuse(emb_parts, emb_rows, 1, kDecDim, false);
        float *nrm = (float *)alloc(D * 4);
        ok = d->tok_emb && nrm;
        if (ok) {
            ok &= cudaMemcpy(nrm, w->norm, D * 4, kind) == cudaSuccess;
            d->norm = nrm;
        }
    }
    cudaFree(stage);
    if (!ok) {
        if (!reported) set_error("decoder_create: weight upload failed (out of device memory?)");
        vox_cuda_decoder_free(d);
        return nullptr;
    }
    return d;
}

extern "C" void vox_cuda_decoder_free(vox_cuda_decoder *d) {
    if (!d) return;
    DevCtx *c = ctx_for(d->device);
    cudaSetDevice(d->device);
    if (c) cudaStreamSynchronize(c->stream);   // also waits for asynchronous steps (see step_batch_dev)
    for (int i = 0; i <= kMaxBatch; i++) free_work(c, d->batch_work[i]);
    free_prefill(c, d->pf);
    if (d->tail) cudaEventDestroy(d->tail);
    for (auto &pr : d->owned)
        if (c) dev_free(c, pr.first, pr.second);
        else cudaFree(pr.first);
    delete d;
}

extern "C" vox_cuda_dec_state *vox_cuda_dec_state_create(vox_cuda_decoder *d, int kv_cap) {
    if (!d || kv_cap <= 0) {
        set_error("dec_state_create: bad arguments");
        return nullptr;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) {
        set_error("dec_state_create: device not initialised");
        return nullptr;
    }
    vox_cuda_dec_state *s = new vox_cuda_dec_state();
    s->dec = d;
    s->cap = kv_cap;
    s->ring_bytes = (size_t)d->n_layers * kv_cap * kKvDim * sizeof(float);
    if (dev_alloc(c, (void **)&s->k_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->v_ring, s->ring_bytes) != cudaSuccess) {
        set_error("dec_state_create: KV ring allocation (%zu bytes x 2) failed", s->ring_bytes);
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    if (cudaMemset(s->k_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->v_ring, 0, s->ring_bytes) != cudaSuccess) {
        set_error("dec_state_create: ring clear failed");
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    s->work = make_work(c, 1, d->vocab);
    if (!s->work) {
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    return s;
}

extern "C" void vox_cuda_dec_state_free(vox_cuda_dec_state *s) {
    if (!s) return;
    DevCtx *c = ctx_for(s->dec->device);
    cudaSetDevice(s->dec->device);
    if (c) cudaStreamSynchronize(c->stream);
    free_work(c, s->work);
    free_work(c, s->prefill_work);
    if (c) {
        dev_free(c, s->k_ring, s->k_ring ? s->ring_bytes : 0);
        dev_free(c, s->v_ring, s->v_ring ? s->ring_bytes : 0);
    }
    delete s;
}

extern "C" int vox_cuda_dec_state_reset(vox_cuda_dec_state *s) {
    if (!s) return VOX_CUDA_ERR_ARG;
    s->pos = 0;
    s->have_logits = false;
    s->last_token = -1;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_dec_state_position(const vox_cuda_dec_state *s) { return s ? s->pos : -1; }

extern "C" int vox_cuda_dec_state_set_position(vox_cuda_dec_state *s, int logical_pos) {
    if (!s || logical_pos < 0) {
        set_error("dec_state_set_position: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    s->pos = logical_pos;
    s->have_logits = false;
    return VOX_CUDA_OK;
}

static int kv_rows_check(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows) {
    if (!s || layer < 0 || layer >= s->dec->n_layers || first_pos < 0 || n_rows <= 0 ||
        n_rows > s->cap) {
        set_error("dec_state kv copy: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    return VOX_CUDA_OK;
}

static int ring_copy(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows, float *host_k,
                     float *host_v, bool to_device) {
    int rc = kv_rows_check(s, layer, first_pos, n_rows);
    if (rc) return rc;
    cudaSetDevice(s->dec->device);
    // the library stream is ordered after pending asynchronous steps, which write the ring
    if (DevCtx *c = ctx_for(s->dec->device)) VC_TRY(cudaStreamSynchronize(c->stream));
    const size_t row = (size_t)kKvDim * sizeof(float);
    int done = 0;
    while (done < n_rows) {
        const int slot = (first_pos + done) % s->cap;
        int run = s->cap - slot;
        if (run > n_rows - done) run = n_rows - done;
        float *dk = s->k_ring + ((size_t)layer * s->cap + slot) * kKvDim;
        float *dv = s->v_ring + ((size_t)layer * s->cap + slot) * kKvDim;
        if (to_device) {
            VC_TRY(cudaMemcpy(dk, host_k + (size_t)done * kKvDim, run * row, cudaMemcpyHostToDevice));
            VC_TRY(cudaMemcpy(dv, host_v + (size_t)done * kKvDim, run * row, cudaMemcpyHostToDevice));
        } else {
            VC_TRY(cudaMemcpy(host_k + (size_t)done * kKvDim, dk, run * row, cudaMemcpyDeviceToHost));
            VC_TRY(cudaMemcpy(host_v + (size_t)done * kKvDim, dv, run * row, cudaMemcpyDeviceToHost));
        }
        done += run;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_dec_state_load_kv(vox_cuda_dec_state *s, int layer, int first_pos,
                                          int n_rows, const float *k_rows, const float *v_rows) {
    if (!k_rows || !v_rows) return VOX_CUDA_ERR_ARG;
    return ring_copy(s, layer, first_pos, n_rows, const_cast<float *>(k_rows),
                     const_cast<float *>(v_rows), true);
}

extern "C" int vox_cuda_dec_state_read_kv(vox_cuda_dec_state *s, int layer, int first_pos,
                                          int n_rows, float *k_rows, float *v_rows) {
    if (!k_rows || !v_rows) return VOX_CUDA_ERR_ARG;
    return ring_copy(s, layer, first_pos, n_rows, k_rows, v_rows, false);
}

extern "C" int vox_cuda_decoder_full_step(vox_cuda_dec_state *s, const float *embed,
                                          const float *rope_freqs, float *logits) {
    if (!s || !embed) {
        set_error("decoder_full_step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = s->dec;
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    int rc = check_capacity(s, s->pos, s->pos);
    if (rc) return rc;
    StepWork *w = s->work;
    fill_slot(s, s->pos, h_slots(w));
    if (rope_freqs) memcpy(h_rope(w), rope_freqs, kHeadDim * sizeof(float));
    else host_rope_table(s->pos, kHeadDim, h_rope(w));
    memcpy(h_x(w), embed, kDecDim * sizeof(float));
    rc = run_step(d, c, w, true, c->stream, logits == nullptr);
    if (rc) return rc;
    if (logits) {
        VC_TRY(cudaMemcpyAsync(logits, w->logits, (size_t)d->vocab * 4, cudaMemcpyDeviceToHost, c->stream));
        VC_TRY(cudaStreamSynchronize(c->stream));
        if ((rc = check_step_error(w, c->stream))) return rc;
    }
    s->pos += 1;
    s->last_token = w->h_tokens[0];
    s->have_logits = true;
    return s->last_token;
}

extern "C" int vox_cuda_decoder_fill_alts(vox_cuda_dec_state *s, int n_alt, float cutoff,
                                          int *alt_ids) {
    if (!s || !alt_ids || n_alt < 1 || n_alt > 4) {
        set_error("decoder_fill_alts: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (!s->have_logits) {
        set_error("decoder_fill_alts: no decode step since the last reset");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = ctx_for(s->dec->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->dec->device);
    StepWork *w = s->work;
    VC_TRY(launch_fill_alts(w->logits, s->dec->vocab, w->tokens, n_alt, cutoff, w->alt_ids, c->stream));
    int ids[4];
    VC_TRY(cudaMemcpyAsync(ids, w->alt_ids, sizeof(ids), cudaMemcpyDeviceToHost, c->stream));
    VC_TRY(cudaStreamSynchronize(c->stream));
    int n = 0;
    for (int i = 0; i < n_alt; i++) {
        if (ids[i] < 0) break;
        alt_ids[n++] = ids[i];
    }
    return n;
}

extern "C" int vox_cuda_decoder_prefill_step(vox_cuda_dec_state *s, const float *x, int seq_len,
                                             const float *rope_freqs) {
    if (!s || !x || seq_len <= 0) {
        set_error("decoder_prefill_step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = s->dec;
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    int rc = VOX_CUDA_OK;
    if (d->tc_prefill) {
        // rows in launch sequences of kPrefillRows on the tensor cores
        for (int r0 = 0; r0 < seq_len; r0 += kPrefillRows) {
            const int last = s->pos + std::min(seq_len, r0 + kPrefillRows) - 1;
            if ((rc = check_capacity(s, s->pos + r0, last))) return rc;
        }
        std::lock_guard<std::mutex> lk(d->mu);
        rc = prefill_tc_rows(d, c, &s, &seq_len, 1, x, rope_freqs);
        if (rc) return rc;
        s->pos += seq_len;
        s->have_logits = false;
        return VOX_CUDA_OK;
    }
    // a row must not overwrite a ring slot still inside the window of an
    // earlier row of the same chunk: positions pos..pos+seq_len-1 all fit
    for (int r0 = 0; r0 < seq_len; r0 += kMaxBatch) {
        const int last = s->pos + ((seq_len - r0 < kMaxBatch) ? seq_len : r0 + kMaxBatch) - 1;
        if ((rc = check_capacity(s, s->pos + r0, last))) return rc;
    }
    // Rows are processed kMaxBatch at a time as parallel "streams" sharing one
    // ring: each row's attention covers positions <= its own, so the causal
    // mask of the prefill (voxtral_decoder.c:321-323) is preserved.
    for (int r0 = 0; r0 < seq_len; r0 += kMaxBatch) {
        const int n = (seq_len - r0 < kMaxBatch) ? seq_len - r0 : kMaxBatch;
        StepWork *&w = (n == kMaxBatch) ? s->prefill_work : d->batch_work[n];
        std::unique_lock<std::mutex> lk(d->mu, std::defer_lock);
        if (n != kMaxBatch) lk.lock();
        if (!w) w = make_work(c, n, d->vocab);
        if (!w) return VOX_CUDA_ERR_OOM;
        if (w->staged_pending) {   // an asynchronous step's upload of the host block
            VC_TRY(cudaEventSynchronize(w->staged));
            w->staged_pending = false;
        }
        for (int i = 0; i < n; i++) {
            const int pos = s->pos + r0 + i;
            fill_slot(s, pos, h_slots(w) + i);
            h_slots(w)[i].fresh = s->pos + r0;   // the chunk's first row
            if (rope_freqs) memcpy(h_rope(w) + i * kHeadDim, rope_freqs + (size_t)(r0 + i) * kHeadDim, kHeadDim * 4);
            else host_rope_table(pos, kHeadDim, h_rope(w) + i * kHeadDim);
        }
        memcpy(h_x(w), x + (size_t)r0 * kDecDim, (size_t)n * kDecDim * sizeof(float));
        rc = run_step(d, c, w, false, c->stream, true);
        if (rc) return rc;
    }
    s->pos += seq_len;
    s->have_logits = false;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_prefill_batch(vox_cuda_dec_state *const *states, int n, const float *x,
                                              const int *seq_lens, const float *rope_freqs) {
    if (!states || n <= 0 || !x || !seq_lens || !states[0]) {
        set_error("decoder_prefill_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = states[0]->dec;
    for (int i = 0; i < n; i++) {
        if (!states[i] || states[i]->dec != d || seq_lens[i] < 0) {
            set_error("decoder_prefill_batch: states must share one decoder, lengths >= 0");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("decoder_prefill_batch: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
    }
    if (!d->tc_prefill) {   // one state after the other through the decode-step kernels
        size_t off = 0;
        for (int i = 0; i < n; i++) {
            if (seq_lens[i] == 0) continue;
            int rc = vox_cuda_decoder_prefill_step(states[i], x + off * kDecDim,
                                                   seq_lens[i], rope_freqs ? rope_freqs + off * kHeadDim : nullptr);
            if (rc) return rc;
            off += seq_lens[i];
        }
        return VOX_CUDA_OK;
    }
    // a launch sequence holds at most kPrefillRows rows: each state's rows in
    // any one of them fit its ring together with the window before them
    for (int i = 0; i < n; i++)
        for (int r0 = 0; r0 < seq_lens[i]; r0 += kPrefillRows) {
            const int last = states[i]->pos + std::min(seq_lens[i], r0 + kPrefillRows) - 1;
            int rc = check_capacity(states[i], states[i]->pos + r0, last);
            if (rc) return rc;
        }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    std::lock_guard<std::mutex> lk(d->mu);
    int rc = prefill_tc_rows(d, c, states, seq_lens, n, x, rope_freqs);
    if (rc) return rc;
    for (int i = 0; i < n; i++) {
        states[i]->pos += seq_lens[i];
        if (seq_lens[i]) states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

static int batch_prepare(vox_cuda_dec_state *const *states, int n, vox_cuda_decoder **pd,
                         DevCtx **pc) {
    if (!states || n <= 0 || n > kMaxBatch) {
        set_error("decoder_step_batch: n must be 1..%d", kMaxBatch);
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = states[0] ? states[0]->dec : nullptr;
    for (int i = 0; i < n; i++) {
        if (!states[i] || states[i]->dec != d) {
            set_error("decoder_step_batch: states must share one decoder");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("decoder_step_batch: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
        int rc = check_capacity(states[i], states[i]->pos, states[i]->pos);
        if (rc) return rc;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    if (!d->batch_work[n]) d->batch_work[n] = make_work(c, n, d->vocab);
    if (!d->batch_work[n]) return VOX_CUDA_ERR_OOM;
    StepWork *w = d->batch_work[n];
    // an asynchronous step's upload of the host block may still be queued
    if (w->staged_pending) {
        VC_TRY(cudaEventSynchronize(w->staged));
        w->staged_pending = false;
    }
    for (int i = 0; i < n; i++) {
        fill_slot(states[i], states[i]->pos, h_slots(w) + i);
        host_rope_table(states[i]->pos, kHeadDim, h_rope(w) + i * kHeadDim);
    }
    *pd = d;
    *pc = c;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_step_batch(vox_cuda_dec_state *const *states, int n,
                                           const float *embeds, int *tokens) {
    if (!embeds || !tokens) {
        set_error("decoder_step_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    memcpy(h_x(w), embeds, (size_t)n * kDecDim * sizeof(float));
    rc = run_step(d, c, w, true, c->stream, true);
    w->err_pending = false;   // this step's error check covered the earlier ones
    if (rc) return rc;
    for (int i = 0; i < n; i++) {
        tokens[i] = w->h_tokens[i];
        states[i]->pos += 1;
        states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_step_batch_dev(vox_cuda_dec_state *const *states, int n,
                                               const float *embeds_dev, int *tokens_dev,
                                               void *stream) {
    if (!embeds_dev || !tokens_dev) {
        set_error("decoder_step_batch_dev: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (((uintptr_t)embeds_dev & 3u) || ((uintptr_t)tokens_dev & 3u)) {
        set_error("decoder_step_batch_dev: misaligned device pointers");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // a timeout raised by an earlier asynchronous step (its error word was
    // copied back behind err_ev) is reported now
    if (w->err_pending && cudaEventQuery(w->err_ev) == cudaSuccess) {
        w->err_pending = false;
        if ((rc = check_step_error(w, st))) return rc;
    }
    if (!d->tail && cudaEventCreateWithFlags(&d->tail, cudaEventDisableTiming) != cudaSuccess) {
        set_error("decoder_step_batch_dev: event creation failed");
        return VOX_CUDA_ERR_CUDA;
    }
    // the previous asynchronous step may have run on another stream
    if (d->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, d->tail, 0));
    // slots + rope tables from the host block; the embeddings from the device
    const size_t head = (char *)w->x - w->dblock;
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st));
    VC_TRY(cudaEventRecord(w->staged, st));
    w->staged_pending = true;
    VC_TRY(cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st));
    cudaGraphExec_t &g = w->graph[1];
    if (!g) {
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_layers(d, w, true, st);
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        VC_TRY(e);
        e = cudaGraphInstantiate(&g, graph, 0);
        cudaGraphDestroy(graph);
        VC_TRY(e);
    }
    VC_TRY(cudaGraphLaunch(g, st));
    VC_TRY(cudaMemcpyAsync(tokens_dev, w->tokens, sizeof(int) * n, cudaMemcpyDeviceToDevice, st));
    if (!w->err_pending) {   // one error-word copy in flight at a time
        VC_TRY(cudaMemcpyAsync(w->h_tokens + n, w->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(w->err_ev, st));
        w->err_pending = true;
    }
    // order the library stream (every synchronous entry point, the frees)
    // after this step, without a host wait
    VC_TRY(cudaEventRecord(d->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, d->tail, 0));
    d->tail_set = true;
    for (int i = 0; i < n; i++) {
        states[i]->pos += 1;
        states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_profile_batch(vox_cuda_dec_state *const *states, int n,
                                              const float *embeds_dev, int iters, float *ms) {
    if (!embeds_dev || !ms || iters <= 0) {
        set_error("decoder_profile_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = c->stream;
    const int n_launch = 5 * d->n_layers + 2;   // prep, 5 per layer, LM head
    std::vector<cudaEvent_t> evs(2 * n_launch);
    for (auto &e : evs)
        if (cudaEventCreate(&e) != cudaSuccess) {
            set_error("profile: event creation failed");
            return VOX_CUDA_ERR_CUDA;
        }
    double acc[VOX_CUDA_PROF_PHASES] = {0};
    const size_t head = (char *)w->x - w->dblock;
    for (int it = 0; it < iters && rc == VOX_CUDA_OK; it++) {
        if (cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess) {
            set_error("profile: staging copy failed");
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        rc = enqueue_layers(d, w, true, st, evs.data());
        if (rc) break;
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            set_error("profile: step failed");
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        for (int i = 0; i < n_launch; i++) {
            float t = 0.f;
            cudaEventElapsedTime(&t, evs[2 * i], evs[2 * i + 1]);
            const int phase = (i == n_launch - 1) ? VOX_CUDA_PROF_LM_HEAD
                              : (i == 0)           ? VOX_CUDA_PROF_QKV
                                                   : ((i - 1) % 5);
            acc[phase] += t;
        }
    }
    for (auto &e : evs) cudaEventDestroy(e);
    if (rc) return rc;
    for (int i = 0; i < VOX_CUDA_PROF_PHASES; i++) ms[i] = (float)(acc[i] / iters);
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_profile_sequence(vox_cuda_dec_state *const *states, int n,
                                                 const float *embeds_dev, int phase, int iters,
                                                 float *ms_per_launch) {
    if (!embeds_dev || !ms_per_launch || iters <= 0 || phase < 0 || phase >= VOX_CUDA_PROF_PHASES) {
        set_error("decoder_profile_sequence: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = c->stream;
    const size_t head = (char *)w->x - w->dblock;
    // one whole step first: every phase's inputs then hold real activations
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st));
    VC_TRY(cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st));
    if ((rc = enqueue_layers(d, w, true, st))) return rc;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_layers(d, w, true, st, nullptr, phase);
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    VC_TRY(e);
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    VC_TRY(e);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float t = 0.f;
    bool ok = cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
    for (int i = 0; ok && i < 2; i++) ok = cudaGraphLaunch(exec, st) == cudaSuccess;   // warm-up
    ok = ok && cudaEventRecord(e0, st) == cudaSuccess;
    for (int i = 0; ok && i < iters; i++) ok = cudaGraphLaunch(exec, st) == cudaSuccess;
    ok = ok && cudaEventRecord(e1, st) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
         cudaEventElapsedTime(&t, e0, e1) == cudaSuccess;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    if (!ok) {
        set_error("decoder_profile_sequence: timing failed");
        return VOX_CUDA_ERR_CUDA;
    }
    VC_TRY(cudaMemcpyAsync(w->h_tokens + n, w->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    VC_TRY(cudaStreamSynchronize(st));
    w->err_pending = false;
    if ((rc = check_step_error(w, st))) return rc;
    const int launches = phase == VOX_CUDA_PROF_LM_HEAD ? 1 : d->n_layers;
    *ms_per_launch = t / ((float)iters * launches);
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

// ---------------------------------------------------------------------------
// encoder chunk + adapter
// ---------------------------------------------------------------------------

namespace {

struct EncLayer {
    const uint16_t *qkv = nullptr;   // [6144, 1280] wq|wk|wv
    const uint16_t *wo = nullptr;    // [1280, 2048]
    const uint16_t *w13 = nullptr;   // [10240, 1280] w1/w3 row-interleaved
    const uint16_t *w2 = nullptr;    // [1280, 5120]
    const float *bq = nullptr, *bv = nullptr, *bo = nullptr, *b2 = nullptr;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

}  // namespace

namespace {

// Workspace of batched encoder launches (several states' chunks as one row
// block, vox_cuda_encoder_step_batch_dev): the row-wise kernels and GEMMs run
// once over all rows; each state's attention runs on its own side stream,
// forked and joined inside the captured graph.
struct EncBatch {
    int cap = 0;                  // rows
    char *ws = nullptr;
    size_t ws_bytes = 0;
    float *x = nullptr;           // [cap][1280]
    uint16_t *xn16 = nullptr;     // [cap][1280] fp16
    uint16_t *att16 = nullptr;    // [cap][2048]
    uint16_t *h16 = nullptr;      // [cap][5120]
    uint16_t *q16 = nullptr;      // [cap][2048]
    float *rope = nullptr;        // planes [64][cap]
    float *split = nullptr;       // split-K partials [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    unsigned *err = nullptr;
    unsigned *h_err = nullptr;    // pinned
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;
    cudaStream_t side[kEncMaxSegs] = {};
    cudaEvent_t fork = nullptr, join[kEncMaxSegs] = {};
    struct Graph {
        cudaGraphExec_t exec = nullptr;
        EncSeg *segs = nullptr;   // device [n]: this key's segments
    };
    // (states, rows) of a launch -> its graph
    std::map<std::vector<std::pair<const void *, int>>, Graph> graphs;
};
void free_enc_batch(DevCtx *c, EncBatch *b);
// Destroy the batched graphs that name `state` (all of them when NULL): a
// graph holds its states' ring and position pointers.
void drop_batch_graphs(EncBatch *b, const void *state);

}  // namespace

struct vox_cuda_encoder {
    int device = 0;
    int n_layers = 0;
    EncLayer L[kEncLayers];
    const float *norm = nullptr;
    const uint16_t *adapter0 = nullptr, *adapter1 = nullptr;
    const float *inv_freq = nullptr;   // [32] RoPE inverse frequencies (head_dim 64)
    std::vector<std::pair<void *, size_t>> owned;
    bool pdl = true;
    EncBatch *batch = nullptr;
    std::mutex mu;   // serialises batched launches (they share `batch`)
};

struct vox_cuda_enc_state {
    vox_cuda_encoder *enc = nullptr;
    int max_chunk = 0, cap = 0, pos = 0;
    uint16_t *k_ring = nullptr, *v_ring = nullptr;   // fp16 [layers][cap][2048]
    size_t ring_bytes = 0;
    char *ws = nullptr;                              // workspace block
    size_t ws_bytes = 0;
    float *x = nullptr;          // [Mx][1280] residual stream (fp32)
    uint16_t *xn16 = nullptr;    // [Mx][1280] bf16 normalised activations
    uint16_t *att16 = nullptr;   // [Mx][2048] bf16 attention output
    uint16_t *h16 = nullptr;     // [Mx][5120] bf16 SwiGLU output
    uint16_t *q16 = nullptr;     // [Mx][2048] fp16 queries
    float *rope = nullptr;       // RoPE planes [64][Mx]: cos of pair d at [d][row], sin at [32 + d][row]
    float *rope_src = nullptr;   // the host's table [Mx][64] (cos, sin pairs), when given
    float *aout = nullptr;       // adapter: [Mx/4][3072] fp32 out (Mx/4 x 5120 fp32 in shares x)
    uint16_t *a16 = nullptr;     // adapter: [Mx/4][5120] bf16 in
    uint16_t *mid16 = nullptr;   // adapter: [Mx/4][3072] bf16 mid
    unsigned *err = nullptr;
    int *pos_dev = nullptr;      // logical position of the chunk's first row
    float *split = nullptr;      // split-K partials of small-M GEMMs [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    float *h_rope = nullptr;     // pinned [Mx][64]
    int *h_pos = nullptr;        // pinned
    unsigned *h_err = nullptr;   // pinned: the error flag as of the last asynchronous step
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;
    cudaEvent_t tail = nullptr;  // the end of the last asynchronous step
    bool tail_set = false;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (rows, rope table?) -> step graph
};

extern "C" vox_cuda_encoder *vox_cuda_encoder_create(const vox_cuda_enc_weights *w) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (!w || w->n_layers <= 0 || w->n_layers > kEncLayers || !w->norm || !w->adapter0 || !w->adapter1) {
        set_error("encoder_create: bad weight descriptor");
        return nullptr;
    }
    for (int l = 0; l < w->n_layers; l++) {
        const vox_cuda_enc_layer_weights &L = w->layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.w1 || !L.w2 || !L.w3 || !L.wq_bias || !L.wv_bias ||
            !L.wo_bias || !L.w2_bias || !L.attention_norm || !L.ffn_norm) {
            set_error("encoder_create: layer %d has a NULL tensor", l);
            return nullptr;
        }
    }
    vox_cuda_encoder *e = new vox_cuda_encoder();
    e->device = c->device;
    e->n_layers = w->n_layers;
    const char *pdl_env = getenv("VOX_CUDA_PDL");
    e->pdl = !(pdl_env && pdl_env[0] == '0');
    const cudaMemcpyKind kind = w->weights_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    bool ok = true;
    Uploader up(c->stream, !w->weights_on_device, c);   // host weights: pinned, pipelined
    auto alloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        if (dev_alloc(c, &p, bytes) != cudaSuccess) return nullptr;
        e->owned.push_back({p, bytes});
        return p;
    };
    auto copy_f32 = [&](const float *src, size_t n) -> const float * {
        float *d = (float *)alloc(n * 4);
        if (!d || cudaMemcpy(d, src, n * 4, kind) != cudaSuccess) {
            ok = false;
            return nullptr;
        }
        return d;
    };
    const size_t D = kEncDim, Q = kEncQkv, H = kEncHidden;
    for (int l = 0; l < w->n_layers && ok; l++) {
        const vox_cuda_enc_layer_weights &L = w->layers[l];
        EncLayer &o = e->L[l];
        for (int j = 0; j < l; j++) {   // aliased layers share device copies
            const vox_cuda_enc_layer_weights &J = w->layers[j];
            if (J.wq == L.wq && J.wk == L.wk && J.wv == L.wv && J.wo == L.wo && J.w1 == L.w1 && J.w2 == L.w2 &&
                J.w3 == L.w3) {
                o.qkv = e->L[j].qkv;
                o.wo = e->L[j].wo;
                o.w13 = e->L[j].w13;
                o.w2 = e->L[j].w2;
                break;
            }
        }
        if (!o.qkv) {
            uint16_t *qkv = (uint16_t *)alloc(3 * Q * D * 2);
            uint16_t *wo = (uint16_t *)alloc(D * Q * 2);
            uint16_t *w13 = (uint16_t *)alloc(2 * H * D * 2);
            uint16_t *w2 = (uint16_t *)alloc(D * H * 2);
            ok = qkv && wo && w13 && w2;
            if (!ok) break;
            ok &= up.copy(qkv, L.wq, Q * D * 2) == cudaSuccess;
            ok &= up.copy(qkv + Q * D, L.wk, Q * D * 2) == cudaSuccess;
            ok &= up.copy(qkv + 2 * Q * D, L.wv, Q * D * 2) == cudaSuccess;
            ok &= up.copy(wo, L.wo, D * Q * 2) == cudaSuccess;
            ok &= up.copy2d(w13, 2 * D * 2, L.w1, D * 2, D * 2, H) == cudaSuccess;
            ok &= up.copy2d(w13 + D, 2 * D * 2, L.w3, D * 2, D * 2, H) == cudaSuccess;
            ok &= up.copy(w2, L.w2, D * H * 2) == cudaSuccess;
            // the tensor-core GEMMs take fp16 operands: activations keep 11
            // mantissa bits instead of bf16's 8 (weights convert exactly
            // except below fp16's normal range, ~6e-5); on the upload stream
            ok &= launch_bf16_to_f16(qkv, 3 * Q * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(wo, D * Q, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(w13, 2 * H * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(w2, D * H, c->stream) == cudaSuccess;
            o.qkv = qkv;
            o.wo = wo;
            o.w13 = w13;
            o.w2 = w2;
        }
        o.bq = copy_f32(L.wq_bias, Q);
        o.bv = copy_f32(L.wv_bias, Q);
        o.bo = copy_f32(L.wo_bias, D);
        o.b2 = copy_f32(L.w2_bias, D);
        o.attn_norm = copy_f32(L.attention_norm, D);
        o.ffn_norm = copy_f32(L.ffn_norm, D);
    }
    if (ok) {
        // RoPE inverse frequencies with the host formula of vox_compute_rope_freqs
        // (voxtral_kernels.c:494); the device forms pos * inv_freq and its cos/sin
        float invf[kEncHeadDim / 2];
        for (int d = 0; d < kEncHeadDim / 2; d++)
            invf[d] = 1.0f / powf(kRopeTheta, (float)(2 * d) / (float)kEncHeadDim);
        float *dinv = (float *)alloc(sizeof(invf));
        ok = dinv && cudaMemcpy(dinv, invf, sizeof(invf), cudaMemcpyHostToDevice) == cudaSuccess;
        e->inv_freq = dinv;
    }
    if (ok) {
        e->norm = copy_f32(w->norm, D);
        uint16_t *a0 = (uint16_t *)alloc((size_t)kDecDim * 4 * D * 2);
        uint16_t *a1 = (uint16_t *)alloc((size_t)kDecDim * kDecDim * 2);
        ok = ok && a0 && a1;
        if (ok) {
            ok &= up.copy(a0, w->adapter0, (size_t)kDecDim * 4 * D * 2) == cudaSuccess;
            ok &= up.copy(a1, w->adapter1, (size_t)kDecDim * kDecDim * 2) == cudaSuccess;
            ok &= launch_bf16_to_f16(a0, (size_t)kDecDim * 4 * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(a1, (size_t)kDecDim * kDecDim, c->stream) == cudaSuccess;
            ok &= cudaStreamSynchronize(c->stream) == cudaSuccess;
            e->adapter0 = a0;
            e->adapter1 = a1;
        }
    }
    if (!ok) {
        set_error("encoder_create: weight upload failed (%s)", cudaGetErrorString(cudaGetLastError()));
        vox_cuda_encoder_free(e);
        return nullptr;
    }
    return e;
}

extern "C" void vox_cuda_encoder_free(vox_cuda_encoder *e) {
    if (!e) return;
    DevCtx *c = ctx_for(e->device);
    cudaSetDevice(e->device);
    if (c) cudaStreamSynchronize(c->stream);
    free_enc_batch(c, e->batch);
    for (auto &pr : e->owned)
        if (c) dev_free(c, pr.first, pr.second);
        else cudaFree(pr.first);
    delete e;
}

extern "C" vox_cuda_enc_state *vox_cuda_enc_state_create(vox_cuda_encoder *e, int max_chunk) {
    if (!e || max_chunk <= 0 || max_chunk > 8192) {
        set_error("enc_state_create: max_chunk must be 1..8192");
        return nullptr;
    }
    DevCtx *c = ctx_for(e->device);
    if (!c) {
        set_error("enc_state_create: device not initialised");
        return nullptr;
    }
    cudaSetDevice(e->device);
    vox_cuda_enc_state *s = new vox_cuda_enc_state();
    s->enc = e;
    s->max_chunk = (max_chunk + 3) / 4 * 4;
    s->cap = (kEncWindow + s->max_chunk + kEncRingAlign - 1) / kEncRingAlign * kEncRingAlign;
    s->ring_bytes = (size_t)e->n_layers * s->cap * kEncQkv * 2;
    const size_t Mx = s->max_chunk;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_x = take(Mx * kEncDim * 4);
    const size_t o_xn = take(Mx * kEncDim * 2);
    const size_t o_att = take(Mx * kEncQkv * 2);
    const size_t o_h = take(Mx * kEncHidden * 2);
    const size_t o_q = take(Mx * kEncQkv * 2);
    const size_t o_rope = take(Mx * kEncHeadDim * 4);
    const size_t o_rope_src = take(Mx * kEncHeadDim * 4);
    const size_t o_aout = take(Mx / 4 * kDecDim * 4);
    const size_t o_a16 = take(Mx / 4 * 4 * kEncDim * 2);
    const size_t o_mid = take(Mx / 4 * kDecDim * 2);
    const size_t o_err = take(sizeof(unsigned));
    const size_t o_pos = take(sizeof(int));
    const size_t o_split = take(kEncSplitFloats * 4);            // split-K partials
    const size_t o_split_cnt = take(kTcSplitCounters * 4);       // split-K tickets
    s->ws_bytes = off;
    if (dev_alloc(c, (void **)&s->k_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->v_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->ws, s->ws_bytes) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_rope, Mx * kEncHeadDim * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_pos, sizeof(int), cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_err, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->err_ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->tail, cudaEventDisableTiming) != cudaSuccess) {
        set_error("enc_state_create: allocation failed");
        vox_cuda_enc_state_free(s);
        return nullptr;
    }
    *s->h_err = 0;
    s->x = (float *)(s->ws + o_x);
    s->xn16 = (uint16_t *)(s->ws + o_xn);
    s->att16 = (uint16_t *)(s->ws + o_att);
    s->h16 = (uint16_t *)(s->ws + o_h);
    s->q16 = (uint16_t *)(s->ws + o_q);
    s->rope = (float *)(s->ws + o_rope);
    s->rope_src = (float *)(s->ws + o_rope_src);
    s->aout = (float *)(s->ws + o_aout);
    s->a16 = (uint16_t *)(s->ws + o_a16);
    s->mid16 = (uint16_t *)(s->ws + o_mid);
    s->err = (unsigned *)(s->ws + o_err);
    s->pos_dev = (int *)(s->ws + o_pos);
    s->split = (float *)(s->ws + o_split);
    s->split_cnt = (unsigned *)(s->ws + o_split_cnt);
    if (cudaMemset(s->k_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->v_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->ws, 0, s->ws_bytes) != cudaSuccess) {
        set_error("enc_state_create: clear failed");
        vox_cuda_enc_state_free(s);
        return nullptr;
    }
    return s;
}

extern "C" void vox_cuda_enc_state_free(vox_cuda_enc_state *s) {
    if (!s) return;
    DevCtx *c = ctx_for(s->enc->device);
    cudaSetDevice(s->enc->device);
    if (c) cudaStreamSynchronize(c->stream);   // also waits for asynchronous steps (see step_dev)
    if (c) {
        dev_free(c, s->k_ring, s->k_ring ? s->ring_bytes : 0);
        dev_free(c, s->v_ring, s->v_ring ? s->ring_bytes : 0);
        dev_free(c, s->ws, s->ws ? s->ws_bytes : 0);
    }
    if (s->h_rope) cudaFreeHost(s->h_rope);
    if (s->h_pos) cudaFreeHost(s->h_pos);
    if (s->h_err) cudaFreeHost(s->h_err);
    if (s->err_ev) cudaEventDestroy(s->err_ev);
    if (s->tail) cudaEventDestroy(s->tail);
    for (auto &kv : s->graphs) cudaGraphExecDestroy(kv.second);
    {   // batched launches captured with this state must not outlive it
        std::lock_guard<std::mutex> lk(s->enc->mu);
        if (s->enc->batch) drop_batch_graphs(s->enc->batch, s);
    }
    delete s;
}

extern "C" int vox_cuda_enc_state_reset(vox_cuda_enc_state *s) {
    if (!s) return VOX_CUDA_ERR_ARG;
    s->pos = 0;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_enc_state_position(const vox_cuda_enc_state *s) { return s ? s->pos : -1; }

namespace {

// The 32 layers + final norm over s->x: M rows at the logical positions
// *s->pos_dev.. (read on the device, so the sequence can be replayed as a
// graph); RoPE from the uploaded table (table) or from a table computed on
// the device for this chunk.  evs (profiling only): 2 events per launch,
// recorded around it.
int enqueue_encoder(vox_cuda_enc_state *s, int M, bool table, cudaStream_t st, cudaEvent_t *evs = nullptr) {
    vox_cuda_encoder *e = s->enc;
    const bool pdl = e->pdl && evs == nullptr;
    int ei = 0;
#define VC_EV_BEGIN() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
#define VC_EV_END() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
    const size_t ring_layer = (size_t)s->cap * kEncQkv;
    VC_TRY(launch_enc_rope_table(s->rope, s->max_chunk, M, table ? s->rope_src : nullptr, s->pos_dev, e->inv_freq,
                                 st, false));
    for (int l = 0; l < e->n_layers; l++) {
        const EncLayer &L = e->L[l];
        VC_EV_BEGIN();
        VC_TRY(launch_rows_to_bf16(s->x, M, kEncDim, kEncDim, L.attn_norm, s->xn16, st, pdl, true));
        VC_EV_END();
        TcGemmParams p = {};
        p.M = M;
        p.N = 3 * kEncQkv;
        p.K = kEncDim;
        p.bias = L.bq;
        p.bias2 = L.bv;
        p.rope = s->rope;
        p.rope_ld = s->max_chunk;
        p.inv_freq = e->inv_freq;
        p.pos0_dev = s->pos_dev;
        p.q_out = s->q16;
        p.k_ring = s->k_ring + l * ring_layer;
        p.v_ring = s->v_ring + l * ring_layer;
        p.cap = s->cap;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        VC_EV_BEGIN();
        VC_TRY(launch_tc_gemm(TC_QKV_ENC, p, s->xn16, L.qkv, st, pdl));
        VC_EV_END();
        EncAttnParams a = {};
        a.q = s->q16;
        a.k_ring = s->k_ring + l * ring_layer;
        a.v_ring = s->v_ring + l * ring_layer;
        a.cap = s->cap;
        a.pos0_dev = s->pos_dev;
        a.M = M;
        a.out = s->att16;
        a.f16 = 1;
        a.err = s->err;
        VC_EV_BEGIN();
        VC_TRY(launch_enc_attn(a, st, pdl));
        VC_EV_END();
        p = TcGemmParams{};
        p.M = M;
        p.N = kEncDim;
        p.K = kEncQkv;
        p.out = s->x;
        p.ldo = kEncDim;
        p.bias = L.bo;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        VC_EV_BEGIN();
        VC_TRY(launch_tc_gemm(TC_RESID, p, s->att16, L.wo, st, pdl));
        VC_EV_END();
        VC_EV_BEGIN();
        VC_TRY(launch_rows_to_bf16(s->x, M, kEncDim, kEncDim, L.ffn_norm, s->xn16, st, pdl, true));
        VC_EV_END();
        p = TcGemmParams{};
        p.M = M;
        p.N = 2 * kEncHidden;
        p.K = kEncDim;
        p.out_bf16 = s->h16;
        p.ldo_bf16 = kEncHidden;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        VC_EV_BEGIN();
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, s->xn16, L.w13, st, pdl));
        VC_EV_END();
        p = TcGemmParams{};
        p.M = M;
        p.N = kEncDim;
        p.K = kEncHidden;
        p.out = s->x;
        p.ldo = kEncDim;
        p.bias = L.b2;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        VC_EV_BEGIN();
        VC_TRY(launch_tc_gemm(TC_RESID, p, s->h16, L.w2, st, pdl));
        VC_EV_END();
    }
    VC_EV_BEGIN();
    VC_TRY(launch_rows_rmsnorm(s->x, M, kEncDim, e->norm, st, pdl));
    VC_EV_END();
#undef VC_EV_BEGIN
#undef VC_EV_END
    return VOX_CUDA_OK;
}

// Upload the chunk position, then replay (capturing on first use) the
// encoder graph for this chunk shape.
int run_encoder(vox_cuda_enc_state *s, int M, bool table, cudaStream_t st) {
    // the position by value: back-to-back asynchronous calls cannot race on it
    VC_TRY(launch_set_int(s->pos_dev, s->pos, st));
    cudaGraphExec_t &g = s->graphs[std::make_pair(M, table ? 1 : 0)];
    if (!g) {
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_encoder(s, M, table, st);
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        VC_TRY(e);
        e = cudaGraphInstantiate(&g, graph, 0);
        cudaGraphDestroy(graph);
        VC_TRY(e);
    }
    VC_TRY(cudaGraphLaunch(g, st));
    return VOX_CUDA_OK;
}

int enc_check(vox_cuda_enc_state *s, int new_len) {
    if (!s || new_len <= 0) {
        set_error("encoder step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (new_len > s->max_chunk) {
        set_error("encoder step: %d rows exceed the state's max_chunk %d", new_len, s->max_chunk);
        return VOX_CUDA_ERR_CAPACITY;
    }
    if (!ctx_for(s->enc->device)) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->enc->device);
    return VOX_CUDA_OK;
}

int enc_err_check(vox_cuda_enc_state *s, cudaStream_t st) {
    unsigned err = 0;
    VC_TRY(cudaMemcpyAsync(&err, s->err, sizeof(err), cudaMemcpyDeviceToHost, st));
    VC_TRY(cudaStreamSynchronize(st));
    s->err_pending = false;   // this check covered the asynchronous steps before it
    if (err) {
        cudaMemset(s->err, 0, sizeof(unsigned));
        set_error("encoder: a device-side wait timed out (results discarded)");
        return VOX_CUDA_ERR_CUDA;
    }
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_encoder_full_step(vox_cuda_enc_state *s, float *x, int new_len,
                                          const float *rope_freqs) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    if (rope_freqs) {
        memcpy(s->h_rope, rope_freqs, (size_t)new_len * kEncHeadDim * 4);
        VC_TRY(cudaMemcpyAsync(s->rope_src, s->h_rope, (size_t)new_len * kEncHeadDim * 4, cudaMemcpyHostToDevice,
                               st));
    }
    VC_TRY(cudaMemcpyAsync(s->x, x, (size_t)new_len * kEncDim * 4, cudaMemcpyHostToDevice, st));
    if ((rc = run_encoder(s, new_len, rope_freqs != nullptr, st))) return rc;
    VC_TRY(cudaMemcpyAsync(x, s->x, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToHost, st));
    if ((rc = enc_err_check(s, st))) return rc;
    s->pos += new_len;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_encoder_step_dev(vox_cuda_enc_state *s, float *x_dev, int new_len, void *stream) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x_dev) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // a timeout raised by an earlier chunk on this state (its flag was copied
    // back behind err_ev) is reported now
    if (s->err_pending && cudaEventQuery(s->err_ev) == cudaSuccess) {
        s->err_pending = false;
        if (*s->h_err) {
            *s->h_err = 0;
            VC_TRY(cudaMemsetAsync(s->err, 0, sizeof(unsigned), st));
            set_error("encoder: a device-side wait of an earlier chunk timed out (its results are invalid)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    // the previous asynchronous chunk may have run on another stream
    if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
    VC_TRY(cudaMemcpyAsync(s->x, x_dev, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st));
    if ((rc = run_encoder(s, new_len, false, st))) return rc;
    VC_TRY(cudaMemcpyAsync(x_dev, s->x, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st));
    if (!s->err_pending) {   // one flag copy in flight at a time
        VC_TRY(cudaMemcpyAsync(s->h_err, s->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(s->err_ev, st));
        s->err_pending = true;
    }
    // order the library stream (every synchronous entry point, the frees)
    // after this chunk, without a host wait
    VC_TRY(cudaEventRecord(s->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
    s->tail_set = true;
    s->pos += new_len;
    return VOX_CUDA_OK;
}

namespace {

void drop_batch_graphs(EncBatch *b, const void *state) {
    for (auto it = b->graphs.begin(); it != b->graphs.end();) {
        bool hit = state == nullptr;
        for (const auto &kv : it->first) hit = hit || kv.first == state;
        if (!hit) {
            ++it;
            continue;
        }
        if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
        if (it->second.segs) cudaFree(it->second.segs);
        it = b->graphs.erase(it);
    }
}

void free_enc_batch(DevCtx *c, EncBatch *b) {
    if (!b) return;
    drop_batch_graphs(b, nullptr);
    if (c) dev_free(c, b->ws, b->ws ? b->ws_bytes : 0);
    if (b->h_err) cudaFreeHost(b->h_err);
    if (b->err_ev) cudaEventDestroy(b->err_ev);
    if (b->fork) cudaEventDestroy(b->fork);
    for (int i = 0; i < kEncMaxSegs; i++) {
        if (b->side[i]) cudaStreamDestroy(b->side[i]);
        if (b->join[i]) cudaEventDestroy(b->join[i]);
    }
    delete b;
}

EncBatch *make_enc_batch(DevCtx *c, int rows) {
    EncBatch *b = new EncBatch();
    b->cap = (int)align_up((size_t)rows, 128);
    const size_t R = (size_t)b->cap;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_x = take(R * kEncDim * 4), o_xn = take(R * kEncDim * 2), o_att = take(R * kEncQkv * 2);
    const size_t o_h = take(R * kEncHidden * 2), o_q = take(R * kEncQkv * 2), o_rope = take(R * kEncHeadDim * 4);
    const size_t o_split = take(kEncSplitFloats * 4), o_cnt = take(kTcSplitCounters * 4), o_err = take(4);
    b->ws_bytes = off;
    bool ok = dev_alloc(c, (void **)&b->ws, b->ws_bytes) == cudaSuccess &&
              cudaMemset(b->ws, 0, b->ws_bytes) == cudaSuccess &&
              cudaHostAlloc((void **)&b->h_err, sizeof(unsigned), cudaHostAllocDefault) == cudaSuccess &&
              cudaEventCreateWithFlags(&b->err_ev, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&b->fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; i < kEncMaxSegs && ok; i++)
        ok = cudaStreamCreateWithFlags(&b->side[i], cudaStreamNonBlocking) == cudaSuccess &&
             cudaEventCreateWithFlags(&b->join[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        set_error("encoder batch workspace: allocation of %zu bytes failed", b->ws_bytes);
        free_enc_batch(c, b);
        return nullptr;
    }
    *b->h_err = 0;
    char *w = b->ws;
    b->x = (float *)(w + o_x);
    b->xn16 = (uint16_t *)(w + o_xn);
    b->att16 = (uint16_t *)(w + o_att);
    b->h16 = (uint16_t *)(w + o_h);
    b->q16 = (uint16_t *)(w + o_q);
    b->rope = (float *)(w + o_rope);
    b->split = (float *)(w + o_split);
    b->split_cnt = (unsigned *)(w + o_cnt);
    b->err = (unsigned *)(w + o_err);
    return b;
}

// The layers of one batched launch over M rows of n states (segments `segs`,
// rows[i] rows of state i from row0[i]): the encoder chunk of
// vox_encoder_forward_incremental (voxtral_encoder.c:452-636) for all of them,
// the row-wise work once, the attention per state on forked side streams.
int enqueue_encoder_batch(vox_cuda_encoder *e, EncBatch *b, vox_cuda_enc_state *const *states, const int *rows,
                          const int *row0, int n, int M, const EncSeg *segs, cudaStream_t st) {
    const bool pdl = e->pdl;
    VC_TRY(launch_enc_rope_table_segs(b->rope, b->cap, M, segs, n, e->inv_freq, st, false));
    auto gemm = [&](int N, int K) {
        TcGemmParams p = {};
        p.M = M;
        p.N = N;
        p.K = K;
        p.err = b->err;
        p.f16 = 1;
        p.ws = b->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = b->split_cnt;
        return p;
    };
    for (int l = 0; l < e->n_layers; l++) {
        const EncLayer &L = e->L[l];
        VC_TRY(launch_rows_to_bf16(b->x, M, kEncDim, kEncDim, L.attn_norm, b->xn16, st, pdl, true));
        TcGemmParams p = gemm(3 * kEncQkv, kEncDim);
        p.bias = L.bq;
        p.bias2 = L.bv;
        p.rope = b->rope;
        p.rope_ld = b->cap;
        p.inv_freq = e->inv_freq;
        p.q_out = b->q16;
        p.segs = segs;
        p.n_segs = n;
        p.layer = l;
        p.cap = 1 << 30;   // (the rings are the segments')
        VC_TRY(launch_tc_gemm(TC_QKV_ENC, p, b->xn16, L.qkv, st, pdl));
        // each state's windowed attention over its own ring, concurrently
        VC_TRY(cudaEventRecord(b->fork, st));
        for (int i = 0; i < n; i++) {
            vox_cuda_enc_state *s = states[i];
            const size_t ring_layer = (size_t)s->cap * kEncQkv;
            VC_TRY(cudaStreamWaitEvent(b->side[i], b->fork, 0));
            EncAttnParams a = {};
            a.q = b->q16 + (size_t)row0[i] * kEncQkv;
            a.k_ring = s->k_ring + l * ring_layer;
            a.v_ring = s->v_ring + l * ring_layer;
            a.cap = s->cap;
            a.pos0_dev = s->pos_dev;
            a.M = rows[i];
            a.out = b->att16 + (size_t)row0[i] * kEncQkv;
            a.f16 = 1;
            a.err = b->err;
            VC_TRY(launch_enc_attn(a, b->side[i], false));
            VC_TRY(cudaEventRecord(b->join[i], b->side[i]));
            VC_TRY(cudaStreamWaitEvent(st, b->join[i], 0));
        }
        p = gemm(kEncDim, kEncQkv);
        p.out = b->x;
        p.ldo = kEncDim;
        p.bias = L.bo;
        VC_TRY(launch_tc_gemm(TC_RESID, p, b->att16, L.wo, st, false));
        VC_TRY(launch_rows_to_bf16(b->x, M, kEncDim, kEncDim, L.ffn_norm, b->xn16, st, pdl, true));
        p = gemm(2 * kEncHidden, kEncDim);
        p.out_bf16 = b->h16;
        p.ldo_bf16 = kEncHidden;
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, b->xn16, L.w13, st, pdl));
        p = gemm(kEncDim, kEncHidden);
        p.out = b->x;
        p.ldo = kEncDim;
        p.bias = L.b2;
        VC_TRY(launch_tc_gemm(TC_RESID, p, b->h16, L.w2, st, pdl));
    }
    VC_TRY(launch_rows_rmsnorm(b->x, M, kEncDim, e->norm, st, pdl));
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_encoder_step_batch_dev(vox_cuda_enc_state *const *states, int n, float *const *x_dev,
                                               const int *new_lens, void *stream) {
    if (!states || n <= 0 || n > kEncMaxSegs || !x_dev || !new_lens || !states[0]) {
        set_error("encoder_step_batch_dev: 1..%d states with their rows", kEncMaxSegs);
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_encoder *e = states[0]->enc;
    int M = 0, row0[kEncMaxSegs];
    for (int i = 0; i < n; i++) {
        int rc = enc_check(states[i], new_lens[i]);
        if (rc) return rc;
        if (!x_dev[i] || states[i]->enc != e) {
            set_error("encoder_step_batch_dev: states must share one encoder, x_dev non-NULL");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("encoder_step_batch_dev: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
        row0[i] = M;
        M += new_lens[i];
    }
    DevCtx *c = ctx_for(e->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    std::lock_guard<std::mutex> lk(e->mu);
    EncBatch *b = e->batch;
    if (b && b->cap < M) {   // grow: the graphs hold the old pointers
        VC_TRY(cudaDeviceSynchronize());
        free_enc_batch(c, b);
        b = e->batch = nullptr;
    }
    if (!b && !(b = e->batch = make_enc_batch(c, std::max(M, 1024)))) return VOX_CUDA_ERR_OOM;
    // a timeout raised by an earlier batched launch is reported now
    if (b->err_pending && cudaEventQuery(b->err_ev) == cudaSuccess) {
        b->err_pending = false;
        if (*b->h_err) {
            *b->h_err = 0;
            VC_TRY(cudaMemsetAsync(b->err, 0, sizeof(unsigned), st));
            set_error("encoder batch: a device-side wait of an earlier launch timed out (its results are invalid)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    std::vector<std::pair<const void *, int>> key;
    for (int i = 0; i < n; i++) key.push_back({states[i], new_lens[i]});
    if (b->graphs.size() >= 64 && !b->graphs.count(key)) {   // bound the cache (ragged chunk sizes)
        VC_TRY(cudaStreamSynchronize(st));
        drop_batch_graphs(b, nullptr);
    }
    EncBatch::Graph &g = b->graphs[key];
    if (!g.exec) {
        EncSeg h[kEncMaxSegs];
        for (int i = 0; i < n; i++) h[i] = EncSeg{states[i]->k_ring, states[i]->v_ring, states[i]->pos_dev,
                                                  states[i]->cap, row0[i]};
        if (cudaMalloc((void **)&g.segs, sizeof(EncSeg) * n) != cudaSuccess ||
            cudaMemcpy(g.segs, h, sizeof(EncSeg) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
            set_error("encoder_step_batch_dev: segment table allocation failed");
            b->graphs.erase(key);
            return VOX_CUDA_ERR_CUDA;
        }
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_encoder_batch(e, b, states, new_lens, row0, n, M, g.segs, st);
        cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (rc == VOX_CUDA_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&g.exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (rc || ce != cudaSuccess) {
            cudaFree(g.segs);
            b->graphs.erase(key);
            if (!rc) set_error("encoder_step_batch_dev: graph capture failed: %s", cudaGetErrorString(ce));
            return rc ? rc : VOX_CUDA_ERR_CUDA;
        }
    }
    for (int i = 0; i < n; i++) {
        vox_cuda_enc_state *s = states[i];
        // the previous asynchronous step of this state may have run on another stream
        if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
        VC_TRY(launch_set_int(s->pos_dev, s->pos, st));
        VC_TRY(cudaMemcpyAsync(b->x + (size_t)row0[i] * kEncDim, x_dev[i], (size_t)new_lens[i] * kEncDim * 4,
                               cudaMemcpyDeviceToDevice, st));
    }
    VC_TRY(cudaGraphLaunch(g.exec, st));
    for (int i = 0; i < n; i++)
        VC_TRY(cudaMemcpyAsync(x_dev[i], b->x + (size_t)row0[i] * kEncDim, (size_t)new_lens[i] * kEncDim * 4,
                               cudaMemcpyDeviceToDevice, st));
    if (!b->err_pending) {   // one flag copy in flight at a time
        VC_TRY(cudaMemcpyAsync(b->h_err, b->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(b->err_ev, st));
        b->err_pending = true;
    }
    // order the library stream after this launch for every state (as step_dev)
    for (int i = 0; i < n; i++) {
        vox_cuda_enc_state *s = states[i];
        VC_TRY(cudaEventRecord(s->tail, st));
        if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
        s->tail_set = true;
        s->pos += new_lens[i];
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_adapter_forward(vox_cuda_enc_state *s, const float *enc, int n, float *out) {
    int rc = enc_check(s, n);
    if (rc) return rc;
    if (!enc || !out || n % 4 != 0) {
        set_error("adapter_forward: n must be a positive multiple of 4");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    vox_cuda_encoder *e = s->enc;
    const int rows = n / 4, K0 = 4 * kEncDim;
    // 4 consecutive [1280] rows are one [5120] row: the same memory
    VC_TRY(cudaMemcpyAsync(s->x, enc, (size_t)n * kEncDim * 4, cudaMemcpyHostToDevice, st));
    VC_TRY(launch_rows_to_bf16(s->x, rows, K0, K0, nullptr, s->a16, st, false, true));
    TcGemmParams p = {};
    p.M = rows;
    p.N = kDecDim;
    p.K = K0;
    p.act = 1;                  // GELU (voxtral_encoder.c:664)
    p.out_bf16 = s->mid16;      // fp16, the next GEMM's A
    p.ldo_bf16 = kDecDim;
    p.err = s->err;
    p.f16 = 1;
    p.ws = s->split;
    p.ws_floats = kEncSplitFloats;
    p.ws_cnt = s->split_cnt;
    VC_TRY(launch_tc_gemm(TC_STORE, p, s->a16, e->adapter0, st, false));
    p = TcGemmParams{};
    p.M = rows;
    p.N = kDecDim;
    p.K = kDecDim;
    p.out = s->aout;
    p.ldo = kDecDim;
    p.err = s->err;
    p.f16 = 1;
    p.ws = s->split;
    p.ws_floats = kEncSplitFloats;
    p.ws_cnt = s->split_cnt;
    VC_TRY(launch_tc_gemm(TC_STORE, p, s->mid16, e->adapter1, st, false));
    VC_TRY(cudaMemcpyAsync(out, s->aout, (size_t)rows * kDecDim * 4, cudaMemcpyDeviceToHost, st));
    return enc_err_check(s, st);
}

extern "C" int vox_cuda_enc_state_set_position(vox_cuda_enc_state *s, int logical_pos) {
    if (!s || logical_pos < 0) {
        set_error("enc_state_set_position: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    s->pos = logical_pos;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_encoder_profile(vox_cuda_enc_state *s, const float *x_dev, int new_len, int iters,
                                        float *ms) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x_dev || !ms || iters <= 0) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    const int n_launch = 7 * s->enc->n_layers + 1;
    std::vector<cudaEvent_t> evs(2 * n_launch);
    for (auto &e : evs)
        if (cudaEventCreate(&e) != cudaSuccess) return VOX_CUDA_ERR_CUDA;
    double acc[VOX_CUDA_EPROF_PHASES] = {0};
    static const int phase_of[7] = {VOX_CUDA_EPROF_NORM, VOX_CUDA_EPROF_QKV, VOX_CUDA_EPROF_ATTN,
                                    VOX_CUDA_EPROF_WO, VOX_CUDA_EPROF_NORM, VOX_CUDA_EPROF_W13,
                                    VOX_CUDA_EPROF_W2};
    for (int it = 0; it < iters && rc == VOX_CUDA_OK; it++) {
        *s->h_pos = s->pos;
        if (cudaMemcpyAsync(s->pos_dev, s->h_pos, sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(s->x, x_dev, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess) {
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        rc = enqueue_encoder(s, new_len, false, st, evs.data());
        if (rc) break;
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        for (int i = 0; i < n_launch; i++) {
            float t = 0.f;
            cudaEventElapsedTime(&t, evs[2 * i], evs[2 * i + 1]);
            acc[(i == n_launch - 1) ? VOX_CUDA_EPROF_NORM : phase_of[i % 7]] += t;
        }
    }
    for (auto &e : evs) cudaEventDestroy(e);
    if (rc) return rc;
    for (int i = 0; i < VOX_CUDA_EPROF_PHASES; i++) ms[i] = (float)(acc[i] / iters);
    return VOX_CUDA_OK;
}

// ---------------------------------------------------------------------------
// Conv stem (stream_conv_stem, voxtral.c:487-665): im2col + tcgen05 GEMM
// with bias + GELU, twice, with the streaming state on the device.
// ---------------------------------------------------------------------------

struct vox_cuda_conv_stem {
    int device = 0;
    int max_mel = 0;
    long long frames = 0;           // mel frames consumed so far
    uint16_t *w0 = nullptr;         // fp16 [1280][384]
    uint16_t *w1 = nullptr;         // fp16 [1280][3840]
    float *b0 = nullptr, *b1 = nullptr;
    char *ws = nullptr;             // workspace block
    size_t ws_bytes = 0;
    float *mel = nullptr;           // [max_mel][128] this chunk's frames
    float *mel_hist = nullptr;      // [2][128]
    uint16_t *c0_hist = nullptr;    // [2][1280] conv0 outputs of the last two frames
    uint16_t *a0 = nullptr;         // [max_mel][384] conv0 im2col
    uint16_t *c0 = nullptr;         // [max_mel][1280] conv0 outputs (fp16)
    uint16_t *a1 = nullptr;         // [max_out][3840] conv1 im2col
    float *out = nullptr;           // [max_out][1280]
    unsigned *err = nullptr;
    // asynchronous steps (step_dev): deferred error flag, ordering event
    unsigned *h_err = nullptr;      // pinned
    cudaEvent_t err_ev = nullptr, tail = nullptr;
    bool err_pending = false, tail_set = false;
};

extern "C" vox_cuda_conv_stem *vox_cuda_conv_stem_create(const float *conv0_weight, const float *conv0_bias,
                                                         const float *conv1_weight, const float *conv1_bias,
                                                         int max_mel) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (!conv0_weight || !conv0_bias || !conv1_weight || !conv1_bias || max_mel <= 0 || max_mel > 1 << 20) {
        set_error("conv_stem_create: bad arguments");
        return nullptr;
    }
    vox_cuda_conv_stem *s = new vox_cuda_conv_stem();
    s->device = c->device;
    s->max_mel = max_mel;
    const size_t Mx = (size_t)max_mel, Ox = Mx / 2 + 2;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t n_w0 = (size_t)kEncDim * 3 * 128, n_w1 = (size_t)kEncDim * 3 * kEncDim;
    const size_t o_w0 = take(n_w0 * 2), o_w1 = take(n_w1 * 2), o_b0 = take(kEncDim * 4), o_b1 = take(kEncDim * 4);
    const size_t o_stage = take(n_w1 * 4);   // fp32 staging of a weight before conversion
    const size_t o_mel = take(Mx * 128 * 4), o_mh = take(2 * 128 * 4), o_ch = take(2 * kEncDim * 2);
    const size_t o_a0 = take(Mx * 3 * 128 * 2), o_c0 = take(Mx * kEncDim * 2);
    const size_t o_a1 = take(Ox * 3 * kEncDim * 2), o_out = take(Ox * kEncDim * 4), o_err = take(4);
    s->ws_bytes = off;
    if (dev_alloc(c, (void **)&s->ws, s->ws_bytes) != cudaSuccess) {
        set_error("conv_stem_create: allocation of %zu bytes failed", s->ws_bytes);
        delete s;
        return nullptr;
    }
    s->w0 = (uint16_t *)(s->ws + o_w0);
    s->w1 = (uint16_t *)(s->ws + o_w1);
    s->b0 = (float *)(s->ws + o_b0);
    s->b1 = (float *)(s->ws + o_b1);
    s->mel = (float *)(s->ws + o_mel);
    s->mel_hist = (float *)(s->ws + o_mh);
    s->c0_hist = (uint16_t *)(s->ws + o_ch);
    s->a0 = (uint16_t *)(s->ws + o_a0);
    s->c0 = (uint16_t *)(s->ws + o_c0);
    s->a1 = (uint16_t *)(s->ws + o_a1);
    s->out = (float *)(s->ws + o_out);
    s->err = (unsigned *)(s->ws + o_err);
    float *stage = (float *)(s->ws + o_stage);
    bool ok = cudaMemset(s->ws, 0, s->ws_bytes) == cudaSuccess &&
              cudaMemcpy(stage, conv0_weight, n_w0 * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              launch_f32_to_f16(stage, s->w0, n_w0, 0) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
              cudaMemcpy(stage, conv1_weight, n_w1 * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              launch_f32_to_f16(stage, s->w1, n_w1, 0) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
              cudaMemcpy(s->b0, conv0_bias, kEncDim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(s->b1, conv1_bias, kEncDim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaHostAlloc((void **)&s->h_err, sizeof(unsigned), cudaHostAllocDefault) == cudaSuccess &&
              cudaEventCreateWithFlags(&s->err_ev, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&s->tail, cudaEventDisableTiming) == cudaSuccess;
    if (s->h_err) *s->h_err = 0;
    if (!ok) {
        set_error("conv_stem_create: weight upload failed");
        vox_cuda_conv_stem_free(s);
        return nullptr;
    }
    return s;
}

extern "C" void vox_cuda_conv_stem_free(vox_cuda_conv_stem *s) {
    if (!s) return;
    DevCtx *c = ctx_for(s->device);
    cudaSetDevice(s->device);
    if (c) {
        cudaStreamSynchronize(c->stream);   // also waits for asynchronous steps (see step_dev)
        dev_free(c, s->ws, s->ws ? s->ws_bytes : 0);
    }
    if (s->h_err) cudaFreeHost(s->h_err);
    if (s->err_ev) cudaEventDestroy(s->err_ev);
    if (s->tail) cudaEventDestroy(s->tail);
    delete s;
}

extern "C" int vox_cuda_conv_stem_reset(vox_cuda_conv_stem *s) {
    if (!s) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->device);
    VC_TRY(cudaMemsetAsync(s->mel_hist, 0, 2 * 128 * 4, c->stream));
    VC_TRY(cudaMemsetAsync(s->c0_hist, 0, 2 * kEncDim * 2, c->stream));
    VC_TRY(cudaStreamSynchronize(c->stream));
    s->frames = 0;
    return VOX_CUDA_OK;
}

namespace {

// One stem step's kernels: mel [n_new][128] (device) -> out [n_out][1280]
// (device), the streaming state updated on the device.  Returns n_out.
int stem_enqueue(vox_cuda_conv_stem *s, const float *mel, int n_new, float *out, cudaStream_t st) {
    const long long f0 = s->frames, u0 = f0 / 2;
    const int n_out = (int)((f0 + n_new) / 2 - u0);
    VC_TRY(launch_stem_im2col0(mel, s->mel_hist, n_new, s->a0, st));
    TcGemmParams p = {};
    p.M = n_new;
    p.N = kEncDim;
    p.K = 3 * 128;
    p.bias = s->b0;
    p.act = 1;                 // GELU (voxtral.c:515)
    p.out_bf16 = s->c0;        // fp16: the conv1 im2col's source
    p.ldo_bf16 = kEncDim;
    p.err = s->err;
    p.f16 = 1;
    VC_TRY(launch_tc_gemm(TC_STORE, p, s->a0, s->w0, st, false));
    if (n_out > 0) {
        VC_TRY(launch_stem_im2col1(s->c0, s->c0_hist, f0, u0, n_out, s->a1, st));
        p = TcGemmParams{};
        p.M = n_out;
        p.N = kEncDim;
        p.K = 3 * kEncDim;
        p.bias = s->b1;
        p.act = 1;             // GELU (voxtral.c:648)
        p.out = out;
        p.ldo = kEncDim;
        p.err = s->err;
        p.f16 = 1;
        VC_TRY(launch_tc_gemm(TC_STORE, p, s->a1, s->w1, st, false));
    }
    VC_TRY(launch_stem_state(mel, n_new, s->mel_hist, s->c0, s->c0_hist, st));
    s->frames += n_new;
    return n_out;
}

int stem_check(vox_cuda_conv_stem *s, const void *mel, int n_new, const void *out, const char *what) {
    if (!s || !mel || !out || n_new <= 0) {
        set_error("%s: bad arguments", what);
        return VOX_CUDA_ERR_ARG;
    }
    if (n_new > s->max_mel) {
        set_error("%s: %d mel frames exceed the state's %d", what, n_new, s->max_mel);
        return VOX_CUDA_ERR_CAPACITY;
    }
    if (!ctx_for(s->device)) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->device);
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_conv_stem_step(vox_cuda_conv_stem *s, const float *mel_new, int n_new, float *out) {
    int rc = stem_check(s, mel_new, n_new, out, "conv_stem_step");
    if (rc) return rc;
    DevCtx *c = ctx_for(s->device);
    std::lock_guard<std::mutex> lk(c->mu);
    cudaStream_t st = c->stream;
    VC_TRY(cudaMemcpyAsync(s->mel, mel_new, (size_t)n_new * 128 * 4, cudaMemcpyHostToDevice, st));
    const int n_out = stem_enqueue(s, s->mel, n_new, s->out, st);
    if (n_out < 0) return n_out;
    if (n_out > 0)
        VC_TRY(cudaMemcpyAsync(out, s->out, (size_t)n_out * kEncDim * 4, cudaMemcpyDeviceToHost, st));
    unsigned h_err = 0;
    VC_TRY(cudaMemcpyAsync(&h_err, s->err, 4, cudaMemcpyDeviceToHost, st));
    VC_TRY(cudaStreamSynchronize(st));
    s->err_pending = false;   // this check covered the asynchronous steps before it
    if (h_err) {
        cudaMemset(s->err, 0, sizeof(unsigned));
        set_error("conv_stem_step: a tensor-core GEMM wait timed out");
        return VOX_CUDA_ERR_CUDA;
    }
    return n_out;
}

extern "C" int vox_cuda_conv_stem_step_dev(vox_cuda_conv_stem *s, const float *mel_dev, int n_new, float *out_dev,
                                           void *stream) {
    int rc = stem_check(s, mel_dev, n_new, out_dev, "conv_stem_step_dev");
    if (rc) return rc;
    DevCtx *c = ctx_for(s->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // a timeout raised by an earlier asynchronous step is reported now
    if (s->err_pending && cudaEventQuery(s->err_ev) == cudaSuccess) {
        s->err_pending = false;
        if (*s->h_err) {
            *s->h_err = 0;
            VC_TRY(cudaMemsetAsync(s->err, 0, sizeof(unsigned), st));
            set_error("conv_stem: a tensor-core GEMM wait of an earlier step timed out (its rows are invalid)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
    const int n_out = stem_enqueue(s, mel_dev, n_new, out_dev, st);
    if (n_out < 0) return n_out;
    if (!s->err_pending) {
        VC_TRY(cudaMemcpyAsync(s->h_err, s->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(s->err_ev, st));
        s->err_pending = true;
    }
    VC_TRY(cudaEventRecord(s->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
    s->tail_set = true;
    return n_out;
}

// ---------------------------------------------------------------------------
// log-mel front end: the incremental context (vox_mel_ctx_t,
// voxtral_audio.c:392-612) and the one-shot spectrogram (:290-395)
// ---------------------------------------------------------------------------

struct vox_cuda_mel {
    int device = 0;
    long long pad = 0;         // logical samples before the first real one (zeros, never stored)
    long long n_samples = 0;   // logical samples so far, pad included
    long long n_frames = 0;    // frames computed (and reported) so far
    bool finished = false;
    int ring_len = 0;          // power of two
    float *block = nullptr;    // tables | ring | reflection | staging
    size_t bytes = 0;
    float *ring = nullptr, *refl = nullptr, *stage = nullptr;
    int stage_frames = 0;
    MelTables t = {};
};

namespace {

long long mel_frames_upto(long long n_samples) {
    return n_samples >= kMelWin ? (n_samples - kMelWin) / kMelHop + 1 : 0;
}

// upload the 4 host tables into dst (win | cos | sin | filt) and point t at them
int mel_upload_tables(float *dst, MelTables *t, cudaStream_t st) {
    const size_t n_tab = kMelWin + 2 * (size_t)kMelWin * kMelFreq + (size_t)kMelFreq * kMelBins;
    std::vector<float> h(n_tab);
    float *win = h.data(), *cs = win + kMelWin, *sn = cs + (size_t)kMelWin * kMelFreq;
    float *ft = sn + (size_t)kMelWin * kMelFreq;
    mel_host_tables(win, cs, sn, ft);
    VC_TRY(cudaMemcpyAsync(dst, h.data(), n_tab * 4, cudaMemcpyHostToDevice, st));
    VC_TRY(cudaStreamSynchronize(st));   // h is on this stack frame
    t->win = dst;
    t->cos_t = dst + kMelWin;
    t->sin_t = t->cos_t + (size_t)kMelWin * kMelFreq;
    t->filt_t = t->sin_t + (size_t)kMelWin * kMelFreq;
    return VOX_CUDA_OK;
}

constexpr size_t kMelTableFloats = kMelWin + 2 * (size_t)kMelWin * kMelFreq + (size_t)kMelFreq * kMelBins;

// Append n samples (src, or zeros when src is NULL) at the stream's end.
int mel_append(vox_cuda_mel *m, const float *src, int n, cudaMemcpyKind kind, cudaStream_t st) {
    long long at = m->n_samples - m->pad;   // ring index of the first new sample
    int done = 0;
    while (done < n) {
        const int slot = (int)(at & (m->ring_len - 1));
        int run = m->ring_len - slot;
        if (run > n - done) run = n - done;
        if (src) VC_TRY(cudaMemcpyAsync(m->ring + slot, src + done, (size_t)run * 4, kind, st));
        else VC_TRY(cudaMemsetAsync(m->ring + slot, 0, (size_t)run * 4, st));
        done += run;
        at += run;
    }
    m->n_samples += n;
    return VOX_CUDA_OK;
}

// Compute every frame that now fits into out; returns the count (or < 0).
int mel_compute(vox_cuda_mel *m, float *out, cudaStream_t st) {
    const long long t1 = mel_frames_upto(m->n_samples);
    const int nf = (int)(t1 - m->n_frames);
    if (nf <= 0) return 0;
    VC_TRY(launch_mel_frames(m->ring, m->ring_len - 1, m->pad, m->n_frames, nf, m->t, out, st));
    m->n_frames = t1;
    return nf;
}

// The largest piece appended at once: the frame in progress keeps < 400
// samples live in the ring.
int mel_piece(const vox_cuda_mel *m) { return m->ring_len - kMelWin; }

// Feed n samples in ring-sized pieces; frames go to out (device) when
// out_dev, else through the staging block to the host buffer.
int mel_feed_impl(vox_cuda_mel *m, const float *samples, int n, float *out, int max_frames, bool dev,
                  cudaStream_t st) {
    if (!m || (!samples && n > 0) || !out || n < 0 || max_frames < 0) {
        set_error("mel_feed: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (m->finished) {
        set_error("mel_feed: the context is finished");
        return VOX_CUDA_ERR_ARG;
    }
    const long long want = mel_frames_upto(m->n_samples + n) - m->n_frames;
    if (want > max_frames) {
        set_error("mel_feed: %lld frames exceed the output's %d", want, max_frames);
        return VOX_CUDA_ERR_CAPACITY;
    }
    cudaSetDevice(m->device);
    const cudaMemcpyKind kind = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    int written = 0, done = 0, rc;
    while (done < n) {
        const int k = std::min(n - done, mel_piece(m));
        if ((rc = mel_append(m, samples + done, k, kind, st))) return rc;
        done += k;
        float *dst = dev ? out + (size_t)written * kMelBins : m->stage;
        const int nf = mel_compute(m, dst, st);
        if (nf < 0) return nf;
        if (!dev && nf > 0)
            VC_TRY(cudaMemcpyAsync(out + (size_t)written * kMelBins, m->stage, (size_t)nf * kMelBins * 4,
                                   cudaMemcpyDeviceToHost, st));
        written += nf;
        if (!dev) VC_TRY(cudaStreamSynchronize(st));   // the staging block is reused by the next piece
    }
    return written;
}

int mel_finish_impl(vox_cuda_mel *m, int right_pad, float *out, int max_frames, bool dev, cudaStream_t st) {
    if (!m || !out || right_pad < 0 || max_frames < 0) {
        set_error("mel_finish: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (m->finished) return 0;
    const long long final_samples = m->n_samples + right_pad + kMelCenterPad;
    const long long computed = mel_frames_upto(final_samples) - m->n_frames;
    const long long report = computed > 0 ? computed - 1 : 0;   // the last frame is dropped
    if (report > max_frames) {
        set_error("mel_finish: %lld frames exceed the output's %d", report, max_frames);
        return VOX_CUDA_ERR_CAPACITY;
    }
    cudaSetDevice(m->device);
    // the reflection of the signal before the right pad, taken first: the pad
    // may overwrite its source in the ring (voxtral_audio.c:583-590)
    VC_TRY(launch_mel_reflect(m->ring, m->ring_len - 1, m->pad, m->n_samples - 2, kMelCenterPad, m->refl, st));
    int written = 0, rc;
    auto emit = [&](int nf) -> int {   // copy the stage's first rows that are reported
        const int keep = (int)std::min<long long>(nf, report - written);
        if (keep > 0)
            VC_TRY(cudaMemcpyAsync(out + (size_t)written * kMelBins, m->stage, (size_t)keep * kMelBins * 4,
                                   dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
        written += keep > 0 ? keep : 0;
        VC_TRY(cudaStreamSynchronize(st));   // the staging block is reused by the next piece
        return VOX_CUDA_OK;
    };
    int left = right_pad;
    while (left > 0) {
        const int k = std::min(left, mel_piece(m));
        if ((rc = mel_append(m, nullptr, k, cudaMemcpyDeviceToDevice, st))) return rc;
        left -= k;
        const int nf = mel_compute(m, m->stage, st);
        if (nf < 0) return nf;
        if ((rc = emit(nf))) return rc;
    }
    if ((rc = mel_append(m, m->refl, kMelCenterPad, cudaMemcpyDeviceToDevice, st))) return rc;
    const int nf = mel_compute(m, m->stage, st);
    if (nf < 0) return nf;
    if ((rc = emit(nf))) return rc;
    if (m->n_frames > 0) m->n_frames -= 1;
    m->finished = true;
    return written;
}

}  // namespace

extern "C" vox_cuda_mel *vox_cuda_mel_create(int left_pad_samples, int max_feed_samples) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (left_pad_samples < 0 || max_feed_samples <= 0) {
        set_error("mel_create: bad arguments");
        return nullptr;
    }
    vox_cuda_mel *m = new vox_cuda_mel();
    m->device = c->device;
    m->pad = kMelCenterPad + (long long)left_pad_samples;
    m->n_samples = m->pad;
    m->ring_len = 1024;
    while (m->ring_len < max_feed_samples + kMelWin) m->ring_len *= 2;
    // the first piece also yields the frames over the leading zeros
    m->stage_frames = (int)((m->pad + m->ring_len) / kMelHop + 4);
    const size_t n = kMelTableFloats + m->ring_len + kMelCenterPad + (size_t)m->stage_frames * kMelBins;
    m->bytes = n * 4;
    if (dev_alloc(c, (void **)&m->block, m->bytes) != cudaSuccess) {
        set_error("mel_create: cudaMalloc(%zu) failed", m->bytes);
        delete m;
        return nullptr;
    }
    m->ring = m->block + kMelTableFloats;
    m->refl = m->ring + m->ring_len;
    m->stage = m->refl + kMelCenterPad;
    if (mel_upload_tables(m->block, &m->t, c->stream) != VOX_CUDA_OK) {
        vox_cuda_mel_free(m);
        return nullptr;
    }
    return m;
}

extern "C" void vox_cuda_mel_free(vox_cuda_mel *m) {
    if (!m) return;
    DevCtx *c = ctx_for(m->device);
    cudaSetDevice(m->device);
    if (c) {
        cudaStreamSynchronize(c->stream);
        dev_free(c, m->block, m->block ? m->bytes : 0);
    }
    delete m;
}

extern "C" int vox_cuda_mel_frames(const vox_cuda_mel *m) { return m ? (int)m->n_frames : VOX_CUDA_ERR_ARG; }

extern "C" int vox_cuda_mel_frames_for(const vox_cuda_mel *m, int n_samples) {
    if (!m || n_samples < 0) return VOX_CUDA_ERR_ARG;
    return (int)(mel_frames_upto(m->n_samples + n_samples) - m->n_frames);
}

extern "C" int vox_cuda_mel_feed(vox_cuda_mel *m, const float *samples, int n_samples, float *mel_out,
                                 int max_frames) {
    DevCtx *c = m ? ctx_for(m->device) : nullptr;
    if (m && !c) return VOX_CUDA_ERR_UNAVAILABLE;
    return mel_feed_impl(m, samples, n_samples, mel_out, max_frames, false, c ? c->stream : nullptr);
}

extern "C" int vox_cuda_mel_feed_dev(vox_cuda_mel *m, const float *samples_dev, int n_samples, float *mel_dev,
                                     int max_frames, void *stream) {
    DevCtx *c = m ? ctx_for(m->device) : nullptr;
    if (m && !c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : (c ? c->stream : nullptr);
    return mel_feed_impl(m, samples_dev, n_samples, mel_dev, max_frames, true, st);
}

extern "C" int vox_cuda_mel_finish(vox_cuda_mel *m, int right_pad_samples, float *mel_out, int max_frames) {
    DevCtx *c = m ? ctx_for(m->device) : nullptr;
    if (m && !c) return VOX_CUDA_ERR_UNAVAILABLE;
    return mel_finish_impl(m, right_pad_samples, mel_out, max_frames, false, c ? c->stream : nullptr);
}

extern "C" int vox_cuda_mel_finish_dev(vox_cuda_mel *m, int right_pad_samples, float *mel_dev, int max_frames,
                                       void *stream) {
    DevCtx *c = m ? ctx_for(m->device) : nullptr;
    if (m && !c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaStream_t st = stream ? (cudaStream_t)stream : (c ? c->stream : nullptr);
    return mel_finish_impl(m, right_pad_samples, mel_dev, max_frames, true, st);
}

extern "C" int vox_cuda_mel_spectrogram(const float *samples, int n_samples, float *mel_out, int max_frames) {
    if (!samples || !mel_out || n_samples <= 0 || max_frames < 0) {
        set_error("mel_spectrogram: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    // center padding by reflection on both sides, the last frame dropped
    const long long padded_len = (long long)n_samples + 2 * kMelCenterPad;
    const long long frames = mel_frames_upto(padded_len) - 1;
    if (frames <= 0) {
        set_error("mel_spectrogram: audio too short (%d samples)", n_samples);
        return VOX_CUDA_ERR_ARG;
    }
    if (frames > max_frames) {
        set_error("mel_spectrogram: %lld frames exceed the output's %d", frames, max_frames);
        return VOX_CUDA_ERR_CAPACITY;
    }
    DevCtx *c = cur_ctx();
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    std::vector<float> padded((size_t)padded_len);
    for (int i = 0; i < kMelCenterPad; i++) {
        const int l = kMelCenterPad - i, r = n_samples - 2 - i;
        padded[i] = l < n_samples ? samples[l] : 0.0f;
        padded[(size_t)kMelCenterPad + n_samples + i] = r >= 0 ? samples[r] : 0.0f;
    }
    memcpy(padded.data() + kMelCenterPad, samples, (size_t)n_samples * 4);
    const size_t n = kMelTableFloats + (size_t)padded_len + (size_t)frames * kMelBins;
    float *block = nullptr;
    if (dev_alloc(c, (void **)&block, n * 4) != cudaSuccess) {
        set_error("mel_spectrogram: cudaMalloc(%zu) failed", n * 4);
        return VOX_CUDA_ERR_OOM;
    }
    MelTables t;
    int rc = mel_upload_tables(block, &t, c->stream);
    float *sig = block + kMelTableFloats, *out = sig + padded_len;
    cudaStream_t st = c->stream;
    if (rc == VOX_CUDA_OK &&
        (cudaMemcpyAsync(sig, padded.data(), (size_t)padded_len * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
         launch_mel_frames(sig, -1, 0, 0, (int)frames, t, out, st) != cudaSuccess ||
         cudaMemcpyAsync(mel_out, out, (size_t)frames * kMelBins * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
         cudaStreamSynchronize(st) != cudaSuccess)) {
        set_error("mel_spectrogram: %s", cudaGetErrorString(cudaGetLastError()));
        rc = VOX_CUDA_ERR_CUDA;
    }
    dev_free(c, block, n * 4);
    return rc == VOX_CUDA_OK ? (int)frames : rc;
}
