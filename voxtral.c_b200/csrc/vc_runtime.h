// vc_runtime.h - shared by the C-ABI runtime files: vc_runtime.cu (device
// contexts, lifecycle, matmul and kernel-level entry points), vc_rt_decoder.cu
// (resident decoder, KV rings, steps, prefill), vc_rt_encoder.cu (encoder
// chunks, batched launches, adapter) and vc_rt_front.cu (conv stem, log-mel).
// Per-device contexts, device-memory accounting, error reporting and the
// pinned weight uploader.
#pragma once

#include "voxtral_cuda.h"

#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

namespace vc {
namespace rt {

// The calling thread's error message (vox_cuda_last_error).
template <typename... A>
inline void set_error(const char *fmt, A... a) {
    set_last_error(fmt, a...);
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

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

int current_device();
DevCtx *ctx_for(int dev);
// The calling thread's device context, or NULL (error set) before vox_cuda_init.
DevCtx *cur_ctx();
// cudaMalloc / cudaFree with the context's byte count kept.
cudaError_t dev_alloc(DevCtx *c, void **p, size_t bytes);
void dev_free(DevCtx *c, void *p, size_t bytes);
// Host RoPE table for one logical position, the same formula as
// vox_compute_rope_freqs (voxtral_kernels.c:488-500).
void host_rope_table(int pos, int head_dim, float *cs);

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

}  // namespace rt
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
