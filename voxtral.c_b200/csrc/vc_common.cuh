// vc_common.cuh - shared device helpers for the sm_100a voxtral backend.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vc {

// Model constants (voxtral.h:18-50).
constexpr int kDecDim = 3072;
constexpr int kDecLayersMax = 26;
constexpr int kDecHeads = 32;
constexpr int kDecKvHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kQDim = kDecHeads * kHeadDim;      // 4096
constexpr int kKvDim = kDecKvHeads * kHeadDim;   // 1024
constexpr int kQkvRows = kQDim + 2 * kKvDim;     // 6144
constexpr int kDecHidden = 9216;
constexpr int kDecWindow = 8192;
constexpr int kVocab = 131072;
constexpr int kEncDim = 1280;
constexpr int kEncLayers = 32;
constexpr int kEncHeads = 32;
constexpr int kEncHeadDim = 64;
constexpr int kEncQkv = kEncHeads * kEncHeadDim; // 2048
constexpr int kEncHidden = 5120;
constexpr int kEncWindow = 750;
constexpr float kNormEps = 1e-5f;
constexpr float kRopeTheta = 1.0e6f;
constexpr int kMaxBatch = 8;                     // streams per batched decode step

// bf16 -> f32 is a 16-bit left shift (voxtral_kernels.c:124-128).
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// Streaming 16-byte load of read-only weights: no L1 allocation, L2
// evict-first so the weight stream does not push the KV cache and the
// activations out of L2.
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t policy) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p), "l"(policy));
    return r;
}

__device__ __forceinline__ uint64_t make_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t make_evict_last_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 8 bf16 weights (one uint4) dotted with 8 fp32 activations, fp32 FMA in
// index order.
__device__ __forceinline__ float dot8(uint4 w, float4 a, float4 b, float acc) {
    acc = fmaf(bf16lo(w.x), a.x, acc);
    acc = fmaf(bf16hi(w.x), a.y, acc);
    acc = fmaf(bf16lo(w.y), a.z, acc);
    acc = fmaf(bf16hi(w.y), a.w, acc);
    acc = fmaf(bf16lo(w.z), b.x, acc);
    acc = fmaf(bf16hi(w.z), b.y, acc);
    acc = fmaf(bf16lo(w.w), b.z, acc);
    acc = fmaf(bf16hi(w.w), b.w, acc);
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (no-op when launched without the attribute) / allow the next one to start.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// This CTA's share of an L2 prefetch of [base, base + bytes): the weights of
// a later kernel in the stream, which depend on nothing this kernel writes.
// One thread per CTA calls it; the bulk prefetches (<= 64 KB each, shares of
// whole 4 KB pages) complete on their own.  base and bytes: multiples of 16.
__device__ __forceinline__ void l2_prefetch_share(const void *base, unsigned long long bytes) {
    if (!base || bytes == 0) return;
    const unsigned long long nb = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    const unsigned long long b =
        blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
    const unsigned long long share = ((bytes + nb - 1) / nb + 4095ull) & ~4095ull;
    const unsigned long long end = min((b + 1) * share, bytes);
    const char *p = static_cast<const char *>(base);
    for (unsigned long long off = b * share; off < end; off += 65536ull) {
        const unsigned n = (unsigned)min(65536ull, end - off);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n) : "memory");
    }
}

// ---------------------------------------------------------------------------
// B-fragment ("xfrag") writers for the decode GEMV's activations: per 16-wide
// k-block, lane 4m + q holds stream m's values at k = 2q, 2q+1 (word 0) and
// 2q+8, 2q+9 (word 1) as bf16 pairs, and the bf16 residuals x - hi of the
// same values in words 2 and 3, so x = hi + lo to ~2^-17 relative.
// Layout: [K/16][32 lanes][4 words].
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t bf16_bits_rn(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);   // round to nearest even; finite inputs
    return u >> 16;
}

// Split-activation layout of the tensor-core prefill: row r of a matrix x
// is stored as bf16 hi = bf16(x_r) at hilo_row(r) and lo = bf16(x_r - hi) at
// hilo_row(r) + 64, i.e. every 64 rows form one 128-row MMA tile [hi; lo].
__host__ __device__ __forceinline__ int hilo_row(int r) { return ((r >> 6) << 7) + (r & 63); }
__host__ __device__ __forceinline__ int hilo_rows(int M) { return ((M + 63) >> 6) << 7; }

__device__ __forceinline__ void split_bf16(float v, uint32_t &hi, uint32_t &lo) {
    hi = bf16_bits_rn(v);
    lo = bf16_bits_rn(v - __uint_as_float(hi << 16));
}

// two consecutive activations (k even) of stream m
__device__ __forceinline__ void xfrag_put2(uint32_t *xfrag, int m, int k, float v0, float v1) {
    const int kb = k >> 4, kk = k & 15;
    const int lane = 4 * m + ((kk & 7) >> 1), word = kk >> 3;
    uint32_t h0, l0, h1, l1;
    split_bf16(v0, h0, l0);
    split_bf16(v1, h1, l1);
    uint32_t *w = xfrag + ((size_t)kb * 32 + lane) * 4;
    w[word] = h0 | (h1 << 16);
    w[2 + word] = l0 | (l1 << 16);
}

// one activation of stream m
__device__ __forceinline__ void xfrag_put1(uint32_t *xfrag, int m, int k, float v) {
    const int kb = k >> 4, kk = k & 15;
    const int lane = 4 * m + ((kk & 7) >> 1), word = kk >> 3, half = kk & 1;
    uint32_t h, l;
    split_bf16(v, h, l);
    uint16_t *w = reinterpret_cast<uint16_t *>(xfrag + ((size_t)kb * 32 + lane) * 4);
    w[2 * word + half] = (uint16_t)h;
    w[2 * (2 + word) + half] = (uint16_t)l;
}

}  // namespace vc
