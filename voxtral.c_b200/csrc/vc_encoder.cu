// vc_encoder.cu - encoder-chunk kernels besides the tensor-core GEMM:
// causal sliding-window flash attention over the encoder's fp16 KV ring
// (vox_causal_attention for seq_q = new_len, window 750, 32 heads x 64;
// voxtral_kernels.c:412-482 as called at voxtral_encoder.c:574-576), and the
// final RMSNorm.
//
// Attention: grid (ceil(M / 64), 32 heads), 128 threads (4 warps x 16 query
// rows).  Q (fp16, RoPE applied by the QKV GEMM epilogue) stays in registers as
// mma.m16n8k16 A fragments; 64-key blocks of K and V are double-buffered in
// shared memory with cp.async; S = Q K^T and O += P V run on the tensor cores
// (fp16 in, fp32 accumulate) with an online softmax in fp32 registers.  Rows
// are masked to keys [pos - 749, pos] of their own logical position.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <cuda_fp16.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

namespace vc {

constexpr int kEaRows = 64;          // query rows per CTA
constexpr int kEaKeys = 64;          // keys per block
constexpr int kEaPitch = 72;         // fp16 row pitch in shared memory (144 B: conflict-free ldmatrix)

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__global__ void __launch_bounds__(128)
enc_attn_kernel(const EncAttnParams p) {
    __shared__ __align__(128) __half sQ[kEaRows * kEaPitch];
    __shared__ __align__(128) __half sK[2][kEaKeys * kEaPitch];
    __shared__ __align__(128) __half sV[2][kEaKeys * kEaPitch];

    grid_dep_wait();
    grid_dep_launch();

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = blockIdx.x * kEaRows, head = blockIdx.y;
    const int M = p.M;
    const int pos0 = p.pos0_dev ? *p.pos0_dev : p.pos0;
    const int p_first = pos0 + r0;
    const int p_last = pos0 + min(r0 + kEaRows, M) - 1;
    const int k_lo = max(0, p_first - (kEncWindow - 1));
    const int n_blocks = (p_last - k_lo) / kEaKeys + 1;

    // ---- Q tile -> shared ----
    for (int c = tid; c < kEaRows * 8; c += 128) {
        const int r = c >> 3, ch = c & 7;
        __half *dst = sQ + r * kEaPitch + ch * 8;
        if (r0 + r < M) cp_async16(dst, p.q + (size_t)(r0 + r) * kEncQkv + head * kEncHeadDim + ch * 8);
        else *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    }
    auto load_kv = [&](int blk, int buf) {
        const int kbase = k_lo + blk * kEaKeys;
        for (int c = tid; c < kEaKeys * 8; c += 128) {
            const int r = c >> 3, ch = c & 7;
            const int kp = kbase + r;
            __half *dk = sK[buf] + r * kEaPitch + ch * 8;
            __half *dv = sV[buf] + r * kEaPitch + ch * 8;
            if (kp <= p_last) {
                const size_t off = (size_t)(kp % p.cap) * kEncQkv + head * kEncHeadDim + ch * 8;
                cp_async16(dk, p.k_ring + off);
                cp_async16(dv, p.v_ring + off);
            } else {
                *reinterpret_cast<uint4 *>(dk) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4 *>(dv) = make_uint4(0, 0, 0, 0);
            }
        }
    };
    load_kv(0, 0);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    // Q A-fragments for this warp's 16 rows, 4 k-steps of 16 dims
    uint32_t qa[4][4];
    {
        const int row = warp * 16 + (lane & 15);
        for (int ks = 0; ks < 4; ks++)
            ldsm_x4(su32(sQ + row * kEaPitch + ks * 16 + (lane >> 4) * 8), qa[ks][0], qa[ks][1], qa[ks][2],
                    qa[ks][3]);
    }

    const int g = lane >> 2, q4 = lane & 3;
    const int row_a = r0 + warp * 16 + g, row_b = row_a + 8;   // this thread's two query rows
    const int pos_a = pos0 + row_a, pos_b = pos0 + row_b;
    const float scale = 1.0f / sqrtf((float)kEncHeadDim);
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
        for (int j = 0; j < 4; j++) o[n][j] = 0.f;

    for (int blk = 0; blk < n_blocks; blk++) {
        const int buf = blk & 1;
        if (blk + 1 < n_blocks) {
            load_kv(blk + 1, buf ^ 1);
            cp_async_commit();
        }
        const int kbase = k_lo + blk * kEaKeys;
        // ---- S = Q K^T (16 x 64 per warp) ----
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[n][j] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {   // pairs of 8-key tiles
                uint32_t b0, b1, b2, b3;
                const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int dim = ks * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(su32(sK[buf] + key * kEaPitch + dim), b0, b1, b2, b3);
                mma_f16_16816(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
                mma_f16_16816(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
            }
        }
        // ---- mask (causal + window of the row's own position), online softmax ----
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int kp = kbase + n * 8 + 2 * q4 + (j & 1);
                const int pq = (j < 2) ? pos_a : pos_b;
                const bool valid = kp <= pq && kp >= pq - (kEncWindow - 1);
                const float v = valid ? s[n][j] * scale : -INFINITY;
                s[n][j] = v;
                if (j < 2) mx_a = fmaxf(mx_a, v);
                else mx_b = fmaxf(mx_b, v);
            }
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float base_a = (mn_a == -INFINITY) ? 0.f : mn_a;
        const float base_b = (mn_b == -INFINITY) ? 0.f : mn_b;
        const float c_a = expf(m_a - base_a), c_b = expf(m_b - base_b);   // 0 when m was -inf
        m_a = mn_a;
        m_b = mn_b;
        float rs_a = 0.f, rs_b = 0.f;
        uint32_t pa[4][4];   // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const float e0 = expf(s[n][0] - base_a), e1 = expf(s[n][1] - base_a);
            const float e2 = expf(s[n][2] - base_b), e3 = expf(s[n][3] - base_b);
            rs_a += e0 + e1;
            rs_b += e2 + e3;
            // C fragment of keys 8n..8n+7 -> A fragment of k-step n/2 (regs 0,1 or 2,3)
            pa[n >> 1][(n & 1) * 2 + 0] = pack_half2(e0, e1);
            pa[n >> 1][(n & 1) * 2 + 1] = pack_half2(e2, e3);
        }
        rs_a += __shfl_xor_sync(0xffffffffu, rs_a, 1);
        rs_a += __shfl_xor_sync(0xffffffffu, rs_a, 2);
        rs_b += __shfl_xor_sync(0xffffffffu, rs_b, 1);
        rs_b += __shfl_xor_sync(0xffffffffu, rs_b, 2);
        l_a = l_a * c_a + rs_a;
        l_b = l_b * c_b + rs_b;
#pragma unroll
        for (int n = 0; n < 8; n++) {
            o[n][0] *= c_a;
            o[n][1] *= c_a;
            o[n][2] *= c_b;
            o[n][3] *= c_b;
        }
        // ---- O += P V ----
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            // A fragment register order: a0 (row g, k 0-7), a1 (row g+8, k 0-7),
            // a2 (row g, k 8-15), a3 (row g+8, k 8-15)
            const uint32_t A0 = pa[ks][0], A1 = pa[ks][1], A2 = pa[ks][2], A3 = pa[ks][3];
#pragma unroll
            for (int np = 0; np < 4; np++) {   // pairs of 8-dim tiles
                uint32_t b0, b1, b2, b3;
                const int key = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int dim = np * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(su32(sV[buf] + key * kEaPitch + dim), b0, b1, b2, b3);
                mma_f16_16816(o[2 * np], A0, A1, A2, A3, b0, b1);
                mma_f16_16816(o[2 * np + 1], A0, A1, A2, A3, b2, b3);
            }
        }
        cp_async_wait<0>();
        __syncthreads();
    }

    // ---- O / l -> fp16 or bf16 (the wo GEMM's A operand) ----
    const float ia = (l_a > 0.f) ? 1.0f / l_a : 0.f, ib = (l_b > 0.f) ? 1.0f / l_b : 0.f;
#pragma unroll
    for (int n = 0; n < 8; n++) {
        const int col = head * kEncHeadDim + n * 8 + 2 * q4;
        if (row_a < M) {
            uint16_t *dst = p.out + (size_t)row_a * kEncQkv + col;
            *reinterpret_cast<uint32_t *>(dst) = p.f16 ? pack_half2(o[n][0] * ia, o[n][1] * ia)
                                                       : (bf16_bits_rn(o[n][0] * ia) | (bf16_bits_rn(o[n][1] * ia) << 16));
        }
        if (row_b < M) {
            uint16_t *dst = p.out + (size_t)row_b * kEncQkv + col;
            *reinterpret_cast<uint32_t *>(dst) = p.f16 ? pack_half2(o[n][2] * ib, o[n][3] * ib)
                                                       : (bf16_bits_rn(o[n][2] * ib) | (bf16_bits_rn(o[n][3] * ib) << 16));
        }
    }
}

cudaError_t launch_enc_attn(const EncAttnParams &p, cudaStream_t st, bool pdl) {
    if (p.M <= 0 || p.cap < p.M + kEncWindow - 1) return cudaErrorInvalidValue;
    const char *sel = getenv("VOX_CUDA_ENC_ATTN");   // "mma" forces the mma.sync kernel
    if (!(sel && strcmp(sel, "mma") == 0) && enc_attn_tc_supported(p)) return launch_enc_attn_tc(p, st, pdl);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.M + kEaRows - 1) / kEaRows, kEncHeads);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, enc_attn_kernel, p);
}

// Final RMSNorm of the encoder output, in place (voxtral_encoder.c:629).
__global__ void __launch_bounds__(256)
rows_rmsnorm_kernel(float *x, int M, int K, const float *w) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    float *xr = x + (size_t)warp * K;
    float ss = 0.f;
    for (int i = lane; i < K; i += 32) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)K + kNormEps);
    for (int i = lane; i < K; i += 32) xr[i] = xr[i] * inv * w[i];
}

// Per-chunk RoPE planes, once for all layers: tab[d][row] = cos and
// tab[32 + d][row] = sin of (pos0 + row) * inv_freq[d], the same angles and
// sincosf the q|k epilogue would otherwise evaluate per pair and per layer
// (vox_compute_rope_freqs, voxtral_kernels.c:488-503, on the device); or the
// host's table src[row][32] (cos, sin) transposed.
__global__ void __launch_bounds__(256)
enc_rope_table_kernel(float *tab, int ld, int M, const float *src, const int *pos0_dev, const float *inv_freq) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // row * 32 + d
    if (i >= M * (kEncHeadDim / 2)) return;
    const int row = i / (kEncHeadDim / 2), d = i % (kEncHeadDim / 2);
    float sn, cs;
    if (src) {
        cs = src[2 * i];
        sn = src[2 * i + 1];
    } else {
        sincosf((float)(*pos0_dev + row) * inv_freq[d], &sn, &cs);
    }
    tab[(size_t)d * ld + row] = cs;
    tab[(size_t)(kEncHeadDim / 2 + d) * ld + row] = sn;
}

cudaError_t launch_enc_rope_table(float *tab, int ld, int M, const float *src, const int *pos0_dev,
                                  const float *inv_freq, cudaStream_t st, bool pdl) {
    const int n = M * (kEncHeadDim / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, enc_rope_table_kernel, tab, ld, M, src, pos0_dev, inv_freq);
}

__global__ void __launch_bounds__(256)
enc_rope_table_segs_kernel(float *tab, int ld, int M, const EncSeg *segs, int n_segs, const float *inv_freq) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // row * 32 + d
    if (i >= M * (kEncHeadDim / 2)) return;
    const int row = i / (kEncHeadDim / 2), d = i % (kEncHeadDim / 2);
    int s = 0;
    while (s + 1 < n_segs && row >= segs[s + 1].row0) s++;
    float sn, cs;
    sincosf((float)(*segs[s].pos0_dev + (row - segs[s].row0)) * inv_freq[d], &sn, &cs);
    tab[(size_t)d * ld + row] = cs;
    tab[(size_t)(kEncHeadDim / 2 + d) * ld + row] = sn;
}

cudaError_t launch_enc_rope_table_segs(float *tab, int ld, int M, const EncSeg *segs, int n_segs,
                                       const float *inv_freq, cudaStream_t st, bool pdl) {
    const int n = M * (kEncHeadDim / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, enc_rope_table_segs_kernel, tab, ld, M, segs, n_segs, inv_freq);
}

__global__ void set_int_kernel(int *dst, int v) { *dst = v; }

cudaError_t launch_set_int(int *dst, int v, cudaStream_t st) {
    set_int_kernel<<<1, 1, 0, st>>>(dst, v);
    return cudaGetLastError();
}

cudaError_t launch_rows_rmsnorm(float *x, int M, int K, const float *w, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_rmsnorm_kernel, x, M, K, w);
}

}  // namespace vc
