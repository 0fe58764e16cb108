// vc_gemm_tc.cu - tcgen05 tensor-core GEMM for the encoder chunk, the adapter
// and M > 8 matmuls: C[M, N] = A[M, K] . W[N, K]^T with bf16 A and W (both
// K-major, row-major as stored), fp32 accumulation in TMEM, fused epilogues.
//
// One CTA computes one 128 x BN output tile:
//   warp 0 (one thread)  TMA producer: 128x64 A and BNx64 W tiles, 128-byte
//                        swizzle, into a STAGES-deep shared-memory ring
//   warp 1 (one thread)  tcgen05.mma issuer (M=128, N=BN, K=16, cta_group::1);
//                        tcgen05.commit releases ring stages and finally
//                        signals the epilogue; warp 1 also owns the TMEM
//                        allocation (BN fp32 columns x 128 lanes)
//   warps 2-5            epilogue: tcgen05.ld of their 32-lane quarter of the
//                        accumulator, bias / residual / activation / RoPE,
//                        stores to global memory
// Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA sets
// the launch's error word and exits after a grace period for in-flight copies.
#include "vc_common.cuh"
#include "vc_internal.h"
#include "vc_tc.cuh"

#include <cuda_fp16.h>
#include <math.h>
#include <stdlib.h>

#include <mutex>
#include <unordered_map>

namespace vc {

using namespace tc;

constexpr int kTcThreads = 192;
constexpr int kBM = 128;
constexpr int kBK = 64;                     // one 128-byte swizzle row of bf16
constexpr uint64_t kTcWaitNs = 2000000000ull;

template <int BN>
struct TcCfg {
    static constexpr int kStages = (BN >= 256) ? 4 : 6;
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kSmem = kStages * (kABytes + kBBytes) + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float gelu_tanh(float v) {
    // tanh-approximated GELU (vox_gelu, voxtral_kernels.c:376-384)
    const float x3 = v * v * v;
    const float inner = 0.7978845608028654f * (v + 0.044715f * x3);
    return 0.5f * v * (1.0f + tanhf(inner));
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const TcGemmParams p) {
    using Cfg = TcCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sA = smem;
    unsigned char *sB = smem + S * Cfg::kABytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + S * Cfg::kBBytes);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    const int KB = (p.K + kBK - 1) / kBK;
    const uint64_t deadline = globaltimer() + kTcWaitNs;
    bool ok = true;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            uint64_t pol_a, pol_b;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_a));
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_b));
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % S;
                if (kb >= S && !mbar_wait(&empty[s], (uint32_t)((kb / S) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(&full[s], Cfg::kABytes + Cfg::kBBytes);
                tma_load_2d(sA + s * Cfg::kABytes, &tmA, kb * kBK, m0, &full[s], pol_a);
                tma_load_2d(sB + s * Cfg::kBBytes, &tmB, kb * kBK, n0, &full[s], pol_b);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kBM, BN);
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % S;
                if (!mbar_wait(&full[s], (uint32_t)(kb / S) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t a0 = smem_desc_sw128(sA + s * Cfg::kABytes);
                const uint64_t b0 = smem_desc_sw128(sB + s * Cfg::kBBytes);
#pragma unroll
                for (int k = 0; k < kBK / 16; k++)   // +32 bytes (2 x 16) per K=16 step
                    tc_mma_bf16(tmem, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
                tc_commit(&empty[s]);
            }
            if (ok) tc_commit(tfull);
        }
    } else {
        // ---- epilogue: warp quarter q owns TMEM lanes 32q..32q+31 = tile rows ----
        const bool got = mbar_wait(tfull, 0u, deadline);
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
        } else {
            tc_fence_after();
            const int q = warp & 3;
            const int row = m0 + 32 * q + lane;
            const bool rv = row < p.M;
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
                const int col0 = n0 + c;
                if (!rv || col0 >= p.N) continue;
                if constexpr (EPI == TC_STORE || EPI == TC_RESID) {
                    float *o = p.out + (size_t)row * p.ldo + col0;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (col0 + j >= p.N) break;
                        float x = v[j];
                        if (p.bias) x += p.bias[col0 + j];
                        if constexpr (EPI == TC_RESID) x += o[j];
                        if (p.act == 1) x = gelu_tanh(x);
                        if (p.out_bf16) p.out_bf16[(size_t)row * p.ldo_bf16 + col0 + j] = (uint16_t)bf16_bits_rn(x);
                        else o[j] = x;
                    }
                } else if constexpr (EPI == TC_SWIGLU) {
                    // columns (2i, 2i+1) = (gate_i, up_i) -> h_i = silu(g) * u
                    // (voxtral_kernels.c:369-374, then :34-36), bf16 for the next GEMM
                    uint16_t *o = p.out_bf16 + (size_t)row * p.ldo_bf16 + (col0 >> 1);
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const float g = v[j], u = v[j + 1];
                        const float sg = g / (1.0f + expf(-g));
                        o[j >> 1] = (uint16_t)bf16_bits_rn(sg * u);
                    }
                } else if constexpr (EPI == TC_QKV_ENC) {
                    // [0,2048): q (+bias, RoPE), [2048,4096): k (RoPE), [4096,6144): v (+bias)
                    // (voxtral_encoder.c:542-559); k and v go to the ring slot of the row
                    const int pos = (p.pos0_dev ? *p.pos0_dev : p.pos0) + row;
                    const size_t slot = (size_t)(pos % p.cap);
                    const float *cs = p.rope ? p.rope + (size_t)row * kEncHeadDim : nullptr;
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const int col = col0 + j;
                        float a = v[j], b = v[j + 1];
                        if (col < 2 * kEncQkv) {
                            if (col < kEncQkv && p.bias) {
                                a += p.bias[col];
                                b += p.bias[col + 1];
                            }
                            const int d = (col & (kEncHeadDim - 1)) >> 1;
                            float c0, s0;
                            if (cs) {
                                c0 = cs[2 * d];
                                s0 = cs[2 * d + 1];
                            } else {   // angle = pos * inv_freq exactly as the host formula
                                sincosf((float)pos * p.inv_freq[d], &s0, &c0);
                            }
                            const float oa = __fsub_rn(__fmul_rn(a, c0), __fmul_rn(b, s0));
                            const float ob = __fadd_rn(__fmul_rn(a, s0), __fmul_rn(b, c0));
                            if (col < kEncQkv) {
                                __half2 *qo = reinterpret_cast<__half2 *>(p.q_out + (size_t)row * kEncQkv + col);
                                static_assert(sizeof(__half2) == 4, "half2");
                                *qo = __floats2half2_rn(oa, ob);
                            } else {
                                __half2 *ko = reinterpret_cast<__half2 *>(p.k_ring + slot * kEncQkv + (col - kEncQkv));
                                *ko = __floats2half2_rn(oa, ob);
                            }
                        } else {
                            const int cv = col - 2 * kEncQkv;
                            if (p.bias2) {
                                a += p.bias2[cv];
                                b += p.bias2[cv + 1];
                            }
                            __half2 *vo = reinterpret_cast<__half2 *>(p.v_ring + slot * kEncQkv + cv);
                            *vo = __floats2half2_rn(a, b);
                        }
                    }
                }
            }
        }
    }

    if (!__all_sync(0xffffffffu, ok)) ok = false;
    if (!ok) {
        if (lane == 0) atomicExch(p.err, 1u);
        const uint64_t grace = globaltimer() + 10000000ull;   // let in-flight copies / MMAs land
        while (globaltimer() < grace) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launches
// ---------------------------------------------------------------------------

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// bf16 row-major [rows, cols] (cols contiguous), box [box_rows, 64], 128B swizzle
bool make_map(CUtensorMap *m, const void *ptr, int rows, int cols, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
cudaError_t launch_bn(const TcGemmParams &p, const void *A, const void *W, cudaStream_t st, bool pdl) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, A, p.M, p.K, kBM) || !make_map(&mb, W, p.N, p.K, BN)) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             TcCfg<BN>::kSmem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.N + BN - 1) / BN, (p.M + kBM - 1) / kBM);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = TcCfg<BN>::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr1[1];
    attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr1[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr1;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, EPI>, ma, mb, p);
}

}  // namespace

// Tile width: enough CTAs to cover the SMs, widest tile otherwise.
int tc_gemm_bn(int M, int N) {
    const int mt = (M + kBM - 1) / kBM;
    if (N % 256 == 0 && mt * (N / 256) >= 148) return 256;
    if (mt * ((N + 127) / 128) >= 100) return 128;
    return 64;
}

cudaError_t launch_tc_gemm(int epi, const TcGemmParams &p, const void *A, const void *W, cudaStream_t st,
                           bool pdl, int bn) {
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.K % 8 != 0 || !p.err || ((uintptr_t)A & 15) || ((uintptr_t)W & 15))
        return cudaErrorInvalidValue;
    if (epi == TC_SWIGLU && (p.N % 32 != 0)) return cudaErrorInvalidValue;
    if (bn == 0) bn = tc_gemm_bn(p.M, p.N);
#define VC_TC_CASE(BN)                                                             \
    if (bn == BN) {                                                                \
        switch (epi) {                                                             \
            case TC_STORE: return launch_bn<BN, TC_STORE>(p, A, W, st, pdl);       \
            case TC_RESID: return launch_bn<BN, TC_RESID>(p, A, W, st, pdl);       \
            case TC_SWIGLU: return launch_bn<BN, TC_SWIGLU>(p, A, W, st, pdl);     \
            case TC_QKV_ENC: return launch_bn<BN, TC_QKV_ENC>(p, A, W, st, pdl);   \
        }                                                                          \
    }
    VC_TC_CASE(64)
    VC_TC_CASE(128)
    VC_TC_CASE(256)
#undef VC_TC_CASE
    return cudaErrorInvalidValue;
}

// fp32 [M, K] (row stride ld) -> bf16 [M, K], optionally RMS-normalised with
// weights w (voxtral_kernels.c:346-363).  One warp per row.
__global__ void __launch_bounds__(256)
rows_to_bf16_kernel(const float *x, int M, int K, int ld, const float *w, uint16_t *out) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float *xr = x + (size_t)warp * ld;
    float inv = 1.0f;
    if (w) {
        float ss = 0.f;
        for (int i = lane; i < K; i += 32) ss = fmaf(xr[i], xr[i], ss);
        ss = warp_sum(ss);
        inv = 1.0f / sqrtf(ss / (float)K + kNormEps);
    }
    uint16_t *o = out + (size_t)warp * K;
    for (int i = lane; i < K; i += 32) {
        const float v = w ? xr[i] * inv * w[i] : xr[i];
        o[i] = (uint16_t)bf16_bits_rn(v);
    }
}

cudaError_t launch_rows_to_bf16(const float *x, int M, int K, int ld, const float *w, uint16_t *out,
                                cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_to_bf16_kernel, x, M, K, ld, w, out);
}

}  // namespace vc
