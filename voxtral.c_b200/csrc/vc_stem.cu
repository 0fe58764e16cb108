// vc_stem.cu - the encoder's conv stem on the device (stream_conv_stem,
// voxtral.c:487-665, over vox_causal_conv1d, voxtral_kernels.c:293-340):
// conv0 (128 -> 1280, kernel 3, stride 1) and conv1 (1280 -> 1280, kernel 3,
// stride 2), each followed by tanh-GELU (voxtral_kernels.c:376-384), as a
// device im2col into fp16 rows plus the tcgen05 GEMM with a bias + GELU
// epilogue.  The reference's weight layout [cout][cin][3] flattened is the
// GEMM's K-major W with K index ic * 3 + k, so the weights need no reordering.
//
// Streaming state between chunks, as the reference keeps it: the last two
// mel frames (after a one-frame chunk the older one is zero, as the
// reference rebuilds its tail, voxtral.c:519-524, 551-556) and the last two
// conv0 outputs by global frame index.  A chunk of n frames after T frames
// yields conv1 rows floor(T / 2) .. floor((T + n) / 2) - 1.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <cuda_fp16.h>

namespace vc {

constexpr int kStemMel = 128;                  // mel bins
constexpr int kStemK0 = 3 * kStemMel;          // conv0 GEMM K
constexpr int kStemK1 = 3 * kEncDim;           // conv1 GEMM K

__device__ __forceinline__ uint16_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// a0[r][ic * 3 + k] = mel frame f0 + r - 2 + k, bin ic: ext = [hist(2) | new(n)]
__global__ void __launch_bounds__(256)
stem_im2col0_kernel(const float *mel_new, const float *mel_hist, int n, uint16_t *a0) {
    const size_t total = (size_t)n * kStemK0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kStemK0), kk = (int)(i % kStemK0);
        const int ic = kk / 3, e = r + kk % 3;
        const float v = e < 2 ? mel_hist[e * kStemMel + ic] : mel_new[(size_t)(e - 2) * kStemMel + ic];
        a0[i] = f16_bits(v);
    }
}

// a1[r][ic * 3 + k] = conv0 output of global frame 2 (u0 + r) - 1 + k (zero
// before frame 0): frames f0 - 2, f0 - 1 from hist, frames >= f0 from c0_new
__global__ void __launch_bounds__(256)
stem_im2col1_kernel(const uint16_t *c0_new, const uint16_t *c0_hist, long long f0, long long u0, int n_out,
                    uint16_t *a1) {
    const size_t total = (size_t)n_out * kStemK1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kStemK1), kk = (int)(i % kStemK1);
        const int ic = kk / 3;
        const long long g = 2 * (u0 + r) - 1 + kk % 3;
        uint16_t v = 0;
        if (g >= f0) v = c0_new[(size_t)(g - f0) * kEncDim + ic];
        else if (g >= 0) v = c0_hist[(size_t)(g - (f0 - 2)) * kEncDim + ic];
        a1[i] = v;
    }
}

// The state after a chunk of n >= 1 frames: thread = channel (reads before
// writes per channel, so the in-place update has no race).
__global__ void __launch_bounds__(256)
stem_state_kernel(const float *mel_new, int n, float *mel_hist, const uint16_t *c0_new, uint16_t *c0_hist) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < kStemMel) {
        const float m1 = mel_new[(size_t)(n - 1) * kStemMel + c];
        const float m0 = n >= 2 ? mel_new[(size_t)(n - 2) * kStemMel + c] : 0.f;   // the reference's [0, frame]
        mel_hist[c] = m0;
        mel_hist[kStemMel + c] = m1;
    }
    if (c < kEncDim) {
        const uint16_t h1 = c0_new[(size_t)(n - 1) * kEncDim + c];
        const uint16_t h0 = n >= 2 ? c0_new[(size_t)(n - 2) * kEncDim + c] : c0_hist[kEncDim + c];
        c0_hist[c] = h0;
        c0_hist[kEncDim + c] = h1;
    }
}

static unsigned stem_blocks(size_t total) {
    const size_t b = (total + 255) / 256;
    return (unsigned)(b < 8192 ? b : 8192);
}

cudaError_t launch_stem_im2col0(const float *mel_new, const float *mel_hist, int n, uint16_t *a0, cudaStream_t st) {
    stem_im2col0_kernel<<<stem_blocks((size_t)n * kStemK0), 256, 0, st>>>(mel_new, mel_hist, n, a0);
    return cudaGetLastError();
}

cudaError_t launch_stem_im2col1(const uint16_t *c0_new, const uint16_t *c0_hist, long long f0, long long u0,
                                int n_out, uint16_t *a1, cudaStream_t st) {
    stem_im2col1_kernel<<<stem_blocks((size_t)n_out * kStemK1), 256, 0, st>>>(c0_new, c0_hist, f0, u0, n_out, a1);
    return cudaGetLastError();
}

cudaError_t launch_stem_state(const float *mel_new, int n, float *mel_hist, const uint16_t *c0_new,
                              uint16_t *c0_hist, cudaStream_t st) {
    stem_state_kernel<<<(kEncDim + 255) / 256, 256, 0, st>>>(mel_new, n, mel_hist, c0_new, c0_hist);
    return cudaGetLastError();
}

// fp32 -> fp16 (the conv weights, once at creation)
__global__ void __launch_bounds__(256) f32_to_f16_kernel(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = f16_bits(src[i]);
}

cudaError_t launch_f32_to_f16(const float *src, uint16_t *dst, size_t n, cudaStream_t st) {
    f32_to_f16_kernel<<<stem_blocks(n), 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

}  // namespace vc

