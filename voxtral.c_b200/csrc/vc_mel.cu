// vc_mel.cu - the log-mel front end on the device (voxtral_audio.c): the
// incremental context's frames (mel_compute_available, voxtral_audio.c:
// 430-482) and the one-shot spectrogram's (vox_mel_spectrogram, :290-395).
//
// Frame t covers samples [160 t, 160 t + 400) of the padded signal: periodic
// Hann window, direct 201-bin DFT power (the reference's tabulated cos / sin of
// the fp32 angle 2 pi k n / 400, not an FFT, so the rounding of the tables
// matches), 128 Slaney mel filters, log10 with the 1e-10 floor and the
// (1.5 - 8) clamp, then (v + 4) / 4.  fp32 on the CUDA cores: a frame is 0.37
// MFLOP, a 2 s chunk (200 frames) 75 MFLOP, far below any tensor-core payoff,
// and fp32 keeps the weak high bands' relative error at the reference's level.
//
// One CTA computes kMelFrames frames: the windowed frames sit in shared
// memory, threads 0..200 accumulate the cos sums and 256..456 the sin sums of
// one bin for every frame (the [400][201] tables are read once per CTA,
// coalesced along the bin, L2-resident), then thread (f, m) applies mel
// filter m to frame f's power.
//
// Samples are addressed by their logical index p in the padded stream: p below
// `pad` (the context's leading zeros) reads 0, else ring[(p - pad) & mask]
// (mask = -1: a linear buffer).
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>

namespace vc {

constexpr int kMelThreads = 512;

__device__ __forceinline__ float mel_sample(const float *ring, long long mask, long long pad, long long p) {
    return p < pad ? 0.f : __ldg(ring + ((p - pad) & mask));
}

__global__ void __launch_bounds__(kMelThreads)
mel_frames_kernel(const float *ring, long long mask, long long pad, long long t0, int n_frames,
                  const float *win, const float *cos_t, const float *sin_t, const float *filt_t,
                  float *out) {
    __shared__ float w[kMelFrames][kMelWin];
    __shared__ float pw[2][kMelFrames][kMelFreq];
    const int tid = threadIdx.x;
    const int f0 = blockIdx.x * kMelFrames;
    for (int i = tid; i < kMelFrames * kMelWin; i += kMelThreads) {
        const int f = i / kMelWin, n = i - f * kMelWin;
        float v = 0.f;
        if (f0 + f < n_frames) v = mel_sample(ring, mask, pad, (t0 + f0 + f) * kMelHop + n) * __ldg(win + n);
        w[f][n] = v;
    }
    __syncthreads();
    // direct DFT: re (threads 0..200) and im (256..456) of one bin per frame
    const int half = tid >> 8, k = tid & 255;
    if (k < kMelFreq) {
        const float *tab = (half ? sin_t : cos_t) + k;
        float acc[kMelFrames];
#pragma unroll
        for (int f = 0; f < kMelFrames; f++) acc[f] = 0.f;
#pragma unroll 8
        for (int n = 0; n < kMelWin; n++) {
            const float c = __ldg(tab + n * kMelFreq);
#pragma unroll
            for (int f = 0; f < kMelFrames; f++) acc[f] = fmaf(w[f][n], c, acc[f]);
        }
#pragma unroll
        for (int f = 0; f < kMelFrames; f++) pw[half][f][k] = acc[f] * acc[f];
    }
    __syncthreads();
    // mel filters + log: thread (f, m)
    const int f = tid >> 7, m = tid & 127;
    if (f < kMelFrames && f0 + f < n_frames) {
        float s = 0.f;
        for (int q = 0; q < kMelFreq; q++) s = fmaf(__ldg(filt_t + q * kMelBins + m), pw[0][f][q] + pw[1][f][q], s);
        float v = log10f(fmaxf(s, 1e-10f));
        v = fmaxf(v, kMelLogMax - 8.f);
        out[(size_t)(f0 + f) * kMelBins + m] = (v + 4.f) * 0.25f;
    }
}

cudaError_t launch_mel_frames(const float *ring, long long mask, long long pad, long long t0, int n_frames,
                              const MelTables &t, float *out, cudaStream_t st) {
    if (n_frames <= 0) return cudaSuccess;
    const int grid = (n_frames + kMelFrames - 1) / kMelFrames;
    mel_frames_kernel<<<grid, kMelThreads, 0, st>>>(ring, mask, pad, t0, n_frames, t.win, t.cos_t, t.sin_t,
                                                    t.filt_t, out);
    return cudaGetLastError();
}

// dst[i] = the sample at logical index src0 - i (0 below `pad`), i < n: the
// reflection appended by vox_mel_finish (voxtral_audio.c:583-590)
__global__ void mel_reflect_kernel(const float *ring, long long mask, long long pad, long long src0, int n,
                                   float *dst) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const long long p = src0 - i;
        dst[i] = p < 0 ? 0.f : mel_sample(ring, mask, pad, p);
    }
}

cudaError_t launch_mel_reflect(const float *ring, long long mask, long long pad, long long src0, int n,
                               float *dst, cudaStream_t st) {
    mel_reflect_kernel<<<(n + 255) / 256, 256, 0, st>>>(ring, mask, pad, src0, n, dst);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// host tables (built once per context, uploaded)
// ---------------------------------------------------------------------------

namespace {

// Slaney mel scale: 3 mel per 200 Hz below 1 kHz, then 27 mel per factor 6.4
// (voxtral_audio.c:220-242)
float hz_to_mel(float hz) {
    if (hz >= 1000.0f) return 15.0f + logf(hz / 1000.0f) * (27.0f / logf(6.4f));
    return 3.0f * hz / 200.0f;
}

float mel_to_hz(float mel) {
    if (mel >= 15.0f) return 1000.0f * expf((logf(6.4f) / 27.0f) * (mel - 15.0f));
    return 200.0f * mel / 3.0f;
}

}  // namespace

void mel_host_tables(float *win, float *cos_t, float *sin_t, float *filt_t) {
    const float two_pi = 2.0f * 3.14159265358979323846f;
    for (int i = 0; i < kMelWin; i++) win[i] = 0.5f * (1.0f - cosf(two_pi * (float)i / (float)kMelWin));
    // [n][k] (bin fastest): the angle as the reference evaluates it, in fp32
    for (int k = 0; k < kMelFreq; k++)
        for (int n = 0; n < kMelWin; n++) {
            const float a = two_pi * (float)k * (float)n / (float)kMelWin;
            cos_t[n * kMelFreq + k] = cosf(a);
            sin_t[n * kMelFreq + k] = sinf(a);
        }
    // triangular filters between consecutive edges, area-normalised by
    // 2 / (upper - lower edge) (voxtral_audio.c:245-283); stored [bin][mel]
    float edges[kMelBins + 2];
    const float lo = hz_to_mel(0.0f), hi = hz_to_mel(kMelRate / 2.0f);
    for (int i = 0; i < kMelBins + 2; i++) edges[i] = mel_to_hz(lo + (hi - lo) * (float)i / (float)(kMelBins + 1));
    for (int m = 0; m < kMelBins; m++) {
        float dl = edges[m + 1] - edges[m], du = edges[m + 2] - edges[m + 1];
        if (dl == 0.0f) dl = 1e-6f;
        if (du == 0.0f) du = 1e-6f;
        const float norm = 2.0f / (edges[m + 2] - edges[m]);
        for (int q = 0; q < kMelFreq; q++) {
            const float hz = (float)q * ((float)kMelRate / 2.0f) / (float)(kMelFreq - 1);
            const float rise = (hz - edges[m]) / dl, fall = (edges[m + 2] - hz) / du;
            float v = rise < fall ? rise : fall;
            if (v < 0.0f) v = 0.0f;
            filt_t[q * kMelBins + m] = v * norm;
        }
    }
}

}  // namespace vc
