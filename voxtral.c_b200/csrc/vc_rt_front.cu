// vc_rt_front.cu - the C ABI of voxtral_cuda.h, part 4: the audio front
// end: the conv stem with its streaming state, and the log-mel context and
// one-shot spectrogram.
#include "vc_runtime.h"

#include <map>

using namespace vc;
using namespace vc::rt;

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

