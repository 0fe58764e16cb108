"""Log-mel spectrogram oracle: a numpy restatement of the reference's audio
front end (voxtral_audio.c).  Test infrastructure only: tests/, smoke() and
bench.py's CPU baseline use it as the checker, the product never does.

Pinned against the reference itself: tests/golden/mel.npz holds the output
of the reference's own vox_mel_ctx_* / vox_mel_spectrogram (compiled from
its sources into oracle/_ref) on seeded synthetic audio.

Constants (voxtral_audio.c:31-37): 16 kHz, 128 mel bins, hop 160, window and
DFT length 400 (201 frequency bins), log-mel ceiling 1.5.
"""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000
N_MEL = 128
HOP = 160
WIN = 400
N_FFT = 400
N_FREQ = N_FFT // 2 + 1
LOG_MEL_MAX = 1.5
CENTER_PAD = 200            # center=True padding (N_FFT / 2)

f32 = np.float32


def hz_to_mel(hz):
    """Slaney mel scale: linear below 1 kHz (3 mel per 200 Hz), logarithmic
    above with 27 mel per factor 6.4 (voxtral_audio.c:220-230)."""
    hz = f32(hz)
    if hz >= f32(1000.0):
        return f32(15.0) + f32(np.log(hz / f32(1000.0))) * (f32(27.0) / f32(np.log(f32(6.4))))
    return f32(3.0) * hz / f32(200.0)


def mel_to_hz(mel):
    """Inverse of hz_to_mel (voxtral_audio.c:232-242)."""
    mel = f32(mel)
    if mel >= f32(15.0):
        return f32(1000.0) * f32(np.exp((f32(np.log(f32(6.4))) / f32(27.0)) * (mel - f32(15.0))))
    return f32(200.0) * mel / f32(3.0)


def mel_filters():
    """[128, 201] triangular Slaney-normalised filters over the FFT bin
    centres 0..8000 Hz (voxtral_audio.c:245-283)."""
    fft_hz = np.array([f32(i) * (f32(SAMPLE_RATE / 2.0) / f32(N_FREQ - 1)) for i in range(N_FREQ)], f32)
    lo, hi = hz_to_mel(0.0), hz_to_mel(SAMPLE_RATE / 2.0)
    edges = np.array([mel_to_hz(lo + (hi - lo) * f32(i) / f32(N_MEL + 1)) for i in range(N_MEL + 2)], f32)
    width = np.diff(edges).astype(f32)
    width[width == 0] = f32(1e-6)
    out = np.zeros((N_MEL, N_FREQ), f32)
    for m in range(N_MEL):
        rise = (fft_hz - edges[m]) / width[m]
        fall = (edges[m + 2] - fft_hz) / width[m + 1]
        tri = np.maximum(np.minimum(rise, fall), f32(0.0)).astype(f32)
        out[m] = tri * (f32(2.0) / (edges[m + 2] - edges[m]))
    return out


def hann_periodic():
    """Periodic Hann window of length 400 (voxtral_audio.c:329-333)."""
    i = np.arange(WIN, dtype=f32)
    return (f32(0.5) * (f32(1.0) - np.cos(f32(2.0) * f32(np.pi) * i / f32(WIN)))).astype(f32)


def dft_tables():
    """cos / sin of the fp32 angle 2 pi k n / 400 as the reference tabulates
    it (voxtral_audio.c:335-344): [201, 400] each."""
    k = np.arange(N_FREQ, dtype=f32)[:, None]
    n = np.arange(N_FFT, dtype=f32)[None, :]
    ang = (f32(2.0) * f32(np.pi)) * k * n / f32(N_FFT)
    return np.cos(ang).astype(f32), np.sin(ang).astype(f32)


_TABLES = None


def _tables():
    global _TABLES
    if _TABLES is None:
        c, s = dft_tables()
        _TABLES = (hann_periodic(), c, s, mel_filters())
    return _TABLES


def frames_to_mel(padded, t0, t1):
    """Log-mel rows for frames t0..t1-1 of a padded signal: window, direct
    DFT power, mel filters, log10 with the 1e-10 floor and the
    (LOG_MEL_MAX - 8) clamp, then (v + 4) / 4 (voxtral_audio.c:353-386)."""
    win, c, s, filt = _tables()
    if t1 <= t0:
        return np.zeros((0, N_MEL), f32)
    idx = (np.arange(t0, t1)[:, None] * HOP + np.arange(N_FFT)[None, :])
    w = padded[idx].astype(f32) * win[None, :]
    re = w @ c.T
    im = w @ s.T
    power = (re * re + im * im).astype(f32)
    mel = power @ filt.T
    mel = np.log10(np.maximum(mel, f32(1e-10))).astype(f32)
    mel = np.maximum(mel, f32(LOG_MEL_MAX - 8.0))
    return ((mel + f32(4.0)) / f32(4.0)).astype(f32)


class StreamingMel:
    """The incremental context (vox_mel_ctx_init / _feed / _finish,
    voxtral_audio.c:392-612): left_pad_samples + 200 zeros first, every
    frame whose 400-sample window fits is computed as samples arrive; finish
    appends right_pad zeros and a 200-sample reflection of the signal before
    them, then drops the last frame."""

    def __init__(self, left_pad_samples):
        self.samples = np.zeros(CENTER_PAD + left_pad_samples, f32)
        self.frames = 0

    def _compute(self):
        n = self.samples.size
        t1 = (n - N_FFT) // HOP + 1 if n >= N_FFT else 0
        out = frames_to_mel(self.samples, self.frames, t1)
        self.frames = max(self.frames, t1)
        return out

    def feed(self, x):
        x = np.asarray(x, f32)
        if x.size == 0:
            return np.zeros((0, N_MEL), f32)
        self.samples = np.concatenate([self.samples, x])
        return self._compute()

    def finish(self, right_pad_samples=0):
        real_end = self.samples.size
        ext = [self.samples, np.zeros(right_pad_samples, f32)]
        src = real_end - 2 - np.arange(CENTER_PAD)
        refl = np.where(src >= 0, self.samples[np.maximum(src, 0)], f32(0.0)).astype(f32)
        self.samples = np.concatenate(ext + [refl])
        out = self._compute()
        if self.frames > 0:          # the last frame is dropped (vLLM convention)
            self.frames -= 1
            out = out[:-1] if out.shape[0] else out
        return out


def mel_spectrogram(x):
    """The one-shot form (vox_mel_spectrogram, voxtral_audio.c:290-395):
    reflect padding of 200 on both sides, the last frame dropped; None when
    no frame remains."""
    x = np.asarray(x, f32)
    n = x.size
    left = np.array([x[CENTER_PAD - i] if CENTER_PAD - i < n else 0.0 for i in range(CENTER_PAD)], f32)
    right = np.array([x[n - 2 - i] if n - 2 - i >= 0 else 0.0 for i in range(CENTER_PAD)], f32)
    padded = np.concatenate([left, x, right])
    total = (padded.size - N_FFT) // HOP + 1
    if total - 1 <= 0:
        return None
    return frames_to_mel(padded, 0, total - 1)
