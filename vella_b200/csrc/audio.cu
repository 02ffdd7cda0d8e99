// Whisper's log-mel input features on the device.
//
// Replaces WhisperAudio.encoderFeatures / logMelSpectrogram (Worker/Sources/MLXAudioSTT/
// Whisper/WhisperAudio.swift:7-93) and MLXAudioCore.melFilters (Worker/Sources/MLXAudioCore/
// DSP.swift:44-135, Slaney scale and norm): each window is padded with zeros or trimmed to
// 480000 samples (30 s at 16 kHz), reflect-padded by 200 samples on each side, cut into
// frames of 400 samples every 160 (3001 frames, the last dropped as torch.stft(center=True)
// gives 3000), multiplied by the periodic Hann window 0.5 (1 - cos(2 pi n / 400)), turned
// into the power spectrum of its 201 real-DFT bins, projected on the mel filterbank,
// log10(max(., 1e-10)), floored at the window's maximum - 8, and mapped to (x + 4) / 4.
//
// Two kernels per call.  mel_frames_kernel: one CTA per 32 frames of one window; the
// windowed frames sit in shared memory (rows of 401 floats, so the 32 lanes of a warp, one
// frame each, read different banks); each warp takes every 8th DFT bin, its lanes sharing
// the twiddle index (k n) mod 400 so the cos/sin table read is a broadcast; the power rows
// then meet the filterbank (read from L2) and the log10 values are written [mel][frame], a
// warp per mel row and 32 consecutive frames.  mel_floor_kernel: one CTA per window reduces
// the window's maximum and maps every value (no atomics, no scratch).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <algorithm>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace vella {
namespace {

constexpr int kNfft = 400, kBins = kNfft / 2 + 1, kHop = 160, kPad = kNfft / 2;
constexpr int64_t kWindow = 480000;  // 30 s at 16 kHz
constexpr int kFrames = 3000;
constexpr int kFramesPerCta = 32, kFrameStride = kNfft + 1, kMelThreads = 256;
constexpr int kPowStride = kBins + 2;  // odd: lanes reading one bin of 32 frames hit 32 banks

// Tables of one mel bin count: filterbank [201][n_mels], cos and sin of 2 pi j / 400, Hann window.
struct MelTables {
  float* filt = nullptr;
  float* cosv = nullptr;
  float* sinv = nullptr;
  float* hann = nullptr;
};

// The reference's filterbank, in fp32 as it computes it (DSP.swift:44-135, Slaney mel scale:
// linear below 1 kHz at 200/3 Hz per mel, logarithmic above with step ln(6.4)/27; triangles
// rising on [low, center), falling on [center, high]; Slaney area norm 2 / (high - low)).
std::vector<float> slaney_filters(int n_mels) {
  const float sr = 16000.0f, fmin = 0.0f, fmax = sr / 2.0f;
  const float f_sp = 200.0f / 3.0f, min_log_hz = 1000.0f, min_log_mel = (min_log_hz - fmin) / f_sp;
  const float log_step = std::log(6.4f) / 27.0f;
  auto hz_to_mel = [&](float f) { return f < min_log_hz ? (f - fmin) / f_sp : min_log_mel + std::log(f / min_log_hz) / log_step; };
  auto mel_to_hz = [&](float m) { return m < min_log_mel ? fmin + f_sp * m : min_log_hz * std::exp(log_step * (m - min_log_mel)); };
  const float m0 = hz_to_mel(fmin), m1 = hz_to_mel(fmax);
  std::vector<float> pts((size_t)n_mels + 2);
  for (int i = 0; i < n_mels + 2; ++i) pts[(size_t)i] = mel_to_hz(m0 + (float)i * (m1 - m0) / (float)(n_mels + 1));
  std::vector<float> fb((size_t)kBins * n_mels, 0.0f);
  for (int i = 0; i < kBins; ++i) {
    const float f = (float)i * sr / (float)kNfft;
    for (int j = 0; j < n_mels; ++j) {
      const float lo = pts[(size_t)j], c = pts[(size_t)j + 1], hi = pts[(size_t)j + 2];
      float v = 0.0f;
      if (f >= lo && f < c) v = (f - lo) / (c - lo);
      else if (f >= c && f <= hi) v = (hi - f) / (hi - c);
      fb[(size_t)i * n_mels + j] = v * (2.0f / (hi - lo));
    }
  }
  return fb;
}

int mel_tables(int device, int n_mels, MelTables* out) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, MelTables> cache;  // held until process exit
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(device, n_mels);
  const auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return VELLA_OK;
  }
  std::vector<float> h = slaney_filters(n_mels);
  const size_t nf = h.size();
  h.resize(nf + 3 * kNfft);
  for (int j = 0; j < kNfft; ++j) {
    const double a = 2.0 * M_PI * (double)j / (double)kNfft;
    h[nf + j] = (float)std::cos(a);
    h[nf + kNfft + j] = (float)std::sin(a);
    // the window as the reference evaluates it in fp32: 0.5 * (1 - cos(2 pi n / N))
    h[nf + 2 * kNfft + j] = 0.5f * (1.0f - std::cos((2.0f * (float)M_PI * (float)j) / (float)kNfft));
  }
  float* d = nullptr;
  VELLA_CUDA_TRY(cudaMalloc(&d, h.size() * sizeof(float)));
  const cudaError_t e = cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "mel tables");
  }
  MelTables t{d, d + nf, d + nf + kNfft, d + nf + 2 * kNfft};
  cache.emplace(key, t);
  *out = t;
  return VELLA_OK;
}

// audio sample j of window s after pad-or-trim and reflect padding; p indexes the padded
// signal [0, 480400)
__device__ __forceinline__ float padded_sample(const float* __restrict__ a, int64_t n_samples, int64_t p) {
  int64_t j = p - kPad;
  if (j < 0) j = -j;
  if (j >= kWindow) j = 2 * (kWindow - 1) - j;
  return j < n_samples ? a[j] : 0.0f;
}

__global__ void __launch_bounds__(kMelThreads) mel_frames_kernel(const float* __restrict__ audio, int64_t audio_stride,
                                                                 int64_t n_samples, int n_mels, MelTables t,
                                                                 float* __restrict__ out) {
  extern __shared__ float sm[];
  float* fr = sm;                                     // [32][401] windowed frames
  float* cs = fr + kFramesPerCta * kFrameStride;      // [400] cos
  float* sn = cs + kNfft;                             // [400] sin
  float* pw = sn + kNfft;                             // [32][203] power
  const int s = blockIdx.y, f0 = blockIdx.x * kFramesPerCta;
  const float* a = audio + (size_t)s * (size_t)audio_stride;
  for (int i = threadIdx.x; i < kNfft; i += kMelThreads) {
    cs[i] = t.cosv[i];
    sn[i] = t.sinv[i];
  }
  for (int i = threadIdx.x; i < kFramesPerCta * kNfft; i += kMelThreads) {
    const int f = i / kNfft, n = i % kNfft, g = f0 + f;
    fr[f * kFrameStride + n] = g < kFrames ? padded_sample(a, n_samples, (int64_t)g * kHop + n) * t.hann[n] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* x = fr + lane * kFrameStride;
  for (int k = warp; k < kBins; k += kMelThreads / 32) {
    float re = 0.0f, im = 0.0f;
    int idx = 0;  // (k * n) mod 400, the same in every lane
    for (int n = 0; n < kNfft; ++n) {
      const float v = x[n];
      re = fmaf(v, cs[idx], re);
      im = fmaf(v, sn[idx], im);
      idx += k;
      if (idx >= kNfft) idx -= kNfft;
    }
    pw[lane * kPowStride + k] = re * re + im * im;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kFramesPerCta * n_mels; i += kMelThreads) {
    const int m = i / kFramesPerCta, f = i % kFramesPerCta, g = f0 + f;
    if (g >= kFrames) continue;
    const float* p = pw + f * kPowStride;
    float acc = 0.0f;
    for (int k = 0; k < kBins; ++k) acc = fmaf(t.filt[k * n_mels + m], p[k], acc);
    out[((size_t)s * n_mels + m) * kFrames + g] = log10f(fmaxf(acc, 1e-10f));
  }
}

constexpr int kFloorThreads = 1024;

// One CTA per window: the window's maximum, then every value floored at maximum - 8 and
// mapped to (x + 4) / 4 (the values are L2-resident: about 1 MB per window).
__global__ void __launch_bounds__(kFloorThreads) mel_floor_kernel(float* __restrict__ out, int n_mels) {
  __shared__ float red[kFloorThreads / 32];
  float* x = out + (size_t)blockIdx.x * n_mels * kFrames;
  const int n = n_mels * kFrames;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += kFloorThreads) mx = fmaxf(mx, x[i]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();  // every thread has read its values before any is rewritten
  mx = -INFINITY;
  for (int i = 0; i < kFloorThreads / 32; ++i) mx = fmaxf(mx, red[i]);
  const float floor_v = mx - 8.0f;
  for (int i = threadIdx.x; i < n; i += kFloorThreads) x[i] = (fmaxf(x[i], floor_v) + 4.0f) / 4.0f;
}

}  // namespace

int launch_log_mel(const float* audio, int64_t audio_stride, int64_t n_samples, int streams, int n_mels, float* out,
                   cudaStream_t stream) {
  int device = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&device));
  MelTables t;
  int rc = mel_tables(device, n_mels, &t);
  if (rc) return rc;
  const size_t smem = (size_t)(kFramesPerCta * kFrameStride + 2 * kNfft + kFramesPerCta * kPowStride) * sizeof(float);
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [&] {
    attr_err = cudaFuncSetAttribute(mel_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "mel_frames_kernel attribute");
  const dim3 grid((kFrames + kFramesPerCta - 1) / kFramesPerCta, (unsigned)streams);
  mel_frames_kernel<<<grid, kMelThreads, smem, stream>>>(audio, audio_stride, n_samples, n_mels, t, out);
  VELLA_CUDA_TRY(cudaGetLastError());
  mel_floor_kernel<<<(unsigned)streams, kFloorThreads, 0, stream>>>(out, n_mels);
  VELLA_CUDA_TRY(cudaGetLastError());
  return VELLA_OK;
}

}  // namespace vella

extern "C" int vella_whisper_mel_filters(int32_t n_mels, float* out) {
  if (!out || n_mels < 1 || n_mels > 512) return vella::fail(VELLA_E_INVALID, "vella_whisper_mel_filters: %d bins", n_mels);
  const std::vector<float> fb = vella::slaney_filters(n_mels);
  std::copy(fb.begin(), fb.end(), out);
  return VELLA_OK;
}

extern "C" int vella_whisper_log_mel(const float* audio, int64_t n_samples, int32_t streams, int32_t n_mels,
                                     float* out, vella_stream_t stream) {
  if (!audio || !out || streams < 1 || n_samples < 0)
    return vella::fail(VELLA_E_INVALID, "vella_whisper_log_mel: NULL pointer or bad sizes");
  if (n_mels != 80 && n_mels != 128)
    return vella::fail(VELLA_E_UNSUPPORTED, "vella_whisper_log_mel: %d mel bins (80 or 128)", n_mels);
  return vella::launch_log_mel(audio, n_samples, n_samples, streams, n_mels, out, (cudaStream_t)stream);
}

