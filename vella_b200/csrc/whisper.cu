// Whisper encoder and decoder step on one GPU (one or more audio streams per handle).
//
// Reference: Worker/Sources/MLXAudioSTT/Whisper/WhisperLayers.swift:11-329 (attention with
// k_proj unbiased, encoder conv1/conv2/positions/pre-LN blocks, decoder layers with self- and
// cross-attention, tied vocabulary projection), WhisperFusedDecode.swift:105-259 (the fused
// decode step: q|k|v as one projection with k's bias zero, the KV append, residual add +
// LayerNorm), WhisperModel.swift:341-400 (the greedy loop with its token rules, :311-372) and
// :218-292 (the temperature fallback's sampled attempts), :554-569 (sinusoid table: double
// trig, rounded to fp32, then to the table dtype).
//
// B200 layout: every weight in one arena; the encoder runs its GEMMs on the tensor cores
// (M = 3000 / 1500 rows) and the attention as the library's clustered flash-decoding kernel
// without a mask; the cross-attention K/V of all decoder layers are projected once per audio
// window into [layers][n_audio][2 * d] (k | v per row) and read in place; the decoder's self
// K/V live in a preallocated [layers][2][heads][max_target][head_dim] cache written at
// absolute positions.  A decoder step is embed, 4 kernels + 8 GEMM/attention launches per
// layer, final LayerNorm, vocabulary GEMM and argmax, captured once into a CUDA graph whose
// positions come from a device scalar.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <initializer_list>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"
#include "model.h"
#include "philox.h"

namespace vella {
namespace {

constexpr int kWRows = 16;      // decoder rows per forward (prompt chunk / teacher-forced chunk)

// ---- kernels -------------------------------------------------------------------------------

// LayerNorm of one row per CTA (ln_row256).
template <typename T>
__global__ void __launch_bounds__(256) layernorm_kernel(T* __restrict__ out, const T* __restrict__ x,
                                                        const T* __restrict__ w, const T* __restrict__ b, int D,
                                                        float eps) {
  __shared__ float red[8];
  pdl_wait();
  pdl_launch_next();
  ln_row256<T>(out + (size_t)blockIdx.x * D, x + (size_t)blockIdx.x * D, w, b, D, eps, threadIdx.x, red,
               [] { __syncthreads(); });
}

template <typename Tin> __device__ __forceinline__ float ld_f(const Tin* p) { return Act<Tin>::to_f(*p); }
template <> __device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }

// im2col of a kernel-3, padding-1 Conv1d: row t = [x(s t - 1), x(s t), x(s t + 1)] over the
// C channels, zero outside [0, T_in) and in the columns 3C..Kp (K padding).  x(t, c) sits at
// x[t * t_stride + c * c_stride].
template <typename Tin, typename T>
__global__ void __launch_bounds__(256) im2col_kernel(T* __restrict__ out, const Tin* __restrict__ x, int C, int stride,
                                                     int T_in, long long t_stride, long long c_stride, int Kp) {
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.x;
  T* orow = out + (size_t)t * Kp;
  for (int e = threadIdx.x; e < Kp; e += blockDim.x) {
    float v = 0.0f;
    if (e < 3 * C) {
      const int j = e / C, c = e % C;
      const int ti = stride * t - 1 + j;
      if (ti >= 0 && ti < T_in) v = ld_f<Tin>(x + (size_t)ti * t_stride + (size_t)c * c_stride);
    }
    orow[e] = Act<T>::from_f(v);
  }
}

// h[m] = T(T(embed[tok[p]]) + dec_pos[p]) at p = *pr.base + pr.off + m; a quantized row is
// T(scale * q + bias) (multiply, then add, each rounded to fp32).  With ln_out set, also
// ln_out[m] = LayerNorm(h[m]) (the first decoder layer's, ln_row256).
template <typename T, int BITS>
__global__ void __launch_bounds__(256) wembed_kernel(T* __restrict__ h, const void* __restrict__ E,
                                                     const T* __restrict__ Es, const T* __restrict__ Eb,
                                                     const T* __restrict__ pos, const int* __restrict__ tok, PosRef pr,
                                                     int d, int vocab, int max_target, int* err, T* ln_out,
                                                     const T* ln_w, const T* ln_b, float eps) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int m = (int)blockIdx.x;
  int p = pr.pos(m);
  if (p < 0 || p >= max_target) {
    if (threadIdx.x == 0) atomicOr(err, 4);
    p = p < 0 ? 0 : max_target - 1;
  }
  int t = tok[(size_t)pr.stream_of(m) * max_target + p];
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0) atomicOr(err, 1);
    t = 0;
  }
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float e;
    if constexpr (BITS == 0) {
      e = A::to_f(static_cast<const T*>(E)[(size_t)t * d + i]);
    } else {
      constexpr int PER = 32 / BITS;
      const uint32_t wd = static_cast<const uint32_t*>(E)[(size_t)t * (d / PER) + i / PER];
      const float q = (float)((wd >> ((i % PER) * BITS)) & ((1u << BITS) - 1));
      const size_t g = (size_t)t * (d / 64) + i / 64;
      e = A::to_f(A::from_f(__fadd_rn(__fmul_rn(A::to_f(Es[g]), q), A::to_f(Eb[g]))));
    }
    h[(size_t)blockIdx.x * d + i] = A::from_f(e + A::to_f(pos[(size_t)p * d + i]));
  }
  if (ln_out) {  // each thread reads back the values it wrote (i = threadIdx.x + 256 j)
    __shared__ float red[8];
    ln_row256<T>(ln_out + (size_t)blockIdx.x * d, h + (size_t)blockIdx.x * d, ln_w, ln_b, d, eps, threadIdx.x, red,
                 [] { __syncthreads(); });
  }
}

// Appends the k and v parts of qkv rows [rows, 3d] to the self-attention cache
// [heads][S][hd] of one layer at position pr.pos(m); row m's stream cache starts kv_ss
// elements per stream after stream 0's.
template <typename T>
__global__ void __launch_bounds__(256) wappend_kernel(const T* __restrict__ qkv, T* __restrict__ kc,
                                                      T* __restrict__ vc, PosRef pr, int d, int hd, int S,
                                                      long long kv_ss) {
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x;
  const int p = pr.pos(m);
  if (p < 0 || p >= S) return;
  const size_t so = (size_t)pr.stream_of(m) * kv_ss;
  kc += so;
  vc += so;
  const T* row = qkv + (size_t)m * 3 * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const int h = i / hd, j = i % hd;
    kc[((size_t)h * S + p) * hd + j] = row[d + i];
    vc[((size_t)h * S + p) * hd + j] = row[2 * d + i];
  }
}

// Stream s (thread s): tok[s][L[s]] = ys[s * ys_stride + ys_off]; L[s] += 1.
__global__ void wcommit_kernel(int* L, int* tok, const int* ys, int max_target, int* err, int streams, int ys_stride,
                               int ys_off) {
  pdl_wait();
  pdl_launch_next();
  const int st = (int)(blockIdx.x * blockDim.x + threadIdx.x);
  if (st >= streams) return;
  const int p = L[st];
  if (p < max_target) tok[(size_t)st * max_target + p] = ys[st * ys_stride + ys_off]; else atomicOr(err, 4);
  L[st] = p + 1;
}

// ---- token rules of the reference's GPU-side greedy (WhisperModel.swift:311-372) --------
struct WRules {
  int eot, no_ts, begin, last_allowed;
};
// Per-decode values the captured step reads from device memory.
struct WDecodeArgs {
  int nprompt;        // prompt length
  float temperature;  // 0: argmax; > 0: a draw from softmax(final row / temperature)
  uint32_t seed_lo, seed_hi;
  uint32_t draw;      // the caller's draw index (Philox counter word)
  int stop;           // end-of-text id of the decode (-1: none): later steps add no log-probability
};
constexpr int kRuleThreads = 512;

// Gumbel noise of token v at a step of stream s: Philox-4x32-10 on counter
// (v / 4, step, s, draw), word v % 4, u = (2*(bits >> 9) + 1) / 2^24 in (0, 1), -log(-log u).
__device__ __forceinline__ float rule_gumbel(const WDecodeArgs& a, int step, int s, int v) {
  const vella::U4 r = vella::philox4x32_10(vella::U4{(uint32_t)v >> 2, (uint32_t)step, (uint32_t)s, a.draw},
                                           a.seed_lo, a.seed_hi);
  const int j = v & 3;
  const uint32_t b = j == 0 ? r.x : j == 1 ? r.y : j == 2 ? r.z : r.w;
  const float u = (float)(2u * (b >> 9) + 1u) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

__device__ __forceinline__ float rule_block_max(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < kRuleThreads / 32; ++i) t = fmaxf(t, red[i]);
  __syncthreads();
  return t;
}
__device__ __forceinline__ float rule_block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < kRuleThreads / 32; ++i) t += red[i];  // warps in order
  __syncthreads();
  return t;
}

// One choice per stream (block s, logits row s * rs + ro): the suppress mask of the step
// (begin-suppress as well at step 0), log-probabilities of the filtered row, the timestamp
// rules, then argmax (lowest index among equal maxima) or, at a temperature, the Gumbel-max
// draw argmax(final / temperature + g); the chosen token's log-probability under the final
// row is added to lpsum[s] until the stream has chosen the decode's end-of-text token (done[s]),
// so steps enqueued past it change nothing the caller reads.  The step is the stream's
// generated-token count L[s] - n_prompt; the rules read the stream's two last generated tokens.
template <typename T>
__global__ void __launch_bounds__(kRuleThreads) wrules_kernel(const T* __restrict__ logits, int vocab, int rs, int ro,
                                                               int* ys, float* lpsum, int* done, int* nonfinite,
                                                               const float* __restrict__ sup_first,
                                                               const float* __restrict__ sup_later, const int* L,
                                                               const int* tok, const WDecodeArgs* da, int max_target,
                                                               WRules r) {
  using A = Act<T>;
  __shared__ float red[kRuleThreads / 32];
  __shared__ int redi[kRuleThreads / 32];
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x, row = s * rs + ro;
  const T* lg = logits + (size_t)row * vocab;
  const WDecodeArgs a = *da;
  const int Ls = L[s], step = Ls - a.nprompt;
  const bool sampled = a.temperature > 0.0f;
  const float* sup = step == 0 ? sup_first : sup_later;
  // maxima of the filtered row (all tokens, text tokens); finiteness of the raw row
  float mall = -INFINITY, mtext = -INFINITY;
  bool bad = false;
  for (int v = threadIdx.x; v < vocab; v += kRuleThreads) {
    const float raw = A::to_f(lg[v]);
    if (!isfinite(raw)) bad = true;
    const float f = raw + sup[v];
    mall = fmaxf(mall, f);
    if (v < r.begin) mtext = fmaxf(mtext, f);
  }
  if (bad) atomicOr(nonfinite, 1);
  mall = rule_block_max(mall, red);
  mtext = rule_block_max(mtext, red);
  float zall = 0.0f, zts = 0.0f;
  for (int v = threadIdx.x; v < vocab; v += kRuleThreads) {
    const float e = expf(A::to_f(lg[v]) + sup[v] - mall);
    zall += e;
    if (v >= r.begin) zts += e;
  }
  zall = rule_block_sum(zall, red);
  zts = rule_block_sum(zts, red);
  const float lse = mall + logf(zall);
  const float ts_mass = logf(zts) + mall - lse, max_text = mtext - lse;
  // the rules of this step
  const bool first = step == 0;
  const bool text_off = first || ts_mass > max_text;
  bool ts_off = false, below_eot_off = false;
  if (step >= 1) {
    // the host keeps n_prompt + max_tokens <= max_target; the clamp keeps the reads in the row
    const int* tk = tok + (size_t)s * max_target;
    const int l1 = min(Ls - 1, max_target - 1), l2 = max(min(Ls - 2, max_target - 1), 0);
    const bool last = tk[l1] >= r.begin;
    const bool pen = step >= 2 ? tk[l2] >= r.begin : true;
    ts_off = last && pen;
    below_eot_off = last && !pen;
  }
  auto final = [&](int v) {
    const float f = A::to_f(lg[v]) + sup[v];
    const bool off = v == r.no_ts || (v < r.begin ? text_off : ts_off) || (below_eot_off && v < r.eot) ||
                     (first && v > r.last_allowed);
    return off ? -INFINITY : f;
  };
  // choice key: the final logit, or final / temperature + Gumbel noise
  float bk = -INFINITY, fmx = -INFINITY;
  int bi = INT32_MAX;
  for (int v = threadIdx.x; v < vocab; v += kRuleThreads) {
    const float f = final(v);
    fmx = fmaxf(fmx, f);
    const float k = sampled ? f / a.temperature + rule_gumbel(a, step, s, v) : f;
    if (k > bk || (k == bk && v < bi)) { bk = k; bi = v; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ok > bk || (ok == bk && oi < bi)) { bk = ok; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { red[threadIdx.x >> 5] = bk; redi[threadIdx.x >> 5] = bi; }
  __syncthreads();
  bk = -INFINITY;
  bi = INT32_MAX;
  for (int i = 0; i < kRuleThreads / 32; ++i)
    if (red[i] > bk || (red[i] == bk && redi[i] < bi)) { bk = red[i]; bi = redi[i]; }
  __syncthreads();
  fmx = rule_block_max(fmx, red);
  float z = 0.0f;
  for (int v = threadIdx.x; v < vocab; v += kRuleThreads) z += expf(final(v) - fmx);
  z = rule_block_sum(z, red);
  if (threadIdx.x == 0) {
    const int t = bi == INT32_MAX ? 0 : bi;
    ys[row] = t;
    if (!done[s]) lpsum[s] += final(t) - fmx - logf(z);
    if (t == a.stop) done[s] = 1;
  }
}

// Zeroes columns [c0, ld) of a row-major [rows, ld] array of 16-bit elements.
__global__ void zero_cols_kernel(uint16_t* w, int ld, int c0) {
  for (int c = c0 + threadIdx.x; c < ld; c += blockDim.x) w[(size_t)blockIdx.x * ld + c] = 0;
}

template <typename T>
__global__ void to_dtype_kernel(T* out, const float* in, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = Act<T>::from_f(in[i]);
}

// ---- the model ---------------------------------------------------------------------------

struct WLin {
  QWeight q;           // w [N, K] dense or packed; s/b for MLX affine
  void* bias = nullptr;
  int bits = 0;
};
struct WNorm {
  void* w = nullptr;
  void* b = nullptr;
};
struct WEnc {
  WNorm ln1, ln2;
  WLin qkv, o, fc1, fc2;
};
struct WDec {
  WNorm ln1, ln2, ln3;
  WLin qkv, o, cq, ckv, co, fc1, fc2;
};

size_t up256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace vella

struct vella_whisper {
  vella_whisper_cfg cfg{};
  int device = 0;
  int S = 1;           // streams
  int R = 0;           // decoder rows per forward: S * kWRows
  size_t elt = 2;
  int kp1 = 0;  // conv1 K padded to a multiple of 64
  void* arena = nullptr;
  size_t arena_bytes = 0;
  vella::WLin conv1, conv2, embed;
  void* enc_pos = nullptr;
  void* dec_pos = nullptr;
  vella::WNorm enc_ln, dec_ln;
  std::vector<vella::WEnc> enc;
  std::vector<vella::WDec> dec;
  // activations
  void* act = nullptr;
  float* mel = nullptr;                          // [S][n_mels][2 n_audio]
  float* audio_buf = nullptr;                    // [S][n_samples] staged audio (encode_audio from the host)
  size_t audio_cap = 0;
  void *col = nullptr, *x0 = nullptr;            // im2col, conv1 output [2A, d]
  void *eh = nullptr, *en = nullptr, *eqkv = nullptr, *eatt = nullptr, *ef = nullptr, *enc_out = nullptr;
  void* xkv = nullptr;                           // [S][dec_layers][A][2d]
  void* kv = nullptr;                            // [S][dec_layers][2][H][max_target][hd]
  void *dh = nullptr, *dn = nullptr, *dqkv = nullptr, *datt = nullptr, *dq2 = nullptr, *df = nullptr;
  void* logits = nullptr;                        // [R, V]
  int *ys = nullptr;                             // [R]
  int *tok = nullptr;                            // [S][max_target]
  int *L = nullptr, *dzero = nullptr;            // [S] lengths, [S] zeros
  int *err = nullptr, *nonfinite = nullptr;
  void* argmax_sc = nullptr;
  // token rules (vella_whisper_set_rules)
  bool rules_on = false;
  vella::WRules rules{};
  float* rule_masks = nullptr;  // [2][vocab]: first step, later steps (0 or -inf)
  float* lpsum = nullptr;       // [S] summed log-probabilities of the current decode
  int* done = nullptr;          // [S] the stream chose the decode's end-of-text token
  vella::WDecodeArgs* dargs = nullptr;  // per-decode values read by the selection kernel
  float temperature = 0.0f;             // following decodes: 0 argmax, > 0 sampled
  uint64_t seed = 0x5eed;
  uint32_t draw = 0;                    // Philox counter word of the sampled decodes
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t step_exec = nullptr;
  bool step_warm = false;
  bool encoded = false;
  // decoder fusions: the first LayerNorm in the embedding kernel, the K/V append in the
  // q|k|v GEMM's epilogue, the other LayerNorms in the preceding GEMM's tail (off with
  // VELLA_WHISPER_FUSE=0 at creation: the same values through separate launches)
  bool fuse = true;
  int step_pos = -1;            // vella_whisper_step: position of the next token (-1: no decode begun)
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr;
  vella_whisper_stats stats{};
};

namespace vella {
namespace {

int plan(vella_whisper* w, const WLin& L, int rows, int epi, vella_qgemm_desc* d, QgemmPlan* p) {
  *d = vella_qgemm_desc{rows, L.q.n, L.q.k, L.bits, 64, w->cfg.dtype, epi};
  if (!qgemm_plan(*d, p)) return fail(VELLA_E_UNSUPPORTED, "whisper gemm %dx%dx%d bits %d", rows, L.q.n, L.q.k, L.bits);
  if (p->workspace > w->gemm_ws_bytes) return fail(VELLA_E_INVALID, "whisper gemm workspace too small");
  return VELLA_OK;
}

// app / norm: the streaming kernel's K/V-append epilogue and LayerNorm tail (the caller
// checks that the plan is a streaming one).
int gemm(vella_whisper* w, const WLin& L, const void* x, int rows, void* out, int epi, const void* residual,
         cudaStream_t s, const KvAppendEpi* app = nullptr, const NormEpi* norm = nullptr) {
  vella_qgemm_desc d;
  QgemmPlan p;
  int rc = plan(w, L, rows, epi, &d, &p);
  if (rc) return rc;
  return qgemm_launch(d, p, x, L.q.w, L.q.s, L.q.b, nullptr, nullptr, nullptr, L.bias, residual, out, w->gemm_ws, s,
                      nullptr, app, norm);
}

template <typename T>
int layernorm_t(void* out, const void* x, const WNorm& n, int rows, int D, float eps, cudaStream_t s) {
  return launch_kernel(layernorm_kernel<T>, dim3(rows), dim3(256), 0, s, static_cast<T*>(out), static_cast<const T*>(x),
                       static_cast<const T*>(n.w), static_cast<const T*>(n.b), D, eps);
}
int layernorm(vella_whisper* w, void* out, const void* x, const WNorm& n, int rows, cudaStream_t s) {
  if (rows <= 0) return VELLA_OK;
  const int D = w->cfg.d_model;
  return w->cfg.dtype == VELLA_BF16 ? layernorm_t<__nv_bfloat16>(out, x, n, rows, D, w->cfg.eps, s)
                                    : layernorm_t<__half>(out, x, n, rows, D, w->cfg.eps, s);
}

// Rows up to which a decoder GEMM's last CTA runs the following LayerNorm (one row after
// another, on its 256 consumer threads); more rows take a LayerNorm launch of a CTA per row.
constexpr int kLnTailRows = 2;

// A residual GEMM into w->dh, then `n` (when set) of its rows into w->dn: in the GEMM's tail
// when the streaming kernel runs it with few rows (*normed = true), else left to the caller.
int gemm_ln(vella_whisper* w, const WLin& L, const void* x, int rows, const WNorm* n, bool* normed, cudaStream_t s) {
  *normed = false;
  vella_qgemm_desc d;
  QgemmPlan p;
  int rc = plan(w, L, rows, VELLA_EPI_BIAS_RESIDUAL, &d, &p);
  if (rc) return rc;
  if (n && w->fuse && p.stream && rows <= kLnTailRows) {
    NormEpi ne;
    ne.out = w->dn; ne.w = n->w; ne.b = n->b; ne.eps = w->cfg.eps;
    *normed = true;
    return gemm(w, L, x, rows, w->dh, VELLA_EPI_BIAS_RESIDUAL, w->dh, s, nullptr, &ne);
  }
  return gemm(w, L, x, rows, w->dh, VELLA_EPI_BIAS_RESIDUAL, w->dh, s);
}

template <typename Tin>
int im2col(vella_whisper* w, void* out, const Tin* x, int C, int stride, int T_in, long long ts, long long cs, int Kp,
           int rows, cudaStream_t s) {
  if (w->cfg.dtype == VELLA_BF16)
    return launch_kernel(im2col_kernel<Tin, __nv_bfloat16>, dim3(rows), dim3(256), 0, s,
                         static_cast<__nv_bfloat16*>(out), x, C, stride, T_in, ts, cs, Kp);
  return launch_kernel(im2col_kernel<Tin, __half>, dim3(rows), dim3(256), 0, s, static_cast<__half*>(out), x, C,
                       stride, T_in, ts, cs, Kp);
}

// The token embedding into w->dh, and with ln set its LayerNorm into w->dn.
template <typename T>
int embed_t(vella_whisper* w, PosRef pr, int rows, const WNorm* ln, cudaStream_t s) {
  const vella_whisper_cfg& c = w->cfg;
  auto* h = static_cast<T*>(w->dh);
  T* lo = ln ? static_cast<T*>(w->dn) : nullptr;
  const T* lw = ln ? static_cast<const T*>(ln->w) : nullptr;
  const T* lb = ln ? static_cast<const T*>(ln->b) : nullptr;
  const auto* es = static_cast<const T*>(w->embed.q.s);
  const auto* eb = static_cast<const T*>(w->embed.q.b);
  const auto* pos = static_cast<const T*>(w->dec_pos);
  if (c.bits == 4)
    return launch_kernel(wembed_kernel<T, 4>, dim3(rows), dim3(256), 0, s, h, (const void*)w->embed.q.w, es, eb, pos,
                         (const int*)w->tok, pr, c.d_model, c.vocab, c.max_target, w->err, lo, lw, lb, c.eps);
  if (c.bits == 8)
    return launch_kernel(wembed_kernel<T, 8>, dim3(rows), dim3(256), 0, s, h, (const void*)w->embed.q.w, es, eb, pos,
                         (const int*)w->tok, pr, c.d_model, c.vocab, c.max_target, w->err, lo, lw, lb, c.eps);
  return launch_kernel(wembed_kernel<T, 0>, dim3(rows), dim3(256), 0, s, h, (const void*)w->embed.q.w, es, eb, pos,
                       (const int*)w->tok, pr, c.d_model, c.vocab, c.max_target, w->err, lo, lw, lb, c.eps);
}

// Elements of one stream's self-attention cache and of its cross-attention K/V.
long long kv_stream_elems(const vella_whisper_cfg& c) {
  return (long long)c.dec_layers * 2 * c.heads * c.max_target * (c.d_model / c.heads);
}
long long xkv_stream_elems(const vella_whisper_cfg& c) { return (long long)c.dec_layers * c.n_audio * 2 * c.d_model; }

template <typename T>
int append_t(vella_whisper* w, int l, PosRef pr, int rows, cudaStream_t s) {
  const vella_whisper_cfg& c = w->cfg;
  const int hd = c.d_model / c.heads;
  const size_t per = (size_t)c.heads * c.max_target * hd;
  T* kc = static_cast<T*>(w->kv) + (size_t)l * 2 * per;
  return launch_kernel(wappend_kernel<T>, dim3(rows), dim3(256), 0, s, static_cast<const T*>(w->dqkv), kc, kc + per, pr,
                       c.d_model, hd, c.max_target, kv_stream_elems(c));
}

void* kcache(vella_whisper* w, int l) {
  const vella_whisper_cfg& c = w->cfg;
  const size_t per = (size_t)c.heads * c.max_target * (c.d_model / c.heads) * w->elt;
  return static_cast<char*>(w->kv) + (size_t)l * 2 * per;
}
void* vcache(vella_whisper* w, int l) {
  const vella_whisper_cfg& c = w->cfg;
  const size_t per = (size_t)c.heads * c.max_target * (c.d_model / c.heads) * w->elt;
  return static_cast<char*>(w->kv) + ((size_t)l * 2 + 1) * per;
}

// Decoder over `rows` rows, `streams` streams of rows / streams consecutive rows each (row m
// at position pr.pos(m) of stream pr.stream_of(m); tokens from w->tok); the last
// `logits_rows` rows go through the vocabulary projection and the argmax, or, with token
// rules set and rule_rs >= 0, stream s's choice comes from logits row s * rule_rs + rule_ro
// under the rules.
int decoder_forward(vella_whisper* w, PosRef pr, int rows, int logits_rows, int streams, cudaStream_t s,
                    int rule_rs = -1, int rule_ro = 0) {
  const vella_whisper_cfg& c = w->cfg;
  if (streams < 1 || rows % streams) return fail(VELLA_E_INVALID, "whisper decoder: %d rows over %d streams", rows, streams);
  const int rps = rows / streams;
  const int d = c.d_model, H = c.heads, hd = d / H, dt = c.dtype;
  const float scale = 1.0f / std::sqrt((float)hd);
  const bool bf = dt == VELLA_BF16;
  int rc;
  // normed: w->dn already holds the LayerNorm that comes next, of the current w->dh
  bool normed = w->fuse && c.dec_layers > 0;
  const WNorm* ln0 = normed ? &w->dec[0].ln1 : nullptr;
  if ((rc = bf ? embed_t<__nv_bfloat16>(w, pr, rows, ln0, s) : embed_t<__half>(w, pr, rows, ln0, s))) return rc;
  for (int l = 0; l < c.dec_layers; ++l) {
    const WDec& L = w->dec[l];
    if (!normed && (rc = layernorm(w, w->dn, w->dh, L.ln1, rows, s))) return rc;
    {
      vella_qgemm_desc qd;
      QgemmPlan qp;
      if ((rc = plan(w, L.qkv, rows, VELLA_EPI_BIAS, &qd, &qp))) return rc;
      if (w->fuse && qp.stream) {
        KvAppendEpi ka;
        ka.kc = kcache(w, l); ka.vc = vcache(w, l); ka.pr = pr;
        ka.d = d; ka.hd = hd; ka.S = c.max_target; ka.kv_ss = kv_stream_elems(c);
        if ((rc = gemm(w, L.qkv, w->dn, rows, w->dqkv, VELLA_EPI_BIAS, nullptr, s, &ka))) return rc;
      } else {
        if ((rc = gemm(w, L.qkv, w->dn, rows, w->dqkv, VELLA_EPI_BIAS, nullptr, s))) return rc;
        if ((rc = bf ? append_t<__nv_bfloat16>(w, l, pr, rows, s) : append_t<__half>(w, l, pr, rows, s))) return rc;
      }
    }
    AttnView sv;
    sv.q = w->dqkv; sv.q_rs = 3LL * d;
    sv.k = kcache(w, l); sv.v = vcache(w, l);
    sv.kv_hs = (long long)c.max_target * hd; sv.kv_rs = hd;
    sv.out = w->datt; sv.o_rs = d;
    sv.q_bs = (long long)rps * 3 * d; sv.o_bs = (long long)rps * d; sv.kv_bs = kv_stream_elems(c);
    if ((rc = launch_attention_ex(dt, sv, streams, pr, 1, rps, H, H, hd, c.max_target, scale, s))) return rc;
    if ((rc = gemm_ln(w, L.o, w->datt, rows, &L.ln2, &normed, s))) return rc;
    if (!normed && (rc = layernorm(w, w->dn, w->dh, L.ln2, rows, s))) return rc;
    if ((rc = gemm(w, L.cq, w->dn, rows, w->dq2, VELLA_EPI_BIAS, nullptr, s))) return rc;
    AttnView cv;
    char* xk = static_cast<char*>(w->xkv) + (size_t)l * c.n_audio * 2 * d * w->elt;
    cv.q = w->dq2; cv.q_rs = d;
    cv.k = xk; cv.v = xk + (size_t)d * w->elt;
    cv.kv_hs = hd; cv.kv_rs = 2LL * d;
    cv.out = w->datt; cv.o_rs = d;
    cv.q_bs = (long long)rps * d; cv.o_bs = (long long)rps * d; cv.kv_bs = xkv_stream_elems(c);
    if ((rc = launch_attention_ex(dt, cv, streams, PosRef{w->dzero, 0}, 0, rps, H, H, hd, c.n_audio, scale, s)))
      return rc;
    if ((rc = gemm_ln(w, L.co, w->datt, rows, &L.ln3, &normed, s))) return rc;
    if (!normed && (rc = layernorm(w, w->dn, w->dh, L.ln3, rows, s))) return rc;
    if ((rc = gemm(w, L.fc1, w->dn, rows, w->df, VELLA_EPI_BIAS_GELU, nullptr, s))) return rc;
    const WNorm& next = l + 1 < c.dec_layers ? w->dec[l + 1].ln1 : w->dec_ln;
    if ((rc = gemm_ln(w, L.fc2, w->df, rows, &next, &normed, s))) return rc;
  }
  if (!normed && (rc = layernorm(w, w->dn, w->dh, w->dec_ln, rows, s))) return rc;
  if (logits_rows > 0) {
    const char* xr = static_cast<const char*>(w->dn) + (size_t)(rows - logits_rows) * d * w->elt;
    if ((rc = gemm(w, w->embed, xr, logits_rows, w->logits, VELLA_EPI_NONE, nullptr, s))) return rc;
    if (w->rules_on && rule_rs >= 0) {
      const float* sf = w->rule_masks;
      const float* sl = w->rule_masks + c.vocab;
      if (bf)
        return launch_kernel(wrules_kernel<__nv_bfloat16>, dim3(streams), dim3(kRuleThreads), 0, s,
                             static_cast<const __nv_bfloat16*>(w->logits), c.vocab, rule_rs, rule_ro, w->ys, w->lpsum, w->done,
                             w->nonfinite, sf, sl, (const int*)w->L, (const int*)w->tok, (const vella::WDecodeArgs*)w->dargs,
                             c.max_target, w->rules);
      return launch_kernel(wrules_kernel<__half>, dim3(streams), dim3(kRuleThreads), 0, s,
                           static_cast<const __half*>(w->logits), c.vocab, rule_rs, rule_ro, w->ys, w->lpsum, w->done,
                           w->nonfinite, sf, sl, (const int*)w->L, (const int*)w->tok, (const vella::WDecodeArgs*)w->dargs,
                           c.max_target, w->rules);
    }
    if ((rc = launch_argmax(dt, w->logits, logits_rows, c.vocab, (size_t)c.vocab, w->ys, w->argmax_sc, w->nonfinite, s)))
      return rc;
  }
  return VELLA_OK;
}

// Encoder of stream `st`'s window, then that stream's cross-attention K/V.
int encoder_forward(vella_whisper* w, int st, cudaStream_t s) {
  const vella_whisper_cfg& c = w->cfg;
  const int d = c.d_model, H = c.heads, hd = d / H, A = c.n_audio, dt = c.dtype;
  const float scale = 1.0f / std::sqrt((float)hd);
  int rc;
  // conv1 over the 2A mel frames (mel is [n_mels][2A]: x(t, c) = mel[c * 2A + t])
  const float* mel = w->mel + (size_t)st * c.n_mels * 2 * A;
  if ((rc = im2col<float>(w, w->col, mel, c.n_mels, 1, 2 * A, 1, 2LL * A, w->kp1, 2 * A, s))) return rc;
  if ((rc = gemm(w, w->conv1, w->col, 2 * A, w->x0, VELLA_EPI_BIAS_GELU, nullptr, s))) return rc;
  // conv2, stride 2, + positions
  if (dt == VELLA_BF16) rc = im2col<__nv_bfloat16>(w, w->col, static_cast<const __nv_bfloat16*>(w->x0), d, 2, 2 * A, d, 1, 3 * d, A, s);
  else rc = im2col<__half>(w, w->col, static_cast<const __half*>(w->x0), d, 2, 2 * A, d, 1, 3 * d, A, s);
  if (rc) return rc;
  if ((rc = gemm(w, w->conv2, w->col, A, w->eh, VELLA_EPI_BIAS_GELU_RESIDUAL, w->enc_pos, s))) return rc;
  for (const WEnc& L : w->enc) {
    if ((rc = layernorm(w, w->en, w->eh, L.ln1, A, s))) return rc;
    if ((rc = gemm(w, L.qkv, w->en, A, w->eqkv, VELLA_EPI_BIAS, nullptr, s))) return rc;
    AttnView v;
    const char* qkv = static_cast<const char*>(w->eqkv);
    v.q = qkv; v.q_rs = 3LL * d;
    v.k = qkv + (size_t)d * w->elt; v.v = qkv + (size_t)2 * d * w->elt;
    v.kv_hs = hd; v.kv_rs = 3LL * d;
    v.out = w->eatt; v.o_rs = d;
    if ((rc = launch_attention_ex(dt, v, 1, PosRef{w->dzero, 0}, 0, A, H, H, hd, A, scale, s))) return rc;
    if ((rc = gemm(w, L.o, w->eatt, A, w->eh, VELLA_EPI_BIAS_RESIDUAL, w->eh, s))) return rc;
    if ((rc = layernorm(w, w->en, w->eh, L.ln2, A, s))) return rc;
    if ((rc = gemm(w, L.fc1, w->en, A, w->ef, VELLA_EPI_BIAS_GELU, nullptr, s))) return rc;
    if ((rc = gemm(w, L.fc2, w->ef, A, w->eh, VELLA_EPI_BIAS_RESIDUAL, w->eh, s))) return rc;
  }
  if ((rc = layernorm(w, w->enc_out, w->eh, w->enc_ln, A, s))) return rc;
  for (int l = 0; l < c.dec_layers; ++l) {
    char* xk = static_cast<char*>(w->xkv) + ((size_t)st * xkv_stream_elems(c) + (size_t)l * A * 2 * d) * w->elt;
    if ((rc = gemm(w, w->dec[l].ckv, w->enc_out, A, xk, VELLA_EPI_BIAS, nullptr, s))) return rc;
  }
  return VELLA_OK;
}

int check_flags(vella_whisper* w, const char* what) {
  int f[2] = {0, 0};
  VELLA_CUDA_TRY(cudaMemcpy(f, w->err, 2 * sizeof(int), cudaMemcpyDeviceToHost));
  if (f[0]) {
    VELLA_CUDA_TRY(cudaMemsetAsync(w->err, 0, sizeof(int), w->stream));
    VELLA_CUDA_TRY(cudaStreamSynchronize(w->stream));
    return fail(VELLA_E_INVALID, "%s: error flags 0x%x (token id out of range or past max_target)", what, f[0]);
  }
  if (f[1]) {
    VELLA_CUDA_TRY(cudaMemsetAsync(w->nonfinite, 0, sizeof(int), w->stream));
    VELLA_CUDA_TRY(cudaStreamSynchronize(w->stream));
    return fail(VELLA_E_NONFINITE, "%s: non-finite logits", what);
  }
  const int st = stream_fault_status(1), tc = tc_fault_status(1);
  if (st < 0 || tc < 0) return fail(VELLA_E_CUDA, "cannot read the kernel fault flags");
  if (st || tc) return fail(VELLA_E_CUDA, "%s: a GEMM pipeline wait timed out (flags 0x%x / 0x%x)", what, st, tc);
  return VELLA_OK;
}

// Byte offsets into one allocation.  Offsets start at 256 so that a planned tensor is never
// offset 0: rebase() treats a null pointer as "tensor absent".
struct Planner {
  size_t off = 256;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += up256(bytes);
    return o;
  }
};

void plan_lin(WLin& L, int n, int k, int bits, size_t elt, Planner& P, bool has_bias) {
  L.bits = bits;
  L.q.n = n;
  L.q.k = k;
  if (bits) {
    L.q.w_bytes = (size_t)n * k * bits / 8;
    L.q.sb_bytes = (size_t)n * (k / 64) * elt;
    L.q.w = reinterpret_cast<void*>(P.take(L.q.w_bytes));
    L.q.s = reinterpret_cast<void*>(P.take(L.q.sb_bytes));
    L.q.b = reinterpret_cast<void*>(P.take(L.q.sb_bytes));
  } else {
    L.q.w_bytes = (size_t)n * k * elt;
    L.q.w = reinterpret_cast<void*>(P.take(L.q.w_bytes));
  }
  if (has_bias) L.bias = reinterpret_cast<void*>(P.take((size_t)n * elt));
}
void plan_norm(WNorm& N, int d, size_t elt, Planner& P) {
  N.w = reinterpret_cast<void*>(P.take((size_t)d * elt));
  N.b = reinterpret_cast<void*>(P.take((size_t)d * elt));
}
template <typename X> void rebase(X*& p, char* base) { if (p) p = reinterpret_cast<X*>(base + reinterpret_cast<uintptr_t>(p)); }
void rebase_lin(WLin& L, char* base) {
  rebase(L.q.w, base); rebase(L.q.s, base); rebase(L.q.b, base); rebase(L.bias, base);
}
void rebase_norm(WNorm& N, char* base) { rebase(N.w, base); rebase(N.b, base); }

int commit(vella_whisper* w, int ys_stride, int ys_off, cudaStream_t s) {
  return launch_kernel(wcommit_kernel, dim3((w->S + 127) / 128), dim3(128), 0, s, w->L, w->tok, (const int*)w->ys,
                       w->cfg.max_target, w->err, w->S, ys_stride, ys_off);
}

// Workspace of a GEMM at each row count it runs at, and at 256 rows below those above it
// (the largest tensor-core call that splits K; the splits keep fp32 sums for every row).
size_t ws_for(const WLin& L, int dtype, int epi, std::initializer_list<int> rows) {
  size_t ws = 0;
  for (int r : rows)
    for (int m : {r, std::min(r, 256)}) {
      vella_qgemm_desc d{m, L.q.n, L.q.k, L.bits, 64, dtype, epi};
      QgemmPlan p;
      if (m > 0 && qgemm_plan(d, &p)) ws = std::max(ws, p.workspace);
    }
  return ws;
}

int run_step(vella_whisper* w) {
  cudaStream_t s = w->stream;
  auto enqueue = [&]() -> int {
    int rc;
    // one row per stream at its last committed token
    if ((rc = decoder_forward(w, PosRef{w->L, -1, 1, 1}, w->S, w->S, w->S, s, 1, 0))) return rc;
    return commit(w, 1, 0, s);
  };
  if (!w->step_warm) {
    const int rc = enqueue();
    if (rc) return rc;
    w->step_warm = true;
    return VELLA_OK;
  }
  if (!w->step_exec) {
    VELLA_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue();
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    const cudaError_t ie = cudaGraphInstantiate(&w->step_exec, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate");
  }
  VELLA_CUDA_TRY(cudaGraphLaunch(w->step_exec, s));
  return VELLA_OK;
}

// The encoder's position table [A][C] in fp32 (WhisperModel.swift:554-569): half = C / 2,
// increment ln(10000) / (half - 1), sin | cos halves of p * exp(-increment * i), in double.
std::vector<float> sinusoid_table(int A, int C) {
  const int half = C / 2;
  std::vector<float> table((size_t)A * C);
  const double inc = std::log(10000.0) / (double)std::max(half - 1, 1);
  for (int p = 0; p < A; ++p)
    for (int i = 0; i < half; ++i) {
      const double t = (double)p * std::exp(-inc * (double)i);
      table[(size_t)p * C + i] = (float)std::sin(t);
      table[(size_t)p * C + half + i] = (float)std::cos(t);
    }
  return table;
}

template <typename T>
int write_sinusoids(vella_whisper* w, cudaStream_t s) {
  const std::vector<float> table = sinusoid_table(w->cfg.n_audio, w->cfg.d_model);
  float* tmp = nullptr;
  VELLA_CUDA_TRY(cudaMalloc(&tmp, table.size() * sizeof(float)));
  cudaError_t e = cudaMemcpyAsync(tmp, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    to_dtype_kernel<T><<<(unsigned)((table.size() + 255) / 256), 256, 0, s>>>(static_cast<T*>(w->enc_pos), tmp, table.size());
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(tmp);
  if (e != cudaSuccess) return cuda_fail(e, "whisper sinusoid table");
  return VELLA_OK;
}

}  // namespace
}  // namespace vella

using namespace vella;

int vella::whisper_weights_loaded(vella_whisper* w) {
  w->encoded = false;
  return VELLA_OK;
}

extern "C" {

int vella_whisper_create(const vella_whisper_cfg* cfg, int32_t device, vella_whisper** out) {
  if (!cfg || !out) return fail(VELLA_E_INVALID, "vella_whisper_create: NULL argument");
  *out = nullptr;
  const vella_whisper_cfg c = *cfg;
  if (c.d_model <= 0 || c.heads <= 0 || c.d_model % 64 || c.d_model % c.heads || c.ffn <= 0 || c.ffn % 64 ||
      c.n_mels <= 0 || c.vocab <= 0 || c.n_audio <= 0 || c.max_target <= 0 || c.enc_layers < 0 || c.dec_layers < 1)
    return fail(VELLA_E_INVALID, "vella_whisper_create: bad dimensions");
  const int hd = c.d_model / c.heads;
  if (hd != 64 && hd != 128) return fail(VELLA_E_UNSUPPORTED, "vella_whisper_create: head_dim %d (64 or 128)", hd);
  if (c.d_model > kLnMaxD) return fail(VELLA_E_UNSUPPORTED, "vella_whisper_create: d_model above %d", kLnMaxD);
  if (c.bits != 0 && c.bits != 4 && c.bits != 8) return fail(VELLA_E_UNSUPPORTED, "vella_whisper_create: bits %d", c.bits);
  if (c.dtype != VELLA_F16 && c.dtype != VELLA_BF16) return fail(VELLA_E_UNSUPPORTED, "vella_whisper_create: dtype");
  if (!(c.eps > 0.0f)) return fail(VELLA_E_INVALID, "vella_whisper_create: eps");
  if (c.streams < 0 || c.streams > 1024) return fail(VELLA_E_INVALID, "vella_whisper_create: %d streams", c.streams);
  VELLA_CUDA_TRY(cudaSetDevice(device));
  auto* w = new vella_whisper();
  w->cfg = c;
  w->device = device;
  if (const char* f = std::getenv("VELLA_WHISPER_FUSE")) w->fuse = std::strcmp(f, "0") != 0;
  w->S = c.streams > 0 ? c.streams : 1;
  w->R = w->S * kWRows;
  w->elt = 2;
  const size_t e = w->elt;
  const int d = c.d_model, A = c.n_audio, F = c.ffn, V = c.vocab, B = c.bits;
  w->kp1 = (3 * c.n_mels + 63) / 64 * 64;
  Planner P;
  plan_lin(w->conv1, d, w->kp1, 0, e, P, true);
  plan_lin(w->conv2, d, 3 * d, 0, e, P, true);
  w->enc_pos = reinterpret_cast<void*>(P.take((size_t)A * d * e));
  w->enc.resize(c.enc_layers);
  for (WEnc& L : w->enc) {
    plan_norm(L.ln1, d, e, P);
    plan_lin(L.qkv, 3 * d, d, 0, e, P, true);
    plan_lin(L.o, d, d, 0, e, P, true);
    plan_norm(L.ln2, d, e, P);
    plan_lin(L.fc1, F, d, 0, e, P, true);
    plan_lin(L.fc2, d, F, 0, e, P, true);
  }
  plan_norm(w->enc_ln, d, e, P);
  w->dec.resize(c.dec_layers);
  for (WDec& L : w->dec) {
    plan_norm(L.ln1, d, e, P);
    plan_lin(L.qkv, 3 * d, d, B, e, P, true);
    plan_lin(L.o, d, d, B, e, P, true);
    plan_norm(L.ln2, d, e, P);
    plan_lin(L.cq, d, d, B, e, P, true);
    plan_lin(L.ckv, 2 * d, d, B, e, P, true);
    plan_lin(L.co, d, d, B, e, P, true);
    plan_norm(L.ln3, d, e, P);
    plan_lin(L.fc1, F, d, B, e, P, true);
    plan_lin(L.fc2, d, F, B, e, P, true);
  }
  plan_norm(w->dec_ln, d, e, P);
  plan_lin(w->embed, V, d, B, e, P, false);
  w->dec_pos = reinterpret_cast<void*>(P.take((size_t)c.max_target * d * e));
  w->arena_bytes = P.off;

  // activations
  size_t ws = 0;
  const int Rd = w->R;  // decoder rows of a forward over every stream
  for (const WDec& L : w->dec) {
    for (const WLin* l : {&L.qkv, &L.cq}) ws = std::max(ws, ws_for(*l, c.dtype, VELLA_EPI_BIAS, {kWRows, Rd}));
    ws = std::max(ws, ws_for(L.ckv, c.dtype, VELLA_EPI_BIAS, {A}));
    for (const WLin* l : {&L.o, &L.co, &L.fc2})
      ws = std::max(ws, ws_for(*l, c.dtype, VELLA_EPI_BIAS_RESIDUAL, {kWRows, Rd}));
    ws = std::max(ws, ws_for(L.fc1, c.dtype, VELLA_EPI_BIAS_GELU, {kWRows, Rd}));
    break;
  }
  ws = std::max(ws, ws_for(w->embed, c.dtype, VELLA_EPI_NONE, {kWRows, Rd}));
  for (const WEnc& L : w->enc) {
    ws = std::max(ws, ws_for(L.qkv, c.dtype, VELLA_EPI_BIAS, {A}));
    ws = std::max(ws, ws_for(L.o, c.dtype, VELLA_EPI_BIAS_RESIDUAL, {A}));
    ws = std::max(ws, ws_for(L.fc2, c.dtype, VELLA_EPI_BIAS_RESIDUAL, {A}));
    ws = std::max(ws, ws_for(L.fc1, c.dtype, VELLA_EPI_BIAS_GELU, {A}));
    break;
  }
  ws = std::max(ws, ws_for(w->conv1, c.dtype, VELLA_EPI_BIAS_GELU, {2 * A}));
  ws = std::max(ws, ws_for(w->conv2, c.dtype, VELLA_EPI_BIAS_GELU_RESIDUAL, {A}));
  w->gemm_ws_bytes = ws;
  const size_t R = (size_t)w->R, S = (size_t)w->S;
  Planner Q;
  const size_t o_mel = Q.take(S * c.n_mels * 2 * A * sizeof(float));
  const size_t o_col = Q.take(std::max((size_t)2 * A * w->kp1, (size_t)A * 3 * d) * e);
  const size_t o_x0 = Q.take((size_t)2 * A * d * e);
  const size_t o_eh = Q.take((size_t)A * d * e), o_en = Q.take((size_t)A * d * e);
  const size_t o_eqkv = Q.take((size_t)A * 3 * d * e), o_eatt = Q.take((size_t)A * d * e);
  const size_t o_ef = Q.take((size_t)A * F * e), o_out = Q.take((size_t)A * d * e);
  const size_t o_xkv = Q.take(S * (size_t)xkv_stream_elems(c) * e);
  const size_t o_kv = Q.take(S * (size_t)kv_stream_elems(c) * e);
  const size_t o_dh = Q.take(R * d * e), o_dn = Q.take(R * d * e), o_dqkv = Q.take(R * 3 * d * e);
  const size_t o_datt = Q.take(R * d * e), o_dq2 = Q.take(R * d * e), o_df = Q.take(R * F * e);
  const size_t o_logits = Q.take(R * (size_t)V * e);
  const size_t o_ints = Q.take((R + S * c.max_target + 2 * S + 8) * sizeof(int));
  const size_t o_amx = Q.take(argmax_scratch_bytes(w->R) + 512);
  const size_t o_rule = Q.take((2 * S + 64) * sizeof(float));
  const size_t o_ws = Q.take(std::max<size_t>(ws, 256));
  auto cleanup = [&]() {
    if (w->act) cudaFree(w->act);
    if (w->arena) cudaFree(w->arena);
    if (w->stream) cudaStreamDestroy(w->stream);
    cudaGetLastError();
    delete w;
  };
  if (cudaMalloc(&w->arena, w->arena_bytes) != cudaSuccess || cudaMalloc(&w->act, Q.off) != cudaSuccess) {
    cleanup();
    return fail(VELLA_E_OOM, "vella_whisper_create: %zu + %zu bytes", P.off, Q.off);
  }
  // the zeroing runs on the handle's own (non-blocking) stream and is waited for here: on the
  // legacy stream it could still be running when the handle's first kernels write the arena
  if (cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMemsetAsync(w->act, 0, Q.off, w->stream) != cudaSuccess ||
      cudaMemsetAsync(w->arena, 0, w->arena_bytes, w->stream) != cudaSuccess ||
      cudaStreamSynchronize(w->stream) != cudaSuccess ||
      cudaEventCreate(&w->ev0) != cudaSuccess || cudaEventCreate(&w->ev1) != cudaSuccess ||
      cudaEventCreate(&w->ev2) != cudaSuccess) {
    cleanup();
    return fail(VELLA_E_CUDA, "vella_whisper_create: stream, events or memset failed");
  }
  char* base = static_cast<char*>(w->arena);
  rebase_lin(w->conv1, base); rebase_lin(w->conv2, base); rebase_lin(w->embed, base);
  rebase(w->enc_pos, base); rebase(w->dec_pos, base);
  rebase_norm(w->enc_ln, base); rebase_norm(w->dec_ln, base);
  for (WEnc& L : w->enc) {
    rebase_norm(L.ln1, base); rebase_norm(L.ln2, base);
    for (WLin* l : {&L.qkv, &L.o, &L.fc1, &L.fc2}) rebase_lin(*l, base);
  }
  for (WDec& L : w->dec) {
    rebase_norm(L.ln1, base); rebase_norm(L.ln2, base); rebase_norm(L.ln3, base);
    for (WLin* l : {&L.qkv, &L.o, &L.cq, &L.ckv, &L.co, &L.fc1, &L.fc2}) rebase_lin(*l, base);
  }
  char* ab = static_cast<char*>(w->act);
  w->mel = reinterpret_cast<float*>(ab + o_mel);
  w->col = ab + o_col; w->x0 = ab + o_x0;
  w->eh = ab + o_eh; w->en = ab + o_en; w->eqkv = ab + o_eqkv; w->eatt = ab + o_eatt; w->ef = ab + o_ef;
  w->enc_out = ab + o_out; w->xkv = ab + o_xkv; w->kv = ab + o_kv;
  w->dh = ab + o_dh; w->dn = ab + o_dn; w->dqkv = ab + o_dqkv; w->datt = ab + o_datt; w->dq2 = ab + o_dq2;
  w->df = ab + o_df; w->logits = ab + o_logits;
  int* ints = reinterpret_cast<int*>(ab + o_ints);
  w->ys = ints;
  w->tok = ints + R;
  w->L = w->tok + S * c.max_target;
  w->dzero = w->L + S;
  w->err = w->dzero + S;  // err and nonfinite are adjacent (check_flags reads both)
  w->nonfinite = w->err + 1;
  w->argmax_sc = ab + o_amx;
  w->lpsum = reinterpret_cast<float*>(ab + o_rule);
  w->done = reinterpret_cast<int*>(w->lpsum + S);
  w->dargs = reinterpret_cast<vella::WDecodeArgs*>(w->done + S);
  w->gemm_ws = ab + o_ws;
  *out = w;
  return VELLA_OK;
}

int vella_whisper_destroy(vella_whisper* w) {
  if (!w) return VELLA_OK;
  cudaSetDevice(w->device);
  if (w->stream) cudaStreamSynchronize(w->stream);
  if (w->step_exec) cudaGraphExecDestroy(w->step_exec);
  if (w->rule_masks) cudaFree(w->rule_masks);
  if (w->audio_buf) cudaFree(w->audio_buf);
  for (cudaEvent_t e : {w->ev0, w->ev1, w->ev2})
    if (e) cudaEventDestroy(e);
  if (w->act) cudaFree(w->act);
  if (w->arena) cudaFree(w->arena);
  if (w->stream) cudaStreamDestroy(w->stream);
  cudaGetLastError();
  delete w;
  return VELLA_OK;
}

int vella_whisper_init_random(vella_whisper* w, uint64_t seed, float std) {
  if (!w) return fail(VELLA_E_INVALID, "vella_whisper_init_random: NULL handle");
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  const vella_whisper_cfg& c = w->cfg;
  cudaStream_t s = w->stream;
  const int dt = c.dtype, d = c.d_model;
  uint32_t tid = 1;
  int rc;
  auto dense = [&](void* p, size_t n, float mean, float sd) { return fill_normal(p, n, dt, seed, tid++, mean, sd, s); };
  auto lin = [&](WLin& L) -> int {
    int r;
    if (L.bits) r = quantize_random(L.q, L.bits, dt, seed, tid++, std, s);
    else r = dense(L.q.w, (size_t)L.q.n * L.q.k, 0.0f, std);
    if (r) return r;
    return L.bias ? dense(L.bias, (size_t)L.q.n, 0.0f, std) : VELLA_OK;
  };
  auto norm = [&](WNorm& N) -> int {
    int r = dense(N.w, (size_t)d, 1.0f, 0.1f);
    return r ? r : dense(N.b, (size_t)d, 0.0f, std);
  };
  if ((rc = lin(w->conv1)) || (rc = lin(w->conv2))) return rc;
  // conv1's K padding columns are zero
  if (w->kp1 > 3 * c.n_mels) {
    zero_cols_kernel<<<d, 64, 0, s>>>(static_cast<uint16_t*>(w->conv1.q.w), w->kp1, 3 * c.n_mels);
    VELLA_CUDA_TRY(cudaGetLastError());
  }
  for (WEnc& L : w->enc) {
    if ((rc = norm(L.ln1)) || (rc = lin(L.qkv)) || (rc = lin(L.o)) || (rc = norm(L.ln2)) || (rc = lin(L.fc1)) ||
        (rc = lin(L.fc2)))
      return rc;
    VELLA_CUDA_TRY(cudaMemsetAsync(static_cast<char*>(L.qkv.bias) + (size_t)d * w->elt, 0, (size_t)d * w->elt, s));
  }
  if ((rc = norm(w->enc_ln))) return rc;
  for (WDec& L : w->dec) {
    if ((rc = norm(L.ln1)) || (rc = lin(L.qkv)) || (rc = lin(L.o)) || (rc = norm(L.ln2)) || (rc = lin(L.cq)) ||
        (rc = lin(L.ckv)) || (rc = lin(L.co)) || (rc = norm(L.ln3)) || (rc = lin(L.fc1)) || (rc = lin(L.fc2)))
      return rc;
    VELLA_CUDA_TRY(cudaMemsetAsync(static_cast<char*>(L.qkv.bias) + (size_t)d * w->elt, 0, (size_t)d * w->elt, s));
    VELLA_CUDA_TRY(cudaMemsetAsync(L.ckv.bias, 0, (size_t)d * w->elt, s));
  }
  if ((rc = norm(w->dec_ln)) || (rc = lin(w->embed))) return rc;
  if ((rc = dense(w->dec_pos, (size_t)c.max_target * d, 0.0f, std))) return rc;
  if ((rc = dt == VELLA_BF16 ? write_sinusoids<__nv_bfloat16>(w, s) : write_sinusoids<__half>(w, s))) return rc;
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  return VELLA_OK;
}

int vella_whisper_sinusoids(int32_t length, int32_t channels, float* out) {
  if (!out || length < 1 || channels < 2 || channels % 2)
    return fail(VELLA_E_INVALID, "vella_whisper_sinusoids: %d x %d (channels even)", length, channels);
  const std::vector<float> t = sinusoid_table(length, channels);
  std::copy(t.begin(), t.end(), out);
  return VELLA_OK;
}

int vella_whisper_get_cfg(const vella_whisper* w, vella_whisper_cfg* out) {
  if (!w || !out) return fail(VELLA_E_INVALID, "vella_whisper_get_cfg: NULL argument");
  *out = w->cfg;
  return VELLA_OK;
}

int vella_whisper_tensor(vella_whisper* w, const char* name, int32_t layer, void** ptr, size_t* bytes) {
  if (!w || !name || !ptr || !bytes) return fail(VELLA_E_INVALID, "vella_whisper_tensor: NULL argument");
  const vella_whisper_cfg& c = w->cfg;
  const size_t e = w->elt;
  const std::string n(name);
  auto ret = [&](void* p, size_t b) {
    *ptr = p;
    *bytes = b;
    return p ? VELLA_OK : fail(VELLA_E_INVALID, "vella_whisper_tensor: '%s' does not exist", name);
  };
  auto lin = [&](const WLin& L, const std::string& part) -> int {
    if (part == "w") return ret(L.q.w, L.q.w_bytes);
    if (part == "s") return ret(L.bits ? L.q.s : nullptr, L.q.sb_bytes);
    if (part == "b") return ret(L.bits ? L.q.b : nullptr, L.q.sb_bytes);
    if (part == "bias") return ret(L.bias, (size_t)L.q.n * e);
    return fail(VELLA_E_INVALID, "vella_whisper_tensor: unknown part '%s'", name);
  };
  auto norm = [&](const WNorm& N, const std::string& part) -> int {
    if (part == "weight") return ret(N.w, (size_t)c.d_model * e);
    if (part == "bias") return ret(N.b, (size_t)c.d_model * e);
    return fail(VELLA_E_INVALID, "vella_whisper_tensor: unknown part '%s'", name);
  };
  const size_t dot = n.rfind('.');
  const std::string head = dot == std::string::npos ? n : n.substr(0, dot);
  const std::string part = dot == std::string::npos ? "" : n.substr(dot + 1);
  if (n == "enc_pos") return ret(w->enc_pos, (size_t)c.n_audio * c.d_model * e);
  if (n == "dec_pos") return ret(w->dec_pos, (size_t)c.max_target * c.d_model * e);
  if (n == "enc_out") return ret(w->enc_out, (size_t)c.n_audio * c.d_model * e);
  if (n == "xkv") return ret(w->xkv, (size_t)w->S * xkv_stream_elems(c) * e);
  if (n == "kv") return ret(w->kv, (size_t)w->S * kv_stream_elems(c) * e);
  if (head == "conv1") return lin(w->conv1, part);
  if (head == "conv2") return lin(w->conv2, part);
  if (head == "embed") return lin(w->embed, part);
  if (head == "enc_ln") return norm(w->enc_ln, part);
  if (head == "dec_ln") return norm(w->dec_ln, part);
  if (head.rfind("enc.", 0) == 0) {
    if (layer < 0 || layer >= c.enc_layers) return fail(VELLA_E_INVALID, "vella_whisper_tensor: encoder layer %d", layer);
    const WEnc& L = w->enc[layer];
    const std::string t = head.substr(4);
    if (t == "ln1") return norm(L.ln1, part);
    if (t == "ln2") return norm(L.ln2, part);
    if (t == "qkv") return lin(L.qkv, part);
    if (t == "o") return lin(L.o, part);
    if (t == "fc1") return lin(L.fc1, part);
    if (t == "fc2") return lin(L.fc2, part);
  }
  if (head.rfind("dec.", 0) == 0) {
    if (layer < 0 || layer >= c.dec_layers) return fail(VELLA_E_INVALID, "vella_whisper_tensor: decoder layer %d", layer);
    const WDec& L = w->dec[layer];
    const std::string t = head.substr(4);
    if (t == "ln1") return norm(L.ln1, part);
    if (t == "ln2") return norm(L.ln2, part);
    if (t == "ln3") return norm(L.ln3, part);
    if (t == "qkv") return lin(L.qkv, part);
    if (t == "o") return lin(L.o, part);
    if (t == "cq") return lin(L.cq, part);
    if (t == "ckv") return lin(L.ckv, part);
    if (t == "co") return lin(L.co, part);
    if (t == "fc1") return lin(L.fc1, part);
    if (t == "fc2") return lin(L.fc2, part);
  }
  return fail(VELLA_E_INVALID, "vella_whisper_tensor: unknown tensor '%s'", name);
}

// The encoder of every stream over the mel features already in w->mel.
static int encode_resident(vella_whisper* w) {
  cudaStream_t s = w->stream;
  w->step_pos = -1;  // a new window ends any token-by-token decode
  int rc = VELLA_OK;
  for (int st = 0; st < w->S && rc == VELLA_OK; ++st) rc = encoder_forward(w, st, s);
  if (rc) return rc;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev1, s));
  VELLA_CUDA_TRY(cudaEventSynchronize(w->ev1));
  cudaEventElapsedTime(&w->stats.encode_ms, w->ev0, w->ev1);
  if ((rc = check_flags(w, "vella_whisper_encode"))) return rc;
  w->encoded = true;
  return VELLA_OK;
}

int vella_whisper_encode(vella_whisper* w, const float* mel, int32_t on_host) {
  if (!w || !mel) return fail(VELLA_E_INVALID, "vella_whisper_encode: NULL argument");
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  const vella_whisper_cfg& c = w->cfg;
  cudaStream_t s = w->stream;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev0, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->mel, mel, (size_t)w->S * c.n_mels * 2 * c.n_audio * sizeof(float),
                                 on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, s));
  return encode_resident(w);
}

int vella_whisper_encode_audio(vella_whisper* w, const float* audio, int64_t n_samples, int32_t on_host) {
  if (!w || !audio || n_samples < 0) return fail(VELLA_E_INVALID, "vella_whisper_encode_audio: NULL argument");
  const vella_whisper_cfg& c = w->cfg;
  if (2 * c.n_audio != 3000 || (c.n_mels != 80 && c.n_mels != 128))
    return fail(VELLA_E_UNSUPPORTED, "vella_whisper_encode_audio: the 30 s log-mel window needs n_audio 1500 and "
                "80 or 128 mel bins");
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  const float* src = audio;
  if (on_host) {
    const size_t need = (size_t)w->S * (size_t)n_samples;
    if (need > w->audio_cap) {
      VELLA_CUDA_TRY(cudaStreamSynchronize(s));
      if (w->audio_buf) cudaFree(w->audio_buf);
      w->audio_buf = nullptr;
      w->audio_cap = 0;
      VELLA_CUDA_TRY(cudaMalloc(&w->audio_buf, std::max<size_t>(need, 1) * sizeof(float)));
      w->audio_cap = need;
    }
    src = w->audio_buf;
  }
  VELLA_CUDA_TRY(cudaEventRecord(w->ev0, s));
  if (on_host && n_samples > 0)
    VELLA_CUDA_TRY(cudaMemcpyAsync(w->audio_buf, audio, (size_t)w->S * (size_t)n_samples * sizeof(float),
                                   cudaMemcpyHostToDevice, s));
  const int rc = launch_log_mel(src, n_samples, n_samples, w->S, c.n_mels, w->mel, s);
  if (rc) return rc;
  return encode_resident(w);
}

// The selection kernel's per-decode values (prompt length, temperature, seed, draw) and
// zeroed log-probability sums.
static int decode_args(vella_whisper* w, int n_prompt, int stop, cudaStream_t s, const char* what) {
  if (w->temperature > 0.0f && !w->rules_on) return fail(VELLA_E_INVALID, "%s: sampling needs token rules", what);
  const WDecodeArgs a{n_prompt, w->temperature, (uint32_t)w->seed, (uint32_t)(w->seed >> 32), w->draw, stop};
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->dargs, &a, sizeof(a), cudaMemcpyHostToDevice, s));
  VELLA_CUDA_TRY(cudaMemsetAsync(w->lpsum, 0, w->S * sizeof(float), s));
  VELLA_CUDA_TRY(cudaMemsetAsync(w->done, 0, w->S * sizeof(int), s));
  return VELLA_OK;
}

// Decoder steps enqueued between two end-of-text checks: the host reads the burst's tokens
// once; steps past an end-of-text token are wasted work but change no returned value.
constexpr int kStopBurst = 8;

int vella_whisper_decode(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens, int32_t eot,
                         int32_t* out_tokens, int32_t* n_out) {
  if (!w || !prompt || !n_out || (max_tokens > 0 && !out_tokens))
    return fail(VELLA_E_INVALID, "vella_whisper_decode: NULL argument");
  const vella_whisper_cfg& c = w->cfg;
  if (!w->encoded) return fail(VELLA_E_INVALID, "vella_whisper_decode: encode first");
  if (w->S != 1) return fail(VELLA_E_INVALID, "vella_whisper_decode: %d streams: use vella_whisper_decode_batch", w->S);
  if (n_prompt < 1 || n_prompt > kWRows) return fail(VELLA_E_INVALID, "vella_whisper_decode: prompt of %d tokens (1..%d)", n_prompt, kWRows);
  if (max_tokens < 0 || n_prompt + max_tokens > c.max_target)
    return fail(VELLA_E_INVALID, "vella_whisper_decode: %d + %d positions exceed max_target %d", n_prompt, max_tokens,
                c.max_target);
  *n_out = 0;
  w->step_pos = -1;  // the token buffer is rewritten
  if (max_tokens == 0) return VELLA_OK;
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  std::vector<int> init(n_prompt + 1);
  std::copy(prompt, prompt + n_prompt, init.begin());
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->tok, init.data(), n_prompt * sizeof(int), cudaMemcpyHostToDevice, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->L, &n_prompt, sizeof(int), cudaMemcpyHostToDevice, s));
  int rc = decode_args(w, n_prompt, eot, s, "vella_whisper_decode");
  if (rc) return rc;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev0, s));
  rc = decoder_forward(w, PosRef{w->dzero, 0}, n_prompt, 1, 1, s, 0, 0);
  if (rc) return rc;
  if ((rc = commit(w, 0, 0, s))) return rc;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev1, s));
  // steps in bursts; with an end-of-text id the host scans each burst's tokens (the first
  // token included) and keeps everything up to the first end-of-text
  int produced = 1, checked = 0, kept = -1;
  std::vector<int> toks((size_t)max_tokens);
  while (kept < 0) {
    const int burst = eot >= 0 ? std::min(kStopBurst, max_tokens - produced) : max_tokens - produced;
    for (int i = 0; i < burst; ++i)
      if ((rc = run_step(w))) return rc;
    produced += burst;
    if (eot < 0) {
      kept = produced;
      break;
    }
    VELLA_CUDA_TRY(cudaMemcpyAsync(toks.data() + checked, w->tok + n_prompt + checked, (produced - checked) * sizeof(int),
                                   cudaMemcpyDeviceToHost, s));
    VELLA_CUDA_TRY(cudaStreamSynchronize(s));
    for (int i = checked; i < produced && kept < 0; ++i)
      if (toks[(size_t)i] == eot) kept = i + 1;
    checked = produced;
    if (produced == max_tokens && kept < 0) kept = produced;
  }
  VELLA_CUDA_TRY(cudaEventRecord(w->ev2, s));
  if (eot < 0)
    VELLA_CUDA_TRY(cudaMemcpyAsync(toks.data(), w->tok + n_prompt, produced * sizeof(int), cudaMemcpyDeviceToHost, s));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  cudaEventElapsedTime(&w->stats.prefill_ms, w->ev0, w->ev1);
  cudaEventElapsedTime(&w->stats.decode_ms, w->ev1, w->ev2);
  w->stats.sum_logprob = 0.0f;
  if (w->rules_on) VELLA_CUDA_TRY(cudaMemcpy(&w->stats.sum_logprob, w->lpsum, sizeof(float), cudaMemcpyDeviceToHost));
  if ((rc = check_flags(w, "vella_whisper_decode"))) return rc;
  int n = kept;
  if (eot >= 0 && n > 0 && toks[(size_t)n - 1] == eot) --n;  // the end-of-text token is not emitted
  std::copy(toks.begin(), toks.begin() + n, out_tokens);
  *n_out = n;
  w->stats.tokens = n;
  return VELLA_OK;
}

int vella_whisper_score(vella_whisper* w, const int32_t* tokens, int32_t T, void* logits, int32_t on_host) {
  if (!w || !tokens || !logits) return fail(VELLA_E_INVALID, "vella_whisper_score: NULL argument");
  const vella_whisper_cfg& c = w->cfg;
  if (!w->encoded) return fail(VELLA_E_INVALID, "vella_whisper_score: encode first");
  if (w->S != 1) return fail(VELLA_E_INVALID, "vella_whisper_score: one-stream handles only");
  if (T < 1 || T > c.max_target) return fail(VELLA_E_INVALID, "vella_whisper_score: %d tokens", T);
  w->step_pos = -1;  // the token buffer is rewritten
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->tok, tokens, (size_t)T * sizeof(int), cudaMemcpyHostToDevice, s));
  const size_t lrow = (size_t)c.vocab * w->elt;
  int rc;
  for (int s0 = 0; s0 < T; s0 += kWRows) {
    const int rows = std::min(kWRows, T - s0);
    if ((rc = decoder_forward(w, PosRef{w->dzero, s0}, rows, rows, 1, s))) return rc;
    VELLA_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(logits) + (size_t)s0 * lrow, w->logits, (size_t)rows * lrow,
                                   on_host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s));
  }
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  return check_flags(w, "vella_whisper_score");
}

// The batched decode: every stream from the same prompt, one decoder forward of S rows per
// token.  With an end-of-text id (eot >= 0) the host scans each burst's tokens of every stream
// and stops once every stream has produced it; n_out[s] counts the tokens before it, and the
// tokens after a stream's end-of-text are -1 in out_tokens.
static int decode_batch_impl(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens, int32_t eot,
                             int32_t* out_tokens, int32_t* n_out, const char* what) {
  if (!w || !prompt || (max_tokens > 0 && !out_tokens)) return fail(VELLA_E_INVALID, "%s: NULL argument", what);
  const vella_whisper_cfg& c = w->cfg;
  if (!w->encoded) return fail(VELLA_E_INVALID, "%s: encode first", what);
  if (n_prompt < 1 || n_prompt > kWRows) return fail(VELLA_E_INVALID, "%s: prompt of %d tokens (1..%d)", what, n_prompt, kWRows);
  if (max_tokens < 0 || n_prompt + max_tokens > c.max_target)
    return fail(VELLA_E_INVALID, "%s: %d + %d positions exceed max_target %d", what, n_prompt, max_tokens, c.max_target);
  const int S = w->S;
  w->step_pos = -1;  // the token buffer is rewritten
  if (n_out)
    for (int st = 0; st < S; ++st) n_out[st] = 0;
  if (max_tokens == 0) return VELLA_OK;
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  std::vector<int> toks((size_t)S * c.max_target, 0), lens(S, n_prompt);
  for (int st = 0; st < S; ++st) std::copy(prompt, prompt + n_prompt, toks.begin() + (size_t)st * c.max_target);
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->tok, toks.data(), toks.size() * sizeof(int), cudaMemcpyHostToDevice, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->L, lens.data(), S * sizeof(int), cudaMemcpyHostToDevice, s));
  int rc = decode_args(w, n_prompt, eot, s, what);
  if (rc) return rc;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev0, s));
  // the prompts of all streams in one forward (stream st: rows st * n_prompt .., positions
  // 0 .. n_prompt - 1), then each stream's first token from its last prompt row
  rc = decoder_forward(w, PosRef{w->dzero, 0, n_prompt, 1}, S * n_prompt, S * n_prompt, S, s, n_prompt,
                       n_prompt - 1);
  if (rc) return rc;
  if ((rc = commit(w, n_prompt, n_prompt - 1, s))) return rc;
  VELLA_CUDA_TRY(cudaEventRecord(w->ev1, s));
  std::vector<int> stop_at(S, -1);  // index of each stream's first end-of-text
  int produced = 1, checked = 0, open = S;
  for (;;) {
    const int burst = eot >= 0 ? std::min(kStopBurst, max_tokens - produced) : max_tokens - produced;
    for (int i = 0; i < burst; ++i)
      if ((rc = run_step(w))) return rc;
    produced += burst;
    if (eot < 0) break;
    const int n = produced - checked;
    VELLA_CUDA_TRY(cudaMemcpy2DAsync(toks.data() + n_prompt + checked, c.max_target * sizeof(int),
                                     w->tok + n_prompt + checked, c.max_target * sizeof(int), n * sizeof(int), S,
                                     cudaMemcpyDeviceToHost, s));
    VELLA_CUDA_TRY(cudaStreamSynchronize(s));
    for (int st = 0; st < S; ++st)
      for (int i = checked; i < produced && stop_at[st] < 0; ++i)
        if (toks[(size_t)st * c.max_target + n_prompt + i] == eot) {
          stop_at[st] = i;
          --open;
        }
    checked = produced;
    if (open == 0 || produced == max_tokens) break;
  }
  VELLA_CUDA_TRY(cudaEventRecord(w->ev2, s));
  if (eot < 0)
    VELLA_CUDA_TRY(cudaMemcpyAsync(toks.data(), w->tok, toks.size() * sizeof(int), cudaMemcpyDeviceToHost, s));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  cudaEventElapsedTime(&w->stats.prefill_ms, w->ev0, w->ev1);
  cudaEventElapsedTime(&w->stats.decode_ms, w->ev1, w->ev2);
  w->stats.sum_logprob = 0.0f;
  if (w->rules_on) VELLA_CUDA_TRY(cudaMemcpy(&w->stats.sum_logprob, w->lpsum, sizeof(float), cudaMemcpyDeviceToHost));
  if ((rc = check_flags(w, what))) return rc;
  int total = 0;
  for (int st = 0; st < S; ++st) {
    const int keep = stop_at[st] >= 0 ? stop_at[st] : produced;
    const int* src = toks.data() + (size_t)st * c.max_target + n_prompt;
    int32_t* dst = out_tokens + (size_t)st * max_tokens;
    for (int i = 0; i < max_tokens; ++i) dst[i] = i < keep ? src[i] : -1;
    if (n_out) n_out[st] = keep;
    total += keep;
  }
  w->stats.tokens = total;
  return VELLA_OK;
}

int vella_whisper_decode_batch(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens,
                               int32_t* out_tokens) {
  return decode_batch_impl(w, prompt, n_prompt, max_tokens, -1, out_tokens, nullptr, "vella_whisper_decode_batch");
}

int vella_whisper_decode_batch_eot(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens,
                                   int32_t eot, int32_t* out_tokens, int32_t* n_out) {
  if (!n_out) return fail(VELLA_E_INVALID, "vella_whisper_decode_batch_eot: NULL n_out");
  return decode_batch_impl(w, prompt, n_prompt, max_tokens, eot, out_tokens, n_out, "vella_whisper_decode_batch_eot");
}

int vella_whisper_begin(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t* first) {
  if (!w || !prompt || !first) return fail(VELLA_E_INVALID, "vella_whisper_begin: NULL argument");
  const vella_whisper_cfg& c = w->cfg;
  w->step_pos = -1;
  if (!w->encoded) return fail(VELLA_E_INVALID, "vella_whisper_begin: encode first");
  if (w->S != 1) return fail(VELLA_E_INVALID, "vella_whisper_begin: %d streams: one-stream handles only", w->S);
  if (n_prompt < 1 || n_prompt > kWRows || n_prompt >= c.max_target)
    return fail(VELLA_E_INVALID, "vella_whisper_begin: prompt of %d tokens (1..%d)", n_prompt, kWRows);
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->tok, prompt, n_prompt * sizeof(int), cudaMemcpyHostToDevice, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(w->L, &n_prompt, sizeof(int), cudaMemcpyHostToDevice, s));
  int rc = decode_args(w, n_prompt, -1, s, "vella_whisper_begin");
  if (rc) return rc;
  if ((rc = decoder_forward(w, PosRef{w->dzero, 0}, n_prompt, 1, 1, s, 0, 0))) return rc;
  if ((rc = commit(w, 0, 0, s))) return rc;
  VELLA_CUDA_TRY(cudaMemcpyAsync(first, w->tok + n_prompt, sizeof(int), cudaMemcpyDeviceToHost, s));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  if ((rc = check_flags(w, "vella_whisper_begin"))) return rc;
  w->step_pos = n_prompt + 1;
  return VELLA_OK;
}

int vella_whisper_step(vella_whisper* w, int32_t* token) {
  if (!w || !token) return fail(VELLA_E_INVALID, "vella_whisper_step: NULL argument");
  if (w->step_pos < 0) return fail(VELLA_E_INVALID, "vella_whisper_step: call vella_whisper_begin first");
  if (w->step_pos >= w->cfg.max_target)
    return fail(VELLA_E_INVALID, "vella_whisper_step: max_target %d positions reached", w->cfg.max_target);
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  cudaStream_t s = w->stream;
  int rc = run_step(w);
  if (rc) return rc;
  VELLA_CUDA_TRY(cudaMemcpyAsync(token, w->tok + w->step_pos, sizeof(int), cudaMemcpyDeviceToHost, s));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  if ((rc = check_flags(w, "vella_whisper_step"))) return rc;
  ++w->step_pos;
  return VELLA_OK;
}

int vella_whisper_get_logprobs(const vella_whisper* w, float* out, int32_t n) {
  if (!w || (n > 0 && !out)) return fail(VELLA_E_INVALID, "vella_whisper_get_logprobs: NULL argument");
  if (n < 0 || n > w->S) return fail(VELLA_E_INVALID, "vella_whisper_get_logprobs: %d of %d streams", n, w->S);
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  VELLA_CUDA_TRY(cudaStreamSynchronize(w->stream));
  if (n > 0) VELLA_CUDA_TRY(cudaMemcpy(out, w->lpsum, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost));
  return VELLA_OK;
}

int vella_whisper_set_rules(vella_whisper* w, const vella_whisper_rules* rules) {
  if (!w) return fail(VELLA_E_INVALID, "vella_whisper_set_rules: NULL handle");
  VELLA_CUDA_TRY(cudaSetDevice(w->device));
  const vella_whisper_cfg& c = w->cfg;
  const int V = c.vocab;
  if (rules) {
    const vella_whisper_rules& r = *rules;
    auto in = [&](int t) { return t >= 0 && t < V; };
    if (!in(r.eot) || !in(r.no_timestamps) || !in(r.timestamp_begin) || r.eot >= r.timestamp_begin ||
        r.n_suppress < 0 || r.n_begin_suppress < 0 || (r.n_suppress > 0 && !r.suppress) ||
        (r.n_begin_suppress > 0 && !r.begin_suppress))
      return fail(VELLA_E_INVALID, "vella_whisper_set_rules: token ids outside the vocabulary of %d or eot >= "
                  "timestamp_begin", V);
  }
  VELLA_CUDA_TRY(cudaStreamSynchronize(w->stream));
  // the captured step holds the previous selection kernel
  if (w->step_exec) {
    cudaGraphExecDestroy(w->step_exec);
    w->step_exec = nullptr;
  }
  w->step_warm = false;
  if (!rules) {
    w->rules_on = false;
    return VELLA_OK;
  }
  const vella_whisper_rules& r = *rules;
  std::vector<float> m(2 * (size_t)V, 0.0f);  // first step, later steps
  for (int i = 0; i < r.n_suppress; ++i)
    if (r.suppress[i] >= 0 && r.suppress[i] < V) m[r.suppress[i]] = m[(size_t)V + r.suppress[i]] = -INFINITY;
  for (int i = 0; i < r.n_begin_suppress; ++i)
    if (r.begin_suppress[i] >= 0 && r.begin_suppress[i] < V) m[r.begin_suppress[i]] = -INFINITY;
  if (!w->rule_masks) VELLA_CUDA_TRY(cudaMalloc(&w->rule_masks, m.size() * sizeof(float)));
  VELLA_CUDA_TRY(cudaMemcpy(w->rule_masks, m.data(), m.size() * sizeof(float), cudaMemcpyHostToDevice));
  // Swift's Double.rounded(): half away from zero (WhisperModel.swift:321)
  w->rules = WRules{r.eot, r.no_timestamps, r.timestamp_begin,
                    r.timestamp_begin + (int)std::floor((double)c.n_audio / 30.0 + 0.5)};
  w->rules_on = true;
  return VELLA_OK;
}

int vella_whisper_set_sampling(vella_whisper* w, float temperature, uint64_t seed, uint32_t draw) {
  if (!w) return fail(VELLA_E_INVALID, "vella_whisper_set_sampling: NULL handle");
  if (!(temperature >= 0.0f) || !std::isfinite(temperature))
    return fail(VELLA_E_INVALID, "vella_whisper_set_sampling: temperature %g", (double)temperature);
  w->temperature = temperature;
  w->seed = seed;
  w->draw = draw;
  return VELLA_OK;
}

int vella_whisper_get_stats(const vella_whisper* w, vella_whisper_stats* out) {
  if (!w || !out) return fail(VELLA_E_INVALID, "vella_whisper_get_stats: NULL argument");
  *out = w->stats;
  return VELLA_OK;
}

}  // extern "C"
