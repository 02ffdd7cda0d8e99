// Draft-and-verify decode loop on one GPU: prefill, one CUDA graph per pass (K draft
// steps, one batched target verify, acceptance, KV rollback), and the host loop with the
// reference's stop rules and fallbacks.
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeModel.swift
//   decodeMTP :306-396 (greedy draft-and-verify: accepted = longest prefix where the
//   target's argmax equals the draft, bonus = the target's token after it, one host sync
//   per pass, non-finite verify logits are an error), decodeGreedy :266-290, decode
//   :412-431 (sticky fallback to plain greedy after a runtime failure), retryingRunaway
//   :436-443, endsInLoop :296-302; NTKVCache.trim NemotronTranscribeDecoder.swift:111-116.
//
// B200 design.  All sequence state lives on the device: token history tok[pos], the
// committed length L and the prefix length P.  Every kernel of a pass reads its positions
// from L, so one captured graph replays every pass.  Draft tokens are written straight into
// tok[L..L+K) (speculatively); the target verifies positions L-1..L+K-1 in one forward and
// appends their K/V; acceptance rewrites tok[L+a] with the bonus token and advances L by
// a+1.  Rolling back the KV cache is free: the cache is valid below L-1 by construction and
// the next pass overwrites everything from there on (no copies, no trims).  The draft runs
// its first step over the two positions L-2, L-1, so it catches up after a full acceptance
// and after a rejection with the same graph.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"
#include "loopguard.h"
#include "model.h"
#include "philox.h"

namespace vella {
namespace {

struct DevState {
  int L;          // committed positions (prefix + emitted tokens)
  int P;          // prefix length
  int pass;       // passes run since the prefill (Philox counter of the oracle draft)
  int n_new;      // tokens committed by the last pass / step (0: the stream is done)
  int nonfinite;  // the last verify logits held NaN/Inf
  int err;        // bit 0 bad token id, bit 1 bad position, bit 2 capacity
  int ref_len;    // length of the oracle reference
  int produced;   // tokens committed since the prefill (its first token included)
  int quota;      // stop advancing once produced >= quota (0: no limit)
  int newtok[16];
};
constexpr int kStateInts = sizeof(DevState) / sizeof(int);  // PosRef stride between streams

__device__ __forceinline__ bool done(const DevState& x) { return x.quota > 0 && x.produced >= x.quota; }

// The decode settings the sampling kernels read.
struct vella_spec_cfg_dev {
  uint64_t seed;
  float temperature;
  float oracle_p;
  int draft_mode;
};

// One stream: st, tok and the logits rows of that stream's prefill forward.
__global__ void prefill_finish_kernel(DevState* st, int* tok, const int* ys, const int* nf, const int* err_t,
                                      int max_seq) {
  pdl_wait();
  pdl_launch_next();
  const int P = st->P, t = ys[0];
  if (P < max_seq) tok[P] = t; else st->err |= 4;
  st->L = P + 1;
  st->n_new = 1;
  st->newtok[0] = t;
  st->pass = 0;
  st->produced = 1;
  st->nonfinite = *nf;
  st->err |= *err_t;
}

// Stream blockIdx.x: commit the argmax of its one verify row.
__global__ void greedy_commit_kernel(DevState* st, int* tok, const int* ys, const int* nf, const int* err_t,
                                     int max_seq) {
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  DevState& x = st[s];
  x.nonfinite = *nf;
  x.err |= *err_t;
  if (done(x)) {
    x.n_new = 0;
    return;
  }
  int* tk = tok + (size_t)s * max_seq;
  const int L = x.L, t = ys[s];
  if (L < max_seq) tk[L] = t; else x.err |= 4;
  x.L = L + 1;
  x.n_new = 1;
  x.newtok[0] = t;
  x.produced += 1;
}

// Draft step i of stream blockIdx.x proposes the token at position L + i.
__global__ void propose_kernel(DevState* st, int* tok, const int* ys_draft, int i, int mode, float p, uint64_t seed,
                               const int* ref, int vocab, int max_seq) {
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  const DevState& x = st[s];
  const int pos = x.L + i;
  int t = ys_draft[s];
  if (mode == VELLA_DRAFT_ORACLE) {
    const U4 r = philox4x32_10(U4{(uint32_t)x.pass, (uint32_t)i, 0x0D4A7u, (uint32_t)s}, (uint32_t)seed,
                               (uint32_t)(seed >> 32));
    const int ri = pos - x.P;
    if (u01(r.x) < p && ri >= 0 && ri < x.ref_len) t = ref[(size_t)s * max_seq + ri];
    else t = min((int)(u01(r.y) * (float)vocab), vocab - 1);
  }
  if (pos < max_seq) tok[(size_t)s * max_seq + pos] = t;
}

// Greedy acceptance of stream blockIdx.x over its verify argmax ys[s(K+1) .. s(K+1)+K]
// (ys[j] predicts position L + j).
__global__ void accept_kernel(DevState* st, int* tok, const int* ys, int K, const int* nf, const int* err_t,
                              const int* err_d, int max_seq) {
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  DevState& x = st[s];
  x.nonfinite = *nf;
  x.err |= *err_t | *err_d;
  if (done(x)) {
    x.n_new = 0;
    return;
  }
  int* tk = tok + (size_t)s * max_seq;
  const int* y = ys + (size_t)s * (K + 1);
  const int L = x.L;
  int a = 0;
  while (a < K && y[a] == tk[L + a]) ++a;
  const int bonus = y[a];
  if (L + a < max_seq) tk[L + a] = bonus; else x.err |= 4;
  for (int j = 0; j <= a; ++j) x.newtok[j] = tk[L + j];
  x.n_new = a + 1;
  x.L = L + a + 1;
  x.pass += 1;
  x.produced += a + 1;
}

// ---- stochastic acceptance (temperature > 0) ------------------------------------------------
// Uniform purposes in the Philox counter (pass or step, position, purpose, stream).
constexpr uint32_t kPurposeDraft = 0x5A3D1u, kPurposeAccept = 0xACC01u, kPurposeResidual = 0xB0B05u,
                   kPurposeFirst = 0xF1257u, kPurposeStep = 0x57E90u;
constexpr int kSampThreads = 512;

struct SampShared {
  float red[kSampThreads / 32];
  float part[kSampThreads];
  float before, stat;
  int seg, idx;
};

__device__ __forceinline__ float uni(const vella_spec_cfg_dev& c, uint32_t a, uint32_t b, uint32_t purpose, int s) {
  return u01(philox4x32_10(U4{a, b, purpose, (uint32_t)s}, (uint32_t)c.seed, (uint32_t)(c.seed >> 32)).x);
}

__device__ float block_max(float v, SampShared& sh) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, sh.red[w]);
    sh.stat = m;
  }
  __syncthreads();
  return sh.stat;
}

__device__ float block_sum(float v, SampShared& sh) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh.red[w];
    sh.stat = t;
  }
  __syncthreads();
  return sh.stat;
}

// (max, sum of exp((l - max) / T)) of one logits row.
template <typename T>
__device__ float2 row_softmax_stats(const T* row, int V, float invT, SampShared& sh) {
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) m = fmaxf(m, Act<T>::to_f(row[v]));
  m = block_max(m, sh);
  float z = 0.0f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) z += expf((Act<T>::to_f(row[v]) - m) * invT);
  z = block_sum(z, sh);
  return make_float2(m, z);
}

// Index drawn from the unnormalised weights w(0..V) with the uniform u: thread t owns the
// contiguous range [t C, (t+1) C); the partial sums are scanned in thread order, so the
// result depends only on the weights and u.  -1 when every weight is zero.
template <typename W>
__device__ int sample_icdf(W w, int V, float u, SampShared& sh) {
  const int C = (V + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = min(V, (int)threadIdx.x * C), hi = min(V, lo + C);
  float ps = 0.0f;
  for (int v = lo; v < hi; ++v) ps += w(v);
  __syncthreads();
  sh.part[threadIdx.x] = ps;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int t = 0; t < (int)blockDim.x; ++t) tot += sh.part[t];
    const float target = u * tot;
    float acc = 0.0f;
    int seg = -1, last = -1;
    for (int t = 0; t < (int)blockDim.x; ++t) {
      const float p = sh.part[t];
      if (p > 0.0f) last = t;
      if (seg < 0 && acc + p > target) {
        seg = t;
        sh.before = acc;
      }
      acc += p;
    }
    if (seg < 0) {  // rounding at the top end: the last range with weight
      seg = last;
      sh.before = -1.0f;
    }
    sh.seg = seg;
    sh.idx = -1;
    sh.stat = target;
  }
  __syncthreads();
  if ((int)threadIdx.x == sh.seg) {
    const float target = sh.stat;
    float acc = sh.before;
    int found = -1, lastv = -1;
    for (int v = lo; v < hi; ++v) {
      const float x = w(v);
      if (x > 0.0f) lastv = v;
      if (found < 0 && sh.before >= 0.0f && acc + x > target) found = v;
      acc += x;
    }
    sh.idx = found >= 0 ? found : lastv;
  }
  __syncthreads();
  return sh.idx;
}

// Draft step i, stream blockIdx.x: x ~ softmax(draft logits / T) for position L + i; the
// row and its (max, sum) are kept for the acceptance test.
template <typename T>
__global__ void __launch_bounds__(kSampThreads) draft_sample_kernel(DevState* st, int* tok, const T* logits, int i,
                                                                    vella_spec_cfg_dev c, int vocab, int max_seq,
                                                                    T* qrows, float2* qstats, int S) {
  __shared__ SampShared sh;
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  const DevState& x = st[s];
  const T* row = logits + (size_t)s * vocab;
  const float invT = 1.0f / c.temperature;
  const float2 mz = row_softmax_stats(row, vocab, invT, sh);
  const float u = uni(c, (uint32_t)x.pass, (uint32_t)i, kPurposeDraft, s);
  int t = sample_icdf([&](int v) { return expf((Act<T>::to_f(row[v]) - mz.x) * invT); }, vocab, u, sh);
  if (t < 0) t = 0;
  T* q = qrows + ((size_t)i * S + s) * vocab;
  for (int v = threadIdx.x; v < vocab; v += blockDim.x) q[v] = row[v];
  if (threadIdx.x == 0) {
    qstats[(size_t)i * S + s] = mz;
    const int pos = x.L + i;
    if (pos < max_seq) tok[(size_t)s * max_seq + pos] = t;
  }
}

// q(v) of draft position j: the model draft's kept row, or the oracle draft's mixture.
template <typename T>
struct DraftQ {
  const T* row;  // null: oracle draft
  float m, z, invT;
  int ref;       // oracle: reference token at this position, -1 when outside the reference
  float p;
  int vocab;
  __device__ float operator()(int v) const {
    if (row) return expf((Act<T>::to_f(row[v]) - m) * invT) / z;
    const float base = (ref >= 0 ? 1.0f - p : 1.0f) / (float)vocab;
    return v == ref ? base + p : base;
  }
};

// Stochastic acceptance of stream blockIdx.x over its K + 1 verify rows.
template <typename T>
__global__ void __launch_bounds__(kSampThreads) accept_sampled_kernel(DevState* st, int* tok, const T* logits, int K,
                                                                      vella_spec_cfg_dev c, int vocab, int max_seq,
                                                                      const T* qrows, const float2* qstats, int S,
                                                                      const int* ref, const int* nf, const int* err_t,
                                                                      const int* err_d) {
  __shared__ SampShared sh;
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  DevState& x = st[s];
  if (done(x)) {  // uniform across the block: every thread returns
    __syncthreads();
    if (threadIdx.x == 0) {
      x.nonfinite = *nf;
      x.err |= *err_t | *err_d;
      x.n_new = 0;
    }
    return;
  }
  int* tk = tok + (size_t)s * max_seq;
  const int L = x.L;
  const float invT = 1.0f / c.temperature;
  int a = 0, bonus = -1;
  for (int j = 0; j < K; ++j) {
    const T* prow = logits + ((size_t)s * (K + 1) + j) * vocab;
    const float2 pm = row_softmax_stats(prow, vocab, invT, sh);
    const int xj = tk[L + j];
    DraftQ<T> q{};
    q.invT = invT;
    q.vocab = vocab;
    q.p = c.oracle_p;
    if (c.draft_mode == VELLA_DRAFT_ORACLE) {
      const int ri = L + j - x.P;
      q.ref = (ri >= 0 && ri < x.ref_len) ? ref[(size_t)s * max_seq + ri] : -1;
    } else {
      q.row = qrows + ((size_t)j * S + s) * vocab;
      const float2 qm = qstats[(size_t)j * S + s];
      q.m = qm.x;
      q.z = qm.y;
    }
    const float px = expf((Act<T>::to_f(prow[xj]) - pm.x) * invT) / pm.y;
    const float qx = q(xj);
    const float u = uni(c, (uint32_t)x.pass, (uint32_t)j, kPurposeAccept, s);
    if (u * qx < px) {  // accept with probability min(1, p / q)
      ++a;
      continue;
    }
    const float u2 = uni(c, (uint32_t)x.pass, (uint32_t)j, kPurposeResidual, s);
    bonus = sample_icdf(
        [&](int v) { return fmaxf(0.0f, expf((Act<T>::to_f(prow[v]) - pm.x) * invT) / pm.y - q(v)); }, vocab, u2, sh);
    if (bonus < 0)  // p == q everywhere: draw from p
      bonus = sample_icdf([&](int v) { return expf((Act<T>::to_f(prow[v]) - pm.x) * invT); }, vocab, u2, sh);
    break;
  }
  if (bonus < 0) {
    const T* prow = logits + ((size_t)s * (K + 1) + K) * vocab;
    const float2 pm = row_softmax_stats(prow, vocab, invT, sh);
    const float u2 = uni(c, (uint32_t)x.pass, (uint32_t)K, kPurposeResidual, s);
    bonus = sample_icdf([&](int v) { return expf((Act<T>::to_f(prow[v]) - pm.x) * invT); }, vocab, u2, sh);
    if (bonus < 0) bonus = 0;
  }
  if (threadIdx.x == 0) {
    x.nonfinite = *nf;
    x.err |= *err_t | *err_d;
    if (L + a < max_seq) tk[L + a] = bonus; else x.err |= 4;
    for (int j = 0; j <= a; ++j) x.newtok[j] = tk[L + j];
    x.n_new = a + 1;
    x.L = L + a + 1;
    x.pass += 1;
    x.produced += a + 1;
  }
}

// Plain sampling step of stream blockIdx.x: tok[L] ~ softmax(logits row s / T).  With
// `first` the row is the stream's prefill logits (one row) and the state is not yet
// advanced past the prefix (the prefill finish kernel already ran).
template <typename T>
__global__ void __launch_bounds__(kSampThreads) sample_commit_kernel(DevState* st, int* tok, const T* logits,
                                                                     vella_spec_cfg_dev c, int vocab, int max_seq,
                                                                     int first, int sbase, const int* nf,
                                                                     const int* err_t) {
  __shared__ SampShared sh;
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  DevState& x = st[s];
  const bool stop = !first && done(x);
  if (stop) {
    __syncthreads();
    if (threadIdx.x == 0) {
      x.nonfinite = *nf;
      x.err |= *err_t;
      x.n_new = 0;
    }
    return;
  }
  const T* row = logits + (size_t)s * vocab;
  const float invT = 1.0f / c.temperature;
  const float2 mz = row_softmax_stats(row, vocab, invT, sh);
  const float u = first ? uni(c, 0u, 0u, kPurposeFirst, sbase + s)
                        : uni(c, (uint32_t)x.produced, 0u, kPurposeStep, sbase + s);
  int t = sample_icdf([&](int v) { return expf((Act<T>::to_f(row[v]) - mz.x) * invT); }, vocab, u, sh);
  if (t < 0) t = 0;
  if (threadIdx.x == 0) {
    int* tk = tok + (size_t)s * max_seq;
    if (first) {  // replace the argmax the prefill finish kernel committed at position P
      tk[x.P] = t;
      x.newtok[0] = t;
    } else {
      x.nonfinite = *nf;
      x.err |= *err_t;
      const int L = x.L;
      if (L < max_seq) tk[L] = t; else x.err |= 4;
      x.L = L + 1;
      x.n_new = 1;
      x.newtok[0] = t;
      x.produced += 1;
    }
  }
}

}  // namespace

struct Spec {
  Model* target = nullptr;
  Model* draft = nullptr;
  vella_spec_cfg cfg{};
  int device = 0;
  int max_seq = 0;
  int streams = 1;
  cudaStream_t stream = nullptr;
  DevState* dstate = nullptr;  // [streams]
  DevState* hstate = nullptr;  // [streams], pinned
  int* tok = nullptr;          // [streams][max_seq]
  int* ref = nullptr;          // [streams][max_seq]
  int ref_len = 0;
  int P = 0;
  cudaGraphExec_t pass_exec = nullptr;
  cudaGraphExec_t greedy_exec = nullptr;
  bool pass_warm = false, greedy_warm = false;
  int fault = VELLA_FAULT_NONE;
  bool draft_disabled = false;
  std::string failure;
  vella_spec_stats stats{};
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, evp = nullptr;  // decode start, end, prefill end
  void* qrows = nullptr;     // [K][streams][vocab] the draft's logits rows (stochastic acceptance)
  float2* qstats = nullptr;  // [K][streams] their (max, sum)

  bool sampled() const { return cfg.temperature > 0.0f; }
  vella_spec_cfg_dev dev_cfg() const {
    return vella_spec_cfg_dev{cfg.seed, cfg.temperature, cfg.oracle_p, cfg.draft_mode};
  }
};

namespace {

// A GEMM pipeline whose wait ran out of time finished without its result: the decode that
// used it is void.  Checked once per prefill and per decode call.
int pipeline_faults() {
  const int st = stream_fault_status(1), tc = tc_fault_status(1);
  if (st < 0 || tc < 0) return fail(VELLA_E_CUDA, "cannot read the kernel fault flags");
  if (st || tc) return fail(VELLA_E_CUDA, "a GEMM pipeline wait timed out (flags 0x%x / 0x%x)", st, tc);
  return VELLA_OK;
}

int sync_state(Spec* s) {
  VELLA_CUDA_TRY(cudaMemcpyAsync(s->hstate, s->dstate, sizeof(DevState) * s->streams, cudaMemcpyDeviceToHost,
                                 s->stream));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int j = 0; j < s->streams; ++j)
    if (s->hstate[j].err)
      return fail(VELLA_E_INVALID, "decode state error flags 0x%x in stream %d (bad token id, position or capacity)",
                  s->hstate[j].err, j);
  return VELLA_OK;
}

PosRef state_pos(Spec* s, int off) { return PosRef{&s->dstate[0].L, off, 0, kStateInts}; }

template <typename T>
int launch_draft_sample(Spec* s, int i) {
  const Model* d = s->draft;
  return launch_kernel(draft_sample_kernel<T>, dim3(s->streams), dim3(kSampThreads), 0, s->stream, s->dstate, s->tok,
                       static_cast<const T*>(d->logits), i, s->dev_cfg(), s->target->cfg.vocab, s->max_seq,
                       static_cast<T*>(s->qrows), s->qstats, s->streams);
}

template <typename T>
int launch_accept_sampled(Spec* s) {
  const Model* t = s->target;
  return launch_kernel(accept_sampled_kernel<T>, dim3(s->streams), dim3(kSampThreads), 0, s->stream, s->dstate,
                       s->tok, static_cast<const T*>(t->logits), s->cfg.draft_k, s->dev_cfg(), t->cfg.vocab,
                       s->max_seq, static_cast<const T*>(s->qrows), (const float2*)s->qstats, s->streams,
                       (const int*)s->ref, (const int*)t->nonfinite, (const int*)t->err, (const int*)s->draft->err);
}

template <typename T>
int launch_sample_commit(Spec* s, DevState* st, int* tok, int streams, int first, int sbase) {
  const Model* t = s->target;
  return launch_kernel(sample_commit_kernel<T>, dim3(streams), dim3(kSampThreads), 0, s->stream, st, tok,
                       static_cast<const T*>(t->logits), s->dev_cfg(), t->cfg.vocab, s->max_seq, first, sbase,
                       (const int*)t->nonfinite, (const int*)t->err);
}

bool bf16_of(const Spec* s) { return s->target->cfg.dtype == VELLA_BF16; }

int enqueue_pass(Spec* s) {
  Model* t = s->target;
  Model* d = s->draft;
  const int K = s->cfg.draft_k, S = s->streams;
  const int* Pp = &s->dstate[0].P;
  int rc;
  for (int i = 0; i < K; ++i) {
    if ((rc = model_forward(d, state_pos(s, i == 0 ? -2 : i - 1), i == 0 ? 2 : 1, S, 0, s->tok, s->max_seq, Pp, 1,
                            s->stream)))
      return rc;
    if (s->sampled() && s->cfg.draft_mode == VELLA_DRAFT_MODEL)
      rc = bf16_of(s) ? launch_draft_sample<__nv_bfloat16>(s, i) : launch_draft_sample<__half>(s, i);
    else
      rc = launch_kernel(propose_kernel, dim3(S), dim3(1), 0, s->stream, s->dstate, s->tok, (const int*)d->ys, i,
                         s->cfg.draft_mode, s->cfg.oracle_p, s->cfg.seed, (const int*)s->ref, t->cfg.vocab, s->max_seq);
    if (rc) return rc;
  }
  if ((rc = model_forward(t, state_pos(s, -1), K + 1, S, 0, s->tok, s->max_seq, Pp, K + 1, s->stream))) return rc;
  if (s->sampled())
    rc = bf16_of(s) ? launch_accept_sampled<__nv_bfloat16>(s) : launch_accept_sampled<__half>(s);
  else
    rc = launch_kernel(accept_kernel, dim3(S), dim3(1), 0, s->stream, s->dstate, s->tok, (const int*)t->ys, K,
                       (const int*)t->nonfinite, (const int*)t->err, (const int*)d->err, s->max_seq);
  if (rc) return rc;
  // the draft's own logits never gate acceptance; the verify flag was copied into the states
  VELLA_CUDA_TRY(cudaMemsetAsync(d->nonfinite, 0, sizeof(int), s->stream));
  VELLA_CUDA_TRY(cudaMemsetAsync(t->nonfinite, 0, sizeof(int), s->stream));
  return VELLA_OK;
}

int enqueue_greedy(Spec* s) {
  Model* t = s->target;
  int rc;
  if ((rc = model_forward(t, state_pos(s, -1), 1, s->streams, 0, s->tok, s->max_seq, &s->dstate[0].P, 1, s->stream)))
    return rc;
  if (s->sampled())
    rc = bf16_of(s) ? launch_sample_commit<__nv_bfloat16>(s, s->dstate, s->tok, s->streams, 0, 0)
                    : launch_sample_commit<__half>(s, s->dstate, s->tok, s->streams, 0, 0);
  else
    rc = launch_kernel(greedy_commit_kernel, dim3(s->streams), dim3(1), 0, s->stream, s->dstate, s->tok,
                       (const int*)t->ys, (const int*)t->nonfinite, (const int*)t->err, s->max_seq);
  if (rc) return rc;
  VELLA_CUDA_TRY(cudaMemsetAsync(t->nonfinite, 0, sizeof(int), s->stream));
  return VELLA_OK;
}

int capture(Spec* s, int (*enqueue)(Spec*), cudaGraphExec_t* exec) {
  VELLA_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue(s);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(s->stream, &g);
  if (rc != VELLA_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  const cudaError_t ie = cudaGraphInstantiate(exec, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate");
  return VELLA_OK;
}

// Runs one unit of work (pass or greedy step), eagerly the first time (kernel attributes
// are configured outside capture), then as a replayed graph.
int run_unit(Spec* s, bool pass) {
  int rc;
  bool& warm = pass ? s->pass_warm : s->greedy_warm;
  cudaGraphExec_t& exec = pass ? s->pass_exec : s->greedy_exec;
  int (*enqueue)(Spec*) = pass ? enqueue_pass : enqueue_greedy;
  if (!s->cfg.use_graphs || !warm) {
    if ((rc = enqueue(s))) return rc;
    warm = true;
  } else {
    if (!exec && (rc = capture(s, enqueue, &exec))) return rc;
    VELLA_CUDA_TRY(cudaGraphLaunch(exec, s->stream));
  }
  return sync_state(s);
}

// Prefill of every stream (one stream at a time), quota = 0 (no limit) or the batch quota.
int prefill_all(Spec* s, int quota) {
  if (s->P < 1) return fail(VELLA_E_INVALID, "prefill: the prefix is empty (vella_spec_set_prefix)");
  std::vector<DevState> init(s->streams);
  for (DevState& x : init) {
    std::memset(&x, 0, sizeof x);
    x.P = x.L = s->P;
    x.ref_len = s->ref_len;
    x.quota = quota;
  }
  VELLA_CUDA_TRY(cudaMemcpyAsync(s->dstate, init.data(), sizeof(DevState) * s->streams, cudaMemcpyHostToDevice,
                                 s->stream));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
  int rc;
  // Chunks of up to kChunkRows positions (tensor-core GEMMs), except the last kMaxRows
  // positions, which run as one small-M forward: the draft's first pass recomputes position
  // P - 1 with the small-M kernels, and a draft that shares the target's weights then holds
  // the target's KV rows bit for bit.
  const int tail = std::min(s->P, kMaxRows);
  Model* t = s->target;
  for (int j = 0; j < s->streams; ++j) {
    const int* Pp = &s->dstate[j].P;
    int* tk = s->tok + (size_t)j * s->max_seq;
    auto run = [&](Model* m, bool logits) -> int {
      int r;
      for (int s0 = 0; s0 < s->P - tail; s0 += kChunkRows) {
        const int rows = std::min(kChunkRows, s->P - tail - s0);
        if ((r = model_forward(m, PosRef{m->dzero, s0}, rows, 1, j, tk, 0, Pp, 0, s->stream))) return r;
      }
      return model_forward(m, PosRef{m->dzero, s->P - tail}, tail, 1, j, tk, 0, Pp, logits ? 1 : 0, s->stream);
    };
    if (s->draft && (rc = run(s->draft, false))) return rc;
    if ((rc = run(t, true))) return rc;
    if ((rc = launch_kernel(prefill_finish_kernel, dim3(1), dim3(1), 0, s->stream, &s->dstate[j], tk,
                            (const int*)t->ys, (const int*)t->nonfinite, (const int*)t->err, s->max_seq)))
      return rc;
    if (s->sampled() &&
        (rc = bf16_of(s) ? launch_sample_commit<__nv_bfloat16>(s, &s->dstate[j], tk, 1, 1, j)
                         : launch_sample_commit<__half>(s, &s->dstate[j], tk, 1, 1, j)))
      return rc;
  }
  VELLA_CUDA_TRY(cudaMemsetAsync(t->nonfinite, 0, sizeof(int), s->stream));
  VELLA_CUDA_TRY(cudaEventRecord(s->evp, s->stream));
  if ((rc = sync_state(s))) return rc;
  return pipeline_faults();
}

int prefill(Spec* s, int* first) {
  int rc;
  if ((rc = prefill_all(s, 0))) return rc;
  *first = s->hstate[0].newtok[0];
  return VELLA_OK;
}

bool is_eos(const Spec* s, int t) {
  for (int i = 0; i < s->cfg.n_eos && i < 8; ++i)
    if (s->cfg.eos[i] == t) return true;
  return false;
}

struct Decoded {
  std::vector<int> tokens;
  bool looped = false;
  bool capacity = false;
};

// decodeGreedy (reference :266-290).
int decode_greedy(Spec* s, int max_tokens, Decoded* out) {
  int y = 0, rc;
  if ((rc = prefill(s, &y))) return rc;
  while ((int)out->tokens.size() < max_tokens) {
    if (is_eos(s, y)) break;
    out->tokens.push_back(y);
    if (ends_in_loop(out->tokens)) {
      out->looped = true;
      break;
    }
    if ((int)out->tokens.size() >= max_tokens) break;
    if (s->hstate->L + 1 > s->max_seq) {
      out->capacity = true;
      break;
    }
    if ((rc = run_unit(s, false))) return rc;
    s->stats.greedy_steps++;
    y = s->hstate->newtok[0];
  }
  return VELLA_OK;
}

// decodeMTP (reference :306-396).
int decode_mtp(Spec* s, int max_tokens, Decoded* out) {
  int t = 0, rc;
  if ((rc = prefill(s, &t))) return rc;
  if (is_eos(s, t) || max_tokens == 0) return VELLA_OK;
  out->tokens.push_back(t);
  const int K = s->cfg.draft_k;
  while ((int)out->tokens.size() < max_tokens) {
    if (s->hstate->L + K + 1 > s->max_seq) {
      out->capacity = true;
      return VELLA_OK;
    }
    if ((rc = run_unit(s, true))) return rc;
    s->stats.passes++;
    const int n = s->hstate->n_new;
    if (n >= 1 && n <= 16) s->stats.accepted[n - 1]++;
    if (s->fault == VELLA_FAULT_THROW) return fail(VELLA_E_INVALID, "injected draft-and-verify fault");
    if (s->hstate->nonfinite || s->fault == VELLA_FAULT_NONFINITE) return fail(VELLA_E_NONFINITE, "non-finite logits");
    for (int j = 0; j < n; ++j) {
      const int tk = s->hstate->newtok[j];
      if (is_eos(s, tk)) return VELLA_OK;
      out->tokens.push_back(tk);
      if ((int)out->tokens.size() >= max_tokens) return VELLA_OK;
      if (ends_in_loop(out->tokens)) {
        out->looped = true;
        return VELLA_OK;
      }
    }
  }
  return VELLA_OK;
}

}  // namespace
}  // namespace vella

using namespace vella;

struct vella_model : Model {};
struct vella_spec : Spec {};

extern "C" {

int vella_quantize(const vella_qgemm_desc* desc, int32_t src_dtype, const void* w, void* packed, void* scales,
                   void* biases, vella_stream_t stream) {
  last_error_slot().clear();
  if (!desc || !w || !packed || !scales || !biases) return fail(VELLA_E_INVALID, "vella_quantize: NULL argument");
  const vella_qgemm_desc& d = *desc;
  if ((d.bits != 4 && d.bits != 8) || d.group_size != 64 || d.n <= 0 || d.k <= 0 || d.k % 64 ||
      (d.dtype != VELLA_BF16 && d.dtype != VELLA_F16) ||
      (src_dtype != VELLA_F32 && src_dtype != VELLA_BF16 && src_dtype != VELLA_F16))
    return fail(VELLA_E_UNSUPPORTED, "vella_quantize: n=%d k=%d bits=%d group=%d dtype=%d src=%d", d.n, d.k, d.bits,
                d.group_size, d.dtype, src_dtype);
  if (!aligned(packed, 4) || !aligned(scales, 2) || !aligned(biases, 2) || !aligned(w, src_dtype == VELLA_F32 ? 4 : 2))
    return fail(VELLA_E_INVALID, "vella_quantize: misaligned pointer");
  return quantize_device(src_dtype, w, d.dtype, d.bits, d.n, d.k, packed, scales, biases,
                         static_cast<cudaStream_t>(stream));
}

int vella_fill_normal(void* out, size_t n, int32_t dtype, uint64_t seed, uint32_t tensor, float mean, float std,
                      vella_stream_t stream) {
  last_error_slot().clear();
  if (!out && n) return fail(VELLA_E_INVALID, "vella_fill_normal: out is NULL");
  return fill_normal(out, n, dtype, seed, tensor, mean, std, static_cast<cudaStream_t>(stream));
}

int vella_model_create(const vella_model_cfg* cfg, int32_t device, vella_model** out) {
  last_error_slot().clear();
  if (!cfg || !out) return fail(VELLA_E_INVALID, "vella_model_create: NULL argument");
  Model* m = nullptr;
  const int rc = model_create(*cfg, device, &m);
  if (rc) return rc;
  *out = static_cast<vella_model*>(m);
  return VELLA_OK;
}

int vella_model_destroy(vella_model* model) {
  model_destroy(model);
  return VELLA_OK;
}

int vella_model_init_random(vella_model* model, uint64_t seed, float std) {
  last_error_slot().clear();
  if (!model) return fail(VELLA_E_INVALID, "vella_model_init_random: NULL model");
  VELLA_CUDA_TRY(cudaSetDevice(model->device));
  return model_init_random(model, seed, std, model->stream);
}

int vella_model_tensor(vella_model* model, const char* name, int32_t layer, void** ptr, size_t* bytes) {
  last_error_slot().clear();
  if (!model || !name || !ptr || !bytes) return fail(VELLA_E_INVALID, "vella_model_tensor: NULL argument");
  return model_tensor(model, name, layer, ptr, bytes);
}

size_t vella_model_weight_bytes(const vella_model* model) { return model ? model->arena_bytes : 0; }

int vella_model_score(vella_model* m, const void* prefix, int32_t P, const int32_t* tokens, int32_t T,
                      void* logits_out, int32_t on_host) {
  last_error_slot().clear();
  if (!m || !logits_out || (T > 0 && !tokens)) return fail(VELLA_E_INVALID, "vella_model_score: NULL argument");
  const vella_model_cfg& c = m->cfg;
  if (P < 1 || P > c.max_prefix || T < 1 || P + T - 1 > c.max_seq)
    return fail(VELLA_E_INVALID, "vella_model_score: P=%d T=%d (max_prefix %d, max_seq %d)", P, T, c.max_prefix, c.max_seq);
  VELLA_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t s = m->stream;
  const size_t row = (size_t)c.d_model * m->elt;
  if (prefix)
    VELLA_CUDA_TRY(cudaMemcpyAsync(m->prefix, prefix, (size_t)P * row,
                                   on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(m->score_tok + P, tokens, (size_t)T * sizeof(int), cudaMemcpyHostToDevice, s));
  VELLA_CUDA_TRY(cudaMemcpyAsync(m->score_P, &P, sizeof(int), cudaMemcpyHostToDevice, s));
  const int last_pos = P + T - 2;  // the last position whose logits are needed
  const size_t lrow = (size_t)c.vocab * m->elt;
  int rc;
  for (int s0 = 0; s0 <= last_pos; s0 += kMaxRows) {
    const int rows = std::min(kMaxRows, last_pos + 1 - s0);
    const int first_scored = std::max(s0, P - 1);
    const int lr = s0 + rows - first_scored;  // rows with position >= P - 1
    if ((rc = model_forward(m, PosRef{m->dzero, s0}, rows, 1, 0, m->score_tok, 0, m->score_P, std::max(lr, 0), s)))
      return rc;
    if (lr > 0) {
      char* dst = static_cast<char*>(logits_out) + (size_t)(first_scored - (P - 1)) * lrow;
      VELLA_CUDA_TRY(cudaMemcpyAsync(dst, m->logits, (size_t)lr * lrow,
                                     on_host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s));
    }
  }
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  int err = 0;
  VELLA_CUDA_TRY(cudaMemcpy(&err, m->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return fail(VELLA_E_INVALID, "vella_model_score: error flags 0x%x (token id out of range?)", err);
  return VELLA_OK;
}

int vella_spec_create(vella_model* target, vella_model* draft, const vella_spec_cfg* cfg, vella_spec** out) {
  last_error_slot().clear();
  if (!target || !cfg || !out) return fail(VELLA_E_INVALID, "vella_spec_create: NULL argument");
  if (draft) {
    if (draft->cfg.vocab != target->cfg.vocab || draft->cfg.dtype != target->cfg.dtype)
      return fail(VELLA_E_INVALID, "vella_spec_create: draft and target must share vocabulary and dtype");
    if (draft->cfg.max_seq < target->cfg.max_seq || draft->device != target->device)
      return fail(VELLA_E_INVALID, "vella_spec_create: the draft needs max_seq >= the target's, on the same device");
    if (draft->streams != target->streams)
      return fail(VELLA_E_INVALID, "vella_spec_create: draft and target must hold the same number of streams");
  }
  if (cfg->draft_k < 1 || cfg->draft_k + 1 > kMaxRows)
    return fail(VELLA_E_UNSUPPORTED, "vella_spec_create: draft_k %d (1..%d)", cfg->draft_k, kMaxRows - 1);
  if (cfg->n_eos < 0 || cfg->n_eos > 8) return fail(VELLA_E_INVALID, "vella_spec_create: n_eos %d", cfg->n_eos);
  if (!(cfg->temperature >= 0.0f)) return fail(VELLA_E_INVALID, "vella_spec_create: temperature %g", cfg->temperature);
  VELLA_CUDA_TRY(cudaSetDevice(target->device));
  vella_spec* s = new vella_spec();
  s->target = target;
  s->draft = draft;
  s->cfg = *cfg;
  s->device = target->device;
  s->max_seq = target->cfg.max_seq;
  s->streams = target->streams;
  const size_t S = (size_t)s->streams;
  int rc = VELLA_OK;
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == VELLA_OK) rc = cuda_fail(e, what);
  };
  cuda(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda(cudaMalloc(&s->dstate, S * sizeof(DevState)), "cudaMalloc(state)");
  cuda(cudaMallocHost(&s->hstate, S * sizeof(DevState)), "cudaMallocHost(state)");
  cuda(cudaMalloc(&s->tok, S * s->max_seq * sizeof(int)), "cudaMalloc(tokens)");
  cuda(cudaMalloc(&s->ref, S * s->max_seq * sizeof(int)), "cudaMalloc(reference)");
  if (cfg->temperature > 0.0f && cfg->draft_mode == VELLA_DRAFT_MODEL && draft) {
    cuda(cudaMalloc(&s->qrows, (size_t)cfg->draft_k * S * target->cfg.vocab * target->elt), "cudaMalloc(draft rows)");
    cuda(cudaMalloc(&s->qstats, (size_t)cfg->draft_k * S * sizeof(float2)), "cudaMalloc(draft stats)");
  }
  cuda(cudaEventCreate(&s->ev0), "cudaEventCreate");
  cuda(cudaEventCreate(&s->ev1), "cudaEventCreate");
  cuda(cudaEventCreate(&s->evp), "cudaEventCreate");
  if (rc == VELLA_OK) {
    std::memset(s->hstate, 0, S * sizeof(DevState));
    cuda(cudaMemset(s->dstate, 0, S * sizeof(DevState)), "cudaMemset");
    cuda(cudaMemset(s->tok, 0, S * s->max_seq * sizeof(int)), "cudaMemset");
  }
  if (rc != VELLA_OK) {
    vella_spec_destroy(s);
    return rc;
  }
  *out = s;
  return VELLA_OK;
}

int vella_spec_destroy(vella_spec* s) {
  if (!s) return VELLA_OK;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  if (s->pass_exec) cudaGraphExecDestroy(s->pass_exec);
  if (s->greedy_exec) cudaGraphExecDestroy(s->greedy_exec);
  if (s->dstate) cudaFree(s->dstate);
  if (s->hstate) cudaFreeHost(s->hstate);
  if (s->tok) cudaFree(s->tok);
  if (s->ref) cudaFree(s->ref);
  if (s->qrows) cudaFree(s->qrows);
  if (s->qstats) cudaFree(s->qstats);
  if (s->ev0) cudaEventDestroy(s->ev0);
  if (s->ev1) cudaEventDestroy(s->ev1);
  if (s->evp) cudaEventDestroy(s->evp);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
  return VELLA_OK;
}

int vella_spec_set_prefix(vella_spec* s, const void* target_embeds, const void* draft_embeds, int32_t T,
                          int32_t on_host) {
  last_error_slot().clear();
  if (!s) return fail(VELLA_E_INVALID, "vella_spec_set_prefix: NULL spec");
  if (T < 1 || T > s->target->cfg.max_prefix || (s->draft && T > s->draft->cfg.max_prefix))
    return fail(VELLA_E_INVALID, "vella_spec_set_prefix: T=%d exceeds max_prefix", T);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  const cudaMemcpyKind kind = on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  // [streams][T][d] into each stream's prefix slot ([streams][max_prefix][d])
  auto put = [&](Model* m, const void* src) -> int {
    const size_t row = (size_t)T * m->cfg.d_model * m->elt;
    VELLA_CUDA_TRY(cudaMemcpy2DAsync(m->prefix, (size_t)m->prefix_ss * m->elt, src, row, row, (size_t)s->streams, kind,
                                     s->stream));
    return VELLA_OK;
  };
  int rc;
  if (target_embeds && (rc = put(s->target, target_embeds))) return rc;
  if (s->draft && draft_embeds && (rc = put(s->draft, draft_embeds))) return rc;
  VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
  s->P = T;
  return VELLA_OK;
}

int vella_spec_set_reference(vella_spec* s, const int32_t* tokens, int32_t n) {
  last_error_slot().clear();
  if (!s || (n > 0 && !tokens)) return fail(VELLA_E_INVALID, "vella_spec_set_reference: NULL argument");
  if (n < 0 || n > s->max_seq) return fail(VELLA_E_INVALID, "vella_spec_set_reference: n=%d", n);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  if (n)
    VELLA_CUDA_TRY(cudaMemcpy2DAsync(s->ref, (size_t)s->max_seq * sizeof(int), tokens, (size_t)n * sizeof(int),
                                     (size_t)n * sizeof(int), (size_t)s->streams, cudaMemcpyHostToDevice, s->stream));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
  s->ref_len = n;
  return VELLA_OK;
}

int vella_spec_prefill(vella_spec* s, int32_t* first) {
  last_error_slot().clear();
  if (!s || !first) return fail(VELLA_E_INVALID, "vella_spec_prefill: NULL argument");
  if (s->streams != 1) return fail(VELLA_E_UNSUPPORTED, "vella_spec_prefill: %d streams (use vella_spec_decode_batch)", s->streams);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  return prefill(s, first);
}

int vella_spec_step(vella_spec* s, int32_t* out_tokens, int32_t* n_out) {
  last_error_slot().clear();
  if (!s || !out_tokens || !n_out) return fail(VELLA_E_INVALID, "vella_spec_step: NULL argument");
  if (!s->draft) return fail(VELLA_E_UNSUPPORTED, "vella_spec_step: no draft model");
  if (s->hstate->L < s->P + 1) return fail(VELLA_E_INVALID, "vella_spec_step: prefill first");
  if (s->hstate->L + s->cfg.draft_k + 1 > s->max_seq) return fail(VELLA_E_INVALID, "vella_spec_step: KV capacity reached");
  if (s->streams != 1) return fail(VELLA_E_UNSUPPORTED, "vella_spec_step: %d streams (use vella_spec_decode_batch)", s->streams);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  const int rc = run_unit(s, true);
  if (rc) return rc;
  s->stats.passes++;
  const int n = s->hstate->n_new;
  if (n >= 1 && n <= 16) s->stats.accepted[n - 1]++;
  *n_out = n;
  for (int j = 0; j < n; ++j) out_tokens[j] = s->hstate->newtok[j];
  if (s->hstate->nonfinite) return fail(VELLA_E_NONFINITE, "non-finite logits in the verify pass");
  return VELLA_OK;
}

int vella_spec_greedy_step(vella_spec* s, int32_t* out_token) {
  last_error_slot().clear();
  if (!s || !out_token) return fail(VELLA_E_INVALID, "vella_spec_greedy_step: NULL argument");
  if (s->hstate->L < s->P + 1) return fail(VELLA_E_INVALID, "vella_spec_greedy_step: prefill first");
  if (s->hstate->L + 1 > s->max_seq) return fail(VELLA_E_INVALID, "vella_spec_greedy_step: KV capacity reached");
  if (s->streams != 1) return fail(VELLA_E_UNSUPPORTED, "vella_spec_greedy_step: %d streams (use vella_spec_decode_batch)", s->streams);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  const int rc = run_unit(s, false);
  if (rc) return rc;
  s->stats.greedy_steps++;
  *out_token = s->hstate->newtok[0];
  if (s->hstate->nonfinite) return fail(VELLA_E_NONFINITE, "non-finite logits");
  return VELLA_OK;
}

int vella_spec_decode(vella_spec* s, int32_t mode, int32_t max_tokens, int32_t* out_tokens, int32_t cap,
                      int32_t* n_out, int32_t* flags) {
  last_error_slot().clear();
  if (!s || !n_out || !flags || (cap > 0 && !out_tokens)) return fail(VELLA_E_INVALID, "vella_spec_decode: NULL argument");
  if (max_tokens < 0) return fail(VELLA_E_INVALID, "vella_spec_decode: max_tokens < 0");
  if (s->streams != 1) return fail(VELLA_E_UNSUPPORTED, "vella_spec_decode: %d streams (use vella_spec_decode_batch)", s->streams);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  *flags = 0;
  Decoded result;
  int rc = VELLA_OK;
  VELLA_CUDA_TRY(cudaEventRecord(s->ev0, s->stream));
  const bool spec_ok = s->draft != nullptr && !s->draft_disabled;
  if (mode == VELLA_DECODE_SPEC) {
    if (!s->draft) return fail(VELLA_E_UNSUPPORTED, "vella_spec_decode: no draft model");
    rc = decode_mtp(s, max_tokens, &result);
  } else if (mode == VELLA_DECODE_GREEDY || !spec_ok) {
    rc = decode_greedy(s, max_tokens, &result);
    if (rc == VELLA_OK && (int)result.tokens.size() >= max_tokens) result.looped = true;
  } else {
    // decode(): draft-and-verify with runaway retry; a runtime failure falls back to greedy, sticky.
    rc = decode_mtp(s, max_tokens, &result);
    if (rc == VELLA_OK && (result.looped || (int)result.tokens.size() >= max_tokens)) {
      s->stats.runaway_retries++;
      *flags |= VELLA_FLAG_RUNAWAY_RETRY;
      result = Decoded();
      rc = decode_greedy(s, max_tokens, &result);
      if (rc == VELLA_OK && (int)result.tokens.size() >= max_tokens) result.looped = true;
    } else if (rc != VELLA_OK && rc != VELLA_E_OOM) {
      s->failure = last_error_slot();
      s->draft_disabled = true;
      s->stats.fallbacks++;
      *flags |= VELLA_FLAG_FELL_BACK;
      VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
      result = Decoded();
      last_error_slot().clear();
      rc = decode_greedy(s, max_tokens, &result);
      if (rc == VELLA_OK && (int)result.tokens.size() >= max_tokens) result.looped = true;
    }
  }
  VELLA_CUDA_TRY(cudaEventRecord(s->ev1, s->stream));
  VELLA_CUDA_TRY(cudaEventSynchronize(s->ev1));
  float ms = 0.0f, pms = 0.0f;
  cudaEventElapsedTime(&pms, s->ev0, s->evp);
  cudaEventElapsedTime(&ms, s->evp, s->ev1);
  s->stats.last_decode_ms = ms;
  s->stats.last_prefill_ms = pms;
  if (rc != VELLA_OK) return rc;
  if ((rc = pipeline_faults())) return rc;
  if (result.looped) *flags |= VELLA_FLAG_LOOPED;
  if (result.capacity) *flags |= VELLA_FLAG_CAPACITY;
  const int n = (int)result.tokens.size();
  *n_out = n;
  s->stats.last_tokens = n;
  for (int i = 0; i < std::min(n, cap); ++i) out_tokens[i] = result.tokens[i];
  return VELLA_OK;
}

int vella_spec_decode_batch(vella_spec* s, int32_t mode, int32_t max_tokens, int32_t* out_tokens, int32_t* n_out) {
  last_error_slot().clear();
  if (!s || !out_tokens || !n_out) return fail(VELLA_E_INVALID, "vella_spec_decode_batch: NULL argument");
  if (mode != VELLA_DECODE_SPEC && mode != VELLA_DECODE_GREEDY)
    return fail(VELLA_E_INVALID, "vella_spec_decode_batch: mode %d (SPEC or GREEDY)", mode);
  if (mode == VELLA_DECODE_SPEC && !s->draft) return fail(VELLA_E_UNSUPPORTED, "vella_spec_decode_batch: no draft model");
  const int K = s->cfg.draft_k;
  if (max_tokens < 1 || s->P + max_tokens + K + 1 > s->max_seq)
    return fail(VELLA_E_INVALID, "vella_spec_decode_batch: prefix %d + %d tokens (+%d) exceed max_seq %d", s->P,
                max_tokens, K + 1, s->max_seq);
  VELLA_CUDA_TRY(cudaSetDevice(s->device));
  VELLA_CUDA_TRY(cudaEventRecord(s->ev0, s->stream));
  int rc;
  if ((rc = prefill_all(s, max_tokens))) return rc;
  const bool spec = mode == VELLA_DECODE_SPEC;
  for (;;) {
    bool all = true;
    for (int j = 0; j < s->streams; ++j) {
      if (s->hstate[j].nonfinite) return fail(VELLA_E_NONFINITE, "non-finite logits in stream %d", j);
      all = all && s->hstate[j].produced >= max_tokens;
    }
    if (all) break;
    if ((rc = run_unit(s, spec))) return rc;
    if (spec) {
      s->stats.passes++;
      for (int j = 0; j < s->streams; ++j) {
        const int n = s->hstate[j].n_new;
        if (n >= 1 && n <= 16) s->stats.accepted[n - 1]++;
      }
    } else {
      s->stats.greedy_steps++;
    }
  }
  VELLA_CUDA_TRY(cudaEventRecord(s->ev1, s->stream));
  VELLA_CUDA_TRY(cudaMemcpy2DAsync(out_tokens, (size_t)max_tokens * sizeof(int), s->tok + s->P,
                                   (size_t)s->max_seq * sizeof(int), (size_t)max_tokens * sizeof(int),
                                   (size_t)s->streams, cudaMemcpyDeviceToHost, s->stream));
  VELLA_CUDA_TRY(cudaStreamSynchronize(s->stream));
  float ms = 0.0f, pms = 0.0f;
  cudaEventElapsedTime(&pms, s->ev0, s->evp);
  cudaEventElapsedTime(&ms, s->evp, s->ev1);
  s->stats.last_decode_ms = ms;
  s->stats.last_prefill_ms = pms;
  s->stats.last_tokens = max_tokens * s->streams;
  for (int j = 0; j < s->streams; ++j) n_out[j] = max_tokens;
  return pipeline_faults();
}

int vella_spec_get_stats(const vella_spec* s, vella_spec_stats* out) {
  if (!s || !out) return fail(VELLA_E_INVALID, "vella_spec_get_stats: NULL argument");
  *out = s->stats;
  out->draft_disabled = s->draft_disabled ? 1 : 0;
  return VELLA_OK;
}

int vella_spec_set_fault(vella_spec* s, int32_t fault) {
  if (!s) return fail(VELLA_E_INVALID, "vella_spec_set_fault: NULL spec");
  s->fault = fault;
  return VELLA_OK;
}

int vella_spec_reset(vella_spec* s) {
  if (!s) return fail(VELLA_E_INVALID, "vella_spec_reset: NULL spec");
  s->draft_disabled = false;
  s->failure.clear();
  s->stats = vella_spec_stats{};
  return VELLA_OK;
}

}  // extern "C"
