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
#include <cooperative_groups.h>
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
  int mm[2 * kSampThreads / 32];  // block_minmax's warp values
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

// Inclusive prefix sums of one value per thread over the block (warp shuffles, then the warp
// totals: a fixed order), and the block total.
__device__ float block_incl_scan(float v, SampShared& sh, float* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (int)(blockDim.x >> 5);
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();  // sh.red is free
  if (lane == 31) sh.red[w] = x;
  __syncthreads();
  if (w == 0) {
    float t = lane < nw ? sh.red[lane] : 0.0f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) sh.red[lane] = t;
  }
  __syncthreads();
  *total = sh.red[nw - 1];
  return x + (w > 0 ? sh.red[w - 1] : 0.0f);
}

// Block-wide min of a (first) and max of b (second) over the threads.
__device__ int2 block_minmax(int a, int b, SampShared& sh) {
  int* scratch = sh.mm;
  a = __reduce_min_sync(0xffffffffu, a);
  b = __reduce_max_sync(0xffffffffu, b);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    scratch[2 * (threadIdx.x >> 5)] = a;
    scratch[2 * (threadIdx.x >> 5) + 1] = b;
  }
  __syncthreads();
  int2 r = make_int2(0x7fffffff, -1);
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    r.x = min(r.x, scratch[2 * w]);
    r.y = max(r.y, scratch[2 * w + 1]);
  }
  return r;
}

// Index drawn from the unnormalised weights w(0..V) with the uniform u: thread t owns the
// contiguous range [t C, (t+1) C); the thread sums are prefix-summed in a fixed order (warp
// shuffles, then the warp totals), the first thread whose running sum passes u * total scans
// its range in vocabulary order.  The result depends only on the weights and u.  -1 when
// every weight is zero.
template <typename W>
__device__ int sample_icdf(W w, int V, float u, SampShared& sh) {
  const int C = (V + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = min(V, (int)threadIdx.x * C), hi = min(V, lo + C);
  float ps = 0.0f;
  for (int v = lo; v < hi; ++v) ps += w(v);
  float total;
  const float incl = block_incl_scan(ps, sh, &total);
  const float target = u * total;
  // the first thread whose running sum passes the target, else the last with weight
  const int2 mm = block_minmax(incl > target ? (int)threadIdx.x : 0x7fffffff, ps > 0.0f ? (int)threadIdx.x : -1, sh);
  if (mm.y < 0) return -1;
  const bool found_seg = mm.x != 0x7fffffff;
  const int tseg = found_seg ? mm.x : mm.y;
  if ((int)threadIdx.x == tseg) {
    float a = found_seg ? incl - ps : -1.0f;
    int found = -1, lastv = -1;
    for (int v = lo; v < hi; ++v) {
      const float x = w(v);
      if (x > 0.0f) lastv = v;
      if (found < 0 && a >= 0.0f && a + x > target) found = v;
      a += x;
    }
    sh.idx = found >= 0 ? found : lastv;
  }
  __syncthreads();
  return sh.idx;
}

// ---- vocabulary sweeps split over a cluster (tree expansion and acceptance) --------------
// A cluster of kTreeCluster CTAs shares one sweep: CTA rank r owns the contiguous range
// [r VC, (r + 1) VC) of the vocabulary.  Each reduction combines one value per CTA, read
// through distributed shared memory in rank order, so every CTA of the cluster gets the same
// value whatever the scheduling, and every decision taken from it is uniform across the
// cluster.  Exchange slots alternate: a slot is written again only after a later cluster
// barrier, which every CTA reaches only once it has read the slot.
constexpr int kTreeCluster = 8;
namespace cg = cooperative_groups;

struct ClSweep {
  cg::cluster_group g;
  int rank, lo, hi;  // this CTA's vocabulary range
  int k;             // reductions so far
  float* xch;        // [2] exchange slots in this CTA's shared memory
  int* xidx;         // the index an inverse-CDF draw found (on the CTA that found it)
  __device__ ClSweep(int V, float* x, int* xi) : g(cg::this_cluster()), k(0), xch(x), xidx(xi) {
    rank = (int)g.block_rank();
    const int VC = (V + kTreeCluster - 1) / kTreeCluster;
    lo = min(V, rank * VC);
    hi = min(V, lo + VC);
  }
  // v: this CTA's value (the same in all its threads); returns the max or the sum over ranks
  __device__ float combine(float v, bool is_max) {
    const int slot = k++ & 1;
    if (threadIdx.x == 0) xch[slot] = v;
    g.sync();
    float r = is_max ? -INFINITY : 0.0f;
    for (int i = 0; i < kTreeCluster; ++i) {
      const float x = *g.map_shared_rank(xch + slot, i);
      r = is_max ? fmaxf(r, x) : r + x;
    }
    return r;
  }
};

// (max, sum of exp((l - max) / T)) of one logits row, over the cluster; the CTA's part of the
// row is its slice (row entries lo .. hi - 1, staged in shared memory).
template <typename T>
__device__ float2 cl_softmax_stats(ClSweep& c, const T* slice, float invT, SampShared& sh) {
  const int n = c.hi - c.lo;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, Act<T>::to_f(slice[i]));
  m = c.combine(block_max(m, sh), true);
  float z = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) z += expf((Act<T>::to_f(slice[i]) - m) * invT);
  z = c.combine(block_sum(z, sh), false);
  return make_float2(m, z);
}

// Copies n elements from src to dst with 16-byte accesses when both are 16-byte aligned (the
// whole block, coalesced), element by element otherwise.
template <typename T>
__device__ __forceinline__ void block_copy(T* dst, const T* src, int n) {
  constexpr int E = 16 / sizeof(T);
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
    const int nv = n / E;
    for (int i = threadIdx.x; i < nv; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    for (int i = nv * E + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// The CTA's part of a row into shared memory (coalesced loads); the caller syncs.
template <typename T>
__device__ __forceinline__ void stage_slice(const ClSweep& c, const T* row, T* slice) {
  block_copy(slice, row + c.lo, c.hi - c.lo);
}
// Dynamic shared memory of the cluster kernels: one CTA's slice of a vocabulary row.
inline size_t cl_slice_bytes(int V, size_t elt) { return (size_t)((V + kTreeCluster - 1) / kTreeCluster) * elt; }

// Index drawn from the unnormalised weights w(0..V) with the uniform u, over the cluster:
// within a CTA each thread sums a contiguous slice, the slices are prefix-summed in a fixed
// order; the CTA totals are scanned in rank order, then the owning CTA finds the first thread
// whose running sum passes the target and that thread its range in vocabulary order.  -1 when
// every weight is zero.
template <typename W>
__device__ int cl_icdf(ClSweep& c, W w, float u, SampShared& sh) {
  const int n = c.hi - c.lo;
  const int C = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = c.lo + min(n, (int)threadIdx.x * C), hi = min(c.hi, lo + C);
  float ps = 0.0f;
  for (int v = lo; v < hi; ++v) ps += w(v);
  float cta_total;
  const float incl = block_incl_scan(ps, sh, &cta_total);
  // the CTA totals, in rank order
  const int slot = c.k++ & 1;
  if (threadIdx.x == 0) c.xch[slot] = cta_total;
  c.g.sync();
  float tots[kTreeCluster];
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < kTreeCluster; ++i) {
    tots[i] = *c.g.map_shared_rank(c.xch + slot, i);
    total += tots[i];
  }
  const float target = u * total;
  float acc = 0.0f, before = -1.0f;
  int seg = -1, last = -1;
#pragma unroll
  for (int i = 0; i < kTreeCluster; ++i) {
    if (tots[i] > 0.0f) last = i;
    if (seg < 0 && acc + tots[i] > target) {
      seg = i;
      before = acc;
    }
    acc += tots[i];
  }
  if (seg < 0) seg = last;  // rounding at the top end (before -1: the last weight of that CTA)
  if (seg < 0) return -1;   // every weight is zero (the same verdict on every CTA)
  if (c.rank == seg) {
    // the first thread whose running sum passes the target, else the last with weight
    const bool hit = before >= 0.0f && before + incl > target;
    const int2 mm = block_minmax(hit ? (int)threadIdx.x : 0x7fffffff, ps > 0.0f ? (int)threadIdx.x : -1, sh);
    const bool found_seg = mm.x != 0x7fffffff;
    const int tseg = found_seg ? mm.x : mm.y;
    if ((int)threadIdx.x == tseg) {
      float a = found_seg ? before + incl - ps : -1.0f;
      int found = -1, lastv = -1;
      for (int v = lo; v < hi; ++v) {
        const float x = w(v);
        if (x > 0.0f) lastv = v;
        if (found < 0 && a >= 0.0f && a + x > target) found = v;
        a += x;
      }
      *c.xidx = found >= 0 ? found : lastv;
    }
  }
  c.g.sync();
  return *c.g.map_shared_rank(c.xidx, seg);
}

// nd draws from the same unnormalised weights with the uniforms u[0..nd) (nd <= 16): the
// per-thread sums, the block scan and the CTA totals are formed once, then each draw finds its
// index exactly as cl_icdf does (the same values in the same order), the finds of all draws
// behind one cluster barrier.  out[d] is -1 when every weight is zero; xidx: nd ints of this
// CTA's shared memory.
template <typename W>
__device__ void cl_icdf_many(ClSweep& c, W w, const float* u, int nd, int* xidx, int* out, SampShared& sh) {
  const int n = c.hi - c.lo;
  const int C = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = c.lo + min(n, (int)threadIdx.x * C), hi = min(c.hi, lo + C);
  float ps = 0.0f;
  for (int v = lo; v < hi; ++v) ps += w(v);
  float cta_total;
  const float incl = block_incl_scan(ps, sh, &cta_total);
  const int slot = c.k++ & 1;
  if (threadIdx.x == 0) c.xch[slot] = cta_total;
  c.g.sync();
  float tots[kTreeCluster];
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < kTreeCluster; ++i) {
    tots[i] = *c.g.map_shared_rank(c.xch + slot, i);
    total += tots[i];
  }
  int segs[16];
  for (int d = 0; d < nd; ++d) {
    const float target = u[d] * total;
    float acc = 0.0f, before = -1.0f;
    int seg = -1, last = -1;
#pragma unroll
    for (int i = 0; i < kTreeCluster; ++i) {
      if (tots[i] > 0.0f) last = i;
      if (seg < 0 && acc + tots[i] > target) {
        seg = i;
        before = acc;
      }
      acc += tots[i];
    }
    if (seg < 0) seg = last;  // rounding at the top end (before -1: the last weight of that CTA)
    segs[d] = seg;
    if (seg >= 0 && c.rank == seg) {
      const bool hit = before >= 0.0f && before + incl > target;
      const int2 mm = block_minmax(hit ? (int)threadIdx.x : 0x7fffffff, ps > 0.0f ? (int)threadIdx.x : -1, sh);
      const bool found_seg = mm.x != 0x7fffffff;
      const int tseg = found_seg ? mm.x : mm.y;
      if ((int)threadIdx.x == tseg) {
        float a = found_seg ? before + incl - ps : -1.0f;
        int found = -1, lastv = -1;
        for (int v = lo; v < hi; ++v) {
          const float x = w(v);
          if (x > 0.0f) lastv = v;
          if (found < 0 && a >= 0.0f && a + x > target) found = v;
          a += x;
        }
        xidx[d] = found >= 0 ? found : lastv;
      }
    }
  }
  c.g.sync();
  for (int d = 0; d < nd; ++d) out[d] = segs[d] < 0 ? -1 : *c.g.map_shared_rank(xidx + d, segs[d]);
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

// ---- tree drafting and verification ---------------------------------------------------------
constexpr uint32_t kPurposeTree = 0x7EE01u;
constexpr int kTreeMaxDepth = 8;

struct TreeTopo {
  int nodes, depth;
  int level_start[kTreeMaxDepth + 2];  // first node of each depth; level_start[depth + 1] = nodes
  const int* dep;                      // [nodes]
  const int* first_child;              // [nodes]
  const int* n_child;                  // [nodes]
};

// One model's KV cache as the compaction sees it: per stream (kv_ss apart) and layer, a K and a
// V plane of kv_heads blocks [max_seq][hd].
template <typename T>
struct KvPlanes {
  T* kv;
  long long kv_ss;
  int layers, kv_heads, max_seq, hd;
};

// The whole block moves the K/V rows of stream s's accepted path (slots root + path[j - 1]) to
// consecutive slots root + j, j = 1..a, in every layer and head; ascending j, one barrier per
// j: a source is never an earlier destination (a node of depth j sits at slot >= root + j).
template <typename T>
__device__ void compact_path(const KvPlanes<T>& p, int s, int root, int a, const int* path, int part = 0,
                             int parts = 1) {
  const size_t plane = (size_t)p.kv_heads * p.max_seq * p.hd;
  T* base = p.kv + (size_t)s * p.kv_ss;
  const int blocks = p.layers * 2 * p.kv_heads;  // (layer, K|V, head) blocks
  const bool vec = (p.hd * (int)sizeof(T)) % 16 == 0;
  const int per_row = vec ? p.hd * (int)sizeof(T) / 16 : p.hd;
  for (int j = 1; j <= a; ++j) {
    const int src = root + path[j - 1], dst = root + j;
    if (src != dst && src < p.max_seq && dst < p.max_seq)
      for (int e = part * blockDim.x + threadIdx.x; e < blocks * per_row; e += parts * blockDim.x) {
        const int b = e / per_row, c = e % per_row;
        T* blk = base + (size_t)(b / p.kv_heads) * plane + (size_t)(b % p.kv_heads) * p.max_seq * p.hd;
        if (vec)
          reinterpret_cast<uint4*>(blk + (size_t)dst * p.hd)[c] = reinterpret_cast<const uint4*>(blk + (size_t)src * p.hd)[c];
        else
          blk[(size_t)dst * p.hd + c] = blk[(size_t)src * p.hd + c];
      }
    __syncthreads();
  }
}

__global__ void tree_root_kernel(const DevState* st, const int* tok, int* ttok, unsigned char* onpath, int N,
                                 int max_seq) {
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x;
  ttok[(size_t)s * N] = tok[(size_t)s * max_seq + st[s].L - 1];
  onpath[(size_t)s * N] = 1;
}

// Block argmax over v in [0, V) excluding `skip[0..n)`, lowest index on ties.
template <typename T>
__device__ int block_argmax_excl(const T* row, int V, const int* skip, int n, SampShared& sh) {
  float bv = -INFINITY;
  int bi = INT32_MAX;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    bool ex = false;
    for (int j = 0; j < n; ++j) ex |= skip[j] == v;
    if (ex) continue;
    const float x = Act<T>::to_f(row[v]);
    if (x > bv || (x == bv && v < bi)) { bv = x; bi = v; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    sh.part[threadIdx.x >> 5] = bv;
    sh.red[threadIdx.x >> 5] = __int_as_float(bi);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v0 = -INFINITY;
    int i0 = INT32_MAX;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      const float ov = sh.part[w];
      const int oi = __float_as_int(sh.red[w]);
      if (ov > v0 || (ov == v0 && oi < i0)) { v0 = ov; i0 = oi; }
    }
    sh.idx = i0 == INT32_MAX ? 0 : i0;
  }
  __syncthreads();
  return sh.idx;
}

// Children of the nodes at `depth` (one cluster = one node of one stream): the draft's logits
// row of the node (row blockIdx.x / kTreeCluster of the stream's rows at this depth) gives
// them.  The sampled form sweeps the vocabulary over the cluster; the greedy and oracle forms
// run on the cluster's first CTA.
template <typename T>
__global__ void __cluster_dims__(kTreeCluster, 1, 1) __launch_bounds__(kSampThreads)
    tree_expand_kernel(const DevState* st, const T* logits, int depth, TreeTopo tt, vella_spec_cfg_dev c,
                       const int* ref, int* ttok, unsigned char* onpath, int vocab, int max_seq, T* qrows,
                       float2* qstats, int S) {
  __shared__ SampShared sh;
  __shared__ int picked[16];
  __shared__ float xch[2];
  __shared__ int xidx;
  pdl_wait();
  pdl_launch_next();
  const int rows = tt.level_start[depth + 1] - tt.level_start[depth];
  const int item = blockIdx.x / kTreeCluster;
  const int node = tt.level_start[depth] + item, s = blockIdx.y;
  const int nc = tt.n_child[node], fc = tt.first_child[node];
  if (nc == 0) return;  // the whole cluster
  const int N = tt.nodes;
  const DevState& x = st[s];
  const T* row = logits + ((size_t)s * rows + item) * vocab;
  const bool first = blockIdx.x % kTreeCluster == 0;
  if (c.draft_mode == VELLA_DRAFT_ORACLE) {
    if (first && threadIdx.x == 0) {
      for (int i = 0; i < nc; ++i) {
        const int ch = fc + i;
        const int ri = x.L - 1 + tt.dep[ch] - x.P;
        const bool valid = onpath[(size_t)s * N + node] && ri >= 0 && ri < x.ref_len;
        const U4 r = philox4x32_10(U4{(uint32_t)x.pass, (uint32_t)ch, kPurposeTree, (uint32_t)s}, (uint32_t)c.seed,
                                   (uint32_t)(c.seed >> 32));
        const int rt = valid ? ref[(size_t)s * max_seq + ri] : -1;
        const int t = (valid && u01(r.x) < c.oracle_p) ? rt : min((int)(u01(r.y) * (float)vocab), vocab - 1);
        ttok[(size_t)s * N + ch] = t;
        onpath[(size_t)s * N + ch] = valid && t == rt;
      }
    }
    return;
  }
  if (c.temperature <= 0.0f) {  // the draft's top-nc tokens
    if (!first) return;
    for (int i = 0; i < nc; ++i) {
      const int t = block_argmax_excl(row, vocab, picked, i, sh);
      if (threadIdx.x == 0) picked[i] = t;
      __syncthreads();
    }
    if (threadIdx.x == 0)
      for (int i = 0; i < nc; ++i) ttok[(size_t)s * N + fc + i] = picked[i];
    return;
  }
  // nc independent samples of softmax(row / T); the row is kept for the acceptance test
  extern __shared__ __align__(16) unsigned char cl_dyn[];
  T* slice = reinterpret_cast<T*>(cl_dyn);
  ClSweep cl(vocab, xch, &xidx);
  stage_slice(cl, row, slice);
  __syncthreads();
  const float invT = 1.0f / c.temperature;
  const float2 mz = cl_softmax_stats(cl, slice, invT, sh);
  float us[16];
  int drawn[16];
  for (int i = 0; i < nc; ++i) us[i] = uni(c, (uint32_t)x.pass, (uint32_t)(fc + i), kPurposeDraft, s);
  cl_icdf_many(cl, [&](int v) { return expf((Act<T>::to_f(slice[v - cl.lo]) - mz.x) * invT); }, us, nc, picked,
               drawn, sh);
  if (first && threadIdx.x == 0)
    for (int i = 0; i < nc; ++i) ttok[(size_t)s * N + fc + i] = drawn[i] < 0 ? 0 : drawn[i];
  T* q = qrows + ((size_t)node * S + s) * vocab;
  block_copy(q + cl.lo, slice, cl.hi - cl.lo);
  if (first && threadIdx.x == 0) qstats[(size_t)node * S + s] = mz;
  cl.g.sync();  // no CTA leaves while another may still read its exchange slots
}

// Tree acceptance of stream blockIdx.x / kTreeCluster over the verify rows of its N nodes,
// then the KV compaction of the accepted path in the target's and the draft's caches (one
// launch after the verify logits).  The sampled walk sweeps the vocabulary over the cluster
// (every decision is taken from cluster-wide values, so all its CTAs walk the same path); the
// residual row lives in global memory, each CTA updating its own range, and single entries of
// other ranges are read through L2 after a cluster barrier.  The compaction is split over the
// cluster; the greedy walk runs on its first CTA.
template <typename T>
__global__ void __cluster_dims__(kTreeCluster, 1, 1) __launch_bounds__(kSampThreads) tree_accept_kernel(
    DevState* st, int* tok, const T* logits, const int* ys, TreeTopo tt, vella_spec_cfg_dev c, const int* ttok,
    const unsigned char* onpath, const int* ref, const T* qrows, const float2* qstats, int S, float* resid,
    KvPlanes<T> kt, KvPlanes<T> kd, int vocab, int max_seq, const int* nf, const int* err_t, const int* err_d) {
  __shared__ SampShared sh;
  __shared__ int s_u, s_a, s_acc, s_bonus, s_path[16];
  __shared__ float xch[2];
  __shared__ int xidx;
  pdl_wait();
  pdl_launch_next();
  const int s = blockIdx.x / kTreeCluster, part = blockIdx.x % kTreeCluster, N = tt.nodes;
  const bool first = part == 0;
  DevState& x = st[s];
  const bool stop = done(x);
  __syncthreads();
  if (stop) {  // the whole cluster
    if (first && threadIdx.x == 0) {
      x.nonfinite = *nf;
      x.err |= *err_t | *err_d;
      x.n_new = 0;
    }
    return;
  }
  const int root = x.L - 1;
  const int* tt_s = ttok + (size_t)s * N;
  int parts = kTreeCluster;
  if (c.temperature <= 0.0f) {
    if (!first) return;
    parts = 1;
    if (threadIdx.x == 0) {
      int u = 0, a = 0, y = 0;
      for (;;) {
        y = ys[(size_t)s * N + u];
        int found = -1;
        for (int i = 0; i < tt.n_child[u] && found < 0; ++i)
          if (tt_s[tt.first_child[u] + i] == y) found = tt.first_child[u] + i;
        if (found < 0) break;
        s_path[a++] = found;
        u = found;
      }
      s_a = a;
      s_bonus = y;
    }
  } else {
    extern __shared__ __align__(16) unsigned char cl_dyn[];
    T* slice = reinterpret_cast<T*>(cl_dyn);  // this CTA's part of the current verify row
    ClSweep cl(vocab, xch, &xidx);
    const float invT = 1.0f / c.temperature;
    float* r = resid + (size_t)s * vocab;
    if (threadIdx.x == 0) {
      s_u = 0;
      s_a = 0;
    }
    __syncthreads();
    for (;;) {
      const int u = s_u;
      const T* prow = logits + ((size_t)s * N + u) * vocab;
      __syncthreads();  // the previous row's slice is no longer read
      stage_slice(cl, prow, slice);
      __syncthreads();
      const float2 pm = cl_softmax_stats(cl, slice, invT, sh);
      for (int v = cl.lo + threadIdx.x; v < cl.hi; v += blockDim.x)
        r[v] = expf((Act<T>::to_f(slice[v - cl.lo]) - pm.x) * invT) / pm.y;
      cl.g.sync();  // the whole row is in place for the tests below
      DraftQ<T> q{};
      q.invT = invT;
      q.vocab = vocab;
      q.p = c.oracle_p;
      const int nc = tt.n_child[u], fc = tt.first_child[u];
      if (c.draft_mode == VELLA_DRAFT_ORACLE) {
        const int ri = root + tt.dep[u] + 1 - x.P;
        q.ref = (nc > 0 && onpath[(size_t)s * N + u] && ri >= 0 && ri < x.ref_len) ? ref[(size_t)s * max_seq + ri] : -1;
      } else if (nc > 0) {
        q.row = qrows + ((size_t)u * S + s) * vocab;
        const float2 qm = qstats[(size_t)u * S + s];
        q.m = qm.x;
        q.z = qm.y;
      }
      int acc = -1;
      for (int i = 0; i < nc; ++i) {
        const int ch = fc + i, xk = tt_s[ch];
        const float uacc = uni(c, (uint32_t)x.pass, (uint32_t)ch, kPurposeAccept, s);
        if (uacc * q(xk) < __ldcg(r + xk)) {
          acc = ch;
          break;
        }
        // rejected: the residual max(0, r - q), renormalised
        float part_sum = 0.0f;
        for (int v = cl.lo + threadIdx.x; v < cl.hi; v += blockDim.x) {
          const float w = fmaxf(0.0f, __ldcg(r + v) - q(v));
          r[v] = w;
          part_sum += w;
        }
        const float tot = cl.combine(block_sum(part_sum, sh), false);
        if (tot > 0.0f)
          for (int v = cl.lo + threadIdx.x; v < cl.hi; v += blockDim.x) r[v] = __ldcg(r + v) / tot;
        cl.g.sync();
      }
      if (acc >= 0) {
        __syncthreads();
        if (threadIdx.x == 0) {
          s_path[s_a] = acc;
          s_a += 1;
          s_u = acc;
        }
        __syncthreads();
        continue;
      }
      const float u2 = uni(c, (uint32_t)x.pass, (uint32_t)u, kPurposeResidual, s);
      int b = cl_icdf(cl, [&](int v) { return __ldcg(r + v); }, u2, sh);
      if (b < 0) b = cl_icdf(cl, [&](int v) { return expf((Act<T>::to_f(slice[v - cl.lo]) - pm.x) * invT); }, u2, sh);
      if (threadIdx.x == 0) s_bonus = b < 0 ? 0 : b;
      break;
    }
    cl.g.sync();  // no CTA leaves while another may still read its exchange slots
  }
  __syncthreads();
  if (first && threadIdx.x == 0) {
    const int a = s_a;
    int* tk = tok + (size_t)s * max_seq;
    x.nonfinite = *nf;
    x.err |= *err_t | *err_d;
    for (int j = 1; j <= a; ++j) {
      const int t = tt_s[s_path[j - 1]];
      if (root + j < max_seq) tk[root + j] = t; else x.err |= 4;
      x.newtok[j - 1] = t;
    }
    if (root + a + 1 < max_seq) tk[root + a + 1] = s_bonus; else x.err |= 4;
    x.newtok[a] = s_bonus;
    x.n_new = a + 1;
    x.L = root + a + 2;
    x.pass += 1;
    x.produced += a + 1;
  }
  compact_path(kt, s, root, s_a, s_path, part, parts);
  compact_path(kd, s, root, s_a, s_path, part, parts);
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
  void* qrows = nullptr;     // [K or tree nodes][streams][vocab] the draft's rows (stochastic acceptance)
  float2* qstats = nullptr;  // [K or tree nodes][streams] their (max, sum)
  // tree verification (cfg.tree_depth > 0)
  int tree_nodes = 0;
  TreeTopo topo{};
  int* tree_dev = nullptr;                  // dep[N] | first_child[N] | n_child[N]
  unsigned long long* tree_mask = nullptr;  // [N] ancestors-or-self
  int* ttok = nullptr;                      // [streams][N] tree tokens
  unsigned char* onpath = nullptr;          // [streams][N] oracle draft: node follows the reference
  float* resid = nullptr;                   // [streams][vocab] running residual (stochastic tree acceptance)

  int span() const { return tree_nodes ? tree_nodes : cfg.draft_k + 1; }  // slots a pass writes from L - 1

  bool sampled() const { return cfg.temperature > 0.0f; }
  vella_spec_cfg_dev dev_cfg() const {
    return vella_spec_cfg_dev{cfg.seed, cfg.temperature, cfg.oracle_p, cfg.draft_mode};
  }
};

namespace {

// A GEMM pipeline whose wait ran out of time finished without its result: the decode that
// used it is void.  Checked once per prefill and per decode call.
int pipeline_faults() {
  const int st = stream_fault_status(1), tc = tc_fault_status(1), fw = fwd_fault_status(1);
  if (st < 0 || tc < 0 || fw < 0) return fail(VELLA_E_CUDA, "cannot read the kernel fault flags");
  if (st || tc || fw)
    return fail(VELLA_E_CUDA, "a pipeline wait timed out (flags 0x%x / 0x%x / 0x%x)", st, tc, fw);
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

TreeView tree_view(Spec* s, int node0) {
  TreeView v;
  v.tok = s->ttok;
  v.dep = s->tree_dev;
  v.mask = s->tree_mask;
  v.nodes = s->tree_nodes;
  v.node0 = node0;
  return v;
}

// Shared memory of a cluster sweep kernel: one CTA's slice of a vocabulary row (above the
// default 48 KB only for vocabularies of more than 196608 entries).
template <typename K>
int cl_smem(K kernel, int vocab, size_t elt, size_t* bytes) {
  *bytes = cl_slice_bytes(vocab, elt);
  if (*bytes > 48 * 1024) VELLA_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)*bytes));
  return VELLA_OK;
}

template <typename T>
int launch_tree_expand(Spec* s, int depth) {
  const int rows = s->topo.level_start[depth + 1] - s->topo.level_start[depth];
  size_t smem;
  int rc;
  if ((rc = cl_smem(tree_expand_kernel<T>, s->target->cfg.vocab, sizeof(T), &smem))) return rc;
  return launch_kernel(tree_expand_kernel<T>, dim3(rows * kTreeCluster, s->streams), dim3(kSampThreads), smem, s->stream,
                       (const DevState*)s->dstate, static_cast<const T*>(s->draft->logits), depth, s->topo,
                       s->dev_cfg(), (const int*)s->ref, s->ttok, s->onpath, s->target->cfg.vocab, s->max_seq,
                       static_cast<T*>(s->qrows), s->qstats, s->streams);
}

template <typename T>
KvPlanes<T> kv_planes(const Model* m) {
  const vella_model_cfg& c = m->cfg;
  return KvPlanes<T>{static_cast<T*>(m->kv), m->kv_ss, c.n_layers, c.n_kv_heads, c.max_seq, c.head_dim};
}

template <typename T>
int launch_tree_accept(Spec* s) {
  const Model* t = s->target;
  size_t smem;
  int rc;
  if ((rc = cl_smem(tree_accept_kernel<T>, t->cfg.vocab, sizeof(T), &smem))) return rc;
  return launch_kernel(tree_accept_kernel<T>, dim3(s->streams * kTreeCluster), dim3(kSampThreads), smem, s->stream,
                       s->dstate, s->tok,
                       static_cast<const T*>(t->logits), (const int*)t->ys, s->topo, s->dev_cfg(),
                       (const int*)s->ttok, (const unsigned char*)s->onpath, (const int*)s->ref,
                       static_cast<const T*>(s->qrows), (const float2*)s->qstats, s->streams, s->resid,
                       kv_planes<T>(t), kv_planes<T>(s->draft),
                       t->cfg.vocab, s->max_seq, (const int*)t->nonfinite, (const int*)t->err,
                       (const int*)s->draft->err);
}

// One tree pass: the draft expands the tree depth by depth (step 0 over the two committed
// positions L-2, L-1 gives the root's children; step k over the nodes of depth k), the target
// verifies every node in one forward, the acceptance walks the tree, and the accepted path's
// K/V move to consecutive slots in both models.
int enqueue_tree_pass(Spec* s) {
  Model* t = s->target;
  Model* d = s->draft;
  const int S = s->streams, N = s->tree_nodes, D = s->topo.depth;
  const int* Pp = &s->dstate[0].P;
  const bool bf = bf16_of(s);
  int rc;
  if ((rc = launch_kernel(tree_root_kernel, dim3(S), dim3(1), 0, s->stream, (const DevState*)s->dstate,
                          (const int*)s->tok, s->ttok, s->onpath, N, s->max_seq)))
    return rc;
  if ((rc = model_forward(d, state_pos(s, -2), 2, S, 0, s->tok, s->max_seq, Pp, 1, s->stream))) return rc;
  if ((rc = bf ? launch_tree_expand<__nv_bfloat16>(s, 0) : launch_tree_expand<__half>(s, 0))) return rc;
  for (int k = 1; k < D; ++k) {
    const int rows = s->topo.level_start[k + 1] - s->topo.level_start[k];
    const TreeView tv = tree_view(s, s->topo.level_start[k]);
    if ((rc = model_forward(d, state_pos(s, -1), rows, S, 0, s->tok, s->max_seq, Pp, rows, s->stream, &tv))) return rc;
    if ((rc = bf ? launch_tree_expand<__nv_bfloat16>(s, k) : launch_tree_expand<__half>(s, k))) return rc;
  }
  const TreeView tv = tree_view(s, 0);
  if ((rc = model_forward(t, state_pos(s, -1), N, S, 0, s->tok, s->max_seq, Pp, N, s->stream, &tv))) return rc;
  if ((rc = bf ? launch_tree_accept<__nv_bfloat16>(s) : launch_tree_accept<__half>(s))) return rc;
  VELLA_CUDA_TRY(cudaMemsetAsync(d->nonfinite, 0, sizeof(int), s->stream));
  VELLA_CUDA_TRY(cudaMemsetAsync(t->nonfinite, 0, sizeof(int), s->stream));
  return VELLA_OK;
}

int enqueue_pass(Spec* s) {
  if (s->tree_nodes) return enqueue_tree_pass(s);
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
    if (s->hstate->L - 1 + s->span() > s->max_seq) {
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

int vella_loop_cut(const int32_t* tokens, int32_t n, int32_t check_every_fourth, int32_t* kept) {
  if ((!tokens && n > 0) || n < 0 || !kept) return fail(VELLA_E_INVALID, "vella_loop_cut: NULL argument");
  std::vector<int> t(tokens, tokens + n);
  const bool looped = check_every_fourth ? ends_in_loop(t) : loop_cut(t);
  *kept = looped ? (int32_t)t.size() : n;
  return looped ? 1 : 0;
}

int vella_rope_table(int32_t max_seq, int32_t head_dim, float theta, float* out) {
  if (!out || max_seq < 1 || head_dim < 2 || head_dim % 2 || !(theta > 0.0f))
    return fail(VELLA_E_INVALID, "vella_rope_table: %d positions, head_dim %d, theta %g", max_seq, head_dim, (double)theta);
  rope_table(max_seq, head_dim, theta, out);
  return VELLA_OK;
}

int vella_model_set_persistent(vella_model* model, int32_t on) {
  last_error_slot().clear();
  if (!model) return fail(VELLA_E_INVALID, "vella_model_set_persistent: NULL model");
  if (on && !model->prog)
    return fail(VELLA_E_UNSUPPORTED, "vella_model_set_persistent: this model's shapes do not suit the persistent forward");
  model->persistent = on != 0;
  return VELLA_OK;
}

int vella_model_get_cfg(const vella_model* model, vella_model_cfg* out) {
  if (!model || !out) return fail(VELLA_E_INVALID, "vella_model_get_cfg: NULL argument");
  *out = model->cfg;
  return VELLA_OK;
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
  // tree topology (breadth-first): dep, parent mask, children ranges, level starts
  std::vector<int> dep, fch, nch;
  std::vector<unsigned long long> mask;
  TreeTopo topo{};
  if (cfg->tree_depth != 0) {
    if (!draft) return fail(VELLA_E_UNSUPPORTED, "vella_spec_create: tree verification needs a draft model");
    if (cfg->tree_depth < 1 || cfg->tree_depth > kTreeMaxDepth)
      return fail(VELLA_E_UNSUPPORTED, "vella_spec_create: tree_depth %d (1..%d)", cfg->tree_depth, kTreeMaxDepth);
    dep = {0};
    mask = {1ull};
    std::vector<int> parent = {-1};
    topo.depth = cfg->tree_depth;
    topo.level_start[0] = 0;
    topo.level_start[1] = 1;
    int maxlevel = 1;
    for (int k = 1; k <= topo.depth; ++k) {
      const int b = cfg->tree_branching[k - 1];
      if (b < 1 || b > 16) return fail(VELLA_E_INVALID, "vella_spec_create: tree_branching[%d] = %d", k - 1, b);
      for (int p = topo.level_start[k - 1]; p < topo.level_start[k]; ++p)
        for (int i = 0; i < b; ++i) {
          const int n = (int)dep.size();
          if (n >= 64) return fail(VELLA_E_UNSUPPORTED, "vella_spec_create: more than 64 tree nodes");
          dep.push_back(k);
          parent.push_back(p);
          mask.push_back(mask[p] | (1ull << n));
        }
      topo.level_start[k + 1] = (int)dep.size();
      maxlevel = std::max(maxlevel, topo.level_start[k + 1] - topo.level_start[k]);
    }
    const int N = (int)dep.size();
    topo.nodes = N;
    fch.assign(N, 0);
    nch.assign(N, 0);
    for (int n = N - 1; n >= 1; --n) {
      fch[parent[n]] = n;  // the lowest child index, scanning downwards
      nch[parent[n]] += 1;
    }
    if (target->rps < N)
      return fail(VELLA_E_INVALID, "vella_spec_create: the target needs rows_per_stream >= %d tree nodes", N);
    if (draft->rps < std::max(2, maxlevel))
      return fail(VELLA_E_INVALID, "vella_spec_create: the draft needs rows_per_stream >= %d", std::max(2, maxlevel));
  }
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
  const size_t qn = topo.nodes ? (size_t)topo.nodes : (size_t)cfg->draft_k;
  if (cfg->temperature > 0.0f && cfg->draft_mode == VELLA_DRAFT_MODEL && draft) {
    cuda(cudaMalloc(&s->qrows, qn * S * target->cfg.vocab * target->elt), "cudaMalloc(draft rows)");
    cuda(cudaMalloc(&s->qstats, qn * S * sizeof(float2)), "cudaMalloc(draft stats)");
  }
  if (topo.nodes) {
    const int N = topo.nodes;
    s->tree_nodes = N;
    s->topo = topo;
    cuda(cudaMalloc(&s->tree_dev, 3 * (size_t)N * sizeof(int)), "cudaMalloc(tree)");
    cuda(cudaMalloc(&s->tree_mask, (size_t)N * sizeof(unsigned long long)), "cudaMalloc(tree mask)");
    cuda(cudaMalloc(&s->ttok, S * N * sizeof(int)), "cudaMalloc(tree tokens)");
    cuda(cudaMalloc(&s->onpath, S * N), "cudaMalloc(tree path flags)");
    if (cfg->temperature > 0.0f)
      cuda(cudaMalloc(&s->resid, S * target->cfg.vocab * sizeof(float)), "cudaMalloc(residual)");
    if (rc == VELLA_OK) {
      std::vector<int> host(3 * (size_t)N);
      std::copy(dep.begin(), dep.end(), host.begin());
      std::copy(fch.begin(), fch.end(), host.begin() + N);
      std::copy(nch.begin(), nch.end(), host.begin() + 2 * N);
      cuda(cudaMemcpy(s->tree_dev, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice), "cudaMemcpy");
      cuda(cudaMemcpy(s->tree_mask, mask.data(), N * sizeof(unsigned long long), cudaMemcpyHostToDevice), "cudaMemcpy");
      s->topo.dep = s->tree_dev;
      s->topo.first_child = s->tree_dev + N;
      s->topo.n_child = s->tree_dev + 2 * N;
    }
  }
  cuda(cudaEventCreate(&s->ev0), "cudaEventCreate");
  cuda(cudaEventCreate(&s->ev1), "cudaEventCreate");
  cuda(cudaEventCreate(&s->evp), "cudaEventCreate");
  if (rc == VELLA_OK) {
    std::memset(s->hstate, 0, S * sizeof(DevState));
    // on the handle's non-blocking stream, waited for: the passes run on that stream
    cuda(cudaMemsetAsync(s->dstate, 0, S * sizeof(DevState), s->stream), "cudaMemsetAsync");
    cuda(cudaMemsetAsync(s->tok, 0, S * s->max_seq * sizeof(int), s->stream), "cudaMemsetAsync");
    cuda(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize");
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
  for (void* p : {(void*)s->tree_dev, (void*)s->tree_mask, (void*)s->ttok, (void*)s->onpath,
                  (void*)s->resid})
    if (p) cudaFree(p);
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
  if (s->hstate->L - 1 + s->span() > s->max_seq) return fail(VELLA_E_INVALID, "vella_spec_step: KV capacity reached");
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
  if (max_tokens < 1 || s->P + max_tokens + s->span() > s->max_seq)
    return fail(VELLA_E_INVALID, "vella_spec_decode_batch: prefix %d + %d tokens (+%d) exceed max_seq %d", s->P,
                max_tokens, s->span(), s->max_seq);
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

int vella_spec_tensor(vella_spec* s, const char* name, void** ptr, size_t* bytes) {
  last_error_slot().clear();
  if (!s || !name || !ptr || !bytes) return fail(VELLA_E_INVALID, "vella_spec_tensor: NULL argument");
  const std::string n(name);
  const size_t S = (size_t)s->streams, V = (size_t)s->target->cfg.vocab;
  const size_t qn = s->tree_nodes ? (size_t)s->tree_nodes : (size_t)s->cfg.draft_k;
  void* p = nullptr;
  size_t b = 0;
  if (n == "draft_rows") { p = s->qrows; b = qn * S * V * s->target->elt; }
  else if (n == "draft_stats") { p = s->qstats; b = qn * S * sizeof(float2); }
  else if (n == "tokens") { p = s->tok; b = S * s->max_seq * sizeof(int); }
  else if (n == "tree_tokens") { p = s->ttok; b = S * s->tree_nodes * sizeof(int); }
  else if (n == "tree_topology") { p = s->tree_dev; b = 3 * (size_t)s->tree_nodes * sizeof(int); }
  else return fail(VELLA_E_INVALID, "vella_spec_tensor: unknown name '%s'", name);
  if (!p) return fail(VELLA_E_INVALID, "vella_spec_tensor: '%s' is not kept by this decoder's settings", name);
  *ptr = p;
  *bytes = b;
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
