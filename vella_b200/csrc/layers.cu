// Transformer decode-step kernels of the draft-and-verify path (Qwen3-style dense GQA
// layer: RMSNorm, RoPE, causal attention over a preallocated KV cache, SwiGLU through the
// GEMM's SiLU-gate epilogue).
//
// Reference: Worker/Sources/MLXAudioSTT/Qwen3ASR/Qwen3ASRTextDecoder.swift:17-214 (layer
// recipe, RoPE with the pre-update cache offset :76-82), NemotronTranscribeDecoder.swift:
// 96-117 (KV cache: append, trim) and :382-390 (causal attention when more than one query).
//
// Every kernel computes each row (token position) with an instruction sequence that does
// not depend on the other rows of the launch: the attention splits keys at absolute
// positions (multiples of kAttnChunk) owned by fixed CTAs of a cluster and combines them
// in a fixed order; masked keys add exact zeros.  So a verify pass over K+1 positions gives bit-identical hidden states,
// logits and tokens to K+1 single-token greedy steps.
#include <cuda_runtime.h>

#include <cooperative_groups.h>

#include <cfloat>
#include <cstdint>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"

namespace vella {
namespace {

namespace cg = cooperative_groups;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = Act<T>::lo(w[i]);
    v[2 * i + 1] = Act<T>::hi(w[i]);
  }
}

// ---------------------------------------------------------------------------------------
// embedding rows: position < P reads the caller's input embeddings, else the token table
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void embed_rows_kernel(T* __restrict__ h, const T* __restrict__ table, const T* __restrict__ prefix,
                                  long long prefix_ss, const int* __restrict__ tok, int tok_ss, PosRef pr,
                                  const int* __restrict__ Pdev, int d, int vocab, int max_seq, int* err, TreeView tv) {
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x;
  const int sidx = pr.stream_of(m);
  int pos = pr.pos(m);
  int node = -1;
  if (tv.tok) {
    const int r = pr.group ? m % pr.group : m;
    node = tv.node0 + r;
    pos = pos - r + tv.dep[node];
  }
  const int P = Pdev[sidx * pr.stride];
  const T* src;
  if (node < 0 && pos >= 0 && pos < P) {
    src = prefix + (size_t)sidx * prefix_ss + (size_t)pos * d;
  } else {
    int t = node >= 0 ? tv.tok[(size_t)sidx * tv.nodes + node]
                      : ((pos >= 0 && pos < max_seq) ? tok[(size_t)sidx * tok_ss + pos] : -1);
    if (t < 0 || t >= vocab) {
      if (threadIdx.x == 0) atomicOr(err, 1);
      t = 0;
    }
    src = table + (size_t)t * d;
  }
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(h + (size_t)m * d);
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) d4[i] = s4[i];
}

// ---------------------------------------------------------------------------------------
// RMSNorm: y = w * T(x * rsqrt(mean(x^2) + eps)), sums in fp32 in a fixed order
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(T* __restrict__ out, const T* __restrict__ x,
                                                      const T* __restrict__ w, int d, float eps, int group, int tail) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int row = blockIdx.x;
  const int src = (row / tail) * group + group - tail + row % tail;
  const T* xr = x + (size_t)src * d;
  float ss = 0.0f;
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    float v[8];
    load8(xr + i, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(red[0] / (float)d + eps);
  T* o = out + (size_t)row * d;
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    float v[8], g[8];
    load8(xr + i, v);
    load8(w + i, g);
    uint32_t pk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = g[2 * j] * A::to_f(A::from_f(v[2 * j] * r));
      const float a1 = g[2 * j + 1] * A::to_f(A::from_f(v[2 * j + 1] * r));
      const T t0 = A::from_f(a0), t1 = A::from_f(a1);
      pk[j] = (uint32_t)reinterpret_cast<const unsigned short&>(t0) |
              ((uint32_t)reinterpret_cast<const unsigned short&>(t1) << 16);
    }
    *reinterpret_cast<uint4*>(o + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
}

// ---------------------------------------------------------------------------------------
// RoPE (half rotation, table of fp32 cos/sin per position) + KV append; optional per-head
// q/k RMSNorm before the rotation (Qwen3 q_norm / k_norm).
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void rope_append_kernel(const T* __restrict__ qkv, T* __restrict__ q_out, T* __restrict__ kc,
                                   T* __restrict__ vc, const float2* __restrict__ cs, const T* __restrict__ qn,
                                   const T* __restrict__ kn, float eps, PosRef pr, int H, int KV, int hd,
                                   int max_seq, int* err, long long kv_ss, TreeView tv) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x, hidx = blockIdx.y, i = threadIdx.x;
  const int half = hd / 2;
  int pos = pr.pos(m);   // RoPE position
  int slot = pos;        // KV-cache slot
  if (tv.dep) {
    const int r = pr.group ? m % pr.group : m;
    const int node = tv.node0 + r;
    slot = pos - r + node;
    pos = pos - r + tv.dep[node];
  }
  if (slot < 0 || slot >= max_seq) {
    if (i == 0) atomicOr(err, 2);
    return;
  }
  const size_t sbase = (size_t)pr.stream_of(m) * kv_ss;
  if (pos < 0 || pos >= max_seq) {
    if (i == 0) atomicOr(err, 2);
    return;
  }
  const T* row = qkv + (size_t)m * (H + 2 * KV) * hd;
  const bool is_q = hidx < H;
  const T* src = row + (size_t)hidx * hd;  // q heads, then k heads
  float x1 = A::to_f(src[i]), x2 = A::to_f(src[i + half]);
  const T* nw = is_q ? qn : kn;
  if (nw != nullptr) {
    __shared__ float red[32];
    float ss = warp_sum(fmaf(x1, x1, x2 * x2));
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (half + 31) / 32; ++w) t += red[w];
    const float r = 1.0f / sqrtf(t / (float)hd + eps);
    x1 = A::to_f(A::from_f(A::to_f(nw[i]) * A::to_f(A::from_f(x1 * r))));
    x2 = A::to_f(A::from_f(A::to_f(nw[i + half]) * A::to_f(A::from_f(x2 * r))));
  }
  const float2 c = cs[(size_t)pos * half + i];
  const float y1 = x1 * c.x - x2 * c.y;
  const float y2 = x1 * c.y + x2 * c.x;
  if (is_q) {
    T* o = q_out + ((size_t)m * H + hidx) * hd;
    o[i] = A::from_f(y1);
    o[i + half] = A::from_f(y2);
  } else {
    const int kv = hidx - H;
    T* ko = kc + sbase + ((size_t)kv * max_seq + slot) * hd;
    ko[i] = A::from_f(y1);
    ko[i + half] = A::from_f(y2);
    const T* vs = row + (size_t)(H + KV + kv) * hd;
    T* vo = vc + sbase + ((size_t)kv * max_seq + slot) * hd;
    vo[i] = vs[i];
    vo[i + half] = vs[i + half];
  }
}

// ---------------------------------------------------------------------------------------
// Decode attention.  One thread-block cluster of kAttnCluster CTAs per (kv head, query
// block).  Keys are cut into chunks of kAttnChunk at absolute positions and chunk c is
// processed by CTA c % kAttnCluster, which keeps a running (max, sum, output) per query
// row over its chunks in chunk order (fp32 scores and probabilities).  The CTAs then
// combine their partial rows through distributed shared memory in rank order.  Query at
// position p sees keys 0..p; a chunk with no visible key leaves a row's state unchanged
// bit for bit (scale exp(0) = 1, added terms exact zeros), so a row's result does not
// depend on the other rows of the launch.
// ---------------------------------------------------------------------------------------
struct AttnArgs {
  AttnView v;
  PosRef pr;   // causal: position of query row 0
  int M, H, KV;
  int S;       // key rows that exist (cache capacity; the key count when not causal)
  int QB;      // query rows per cluster (QB * H / KV <= kAttnRows)
  int causal;  // 1: the query at position p sees keys 0..p; 0: all S keys
  float scale;
};

template <typename T, int HD>
__global__ void __cluster_dims__(kAttnCluster, 1, 1) __launch_bounds__(256) attn_kernel(const AttnArgs a) {
  constexpr int C = kAttnChunk;
  constexpr int CS = kAttnCluster;
  constexpr int KS = HD + 4;  // padded fp32 row stride of K/V/Q/O in shared memory
  constexpr int PS = C + 4;
  constexpr int V8 = HD / 8;            // 16-byte vectors per key row
  constexpr int LDI = C * V8 / 256;     // vectors of K (and of V) per thread and chunk
  static_assert(LDI * 256 == C * V8, "chunk loads must tile the block");
  extern __shared__ __align__(16) float sm[];
  const int GQ = a.H / a.KV;
  const int QB = a.QB;
  constexpr int QRmax = kAttnRows;
  float* Ks = sm;
  float* Vs = Ks + C * KS;
  float* Qs = Vs + C * KS;
  float* Os = Qs + QRmax * KS;
  float* Ps = Os + QRmax * KS;
  float* Mx = Ps + QRmax * PS;  // running max per row
  float* Ls = Mx + QRmax;       // running sum of probabilities
  float* Al = Ls + QRmax;       // rescale factor of the current chunk

  cg::cluster_group cl = cg::this_cluster();
  const int r = (int)cl.block_rank();
  const int kvh = blockIdx.x / CS, qb = blockIdx.y, bz = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_launch_next();
  const int pos0 = a.causal ? a.pr.base[bz * a.pr.stride] + a.pr.off : 0;
  const int mq0 = qb * QB;
  const int nq = min(QB, a.M - mq0);
  const int QR = nq * GQ;
  // keys needed by the last query of this block (tree mode: pos0 is the root slot, the rows
  // are nodes tnode0 + mq0 .. and see keys up to their own slot)
  const int tmax = a.causal ? pos0 + (a.v.tmask ? a.v.tnode0 : 0) + mq0 + nq : a.S;
  const int nact = (tmax + C - 1) / C;
  const int kend = min(tmax, a.S);   // key rows that exist
  const T* q = static_cast<const T*>(a.v.q) + (size_t)bz * a.v.q_bs;
  const T* kbase = static_cast<const T*>(a.v.k) + (size_t)bz * a.v.kv_bs + (size_t)kvh * a.v.kv_hs;
  const T* vbase = static_cast<const T*>(a.v.v) + (size_t)bz * a.v.kv_bs + (size_t)kvh * a.v.kv_hs;

  for (int i = tid; i < QR * KS; i += 256) Os[i] = 0.0f;
  for (int i = tid; i < QR; i += 256) { Mx[i] = -INFINITY; Ls[i] = 0.0f; }
  for (int e0 = 0; e0 < QR * V8; e0 += 4 * 256) {
    uint4 raw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * 256 + tid;
      if (e < QR * V8) {
        const int qr = e / V8, d8 = (e % V8) * 8;
        raw[u] = *reinterpret_cast<const uint4*>(q + (size_t)(mq0 + qr / GQ) * a.v.q_rs + (size_t)(kvh * GQ + qr % GQ) * HD + d8);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * 256 + tid;
      if (e < QR * V8) {
        const int qr = e / V8, d8 = (e % V8) * 8;
        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          Qs[qr * KS + d8 + 2 * t] = Act<T>::lo(w[t]);
          Qs[qr * KS + d8 + 2 * t + 1] = Act<T>::hi(w[t]);
        }
      }
    }
  }

  // K/V of a chunk travel through registers so that the next chunk's loads overlap this
  // chunk's arithmetic; keys at or past tmax read as zeros (their rows may be stale).
  uint4 kr[LDI], vr[LDI];
  auto fetch = [&](int c) {
    const int k0 = c * C;
#pragma unroll
    for (int u = 0; u < LDI; ++u) {
      const int e = u * 256 + tid, j = e / V8, d8 = (e % V8) * 8;
      if (k0 + j < kend) {
        kr[u] = *reinterpret_cast<const uint4*>(kbase + (size_t)(k0 + j) * a.v.kv_rs + d8);
        vr[u] = *reinterpret_cast<const uint4*>(vbase + (size_t)(k0 + j) * a.v.kv_rs + d8);
      } else {
        kr[u] = vr[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int u = 0; u < LDI; ++u) {
      const int e = u * 256 + tid, j = e / V8, d8 = (e % V8) * 8;
      const uint32_t kw[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
      const uint32_t vw[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        Ks[j * KS + d8 + 2 * t] = Act<T>::lo(kw[t]);
        Ks[j * KS + d8 + 2 * t + 1] = Act<T>::hi(kw[t]);
        Vs[j * KS + d8 + 2 * t] = Act<T>::lo(vw[t]);
        Vs[j * KS + d8 + 2 * t + 1] = Act<T>::hi(vw[t]);
      }
    }
  };

  constexpr int RS = 256 / HD;
  const int d = tid % HD, rset = tid / HD;
  if (r < nact) fetch(r);
  for (int c = r; c < nact; c += CS) {
    const int k0 = c * C;
    __syncthreads();  // the previous chunk's P.V has finished reading Ks/Vs
    stash();
    if (c + CS < nact) fetch(c + CS);
    __syncthreads();

    // ---- scores: warp w takes 4-row blocks, lane j takes keys j and j + 32 -----------
    for (int rb = warp * 4; rb < QR; rb += 32) {
      float s[4][2];
#pragma unroll
      for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.0f;
      for (int dd = 0; dd < HD; dd += 4) {
        const float4 ka = *reinterpret_cast<const float4*>(Ks + lane * KS + dd);
        const float4 kb = *reinterpret_cast<const float4*>(Ks + (lane + 32) * KS + dd);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 qv = *reinterpret_cast<const float4*>(Qs + min(rb + i, QR - 1) * KS + dd);
          s[i][0] = fmaf(qv.x, ka.x, s[i][0]); s[i][0] = fmaf(qv.y, ka.y, s[i][0]);
          s[i][0] = fmaf(qv.z, ka.z, s[i][0]); s[i][0] = fmaf(qv.w, ka.w, s[i][0]);
          s[i][1] = fmaf(qv.x, kb.x, s[i][1]); s[i][1] = fmaf(qv.y, kb.y, s[i][1]);
          s[i][1] = fmaf(qv.z, kb.z, s[i][1]); s[i][1] = fmaf(qv.w, kb.w, s[i][1]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int qr = rb + i;
        if (qr < QR) {
          bool v0, v1;
          if (a.v.tmask) {  // committed keys below the root, then the node's ancestors and itself
            const unsigned long long mk = a.v.tmask[a.v.tnode0 + mq0 + qr / GQ];
            const int j0 = k0 + lane - pos0, j1 = j0 + 32;
            v0 = j0 < 0 || (j0 < 64 && ((mk >> j0) & 1ull));
            v1 = j1 < 0 || (j1 < 64 && ((mk >> j1) & 1ull));
          } else {
            const int lim = a.causal ? pos0 + mq0 + qr / GQ : a.S - 1;  // last visible key
            v0 = k0 + lane <= lim;
            v1 = k0 + lane + 32 <= lim;
          }
          Ps[qr * PS + lane] = v0 ? s[i][0] * a.scale : -INFINITY;
          Ps[qr * PS + lane + 32] = v1 ? s[i][1] * a.scale : -INFINITY;
        }
      }
    }
    __syncthreads();

    // ---- running softmax: warp per row --------------------------------------------------
    for (int qr = warp; qr < QR; qr += 8) {
      const float v0 = Ps[qr * PS + lane], v1 = Ps[qr * PS + lane + 32];
      const float mo = Mx[qr];
      const float mn = fmaxf(mo, warp_max(fmaxf(v0, v1)));
      float p0 = 0.0f, p1 = 0.0f, alpha = 1.0f;
      if (mn != -INFINITY) {
        p0 = v0 == -INFINITY ? 0.0f : expf(v0 - mn);
        p1 = v1 == -INFINITY ? 0.0f : expf(v1 - mn);
        alpha = mo == -INFINITY ? 0.0f : expf(mo - mn);
      }
      const float l = warp_sum(p0 + p1);
      Ps[qr * PS + lane] = p0;
      Ps[qr * PS + lane + 32] = p1;
      if (lane == 0) {
        Mx[qr] = mn;
        Ls[qr] = fmaf(Ls[qr], alpha, l);
        Al[qr] = alpha;
      }
    }
    __syncthreads();

    // ---- O = O * alpha + P.V: thread (d, row set), 4 rows at a time --------------------
    for (int rb = rset * 4; rb < QR; rb += RS * 4) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int j = 0; j < C; j += 4) {
        const float v0 = Vs[j * KS + d], v1 = Vs[(j + 1) * KS + d], v2 = Vs[(j + 2) * KS + d],
                    v3 = Vs[(j + 3) * KS + d];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 p = *reinterpret_cast<const float4*>(Ps + min(rb + i, QR - 1) * PS + j);
          acc[i] = fmaf(p.x, v0, acc[i]); acc[i] = fmaf(p.y, v1, acc[i]);
          acc[i] = fmaf(p.z, v2, acc[i]); acc[i] = fmaf(p.w, v3, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (rb + i < QR) Os[(rb + i) * KS + d] = fmaf(Os[(rb + i) * KS + d], Al[rb + i], acc[i]);
    }
  }

  // ---- combine the cluster's partial rows in rank order; CTA r owns rows r, r + CS, … --
  cl.sync();
  T* out = static_cast<T*>(a.v.out) + (size_t)bz * a.v.o_bs;
  for (int qr = r + CS * rset; qr < QR; qr += CS * RS) {
    float mr[CS], lr[CS], orr[CS];
#pragma unroll
    for (int i = 0; i < CS; ++i) {
      mr[i] = *cl.map_shared_rank(Mx + qr, i);
      lr[i] = *cl.map_shared_rank(Ls + qr, i);
      orr[i] = *cl.map_shared_rank(Os + qr * KS + d, i);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < CS; ++i) mx = fmaxf(mx, mr[i]);
    float o = 0.0f, l = 0.0f;
#pragma unroll
    for (int i = 0; i < CS; ++i) {
      const float w = mr[i] == -INFINITY ? 0.0f : expf(mr[i] - mx);
      o = fmaf(w, orr[i], o);
      l = fmaf(w, lr[i], l);
    }
    out[(size_t)(mq0 + qr / GQ) * a.v.o_rs + (size_t)(kvh * GQ + qr % GQ) * HD + d] = Act<T>::from_f(o / l);
  }
  cl.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---------------------------------------------------------------------------------------
// argmax per row with the lowest index on ties; NaN/Inf anywhere sets the flag
// ---------------------------------------------------------------------------------------
constexpr int kArgBlocks = 32;
constexpr int kArgRowBytes = kArgBlocks * 8 + 16;  // partials (float2 each) + counter, 16-byte slots

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_kernel(const T* __restrict__ logits, int V, size_t ld,
                                                     int* __restrict__ ys, char* scratch, int* nonfinite) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x, b = blockIdx.y;
  const int per = ((V + kArgBlocks - 1) / kArgBlocks + 7) / 8 * 8;
  const int lo = b * per, hi = min(V, lo + per);
  const T* row = logits + (size_t)m * ld;
  float bv = -INFINITY;
  int bi = INT32_MAX;
  bool bad = false;
  const bool vec = (ld % 8 == 0);
  for (int i = lo + threadIdx.x * 8; i < hi; i += 256 * 8) {
    if (vec && i + 8 <= hi) {
      float v[8];
      load8(row + i, v);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (!isfinite(v[t])) { bad = true; if (isnan(v[t])) continue; }
        better(bv, bi, v[t], i + t);
      }
    } else {
      for (int t = i; t < min(i + 8, hi); ++t) {
        const float v = A::to_f(row[t]);
        if (!isfinite(v)) { bad = true; if (isnan(v)) continue; }
        better(bv, bi, v, t);
      }
    }
  }
  if (bad) atomicOr(nonfinite, 1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ int s_last;
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) better(bv, bi, sv[w], si[w]);
    float2* part = reinterpret_cast<float2*>(scratch + (size_t)m * kArgRowBytes);
    int* ctr = reinterpret_cast<int*>(part + kArgBlocks);
    part[b] = make_float2(bv, __int_as_float(bi));
    __threadfence();
    const int prev = atomicAdd(ctr, 1);
    s_last = prev == kArgBlocks - 1;
    if (s_last) {
      *ctr = 0;
      __threadfence();
      float fv = -INFINITY;
      int fi = INT32_MAX;
      for (int k = 0; k < kArgBlocks; ++k) {
        const float2 p = __ldcg(part + k);
        better(fv, fi, p.x, __float_as_int(p.y));
      }
      ys[m] = fi == INT32_MAX ? 0 : fi;
    }
  }
}

size_t attn_smem_bytes(int hd) {
  const size_t ks = hd + 4, ps = kAttnChunk + 4, qr = kAttnRows;
  return (2 * kAttnChunk * ks + 2 * qr * ks + qr * ps + 3 * qr) * sizeof(float);
}

template <typename T, int HD>
int launch_attn_t(const AttnArgs& a, int batch, cudaStream_t s) {
  const size_t smem = attn_smem_bytes(HD);
  static int configured[64] = {0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(attn_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)attn_smem_bytes(HD)));
    configured[dev & 63] = 1;
  }
  const int nqb = (a.M + a.QB - 1) / a.QB;
  return launch_kernel(attn_kernel<T, HD>, dim3(a.KV * kAttnCluster, nqb, batch), dim3(256), smem, s, a);
}

}  // namespace

int launch_embed_rows_dev(int dtype, void* h, const void* table, const void* prefix, long long prefix_ss,
                          const int* tok, int tok_ss, PosRef pr, int rows, const int* P, int d, int vocab, int max_seq,
                          int* err, cudaStream_t s, TreeView tv) {
  if (rows <= 0) return VELLA_OK;
  if (dtype == VELLA_BF16)
    return launch_kernel(embed_rows_kernel<__nv_bfloat16>, dim3(rows), dim3(256), 0, s, static_cast<__nv_bfloat16*>(h),
                         static_cast<const __nv_bfloat16*>(table), static_cast<const __nv_bfloat16*>(prefix), prefix_ss,
                         tok, tok_ss, pr, P, d, vocab, max_seq, err, tv);
  return launch_kernel(embed_rows_kernel<__half>, dim3(rows), dim3(256), 0, s, static_cast<__half*>(h),
                       static_cast<const __half*>(table), static_cast<const __half*>(prefix), prefix_ss, tok, tok_ss,
                       pr, P, d, vocab, max_seq, err, tv);
}

int launch_rmsnorm(int dtype, void* out, const void* x, const void* w, int rows, int d, float eps,
                   cudaStream_t s, int group, int tail) {
  if (rows <= 0) return VELLA_OK;
  if (group <= 0 || tail <= 0) group = tail = rows;
  if (tail > group) return fail(VELLA_E_INVALID, "rmsnorm: tail %d of groups of %d rows", tail, group);
  if (dtype == VELLA_BF16)
    return launch_kernel(rmsnorm_kernel<__nv_bfloat16>, dim3(rows), dim3(256), 0, s, static_cast<__nv_bfloat16*>(out),
                         static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), d, eps, group, tail);
  return launch_kernel(rmsnorm_kernel<__half>, dim3(rows), dim3(256), 0, s, static_cast<__half*>(out),
                       static_cast<const __half*>(x), static_cast<const __half*>(w), d, eps, group, tail);
}

int launch_rope_append(int dtype, const void* qkv, void* q_out, void* kc, void* vc, const float2* cs,
                       const void* qn, const void* kn, float eps, PosRef pr, int rows, int H, int KV, int hd,
                       int max_seq, int* err, cudaStream_t s, long long kv_ss, TreeView tv) {
  if (rows <= 0) return VELLA_OK;
  const dim3 grid(rows, H + KV);
  if (dtype == VELLA_BF16)
    return launch_kernel(rope_append_kernel<__nv_bfloat16>, grid, dim3(hd / 2), 0, s,
                         static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(q_out),
                         static_cast<__nv_bfloat16*>(kc), static_cast<__nv_bfloat16*>(vc), cs,
                         static_cast<const __nv_bfloat16*>(qn), static_cast<const __nv_bfloat16*>(kn), eps, pr, H, KV,
                         hd, max_seq, err, kv_ss, tv);
  return launch_kernel(rope_append_kernel<__half>, grid, dim3(hd / 2), 0, s, static_cast<const __half*>(qkv),
                       static_cast<__half*>(q_out), static_cast<__half*>(kc), static_cast<__half*>(vc), cs,
                       static_cast<const __half*>(qn), static_cast<const __half*>(kn), eps, pr, H, KV, hd, max_seq,
                       err, kv_ss, tv);
}

int launch_attention_ex(int dtype, const AttnView& v, int batch, PosRef pr, int causal, int rows, int H, int KV,
                        int hd, int S, float scale, cudaStream_t s) {
  if (rows <= 0 || batch <= 0) return VELLA_OK;
  const int gq = KV > 0 ? H / KV : 0;
  if (gq < 1 || gq * KV != H || gq > kAttnMaxGQ)
    return fail(VELLA_E_UNSUPPORTED, "attention: H/KV = %d/%d not supported", H, KV);
  if (S < 1 || batch > 65535) return fail(VELLA_E_INVALID, "attention: %d keys, batch %d", S, batch);
  AttnArgs a{};
  a.v = v;
  a.pr = pr; a.M = rows; a.H = H; a.KV = KV; a.S = S;
  a.QB = kAttnRows / gq;
  a.causal = causal ? 1 : 0;
  a.scale = scale;
  if (dtype == VELLA_BF16) {
    if (hd == 128) return launch_attn_t<__nv_bfloat16, 128>(a, batch, s);
    if (hd == 64) return launch_attn_t<__nv_bfloat16, 64>(a, batch, s);
  } else {
    if (hd == 128) return launch_attn_t<__half, 128>(a, batch, s);
    if (hd == 64) return launch_attn_t<__half, 64>(a, batch, s);
  }
  return fail(VELLA_E_UNSUPPORTED, "attention: head_dim %d not supported", hd);
}

int launch_attention(int dtype, const void* q, const void* kc, const void* vc, void* out, PosRef pr, int rows,
                     int H, int KV, int hd, int max_seq, float scale, cudaStream_t s) {
  AttnView v{};
  v.q = q; v.k = kc; v.v = vc; v.out = out;
  v.q_rs = v.o_rs = (long long)H * hd;
  v.kv_hs = (long long)max_seq * hd;
  v.kv_rs = hd;
  return launch_attention_ex(dtype, v, 1, pr, 1, rows, H, KV, hd, max_seq, scale, s);
}

// One slot per logits row, at a fixed offset whatever the launch's row count: the row's
// kArgBlocks partial maxima, then its ticket counter (zero between launches).
size_t argmax_scratch_bytes(int max_rows) { return (size_t)max_rows * kArgRowBytes + 256; }

int launch_argmax(int dtype, const void* logits, int rows, int V, size_t ld, int* ys, void* scratch,
                  int* nonfinite, cudaStream_t s) {
  if (rows <= 0) return VELLA_OK;
  char* sc = static_cast<char*>(scratch);
  const dim3 grid(rows, kArgBlocks);
  if (dtype == VELLA_BF16)
    return launch_kernel(argmax_kernel<__nv_bfloat16>, grid, dim3(256), 0, s,
                         static_cast<const __nv_bfloat16*>(logits), V, ld, ys, sc, nonfinite);
  return launch_kernel(argmax_kernel<__half>, grid, dim3(256), 0, s, static_cast<const __half*>(logits), V, ld, ys, sc,
                       nonfinite);
}

}  // namespace vella
