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
  const float y1 = rope_rot1(x1, x2, c), y2 = rope_rot2(x1, x2, c);
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
// Attention on the tensor cores (mma.sync m16n8k16, fp32 accumulation).  One thread-block
// cluster of kAttnCluster CTAs per (kv head, query block, batch); a query block is up to 64
// "head rows" (query rows x the GQ query heads of the kv head), 16 per warp.  Keys are cut
// into chunks of kAttnChunk at absolute positions and chunk c is processed by CTA
// c % kAttnCluster, which keeps a running (max, sum, output) per head row over its chunks in
// chunk order: S = Q.K^T on the tensor cores, scale and mask in fp32, the online softmax in
// fp32, and O += P.V with P split into two activation-dtype terms (P = hi + lo, both
// multiplied on the tensor cores), so P keeps about 16 significant bits.  The CTAs then
// combine their partial rows through distributed shared memory in rank order.  The query at
// position p sees keys 0..p (tree mode: the keys below the root slot plus its ancestors and
// itself); a chunk with no visible key leaves a row's state unchanged bit for bit (scale
// exp(0) = 1, added terms exact zeros), and every row's arithmetic is independent of the
// other rows of the launch.  K/V chunks travel by cp.async into a double buffer; keys past
// the last needed one are zero-filled (stale cache rows are never multiplied).
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

template <int HD>
struct AttnLayout {
  static constexpr int RS = HD + 8;                         // padded row stride (elements): ldmatrix conflict-free
  static constexpr int TILE = kAttnChunk * RS * 2;           // one [64 x HD] activation tile (bytes)
  static constexpr int Q_OFF = 0, K_OFF = TILE, V_OFF = 3 * TILE;  // Q, K[2], V[2]
  static constexpr int OS = HD + 4;                          // combine: fp32 row stride
  static constexpr int BYTES = 5 * TILE + 2 * kAttnRows * 4;  // + running max / sum per row
  static_assert(kAttnRows * OS * 4 <= 4 * TILE, "combine rows fit over the K/V buffers");
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (sizeof(T) == 2 && Act<T>::kMagic == 128.0f) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

// CS = kAttnCluster: the key chunks of a query block are split over a cluster (decode: one
// query block per stream); CS = 1: one CTA walks all chunks of its query block (launches
// with several query blocks per stream: tree verification, prefill, the Whisper encoder).
template <typename T, int HD, int CS>
__global__ void __cluster_dims__(CS, 1, 1) __launch_bounds__(128) attn_kernel(const AttnArgs a) {
  using LY = AttnLayout<HD>;
  constexpr int C = kAttnChunk;
  constexpr int RS = LY::RS;
  constexpr int NK = HD / 16;  // k16 steps of Q.K^T
  constexpr int ND = HD / 8;   // n8 tiles of the output
  extern __shared__ __align__(128) unsigned char asmem[];
  T* Qs = reinterpret_cast<T*>(asmem + LY::Q_OFF);
  T* Ks = reinterpret_cast<T*>(asmem + LY::K_OFF);
  T* Vs = reinterpret_cast<T*>(asmem + LY::V_OFF);
  float* Mx = reinterpret_cast<float*>(asmem + 5 * LY::TILE);
  float* Ls = Mx + kAttnRows;
  float* Os = reinterpret_cast<float*>(asmem + LY::K_OFF);  // combine: reuses the K/V buffers

  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int kvh = blockIdx.x / CS, qb = blockIdx.y, bz = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, cq = lane & 3;
  pdl_wait();
  pdl_launch_next();
  const int GQ = a.H / a.KV;
  const int QB = a.QB;
  const int pos0 = a.causal ? a.pr.base[bz * a.pr.stride] + a.pr.off : 0;
  const int mq0 = qb * QB;
  const int nq = min(QB, a.M - mq0);
  const int QR = nq * GQ;
  // keys needed by the last query of this block (tree mode: pos0 is the root slot, the rows
  // are nodes tnode0 + mq0 .. and see keys up to their own slot)
  const int tmax = a.causal ? pos0 + (a.v.tmask ? a.v.tnode0 : 0) + mq0 + nq : a.S;
  const int nact = (tmax + C - 1) / C;
  const int kend = min(tmax, a.S);  // key rows that exist
  const T* q = static_cast<const T*>(a.v.q) + (size_t)bz * a.v.q_bs;
  const T* kbase = static_cast<const T*>(a.v.k) + (size_t)bz * a.v.kv_bs + (size_t)kvh * a.v.kv_hs;
  const T* vbase = static_cast<const T*>(a.v.v) + (size_t)bz * a.v.kv_bs + (size_t)kvh * a.v.kv_hs;

  // Q block: head row hr = query mq0 + hr / GQ, head kvh * GQ + hr % GQ; rows >= QR are zeros
  for (int e = tid; e < kAttnRows * (HD / 8); e += 128) {
    const int hr = e / (HD / 8), d8 = (e % (HD / 8)) * 8;
    const bool ok = hr < QR;
    const T* src = ok ? q + (size_t)(mq0 + hr / GQ) * a.v.q_rs + (size_t)(kvh * GQ + hr % GQ) * HD + d8 : q;
    cp_async16(Qs + hr * RS + d8, src, ok);
  }
  cp_async_commit();
  auto fetch = [&](int c, int buf) {
    const int k0 = c * C;
    T* kd = Ks + buf * C * RS;
    T* vd = Vs + buf * C * RS;
    for (int e = tid; e < C * (HD / 8); e += 128) {
      const int j = e / (HD / 8), d8 = (e % (HD / 8)) * 8;
      const bool ok = k0 + j < kend;
      const size_t off = ok ? (size_t)(k0 + j) * a.v.kv_rs + d8 : 0;
      cp_async16(kd + j * RS + d8, kbase + off, ok);
      cp_async16(vd + j * RS + d8, vbase + off, ok);
    }
    cp_async_commit();
  };
  if (rank < nact) fetch(rank, 0);

  // per thread: head rows w*16 + r (accumulator elements 0, 1) and + 8 (elements 2, 3)
  const int hr0 = warp * 16 + r, hr1 = hr0 + 8;
  const bool live = warp * 16 < QR;  // this warp has at least one real row
  float o[ND][4];
#pragma unroll
  for (int u = 0; u < ND; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  // last visible key of the two rows (causal, non-tree), their tree masks
  const int qi0 = mq0 + hr0 / GQ, qi1 = mq0 + hr1 / GQ;
  const int lim0 = a.causal ? pos0 + qi0 : a.S - 1, lim1 = a.causal ? pos0 + qi1 : a.S - 1;
  unsigned long long mk0 = 0, mk1 = 0;
  if (a.v.tmask) {
    mk0 = hr0 < QR ? a.v.tmask[a.v.tnode0 + qi0] : 0ull;
    mk1 = hr1 < QR ? a.v.tmask[a.v.tnode0 + qi1] : 0ull;
  }
  uint32_t qf[NK][4];

  int buf = 0;
  bool first = true;
  for (int c = rank; c < nact; c += CS, buf ^= 1) {
    const int k0 = c * C;
    if (c + CS < nact) {
      fetch(c + CS, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (first) {
      first = false;
      if (live) {
#pragma unroll
        for (int kk = 0; kk < NK; ++kk) {
          const int idx = lane >> 3;
          ldsm4(qf[kk], Qs + (warp * 16 + (idx & 1) * 8 + (lane & 7)) * RS + kk * 16 + (idx >> 1) * 8);
        }
      }
    }
    if (live) {
      const T* kt = Ks + buf * C * RS;
      const T* vt = Vs + buf * C * RS;
      // ---- S = Q K^T: 8 n8 tiles of keys -------------------------------------------------
      float sc[C / 8][4];
#pragma unroll
      for (int t = 0; t < C / 8; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < NK; ++kk)
#pragma unroll
        for (int t = 0; t < C / 8; t += 2) {
          uint32_t b[4];
          const int idx = lane >> 3;
          ldsm4(b, kt + (8 * (t + (idx >> 1)) + (lane & 7)) * RS + kk * 16 + (idx & 1) * 8);
          mma16816<T>(sc[t], qf[kk], b[0], b[1]);
          mma16816<T>(sc[t + 1], qf[kk], b[2], b[3]);
        }
      // ---- scale, mask, online softmax (rows hr0: elements 0,1; hr1: elements 2,3) ---------
      float cm0 = -INFINITY, cm1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < C / 8; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + 8 * t + 2 * cq + (e & 1);
          bool vis;
          if (a.v.tmask) {
            const int j = key - pos0;
            const unsigned long long mk = (e >> 1) ? mk1 : mk0;
            vis = j < 0 || (j < 64 && ((mk >> j) & 1ull));
          } else {
            vis = key <= ((e >> 1) ? lim1 : lim0);
          }
          const float v = vis ? sc[t][e] * a.scale : -INFINITY;
          sc[t][e] = v;
          if (e >> 1) cm1 = fmaxf(cm1, v); else cm0 = fmaxf(cm0, v);
        }
      cm0 = fmaxf(cm0, __shfl_xor_sync(0xffffffffu, cm0, 1));
      cm0 = fmaxf(cm0, __shfl_xor_sync(0xffffffffu, cm0, 2));
      cm1 = fmaxf(cm1, __shfl_xor_sync(0xffffffffu, cm1, 1));
      cm1 = fmaxf(cm1, __shfl_xor_sync(0xffffffffu, cm1, 2));
      const float mn0 = fmaxf(m0, cm0), mn1 = fmaxf(m1, cm1);
      const float al0 = mn0 == -INFINITY ? 1.0f : (m0 == -INFINITY ? 0.0f : expf(m0 - mn0));
      const float al1 = mn1 == -INFINITY ? 1.0f : (m1 == -INFINITY ? 0.0f : expf(m1 - mn1));
      float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
      for (int t = 0; t < C / 8; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = (e >> 1) ? mn1 : mn0;
          const float v = sc[t][e];
          const float pe = (mn == -INFINITY || v == -INFINITY) ? 0.0f : expf(v - mn);
          sc[t][e] = pe;
          if (e >> 1) ps1 += pe; else ps0 += pe;
        }
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
      l0 = fmaf(l0, al0, ps0);
      l1 = fmaf(l1, al1, ps1);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int u = 0; u < ND; ++u) {
        o[u][0] *= al0; o[u][1] *= al0;
        o[u][2] *= al1; o[u][3] *= al1;
      }
      // ---- O += P V, P = hi + lo in the activation dtype ---------------------------------
#pragma unroll
      for (int j = 0; j < C / 16; ++j) {
        uint32_t ph[4], pl[4];
        const float* s0 = sc[2 * j];
        const float* s1 = sc[2 * j + 1];
        const float f[4][2] = {{s0[0], s0[1]}, {s0[2], s0[3]}, {s1[0], s1[1]}, {s1[2], s1[3]}};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ph[i] = pack2<T>(f[i][0], f[i][1]);
          const T* hv = reinterpret_cast<const T*>(&ph[i]);
          pl[i] = pack2<T>(f[i][0] - Act<T>::to_f(hv[0]), f[i][1] - Act<T>::to_f(hv[1]));
        }
#pragma unroll
        for (int u = 0; u < ND; u += 2) {
          uint32_t b[4];
          const int idx = lane >> 3;
          ldsm4t(b, vt + (16 * j + (idx & 1) * 8 + (lane & 7)) * RS + 8 * (u + (idx >> 1)));
          mma16816<T>(o[u], ph, b[0], b[1]);
          mma16816<T>(o[u], pl, b[0], b[1]);
          mma16816<T>(o[u + 1], ph, b[2], b[3]);
          mma16816<T>(o[u + 1], pl, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- partial rows to shared memory, combine across the cluster in rank order -----------
  if (cq == 0) {
    Mx[hr0] = m0; Ls[hr0] = l0;
    Mx[hr1] = m1; Ls[hr1] = l1;
  }
#pragma unroll
  for (int u = 0; u < ND; ++u) {
    const int d = 8 * u + 2 * cq;
    Os[hr0 * LY::OS + d] = o[u][0];
    Os[hr0 * LY::OS + d + 1] = o[u][1];
    Os[hr1 * LY::OS + d] = o[u][2];
    Os[hr1 * LY::OS + d + 1] = o[u][3];
  }
  cl.sync();
  T* out = static_cast<T*>(a.v.out) + (size_t)bz * a.v.o_bs;
  constexpr int RSETS = 128 / HD;
  const int d = tid % HD, rset = tid / HD;
  for (int qr = rank + CS * rset; qr < QR; qr += CS * RSETS) {
    float mr[CS], lr[CS], orr[CS];
#pragma unroll
    for (int i = 0; i < CS; ++i) {
      mr[i] = *cl.map_shared_rank(Mx + qr, i);
      lr[i] = *cl.map_shared_rank(Ls + qr, i);
      orr[i] = *cl.map_shared_rank(Os + qr * LY::OS + d, i);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < CS; ++i) mx = fmaxf(mx, mr[i]);
    float ov = 0.0f, l = 0.0f;
#pragma unroll
    for (int i = 0; i < CS; ++i) {
      const float w = mr[i] == -INFINITY ? 0.0f : expf(mr[i] - mx);
      ov = fmaf(w, orr[i], ov);
      l = fmaf(w, lr[i], l);
    }
    out[(size_t)(mq0 + qr / GQ) * a.v.o_rs + (size_t)(kvh * GQ + qr % GQ) * HD + d] = Act<T>::from_f(ov / l);
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

size_t attn_smem_bytes(int hd) { return hd == 128 ? AttnLayout<128>::BYTES : AttnLayout<64>::BYTES; }

template <typename T, int HD, int CS>
int launch_attn_cs(const AttnArgs& a, int nqb, int batch, cudaStream_t s) {
  const size_t smem = attn_smem_bytes(HD);
  static int configured[64] = {0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(attn_kernel<T, HD, CS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)attn_smem_bytes(HD)));
    configured[dev & 63] = 1;
  }
  return launch_kernel(attn_kernel<T, HD, CS>, dim3(a.KV * CS, nqb, batch), dim3(128), smem, s, a);
}

template <typename T, int HD>
int launch_attn_t(const AttnArgs& a, int batch, cudaStream_t s) {
  const int nqb = (a.M + a.QB - 1) / a.QB;
  // one query block per stream: split its keys over a cluster; several: a CTA per block
  return nqb > 1 ? launch_attn_cs<T, HD, 1>(a, nqb, batch, s) : launch_attn_cs<T, HD, kAttnCluster>(a, nqb, batch, s);
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
