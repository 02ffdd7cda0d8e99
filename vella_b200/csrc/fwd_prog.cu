// Persistent decode forward: one cooperative launch runs a decode-sized forward (at most 16
// rows) of a whole model, instead of seven launches per layer.
//
// Why: at decode sizes every kernel boundary costs several microseconds (the dependent launch's
// release after the previous grid has drained, the activations' first load, the slowest CTA),
// which is most of a 14.8 MB GEMM's time and more than a norm's or an attention's work.  Here a
// grid of one CTA per SM runs the layer program
//
//   NORM (RMSNorm of h into xn) -> GEMM q|k|v (+ RoPE, K/V append) -> ATTN (partial softmax
//   sums per key split) -> COMBINE -> GEMM o (+ residual into h) -> NORM -> GEMM gate/up
//   (SiLU gate) -> GEMM down (+ residual into h), layer after layer, then NORM of the logits
//   rows and the LM head GEMM,
//
// with a grid barrier between ops (an arrival counter: op i starts once every CTA has finished
// op i - 1).  Each CTA keeps the streaming GEMM's roles: a TMA producer thread, an x-preparation
// warp and eight consumer warps.  The producer walks every GEMM unit of the whole program and
// issues a unit's weight copies as soon as its ring stage is free -- weights do not depend on
// the activations, so they keep streaming across barriers and non-GEMM ops -- and the unit's x
// copies once the barrier before its op has passed.  The consumer warps run the GEMM units and
// the NORM / ATTN / COMBINE ops.
//
// Every op reuses the per-op kernels' arithmetic: the GEMM units, their split-K order and
// epilogues are the streaming GEMM's (stream_core.cuh); NORM is rmsnorm_kernel's 256-thread
// reduction; ATTN / COMBINE are the decode attention's eight-way key split (chunk c at split
// c % 8, combined in split order) with the partial rows in global memory instead of cluster
// shared memory.  The GEMM units are split over this grid's one CTA per SM; the per-op path
// runs its large int4 GEMMs at two CTAs per SM, so their split-K boundaries (and the last bits
// of their sums) differ, while every other op -- the dense GEMMs included -- gives the per-op
// path's bits.  A row's result never depends on the other rows of the forward, so every
// decode-sized forward of a model (greedy step, draft step, verify) agrees bit for bit.
//
// Waits: every wait (ring stages, the barrier counter, split-K flags) is bounded; one that runs
// out sets a fault bit and an abort flag, after which no thread waits again and the kernel
// ends (the host reports the fault).  Reads of activations written earlier in the same launch
// by other CTAs bypass L1 (TMA, cp.async.cg, ld.global.cg).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"
#include "model.h"
#include "sm100.cuh"
#include "stream_core.cuh"

namespace vella {

__device__ int g_fwd_fault = 0;  // bits: 1 ring, 2 copies in flight, 4 consumer, 8 prep, 16 gather, 32 barrier

namespace {

using namespace sk;

enum : int { kOpNorm = 1, kOpGemm = 2, kOpAttn = 3, kOpCombine = 4 };
constexpr int kMaps = 8;  // w, up, scales, biases, up scales, up biases, x (NT = 1), x (NT = 2)
constexpr int kSplit = kAttnCluster;  // key splits of the decode attention
constexpr int kHD = 128;

struct ProgOp {
  int kind;
  // GEMM
  int N, K, rowblocks, nkc, gate, has_res, rope, head;
  const CUtensorMap* maps;  // kMaps tensor maps (device memory)
  void* out;
  const void* res;
  // NORM: y = rmsnorm(x) * w over d, all rows or the logits rows (tail)
  const void* x;
  void* y;
  const void* w;
  int d, tail;
  float eps;
  // ATTN / COMBINE / RoPE: the layer's caches (stream 0)
  void* kc;
  void* vc;
};

// Per launch: the rows, their positions and the shared buffers.
struct FwdArgs {
  const ProgOp* ops;
  int nops;
  int M;            // rows = rows_per_stream * streams, stream-major
  int rows, streams, logits_rows;
  PosRef pr;
  const void* q;    // [M][H][128]
  void* attn;       // [M][H][128]
  int H, KV, max_seq;
  long long kv_ss;  // elements between streams' caches
  long long kv0;    // element offset of the first stream's cache
  float scale;
  const float2* rope_cs;
  int* err;
  float* apart;     // attention partial rows [streams][KV][kSplit][2 * 64 + 64 * 128]
  float* partial;   // split-K partial sums [P][16][128]
  int* flags;       // [P][kRowWarps]
  unsigned* bar;    // [0] arrivals, [1] abort; zeroed before the launch
  int P;
};

// ---------------------------------------------------------------------------------------
// shared memory
// ---------------------------------------------------------------------------------------
constexpr int kAttnRS = kHD + 8;                       // padded row stride of the attention tiles
constexpr int kAttnTile = kAttnChunk * kAttnRS * 2;    // one [64 x 128] tile (bytes)

template <int BITS, int NT>
struct FwdLayout : Tile<BITS, NT> {
  using TL = Tile<BITS, NT>;
  static constexpr int NS = 2;
  static constexpr int KVB_TRY = 2;
  static constexpr int bar_bytes() { return 4 * NS * 8 + 64; }
  static constexpr int attn_bytes(int kvb) { return (1 + 2 * kvb) * kAttnTile + 2 * kAttnRows * 4; }
  static constexpr int total(int kvb) { return 1024 + NS * TL::STAGE + TL::RED + attn_bytes(kvb) + 32 * 4 + bar_bytes(); }
  static constexpr int KVB = total(2) <= 227 * 1024 ? 2 : 1;  // K/V double buffering when it fits
  static constexpr int ATTN = attn_bytes(KVB);
  static constexpr int RING = 0;
  static constexpr int RED_OFF = NS * TL::STAGE;
  static constexpr int ATTN_OFF = RED_OFF + TL::RED;
  static constexpr int NRED_OFF = ATTN_OFF + ATTN;   // the norm's 32 floats
  static constexpr int BAR_OFF = NRED_OFF + 32 * 4;
  static constexpr int TOTAL = 1024 + BAR_OFF + bar_bytes();
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ void load8_cg(const T* p, float (&v)[8]) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = Act<T>::lo(w[i]);
    v[2 * i + 1] = Act<T>::hi(w[i]);
  }
}
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

// The GEMM units of this CTA across the whole program, in program order.
struct GemmCursor {
  int op;           // current GEMM op (nops: done)
  long long u0, u1; // this CTA's unit range of that op
  UnitWalk w;
  int i;            // units of the op done
  __device__ GemmCursor() : op(-1), u0(0), u1(0), w(0, 0, 1), i(0) {}
};

__device__ __forceinline__ bool op_has_units(const ProgOp& o, int c, int P, long long* u0, long long* u1) {
  const long long U = (long long)o.rowblocks * o.nkc;
  *u0 = unit0(c, U, P);
  *u1 = unit0(c + 1, U, P);
  return *u1 > *u0;
}

// Moves the cursor to its next unit (the first unit of the next GEMM op with units when the
// current op is done).  Returns false at the end of the program.
__device__ __forceinline__ bool cursor_next(GemmCursor& g, const FwdArgs& a, int c, int nops) {
  if (g.op >= 0 && g.op < nops) {
    ++g.i;
    g.w.next(a.ops[g.op].nkc);
    if (g.i < (int)(g.u1 - g.u0)) return true;
  }
  for (int o = g.op + 1; o < nops; ++o) {
    const ProgOp& op = a.ops[o];
    if (op.kind != kOpGemm) continue;
    long long u0, u1;
    if (!op_has_units(op, c, a.P, &u0, &u1)) continue;
    g.op = o;
    g.u0 = u0;
    g.u1 = u1;
    g.w = UnitWalk(u0, u1, op.nkc);
    g.i = 0;
    return true;
  }
  g.op = nops;
  return false;
}

// Barrier: op i may start once all P CTAs have arrived i times.  Bounded; false on abort.
__device__ __forceinline__ bool barrier_ready(const FwdArgs& a, int i, bool spin) {
  if (i <= 0) return true;
  const unsigned need = (unsigned)i * (unsigned)a.P;
  if (ld_acquire(a.bar) >= need) return true;
  if (!spin) return false;
  const long long t0 = clock64();
  while (ld_acquire(a.bar) < need) {
    if (*reinterpret_cast<volatile unsigned*>(a.bar + 1)) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_fwd_fault, 32);
      atomicExch(a.bar + 1, 1u);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ bool aborted(const FwdArgs& a) {
  return *reinterpret_cast<volatile unsigned*>(a.bar + 1) != 0;
}
__device__ __forceinline__ void set_abort(const FwdArgs& a, int bit) {
  atomicOr(&g_fwd_fault, bit);
  atomicExch(a.bar + 1, 1u);
}

// ---------------------------------------------------------------------------------------
// NORM: rmsnorm_kernel's arithmetic with the 256 consumer threads (ct = 0..255)
// ---------------------------------------------------------------------------------------
template <typename T>
__device__ void norm_row(const ProgOp& o, const FwdArgs& a, int row, int ct, float* nred) {
  using A = Act<T>;
  const int d = o.d;
  int src = row;
  if (o.tail) {  // the last logits_rows rows of every stream
    const int group = a.rows, tail = a.logits_rows;
    src = (row / tail) * group + group - tail + row % tail;
  }
  const T* xr = static_cast<const T*>(o.x) + (size_t)src * d;
  float ss = 0.0f;
  for (int i = ct * 8; i < d; i += 256 * 8) {
    float v[8];
    load8_cg(xr + i, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
  }
  ss = warp_sum(ss);
  if ((ct & 31) == 0) nred[ct >> 5] = ss;
  named_sync(1, 256);
  if (ct < 32) {
    float t = ct < 8 ? nred[ct] : 0.0f;
    t = warp_sum(t);
    if (ct == 0) nred[8] = t;
  }
  named_sync(1, 256);
  const float r = 1.0f / sqrtf(nred[8] / (float)d + o.eps);
  T* out = static_cast<T*>(o.y) + (size_t)row * d;
  const T* w = static_cast<const T*>(o.w);
  for (int i = ct * 8; i < d; i += 256 * 8) {
    float v[8], g[8];
    load8_cg(xr + i, v);
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
    *reinterpret_cast<uint4*>(out + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  named_sync(1, 256);  // nred is reused by the next row
}

// ---------------------------------------------------------------------------------------
// ATTN / COMBINE: the decode attention (one query block per stream, keys split 8 ways) with
// the 128 threads of consumer warps 0..3 (t = 0..127)
// ---------------------------------------------------------------------------------------
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
  if constexpr (Act<T>::kMagic == 128.0f) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

__device__ __forceinline__ size_t apart_item(const FwdArgs& a, int bz, int kvh, int split) {
  return (((size_t)bz * a.KV + kvh) * kSplit + split) * (size_t)(2 * kAttnRows + kAttnRows * kHD);
}

// One key split of one (stream, kv head): the running (max, sum, output) of its head rows over
// the chunks c = split, split + 8, ... in order, written to a.apart.
template <typename T, int KVB>
__device__ void attn_split(const ProgOp& o, const FwdArgs& a, int bz, int kvh, int split, int t, unsigned char* sm) {
  constexpr int C = kAttnChunk, RS = kAttnRS, HD = kHD;
  constexpr int NK = HD / 16, ND = HD / 8;
  T* Qs = reinterpret_cast<T*>(sm);
  T* Ks = reinterpret_cast<T*>(sm + kAttnTile);
  T* Vs = reinterpret_cast<T*>(sm + (1 + KVB) * kAttnTile);
  const int warp = t >> 5, lane = t & 31;
  const int r = lane >> 2, cq = lane & 3;
  const int GQ = a.H / a.KV;
  const int pos0 = a.pr.group ? a.pr.base[bz * a.pr.stride] + a.pr.off : *a.pr.base + a.pr.off;
  const int nq = a.rows;  // one query block per stream
  const int QR = nq * GQ;
  const int tmax = pos0 + nq;
  const int nact = (tmax + C - 1) / C;
  const int kend = min(tmax, a.max_seq);
  const T* q = static_cast<const T*>(a.q) + (size_t)bz * a.rows * a.H * HD;
  const long long kvo = a.kv0 + (long long)bz * a.kv_ss + (long long)kvh * a.max_seq * HD;
  const T* kbase = static_cast<const T*>(o.kc) + kvo;
  const T* vbase = static_cast<const T*>(o.vc) + kvo;
  for (int e = t; e < kAttnRows * (HD / 8); e += 128) {
    const int hr = e / (HD / 8), d8 = (e % (HD / 8)) * 8;
    const bool ok = hr < QR;
    const T* src = ok ? q + (size_t)(hr / GQ) * a.H * HD + (size_t)(kvh * GQ + hr % GQ) * HD + d8 : q;
    cp_async16(Qs + hr * RS + d8, src, ok);
  }
  cp_async_commit();
  auto fetch = [&](int c, int buf) {
    const int k0 = c * C;
    T* kd = Ks + buf * C * RS;
    T* vd = Vs + buf * C * RS;
    for (int e = t; e < C * (HD / 8); e += 128) {
      const int j = e / (HD / 8), d8 = (e % (HD / 8)) * 8;
      const bool ok = k0 + j < kend;
      const size_t off = ok ? (size_t)(k0 + j) * HD + d8 : 0;
      cp_async16(kd + j * RS + d8, kbase + off, ok);
      cp_async16(vd + j * RS + d8, vbase + off, ok);
    }
    cp_async_commit();
  };
  const int hr0 = warp * 16 + r, hr1 = hr0 + 8;
  const bool live = warp * 16 < QR;
  float ov[ND][4];
#pragma unroll
  for (int u = 0; u < ND; ++u) ov[u][0] = ov[u][1] = ov[u][2] = ov[u][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const int qi0 = hr0 / GQ, qi1 = hr1 / GQ;
  const int lim0 = pos0 + qi0, lim1 = pos0 + qi1;
  uint32_t qf[NK][4];
  int buf = 0;
  bool first = true;
  if (KVB == 2 && split < nact) fetch(split, 0);
  for (int c = split; c < nact; c += kSplit) {
    const int k0 = c * C;
    if constexpr (KVB == 2) {
      if (c + kSplit < nact) {
        fetch(c + kSplit, buf ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
    } else {
      fetch(c, 0);
      cp_async_wait<0>();
    }
    named_sync(6, 128);
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
      float sc[C / 8][4];
#pragma unroll
      for (int tt = 0; tt < C / 8; ++tt) sc[tt][0] = sc[tt][1] = sc[tt][2] = sc[tt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < NK; ++kk)
#pragma unroll
        for (int tt = 0; tt < C / 8; tt += 2) {
          uint32_t b[4];
          const int idx = lane >> 3;
          ldsm4(b, kt + (8 * (tt + (idx >> 1)) + (lane & 7)) * RS + kk * 16 + (idx & 1) * 8);
          mma16816<T>(sc[tt], qf[kk], b[0], b[1]);
          mma16816<T>(sc[tt + 1], qf[kk], b[2], b[3]);
        }
      float cm0 = -INFINITY, cm1 = -INFINITY;
#pragma unroll
      for (int tt = 0; tt < C / 8; ++tt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + 8 * tt + 2 * cq + (e & 1);
          const bool vis = key <= ((e >> 1) ? lim1 : lim0);
          const float v = vis ? sc[tt][e] * a.scale : -INFINITY;
          sc[tt][e] = v;
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
      for (int tt = 0; tt < C / 8; ++tt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = (e >> 1) ? mn1 : mn0;
          const float v = sc[tt][e];
          const float pe = (mn == -INFINITY || v == -INFINITY) ? 0.0f : expf(v - mn);
          sc[tt][e] = pe;
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
        ov[u][0] *= al0; ov[u][1] *= al0;
        ov[u][2] *= al1; ov[u][3] *= al1;
      }
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
          mma16816<T>(ov[u], ph, b[0], b[1]);
          mma16816<T>(ov[u], pl, b[0], b[1]);
          mma16816<T>(ov[u + 1], ph, b[2], b[3]);
          mma16816<T>(ov[u + 1], pl, b[2], b[3]);
        }
      }
    }
    named_sync(6, 128);  // every warp is done with this buffer before it is refilled
    if constexpr (KVB == 2) buf ^= 1;
  }
  cp_async_wait<0>();
  named_sync(6, 128);
  // partial rows to global memory (every head row of the block, zeros where no key was seen)
  float* pp = a.apart + apart_item(a, bz, kvh, split);
  float* Mx = pp;
  float* Ls = pp + kAttnRows;
  float* Os = pp + 2 * kAttnRows;
  if (cq == 0) {
    Mx[hr0] = m0; Ls[hr0] = l0;
    Mx[hr1] = m1; Ls[hr1] = l1;
  }
#pragma unroll
  for (int u = 0; u < ND; ++u) {
    const int dd = 8 * u + 2 * cq;
    *reinterpret_cast<float2*>(Os + hr0 * HD + dd) = make_float2(ov[u][0], ov[u][1]);
    *reinterpret_cast<float2*>(Os + hr1 * HD + dd) = make_float2(ov[u][2], ov[u][3]);
  }
}

// The rows qr = split, split + 8, ... of one (stream, kv head): the split partials combined in
// split order into the attention output.
template <typename T>
__device__ void attn_combine(const FwdArgs& a, int bz, int kvh, int split, int t) {
  constexpr int HD = kHD;
  const int GQ = a.H / a.KV;
  const int QR = a.rows * GQ;
  const int d = t % HD, rset = t / HD;
  constexpr int RSETS = 128 / HD;
  T* out = static_cast<T*>(a.attn) + (size_t)bz * a.rows * a.H * HD;
  for (int qr = split + kSplit * rset; qr < QR; qr += kSplit * RSETS) {
    float mr[kSplit], lr[kSplit], orr[kSplit];
#pragma unroll
    for (int i = 0; i < kSplit; ++i) {
      const float* pp = a.apart + apart_item(a, bz, kvh, i);
      mr[i] = __ldcg(pp + qr);
      lr[i] = __ldcg(pp + kAttnRows + qr);
      orr[i] = __ldcg(pp + 2 * kAttnRows + (size_t)qr * HD + d);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kSplit; ++i) mx = fmaxf(mx, mr[i]);
    float ov = 0.0f, l = 0.0f;
#pragma unroll
    for (int i = 0; i < kSplit; ++i) {
      const float w = mr[i] == -INFINITY ? 0.0f : expf(mr[i] - mx);
      ov = fmaf(w, orr[i], ov);
      l = fmaf(w, lr[i], l);
    }
    out[(size_t)(qr / GQ) * a.H * HD + (size_t)(kvh * GQ + qr % GQ) * HD + d] = Act<T>::from_f(ov / l);
  }
}

// ---------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------
template <typename T, int BITS, int NT>
__global__ void __launch_bounds__(kThreads, 1) fwd_kernel(const __grid_constant__ FwdArgs a) {
  using LY = FwdLayout<BITS, NT>;
  constexpr int NS = LY::NS, UG = LY::UG, BPG = SFmt<BITS>::BPG;
  constexpr bool kQuant = BITS != 0;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  float* red = reinterpret_cast<float*>(smem + LY::RED_OFF);
  unsigned char* asm_ = smem + LY::ATTN_OFF;
  float* nred = reinterpret_cast<float*>(smem + LY::NRED_OFF);
  uint64_t* fullw = reinterpret_cast<uint64_t*>(smem + LY::BAR_OFF);
  uint64_t* fullx = fullw + NS;
  uint64_t* empty = fullx + NS;
  uint64_t* prepared = empty + NS;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, P = a.P, nops = a.nops;
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&fullw[s], 1);
      mbar_init(&fullx[s], 1);
      mbar_init(&empty[s], kRowWarps);
      mbar_init(&prepared[s], 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ------------------------------- producer (one thread) ------------------------------
    if (lane != 0) return;
    GemmCursor gw, gx;  // next unit whose weights / x are to be issued
    bool w_more = cursor_next(gw, a, c, nops), x_more = cursor_next(gx, a, c, nops);
    long long wi = 0, xi = 0;  // units issued (weights / x); unit j uses stage j % NS
    int ready_op = 0;          // ops known to have their inputs ready
    const long long t0 = clock64();
    while (x_more) {
      if (aborted(a)) break;
      bool progress = false;
      if (xi < wi) {  // x of the oldest unit whose weights are in flight
        const int op = gx.op;
        if (op < ready_op || barrier_ready(a, op, false)) {
          if (op >= ready_op) {
            ready_op = op + 1;
            fence_proxy_async_global();
          }
          const ProgOp& o = a.ops[op];
          const int s = (int)(xi % NS);
          unsigned char* st = smem + s * LY::STAGE;
          const CUtensorMap* xm = o.maps + (NT == 1 ? 6 : 7);
          mbar_expect_tx(&fullx[s], LY::TX_X);
#pragma unroll
          for (int j = 0; j < SFmt<BITS>::XCH; ++j)
            tma2d(st + LY::XOFF + j * LY::XCHUNK, xm, gx.w.kc * UG * 64 + j * 256, 0, &fullx[s]);
          ++xi;
          x_more = cursor_next(gx, a, c, nops);
          progress = true;
        }
      }
      if (w_more && wi - xi < NS) {
        const int s = (int)(wi % NS);
        const long long use = wi / NS;
        if (use == 0 || mbar_try(&empty[s], (uint32_t)((use - 1) & 1))) {
          const ProgOp& o = a.ops[gw.op];
          const int rb = gw.w.rb, kc = gw.w.kc;
          unsigned char* st = smem + s * LY::STAGE;
          const int w0 = kc * UG * BPG / 4;
          mbar_expect_tx(&fullw[s], LY::TX_W);
#pragma unroll
          for (int j = 0; j < SFmt<BITS>::WCH; ++j) {
            unsigned char* dst = st + j * LY::WCHUNK;
            if (o.gate) {
              tma2d(dst, o.maps + 0, w0 + j * 32, rb * 64, &fullw[s]);
              tma2d(dst + 64 * 128, o.maps + 1, w0 + j * 32, rb * 64, &fullw[s]);
            } else {
              tma2d(dst, o.maps + 0, w0 + j * 32, rb * 128, &fullw[s]);
            }
          }
          if constexpr (kQuant) {
            unsigned char* ssb = st + LY::W_BYTES;
            if (o.gate) {
              tma2d(ssb, o.maps + 2, kc * 8, rb * 64, &fullw[s]);
              tma2d(ssb + 64 * 16, o.maps + 4, kc * 8, rb * 64, &fullw[s]);
              tma2d(ssb + kSlots * 16, o.maps + 3, kc * 8, rb * 64, &fullw[s]);
              tma2d(ssb + kSlots * 16 + 64 * 16, o.maps + 5, kc * 8, rb * 64, &fullw[s]);
            } else {
              tma2d(ssb, o.maps + 2, kc * 8, rb * 128, &fullw[s]);
              tma2d(ssb + kSlots * 16, o.maps + 3, kc * 8, rb * 128, &fullw[s]);
            }
          }
          ++wi;
          w_more = cursor_next(gw, a, c, nops);
          progress = true;
        }
      }
      if (!progress) {
        if (clock64() - t0 > 8 * kWaitCycles) {  // the whole program: far above any real forward
          set_abort(a, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    // never leave with copies in flight: the last weight and x fill of every stage
    for (int q = 0; q < NS; ++q) {
      const long long fw = wi > q ? (wi - 1 - q) / NS + 1 : 0, fx = xi > q ? (xi - 1 - q) / NS + 1 : 0;
      if (fw > 0 && !mbar_wait(&fullw[q], (uint32_t)((fw - 1) & 1))) atomicOr(&g_fwd_fault, 2);
      if (fx > 0 && !mbar_wait(&fullx[q], (uint32_t)((fx - 1) & 1))) atomicOr(&g_fwd_fault, 2);
    }
    return;
  }

  if (warp == kPrepWarp) {
    // ----------------- x preparation: B fragments and group sums, once per stage -----------
    if constexpr (kQuant) {
      GemmCursor g;
      long long j = 0;
      for (bool more = cursor_next(g, a, c, nops); more; more = cursor_next(g, a, c, nops), ++j) {
        const int s = (int)(j % NS);
        const uint32_t ph = (uint32_t)((j / NS) & 1);
        if (!aborted(a) && !(mbar_wait(&fullw[s], ph) && mbar_wait(&fullx[s], ph))) set_abort(a, 8);
        if (!aborted(a)) prep_stage<T, BITS, NT>(smem + s * LY::STAGE, lane);
        mbar_arrive(&prepared[s]);  // also after a fault, so that no consumer waits for it
      }
    }
    return;
  }

  // --------------------------------- consumers ------------------------------------------
  const int ct = tid;  // 0..255
  const int r = lane >> 2, cq = lane & 3;
  const int slot0 = 16 * warp + r, slot1 = slot0 + 8;
  const WOff<BITS> woff(slot0, r, cq);
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
  long long j = 0;  // GEMM units consumed (ring position)
  const int LR = a.logits_rows * a.streams;
  __shared__ int s_ok;
  for (int i = 0; i < nops; ++i) {
    // ---- wait for op i's inputs (every CTA done with op i - 1); one CTA-wide verdict, so every
    // branch below that reaches a named barrier is taken by all consumer threads or none ----
    if (ct == 0) s_ok = !aborted(a) && barrier_ready(a, i, true) && !aborted(a);
    named_sync(1, 256);
    const bool ok = s_ok != 0;
    const ProgOp& o = a.ops[i];
    if (o.kind == kOpGemm) {
      long long u0, u1;
      if (op_has_units(o, c, P, &u0, &u1)) {
        const int nkc = o.nkc;
        RopeEpi re;
        Epi ep;
        ep.bias = nullptr; ep.res = o.res; ep.out = o.out; ep.partial = a.partial; ep.flags = a.flags;
        ep.N = o.N; ep.mc = o.head ? LR : a.M; ep.P = P; ep.U = (long long)o.rowblocks * nkc; ep.nkc = nkc;
        ep.gate = o.gate; ep.has_bias = 0; ep.has_res = o.has_res; ep.gelu = 0; ep.rope = o.rope;
        ep.re = &re; ep.fault = &g_fwd_fault; ep.abort = a.bar + 1;
        if (o.rope) {
          re.cs = a.rope_cs; re.q = const_cast<void*>(a.q);
          re.kc = static_cast<T*>(o.kc) + a.kv0; re.vc = static_cast<T*>(o.vc) + a.kv0;
          re.pr = a.pr; re.H = a.H; re.KV = a.KV; re.max_seq = a.max_seq; re.kv_ss = a.kv_ss; re.err = a.err;
        }
        const int rf = (int)(u0 / nkc), rl = (int)((u1 - 1) / nkc);
        const bool head_shared = u0 % nkc != 0, tail_shared = u1 % nkc != 0;
        UnitWalk cur(u0, u1, nkc);
        const int nunits = (int)(u1 - u0);
        for (int k = 0; k < nunits; ++k, ++j) {
          const int s = (int)(j % NS);
          const uint32_t ph = (uint32_t)((j / NS) & 1);
          bool have = ok && !aborted(a);
          if (have) {
            have = mbar_wait(&fullw[s], ph) && mbar_wait(&fullx[s], ph) && (!kQuant || mbar_wait(&prepared[s], ph));
            if (!have) set_abort(a, 4);
          }
          if (have) consume_stage<T, BITS, NT>(smem + s * LY::STAGE, acc, woff, lane, slot0, slot1);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          const int rb = cur.rb;
          const bool flush = cur.seg_last() || cur.kc + 1 == nkc;
          cur.next(nkc);
          // every consumer warp flushes at the same row-block ends (the gate / RoPE pairing
          // synchronises warps w and w + 4), aborted or not
          if (flush)
            flush_rowblock<T, NT>(ep, c, rb, rb == rl && tail_shared, rb == rf && head_shared, acc, red, warp, lane);
        }
      }
    } else if (o.kind == kOpNorm && ok) {
      const int rows = o.tail ? LR : a.M;
      for (int row = c; row < rows; row += P) norm_row<T>(o, a, row, ct, nred);
    } else if (o.kind == kOpAttn && ok) {
      const int items = a.streams * a.KV * kSplit;
      for (int it = c; it < items; it += P) {
        if (warp < 4) attn_split<T, LY::KVB>(o, a, it / (a.KV * kSplit), (it / kSplit) % a.KV, it % kSplit, ct, asm_);
        named_sync(1, 256);
      }
    } else if (o.kind == kOpCombine && ok) {
      const int items = a.streams * a.KV * kSplit;
      for (int it = c; it < items; it += P)
        if (warp < 4) attn_combine<T>(a, it / (a.KV * kSplit), (it / kSplit) % a.KV, it % kSplit, ct);
    }
    // ---- arrive: this CTA is done with op i ----
    named_sync(1, 256);
    if (ct == 0) {
      __threadfence();
      atomicAdd(a.bar, 1u);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------
// host side: the program of a model, built once
// ---------------------------------------------------------------------------------------
struct FwdProg {
  int device = -1;
  int P = 0;
  std::vector<ProgOp> host_ops;
  ProgOp* ops = nullptr;
  CUtensorMap* maps = nullptr;
  float* apart = nullptr;
  float* partial = nullptr;
  int* scratch = nullptr;  // bar[2] + pad, then flags [P][kRowWarps]
  size_t scratch_bytes = 0;
  int nops = 0;
};

namespace {

int ptr_ok(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int build_maps(const Model* m, const QWeight& w, const QWeight* up, const void* x, CUtensorMap* out) {
  const vella_model_cfg& c = m->cfg;
  const bool gate = up != nullptr;
  const int rows_box = gate ? 64 : 128;
  const int wbits = c.bits ? c.bits : 16;
  const uint64_t words = (uint64_t)w.k * wbits / 32, row_bytes = (uint64_t)w.k * wbits / 8;
  const uint64_t G = w.k / 64;
  std::memset(out, 0, sizeof(CUtensorMap) * kMaps);
  int rc;
  if ((rc = make_tensor_map(&out[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, w.w, words, w.n, row_bytes, 32, rows_box,
                            CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (gate && (rc = make_tensor_map(&out[1], CU_TENSOR_MAP_DATA_TYPE_UINT32, up->w, words, up->n, row_bytes, 32,
                                    rows_box, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (c.bits) {
    if ((rc = make_tensor_map(&out[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, w.s, G, w.n, G * 2, 8, rows_box,
                              CU_TENSOR_MAP_SWIZZLE_NONE)) ||
        (rc = make_tensor_map(&out[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, w.b, G, w.n, G * 2, 8, rows_box,
                              CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    if (gate && ((rc = make_tensor_map(&out[4], CU_TENSOR_MAP_DATA_TYPE_UINT16, up->s, G, up->n, G * 2, 8, rows_box,
                                       CU_TENSOR_MAP_SWIZZLE_NONE)) ||
                 (rc = make_tensor_map(&out[5], CU_TENSOR_MAP_DATA_TYPE_UINT16, up->b, G, up->n, G * 2, 8, rows_box,
                                       CU_TENSOR_MAP_SWIZZLE_NONE))))
      return rc;
  }
  // x: the activation buffer's rows (garbage rows beyond a call's M feed output columns that
  // are never stored); one map per token tile height
  for (int nt = 1; nt <= 2; ++nt)
    if ((rc = make_tensor_map(&out[5 + nt], CU_TENSOR_MAP_DATA_TYPE_UINT16, x, w.k, m->max_rows, (uint64_t)w.k * 2, 256,
                              nt * 8, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
  return VELLA_OK;
}

ProgOp gemm_op(const QWeight& w, const QWeight* up, void* out, const void* res, int rope, int head, int bits) {
  ProgOp o{};
  o.kind = kOpGemm;
  o.gate = up != nullptr;
  o.N = w.n;
  o.K = w.k;
  o.rowblocks = (w.n + (o.gate ? 63 : 127)) / (o.gate ? 64 : 128);
  o.nkc = w.k / 64 / (bits ? 8 : 4);
  o.out = out;
  o.res = res;
  o.has_res = res != nullptr;
  o.rope = rope;
  o.head = head;
  return o;
}

ProgOp norm_op(const void* x, void* y, const void* w, int d, float eps, int tail) {
  ProgOp o{};
  o.kind = kOpNorm;
  o.x = x; o.y = y; o.w = w; o.d = d; o.eps = eps; o.tail = tail;
  return o;
}

}  // namespace

// Shapes the persistent forward serves: dense or int4 bf16/fp16 weights of a model whose every
// GEMM suits the streaming kernel, head_dim 128, no q/k norm.
bool fwd_prog_model_ok(const Model* m) {
  const vella_model_cfg& c = m->cfg;
  if ((c.bits != 0 && c.bits != 4) || c.head_dim != kHD || c.qk_norm || c.n_heads % c.n_kv_heads ||
      c.n_heads / c.n_kv_heads > kAttnMaxGQ)
    return false;
  const int kq = c.bits ? 512 : 256;
  return c.d_model % kq == 0 && (c.n_heads * kHD) % kq == 0 && c.ffn % kq == 0 && c.d_model % 8 == 0;
}

void fwd_prog_destroy(FwdProg* p) {
  if (!p) return;
  if (p->device >= 0) cudaSetDevice(p->device);
  for (void* q : {(void*)p->ops, (void*)p->maps, (void*)p->apart, (void*)p->partial, (void*)p->scratch})
    if (q) cudaFree(q);
  delete p;
}

int fwd_prog_build(Model* m, FwdProg** out) {
  *out = nullptr;
  const vella_model_cfg& c = m->cfg;
  auto* p = new FwdProg();
  p->device = m->device;
  p->P = num_sms(m->device);
  const int L = c.n_layers;
  const int nops = 8 * L + 2;
  std::vector<CUtensorMap> maps((size_t)(4 * L + 1) * kMaps);
  std::vector<ProgOp> ops;
  ops.reserve(nops);
  const int bits = c.bits;
  int rc = VELLA_OK;
  int mi = 0;  // GEMM index (tensor maps)
  auto add_gemm = [&](ProgOp o, const QWeight& w, const QWeight* up, const void* x) {
    if (rc) return;
    rc = build_maps(m, w, up, x, &maps[(size_t)mi * kMaps]);
    o.maps = reinterpret_cast<const CUtensorMap*>((size_t)mi * kMaps);  // index, rebased after the upload
    ++mi;
    ops.push_back(o);
  };
  for (int l = 0; l < L; ++l) {
    Layer& Ly = m->layers[l];
    ops.push_back(norm_op(m->h, m->xn, Ly.attn_norm, c.d_model, c.rms_eps, 0));
    ProgOp qkv = gemm_op(Ly.qkv, nullptr, m->qkv_out, nullptr, 1, 0, bits);
    qkv.kc = m->kcache(l);
    qkv.vc = m->vcache(l);
    add_gemm(qkv, Ly.qkv, nullptr, m->xn);
    ProgOp at{};
    at.kind = kOpAttn;
    at.kc = m->kcache(l);
    at.vc = m->vcache(l);
    ops.push_back(at);
    at.kind = kOpCombine;
    ops.push_back(at);
    add_gemm(gemm_op(Ly.o, nullptr, m->h, m->h, 0, 0, bits), Ly.o, nullptr, m->attn);
    ops.push_back(norm_op(m->h, m->xn, Ly.mlp_norm, c.d_model, c.rms_eps, 0));
    add_gemm(gemm_op(Ly.gate, &Ly.up, m->mlp, nullptr, 0, 0, bits), Ly.gate, &Ly.up, m->xn);
    add_gemm(gemm_op(Ly.down, nullptr, m->h, m->h, 0, 0, bits), Ly.down, nullptr, m->mlp);
  }
  ops.push_back(norm_op(m->h, m->xn, m->final_norm, c.d_model, c.rms_eps, 1));
  add_gemm(gemm_op(m->lm_head, nullptr, m->logits, nullptr, 0, 1, bits), m->lm_head, nullptr, m->xn);
  if (rc) {
    fwd_prog_destroy(p);
    return rc;
  }
  const int P = p->P;
  const size_t apart_bytes =
      (size_t)m->streams * c.n_kv_heads * kSplit * (2 * kAttnRows + kAttnRows * kHD) * sizeof(float);
  p->scratch_bytes = 256 + (size_t)P * kRowWarps * sizeof(int);
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == VELLA_OK) rc = cuda_fail(e, what);
  };
  cuda(cudaSetDevice(m->device), "cudaSetDevice");
  cuda(cudaMalloc(&p->maps, maps.size() * sizeof(CUtensorMap)), "cudaMalloc(tensor maps)");
  cuda(cudaMalloc(&p->ops, ops.size() * sizeof(ProgOp)), "cudaMalloc(program)");
  cuda(cudaMalloc(&p->apart, apart_bytes), "cudaMalloc(attention partials)");
  cuda(cudaMalloc(&p->partial, (size_t)P * kTokMax * kSlots * sizeof(float)), "cudaMalloc(partials)");
  cuda(cudaMalloc(&p->scratch, p->scratch_bytes), "cudaMalloc(barrier)");
  if (rc == VELLA_OK) {
    for (ProgOp& o : ops)
      if (o.kind == kOpGemm) o.maps = p->maps + reinterpret_cast<size_t>(o.maps);
    cuda(cudaMemcpyAsync(p->maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, m->stream),
         "cudaMemcpy(tensor maps)");
    cuda(cudaMemcpyAsync(p->ops, ops.data(), ops.size() * sizeof(ProgOp), cudaMemcpyHostToDevice, m->stream),
         "cudaMemcpy(program)");
    cuda(cudaMemsetAsync(p->scratch, 0, p->scratch_bytes, m->stream), "cudaMemset(barrier)");
    cuda(cudaStreamSynchronize(m->stream), "cudaStreamSynchronize");
  }
  if (rc) {
    fwd_prog_destroy(p);
    return rc;
  }
  p->nops = (int)ops.size();
  p->host_ops = std::move(ops);
  *out = p;
  return VELLA_OK;
}

namespace {

template <typename T, int BITS, int NT>
int launch_fwd(const FwdArgs& a, cudaStream_t s) {
  using LY = FwdLayout<BITS, NT>;
  auto k = fwd_kernel<T, BITS, NT>;
  static int configured[64] = {0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::TOTAL));
    int per_sm = 0;
    VELLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, LY::TOTAL));
    if (per_sm < 1) return fail(VELLA_E_CUDA, "persistent forward: no CTA fits an SM");
    configured[dev & 63] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.P);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = LY::TOTAL;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k, a);
  if (e != cudaSuccess) return cuda_fail(e, "persistent forward launch");
  return VELLA_OK;
}

}  // namespace

// The rows of model_forward (no tree) through the persistent kernel; the caller has written
// the rows' embeddings into m->h.  logits_rows > 0 runs the final norm and the LM head of the
// last logits_rows rows of every stream into m->logits.
int fwd_prog_run(Model* m, FwdProg* p, PosRef pr, int rows, int streams, int stream0, int logits_rows, cudaStream_t s) {
  const vella_model_cfg& c = m->cfg;
  const int M = rows * streams;
  const int GQ = c.n_heads / c.n_kv_heads;
  if (M < 1 || M > kTokMax || rows * GQ > kAttnRows)
    return fail(VELLA_E_INVALID, "persistent forward: %d rows x %d streams", rows, streams);
  FwdArgs a{};
  a.ops = p->ops;
  a.nops = logits_rows > 0 ? p->nops : p->nops - 2;
  a.M = M;
  a.rows = rows;
  a.streams = streams;
  a.logits_rows = logits_rows;
  a.pr = pr;
  a.pr.group = streams > 1 ? rows : 0;
  a.q = m->q;
  a.attn = m->attn;
  a.H = c.n_heads;
  a.KV = c.n_kv_heads;
  a.max_seq = c.max_seq;
  a.kv_ss = m->kv_ss;
  a.kv0 = (long long)stream0 * m->kv_ss;
  a.scale = 1.0f / std::sqrt((float)c.head_dim);
  a.rope_cs = m->rope;
  a.err = m->err;
  a.apart = p->apart;
  a.partial = p->partial;
  a.bar = reinterpret_cast<unsigned*>(p->scratch);
  a.flags = reinterpret_cast<int*>(reinterpret_cast<char*>(p->scratch) + 256);
  a.P = p->P;
  VELLA_CUDA_TRY(cudaMemsetAsync(p->scratch, 0, p->scratch_bytes, s));
  const bool bf = c.dtype == VELLA_BF16;
  const bool nt2 = M > 8;
  if (c.bits == 4) {
    if (bf) return nt2 ? launch_fwd<__nv_bfloat16, 4, 2>(a, s) : launch_fwd<__nv_bfloat16, 4, 1>(a, s);
    return nt2 ? launch_fwd<__half, 4, 2>(a, s) : launch_fwd<__half, 4, 1>(a, s);
  }
  if (bf) return nt2 ? launch_fwd<__nv_bfloat16, 0, 2>(a, s) : launch_fwd<__nv_bfloat16, 0, 1>(a, s);
  return nt2 ? launch_fwd<__half, 0, 2>(a, s) : launch_fwd<__half, 0, 1>(a, s);
}

int fwd_fault_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fwd_fault, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_fwd_fault, &z, sizeof(int));
  }
  return v;
}

}  // namespace vella
