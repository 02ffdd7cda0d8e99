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
// The program's tensor maps, kernel parameters like the per-op kernels' (a descriptor in global
// memory costs the TMA unit a fetch whenever it falls out of its cache): per weight kind its
// weights, scales and biases over every layer (3D: element, row, layer; the layers' tensors
// sit a constant stride apart in the weights arena).
enum : int {
  kMapQkv = 0, kMapO = 3, kMapGate = 6, kMapUp = 9, kMapDown = 12, kMapHead = 15,
  kProgMaps = 18
};
constexpr int kSplit = 16;  // key splits of the decode attention (chunk c at split c % kSplit)
constexpr int kHD = 128;
constexpr int kPrepWarps = 2;  // x preparation warps (alternate units), after the producer warp
constexpr int kFwdThreads = (kRowWarps + 1 + kPrepWarps) * 32;

struct ProgOp {
  int kind;
  // GEMM
  int N, K, rowblocks, nkc, gate, has_res, rope, head;
  int wm, um, layer;        // tensor maps: weights (+1 scales, +2 biases), up rows (gate); layer plane
  void* out;
  const void* res;
  // GEMM: x = the activation rows; NORM: y = rmsnorm(x) * w over d, all rows or the logits rows (tail)
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
  CUtensorMap tm[kProgMaps];
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
constexpr int kAttnRS = kHD + 8;                    // padded row stride of the attention tiles
constexpr int kFwdChunk = 32;                       // keys per attention chunk
constexpr int kQTile = kAttnRows * kAttnRS * 2;     // the [64 head rows x 128] query tile (bytes)
constexpr int kKVTile = kFwdChunk * kAttnRS * 2;    // one [32 keys x 128] K or V tile (bytes)

// Each ring stage is split in two: the weight part (weights, scales, biases; TMA) and the x part
// (quantized: the prepared B fragments and x sums; dense: the raw x slice the consumers read
// their fragments from; written by the prep warps), in two separate rings with the same stage
// index.  The attention tiles overlay the x ring when it is large enough: during ATTN / COMBINE
// no x part is written (the next GEMM op's preparation waits for the barrier after COMBINE),
// while the weight ring keeps filling.  Stage counts: as many as fit (int4: 5 at up to 8 rows,
// 180 KB of weights in flight per SM -- the ring must cover the weights' landing latency plus
// the time the consumers hold a stage).
template <int BITS, int NT>
struct FwdLayout : Tile<BITS, NT> {
  using TL = Tile<BITS, NT>;
  static constexpr int WST = (TL::TX_W + 1023) / 1024 * 1024;                // weight part of a stage
  static constexpr int XS = BITS ? TL::PB_BYTES + TL::PX_BYTES : TL::X_BYTES;  // x part of a stage
  static constexpr int XST = (XS + 127) / 128 * 128;
  static constexpr int PREL = BITS ? 0 : TL::P_REL;  // B fragments within the x part
  static constexpr int kLimit = 227 * 1024;
  static constexpr int bar_bytes(int ns) { return 4 * ns * 8 + 64; }  // fullw, wempty, prepared, xempty
  static constexpr int attn_bytes(int kvb) { return kQTile + 2 * kvb * kKVTile + 2 * kAttnRows * 4; }
  static constexpr int total(int ns, int kvb) {
    return 1024 + ns * (WST + XST) + TL::RED + (ns * XST >= attn_bytes(kvb) ? 0 : attn_bytes(kvb)) + 32 * 4 +
           bar_bytes(ns);
  }
  static constexpr int NS = total(5, 1) <= kLimit ? 5 : total(4, 1) <= kLimit ? 4 : total(3, 1) <= kLimit ? 3 : 2;
  static constexpr int KVB = total(NS, 2) <= kLimit ? 2 : 1;  // K/V double buffering when it fits
  static constexpr int ATTN = attn_bytes(KVB);
  static constexpr bool OVERLAY = NS * XST >= ATTN;
  static constexpr int W_OFF = 0;
  static constexpr int X_OFF = NS * WST;
  static constexpr int RED_OFF = X_OFF + NS * XST;
  static constexpr int ATTN_OFF = OVERLAY ? X_OFF : RED_OFF + TL::RED;
  static constexpr int NRED_OFF = RED_OFF + TL::RED + (OVERLAY ? 0 : ATTN);  // the norm's 32 floats
  static constexpr int BAR_OFF = NRED_OFF + 32 * 4;
  static constexpr int TOTAL = 1024 + BAR_OFF + bar_bytes(NS);
  static_assert(TOTAL <= kLimit, "shared memory");
  static_assert(total(2, 1) <= kLimit, "two stages must fit");
  static_assert(XST % 16 == 0 && RED_OFF % 16 == 0 && BAR_OFF % 8 == 0, "alignment");
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Shared-memory release / acquire between the threads of a CTA (a barrier seen by one thread
// handed to another: causality is transitive through the pair).
__device__ __forceinline__ void st_release_cta(unsigned* p, unsigned v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(saddr(p)), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(saddr(p)) : "memory");
  return v;
}

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

// The raw x slice of a dense unit ([TOK rows][256 elements], the layout the consumers read
// their B fragments from) by one warp: rows [0, rows) of a row-major [.. x K] array from
// column k0, zeros above.
template <typename T, int NT>
__device__ __forceinline__ void stage_x_dense(unsigned char* xs, const T* x, int K, int rows, int k0, int lane) {
  constexpr int TOK = NT * 8;
  uint4 v[TOK];
#pragma unroll
  for (int row = 0; row < TOK; ++row)
    v[row] = row < rows ? __ldcg(reinterpret_cast<const uint4*>(x + (size_t)row * K + k0) + lane) : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int row = 0; row < TOK; ++row) reinterpret_cast<uint4*>(xs + row * 512)[lane] = v[row];
}

// The GEMM units of this CTA across the whole program, in program order.  The fields of the
// current op that the unit paths need are kept here (no global load per unit).
struct GemmCursor {
  int op;           // current GEMM op (nops: done)
  long long u0, u1; // this CTA's unit range of that op
  UnitWalk w;
  int i, n;         // units of the op done, of the op in this CTA
  int nkc, gate, wm, um, layer, K, head;
  const void* x;    // the op's activation rows
  __device__ GemmCursor()
      : op(-1), u0(0), u1(0), w(0, 0, 1), i(0), n(0), nkc(1), gate(0), wm(0), um(0), layer(0), K(0), head(0), x(nullptr) {}
};

// A GEMM op's units are spread over its first min(P, U) CTAs, as the per-op kernel caps its grid
// at the unit count: every CTA between a row block's first and last owner then holds some of
// its units and publishes its partial sums (a CTA without units never would, and the row
// block's gather would wait for it).
__device__ __forceinline__ int op_ctas(const ProgOp& o, int P) {
  const long long U = (long long)o.rowblocks * o.nkc;
  return U < P ? (int)U : P;
}
__device__ __forceinline__ bool op_has_units(const ProgOp& o, int c, int P, long long* u0, long long* u1) {
  const long long U = (long long)o.rowblocks * o.nkc;
  const int Pe = op_ctas(o, P);
  if (c >= Pe) return false;
  *u0 = unit0(c, U, Pe);
  *u1 = unit0(c + 1, U, Pe);
  return *u1 > *u0;
}

// Moves the cursor to its next unit (the first unit of the next GEMM op with units when the
// current op is done).  Returns false at the end of the program.
__device__ __forceinline__ bool cursor_next(GemmCursor& g, const FwdArgs& a, int c, int nops) {
  if (g.op >= 0 && g.op < nops) {
    ++g.i;
    g.w.next(g.nkc);
    if (g.i < g.n) return true;
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
    g.n = (int)(u1 - u0);
    g.nkc = op.nkc;
    g.gate = op.gate;
    g.wm = op.wm;
    g.um = op.um;
    g.layer = op.layer;
    g.K = op.K;
    g.head = op.head;
    g.x = op.x;
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

// Abort: the grid-wide flag a.bar[1] (an L2 round trip: read at op barriers and while idle)
// and this CTA's copy in shared memory (read on the per-unit paths).
__device__ __forceinline__ bool aborted(const FwdArgs& a) {
  return *reinterpret_cast<volatile unsigned*>(a.bar + 1) != 0;
}
__device__ __forceinline__ void set_abort(const FwdArgs& a, int bit, volatile int* local) {
  atomicOr(&g_fwd_fault, bit);
  atomicExch(a.bar + 1, 1u);
  *local = 1;
}

// ---------------------------------------------------------------------------------------
// NORM: rmsnorm_kernel's arithmetic with the 256 consumer threads (ct = 0..255)
// ---------------------------------------------------------------------------------------
constexpr int kNormChunks = 4;  // 8-element chunks of a row per thread: d <= 256 * 8 * 4

// The norm weight slices of consumer thread ct (a constant: loaded before the barrier wait).
template <typename T>
__device__ __forceinline__ void norm_weights(const ProgOp& o, int ct, uint4 (&wv)[kNormChunks]) {
  const T* w = static_cast<const T*>(o.w);
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int i = ct * 8 + k * 2048;
    wv[k] = i < o.d ? *reinterpret_cast<const uint4*>(w + i) : make_uint4(0, 0, 0, 0);
  }
}

template <typename T>
__device__ void norm_row(const ProgOp& o, const FwdArgs& a, int row, int ct, float* nred,
                         const uint4 (&wv)[kNormChunks]) {
  using A = Act<T>;
  const int d = o.d;
  int src = row;
  if (o.tail) {  // the last logits_rows rows of every stream
    const int group = a.rows, tail = a.logits_rows;
    src = (row / tail) * group + group - tail + row % tail;
  }
  const T* xr = static_cast<const T*>(o.x) + (size_t)src * d;
  uint4 xv[kNormChunks];
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int i = ct * 8 + k * 2048;
    xv[k] = i < d ? __ldcg(reinterpret_cast<const uint4*>(xr + i)) : make_uint4(0, 0, 0, 0);
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    if (ct * 8 + k * 2048 >= d) break;
    const uint32_t w4[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v0 = A::lo(w4[j]), v1 = A::hi(w4[j]);
      ss = fmaf(v0, v0, ss);
      ss = fmaf(v1, v1, ss);
    }
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
#pragma unroll
  for (int k = 0; k < kNormChunks; ++k) {
    const int i = ct * 8 + k * 2048;
    if (i >= d) break;
    const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
    const uint32_t gw[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
    uint32_t pk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = A::lo(gw[j]) * A::to_f(A::from_f(A::lo(xw[j]) * r));
      const float a1 = A::hi(gw[j]) * A::to_f(A::from_f(A::hi(xw[j]) * r));
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
// the 256 consumer threads (t = 0..255).  Warps 2r and 2r + 1 hold the same 16 head rows: both
// compute their scores and softmax (the same operations, so the same values), and each
// accumulates one half of the head dimension -- every output element gets the per-op
// kernel's arithmetic with half its accumulator registers.
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

// L2 prefetch of the K and V rows one key split of one (stream, kv head) reads: issued at the
// start of the layer, so that the attention, which follows the q|k|v GEMM, reads its keys from
// L2 instead of queueing behind that GEMM's weight traffic in HBM.
template <typename T>
__device__ void attn_prefetch(const ProgOp& o, const FwdArgs& a, int bz, int kvh, int split) {
  constexpr int C = kFwdChunk, HD = kHD;
  const int pos0 = a.pr.group ? a.pr.base[bz * a.pr.stride] + a.pr.off : *a.pr.base + a.pr.off;
  const int tmax = pos0 + a.rows, kend = min(tmax, a.max_seq);
  const long long kvo = a.kv0 + (long long)bz * a.kv_ss + (long long)kvh * a.max_seq * HD;
  const T* kb = static_cast<const T*>(o.kc) + kvo;
  const T* vb = static_cast<const T*>(o.vc) + kvo;
  for (int c = split; c * C < kend; c += kSplit) {
    const int n = min(C, kend - c * C);
    const uint32_t bytes = (uint32_t)(n * HD * sizeof(T));
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kb + (size_t)c * C * HD), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vb + (size_t)c * C * HD), "r"(bytes) : "memory");
  }
}

__device__ __forceinline__ size_t apart_item(const FwdArgs& a, int bz, int kvh, int split) {
  return (((size_t)bz * a.KV + kvh) * kSplit + split) * (size_t)(2 * kAttnRows + kAttnRows * kHD);
}

// One key split of one (stream, kv head): the running (max, sum, output) of its head rows over
// the chunks c = split, split + 8, ... in order, written to a.apart.
template <typename T, int KVB>
__device__ void attn_split(const ProgOp& o, const FwdArgs& a, int bz, int kvh, int split, int t, unsigned char* sm) {
  constexpr int C = kFwdChunk, RS = kAttnRS, HD = kHD;
  constexpr int NK = HD / 16, ND = HD / 8, NH = ND / 2;  // NH: 8-column output tiles per half
  T* Qs = reinterpret_cast<T*>(sm);
  T* Ks = reinterpret_cast<T*>(sm + kQTile);
  T* Vs = reinterpret_cast<T*>(sm + kQTile + KVB * kKVTile);
  const int warp = t >> 5, lane = t & 31;
  const int rw = warp >> 1, dh = warp & 1;  // row warp (16 head rows), head-dimension half: the two
                                            // warps of a row warp sit on different SMSPs
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
  for (int e = t; e < kAttnRows * (HD / 8); e += 256) {
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
    for (int e = t; e < C * (HD / 8); e += 256) {
      const int j = e / (HD / 8), d8 = (e % (HD / 8)) * 8;
      const bool ok = k0 + j < kend;
      const size_t off = ok ? (size_t)(k0 + j) * HD + d8 : 0;
      cp_async16(kd + j * RS + d8, kbase + off, ok);
      cp_async16(vd + j * RS + d8, vbase + off, ok);
    }
    cp_async_commit();
  };
  const int hr0 = rw * 16 + r, hr1 = hr0 + 8;
  const bool live = rw * 16 < QR;
  float ov[NH][4];
#pragma unroll
  for (int u = 0; u < NH; ++u) ov[u][0] = ov[u][1] = ov[u][2] = ov[u][3] = 0.0f;
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
    named_sync(6, 256);
    if (first) {
      first = false;
      if (live) {
#pragma unroll
        for (int kk = 0; kk < NK; ++kk) {
          const int idx = lane >> 3;
          ldsm4(qf[kk], Qs + (rw * 16 + (idx & 1) * 8 + (lane & 7)) * RS + kk * 16 + (idx >> 1) * 8);
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
      for (int u = 0; u < NH; ++u) {
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
        for (int u = 0; u < NH; u += 2) {
          uint32_t b[4];
          const int idx = lane >> 3;
          ldsm4t(b, vt + (16 * j + (idx & 1) * 8 + (lane & 7)) * RS + 8 * (dh * NH + u + (idx >> 1)));
          mma16816<T>(ov[u], ph, b[0], b[1]);
          mma16816<T>(ov[u], pl, b[0], b[1]);
          mma16816<T>(ov[u + 1], ph, b[2], b[3]);
          mma16816<T>(ov[u + 1], pl, b[2], b[3]);
        }
      }
    }
    named_sync(6, 256);  // every warp is done with this buffer before it is refilled
    if constexpr (KVB == 2) buf ^= 1;
  }
  cp_async_wait<0>();
  named_sync(6, 256);
  // partial rows to global memory (every head row of the block, zeros where no key was seen)
  float* pp = a.apart + apart_item(a, bz, kvh, split);
  float* Mx = pp;
  float* Ls = pp + kAttnRows;
  float* Os = pp + 2 * kAttnRows;
  if (cq == 0 && dh == 0) {
    Mx[hr0] = m0; Ls[hr0] = l0;
    Mx[hr1] = m1; Ls[hr1] = l1;
  }
#pragma unroll
  for (int u = 0; u < NH; ++u) {
    const int dd = 8 * (dh * NH + u) + 2 * cq;
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
  constexpr int RSETS = 256 / HD;
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
__global__ void __launch_bounds__(kFwdThreads, 1) fwd_kernel(const __grid_constant__ FwdArgs a) {
  using LY = FwdLayout<BITS, NT>;
  constexpr int NS = LY::NS, UG = LY::UG, BPG = SFmt<BITS>::BPG;
  constexpr bool kQuant = BITS != 0;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  unsigned char* wring = smem + LY::W_OFF;
  unsigned char* xring = smem + LY::X_OFF;
  float* red = reinterpret_cast<float*>(smem + LY::RED_OFF);
  unsigned char* asm_ = smem + LY::ATTN_OFF;
  float* nred = reinterpret_cast<float*>(smem + LY::NRED_OFF);
  uint64_t* fullw = reinterpret_cast<uint64_t*>(smem + LY::BAR_OFF);
  uint64_t* wempty = fullw + NS;     // a stage's weight part consumed (copied to registers)
  uint64_t* prepared = wempty + NS;
  uint64_t* xempty = prepared + NS;  // a stage's x part consumed

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, P = a.P, nops = a.nops;
  __shared__ int s_abort_;
  __shared__ unsigned s_passed_;  // the last op whose barrier a consumer thread saw pass (+ 1)
  volatile int* s_abort = &s_abort_;
  unsigned* s_passed = &s_passed_;
  if (tid == 0) {
    s_abort_ = 0;
    s_passed_ = 0;
    for (int s = 0; s < NS; ++s) {
      mbar_init(&fullw[s], 1);
      mbar_init(&wempty[s], kRowWarps);
      mbar_init(&xempty[s], kRowWarps);
      mbar_init(&prepared[s], 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ----------------------- weight producer (one thread) -----------------------------
    // Weights do not depend on the activations: unit j's copies go out as soon as its stage is
    // free (unit j - NS consumed), across barriers and non-GEMM ops.
    if (lane != 0) return;
    GemmCursor g;
    long long wi = 0;  // units issued; unit j uses stage j % NS
    for (bool more = cursor_next(g, a, c, nops); more && !*s_abort; more = cursor_next(g, a, c, nops), ++wi) {
      const int s = (int)(wi % NS);
      if (wi >= NS && !mbar_wait(&wempty[s], (uint32_t)((wi / NS - 1) & 1))) {
        set_abort(a, 1, s_abort);
        break;
      }
      uint64_t* bar = &fullw[s];
      mbar_expect_tx(bar, LY::TX_W);
      unsigned char* st = wring + s * LY::WST;
      const int rb = g.w.rb, kc = g.w.kc, layer = g.layer;
      const int w0 = kc * UG * BPG / 4;
#pragma unroll
      for (int q = 0; q < SFmt<BITS>::WCH; ++q) {
        unsigned char* dst = st + q * LY::WCHUNK;
        if (g.gate) {
          tma3d(dst, &a.tm[g.wm], w0 + q * 32, rb * 64, layer, bar);
          tma3d(dst + 64 * 128, &a.tm[g.um], w0 + q * 32, rb * 64, layer, bar);
        } else {
          tma3d(dst, &a.tm[g.wm], w0 + q * 32, rb * 128, layer, bar);
        }
      }
      if constexpr (kQuant) {
        unsigned char* ssb = st + LY::W_BYTES;
        if (g.gate) {
          tma3d(ssb, &a.tm[g.wm + 1], kc * 8, rb * 64, layer, bar);
          tma3d(ssb + 64 * 16, &a.tm[g.um + 1], kc * 8, rb * 64, layer, bar);
          tma3d(ssb + kSlots * 16, &a.tm[g.wm + 2], kc * 8, rb * 64, layer, bar);
          tma3d(ssb + kSlots * 16 + 64 * 16, &a.tm[g.um + 2], kc * 8, rb * 64, layer, bar);
        } else {
          tma3d(ssb, &a.tm[g.wm + 1], kc * 8, rb * 128, layer, bar);
          tma3d(ssb + kSlots * 16, &a.tm[g.wm + 2], kc * 8, rb * 128, layer, bar);
        }
      }
    }
    // never leave with copies in flight: the last fill of every stage
    for (int q = 0; q < NS; ++q) {
      const long long f = wi > q ? (wi - 1 - q) / NS + 1 : 0;
      if (f > 0 && !mbar_wait(&fullw[q], (uint32_t)((f - 1) & 1))) atomicOr(&g_fwd_fault, 2);
    }
    return;
  }

  const int LR = a.logits_rows * a.streams;
  if (warp >= kPrepWarp) {
    // ------------------ x preparation (two warps, alternate units) -----------------------
    // Unit j's x slice is read from L2 (plain loads: the SM's TMA queue is busy with weights,
    // and a slice behind them would land only when they do) once its stage is free (unit
    // j - NS consumed) and the barrier before its op has passed (published by the consumer
    // thread that waits on it, or waited on here).  Quantized: the B fragments and group sums;
    // dense: the raw slice the consumers read their fragments from.  Rows >= M read as zeros.
    const int pw = warp - kPrepWarp;
    GemmCursor g;
    long long j = 0;
    int ready_op = 0;  // ops whose barrier this warp has seen pass
    for (bool more = cursor_next(g, a, c, nops); more; more = cursor_next(g, a, c, nops), ++j) {
      if ((int)(j % kPrepWarps) != pw) continue;
      const int s = (int)(j % NS);
      int go = !*s_abort;
      if (lane == 0 && go) {
        if (j >= NS && !mbar_wait(&xempty[s], (uint32_t)((j / NS - 1) & 1))) {
          set_abort(a, 8, s_abort);
          go = 0;
        }
        if (go && g.op >= ready_op) {
          if (ld_acquire_cta(s_passed) < (unsigned)g.op && !barrier_ready(a, g.op, true)) {  // bounded
            *s_abort = 1;
            go = 0;
          } else {
            ready_op = g.op + 1;
          }
        }
      }
      __syncwarp();  // orders the other lanes' loads after lane 0's acquire
      go = __shfl_sync(0xffffffffu, go, 0);
      if (go) {
        unsigned char* xs = xring + s * LY::XST;
        const T* x = static_cast<const T*>(g.x);
        const int rows = g.head ? LR : a.M, k0 = g.w.kc * UG * 64;
        if constexpr (kQuant) prep_global<T, BITS, NT, LY::PREL>(xs, x, g.K, rows, k0, lane);
        else stage_x_dense<T, NT>(xs, x, g.K, rows, k0, lane);
      }
      mbar_arrive(&prepared[s]);  // also after a fault, so that no consumer waits for it
    }
    return;
  }

  // --------------------------------- consumers ------------------------------------------
  const int ct = tid;  // 0..255
  const int r = lane >> 2, cq = lane & 3;
  const int slot0 = 16 * warp + r, slot1 = slot0 + 8;
  long long j = 0;  // GEMM units consumed (ring position)
  __shared__ int s_ok;
  __shared__ Epi s_ep;
  __shared__ RopeEpi s_re;
  for (int i = 0; i < nops; ++i) {
    // ---- wait for op i's inputs (every CTA done with op i - 1); one CTA-wide verdict, so every
    // branch below that reaches a named barrier is taken by all consumer threads or none ----
    // the op's descriptor into L1 while the barrier is waited on (its fields are read right after)
    if (ct * 128 < (int)sizeof(ProgOp))
      asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char*>(&a.ops[i]) + ct * 128));
    const ProgOp& o = a.ops[i];
    uint4 wv[kNormChunks];
    const int norm_rows = o.tail ? LR : a.M;
    if (o.kind == kOpNorm && c < norm_rows) norm_weights<T>(o, ct, wv);  // in flight across the wait
    if (ct == 0) {
      s_ok = !*s_abort && !aborted(a) && barrier_ready(a, i, true) && !aborted(a);
      if (!s_ok) *s_abort = 1;
      else st_release_cta(s_passed, (unsigned)i);  // after the gpu-scope acquire of the barrier
    }
    named_sync(1, 256);
    const bool ok = s_ok != 0;
    if (o.kind == kOpGemm) {
      long long u0, u1;
      if (op_has_units(o, c, P, &u0, &u1)) {
        // accumulators and fragment offsets live for this op only (every row block's flush
        // leaves acc at zero), so the other ops' code has the registers
        const WOff<BITS> woff(slot0, r, cq);
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
        const int nkc = o.nkc;
        // the op's epilogue descriptors live in shared memory (read at row-block ends only), so
        // the unit loop keeps its registers for the weights
        if (ct == 0) {
          Epi& ep = s_ep;
          RopeEpi& re = s_re;
          ep.bias = nullptr; ep.res = o.res; ep.out = o.out; ep.partial = a.partial; ep.flags = a.flags;
          ep.N = o.N; ep.mc = o.head ? LR : a.M; ep.P = op_ctas(o, P); ep.U = (long long)o.rowblocks * nkc; ep.nkc = nkc;
          ep.gate = o.gate; ep.has_bias = 0; ep.has_res = o.has_res; ep.gelu = 0; ep.rope = o.rope;
          ep.re = &s_re; ep.fault = &g_fwd_fault; ep.abort = a.bar + 1; ep.ka = nullptr;
          if (o.rope) {
            re.cs = a.rope_cs; re.q = const_cast<void*>(a.q);
            re.kc = static_cast<T*>(o.kc) + a.kv0; re.vc = static_cast<T*>(o.vc) + a.kv0;
            re.pr = a.pr; re.H = a.H; re.KV = a.KV; re.max_seq = a.max_seq; re.kv_ss = a.kv_ss; re.err = a.err;
          }
        }
        named_sync(1, 256);
        const int rf = (int)(u0 / nkc), rl = (int)((u1 - 1) / nkc);
        const bool head_shared = u0 % nkc != 0, tail_shared = u1 % nkc != 0;
        UnitWalk cur(u0, u1, nkc);
        const int nunits = (int)(u1 - u0);
        for (int k = 0; k < nunits; ++k, ++j) {
          const int s = (int)(j % NS);
          const uint32_t ph = (uint32_t)((j / NS) & 1);
          bool have = ok && !*s_abort;
          if (have) {
            have = mbar_wait(&fullw[s], ph) && mbar_wait(&prepared[s], ph);
            if (!have) set_abort(a, 4, s_abort);
          }
          if (have)
            consume_stage<T, BITS, NT, LY::PREL>(wring + s * LY::WST, xring + s * LY::XST, acc, woff, lane, slot0, slot1);
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&wempty[s]);
            mbar_arrive(&xempty[s]);
          }
          const int rb = cur.rb;
          const bool flush = cur.seg_last() || cur.kc + 1 == nkc;
          cur.next(nkc);
          // every consumer warp flushes at the same row-block ends (the gate / RoPE pairing
          // synchronises warps w and w + 4), aborted or not
          if (flush)
            flush_rowblock<T, NT>(s_ep, c, rb, rb == rl && tail_shared, rb == rf && head_shared, acc, red, warp, lane);
        }
      }
    } else if (o.kind == kOpNorm && ok) {
      for (int row = c; row < norm_rows; row += P) norm_row<T>(o, a, row, ct, nred, wv);
      if (ct == 0 && i + 2 < nops && !o.tail) {  // a layer's first norm: its attention's keys into L2
        const ProgOp& at = a.ops[i + 2];
        if (at.kind == kOpAttn)
          for (int it = c; it < a.streams * a.KV * kSplit; it += P)
            attn_prefetch<T>(at, a, it / (a.KV * kSplit), (it / kSplit) % a.KV, it % kSplit);
      }
    } else if (o.kind == kOpAttn && ok) {
      const int items = a.streams * a.KV * kSplit;
      for (int it = c; it < items; it += P) {
        attn_split<T, LY::KVB>(o, a, it / (a.KV * kSplit), (it / kSplit) % a.KV, it % kSplit, ct, asm_);
        named_sync(1, 256);
      }
    } else if (o.kind == kOpCombine && ok) {
      const int items = a.streams * a.KV * kSplit;
      for (int it = c; it < items; it += P)
        attn_combine<T>(a, it / (a.KV * kSplit), (it / kSplit) % a.KV, it % kSplit, ct);
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
  CUtensorMap tm[kProgMaps];  // copied into every launch's parameters
  float* apart = nullptr;
  float* partial = nullptr;
  int* scratch = nullptr;  // bar[2] + pad, then flags [P][kRowWarps]
  size_t scratch_bytes = 0;
  int nops = 0;
};

namespace {

// The weight maps of one kind (weights, scales, biases of every layer at maps[idx..idx + 2]):
// 3D over (element, row, layer) with the layers' constant stride in the arena; a single
// tensor (the LM head) is one plane.
int kind_maps(const Model* m, int idx, const QWeight* const* per_layer, int layers, int rows_box, CUtensorMap* maps) {
  const vella_model_cfg& c = m->cfg;
  const QWeight& w = *per_layer[0];
  const int wbits = c.bits ? c.bits : 16;
  const uint64_t words = (uint64_t)w.k * wbits / 32, row_bytes = (uint64_t)w.k * wbits / 8, G = w.k / 64;
  auto stride = [&](void* QWeight::*f, uint64_t one) -> uint64_t {
    if (layers == 1) return (one + 15) / 16 * 16;
    const uint64_t st = (uint64_t)(static_cast<char*>(per_layer[1]->*f) - static_cast<char*>(per_layer[0]->*f));
    for (int l = 1; l < layers; ++l)
      if ((uint64_t)(static_cast<char*>(per_layer[l]->*f) - static_cast<char*>(per_layer[0]->*f)) != st * l) return 0;
    return st % 16 == 0 ? st : 0;
  };
  const uint64_t sw = stride(&QWeight::w, w.n * row_bytes);
  if (!sw) return fail(VELLA_E_UNSUPPORTED, "persistent forward: layer weights not a constant stride apart");
  int rc = make_tensor_map_3d(&maps[idx], CU_TENSOR_MAP_DATA_TYPE_UINT32, w.w, words, w.n, layers, row_bytes, sw, 32,
                              rows_box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc || !c.bits) return rc;
  const uint64_t ss = stride(&QWeight::s, w.n * G * 2), sb = stride(&QWeight::b, w.n * G * 2);
  if (!ss || !sb) return fail(VELLA_E_UNSUPPORTED, "persistent forward: layer scales not a constant stride apart");
  if ((rc = make_tensor_map_3d(&maps[idx + 1], CU_TENSOR_MAP_DATA_TYPE_UINT16, w.s, G, w.n, layers, G * 2, ss, 8,
                               rows_box, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  return make_tensor_map_3d(&maps[idx + 2], CU_TENSOR_MAP_DATA_TYPE_UINT16, w.b, G, w.n, layers, G * 2, sb, 8, rows_box,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
}

int build_prog_maps(const Model* m, CUtensorMap* maps) {
  const vella_model_cfg& c = m->cfg;
  const int L = c.n_layers;
  std::memset(maps, 0, sizeof(CUtensorMap) * kProgMaps);
  std::vector<const QWeight*> per(L);
  const struct { int idx; QWeight Layer::*f; int rows_box; } kinds[] = {
      {kMapQkv, &Layer::qkv, 128}, {kMapO, &Layer::o, 128}, {kMapGate, &Layer::gate, 64},
      {kMapUp, &Layer::up, 64},    {kMapDown, &Layer::down, 128}};
  int rc;
  for (const auto& k : kinds) {
    for (int l = 0; l < L; ++l) per[l] = &(m->layers[l].*(k.f));
    if ((rc = kind_maps(m, k.idx, per.data(), L, k.rows_box, maps))) return rc;
  }
  const QWeight* head = &m->lm_head;
  if ((rc = kind_maps(m, kMapHead, &head, 1, 128, maps))) return rc;
  return VELLA_OK;
}

ProgOp gemm_op(const QWeight& w, const QWeight* up, const void* x, void* out, const void* res, int rope, int head,
               int bits, int wm, int layer) {
  ProgOp o{};
  o.kind = kOpGemm;
  o.wm = wm;
  o.um = kMapUp;
  o.x = x;
  o.layer = layer;
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
  return c.d_model % kq == 0 && (c.n_heads * kHD) % kq == 0 && c.ffn % kq == 0 && c.d_model % 8 == 0 &&
         c.d_model <= 256 * 8 * kNormChunks;
}

void fwd_prog_destroy(FwdProg* p) {
  if (!p) return;
  if (p->device >= 0) cudaSetDevice(p->device);
  for (void* q : {(void*)p->ops, (void*)p->apart, (void*)p->partial, (void*)p->scratch})
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
  std::vector<ProgOp> ops;
  ops.reserve(nops);
  const int bits = c.bits;
  int rc = build_prog_maps(m, p->tm);
  for (int l = 0; l < L; ++l) {
    Layer& Ly = m->layers[l];
    ops.push_back(norm_op(m->h, m->xn, Ly.attn_norm, c.d_model, c.rms_eps, 0));
    ProgOp qkv = gemm_op(Ly.qkv, nullptr, m->xn, m->qkv_out, nullptr, 1, 0, bits, kMapQkv, l);
    qkv.kc = m->kcache(l);
    qkv.vc = m->vcache(l);
    ops.push_back(qkv);
    ProgOp at{};
    at.kind = kOpAttn;
    at.kc = m->kcache(l);
    at.vc = m->vcache(l);
    ops.push_back(at);
    at.kind = kOpCombine;
    ops.push_back(at);
    ops.push_back(gemm_op(Ly.o, nullptr, m->attn, m->h, m->h, 0, 0, bits, kMapO, l));
    ops.push_back(norm_op(m->h, m->xn, Ly.mlp_norm, c.d_model, c.rms_eps, 0));
    ops.push_back(gemm_op(Ly.gate, &Ly.up, m->xn, m->mlp, nullptr, 0, 0, bits, kMapGate, l));
    ops.push_back(gemm_op(Ly.down, nullptr, m->mlp, m->h, m->h, 0, 0, bits, kMapDown, l));
  }
  ops.push_back(norm_op(m->h, m->xn, m->final_norm, c.d_model, c.rms_eps, 1));
  ops.push_back(gemm_op(m->lm_head, nullptr, m->xn, m->logits, nullptr, 0, 1, bits, kMapHead, 0));
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
  cuda(cudaMalloc(&p->ops, ops.size() * sizeof(ProgOp)), "cudaMalloc(program)");
  cuda(cudaMalloc(&p->apart, apart_bytes), "cudaMalloc(attention partials)");
  cuda(cudaMalloc(&p->partial, (size_t)P * kTokMax * kSlots * sizeof(float)), "cudaMalloc(partials)");
  cuda(cudaMalloc(&p->scratch, p->scratch_bytes), "cudaMalloc(barrier)");
  if (rc == VELLA_OK) {
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
    VELLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kFwdThreads, LY::TOTAL));
    if (per_sm < 1) return fail(VELLA_E_CUDA, "persistent forward: no CTA fits an SM");
    configured[dev & 63] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.P);
  cfg.blockDim = dim3(kFwdThreads);
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
  std::memcpy(a.tm, p->tm, sizeof(a.tm));
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
