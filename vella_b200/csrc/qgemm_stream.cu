// K1, streaming form: the small-M GEMM as a persistent, warp-specialised TMA pipeline (one
// CTA per SM).  Same arithmetic as qgemm.cu (reference SmallMGEMM.swift:662-755 product form;
// m16n8k16 with the weights as the A operand, 4-bit codes dequantized with one LOP3 per pair,
// sum(x) through an all-ones MMA), different data movement:
//
//   * a producer thread moves, per work unit, the weight tile [128 rows x UG groups] with
//     2D tensor-map TMA copies (boxes of 128 rows x 128 bytes, 128-byte swizzle), the
//     unit's scales and biases (boxes of 128 rows x 16 bytes) and the x slice (boxes of
//     TOK tokens x 256 elements, out-of-range tokens and rows zero-filled by the TMA unit)
//     into a ring of NS shared-memory stages; mbarriers (expect_tx / complete_tx) mark a
//     stage full, consumer arrivals mark it empty.  Every wait is bounded by a clock limit,
//     after which the kernel records a fault and runs to its end without waiting.
//   * for the quantized formats an x-preparation warp turns each stage's x slice into the
//     MMA's B fragments in the order the nibble/byte unpacking produces the A fragments, and
//     sums x per group and token (the bias term of the product form), once per stage for
//     all consumers; it marks the stage "prepared" on a third mbarrier.
//   * eight consumer warps each own 16 weight rows of the unit across all its groups, so a
//     row block's sums never cross warps: every warp runs its own epilogue from registers
//     (with the SiLU gate, up-row warp w + 4 hands its sums to gate-row warp w).
//   * work unit u = (row block, k chunk); CTA c streams units [c U/P, (c+1) U/P), i.e. a
//     few whole row blocks plus a partial one at each end.  A row block split between CTAs
//     is finished by the CTA holding its last unit (the "gatherer"); the others publish
//     their partial sums.  Each CTA works its own last row block first when it continues in
//     the next CTA (publishing early, one flag per warp), then its whole row blocks, and its
//     first row block last when it began in earlier CTAs: the partial sums it then gathers
//     (in CTA order, from lower-numbered CTAs only) were published at their start.
//
// The unit ranges depend on (N, K, format, SM count) only, never on M, and every output
// row is computed by the same instruction sequence whatever the other rows are: a row of
// a batched call is bit-identical to the same row computed alone.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"
#include "sm100.cuh"

namespace vella {

__device__ int g_stream_fault = 0;  // set when a pipeline wait ran out of time

namespace {

constexpr int kRowWarps = 8;                 // consumer warps, 16 weight rows each
constexpr int kProducerWarp = kRowWarps;     // one TMA thread
constexpr int kPrepWarp = kRowWarps + 1;     // x preparation (quantized formats)
constexpr int kThreads = (kRowWarps + 2) * 32;
constexpr int kSlots = 128;
constexpr int kTokMax = 16;
constexpr int kBarPair0 = 2;  // named barriers 2..5: gate-row warp w with up-row warp w + 4

// UG groups of 64 per unit; BPG bytes per row and group; WCH 128-byte column chunks of the
// weight tile; XCH 256-element chunks of the x slice.
template <int BITS> struct SFmt;
template <> struct SFmt<4> { static constexpr int UG = 8, BPG = 32, WCH = 2, XCH = 2; };
template <> struct SFmt<8> { static constexpr int UG = 8, BPG = 64, WCH = 4, XCH = 2; };
template <> struct SFmt<0> { static constexpr int UG = 4, BPG = 128, WCH = 4, XCH = 1; };

// LIGHT: the compact layout (96 registers a thread, two stages), two of which fit one SM: the
// int4 calls run two CTAs per SM when their units keep both busy, else one, which leaves room
// for the next kernel's CTA to start its weight copies before this call ends.
template <int BITS, int NT, bool LIGHT = false>
struct Layout {
  static constexpr int TOK = NT * 8;
  static constexpr int UG = SFmt<BITS>::UG;
  static constexpr int WCHUNK = kSlots * 128;                 // one [128 rows x 128 B] box
  static constexpr int W_BYTES = SFmt<BITS>::WCH * WCHUNK;
  static constexpr int SB_BYTES = BITS ? 2 * kSlots * 16 : 0;  // scales [128][16 B], biases [128][16 B]
  static constexpr int XCHUNK = TOK * 512;                    // one [TOK x 256 elements] box
  static constexpr int X_BYTES = SFmt<BITS>::XCH * XCHUNK;
  static constexpr int PB_BYTES = BITS ? UG * NT * 1024 : 0;  // B fragments [g][nt][half][lane] x 16 B
  static constexpr int PX_BYTES = BITS ? UG * TOK * 4 : 0;    // x group sums [g][token], fp32
  static constexpr int TX = W_BYTES + SB_BYTES + X_BYTES;     // bytes the TMA unit delivers per stage
  static constexpr int STAGE = (TX + PB_BYTES + PX_BYTES + 1023) / 1024 * 1024;
  static constexpr int RED = 64 * TOK * 4;                    // up-row sums handed to the gate warps
  static constexpr int fixed(int ns) { return 1024 + RED + 3 * ns * 8 + 16; }
  static constexpr int NS =
      LIGHT ? 2 : (fixed(4) + 4 * STAGE <= 227 * 1024) ? 4 : (fixed(3) + 3 * STAGE <= 227 * 1024) ? 3 : 2;
  static constexpr int TOTAL = fixed(NS) + NS * STAGE;
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

struct SArgs {
  CUtensorMap tw, tu, ts, tb, tus, tub, tx;
  const void* bias;
  const void* res;
  void* out;
  float* partial;  // [P][16][128]: a CTA's partial sums of its last row block
  int* flags;      // [P][kRowWarps]: partial published, per warp (reset by the gatherer)
  int M, N, K, G, rowblocks, nkc, P;
  int has_bias, has_res, gelu;
  int rope;     // RoPE + KV-append epilogue (q|k|v projection, 128-row blocks = heads)
  RopeEpi re;
};

using namespace sm100;

// CTA holding unit u when U units are split over P CTAs as [c U/P, (c+1) U/P) (U >= P).
__device__ __forceinline__ int cta_of(long long u, long long U, int P) { return (int)(((u + 1) * P - 1) / U); }
__device__ __forceinline__ long long unit0(int c, long long U, int P) { return (long long)c * U / P; }

// The units [u0, u1) of a CTA in processing order: its last row block first when that
// continues in the next CTA, then the row blocks it holds whole, then its first row block
// when that began in an earlier CTA.  (row block, k chunk) advance one unit at a time; the
// chunk count is divided by once per segment only.
struct UnitWalk {
  // the current segment ends at e; up to two more segments [b1, e1), [b2, e2) follow (scalars,
  // not arrays: a runtime-indexed array would live in local memory)
  long long e, b1, e1, b2, e2;
  int left;
  long long u;
  int rb, kc;
  __device__ UnitWalk(long long u0, long long u1, int nkc) : e(u1), b1(0), e1(0), b2(0), e2(0), left(0), u(u0) {
    const long long rf = u0 / nkc, rl = (u1 - 1) / nkc;
    if (rl != rf) {
      const bool tail = u1 % nkc != 0, head = u0 % nkc != 0;
      const long long mb = head ? (rf + 1) * nkc : u0, me = tail ? rl * nkc : u1;
      int n = 0;
      long long b0 = 0, e0 = 0;
      auto push = [&](long long bb, long long ee) {
        if (n == 0) { b0 = bb; e0 = ee; }
        else if (n == 1) { b1 = bb; e1 = ee; }
        else { b2 = bb; e2 = ee; }
        ++n;
      };
      if (tail) push(rl * nkc, u1);
      if (me > mb) push(mb, me);
      if (head) push(u0, (rf + 1) * nkc);
      u = b0;
      e = e0;
      left = n - 1;
    }
    rb = (int)(u / nkc);
    kc = (int)(u % nkc);
  }
  __device__ __forceinline__ bool seg_last() const { return u + 1 == e; }
  __device__ __forceinline__ void next(int nkc) {
    if (++u == e) {
      if (left > 0) {
        u = b1;
        e = e1;
        b1 = b2;
        e1 = e2;
        --left;
        rb = (int)(u / nkc);
        kc = (int)(u % nkc);
      }
    } else if (++kc == nkc) {
      kc = 0;
      ++rb;
    }
  }
};

template <int BITS>
__device__ __forceinline__ void permute_xs(uint32_t (&p)[8], const uint32_t (&n)[8]) {
  if constexpr (BITS == 4) {
    p[0] = __byte_perm(n[0], n[2], 0x5410); p[1] = __byte_perm(n[0], n[2], 0x7632);
    p[2] = __byte_perm(n[1], n[3], 0x5410); p[3] = __byte_perm(n[1], n[3], 0x7632);
    p[4] = __byte_perm(n[4], n[6], 0x5410); p[5] = __byte_perm(n[4], n[6], 0x7632);
    p[6] = __byte_perm(n[5], n[7], 0x5410); p[7] = __byte_perm(n[5], n[7], 0x7632);
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[2 * j] = __byte_perm(n[2 * j], n[2 * j + 1], 0x5410);
      p[2 * j + 1] = __byte_perm(n[2 * j], n[2 * j + 1], 0x7632);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = n[i];
  }
}

__device__ __forceinline__ int ld_flag(const int* p) {
  int v;
  asm volatile("ld.volatile.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T, int BITS, int NT, bool GATE, bool LIGHT>
__global__ void __launch_bounds__(kThreads, LIGHT ? 2 : 1) qgemm_stream_kernel(const __grid_constant__ SArgs a) {
  using A = Act<T>;
  using LY = Layout<BITS, NT, LIGHT>;
  constexpr int UG = LY::UG, BPG = SFmt<BITS>::BPG, NS = LY::NS, TOK = LY::TOK;
  constexpr bool kQuant = BITS != 0;
  constexpr uint32_t kMask = 0x000F000Fu;
  constexpr uint32_t kMag = A::kMagic2;
  constexpr float kOff = BITS == 4 ? A::kMagic : 17.0f * A::kMagic;
  constexpr uint32_t kOne2 = A::kMagic == 128.0f ? 0x3F803F80u : 0x3C003C00u;
  constexpr int XOFF = LY::W_BYTES + LY::SB_BYTES;  // raw x slice within a stage
  constexpr int POFF = XOFF + LY::X_BYTES;          // prepared B fragments, then x sums

  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle
  // (offsetting the shared array itself keeps its address space: shared loads, not generic ones)
  unsigned char* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  float* red = reinterpret_cast<float*>(smem + NS * LY::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * LY::STAGE + LY::RED);
  uint64_t* empty = full + NS;
  uint64_t* prepared = empty + NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(prepared + NS);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, P = a.P, nkc = a.nkc;
  const long long U = (long long)a.rowblocks * nkc;
  const long long u0 = unit0(c, U, P), u1 = unit0(c + 1, U, P);
  const int nunits = (int)(u1 - u0);
  const int mc = min(a.M, kTokMax);
  const int N = a.N;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRowWarps);
      mbar_init(&prepared[s], 32);
    }
    abort_flag[0] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_next();

  if (warp == kProducerWarp) {
    // ------------------------------- producer (one thread) ------------------------------
    if (lane != 0) return;
    int issued = 0;  // units whose copies were issued; unit i fills stage i % NS
    // weights, scales and biases of a unit (constant data: may be read before the
    // preceding kernel has finished)
    auto issue_w = [&](const UnitWalk& w, int s) {
      const int rb = w.rb, kc = w.kc;
      unsigned char* st = smem + s * LY::STAGE;
      const int w0 = kc * UG * BPG / 4;  // first 32-bit word of the unit in a weight row
#pragma unroll
      for (int j = 0; j < SFmt<BITS>::WCH; ++j) {
        unsigned char* dst = st + j * LY::WCHUNK;
        if constexpr (GATE) {
          tma2d(dst, &a.tw, w0 + j * 32, rb * 64, &full[s]);
          tma2d(dst + 64 * 128, &a.tu, w0 + j * 32, rb * 64, &full[s]);
        } else {
          tma2d(dst, &a.tw, w0 + j * 32, rb * 128, &full[s]);
        }
      }
      if constexpr (kQuant) {
        unsigned char* ssb = st + LY::W_BYTES;
        if constexpr (GATE) {
          tma2d(ssb, &a.ts, kc * 8, rb * 64, &full[s]);
          tma2d(ssb + 64 * 16, &a.tus, kc * 8, rb * 64, &full[s]);
          tma2d(ssb + kSlots * 16, &a.tb, kc * 8, rb * 64, &full[s]);
          tma2d(ssb + kSlots * 16 + 64 * 16, &a.tub, kc * 8, rb * 64, &full[s]);
        } else {
          tma2d(ssb, &a.ts, kc * 8, rb * 128, &full[s]);
          tma2d(ssb + kSlots * 16, &a.tb, kc * 8, rb * 128, &full[s]);
        }
      }
    };
    // the x slice of a unit (written by the preceding kernel)
    auto issue_x = [&](const UnitWalk& w, int s) {
      unsigned char* st = smem + s * LY::STAGE;
#pragma unroll
      for (int j = 0; j < SFmt<BITS>::XCH; ++j)
        tma2d(st + XOFF + j * LY::XCHUNK, &a.tx, w.kc * UG * 64 + j * 256, 0, &full[s]);
    };
    // first round of the ring: weights before the dependency wait, x after it
    const int npre = nunits < NS ? nunits : NS;
    UnitWalk cur(u0, u1, nkc);
    {
      UnitWalk cw = cur;
      for (int j = 0; j < npre; ++j, cw.next(nkc)) {
        mbar_expect_tx(&full[j], LY::TX);
        ++issued;
        issue_w(cw, j);
      }
    }
    pdl_wait();
    for (int j = 0; j < npre; ++j, cur.next(nkc)) issue_x(cur, j);
    int s = npre % NS;
    uint32_t ph = npre == NS ? 1u : 0u;
    for (int i = npre; i < nunits; ++i, cur.next(nkc)) {
      if (abort_flag[0]) break;
      if (!mbar_wait(&empty[s], ph ^ 1)) {
        abort_flag[0] = 1;
        atomicOr(&g_stream_fault, 1);
        break;
      }
      mbar_expect_tx(&full[s], LY::TX);
      ++issued;
      issue_w(cur, s);
      issue_x(cur, s);
      if (++s == NS) {
        s = 0;
        ph ^= 1u;
      }
    }
    // Never leave with copies in flight: wait for the last fill of every stage.
    for (int q = 0; q < NS; ++q) {
      const int fq = issued > q ? (issued - 1 - q) / NS + 1 : 0;  // fills of stage q
      if (fq > 0 && !mbar_wait(&full[q], (uint32_t)((fq - 1) & 1))) atomicOr(&g_stream_fault, 2);
    }
    return;
  }

  const int r = lane >> 2, cq = lane & 3;
  const uint32_t ones[4] = {kOne2, kOne2, kOne2, kOne2};

  if (warp == kPrepWarp) {
    // ----------------- x preparation: B fragments and group sums, once per stage -----------
    if constexpr (kQuant) {
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nunits; ++i) {
        if (!abort_flag[0] && !mbar_wait(&full[s], ph)) {
          abort_flag[0] = 1;
          atomicOr(&g_stream_fault, 8);
        }
        if (!abort_flag[0]) {
          unsigned char* st = smem + s * LY::STAGE;
          float* px = reinterpret_cast<float*>(st + POFF + LY::PB_BYTES);
#pragma unroll
          for (int g = 0; g < UG; ++g)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const unsigned char* xp = st + XOFF + (g >> 2) * LY::XCHUNK + (nt * 8 + r) * 512 + (g & 3) * 128 + cq * 32;
              const uint4 v0 = reinterpret_cast<const uint4*>(xp)[0], v1 = reinterpret_cast<const uint4*>(xp)[1];
              const uint32_t nat[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
              uint32_t B[8];
              permute_xs<BITS>(B, nat);
              uint4* pb = reinterpret_cast<uint4*>(st + POFF + (g * NT + nt) * 1024);
              pb[lane] = make_uint4(B[0], B[1], B[2], B[3]);
              pb[32 + lane] = make_uint4(B[4], B[5], B[6], B[7]);
              float X[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
              for (int j = 0; j < 4; ++j) mma16816<T>(X, ones, B[2 * j], B[2 * j + 1]);
              if (r == 0) *reinterpret_cast<float2*>(px + g * TOK + nt * 8 + 2 * cq) = make_float2(X[0], X[1]);
            }
        }
        mbar_arrive(&prepared[s]);  // also after a fault, so that no consumer waits for it
        if (++s == NS) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    return;
  }

  // --------------------------------- consumers ------------------------------------------
  pdl_wait();  // outputs, residuals and the workspace belong to the preceding kernel until now
  const int slot0 = 16 * warp + r, slot1 = slot0 + 8;  // this warp's weight rows in the unit
  // Byte offsets of this thread's weight fragments in a stage (row slot0; slot1 is 1024 bytes
  // further): the 16-byte unit of a [128 x 128 B] box is swizzled by row % 8 == r.  The
  // group pattern repeats every WPAT groups, and the box index is g / WPAT.
  constexpr int WPAT = BITS == 4 ? 4 : (BITS == 8 ? 2 : 1);
  int woff[BITS ? WPAT : 2];
  if constexpr (BITS == 4) {
#pragma unroll
    for (int G = 0; G < 4; ++G) woff[G] = slot0 * 128 + ((((2 * G) | (cq >> 1)) ^ r) << 4) + (cq & 1) * 8;
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int G = 0; G < 2; ++G) woff[G] = slot0 * 128 + (((4 * G + cq) ^ r) << 4);
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) woff[h] = slot0 * 128 + (((2 * cq + h) ^ r) << 4);
  }
  const int rf = (int)(u0 / nkc), rl = (int)((u1 - 1) / nkc);
  const bool head_shared = u0 % nkc != 0, tail_shared = u1 % nkc != 0;
  float acc[NT][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
  };
  zero_acc();
  const T* bias = static_cast<const T*>(a.bias);
  const T* res = static_cast<const T*>(a.res);
  T* out = static_cast<T*>(a.out);

  // epilogue from registers: GATE -> bias -> GELU -> residual, one rounding.  `up` holds the
  // matching up-row sums with the SiLU gate.
  auto epilogue = [&](int rb, const float (&up)[NT][4]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = nt * 8 + 2 * cq + (e & 1);
        const int n = rb * (GATE ? 64 : 128) + ((e >> 1) ? slot1 : slot0);
        if (tok >= mc || n >= N) continue;
        float v = acc[nt][e];
        if constexpr (GATE) v = v / (1.0f + expf(-v)) * up[nt][e];
        const size_t o = (size_t)tok * N + n;
        if (a.has_bias) v += A::to_f(bias[n]);
        if (a.gelu) v = gelu_erf(v);
        if (a.has_res) v += A::to_f(res[o]);
        out[o] = A::from_f(v);
      }
  };

  UnitWalk cur(u0, u1, nkc);
  int s = 0;
  uint32_t ph = 0;
  for (int i = 0; i < nunits; ++i) {
    if (!abort_flag[0]) {
      const bool ok = mbar_wait(&full[s], ph) && (!kQuant || mbar_wait(&prepared[s], ph));
      if (!ok) {
        abort_flag[0] = 1;
        atomicOr(&g_stream_fault, 4);
      }
    }
    if (!abort_flag[0]) {
      const unsigned char* st = smem + s * LY::STAGE;
      if constexpr (kQuant) {
        // this warp's scales and biases of the unit's UG groups: 16 bytes per row
        const uint4 sv0 = *reinterpret_cast<const uint4*>(st + LY::W_BYTES + slot0 * 16);
        const uint4 sv1 = *reinterpret_cast<const uint4*>(st + LY::W_BYTES + slot1 * 16);
        const uint4 bv0 = *reinterpret_cast<const uint4*>(st + LY::W_BYTES + kSlots * 16 + slot0 * 16);
        const uint4 bv1 = *reinterpret_cast<const uint4*>(st + LY::W_BYTES + kSlots * 16 + slot1 * 16);
        const uint32_t sw0[4] = {sv0.x, sv0.y, sv0.z, sv0.w}, sw1[4] = {sv1.x, sv1.y, sv1.z, sv1.w};
        const uint32_t bw0[4] = {bv0.x, bv0.y, bv0.z, bv0.w}, bw1[4] = {bv1.x, bv1.y, bv1.z, bv1.w};
        const uint4* pb = reinterpret_cast<const uint4*>(st + POFF);
        const float* px = reinterpret_cast<const float*>(st + POFF + LY::PB_BYTES);
#pragma unroll
        for (int g = 0; g < UG; ++g) {
          uint32_t B[NT][8];
          float X[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint4 lo = pb[(g * NT + nt) * 64 + lane], hi = pb[(g * NT + nt) * 64 + 32 + lane];
            B[nt][0] = lo.x; B[nt][1] = lo.y; B[nt][2] = lo.z; B[nt][3] = lo.w;
            B[nt][4] = hi.x; B[nt][5] = hi.y; B[nt][6] = hi.z; B[nt][7] = hi.w;
            const float2 xv = *reinterpret_cast<const float2*>(px + g * TOK + nt * 8 + 2 * cq);
            X[nt][0] = xv.x;
            X[nt][1] = xv.y;
          }
          const unsigned char* wrow = st + (g / WPAT) * LY::WCHUNK + woff[g % WPAT];  // row slot0
          float d[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
          if constexpr (BITS == 4) {
            const uint2 u0v = *reinterpret_cast<const uint2*>(wrow);
            const uint2 u1v = *reinterpret_cast<const uint2*>(wrow + 1024);
            const uint32_t w0[2] = {u0v.x, u0v.y}, w1[2] = {u1v.x, u1v.y};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int sh = (j & 1) * 8;
              const uint32_t p0 = w0[j >> 1], p1 = w1[j >> 1];
              const uint32_t af[4] = {and_or(p0 >> sh, kMask, kMag), and_or(p1 >> sh, kMask, kMag),
                                      and_or(p0 >> (sh + 4), kMask, kMag), and_or(p1 >> (sh + 4), kMask, kMag)};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma16816<T>(d[nt], af, B[nt][2 * j], B[nt][2 * j + 1]);
            }
          } else {
            const uint4 u0v = *reinterpret_cast<const uint4*>(wrow);
            const uint4 u1v = *reinterpret_cast<const uint4*>(wrow + 1024);
            const uint32_t w0[4] = {u0v.x, u0v.y, u0v.z, u0v.w}, w1[4] = {u1v.x, u1v.y, u1v.z, u1v.w};
            float dh[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) dh[nt][e] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t p0 = w0[j], p1 = w1[j];
              const uint32_t lo[4] = {and_or(p0, kMask, kMag), and_or(p1, kMask, kMag), and_or(p0 >> 8, kMask, kMag),
                                      and_or(p1 >> 8, kMask, kMag)};
              const uint32_t hi[4] = {and_or(p0 >> 4, kMask, kMag), and_or(p1 >> 4, kMask, kMag),
                                      and_or(p0 >> 12, kMask, kMag), and_or(p1 >> 12, kMask, kMag)};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                mma16816<T>(d[nt], lo, B[nt][2 * j], B[nt][2 * j + 1]);
                mma16816<T>(dh[nt], hi, B[nt][2 * j], B[nt][2 * j + 1]);
              }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) d[nt][e] = fmaf(16.0f, dh[nt][e], d[nt][e]);
          }
          // scale/bias of group g: 16-bit half (g & 1) of word (g >> 1)
          const float s0 = (g & 1) ? A::hi(sw0[g >> 1]) : A::lo(sw0[g >> 1]);
          const float s1 = (g & 1) ? A::hi(sw1[g >> 1]) : A::lo(sw1[g >> 1]);
          const float b0 = fmaf(-kOff, s0, (g & 1) ? A::hi(bw0[g >> 1]) : A::lo(bw0[g >> 1]));
          const float b1 = fmaf(-kOff, s1, (g & 1) ? A::hi(bw1[g >> 1]) : A::lo(bw1[g >> 1]));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = fmaf(s0, d[nt][0], fmaf(b0, X[nt][0], acc[nt][0]));
            acc[nt][1] = fmaf(s0, d[nt][1], fmaf(b0, X[nt][1], acc[nt][1]));
            acc[nt][2] = fmaf(s1, d[nt][2], fmaf(b1, X[nt][0], acc[nt][2]));
            acc[nt][3] = fmaf(s1, d[nt][3], fmaf(b1, X[nt][1], acc[nt][3]));
          }
        }
      } else {
        // dense weights: B fragments straight from the x slice (natural order)
        const unsigned char* sx = st + XOFF;
#pragma unroll
        for (int g = 0; g < UG; ++g) {
          uint32_t B[NT][8];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const unsigned char* xp = sx + (g >> 2) * LY::XCHUNK + (nt * 8 + r) * 512 + (g & 3) * 128 + cq * 32;
            const uint4 v0 = reinterpret_cast<const uint4*>(xp)[0], v1 = reinterpret_cast<const uint4*>(xp)[1];
            B[nt][0] = v0.x; B[nt][1] = v0.y; B[nt][2] = v0.z; B[nt][3] = v0.w;
            B[nt][4] = v1.x; B[nt][5] = v1.y; B[nt][6] = v1.z; B[nt][7] = v1.w;
          }
          const unsigned char* wbox = st + g * LY::WCHUNK;
          const uint4 a0 = *reinterpret_cast<const uint4*>(wbox + woff[0]);
          const uint4 a1 = *reinterpret_cast<const uint4*>(wbox + woff[1]);
          const uint4 b0 = *reinterpret_cast<const uint4*>(wbox + woff[0] + 1024);
          const uint4 b1 = *reinterpret_cast<const uint4*>(wbox + woff[1] + 1024);
          const uint32_t w0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const uint32_t w1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t af[4] = {w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1]};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816<T>(acc[nt], af, B[nt][2 * j], B[nt][2 * j + 1]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == NS) {
      s = 0;
      ph ^= 1u;
    }

    // ---- end of a row block (or of a segment of this CTA's range) -----------------------
    const int rb = cur.rb;
    const bool flush = cur.seg_last() || cur.kc + 1 == nkc;
    cur.next(nkc);
    if (!flush) continue;
    int* wflags = a.flags + warp;  // this warp's flag of every CTA: wflags[c * kRowWarps]
    if (rb == rl && tail_shared) {
      // publish: the row block continues in the next CTA, which gathers it
      float* part = a.partial + (size_t)c * kTokMax * kSlots;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = nt * 8 + 2 * cq + (e & 1);
          if (tok < mc) part[tok * kSlots + ((e >> 1) ? slot1 : slot0)] = acc[nt][e];
        }
      __syncwarp();
      if (lane == 0) {
        __threadfence();
        *reinterpret_cast<volatile int*>(wflags + (size_t)c * kRowWarps) = 1;
      }
      zero_acc();
      continue;
    }
    if (rb == rf && head_shared) {
      // gather: add the partial sums of the earlier CTAs (in CTA order), then this CTA's
      const int cf = cta_of((long long)rb * nkc, U, P);
      if (lane == 0) {
        for (int c2 = cf; c2 < c; ++c2) {
          const int* f = wflags + (size_t)c2 * kRowWarps;
          if (ld_flag(f) == 0) {
            const long long t0 = clock64();
            while (ld_flag(f) == 0) {
              if (clock64() - t0 > kWaitCycles) {
                atomicOr(&g_stream_fault, 16);
                break;
              }
            }
          }
        }
        __threadfence();
      }
      __syncwarp();
      float sum[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sum[nt][e] = 0.0f;
      constexpr int RQ = 4;  // contributors whose loads are in flight together
#pragma unroll 1
      for (int cc = cf; cc < c; cc += RQ) {
        float tmp[RQ][NT][4];
#pragma unroll
        for (int q = 0; q < RQ; ++q) {
          const float* pp = a.partial + (size_t)min(cc + q, c - 1) * kTokMax * kSlots;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int tok = nt * 8 + 2 * cq + (e & 1);
              tmp[q][nt][e] = (cc + q < c && tok < mc) ? __ldcg(pp + tok * kSlots + ((e >> 1) ? slot1 : slot0)) : 0.0f;
            }
        }
#pragma unroll
        for (int q = 0; q < RQ; ++q)
          if (cc + q < c)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) sum[nt][e] += tmp[q][nt][e];
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = sum[nt][e] + acc[nt][e];
      __syncwarp();
      if (lane == 0)  // consumed: leave the flags at zero for the next call
        for (int c2 = cf; c2 < c; ++c2) wflags[(size_t)c2 * kRowWarps] = 0;
    }
    if constexpr (GATE) {
      // up-row warp w + 4 hands its sums to gate-row warp w
      const int pw = warp & 3;
      float* rp = red + pw * 16 * TOK;
      if (warp >= 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) rp[((e >> 1) * 8 + r) * TOK + nt * 8 + 2 * cq + (e & 1)] = acc[nt][e];
      }
      named_sync(kBarPair0 + pw, 64);
      if (warp < 4) {
        float up[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) up[nt][e] = rp[((e >> 1) * 8 + r) * TOK + nt * 8 + 2 * cq + (e & 1)];
        epilogue(rb, up);
      }
      named_sync(kBarPair0 + pw, 64);  // the exchange area is free again
    } else if (a.rope) {
      // head rb: dims 0..63 live in warps 0..3, their rotation partners 64..127 in warps
      // 4..7; both are rounded to T first (the projection's output), then rotated
      const int pw = warp & 3;
      float* rp = red + pw * 16 * TOK;
      if (warp >= 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) rp[((e >> 1) * 8 + r) * TOK + nt * 8 + 2 * cq + (e & 1)] = acc[nt][e];
      }
      named_sync(kBarPair0 + pw, 64);
      if (warp < 4) {
        const RopeEpi& re = a.re;
        const int H = re.H, KV = re.KV;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = nt * 8 + 2 * cq + (e & 1);
            if (tok >= mc) continue;
            const int i = (e >> 1) ? slot1 : slot0;  // 0..63
            const float x1 = A::to_f(A::from_f(acc[nt][e]));
            const float x2 = A::to_f(A::from_f(rp[((e >> 1) * 8 + r) * TOK + nt * 8 + 2 * cq + (e & 1)]));
            const int pos = re.pr.pos(tok);
            if (pos < 0 || pos >= re.max_seq) {
              atomicOr(re.err, 2);
              continue;
            }
            float y1 = x1, y2 = x2;
            if (rb < H + KV) {
              const float2 c = re.cs[(size_t)pos * 64 + i];
              y1 = rope_rot1(x1, x2, c);
              y2 = rope_rot2(x1, x2, c);
            }
            T* dst;
            if (rb < H) {
              dst = static_cast<T*>(re.q) + ((size_t)tok * H + rb) * 128;
            } else {
              const size_t so = (size_t)re.pr.stream_of(tok) * re.kv_ss;
              T* base = static_cast<T*>(rb < H + KV ? re.kc : re.vc) + so;
              dst = base + ((size_t)(rb < H + KV ? rb - H : rb - H - KV) * re.max_seq + pos) * 128;
            }
            dst[i] = A::from_f(y1);
            dst[i + 64] = A::from_f(y2);
          }
      }
      named_sync(kBarPair0 + pw, 64);
    } else {
      epilogue(rb, acc);
    }
    zero_acc();
  }
}

template <typename T, int BITS, int NT, bool GATE, bool LIGHT>
int launch_stream_t(const SArgs& a, cudaStream_t stream) {
  using LY = Layout<BITS, NT, LIGHT>;
  auto k = qgemm_stream_kernel<T, BITS, NT, GATE, LIGHT>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::TOTAL));
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  return launch_kernel(k, dim3(a.P), dim3(kThreads), LY::TOTAL, stream, a);
}

template <typename T, int BITS, bool LIGHT>
int dispatch_stream(const SArgs& a, bool gate, int nt, cudaStream_t s) {
  if (gate)
    return nt == 1 ? launch_stream_t<T, BITS, 1, true, LIGHT>(a, s) : launch_stream_t<T, BITS, 2, true, LIGHT>(a, s);
  return nt == 1 ? launch_stream_t<T, BITS, 1, false, LIGHT>(a, s) : launch_stream_t<T, BITS, 2, false, LIGHT>(a, s);
}

}  // namespace

// The streaming kernel takes calls of 1 <= M <= 16 whose K suits its unit: K % 512 == 0
// for the quantized formats (scales/biases move in 16-byte rows), K % 256 == 0 for dense.
bool stream_eligible(const vella_qgemm_desc& d) {
  if (d.m < 1 || d.m > kTokMax) return false;
  if (d.bits == 0) return d.k % 256 == 0;
  return d.k % 512 == 0;
}

int stream_units(const vella_qgemm_desc& d, int* rowblocks, int* nkc) {
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  *rowblocks = (d.n + (gate ? 63 : 127)) / (gate ? 64 : 128);
  *nkc = d.k / 64 / (d.bits ? 8 : 4);
  return VELLA_OK;
}

// Two CTAs per SM pay off for int4 once every CTA streams four or more units; the M <= 8
// and M <= 16 forms both follow this rule, so the K split (and with it every row's value)
// never depends on M.  The M <= 16 form's two stages do not fit twice in an SM: its CTAs
// then run in two waves, which the gather order allows (a CTA waits on lower-numbered ones
// only).
bool stream_light(const vella_qgemm_desc& d, int rowblocks, int nkc, int sms) {
  return d.bits == 4 && (long long)rowblocks * nkc >= 8LL * sms;
}

size_t stream_partial_bytes(int P) { return (size_t)P * kTokMax * kSlots * sizeof(float); }

int stream_flag_count(int P) { return P * kRowWarps; }

int stream_launch(const vella_qgemm_desc& d, int P, bool light, const void* x, const void* w, const void* scales,
                  const void* biases, const void* up_w, const void* up_scales, const void* up_biases,
                  const void* bias, const void* residual, void* out, int* flags, float* partial,
                  cudaStream_t stream, const RopeEpi* rope) {
  SArgs a;
  std::memset(&a, 0, sizeof a);
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  const int nt = d.m <= 8 ? 1 : 2;
  const int rows_box = gate ? 64 : 128;
  const int wbits = d.bits ? d.bits : 16;
  const uint64_t words = (uint64_t)d.k * wbits / 32, row_bytes = (uint64_t)d.k * wbits / 8;
  const uint64_t G = d.k / 64;
  int rc;
  if ((rc = make_tensor_map(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, words, d.n, row_bytes, 32, rows_box,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (gate && (rc = make_tensor_map(&a.tu, CU_TENSOR_MAP_DATA_TYPE_UINT32, up_w, words, d.n, row_bytes, 32, rows_box,
                             CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (d.bits) {
    if ((rc = make_tensor_map(&a.ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, scales, G, d.n, G * 2, 8, rows_box,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    if ((rc = make_tensor_map(&a.tb, CU_TENSOR_MAP_DATA_TYPE_UINT16, biases, G, d.n, G * 2, 8, rows_box,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    if (gate) {
      if ((rc = make_tensor_map(&a.tus, CU_TENSOR_MAP_DATA_TYPE_UINT16, up_scales, G, d.n, G * 2, 8, rows_box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
      if ((rc = make_tensor_map(&a.tub, CU_TENSOR_MAP_DATA_TYPE_UINT16, up_biases, G, d.n, G * 2, 8, rows_box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    }
  }
  if ((rc = make_tensor_map(&a.tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, x, d.k, d.m, (uint64_t)d.k * 2, 256, nt * 8,
                     CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  a.bias = bias; a.res = residual; a.out = out;
  a.partial = partial; a.flags = flags;
  a.M = d.m; a.N = d.n; a.K = d.k; a.G = d.k / 64; a.P = P;
  stream_units(d, &a.rowblocks, &a.nkc);
  a.has_bias = epi_bias(d.epilogue);
  a.has_res = epi_residual(d.epilogue);
  a.gelu = epi_gelu(d.epilogue);
  if (rope) {
    if (gate || d.epilogue != VELLA_EPI_NONE || d.n % 128 != 0 || d.n / 128 != rope->H + 2 * rope->KV)
      return fail(VELLA_E_INVALID, "stream GEMM: RoPE epilogue needs a plain q|k|v projection of 128-row heads");
    a.rope = 1;
    a.re = *rope;
  }
  if (light && d.bits != 4) return fail(VELLA_E_INVALID, "stream GEMM: the compact layout is int4 only");
  if (d.dtype == VELLA_BF16) {
    switch (d.bits) {
      case 4:
        return light ? dispatch_stream<__nv_bfloat16, 4, true>(a, gate, nt, stream)
                     : dispatch_stream<__nv_bfloat16, 4, false>(a, gate, nt, stream);
      case 8: return dispatch_stream<__nv_bfloat16, 8, false>(a, gate, nt, stream);
      default: return dispatch_stream<__nv_bfloat16, 0, false>(a, gate, nt, stream);
    }
  }
  switch (d.bits) {
    case 4:
      return light ? dispatch_stream<__half, 4, true>(a, gate, nt, stream)
                   : dispatch_stream<__half, 4, false>(a, gate, nt, stream);
    case 8: return dispatch_stream<__half, 8, false>(a, gate, nt, stream);
    default: return dispatch_stream<__half, 0, false>(a, gate, nt, stream);
  }
}

int stream_fault_status(int clear) {  // the flags, or -1 when they cannot be read
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_stream_fault, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_stream_fault, &zero, sizeof(int)) != cudaSuccess) cudaGetLastError();
  }
  return v;
}

}  // namespace vella
