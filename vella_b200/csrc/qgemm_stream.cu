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
//   * eight consumer warps (4 row sets x 2 group sets) run the MMAs out of shared memory.
//   * work unit u = (row block, k chunk); CTA c streams units [c U/P, (c+1) U/P), i.e. a
//     few whole row blocks plus a partial one at each end, so K-split partial sums only
//     exist at range edges.  A row block split between CTAs is finished by the CTA that
//     takes the last ticket, which adds the partials in CTA order.
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
#include "sm100.cuh"

namespace vella {

__device__ int g_stream_fault = 0;  // set when a pipeline wait ran out of time

namespace {

constexpr int kGroupSets = 2;                  // consumer warps split each unit's groups this many ways
constexpr int kConsumerWarps = 4 * kGroupSets;  // 4 row sets x kGroupSets group sets
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSlots = 128;
constexpr int kTokMax = 16;

// UG groups of 64 per unit; BPG bytes per row and group; WCH 128-byte column chunks of the
// weight tile; XCH 256-element chunks of the x slice.
template <int BITS> struct SFmt;
template <> struct SFmt<4> { static constexpr int UG = 8, BPG = 32, WCH = 2, XCH = 2; };
template <> struct SFmt<8> { static constexpr int UG = 8, BPG = 64, WCH = 4, XCH = 2; };
template <> struct SFmt<0> { static constexpr int UG = 4, BPG = 128, WCH = 4, XCH = 1; };

template <int BITS, int NT>
struct Layout {
  static constexpr int TOK = NT * 8;
  static constexpr int WCHUNK = kSlots * 128;                 // one [128 rows x 128 B] box
  static constexpr int W_BYTES = SFmt<BITS>::WCH * WCHUNK;
  static constexpr int SB_BYTES = BITS ? 2 * kSlots * 16 : 0;  // scales [128][16 B], biases [128][16 B]
  static constexpr int XCHUNK = TOK * 512;                    // one [TOK x 256 elements] box
  static constexpr int X_BYTES = SFmt<BITS>::XCH * XCHUNK;
  static constexpr int STAGE = W_BYTES + SB_BYTES + X_BYTES;  // multiple of 1024
  static constexpr int NS = BITS == 8 ? 2 : (BITS == 4 ? (NT == 1 ? 4 : 3) : (NT == 1 ? 3 : 2));
  static constexpr int RED = (kGroupSets - 1) * TOK * (kSlots + 4) * 4;  // partial tiles of group sets 1..3
  static constexpr int TOTAL = 1024 + NS * STAGE + RED + 2 * NS * 8 + 16;
};

struct SArgs {
  CUtensorMap tw, tu, ts, tb, tus, tub, tx;
  const void* bias;
  const void* res;
  void* out;
  float* partial;  // [P][2][16][128]
  int* counters;   // [rowblocks]
  int M, N, K, G, rowblocks, nkc, P;
  int has_bias, has_res, gelu;
};

using namespace sm100;

// CTA holding unit u when U units are split over P CTAs as [c U/P, (c+1) U/P) (U >= P).
__device__ __forceinline__ int cta_of(long long u, long long U, int P) { return (int)(((u + 1) * P - 1) / U); }
__device__ __forceinline__ long long unit0(int c, long long U, int P) { return (long long)c * U / P; }

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

// Byte address in a swizzled [128 rows x 128 B] box: 16-byte unit u of row `row` sits at
// unit u ^ (row % 8).
__device__ __forceinline__ const unsigned char* swz(const unsigned char* box, int row, int byte) {
  return box + row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15));
}

template <typename T, int BITS, int NT, bool GATE>
__global__ void __launch_bounds__(kThreads, 1) qgemm_stream_kernel(const __grid_constant__ SArgs a) {
  using A = Act<T>;
  using LY = Layout<BITS, NT>;
  constexpr int UG = SFmt<BITS>::UG, BPG = SFmt<BITS>::BPG, NS = LY::NS, TOK = LY::TOK;
  constexpr int GPW = UG / kGroupSets;  // groups per consumer warp and unit
  constexpr int REDSET = LY::TOK * (kSlots + 4);
  constexpr bool kQuant = BITS != 0;
  constexpr uint32_t kMask = 0x000F000Fu;
  constexpr uint32_t kMag = A::kMagic2;
  constexpr float kOff = BITS == 4 ? A::kMagic : 17.0f * A::kMagic;
  constexpr uint32_t kOne2 = A::kMagic == 128.0f ? 0x3F803F80u : 0x3C003C00u;
  constexpr uint32_t kBytes = LY::STAGE;  // every box is counted whole (out-of-range parts are zero-filled)

  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + NS * LY::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * LY::STAGE + LY::RED);
  uint64_t* empty = full + NS;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + NS);  // [0] abort, [1] last ticket

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, P = a.P;
  const long long U = (long long)a.rowblocks * a.nkc;
  const long long u0 = unit0(c, U, P), u1 = unit0(c + 1, U, P);
  const int mc = min(a.M, kTokMax);
  const int N = a.N;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_next();

  if (warp == kConsumerWarps) {
    // ------------------------------- producer (one thread) ------------------------------
    if (lane != 0) return;
    int fills[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) fills[s] = 0;
    // weights, scales and biases of a unit (constant data: may be read before the
    // preceding kernel has finished)
    auto issue_w = [&](long long u, int s) {
      const int rb = (int)(u / a.nkc), kc = (int)(u % a.nkc);
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
    auto issue_x = [&](long long u, int s) {
      const int kc = (int)(u % a.nkc);
      unsigned char* st = smem + s * LY::STAGE;
#pragma unroll
      for (int j = 0; j < SFmt<BITS>::XCH; ++j)
        tma2d(st + LY::W_BYTES + LY::SB_BYTES + j * LY::XCHUNK, &a.tx, kc * UG * 64 + j * 256, 0, &full[s]);
    };
    // first round of the ring: weights before the dependency wait, x after it
    const long long npre = (u1 - u0) < NS ? (u1 - u0) : NS;
    for (long long j = 0; j < npre; ++j) {
      mbar_expect_tx(&full[j], kBytes);
      fills[j]++;
      issue_w(u0 + j, (int)j);
    }
    pdl_wait();
    for (long long j = 0; j < npre; ++j) issue_x(u0 + j, (int)j);
    long long i = npre;
    for (long long u = u0 + npre; u < u1; ++u, ++i) {
      const int s = (int)(i % NS);
      const uint32_t ph = (uint32_t)((i / NS) & 1);
      if (flags[0]) break;
      if (!mbar_wait(&empty[s], ph ^ 1)) {
        flags[0] = 1;
        atomicOr(&g_stream_fault, 1);
        break;
      }
      mbar_expect_tx(&full[s], kBytes);
      fills[s]++;
      issue_w(u, s);
      issue_x(u, s);
    }
    // Never leave with copies in flight: wait for the last fill of every stage.
    for (int s = 0; s < NS; ++s)
      if (fills[s] > 0 && !mbar_wait(&full[s], (uint32_t)((fills[s] - 1) & 1))) atomicOr(&g_stream_fault, 2);
    return;
  }

  // --------------------------------- consumers ------------------------------------------
  pdl_wait();  // outputs, residuals and the workspace belong to the preceding kernel until now
  const int r = lane >> 2, cq = lane & 3;
  const int rs = warp & 3, gs = warp >> 2;
  int slot[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t = q >> 1, h = q & 1;
    slot[q] = GATE ? t * 64 + rs * 16 + h * 8 + r : rs * 32 + t * 16 + h * 8 + r;
  }
  const uint32_t ones[4] = {kOne2, kOne2, kOne2, kOne2};
  float acc[2][NT][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][nt][e] = 0.0f;
  };
  zero_acc();
  const T* bias = static_cast<const T*>(a.bias);
  const T* res = static_cast<const T*>(a.res);
  T* out = static_cast<T*>(a.out);

  // epilogue from registers (group-set 0 warps only): GATE -> bias -> residual, one rounding
  auto epilogue = [&](int rb) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = nt * 8 + 2 * cq + (e & 1);
        if (tok >= mc) continue;
#pragma unroll
        for (int t = 0; t < (GATE ? 1 : 2); ++t) {
          const int sl = GATE ? rs * 16 + (e >> 1) * 8 + r : rs * 32 + t * 16 + (e >> 1) * 8 + r;
          const int n = rb * (GATE ? 64 : 128) + sl;
          if (n >= N) continue;
          float v = acc[t][nt][e];
          if constexpr (GATE) v = v / (1.0f + expf(-v)) * acc[1][nt][e];
          const size_t o = (size_t)tok * N + n;
          if (a.has_bias) v += A::to_f(bias[n]);
          if (a.gelu) v = gelu_erf(v);
          if (a.has_res) v += A::to_f(res[o]);
          out[o] = A::from_f(v);
        }
      }
  };

  long long i = 0;
  for (long long u = u0; u < u1; ++u, ++i) {
    const int s = (int)(i % NS);
    const uint32_t ph = (uint32_t)((i / NS) & 1);
    if (!flags[0] && !mbar_wait(&full[s], ph)) {
      flags[0] = 1;
      atomicOr(&g_stream_fault, 4);
    }
    if (!flags[0]) {
      const unsigned char* st = smem + s * LY::STAGE;
      const unsigned char* sx = st + LY::W_BYTES + LY::SB_BYTES;
      // this warp's scales and biases for its GPW groups, 4 rows
      constexpr int SBW = (GPW + 1) / 2;  // 32-bit words holding this warp's GPW scales (biases)
      uint32_t sw[4][SBW], bw[4][SBW];
      if constexpr (kQuant) {
        static_assert(GPW % 2 == 0, "quantized group sets own whole 32-bit words of scales");
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int wd = 0; wd < SBW; ++wd) {
            sw[q][wd] = *reinterpret_cast<const uint32_t*>(st + LY::W_BYTES + slot[q] * 16 + gs * GPW * 2 + 4 * wd);
            bw[q][wd] =
                *reinterpret_cast<const uint32_t*>(st + LY::W_BYTES + kSlots * 16 + slot[q] * 16 + gs * GPW * 2 + 4 * wd);
          }
      }
#pragma unroll
      for (int gi = 0; gi < GPW; ++gi) {
        const int g = gs * GPW + gi;
        uint32_t B[NT][8];
        float X[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const unsigned char* xp = sx + (g >> 2) * LY::XCHUNK + (nt * 8 + r) * 512 + (g & 3) * 128 + cq * 32;
          const uint4 v0 = reinterpret_cast<const uint4*>(xp)[0], v1 = reinterpret_cast<const uint4*>(xp)[1];
          const uint32_t nat[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
          permute_xs<BITS>(B[nt], nat);
          if constexpr (kQuant) {
#pragma unroll
            for (int e = 0; e < 4; ++e) X[nt][e] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) mma16816<T>(X[nt], ones, B[nt][2 * j], B[nt][2 * j + 1]);
          }
        }
        // weight fragment location: 128-byte column chunk and byte within the row
        const int wbyte = g * BPG + cq * (BPG / 4);
        const unsigned char* wbox = st + (wbyte >> 7) * LY::WCHUNK;
        const int wb = wbyte & 127;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int r0 = slot[2 * t], r1 = slot[2 * t + 1];
          if constexpr (BITS == 0) {
            const uint4 a0 = *reinterpret_cast<const uint4*>(swz(wbox, r0, wb));
            const uint4 a1 = *reinterpret_cast<const uint4*>(swz(wbox, r0, wb + 16));
            const uint4 b0 = *reinterpret_cast<const uint4*>(swz(wbox, r1, wb));
            const uint4 b1 = *reinterpret_cast<const uint4*>(swz(wbox, r1, wb + 16));
            const uint32_t w0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const uint32_t w1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t af[4] = {w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1]};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma16816<T>(acc[t][nt], af, B[nt][2 * j], B[nt][2 * j + 1]);
            }
          } else {
            float d[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
            if constexpr (BITS == 4) {
              const uint2 u0v = *reinterpret_cast<const uint2*>(swz(wbox, r0, wb));
              const uint2 u1v = *reinterpret_cast<const uint2*>(swz(wbox, r1, wb));
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
              const uint4 u0v = *reinterpret_cast<const uint4*>(swz(wbox, r0, wb));
              const uint4 u1v = *reinterpret_cast<const uint4*>(swz(wbox, r1, wb));
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
            // scale/bias of group gi: 16-bit half (gi & 1) of word (gi >> 1)
            const uint32_t s0w = sw[2 * t][gi >> 1], s1w = sw[2 * t + 1][gi >> 1];
            const uint32_t b0w = bw[2 * t][gi >> 1], b1w = bw[2 * t + 1][gi >> 1];
            const float s0 = (gi & 1) ? A::hi(s0w) : A::lo(s0w), s1 = (gi & 1) ? A::hi(s1w) : A::lo(s1w);
            const float b0 = fmaf(-kOff, s0, (gi & 1) ? A::hi(b0w) : A::lo(b0w));
            const float b1 = fmaf(-kOff, s1, (gi & 1) ? A::hi(b1w) : A::lo(b1w));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[t][nt][0] = fmaf(s0, d[nt][0], fmaf(b0, X[nt][0], acc[t][nt][0]));
              acc[t][nt][1] = fmaf(s0, d[nt][1], fmaf(b0, X[nt][1], acc[t][nt][1]));
              acc[t][nt][2] = fmaf(s1, d[nt][2], fmaf(b1, X[nt][0], acc[t][nt][2]));
              acc[t][nt][3] = fmaf(s1, d[nt][3], fmaf(b1, X[nt][1], acc[t][nt][3]));
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // ---- flush at the end of a row block (or of this CTA's range) ---------------------
    const int rb = (int)(u / a.nkc);
    if (u + 1 == u1 || (u + 1) / a.nkc != rb) {
      const long long rb_u0 = (long long)rb * a.nkc, rb_u1 = rb_u0 + a.nkc - 1;
      const int cf = cta_of(rb_u0, U, P), cl = cta_of(rb_u1, U, P);
      if (gs > 0) {
        float* rd = red + (gs - 1) * REDSET;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e)
              rd[(nt * 8 + 2 * cq + (e & 1)) * (kSlots + 4) + slot[2 * t + (e >> 1)]] = acc[t][nt][e];
      }
      named_sync(1, kConsumerWarps * 32);
      if (gs == 0) {
        // group sets added in order 0 + 1 + 2 + 3
#pragma unroll
        for (int gsi = 0; gsi < kGroupSets - 1; ++gsi)
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                acc[t][nt][e] += red[gsi * REDSET + (nt * 8 + 2 * cq + (e & 1)) * (kSlots + 4) + slot[2 * t + (e >> 1)]];
        if (cf == cl) {
          epilogue(rb);
        } else {
          const int sidx = (rb == (int)(u0 / a.nkc)) ? 0 : 1;
          float* part = a.partial + ((size_t)c * 2 + sidx) * kTokMax * kSlots;
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int tok = nt * 8 + 2 * cq + (e & 1);
                if (tok < mc) part[tok * kSlots + slot[2 * t + (e >> 1)]] = acc[t][nt][e];
              }
          __threadfence();
          named_sync(2, 4 * 32);
          if (tid == 0) {
            const int prev = atomicAdd(&a.counters[rb], 1);
            const int last = prev == cl - cf;
            if (last) a.counters[rb] = 0;
            flags[1] = last;
          }
          named_sync(2, 4 * 32);
          if (flags[1]) {
            __threadfence();
            zero_acc();
            // the contributors' partials, added in CTA order; loads of four CTAs in flight at once
#pragma unroll 1
            for (int cc = cf; cc <= cl; cc += 4) {
              float tmp[4][2][NT][4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int c2 = cc + q;
                const int si = (c2 <= cl && rb == (int)(unit0(c2, U, P) / a.nkc)) ? 0 : 1;
                const float* pp = a.partial + ((size_t)min(c2, cl) * 2 + si) * kTokMax * kSlots;
#pragma unroll
                for (int t = 0; t < 2; ++t)
#pragma unroll
                  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const int tok = nt * 8 + 2 * cq + (e & 1);
                      tmp[q][t][nt][e] = (c2 <= cl && tok < mc) ? __ldcg(pp + tok * kSlots + slot[2 * t + (e >> 1)]) : 0.0f;
                    }
              }
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (cc + q <= cl)
#pragma unroll
                  for (int t = 0; t < 2; ++t)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                      for (int e = 0; e < 4; ++e) acc[t][nt][e] += tmp[q][t][nt][e];
            }
            epilogue(rb);
          }
        }
      }
      named_sync(1, kConsumerWarps * 32);
      zero_acc();
    }
  }
}

template <typename T, int BITS, int NT, bool GATE>
int launch_stream_t(const SArgs& a, cudaStream_t stream) {
  using LY = Layout<BITS, NT>;
  auto k = qgemm_stream_kernel<T, BITS, NT, GATE>;
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

template <typename T, int BITS>
int dispatch_stream(const SArgs& a, bool gate, int nt, cudaStream_t s) {
  if (gate) return nt == 1 ? launch_stream_t<T, BITS, 1, true>(a, s) : launch_stream_t<T, BITS, 2, true>(a, s);
  return nt == 1 ? launch_stream_t<T, BITS, 1, false>(a, s) : launch_stream_t<T, BITS, 2, false>(a, s);
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

size_t stream_partial_bytes(int P) { return (size_t)P * 2 * kTokMax * kSlots * sizeof(float); }

int stream_launch(const vella_qgemm_desc& d, int P, const void* x, const void* w, const void* scales,
                  const void* biases, const void* up_w, const void* up_scales, const void* up_biases,
                  const void* bias, const void* residual, void* out, int* counters, float* partial,
                  cudaStream_t stream) {
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
  a.partial = partial; a.counters = counters;
  a.M = d.m; a.N = d.n; a.K = d.k; a.G = d.k / 64; a.P = P;
  stream_units(d, &a.rowblocks, &a.nkc);
  a.has_bias = epi_bias(d.epilogue);
  a.has_res = epi_residual(d.epilogue);
  a.gelu = epi_gelu(d.epilogue);
  if (d.dtype == VELLA_BF16) {
    switch (d.bits) {
      case 4: return dispatch_stream<__nv_bfloat16, 4>(a, gate, nt, stream);
      case 8: return dispatch_stream<__nv_bfloat16, 8>(a, gate, nt, stream);
      default: return dispatch_stream<__nv_bfloat16, 0>(a, gate, nt, stream);
    }
  }
  switch (d.bits) {
    case 4: return dispatch_stream<__half, 4>(a, gate, nt, stream);
    case 8: return dispatch_stream<__half, 8>(a, gate, nt, stream);
    default: return dispatch_stream<__half, 0>(a, gate, nt, stream);
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
