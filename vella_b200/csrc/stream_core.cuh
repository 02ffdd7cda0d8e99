// The small-M streaming GEMM's per-role device code, shared by the one-GEMM kernel
// (qgemm_stream.cu) and the persistent decode forward (fwd_prog.cu): stage layout, the unit
// walk, the x preparation of a stage, one stage's MMA work of a consumer warp, and the end
// of a row block (split-K publish / gather, SiLU-gate pairing, RoPE + KV append, epilogue).
//
// Arithmetic (reference SmallMGEMM.swift:662-755, product form): per group of 64,
// acc += s * sum(x * q) + b' * sum(x) with b' = b - magic * s, sum(x * (magic + q)) on
// m16n8k16 with the weights as the A operand (swap-AB), sum(x) through an all-ones MMA, fp32
// throughout, the epilogue (SiLU gate, bias, GELU, residual) rounded once.  A row's sums
// never depend on the other rows of the call.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "layers.cuh"
#include "sm100.cuh"

namespace vella {
namespace sk {

using namespace sm100;

constexpr int kRowWarps = 8;                 // consumer warps, 16 weight rows each
constexpr int kProducerWarp = kRowWarps;     // one TMA thread
constexpr int kPrepWarp = kRowWarps + 1;     // x preparation (quantized formats)
constexpr int kThreads = (kRowWarps + 2) * 32;
constexpr int kSlots = 128;
constexpr int kTokMax = 16;
constexpr int kBarPair0 = 2;  // named barriers 2..5: gate-row warp w with up-row warp w + 4
constexpr int kBarConsumers = 6;  // named barrier 6: the kRowWarps consumer warps

// UG groups of 64 per unit; BPG bytes per row and group; WCH 128-byte column chunks of the
// weight tile; XCH 256-element chunks of the x slice.
template <int BITS> struct SFmt;
template <> struct SFmt<4> { static constexpr int UG = 8, BPG = 32, WCH = 2, XCH = 2; };
template <> struct SFmt<8> { static constexpr int UG = 8, BPG = 64, WCH = 4, XCH = 2; };
template <> struct SFmt<0> { static constexpr int UG = 4, BPG = 128, WCH = 4, XCH = 1; };

// One ring stage: weights [128 rows x UG groups] (128-byte swizzled boxes), scales and biases,
// the raw x slice, then (quantized) the prepared B fragments and the x group sums.
template <int BITS, int NT>
struct Tile {
  static constexpr int TOK = NT * 8;
  static constexpr int UG = SFmt<BITS>::UG;
  static constexpr int WCHUNK = kSlots * 128;                 // one [128 rows x 128 B] box
  static constexpr int W_BYTES = SFmt<BITS>::WCH * WCHUNK;
  static constexpr int SB_BYTES = BITS ? 2 * kSlots * 16 : 0;  // scales [128][16 B], biases [128][16 B]
  static constexpr int XCHUNK = TOK * 512;                    // one [TOK x 256 elements] box
  static constexpr int X_BYTES = SFmt<BITS>::XCH * XCHUNK;
  static constexpr int PB_BYTES = BITS ? UG * NT * 1024 : 0;  // B fragments [g][nt][half][lane] x 16 B
  static constexpr int PX_BYTES = BITS ? UG * TOK * 4 : 0;    // x group sums [g][token], fp32
  static constexpr int TX_W = W_BYTES + SB_BYTES;             // bytes of the weight copies of a stage
  static constexpr int TX_X = X_BYTES;                        // bytes of the x copies of a stage
  static constexpr int TX = TX_W + TX_X;
  static constexpr int STAGE = (TX + PB_BYTES + PX_BYTES + 1023) / 1024 * 1024;
  static constexpr int XOFF = W_BYTES + SB_BYTES;             // raw x slice within a stage
  static constexpr int POFF = XOFF + X_BYTES;                 // prepared B fragments, then x sums
  // The x part of a stage (raw x slice, B fragments, x sums) may also live apart from the
  // weight part: XS bytes, the B fragments P_REL bytes into it (a layout without the raw slice
  // passes its own offset, 0, to the functions below).
  static constexpr int XS = X_BYTES + PB_BYTES + PX_BYTES;
  static constexpr int P_REL = X_BYTES;
  static constexpr int RED = 64 * TOK * 4;                    // up-row sums handed to the gate warps
};

// CTA holding unit u when U units are split over P CTAs as [c U/P, (c+1) U/P).
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
    const long long rf = u0 / nkc, rl = u1 > u0 ? (u1 - 1) / nkc : rf;
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

// x preparation of one (group, token tile) of a stage by the prep warp: the MMA's B fragments
// of the lane's 16 x values (v0, v1: row nt * 8 + r, columns g * 64 + cq * 16 ..) in the order
// the code unpacking produces the A fragments, and sum(x) per group and token.
template <typename T, int BITS, int NT, int PREL = Tile<BITS, NT>::P_REL>
__device__ __forceinline__ void prep_one(unsigned char* xs, int g, int nt, int lane, uint4 v0, uint4 v1) {
  using A = Act<T>;
  using TL = Tile<BITS, NT>;
  constexpr uint32_t kOne2 = A::kMagic == 128.0f ? 0x3F803F80u : 0x3C003C00u;
  const uint32_t ones[4] = {kOne2, kOne2, kOne2, kOne2};
  const int r = lane >> 2, cq = lane & 3;
  float* px = reinterpret_cast<float*>(xs + PREL + TL::PB_BYTES);
  const uint32_t nat[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  uint32_t B[8];
  permute_xs<BITS>(B, nat);
  uint4* pb = reinterpret_cast<uint4*>(xs + PREL + (g * NT + nt) * 1024);
  pb[lane] = make_uint4(B[0], B[1], B[2], B[3]);
  pb[32 + lane] = make_uint4(B[4], B[5], B[6], B[7]);
  float X[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int j = 0; j < 4; ++j) mma16816<T>(X, ones, B[2 * j], B[2 * j + 1]);
  if (r == 0) *reinterpret_cast<float2*>(px + g * TL::TOK + nt * 8 + 2 * cq) = make_float2(X[0], X[1]);
}

// x preparation of one stage from the raw x slice in shared memory.  xs: the stage's x part
// (raw x slice, then B fragments and x sums).
template <typename T, int BITS, int NT>
__device__ __forceinline__ void prep_stage(unsigned char* xs, int lane) {
  using TL = Tile<BITS, NT>;
  const int r = lane >> 2, cq = lane & 3;
#pragma unroll
  for (int g = 0; g < TL::UG; ++g)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const unsigned char* xp = xs + (g >> 2) * TL::XCHUNK + (nt * 8 + r) * 512 + (g & 3) * 128 + cq * 32;
      prep_one<T, BITS, NT>(xs, g, nt, lane, reinterpret_cast<const uint4*>(xp)[0], reinterpret_cast<const uint4*>(xp)[1]);
    }
}

// The same from x in global memory: rows [0, rows) of a row-major [.. x K] array, columns k0 ..
// k0 + UG * 64 (rows >= rows read as zeros).  L2 loads, one token tile's issued together
// before its work.
template <typename T, int BITS, int NT, int PREL = Tile<BITS, NT>::P_REL>
__device__ __forceinline__ void prep_global(unsigned char* xs, const T* x, int K, int rows, int k0, int lane) {
  using TL = Tile<BITS, NT>;
  const int r = lane >> 2, cq = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    uint4 v[TL::UG][2];
    const bool live = nt * 8 + r < rows;
    const uint4* p = reinterpret_cast<const uint4*>(x + (size_t)(live ? nt * 8 + r : 0) * K + k0 + cq * 16);
#pragma unroll
    for (int g = 0; g < TL::UG; ++g) {
      v[g][0] = live ? __ldcg(p + g * 8) : make_uint4(0, 0, 0, 0);
      v[g][1] = live ? __ldcg(p + g * 8 + 1) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int g = 0; g < TL::UG; ++g) prep_one<T, BITS, NT, PREL>(xs, g, nt, lane, v[g][0], v[g][1]);
  }
}

// Byte offsets of a consumer thread's weight fragments in a stage (row slot0; slot1 is 1024
// bytes further): the 16-byte unit of a [128 x 128 B] box is swizzled by row % 8 == r.  The
// group pattern repeats every WPAT groups, and the box index is g / WPAT.
template <int BITS> struct WOff {
  static constexpr int WPAT = BITS == 4 ? 4 : (BITS == 8 ? 2 : 1);
  int v[BITS ? WPAT : 2];
  __device__ __forceinline__ WOff(int slot0, int r, int cq) {
    if constexpr (BITS == 4) {
#pragma unroll
      for (int G = 0; G < 4; ++G) v[G] = slot0 * 128 + ((((2 * G) | (cq >> 1)) ^ r) << 4) + (cq & 1) * 8;
    } else if constexpr (BITS == 8) {
#pragma unroll
      for (int G = 0; G < 2; ++G) v[G] = slot0 * 128 + (((4 * G + cq) ^ r) << 4);
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) v[h] = slot0 * 128 + (((2 * cq + h) ^ r) << 4);
    }
  }
};

// The weight words of one group for a consumer thread: rows slot0 (w0) and slot1 (w1), WPG
// 32-bit words each (int4: 2, int8: 4, dense: 8), read from a stage as the MMA wants them.
template <int BITS> struct WGroup {
  static constexpr int WPG = BITS == 4 ? 2 : (BITS == 8 ? 4 : 8);
};
template <int BITS, int NT>
__device__ __forceinline__ void stage_wgroup(const unsigned char* st, const WOff<BITS>& woff, int g, uint32_t (&w0)[WGroup<BITS>::WPG],
                                             uint32_t (&w1)[WGroup<BITS>::WPG]) {
  using TL = Tile<BITS, NT>;
  if constexpr (BITS == 4) {
    const unsigned char* wrow = st + (g / 4) * TL::WCHUNK + woff.v[g % 4];
    const uint2 u0v = *reinterpret_cast<const uint2*>(wrow);
    const uint2 u1v = *reinterpret_cast<const uint2*>(wrow + 1024);
    w0[0] = u0v.x; w0[1] = u0v.y; w1[0] = u1v.x; w1[1] = u1v.y;
  } else if constexpr (BITS == 8) {
    const unsigned char* wrow = st + (g / 2) * TL::WCHUNK + woff.v[g % 2];
    const uint4 u0v = *reinterpret_cast<const uint4*>(wrow);
    const uint4 u1v = *reinterpret_cast<const uint4*>(wrow + 1024);
    w0[0] = u0v.x; w0[1] = u0v.y; w0[2] = u0v.z; w0[3] = u0v.w;
    w1[0] = u1v.x; w1[1] = u1v.y; w1[2] = u1v.z; w1[3] = u1v.w;
  } else {
    const unsigned char* wbox = st + g * TL::WCHUNK;
    const uint4 a0 = *reinterpret_cast<const uint4*>(wbox + woff.v[0]);
    const uint4 a1 = *reinterpret_cast<const uint4*>(wbox + woff.v[1]);
    const uint4 b0 = *reinterpret_cast<const uint4*>(wbox + woff.v[0] + 1024);
    const uint4 b1 = *reinterpret_cast<const uint4*>(wbox + woff.v[1] + 1024);
    w0[0] = a0.x; w0[1] = a0.y; w0[2] = a0.z; w0[3] = a0.w; w0[4] = a1.x; w0[5] = a1.y; w0[6] = a1.z; w0[7] = a1.w;
    w1[0] = b0.x; w1[1] = b0.y; w1[2] = b0.z; w1[3] = b0.w; w1[4] = b1.x; w1[5] = b1.y; w1[6] = b1.z; w1[7] = b1.w;
  }
}
// This warp's scales and biases of the unit's UG groups (quantized): 16 bytes per row, rows
// slot0 / slot1: sb = {scales slot0, scales slot1, biases slot0, biases slot1} x 4 words.
template <int BITS, int NT>
__device__ __forceinline__ void stage_sb(const unsigned char* st, int slot0, int slot1, uint32_t (&sb)[16]) {
  using TL = Tile<BITS, NT>;
  const uint4 v[4] = {*reinterpret_cast<const uint4*>(st + TL::W_BYTES + slot0 * 16),
                      *reinterpret_cast<const uint4*>(st + TL::W_BYTES + slot1 * 16),
                      *reinterpret_cast<const uint4*>(st + TL::W_BYTES + kSlots * 16 + slot0 * 16),
                      *reinterpret_cast<const uint4*>(st + TL::W_BYTES + kSlots * 16 + slot1 * 16)};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sb[4 * i] = v[i].x; sb[4 * i + 1] = v[i].y; sb[4 * i + 2] = v[i].z; sb[4 * i + 3] = v[i].w;
  }
}

// One stage's MMA work of a consumer warp: its 16 weight rows (slot0, slot1 = slot0 + 8 per
// thread) across the unit's UG groups, accumulated into acc.  The weight words of group g come
// from wf(g, w0, w1); sb: the scales and biases (quantized); xs: the stage's x part, its B
// fragments PREL bytes in.
template <typename T, int BITS, int NT, int PREL, typename WF>
__device__ __forceinline__ void consume_core(const unsigned char* xs, float (&acc)[NT][4], int lane,
                                             const uint32_t (&sb)[16], const WF& wf) {
  using A = Act<T>;
  using TL = Tile<BITS, NT>;
  constexpr int UG = TL::UG, TOK = TL::TOK, WPG = WGroup<BITS>::WPG;
  constexpr uint32_t kMask = 0x000F000Fu;
  constexpr uint32_t kMag = A::kMagic2;
  constexpr float kOff = BITS == 4 ? A::kMagic : 17.0f * A::kMagic;
  const int r = lane >> 2, cq = lane & 3;
  if constexpr (BITS != 0) {
    const uint32_t* sw0 = sb;
    const uint32_t* sw1 = sb + 4;
    const uint32_t* bw0 = sb + 8;
    const uint32_t* bw1 = sb + 12;
    const uint4* pb = reinterpret_cast<const uint4*>(xs + PREL);
    const float* px = reinterpret_cast<const float*>(xs + PREL + TL::PB_BYTES);
    // Groups in pairs: the two groups' MMA chains are issued interleaved (each group's own sums
    // keep their order, and acc takes group g before group g + 1).
    constexpr int GP = 2;
#pragma unroll
    for (int g0 = 0; g0 < UG; g0 += GP) {
      uint32_t B[GP][NT][8];
      float X[GP][NT][2];
      uint32_t w0[GP][WPG], w1[GP][WPG];
      float d[GP][NT][4];
#pragma unroll
      for (int h = 0; h < GP; ++h) {
        const int g = g0 + h;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 lo = pb[(g * NT + nt) * 64 + lane], hi = pb[(g * NT + nt) * 64 + 32 + lane];
          B[h][nt][0] = lo.x; B[h][nt][1] = lo.y; B[h][nt][2] = lo.z; B[h][nt][3] = lo.w;
          B[h][nt][4] = hi.x; B[h][nt][5] = hi.y; B[h][nt][6] = hi.z; B[h][nt][7] = hi.w;
          const float2 xv = *reinterpret_cast<const float2*>(px + g * TOK + nt * 8 + 2 * cq);
          X[h][nt][0] = xv.x;
          X[h][nt][1] = xv.y;
#pragma unroll
          for (int e = 0; e < 4; ++e) d[h][nt][e] = 0.0f;
        }
        wf(g, w0[h], w1[h]);
      }
      if constexpr (BITS == 4) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int h = 0; h < GP; ++h) {
            const int sh = (j & 1) * 8;
            const uint32_t p0 = w0[h][j >> 1], p1 = w1[h][j >> 1];
            const uint32_t af[4] = {and_or(p0 >> sh, kMask, kMag), and_or(p1 >> sh, kMask, kMag),
                                    and_or(p0 >> (sh + 4), kMask, kMag), and_or(p1 >> (sh + 4), kMask, kMag)};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816<T>(d[h][nt], af, B[h][nt][2 * j], B[h][nt][2 * j + 1]);
          }
      } else {
        float dh[GP][NT][4];
#pragma unroll
        for (int h = 0; h < GP; ++h)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) dh[h][nt][e] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int h = 0; h < GP; ++h) {
            const uint32_t p0 = w0[h][j], p1 = w1[h][j];
            const uint32_t lo[4] = {and_or(p0, kMask, kMag), and_or(p1, kMask, kMag), and_or(p0 >> 8, kMask, kMag),
                                    and_or(p1 >> 8, kMask, kMag)};
            const uint32_t hi[4] = {and_or(p0 >> 4, kMask, kMag), and_or(p1 >> 4, kMask, kMag),
                                    and_or(p0 >> 12, kMask, kMag), and_or(p1 >> 12, kMask, kMag)};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma16816<T>(d[h][nt], lo, B[h][nt][2 * j], B[h][nt][2 * j + 1]);
              mma16816<T>(dh[h][nt], hi, B[h][nt][2 * j], B[h][nt][2 * j + 1]);
            }
          }
#pragma unroll
        for (int h = 0; h < GP; ++h)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[h][nt][e] = fmaf(16.0f, dh[h][nt][e], d[h][nt][e]);
      }
#pragma unroll
      for (int h = 0; h < GP; ++h) {
        const int g = g0 + h;
        // scale/bias of group g: 16-bit half (g & 1) of word (g >> 1)
        const float s0 = (g & 1) ? A::hi(sw0[g >> 1]) : A::lo(sw0[g >> 1]);
        const float s1 = (g & 1) ? A::hi(sw1[g >> 1]) : A::lo(sw1[g >> 1]);
        const float b0 = fmaf(-kOff, s0, (g & 1) ? A::hi(bw0[g >> 1]) : A::lo(bw0[g >> 1]));
        const float b1 = fmaf(-kOff, s1, (g & 1) ? A::hi(bw1[g >> 1]) : A::lo(bw1[g >> 1]));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[nt][0] = fmaf(s0, d[h][nt][0], fmaf(b0, X[h][nt][0], acc[nt][0]));
          acc[nt][1] = fmaf(s0, d[h][nt][1], fmaf(b0, X[h][nt][1], acc[nt][1]));
          acc[nt][2] = fmaf(s1, d[h][nt][2], fmaf(b1, X[h][nt][0], acc[nt][2]));
          acc[nt][3] = fmaf(s1, d[h][nt][3], fmaf(b1, X[h][nt][1], acc[nt][3]));
        }
      }
    }
  } else {
    // dense weights: B fragments straight from the x slice (natural order)
#pragma unroll
    for (int g = 0; g < UG; ++g) {
      uint32_t B[NT][8];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const unsigned char* xp = xs + (g >> 2) * TL::XCHUNK + (nt * 8 + r) * 512 + (g & 3) * 128 + cq * 32;
        const uint4 v0 = reinterpret_cast<const uint4*>(xp)[0], v1 = reinterpret_cast<const uint4*>(xp)[1];
        B[nt][0] = v0.x; B[nt][1] = v0.y; B[nt][2] = v0.z; B[nt][3] = v0.w;
        B[nt][4] = v1.x; B[nt][5] = v1.y; B[nt][6] = v1.z; B[nt][7] = v1.w;
      }
      uint32_t w0[WPG], w1[WPG];
      wf(g, w0, w1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t af[4] = {w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<T>(acc[nt], af, B[nt][2 * j], B[nt][2 * j + 1]);
      }
    }
  }
}

// The weight fetcher of consume_core (a functor, so that it is inlined and the words stay in
// registers): from the stage in shared memory.
template <int BITS, int NT>
struct StageW {
  const unsigned char* st;
  const WOff<BITS>& woff;
  __device__ __forceinline__ void operator()(int g, uint32_t (&w0)[WGroup<BITS>::WPG], uint32_t (&w1)[WGroup<BITS>::WPG]) const {
    stage_wgroup<BITS, NT>(st, woff, g, w0, w1);
  }
};

// consume_core with the weights read from the stage as they are used.  st: the stage's weight
// part (weights, scales, biases); xs: its x part.
template <typename T, int BITS, int NT, int PREL = Tile<BITS, NT>::P_REL>
__device__ __forceinline__ void consume_stage(const unsigned char* st, const unsigned char* xs, float (&acc)[NT][4],
                                              const WOff<BITS>& woff, int lane, int slot0, int slot1) {
  uint32_t sb[16];
  if constexpr (BITS != 0) stage_sb<BITS, NT>(st, slot0, slot1, sb);
  consume_core<T, BITS, NT, PREL>(xs, acc, lane, sb, StageW<BITS, NT>{st, woff});
}

// What happens to a finished row block.
struct Epi {
  const void* bias;
  const void* res;
  void* out;
  float* partial;  // [P][16][128]: a CTA's partial sums of its last row block
  int* flags;      // [P][kRowWarps]: partial published, per warp (reset by the gatherer)
  int N, mc, P;
  long long U;     // units of the call
  int nkc;
  int gate, has_bias, has_res, gelu, rope;
  const RopeEpi* re;  // the RoPE epilogue's operands (rope != 0)
  const KvAppendEpi* ka = nullptr;  // the K/V-append epilogue's operands, when set
  int* fault;      // the kernel's fault flags (bit 4: a gather wait ran out of time)
  const unsigned* abort = nullptr;  // when set and nonzero, a gather stops waiting
};

// End of a row block (or of a segment of this CTA's range) for one consumer warp: publish the
// partial sums when the row block continues in the next CTA, else gather the earlier CTAs'
// partial sums (rf == rb && head_shared) and run the epilogue.  Returns with acc zeroed.
// `red` is the gate / RoPE exchange area (RED bytes).  Residuals are read with L2 loads (rows
// written earlier in the same persistent kernel by other CTAs may sit stale in L1).
template <typename T, int NT>
__device__ __forceinline__ void flush_rowblock(const Epi& a, int c, int rb, bool publish, bool gather, float (&acc)[NT][4],
                                               float* red, int warp, int lane) {
  using A = Act<T>;
  constexpr int TOK = NT * 8;
  const int r = lane >> 2, cq = lane & 3;
  const int slot0 = 16 * warp + r, slot1 = slot0 + 8;
  const int mc = a.mc, N = a.N;
  int* wflags = a.flags + warp;  // this warp's flag of every CTA: wflags[c * kRowWarps]
  auto zero_acc = [&]() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
  };
  if (publish) {
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
    return;
  }
  if (gather) {
    // add the partial sums of the earlier CTAs (in CTA order), then this CTA's
    const int cf = cta_of((long long)rb * a.nkc, a.U, a.P);
    // each lane reads one contributor's flag, so that up to 32 flags cost one round trip
    // instead of one each; a lane whose flag is not yet set polls it, with the clock limit
    for (int c2 = cf + lane; c2 < c; c2 += 32) {
      const int* f = wflags + (size_t)c2 * kRowWarps;
      if (ld_flag(f) == 0) {
        const long long t0 = clock64();
        while (ld_flag(f) == 0) {
          if ((a.abort && *reinterpret_cast<const volatile unsigned*>(a.abort)) || clock64() - t0 > kWaitCycles) {
            atomicOr(a.fault, 16);
            break;
          }
        }
      }
    }
    __threadfence();
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
    for (int c2 = cf + lane; c2 < c; c2 += 32) wflags[(size_t)c2 * kRowWarps] = 0;  // consumed: zero for the next call
  }
  const T* bias = static_cast<const T*>(a.bias);
  const T* res = static_cast<const T*>(a.res);
  T* out = static_cast<T*>(a.out);
  // epilogue from registers: GATE -> bias -> GELU -> residual, one rounding.  `up` holds the
  // matching up-row sums with the SiLU gate.
  auto epilogue = [&](const float (&up)[NT][4]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = nt * 8 + 2 * cq + (e & 1);
        const int n = rb * (a.gate ? 64 : 128) + ((e >> 1) ? slot1 : slot0);
        if (tok >= mc || n >= N) continue;
        float v = acc[nt][e];
        if (a.gate) v = v / (1.0f + expf(-v)) * up[nt][e];
        const size_t o = (size_t)tok * N + n;
        if (a.has_bias) v += A::to_f(bias[n]);
        if (a.gelu) v = gelu_erf(v);
        if (a.has_res) v += A::to_f(__ldcg(res + o));
        const T tv = A::from_f(v);
        out[o] = tv;
        if (a.ka && n >= a.ka->d) {
          const KvAppendEpi& ka = *a.ka;
          const int p = ka.pr.pos(tok);
          if (p >= 0 && p < ka.S) {
            const bool isv = n >= 2 * ka.d;
            const int i = n - (isv ? 2 : 1) * ka.d;
            T* base = static_cast<T*>(isv ? ka.vc : ka.kc) + (size_t)ka.pr.stream_of(tok) * ka.kv_ss;
            base[((size_t)(i / ka.hd) * ka.S + p) * ka.hd + i % ka.hd] = tv;
          }
        }
      }
  };
  if (a.gate) {
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
      epilogue(up);
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
      const RopeEpi& re = *a.re;
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
            const float2 cs = re.cs[(size_t)pos * 64 + i];
            y1 = rope_rot1(x1, x2, cs);
            y2 = rope_rot2(x1, x2, cs);
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
    epilogue(acc);
  }
  zero_acc();
}

}  // namespace sk
}  // namespace vella
