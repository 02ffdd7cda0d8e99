// K2: tensor-core GEMM for calls of more than 16 rows (prefill chunks, batched verify,
// encoder projections) on the 5th-generation tensor core (tcgen05, accumulators in tensor
// memory, operands staged in shared memory by TMA).
//
//   out[m, n] = epilogue( sum_k x[m, k] * W'[n, k] ),   fp32 accumulation,
//
// with W' = T(scale * q + bias) (T = activation dtype, one rounding per weight) for the
// MLX-affine formats (reference SmallMGEMM.swift:491-498 layout) and W' = W for dense weights;
// the epilogue is the library's: SiLU gate, then bias, then GELU, then residual, one rounding
// (SmallMGEMM.swift:745-753).
//
// CTA tile: 128 weight rows (the MMA's M side) x up to 256 tokens (its N side: the call's
// remaining rows rounded up to 16, so a small call spends no tensor time on padding) x all
// of K, streamed in stages of 64 K elements (one quantization group); each weight tile is
// dequantised once per 256 tokens:
//   warp 0      TMA producer: the x tile [256 tokens x 64] (128-byte swizzle, out-of-range
//               tokens zero-filled) and the stage's weights (dense: directly into the MMA's
//               operand tile; quantized: the raw code rows).
//   warp 1      allocates tensor memory; one thread issues 4 MMAs (K = 16 each) per stage and
//               commits them to the stage's "empty" barrier; frees tensor memory at the end.
//   warps 2..   four threads per weight row (warps w, w + 4, ..
//               share the row window of
//               tensor-memory lanes 32 (w % 4) ..): each turns a slice of the stage's codes
//               of its row into the operand tile (128-byte swizzled K-major rows; scales and
//               biases read 8 groups at a time, a block ahead), then they run the epilogue
//               out of tensor memory on interleaved 32-column chunks.
// A call of at most 256 rows whose row tiles leave SMs idle splits K over blockIdx.z (the
// split count from N and K only): each split writes its fp32 sums to the workspace, and the
// tile's last split to arrive adds the splits' sums in split order and runs the epilogue.
// Every wait is bounded (sm100::kWaitCycles); a wait that runs out records a fault
// (vella_qgemm reports it) and the kernel finishes without waiting again.
//
// A row m of the output depends only on x[m, :] and the weights: the tensor core's per-
// element accumulation order does not involve other tokens, so a row of a batched call is
// bit-identical to the same row in any other call of 17-256 rows (or of more than 256 rows:
// the K split differs between the two classes).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"

namespace vella {

__device__ int g_tc_fault = 0;  // set when a pipeline wait ran out of time

namespace {

using namespace sm100;

constexpr int kTcRows = 128;     // weight rows per CTA (MMA M)
constexpr int kTcTok = 256;      // tokens per CTA (largest MMA N)
constexpr int kTcK = 64;         // K elements per stage
// K splits of a call of at most kTcSplitRows rows, from (N, K) only: as many as keep two
// 128-token tiles within one wave of 148 CTAs, at least 16 stages per split, at most 4.  Calls
// whose row tiles alone fill the GPU (the 30B target's projections) and calls of more rows
// (their token tiles fill it) take one.
constexpr int kTcSplitRows = 256;
constexpr int kTcWave = 148;
constexpr int kTcMaxSplits = 4;
constexpr int kTcMinSplitStages = 16;
// Transform/epilogue warps: 16, four threads per weight row (quantized: each dequantises a
// quarter of the row's codes per stage -- with 8 the transform's latency left the tensor pipe
// idle half the time; dense: no transform, the four share the epilogue).
template <int BITS> constexpr int tc_xw() { return 16; }
template <int BITS> constexpr int tc_threads() { return 64 + 32 * tc_xw<BITS>(); }

template <int BITS, bool GATE>
struct TcLayout {
  static constexpr int NA = GATE ? 2 : 1;                         // operand tiles (gate, up)
  static constexpr int A_BYTES = kTcRows * 128;                   // [128 rows x 64] bf16/fp16
  static constexpr int B_BYTES = kTcTok * 128;                    // [128 tokens x 64]
  static constexpr int RAW_BYTES = BITS ? kTcRows * kTcK * BITS / 8 : 0;
  static constexpr int STAGE = NA * A_BYTES + B_BYTES + NA * RAW_BYTES;  // multiple of 1024
  static constexpr int total(int ns) { return 1024 + ns * STAGE + (3 * ns + 1) * 8 + 16; }
  static constexpr int NS =
      total(5) <= 227 * 1024 ? 5 : (total(4) <= 227 * 1024 ? 4 : (total(3) <= 227 * 1024 ? 3 : 2));
  static constexpr int TX = B_BYTES + (BITS ? NA * RAW_BYTES : NA * A_BYTES);
  static constexpr int BAR = NS * STAGE;  // barrier block offset
  static constexpr int TOTAL = total(NS);
  static constexpr uint32_t COLS = GATE ? 2 * kTcTok : kTcTok;  // tensor-memory columns
  static_assert(STAGE % 1024 == 0, "stage tiles must stay 1024-byte aligned");
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

struct TcArgs {
  CUtensorMap tx, tw, tu;  // x; weights (dense tile or raw codes); up weights (gate)
  const void* s;           // scales  [N, K/64]
  const void* b;           // biases  [N, K/64]
  const void* us;          // up scales
  const void* ub;          // up biases
  const void* bias;        // [N] or null
  const void* res;         // [M, N] or null
  int gelu;                // GELU after the bias
  void* out;               // [M, N]
  int M, N, K, G;
  int tt;                  // tokens per CTA: 128 or 256 (the x box height)
  int S;                   // K splits (blockIdx.z); above 1 the fp32 sums go through `part`
  int Mp;                  // rows of a split's slice of `part` (M rounded up to tt)
  float* part;             // [S][NA][Mp][N] fp32 sums of each split
  int* cnt;                // [token tiles x row tiles] splits done (the last resets it)
};

// CH chunks of 8 codes of one weight row (8: the stage's 64, 4: half of them) -> CH chunks
// of 8 operand elements (16 bytes each).
// Codes are exact in T as magic + q (bf16: 128 + q for 4-bit codes; fp16: 1024 + q for 4- and
// 8-bit codes); subtracting the magic is exact, the fma rounds once.  8-bit codes with bf16
// go through fp32 (bf16 cannot hold 128 + q for q >= 128).
template <typename T, int BITS, int CH>
__device__ __forceinline__ void dequant_row(const uint32_t* raw, T s, T b, uint4 (&o)[CH]) {
  using A = Act<T>;
  if constexpr (BITS == 8 && sizeof(T) == 2 && A::kMagic == 128.0f) {  // bf16, 8-bit codes
    const float fs = A::to_f(s), fb = A::to_f(b);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint32_t w2[2] = {raw[2 * c], raw[2 * c + 1]};
      uint32_t r[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float f0 = __uint_as_float(__byte_perm(w2[h], 0x4B000000u, 0x7440 + 2 * p)) - 8388608.0f;
          const float f1 = __uint_as_float(__byte_perm(w2[h], 0x4B000000u, 0x7441 + 2 * p)) - 8388608.0f;
          const __nv_bfloat162 v = __floats2bfloat162_rn(fmaf(f0, fs, fb), fmaf(f1, fs, fb));
          r[2 * h + p] = *reinterpret_cast<const uint32_t*>(&v);
        }
      }
      o[c] = make_uint4(r[0], r[1], r[2], r[3]);
    }
  } else {
    using V2 = typename std::conditional<sizeof(T) == 2 && A::kMagic == 128.0f, __nv_bfloat162, __half2>::type;
    const uint32_t mag = A::kMagic2;
    V2 s2, b2, m2;
    *reinterpret_cast<T*>(&s2) = s; *(reinterpret_cast<T*>(&s2) + 1) = s;
    *reinterpret_cast<T*>(&b2) = b; *(reinterpret_cast<T*>(&b2) + 1) = b;
    *reinterpret_cast<uint32_t*>(&m2) = mag;
    auto fin = [&](uint32_t v) {
      V2 q = *reinterpret_cast<V2*>(&v);
      q = __hsub2(q, m2);
      const V2 r = __hfma2(q, s2, b2);
      return *reinterpret_cast<const uint32_t*>(&r);
    };
    if constexpr (BITS == 4) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint32_t w = raw[c];  // elements 8c .. 8c+7, low nibble first
        const uint32_t p04 = and_or(w, 0x000F000Fu, mag), p15 = and_or(w >> 4, 0x000F000Fu, mag);
        const uint32_t p26 = and_or(w >> 8, 0x000F000Fu, mag), p37 = and_or(w >> 12, 0x000F000Fu, mag);
        o[c] = make_uint4(fin(__byte_perm(p04, p15, 0x5410)), fin(__byte_perm(p26, p37, 0x5410)),
                          fin(__byte_perm(p04, p15, 0x7632)), fin(__byte_perm(p26, p37, 0x7632)));
      }
    } else {  // fp16, 8-bit codes
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        uint32_t r[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t w = raw[2 * c + h];  // elements 8c + 4h .. +3, low byte first
          const uint32_t p02 = and_or(w, 0x00FF00FFu, mag), p13 = and_or(w >> 8, 0x00FF00FFu, mag);
          r[2 * h] = fin(__byte_perm(p02, p13, 0x5410));
          r[2 * h + 1] = fin(__byte_perm(p02, p13, 0x7632));
        }
        o[c] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
  }
}

template <typename T, int BITS, bool GATE>
__global__ void __launch_bounds__(tc_threads<BITS>(), 1) tc_gemm_kernel(const __grid_constant__ TcArgs a) {
  using A = Act<T>;
  constexpr int kTcXW = tc_xw<BITS>();
  constexpr int kTcParts = kTcXW / 4;  // threads per weight row (each a slice of its codes)
  using LY = TcLayout<BITS, GATE>;
  constexpr int NS = LY::NS;
  constexpr int WPG = BITS ? kTcK * BITS / 32 : 0;  // 32-bit code words per row and stage

  extern __shared__ unsigned char smem_raw[];
  // (offsetting the shared array itself keeps its address space: shared loads, not generic ones)
  unsigned char* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY::BAR);
  uint64_t* ready = full + NS;
  uint64_t* empty = ready + NS;
  uint64_t* accf = empty + NS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  auto tileA = [&](int st, int i) { return smem + st * LY::STAGE + i * LY::A_BYTES; };
  auto tileB = [&](int st) { return smem + st * LY::STAGE + LY::NA * LY::A_BYTES; };
  auto tileR = [&](int st, int i) { return smem + st * LY::STAGE + LY::NA * LY::A_BYTES + LY::B_BYTES + i * LY::RAW_BYTES; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tok0 = blockIdx.x * a.tt, row0 = blockIdx.y * kTcRows;
  const int G = a.G;
  // this split's stages [g0, g1): whole blocks of 8 groups (the scale/bias loads' unit)
  const int z = blockIdx.z, nblk = (G + 7) / 8;
  const int g0 = 8 * (z * nblk / a.S), g1 = min(G, 8 * ((z + 1) * nblk / a.S));
  const int NG = g1 - g0;
  // MMA N: this tile's tokens rounded up to 16 (a row's sums do not depend on N)
  const int ntok = min(a.tt, (a.M - tok0 + 15) / 16 * 16);
  const uint32_t tx = (uint32_t)(a.tt * 128 + (BITS ? LY::NA * LY::RAW_BYTES : LY::NA * LY::A_BYTES));
  const uint32_t idesc = f16_idesc(A::kMagic == 128.0f, kTcRows, ntok);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 32 * kTcXW);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tslot, LY::COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_next();

  if (warp == 0) {
    // ---- TMA producer ---------------------------------------------------------------------
    if (lane == 0) {
      auto weights = [&](int g, int st) {
        if constexpr (BITS == 0) {
          tma2d(tileA(st, 0), &a.tw, g * kTcK, row0, &full[st]);
          if constexpr (GATE) tma2d(tileA(st, 1), &a.tu, g * kTcK, row0, &full[st]);
        } else {
          tma2d(tileR(st, 0), &a.tw, g * WPG, row0, &full[st]);
          if constexpr (GATE) tma2d(tileR(st, 1), &a.tu, g * WPG, row0, &full[st]);
        }
      };
      // stage l of this split holds group g0 + l in ring slot l % NS
      const int npre = min(NG, NS);
      for (int l = 0; l < npre; ++l) {
        mbar_expect_tx(&full[l], tx);
        weights(g0 + l, l);
      }
      pdl_wait();  // x is written by the previous kernel
      for (int l = 0; l < npre; ++l) tma2d(tileB(l), &a.tx, (g0 + l) * kTcK, tok0, &full[l]);
      int issued = npre;
      for (int l = npre; l < NG; ++l) {
        const int st = l % NS, use = l / NS;
        if (!mbar_wait(&empty[st], (uint32_t)((use - 1) & 1))) {
          atomicOr(&g_tc_fault, 1);
          break;
        }
        mbar_expect_tx(&full[st], tx);
        weights(g0 + l, st);
        tma2d(tileB(st), &a.tx, (g0 + l) * kTcK, tok0, &full[st]);
        issued = l + 1;
      }
      // every copy issued must land before the CTA may exit
      for (int l = max(0, issued - NS); l < issued; ++l)
        if (!mbar_wait(&full[l % NS], (uint32_t)((l / NS) & 1))) atomicOr(&g_tc_fault, 2);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ---------------------------------------------------------------------
    pdl_wait();
    if (lane == 0) {
      for (int l = 0; l < NG; ++l) {
        const int st = l % NS;
        const uint32_t par = (uint32_t)((l / NS) & 1);
        if (!mbar_wait(BITS ? &ready[st] : &full[st], par)) {
          atomicOr(&g_tc_fault, 4);
          break;
        }
        tc_fence_after();
        const uint32_t a0 = saddr(tileA(st, 0)), b0 = saddr(tileB(st));
#pragma unroll
        for (int kk = 0; kk < kTcK / 16; ++kk) {
          const uint64_t bd = kmajor_sw128_desc(b0 + kk * 32);
          const uint32_t acc = (l > 0 || kk > 0) ? 1u : 0u;
          mma_f16_ss(tmem, kmajor_sw128_desc(a0 + kk * 32), bd, idesc, acc);
          if constexpr (GATE) mma_f16_ss(tmem + kTcTok, kmajor_sw128_desc(saddr(tileA(st, 1)) + kk * 32), bd, idesc, acc);
        }
        mma_commit(&empty[st]);
      }
      mma_commit(accf);  // arrives when every MMA above has completed
    }
    __syncwarp();
  } else {
    // ---- transform (quantized formats) and epilogue: four threads per weight row -----------
    pdl_wait();
    const int r = 32 * (warp & 3) + lane;  // tensor-memory lane of this warp's window
    const int hf = (warp - 2) >> 2;        // which slice of the row's codes / which column chunks
    const int n = row0 + r;
    const bool nv = n < a.N;
    if constexpr (BITS != 0) {
      // transform mapping: adjacent lanes take the slices of one weight row, so the lanes of
      // a quarter-warp read contiguous code bytes (the epilogue keeps thread = tensor-memory
      // lane); the swizzled operand writes of those lanes fall in distinct 16-byte units
      const int xi = (warp - 2) * 32 + lane;
      const int tr = xi / kTcParts, tp = xi % kTcParts;
      const int tn = row0 + tr;
      const bool tnv = tn < a.N;
      // scales/biases of this row: blocks of 8 groups (two 32-bit words = 4 packed values
      // each half), the next block's loads in flight while this one is used
      const size_t rowg = (size_t)(tnv ? tn : 0) * G;
      const bool vec = (G % 8) == 0;  // rows start 16-byte aligned: one 16-byte load per array
      auto load_block = [&](const void* base, int gb, uint32_t (&wv)[4]) {
        const T* p = static_cast<const T*>(base) + rowg + gb;
        if (!tnv || gb >= G) {
          wv[0] = wv[1] = wv[2] = wv[3] = 0u;
        } else if (vec) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
          wv[0] = v.x; wv[1] = v.y; wv[2] = v.z; wv[3] = v.w;
        } else {
          const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lo = gb + 2 * j < G ? q[2 * j] : 0u, hi = gb + 2 * j + 1 < G ? q[2 * j + 1] : 0u;
            wv[j] = lo | (hi << 16);
          }
        }
      };
      auto half_of = [](const uint32_t (&wv)[4], int j) {
        const uint32_t w2 = wv[j >> 1];
        const uint16_t h = (j & 1) ? (uint16_t)(w2 >> 16) : (uint16_t)(w2 & 0xFFFFu);
        return *reinterpret_cast<const T*>(&h);
      };
      uint32_t sc[4], bc[4], sn[4], bn[4], usc[4], ubc[4], usn[4], ubn[4];
      load_block(a.s, g0, sc);
      load_block(a.b, g0, bc);
      if constexpr (GATE) { load_block(a.us, g0, usc); load_block(a.ub, g0, ubc); }
      bool ok = true;
      for (int gb = g0; gb < g1 && ok; gb += 8) {
        load_block(a.s, gb + 8, sn);
        load_block(a.b, gb + 8, bn);
        if constexpr (GATE) { load_block(a.us, gb + 8, usn); load_block(a.ub, gb + 8, ubn); }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int g = gb + j;
          if (g >= g1) break;
          const int st = (g - g0) % NS;
          if (!mbar_wait(&full[st], (uint32_t)(((g - g0) / NS) & 1))) {
            atomicOr(&g_tc_fault, 8);
            ok = false;
            break;
          }
#pragma unroll
          for (int i = 0; i < LY::NA; ++i) {
            constexpr int HW = WPG / kTcParts;  // code words of this thread's slice
            constexpr int CH = 8 / kTcParts;    // 8-element chunks of the slice
            const unsigned char* sp0 = tileR(st, i) + tr * WPG * 4 + tp * HW * 4;
            uint32_t raw[HW];
            if constexpr (HW >= 4) {
#pragma unroll
              for (int v = 0; v < HW / 4; ++v) {
                const uint4 q = reinterpret_cast<const uint4*>(sp0)[v];
                raw[4 * v] = q.x; raw[4 * v + 1] = q.y; raw[4 * v + 2] = q.z; raw[4 * v + 3] = q.w;
              }
            } else {
              const uint2 q = *reinterpret_cast<const uint2*>(sp0);
              raw[0] = q.x; raw[1] = q.y;
            }
            uint4 o[CH];
            const T sj = i ? half_of(usc, j) : half_of(sc, j);
            const T bj = i ? half_of(ubc, j) : half_of(bc, j);
            dequant_row<T, BITS, CH>(raw, sj, bj, o);
            unsigned char* dst = tileA(st, i) + tr * 128;
#pragma unroll
            for (int c = 0; c < CH; ++c) *reinterpret_cast<uint4*>(dst + (((CH * tp + c) ^ (tr & 7)) << 4)) = o[c];
          }
          fence_proxy_async();
          mbar_arrive(&ready[st]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[j] = sn[j]; bc[j] = bn[j];
          if constexpr (GATE) { usc[j] = usn[j]; ubc[j] = ubn[j]; }
        }
      }
    }
    // ---- epilogue ------------------------------------------------------------------------
    const bool ok = mbar_wait(accf, 0);
    tc_fence_after();
    if (!ok) atomicOr(&g_tc_fault, 16);
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const T* bias = static_cast<const T*>(a.bias);
    const T* res = static_cast<const T*>(a.res);
    T* out = static_cast<T*>(a.out);
    // GATE -> bias -> GELU -> residual, one rounding
    auto finish = [&](int m, int col, float y, float up, float bcol) {
      if constexpr (GATE) y = y / (1.0f + expf(-y)) * up;
      y += bcol;
      if (a.gelu) y = gelu_erf(y);
      if (res) y += A::to_f(res[(size_t)m * a.N + col]);
      out[(size_t)m * a.N + col] = A::from_f(y);
    };
    if (a.S == 1) {
      const float bn = (bias && nv) ? A::to_f(bias[n]) : 0.0f;
      if (ok) {
        for (int c0 = 32 * hf; c0 < ntok && tok0 + c0 < a.M; c0 += 32 * kTcParts) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + c0, v);
          uint32_t u[32];
          if constexpr (GATE) tmem_ld32(tmem + lane_base + kTcTok + c0, u);
          if (nv) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = tok0 + c0 + j;
              if (m < a.M) finish(m, n, __uint_as_float(v[j]), GATE ? __uint_as_float(u[j]) : 0.0f, bn);
            }
          }
        }
      }
    } else {
      // K split: this split's fp32 sums go to `part`; the tile's last split to arrive adds the
      // splits' sums in split order and runs the epilogue (no split waits for another)
      const size_t plane = (size_t)a.Mp * a.N;
      float* pz = a.part + (size_t)z * LY::NA * plane;
      if (ok) {
        for (int c0 = 32 * hf; c0 < ntok && tok0 + c0 < a.M; c0 += 32 * kTcParts) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + c0, v);
          uint32_t u[32];
          if constexpr (GATE) tmem_ld32(tmem + lane_base + kTcTok + c0, u);
          if (nv) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = tok0 + c0 + j;
              if (m < a.M) {
                pz[(size_t)m * a.N + n] = __uint_as_float(v[j]);
                if constexpr (GATE) pz[plane + (size_t)m * a.N + n] = __uint_as_float(u[j]);
              }
            }
          }
        }
      }
      __threadfence();
      named_sync(1, 32 * kTcXW);
      volatile uint32_t* s_last = tslot + 1;
      if (tid == 64) {
        int* cp = a.cnt + blockIdx.y * gridDim.x + blockIdx.x;
        const bool last = atomicAdd(cp, 1) == a.S - 1;
        if (last) {
          __threadfence();
          *cp = 0;  // every split has arrived: zero for the next call
        }
        *s_last = last ? 1u : 0u;
      }
      named_sync(1, 32 * kTcXW);
      if (*s_last) {
        // the whole tile over the epilogue warps, a weight row per lane (coalesced along N);
        // RB elements a thread at a time, their loads all in flight before any is added
        constexpr int RB = 8;
        const int et = tid - 64, rows = min(a.tt, a.M - tok0), total = rows * kTcRows;
        for (int e0 = et; e0 < total; e0 += RB * 32 * kTcXW) {
          float pv[RB][kTcMaxSplits], pu[RB][kTcMaxSplits];
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            const int e = e0 + r * 32 * kTcXW;
            const int m = tok0 + (e >> 7), col = row0 + (e & (kTcRows - 1));
            const bool in = e < total && col < a.N;
            const size_t o = in ? (size_t)m * a.N + col : 0;
#pragma unroll
            for (int q = 0; q < kTcMaxSplits; ++q) {
              pv[r][q] = in && q < a.S ? __ldcg(a.part + (size_t)q * LY::NA * plane + o) : 0.0f;
              pu[r][q] = GATE && in && q < a.S ? __ldcg(a.part + ((size_t)q * LY::NA + 1) * plane + o) : 0.0f;
            }
          }
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            const int e = e0 + r * 32 * kTcXW;
            const int m = tok0 + (e >> 7), col = row0 + (e & (kTcRows - 1));
            if (e >= total || col >= a.N) continue;
            float y = pv[r][0], up = pu[r][0];
#pragma unroll
            for (int q = 1; q < kTcMaxSplits; ++q)
              if (q < a.S) {
                y += pv[r][q];
                up += pu[r][q];
              }
            finish(m, col, y, up, bias ? A::to_f(bias[col]) : 0.0f);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, LY::COLS);
}

template <typename T, int BITS, bool GATE>
int launch_tc_t(const TcArgs& a, cudaStream_t stream) {
  using LY = TcLayout<BITS, GATE>;
  auto k = tc_gemm_kernel<T, BITS, GATE>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::TOTAL));
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const dim3 grid((a.M + a.tt - 1) / a.tt, (a.N + kTcRows - 1) / kTcRows, a.S);
  return launch_kernel(k, grid, dim3(tc_threads<BITS>()), LY::TOTAL, stream, a);
}

template <typename T, int BITS>
int dispatch_tc(const TcArgs& a, bool gate, cudaStream_t s) {
  return gate ? launch_tc_t<T, BITS, true>(a, s) : launch_tc_t<T, BITS, false>(a, s);
}

}  // namespace

// Calls of more than 16 rows with K % 64 == 0 (and every pointer 16-byte aligned, checked by
// the caller).
bool tc_eligible(const vella_qgemm_desc& d) {
  return d.m > 16 && d.k >= kTcK && d.k % kTcK == 0 && (d.bits == 0 || d.bits == 4 || d.bits == 8) &&
         (d.dtype == VELLA_BF16 || d.dtype == VELLA_F16);
}

int tc_splits(const vella_qgemm_desc& d) {
  if (d.m > kTcSplitRows) return 1;
  const int rtiles = (d.n + kTcRows - 1) / kTcRows;
  const int by_wave = kTcWave / (2 * rtiles);
  const int by_stages = d.k / kTcK / kTcMinSplitStages;
  int splits = std::max(1, std::min(std::min(by_wave, by_stages), kTcMaxSplits));
  // a long K (a split keeps at least 100 stages: the 30B target's down projection) takes three
  // splits while one token tile's splits fit one wave, even though two tiles then take two
  if (d.k / kTcK / 3 >= 100 && 3 * rtiles <= kTcWave) splits = std::max(splits, 3);
  return splits;
}

// Counters for every (token tile, row tile) at 128-token tiles, then [S][NA][Mp][N] fp32 with Mp
// the rows rounded up to 256 (either tile height fits).
size_t tc_workspace(const vella_qgemm_desc& d, int splits) {
  if (splits <= 1) return 0;
  const size_t rtiles = (d.n + kTcRows - 1) / kTcRows, ttiles = (d.m + kTcTok / 2 - 1) / (kTcTok / 2);
  const size_t mp = (size_t)(d.m + kTcTok - 1) / kTcTok * kTcTok;
  const size_t na = d.epilogue == VELLA_EPI_SILU_GATE ? 2 : 1;
  return counter_region(rtiles * ttiles) + (size_t)splits * na * mp * d.n * sizeof(float);
}

int tc_launch(const vella_qgemm_desc& d, int splits, const void* x, const void* w, const void* scales,
              const void* biases, const void* up_w, const void* up_scales, const void* up_biases, const void* bias,
              const void* residual, void* out, void* ws, cudaStream_t stream) {
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  TcArgs a{};
  a.s = scales; a.b = biases; a.us = up_scales; a.ub = up_biases;
  a.bias = epi_bias(d.epilogue) ? bias : nullptr;
  a.res = epi_residual(d.epilogue) ? residual : nullptr;
  a.gelu = epi_gelu(d.epilogue);
  a.out = out;
  a.M = d.m; a.N = d.n; a.K = d.k; a.G = d.k / kTcK;
  // 256 tokens per CTA dequantise each weight tile half as often; 128 when the wide tiles
  // would leave SMs idle (a row's value is the same either way)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  const long long rtiles = (d.n + kTcRows - 1) / kTcRows;
  a.tt = ((long long)(d.m + kTcTok - 1) / kTcTok) * rtiles >= num_sms(dev) ? kTcTok : kTcTok / 2;
  a.S = std::max(1, splits);
  if (a.S > 1) {
    if (!ws) return fail(VELLA_E_INVALID, "tensor-core GEMM: %d K splits need a workspace", a.S);
    const size_t ttiles = (d.m + kTcTok / 2 - 1) / (kTcTok / 2);
    a.cnt = static_cast<int*>(ws);
    a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + counter_region((size_t)rtiles * ttiles));
    a.Mp = (d.m + a.tt - 1) / a.tt * a.tt;
  }
  int rc;
  const uint64_t xrow = (uint64_t)d.k * 2;
  if ((rc = make_tensor_map(&a.tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, x, d.k, d.m, xrow, kTcK, a.tt,
                            CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (d.bits == 0) {
    if ((rc = make_tensor_map(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, d.k, d.n, xrow, kTcK, kTcRows,
                              CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (gate && (rc = make_tensor_map(&a.tu, CU_TENSOR_MAP_DATA_TYPE_UINT16, up_w, d.k, d.n, xrow, kTcK, kTcRows,
                                      CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  } else {
    const uint64_t words = (uint64_t)d.k * d.bits / 32;
    const uint32_t wpg = kTcK * d.bits / 32;
    if ((rc = make_tensor_map(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, words, d.n, words * 4, wpg, kTcRows,
                              CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
    if (gate && (rc = make_tensor_map(&a.tu, CU_TENSOR_MAP_DATA_TYPE_UINT32, up_w, words, d.n, words * 4, wpg,
                                      kTcRows, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
  }
  const bool bf = d.dtype == VELLA_BF16;
  switch (d.bits) {
    case 0: return bf ? dispatch_tc<__nv_bfloat16, 0>(a, gate, stream) : dispatch_tc<__half, 0>(a, gate, stream);
    case 4: return bf ? dispatch_tc<__nv_bfloat16, 4>(a, gate, stream) : dispatch_tc<__half, 4>(a, gate, stream);
    default: return bf ? dispatch_tc<__nv_bfloat16, 8>(a, gate, stream) : dispatch_tc<__half, 8>(a, gate, stream);
  }
}

int tc_fault_status(int clear) {  // the flags, or -1 when they cannot be read
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_fault, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_tc_fault, &zero, sizeof(int)) != cudaSuccess) cudaGetLastError();
  }
  return v;
}

}  // namespace vella
