// K1: small-M (1-16 rows per pass) GEMM over MLX-affine int4/int8 or dense bf16/fp16
// weights, out[M, N] = epilogue(x[M, K] . W^T).
//
// Reference: Worker/Sources/SmallMGEMM/SmallMGEMM.swift:662-755 (smallm_gemv_affine, the
// product form acc += s * sum(x*q) + b * sum(x), fp32 accumulation, epilogue GATE -> bias
// -> residual, one rounding) and :585-656 (dense GEMV).
//
// B200 design.  The kernel streams the weights once from HBM; x is tiny.  Each warp owns
// 32 weight rows (two m16 tiles; with the SiLU gate: 16 gate rows + the same 16 up rows)
// and issues tensor-core m16n8k16 MMAs with the *weights as the A operand* and x^T as B,
// so M <= 8 needs one n8 tile and M <= 16 two.  Weights are dequantized in registers:
// (word >> s) & 0x000F000F | 0x43004300 turns two 4-bit codes into the bf16 pair
// (128 + q_a, 128 + q_b) in one LOP3, which is exact; the 128 offset is removed in the
// per-group scale step, acc += s * D + (b - 128 s) * sum(x), i.e. the reference's product
// form with D = sum(x * (128 + q)).  sum(x) per group comes from the same MMA with an
// all-ones A operand.  8-bit codes are split into low and high nibbles (two MMAs,
// D = D_lo + 16 D_hi).  Within one MMA the k positions may be permuted freely as long as
// A and B agree, so each thread's k slots are the nibbles its own 8/16-byte load
// delivers, and x is permuted to match when its fragment is read from shared memory.
//
// Pipeline: weights and their scales/biases for the next PF groups are in flight in
// registers (no shared-memory staging of the weight stream); x for the CTA's K range is
// copied to shared memory once with cp.async.
//
// Work split: a CTA (4 warps) covers 128 output rows (64 with the gate) x KC groups of
// 64 along K; `splits` CTAs along K write fp32 partial tiles to a workspace and the CTA
// that arrives last (atomic ticket, no waiting) adds them in split order and runs the
// epilogue.  The plan depends on (N, K, bits, gate) only, never on M, and every output
// row is computed by the same instruction sequence whatever the other rows are: a row of
// a batched call is bit-identical to the same row computed alone (verify == greedy).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "internal.h"

namespace vella {

// The ticket counters sit at the front of the workspace in a region of this fixed size
// (32768 counters), and the fp32 partials after it, so that calls of different shapes can
// share one workspace: no shape's partials ever overwrite another shape's counters.
constexpr size_t kCounterRegion = size_t(128) << 10;

size_t counter_region(size_t counters) {
  const size_t bytes = (counters * sizeof(int) + 255) / 256 * 256;
  return bytes > kCounterRegion ? bytes : kCounterRegion;
}

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kSlots = 128;  // weight rows per CTA (gate: 64 gate + 64 up)
constexpr int kKCMax = 32;
constexpr int kTokMax = 16;  // tokens per pass (z chunk)
constexpr int kAccStride = kSlots + 4;

struct Args {
  const void* x;
  const uint32_t* w;
  const void* sc;
  const void* bi;
  const uint32_t* uw;
  const void* usc;
  const void* ubi;
  const void* bias;
  const void* res;
  void* out;
  float* partial;
  int* counters;
  int M, N, K, G, KC, S, rowblocks;
  int has_bias, has_res, gelu;
};

// Words of packed weight per row and group of 64, and per thread (k quarter) of a group.
template <int BITS> struct Fmt;
template <> struct Fmt<4> { static constexpr int kWordsPerGroup = 8, kWordsPerThread = 2, kPF = 4; };
template <> struct Fmt<8> { static constexpr int kWordsPerGroup = 16, kWordsPerThread = 4, kPF = 3; };
template <> struct Fmt<0> { static constexpr int kWordsPerGroup = 32, kWordsPerThread = 8, kPF = 2; };

template <int BITS>
__device__ __forceinline__ void load_words(uint32_t* dst, const uint32_t* p) {
  if constexpr (BITS == 4) {
    uint2 v = ld_stream2(p);
    dst[0] = v.x; dst[1] = v.y;
  } else if constexpr (BITS == 8) {
    uint4 v = ld_stream4(p);
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  } else {
    uint4 v = ld_stream4(p);
    uint4 u = ld_stream4(p + 4);
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
    dst[4] = u.x; dst[5] = u.y; dst[6] = u.z; dst[7] = u.w;
  }
}

__device__ __forceinline__ uint32_t ld_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Natural x words n[0..7] (n[i] = x[2i], x[2i+1]) -> the k order the A dequant delivers.
template <int BITS>
__device__ __forceinline__ void permute_x(uint32_t (&p)[8], const uint32_t (&n)[8]) {
  if constexpr (BITS == 4) {
    // pairs (0,4) (1,5) (2,6) (3,7) (8,12) (9,13) (10,14) (11,15)
    p[0] = __byte_perm(n[0], n[2], 0x5410); p[1] = __byte_perm(n[0], n[2], 0x7632);
    p[2] = __byte_perm(n[1], n[3], 0x5410); p[3] = __byte_perm(n[1], n[3], 0x7632);
    p[4] = __byte_perm(n[4], n[6], 0x5410); p[5] = __byte_perm(n[4], n[6], 0x7632);
    p[6] = __byte_perm(n[5], n[7], 0x5410); p[7] = __byte_perm(n[5], n[7], 0x7632);
  } else if constexpr (BITS == 8) {
    // pairs (0,2) (1,3) (4,6) (5,7) ...
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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}

template <typename T, int BITS, int NT, bool GATE>
__global__ void __launch_bounds__(kThreads) qgemm_kernel(const Args a) {
  using A = Act<T>;
  constexpr bool kQuant = BITS != 0;
  constexpr int WPG = Fmt<BITS>::kWordsPerGroup;
  constexpr int WPT = Fmt<BITS>::kWordsPerThread;
  constexpr int PF = Fmt<BITS>::kPF;
  constexpr int TOK = NT * 8;
  constexpr uint32_t kMask = 0x000F000Fu;
  constexpr uint32_t kMag = A::kMagic2;
  constexpr float kOff = BITS == 4 ? A::kMagic : 17.0f * A::kMagic;
  constexpr int kRowsOut = GATE ? 64 : 128;
  // all-ones A operand (1.0 in both halves) for sum(x) through the tensor core
  constexpr uint32_t kOne2 = sizeof(T) == 2 && A::kMagic == 128.0f ? 0x3F803F80u : 0x3C003C00u;

  extern __shared__ __align__(16) unsigned char smem[];
  const int KC = a.KC;
  const int xs_stride = KC * 64 + 8;  // elements per token row of the staged x (16-byte bank offset)
  T* sx = reinterpret_cast<T*>(smem);
  float* sacc = reinterpret_cast<float*>(smem);  // reused after the main loop: [16][kAccStride]
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, c = lane & 3;
  const int nb = blockIdx.x, split = blockIdx.y, z = blockIdx.z;
  const int g0 = split * KC;
  const int ng = min(KC, a.G - g0);
  const int m0 = z * kTokMax;
  const int mc = min(kTokMax, a.M - m0);
  const int N = a.N;
  const int wpr = a.K / 64 * WPG;  // words per weight row

  pdl_wait();
  pdl_launch_next();
  // ---- x for this CTA's K range -> shared memory (natural order), one async copy -------
  {
    const T* x = static_cast<const T*>(a.x);
    const int chunks = ng * 8;  // 16-byte chunks per token row
    for (int e = tid; e < TOK * chunks; e += kThreads) {
      const int m = e / chunks, i = e % chunks;
      const bool ok = m < mc;
      const T* src = ok ? x + (size_t)(m0 + m) * a.K + (size_t)g0 * 64 + i * 8 : x;
      cp_async16(sx + m * xs_stride + i * 8, src, ok ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }

  // ---- the four weight rows of this thread: q = tile * 2 + half --------------------
  const uint32_t* rowp[4];
  const unsigned short* sp[4];
  const unsigned short* bp[4];
  int slot[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t = q >> 1, h = q & 1;
    int n;
    const uint32_t* base;
    const void* sbase = a.sc;
    const void* bbase = a.bi;
    if constexpr (GATE) {
      slot[q] = t * 64 + warp * 16 + h * 8 + r;
      n = nb * 64 + warp * 16 + h * 8 + r;
      base = t == 0 ? a.w : a.uw;
      if (t == 1) { sbase = a.usc; bbase = a.ubi; }
    } else {
      slot[q] = warp * 32 + t * 16 + h * 8 + r;
      n = nb * 128 + slot[q];
      base = a.w;
    }
    n = min(n, N - 1);
    rowp[q] = base + (size_t)n * wpr + (size_t)g0 * WPG + c * WPT;
    sp[q] = bp[q] = nullptr;
    if constexpr (kQuant) {
      sp[q] = static_cast<const unsigned short*>(sbase) + (size_t)n * a.G + g0;
      bp[q] = static_cast<const unsigned short*>(bbase) + (size_t)n * a.G + g0;
    }
  }

  // ---- register ring: weights (+ scale, bias) of the next PF groups ------------------
  uint32_t st[PF][4][WPT];
  uint32_t sb[PF][4][2];
#pragma unroll
  for (int s = 0; s < PF; ++s)
    if (s < ng) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        load_words<BITS>(st[s][q], rowp[q] + s * WPG);
        if constexpr (kQuant) { sb[s][q][0] = ld_u16(sp[q] + s); sb[s][q][1] = ld_u16(bp[q] + s); }
      }
    }

  asm volatile("cp.async.wait_all;\n" ::);
  __syncthreads();

  float acc[2][NT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][nt][i] = 0.0f;

  const uint32_t ones[4] = {kOne2, kOne2, kOne2, kOne2};

  for (int gb = 0; gb < ng; gb += PF) {
#pragma unroll
    for (int s = 0; s < PF; ++s) {
      const int g = gb + s;
      if (g < ng) {
        // x fragments of this group (token r of each n8 tile, k quarter c), permuted
        uint32_t B[NT][8];
        float X[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4* src = reinterpret_cast<const uint4*>(sx + (nt * 8 + r) * xs_stride + g * 64 + c * 16);
          const uint4 v0 = src[0], v1 = src[1];
          const uint32_t nat[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
          permute_x<BITS>(B[nt], nat);
          if constexpr (kQuant) {
#pragma unroll
            for (int i = 0; i < 4; ++i) X[nt][i] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) mma16816<T>(X[nt], ones, B[nt][2 * j], B[nt][2 * j + 1]);
          }
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t* w0 = st[s][2 * t];      // row r of tile t
          const uint32_t* w1 = st[s][2 * t + 1];  // row r + 8 of tile t
          if constexpr (BITS == 0) {
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
              for (int i = 0; i < 4; ++i) d[nt][i] = 0.0f;
            if constexpr (BITS == 4) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int sh = (j & 1) * 8;
                const uint32_t u0 = w0[j >> 1], u1 = w1[j >> 1];
                const uint32_t af[4] = {and_or(u0 >> sh, kMask, kMag), and_or(u1 >> sh, kMask, kMag),
                                        and_or(u0 >> (sh + 4), kMask, kMag), and_or(u1 >> (sh + 4), kMask, kMag)};
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<T>(d[nt], af, B[nt][2 * j], B[nt][2 * j + 1]);
              }
            } else {
              float dh[NT][4];
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) dh[nt][i] = 0.0f;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t u0 = w0[j], u1 = w1[j];
                const uint32_t lo[4] = {and_or(u0, kMask, kMag), and_or(u1, kMask, kMag),
                                        and_or(u0 >> 8, kMask, kMag), and_or(u1 >> 8, kMask, kMag)};
                const uint32_t hi[4] = {and_or(u0 >> 4, kMask, kMag), and_or(u1 >> 4, kMask, kMag),
                                        and_or(u0 >> 12, kMask, kMag), and_or(u1 >> 12, kMask, kMag)};
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  mma16816<T>(d[nt], lo, B[nt][2 * j], B[nt][2 * j + 1]);
                  mma16816<T>(dh[nt], hi, B[nt][2 * j], B[nt][2 * j + 1]);
                }
              }
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) d[nt][i] = fmaf(16.0f, dh[nt][i], d[nt][i]);
            }
            const float s0 = A::lo(sb[s][2 * t][0]), s1 = A::lo(sb[s][2 * t + 1][0]);
            const float b0 = fmaf(-kOff, s0, A::lo(sb[s][2 * t][1]));
            const float b1 = fmaf(-kOff, s1, A::lo(sb[s][2 * t + 1][1]));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[t][nt][0] = fmaf(s0, d[nt][0], fmaf(b0, X[nt][0], acc[t][nt][0]));
              acc[t][nt][1] = fmaf(s0, d[nt][1], fmaf(b0, X[nt][1], acc[t][nt][1]));
              acc[t][nt][2] = fmaf(s1, d[nt][2], fmaf(b1, X[nt][0], acc[t][nt][2]));
              acc[t][nt][3] = fmaf(s1, d[nt][3], fmaf(b1, X[nt][1], acc[t][nt][3]));
            }
          }
        }
        if (g + PF < ng) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            load_words<BITS>(st[s][q], rowp[q] + (g + PF) * WPG);
            if constexpr (kQuant) { sb[s][q][0] = ld_u16(sp[q] + g + PF); sb[s][q][1] = ld_u16(bp[q] + g + PF); }
          }
        }
      }
    }
  }

  // ---- CTA tile -> shared memory [token][slot] (x is no longer needed) -----------------
  __syncthreads();
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tk = nt * 8 + 2 * c;
      sacc[tk * kAccStride + slot[2 * t]] = acc[t][nt][0];
      sacc[(tk + 1) * kAccStride + slot[2 * t]] = acc[t][nt][1];
      sacc[tk * kAccStride + slot[2 * t + 1]] = acc[t][nt][2];
      sacc[(tk + 1) * kAccStride + slot[2 * t + 1]] = acc[t][nt][3];
    }
  __syncthreads();

  // ---- split-K: publish the partial tile; the last CTA of the row block adds them ----
  if (a.S > 1) {
    const int wd = a.rowblocks * kSlots;
    float* part = a.partial + (size_t)(z * a.S + split) * kTokMax * wd + (size_t)nb * kSlots;
    for (int e = tid; e < mc * kSlots; e += kThreads) {
      const int m = e / kSlots, sl = e % kSlots;
      part[(size_t)m * wd + sl] = sacc[m * kAccStride + sl];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      int* ctr = a.counters + z * a.rowblocks + nb;
      const int prev = atomicAdd(ctr, 1);
      const int last = prev == a.S - 1;
      if (last) *ctr = 0;  // every CTA of this row block has arrived: reset for the next call
      s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = a.partial + (size_t)z * a.S * kTokMax * wd + (size_t)nb * kSlots;
    for (int e = tid; e < mc * kSlots; e += kThreads) {
      const int m = e / kSlots, sl = e % kSlots;
      float v = 0.0f;
      for (int sp2 = 0; sp2 < a.S; ++sp2) v += __ldcg(base + ((size_t)sp2 * kTokMax + m) * wd + sl);
      sacc[m * kAccStride + sl] = v;
    }
    __syncthreads();
  }

  // ---- epilogue: GATE -> bias -> residual, one rounding --------------------------------
  const T* bias = static_cast<const T*>(a.bias);
  const T* res = static_cast<const T*>(a.res);
  T* out = static_cast<T*>(a.out);
  for (int e = tid; e < mc * kRowsOut; e += kThreads) {
    const int m = e / kRowsOut, j = e % kRowsOut;
    const int n = nb * kRowsOut + j;
    if (n >= N) continue;
    float v = sacc[m * kAccStride + j];
    if constexpr (GATE) {
      const float u = sacc[m * kAccStride + 64 + j];
      v = v / (1.0f + expf(-v)) * u;
    }
    const size_t o = (size_t)(m0 + m) * N + n;
    if (a.has_bias) v += A::to_f(bias[n]);
    if (a.gelu) v = gelu_erf(v);
    if (a.has_res) v += A::to_f(res[o]);
    out[o] = A::from_f(v);
  }
}

size_t smem_bytes(int nt, int kc) {
  const size_t x = (size_t)nt * 8 * (kc * 64 + 8) * 2;
  const size_t accb = (size_t)kTokMax * kAccStride * 4;
  return std::max(x, accb);
}

template <typename T, int BITS, int NT, bool GATE>
int launch_t(const Args& a, dim3 grid, size_t smem, cudaStream_t stream) {
  auto k = qgemm_kernel<T, BITS, NT, GATE>;
  // One attribute call per instantiation and device.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes(2, kKCMax)));
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  return launch_kernel(k, grid, dim3(kThreads), smem, stream, a);
}

template <typename T, int BITS>
int dispatch_nt(const Args& a, bool gate, int nt, dim3 grid, size_t smem, cudaStream_t s) {
  if (gate) return nt == 1 ? launch_t<T, BITS, 1, true>(a, grid, smem, s) : launch_t<T, BITS, 2, true>(a, grid, smem, s);
  return nt == 1 ? launch_t<T, BITS, 1, false>(a, grid, smem, s) : launch_t<T, BITS, 2, false>(a, grid, smem, s);
}

}  // namespace

bool qgemm_plan(const vella_qgemm_desc& d, QgemmPlan* p) {
  if (d.m < 0 || d.n < 0 || d.k <= 0) return false;
  if (d.bits != 0 && d.bits != 4 && d.bits != 8) return false;
  if (d.bits != 0 && d.group_size != 64) return false;
  if (d.k % 64 != 0) return false;
  if (d.dtype != VELLA_BF16 && d.dtype != VELLA_F16) return false;
  if (!epi_valid(d.epilogue)) return false;
  p->stream = false;
  p->tc = false;
  if (tc_eligible(d) && d.m <= (1 << 24)) {  // more than 16 rows: tensor cores
    p->tc = true;
    p->splits = tc_splits(d);
    p->workspace = tc_workspace(d, p->splits);
    return true;
  }
  if (d.m > 256) return false;
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  p->rows_out = gate ? 64 : 128;
  p->rowblocks = (d.n + p->rows_out - 1) / p->rows_out;
  const int G = d.k / 64;
  // Enough CTAs for ~4 per SM on a 148-SM B200; depends on (N, K, gate) only.
  const int target = 4 * 148;
  int want = (target + std::max(p->rowblocks, 1) - 1) / std::max(p->rowblocks, 1);
  want = std::max(1, std::min(want, G));
  int kc = (G + want - 1) / want;
  kc = std::max(kc, std::min(G, 4));
  kc = std::min(kc, kKCMax);
  p->kc = kc;
  p->splits = (G + kc - 1) / kc;
  p->zchunks = std::max(1, (d.m + kTokMax - 1) / kTokMax);
  p->stream = false;
  if (stream_eligible(d)) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
      cudaGetLastError();
      dev = -1;
    }
    int rb = 0, nkc = 0;
    stream_units(d, &rb, &nkc);
    p->stream = true;
    // one CTA per SM, but never more CTAs than units: every CTA owns at least one unit
    const int sms = num_sms(dev);
    // int4: the compact two-stage layout (96 registers, ~112 KB), two CTAs per SM for calls with
    // many units; with one CTA per SM the other half of the SM takes the next kernel's CTA, which
    // fetches its first weight stages while this call finishes
    p->light = d.bits == 4;
    p->ctas = (int)std::min<long long>((stream_light(d, rb, nkc, sms) ? 2 : 1) * (long long)sms, (long long)rb * nkc);
    p->rowblocks = rb;
    p->workspace = counter_region((size_t)stream_flag_count(p->ctas)) + stream_partial_bytes(p->ctas);
    return true;
  }
  if (p->splits > 1) {
    const size_t part = (size_t)p->zchunks * p->splits * kTokMax * (size_t)p->rowblocks * kSlots * sizeof(float);
    p->workspace = counter_region((size_t)p->zchunks * p->rowblocks) + part;
  } else {
    p->workspace = 0;
  }
  return true;
}

int qgemm_launch(const vella_qgemm_desc& d, const QgemmPlan& p, const void* x, const void* w,
                 const void* scales, const void* biases, const void* up_w, const void* up_scales,
                 const void* up_biases, const void* bias, const void* residual, void* out, void* ws,
                 cudaStream_t stream, const RopeEpi* rope, const KvAppendEpi* app, const NormEpi* norm) {
  if (d.m == 0 || d.n == 0) return VELLA_OK;
  if ((rope || app || norm) && !p.stream)
    return fail(VELLA_E_INVALID, "qgemm: the RoPE, K/V-append and LayerNorm epilogues run on the streaming kernel only");
  if (p.tc)
    return tc_launch(d, p.splits, x, w, scales, biases, up_w, up_scales, up_biases, bias, residual, out, ws, stream);
  if (p.stream) {
    int* flags = static_cast<int*>(ws);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) + counter_region((size_t)stream_flag_count(p.ctas)));
    // the LayerNorm tail's arrival counter: the last int of the counter region (the stream
    // flags take stream_flag_count(ctas) ints from its start)
    int* done = flags + kCounterRegion / sizeof(int) - 1;
    return stream_launch(d, p.ctas, p.light, x, w, scales, biases, up_w, up_scales, up_biases, bias, residual, out, flags,
                         partial, stream, rope, app, norm, done);
  }
  Args a{};
  a.x = x; a.w = static_cast<const uint32_t*>(w); a.sc = scales; a.bi = biases;
  a.uw = static_cast<const uint32_t*>(up_w); a.usc = up_scales; a.ubi = up_biases;
  a.bias = bias; a.res = residual; a.out = out;
  a.M = d.m; a.N = d.n; a.K = d.k; a.G = d.k / 64; a.KC = p.kc; a.S = p.splits; a.rowblocks = p.rowblocks;
  a.has_bias = epi_bias(d.epilogue);
  a.has_res = epi_residual(d.epilogue);
  a.gelu = epi_gelu(d.epilogue);
  if (p.splits > 1) {
    a.counters = static_cast<int*>(ws);
    a.partial = reinterpret_cast<float*>(static_cast<char*>(ws) + counter_region((size_t)p.zchunks * p.rowblocks));
  }
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  const int nt = d.m <= 8 ? 1 : 2;
  const size_t smem = smem_bytes(nt, p.kc);
  const dim3 grid(p.rowblocks, p.splits, p.zchunks);
  if (d.dtype == VELLA_BF16) {
    switch (d.bits) {
      case 4: return dispatch_nt<__nv_bfloat16, 4>(a, gate, nt, grid, smem, stream);
      case 8: return dispatch_nt<__nv_bfloat16, 8>(a, gate, nt, grid, smem, stream);
      default: return dispatch_nt<__nv_bfloat16, 0>(a, gate, nt, grid, smem, stream);
    }
  }
  switch (d.bits) {
    case 4: return dispatch_nt<__half, 4>(a, gate, nt, grid, smem, stream);
    case 8: return dispatch_nt<__half, 8>(a, gate, nt, grid, smem, stream);
    default: return dispatch_nt<__half, 0>(a, gate, nt, grid, smem, stream);
  }
}

}  // namespace vella
