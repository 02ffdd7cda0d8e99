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
#include "stream_core.cuh"

namespace vella {

__device__ int g_stream_fault = 0;  // set when a pipeline wait ran out of time

namespace {

using namespace sk;

// LIGHT: the compact layout (96 registers a thread, two stages), two of which fit one SM: the
// int4 calls run two CTAs per SM when their units keep both busy, else one, which leaves room
// for the next kernel's CTA to start its weight copies before this call ends.
template <int BITS, int NT, bool LIGHT = false>
struct Layout : Tile<BITS, NT> {
  using TL = Tile<BITS, NT>;
  static constexpr int fixed(int ns) { return 1024 + TL::RED + 3 * ns * 8 + 16; }
  static constexpr int NS = LIGHT ? 2
                            : (fixed(4) + 4 * TL::STAGE <= 227 * 1024) ? 4
                            : (fixed(3) + 3 * TL::STAGE <= 227 * 1024) ? 3
                                                                        : 2;
  static constexpr int TOTAL = fixed(NS) + NS * TL::STAGE;
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
  int app;      // K/V-append epilogue (q|k|v projection without RoPE)
  KvAppendEpi ka;
  int norm;     // LayerNorm of the output rows by the last CTA
  NormEpi ne;
  int* done;    // CTAs past their epilogue (the last one resets it to zero)
};

template <typename T, int BITS, int NT, bool GATE, bool LIGHT>
__global__ void __launch_bounds__(kThreads, LIGHT ? 2 : 1) qgemm_stream_kernel(const __grid_constant__ SArgs a) {
  using LY = Layout<BITS, NT, LIGHT>;
  constexpr int UG = LY::UG, BPG = SFmt<BITS>::BPG, NS = LY::NS;
  constexpr bool kQuant = BITS != 0;
  constexpr int XOFF = LY::XOFF;

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
        if (!abort_flag[0]) prep_stage<T, BITS, NT>(smem + s * LY::STAGE + XOFF, lane);
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
  const int r = lane >> 2, cq = lane & 3;
  const int slot0 = 16 * warp + r, slot1 = slot0 + 8;  // this warp's weight rows in the unit
  const WOff<BITS> woff(slot0, r, cq);
  const int rf = (int)(u0 / nkc), rl = (int)((u1 - 1) / nkc);
  const bool head_shared = u0 % nkc != 0, tail_shared = u1 % nkc != 0;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
  Epi ep;
  ep.bias = a.bias; ep.res = a.res; ep.out = a.out; ep.partial = a.partial; ep.flags = a.flags;
  ep.N = a.N; ep.mc = min(a.M, kTokMax); ep.P = P; ep.U = U; ep.nkc = nkc;
  ep.gate = GATE; ep.has_bias = a.has_bias; ep.has_res = a.has_res; ep.gelu = a.gelu; ep.rope = a.rope;
  ep.re = &a.re; ep.fault = &g_stream_fault;
  ep.ka = a.app ? &a.ka : nullptr;

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
    if (!abort_flag[0]) consume_stage<T, BITS, NT>(smem + s * LY::STAGE, smem + s * LY::STAGE + XOFF, acc, woff, lane, slot0, slot1);
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
    flush_rowblock<T, NT>(ep, c, rb, rb == rl && tail_shared, rb == rf && head_shared, acc, red, warp, lane);
  }
  if (a.norm) {
    // The output rows are complete once every CTA has arrived here; the last to arrive
    // normalises them (no CTA waits for another).
    __threadfence();
    named_sync(kBarConsumers, kRowWarps * 32);
    if (tid == 0) {
      const int last = atomicAdd(a.done, 1) == P - 1;
      if (last) {
        __threadfence();
        *a.done = 0;  // every CTA has arrived: zero for the next call
      }
      abort_flag[1] = last;
    }
    named_sync(kBarConsumers, kRowWarps * 32);
    if (abort_flag[1]) {
      const int D = a.N;
      for (int m = 0; m < ep.mc; ++m)
        ln_row256<T>(static_cast<T*>(a.ne.out) + (size_t)m * D, static_cast<const T*>(a.out) + (size_t)m * D,
                     static_cast<const T*>(a.ne.w), static_cast<const T*>(a.ne.b), D, a.ne.eps, tid, red,
                     [] { named_sync(kBarConsumers, kRowWarps * 32); });
    }
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
                  cudaStream_t stream, const RopeEpi* rope, const KvAppendEpi* app, const NormEpi* norm, int* done) {
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
  if (app) {
    if (gate || rope || app->d <= 0 || app->hd <= 0 || app->d % app->hd || d.n != 3 * app->d)
      return fail(VELLA_E_INVALID, "stream GEMM: the K/V-append epilogue needs a q|k|v projection of 3 x d rows");
    a.app = 1;
    a.ka = *app;
  }
  if (norm) {
    if (gate || rope || d.n > kLnMaxD || !done || !norm->out || !norm->w || !norm->b)
      return fail(VELLA_E_INVALID, "stream GEMM: the LayerNorm tail needs at most %d output columns", kLnMaxD);
    a.norm = 1;
    a.ne = *norm;
    a.done = done;
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
