// Nemotron-H's routed experts on the device: y[m] = sum_j w[m][j] * fc2_e(relu(fc1_e(x[m]))^2)
// with e = expert_idx[m][j], the experts' weights MLX-affine (int4 / int8, group 64) or dense.
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeDecoder.swift:
// NTSwitchMLP (:435-462: fc1, relu, square, fc2 through gatherQuantizedMM / gatherMM over the
// stacked [experts, out, in] weights) and NTMoE's weighted sum over the chosen experts
// (:497-499).  The shared expert (NTMLP, relu^2 as well) is the same computation with one
// expert chosen by every row at weight 1.
//
// Four launches, for decode-sized batches (rows * top_k pairs, a few hundred at most):
//   moe_sort_kernel     one thread: counting sort of the (row, slot) pairs by expert (stable:
//                       row, then slot; O(pairs + experts)), per-expert offsets and each pair's
//                       sorted position.
//   moe_fc_kernel<1>    CTA (64-row output tile, expert): the expert's weight rows are read
//                       once per chunk of 4 of its pairs (a warp per 8 output rows, lanes
//                       splitting K, codes dequantized as scale * q + bias in registers), the
//                       pairs' input rows staged in shared memory as fp32; relu^2 into an fp32
//                       scratch row per pair.  Experts no pair chose exit at once.
//   moe_fc_kernel<2>    the same over fc2, input the scratch rows, output fp32 per pair.
//   moe_combine_kernel  out[m] (+)= sum_j w[m][j] * y[pair(m, j)], slots in order.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace vella {
namespace {

constexpr int kFcRows = 64, kFcThreads = 256, kFcPairs = 4;
constexpr int kMaxPairs = 4096, kMaxMoeK = 8192;  // 4 staged rows of K fp32 fit shared memory

struct MoeArgs {
  int rows, hidden, inter, E, k, bits;
  int* order;    // [pairs] pair ids (row * k + slot) sorted by expert
  int* pos;      // [pairs] sorted position of pair id
  int* offsets;  // [E + 1]
  int* cursor;   // [E] fill cursors of the sort
  float* h;      // [pairs][inter] relu^2(fc1), in sorted order
  float* y;      // [pairs][hidden] fc2, in sorted order
};

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t moe_ws_bytes(int rows, int k, int E, int hidden, int inter) {
  const size_t P = (size_t)rows * k;
  return align256(P * sizeof(int)) * 2 + align256((size_t)(E + 1) * sizeof(int)) + align256((size_t)E * sizeof(int)) +
         align256(P * inter * sizeof(float)) + align256(P * hidden * sizeof(float));
}

__global__ void moe_sort_kernel(MoeArgs a, const int32_t* __restrict__ idx) {
  pdl_wait();
  pdl_launch_next();
  if (threadIdx.x != 0) return;
  const int P = a.rows * a.k;
  for (int e = 0; e <= a.E; ++e) a.offsets[e] = 0;
  for (int p = 0; p < P; ++p) {
    const int e = idx[p];
    if (e >= 0 && e < a.E) a.offsets[e + 1] += 1;
  }
  for (int e = 0; e < a.E; ++e) {
    a.offsets[e + 1] += a.offsets[e];
    a.cursor[e] = a.offsets[e];
  }
  // stable fill: pairs in id order (row, then slot) within each expert
  for (int p = 0; p < P; ++p) {
    const int e = idx[p];
    if (e >= 0 && e < a.E) {
      const int sp = a.cursor[e]++;
      a.order[sp] = p;
      a.pos[p] = sp;
    } else {
      a.pos[p] = -1;  // an expert id out of range contributes nothing
    }
  }
}

template <typename T, int BITS>
__device__ __forceinline__ float weight_at(const void* w, const T* s, const T* b, size_t row, int K, int kk) {
  using A = Act<T>;
  if constexpr (BITS == 0) {
    return A::to_f(static_cast<const T*>(w)[row * K + kk]);
  } else {
    constexpr int per = 32 / BITS;
    const uint32_t word = static_cast<const uint32_t*>(w)[row * (size_t)(K / per) + kk / per];
    const float q = (float)((word >> ((kk % per) * BITS)) & ((1u << BITS) - 1u));
    const size_t g = row * (size_t)(K / 64) + kk / 64;
    return __fadd_rn(__fmul_rn(A::to_f(s[g]), q), A::to_f(b[g]));
  }
}

// STAGE 1: out rows = inter, input = x rows (act dtype, gathered by pair); relu^2 -> a.h.
// STAGE 2: out rows = hidden, input = a.h rows (fp32, sorted order) -> a.y.
template <typename T, int BITS, int STAGE>
__global__ void __launch_bounds__(kFcThreads) moe_fc_kernel(MoeArgs a, const T* __restrict__ x, const void* __restrict__ w,
                                                            const T* __restrict__ ws, const T* __restrict__ wb) {
  using A = Act<T>;
  extern __shared__ float xs[];  // [kFcPairs][K]
  pdl_wait();
  pdl_launch_next();
  const int e = blockIdx.y, n0 = blockIdx.x * kFcRows;
  const int N = STAGE == 1 ? a.inter : a.hidden, K = STAGE == 1 ? a.hidden : a.inter;
  const int beg = a.offsets[e], end = a.offsets[e + 1];
  if (beg == end || n0 >= N) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t ebase = (size_t)e * N;  // the expert's first weight row
  for (int c0 = beg; c0 < end; c0 += kFcPairs) {
    const int np = min(kFcPairs, end - c0);
    __syncthreads();  // the previous chunk's rows are no longer read
    for (int i = threadIdx.x; i < np * K; i += kFcThreads) {
      const int pi = i / K, kk = i % K, sp = c0 + pi;
      float v;
      if constexpr (STAGE == 1) v = A::to_f(x[(size_t)(a.order[sp] / a.k) * K + kk]);
      else v = a.h[(size_t)sp * K + kk];
      xs[pi * K + kk] = v;
    }
    __syncthreads();
    for (int r = warp; r < kFcRows; r += kFcThreads / 32) {
      const int n = n0 + r;
      if (n >= N) break;
      float acc[kFcPairs] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int kk = lane; kk < K; kk += 32) {
        const float wv = weight_at<T, BITS>(w, ws, wb, ebase + n, K, kk);
#pragma unroll
        for (int pi = 0; pi < kFcPairs; ++pi) acc[pi] = fmaf(wv, xs[pi * K + kk], acc[pi]);
      }
#pragma unroll
      for (int pi = 0; pi < kFcPairs; ++pi) acc[pi] = warp_sum(acc[pi]);
      if (lane < np) {
        const float v = acc[lane];
        const int sp = c0 + lane;
        if constexpr (STAGE == 1) {
          const float rl = fmaxf(v, 0.0f);
          a.h[(size_t)sp * N + n] = rl * rl;
        } else {
          a.y[(size_t)sp * N + n] = v;
        }
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) moe_combine_kernel(MoeArgs a, const float* __restrict__ wgt, T* __restrict__ out,
                                                          int accumulate) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x;
  for (int n = threadIdx.x; n < a.hidden; n += blockDim.x) {
    float acc = accumulate ? A::to_f(out[(size_t)m * a.hidden + n]) : 0.0f;
    for (int j = 0; j < a.k; ++j) {
      const int sp = a.pos[m * a.k + j];
      if (sp >= 0) acc = fmaf(wgt[m * a.k + j], a.y[(size_t)sp * a.hidden + n], acc);
    }
    out[(size_t)m * a.hidden + n] = A::from_f(acc);
  }
}

template <typename T, int BITS>
int run_moe(const vella_moe_experts_desc* d, MoeArgs a, const void* x, const int32_t* idx, const float* wgt,
            const void* f1w, const void* f1s, const void* f1b, const void* f2w, const void* f2s, const void* f2b,
            void* out, int accumulate, cudaStream_t s) {
  int rc = launch_kernel(moe_sort_kernel, dim3(1), dim3(32), 0, s, a, idx);
  if (rc) return rc;
  const size_t sm1 = (size_t)kFcPairs * a.hidden * sizeof(float), sm2 = (size_t)kFcPairs * a.inter * sizeof(float);
  VELLA_CUDA_TRY(cudaFuncSetAttribute(moe_fc_kernel<T, BITS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1));
  VELLA_CUDA_TRY(cudaFuncSetAttribute(moe_fc_kernel<T, BITS, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2));
  rc = launch_kernel(moe_fc_kernel<T, BITS, 1>, dim3((a.inter + kFcRows - 1) / kFcRows, a.E), dim3(kFcThreads), sm1,
                     s, a, static_cast<const T*>(x), f1w, static_cast<const T*>(f1s), static_cast<const T*>(f1b));
  if (rc) return rc;
  rc = launch_kernel(moe_fc_kernel<T, BITS, 2>, dim3((a.hidden + kFcRows - 1) / kFcRows, a.E), dim3(kFcThreads), sm2,
                     s, a, static_cast<const T*>(x), f2w, static_cast<const T*>(f2s), static_cast<const T*>(f2b));
  if (rc) return rc;
  (void)d;
  return launch_kernel(moe_combine_kernel<T>, dim3(a.rows), dim3(256), 0, s, a, wgt, static_cast<T*>(out), accumulate);
}

}  // namespace
}  // namespace vella

using namespace vella;

extern "C" {

size_t vella_moe_experts_workspace_size(const vella_moe_experts_desc* d) {
  if (!d || d->rows < 1 || d->top_k < 1 || d->experts < 1 || d->hidden < 1 || d->inter < 1) return 0;
  return moe_ws_bytes(d->rows, d->top_k, d->experts, d->hidden, d->inter);
}

int vella_moe_experts(const vella_moe_experts_desc* d, const void* x, const int32_t* expert_idx, const float* expert_w,
                      const void* fc1_w, const void* fc1_scales, const void* fc1_biases, const void* fc2_w,
                      const void* fc2_scales, const void* fc2_biases, void* out, int32_t accumulate, void* workspace,
                      size_t workspace_bytes, vella_stream_t stream) {
  if (!d || !x || !expert_idx || !expert_w || !fc1_w || !fc2_w || !out || !workspace)
    return fail(VELLA_E_INVALID, "vella_moe_experts: NULL argument");
  const bool q = d->bits != 0;
  if ((d->bits != 0 && d->bits != 4 && d->bits != 8) || (q && (!fc1_scales || !fc1_biases || !fc2_scales || !fc2_biases)))
    return fail(VELLA_E_INVALID, "vella_moe_experts: bits %d needs scales and biases", d->bits);
  if (d->rows < 1 || d->top_k < 1 || d->experts < 1 || (long long)d->rows * d->top_k > kMaxPairs || d->hidden < 64 ||
      d->inter < 64 || d->hidden > kMaxMoeK || d->inter > kMaxMoeK || (q && (d->hidden % 64 || d->inter % 64)) ||
      (d->dtype != VELLA_BF16 && d->dtype != VELLA_F16))
    return fail(VELLA_E_INVALID, "vella_moe_experts: rows %d top_k %d (pairs <= %d) experts %d hidden %d inter %d "
                "(64..%d, multiples of 64 when quantized)", d->rows, d->top_k, kMaxPairs, d->experts, d->hidden,
                d->inter, kMaxMoeK);
  const size_t need = moe_ws_bytes(d->rows, d->top_k, d->experts, d->hidden, d->inter);
  if (workspace_bytes < need) return fail(VELLA_E_INVALID, "vella_moe_experts: workspace %zu < %zu bytes", workspace_bytes, need);
  char* p = static_cast<char*>(workspace);
  const size_t P = (size_t)d->rows * d->top_k;
  MoeArgs a{d->rows, d->hidden, d->inter, d->experts, d->top_k, d->bits, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  a.order = reinterpret_cast<int*>(p); p += align256(P * sizeof(int));
  a.pos = reinterpret_cast<int*>(p); p += align256(P * sizeof(int));
  a.offsets = reinterpret_cast<int*>(p); p += align256((size_t)(d->experts + 1) * sizeof(int));
  a.cursor = reinterpret_cast<int*>(p); p += align256((size_t)d->experts * sizeof(int));
  a.h = reinterpret_cast<float*>(p); p += align256(P * d->inter * sizeof(float));
  a.y = reinterpret_cast<float*>(p);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = d->dtype == VELLA_BF16;
#define VELLA_MOE_RUN(T, B)                                                                                      \
  return run_moe<T, B>(d, a, x, expert_idx, expert_w, fc1_w, fc1_scales, fc1_biases, fc2_w, fc2_scales, fc2_biases, \
                       out, accumulate, s)
  if (d->bits == 4) {
    if (bf) VELLA_MOE_RUN(__nv_bfloat16, 4);
    VELLA_MOE_RUN(__half, 4);
  }
  if (d->bits == 8) {
    if (bf) VELLA_MOE_RUN(__nv_bfloat16, 8);
    VELLA_MOE_RUN(__half, 8);
  }
  if (bf) VELLA_MOE_RUN(__nv_bfloat16, 0);
  VELLA_MOE_RUN(__half, 0);
#undef VELLA_MOE_RUN
}

}  // extern "C"
