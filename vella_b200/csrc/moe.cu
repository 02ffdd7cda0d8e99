// Nemotron-H's MoE router on the device: fp32 router logits, sigmoid scores, top-k selection
// by score plus the correction bias, weights from the unbiased scores.
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeDecoder.swift:
// NTMoE.callAsFunction (:487-496): original = sigmoid(x . W^T) in fp32, biased = original +
// e_score_correction_bias, the top_k experts of biased (argPartition; ties here go to the lower
// expert index, the chosen experts listed by descending biased score), scores = original at
// them, / (sum + 1e-20) when norm_topk_prob and top_k > 1, * routed_scaling_factor.
//
// One CTA per row: the row of x staged in shared memory as fp32, each warp takes every 8th
// expert's dot product (lanes split the hidden dimension, warp sum), then top_k rounds of a
// block argmax with the lowest index on ties.  The router is tiny next to the experts'
// GEMMs (E x hidden fp32 read per row, from L2 after the first row).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace vella {
namespace {

constexpr int kRouteThreads = 256, kMaxExperts = 1024, kMaxTopK = 32, kMaxHidden = 16384;

struct RouteArgs {
  int M, hidden, E, k, norm;
  float scaling;
};

template <typename T>
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(RouteArgs a, const T* __restrict__ x,
                                                                  const float* __restrict__ W,
                                                                  const float* __restrict__ bias,
                                                                  int32_t* __restrict__ idx, float* __restrict__ wout) {
  using A = Act<T>;
  extern __shared__ float sm[];
  float* xs = sm;                  // [hidden]
  float* p = xs + a.hidden;        // [E] sigmoid scores
  float* q = p + a.E;              // [E] biased scores, -inf once chosen
  __shared__ float rv[kRouteThreads / 32];
  __shared__ int ri[kRouteThreads / 32];
  __shared__ int chosen[kMaxTopK];
  pdl_wait();
  pdl_launch_next();
  const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < a.hidden; i += kRouteThreads) xs[i] = A::to_f(x[(size_t)m * a.hidden + i]);
  __syncthreads();
  for (int e = warp; e < a.E; e += kRouteThreads / 32) {
    const float* w = W + (size_t)e * a.hidden;
    float acc = 0.0f;
    for (int i = lane; i < a.hidden; i += 32) acc = fmaf(xs[i], w[i], acc);
    acc = warp_sum(acc);
    if (lane == 0) {
      const float s = 1.0f / (1.0f + expf(-acc));
      p[e] = s;
      q[e] = s + bias[e];
    }
  }
  __syncthreads();
  for (int j = 0; j < a.k; ++j) {
    float bv = -INFINITY;
    int bi = INT32_MAX;
    for (int e = threadIdx.x; e < a.E; e += kRouteThreads)
      if (q[e] > bv || (q[e] == bv && e < bi)) { bv = q[e]; bi = e; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = -INFINITY;
      int b = INT32_MAX;
      for (int i = 0; i < kRouteThreads / 32; ++i)
        if (rv[i] > v || (rv[i] == v && ri[i] < b)) { v = rv[i]; b = ri[i]; }
      if (b == INT32_MAX) b = 0;  // every score non-finite: expert 0
      chosen[j] = b;
      q[b] = -INFINITY;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int j = 0; j < a.k; ++j) sum += p[chosen[j]];
    const float div = (a.norm && a.k > 1) ? sum + 1e-20f : 1.0f;
    for (int j = 0; j < a.k; ++j) {
      idx[(size_t)m * a.k + j] = chosen[j];
      wout[(size_t)m * a.k + j] = p[chosen[j]] / div * a.scaling;
    }
  }
}

}  // namespace
}  // namespace vella

using namespace vella;

extern "C" int vella_moe_route(const vella_moe_route_desc* d, const void* x, const float* router_w, const float* bias,
                               int32_t* expert_idx, float* expert_w, vella_stream_t stream) {
  if (!d || !x || !router_w || !bias || !expert_idx || !expert_w)
    return fail(VELLA_E_INVALID, "vella_moe_route: NULL argument");
  if (d->rows < 1 || d->hidden < 1 || d->hidden > kMaxHidden || d->experts < 1 || d->experts > kMaxExperts ||
      d->top_k < 1 || d->top_k > kMaxTopK || d->top_k > d->experts || (d->dtype != VELLA_BF16 && d->dtype != VELLA_F16))
    return fail(VELLA_E_INVALID, "vella_moe_route: rows %d hidden %d (<= %d) experts %d (<= %d) top_k %d (<= %d)",
                d->rows, d->hidden, kMaxHidden, d->experts, kMaxExperts, d->top_k, kMaxTopK);
  const RouteArgs a{d->rows, d->hidden, d->experts, d->top_k, d->norm_topk ? 1 : 0, d->scaling};
  const size_t smem = (size_t)(d->hidden + 2 * d->experts) * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the opt-in shared-memory size is set on every call (cheap; per device and thread safe)
  if (d->dtype == VELLA_BF16) {
    VELLA_CUDA_TRY(cudaFuncSetAttribute(moe_route_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    return launch_kernel(moe_route_kernel<__nv_bfloat16>, dim3(a.M), dim3(kRouteThreads), smem, s, a,
                         static_cast<const __nv_bfloat16*>(x), router_w, bias, expert_idx, expert_w);
  }
  VELLA_CUDA_TRY(cudaFuncSetAttribute(moe_route_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_kernel(moe_route_kernel<__half>, dim3(a.M), dim3(kRouteThreads), smem, s, a,
                       static_cast<const __half*>(x), router_w, bias, expert_idx, expert_w);
}
