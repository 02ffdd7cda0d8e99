// Nemotron-H's Mamba-2 mixer core on the device: the stateful causal depthwise conv with SiLU,
// the selective scan with an fp32 state, and the gated group RMSNorm.  The in_proj and
// out_proj GEMMs around them are vella_qgemm calls.
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeDecoder.swift:
// NTMamba (:318-360: in_proj -> gate | conv input | dt; conv over the cached K - 1 inputs, SiLU;
// x | B | C), ntComputeDt (:214-216: clip(softplus(dt + dt_bias))), nt_ssm_kernel and
// nt_ssm_initial_kernel (:126-194: per head and channel d, lanes splitting the state dimension,
// state = exp(-exp(A_log) dt) state + x dt B, y = state . C + x D, fp32 state), ntSSMAttn
// (:225-276: the SSD chunk form the reference uses for several tokens with a state; the same
// recurrence, computed here sequentially in fp32), NTGatedRMSNorm (:301-316).
//
// Layout: rows are stream-major (row s * T + t).  The in_proj output ("zxbcdt") has rows of
// in_stride elements: gate [0, I), conv input [I, I + convDim), dt [I + convDim, + H), with
// I = heads * head_dim and convDim = I + 2 * groups * state_dim.  conv_state [S][K-1][convDim]
// (activation dtype, the last K - 1 conv inputs), ssm_state [S][H][Dh][Ds] fp32.
//
// Kernels (HBM/latency-bound elementwise and scan work, no tensor cores):
//   mamba_conv_kernel   one thread per channel of one stream, the K-tap window in registers,
//                       T rows in order; the window goes back to conv_state at the end.
//   mamba_ssm_kernel    one warp per (stream, head, channel d), Ds / 32 states per lane in
//                       registers for all T rows (state read once, written once), warp-sum
//                       of state . C per row.
//   mamba_norm_kernel   one CTA per (row, group): y * silu(gate), mean square, scale, weight.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace vella {
namespace {

constexpr int kMaxConvK = 8;
constexpr int kMaxStatePerLane = 8;  // state_dim <= 256

struct MambaDims {
  int S, T, H, Dh, G, Ds, K, I, conv_dim, in_stride;
  float dt_min, dt_max, eps;
};

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float softplus_f(float v) { return v > 20.0f ? v : log1pf(expf(v)); }

// K taps in registers (a template parameter, so the window shifts stay in registers)
template <typename T, int K>
__global__ void __launch_bounds__(128) mamba_conv_kernel(MambaDims m, const T* __restrict__ zx, const T* __restrict__ w,
                                                         const T* __restrict__ bias, T* __restrict__ cstate,
                                                         T* __restrict__ xbc) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int c = blockIdx.x * blockDim.x + threadIdx.x, s = blockIdx.y;
  if (c >= m.conv_dim) return;
  float wk[K], win[K];  // win[0 .. K-2]: the last K - 1 inputs, oldest first
#pragma unroll
  for (int k = 0; k < K; ++k) wk[k] = A::to_f(w[(size_t)c * K + k]);
  T* st = cstate + (size_t)s * (K - 1) * m.conv_dim;
#pragma unroll
  for (int k = 0; k < K - 1; ++k) win[k] = A::to_f(st[(size_t)k * m.conv_dim + c]);
  const float b = bias ? A::to_f(bias[c]) : 0.0f;
  for (int t = 0; t < m.T; ++t) {
    const size_t row = (size_t)s * m.T + t;
    const float xin = A::to_f(zx[row * m.in_stride + m.I + c]);
    float acc = b;
#pragma unroll
    for (int k = 0; k < K - 1; ++k) acc = fmaf(wk[k], win[k], acc);
    acc = fmaf(wk[K - 1], xin, acc);
    xbc[row * m.conv_dim + c] = A::from_f(silu_f(acc));
#pragma unroll
    for (int k = 0; k + 1 < K - 1; ++k) win[k] = win[k + 1];
    if constexpr (K > 1) win[K - 2] = xin;
  }
#pragma unroll
  for (int k = 0; k < K - 1; ++k) st[(size_t)k * m.conv_dim + c] = A::from_f(win[k]);
}

template <typename T, int K = 1>
int launch_conv(const MambaDims& m, const void* zx, const void* w, const void* b, void* cs, void* xbc, cudaStream_t s) {
  if (m.K != K) {
    if constexpr (K < kMaxConvK) return launch_conv<T, K + 1>(m, zx, w, b, cs, xbc, s);
    else return fail(VELLA_E_INVALID, "vella_mamba_conv: conv_kernel %d", m.K);
  }
  const dim3 grid((m.conv_dim + 127) / 128, m.S);
  return launch_kernel(mamba_conv_kernel<T, K>, grid, dim3(128), 0, s, m, static_cast<const T*>(zx),
                       static_cast<const T*>(w), static_cast<const T*>(b), static_cast<T*>(cs), static_cast<T*>(xbc));
}

template <typename T>
__global__ void __launch_bounds__(256) mamba_ssm_kernel(MambaDims m, const T* __restrict__ xbc, const T* __restrict__ zx,
                                                        const float* __restrict__ a_log,
                                                        const float* __restrict__ dt_bias, const float* __restrict__ Dv,
                                                        float* __restrict__ state, T* __restrict__ y) {
  using A = Act<T>;
  pdl_wait();
  pdl_launch_next();
  const int warps_per_head = (m.Dh + 7) / 8;
  const int h = blockIdx.x / warps_per_head;
  const int d = (blockIdx.x % warps_per_head) * 8 + threadIdx.y;
  const int s = blockIdx.y, lane = threadIdx.x;
  if (d >= m.Dh) return;
  const int per = m.Ds / 32, g = h / (m.H / m.G);
  float* st = state + (((size_t)s * m.H + h) * m.Dh + d) * m.Ds + (size_t)lane * per;
  float reg[kMaxStatePerLane];
#pragma unroll
  for (int i = 0; i < kMaxStatePerLane; ++i) reg[i] = i < per ? st[i] : 0.0f;
  const float A_h = -expf(a_log[h]), D_h = Dv[h], bias_h = dt_bias[h];
  for (int t = 0; t < m.T; ++t) {
    const size_t row = (size_t)s * m.T + t;
    const float dt = fminf(fmaxf(softplus_f(A::to_f(zx[row * m.in_stride + m.I + m.conv_dim + h]) + bias_h), m.dt_min),
                           m.dt_max);
    const float dA = expf(A_h * dt);
    const T* r = xbc + row * m.conv_dim;
    const float x = A::to_f(r[h * m.Dh + d]);
    const T* Bp = r + m.I + (size_t)g * m.Ds + (size_t)lane * per;
    const T* Cp = r + m.I + (size_t)m.G * m.Ds + (size_t)g * m.Ds + (size_t)lane * per;
    const float xdt = x * dt;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxStatePerLane; ++i)
      if (i < per) {
        reg[i] = fmaf(dA, reg[i], xdt * A::to_f(Bp[i]));
        acc = fmaf(reg[i], A::to_f(Cp[i]), acc);
      }
    acc = warp_sum(acc);
    if (lane == 0) y[row * m.I + h * m.Dh + d] = A::from_f(fmaf(x, D_h, acc));
  }
#pragma unroll
  for (int i = 0; i < kMaxStatePerLane; ++i)
    if (i < per) st[i] = reg[i];
}

constexpr int kNormThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) mamba_norm_kernel(MambaDims m, const T* __restrict__ yv,
                                                                  const T* __restrict__ zx, const T* __restrict__ w,
                                                                  T* __restrict__ out) {
  using A = Act<T>;
  __shared__ float red[kNormThreads / 32];
  pdl_wait();
  pdl_launch_next();
  const size_t row = blockIdx.x;
  const int gs = m.I / m.G, c0 = blockIdx.y * gs;
  const T* yr = yv + row * m.I + c0;
  const T* gr = zx + row * m.in_stride + c0;  // the gate is the first I columns of the in_proj output
  float ss = 0.0f;
  for (int i = threadIdx.x; i < gs; i += kNormThreads) {
    const float v = A::to_f(yr[i]) * silu_f(A::to_f(gr[i]));
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)gs + m.eps);
  T* o = out + row * m.I + c0;
  for (int i = threadIdx.x; i < gs; i += kNormThreads) {
    const float v = A::to_f(yr[i]) * silu_f(A::to_f(gr[i]));
    o[i] = A::from_f(v * r * A::to_f(w[c0 + i]));
  }
}

int mamba_dims(const vella_mamba_desc* d, MambaDims* m, const char* what) {
  if (!d) return fail(VELLA_E_INVALID, "%s: NULL descriptor", what);
  MambaDims x{};
  x.S = d->streams; x.T = d->tokens; x.H = d->heads; x.Dh = d->head_dim; x.G = d->groups; x.Ds = d->state_dim;
  x.K = d->conv_kernel;
  x.I = x.H * x.Dh;
  x.conv_dim = x.I + 2 * x.G * x.Ds;
  x.in_stride = d->in_stride;
  x.dt_min = d->dt_min; x.dt_max = d->dt_max; x.eps = d->eps;
  if (x.S < 1 || x.T < 1 || x.H < 1 || x.Dh < 1 || x.G < 1 || x.H % x.G || x.Ds < 32 || x.Ds % 32 ||
      x.Ds > 32 * kMaxStatePerLane || x.K < 1 || x.K > kMaxConvK || x.in_stride < x.I + x.conv_dim + x.H ||
      (d->dtype != VELLA_BF16 && d->dtype != VELLA_F16) || !(x.dt_min <= x.dt_max) || !(x.eps >= 0.0f))
    return fail(VELLA_E_INVALID, "%s: streams %d tokens %d heads %d head_dim %d groups %d state_dim %d (a multiple "
                "of 32 up to %d) conv_kernel %d (1..%d) in_stride %d", what, x.S, x.T, x.H, x.Dh, x.G, x.Ds,
                32 * kMaxStatePerLane, x.K, kMaxConvK, x.in_stride);
  *m = x;
  return VELLA_OK;
}

}  // namespace
}  // namespace vella

using namespace vella;

extern "C" {

int vella_mamba_conv(const vella_mamba_desc* desc, const void* zxbcdt, const void* conv_w, const void* conv_b,
                     void* conv_state, void* xbc, vella_stream_t stream) {
  MambaDims m;
  int rc = mamba_dims(desc, &m, "vella_mamba_conv");
  if (rc) return rc;
  if (!zxbcdt || !conv_w || !xbc || (m.K > 1 && !conv_state))
    return fail(VELLA_E_INVALID, "vella_mamba_conv: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == VELLA_BF16) return launch_conv<__nv_bfloat16>(m, zxbcdt, conv_w, conv_b, conv_state, xbc, s);
  return launch_conv<__half>(m, zxbcdt, conv_w, conv_b, conv_state, xbc, s);
}

int vella_mamba_ssm(const vella_mamba_desc* desc, const void* xbc, const void* zxbcdt, const float* a_log,
                    const float* dt_bias, const float* D, float* ssm_state, void* y, vella_stream_t stream) {
  MambaDims m;
  int rc = mamba_dims(desc, &m, "vella_mamba_ssm");
  if (rc) return rc;
  if (!xbc || !zxbcdt || !a_log || !dt_bias || !D || !ssm_state || !y)
    return fail(VELLA_E_INVALID, "vella_mamba_ssm: NULL pointer");
  const dim3 grid(m.H * ((m.Dh + 7) / 8), m.S), block(32, 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == VELLA_BF16)
    return launch_kernel(mamba_ssm_kernel<__nv_bfloat16>, grid, block, 0, s, m, static_cast<const __nv_bfloat16*>(xbc),
                         static_cast<const __nv_bfloat16*>(zxbcdt), a_log, dt_bias, D, ssm_state,
                         static_cast<__nv_bfloat16*>(y));
  return launch_kernel(mamba_ssm_kernel<__half>, grid, block, 0, s, m, static_cast<const __half*>(xbc),
                       static_cast<const __half*>(zxbcdt), a_log, dt_bias, D, ssm_state, static_cast<__half*>(y));
}

int vella_mamba_gated_norm(const vella_mamba_desc* desc, const void* y, const void* zxbcdt, const void* norm_w,
                           void* out, vella_stream_t stream) {
  MambaDims m;
  int rc = mamba_dims(desc, &m, "vella_mamba_gated_norm");
  if (rc) return rc;
  if (!y || !zxbcdt || !norm_w || !out) return fail(VELLA_E_INVALID, "vella_mamba_gated_norm: NULL pointer");
  if (m.I % m.G) return fail(VELLA_E_INVALID, "vella_mamba_gated_norm: %d channels in %d groups", m.I, m.G);
  const dim3 grid((unsigned)(m.S * m.T), m.G);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == VELLA_BF16)
    return launch_kernel(mamba_norm_kernel<__nv_bfloat16>, grid, dim3(kNormThreads), 0, s, m,
                         static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(zxbcdt),
                         static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(out));
  return launch_kernel(mamba_norm_kernel<__half>, grid, dim3(kNormThreads), 0, s, m, static_cast<const __half*>(y),
                       static_cast<const __half*>(zxbcdt), static_cast<const __half*>(norm_w),
                       static_cast<__half*>(out));
}

}  // extern "C"
