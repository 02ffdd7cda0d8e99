// Shared device helpers for the sm_100a kernels of the decode path.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "vella_cuda.h"

namespace vella {

// ---------------------------------------------------------------------------------------
// activation dtypes
// ---------------------------------------------------------------------------------------

template <typename T> struct Act;

template <> struct Act<__nv_bfloat16> {
  // 0x4300 is 128.0 in bf16: OR-ing a 4-bit code into the mantissa gives 128 + q exactly.
  static constexpr uint32_t kMagic2 = 0x43004300u;
  static constexpr float kMagic = 128.0f;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
};

template <> struct Act<__half> {
  // 0x6400 is 1024.0 in fp16: OR-ing a 4-bit code into the mantissa gives 1024 + q exactly.
  static constexpr uint32_t kMagic2 = 0x64006400u;
  static constexpr float kMagic = 1024.0f;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
};

// ---------------------------------------------------------------------------------------
// tensor core: m16n8k16, fp32 accumulate (legacy warp-level MMA; used where M <= 16 and the
// kernel is bound by HBM, not by the tensor pipe)
// ---------------------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (a & m) | c in one instruction.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(c));
  return r;
}

// ---------------------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------------------

// Weight stream: read once, never reused by this CTA -> bypass L1, ask L2 for 256-byte fills.
__device__ __forceinline__ uint2 ld_stream2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Programmatic dependent launch: wait until the preceding kernel of the stream has finished
// and its writes are visible (a no-op when launched without the attribute), and let the
// next kernel start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// GELU, erf form: 0.5 x (1 + erf(x / sqrt(2))) (MLX's default gelu).
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

constexpr int kLnMaxD = 2048;  // LayerNorm row length limit (8 values per thread)

// LayerNorm of one row of D <= kLnMaxD values by 256 threads t = 0..255 (value i on thread
// i % 256): fp32 mean and centred variance, x_hat rounded to T, then T(w * x_hat + b)
// (WhisperFusedDecode.swift:204-251 row algorithm, one final rounding).  The row is read
// with L2 loads (it may have been written by other CTAs of the same kernel); `sync` is the
// 256 threads' barrier and `red` 8 floats of shared memory.  Every caller runs this same
// sequence, so a row's result does not depend on which kernel normalises it.
template <typename T, typename Sync>
__device__ __forceinline__ void ln_row256(T* __restrict__ orow, const T* xr, const T* __restrict__ w,
                                          const T* __restrict__ b, int D, float eps, int t, float* red, Sync sync) {
  using A = Act<T>;
  const int warp = t >> 5, lane = t & 31;
  auto bsum = [&](float v) {
    v = warp_sum(v);
    sync();
    if (lane == 0) red[warp] = v;
    sync();
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k];
    return s;
  };
  float v[kLnMaxD / 256];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < kLnMaxD / 256; ++j) {
    const int i = t + 256 * j;
    v[j] = i < D ? A::to_f(__ldcg(xr + i)) : 0.0f;
    s += v[j];
  }
  const float mean = bsum(s) / (float)D;
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kLnMaxD / 256; ++j) {
    const int i = t + 256 * j;
    if (i < D) {
      v[j] -= mean;
      ss = fmaf(v[j], v[j], ss);
    }
  }
  const float r = sqrtf(bsum(ss) / (float)D + eps);
#pragma unroll
  for (int j = 0; j < kLnMaxD / 256; ++j) {
    const int i = t + 256 * j;
    if (i < D) {
      const float xh = A::to_f(A::from_f(v[j] / r));
      orow[i] = A::from_f(fmaf(A::to_f(w[i]), xh, A::to_f(b[i])));
    }
  }
}

}  // namespace vella
