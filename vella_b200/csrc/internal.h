// Host-side helpers shared by the library's translation units (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <string>
#include <utility>

#include "vella_cuda.h"

namespace vella {

// Per-thread message of the last failing call (vella_last_error).
std::string& last_error_slot();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  last_error_slot() = buf;
  return code;
}

inline int cuda_fail(cudaError_t e, const char* what) {
  return fail(VELLA_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define VELLA_CUDA_TRY(call)                                   \
  do {                                                         \
    cudaError_t e_ = (call);                                   \
    if (e_ != cudaSuccess) return ::vella::cuda_fail(e_, #call); \
  } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Epilogue parts of a VELLA_EPI_* code, applied in the order gate, bias, GELU, residual.
inline bool epi_valid(int e) { return e >= VELLA_EPI_NONE && e <= VELLA_EPI_BIAS_GELU_RESIDUAL; }
inline bool epi_bias(int e) {
  return e == VELLA_EPI_BIAS || e == VELLA_EPI_BIAS_RESIDUAL || e == VELLA_EPI_BIAS_GELU ||
         e == VELLA_EPI_BIAS_GELU_RESIDUAL;
}
inline bool epi_residual(int e) {
  return e == VELLA_EPI_RESIDUAL || e == VELLA_EPI_BIAS_RESIDUAL || e == VELLA_EPI_BIAS_GELU_RESIDUAL;
}
inline bool epi_gelu(int e) { return e == VELLA_EPI_BIAS_GELU || e == VELLA_EPI_BIAS_GELU_RESIDUAL; }

int num_sms(int device);

// Launch with programmatic stream serialization (the kernel overlaps the tail of the
// preceding kernel and calls griddepcontrol.wait before touching its results).  Set
// VELLA_PDL=0 to launch with plain stream order.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return VELLA_OK;
}

// Library-owned per-device workspace (vella_qgemm with workspace == NULL).  Grows on
// demand; the returned memory is zero-filled when first handed out.
int device_workspace(size_t bytes, void** out);

// ---- GEMM (qgemm.cu) -------------------------------------------------------------------
struct RopeEpi;      // layers.cuh
struct KvAppendEpi;  // layers.cuh
struct NormEpi;      // layers.cuh
struct QgemmPlan {
  int rows_out;   // output rows per CTA (128, or 64 with the SiLU gate)
  int rowblocks;  // ceil(N / rows_out)
  int kc;         // groups of 64 per CTA
  int splits;     // CTAs along K
  int zchunks;    // ceil(M / 16)
  size_t workspace;
  bool stream = false;  // persistent bulk-copy kernel (qgemm_stream.cu)
  int ctas = 0;         // its grid: one CTA per SM, or two for int4 calls with many units
  bool light = false;   // the compact 96-register, two-stage layout (int4): two fit one SM
  bool tc = false;      // tensor-core kernel for M > 16 (tc_gemm.cu)
};

// qgemm_stream.cu
bool stream_eligible(const vella_qgemm_desc& d);
int stream_units(const vella_qgemm_desc& d, int* rowblocks, int* nkc);
// True when an int4 call runs two CTAs per SM; depends on (N, K, format, SM count) only.
bool stream_light(const vella_qgemm_desc& d, int rowblocks, int nkc, int sms);
size_t stream_partial_bytes(int P);
int stream_flag_count(int P);  // ints of the flag region (zero between calls)
int stream_launch(const vella_qgemm_desc& d, int P, bool light, const void* x, const void* w, const void* scales,
                  const void* biases, const void* up_w, const void* up_scales, const void* up_biases,
                  const void* bias, const void* residual, void* out, int* flags, float* partial,
                  cudaStream_t stream, const RopeEpi* rope = nullptr, const KvAppendEpi* app = nullptr,
                  const NormEpi* norm = nullptr, int* done = nullptr);
int stream_fault_status(int clear);
int fwd_fault_status(int clear);  // fwd_prog.cu: the persistent decode forward's flags

// Bytes of a workspace's counter region (at least the fixed 128 KiB at its front) for
// `counters` ints; scratch follows it (qgemm.cu).
size_t counter_region(size_t counters);

// tc_gemm.cu
bool tc_eligible(const vella_qgemm_desc& d);
// K splits of a tensor-core call (a function of N, K and the call's row class only, so that a
// row's value does not depend on M within the class) and the workspace they need (zero for
// one split).
int tc_splits(const vella_qgemm_desc& d);
size_t tc_workspace(const vella_qgemm_desc& d, int splits);
int tc_launch(const vella_qgemm_desc& d, int splits, const void* x, const void* w, const void* scales,
              const void* biases, const void* up_w, const void* up_scales, const void* up_biases, const void* bias,
              const void* residual, void* out, void* ws, cudaStream_t stream);
int tc_fault_status(int clear);

bool qgemm_plan(const vella_qgemm_desc& d, QgemmPlan* plan);

// Small-M streaming plans only: rope, RoPE + KV append instead of writing `out`; app, the
// K/V append besides writing `out`; norm, LayerNorm of the output rows after the call.
int qgemm_launch(const vella_qgemm_desc& d, const QgemmPlan& plan, const void* x, const void* w,
                 const void* scales, const void* biases, const void* up_w, const void* up_scales,
                 const void* up_biases, const void* bias, const void* residual, void* out, void* ws,
                 cudaStream_t stream, const RopeEpi* rope = nullptr, const KvAppendEpi* app = nullptr,
                 const NormEpi* norm = nullptr);

// 2D tensor map over a row-major array of `rows` rows of `inner` elements (`row_bytes`
// apart), copied in boxes of box_inner x box_rows with the given swizzle; out-of-range
// elements read as zeros (tma.cu).
int make_tensor_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz);
// 3D: `planes` such arrays plane_bytes apart (the same tensor of every layer), boxes one plane
// deep.
int make_tensor_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                       uint64_t planes, uint64_t row_bytes, uint64_t plane_bytes, uint32_t box_inner, uint32_t box_rows,
                       CUtensorMapSwizzle swz);

// The RoPE table [max_seq][head_dim / 2] of (cos, sin) pairs: angle = pos * theta^(-2i/hd) in
// double, rounded once to fp32 (model.cu).
void rope_table(int max_seq, int head_dim, float theta, float* out);

// Whisper log-mel features of `streams` windows (audio window s at audio + s * audio_stride,
// n_samples long, padded or trimmed to 30 s) into out [streams][n_mels][3000] (audio.cu).
int launch_log_mel(const float* audio, int64_t audio_stride, int64_t n_samples, int streams, int n_mels, float* out,
                   cudaStream_t stream);

// After a checkpoint load: the encoder output and cross-attention K/V are stale until the
// next vella_whisper_encode (whisper.cu).
int whisper_weights_loaded(vella_whisper* w);

}  // namespace vella
