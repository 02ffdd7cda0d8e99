// vella_qgemm_noalloc: the small-M GEMM for callers that cannot allocate device memory.
//
// Some hosts of this library must not call cudaMalloc themselves or have it called on
// their behalf: code that runs while a CUDA graph is being captured, a real-time audio
// thread that cannot block on the device synchronisation an allocation may imply, or an
// embedder whose device memory is owned by another allocator under a fixed budget.  For
// them this entry point takes the split-K scratch of the GEMM from one file-scope device
// array of kNoAllocScratchBytes (32 MiB) instead of a workspace argument or the library's
// growable workspace.  Every GPU that loads the library holds that array until exit.
//
// The array's name in host code is only a host-side stand-in: its device address is
// looked up with cudaGetSymbolAddress once per device, with that device current, on the
// first call made on that device.  That first call also clears the array and waits for
// the clear on its stream, so it should come before any stream capture.  All calls share
// the one array and each leaves its ticket counters at zero; calls that overlap on the
// GPU (different streams, or concurrent graphs) race on it and must be serialised by the
// caller.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"
#include "vella_cuda.h"

namespace vella {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the static scratch on the current device (set-up on first use).
int noalloc_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "vella_qgemm_noalloc: cudaGetSymbolAddress");
    VELLA_CUDA_TRY(cudaMemsetAsync(p, 0, kNoAllocScratchBytes, stream));
    VELLA_CUDA_TRY(cudaStreamSynchronize(stream));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return VELLA_OK;
}

}  // namespace
}  // namespace vella

using namespace vella;

extern "C" int vella_qgemm_noalloc(const vella_qgemm_desc* desc, const void* x, const void* w, const void* scales,
                                   const void* biases, const void* up_w, const void* up_scales,
                                   const void* up_biases, const void* bias, const void* residual, void* out,
                                   vella_stream_t stream) {
  last_error_slot().clear();
  if (!desc) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: desc is NULL");
  const vella_qgemm_desc& d = *desc;
  QgemmPlan plan;
  if (!qgemm_plan(d, &plan))
    return fail(VELLA_E_UNSUPPORTED, "vella_qgemm_noalloc: unsupported call (m=%d n=%d k=%d bits=%d group=%d dtype=%d epilogue=%d)",
                d.m, d.n, d.k, d.bits, d.group_size, d.dtype, d.epilogue);
  if (plan.workspace > kNoAllocScratchBytes)
    return fail(VELLA_E_INVALID,
                "vella_qgemm_noalloc: this shape needs %zu bytes of scratch, more than the %zu-byte static array "
                "(m=%d n=%d k=%d); use vella_qgemm with a workspace",
                plan.workspace, kNoAllocScratchBytes, d.m, d.n, d.k);
  if (d.m == 0 || d.n == 0) return VELLA_OK;
  const bool quant = d.bits != 0;
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  const bool has_bias = epi_bias(d.epilogue);
  const bool has_res = epi_residual(d.epilogue);
  if (!x || !w || !out) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: x, w and out must be non-NULL");
  if (quant && (!scales || !biases))
    return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: scales and biases are required for bits=%d", d.bits);
  if (gate && (!up_w || (quant && (!up_scales || !up_biases))))
    return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: the SiLU gate needs the up projection");
  if (has_bias && !bias) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: bias is NULL");
  if (has_res && !residual) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: residual is NULL");
  if (!aligned(x, 16)) return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: x must be 16-byte aligned");
  if (!aligned(w, 16) || (gate && !aligned(up_w, 16)))
    return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: weights must be 16-byte aligned");
  if (!aligned(out, 2) || (has_bias && !aligned(bias, 2)) || (has_res && !aligned(residual, 2)) ||
      (quant && (!aligned(scales, 2) || !aligned(biases, 2))))
    return fail(VELLA_E_INVALID, "vella_qgemm_noalloc: 16-bit operands must be 2-byte aligned");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the set-up runs on every call, whether or not this shape's plan uses the scratch, so the
  // first call on a device (whatever its shape) is the one that looks the array up and clears it
  void* scratch = nullptr;
  const int rc = noalloc_scratch(s, &scratch);
  if (rc != VELLA_OK) return rc;
  void* ws = plan.workspace ? scratch : nullptr;
  return qgemm_launch(d, plan, x, w, scales, biases, up_w, up_scales, up_biases, bias, residual, out, ws, s);
}
