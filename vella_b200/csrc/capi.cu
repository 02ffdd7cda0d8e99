// extern "C" entry points of the GEMM boundary, argument checks, error reporting and
// the library-owned per-device workspace.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "vella_cuda.h"

namespace vella {

std::string& last_error_slot() {
  static thread_local std::string msg;
  return msg;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VELLA_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int num_sms(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) return 148;
  if ((int)cache.size() <= device) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cache[device] = v;
  }
  return cache[device];
}

namespace {
struct DeviceWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  // Buffers replaced by a larger one.  They are never freed: a CUDA graph captured with an
  // earlier call still holds their address and must stay valid when it is replayed.
  std::vector<void*> retired;
};
std::mutex g_ws_mu;
std::vector<DeviceWorkspace> g_ws;
}  // namespace

int device_workspace(size_t bytes, void** out) {
  int dev = 0;
  VELLA_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_ws_mu);
  if ((int)g_ws.size() <= dev) g_ws.resize(dev + 1);
  DeviceWorkspace& ws = g_ws[dev];
  if (ws.bytes < bytes) {
    size_t want = std::max(bytes, ws.bytes * 2);
    want = std::max<size_t>(want, 1 << 20);
    if (ws.ptr) {
      ws.retired.push_back(ws.ptr);
      ws.ptr = nullptr;
      ws.bytes = 0;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
      cudaGetLastError();
      return fail(VELLA_E_OOM, "workspace allocation of %zu bytes failed", want);
    }
    // zeroed before any stream uses it (callers' streams may be non-blocking)
    VELLA_CUDA_TRY(cudaMemset(p, 0, want));
    VELLA_CUDA_TRY(cudaDeviceSynchronize());
    ws.ptr = p;
    ws.bytes = want;
  }
  *out = ws.ptr;
  return VELLA_OK;
}

}  // namespace vella

using namespace vella;

extern "C" {

size_t vella_last_error(char* buf, size_t cap) {
  const std::string& m = last_error_slot();
  if (buf && cap) {
    const size_t n = std::min(cap - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = 0;
  }
  return m.size();
}

int32_t vella_fault_flags(int32_t clear) {
  const int st = stream_fault_status(clear);
  const int tc = tc_fault_status(clear);
  const int fw = fwd_fault_status(clear);
  if (st < 0 || tc < 0 || fw < 0) return -1;
  return (st & 0xFF) | ((tc & 0xFF) << 8) | ((fw & 0xFF) << 16);
}

const char* vella_version(void) { return "vella-b200 0.1 sm_100a"; }

int vella_qgemm_supports(const vella_qgemm_desc* desc) {
  if (!desc) return 0;
  QgemmPlan p;
  return qgemm_plan(*desc, &p) ? 1 : 0;
}

size_t vella_qgemm_workspace_size(const vella_qgemm_desc* desc) {
  if (!desc) return 0;
  QgemmPlan p;
  if (!qgemm_plan(*desc, &p)) return 0;
  return p.workspace;
}

int vella_qgemm(const vella_qgemm_desc* desc, const void* x, const void* w, const void* scales,
                const void* biases, const void* up_w, const void* up_scales, const void* up_biases,
                const void* bias, const void* residual, void* out, void* workspace, size_t workspace_bytes,
                vella_stream_t stream) {
  last_error_slot().clear();
  if (!desc) return fail(VELLA_E_INVALID, "vella_qgemm: desc is NULL");
  const vella_qgemm_desc& d = *desc;
  QgemmPlan plan;
  if (!qgemm_plan(d, &plan))
    return fail(VELLA_E_UNSUPPORTED, "vella_qgemm: unsupported call (m=%d n=%d k=%d bits=%d group=%d dtype=%d epilogue=%d)",
                d.m, d.n, d.k, d.bits, d.group_size, d.dtype, d.epilogue);
  if (d.m == 0 || d.n == 0) return VELLA_OK;
  const bool quant = d.bits != 0;
  const bool gate = d.epilogue == VELLA_EPI_SILU_GATE;
  const bool has_bias = epi_bias(d.epilogue);
  const bool has_res = epi_residual(d.epilogue);
  if (!x || !w || !out) return fail(VELLA_E_INVALID, "vella_qgemm: x, w and out must be non-NULL");
  if (quant && (!scales || !biases)) return fail(VELLA_E_INVALID, "vella_qgemm: scales and biases are required for bits=%d", d.bits);
  if (gate && (!up_w || (quant && (!up_scales || !up_biases))))
    return fail(VELLA_E_INVALID, "vella_qgemm: the SiLU gate needs the up projection");
  if (has_bias && !bias) return fail(VELLA_E_INVALID, "vella_qgemm: bias is NULL");
  if (has_res && !residual) return fail(VELLA_E_INVALID, "vella_qgemm: residual is NULL");
  if (!aligned(x, 16)) return fail(VELLA_E_INVALID, "vella_qgemm: x must be 16-byte aligned");
  if (!aligned(w, 16) || (gate && !aligned(up_w, 16))) return fail(VELLA_E_INVALID, "vella_qgemm: weights must be 16-byte aligned");
  if (!aligned(out, 2) || (has_bias && !aligned(bias, 2)) || (has_res && !aligned(residual, 2)) ||
      (quant && (!aligned(scales, 2) || !aligned(biases, 2))))
    return fail(VELLA_E_INVALID, "vella_qgemm: 16-bit operands must be 2-byte aligned");
  void* ws = nullptr;
  if (plan.workspace) {
    if (workspace) {
      if (workspace_bytes < plan.workspace)
        return fail(VELLA_E_INVALID, "vella_qgemm: workspace of %zu bytes is smaller than the %zu required",
                    workspace_bytes, plan.workspace);
      if (!aligned(workspace, 256)) return fail(VELLA_E_INVALID, "vella_qgemm: workspace must be 256-byte aligned");
      ws = workspace;
    } else {
      const int rc = device_workspace(plan.workspace, &ws);
      if (rc != VELLA_OK) return rc;
    }
  }
  return qgemm_launch(d, plan, x, w, scales, biases, up_w, up_scales, up_biases, bias, residual, out, ws,
                      static_cast<cudaStream_t>(stream));
}

}  // extern "C"
