/*
 * vella_cuda.h — C ABI of the B200 (sm_100a) decode path: MLX-affine int4/int8 small-M
 * dequant GEMM, the draft-and-verify decode loop and the fused Whisper decoder step.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and returns a status
 * code.  Device pointers are caller-owned CUDA device memory on the current device;
 * `vella_stream_t` is a `cudaStream_t` (NULL = the legacy default stream).  Calls are
 * asynchronous on the stream unless stated otherwise.  On any status other than VELLA_OK
 * `vella_last_error` returns a message for the calling thread.
 *
 * Reference interfaces replaced (paths inside the Vella repository):
 *   vella_qgemm / vella_qgemm_supports
 *       SmallMGEMM.matmul(_:_:epilogue:native:) -> MLXArray?   Worker/Sources/SmallMGEMM/SmallMGEMM.swift:126
 *       SmallMGEMM.supports(m:n:k:dtype:format:epilogue:native:) SmallMGEMM.swift:113
 *       (VELLA_E_UNSUPPORTED plays the role of the `nil` return: the caller keeps its own path)
 *   vella_spec_*  NemotronTranscribeModel.decodeMTP / decodeGreedy / decode
 *       Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeModel.swift:266-443
 *   vella_whisper_*  WhisperFusedDecoder.step, WhisperModel.pipelinedGreedy
 *       Worker/Sources/MLXAudioSTT/Whisper/WhisperFusedDecode.swift:105-141,
 *       Worker/Sources/MLXAudioSTT/Whisper/WhisperModel.swift:341-400
 */
#ifndef VELLA_CUDA_H
#define VELLA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VELLA_API __attribute__((visibility("default")))
#else
#define VELLA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* vella_stream_t; /* cudaStream_t */

/* ---- status codes ------------------------------------------------------------------- */
enum {
  VELLA_OK = 0,
  VELLA_E_UNSUPPORTED = 1, /* shape/format not handled: the caller uses its own path     */
  VELLA_E_INVALID = 2,     /* bad argument (null pointer, misaligned, inconsistent sizes) */
  VELLA_E_CUDA = 3,        /* a CUDA runtime call failed                                  */
  VELLA_E_NONFINITE = 4,   /* a verify pass produced NaN/Inf logits                       */
  VELLA_E_OOM = 5          /* device allocation failed                                    */
};

/* ---- element types ------------------------------------------------------------------ */
enum { VELLA_BF16 = 0, VELLA_F16 = 1 };

/* ---- GEMM epilogues (reference SmallMGEMM.EpilogueKind, SmallMGEMM.swift:41) --------- */
enum {
  VELLA_EPI_NONE = 0,
  VELLA_EPI_BIAS = 1,          /* + bias[n]                                               */
  VELLA_EPI_RESIDUAL = 2,      /* + residual[m, n]                                        */
  VELLA_EPI_BIAS_RESIDUAL = 3, /* + bias[n] + residual[m, n]                              */
  VELLA_EPI_SILU_GATE = 4      /* silu(x . Wg^T) * (x . Wu^T); W = gate, `up_*` = up      */
};

/*
 * out[M, N] = epilogue(x[M, K] . W^T), fp32 accumulation, one rounding to `dtype`.
 *   bits = 0     W is dense [N, K] in `dtype` (scales/biases unused).
 *   bits = 4 | 8 W is MLX-affine: packed uint32 [N, K*bits/32] (element i of a word at bits
 *                [bits*i, bits*(i+1)), low first), scales and biases [N, K/64] in `dtype`,
 *                element = scale * q + bias; accumulated in the product form
 *                sum_g (scale * sum(x*q) + bias * sum(x)) as SmallMGEMM.swift:724.
 * group_size must be 64 when bits != 0.  x, residual, out are row-major with row stride K
 * (x) or N (residual, out).
 */
typedef struct vella_qgemm_desc {
  int32_t m, n, k;
  int32_t bits;       /* 0, 4 or 8 */
  int32_t group_size; /* 64        */
  int32_t dtype;      /* VELLA_BF16 | VELLA_F16 */
  int32_t epilogue;   /* VELLA_EPI_* */
} vella_qgemm_desc;

/* Pure query: 1 when vella_qgemm runs this call, else 0 (no device work). */
VELLA_API int vella_qgemm_supports(const vella_qgemm_desc* desc);

/* Bytes of workspace vella_qgemm needs for this shape (0 when none). */
VELLA_API size_t vella_qgemm_workspace_size(const vella_qgemm_desc* desc);

/*
 * Runs the GEMM.  `up_w/up_scales/up_biases` are read only for VELLA_EPI_SILU_GATE,
 * `bias` only for the bias epilogues, `residual` only for the residual epilogues.
 * `workspace`: device memory of at least vella_qgemm_workspace_size bytes, 256-byte
 * aligned, zero-filled before its first use (every completed call leaves its counter words
 * zero again), used by one stream at a time.  NULL selects a per-device workspace owned
 * by the library: it is allocated or grown by the first call that needs more, so that
 * call must not be inside CUDA graph capture; a grown workspace keeps the old buffer
 * alive, so graphs captured earlier stay valid, but they all share one buffer and must
 * not run concurrently.
 * The reduction order of a row depends only on (N, K, bits): a row of a batched call is
 * bit-identical to the same row computed alone.
 */
VELLA_API int vella_qgemm(const vella_qgemm_desc* desc, const void* x, const void* w, const void* scales,
                const void* biases, const void* up_w, const void* up_scales, const void* up_biases,
                const void* bias, const void* residual, void* out, void* workspace,
                size_t workspace_bytes, vella_stream_t stream);

/*
 * vella_qgemm without any device allocation, for callers that cannot allocate: code that
 * runs during CUDA graph capture, a real-time audio thread that must not block on an
 * allocation, or an embedder whose device memory belongs to another allocator.  It has no
 * counterpart in the reference (MLX allocates for its caller).  Same arguments and result
 * as vella_qgemm minus the workspace: the split-K scratch is one static device array of
 * 32 MiB inside the library, held by every GPU that loads the library until exit.  A
 * shape whose scratch (vella_qgemm_workspace_size) exceeds 32 MiB is rejected with
 * VELLA_E_INVALID.  The first call on a device looks the array up and clears it, waiting
 * on `stream`, so make it before any stream capture.  All calls share the array: calls
 * that overlap on the GPU race and must be serialised by the caller.
 */
VELLA_API int vella_qgemm_noalloc(const vella_qgemm_desc* desc, const void* x, const void* w, const void* scales,
                                  const void* biases, const void* up_w, const void* up_scales,
                                  const void* up_biases, const void* bias, const void* residual, void* out,
                                  vella_stream_t stream);

/* Message of the last failing call on this thread ("" when none); returns its length. */
VELLA_API size_t vella_last_error(char* buf, size_t cap);

/* Library version string, e.g. "vella-b200 0.1 sm_100a". */
VELLA_API const char* vella_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VELLA_CUDA_H */
