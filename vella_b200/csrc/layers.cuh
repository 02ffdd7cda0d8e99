// Kernel launchers of the transformer decode step (layers.cu).  Host-only declarations.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace vella {

// Position of row 0 of a launch = *base + off (device scalar, so captured graphs can be
// replayed while the sequence grows).
struct PosRef {
  const int* base;
  int off;
};

constexpr int kAttnChunk = 64;   // keys per chunk (absolute-position aligned)
constexpr int kAttnRows = 64;    // query rows x query heads per cluster (query block = 64 / GQ rows)
constexpr int kAttnCluster = 8;  // CTAs per (kv head, query block); chunk c goes to CTA c % 8
constexpr int kAttnMaxGQ = 8;    // query heads per kv head

// Operands of an attention launch (element strides).  q/out rows hold the heads
// [H][hd] contiguously; K/V of kv head h, key row j at k + h * kv_hs + j * kv_rs; launch
// batch b adds b * {q,o,kv}_bs (independent streams).
struct AttnView {
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  void* out = nullptr;
  long long q_rs = 0, o_rs = 0;
  long long kv_hs = 0, kv_rs = 0;
  long long q_bs = 0, o_bs = 0, kv_bs = 0;
};

// dtype: 0 = bf16, 1 = fp16 everywhere below.
// Row m holds position p = *pr.base + pr.off + m: the caller's input embedding p when
// p < *P (device scalar), else the token table row tok[p].
int launch_embed_rows_dev(int dtype, void* h, const void* table, const void* prefix, const int* tok, PosRef pr,
                          int rows, const int* P, int d, int vocab, int max_seq, int* err, cudaStream_t s);
int launch_rmsnorm(int dtype, void* out, const void* x, const void* w, int rows, int d, float eps,
                   cudaStream_t s);
int launch_rope_append(int dtype, const void* qkv, void* q_out, void* kc, void* vc, const float2* cs,
                       const void* qn, const void* kn, float eps, PosRef pr, int rows, int H, int KV, int hd,
                       int max_seq, int* err, cudaStream_t s);
int launch_attention(int dtype, const void* q, const void* kc, const void* vc, void* out, PosRef pr, int rows,
                     int H, int KV, int hd, int max_seq, float scale, cudaStream_t s);
// General form: causal (query at position *pr.base + pr.off + m sees keys 0..that) or not
// (every query sees the S keys), strided operands, `batch` independent streams.
int launch_attention_ex(int dtype, const AttnView& v, int batch, PosRef pr, int causal, int rows, int H, int KV,
                        int hd, int S, float scale, cudaStream_t s);
// ys[m] = first index of the row maximum of logits[m][0..V) (row stride ld); any NaN/Inf
// sets *nonfinite.  `part`/`counters` scratch from argmax_scratch_bytes.
size_t argmax_scratch_bytes(int max_rows);
int launch_argmax(int dtype, const void* logits, int rows, int V, size_t ld, int* ys, void* scratch,
                  int* nonfinite, cudaStream_t s);

}  // namespace vella
