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
constexpr int kAttnQBlock = 8;   // query rows per cluster
constexpr int kAttnCluster = 8;  // CTAs per (kv head, query block); chunk c goes to CTA c % 8
constexpr int kAttnMaxGQ = 8;    // query heads per kv head

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
// ys[m] = first index of the row maximum of logits[m][0..V) (row stride ld); any NaN/Inf
// sets *nonfinite.  `part`/`counters` scratch from argmax_scratch_bytes.
size_t argmax_scratch_bytes(int max_rows);
int launch_argmax(int dtype, const void* logits, int rows, int V, size_t ld, int* ys, void* scratch,
                  int* nonfinite, cudaStream_t s);

}  // namespace vella
