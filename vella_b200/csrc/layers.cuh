// Kernel launchers of the transformer decode step (layers.cu).  Host-only declarations.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace vella {

// Positions of the rows of a launch, read from device scalars so that captured graphs can
// be replayed while the sequences grow.  One stream (group == 0): row m sits at position
// *base + off + m.  Several streams in one launch (group = rows per stream): row m belongs
// to stream m / group and sits at base[(m / group) * stride] + off + m % group.
struct PosRef {
  const int* base;
  int off;
  int group = 0;
  int stride = 0;
  __host__ __device__ int stream_of(int m) const { return group ? m / group : 0; }
  __device__ int pos(int m) const { return group ? base[(m / group) * stride] + off + m % group : *base + off + m; }
};

// Tree-mode rows (tree verification and tree drafting): row m of a stream is node
// n = node0 + (m mod rows per stream) of that stream's draft tree, whose root sits at the
// PosRef position of the row's stream minus its row index (the tree's root slot R).  The node's
// token is tok[stream * nodes + n], its RoPE position R + dep[n] and its KV-cache slot R + n;
// it attends to every key below R and to the tree keys of its ancestors and itself
// (mask[n] bit j = node j).
struct TreeView {
  const int* tok = nullptr;
  const int* dep = nullptr;
  const unsigned long long* mask = nullptr;
  int nodes = 0;
  int node0 = 0;
};

// Half rotation of RoPE with one rounding order everywhere (the standalone kernel and the
// fused GEMM epilogue): y1 = x1 cos - x2 sin, y2 = x1 sin + x2 cos.
__device__ __forceinline__ float rope_rot1(float x1, float x2, float2 c) {
  return __fmaf_rn(x1, c.x, -__fmul_rn(x2, c.y));
}
__device__ __forceinline__ float rope_rot2(float x1, float x2, float2 c) {
  return __fmaf_rn(x1, c.y, __fmul_rn(x2, c.x));
}

// RoPE + KV-append epilogue of the q|k|v projection (head_dim 128, no q/k norm, no tree),
// fused into the small-M streaming GEMM: output rows of head h < H go to q [M][H][128]
// rotated, h < H + KV to the K cache at the row's position rotated, the rest to the V cache.
struct RopeEpi {
  const float2* cs = nullptr;  // [positions][64] (cos, sin)
  void* q = nullptr;
  void* kc = nullptr;          // layer's K cache of stream 0; stream s adds s * kv_ss elements
  void* vc = nullptr;
  PosRef pr{};
  int H = 0, KV = 0, max_seq = 0;
  long long kv_ss = 0;
  int* err = nullptr;          // bit 1: a position past the cache
};

// K/V-append epilogue of a q|k|v projection without RoPE (the Whisper decoder's), fused into
// the small-M streaming GEMM: output columns [d, 2d) of row m also go to the K cache
// [heads][S][hd] of the row's stream at position pr.pos(m), columns [2d, 3d) to the V
// cache (rows whose position lies outside [0, S) append nothing); `out` keeps all columns.
struct KvAppendEpi {
  void* kc = nullptr;  // the layer's K cache of stream 0; stream s adds s * kv_ss elements
  void* vc = nullptr;
  PosRef pr{};
  int d = 0, hd = 0, S = 0;
  long long kv_ss = 0;
};

// LayerNorm of a streaming GEMM's output rows (N <= 2048 columns, weight w and bias b of N
// elements) into `out`, run once the whole GEMM has finished by its last CTA to finish.
struct NormEpi {
  void* out = nullptr;
  const void* w = nullptr;
  const void* b = nullptr;
  float eps = 0.0f;
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
  const unsigned long long* tmask = nullptr;  // tree mode: ancestors-or-self mask per node
  int tnode0 = 0;                             // tree mode: node of row 0 of every batch
};

// dtype: 0 = bf16, 1 = fp16 everywhere below.
// Row m of stream s = pr.stream_of(m) holds position p = pr.pos(m): the stream's input
// embedding p (prefix + s * prefix_ss) when p < P[s * pr.stride], else the token table row
// of tok[s * tok_ss + p].
int launch_embed_rows_dev(int dtype, void* h, const void* table, const void* prefix, long long prefix_ss,
                          const int* tok, int tok_ss, PosRef pr, int rows, const int* P, int d, int vocab, int max_seq,
                          int* err, cudaStream_t s, TreeView tv = TreeView{});
// out row i = RMSNorm(x row src(i)), src(i) = (i / tail) * group + group - tail + i % tail:
// the last `tail` rows of every `group` rows (group == tail: every row).
int launch_rmsnorm(int dtype, void* out, const void* x, const void* w, int rows, int d, float eps,
                   cudaStream_t s, int group = 0, int tail = 0);
// RoPE of q/k and K/V append; stream s's cache starts kv_ss elements after stream 0's.
int launch_rope_append(int dtype, const void* qkv, void* q_out, void* kc, void* vc, const float2* cs,
                       const void* qn, const void* kn, float eps, PosRef pr, int rows, int H, int KV, int hd,
                       int max_seq, int* err, cudaStream_t s, long long kv_ss = 0, TreeView tv = TreeView{});
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
