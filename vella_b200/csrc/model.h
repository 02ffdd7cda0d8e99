// Dense GQA transformer (Qwen3-style recipe) resident on one GPU: weights, KV cache,
// activation buffers and the decode-step forward.  Internal C++ API behind vella_model_*.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "internal.h"
#include "layers.cuh"
#include "vella_cuda.h"

namespace vella {

constexpr int kMaxRows = 16;     // rows per decode forward and per logits launch
constexpr int kChunkRows = 256;  // rows per prefill forward (tensor-core GEMMs above 16 rows)

struct QWeight {
  void* w = nullptr;  // packed uint32 [N, K*bits/32] or dense [N, K]
  void* s = nullptr;  // scales [N, K/64]
  void* b = nullptr;  // biases [N, K/64]
  int n = 0, k = 0;
  size_t w_bytes = 0, sb_bytes = 0;
};

struct Layer {
  void* attn_norm = nullptr;
  void* mlp_norm = nullptr;
  void* q_norm = nullptr;
  void* k_norm = nullptr;
  QWeight qkv, o, gate, up, down;
};

struct FwdProg;  // fwd_prog.cu: the persistent decode forward's program of a model

struct Model {
  vella_model_cfg cfg{};
  int device = 0;
  int elt = 2;  // bytes per activation element
  // weights
  void* arena = nullptr;
  size_t arena_bytes = 0;
  void* embed = nullptr;       // [V, d]
  void* final_norm = nullptr;  // [d]
  QWeight lm_head;             // [V, d]
  std::vector<Layer> layers;
  // per-sequence state (streams = max(1, cfg.streams) independent sequences)
  int streams = 1;
  void* kv = nullptr;  // [streams][L][2][KV][max_seq][hd]
  size_t kv_bytes = 0;
  long long kv_ss = 0;      // elements between consecutive streams' caches
  void* prefix = nullptr;  // [streams][max_prefix][d]
  long long prefix_ss = 0;  // elements between consecutive streams' prefixes
  int rps = kMaxRows;       // decode rows per stream (cfg.rows_per_stream, default kMaxRows)
  int max_rows = 0;         // rows of the activation buffers (max(kChunkRows, streams * rps))
  float2* rope = nullptr;  // [S][hd/2] (cos, sin)
  // activations and scratch
  void* act_arena = nullptr;
  void *h = nullptr, *xn = nullptr, *qkv_out = nullptr, *q = nullptr, *attn = nullptr, *mlp = nullptr;
  void* logits = nullptr;  // [streams * rps, V]
  int* ys = nullptr;       // [streams * rps]
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  void* argmax_sc = nullptr;
  int* err = nullptr;        // bit flags set by kernels (bad token, bad position)
  int* nonfinite = nullptr;  // set by argmax over logits
  int* dzero = nullptr;      // device 0 (position base of prefill chunks)
  int* score_tok = nullptr;  // [max_seq] token ids of vella_model_score
  int* score_P = nullptr;    // prefix length of vella_model_score
  cudaStream_t stream = nullptr;  // stream of the model-level calls (init, score)
  FwdProg* prog = nullptr;        // persistent decode forward (null: the model's shapes do not suit it)
  bool persistent = false;        // decode-sized forwards run the persistent kernel (needs prog)

  void* kcache(int l) const;
  void* vcache(int l) const;
  int qkv_n() const { return (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim; }
};

int model_create(const vella_model_cfg& cfg, int device, Model** out);
int fill_normal(void* out, size_t n, int dtype, uint64_t seed, uint32_t tensor, float mean, float std, cudaStream_t s);
// Random MLX-affine weights: each group drawn ~N(0, std) and quantized on the device.
int quantize_random(const QWeight& w, int bits, int dtype, uint64_t seed, uint32_t tensor, float std, cudaStream_t s);
int quantize_device(int src_dtype, const void* w, int dtype, int bits, int N, int K, void* packed, void* scales,
                    void* biases, cudaStream_t s);
void model_destroy(Model* m);
int model_init_random(Model* m, uint64_t seed, float std, cudaStream_t s);
int model_tensor(Model* m, const std::string& name, int layer, void** ptr, size_t* bytes);

// Runs `rows` positions of each of `streams` streams (stream0, stream0 + 1, ...) through every
// layer in one batch of rows * streams rows, appending their K/V to each stream's cache.
// Stream j's rows start at pr.base[j * pr.stride] + pr.off (pr.base, tok and P point at
// stream0's values; tok advances tok_ss ints per stream, P pr.stride ints).  Token ids come
// from tok (pos >= P) or the stream's prefix embeddings (pos < P).  When logits_rows > 0 the
// last `logits_rows` rows of every stream go through the final norm and the LM head into
// m->logits (stream-major) and their argmax into m->ys.
// With `tree`, the rows are tree nodes (TreeView): pr then gives each stream's root slot.
int model_forward(Model* m, PosRef pr, int rows, int streams, int stream0, const int* tok, int tok_ss, const int* P,
                  int logits_rows, cudaStream_t s, const TreeView* tree = nullptr);

// Persistent decode forward (fwd_prog.cu): one cooperative launch per forward of at most 16
// rows, bit-identical to the per-op kernels.  fwd_prog_run expects the rows' embeddings in m->h
// and leaves the logits of the last logits_rows rows of every stream in m->logits.
bool fwd_prog_model_ok(const Model* m);
int fwd_prog_build(Model* m, FwdProg** out);
void fwd_prog_destroy(FwdProg* p);
int fwd_prog_run(Model* m, FwdProg* p, PosRef pr, int rows, int streams, int stream0, int logits_rows, cudaStream_t s);
int fwd_fault_status(int clear);

// GEMM with the model's workspace (rope: the streaming kernel's RoPE + KV-append epilogue).
int model_gemm(Model* m, const QWeight& w, const void* x, int rows, void* out, int epilogue, const void* residual,
               const QWeight* up, cudaStream_t s, const RopeEpi* rope = nullptr);

}  // namespace vella
