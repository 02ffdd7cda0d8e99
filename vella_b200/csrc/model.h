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
  // per-sequence state
  void* kv = nullptr;  // [L][2][KV][S][hd]
  size_t kv_bytes = 0;
  void* prefix = nullptr;  // [max_prefix][d]
  float2* rope = nullptr;  // [S][hd/2] (cos, sin)
  // activations and scratch
  void* act_arena = nullptr;
  void *h = nullptr, *xn = nullptr, *qkv_out = nullptr, *q = nullptr, *attn = nullptr, *mlp = nullptr;
  void* logits = nullptr;  // [kMaxRows, V]
  int* ys = nullptr;       // [kMaxRows]
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  void* argmax_sc = nullptr;
  int* err = nullptr;        // bit flags set by kernels (bad token, bad position)
  int* nonfinite = nullptr;  // set by argmax over logits
  int* dzero = nullptr;      // device 0 (position base of prefill chunks)
  int* score_tok = nullptr;  // [max_seq] token ids of vella_model_score
  int* score_P = nullptr;    // prefix length of vella_model_score
  cudaStream_t stream = nullptr;  // stream of the model-level calls (init, score)

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

// Runs `rows` (<= kMaxRows) positions starting at *pr.base + pr.off through every layer,
// appending their K/V.  Token ids come from tok[pos] (pos >= *P) or the prefix embeddings
// (pos < *P).  When logits_rows > 0 the last `logits_rows` rows go through the final norm
// and the LM head into m->logits[0..logits_rows) and their argmax into m->ys.
int model_forward(Model* m, PosRef pr, int rows, const int* tok, const int* P, int logits_rows, cudaStream_t s);

// GEMM with the model's workspace.
int model_gemm(Model* m, const QWeight& w, const void* x, int rows, void* out, int epilogue, const void* residual,
               const QWeight* up, cudaStream_t s);

}  // namespace vella
