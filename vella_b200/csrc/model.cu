// Dense GQA transformer resident on one GPU (weights, KV cache, buffers) and its decode
// forward over the layer kernels; synthetic weight initialisation and the MLX-affine
// quantizer on the device.
//
// Layer recipe (reference Worker/Sources/MLXAudioSTT/Qwen3ASR/Qwen3ASRTextDecoder.swift:
// 124-149): h += o_proj(attn(rope(q), rope(k), v)) over input_layernorm(h), then
// h += down(silu(gate(x)) * up(x)) over post_attention_layernorm(h); final RMSNorm, LM head.
// q|k|v share one GEMM (rows concatenated, as WhisperFusedDecode.swift:67-88 fuses them),
// the SwiGLU product is the GEMM's SiLU-gate epilogue, both residual adds are GEMM
// epilogues writing the residual stream in place.
//
// Quantizer: MLX's affine quantize, restated (third-party mlx, pinned through mlx-swift
// 901941965d82e4a216d4d117231d847d194c563d): per group of 64, scale = max((max-min)/n_bins,
// 1e-7) signed toward the larger-magnitude edge, the edge snapped to an integer code, codes
// = clip(round((w - bias)/scale), 0, n_bins) with the fp32 scale and bias, which are then
// stored in the activation dtype (reference call sites NemotronTranscribeRecipe.swift:48,
// DerivedPrecision.swift:146).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"
#include "model.h"
#include "philox.h"

namespace vella {
namespace {

__device__ __forceinline__ float round_half_away(float x) { return copysignf(floorf(fabsf(x) + 0.5f), x); }

// 4 normals from one Philox block (Box-Muller).
__device__ __forceinline__ void normal4(uint64_t seed, uint32_t tensor, uint64_t ctr, float (&z)[4]) {
  const U4 r = philox4x32_10(U4{(uint32_t)ctr, (uint32_t)(ctr >> 32), tensor, 0x51EDu}, (uint32_t)seed,
                             (uint32_t)(seed >> 32));
  const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float u1 = ((u[2 * p] >> 8) + 1u) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = (u[2 * p + 1] >> 8) * (1.0f / 16777216.0f);      // [0, 1)
    const float rad = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    z[2 * p] = rad * cs;
    z[2 * p + 1] = rad * sn;
  }
}

template <typename T> __device__ __forceinline__ T cvt_from(float v) { return Act<T>::from_f(v); }
template <> __device__ __forceinline__ float cvt_from<float>(float v) { return v; }
template <typename T> __device__ __forceinline__ float cvt_to(T v) { return Act<T>::to_f(v); }
template <> __device__ __forceinline__ float cvt_to<float>(float v) { return v; }

// One group of 64 values -> packed codes, scale, bias (MLX affine).
template <typename T, int BITS>
__device__ void quantize_group(const float (&v)[64], uint32_t* packed, T* s_out, T* b_out) {
  float wmax = v[0], wmin = v[0];
#pragma unroll
  for (int i = 1; i < 64; ++i) { wmax = fmaxf(wmax, v[i]); wmin = fminf(wmin, v[i]); }
  const float n_bins = (float)((1 << BITS) - 1);
  float scale = fmaxf(__fdiv_rn(wmax - wmin, n_bins), 1e-7f);
  const bool side = fabsf(wmin) > fabsf(wmax);
  scale = side ? scale : -scale;
  const float edge = side ? wmin : wmax;
  const float q0 = round_half_away(__fdiv_rn(edge, scale));
  const bool at_zero = q0 == 0.0f;
  scale = at_zero ? scale : __fdiv_rn(edge, q0);
  const float bias = at_zero ? 0.0f : edge;
  constexpr int PER = 32 / BITS;
#pragma unroll
  for (int wd = 0; wd < 64 / PER; ++wd) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      float c = round_half_away(__fdiv_rn(__fsub_rn(v[wd * PER + j], bias), scale));
      c = fminf(fmaxf(c, 0.0f), n_bins);
      word |= (uint32_t)c << (BITS * j);
    }
    packed[wd] = word;
  }
  *s_out = Act<T>::from_f(scale);
  *b_out = Act<T>::from_f(bias);
}

template <typename T, int BITS>
__global__ void init_quant_kernel(uint32_t* packed, T* scales, T* biases, int N, int K, uint64_t seed,
                                  uint32_t tensor, float mean, float std) {
  const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int G = K / 64;
  if (gid >= (size_t)N * G) return;
  float v[64];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float z[4];
    normal4(seed, tensor, gid * 16 + i, z);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[4 * i + j] = fmaf(z[j], std, mean);
  }
  quantize_group<T, BITS>(v, packed + gid * (64 * BITS / 32), scales + gid, biases + gid);
}

template <typename Tin, typename T, int BITS>
__global__ void quantize_kernel(const Tin* w, uint32_t* packed, T* scales, T* biases, int N, int K) {
  const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int G = K / 64;
  if (gid >= (size_t)N * G) return;
  float v[64];
  const Tin* src = w + gid * 64;
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = cvt_to<Tin>(src[i]);
  quantize_group<T, BITS>(v, packed + gid * (64 * BITS / 32), scales + gid, biases + gid);
}

template <typename T>
__global__ void init_dense_kernel(T* out, size_t n, uint64_t seed, uint32_t tensor, float mean, float std) {
  const size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q * 4 >= n) return;
  float z[4];
  normal4(seed, tensor, q, z);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (q * 4 + j < n) out[q * 4 + j] = cvt_from<T>(fmaf(z[j], std, mean));
}

size_t up256(size_t b) { return (b + 255) / 256 * 256; }

template <typename T>
int fill_normal_t(void* out, size_t n, uint64_t seed, uint32_t tensor, float mean, float std, cudaStream_t s) {
  const size_t q = (n + 3) / 4;
  init_dense_kernel<T><<<(unsigned)((q + 255) / 256), 256, 0, s>>>(static_cast<T*>(out), n, seed, tensor, mean, std);
  VELLA_CUDA_TRY(cudaGetLastError());
  return VELLA_OK;
}

}  // namespace

int fill_normal(void* out, size_t n, int dtype, uint64_t seed, uint32_t tensor, float mean, float std,
                cudaStream_t s) {
  if (n == 0) return VELLA_OK;
  switch (dtype) {
    case VELLA_BF16: return fill_normal_t<__nv_bfloat16>(out, n, seed, tensor, mean, std, s);
    case VELLA_F16: return fill_normal_t<__half>(out, n, seed, tensor, mean, std, s);
    case VELLA_F32: return fill_normal_t<float>(out, n, seed, tensor, mean, std, s);
  }
  return fail(VELLA_E_INVALID, "fill_normal: dtype %d", dtype);
}

int quantize_random(const QWeight& w, int bits, int dtype, uint64_t seed, uint32_t tensor, float std, cudaStream_t s) {
  const size_t groups = (size_t)w.n * (w.k / 64);
  const unsigned blocks = (unsigned)((groups + 127) / 128);
  auto* p = static_cast<uint32_t*>(w.w);
  if (dtype == VELLA_BF16) {
    auto* sc = static_cast<__nv_bfloat16*>(w.s);
    auto* bi = static_cast<__nv_bfloat16*>(w.b);
    if (bits == 4) init_quant_kernel<__nv_bfloat16, 4><<<blocks, 128, 0, s>>>(p, sc, bi, w.n, w.k, seed, tensor, 0.0f, std);
    else init_quant_kernel<__nv_bfloat16, 8><<<blocks, 128, 0, s>>>(p, sc, bi, w.n, w.k, seed, tensor, 0.0f, std);
  } else {
    auto* sc = static_cast<__half*>(w.s);
    auto* bi = static_cast<__half*>(w.b);
    if (bits == 4) init_quant_kernel<__half, 4><<<blocks, 128, 0, s>>>(p, sc, bi, w.n, w.k, seed, tensor, 0.0f, std);
    else init_quant_kernel<__half, 8><<<blocks, 128, 0, s>>>(p, sc, bi, w.n, w.k, seed, tensor, 0.0f, std);
  }
  VELLA_CUDA_TRY(cudaGetLastError());
  return VELLA_OK;
}

int quantize_device(int src_dtype, const void* w, int dtype, int bits, int N, int K, void* packed, void* scales,
                    void* biases, cudaStream_t s) {
  const size_t groups = (size_t)N * (K / 64);
  const unsigned blocks = (unsigned)((groups + 127) / 128);
  auto* p = static_cast<uint32_t*>(packed);
#define VELLA_Q(TIN, TOUT, B)                                                                                  \
  quantize_kernel<TIN, TOUT, B><<<blocks, 128, 0, s>>>(static_cast<const TIN*>(w), p, static_cast<TOUT*>(scales), \
                                                       static_cast<TOUT*>(biases), N, K)
#define VELLA_QB(TIN, TOUT) \
  if (bits == 4) VELLA_Q(TIN, TOUT, 4); else VELLA_Q(TIN, TOUT, 8)
#define VELLA_QT(TIN)                                      \
  if (dtype == VELLA_BF16) { VELLA_QB(TIN, __nv_bfloat16); } \
  else { VELLA_QB(TIN, __half); }
  if (src_dtype == VELLA_F32) { VELLA_QT(float); }
  else if (src_dtype == VELLA_BF16) { VELLA_QT(__nv_bfloat16); }
  else { VELLA_QT(__half); }
#undef VELLA_QT
#undef VELLA_QB
#undef VELLA_Q
  VELLA_CUDA_TRY(cudaGetLastError());
  return VELLA_OK;
}

void* Model::kcache(int l) const {
  const size_t per = (size_t)cfg.n_kv_heads * cfg.max_seq * cfg.head_dim * elt;
  return static_cast<char*>(kv) + (size_t)l * 2 * per;
}
void* Model::vcache(int l) const {
  const size_t per = (size_t)cfg.n_kv_heads * cfg.max_seq * cfg.head_dim * elt;
  return static_cast<char*>(kv) + ((size_t)l * 2 + 1) * per;
}

namespace {

void plan_qweight(QWeight& q, int n, int k, int bits, int elt, size_t* off) {
  q.n = n;
  q.k = k;
  q.w_bytes = bits ? (size_t)n * k * bits / 8 : (size_t)n * k * elt;
  q.sb_bytes = bits ? (size_t)n * (k / 64) * elt : 0;
  q.w = reinterpret_cast<void*>(*off);
  *off += up256(q.w_bytes);
  if (bits) {
    q.s = reinterpret_cast<void*>(*off);
    *off += up256(q.sb_bytes);
    q.b = reinterpret_cast<void*>(*off);
    *off += up256(q.sb_bytes);
  }
}

void rebase_q(QWeight& q, char* base, bool quant) {
  q.w = base + reinterpret_cast<uintptr_t>(q.w);
  if (quant) {
    q.s = base + reinterpret_cast<uintptr_t>(q.s);
    q.b = base + reinterpret_cast<uintptr_t>(q.b);
  }
}

// Workspace of a GEMM at the streaming kernel's largest call (16 rows), at the largest
// tensor-core call that splits K (at most 256 rows; the splits keep fp32 sums for every row)
// and at the model's largest call.
size_t gemm_ws_for(const QWeight& w, int bits, int dtype, int epi, int rows) {
  size_t ws = 0;
  for (int m : {kMaxRows, std::min(rows, 256), rows}) {
    vella_qgemm_desc d{m, w.n, w.k, bits, 64, dtype, epi};
    QgemmPlan p;
    if (qgemm_plan(d, &p)) ws = std::max(ws, p.workspace);
  }
  return ws;
}

}  // namespace

void rope_table(int max_seq, int head_dim, float theta, float* out) {
  const int half = head_dim / 2;
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const double inv = std::pow((double)theta, -2.0 * i / (double)head_dim);
      const double ang = (double)pos * inv;
      out[((size_t)pos * half + i) * 2] = (float)std::cos(ang);
      out[((size_t)pos * half + i) * 2 + 1] = (float)std::sin(ang);
    }
}

int model_create(const vella_model_cfg& c, int device, Model** out) {
  if (c.n_layers <= 0 || c.d_model <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
      c.ffn <= 0 || c.vocab <= 0 || c.max_seq <= 0 || c.max_prefix < 0)
    return fail(VELLA_E_INVALID, "vella_model_create: sizes must be positive");
  if (c.n_heads % c.n_kv_heads != 0 || c.n_heads / c.n_kv_heads > 8)
    return fail(VELLA_E_UNSUPPORTED, "vella_model_create: n_heads/n_kv_heads = %d/%d", c.n_heads, c.n_kv_heads);
  if (c.head_dim != 64 && c.head_dim != 128) return fail(VELLA_E_UNSUPPORTED, "vella_model_create: head_dim %d", c.head_dim);
  if (c.bits != 0 && c.bits != 4 && c.bits != 8) return fail(VELLA_E_UNSUPPORTED, "vella_model_create: bits %d", c.bits);
  if (c.dtype != VELLA_BF16 && c.dtype != VELLA_F16) return fail(VELLA_E_UNSUPPORTED, "vella_model_create: dtype %d", c.dtype);
  if (c.d_model % 64 || c.ffn % 64 || (c.n_heads * c.head_dim) % 64)
    return fail(VELLA_E_UNSUPPORTED, "vella_model_create: d_model, ffn and n_heads*head_dim must be multiples of 64");
  if (c.max_prefix > c.max_seq) return fail(VELLA_E_INVALID, "vella_model_create: max_prefix > max_seq");
  if (c.streams < 0 || c.streams > 4096) return fail(VELLA_E_INVALID, "vella_model_create: streams %d", c.streams);
  if (c.rows_per_stream < 0 || c.rows_per_stream > 64)
    return fail(VELLA_E_INVALID, "vella_model_create: rows_per_stream %d (0..64)", c.rows_per_stream);
  VELLA_CUDA_TRY(cudaSetDevice(device));
  Model* m = new Model();
  m->cfg = c;
  m->device = device;
  m->elt = 2;
  m->streams = std::max(1, c.streams);
  const int d = c.d_model, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads, bits = c.bits, e = m->elt;
  // ---- weights arena ------------------------------------------------------------------
  size_t off = 0;
  m->embed = reinterpret_cast<void*>(off); off += up256((size_t)c.vocab * d * e);
  m->final_norm = reinterpret_cast<void*>(off); off += up256((size_t)d * e);
  plan_qweight(m->lm_head, c.vocab, d, bits, e, &off);
  m->layers.resize(c.n_layers);
  for (Layer& L : m->layers) {
    L.attn_norm = reinterpret_cast<void*>(off); off += up256((size_t)d * e);
    L.mlp_norm = reinterpret_cast<void*>(off); off += up256((size_t)d * e);
    if (c.qk_norm) {
      L.q_norm = reinterpret_cast<void*>(off); off += up256((size_t)hd * e);
      L.k_norm = reinterpret_cast<void*>(off); off += up256((size_t)hd * e);
    }
    plan_qweight(L.qkv, (H + 2 * KV) * hd, d, bits, e, &off);
    plan_qweight(L.o, d, H * hd, bits, e, &off);
    plan_qweight(L.gate, c.ffn, d, bits, e, &off);
    plan_qweight(L.up, c.ffn, d, bits, e, &off);
    plan_qweight(L.down, d, c.ffn, bits, e, &off);
  }
  m->arena_bytes = off;
  if (cudaMalloc(&m->arena, off) != cudaSuccess) {
    cudaGetLastError();
    delete m;
    return fail(VELLA_E_OOM, "vella_model_create: %zu bytes of weights", off);
  }
  char* base = static_cast<char*>(m->arena);
  m->embed = base + reinterpret_cast<uintptr_t>(m->embed);
  m->final_norm = base + reinterpret_cast<uintptr_t>(m->final_norm);
  rebase_q(m->lm_head, base, bits != 0);
  for (Layer& L : m->layers) {
    L.attn_norm = base + reinterpret_cast<uintptr_t>(L.attn_norm);
    L.mlp_norm = base + reinterpret_cast<uintptr_t>(L.mlp_norm);
    if (c.qk_norm) {
      L.q_norm = base + reinterpret_cast<uintptr_t>(L.q_norm);
      L.k_norm = base + reinterpret_cast<uintptr_t>(L.k_norm);
    }
    for (QWeight* q : {&L.qkv, &L.o, &L.gate, &L.up, &L.down}) rebase_q(*q, base, bits != 0);
  }
  // ---- KV cache, prefix, rope table -----------------------------------------------------
  m->kv_ss = (long long)c.n_layers * 2 * KV * c.max_seq * hd;
  m->kv_bytes = (size_t)m->streams * m->kv_ss * e;
  m->prefix_ss = (long long)std::max(c.max_prefix, 1) * d;
  m->rps = c.rows_per_stream > 0 ? c.rows_per_stream : kMaxRows;
  m->max_rows = std::max(kChunkRows, m->streams * m->rps);
  // ---- activations and scratch ------------------------------------------------------------
  size_t ws = 0;
  for (const Layer& L : m->layers) {
    const int R = m->max_rows;
    ws = std::max(ws, gemm_ws_for(L.qkv, bits, c.dtype, VELLA_EPI_NONE, R));
    ws = std::max(ws, gemm_ws_for(L.o, bits, c.dtype, VELLA_EPI_RESIDUAL, R));
    ws = std::max(ws, gemm_ws_for(L.gate, bits, c.dtype, VELLA_EPI_SILU_GATE, R));
    ws = std::max(ws, gemm_ws_for(L.down, bits, c.dtype, VELLA_EPI_RESIDUAL, R));
    break;  // every layer has the same shapes
  }
  ws = std::max(ws, gemm_ws_for(m->lm_head, bits, c.dtype, VELLA_EPI_NONE, m->max_rows));
  m->gemm_ws_bytes = ws;
  const size_t R = m->max_rows, RL = (size_t)m->streams * m->rps;
  const size_t sizes[] = {
      m->kv_bytes,                                  // 0 kv
      (size_t)m->streams * m->prefix_ss * e,        // 1 prefix
      (size_t)c.max_seq * (hd / 2) * sizeof(float2),// 2 rope
      R * d * e, R * d * e,                         // 3 h, 4 xn
      R * m->qkv_n() * e,                           // 5 qkv
      R * H * hd * e, R * H * hd * e,               // 6 q, 7 attn
      R * c.ffn * e,                                // 8 mlp
      RL * (size_t)c.vocab * e,                     // 9 logits
      RL * sizeof(int),                             // 10 ys
      ws,                                           // 11 gemm workspace
      0,                                            // 12 (unused)
      argmax_scratch_bytes((int)RL) + 512,          // 13 argmax scratch
      4 * sizeof(int),                              // 14 flags
      (size_t)c.max_seq * sizeof(int),              // 15 scoring token ids
  };
  size_t total = 0;
  for (size_t s : sizes) total += up256(s);
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(m->arena);
    delete m;
    return fail(VELLA_E_CUDA, "vella_model_create: stream creation failed");
  }
  if (cudaMalloc(&m->act_arena, total) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(m->arena);
    delete m;
    return fail(VELLA_E_OOM, "vella_model_create: %zu bytes of cache and buffers", total);
  }
  // zeroed on the model's non-blocking stream and waited for before any kernel uses it
  VELLA_CUDA_TRY(cudaMemsetAsync(m->act_arena, 0, total, m->stream));
  VELLA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  char* p = static_cast<char*>(m->act_arena);
  void* slots[16];
  for (int i = 0; i < 16; ++i) { slots[i] = p; p += up256(sizes[i]); }
  m->kv = slots[0];
  m->prefix = slots[1];
  m->rope = static_cast<float2*>(slots[2]);
  m->h = slots[3]; m->xn = slots[4]; m->qkv_out = slots[5]; m->q = slots[6]; m->attn = slots[7]; m->mlp = slots[8];
  m->logits = slots[9];
  m->ys = static_cast<int*>(slots[10]);
  m->gemm_ws = ws ? slots[11] : nullptr;
  m->argmax_sc = slots[13];
  int* flags = static_cast<int*>(slots[14]);
  m->err = flags;
  m->nonfinite = flags + 1;
  m->dzero = flags + 2;
  m->score_P = flags + 3;
  m->score_tok = static_cast<int*>(slots[15]);
  std::vector<float> table((size_t)c.max_seq * hd);
  rope_table(c.max_seq, hd, c.rope_theta, table.data());
  VELLA_CUDA_TRY(cudaMemcpy(m->rope, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (fwd_prog_model_ok(m)) {  // built now: a forward may first run under graph capture
    const int rc = fwd_prog_build(m, &m->prog);
    if (rc) {
      model_destroy(m);
      return rc;
    }
  }
  *out = m;
  return VELLA_OK;
}

void model_destroy(Model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  cudaDeviceSynchronize();
  if (m->prog) fwd_prog_destroy(m->prog);
  if (m->arena) cudaFree(m->arena);
  if (m->act_arena) cudaFree(m->act_arena);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int model_init_random(Model* m, uint64_t seed, float std, cudaStream_t s) {
  const vella_model_cfg& c = m->cfg;
  const int dt = c.dtype;
  uint32_t tid = 1;
  int rc;
  auto dense = [&](void* p, size_t n, float mean, float sd) { return fill_normal(p, n, dt, seed, tid++, mean, sd, s); };
  auto weight = [&](const QWeight& q) {
    if (c.bits) return quantize_random(q, c.bits, dt, seed, tid++, std, s);
    return fill_normal(q.w, (size_t)q.n * q.k, dt, seed, tid++, 0.0f, std, s);
  };
  if ((rc = dense(m->embed, (size_t)c.vocab * c.d_model, 0.0f, 1.0f))) return rc;
  if ((rc = dense(m->final_norm, c.d_model, 1.0f, 0.1f))) return rc;
  if ((rc = weight(m->lm_head))) return rc;
  for (Layer& L : m->layers) {
    if ((rc = dense(L.attn_norm, c.d_model, 1.0f, 0.1f))) return rc;
    if ((rc = dense(L.mlp_norm, c.d_model, 1.0f, 0.1f))) return rc;
    if (c.qk_norm) {
      if ((rc = dense(L.q_norm, c.head_dim, 1.0f, 0.1f))) return rc;
      if ((rc = dense(L.k_norm, c.head_dim, 1.0f, 0.1f))) return rc;
    }
    for (QWeight* q : {&L.qkv, &L.o, &L.gate, &L.up, &L.down})
      if ((rc = weight(*q))) return rc;
  }
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  return VELLA_OK;
}

int model_tensor(Model* m, const std::string& name, int layer, void** ptr, size_t* bytes) {
  const vella_model_cfg& c = m->cfg;
  const size_t e = m->elt;
  auto ret = [&](void* p, size_t b) {
    *ptr = p;
    *bytes = b;
    return VELLA_OK;
  };
  auto qw = [&](const QWeight& q, const std::string& part) -> int {
    if (part == "w") return ret(q.w, q.w_bytes);
    if (part == "s" && c.bits) return ret(q.s, q.sb_bytes);
    if (part == "b" && c.bits) return ret(q.b, q.sb_bytes);
    return fail(VELLA_E_INVALID, "vella_model_tensor: no part '%s'", part.c_str());
  };
  if (name == "embed") return ret(m->embed, (size_t)c.vocab * c.d_model * e);
  if (name == "final_norm") return ret(m->final_norm, (size_t)c.d_model * e);
  if (name == "prefix") return ret(m->prefix, (size_t)m->streams * m->prefix_ss * e);  // [streams][max_prefix][d]
  if (name == "logits") return ret(m->logits, (size_t)m->streams * m->rps * c.vocab * e);
  if (name == "kv") return ret(m->kv, m->kv_bytes);
  const size_t dot = name.find('.');
  const std::string head = name.substr(0, dot), part = dot == std::string::npos ? "" : name.substr(dot + 1);
  if (head == "lm_head") return qw(m->lm_head, part);
  if (layer < 0 || layer >= c.n_layers) return fail(VELLA_E_INVALID, "vella_model_tensor: layer %d out of range", layer);
  Layer& L = m->layers[layer];
  if (name == "attn_norm") return ret(L.attn_norm, (size_t)c.d_model * e);
  if (name == "mlp_norm") return ret(L.mlp_norm, (size_t)c.d_model * e);
  if (name == "q_norm" && c.qk_norm) return ret(L.q_norm, (size_t)c.head_dim * e);
  if (name == "k_norm" && c.qk_norm) return ret(L.k_norm, (size_t)c.head_dim * e);
  if (head == "qkv") return qw(L.qkv, part);
  if (head == "o") return qw(L.o, part);
  if (head == "gate") return qw(L.gate, part);
  if (head == "up") return qw(L.up, part);
  if (head == "down") return qw(L.down, part);
  return fail(VELLA_E_INVALID, "vella_model_tensor: unknown tensor '%s'", name.c_str());
}

int model_gemm(Model* m, const QWeight& w, const void* x, int rows, void* out, int epilogue, const void* residual,
               const QWeight* up, cudaStream_t s, const RopeEpi* rope) {
  vella_qgemm_desc d{rows, w.n, w.k, m->cfg.bits, 64, m->cfg.dtype, epilogue};
  QgemmPlan p;
  if (!qgemm_plan(d, &p)) return fail(VELLA_E_UNSUPPORTED, "model gemm %dx%dx%d", rows, w.n, w.k);
  if (p.workspace > m->gemm_ws_bytes) return fail(VELLA_E_INVALID, "model gemm workspace too small");
  return qgemm_launch(d, p, x, w.w, w.s, w.b, up ? up->w : nullptr, up ? up->s : nullptr, up ? up->b : nullptr,
                      nullptr, residual, out, m->gemm_ws, s, rope);
}

// True when the q|k|v projection of M rows runs on the streaming kernel, which can apply
// RoPE and append K/V in its epilogue (head_dim 128, no q/k norm, no tree rows).
bool fuse_rope(Model* m, const Layer& L, int M, const TreeView* tree) {
  const vella_model_cfg& c = m->cfg;
  if (tree || L.q_norm || L.k_norm || c.head_dim != 128) return false;
  vella_qgemm_desc d{M, L.qkv.n, L.qkv.k, c.bits, 64, c.dtype, VELLA_EPI_NONE};
  QgemmPlan p;
  return qgemm_plan(d, &p) && p.stream;
}

int model_forward(Model* m, PosRef pr, int rows, int streams, int stream0, const int* tok, int tok_ss, const int* P,
                  int logits_rows, cudaStream_t s, const TreeView* tree) {
  const vella_model_cfg& c = m->cfg;
  const int M = rows * streams;
  if (rows <= 0 || streams <= 0 || stream0 < 0 || stream0 + streams > m->streams || M > m->max_rows ||
      logits_rows > std::min(rows, m->rps) || logits_rows < 0)
    return fail(VELLA_E_INVALID, "forward: %d rows x %d streams from %d, %d logits rows", rows, streams, stream0,
                logits_rows);
  const int d = c.d_model, H = c.n_heads, KV = c.n_kv_heads, hd = c.head_dim, dt = c.dtype;
  const float scale = 1.0f / std::sqrt((float)hd);
  pr.group = streams > 1 ? rows : 0;
  const size_t e = m->elt;
  const char* prefix = static_cast<const char*>(m->prefix) + (size_t)stream0 * m->prefix_ss * e;
  const size_t kv0 = (size_t)stream0 * m->kv_ss * e;
  const TreeView tv = tree ? *tree : TreeView{};
  if (tree && (!tree->tok || !tree->dep || !tree->mask || tree->node0 + rows > tree->nodes || tree->nodes > 64))
    return fail(VELLA_E_INVALID, "forward: tree rows %d from node %d of %d", rows, tree->node0, tree->nodes);
  int rc;
  if ((rc = launch_embed_rows_dev(dt, m->h, m->embed, prefix, m->prefix_ss, tok, tok_ss, pr, M, P, d, c.vocab,
                                  c.max_seq, m->err, s, tv)))
    return rc;
  if (!tree && m->prog && m->persistent && M <= kMaxRows && rows * (H / KV) <= kAttnRows) {
    if ((rc = fwd_prog_run(m, m->prog, pr, rows, streams, stream0, logits_rows, s))) return rc;
    if (logits_rows > 0)
      return launch_argmax(dt, m->logits, logits_rows * streams, c.vocab, (size_t)c.vocab, m->ys, m->argmax_sc,
                           m->nonfinite, s);
    return VELLA_OK;
  }
  for (int l = 0; l < c.n_layers; ++l) {
    Layer& L = m->layers[l];
    char* kc = static_cast<char*>(m->kcache(l)) + kv0;
    char* vc = static_cast<char*>(m->vcache(l)) + kv0;
    if ((rc = launch_rmsnorm(dt, m->xn, m->h, L.attn_norm, M, d, c.rms_eps, s))) return rc;
    if (fuse_rope(m, L, M, tree)) {
      RopeEpi re;
      re.cs = m->rope; re.q = m->q; re.kc = kc; re.vc = vc; re.pr = pr;
      re.H = H; re.KV = KV; re.max_seq = c.max_seq; re.kv_ss = m->kv_ss; re.err = m->err;
      if ((rc = model_gemm(m, L.qkv, m->xn, M, m->qkv_out, VELLA_EPI_NONE, nullptr, nullptr, s, &re))) return rc;
    } else {
      if ((rc = model_gemm(m, L.qkv, m->xn, M, m->qkv_out, VELLA_EPI_NONE, nullptr, nullptr, s))) return rc;
      if ((rc = launch_rope_append(dt, m->qkv_out, m->q, kc, vc, m->rope, L.q_norm, L.k_norm, c.rms_eps, pr, M, H, KV,
                                   hd, c.max_seq, m->err, s, m->kv_ss, tv)))
        return rc;
    }
    AttnView v;
    v.q = m->q; v.out = m->attn;
    v.q_rs = v.o_rs = (long long)H * hd;
    v.q_bs = v.o_bs = (long long)rows * H * hd;
    v.k = kc; v.v = vc;
    v.kv_hs = (long long)c.max_seq * hd; v.kv_rs = hd; v.kv_bs = m->kv_ss;
    v.tmask = tv.mask; v.tnode0 = tv.node0;
    if ((rc = launch_attention_ex(dt, v, streams, pr, 1, rows, H, KV, hd, c.max_seq, scale, s))) return rc;
    if ((rc = model_gemm(m, L.o, m->attn, M, m->h, VELLA_EPI_RESIDUAL, m->h, nullptr, s))) return rc;
    if ((rc = launch_rmsnorm(dt, m->xn, m->h, L.mlp_norm, M, d, c.rms_eps, s))) return rc;
    if ((rc = model_gemm(m, L.gate, m->xn, M, m->mlp, VELLA_EPI_SILU_GATE, nullptr, &L.up, s))) return rc;
    if ((rc = model_gemm(m, L.down, m->mlp, M, m->h, VELLA_EPI_RESIDUAL, m->h, nullptr, s))) return rc;
  }
  if (logits_rows > 0) {
    const int LR = logits_rows * streams;  // the last logits_rows rows of every stream, stream-major
    if ((rc = launch_rmsnorm(dt, m->xn, m->h, m->final_norm, LR, d, c.rms_eps, s, rows, logits_rows))) return rc;
    if ((rc = model_gemm(m, m->lm_head, m->xn, LR, m->logits, VELLA_EPI_NONE, nullptr, nullptr, s))) return rc;
    if ((rc = launch_argmax(dt, m->logits, LR, c.vocab, (size_t)c.vocab, m->ys, m->argmax_sc, m->nonfinite, s)))
      return rc;
  }
  return VELLA_OK;
}

}  // namespace vella
