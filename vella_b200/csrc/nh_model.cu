// A Nemotron-H backbone on one GPU: the reference's hybrid stack of Mamba-2, attention and MoE
// blocks (pattern string, one character per layer), final norm, LM head and argmax.
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeDecoder.swift:
// NTBlock (:508-531: x + mixer(rmsnorm(x))), NTMamba (:318-360), NTAttention (:362-392: GQA
// without positional encoding, causal over the cache), NTMoE (:464-499: routed relu^2 experts
// plus the shared relu^2 expert), NTBackbone (:533-562: embeddings, layers, norm_f) and the LM
// head (:564-571, argmax in NemotronTranscribeModel.head :263).
//
// Every block runs on the library's kernels: RMSNorm, the MLX-affine / dense GEMM (vella_qgemm
// with the residual epilogue for the output projections), the Mamba-2 conv / scan / gated
// norm, the attention kernel after the K/V append (the RoPE append with an identity table: no
// positional encoding), the MoE router and experts (accumulating into the residual stream).
// The Mamba states and the attention caches live in the handle; a caller that rolls a
// verify pass back copies the Mamba states back from its own snapshot (vella_nh_tensor) and
// forwards the next rows from the accepted position, which overwrites the attention rows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "layers.cuh"

namespace vella {
namespace {

struct NhLin {  // one Linear [n][k] (stacked over `count` experts), MLX-affine or dense
  void *w = nullptr, *s = nullptr, *b = nullptr;
  int n = 0, k = 0, count = 1;
  size_t w_bytes = 0, sb_bytes = 0;
};

struct NhLayer {
  char kind = 'M';
  void* norm = nullptr;
  // M
  NhLin in_proj, out_proj;
  void *conv_w = nullptr, *conv_b = nullptr, *gnorm = nullptr, *conv_state = nullptr;
  float *a_log = nullptr, *dt_bias = nullptr, *Dv = nullptr, *ssm_state = nullptr;
  // *
  NhLin qkv, o;
  void* kv = nullptr;  // [2][KV][max_seq][hd]
  // E
  float *router = nullptr, *rbias = nullptr;
  NhLin fc1, fc2, sup, sdown;
};

// The MTP head (NTMTP, NemotronTranscribeDecoder.swift:578-606):
// x = eh_proj(concat(enorm(e), hnorm(h))); x += attention(attn_norm(x)); x += MoE(moe_norm(x));
// its own attention cache.
struct NhMtp {
  NhLin eh;
  void *enorm = nullptr, *hnorm = nullptr, *final_norm = nullptr;
  NhLayer attn, moe;  // kind '*' and 'E'
};

__global__ void nh_embed_kernel(uint16_t* h, const uint16_t* __restrict__ table, const int* __restrict__ tok, int d,
                                int vocab, int* err) {
  pdl_wait();
  pdl_launch_next();
  int t = tok[blockIdx.x];
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0) atomicOr(err, 1);
    t = 0;
  }
  for (int i = threadIdx.x; i < d; i += blockDim.x) h[(size_t)blockIdx.x * d + i] = table[(size_t)t * d + i];
}

}  // namespace
}  // namespace vella

using namespace vella;

struct vella_nh {
  vella_nh_cfg cfg{};
  int device = 0, L = 0, I = 0, conv_dim = 0, in_w = 0, qkv_n = 0;
  size_t elt = 2;
  cudaStream_t stream = nullptr;
  std::vector<NhLayer> layers;
  bool has_mtp = false;
  NhMtp mtp;
  void *cat = nullptr, *x2 = nullptr;  // MTP [rows][2 hidden] input, [rows][hidden] stream
  std::vector<void*> allocs;
  void *embed = nullptr, *norm_f = nullptr;
  NhLin lm_head;
  // activations [max_rows][...]
  void *h = nullptr, *xn = nullptr, *big = nullptr, *xbc = nullptr, *y = nullptr, *yn = nullptr, *q = nullptr,
       *attn = nullptr, *logits = nullptr, *ident = nullptr, *gemm_ws = nullptr, *moe_ws = nullptr,
       *argmax_sc = nullptr;
  size_t gemm_ws_bytes = 0, moe_ws_bytes = 0;
  int *tok = nullptr, *ys = nullptr, *dpos = nullptr, *err = nullptr, *nonfinite = nullptr, *eidx = nullptr,
      *zidx = nullptr;
  float *ew = nullptr, *ones = nullptr;

  void* alloc(size_t bytes, int* rc) {
    void* p = nullptr;
    if (*rc) return nullptr;
    if (cudaMalloc(&p, std::max<size_t>(bytes, 16)) != cudaSuccess) {
      cudaGetLastError();
      *rc = fail(VELLA_E_OOM, "vella_nh_create: %zu bytes", bytes);
      return nullptr;
    }
    allocs.push_back(p);
    if (cudaMemsetAsync(p, 0, std::max<size_t>(bytes, 16), stream) != cudaSuccess) *rc = fail(VELLA_E_CUDA, "memset");
    return p;
  }
  void lin(NhLin& l, int n, int k, int count, int* rc) {
    l.n = n; l.k = k; l.count = count;
    const int bits = cfg.bits;
    l.w_bytes = bits ? (size_t)count * n * k * bits / 8 : (size_t)count * n * k * elt;
    l.sb_bytes = bits ? (size_t)count * n * (k / 64) * elt : 0;
    l.w = alloc(l.w_bytes, rc);
    if (bits) { l.s = alloc(l.sb_bytes, rc); l.b = alloc(l.sb_bytes, rc); }
  }
};

namespace {

int nh_gemm(vella_nh* m, const NhLin& l, const void* x, int rows, void* out, bool residual) {
  vella_qgemm_desc d{rows, l.n, l.k, m->cfg.bits, 64, m->cfg.dtype, residual ? VELLA_EPI_RESIDUAL : VELLA_EPI_NONE};
  return vella_qgemm(&d, x, l.w, l.s, l.b, nullptr, nullptr, nullptr, nullptr, residual ? out : nullptr, out,
                     m->gemm_ws, m->gemm_ws_bytes, m->stream);
}

// At the streaming kernel's largest call, at the largest tensor-core call that splits K (at
// most 256 rows; the splits keep fp32 sums for every row) and at the largest call.
size_t gemm_ws_for(const vella_nh* m, int n, int k) {
  size_t ws = 0;
  for (int rows : {std::min(16, m->cfg.max_rows), std::min(256, m->cfg.max_rows), m->cfg.max_rows}) {
    vella_qgemm_desc d{rows, n, k, m->cfg.bits, 64, m->cfg.dtype, VELLA_EPI_RESIDUAL};
    ws = std::max(ws, vella_qgemm_workspace_size(&d));
  }
  return ws;
}

vella_mamba_desc mamba_desc(const vella_nh* m, int rows) {
  const vella_nh_cfg& c = m->cfg;
  vella_mamba_desc d{};
  d.streams = 1; d.tokens = rows; d.heads = c.m_heads; d.head_dim = c.m_head_dim; d.groups = c.groups;
  d.state_dim = c.state_dim; d.conv_kernel = c.conv_kernel; d.dtype = c.dtype; d.in_stride = m->in_w;
  d.dt_min = c.dt_min; d.dt_max = c.dt_max; d.eps = c.eps;
  return d;
}

// Device tokens of `rows` host ids, then the embedding rows into `out`.
int nh_embed(vella_nh* m, const int32_t* tokens, int rows, void* out) {
  const vella_nh_cfg& c = m->cfg;
  VELLA_CUDA_TRY(cudaMemcpyAsync(m->tok, tokens, rows * sizeof(int), cudaMemcpyHostToDevice, m->stream));
  return launch_kernel(nh_embed_kernel, dim3(rows), dim3(128), 0, m->stream, static_cast<uint16_t*>(out),
                       static_cast<const uint16_t*>(m->embed), (const int*)m->tok, c.hidden, c.vocab, m->err);
}

// x += out_proj(gated_norm(ssm(conv(in_proj(rmsnorm(x))))))
int nh_mamba_block(vella_nh* m, NhLayer& Ly, void* x, int rows) {
  const vella_nh_cfg& c = m->cfg;
  cudaStream_t s = m->stream;
  const vella_mamba_desc md = mamba_desc(m, rows);
  int rc;
  if ((rc = launch_rmsnorm(c.dtype, m->xn, x, Ly.norm, rows, c.hidden, c.eps, s)) ||
      (rc = nh_gemm(m, Ly.in_proj, m->xn, rows, m->big, false)) ||
      (rc = vella_mamba_conv(&md, m->big, Ly.conv_w, Ly.conv_b, Ly.conv_state, m->xbc, s)) ||
      (rc = vella_mamba_ssm(&md, m->xbc, m->big, Ly.a_log, Ly.dt_bias, Ly.Dv, Ly.ssm_state, m->y, s)) ||
      (rc = vella_mamba_gated_norm(&md, m->y, m->big, Ly.gnorm, m->yn, s)))
    return rc;
  return nh_gemm(m, Ly.out_proj, m->yn, rows, x, true);
}

// x += o(attention(q, K/V cache)) of rmsnorm(x), keys appended at positions *dpos ..
int nh_attention_block(vella_nh* m, NhLayer& Ly, void* x, int rows) {
  const vella_nh_cfg& c = m->cfg;
  cudaStream_t s = m->stream;
  const int H = c.heads, KV = c.kv_heads, hd = c.head_dim, dt = c.dtype;
  char* kc = static_cast<char*>(Ly.kv);
  char* vc = kc + (size_t)KV * c.max_seq * hd * m->elt;
  const PosRef pr{m->dpos, 0};
  int rc;
  if ((rc = launch_rmsnorm(dt, m->xn, x, Ly.norm, rows, c.hidden, c.eps, s)) ||
      (rc = nh_gemm(m, Ly.qkv, m->xn, rows, m->big, false)) ||
      (rc = launch_rope_append(dt, m->big, m->q, kc, vc, static_cast<const float2*>(m->ident), nullptr, nullptr, c.eps,
                               pr, rows, H, KV, hd, c.max_seq, m->err, s)))
    return rc;
  AttnView v;
  v.q = m->q; v.out = m->attn;
  v.q_rs = v.o_rs = (long long)H * hd;
  v.q_bs = v.o_bs = (long long)rows * H * hd;
  v.k = kc; v.v = vc;
  v.kv_hs = (long long)c.max_seq * hd; v.kv_rs = hd; v.kv_bs = 0;
  if ((rc = launch_attention_ex(dt, v, 1, pr, 1, rows, H, KV, hd, c.max_seq, 1.0f / std::sqrt((float)hd), s)))
    return rc;
  return nh_gemm(m, Ly.o, m->attn, rows, x, true);
}

// x += routed experts + shared expert of rmsnorm(x)
int nh_moe_block(vella_nh* m, NhLayer& Ly, void* x, int rows) {
  const vella_nh_cfg& c = m->cfg;
  cudaStream_t s = m->stream;
  const int d = c.hidden, dt = c.dtype;
  vella_moe_route_desc rd{rows, d, c.experts, c.top_k, c.norm_topk, c.routed_scaling, dt};
  vella_moe_experts_desc xd{rows, d, c.moe_inter, c.experts, c.top_k, c.bits, dt};
  vella_moe_experts_desc sd{rows, d, c.shared_inter, 1, 1, c.bits, dt};
  int rc;
  if ((rc = launch_rmsnorm(dt, m->xn, x, Ly.norm, rows, d, c.eps, s)) ||
      (rc = vella_moe_route(&rd, m->xn, Ly.router, Ly.rbias, m->eidx, m->ew, s)) ||
      (rc = vella_moe_experts(&xd, m->xn, m->eidx, m->ew, Ly.fc1.w, Ly.fc1.s, Ly.fc1.b, Ly.fc2.w, Ly.fc2.s, Ly.fc2.b,
                              x, 1, m->moe_ws, m->moe_ws_bytes, s)))
    return rc;
  return vella_moe_experts(&sd, m->xn, m->zidx, m->ones, Ly.sup.w, Ly.sup.s, Ly.sup.b, Ly.sdown.w, Ly.sdown.s,
                           Ly.sdown.b, x, 1, m->moe_ws, m->moe_ws_bytes, s);
}

// norm, LM head and argmax of the last logits_rows of `rows` rows of x
int nh_head(vella_nh* m, const void* x, const void* norm, int rows, int logits_rows, int32_t* argmax_out,
            void* logits_out) {
  if (logits_rows <= 0) return VELLA_OK;
  const vella_nh_cfg& c = m->cfg;
  cudaStream_t s = m->stream;
  int rc;
  if ((rc = launch_rmsnorm(c.dtype, m->xn, x, norm, logits_rows, c.hidden, c.eps, s, rows, logits_rows)) ||
      (rc = nh_gemm(m, m->lm_head, m->xn, logits_rows, m->logits, false)) ||
      (rc = launch_argmax(c.dtype, m->logits, logits_rows, c.vocab, (size_t)c.vocab, m->ys, m->argmax_sc, m->nonfinite,
                          s)))
    return rc;
  VELLA_CUDA_TRY(cudaMemcpyAsync(argmax_out, m->ys, logits_rows * sizeof(int), cudaMemcpyDeviceToHost, s));
  if (logits_out)
    VELLA_CUDA_TRY(cudaMemcpyAsync(logits_out, m->logits, (size_t)logits_rows * c.vocab * m->elt,
                                   cudaMemcpyDeviceToDevice, s));
  return VELLA_OK;
}

// waits for the handle's work and reports its flags
int nh_finish(vella_nh* m, const char* what) {
  cudaStream_t s = m->stream;
  VELLA_CUDA_TRY(cudaStreamSynchronize(s));
  int f[2] = {0, 0};
  VELLA_CUDA_TRY(cudaMemcpy(f, m->err, sizeof(f), cudaMemcpyDeviceToHost));
  if (f[0] || f[1]) {
    VELLA_CUDA_TRY(cudaMemsetAsync(m->err, 0, sizeof(f), s));
    VELLA_CUDA_TRY(cudaStreamSynchronize(s));
    return fail(f[1] ? VELLA_E_NONFINITE : VELLA_E_INVALID, "%s: flags 0x%x 0x%x", what, f[0], f[1]);
  }
  return VELLA_OK;
}

}  // namespace

extern "C" {

int vella_nh_create(const vella_nh_cfg* cfg, int32_t device, vella_nh** out) {
  if (!cfg || !out) return fail(VELLA_E_INVALID, "vella_nh_create: NULL argument");
  *out = nullptr;
  const vella_nh_cfg& c = *cfg;
  const int L = (int)strnlen(c.pattern, sizeof(c.pattern));
  if (L < 1 || L >= (int)sizeof(c.pattern) || c.hidden % 64 || c.vocab < 1 || c.max_rows < 1 || c.max_rows > 512 ||
      c.max_seq < c.max_rows || (c.bits != 0 && c.bits != 4 && c.bits != 8) ||
      (c.dtype != VELLA_BF16 && c.dtype != VELLA_F16))
    return fail(VELLA_E_INVALID, "vella_nh_create: pattern of %d layers, hidden %d (multiple of 64), max_rows %d "
                "(1..512), max_seq %d, bits %d", L, c.hidden, c.max_rows, c.max_seq, c.bits);
  for (int l = 0; l < L; ++l)
    if (c.pattern[l] != 'M' && c.pattern[l] != '*' && c.pattern[l] != 'E')
      return fail(VELLA_E_INVALID, "vella_nh_create: layer %d kind '%c' (M, * or E)", l, c.pattern[l]);
  VELLA_CUDA_TRY(cudaSetDevice(device));
  auto* m = new vella_nh();
  m->cfg = c;
  m->device = device;
  m->L = L;
  m->I = c.m_heads * c.m_head_dim;
  m->conv_dim = m->I + 2 * c.groups * c.state_dim;
  m->in_w = m->I + m->conv_dim + c.m_heads;
  m->qkv_n = (c.heads + 2 * c.kv_heads) * c.head_dim;
  int rc = VELLA_OK;
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete m;
    return fail(VELLA_E_CUDA, "vella_nh_create: stream");
  }
  const int d = c.hidden, R = c.max_rows, e = (int)m->elt;
  m->embed = m->alloc((size_t)c.vocab * d * e, &rc);
  m->norm_f = m->alloc((size_t)d * e, &rc);
  m->lin(m->lm_head, c.vocab, d, 1, &rc);
  size_t ws = gemm_ws_for(m, c.vocab, d);
  int moe_inter = 1;
  m->layers.resize(L);
  for (int l = 0; l < L; ++l) {
    NhLayer& Ly = m->layers[l];
    Ly.kind = c.pattern[l];
    Ly.norm = m->alloc((size_t)d * e, &rc);
    if (Ly.kind == 'M') {
      m->lin(Ly.in_proj, m->in_w, d, 1, &rc);
      m->lin(Ly.out_proj, d, m->I, 1, &rc);
      Ly.conv_w = m->alloc((size_t)m->conv_dim * c.conv_kernel * e, &rc);
      Ly.conv_b = m->alloc((size_t)m->conv_dim * e, &rc);
      Ly.gnorm = m->alloc((size_t)m->I * e, &rc);
      Ly.conv_state = m->alloc((size_t)std::max(c.conv_kernel - 1, 1) * m->conv_dim * e, &rc);
      Ly.a_log = static_cast<float*>(m->alloc((size_t)c.m_heads * 4, &rc));
      Ly.dt_bias = static_cast<float*>(m->alloc((size_t)c.m_heads * 4, &rc));
      Ly.Dv = static_cast<float*>(m->alloc((size_t)c.m_heads * 4, &rc));
      Ly.ssm_state = static_cast<float*>(m->alloc((size_t)c.m_heads * c.m_head_dim * c.state_dim * 4, &rc));
      ws = std::max({ws, gemm_ws_for(m, m->in_w, d), gemm_ws_for(m, d, m->I)});
    } else if (Ly.kind == '*') {
      m->lin(Ly.qkv, m->qkv_n, d, 1, &rc);
      m->lin(Ly.o, d, c.heads * c.head_dim, 1, &rc);
      Ly.kv = m->alloc((size_t)2 * c.kv_heads * c.max_seq * c.head_dim * e, &rc);
      ws = std::max({ws, gemm_ws_for(m, m->qkv_n, d), gemm_ws_for(m, d, c.heads * c.head_dim)});
    } else {
      Ly.router = static_cast<float*>(m->alloc((size_t)c.experts * d * 4, &rc));
      Ly.rbias = static_cast<float*>(m->alloc((size_t)c.experts * 4, &rc));
      m->lin(Ly.fc1, c.moe_inter, d, c.experts, &rc);
      m->lin(Ly.fc2, d, c.moe_inter, c.experts, &rc);
      m->lin(Ly.sup, c.shared_inter, d, 1, &rc);
      m->lin(Ly.sdown, d, c.shared_inter, 1, &rc);
      moe_inter = std::max({moe_inter, c.moe_inter, c.shared_inter});
    }
  }
  if (c.mtp) {
    m->has_mtp = true;
    NhMtp& t = m->mtp;
    m->lin(t.eh, d, 2 * d, 1, &rc);
    t.enorm = m->alloc((size_t)d * e, &rc);
    t.hnorm = m->alloc((size_t)d * e, &rc);
    t.final_norm = m->alloc((size_t)d * e, &rc);
    t.attn.kind = '*';
    t.attn.norm = m->alloc((size_t)d * e, &rc);
    m->lin(t.attn.qkv, m->qkv_n, d, 1, &rc);
    m->lin(t.attn.o, d, c.heads * c.head_dim, 1, &rc);
    t.attn.kv = m->alloc((size_t)2 * c.kv_heads * c.max_seq * c.head_dim * e, &rc);
    t.moe.kind = 'E';
    t.moe.norm = m->alloc((size_t)d * e, &rc);
    t.moe.router = static_cast<float*>(m->alloc((size_t)c.experts * d * 4, &rc));
    t.moe.rbias = static_cast<float*>(m->alloc((size_t)c.experts * 4, &rc));
    m->lin(t.moe.fc1, c.moe_inter, d, c.experts, &rc);
    m->lin(t.moe.fc2, d, c.moe_inter, c.experts, &rc);
    m->lin(t.moe.sup, c.shared_inter, d, 1, &rc);
    m->lin(t.moe.sdown, d, c.shared_inter, 1, &rc);
    moe_inter = std::max({moe_inter, c.moe_inter, c.shared_inter});
    ws = std::max({ws, gemm_ws_for(m, d, 2 * d), gemm_ws_for(m, m->qkv_n, d), gemm_ws_for(m, d, c.heads * c.head_dim)});
    m->cat = m->alloc((size_t)R * 2 * d * e, &rc);
    m->x2 = m->alloc((size_t)R * d * e, &rc);
  }
  const int wide = std::max({m->in_w, m->qkv_n, d});
  m->h = m->alloc((size_t)R * d * e, &rc);
  m->xn = m->alloc((size_t)R * d * e, &rc);
  m->big = m->alloc((size_t)R * wide * e, &rc);
  m->xbc = m->alloc((size_t)R * m->conv_dim * e, &rc);
  m->y = m->alloc((size_t)R * m->I * e, &rc);
  m->yn = m->alloc((size_t)R * m->I * e, &rc);
  m->q = m->alloc((size_t)R * c.heads * c.head_dim * e, &rc);
  m->attn = m->alloc((size_t)R * c.heads * c.head_dim * e, &rc);
  m->logits = m->alloc((size_t)R * c.vocab * e, &rc);
  m->argmax_sc = m->alloc(argmax_scratch_bytes(R), &rc);
  m->tok = static_cast<int*>(m->alloc((size_t)R * 4, &rc));
  m->ys = static_cast<int*>(m->alloc((size_t)R * 4, &rc));
  m->dpos = static_cast<int*>(m->alloc(16, &rc));
  m->err = static_cast<int*>(m->alloc(16, &rc));
  m->nonfinite = m->err + 1;
  if (c.experts > 0 && c.top_k > 0) {
    m->eidx = static_cast<int*>(m->alloc((size_t)R * c.top_k * 4, &rc));
    m->ew = static_cast<float*>(m->alloc((size_t)R * c.top_k * 4, &rc));
    m->zidx = static_cast<int*>(m->alloc((size_t)R * 4, &rc));  // zeros: every row's shared expert
    m->ones = static_cast<float*>(m->alloc((size_t)R * 4, &rc));
    vella_moe_experts_desc md{R, d, moe_inter, std::max(c.experts, 1), c.top_k, c.bits, c.dtype};
    m->moe_ws_bytes = vella_moe_experts_workspace_size(&md);
    m->moe_ws = m->alloc(m->moe_ws_bytes, &rc);
  }
  m->gemm_ws_bytes = ws;
  if (ws) m->gemm_ws = m->alloc(ws, &rc);
  // identity rotation: the attention has no positional encoding
  m->ident = m->alloc((size_t)c.max_seq * (c.head_dim / 2) * sizeof(float2), &rc);
  if (!rc) {
    std::vector<float2> id((size_t)c.max_seq * (c.head_dim / 2), make_float2(1.0f, 0.0f));
    if (cudaMemcpyAsync(m->ident, id.data(), id.size() * sizeof(float2), cudaMemcpyHostToDevice, m->stream) !=
        cudaSuccess)
      rc = fail(VELLA_E_CUDA, "vella_nh_create: identity table");
    if (!rc && m->ones) {
      std::vector<float> one((size_t)R, 1.0f);
      if (cudaMemcpyAsync(m->ones, one.data(), one.size() * 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
        rc = fail(VELLA_E_CUDA, "vella_nh_create: ones");
    }
    if (!rc && cudaStreamSynchronize(m->stream) != cudaSuccess) rc = fail(VELLA_E_CUDA, "vella_nh_create: sync");
  }
  if (rc) {
    vella_nh_destroy(m);
    return rc;
  }
  *out = m;
  return VELLA_OK;
}

int vella_nh_get_cfg(const vella_nh* m, vella_nh_cfg* out) {
  if (!m || !out) return fail(VELLA_E_INVALID, "vella_nh_get_cfg: NULL argument");
  *out = m->cfg;
  return VELLA_OK;
}

int vella_nh_destroy(vella_nh* m) {
  if (!m) return VELLA_OK;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (void* p : m->allocs) cudaFree(p);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
  return VELLA_OK;
}

int vella_nh_tensor(vella_nh* m, const char* name, int32_t layer, void** ptr, size_t* bytes) {
  if (!m || !name || !ptr || !bytes) return fail(VELLA_E_INVALID, "vella_nh_tensor: NULL argument");
  const vella_nh_cfg& c = m->cfg;
  const std::string n(name);
  const size_t e = m->elt, d = (size_t)c.hidden;
  auto ret = [&](void* p, size_t b) -> int {
    if (!p) return fail(VELLA_E_INVALID, "vella_nh_tensor: '%s' does not exist in layer %d", name, layer);
    *ptr = p;
    *bytes = b;
    return VELLA_OK;
  };
  auto lin = [&](const NhLin& l, const std::string& part) -> int {
    if (part == "w") return ret(l.w, l.w_bytes);
    if (part == "s") return ret(l.s, l.sb_bytes);
    if (part == "b") return ret(l.b, l.sb_bytes);
    return fail(VELLA_E_INVALID, "vella_nh_tensor: part '%s'", part.c_str());
  };
  const size_t dot = n.rfind('.');
  const std::string head = dot == std::string::npos ? n : n.substr(0, dot);
  const std::string part = dot == std::string::npos ? "" : n.substr(dot + 1);
  if (n == "embed") return ret(m->embed, (size_t)c.vocab * d * e);
  if (n == "norm_f") return ret(m->norm_f, d * e);
  if (head == "lm_head") return lin(m->lm_head, part);
  if (n.rfind("mtp.", 0) == 0) {
    if (!m->has_mtp) return fail(VELLA_E_INVALID, "vella_nh_tensor: '%s': the model has no MTP head", name);
    NhMtp& t = m->mtp;
    const std::string r = n.substr(4);
    const size_t rdot = r.rfind('.');
    const std::string rh = rdot == std::string::npos ? r : r.substr(0, rdot);
    const std::string rp = rdot == std::string::npos ? "" : r.substr(rdot + 1);
    if (rh == "eh_proj") return lin(t.eh, rp);
    if (r == "enorm") return ret(t.enorm, d * e);
    if (r == "hnorm") return ret(t.hnorm, d * e);
    if (r == "final_norm") return ret(t.final_norm, d * e);
    if (r == "attn_norm") return ret(t.attn.norm, d * e);
    if (rh == "qkv") return lin(t.attn.qkv, rp);
    if (rh == "o") return lin(t.attn.o, rp);
    if (r == "kv") return ret(t.attn.kv, (size_t)2 * c.kv_heads * c.max_seq * c.head_dim * e);
    if (r == "moe_norm") return ret(t.moe.norm, d * e);
    if (r == "router") return ret(t.moe.router, (size_t)c.experts * d * 4);
    if (r == "router_bias") return ret(t.moe.rbias, (size_t)c.experts * 4);
    if (rh == "fc1") return lin(t.moe.fc1, rp);
    if (rh == "fc2") return lin(t.moe.fc2, rp);
    if (rh == "shared_up") return lin(t.moe.sup, rp);
    if (rh == "shared_down") return lin(t.moe.sdown, rp);
    return fail(VELLA_E_INVALID, "vella_nh_tensor: '%s' is not an MTP tensor", name);
  }
  if (layer < 0 || layer >= m->L) return fail(VELLA_E_INVALID, "vella_nh_tensor: layer %d of %d", layer, m->L);
  NhLayer& Ly = m->layers[layer];
  if (n == "norm") return ret(Ly.norm, d * e);
  if (Ly.kind == 'M') {
    if (head == "in_proj") return lin(Ly.in_proj, part);
    if (head == "out_proj") return lin(Ly.out_proj, part);
    if (n == "conv_w") return ret(Ly.conv_w, (size_t)m->conv_dim * c.conv_kernel * e);
    if (n == "conv_b") return ret(Ly.conv_b, (size_t)m->conv_dim * e);
    if (n == "gnorm") return ret(Ly.gnorm, (size_t)m->I * e);
    if (n == "a_log") return ret(Ly.a_log, (size_t)c.m_heads * 4);
    if (n == "dt_bias") return ret(Ly.dt_bias, (size_t)c.m_heads * 4);
    if (n == "D") return ret(Ly.Dv, (size_t)c.m_heads * 4);
    if (n == "conv_state") return ret(Ly.conv_state, (size_t)std::max(c.conv_kernel - 1, 1) * m->conv_dim * e);
    if (n == "ssm_state") return ret(Ly.ssm_state, (size_t)c.m_heads * c.m_head_dim * c.state_dim * 4);
  } else if (Ly.kind == '*') {
    if (head == "qkv") return lin(Ly.qkv, part);
    if (head == "o") return lin(Ly.o, part);
    if (n == "kv") return ret(Ly.kv, (size_t)2 * c.kv_heads * c.max_seq * c.head_dim * e);
  } else {
    if (n == "router") return ret(Ly.router, (size_t)c.experts * d * 4);
    if (n == "router_bias") return ret(Ly.rbias, (size_t)c.experts * 4);
    if (head == "fc1") return lin(Ly.fc1, part);
    if (head == "fc2") return lin(Ly.fc2, part);
    if (head == "shared_up") return lin(Ly.sup, part);
    if (head == "shared_down") return lin(Ly.sdown, part);
  }
  return fail(VELLA_E_INVALID, "vella_nh_tensor: '%s' is not a tensor of layer %d ('%c')", name, layer, Ly.kind);
}

int vella_nh_forward(vella_nh* m, const int32_t* tokens, const void* embeds, int32_t rows, int32_t pos,
                     int32_t logits_rows, int32_t* argmax_out, void* logits_out, void* hidden_out) {
  if (!m || (!tokens == !embeds)) return fail(VELLA_E_INVALID, "vella_nh_forward: tokens or embeddings, one of them");
  const vella_nh_cfg& c = m->cfg;
  if (rows < 1 || rows > c.max_rows || pos < 0 || pos + rows > c.max_seq || logits_rows < 0 || logits_rows > rows ||
      (logits_rows > 0 && !argmax_out))
    return fail(VELLA_E_INVALID, "vella_nh_forward: %d rows at %d (max_rows %d, max_seq %d), %d logits rows", rows, pos,
                c.max_rows, c.max_seq, logits_rows);
  VELLA_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t s = m->stream;
  const int d = c.hidden, dt = c.dtype;
  const size_t e = m->elt;
  int rc;
  VELLA_CUDA_TRY(cudaMemcpyAsync(m->dpos, &pos, sizeof(int), cudaMemcpyHostToDevice, s));
  if (tokens) {
    if ((rc = nh_embed(m, tokens, rows, m->h))) return rc;
  } else {
    VELLA_CUDA_TRY(cudaMemcpyAsync(m->h, embeds, (size_t)rows * d * e, cudaMemcpyDeviceToDevice, s));
  }
  for (int l = 0; l < m->L; ++l) {
    NhLayer& Ly = m->layers[l];
    if (Ly.kind == 'M') rc = nh_mamba_block(m, Ly, m->h, rows);
    else if (Ly.kind == '*') rc = nh_attention_block(m, Ly, m->h, rows);
    else rc = nh_moe_block(m, Ly, m->h, rows);
    if (rc) return rc;
  }
  if (hidden_out) {  // the post-norm hidden states of every row (the MTP head's input)
    if ((rc = launch_rmsnorm(dt, m->xn, m->h, m->norm_f, rows, d, c.eps, s))) return rc;
    VELLA_CUDA_TRY(cudaMemcpyAsync(hidden_out, m->xn, (size_t)rows * d * e, cudaMemcpyDeviceToDevice, s));
  }
  if ((rc = nh_head(m, m->h, m->norm_f, rows, logits_rows, argmax_out, logits_out))) return rc;
  return nh_finish(m, "vella_nh_forward");
}

int vella_nh_mtp_forward(vella_nh* m, const int32_t* next_tokens, const void* next_embeds, const void* hidden,
                         int32_t rows, int32_t pos, int32_t logits_rows, int32_t* argmax_out, void* x_out) {
  if (!m || !hidden || (!next_tokens == !next_embeds))
    return fail(VELLA_E_INVALID, "vella_nh_mtp_forward: a hidden row and one of next tokens / next embeddings");
  if (!m->has_mtp) return fail(VELLA_E_INVALID, "vella_nh_mtp_forward: the model has no MTP head");
  const vella_nh_cfg& c = m->cfg;
  if (rows < 1 || rows > c.max_rows || pos < 0 || pos + rows > c.max_seq || logits_rows < 0 || logits_rows > rows ||
      (logits_rows > 0 && !argmax_out))
    return fail(VELLA_E_INVALID, "vella_nh_mtp_forward: %d rows at %d, %d logits rows", rows, pos, logits_rows);
  VELLA_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t s = m->stream;
  const int d = c.hidden, dt = c.dtype;
  const size_t e = m->elt, row = (size_t)d * e;
  NhMtp& t = m->mtp;
  int rc;
  VELLA_CUDA_TRY(cudaMemcpyAsync(m->dpos, &pos, sizeof(int), cudaMemcpyHostToDevice, s));
  // concat(enorm(embed(next)), hnorm(hidden)) -> eh_proj
  if (next_tokens) {
    if ((rc = nh_embed(m, next_tokens, rows, m->x2))) return rc;
  } else {
    VELLA_CUDA_TRY(cudaMemcpyAsync(m->x2, next_embeds, (size_t)rows * row, cudaMemcpyDeviceToDevice, s));
  }
  if ((rc = launch_rmsnorm(dt, m->xn, m->x2, t.enorm, rows, d, c.eps, s))) return rc;
  VELLA_CUDA_TRY(cudaMemcpy2DAsync(m->cat, 2 * row, m->xn, row, row, rows, cudaMemcpyDeviceToDevice, s));
  if ((rc = launch_rmsnorm(dt, m->xn, hidden, t.hnorm, rows, d, c.eps, s))) return rc;
  VELLA_CUDA_TRY(cudaMemcpy2DAsync(static_cast<char*>(m->cat) + row, 2 * row, m->xn, row, row, rows,
                                   cudaMemcpyDeviceToDevice, s));
  if ((rc = nh_gemm(m, t.eh, m->cat, rows, m->x2, false)) || (rc = nh_attention_block(m, t.attn, m->x2, rows)) ||
      (rc = nh_moe_block(m, t.moe, m->x2, rows)))
    return rc;
  if (x_out) VELLA_CUDA_TRY(cudaMemcpyAsync(x_out, m->x2, (size_t)rows * row, cudaMemcpyDeviceToDevice, s));
  if ((rc = nh_head(m, m->x2, t.final_norm, rows, logits_rows, argmax_out, nullptr))) return rc;
  return nh_finish(m, "vella_nh_mtp_forward");
}

}  // extern "C"
