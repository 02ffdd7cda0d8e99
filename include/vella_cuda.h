/*
 * vella_cuda.h — C ABI of the B200 (sm_100a) decode path: MLX-affine int4/int8 small-M
 * dequant GEMM, the draft-and-verify decode loop and the fused Whisper decoder step.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and returns a status
 * code.  Device pointers are caller-owned CUDA device memory on the current device;
 * `vella_stream_t` is a `cudaStream_t` (NULL = the legacy default stream).  Calls are
 * asynchronous on the stream unless stated otherwise.  The handle entry points (vella_spec_*,
 * vella_model_*, vella_whisper_*) work on the handle's own non-blocking stream and return when
 * their work is done; that stream does not wait for other streams, so device inputs passed to
 * them must be complete when the call is made.  On any status other than VELLA_OK
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
enum { VELLA_BF16 = 0, VELLA_F16 = 1, VELLA_F32 = 2 };

/* ---- GEMM epilogues (reference SmallMGEMM.EpilogueKind, SmallMGEMM.swift:41) --------- */
enum {
  VELLA_EPI_NONE = 0,
  VELLA_EPI_BIAS = 1,          /* + bias[n]                                               */
  VELLA_EPI_RESIDUAL = 2,      /* + residual[m, n]                                        */
  VELLA_EPI_BIAS_RESIDUAL = 3, /* + bias[n] + residual[m, n]                              */
  VELLA_EPI_SILU_GATE = 4,     /* silu(x . Wg^T) * (x . Wu^T); W = gate, `up_*` = up      */
  /* Whisper's fc1 and convolutions (no counterpart in SmallMGEMM, whose epilogues end above):
   * gelu(acc + bias[n]) with the erf form of GELU, optionally + residual[m, n] after it. */
  VELLA_EPI_BIAS_GELU = 5,
  VELLA_EPI_BIAS_GELU_RESIDUAL = 6
};

/*
 * out[M, N] = epilogue(x[M, K] . W^T), fp32 accumulation, one rounding to `dtype`.
 *   bits = 0     W is dense [N, K] in `dtype` (scales/biases unused).
 *   bits = 4 | 8 W is MLX-affine: packed uint32 [N, K*bits/32] (element i of a word at bits
 *                [bits*i, bits*(i+1)), low first), scales and biases [N, K/64] in `dtype`,
 *                element = scale * q + bias.  M <= 16: accumulated in the product form
 *                sum_g (scale * sum(x*q) + bias * sum(x)) as SmallMGEMM.swift:724.
 *                M > 16 (tensor cores): each weight is rounded once to `dtype` as
 *                scale * q + bias, then accumulated in fp32.
 * group_size must be 64 when bits != 0.  x, residual, out are row-major with row stride K
 * (x) or N (residual, out).  M may be any size; K a multiple of 64.
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
 * zero again), used by one stream at a time; calls of different shapes may share it (the
 * counters occupy a fixed 128 KiB region at its front).  NULL selects a per-device workspace owned
 * by the library: it is allocated or grown by the first call that needs more, so that
 * call must not be inside CUDA graph capture; a grown workspace keeps the old buffer
 * alive, so graphs captured earlier stay valid, but they all share one buffer and must
 * not run concurrently.
 * The reduction order of a row depends only on (N, K, bits) and on the call's row class
 * (1-16, 17-256, above 256 rows): a row of a call of M <= 16 rows is bit-identical to the same
 * row computed alone, and a row of a call of 17-256 rows (above 256) to the same row in any
 * other call of 17-256 rows (above 256).
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

/* ---- weight preparation ------------------------------------------------------------- */

/*
 * MLX-affine quantize on the device (quantize-at-load): w [N, K] in `src_dtype` (VELLA_F32,
 * VELLA_BF16 or VELLA_F16) -> packed uint32 [N, K*bits/32], scales and biases [N, K/64] in
 * desc->dtype.  desc supplies n, k, bits (4 | 8), group_size (64), dtype; m and epilogue are
 * ignored.  Replaces MLX.quantized(_:groupSize:bits:mode: .affine) at
 * Worker/Sources/MLXAudioSTT/Precision/DerivedPrecision.swift:138 and
 * NemotronTranscribe/NemotronTranscribeRecipe.swift:48.
 */
VELLA_API int vella_quantize(const vella_qgemm_desc* desc, int32_t src_dtype, const void* w, void* packed,
                             void* scales, void* biases, vella_stream_t stream);

/* n values ~ N(mean, std^2) in `dtype` from Philox-4x32-10 keyed by (seed, tensor): the
 * synthetic inputs and weights of the benchmarks (value i uses counter i/4, lane i%4). */
VELLA_API int vella_fill_normal(void* out, size_t n, int32_t dtype, uint64_t seed, uint32_t tensor, float mean,
                                float std, vella_stream_t stream);

/* ---- resident decoder model ------------------------------------------------------------
 * A dense GQA transformer (Qwen3 text-decoder recipe, Worker/Sources/MLXAudioSTT/Qwen3ASR/
 * Qwen3ASRTextDecoder.swift:17-214): RMSNorm, RoPE (half rotation, base rope_theta),
 * optional per-head q/k RMSNorm, SwiGLU MLP, final RMSNorm, LM head.  Every linear
 * (q|k|v, o, gate, up, down, lm_head) is `bits` = 0 (dense) or MLX-affine 4/8-bit g64; the
 * token embedding is dense.  The model owns its weights, one KV cache of max_seq positions
 * and a buffer of max_prefix input embeddings (positions below the prefix length take
 * their input embedding from it, later positions from the token table).
 */
typedef struct vella_model_cfg {
  int32_t n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn, vocab;
  int32_t bits;       /* 0, 4 or 8 */
  int32_t dtype;      /* VELLA_BF16 | VELLA_F16 */
  int32_t qk_norm;    /* 1: RMSNorm over head_dim on q and k before RoPE */
  int32_t max_seq;    /* KV capacity in positions */
  int32_t max_prefix; /* capacity of the input-embedding prefix */
  float rms_eps;
  float rope_theta;
  int32_t streams;    /* independent sequences held at once (0 or 1: one); each has its own KV
                         cache [max_seq] and prefix buffer [max_prefix] */
  int32_t rows_per_stream; /* decode rows per stream and forward, logits included (0: 16; up to
                              64: tree verification needs one row per tree node) */
} vella_model_cfg;

typedef struct vella_model vella_model;

VELLA_API int vella_model_create(const vella_model_cfg* cfg, int32_t device, vella_model** out);
VELLA_API int vella_model_destroy(vella_model* model);
/* Synthetic weights: linears ~N(0, std^2) (quantized on the device when bits != 0), norm
 * weights ~N(1, 0.1^2), token embedding ~N(0, 1); Philox keyed by `seed`. */
VELLA_API int vella_model_init_random(vella_model* model, uint64_t seed, float std);
/* Device pointer and size of a tensor, for loading real weights or reading them back.
 * Names: "embed", "final_norm", "prefix", "logits", "kv", "lm_head.w|s|b", and per layer
 * "attn_norm", "mlp_norm", "q_norm", "k_norm", "qkv.w|s|b" (rows q, then k, then v),
 * "o.w|s|b", "gate.w|s|b", "up.w|s|b", "down.w|s|b". */
VELLA_API int vella_model_tensor(vella_model* model, const char* name, int32_t layer, void** ptr, size_t* bytes);
/* The decode loop's repetition guard on host tokens (host-only): returns 1 when the tokens end
 * in one block of at most 64 tokens repeated at least 20 times, and sets *kept to the length
 * up to and including the block's first copy (NemotronTranscribeLoop.tail / cut,
 * NemotronTranscribeText.swift:98-127); else 0 and *kept = n.  check_every_fourth: only when
 * n >= 20 and n % 4 == 0 (endsInLoop, NemotronTranscribeModel.swift:296-302).  A negative
 * status is an error. */
VELLA_API int vella_loop_cut(const int32_t* tokens, int32_t n, int32_t check_every_fourth, int32_t* kept);
/* The RoPE table the model handles use, [max_seq][head_dim / 2] (cos, sin) fp32 pairs (host memory;
 * host-only): angle = pos * theta^(-2i / head_dim) in double, rounded once to fp32 (the
 * non-traditional RoPE of Qwen3ASRTextDecoder.swift:47 and :76-82). */
VELLA_API int vella_rope_table(int32_t max_seq, int32_t head_dim, float theta, float* out);
/* Decode-sized forwards (at most 16 rows, no tree) of a model whose shapes suit it (dense or
 * int4 weights whose GEMMs take the streaming kernel, head_dim 128, no q/k norm) run as one
 * persistent cooperative launch -- every layer's ops separated by grid barriers, the weights
 * streaming across them -- instead of seven launches per layer; off by default (the per-op
 * kernels are faster at the benchmark's 30B-class shapes).  It computes the
 * per-op kernels' arithmetic (bit for bit for dense weights; for int4 GEMMs that the per-op
 * path splits over two CTAs per SM, the split-K boundaries differ, a rounding-level difference);
 * every decode-sized forward agrees with every other bit for bit, so draft-and-verify still
 * equals greedy.  on = 0 selects the per-op kernels (for comparisons);
 * on = 1 for a model that cannot take it returns VELLA_E_UNSUPPORTED.  No counterpart in the
 * reference (MLX schedules its own kernels). */
VELLA_API int vella_model_set_persistent(vella_model* model, int32_t on);
/* The configuration the model was created with. */
VELLA_API int vella_model_get_cfg(const vella_model* model, vella_model_cfg* out);
VELLA_API size_t vella_model_weight_bytes(const vella_model* model);
/*
 * Teacher-forced scoring (the backbone over a whole prompt, as llm.backbone(...) +
 * lmHead in NemotronTranscribeModel.swift:316-322): runs the prefix embeddings [P, d]
 * (host or device, model dtype) then tokens[0..T-1] (host) through a fresh cache and
 * writes the logits that predict each token, rows for positions P-1 .. P+T-2, to
 * logits_out [T, vocab] (host when on_host, else device).  Synchronous.
 */
VELLA_API int vella_model_score(vella_model* model, const void* prefix, int32_t P, const int32_t* tokens, int32_t T,
                                void* logits_out, int32_t on_host);

/* ---- draft-and-verify decode (NemotronTranscribeModel.decodeMTP, :306-396) ---------- */
enum { VELLA_DRAFT_MODEL = 0, VELLA_DRAFT_ORACLE = 1 };
enum { VELLA_DECODE_AUTO = 0, VELLA_DECODE_SPEC = 1, VELLA_DECODE_GREEDY = 2 };
enum { VELLA_FAULT_NONE = 0, VELLA_FAULT_THROW = 1, VELLA_FAULT_NONFINITE = 2 };
enum { VELLA_FLAG_LOOPED = 1, VELLA_FLAG_FELL_BACK = 2, VELLA_FLAG_RUNAWAY_RETRY = 4, VELLA_FLAG_CAPACITY = 8 };

typedef struct vella_spec_cfg {
  int32_t draft_k;    /* drafts per pass, 1..15 (reference draftDepth, :23-24) */
  int32_t draft_mode; /* VELLA_DRAFT_MODEL: the draft model's greedy tokens;
                         VELLA_DRAFT_ORACLE: each proposal is the reference token with
                         probability oracle_p, else uniform over the vocabulary (Philox) */
  float oracle_p;
  uint64_t seed;      /* Philox key of the oracle proposals */
  int32_t n_eos;
  int32_t eos[8];
  int32_t use_graphs; /* 1: replay each pass as one CUDA graph */
  /* 0: greedy acceptance (argmax; the reference's decodeMTP, :364-369).  > 0: stochastic
   * acceptance at this temperature, which the reference does not have (speculative sampling:
   * Leviathan et al. 2023, Chen et al. 2023): tokens follow softmax(logits / temperature) of
   * the target exactly.  The draft samples its proposals from softmax(draft logits /
   * temperature) (the oracle draft keeps its mixture: reference token with probability
   * oracle_p, else uniform); draft j is accepted when u < p(x_j) / q(x_j); at the first
   * rejection the token is drawn from max(0, p - q) renormalised; after K acceptances the
   * bonus token is drawn from p.  The first token after the prefill and plain (greedy-mode)
   * steps are drawn from p.  Uniforms are Philox-4x32-10 keyed by `seed`, with counters
   * (pass or step, position, purpose, stream), so a run is reproducible. */
  float temperature;
  /* Tree verification when tree_depth > 0 (the reference verifies one chain; tree attention
   * after SpecInfer, Miao et al. 2023): the draft expands a tree depth by depth, node i at
   * depth d having tree_branching[d] children (nodes in breadth-first order, at most 64 with
   * the root); with temperature 0 the children are the draft's top-b tokens, with temperature
   * > 0 b independent samples (the oracle draft: each child the reference token with
   * probability oracle_p while its ancestors follow the reference, else uniform).  One
   * target forward verifies every node (each attends to the committed tokens and its own
   * ancestors); greedy acceptance follows the child equal to the target's argmax, stochastic
   * acceptance tries the children in order against the running residual; the accepted
   * path's K/V are moved to consecutive cache slots.  draft_k is ignored.  The target must be
   * created with rows_per_stream >= the node count.  Greedy tree decoding follows the same
   * argmax rule as a chain but sums a node's ancestor keys in another order, so its tokens
   * can differ from a chain decode's where two logits tie to rounding. */
  int32_t tree_depth;
  int32_t tree_branching[8];
} vella_spec_cfg;

typedef struct vella_spec_stats {
  int64_t passes;          /* draft+verify passes          */
  int64_t greedy_steps;    /* single-token target steps    */
  int64_t accepted[16];    /* passes that accepted i drafts */
  int64_t fallbacks;       /* runtime failures -> greedy (sticky) */
  int64_t runaway_retries; /* looping draft-and-verify runs decoded again greedy */
  int32_t draft_disabled;  /* sticky fallback in force */
  float last_decode_ms;    /* device time of the last vella_spec_decode after its prefill */
  int32_t last_tokens;
  float last_prefill_ms;   /* device time of the last prefill */
} vella_spec_stats;

typedef struct vella_spec vella_spec;

/* target: the verifying model; draft: the proposing model (NULL: greedy only).  Both
 * must share the vocabulary; the handle owns its stream and is single-threaded. */
VELLA_API int vella_spec_create(vella_model* target, vella_model* draft, const vella_spec_cfg* cfg, vella_spec** out);
VELLA_API int vella_spec_destroy(vella_spec* spec);
/* Input embeddings of the request: [T, d_target] and [T, d_draft] (NULL keeps what is
 * already in the models' "prefix" buffers). */
VELLA_API int vella_spec_set_prefix(vella_spec* spec, const void* target_embeds, const void* draft_embeds, int32_t T,
                                    int32_t on_host);
/* Reference continuation for VELLA_DRAFT_ORACLE (token i is the one at position T + i). */
VELLA_API int vella_spec_set_reference(vella_spec* spec, const int32_t* tokens, int32_t n);
/* Prefill both models over the prefix; *first = the target's greedy token after it. */
VELLA_API int vella_spec_prefill(vella_spec* spec, int32_t* first);
/* One pass: K draft steps, one target forward over K+1 positions (causal KV append),
 * greedy acceptance, KV rollback past the first mismatch.  Writes the accepted drafts and
 * the target's bonus token (1..K+1 tokens).  VELLA_E_NONFINITE when the verify logits
 * hold NaN/Inf (reference :356-363). */
VELLA_API int vella_spec_step(vella_spec* spec, int32_t* out_tokens, int32_t* n_out);
/* One plain greedy target step (reference decodeGreedy, :266-290). */
VELLA_API int vella_spec_greedy_step(vella_spec* spec, int32_t* out_token);
/*
 * A whole decode (reference decode/decodeMTP/decodeGreedy/retryingRunaway, :266-443):
 * prefill, then passes (SPEC), single steps (GREEDY) or, for AUTO, draft-and-verify with
 * the reference's fallbacks: a runtime failure re-decodes plain greedy and keeps the draft
 * off until vella_spec_reset (sticky); a run that loops or reaches max_tokens is decoded
 * again greedy.  Stops at an EOS token (not emitted), at max_tokens, or at a repetition
 * loop (cut to one copy).  *flags: VELLA_FLAG_*.
 */
VELLA_API int vella_spec_decode(vella_spec* spec, int32_t mode, int32_t max_tokens, int32_t* out_tokens, int32_t cap,
                                int32_t* n_out, int32_t* flags);
/*
 * Several independent streams at once (models created with cfg.streams = S > 1; the single-
 * stream calls above then return VELLA_E_UNSUPPORTED).  vella_spec_set_prefix takes the
 * embeddings stream-major [S][T][d], vella_spec_set_reference the continuations [S][n].
 * Every pass runs the draft steps and the verify of all S streams as one batch (verify rows
 * S * (K + 1)); each stream accepts on its own and stops advancing once it has max_tokens
 * tokens.  out_tokens [S][max_tokens] receives each stream's first max_tokens tokens (no EOS
 * or loop stop: the caller applies its own rules per stream); n_out[S] = max_tokens.
 * mode: VELLA_DECODE_SPEC or VELLA_DECODE_GREEDY (one batched greedy step per token).
 * Batching changes which GEMM path a row takes (at most 16 rows: the small-M kernels; above:
 * tensor cores), so SPEC and GREEDY give bit-identical tokens when their batches fall on the
 * same side (S * (K + 1) <= 16, or S > 16), and a stream's tokens can differ in rounding from
 * a single-stream decode of the same prefix.
 */
VELLA_API int vella_spec_decode_batch(vella_spec* spec, int32_t mode, int32_t max_tokens, int32_t* out_tokens,
                                      int32_t* n_out);
VELLA_API int vella_spec_get_stats(const vella_spec* spec, vella_spec_stats* out);
/* Device pointer and size of a decoder buffer, for inspecting the last pass (no counterpart in
 * the reference, whose decode state is MLX arrays the caller can read; the parity tests replay
 * a pass's acceptance from these).  Names: "draft_rows" [K or tree nodes][S][vocab] the draft
 * logits rows the last pass sampled from (temperature > 0 with the model draft), "draft_stats"
 * their (max, sum) float pairs, "tokens" [S][max_seq] int32 (committed tokens, and beyond the
 * committed length the last pass's rejected drafts), "tree_tokens" [S][nodes] int32,
 * "tree_topology" int32 depth[nodes] | first_child[nodes] | n_child[nodes].  The buffers
 * belong to the decoder; the next call rewrites them. */
VELLA_API int vella_spec_tensor(vella_spec* spec, const char* name, void** ptr, size_t* bytes);
/* Test hook mirroring VELLA_TEST_OPTIMIZED_FAULT (NemotronTranscribeModel.swift:398-399). */
VELLA_API int vella_spec_set_fault(vella_spec* spec, int32_t fault);
/* Clear the sticky fallback and the statistics. */
VELLA_API int vella_spec_reset(vella_spec* spec);

/* ---- Whisper encoder + decoder step ------------------------------------------------------
 *
 * Replaces WhisperModel's encoder call and WhisperFusedDecoder.step / pipelinedGreedy
 * (Worker/Sources/MLXAudioSTT/Whisper/WhisperLayers.swift:110-329, WhisperFusedDecode.swift:
 * 105-141, WhisperModel.swift:341-400) for one audio stream: the encoder (conv1 -> GELU ->
 * conv2 -> GELU -> + sinusoid positions -> pre-LN blocks -> LayerNorm), the cross-attention
 * K/V of every decoder layer projected once, then decoder steps (self-attention over the KV
 * cache, cross-attention over the encoder frames, GELU MLP, tied vocabulary projection) with
 * the token choice on the device, one CUDA graph per step: plain argmax, or the reference's
 * token rules (vella_whisper_set_rules) and sampled fallback attempts
 * (vella_whisper_set_sampling).
 */
typedef struct vella_whisper_cfg {
  int32_t n_mels;      /* mel bins (80 | 128)                                           */
  int32_t d_model;     /* multiple of 64; head_dim = d_model / heads must be 64 or 128   */
  int32_t heads;
  int32_t enc_layers;
  int32_t dec_layers;
  int32_t ffn;         /* multiple of 64 */
  int32_t vocab;
  int32_t n_audio;     /* encoder frames = mel frames / 2 (1500 for 30 s) */
  int32_t max_target;  /* decoder positions (448) */
  int32_t bits;        /* decoder Linears and token embedding: 0 (dense), 4 or 8 (MLX affine, g64) */
  int32_t dtype;       /* VELLA_F16 | VELLA_BF16 */
  float eps;           /* LayerNorm epsilon (1e-5) */
  /* Independent audio streams held by the handle (0 or 1: one).  Each has its own window,
   * cross-attention K/V, self-attention cache and tokens; vella_whisper_decode_batch steps
   * all of them with one decoder forward per token (one row per stream).  The reference runs
   * one window per model call (WhisperModel.swift:341-400). */
  int32_t streams;
} vella_whisper_cfg;

typedef struct vella_whisper_stats {
  float encode_ms;   /* last vella_whisper_encode: encoder + cross K/V projections (device time) */
  float prefill_ms;  /* last decode: the prompt's forward and first token                     */
  float decode_ms;   /* last decode: every following step                                     */
  int32_t tokens;    /* tokens produced by the last decode                                    */
  float sum_logprob; /* with token rules set: the log-probabilities of the chosen tokens of the
                        last decode (end-of-text included), summed in step order (stream 0)    */
} vella_whisper_stats;

/* Token rules of the reference's GPU-side greedy (WhisperModel.pipelinedGreedy with its rule
 * masks, WhisperModel.swift:311-372): per step the suppress list (and at the first step the
 * begin-suppress list) is masked; the token's log-probability is taken under the final row;
 * no-timestamps is never chosen; the first token is a timestamp in
 * [timestamp_begin, timestamp_begin + round(n_audio / 30)]; text is masked when the
 * timestamps' total probability beats every text token; after a timestamp, timestamps are
 * masked when the token before it was one too (or there is none), else text below eot. */
typedef struct vella_whisper_rules {
  int32_t eot;
  int32_t no_timestamps;
  int32_t timestamp_begin;
  const int32_t* suppress;        /* host array of token ids */
  int32_t n_suppress;
  const int32_t* begin_suppress;  /* host array of token ids, first step only */
  int32_t n_begin_suppress;
} vella_whisper_rules;

typedef struct vella_whisper vella_whisper;

VELLA_API int vella_whisper_create(const vella_whisper_cfg* cfg, int32_t device, vella_whisper** out);
VELLA_API int vella_whisper_destroy(vella_whisper* w);
/* Synthetic weights: Linears ~N(0, std) (decoder Linears and the token embedding quantized
 * when bits != 0), biases ~N(0, std) except k_proj's (zero), LayerNorm gains ~N(1, 0.1) and
 * offsets ~N(0, std), encoder positions = the sinusoid table, decoder positions ~N(0, std). */
VELLA_API int vella_whisper_init_random(vella_whisper* w, uint64_t seed, float std);
/* Device view of a tensor (layer = -1 for whole-model tensors).  Linears: "<name>.w" (dense
 * [N, K] or packed codes), "<name>.s", "<name>.b" (MLX scales/biases), "<name>.bias";
 * LayerNorms: "<name>.weight", "<name>.bias".  Encoder layers: enc.ln1, enc.qkv (q|k|v rows,
 * k's bias zero), enc.o, enc.ln2, enc.fc1, enc.fc2; decoder layers: dec.ln1, dec.qkv, dec.o,
 * dec.ln2, dec.cq, dec.ckv (cross k|v rows, k's bias zero), dec.co, dec.ln3, dec.fc1, dec.fc2;
 * whole model: conv1 (K padded to a multiple of 64 with zero columns), conv2, enc_pos,
 * enc_ln, dec_ln, embed (token embedding = vocabulary projection), dec_pos, and the
 * activations enc_out [n_audio, d_model] (the last encoded window), xkv (the cross-
 * attention K|V of every stream and decoder layer, [streams][dec_layers][n_audio][2 d_model])
 * and kv (the self-attention cache, [streams][dec_layers][K, V][heads][max_target][head_dim]).
 * Setting VELLA_WHISPER_FUSE=0 in the environment before vella_whisper_create gives a handle
 * that runs the decoder's LayerNorms and K/V appends as launches of their own instead of in
 * the neighbouring kernels (the same values; for comparisons). */
/* Whisper's log-mel input features of `streams` windows of 16 kHz mono audio (device
 * pointers; window s at audio + s * n_samples), each padded with zeros or trimmed to 30 s
 * (480000 samples): reflect-padded STFT (400-point periodic Hann window, hop 160, 3000
 * frames), power spectrum, Slaney mel filterbank (80 or 128 bins), log10 floored at the
 * window's maximum - 8, (x + 4) / 4; out [streams][n_mels][3000] fp32, the layout
 * vella_whisper_encode reads.  Replaces WhisperAudio.encoderFeatures (WhisperAudio.swift:
 * 7-93) with MLXAudioCore.melFilters (MLXAudioCore/DSP.swift:44-135). */
/* The Slaney mel filterbank vella_whisper_log_mel projects on, [201][n_mels] fp32 row-major
 * (host memory; host-only): MLXAudioCore.melFilters(sampleRate: 16000, nFft: 400, nMels:,
 * fMin: 0, fMax: 8000, norm: "slaney", melScale: .slaney), MLXAudioCore/DSP.swift:44-135. */
VELLA_API int vella_whisper_mel_filters(int32_t n_mels, float* out);
VELLA_API int vella_whisper_log_mel(const float* audio, int64_t n_samples, int32_t streams, int32_t n_mels,
                                    float* out, vella_stream_t stream);
/* The log-mel features of every stream's window (audio [streams][n_samples], on the host or
 * the device), then vella_whisper_encode over them. */
VELLA_API int vella_whisper_encode_audio(vella_whisper* w, const float* audio, int64_t n_samples, int32_t on_host);
/* The encoder position table the handle computes, [length][channels] fp32 before its rounding to
 * the activation dtype (host memory; host-only): WhisperModel.whisperSinusoids (WhisperModel.swift:
 * 554-569), double trig rounded once to fp32. */
VELLA_API int vella_whisper_sinusoids(int32_t length, int32_t channels, float* out);
/* The configuration the handle was created with. */
VELLA_API int vella_whisper_get_cfg(const vella_whisper* w, vella_whisper_cfg* out);
VELLA_API int vella_whisper_tensor(vella_whisper* w, const char* name, int32_t layer, void** ptr, size_t* bytes);
/* Encoder over one window per stream: mel fp32 [streams][n_mels][2 * n_audio] (host or
 * device), then the cross-attention K/V of every decoder layer, per stream. */
VELLA_API int vella_whisper_encode(vella_whisper* w, const float* mel, int32_t on_host);
/* Greedy decode after the prompt (n_prompt <= 16 tokens): up to max_tokens tokens, stopping
 * after `eot` when eot >= 0 (not emitted).  out_tokens (host) receives *n_out tokens. */
VELLA_API int vella_whisper_decode(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t max_tokens,
                                   int32_t eot, int32_t* out_tokens, int32_t* n_out);
/* Greedy decode of every stream (streams > 1 or 1): the same prompt (n_prompt <= 16) for
 * each, then max_tokens tokens per stream, one decoder forward of `streams` rows per token
 * (one CUDA graph), no end-of-text stop.  out_tokens (host) [streams][max_tokens].  The
 * stats' tokens field counts all streams' tokens. */
VELLA_API int vella_whisper_decode_batch(vella_whisper* w, const int32_t* prompt, int32_t n_prompt,
                                         int32_t max_tokens, int32_t* out_tokens);
/* The same with an end-of-text id: the host checks every stream's tokens once per burst of 8
 * steps and stops when every stream has produced `eot` (or after max_tokens); n_out[s] counts
 * stream s's tokens before its end-of-text, later entries of its out_tokens row are -1.  With
 * token rules set each stream's log-probability sum stops at its end-of-text step. */
VELLA_API int vella_whisper_decode_batch_eot(vella_whisper* w, const int32_t* prompt, int32_t n_prompt,
                                             int32_t max_tokens, int32_t eot, int32_t* out_tokens, int32_t* n_out);
/* The summed log-probabilities of the last decode's first n streams (token rules set; zeros
 * otherwise). */
VELLA_API int vella_whisper_get_logprobs(const vella_whisper* w, float* out, int32_t n);
/* Token by token (the reference's step-by-step loop for streaming callers, WhisperModel.swift:
 * 244-276): vella_whisper_begin runs the prompt and returns the first token; each
 * vella_whisper_step runs one decoder step (the captured graph) and returns the next.  The
 * token rules, sampling and log-probability sum apply as in vella_whisper_decode; the caller
 * stops at end-of-text.  One-stream handles. */
VELLA_API int vella_whisper_begin(vella_whisper* w, const int32_t* prompt, int32_t n_prompt, int32_t* first);
VELLA_API int vella_whisper_step(vella_whisper* w, int32_t* token);
/* Token rules for the following decodes (NULL: plain argmax, the default).  The ids must lie
 * in the vocabulary with eot < timestamp_begin; the masks are built on the device here. */
VELLA_API int vella_whisper_set_rules(vella_whisper* w, const vella_whisper_rules* rules);
/* Temperature of the following decodes (the reference's fallback attempts, WhisperModel.swift:
 * 218-292, and its sample() at :447-454): 0 is argmax; at temperature > 0 (token rules
 * required) each step draws argmax(final / temperature + Gumbel noise), the noise from
 * Philox-4x32-10 keyed by `seed` on counter (token / 4, step, stream, draw), word token % 4,
 * u = (2 * (bits >> 9) + 1) / 2^24, noise -log(-log u).  The caller picks `draw` (e.g. the
 * attempt index) so that attempts draw different noise and a request replays exactly.  The
 * log-probability sum in the stats stays that of the unscaled final row, as the reference's. */
VELLA_API int vella_whisper_set_sampling(vella_whisper* w, float temperature, uint64_t seed, uint32_t draw);
/* Teacher-forced logits [T, vocab] (dtype) of the token sequence (positions 0..T-1); one-
 * stream handles only (as vella_whisper_decode). */
VELLA_API int vella_whisper_score(vella_whisper* w, const int32_t* tokens, int32_t T, void* logits, int32_t on_host);
VELLA_API int vella_whisper_get_stats(const vella_whisper* w, vella_whisper_stats* out);

/* Message of the last failing call on this thread ("" when none); returns its length. */
VELLA_API size_t vella_last_error(char* buf, size_t cap);

/* Diagnostic with no counterpart in the reference: nonzero when a TMA/tensor-core pipeline
 * wait inside a kernel ran out of time since the last clear (bits 0-7: small-M streaming GEMM,
 * bits 8-15: tensor-core GEMM, bits 16-23: persistent decode forward).  The kernel that gave
 * up finished without its result.
 * Synchronises with the device; clear != 0 resets the flags. */
VELLA_API int32_t vella_fault_flags(int32_t clear);

/* Library version string, e.g. "vella-b200 0.1 sm_100a". */
VELLA_API const char* vella_version(void);

/* ---- checkpoints (safetensors) ----------------------------------------------------------
 *
 * Replaces MLX.loadArrays over a model directory's *.safetensors shards (merged in the
 * caller's order, later keys winning: WhisperModel.swift:676-684) and WhisperModel's key
 * sanitising and derived precision (:483-651, :686-701).  Files are memory-mapped; tensor
 * data pointers stay valid until vella_st_close.  Host-only: no device work.
 */
enum {
  VELLA_ST_BF16 = 0, VELLA_ST_F16 = 1, VELLA_ST_F32 = 2, VELLA_ST_U32 = 3, VELLA_ST_I32 = 4, VELLA_ST_U8 = 5,
  VELLA_ST_I8 = 6, VELLA_ST_I64 = 7, VELLA_ST_F64 = 8, VELLA_ST_U16 = 9, VELLA_ST_I16 = 10, VELLA_ST_BOOL = 11,
  VELLA_ST_U64 = 12, VELLA_ST_F8_E4M3 = 13, VELLA_ST_F8_E5M2 = 14
};
typedef struct vella_st vella_st;
VELLA_API int vella_st_open(const char* const* paths, int32_t n_paths, vella_st** out);
VELLA_API int vella_st_close(vella_st* st);
VELLA_API int vella_st_count(const vella_st* st, int32_t* n);
/* index of `name`, or -1 */
VELLA_API int vella_st_find(const vella_st* st, const char* name, int32_t* index);
/* any output may be NULL; shape holds up to 8 dimensions */
VELLA_API int vella_st_info(const vella_st* st, int32_t index, const char** name, int32_t* dtype, int32_t* ndim,
                            int64_t* shape, const void** data, size_t* bytes);
/* Whether a Hugging Face (model.encoder.layers.N...) or OpenAI/mlx-whisper (encoder.blocks.N...)
 * checkpoint holds every tensor a handle of `cfg` needs, with matching shapes (float, or
 * MLX-affine group 64 with the handle's bits for the decoder Linears and token embedding).
 * A float checkpoint loaded into an int4/int8 handle is the reference's derived precision
 * (WhisperModel.swift:694-701): the decoder Linears and the token embedding are quantized at
 * load, and the encoder Linears, which the handle runs dense, hold their quantized values
 * dequantized; the convolutions and position tables stay float.  Quantized encoder Linears of
 * an already-quantized checkpoint are dequantized, its float ones kept.  Host-only;
 * VELLA_E_INVALID names the first problem. */
VELLA_API int vella_whisper_check_checkpoint(const vella_st* st, const vella_whisper_cfg* cfg);
/* Fills the handle's weights from the checkpoint (checked first: a failed check leaves the
 * handle unchanged).  q|k|v rows are concatenated with k's bias zero, cross k|v likewise;
 * conv weights are read as PyTorch [out, in, 3] (Hugging Face) or [out, 3, in] (mlx-whisper);
 * the encoder position table is kept (computed) unless the checkpoint supplies one.  The
 * next decode needs a new vella_whisper_encode. */
VELLA_API int vella_whisper_load(vella_whisper* w, const vella_st* st);
/* The same for a Qwen3-style decoder model (Qwen3ASRTextDecoder.swift:17-214, keys as
 * Qwen3ASRModel.sanitize leaves them, :682-708, a "thinker." prefix stripped):
 * model.embed_tokens (dense in the handle: an MLX-affine embedding is dequantized),
 * model.norm, lm_head (the embedding when the checkpoint has none: tied), and per layer
 * input_layernorm, post_attention_layernorm, self_attn.{q,k,v,o}_proj (q|k|v rows
 * concatenated), self_attn.{q,k}_norm when cfg.qk_norm, mlp.{gate,up,down}_proj; float
 * Linears of an int4/int8 model are quantized at load. */
VELLA_API int vella_model_check_checkpoint(const vella_st* st, const vella_model_cfg* cfg);
VELLA_API int vella_model_load(vella_model* model, const vella_st* st);

/* ---- Nemotron-H Mamba-2 mixer core ------------------------------------------------------
 *
 * Replaces NTMamba's conv, SSM and gated norm (Worker/Sources/MLXAudioSTT/NemotronTranscribe/
 * NemotronTranscribeDecoder.swift:126-360: nt_ssm_kernel, nt_ssm_initial_kernel, ntSSMAttn,
 * ntComputeDt, NTGatedRMSNorm).  Rows are stream-major (row s * tokens + t).  `zxbcdt` is the
 * in_proj output, rows of in_stride elements: gate [0, I), conv input [I, I + convDim), dt
 * [I + convDim, I + convDim + heads), I = heads * head_dim, convDim = I + 2 * groups *
 * state_dim.  Device pointers, asynchronous on `stream`; the in_proj / out_proj GEMMs are
 * vella_qgemm calls.
 */
typedef struct vella_mamba_desc {
  int32_t streams, tokens;  /* S sequences, T new positions each (1: decode step; more: chunk)  */
  int32_t heads, head_dim;  /* mamba_num_heads, mamba_head_dim                                  */
  int32_t groups;           /* n_groups (divides heads)                                         */
  int32_t state_dim;        /* ssm_state_size: a multiple of 32, at most 256                    */
  int32_t conv_kernel;      /* conv_kernel (1..8)                                               */
  int32_t dtype;            /* VELLA_BF16 | VELLA_F16 (activations, conv weight and state)      */
  int32_t in_stride;        /* elements between rows of zxbcdt (>= I + convDim + heads)         */
  float dt_min, dt_max;     /* time_step_limit                                                  */
  float eps;                /* layer_norm_epsilon of the gated norm                             */
} vella_mamba_desc;
/* xbc [S*T][convDim] = silu(causal depthwise conv over conv_state [S][K-1][convDim] then the T
 * conv inputs; conv_w [convDim][K], conv_b [convDim] or NULL); conv_state keeps the last K-1
 * conv inputs. */
VELLA_API int vella_mamba_conv(const vella_mamba_desc* desc, const void* zxbcdt, const void* conv_w,
                               const void* conv_b, void* conv_state, void* xbc, vella_stream_t stream);
/* y [S*T][I]: per head h (group h / (heads / groups)) and channel d, for each row in order,
 * dt = clip(softplus(dt_raw + dt_bias[h]), dt_min, dt_max), state = exp(-exp(a_log[h]) dt)
 * state + x dt B, y = state . C + x D[h]; ssm_state [S][H][Dh][Ds] fp32, read and written. */
VELLA_API int vella_mamba_ssm(const vella_mamba_desc* desc, const void* xbc, const void* zxbcdt, const float* a_log,
                              const float* dt_bias, const float* D, float* ssm_state, void* y, vella_stream_t stream);
/* out [S*T][I] = rms_norm(y * silu(gate)) over groups of I / groups channels, times norm_w [I]. */
VELLA_API int vella_mamba_gated_norm(const vella_mamba_desc* desc, const void* y, const void* zxbcdt,
                                     const void* norm_w, void* out, vella_stream_t stream);

/* ---- Nemotron-H MoE router -------------------------------------------------------------
 *
 * Replaces NTMoE's routing (NemotronTranscribeDecoder.swift:487-496): p = sigmoid(x . W^T) in
 * fp32; the top_k experts of p + e_score_correction_bias (ties: lower expert index), listed by
 * descending biased score; weights p at them, divided by their sum (+ 1e-20) when norm_topk
 * and top_k > 1, times `scaling`.  x [rows][hidden] (dtype), router_w [experts][hidden] fp32,
 * bias [experts] fp32; expert_idx [rows][top_k] int32, expert_w [rows][top_k] fp32.
 */
typedef struct vella_moe_route_desc {
  int32_t rows, hidden, experts, top_k;  /* hidden <= 16384, experts <= 1024, top_k <= 32 */
  int32_t norm_topk;                     /* norm_topk_prob */
  float scaling;                         /* routed_scaling_factor */
  int32_t dtype;                         /* VELLA_BF16 | VELLA_F16 */
} vella_moe_route_desc;
VELLA_API int vella_moe_route(const vella_moe_route_desc* desc, const void* x, const float* router_w,
                              const float* bias, int32_t* expert_idx, float* expert_w, vella_stream_t stream);

/* ---- Nemotron-H routed experts -----------------------------------------------------------
 *
 * Replaces NTSwitchMLP + NTMoE's weighted sum (NemotronTranscribeDecoder.swift:435-499):
 * out[m] (+)= sum_j expert_w[m][j] * fc2_e(relu(fc1_e(x[m]))^2), e = expert_idx[m][j].  The
 * experts' weights are stacked [experts][out][in]: MLX-affine (bits 4 | 8, group 64: packed
 * uint32 [E][out][in*bits/32], scales and biases [E][out][in/64] in dtype) or dense (bits 0,
 * [E][out][in] in dtype).  fc1 is [E][inter][hidden], fc2 [E][hidden][inter].  The shared
 * expert (NTMLP, relu^2) is the same call with one expert, every row choosing it at weight 1,
 * and accumulate = 1.  rows * top_k <= 4096 pairs; hidden and inter in 64..8192.
 */
typedef struct vella_moe_experts_desc {
  int32_t rows, hidden, inter, experts, top_k;
  int32_t bits;   /* 0, 4 or 8 */
  int32_t dtype;  /* VELLA_BF16 | VELLA_F16 */
} vella_moe_experts_desc;
VELLA_API size_t vella_moe_experts_workspace_size(const vella_moe_experts_desc* desc);
VELLA_API int vella_moe_experts(const vella_moe_experts_desc* desc, const void* x, const int32_t* expert_idx,
                                const float* expert_w, const void* fc1_w, const void* fc1_scales,
                                const void* fc1_biases, const void* fc2_w, const void* fc2_scales,
                                const void* fc2_biases, void* out, int32_t accumulate, void* workspace,
                                size_t workspace_bytes, vella_stream_t stream);

/* ---- Nemotron-H backbone -----------------------------------------------------------------
 *
 * Replaces NTBackbone + the LM head (NemotronTranscribeDecoder.swift:508-571): a stack of
 * Mamba-2 ('M'), attention without positional encoding ('*') and MoE ('E') blocks, each
 * x + mixer(rmsnorm(x)), then norm_f, lm_head and argmax; one sequence per handle, the Mamba
 * states and attention caches held in it.  Weights and states are filled / read through
 * vella_nh_tensor: "embed" [vocab][hidden], "norm_f", "lm_head.w|s|b"; per layer "norm" and
 * M: "in_proj.w|s|b" [I + convDim + m_heads][hidden], "out_proj.w|s|b", "conv_w", "conv_b",
 *    "gnorm", "a_log", "dt_bias", "D" (fp32), "conv_state", "ssm_state" (fp32);
 * *: "qkv.w|s|b" [(heads + 2 kv_heads) head_dim][hidden] (rows q | k | v), "o.w|s|b", "kv";
 * E: "router", "router_bias" (fp32), "fc1.w|s|b" [experts][moe_inter][hidden], "fc2.w|s|b",
 *    "shared_up.w|s|b" [shared_inter][hidden], "shared_down.w|s|b".
 * Linears are MLX-affine at `bits` (4 | 8, group 64) or dense (0).
 */
typedef struct vella_nh_cfg {
  int32_t vocab, hidden, heads, kv_heads, head_dim;        /* head_dim 64 | 128            */
  int32_t m_heads, m_head_dim, state_dim, conv_kernel, groups;
  int32_t moe_inter, shared_inter, experts, top_k, norm_topk;
  float routed_scaling, dt_min, dt_max, eps;
  int32_t bits, dtype;
  int32_t max_seq;   /* attention cache positions */
  int32_t max_rows;  /* rows per forward (1..512)  */
  int32_t mtp;       /* 1: the MTP head (NTMTP: eh_proj, norms, attention + MoE block, own cache) */
  char pattern[128]; /* one of M, *, E per layer, NUL-terminated */
} vella_nh_cfg;
typedef struct vella_nh vella_nh;
VELLA_API int vella_nh_create(const vella_nh_cfg* cfg, int32_t device, vella_nh** out);
VELLA_API int vella_nh_destroy(vella_nh* model);
VELLA_API int vella_nh_tensor(vella_nh* model, const char* name, int32_t layer, void** ptr, size_t* bytes);
VELLA_API int vella_nh_get_cfg(const vella_nh* model, vella_nh_cfg* out);
/* A Nemotron-H checkpoint: NVIDIA's NeMo keys (llm.model.*, experts stored [E][in][out], the MTP
 * head's llm.mtp.* keys) or the MLX module tree (llm.backbone.*, lm_head, mtp.*), float (quantized
 * at load for an int4/int8 handle) or MLX-affine at the handle's bits (NemotronTranscribeKeys.map,
 * NemotronTranscribeText.swift:369-397; NemotronTranscribeModel.loadWeights :127-175). */
VELLA_API int vella_nh_check_checkpoint(const vella_st* st, const vella_nh_cfg* cfg);
VELLA_API int vella_nh_load(vella_nh* model, const vella_st* st);
/* Runs `rows` new positions pos .. pos + rows - 1 (host tokens, or device embeddings [rows][hidden]:
 * exactly one of them); the argmax of the last logits_rows rows into argmax_out (host), their
 * logits into logits_out (device, may be NULL), the post-norm_f hidden states of every row into
 * hidden_out (device [rows][hidden], may be NULL).  Synchronous. */
VELLA_API int vella_nh_forward(vella_nh* model, const int32_t* tokens, const void* embeds, int32_t rows, int32_t pos,
                               int32_t logits_rows, int32_t* argmax_out, void* logits_out, void* hidden_out);
/* The MTP head over `rows` pairs (next token or next embedding row, hidden row): x =
 * eh_proj(concat(enorm(embed(next)),
 * hnorm(hidden))), then its attention block (cache positions pos ..) and MoE block; x into
 * x_out (device [rows][hidden], may be NULL: the next chained call's hidden), the argmax of
 * lm_head(final_norm(x)) of the last logits_rows rows into argmax_out (host).  MTP tensors are
 * "mtp.eh_proj.w|s|b", "mtp.enorm", "mtp.hnorm", "mtp.attn_norm", "mtp.qkv.w|s|b", "mtp.o.w|s|b",
 * "mtp.kv", "mtp.moe_norm", "mtp.router", "mtp.router_bias", "mtp.fc1/fc2/shared_up/shared_down.w|s|b",
 * "mtp.final_norm".  Synchronous. */
VELLA_API int vella_nh_mtp_forward(vella_nh* model, const int32_t* next_tokens, const void* next_embeds,
                                   const void* hidden, int32_t rows, int32_t pos, int32_t logits_rows,
                                   int32_t* argmax_out, void* x_out);

#ifdef __cplusplus
}
#endif

#endif /* VELLA_CUDA_H */
