"""CPU restatement of the speech-LM decode path (test infrastructure only).

* ``forward`` — the dense GQA decoder layer recipe of the reference's Qwen3 text decoder
  (``Worker/Sources/MLXAudioSTT/Qwen3ASR/Qwen3ASRTextDecoder.swift:17-214``): RMSNorm,
  q|k|v projections, optional per-head q/k RMSNorm (``:59-60``), RoPE with the cache
  offset (non-traditional half rotation, ``:76-82``), causal GQA attention (the mask of
  ``NemotronTranscribeDecoder.swift:387-388``), o_proj + residual, RMSNorm, SwiGLU MLP
  (``:110-112``) + residual, final RMSNorm, LM head.  Values are rounded to the activation
  dtype wherever a kernel of the library stores them (after each GEMM, norm, RoPE and the
  attention output); reductions are fp32 in numpy's order.
* ``greedy`` / ``draft_and_verify`` — ``NemotronTranscribeModel.swift:266-290`` and
  ``:306-396``: greedy acceptance (the longest prefix of drafts equal to the target's
  argmax, then the target's bonus token), stop at EOS / max tokens / a repetition loop.
* ``loop_tail`` / ``loop_cut`` / ``ends_in_loop`` — ``NemotronTranscribeText.swift:98-127``
  and ``NemotronTranscribeModel.swift:296-302``; ``retrying_runaway`` — ``:436-443``.
* ``philox4x32_10`` — the counter-based generator (Salmon et al., SC'11) that draws the
  oracle-draft proposals.

Parity: the integer parts are pinned by the reference's known-answer tests
(``tests/test_oracle_pins.py``); the floating-point parts are parity unpinned against MLX
(no MLX outputs exist in the reference repository).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import affine as A

MIN_REPEATS = 20
MAX_PERIOD = 64


# ---------------------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------------------

@dataclass
class Config:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    bits: int = 4
    dtype: str = "bf16"
    qk_norm: bool = False
    rms_eps: float = 1e-6
    rope_theta: float = 1e6


def rope_table(max_seq: int, head_dim: int, theta: float) -> np.ndarray:
    """cos/sin [max_seq, head_dim/2, 2]: angle = pos * theta^(-2i/hd) in double, rounded once
    to fp32."""
    half = head_dim // 2
    t = np.empty((max_seq, half, 2), np.float32)
    inv = [math.pow(theta, -2.0 * i / head_dim) for i in range(half)]
    for pos in range(max_seq):
        for i in range(half):
            a = pos * inv[i]
            t[pos, i, 0] = math.cos(a)
            t[pos, i, 1] = math.sin(a)
    return t


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """y = w * T(x * rsqrt(mean(x^2) + eps)), x and w already rounded to T (fp32 arrays)."""
    ss = (x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True).astype(np.float32)
    r = (np.float32(1) / np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps))).astype(np.float32)
    return A.round_to(w * A.round_to(x * r, dtype), dtype)


# Quantized GEMMs of more than this many rows take the dequantize-then-multiply form (the
# library's tensor-core GEMM; stock MLX quantizedMM at large row counts); up to it, the GEMV's
# product form (SmallMGEMM.swift:662-755).
TILE_ROWS = 16


def linear(x: np.ndarray, W: dict, bits: int, dtype: str, epilogue="none", residual=None, up=None,
           raw: bool = False, call_rows: int = 0) -> np.ndarray:
    """The library GEMM's arithmetic: fp32 accumulation, epilogue, one rounding (none with raw).
    The form follows the row count of the library's call (call_rows, else the rows of x)."""
    xs = A.to_storage(x, dtype)
    res = A.to_storage(residual, dtype) if residual is not None else None
    u = (up["w"], up.get("s"), up.get("b")) if up is not None else None
    form = "tile" if (call_rows or xs.shape[0]) > TILE_ROWS else "product"
    out = A.qgemm(xs, W["w"], W.get("s"), W.get("b"), bits=bits, dtype=dtype, epilogue=epilogue, residual=res, up=u,
                  form=form, raw=raw)
    return out if raw else A.from_storage(out, dtype)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, pos_q: np.ndarray, scale: float, dtype: str):
    """q [Tq, H, hd], k/v [Tk, KV, hd] (positions 0..Tk-1); query at position p sees keys <= p."""
    H, KV = q.shape[1], k.shape[1]
    g = H // KV
    out = np.empty_like(q)
    for h in range(H):
        kh, vh = k[:, h // g, :], v[:, h // g, :]
        s = (q[:, h, :] @ kh.T) * np.float32(scale)
        mask = np.arange(k.shape[0])[None, :] <= pos_q[:, None]
        s = np.where(mask, s, -np.inf).astype(np.float32)
        mx = s.max(axis=1, keepdims=True)
        p = np.where(mask, np.exp(s - mx), 0).astype(np.float32)
        out[:, h, :] = (p @ vh) / p.sum(axis=1, keepdims=True)
    return A.round_to(out, dtype)


def rope(x: np.ndarray, pos: np.ndarray, table: np.ndarray, dtype: str) -> np.ndarray:
    half = x.shape[-1] // 2
    c = table[pos, :, 0][:, None, :]
    s = table[pos, :, 1][:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return A.round_to(np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1), dtype)


def forward(cfg: Config, W: dict, embeds: np.ndarray, table: np.ndarray, raw_logits: bool = False,
            logits_from: int = 0, call_rows: int = 0) -> np.ndarray:
    """Causal forward of the whole sequence of input embeddings [T, d] (fp32, rounded to T);
    returns the logits [T - logits_from, V] of the rows from logits_from on (fp32 values of T;
    with raw_logits, before their final rounding).  The LM head is one GEMM over those rows
    only, as the library runs it, so its row count picks its form; call_rows > 0 says the library
    runs the sequence in calls of at most that many rows, which picks the layers' GEMM form."""
    dt = cfg.dtype
    T = embeds.shape[0]
    H, KV, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    pos = np.arange(T)
    h = embeds.astype(np.float32)
    rows = min(T, call_rows) if call_rows > 0 else T
    for L in W["layers"]:
        xn = rmsnorm(h, L["attn_norm"], cfg.rms_eps, dt)
        qkv = linear(xn, L["qkv"], cfg.bits, dt, call_rows=rows)
        q = qkv[:, :H * hd].reshape(T, H, hd)
        k = qkv[:, H * hd:(H + KV) * hd].reshape(T, KV, hd)
        v = qkv[:, (H + KV) * hd:].reshape(T, KV, hd)
        if cfg.qk_norm:
            q = rmsnorm(q, L["q_norm"], cfg.rms_eps, dt)
            k = rmsnorm(k, L["k_norm"], cfg.rms_eps, dt)
        q = rope(q, pos, table, dt)
        k = rope(k, pos, table, dt)
        att = attention(q, k, v, pos, 1.0 / math.sqrt(hd), dt).reshape(T, H * hd)
        h = linear(att, L["o"], cfg.bits, dt, "residual", residual=h, call_rows=rows)
        xn = rmsnorm(h, L["mlp_norm"], cfg.rms_eps, dt)
        act = linear(xn, L["gate"], cfg.bits, dt, "siluGate", up=L["up"], call_rows=rows)
        h = linear(act, L["down"], cfg.bits, dt, "residual", residual=h, call_rows=rows)
    xn = rmsnorm(h[logits_from:], W["final_norm"], cfg.rms_eps, dt)
    return linear(xn, W["lm_head"], cfg.bits, dt, raw=raw_logits)


def embed_sequence(W: dict, prefix: np.ndarray, tokens) -> np.ndarray:
    rows = [prefix.astype(np.float32)]
    if len(tokens):
        rows.append(W["embed"][np.asarray(tokens, dtype=np.int64)])
    return np.concatenate(rows, axis=0)


SCORE_ROWS = 16  # the library's teacher-forced score runs its positions in calls of 16 rows


def score(cfg: Config, W: dict, prefix: np.ndarray, tokens, table: np.ndarray, raw_logits: bool = False) -> np.ndarray:
    """Logits predicting tokens[0..T) (positions P-1 .. P+T-2), teacher forced, with the GEMM form
    of the library's score (calls of at most SCORE_ROWS rows)."""
    x = embed_sequence(W, prefix, list(tokens)[:-1])
    return forward(cfg, W, x, table, raw_logits, logits_from=prefix.shape[0] - 1, call_rows=SCORE_ROWS)


def first_argmax(row: np.ndarray) -> int:
    return int(np.argmax(row))  # the first index of the maximum, as the library's argmax


# ---------------------------------------------------------------------------------------
# decode loops (integer logic; the target is any callable giving argmax tokens)
# ---------------------------------------------------------------------------------------

def loop_tail(tokens, min_repeats=MIN_REPEATS, max_period=MAX_PERIOD):
    n = len(tokens)
    if min_repeats < 2:
        return None
    for period in range(1, max_period + 1):
        if period * min_repeats > n:
            break
        if all(tokens[n - 1 - i] == tokens[n - 1 - i - period] for i in range(period * (min_repeats - 1))):
            start = n - period * min_repeats
            while start > 0 and tokens[start - 1] == tokens[start - 1 + period]:
                start -= 1
            return start, period
    return None


def loop_cut(tokens):
    t = loop_tail(tokens)
    if t is None:
        return list(tokens), False
    return list(tokens[:t[0] + t[1]]), True


def ends_in_loop(out: list) -> bool:
    if len(out) < MIN_REPEATS or len(out) % 4 != 0:
        return False
    cut, looped = loop_cut(out)
    if looped:
        out[:] = cut
    return looped


def retrying_runaway(max_tokens, draft_and_verify, greedy):
    """Returns (tokens, looped, retried)."""
    first = draft_and_verify()
    if not (first[1] or len(first[0]) >= max_tokens):
        return first[0], first[1], False
    g = greedy()
    return g[0], g[1], True


def greedy(next_token, first: int, max_tokens: int, eos=()):
    """decodeGreedy: ``next_token(seq)`` returns the target's argmax after ``seq``."""
    out, y, looped = [], first, False
    while len(out) < max_tokens:
        if y in eos:
            break
        out.append(y)
        if ends_in_loop(out):
            looped = True
            break
        if len(out) >= max_tokens:
            break
        y = next_token(out)
    return out, looped


def accept(ys, drafts):
    """Greedy acceptance: (accepted count, bonus token)."""
    a = 0
    while a < len(drafts) and ys[a] == drafts[a]:
        a += 1
    return a, ys[a]


def draft_and_verify(verify, propose, first: int, max_tokens: int, k: int, eos=()):
    """decodeMTP with a separate draft: ``propose(out, pass_index)`` -> k drafts,
    ``verify(out, drafts)`` -> the target's k+1 argmax tokens.  Returns (tokens, looped,
    accepted counts per pass)."""
    out, hist = [], []
    if first in eos or max_tokens == 0:
        return out, False, hist
    out.append(first)
    p = 0
    while len(out) < max_tokens:
        drafts = propose(out, p)
        ys = verify(out, drafts)
        a, bonus = accept(ys, drafts)
        hist.append(a)
        p += 1
        for t in list(drafts[:a]) + [bonus]:
            if t in eos:
                return out, False, hist
            out.append(t)
            if len(out) >= max_tokens:
                return out, False, hist
            if ends_in_loop(out):
                return out, True, hist
    return out, False, hist


# ---------------------------------------------------------------------------------------
# Philox-4x32-10 and the oracle-draft proposal rule
# ---------------------------------------------------------------------------------------

M32 = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    c0, c1, c2, c3 = [int(v) & M32 for v in ctr]
    k0, k1 = [int(v) & M32 for v in key]
    for _ in range(10):
        p0 = 0xD2511F53 * c0
        p1 = 0xCD9E8D57 * c2
        hi0, lo0 = p0 >> 32, p0 & M32
        hi1, lo1 = p1 >> 32, p1 & M32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & M32, lo1, (hi0 ^ c3 ^ k1) & M32, lo0
        k0 = (k0 + 0x9E3779B9) & M32
        k1 = (k1 + 0xBB67AE85) & M32
    return c0, c1, c2, c3


def u01(v: int) -> float:
    return float(np.float32(v >> 8) * np.float32(1.0 / 16777216.0))


def oracle_proposal(seed: int, pass_index: int, depth: int, reference_token, p: float, vocab: int) -> int:
    """Draft token at depth ``depth`` of pass ``pass_index``: the reference token with
    probability p, else uniform over the vocabulary (the library's propose kernel)."""
    r = philox4x32_10((pass_index, depth, 0x0D4A7, 0), (seed & M32, seed >> 32))
    if u01(r[0]) < np.float32(p) and reference_token is not None:
        return int(reference_token)
    return min(int(np.float32(u01(r[1])) * np.float32(vocab)), vocab - 1)


# ---------------------------------------------------------------------------------------
# Stochastic acceptance (temperature > 0) and tree verification
# ---------------------------------------------------------------------------------------
# The reference's draft-and-verify is greedy only (NemotronTranscribeModel.swift:364-369).
# The sampled forms follow the published algorithms: speculative sampling (Leviathan, Kalman
# and Matias, ICML 2023; Chen et al. 2023) -- draft x ~ q, accept with probability
# min(1, p(x) / q(x)), on rejection draw from the normalised max(0, p - q), after K
# acceptances draw the bonus from p -- and multi-candidate tree verification (SpecInfer,
# Miao et al. 2023) -- the children of a node are tried in order against the running
# residual r (r = p at the node; after a rejected child, r = normalise(max(0, r - q))); if
# every child is rejected the bonus is drawn from r.  The uniforms are Philox-4x32-10 draws
# on the counter (pass or step, position or node, purpose, stream) with the key (seed low,
# seed high), the first 32-bit word mapped to [0, 1) by its top 24 bits.  Draws from a
# distribution use the inverse CDF in vocabulary order: the first index whose running sum
# exceeds u times the total.  Arithmetic here is float64; every decision also reports its
# margin (the distance of the compared quantities, relative to their scale), so a caller
# comparing with a float32 implementation can tell a rounding-level tie from a real
# difference.

PURPOSE_DRAFT, PURPOSE_ACCEPT, PURPOSE_RESIDUAL = 0x5A3D1, 0xACC01, 0xB0B05
PURPOSE_FIRST, PURPOSE_STEP, PURPOSE_TREE, PURPOSE_PROPOSAL = 0xF1257, 0x57E90, 0x7EE01, 0x0D4A7


def uniform(seed: int, a: int, b: int, purpose: int, stream: int) -> float:
    """u in [0, 1) for the counter (a, b, purpose, stream)."""
    r = philox4x32_10((a, b, purpose, stream), (seed & M32, (seed >> 32) & M32))
    return u01(r[0])


def softmax_t(logits_row, temperature: float) -> np.ndarray:
    """softmax(l / T) in float64 of a logits row (values of the activation dtype)."""
    z = np.asarray(logits_row, np.float64) / float(np.float32(temperature))
    w = np.exp(z - z.max())
    return w / w.sum()


def icdf(weights, u: float):
    """(index, margin) of the inverse-CDF draw from unnormalised weights w >= 0: the first v with
    cumsum(w)[v] > u * sum(w) (the last positive weight when rounding leaves none), -1 when every
    weight is zero.  margin = distance of u * sum(w) to the nearest bin edge / sum(w)."""
    w = np.maximum(np.asarray(weights, np.float64), 0.0)
    tot = w.sum()
    if not tot > 0:
        return -1, np.inf
    cum = np.cumsum(w)
    target = u * tot
    idx = int(np.searchsorted(cum, target, side="right"))
    if idx >= len(w):
        idx = int(np.nonzero(w)[0][-1])
    lo = cum[idx] - w[idx]
    return idx, min(target - lo, cum[idx] - target) / tot


def oracle_draft_q(vocab: int, ref_token, p: float) -> np.ndarray:
    """q of the oracle draft: the reference token with probability p, else uniform (all uniform
    when the position has no reference token)."""
    q = np.full(vocab, (1.0 - p if ref_token is not None else 1.0) / vocab)
    if ref_token is not None:
        q[ref_token] += p
    return q


def sample_drafts(q_rows, temperature: float, seed: int, pass_index: int, stream: int = 0):
    """K draft tokens of a pass, x_i ~ softmax(q_row_i / T) with u(pass, i, DRAFT, stream);
    returns (tokens, min margin)."""
    toks, margin = [], np.inf
    for i, row in enumerate(q_rows):
        t, m = icdf(softmax_t(row, temperature), uniform(seed, pass_index, i, PURPOSE_DRAFT, stream))
        toks.append(max(t, 0))
        margin = min(margin, m)
    return toks, margin


def sampled_accept(p_rows, qs, drafts, temperature: float, seed: int, pass_index: int, stream: int = 0):
    """Speculative sampling over one pass: p_rows are the K + 1 target logits rows (row j at the
    draft's position j), qs the K draft distributions (arrays over the vocabulary), drafts the
    K drafted tokens.  Returns (accepted count a, bonus token, min margin)."""
    K = len(drafts)
    margin = np.inf
    for j in range(K):
        p = softmax_t(p_rows[j], temperature)
        x = drafts[j]
        u = uniform(seed, pass_index, j, PURPOSE_ACCEPT, stream)
        lhs, rhs = u * qs[j][x], p[x]
        margin = min(margin, abs(lhs - rhs) / max(lhs, rhs, 1e-300))
        if lhs < rhs:
            continue
        u2 = uniform(seed, pass_index, j, PURPOSE_RESIDUAL, stream)
        b, m = icdf(np.maximum(p - qs[j], 0.0), u2)
        if b < 0:
            b, m = icdf(p, u2)
        return j, b, min(margin, m)
    p = softmax_t(p_rows[K], temperature)
    b, m = icdf(p, uniform(seed, pass_index, K, PURPOSE_RESIDUAL, stream))
    return K, max(b, 0), min(margin, m)


def tree_topology(branching):
    """Breadth-first tree of the branching factors per depth: (depth, first_child, n_child) per
    node, node 0 the root (the last committed token)."""
    dep, first, nch = [0], [0], [0]
    level = [0]
    for d, b in enumerate(branching):
        nxt = []
        for u in level:
            first[u], nch[u] = len(dep), b
            for _ in range(b):
                nxt.append(len(dep))
                dep.append(d + 1)
                first.append(0)
                nch.append(0)
        level = nxt
    return np.array(dep), np.array(first), np.array(nch)


def tree_children(q_rows, branching, temperature: float, seed: int, pass_index: int, stream: int = 0):
    """Tree tokens of a pass drafted by sampling: every child c of node u is an independent draw
    from softmax(q_rows[u] / T) with u(pass, c, DRAFT, stream).  q_rows maps each node with
    children to its draft logits row.  Returns (tokens of nodes 1.., min margin)."""
    dep, first, nch = tree_topology(branching)
    toks = np.zeros(len(dep), np.int64)
    margin = np.inf
    for u in range(len(dep)):
        if nch[u] == 0:
            continue
        q = softmax_t(q_rows[u], temperature)
        for i in range(nch[u]):
            c = first[u] + i
            t, m = icdf(q, uniform(seed, pass_index, c, PURPOSE_DRAFT, stream))
            toks[c] = max(t, 0)
            margin = min(margin, m)
    return toks, margin


def tree_accept(p_rows, q_of, tokens, branching, temperature: float, seed: int, pass_index: int, stream: int = 0):
    """Multi-candidate acceptance along the tree: p_rows[u] is the target's logits row at node u,
    q_of(u) the draft distribution its children were drawn from, tokens[c] node c's token.
    From the root, the children of the current node are tried in order: child c is accepted
    when u(pass, c, ACCEPT) * q(x_c) < r(x_c), r the running residual (p at the node); after a
    rejection r = normalise(max(0, r - q)).  The first accepted child becomes the current node;
    when all are rejected, the bonus is drawn from r with u(pass, node, RESIDUAL) (from p when r
    is all zero).  Returns (accepted path of nodes, bonus token, min margin)."""
    dep, first, nch = tree_topology(branching)
    path, u, margin = [], 0, np.inf
    while True:
        p = softmax_t(p_rows[u], temperature)
        r = p.copy()
        acc = -1
        if nch[u]:
            q = q_of(u)
            for i in range(nch[u]):
                c = first[u] + i
                x = int(tokens[c])
                ua = uniform(seed, pass_index, c, PURPOSE_ACCEPT, stream)
                lhs, rhs = ua * q[x], r[x]
                margin = min(margin, abs(lhs - rhs) / max(lhs, rhs, 1e-300))
                if lhs < rhs:
                    acc = c
                    break
                r = np.maximum(r - q, 0.0)
                tot = r.sum()
                if tot > 0:
                    r = r / tot
        if acc >= 0:
            path.append(acc)
            u = acc
            continue
        u2 = uniform(seed, pass_index, u, PURPOSE_RESIDUAL, stream)
        b, m = icdf(r, u2)
        if b < 0:
            b, m = icdf(p, u2)
        return path, max(b, 0), min(margin, m)
