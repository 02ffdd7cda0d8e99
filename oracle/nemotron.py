"""CPU restatement of Nemotron-H's Mamba-2 mixer core and MoE routing (test infrastructure only).

Follows ``Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeDecoder.swift``:
  * ``NTMamba.callAsFunction`` (:340-360): the in_proj output splits into gate [I], the conv
    input [convDim = I + 2 G Ds] and dt [H]; the conv input runs through a causal depthwise
    Conv1d of kernel K over the cached K - 1 previous inputs (the cache keeps the last K - 1),
    then SiLU; the result splits into x [H, Dh], B [G, Ds], C [G, Ds];
  * ``ntComputeDt`` (:214-216): dt = clip(softplus(dt + dt_bias), lo, hi) in fp32;
  * the SSM (``nt_ssm_kernel`` :126-152 for one token, ``nt_ssm_initial_kernel`` :154-194 for
    a chunk without a state, ``ntSSMAttn`` :225-276, the SSD chunk form, with a state): per
    head h of group g = h / (H / G), state[d, s] <- exp(-exp(A_log[h]) dt) state[d, s] +
    x[d] dt B[g, s]; y[d] = sum_s state[d, s] C[g, s] + x[d] D[h]; the state is fp32;
  * ``NTGatedRMSNorm`` (:301-316): v = y * silu(gate) in fp32, RMS-normalised over groups of
    I / G elements (no weight), then times the weight.
  * ``NTMoE`` routing (:487-496): sigmoid router scores in fp32, top-k by score plus the
    correction bias, weights from the unbiased scores (optionally normalised), times the
    routed scaling factor.

``ssm_scan`` is the sequential form the library's kernel computes; ``ssm_ssd`` restates the
reference's SSD chunk form, and the tests check that the two agree in float64.  The whole
hybrid model (Mamba, attention without positional encoding, MoE blocks; the MTP head) and the
reference's greedy and MTP draft-and-verify loops, with the Mamba snapshot/restore rollback,
are restated at the end; the tests check that the draft-and-verify tokens equal greedy's.
Parity unpinned: the reference has no numeric fixtures for these layers.
"""
from __future__ import annotations

import numpy as np

from .decoder import ends_in_loop


def silu(x):
    x = np.asarray(x, np.float64)
    return x / (1.0 + np.exp(-x))


def softplus(x):
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def compute_dt(dt_raw, dt_bias, lo: float, hi: float):
    """[T, H] raw dt from in_proj -> clip(softplus(dt + bias), lo, hi)."""
    return np.clip(softplus(np.asarray(dt_raw, np.float64) + np.asarray(dt_bias, np.float64)), lo, hi)


def conv_step(x, weight, bias, state):
    """Causal depthwise conv of x [T, C] after the cached state [K-1, C] (weight [C, K], bias
    [C] or None), then SiLU.  Returns (out [T, C], new state [K-1, C])."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    K = w.shape[1]
    padded = np.concatenate([np.asarray(state, np.float64), x], axis=0)  # [K-1+T, C]
    T = x.shape[0]
    out = np.zeros_like(x)
    for t in range(T):
        out[t] = (padded[t:t + K] * w.T).sum(axis=0)
    if bias is not None:
        out = out + np.asarray(bias, np.float64)
    return silu(out), padded[T:].copy() if K > 1 else padded[:0].copy()


def split_xbc(xbc, H: int, Dh: int, G: int, Ds: int):
    """[T, convDim] -> x [T, H, Dh], B [T, G, Ds], C [T, G, Ds]."""
    T = xbc.shape[0]
    I = H * Dh
    x = xbc[:, :I].reshape(T, H, Dh)
    B = xbc[:, I:I + G * Ds].reshape(T, G, Ds)
    C = xbc[:, I + G * Ds:I + 2 * G * Ds].reshape(T, G, Ds)
    return x, B, C


def ssm_scan(x, B, C, dt, a_log, D, state):
    """Sequential selective scan: x [T, H, Dh], B/C [T, G, Ds], dt [T, H] (already through
    compute_dt), a_log/D [H], state [H, Dh, Ds].  Returns (y [T, H, Dh], state)."""
    x = np.asarray(x, np.float64)
    T, H, Dh = x.shape
    G = B.shape[1]
    hpg = H // G
    st = np.asarray(state, np.float64).copy()
    y = np.zeros_like(x)
    A = -np.exp(np.asarray(a_log, np.float64))
    for t in range(T):
        for h in range(H):
            g = h // hpg
            dA = np.exp(A[h] * dt[t, h])
            st[h] = dA * st[h] + (x[t, h] * dt[t, h])[:, None] * np.asarray(B[t, g], np.float64)[None, :]
            y[t, h] = st[h] @ np.asarray(C[t, g], np.float64) + x[t, h] * float(D[h])
    return y, st


def ssm_ssd(x, B, C, dt, a_log, D, state):
    """The reference's SSD chunk form (``ntSSMAttn``): within the chunk y = (L o C B^T) (dt x)
    with L[i, j] = exp(sum_{j<k<=i} dt_k A) for j <= i, plus the carried state's contribution
    exp(cumsum(dt A)) C . state; the new state is sum_j exp(sum_{j<k} dt_k A) dt_j x_j B_j^T
    plus exp(sum dt A) . state."""
    x = np.asarray(x, np.float64)
    T, H, Dh = x.shape
    G = B.shape[1]
    hpg = H // G
    A = -np.exp(np.asarray(a_log, np.float64))
    y = np.zeros_like(x)
    new = np.zeros((H, Dh, B.shape[2]))
    for h in range(H):
        g = h // hpg
        a = dt[:, h] * A[h]                        # [T]
        cs = np.cumsum(a)                          # inclusive
        Lm = np.zeros((T, T))
        for i in range(T):
            for j in range(i + 1):
                Lm[i, j] = np.exp(cs[i] - cs[j])
        CB = np.asarray(C[:, g], np.float64) @ np.asarray(B[:, g], np.float64).T   # [T, T]
        dtx = dt[:, h][:, None] * x[:, h]          # [T, Dh]
        y[:, h] = (Lm * CB) @ dtx
        y[:, h] += np.exp(cs)[:, None] * (np.asarray(C[:, g], np.float64) @ np.asarray(state[h], np.float64).T)
        w = np.exp(cs[-1] - cs)                    # decay from step j to the chunk end
        new[h] = (dtx * w[:, None]).T @ np.asarray(B[:, g], np.float64) + np.exp(cs[-1]) * np.asarray(state[h], np.float64)
        y[:, h] += x[:, h] * float(D[h])
    return y, new


def gated_rmsnorm(y, gate, weight, groups: int, eps: float):
    """[T, I] y and gate -> rms_norm(y * silu(gate)) over groups of I / groups, times weight."""
    v = np.asarray(y, np.float64) * silu(gate)
    T, I = v.shape
    gs = I // groups
    v = v.reshape(T, groups, gs)
    v = v / np.sqrt((v * v).mean(axis=-1, keepdims=True) + eps)
    return v.reshape(T, I) * np.asarray(weight, np.float64)


def mixer(zxbcdt, conv_w, conv_b, a_log, dt_bias, D, norm_w, conv_state, ssm_state, *, H, Dh, G, Ds, lo, hi, eps):
    """The mixer between in_proj and out_proj for one stream: zxbcdt [T, I + convDim + H].
    Returns (normalised gated output [T, I], conv state, ssm state)."""
    I = H * Dh
    conv_dim = I + 2 * G * Ds
    gate = zxbcdt[:, :I]
    conv_in = zxbcdt[:, I:I + conv_dim]
    dt_raw = zxbcdt[:, I + conv_dim:I + conv_dim + H]
    xbc, conv_state = conv_step(conv_in, conv_w, conv_b, conv_state)
    x, B, C = split_xbc(xbc, H, Dh, G, Ds)
    dt = compute_dt(dt_raw, dt_bias, lo, hi)
    y, ssm_state = ssm_scan(x, B, C, dt, a_log, D, ssm_state)
    out = gated_rmsnorm(y.reshape(-1, I), gate, norm_w, G, eps)
    return out, conv_state, ssm_state


def moe_route(x, router_w, bias, top_k: int, norm_topk: bool, scaling: float):
    """``NTMoE`` routing (NemotronTranscribeDecoder.swift:487-496): p = sigmoid(x . W^T) in
    fp32, experts chosen by the top_k of p + e_score_correction_bias (ties: lowest index; the
    reference's argPartition leaves their order unspecified), weights p at the chosen experts,
    divided by their sum (+ 1e-20) when norm_topk and top_k > 1, times the routed scaling
    factor.  x [M, hidden], router_w [E, hidden].  Returns (idx [M, k] in descending biased
    score, weight [M, k], biased scores [M, E])."""
    logits = np.asarray(x, np.float64) @ np.asarray(router_w, np.float64).T
    p = 1.0 / (1.0 + np.exp(-logits))
    biased = p + np.asarray(bias, np.float64)
    M, E = biased.shape
    idx = np.zeros((M, top_k), np.int64)
    for m in range(M):
        order = sorted(range(E), key=lambda e: (-biased[m, e], e))
        idx[m] = order[:top_k]
    w = np.take_along_axis(p, idx, axis=1)
    if top_k > 1 and norm_topk:
        w = w / (w.sum(axis=1, keepdims=True) + 1e-20)
    return idx, w * scaling, biased


# ---------------------------------------------------------------------------------------
# A whole hybrid model (NemotronTranscribeDecoder.swift:330-627) and its greedy and MTP
# draft-and-verify loops (NemotronTranscribeModel.swift:263-396), in float64, for small
# random models: the reference's rollback (Mamba states restored from a snapshot, attention
# caches trimmed, the accepted prefix fed again) must give exactly the greedy tokens.
# ---------------------------------------------------------------------------------------

from dataclasses import dataclass, field  # noqa: E402


@dataclass
class HybridConfig:
    vocab: int = 12
    hidden: int = 32
    heads: int = 4
    kv_heads: int = 2
    head_dim: int = 8
    m_heads: int = 4
    m_head_dim: int = 8
    state: int = 32
    conv_k: int = 4
    groups: int = 2
    eps: float = 1e-5
    moe_inter: int = 16
    shared_inter: int = 24
    experts: int = 8
    top_k: int = 2
    norm_topk: bool = True
    scaling: float = 1.5
    dt_lo: float = 0.0
    dt_hi: float = float("inf")
    pattern: str = "M*EM*E"

    @property
    def m_inner(self):
        return self.m_heads * self.m_head_dim

    @property
    def conv_dim(self):
        return self.m_inner + 2 * self.groups * self.state


def random_hybrid(c: HybridConfig, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    r = lambda *s, sc=0.3: rng.standard_normal(s) * sc  # noqa: E731
    d = c.hidden

    def attn():
        return {"q": r(c.heads * c.head_dim, d), "k": r(c.kv_heads * c.head_dim, d),
                "v": r(c.kv_heads * c.head_dim, d), "o": r(d, c.heads * c.head_dim)}

    def moe():
        return {"router": r(c.experts, d), "bias": r(c.experts, sc=0.1), "fc1": r(c.experts, c.moe_inter, d),
                "fc2": r(c.experts, d, c.moe_inter), "up": r(c.shared_inter, d), "down": r(d, c.shared_inter)}

    layers = []
    for kind in c.pattern:
        L = {"kind": kind, "norm": 1.0 + r(d, sc=0.1)}
        if kind == "M":
            L.update(in_proj=r(c.m_inner + c.conv_dim + c.m_heads, d), out_proj=r(d, c.m_inner),
                     conv_w=r(c.conv_dim, c.conv_k), conv_b=r(c.conv_dim, sc=0.1), a_log=r(c.m_heads),
                     dt_bias=r(c.m_heads), D=r(c.m_heads), norm_w=1.0 + r(c.m_inner, sc=0.1))
        elif kind == "*":
            L.update(attn())
        else:
            L.update(moe())
        layers.append(L)
    mtp = {"eh": r(d, 2 * d), "enorm": 1.0 + r(d, sc=0.1), "hnorm": 1.0 + r(d, sc=0.1),
           "attn_norm": 1.0 + r(d, sc=0.1), "attn": attn(), "moe_norm": 1.0 + r(d, sc=0.1), "moe": moe(),
           "final_norm": 1.0 + r(d, sc=0.1)}
    return {"embed": r(c.vocab, d, sc=1.0), "layers": layers, "norm_f": 1.0 + r(d, sc=0.1),
            "lm_head": r(c.vocab, d), "mtp": mtp}


def rmsnorm(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * w


class KV:
    """An attention cache: rows appended, trim(n) drops the last n (NTKVCache.update/trim)."""

    def __init__(self):
        self.k = None
        self.v = None

    def append(self, k, v):
        self.k = k if self.k is None else np.concatenate([self.k, k])
        self.v = v if self.v is None else np.concatenate([self.v, v])
        return self.k, self.v

    def trim(self, n):
        if n > 0 and self.k is not None:
            self.k, self.v = self.k[:-n], self.v[:-n]


def attention(c: HybridConfig, W, x, kv: KV):
    """No positional encoding; causal when several rows (NTAttention, :384-391)."""
    T = x.shape[0]
    q = (x @ W["q"].T).reshape(T, c.heads, c.head_dim)
    keys, vals = kv.append((x @ W["k"].T).reshape(T, c.kv_heads, c.head_dim),
                           (x @ W["v"].T).reshape(T, c.kv_heads, c.head_dim))
    S = keys.shape[0]
    g = c.heads // c.kv_heads
    out = np.zeros((T, c.heads, c.head_dim))
    for h in range(c.heads):
        s = q[:, h] @ keys[:, h // g].T / np.sqrt(c.head_dim)      # [T, S]
        if T > 1:
            pos = S - T + np.arange(T)
            s = np.where(np.arange(S)[None, :] <= pos[:, None], s, -np.inf)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h] = (p / p.sum(axis=1, keepdims=True)) @ vals[:, h // g]
    return out.reshape(T, -1) @ W["o"].T


def moe_experts(x, idx, w, fc1, fc2):
    """NTSwitchMLP and the weighted sum (:435-499): out[m] = sum_j w[m, j] fc2[e] (relu(fc1[e]
    x[m])^2), e = idx[m, j]; fc1 [E, inter, hidden], fc2 [E, hidden, inter]."""
    x = np.asarray(x, np.float64)
    out = np.zeros_like(x)
    for m in range(x.shape[0]):
        for j in range(idx.shape[1]):
            e = idx[m, j]
            h = np.maximum(np.asarray(fc1[e], np.float64) @ x[m], 0.0)
            out[m] += w[m, j] * (np.asarray(fc2[e], np.float64) @ (h * h))
    return out


def moe(c: HybridConfig, W, x):
    """NTMoE: routed relu^2 experts weighted, plus the shared relu^2 MLP (:435-496)."""
    idx, w, _ = moe_route(x, W["router"], W["bias"], c.top_k, c.norm_topk, c.scaling)
    sh = np.maximum(x @ W["up"].T, 0.0)
    return moe_experts(x, idx, w, W["fc1"], W["fc2"]) + (sh * sh) @ W["down"].T


def make_cache(c: HybridConfig):
    return [{"conv": np.zeros((c.conv_k - 1, c.conv_dim)), "state": np.zeros((c.m_heads, c.m_head_dim, c.state))}
            if k == "M" else (KV() if k == "*" else None) for k in c.pattern]


def backbone(c: HybridConfig, P, x, cache):
    """NTBackbone over rows x [T, hidden] with the caches; hidden states after norm_f."""
    h = np.asarray(x, np.float64)
    for L, lc in zip(P["layers"], cache):
        z = rmsnorm(h, L["norm"], c.eps)
        if L["kind"] == "M":
            zx = z @ L["in_proj"].T
            o, lc["conv"], lc["state"] = mixer(zx, L["conv_w"], L["conv_b"], L["a_log"], L["dt_bias"], L["D"],
                                               L["norm_w"], lc["conv"], lc["state"], H=c.m_heads, Dh=c.m_head_dim,
                                               G=c.groups, Ds=c.state, lo=c.dt_lo, hi=c.dt_hi, eps=c.eps)
            h = h + o @ L["out_proj"].T
        elif L["kind"] == "*":
            h = h + attention(c, L, z, lc)
        else:
            h = h + moe(c, L, z)
    return rmsnorm(h, P["norm_f"], c.eps)


def head(P, h):
    return np.argmax(np.asarray(h) @ P["lm_head"].T, axis=-1)


def mtp_forward(c: HybridConfig, P, e, h, kv: KV):
    """NTMTP (:585-606): x = eh_proj(concat(enorm(e), hnorm(h))); + attention; + MoE; returns
    (x, final_norm(x))."""
    M = P["mtp"]
    x = np.concatenate([rmsnorm(e, M["enorm"], c.eps), rmsnorm(h, M["hnorm"], c.eps)], axis=-1) @ M["eh"].T
    x = x + attention(c, M["attn"], rmsnorm(x, M["attn_norm"], c.eps), kv)
    x = x + moe(c, M["moe"], rmsnorm(x, M["moe_norm"], c.eps))
    return x, rmsnorm(x, M["final_norm"], c.eps)


def decode_greedy(c: HybridConfig, P, embeddings, max_tokens: int, eos=(), info=None):
    """decodeGreedy (:266-290): the prefix, then one token per backbone step, stopping at a
    repetition loop (endsInLoop, :285 and :296-302; ``info["looped"]`` is set)."""
    cache = make_cache(c)
    t = int(head(P, backbone(c, P, embeddings, cache)[-1]))
    out = []
    if info is not None:
        info["looped"] = False
    while len(out) < max_tokens and t not in eos:
        out.append(t)
        if ends_in_loop(out):
            if info is not None:
                info["looped"] = True
            break
        t = int(head(P, backbone(c, P, P["embed"][[t]], cache)[-1]))
    return out


def decode_mtp(c: HybridConfig, P, embeddings, max_tokens: int, depth: int, eos=(), info=None):
    """decodeMTP (:306-396): depth chained MTP drafts verified by one backbone pass; on a
    partial acceptance the Mamba states go back to the pass's snapshot, the attention caches
    drop the whole feed, and the accepted prefix is fed again with the next drafts; the MTP
    cache drops its depth - 1 chain entries every pass; the decode stops at a repetition loop
    (endsInLoop, :390; ``info["looped"]`` is set).  Returns (tokens, accepted counts)."""
    if info is not None:
        info["looped"] = False
    cache, mcache = make_cache(c), KV()
    post = backbone(c, P, embeddings, cache)
    t = int(head(P, post[-1]))
    out, hist = [], []
    if t in eos or max_tokens == 0:
        return out, hist
    out.append(t)
    embed = lambda toks: P["embed"][np.asarray(toks, np.int64)]  # noqa: E731

    def chain(x0, first):
        drafts, token, x = [first], first, x0
        for _ in range(depth - 1):
            nx, xo = mtp_forward(c, P, embed([token]), x, mcache)
            x, token = nx, int(head(P, xo[-1]))
            drafts.append(token)
        return drafts

    nxt = np.concatenate([np.asarray(embeddings, np.float64)[1:], embed([t])])
    x, xo = mtp_forward(c, P, nxt, post, mcache)
    drafts = chain(x[-1:], int(head(P, xo[-1])))
    pending, mtp_done = [t], 0
    while len(out) < max_tokens:
        snapshot = [(lc["conv"].copy(), lc["state"].copy()) if isinstance(lc, dict) else None for lc in cache]
        fed = pending + drafts
        verified = backbone(c, P, embed(fed), cache)
        ys = head(P, verified)
        k, a = len(pending), 0
        while a < len(drafts) and ys[k - 1 + a] == drafts[a]:
            a += 1
        bonus = int(ys[k - 1 + a])
        new = drafts[:a] + [bonus]
        hist.append(a)
        mcache.trim(depth - 1)
        upto = k + a
        e_next = (fed[1:upto] + [bonus])[mtp_done:]
        nx, nxo = mtp_forward(c, P, embed(e_next), verified[mtp_done:upto], mcache)
        drafts = chain(nx[-1:], int(head(P, nxo[-1])))
        if a == len(fed) - k:
            pending, mtp_done = [bonus], 0
        else:
            for lc, snap in zip(cache, snapshot):
                if isinstance(lc, dict):
                    lc["conv"], lc["state"] = snap
                elif isinstance(lc, KV):
                    lc.trim(len(fed))
            pending, mtp_done = fed[:upto] + [bonus], upto
        for tok in new:
            if tok in eos:
                return out, hist
            out.append(tok)
            if len(out) >= max_tokens:
                return out, hist
            if ends_in_loop(out):
                if info is not None:
                    info["looped"] = True
                return out, hist
    return out, hist
