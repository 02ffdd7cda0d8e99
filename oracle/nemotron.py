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
reference's SSD chunk form, and the tests check that the two agree in float64.  Parity
unpinned: the reference has no numeric fixtures for these layers.
"""
from __future__ import annotations

import numpy as np


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
