"""CPU restatement of the Whisper encoder and decoder step (test infrastructure only).

Follows the reference's Whisper layers and fused decode step:
  * encoder — ``Worker/Sources/MLXAudioSTT/Whisper/WhisperLayers.swift:110-157``: conv1 (k 3,
    s 1, p 1) -> GELU -> conv2 (k 3, s 2, p 1) -> GELU -> + sinusoid positions -> pre-LN
    blocks (self-attention without mask, GELU MLP) -> final LayerNorm;
  * attention — ``:11-73``: k_proj has no bias, scale head_dim ** -0.5;
  * decoder — ``:170-329`` and the fused step ``WhisperFusedDecode.swift:105-141``: token +
    learned position embedding, per layer self-attention over the KV cache (causal), cross-
    attention over the encoder output (K/V projected once), GELU MLP, each behind a
    LayerNorm with a residual add; final LayerNorm; logits through the tied token embedding
    (``:326-328``); q|k|v of the self-attention as one projection with k's bias zero
    (``WhisperFusedDecode.swift:67-88``);
  * sinusoids — ``WhisperModel.swift:554-569``: double-precision trig rounded to fp32, then
    to the table dtype;
  * quantization recipe of config 1 — ``WhisperModel.swift:697-703``: every decoder Linear and
    the token embedding MLX-affine (group 64), positional tables float.

Arithmetic as the library's kernels store it: every GEMM accumulates in fp32 and rounds
once after its epilogue (bias, GELU, residual); LayerNorm statistics in fp32 with the
normalised value rounded to the activation dtype before ``w * x + b`` (``WhisperFusedDecode
.swift:204-251``, the MLX row algorithm, here with one final rounding); GELU is the erf form.
Greedy argmax, plain or under the token rules of the reference's GPU-side greedy
(``WhisperModel.swift:311-372``, ``rule_select`` below); the temperature fallback's sampled
attempts, compression ratio and attempt verdict (``WhisperModel.swift:218-292, 434-454``,
``rule_sample`` / ``attempt_verdict`` below).

Parity: the reference (Swift + MLX) cannot run on this machine; the floating-point
arithmetic is parity unpinned against MLX.  The sinusoid table rule is pinned by the
reference test ``WhisperStockDTypeTests.swift:42-46`` (table shape and dtype).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import affine as A
from . import decoder as D


@dataclass
class WhisperConfig:
    n_mels: int = 80
    d_model: int = 384
    heads: int = 6
    enc_layers: int = 4
    dec_layers: int = 4
    ffn: int = 1536
    vocab: int = 51865
    n_audio: int = 1500        # encoder frames (3000 mel frames / 2)
    max_target: int = 448
    bits: int = 4              # decoder Linears and token embedding (0: dense)
    dtype: str = "f16"
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads


def sinusoids(length: int, channels: int, dtype: str = "f16") -> np.ndarray:
    """WhisperModel.swift:554-569: Double trig -> Float32, rounded once to the table dtype."""
    half = channels // 2
    inc = math.log(10000.0) / max(half - 1, 1)
    out = np.empty((length, channels), np.float32)
    for i in range(half):
        t = np.arange(length, dtype=np.float64) * math.exp(-inc * i)
        out[:, i] = np.sin(t).astype(np.float32)
        out[:, half + i] = np.cos(t).astype(np.float32)
    return A.from_storage(A.to_storage(out, dtype), dtype)


def rnd(x: np.ndarray, dtype: str) -> np.ndarray:
    return A.from_storage(A.to_storage(np.asarray(x, np.float32), dtype), dtype)


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    x = x.astype(np.float32)
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    c = x - mean
    var = (c * c).mean(axis=-1, keepdims=True, dtype=np.float32)
    xh = rnd(c / np.sqrt(var + np.float32(eps)), dtype)
    return rnd(w.astype(np.float32) * xh + b.astype(np.float32), dtype)


def linear(x, W, bits, dtype, bias=None, gelu_out=False, residual=None):
    """GEMM with the library's epilogue: fp32 accumulation, + bias, GELU, + residual, one rounding."""
    xs = A.to_storage(x, dtype)
    acc = A.qgemm(xs, W["w"], W.get("s"), W.get("b"), bits=bits, dtype=dtype, raw=True)
    if bias is not None:
        acc = acc + bias.astype(np.float32)[None, :]
    if gelu_out:
        acc = A.gelu(acc)
    if residual is not None:
        acc = acc + residual.astype(np.float32)
    return rnd(acc, dtype)


def attention(q, k, v, heads, causal_pos=None):
    """q [Tq, d], k/v [Tk, d] (rows = positions); causal_pos[i] = position of query i (keys
    <= it visible) or None (all keys)."""
    Tq, d = q.shape
    hd = d // heads
    pos = causal_pos if causal_pos is not None else np.full(Tq, k.shape[0] - 1)
    out = D.attention(q.reshape(Tq, heads, hd), k.reshape(-1, heads, hd), v.reshape(-1, heads, hd),
                      np.asarray(pos), hd ** -0.5, "f32")
    return out.reshape(Tq, d)


def im2col(x: np.ndarray, stride: int) -> np.ndarray:
    """x [T, C] channels-last -> [T_out, 3*C] rows [x[s*t-1], x[s*t], x[s*t+1]] (zero padded)."""
    T, C = x.shape
    xp = np.zeros((T + 2, C), np.float32)
    xp[1:-1] = x
    To = (T + 2 - 3) // stride + 1
    idx = np.arange(To) * stride
    return np.concatenate([xp[idx], xp[idx + 1], xp[idx + 2]], axis=1)


def encoder(cfg: WhisperConfig, W: dict, mel: np.ndarray) -> np.ndarray:
    """mel [n_mels, 2 * n_audio] -> encoder output [n_audio, d] (values of the activation dtype)."""
    dt = cfg.dtype
    x = rnd(mel.T, dt)
    c1 = im2col(x, 1)
    kp = W["conv1"]["w"].shape[1]  # conv1's K padded to a multiple of 64 with zero columns
    c1 = np.pad(c1, ((0, 0), (0, kp - c1.shape[1])))
    h = linear(c1, W["conv1"], 0, dt, bias=W["conv1_b"], gelu_out=True)
    h = linear(im2col(h, 2), W["conv2"], 0, dt, bias=W["conv2_b"], gelu_out=True, residual=W["enc_pos"])
    d = cfg.d_model
    for L in W["enc"]:
        n = layernorm(h, L["ln1_w"], L["ln1_b"], cfg.eps, dt)
        qkv = linear(n, L["qkv"], 0, dt, bias=L["qkv_b"])
        a = rnd(attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], cfg.heads), dt)
        h = linear(a, L["o"], 0, dt, bias=L["o_b"], residual=h)
        n = layernorm(h, L["ln2_w"], L["ln2_b"], cfg.eps, dt)
        f = linear(n, L["fc1"], 0, dt, bias=L["fc1_b"], gelu_out=True)
        h = linear(f, L["fc2"], 0, dt, bias=L["fc2_b"], residual=h)
    return layernorm(h, W["enc_ln_w"], W["enc_ln_b"], cfg.eps, dt)


def cross_kv(cfg: WhisperConfig, W: dict, enc: np.ndarray):
    """Cross-attention K/V of every decoder layer (k|v as one projection, k's bias zero),
    projected once per audio window."""
    d = cfg.d_model
    out = []
    for L in W["dec"]:
        kv = linear(enc, L["ckv"], cfg.bits, cfg.dtype, bias=L["ckv_b"])
        out.append((kv[:, :d], kv[:, d:]))
    return out


def token_embedding(cfg: WhisperConfig, W: dict, tokens) -> np.ndarray:
    E = W["embed"]
    toks = np.asarray(tokens)
    if cfg.bits:
        q = A.unpack(E["w"][toks], cfg.bits).astype(np.float32)
        s = A.from_storage(E["s"][toks], cfg.dtype).repeat(64, axis=1)
        b = A.from_storage(E["b"][toks], cfg.dtype).repeat(64, axis=1)
        return rnd(s * q + b, cfg.dtype)
    return A.from_storage(E["w"][toks], cfg.dtype)


def decoder_forward(cfg: WhisperConfig, W: dict, xkv, tokens, start: int, cache: list) -> np.ndarray:
    """Runs `tokens` at positions start.. through the decoder; appends to `cache` (per layer
    [K rows, V rows]); returns the final-LayerNorm hidden states [T, d]."""
    dt = cfg.dtype
    T = len(tokens)
    pos = np.arange(start, start + T)
    h = rnd(token_embedding(cfg, W, tokens) + W["dec_pos"][pos], dt)
    d = cfg.d_model
    for li, L in enumerate(W["dec"]):
        n = layernorm(h, L["ln1_w"], L["ln1_b"], cfg.eps, dt)
        qkv = linear(n, L["qkv"], cfg.bits, dt, bias=L["qkv_b"])
        q, k, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]
        cache[li][0] = np.concatenate([cache[li][0], k]) if cache[li][0] is not None else k
        cache[li][1] = np.concatenate([cache[li][1], v]) if cache[li][1] is not None else v
        a = rnd(attention(q, cache[li][0], cache[li][1], cfg.heads, pos), dt)
        h = linear(a, L["o"], cfg.bits, dt, bias=L["o_b"], residual=h)
        n = layernorm(h, L["ln2_w"], L["ln2_b"], cfg.eps, dt)
        q2 = linear(n, L["cq"], cfg.bits, dt, bias=L["cq_b"])
        a = rnd(attention(q2, xkv[li][0], xkv[li][1], cfg.heads), dt)
        h = linear(a, L["co"], cfg.bits, dt, bias=L["co_b"], residual=h)
        n = layernorm(h, L["ln3_w"], L["ln3_b"], cfg.eps, dt)
        f = linear(n, L["fc1"], cfg.bits, dt, bias=L["fc1_b"], gelu_out=True)
        h = linear(f, L["fc2"], cfg.bits, dt, bias=L["fc2_b"], residual=h)
    return layernorm(h, W["dec_ln_w"], W["dec_ln_b"], cfg.eps, dt)


def logits(cfg: WhisperConfig, W: dict, hidden: np.ndarray) -> np.ndarray:
    return linear(hidden, W["embed"], cfg.bits, cfg.dtype)


def score(cfg: WhisperConfig, W: dict, enc: np.ndarray, tokens) -> np.ndarray:
    """Teacher-forced logits of every position of `tokens` (prompt included), [T, vocab]."""
    xkv = cross_kv(cfg, W, enc)
    cache = [[None, None] for _ in W["dec"]]
    return logits(cfg, W, decoder_forward(cfg, W, xkv, list(tokens), 0, cache))


def greedy(cfg: WhisperConfig, W: dict, enc: np.ndarray, prompt, n_tokens: int):
    """Prefill the prompt, then `n_tokens` greedy choices (no end-of-text stop); returns the
    tokens and the logits rows that chose them."""
    xkv = cross_kv(cfg, W, enc)
    cache = [[None, None] for _ in W["dec"]]
    hid = decoder_forward(cfg, W, xkv, list(prompt), 0, cache)
    row = logits(cfg, W, hid[-1:])[0]
    toks, rows = [], []
    pos = len(prompt)
    for i in range(n_tokens):
        t = int(np.argmax(row))
        toks.append(t)
        rows.append(row)
        if i + 1 == n_tokens:
            break
        hid = decoder_forward(cfg, W, xkv, [t], pos, cache)
        row = logits(cfg, W, hid)[0]
        pos += 1
    return toks, np.stack(rows)


# ---------------------------------------------------------------------------------------
# Token rules of the reference's GPU-side greedy decode (WhisperModel.swift:311-372)
# ---------------------------------------------------------------------------------------

@dataclass
class TokenRules:
    """Token ids and suppress lists of a checkpoint's tokenizer and generation config."""
    eot: int
    no_timestamps: int
    timestamp_begin: int
    suppress: tuple = ()
    begin_suppress: tuple = ()
    max_source_positions: int = 1500  # encoder frames; 30 s windows

    def last_allowed(self) -> int:
        # Swift's Double.rounded() rounds half away from zero (WhisperModel.swift:321)
        q = self.max_source_positions / 30.0
        return self.timestamp_begin + int(math.floor(q + 0.5))


def _lse(x: np.ndarray) -> float:
    m = float(np.max(x))
    if m == -math.inf:
        return -math.inf
    return m + math.log(float(np.sum(np.exp((x - m).astype(np.float64)))))


def rule_select(row: np.ndarray, step: int, prev, before_prev, r: TokenRules):
    """One choice of the rules (``select`` at WhisperModel.swift:340-359): the suppress mask
    (begin-suppress too at step 0), log-probabilities of the filtered row, text masked when the
    timestamp tokens' total probability beats every text token, no-timestamps always masked,
    step 0 limited to the first timestamps; after a timestamp, timestamps are masked when the
    token before it was one as well (or there is none), else text up to end-of-text.  Returns
    the token (lowest index among equal maxima) and its log-probability under the final row."""
    f = np.asarray(row, np.float64).copy()
    V = f.shape[0]
    begin = r.timestamp_begin
    sup = list(r.suppress) + (list(r.begin_suppress) if step == 0 else [])
    for t in sup:
        if 0 <= t < V:
            f[t] = -math.inf
    lse = _lse(f)
    lp = f - lse
    ts_mass = _lse(lp[begin:])
    max_text = float(np.max(lp[:begin]))
    mask = np.zeros(V)
    mask[r.no_timestamps] = -math.inf
    if step == 0:
        mask[:begin] = -math.inf
        la = r.last_allowed()
        if la + 1 < V:
            mask[la + 1:] = -math.inf
    if ts_mass > max_text:
        mask[:begin] = -math.inf
    if prev is not None:
        last = prev >= begin
        pen = before_prev >= begin if before_prev is not None else True
        if last and pen:
            mask[begin:] = -math.inf
        if last and not pen:
            mask[:r.eot] = -math.inf
    final = f + mask
    tok = int(np.argmax(final))
    return tok, float(final[tok] - _lse(final)), final


# ---------------------------------------------------------------------------------------
# Temperature fallback (WhisperModel.swift:218-292, sample() :447-454, compressionRatio
# :434-445): an attempt at temperature T > 0 draws each token from softmax(final / T); the
# library's draw is Gumbel-max with Philox-4x32-10 noise (MLX's categorical is Gumbel-max
# as well, on its own generator, so the draws themselves are not comparable with MLX's).
# ---------------------------------------------------------------------------------------

_PHILOX_M0, _PHILOX_M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)


def philox4x32_10_np(c0, c1, c2, c3, k0: int, k1: int):
    """Philox-4x32-10 over arrays of counters (uint32 words), the same rounds as
    ``oracle.decoder.philox4x32_10``; returns four uint32 arrays."""
    M = np.uint64(0xFFFFFFFF)
    c0, c1, c2, c3 = (np.asarray(v, np.uint64) & M for v in (c0, c1, c2, c3))
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    k0, k1 = int(k0) & 0xFFFFFFFF, int(k1) & 0xFFFFFFFF
    for _ in range(10):
        p0 = _PHILOX_M0 * c0
        p1 = _PHILOX_M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & M
        hi1, lo1 = p1 >> np.uint64(32), p1 & M
        c0, c1, c2, c3 = (hi1 ^ c1 ^ np.uint64(k0)) & M, lo1, (hi0 ^ c3 ^ np.uint64(k1)) & M, lo0
        k0 = (k0 + 0x9E3779B9) & 0xFFFFFFFF
        k1 = (k1 + 0xBB67AE85) & 0xFFFFFFFF
    return [x.astype(np.uint32) for x in (c0, c1, c2, c3)]


def gumbel_noise(seed: int, draw: int, step: int, stream: int, vocab: int) -> np.ndarray:
    """Noise of every token at one step: Philox on counter (v // 4, step, stream, draw) keyed
    by the seed, word v % 4, u = (2 * (bits >> 9) + 1) / 2**24 (exact in fp32), -log(-log u)."""
    v = np.arange(vocab, dtype=np.uint64)
    words = philox4x32_10_np(v >> np.uint64(2), step, stream, draw, seed & 0xFFFFFFFF, seed >> 32)
    bits = np.choose((v & np.uint64(3)).astype(np.int64), words).astype(np.uint64)
    u = (np.uint64(2) * (bits >> np.uint64(9)) + np.uint64(1)).astype(np.float64) / 16777216.0
    return -np.log(-np.log(u))


def rule_sample(row, step: int, prev, before_prev, r: TokenRules, temperature: float, seed: int, draw: int,
                stream: int = 0):
    """One sampled choice under the rules: argmax(final / temperature + noise) and the token's
    log-probability under the unscaled final row (the reference adds ``filtered[next] -
    logSumExp(filtered)``, WhisperModel.swift:264-265).  Returns (token, logprob, keys, final)."""
    _, _, final = rule_select(row, step, prev, before_prev, r)
    keys = final / temperature + gumbel_noise(seed, draw, step, stream, final.shape[0])
    tok = int(np.argmax(keys))
    return tok, float(final[tok] - _lse(final)), keys, final


def compression_ratio(text: str) -> float:
    """UTF-8 bytes over zlib-compressed bytes at the default level; 0 for empty text
    (WhisperModel.swift:434-445)."""
    import zlib
    raw = text.encode("utf-8")
    return 0.0 if not raw else len(raw) / len(zlib.compress(raw, 6))


def attempt_verdict(sum_logprob: float, n_tokens: int, text: str, no_speech_prob: float = 0.0) -> str:
    """After one attempt (WhisperModel.swift:285-291): the average log-probability counts the
    end-of-text step (n_tokens + 1); 'empty' when the window is probably silence, 'accept' when
    the average is >= -1 and the compression ratio <= 2.4, else 'retry' at the next temperature
    (the last temperature's attempt stands if every one asks for a retry)."""
    average = sum_logprob / (n_tokens + 1)
    if no_speech_prob > 0.6 and average < -1:
        return "empty"
    if average >= -1 and compression_ratio(text) <= 2.4:
        return "accept"
    return "retry"


FALLBACK_TEMPERATURES = (0.0, 0.2, 0.4, 0.6, 0.8, 1.0)  # WhisperModel.swift:218-219


# ---------------------------------------------------------------------------------------
# Log-mel input features (WhisperAudio.swift:7-93; MLXAudioCore/DSP.swift:44-135)
# ---------------------------------------------------------------------------------------

SAMPLE_RATE, N_FFT, HOP, WINDOW_SAMPLES = 16000, 400, 160, 480000


def mel_filters(n_mels: int) -> np.ndarray:
    """The reference's Slaney filterbank [201, n_mels], evaluated in fp32 as it does
    (DSP.swift:44-135): mel points uniform between hz_to_mel(0) and hz_to_mel(8000), rising
    edge on [low, center), falling on [center, high], each filter scaled by 2 / (high - low)."""
    f32 = np.float32
    sr, fmin, fmax = f32(SAMPLE_RATE), f32(0.0), f32(SAMPLE_RATE / 2.0)
    f_sp, min_log_hz = f32(200.0) / f32(3.0), f32(1000.0)
    min_log_mel = (min_log_hz - fmin) / f_sp
    log_step = f32(np.log(f32(6.4))) / f32(27.0)

    def hz_to_mel(f):
        f = f32(f)
        return (f - fmin) / f_sp if f < min_log_hz else min_log_mel + f32(np.log(f / min_log_hz)) / log_step

    def mel_to_hz(m):
        m = f32(m)
        return fmin + f_sp * m if m < min_log_mel else min_log_hz * f32(np.exp(log_step * (m - min_log_mel)))

    m0, m1 = hz_to_mel(fmin), hz_to_mel(fmax)
    pts = [mel_to_hz(m0 + f32(i) * (m1 - m0) / f32(n_mels + 1)) for i in range(n_mels + 2)]
    fb = np.zeros((N_FFT // 2 + 1, n_mels), np.float32)
    for i in range(N_FFT // 2 + 1):
        f = f32(i) * sr / f32(N_FFT)
        for j in range(n_mels):
            lo, c, hi = pts[j], pts[j + 1], pts[j + 2]
            v = f32(0.0)
            if lo <= f < c:
                v = (f - lo) / (c - lo)
            elif c <= f <= hi:
                v = (hi - f) / (hi - c)
            fb[i, j] = v * (f32(2.0) / (hi - lo))
    return fb


def log_mel(audio: np.ndarray, n_mels: int) -> np.ndarray:
    """[n_mels, 3000] features of one window: pad with zeros or trim to 30 s, reflect-pad
    200, frames of 400 every 160 (the last of 3001 dropped), periodic Hann window, |rfft|^2
    (float64 here), mel projection, log10(max(., 1e-10)), floor at max - 8, (x + 4) / 4."""
    a = np.zeros(WINDOW_SAMPLES, np.float32)
    src = np.asarray(audio, np.float32).reshape(-1)[:WINDOW_SAMPLES]
    a[:src.size] = src
    padded = np.pad(a, N_FFT // 2, mode="reflect")
    n_frames = 1 + (padded.size - N_FFT) // HOP
    idx = np.arange(n_frames)[:, None] * HOP + np.arange(N_FFT)[None, :]
    n = np.arange(N_FFT, dtype=np.float32)
    win = np.float32(0.5) * (np.float32(1.0) - np.cos(np.float32(2.0 * np.pi) * n / np.float32(N_FFT)))
    spec = np.fft.rfft(padded[idx].astype(np.float64) * win.astype(np.float64), axis=-1)
    power = (spec.real ** 2 + spec.imag ** 2)[:-1]
    mel = (power @ mel_filters(n_mels).astype(np.float64)).T
    logs = np.log10(np.maximum(mel, 1e-10))
    logs = np.maximum(logs, logs.max() - 8.0)
    return ((logs + 4.0) / 4.0).astype(np.float32)
