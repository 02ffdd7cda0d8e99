"""Parity of the Whisper encoder and decoder step (vella_whisper_* through the C ABI) with
the CPU oracle, at the Whisper-tiny shapes of config 1 (int4 decoder, fp16) and a dense one.

Bars: encoder output relative RMS <= 1e-2; teacher-forced logits max |error| <= 2e-2;
greedy tokens equal the oracle's argmax wherever its top-2 margin exceeds that tolerance;
a replayed decoder-step graph gives the same tokens as the first (eager) step sequence.
"""
import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle import whisper as Wh

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


class _Dev:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def download(model, name, layer=-1):
    ptr, nbytes = model.tensor(name, layer)
    return torch.as_tensor(_Dev(ptr, nbytes), device="cuda").cpu().numpy()


def f16(raw):
    return raw.view(np.float16)


def oracle_weights(model, c):
    d, F = c.d_model, c.ffn
    val = lambda name, layer=-1: f16(download(model, name, layer)).astype(np.float32)  # noqa: E731

    def lin(name, layer, n, k, bits):
        w = download(model, f"{name}.w", layer)
        if bits:
            return {"w": w.view(np.uint32).reshape(n, k * bits // 32),
                    "s": f16(download(model, f"{name}.s", layer)).reshape(n, k // 64),
                    "b": f16(download(model, f"{name}.b", layer)).reshape(n, k // 64)}
        return {"w": f16(w).reshape(n, k)}

    kp1 = (3 * c.n_mels + 63) // 64 * 64
    W = {"conv1": lin("conv1", -1, d, kp1, 0), "conv1_b": val("conv1.bias"),
         "conv2": lin("conv2", -1, d, 3 * d, 0), "conv2_b": val("conv2.bias"),
         "enc_pos": val("enc_pos").reshape(c.n_audio, d),
         "enc_ln_w": val("enc_ln.weight"), "enc_ln_b": val("enc_ln.bias"),
         "dec_ln_w": val("dec_ln.weight"), "dec_ln_b": val("dec_ln.bias"),
         "embed": lin("embed", -1, c.vocab, d, c.bits), "dec_pos": val("dec_pos").reshape(c.max_target, d),
         "enc": [], "dec": []}
    for l in range(c.enc_layers):
        W["enc"].append({"ln1_w": val("enc.ln1.weight", l), "ln1_b": val("enc.ln1.bias", l),
                         "qkv": lin("enc.qkv", l, 3 * d, d, 0), "qkv_b": val("enc.qkv.bias", l),
                         "o": lin("enc.o", l, d, d, 0), "o_b": val("enc.o.bias", l),
                         "ln2_w": val("enc.ln2.weight", l), "ln2_b": val("enc.ln2.bias", l),
                         "fc1": lin("enc.fc1", l, F, d, 0), "fc1_b": val("enc.fc1.bias", l),
                         "fc2": lin("enc.fc2", l, d, F, 0), "fc2_b": val("enc.fc2.bias", l)})
    b = c.bits
    for l in range(c.dec_layers):
        L = {}
        for ln in ("ln1", "ln2", "ln3"):
            L[f"{ln}_w"], L[f"{ln}_b"] = val(f"dec.{ln}.weight", l), val(f"dec.{ln}.bias", l)
        for name, n, k in (("qkv", 3 * d, d), ("o", d, d), ("cq", d, d), ("ckv", 2 * d, d), ("co", d, d),
                           ("fc1", F, d), ("fc2", d, F)):
            L[name] = lin(f"dec.{name}", l, n, k, b)
            L[f"{name}_b"] = val(f"dec.{name}.bias", l)
        W["dec"].append(L)
    return W


def make(cfg, seed=1):
    from vella_b200 import whisper as VW
    m = VW.Whisper(cfg)
    m.init_random(seed, 0.02)
    oc = Wh.WhisperConfig(cfg.n_mels, cfg.d_model, cfg.heads, cfg.enc_layers, cfg.dec_layers, cfg.ffn, cfg.vocab,
                          cfg.n_audio, cfg.max_target, cfg.bits, "f16", cfg.eps)
    return m, oc


def mel_of(cfg, seed):
    return np.random.default_rng(seed).standard_normal((cfg.n_mels, 2 * cfg.n_audio)).astype(np.float32)


@pytest.fixture(scope="module")
def tiny():
    from vella_b200 import whisper as VW
    m, oc = make(VW.TINY, seed=5)
    W = oracle_weights(m, oc)
    mel = mel_of(oc, 7)
    m.encode(mel)
    enc_ref = Wh.encoder(oc, W, mel)
    yield m, oc, W, mel, enc_ref
    m.close()


def test_encoder_matches_oracle(tiny):
    m, oc, W, mel, enc_ref = tiny
    got = f16(download(m, "enc_out")).astype(np.float32).reshape(oc.n_audio, oc.d_model)
    assert np.isfinite(got).all()
    assert A.relative_rms(got, enc_ref) <= 1e-2


def test_teacher_forced_logits_match_oracle(tiny):
    m, oc, W, mel, enc_ref = tiny
    toks = [50258, 50259, 50359, 50363] + list(np.random.default_rng(3).integers(0, 50000, 20))
    got = m.score(toks).astype(np.float32)
    ref = Wh.score(oc, W, enc_ref, toks)
    assert got.shape == ref.shape == (len(toks), oc.vocab)
    err = float(np.abs(got - ref).max())
    assert err <= LOGIT_TOL, err


def test_greedy_decode_matches_oracle_and_replays(tiny):
    m, oc, W, mel, enc_ref = tiny
    prompt = [50258, 50259, 50359, 50363]
    res = m.decode(prompt, 24)
    assert len(res.tokens) == 24
    # teacher-forced oracle logits along the produced sequence: each token is the argmax
    # wherever the oracle's top-2 margin exceeds the logits tolerance
    logits = Wh.score(oc, W, enc_ref, prompt + res.tokens[:-1])[len(prompt) - 1:]
    for j, t in enumerate(res.tokens):
        row = logits[j]
        best = int(np.argmax(row))
        assert t == best or row[best] - row[t] <= LOGIT_TOL, (j, t, best)
    # the second decode replays the captured step graph: identical tokens
    again = m.decode(prompt, 24)
    assert again.tokens == res.tokens


def test_end_of_text_stops_and_is_not_emitted(tiny):
    m, oc, W, mel, enc_ref = tiny
    prompt = [50258, 50259, 50359, 50363]
    full = m.decode(prompt, 12).tokens
    eot = full[5]
    first = full.index(eot)
    cut = m.decode(prompt, 12, eot=eot).tokens
    assert cut == full[:first]


def test_dense_fp16_model_matches_oracle():
    """The dense (config 3 style) decoder path at reduced sizes, encoder included."""
    from vella_b200 import whisper as VW
    cfg = VW.WhisperConfig(n_mels=128, d_model=256, heads=4, enc_layers=2, dec_layers=2, ffn=1024, vocab=4000,
                           n_audio=300, max_target=64, bits=0)
    m, oc = make(cfg, seed=9)
    W = oracle_weights(m, oc)
    mel = mel_of(oc, 11)
    m.encode(mel)
    enc_ref = Wh.encoder(oc, W, mel)
    got = f16(download(m, "enc_out")).astype(np.float32).reshape(oc.n_audio, oc.d_model)
    assert A.relative_rms(got, enc_ref) <= 1e-2
    toks = [1, 2, 3, 4] + list(np.random.default_rng(12).integers(0, 4000, 12))
    err = float(np.abs(m.score(toks).astype(np.float32) - Wh.score(oc, W, enc_ref, toks)).max())
    assert err <= LOGIT_TOL, err
    m.close()


def test_bad_arguments_are_rejected():
    from vella_b200 import _lib
    from vella_b200 import whisper as VW
    cfg = VW.WhisperConfig(n_mels=16, d_model=128, heads=2, enc_layers=1, dec_layers=1, ffn=256, vocab=500,
                           n_audio=40, max_target=32, bits=4)
    m = VW.Whisper(cfg)
    m.init_random(1)
    with pytest.raises(_lib.VellaError):
        m.decode([1, 2], 4)                      # decode before encode
    m.encode(mel_of(cfg, 1))
    with pytest.raises(_lib.VellaError):
        m.decode([1, 2], 31)                     # past max_target
    with pytest.raises(_lib.VellaError):
        m.score([1, 2, 700])                     # token id out of range
    assert len(m.decode([1, 2], 8).tokens) == 8  # the handle still works afterwards
    m.close()


def test_batched_streams_equal_single_stream_decodes():
    """Three streams in one handle (one decoder row per stream per step, the small-M GEMM path):
    each stream's cross-attention K/V equal, bit for bit, those of a one-stream handle that
    encoded its window alone, the windows give different tokens (weights std 0.1, so the
    audio steers the decoder), each stream's tokens are exactly the one-stream decode's, and
    a second batched decode (graph replay) repeats them."""
    from dataclasses import replace

    from vella_b200 import whisper as VW
    S, n, std = 3, 16, 0.1
    prompt = [50258, 50259, 50359, 50363]
    mels = np.stack([mel_of(VW.TINY, 30 + st) for st in range(S)])
    mb = VW.Whisper(replace(VW.TINY, streams=S))
    mb.init_random(5, std)
    mb.encode(mels)
    xkv = download(mb, "xkv").reshape(S, -1)
    got = mb.decode_batch(prompt, n)
    assert got.shape == (S, n)
    assert len({tuple(r) for r in got.tolist()}) > 1, got
    assert np.array_equal(mb.decode_batch(prompt, n), got)
    st_ = mb.stats()
    assert st_["tokens"] == S * n and st_["decode_ms"] > 0
    mb.close()
    single = VW.Whisper(VW.TINY)
    single.init_random(5, std)
    for st in range(S):
        single.encode(mels[st])
        assert np.array_equal(download(single, "xkv").reshape(-1), xkv[st]), st
        assert single.decode(prompt, n).tokens == list(got[st]), st
    single.close()


def test_many_streams_follow_the_oracle():
    """Twenty streams (decoder rows on the tensor-core GEMM): the first and last streams'
    tokens are the oracle's argmax wherever its top-2 margin exceeds the logits tolerance."""
    from dataclasses import replace

    from vella_b200 import _lib
    from vella_b200 import whisper as VW
    S, n = 20, 12
    prompt = [50258, 50259, 50359, 50363]
    m, oc = make(replace(VW.TINY, streams=S), seed=6)
    W = oracle_weights(m, oc)
    mels = np.stack([mel_of(oc, 50 + st) for st in range(S)])
    m.encode(mels)
    got = m.decode_batch(prompt, n)
    for st in (0, S - 1):
        enc_ref = Wh.encoder(oc, W, mels[st])
        logits = Wh.score(oc, W, enc_ref, prompt + list(got[st][:-1]))[len(prompt) - 1:]
        for j, t in enumerate(got[st]):
            row = logits[j]
            best = int(np.argmax(row))
            assert t == best or row[best] - row[t] <= LOGIT_TOL, (st, j, t, best)
    with pytest.raises(_lib.VellaError):
        m.decode(prompt, 4)  # one-stream entry point on a multi-stream handle
    m.close()


def _rule_choices(row, step, prev, before_prev, r, tol):
    """Tokens the rules may choose from a row known to within `tol` per logit: the oracle's
    choice and every token within 2*tol of it, for the row as given and with the timestamp
    block moved by +-2*tol (which covers a flip of the timestamp-mass comparison)."""
    ok = set()
    for shift in (0.0, 2 * tol, -2 * tol):
        x = np.asarray(row, np.float64).copy()
        x[r.timestamp_begin:] += shift
        tok, _, final = Wh.rule_select(x, step, prev, before_prev, r)
        if np.isfinite(final[tok]):
            ok |= set(np.nonzero(final >= final[tok] - 2 * tol)[0].tolist())
    return ok


def test_token_rules_follow_the_oracle(tiny):
    """Decode with the reference's token rules (suppress and begin-suppress masks, timestamp
    rules, no-timestamps masked): every token is one the oracle's rules allow on the
    teacher-forced row, the first token is a timestamp and the second is not, the summed
    log-probability matches the oracle's, a two-stream handle's stream 0 repeats the
    one-stream decode, and clearing the rules restores plain argmax."""
    from dataclasses import replace

    from vella_b200 import _lib
    from vella_b200 import whisper as VW
    m, oc, W, mel, enc_ref = tiny
    prompt = [50258, 50259, 50359, 50363]
    n = 16
    plain = m.decode(prompt, n).tokens
    V = oc.vocab
    r = Wh.TokenRules(eot=50257, no_timestamps=V - 3, timestamp_begin=V - 2,
                      suppress=[220, 50256, plain[1], plain[3]], begin_suppress=[50257, 220])
    with pytest.raises(_lib.VellaError):
        m.set_rules(eot=V, no_timestamps=V - 3, timestamp_begin=V - 2)
    with pytest.raises(_lib.VellaError):
        m.set_rules(eot=V - 1, no_timestamps=V - 3, timestamp_begin=V - 2)
    m.set_rules(r.eot, r.no_timestamps, r.timestamp_begin, r.suppress, r.begin_suppress)
    try:
        got = m.decode(prompt, n).tokens
        lp_gpu = m.stats()["sum_logprob"]
        assert len(got) == n
        assert got[0] >= r.timestamp_begin and got[1] < r.timestamp_begin, got[:2]
        logits = Wh.score(oc, W, enc_ref, prompt + got[:-1])[len(prompt) - 1:]
        lps = []
        for j, t in enumerate(got):
            prev = got[j - 1] if j >= 1 else None
            bprev = got[j - 2] if j >= 2 else None
            assert t in _rule_choices(logits[j], j, prev, bprev, r, LOGIT_TOL), (j, t)
            _, _, final = Wh.rule_select(logits[j], j, prev, bprev, r)
            lps.append(float(final[t] - Wh._lse(final)))
        lp_ref = sum(lps)
        assert abs(lp_gpu - lp_ref) <= 2 * LOGIT_TOL * n, (lp_gpu, lp_ref)
        assert m.decode(prompt, n).tokens == got  # replayed step graph
        # stopping at an end-of-text id: the tokens before it, and the sum up to it included
        # (steps enqueued past it add nothing)
        stop = got[9]
        first = got.index(stop)
        cut = m.decode(prompt, n, eot=stop)
        assert cut.tokens == got[:first]
        assert abs(m.stats()["sum_logprob"] - sum(lps[:first + 1])) <= 2 * LOGIT_TOL * (first + 1)
    finally:
        m.set_rules(None)
    assert m.decode(prompt, n).tokens == plain
    mb = VW.Whisper(replace(VW.TINY, streams=2))
    mb.init_random(5, 0.02)
    mb.encode(np.stack([mel, mel_of(oc, 8)]))
    mb.set_rules(r.eot, r.no_timestamps, r.timestamp_begin, r.suppress, r.begin_suppress)
    both = mb.decode_batch(prompt, n)
    assert list(both[0]) == got
    assert abs(mb.stats()["sum_logprob"] - lp_gpu) <= 1e-3 * max(1.0, abs(lp_gpu))
    mb.close()


def test_sampled_attempts_follow_the_oracle(tiny):
    """Temperature 0.7 under the token rules: every token is within the logits tolerance of
    the oracle's Gumbel-max draw (same Philox noise) on the teacher-forced row, the summed
    log-probability is the oracle's for those tokens, the same (seed, draw) replays, another
    draw gives another sequence, and the fallback loop ends on its last temperature when
    every attempt's average log-probability is below -1."""
    m, oc, W, mel, enc_ref = tiny
    prompt = [50258, 50259, 50359, 50363]
    n, T, seed = 12, 0.7, 0x5EED
    V = oc.vocab
    r = Wh.TokenRules(eot=50257, no_timestamps=V - 3, timestamp_begin=V - 2, suppress=[220, 50256],
                      begin_suppress=[50257, 220])
    m.set_rules(r.eot, r.no_timestamps, r.timestamp_begin, r.suppress, r.begin_suppress)
    try:
        m.set_sampling(T, seed, 3)
        got = m.decode(prompt, n).tokens
        lp_gpu = m.stats()["sum_logprob"]
        assert m.decode(prompt, n).tokens == got
        m.set_sampling(T, seed, 4)
        assert m.decode(prompt, n).tokens != got
        logits = Wh.score(oc, W, enc_ref, prompt + got[:-1])[len(prompt) - 1:]
        lp_ref = 0.0
        tol = 2 * LOGIT_TOL / T + 1e-3
        for j, t in enumerate(got):
            prev = got[j - 1] if j >= 1 else None
            bprev = got[j - 2] if j >= 2 else None
            ok = set()
            for shift in (0.0, 2 * LOGIT_TOL, -2 * LOGIT_TOL):
                x = np.asarray(logits[j], np.float64).copy()
                x[r.timestamp_begin:] += shift
                tok, _, keys, _ = Wh.rule_sample(x, j, prev, bprev, r, T, seed, 3)
                ok |= set(np.nonzero(keys >= keys[tok] - tol)[0].tolist())
            assert t in ok, (j, t)
            _, _, final = Wh.rule_select(logits[j], j, prev, bprev, r)
            lp_ref += float(final[t] - Wh._lse(final))
        assert abs(lp_gpu - lp_ref) <= 2 * LOGIT_TOL * n, (lp_gpu, lp_ref)
        res = m.decode_with_fallback(prompt, n, eot=-1, seed=seed)
        assert res.attempts == 6 and res.temperature == 1.0 and res.avg_logprob < -1
        m.set_sampling(1.0, seed, 5)
        assert m.decode(prompt, n).tokens == res.tokens
    finally:
        m.set_sampling(0.0)
        m.set_rules(None)


def test_log_mel_matches_the_oracle_and_feeds_the_encoder(tiny):
    """Log-mel features on the device (two windows at once, 80 bins; a window longer than
    30 s at 128 bins) match the oracle within 5e-3 (mean 1e-4: the device DFT accumulates in
    fp32, the oracle's rfft in fp64), and encode_audio gives, bit for bit, the encoder output
    of encode() on those features."""
    from vella_b200 import whisper as VW
    m, oc, W, mel, enc_ref = tiny
    rng = np.random.default_rng(9)
    t = np.arange(16000 * 12) / 16000.0
    a = (0.3 * np.sin(2 * np.pi * 440.0 * t) + 0.1 * np.sin(2 * np.pi * 3000.0 * t) * np.exp(-t)
         + 0.01 * rng.standard_normal(t.size)).astype(np.float32)
    b = (0.05 * rng.standard_normal(480000 + 7000)).astype(np.float32)
    got = VW.log_mel(np.stack([a, b[:a.size]]), 80).cpu().numpy()
    for st, x in enumerate((a, b[:a.size])):
        err = np.abs(got[st] - Wh.log_mel(x, 80))
        assert err.max() <= 5e-3 and err.mean() <= 1e-4, (st, err.max(), err.mean())
    err = np.abs(VW.log_mel(b, 128).cpu().numpy()[0] - Wh.log_mel(b, 128))
    assert err.max() <= 5e-3 and err.mean() <= 1e-4, (err.max(), err.mean())
    m.encode_audio(a)
    from_audio = download(m, "enc_out")
    m.encode(got[0])
    assert np.array_equal(download(m, "enc_out"), from_audio)
    m.encode(mel)  # the fixture's window again


def test_batched_end_of_text_and_log_probabilities_follow_single_streams():
    """Three streams under the token rules with an end-of-text id: each stream's tokens and
    summed log-probability equal those of a one-stream handle decoding its window alone."""
    from dataclasses import replace

    from vella_b200 import whisper as VW
    S, n, std = 3, 16, 0.1
    prompt = [50258, 50259, 50359, 50363]
    V = VW.TINY.vocab
    rules = dict(eot=50257, no_timestamps=V - 3, timestamp_begin=V - 2, suppress=[220], begin_suppress=[50257, 220])
    mels = np.stack([mel_of(VW.TINY, 40 + st) for st in range(S)])
    mb = VW.Whisper(replace(VW.TINY, streams=S))
    mb.init_random(5, std)
    mb.set_rules(**rules)
    mb.encode(mels)
    full = mb.decode_batch(prompt, n)
    stop = int(full[0][5])  # ends stream 0 at its first occurrence; the others wherever it appears
    got = mb.decode_batch(prompt, n, eot=stop)
    lps = mb.logprobs()
    single = VW.Whisper(VW.TINY)
    single.init_random(5, std)
    single.set_rules(**rules)
    for st in range(S):
        row = list(full[st])
        want = row[:row.index(stop)] if stop in row else row
        assert got[st] == want, st
        single.encode(mels[st])
        assert single.decode(prompt, n, eot=stop).tokens == want, st
        assert abs(single.stats()["sum_logprob"] - lps[st]) <= 1e-4 * max(1.0, abs(lps[st])), st
    single.close()
    mb.close()



def test_fused_decoder_step_equals_unfused_launches(monkeypatch):
    """The decoder's fusions (the first LayerNorm in the embedding kernel, the K/V append in
    the q|k|v GEMM's epilogue, the other LayerNorms in the preceding GEMM's last CTA) change
    no value: a handle created with VELLA_WHISPER_FUSE=0 (separate launches) decodes the same
    tokens, leaves a bit-equal self-attention cache, and gives bit-equal logits for one- and
    two-row forwards (the rows the LayerNorm tail takes), int4 and dense fp16."""
    from dataclasses import replace

    from vella_b200 import whisper as VW
    prompt = [50258, 50259, 50359, 50363]
    for cfg in (VW.TINY, replace(VW.TINY, bits=0)):
        mel = mel_of(cfg, 41)
        handles = []
        for fuse in ("1", "0"):
            monkeypatch.setenv("VELLA_WHISPER_FUSE", fuse)
            h = VW.Whisper(cfg)
            h.init_random(8, 0.1)
            h.encode(mel)
            handles.append(h)
        monkeypatch.delenv("VELLA_WHISPER_FUSE")
        fused, plain = handles
        try:
            a, b = fused.decode(prompt, 24), plain.decode(prompt, 24)
            assert a.tokens == b.tokens
            assert np.array_equal(download(fused, "kv"), download(plain, "kv"))
            for toks in ([50258], [50258, 50259]):
                assert np.array_equal(fused.score(toks), plain.score(toks)), toks
        finally:
            fused.close()
            plain.close()
