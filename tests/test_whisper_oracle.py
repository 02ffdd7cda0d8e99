"""The Whisper oracle's building blocks against the reference's rules (CPU only)."""
import math

import numpy as np

from oracle import whisper as Wh


def test_sinusoid_table_rule():
    # WhisperModel.swift:554-569: half = C/2, increment ln(10000)/(half-1), sin | cos halves
    t = Wh.sinusoids(3, 4, "f32")
    inc = math.log(10000.0)
    expect = np.array([[math.sin(p), math.sin(p * math.exp(-inc)), math.cos(p), math.cos(p * math.exp(-inc))]
                       for p in range(3)], np.float32)
    assert t.shape == (3, 4)
    assert np.array_equal(t, expect)
    # the table dtype rounds once (fp16 here)
    assert np.array_equal(Wh.sinusoids(3, 4, "f16"), expect.astype(np.float16).astype(np.float32))


def test_conv_geometry():
    x = np.arange(10 * 2, dtype=np.float32).reshape(10, 2)
    c1 = Wh.im2col(x, 1)
    assert c1.shape == (10, 6)
    assert np.array_equal(c1[0], [0, 0, 0, 1, 2, 3])          # left padding
    assert np.array_equal(c1[9], [16, 17, 18, 19, 0, 0])      # right padding
    c2 = Wh.im2col(x, 2)
    assert c2.shape == (5, 6)                                  # 3000 frames -> 1500 at stride 2
    assert np.array_equal(c2[1], [2, 3, 4, 5, 6, 7])          # taps 2t-1, 2t, 2t+1


def test_gelu_is_the_erf_form():
    g = Wh.A.gelu(np.array([0.0, 1.0, -1.0, 3.0], np.float32))
    ref = [0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in (0.0, 1.0, -1.0, 3.0)]
    assert np.allclose(g, ref, rtol=1e-6, atol=1e-7)


def test_layernorm_normalises_rows():
    x = np.random.default_rng(0).standard_normal((4, 384)).astype(np.float32) * 3 + 1
    y = Wh.layernorm(x, np.ones(384, np.float32), np.zeros(384, np.float32), 1e-5, "f32")
    assert np.allclose(y.mean(axis=1), 0, atol=1e-5)
    assert np.allclose(y.var(axis=1), 1, atol=1e-3)


def test_token_rules_known_answers():
    """Each rule of the reference's GPU-side greedy (WhisperModel.swift:311-372) on hand-made
    rows: suppress lists, no-timestamps, step 0 limited to [begin, begin + frames / 30], text
    masked when the timestamps' total probability beats every text token, and the two rules
    after a timestamp."""
    from oracle import whisper as Wh
    r = Wh.TokenRules(eot=90, no_timestamps=99, timestamp_begin=100, suppress=(5,), begin_suppress=(7,),
                      max_source_positions=300)
    assert r.last_allowed() == 110
    V = 130
    row = np.full(V, -5.0, np.float32)
    # step 0: text, end-of-text and late timestamps are masked; the best early timestamp wins
    row0 = row.copy(); row0[3] = 9.0; row0[120] = 8.0; row0[104] = 2.0
    tok, lp, final = Wh.rule_select(row0, 0, None, None, r)
    assert tok == 104 and np.isneginf(final[:100]).all() and np.isneginf(final[111:]).all()
    assert lp < 0
    # later steps, text dominates: the suppressed token loses, the next best text token wins
    row1 = row.copy(); row1[5] = 20.0; row1[6] = 19.0
    assert Wh.rule_select(row1, 3, 10, 11, r)[0] == 6
    row1[7] = 30.0  # begin-suppress applies at step 0 only
    assert Wh.rule_select(row1, 3, 10, 11, r)[0] == 7
    # no-timestamps is never chosen
    row2 = row.copy(); row2[99] = 50.0; row2[40] = 1.0
    assert Wh.rule_select(row2, 2, 10, 11, r)[0] == 40
    # timestamp mass beats the best text token: text is masked
    row3 = row.copy(); row3[100:] = 3.0; row3[40] = 4.0
    assert Wh.rule_select(row3, 2, 10, 11, r)[0] >= 100
    # after a timestamp preceded by text: text up to end-of-text masked (end-of-text allowed)
    row4 = row.copy(); row4[40] = 9.0; row4[90] = 1.0; row4[95] = 2.0
    assert Wh.rule_select(row4, 2, 105, 11, r)[0] == 95
    # after two timestamps: every timestamp masked, text allowed
    row5 = row.copy(); row5[40] = 3.0; row5[120] = 2.0
    tok, lp, final = Wh.rule_select(row5, 3, 105, 104, r)
    assert tok == 40 and np.isneginf(final[100:]).all() and np.isfinite(lp)


def test_vectorised_philox_matches_the_scalar_rounds():
    from oracle import decoder as D
    rng = np.random.default_rng(4)
    for _ in range(20):
        c = [int(x) for x in rng.integers(0, 2**32, 4, dtype=np.uint64)]
        k = [int(x) for x in rng.integers(0, 2**32, 2, dtype=np.uint64)]
        got = Wh.philox4x32_10_np(*[np.array([x], np.uint64) for x in c], *k)
        assert tuple(int(g[0]) for g in got) == D.philox4x32_10(c, k)


def test_gumbel_noise_word_layout_and_moments():
    from oracle import decoder as D
    g = Wh.gumbel_noise(0x5EED, 2, 7, 3, 4099)
    # token 4098: counter (1024, step 7, stream 3, draw 2), word 2
    w = D.philox4x32_10((1024, 7, 3, 2), (0x5EED, 0))[2]
    u = (2 * (w >> 9) + 1) / 2**24
    assert g[4098] == -math.log(-math.log(u))
    big = Wh.gumbel_noise(1, 0, 0, 0, 200000)
    assert abs(big.mean() - np.euler_gamma) < 0.01 and abs(big.std() - math.pi / math.sqrt(6)) < 0.01


def test_rule_sample_draws_from_the_tempered_final_row():
    """Frequencies of Gumbel-max draws over many (step, draw) counters follow
    softmax(final / T) on a small row; tokens the rules mask are never drawn."""
    r = Wh.TokenRules(eot=5, no_timestamps=6, timestamp_begin=7, suppress=(1,), max_source_positions=30)
    row = np.array([0.0, 3.0, 0.5, 1.0, -1.0, 0.2, 4.0, -9.0, -9.0, -9.0])
    T = 0.7
    counts = np.zeros(row.size)
    for d in range(3000):
        tok, lp, keys, final = Wh.rule_sample(row, 5, 2, 3, r, T, 99, d)
        counts[tok] += 1
        assert math.isclose(lp, final[tok] - Wh._lse(final))
    _, _, final = Wh.rule_select(row, 5, 2, 3, r)
    p = np.exp(final / T - Wh._lse(final / T))
    assert counts[1] == counts[6] == 0
    assert np.abs(counts / counts.sum() - p).max() < 0.03


def test_attempt_verdict_and_compression_ratio_match_the_library():
    import zlib

    from vella_b200 import whisper as VW
    assert Wh.compression_ratio("") == VW.compression_ratio("") == 0.0
    text = "the cat sat on the mat " * 12
    assert Wh.compression_ratio(text) == VW.compression_ratio(text) == len(text) / len(zlib.compress(text.encode()))
    assert Wh.compression_ratio(text) > 2.4
    for lp, n, t, ns in [(-3.0, 5, "", 0.0), (-7.0, 5, "", 0.0), (-7.0, 5, "", 0.9), (-3.0, 5, "", 0.9),
                         (-3.0, 5, text, 0.0), (-6.0, 5, "short text", 0.0)]:
        assert Wh.attempt_verdict(lp, n, t, ns) == VW.attempt_verdict(lp, n, t, ns)
    assert Wh.attempt_verdict(-6.0, 5, "", 0.0) == "accept"      # average -1 is kept
    assert Wh.attempt_verdict(-6.1, 5, "", 0.0) == "retry"
    assert Wh.attempt_verdict(-6.1, 5, "", 0.61) == "empty"
    assert Wh.attempt_verdict(-3.0, 5, text, 0.0) == "retry"     # compression ratio above 2.4


class _FakeHandle:
    """The decode / stats / set_sampling surface of a Whisper handle, scripted per temperature."""

    def __init__(self, script):
        self.script, self.calls, self.temp = script, [], None

    def set_sampling(self, temperature, seed=0x5EED, draw=0):
        self.calls.append((temperature, seed, draw))
        self.temp = temperature

    def decode(self, prompt, max_tokens, eot=-1):
        from vella_b200.whisper import DecodeResult
        return DecodeResult(list(self.script[self.temp][0]), 0.0, 0.0)

    def stats(self):
        return {"sum_logprob": self.script[self.temp][1]}


def test_fallback_loop_follows_the_reference_order():
    from vella_b200 import whisper as VW
    run = VW.Whisper.decode_with_fallback
    repeat = "la la la la la la la la la la la la la la la la la la"
    script = {0.0: ([1, 2, 3], -9.0), 0.2: ([4, 4], -1.0), 0.4: ([5], -0.1), 0.6: ([6], -0.1), 0.8: ([7], -0.1),
              1.0: ([8], -0.1)}
    h = _FakeHandle(script)
    res = run(h, [1], 8, 50257, seed=7)
    assert res.tokens == [4, 4] and res.temperature == 0.2 and res.attempts == 2 and res.verdict == "accept"
    assert h.calls == [(0.0, 7, 0), (0.2, 7, 1), (0.0, 7, 0)]  # back to argmax afterwards
    # a repetitive text is rejected by the compression ratio: every attempt retries, the last stands
    h = _FakeHandle(script)
    res = run(h, [1], 8, 50257, detokenize=lambda t: repeat, seed=7)
    assert res.attempts == 6 and res.temperature == 1.0 and res.tokens == [8] and res.verdict == "retry"
    # probable silence empties the window at the first low-confidence attempt
    res = run(_FakeHandle(script), [1], 8, 50257, no_speech_prob=0.9)
    assert res.tokens == [] and res.attempts == 1 and res.verdict == "empty"


def test_mel_filterbank_shape_and_peaks():
    for n in (80, 128):
        fb = Wh.mel_filters(n)
        assert fb.shape == (201, n) and (fb >= 0).all()
        # each triangle peaks at the bin nearest its center and is nonzero somewhere
        assert (fb.max(axis=0) > 0).all()
        peaks = fb.argmax(axis=0)
        assert (np.diff(peaks) >= 0).all()
    # Slaney area norm: each triangle has unit area in Hz, so its weights times the 40 Hz bin
    # spacing sum to about 1
    fb = Wh.mel_filters(80)
    assert np.allclose(fb.sum(axis=0)[:10] * 40.0, 1.0, atol=0.05)


def test_log_mel_properties():
    # silence: every value at the floor of log10(1e-10) = -10, mapped to -1.5
    assert np.array_equal(np.unique(Wh.log_mel(np.zeros(16000), 80)), np.array([-1.5], np.float32))
    t = np.arange(16000 * 5) / 16000.0
    tone = 0.5 * np.sin(2 * np.pi * 1000.0 * t)
    m = Wh.log_mel(tone, 80)
    assert m.shape == (80, 3000)
    centers = Wh.mel_filters(80).argmax(axis=0) * 40.0
    assert abs(centers[int(np.argmax(m[:, 100]))] - 1000.0) <= 80.0  # the 1 kHz tone's mel bin
    assert m.max() - m.min() <= 2.0 + 1e-6  # floored 8 decades below the maximum, / 4
    # trimming: samples past 30 s change nothing
    long = np.concatenate([tone, np.zeros(480000), np.ones(1000)])
    assert np.array_equal(Wh.log_mel(long, 80), Wh.log_mel(np.concatenate([tone, np.zeros(480000)])[:480000], 80))


class _FakeWhisperHandle:
    """encode_audio / decode_with_fallback of a Whisper handle, scripted per window."""

    def __init__(self, results):
        from vella_b200.whisper import WhisperConfig
        self.cfg = WhisperConfig()
        self.results, self.encoded, self.calls = list(results), [], []

    def encode_audio(self, audio):
        self.encoded.append(np.asarray(audio).copy())

    def decode_with_fallback(self, prompt, max_tokens, eot, detokenize, temps, seed, no_speech_prob, draw_base=0):
        self.calls.append((list(prompt), max_tokens, eot, tuple(temps), seed, no_speech_prob, draw_base))
        return self.results.pop(0)


def test_generate_windows_prompt_and_text():
    from vella_b200 import whisper as VW
    from vella_b200.checkpoint import WhisperTokens
    tok = WhisperTokens(sot=50258, eot=50257, no_timestamps=50364, timestamp_begin=50365, transcribe=50360,
                        languages={"en": 50259}, multilingual=True)
    mk = lambda t: VW.FallbackResult(t, 0.0, -1.0, -0.5, 1.0, 1, "accept")  # noqa: E731
    fake = _FakeWhisperHandle([mk([1, 2]), mk([]), mk([7])])
    words = {1: "hello", 2: " world", 7: " again "}
    stt = VW.WhisperSTT(fake, tok, lambda ts: "".join(words[t] for t in ts), seed=9)
    stereo = np.random.default_rng(0).standard_normal((16000 * 65, 2)).astype(np.float32)
    out = stt.generate(stereo, language="en", max_tokens=1024)
    # 65 s: windows of 30, 30 and 5 s, each the channel mean
    assert [e.shape[0] for e in fake.encoded] == [480000, 480000, 80000]
    assert np.allclose(fake.encoded[2], stereo[960000:].mean(axis=1))
    assert all(c[0] == [50258, 50259, 50360] for c in fake.calls)
    assert fake.calls[0][1] == 224 and fake.calls[0][3] == VW.FALLBACK_TEMPERATURES  # n_text_ctx / 2
    assert [c[6] for c in fake.calls] == [0, 6, 12] and all(c[4] == 9 for c in fake.calls)
    assert out.text == "hello world again"
    assert out.segments == [{"text": "hello world", "start": 0.0, "end": 30.0},
                            {"text": "again", "start": 60.0, "end": 65.0}]
    assert (out.prompt_tokens, out.generation_tokens, out.total_tokens) == (9, 3, 12)
    # a fixed temperature is the only attempt
    fake = _FakeWhisperHandle([mk([1])])
    VW.WhisperSTT(fake, tok, lambda ts: "x").generate(np.zeros(1000, np.float32), temperature=0.4)
    assert fake.calls[0][3] == (0.4,)


def test_library_mel_filterbank_matches_the_oracle():
    """The library's host-side filterbank (the one the device log-mel projects on) against the
    oracle's restatement of MLXAudioCore.melFilters: fp32 on both sides, libm and numpy may
    differ by an ulp in log/exp."""
    import ctypes

    from vella_b200 import _lib
    _lib.declare("vella_whisper_mel_filters", ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_float)])
    for n in (80, 128):
        out = np.zeros((201, n), np.float32)
        _lib.check(_lib.lib().vella_whisper_mel_filters(n, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        ref = Wh.mel_filters(n)
        # relative to each filter's peak: near a triangle's foot a weight is a difference of nearly
        # equal frequencies, where an ulp in a mel point is a large relative change
        assert (np.abs(out - ref) <= 1e-5 * ref.max(axis=0, keepdims=True)).all(), np.abs(out - ref).max()
        assert ((out > 0) == (ref > 0)).all()


def test_library_sinusoid_table_matches_the_oracle():
    """The library's host-side encoder position table against the oracle's statement of the
    reference rule (double trig, rounded once to fp32): bit for bit."""
    import ctypes

    from vella_b200 import _lib
    _lib.declare("vella_whisper_sinusoids", ctypes.c_int, [ctypes.c_int32, ctypes.c_int32,
                                                           ctypes.POINTER(ctypes.c_float)])
    for A, C in ((1500, 384), (1500, 1280), (3, 4)):
        out = np.zeros((A, C), np.float32)
        _lib.check(_lib.lib().vella_whisper_sinusoids(A, C, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        assert np.array_equal(out, Wh.sinusoids(A, C, "f32"))
