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
