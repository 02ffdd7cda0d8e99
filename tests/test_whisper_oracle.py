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
