"""ctypes binding of the Whisper encoder + decoder step (``vella_whisper_*`` in
``include/vella_cuda.h``).

The model runs in the library (C++ host code, CUDA kernels, one CUDA graph per decoder step);
this module marshals arguments for the tests and the benchmark.  Names follow the reference's
``WhisperModel`` (``Worker/Sources/MLXAudioSTT/Whisper/WhisperModel.swift``): ``encode`` runs
the encoder and projects the cross-attention K/V, ``decode`` the greedy loop.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib


class WhisperCfg(ctypes.Structure):
    _fields_ = [("n_mels", ctypes.c_int32), ("d_model", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("enc_layers", ctypes.c_int32), ("dec_layers", ctypes.c_int32), ("ffn", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("n_audio", ctypes.c_int32), ("max_target", ctypes.c_int32),
                ("bits", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
                ("streams", ctypes.c_int32)]


class WhisperStats(ctypes.Structure):
    _fields_ = [("encode_ms", ctypes.c_float), ("prefill_ms", ctypes.c_float), ("decode_ms", ctypes.c_float),
                ("tokens", ctypes.c_int32), ("sum_logprob", ctypes.c_float)]


class WhisperRules(ctypes.Structure):
    _fields_ = [("eot", ctypes.c_int32), ("no_timestamps", ctypes.c_int32), ("timestamp_begin", ctypes.c_int32),
                ("suppress", ctypes.POINTER(ctypes.c_int32)), ("n_suppress", ctypes.c_int32),
                ("begin_suppress", ctypes.POINTER(ctypes.c_int32)), ("n_begin_suppress", ctypes.c_int32)]


_vp, _i32, _pi32 = ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)
for _name, _res, _args in [
    ("vella_whisper_create", ctypes.c_int, [ctypes.POINTER(WhisperCfg), _i32, ctypes.POINTER(_vp)]),
    ("vella_whisper_destroy", ctypes.c_int, [_vp]),
    ("vella_whisper_init_random", ctypes.c_int, [_vp, ctypes.c_uint64, ctypes.c_float]),
    ("vella_whisper_tensor", ctypes.c_int, [_vp, ctypes.c_char_p, _i32, ctypes.POINTER(_vp),
                                            ctypes.POINTER(ctypes.c_size_t)]),
    ("vella_whisper_encode", ctypes.c_int, [_vp, _vp, _i32]),
    ("vella_whisper_decode", ctypes.c_int, [_vp, _pi32, _i32, _i32, _i32, _pi32, _pi32]),
    ("vella_whisper_decode_batch", ctypes.c_int, [_vp, _pi32, _i32, _i32, _pi32]),
    ("vella_whisper_score", ctypes.c_int, [_vp, _pi32, _i32, _vp, _i32]),
    ("vella_whisper_get_stats", ctypes.c_int, [_vp, ctypes.POINTER(WhisperStats)]),
    ("vella_whisper_set_rules", ctypes.c_int, [_vp, ctypes.POINTER(WhisperRules)]),
]:
    _lib.declare(_name, _res, _args)


@dataclass
class WhisperConfig:
    n_mels: int = 80
    d_model: int = 384
    heads: int = 6
    enc_layers: int = 4
    dec_layers: int = 4
    ffn: int = 1536
    vocab: int = 51865
    n_audio: int = 1500
    max_target: int = 448
    bits: int = 4
    dtype: int = _lib.F16
    eps: float = 1e-5
    streams: int = 1  # independent windows decoded together (decode_batch)

    def c(self) -> WhisperCfg:
        return WhisperCfg(self.n_mels, self.d_model, self.heads, self.enc_layers, self.dec_layers, self.ffn,
                          self.vocab, self.n_audio, self.max_target, self.bits, self.dtype, self.eps, self.streams)


TINY = WhisperConfig()  # Whisper-tiny shapes, int4 decoder (config 1)
TURBO = WhisperConfig(n_mels=128, d_model=1280, heads=20, enc_layers=32, dec_layers=4, ffn=5120, vocab=51866,
                      bits=0)  # large-v3-turbo shapes, fp16 dense (config 3)


@dataclass
class DecodeResult:
    tokens: list
    prefill_ms: float
    decode_ms: float


class Whisper:
    def __init__(self, cfg: WhisperConfig, device: int = 0):
        self.cfg = cfg
        h = _vp()
        _lib.check(_lib.lib().vella_whisper_create(ctypes.byref(cfg.c()), device, ctypes.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            _lib.lib().vella_whisper_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed: int, std: float = 0.02):
        _lib.check(_lib.lib().vella_whisper_init_random(self.h, seed, std))

    def tensor(self, name: str, layer: int = -1):
        p, n = _vp(), ctypes.c_size_t()
        _lib.check(_lib.lib().vella_whisper_tensor(self.h, name.encode(), layer, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def encode(self, mel, on_host: Optional[bool] = None):
        """mel: numpy fp32 [n_mels, 2 * n_audio] ([streams, n_mels, 2 * n_audio] with several
        streams) on the host, or a device pointer / torch tensor."""
        if isinstance(mel, np.ndarray):
            m = np.ascontiguousarray(mel, np.float32)
            shape = (self.cfg.n_mels, 2 * self.cfg.n_audio)
            assert m.shape[-2:] == shape and m.size == max(self.cfg.streams, 1) * shape[0] * shape[1], m.shape
            _lib.check(_lib.lib().vella_whisper_encode(self.h, m.ctypes.data, 1))
        else:
            ptr = mel if isinstance(mel, int) else mel.data_ptr()
            _lib.check(_lib.lib().vella_whisper_encode(self.h, ptr, 0 if on_host is None else int(on_host)))

    def decode(self, prompt: Sequence[int], max_tokens: int, eot: int = -1) -> DecodeResult:
        pr = (ctypes.c_int32 * len(prompt))(*prompt)
        out = (ctypes.c_int32 * max(max_tokens, 1))()
        n = ctypes.c_int32()
        _lib.check(_lib.lib().vella_whisper_decode(self.h, pr, len(prompt), max_tokens, eot, out, ctypes.byref(n)))
        st = self.stats()
        return DecodeResult(list(out[: n.value]), st["prefill_ms"], st["decode_ms"])

    def decode_batch(self, prompt: Sequence[int], max_tokens: int) -> np.ndarray:
        """Greedy tokens [streams, max_tokens] of every stream after the same prompt."""
        S = max(self.cfg.streams, 1)
        pr = (ctypes.c_int32 * len(prompt))(*prompt)
        out = np.zeros((S, max(max_tokens, 1)), np.int32)
        _lib.check(_lib.lib().vella_whisper_decode_batch(self.h, pr, len(prompt), max_tokens,
                                                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out[:, :max_tokens]

    def set_rules(self, eot: Optional[int] = None, no_timestamps: int = 0, timestamp_begin: int = 0,
                  suppress: Sequence[int] = (), begin_suppress: Sequence[int] = ()):
        """Token rules of the reference's GPU-side greedy for the following decodes (suppress
        and begin-suppress masks, timestamp rules, summed log-probabilities in the stats);
        ``eot=None`` returns to plain argmax."""
        if eot is None:
            _lib.check(_lib.lib().vella_whisper_set_rules(self.h, None))
            return
        sup = (ctypes.c_int32 * max(len(suppress), 1))(*suppress)
        bsup = (ctypes.c_int32 * max(len(begin_suppress), 1))(*begin_suppress)
        r = WhisperRules(eot, no_timestamps, timestamp_begin, sup, len(suppress), bsup, len(begin_suppress))
        _lib.check(_lib.lib().vella_whisper_set_rules(self.h, ctypes.byref(r)))

    def score(self, tokens: Sequence[int]) -> np.ndarray:
        """Teacher-forced logits [T, vocab] as storage (float16, or bf16 bits as uint16)."""
        T = len(tokens)
        tk = (ctypes.c_int32 * T)(*tokens)
        dt = np.float16 if self.cfg.dtype == _lib.F16 else np.uint16
        out = np.empty((T, self.cfg.vocab), dt)
        _lib.check(_lib.lib().vella_whisper_score(self.h, tk, T, out.ctypes.data, 1))
        return out

    def stats(self) -> dict:
        s = WhisperStats()
        _lib.check(_lib.lib().vella_whisper_get_stats(self.h, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in WhisperStats._fields_}
