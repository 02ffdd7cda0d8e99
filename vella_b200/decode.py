"""ctypes binding of the resident decoder model and the draft-and-verify loop
(``vella_model_*`` / ``vella_spec_*`` in ``include/vella_cuda.h``).

The loop itself runs in the library (C++ host code + CUDA graphs); this module only
marshals arguments for tests and the benchmark.  Method names follow the reference's
decoder (``NemotronTranscribeModel.decodeMTP / decodeGreedy / decode``,
``Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeModel.swift:266-443``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib

DRAFT_MODEL, DRAFT_ORACLE = 0, 1
DECODE_AUTO, DECODE_SPEC, DECODE_GREEDY = 0, 1, 2
FAULT_NONE, FAULT_THROW, FAULT_NONFINITE = 0, 1, 2
FLAG_LOOPED, FLAG_FELL_BACK, FLAG_RUNAWAY_RETRY, FLAG_CAPACITY = 1, 2, 4, 8


class ModelCfg(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("d_model", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("ffn", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("bits", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("qk_norm", ctypes.c_int32), ("max_seq", ctypes.c_int32), ("max_prefix", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("streams", ctypes.c_int32),
                ("rows_per_stream", ctypes.c_int32)]


class SpecCfg(ctypes.Structure):
    _fields_ = [("draft_k", ctypes.c_int32), ("draft_mode", ctypes.c_int32), ("oracle_p", ctypes.c_float),
                ("seed", ctypes.c_uint64), ("n_eos", ctypes.c_int32), ("eos", ctypes.c_int32 * 8),
                ("use_graphs", ctypes.c_int32), ("temperature", ctypes.c_float), ("tree_depth", ctypes.c_int32),
                ("tree_branching", ctypes.c_int32 * 8)]


class SpecStats(ctypes.Structure):
    _fields_ = [("passes", ctypes.c_int64), ("greedy_steps", ctypes.c_int64), ("accepted", ctypes.c_int64 * 16),
                ("fallbacks", ctypes.c_int64), ("runaway_retries", ctypes.c_int64),
                ("draft_disabled", ctypes.c_int32), ("last_decode_ms", ctypes.c_float),
                ("last_tokens", ctypes.c_int32), ("last_prefill_ms", ctypes.c_float)]


_vp, _i32, _pi32 = ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)
for _name, _res, _args in [
    ("vella_quantize", ctypes.c_int, [ctypes.POINTER(_lib.QgemmDesc), _i32, _vp, _vp, _vp, _vp, _vp]),
    ("vella_fill_normal", ctypes.c_int, [_vp, ctypes.c_size_t, _i32, ctypes.c_uint64, ctypes.c_uint32,
                                         ctypes.c_float, ctypes.c_float, _vp]),
    ("vella_model_create", ctypes.c_int, [ctypes.POINTER(ModelCfg), _i32, ctypes.POINTER(_vp)]),
    ("vella_model_destroy", ctypes.c_int, [_vp]),
    ("vella_model_init_random", ctypes.c_int, [_vp, ctypes.c_uint64, ctypes.c_float]),
    ("vella_model_tensor", ctypes.c_int, [_vp, ctypes.c_char_p, _i32, ctypes.POINTER(_vp),
                                          ctypes.POINTER(ctypes.c_size_t)]),
    ("vella_model_weight_bytes", ctypes.c_size_t, [_vp]),
    ("vella_model_score", ctypes.c_int, [_vp, _vp, _i32, _pi32, _i32, _vp, _i32]),
    ("vella_spec_create", ctypes.c_int, [_vp, _vp, ctypes.POINTER(SpecCfg), ctypes.POINTER(_vp)]),
    ("vella_spec_destroy", ctypes.c_int, [_vp]),
    ("vella_spec_set_prefix", ctypes.c_int, [_vp, _vp, _vp, _i32, _i32]),
    ("vella_spec_set_reference", ctypes.c_int, [_vp, _pi32, _i32]),
    ("vella_spec_prefill", ctypes.c_int, [_vp, _pi32]),
    ("vella_spec_step", ctypes.c_int, [_vp, _pi32, _pi32]),
    ("vella_spec_greedy_step", ctypes.c_int, [_vp, _pi32]),
    ("vella_spec_decode", ctypes.c_int, [_vp, _i32, _i32, _pi32, _i32, _pi32, _pi32]),
    ("vella_spec_decode_batch", ctypes.c_int, [_vp, _i32, _i32, _pi32, _pi32]),
    ("vella_spec_get_stats", ctypes.c_int, [_vp, ctypes.POINTER(SpecStats)]),
    ("vella_spec_set_fault", ctypes.c_int, [_vp, _i32]),
    ("vella_model_set_persistent", ctypes.c_int, [_vp, _i32]),
    ("vella_spec_tensor", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_size_t)]),
    ("vella_spec_reset", ctypes.c_int, [_vp]),
]:
    _lib.declare(_name, _res, _args)


def _i32_array(values: Sequence[int]):
    arr = np.ascontiguousarray(np.asarray(values, dtype=np.int32))
    return arr, arr.ctypes.data_as(_pi32)


@dataclass
class ModelConfig:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    bits: int = 4
    dtype: int = _lib.BF16
    qk_norm: bool = False
    max_seq: int = 2048
    max_prefix: int = 1024
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    streams: int = 1
    rows_per_stream: int = 16

    def c(self) -> ModelCfg:
        return ModelCfg(self.n_layers, self.d_model, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn,
                        self.vocab, self.bits, self.dtype, int(self.qk_norm), self.max_seq, self.max_prefix,
                        self.rms_eps, self.rope_theta, self.streams, self.rows_per_stream)


class Model:
    """A resident decoder on one GPU (weights + KV cache + prefix buffer)."""

    def __init__(self, cfg: ModelConfig, device: int = 0):
        self.cfg = cfg
        self.handle = _vp()
        c = cfg.c()
        _lib.check(_lib.lib().vella_model_create(ctypes.byref(c), device, ctypes.byref(self.handle)))

    def close(self):
        if self.handle:
            _lib.lib().vella_model_destroy(self.handle)
            self.handle = _vp()

    __del__ = close

    def init_random(self, seed: int, std: float = 0.02):
        _lib.check(_lib.lib().vella_model_init_random(self.handle, seed, std))

    def tensor(self, name: str, layer: int = -1):
        p, n = _vp(), ctypes.c_size_t()
        _lib.check(_lib.lib().vella_model_tensor(self.handle, name.encode(), layer, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def set_persistent(self, on: bool):
        """Decode-sized forwards as one persistent launch (where the shapes allow) or as per-op
        kernels (the default).  Same arithmetic; int4 GEMMs may differ in the last bits."""
        _lib.check(_lib.lib().vella_model_set_persistent(self.handle, int(bool(on))))

    def weight_bytes(self) -> int:
        return int(_lib.lib().vella_model_weight_bytes(self.handle))

    def score(self, prefix: np.ndarray, tokens: Sequence[int]) -> np.ndarray:
        """Teacher-forced logits [T, V] (storage dtype: uint16 bf16 bits / float16)."""
        prefix = np.ascontiguousarray(prefix)
        arr, ptr = _i32_array(tokens)
        out = np.empty((len(arr), self.cfg.vocab), dtype=np.uint16 if self.cfg.dtype == _lib.BF16 else np.float16)
        _lib.check(_lib.lib().vella_model_score(self.handle, prefix.ctypes.data, prefix.shape[0], ptr, len(arr),
                                                out.ctypes.data, 1))
        return out


@dataclass
class DecodeResult:
    tokens: list
    flags: int
    ms: float = 0.0
    stats: Optional[dict] = field(default=None)

    @property
    def looped(self) -> bool:
        return bool(self.flags & FLAG_LOOPED)


class SpecDecoder:
    """Draft-and-verify decoding over a target (verifier) and an optional draft model."""

    def __init__(self, target: Model, draft: Optional[Model], k: int = 4, mode: int = DRAFT_MODEL,
                 oracle_p: float = 0.0, seed: int = 0, eos: Sequence[int] = (), use_graphs: bool = True,
                 temperature: float = 0.0, tree: Sequence[int] = ()):
        eos_arr = (ctypes.c_int32 * 8)(*list(eos)[:8])
        br = (ctypes.c_int32 * 8)(*list(tree)[:8])
        self.cfg = SpecCfg(k, mode, oracle_p, seed, len(list(eos)[:8]), eos_arr, int(use_graphs), temperature,
                           len(list(tree)[:8]), br)
        self.handle = _vp()
        self.target, self.draft = target, draft
        _lib.check(_lib.lib().vella_spec_create(target.handle, draft.handle if draft else None,
                                                ctypes.byref(self.cfg), ctypes.byref(self.handle)))

    def close(self):
        if self.handle:
            _lib.lib().vella_spec_destroy(self.handle)
            self.handle = _vp()

    __del__ = close

    def set_prefix(self, target_embeds: Optional[np.ndarray], draft_embeds: Optional[np.ndarray], T: int = None):
        t = None if target_embeds is None else np.ascontiguousarray(target_embeds)
        d = None if draft_embeds is None else np.ascontiguousarray(draft_embeds)
        n = T if T is not None else t.shape[-2]  # [T, d], or [streams, T, d] stream-major
        _lib.check(_lib.lib().vella_spec_set_prefix(self.handle, None if t is None else t.ctypes.data,
                                                    None if d is None else d.ctypes.data, n, 1))

    def set_reference(self, tokens):
        """Oracle-draft continuation: [n] tokens, or [streams, n] for several streams."""
        arr = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        _lib.check(_lib.lib().vella_spec_set_reference(self.handle, arr.ctypes.data_as(_pi32), arr.shape[-1]))

    def prefill(self) -> int:
        v = ctypes.c_int32()
        _lib.check(_lib.lib().vella_spec_prefill(self.handle, ctypes.byref(v)))
        return v.value

    def step(self) -> list:
        out = (ctypes.c_int32 * 16)()
        n = ctypes.c_int32()
        _lib.check(_lib.lib().vella_spec_step(self.handle, out, ctypes.byref(n)))
        return list(out[:n.value])

    def greedy_step(self) -> int:
        v = ctypes.c_int32()
        _lib.check(_lib.lib().vella_spec_greedy_step(self.handle, ctypes.byref(v)))
        return v.value

    def decode(self, max_tokens: int, mode: int = DECODE_AUTO) -> DecodeResult:
        """One decode through vella_spec_decode.  The result's stats count this call only
        (passes, greedy steps, fallbacks, runaway retries and the accepted-length histogram are
        the differences of the handle's cumulative counters, which stats() returns)."""
        cap = max(max_tokens, 1)
        out = (ctypes.c_int32 * cap)()
        n, flags = ctypes.c_int32(), ctypes.c_int32()
        before = self.stats()
        _lib.check(_lib.lib().vella_spec_decode(self.handle, mode, max_tokens, out, cap, ctypes.byref(n),
                                                ctypes.byref(flags)))
        st = self.stats()
        for key in ("passes", "greedy_steps", "fallbacks", "runaway_retries"):
            st[key] -= before[key]
        st["accepted"] = [a - b for a, b in zip(st["accepted"], before["accepted"])]
        return DecodeResult(list(out[:n.value]), flags.value, st["last_decode_ms"], st)

    def decode_greedy(self, max_tokens: int) -> DecodeResult:
        return self.decode(max_tokens, DECODE_GREEDY)

    def decode_mtp(self, max_tokens: int) -> DecodeResult:
        return self.decode(max_tokens, DECODE_SPEC)

    def decode_batch(self, max_tokens: int, mode: int = DECODE_SPEC) -> np.ndarray:
        """Every stream's first max_tokens tokens, [streams, max_tokens] (models with streams > 1)."""
        streams = self.target.cfg.streams
        out = np.zeros((streams, max_tokens), np.int32)
        n = np.zeros(streams, np.int32)
        _lib.check(_lib.lib().vella_spec_decode_batch(self.handle, mode, max_tokens, out.ctypes.data_as(_pi32),
                                                      n.ctypes.data_as(_pi32)))
        return out

    def stats(self) -> dict:
        s = SpecStats()
        _lib.check(_lib.lib().vella_spec_get_stats(self.handle, ctypes.byref(s)))
        return {"passes": s.passes, "greedy_steps": s.greedy_steps, "accepted": list(s.accepted),
                "fallbacks": s.fallbacks, "runaway_retries": s.runaway_retries,
                "draft_disabled": bool(s.draft_disabled), "last_decode_ms": s.last_decode_ms,
                "last_tokens": s.last_tokens, "last_prefill_ms": s.last_prefill_ms}

    def tensor(self, name: str):
        """(device pointer, bytes) of a decoder buffer (vella_spec_tensor)."""
        p, n = _vp(), ctypes.c_size_t()
        _lib.check(_lib.lib().vella_spec_tensor(self.handle, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def set_fault(self, fault: int):
        _lib.check(_lib.lib().vella_spec_set_fault(self.handle, fault))

    def reset(self):
        _lib.check(_lib.lib().vella_spec_reset(self.handle))
