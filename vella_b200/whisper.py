"""ctypes binding of the Whisper encoder + decoder step (``vella_whisper_*`` in
``include/vella_cuda.h``).

The model runs in the library (C++ host code, CUDA kernels, one CUDA graph per decoder step);
this module marshals arguments for the tests and the benchmark.  Names follow the reference's
``WhisperModel`` (``Worker/Sources/MLXAudioSTT/Whisper/WhisperModel.swift``): ``encode`` runs
the encoder and projects the cross-attention K/V (``encode_audio`` computes the log-mel
features first), ``decode`` the greedy loop, under the token rules once ``set_rules`` is
called, ``decode_with_fallback`` the temperature fallback.
"""
from __future__ import annotations

import ctypes
import zlib
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _lib


FALLBACK_TEMPERATURES = (0.0, 0.2, 0.4, 0.6, 0.8, 1.0)  # WhisperModel.swift:218-219


def log_mel(audio, n_mels: int = 80):
    """Whisper's log-mel features [streams, n_mels, 3000] of windows of 16 kHz mono audio
    ([streams, n] or [n]; CUDA tensors stay on their device), computed by the library."""
    import torch
    a = torch.as_tensor(audio, dtype=torch.float32)
    if not a.is_cuda:
        a = a.cuda()
    a = a.reshape(-1, a.shape[-1]).contiguous()
    out = torch.empty((a.shape[0], n_mels, 3000), dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        st = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().vella_whisper_log_mel(a.data_ptr(), a.shape[1], a.shape[0], n_mels, out.data_ptr(), st))
    return out


def compression_ratio(text: str) -> float:
    """UTF-8 bytes over zlib-compressed bytes (default level); 0 for empty text
    (``compressionRatio``, WhisperModel.swift:434-445)."""
    raw = text.encode("utf-8")
    return 0.0 if not raw else len(raw) / len(zlib.compress(raw, 6))


def attempt_verdict(sum_logprob: float, n_tokens: int, text: str, no_speech_prob: float = 0.0) -> str:
    """'empty', 'accept' or 'retry' after one attempt (WhisperModel.swift:285-291): the
    average log-probability counts the end-of-text step; no-speech above 0.6 with an average
    below -1 empties the window; an average >= -1 with a compression ratio <= 2.4 accepts."""
    average = sum_logprob / (n_tokens + 1)
    if no_speech_prob > 0.6 and average < -1:
        return "empty"
    if average >= -1 and compression_ratio(text) <= 2.4:
        return "accept"
    return "retry"


@dataclass
class FallbackResult:
    tokens: List[int]
    temperature: float
    sum_logprob: float
    avg_logprob: float
    compression_ratio: float
    attempts: int
    verdict: str


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
    ("vella_whisper_encode_audio", ctypes.c_int, [_vp, _vp, ctypes.c_int64, _i32]),
    ("vella_whisper_log_mel", ctypes.c_int, [_vp, ctypes.c_int64, _i32, _i32, _vp, _vp]),
    ("vella_whisper_decode", ctypes.c_int, [_vp, _pi32, _i32, _i32, _i32, _pi32, _pi32]),
    ("vella_whisper_decode_batch", ctypes.c_int, [_vp, _pi32, _i32, _i32, _pi32]),
    ("vella_whisper_decode_batch_eot", ctypes.c_int, [_vp, _pi32, _i32, _i32, _i32, _pi32, _pi32]),
    ("vella_whisper_get_logprobs", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_float), _i32]),
    ("vella_whisper_begin", ctypes.c_int, [_vp, _pi32, _i32, _pi32]),
    ("vella_whisper_step", ctypes.c_int, [_vp, _pi32]),
    ("vella_whisper_score", ctypes.c_int, [_vp, _pi32, _i32, _vp, _i32]),
    ("vella_whisper_get_stats", ctypes.c_int, [_vp, ctypes.POINTER(WhisperStats)]),
    ("vella_whisper_set_rules", ctypes.c_int, [_vp, ctypes.POINTER(WhisperRules)]),
    ("vella_whisper_set_sampling", ctypes.c_int, [_vp, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint32]),
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
            if not isinstance(mel, int) and getattr(mel, "is_cuda", False):
                import torch
                # the handle's stream does not wait for torch's: the features must be complete
                torch.cuda.current_stream(mel.device).synchronize()
            ptr = mel if isinstance(mel, int) else mel.data_ptr()
            _lib.check(_lib.lib().vella_whisper_encode(self.h, ptr, 0 if on_host is None else int(on_host)))

    def encode_audio(self, audio):
        """Log-mel features of every stream's window of 16 kHz mono audio ([streams, n] or [n],
        a numpy array or a CUDA tensor), then the encoder."""
        import torch
        if isinstance(audio, torch.Tensor) and audio.is_cuda:
            a = audio.float().contiguous()
            torch.cuda.current_stream(a.device).synchronize()  # the handle's stream does not wait for torch's
            _lib.check(_lib.lib().vella_whisper_encode_audio(self.h, a.data_ptr(), a.shape[-1], 0))
            return
        a = np.ascontiguousarray(np.asarray(audio, np.float32))
        _lib.check(_lib.lib().vella_whisper_encode_audio(self.h, a.ctypes.data, a.shape[-1], 1))

    def decode(self, prompt: Sequence[int], max_tokens: int, eot: int = -1) -> DecodeResult:
        pr = (ctypes.c_int32 * len(prompt))(*prompt)
        out = (ctypes.c_int32 * max(max_tokens, 1))()
        n = ctypes.c_int32()
        _lib.check(_lib.lib().vella_whisper_decode(self.h, pr, len(prompt), max_tokens, eot, out, ctypes.byref(n)))
        st = self.stats()
        return DecodeResult(list(out[: n.value]), st["prefill_ms"], st["decode_ms"])

    def decode_batch(self, prompt: Sequence[int], max_tokens: int, eot: int = -1):
        """Tokens of every stream after the same prompt: [streams, max_tokens] without an
        end-of-text id, else one list per stream of its tokens before ``eot``."""
        S = max(self.cfg.streams, 1)
        pr = (ctypes.c_int32 * len(prompt))(*prompt)
        out = np.zeros((S, max(max_tokens, 1)), np.int32)
        optr = out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
        if eot < 0:
            _lib.check(_lib.lib().vella_whisper_decode_batch(self.h, pr, len(prompt), max_tokens, optr))
            return out[:, :max_tokens]
        n = np.zeros(S, np.int32)
        _lib.check(_lib.lib().vella_whisper_decode_batch_eot(self.h, pr, len(prompt), max_tokens, eot, optr,
                                                             n.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return [list(out[st, :n[st]]) for st in range(S)]

    def begin(self, prompt: Sequence[int]) -> int:
        """Runs the prompt; returns the first token (then ``step()`` for each next one)."""
        pr = (ctypes.c_int32 * len(prompt))(*prompt)
        t = ctypes.c_int32()
        _lib.check(_lib.lib().vella_whisper_begin(self.h, pr, len(prompt), ctypes.byref(t)))
        return t.value

    def step(self) -> int:
        """One decoder step after ``begin``; returns the next token."""
        t = ctypes.c_int32()
        _lib.check(_lib.lib().vella_whisper_step(self.h, ctypes.byref(t)))
        return t.value

    def logprobs(self) -> np.ndarray:
        """Each stream's summed log-probability over the last decode (token rules set)."""
        S = max(self.cfg.streams, 1)
        out = np.zeros(S, np.float32)
        _lib.check(_lib.lib().vella_whisper_get_logprobs(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), S))
        return out

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

    def set_sampling(self, temperature: float, seed: int = 0x5EED, draw: int = 0):
        """Temperature of the following decodes (0: argmax; > 0 draws under the token rules,
        Philox noise keyed by ``seed`` with counter word ``draw``)."""
        _lib.check(_lib.lib().vella_whisper_set_sampling(self.h, float(temperature), int(seed) & (2**64 - 1),
                                                         int(draw) & 0xFFFFFFFF))

    def decode_with_fallback(self, prompt: Sequence[int], max_tokens: int, eot: int,
                             detokenize: Optional[Callable[[List[int]], str]] = None,
                             temperatures: Sequence[float] = FALLBACK_TEMPERATURES, seed: int = 0x5EED,
                             no_speech_prob: float = 0.0, draw_base: int = 0) -> FallbackResult:
        """The reference's temperature fallback for one window (``transcribeChunk``,
        WhisperModel.swift:218-292): attempts at 0, 0.2, .. 1.0 until the average
        log-probability (end-of-text step counted) is >= -1 and the compression ratio of
        ``detokenize(tokens)`` is <= 2.4; an attempt whose average is < -1 while
        ``no_speech_prob`` > 0.6 gives an empty window; if every attempt asks for a retry the
        last one stands.  Token rules must be set.  Attempt i draws with counter word
        draw_base + i.
        Without ``detokenize`` the compression test passes (ratio 0, the reference's value for
        empty text)."""
        res = None
        try:
            for i, temp in enumerate(temperatures):
                self.set_sampling(temp, seed, draw_base + i)
                out = self.decode(prompt, max_tokens, eot)
                lp = float(self.stats()["sum_logprob"])
                text = detokenize(out.tokens) if detokenize is not None else ""
                verdict = attempt_verdict(lp, len(out.tokens), text, no_speech_prob)
                res = FallbackResult(list(out.tokens), float(temp), lp, lp / (len(out.tokens) + 1),
                                     compression_ratio(text), i + 1, verdict)
                if verdict == "empty":
                    res.tokens = []
                if verdict != "retry":
                    break
        finally:
            self.set_sampling(0.0, seed, 0)
        return res

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


# ---------------------------------------------------------------------------------------
# The plugin boundary: generate(audio:) of the reference's STTGenerationModel
# ---------------------------------------------------------------------------------------

SAMPLE_RATE, WINDOW_SAMPLES = 16000, 480000  # WhisperAudioConfig: 16 kHz, 30 s windows


@dataclass
class STTOutput:
    """The fields of the reference's STTOutput (Shared/STTOutput.swift:34-88) this path fills."""
    text: str
    segments: Optional[List[dict]]
    language: Optional[str]
    prompt_tokens: int
    generation_tokens: int
    total_tokens: int
    prompt_tps: float
    generation_tps: float
    total_time: float


def chunk_audio(audio: np.ndarray) -> List[tuple]:
    """``chunkAudioFor30sWindows`` (WhisperModel.swift:150-166): consecutive 30 s windows, the
    last one shorter; (samples, offset in seconds) each."""
    n = audio.shape[0]
    if n <= WINDOW_SAMPLES:
        return [(audio, 0.0)]
    return [(audio[i:min(n, i + WINDOW_SAMPLES)], i / SAMPLE_RATE) for i in range(0, n, WINDOW_SAMPLES)]


class WhisperSTT:
    """``WhisperModel.generate(audio:generationParameters:)`` (WhisperModel.swift:84-140) over a
    one-stream handle with its token rules set: mono mix-down, 30 s windows, per window the
    log-mel features and the encoder on the device, the prompt, and the decode with the
    temperature fallback (``decode_with_fallback``); the windows' trimmed texts joined by
    spaces, a segment per non-empty window.  ``detokenize`` maps token ids to text (the
    tokenizer is not part of this library).  Language detection is the caller's: pass the
    language; ``no_speech_prob`` of a window, when known, comes through ``no_speech``."""

    def __init__(self, model, tokens, detokenize: Callable[[List[int]], str], seed: int = 0x5EED,
                 no_speech: Optional[Callable[[int], float]] = None):
        self.model, self.tokens, self.detokenize, self.seed = model, tokens, detokenize, seed
        self.no_speech = no_speech

    def generate(self, audio, temperature: float = 0.0, language: Optional[str] = None,
                 max_tokens: int = 1024) -> STTOutput:
        import time
        t0 = time.perf_counter()
        a = np.asarray(audio, np.float32)
        mono = a.mean(axis=-1) if a.ndim > 1 else a
        # the reference hands Whisper its default sample_len, n_text_ctx / 2 (WhisperModel.swift:215-217)
        limit = max(1, min(max_tokens, self.model.cfg.max_target // 2))
        prompt = self.tokens.prompt(language, "transcribe", without_timestamps=False)
        temps = FALLBACK_TEMPERATURES if temperature == 0 else (temperature,)
        texts, segments, n_prompt, n_gen = [], [], 0, 0
        for i, (chunk, offset) in enumerate(chunk_audio(mono)):
            self.model.encode_audio(chunk)
            # one seed per request; every window and attempt draws its own Philox counter word
            res = self.model.decode_with_fallback(
                prompt, min(limit, self.model.cfg.max_target - len(prompt)), self.tokens.eot, self.detokenize,
                temps, self.seed, self.no_speech(i) if self.no_speech else 0.0, draw_base=i * len(temps))
            n_prompt += len(prompt)
            n_gen += len(res.tokens)
            text = self.detokenize(res.tokens).strip() if res.tokens else ""
            if text:
                texts.append(text)
                segments.append({"text": text, "start": offset, "end": offset + chunk.shape[0] / SAMPLE_RATE})
        elapsed = time.perf_counter() - t0
        return STTOutput(" ".join(texts), segments or None, language, n_prompt, n_gen, n_prompt + n_gen,
                         n_prompt / elapsed if elapsed > 0 else 0.0, n_gen / elapsed if elapsed > 0 else 0.0, elapsed)

