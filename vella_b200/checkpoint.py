"""Model directories: safetensors shards, config.json, the Whisper token ids, and the
Qwen3-style decoder models of the draft-and-verify path.

Mirrors the reference's ``WhisperModel.fromDirectory`` (``Worker/Sources/MLXAudioSTT/Whisper/
WhisperModel.swift:653-723``): ``config.json`` (Hugging Face or OpenAI/mlx-whisper keys,
``WhisperConfig.swift:95-140``), every ``*.safetensors`` file in file-name order (later keys
win), an optional ``quantization`` block (already-quantized checkpoint) or a derived
precision made at load (``bits``), and the tokenizer's special ids and suppress lists
(``WhisperTokenizer.swift:20-118``, ``WhisperModel.swift:209-214``).  The tensors are read and
placed by the library (``vella_st_*``, ``vella_whisper_load`` in ``include/vella_cuda.h``).
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib

_vp, _i32 = ctypes.c_void_p, ctypes.c_int32
for _name, _res, _args in [
    ("vella_st_open", ctypes.c_int, [ctypes.POINTER(ctypes.c_char_p), _i32, ctypes.POINTER(_vp)]),
    ("vella_st_close", ctypes.c_int, [_vp]),
    ("vella_st_count", ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    ("vella_st_find", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_i32)]),
    ("vella_st_info", ctypes.c_int, [_vp, _i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i32),
                                     ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_vp),
                                     ctypes.POINTER(ctypes.c_size_t)]),
    ("vella_whisper_check_checkpoint", ctypes.c_int, [_vp, _vp]),
    ("vella_whisper_load", ctypes.c_int, [_vp, _vp]),
    ("vella_model_check_checkpoint", ctypes.c_int, [_vp, _vp]),
    ("vella_model_load", ctypes.c_int, [_vp, _vp]),
    ("vella_nh_check_checkpoint", ctypes.c_int, [_vp, _vp]),
    ("vella_nh_load", ctypes.c_int, [_vp, _vp]),
]:
    _lib.declare(_name, _res, _args)

ST_DTYPES = {0: "BF16", 1: "F16", 2: "F32", 3: "U32", 4: "I32", 5: "U8", 6: "I8", 7: "I64", 8: "F64", 9: "U16",
             10: "I16", 11: "BOOL", 12: "U64", 13: "F8_E4M3", 14: "F8_E5M2"}
_NP = {"F16": np.float16, "F32": np.float32, "U32": np.uint32, "I32": np.int32, "U8": np.uint8, "I8": np.int8,
       "I64": np.int64, "F64": np.float64, "U16": np.uint16, "I16": np.int16, "BOOL": np.bool_, "U64": np.uint64,
       "BF16": np.uint16, "F8_E4M3": np.uint8, "F8_E5M2": np.uint8}


class SafeTensors:
    """Memory-mapped safetensors shards merged in the given order (later keys win)."""

    def __init__(self, paths: Sequence[str]):
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        self.h = ctypes.c_void_p()
        _lib.check(_lib.lib().vella_st_open(arr, len(paths), ctypes.byref(self.h)))

    def close(self):
        if self.h:
            _lib.lib().vella_st_close(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = _i32()
        _lib.check(_lib.lib().vella_st_count(self.h, ctypes.byref(n)))
        return n.value

    def _info(self, i: int):
        name, dt, nd = ctypes.c_char_p(), _i32(), _i32()
        shape = (ctypes.c_int64 * 8)()
        data, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        _lib.check(_lib.lib().vella_st_info(self.h, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd), shape,
                                            ctypes.byref(data), ctypes.byref(nbytes)))
        return name.value.decode(), ST_DTYPES[dt.value], tuple(shape[: nd.value]), data.value, nbytes.value

    def keys(self) -> List[str]:
        return [self._info(i)[0] for i in range(len(self))]

    def index(self, name: str) -> int:
        i = _i32()
        _lib.check(_lib.lib().vella_st_find(self.h, name.encode(), ctypes.byref(i)))
        return i.value

    def info(self, name: str):
        """(dtype name, shape) of a tensor."""
        i = self.index(name)
        if i < 0:
            raise KeyError(name)
        _, dt, shape, _, _ = self._info(i)
        return dt, shape

    def array(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes as numpy (bf16 and fp8 as their raw integer words)."""
        i = self.index(name)
        if i < 0:
            raise KeyError(name)
        _, dt, shape, ptr, nbytes = self._info(i)
        raw = ctypes.string_at(ptr, nbytes) if nbytes else b""
        return np.frombuffer(raw, dtype=_NP[dt]).reshape(shape).copy()


# ---------------------------------------------------------------------------------------
# Whisper
# ---------------------------------------------------------------------------------------

def whisper_config(cfg: dict, bits: Optional[int] = None, dtype: Optional[int] = None, streams: int = 1):
    """A ``WhisperConfig`` from config.json: Hugging Face keys first, then the OpenAI/mlx-whisper
    ones, then the reference's defaults (``WhisperConfig.swift:95-140``).  ``bits`` is the
    decoder's precision: the checkpoint's ``quantization.bits`` when it has one, else the
    argument (a derived precision, quantized at load), else 0 (dense)."""
    from .whisper import WhisperConfig

    def pick(*keys, default):
        for k in keys:
            if cfg.get(k) is not None:
                return cfg[k]
        return default

    d = pick("d_model", "n_audio_state", "n_text_state", default=384)
    q = cfg.get("quantization") or cfg.get("quantization_config")
    if q:
        if int(q.get("group_size", 64)) != 64:
            raise ValueError(f"quantized checkpoint with group size {q.get('group_size')} (the kernels use 64)")
        if bits is not None and bits != int(q["bits"]):
            raise ValueError("the checkpoint is already quantized")  # WhisperModel.swift:692-694
        bits = int(q["bits"])
    return WhisperConfig(
        n_mels=pick("num_mel_bins", "n_mels", default=80), d_model=d,
        heads=pick("encoder_attention_heads", "n_audio_head", default=6),
        enc_layers=pick("encoder_layers", "n_audio_layer", default=4),
        dec_layers=pick("decoder_layers", "n_text_layer", default=4),
        ffn=pick("encoder_ffn_dim", default=4 * d),
        vocab=pick("vocab_size", "n_vocab", default=51865),
        n_audio=pick("max_source_positions", "n_audio_ctx", default=1500),
        max_target=pick("max_target_positions", "n_text_ctx", default=448),
        bits=int(bits or 0), dtype=_lib.F16 if dtype is None else dtype, streams=streams)


def safetensors_files(model_dir) -> List[Path]:
    files = sorted(Path(model_dir).glob("*.safetensors"), key=lambda p: p.name)
    if not files:
        raise FileNotFoundError(f"No .safetensors files found in {model_dir}.")
    return files


def check_whisper_checkpoint(st: SafeTensors, cfg) -> None:
    """Raises VellaError naming the first missing or mis-shaped tensor."""
    c = cfg.c()
    _lib.check(_lib.lib().vella_whisper_check_checkpoint(st.h, ctypes.byref(c)))


def load_whisper(model_dir, bits: Optional[int] = None, dtype: Optional[int] = None, streams: int = 1,
                 device: int = 0):
    """A Whisper handle with the directory's weights (not yet encoded)."""
    from .whisper import Whisper
    model_dir = Path(model_dir)
    cfg = whisper_config(json.loads((model_dir / "config.json").read_text()), bits, dtype, streams)
    with SafeTensors([str(p) for p in safetensors_files(model_dir)]) as st:
        check_whisper_checkpoint(st, cfg)
        m = Whisper(cfg, device)
        try:
            _lib.check(_lib.lib().vella_whisper_load(m.h, st.h))
        except Exception:
            m.close()
            raise
    return m


@dataclass
class WhisperTokens:
    """Special ids, suppress lists and prompt of a checkpoint's tokenizer."""
    sot: int
    eot: int
    no_timestamps: int
    timestamp_begin: int
    transcribe: Optional[int] = None
    translate: Optional[int] = None
    prev_sot: Optional[int] = None
    sot_lm: Optional[int] = None
    no_speech: Optional[int] = None
    languages: Dict[str, int] = field(default_factory=dict)
    multilingual: bool = False
    suppress: List[int] = field(default_factory=list)
    begin_suppress: List[int] = field(default_factory=list)

    def prompt(self, language: Optional[str] = None, task: str = "transcribe",
               without_timestamps: bool = False) -> List[int]:
        """``buildPromptTokens`` (WhisperTokenizer.swift:99-118)."""
        toks = [self.sot]
        if self.multilingual:
            lang = self.languages.get(_lang_key(language)) if language else None
            if lang is not None:
                toks.append(lang)
            task_id = self.translate if task.lower() == "translate" else self.transcribe
            if task_id is not None:
                toks.append(task_id)
        if without_timestamps:
            toks.append(self.no_timestamps)
        return toks

    def rules(self) -> dict:
        """Keyword arguments of ``Whisper.set_rules``."""
        return {"eot": self.eot, "no_timestamps": self.no_timestamps, "timestamp_begin": self.timestamp_begin,
                "suppress": self.suppress, "begin_suppress": self.begin_suppress}


def _lang_key(s: str) -> str:
    s = s.strip().lower()
    if s.startswith("<|") and s.endswith("|>"):
        s = s[2:-2]
    return s


def whisper_tokens(model_dir) -> WhisperTokens:
    """Special ids from generation_config.json, then tokenizer_config.json's
    ``added_tokens_decoder``, then config.json (WhisperTokenizer.swift:20-90); suppress lists as
    ``transcribeChunk`` builds them (WhisperModel.swift:209-214)."""
    model_dir = Path(model_dir)

    def read(name):
        p = model_dir / name
        return json.loads(p.read_text()) if p.exists() else {}

    base, gen = read("config.json"), read("generation_config.json")
    added = {int(k): v.get("content") for k, v in (read("tokenizer_config.json").get("added_tokens_decoder") or {}).items()
             if isinstance(v, dict)}
    by_name = {v: k for k, v in sorted(added.items())}
    vocab = base.get("vocab_size", base.get("n_vocab", 51865))
    start = base.get("decoder_start_token_id", 50258)

    def first(*vals):
        for v in vals:
            if v is not None:
                return v
        return None

    sot = first(gen.get("decoder_start_token_id"), by_name.get("<|startoftranscript|>"), start)
    eot = first(gen.get("eos_token_id"), by_name.get("<|endoftext|>"), base.get("eos_token_id", 50257))
    no_ts = first(gen.get("no_timestamps_token_id"), by_name.get("<|notimestamps|>"),
                  start + (105 if vocab > 51864 else 104))
    task = gen.get("task_to_id") or {}
    langs = {_lang_key(k): v for k, v in (gen.get("lang_to_id") or {}).items()}
    for tid, name in added.items():
        key = _lang_key(name or "")
        if name and name.startswith("<|") and 2 <= len(key) <= 3 and key.isalpha():
            langs[key] = tid
    t = WhisperTokens(sot=sot, eot=eot, no_timestamps=no_ts, timestamp_begin=no_ts + 1,
                      transcribe=first(task.get("transcribe"), by_name.get("<|transcribe|>")),
                      translate=first(task.get("translate"), by_name.get("<|translate|>")),
                      prev_sot=first(gen.get("prev_sot_token_id"), by_name.get("<|startofprev|>")),
                      sot_lm=by_name.get("<|startoflm|>"), no_speech=by_name.get("<|nospeech|>"),
                      languages=langs,
                      multilingual=bool(gen["is_multilingual"]) if "is_multilingual" in gen else bool(langs))
    t.begin_suppress = list(gen.get("begin_suppress_tokens") or [220, eot])
    sup = list(gen.get("suppress_tokens") or [])
    sup += [x for x in (t.transcribe, t.translate, t.prev_sot, t.sot_lm, t.no_speech, t.sot) if x is not None]
    t.suppress = sorted(set(sup))
    return t


# ---------------------------------------------------------------------------------------
# Qwen3-style decoder (the draft-and-verify target and draft)
# ---------------------------------------------------------------------------------------

def model_config(cfg: dict, bits: Optional[int] = None, dtype: Optional[int] = None, qk_norm: bool = True,
                 **kw):
    """A ``decode.ModelConfig`` from a Qwen3 config.json (or a Qwen3-ASR one, whose text model
    sits under ``thinker_config.text_config``); ``bits`` as in ``whisper_config``; the dtype
    from ``torch_dtype`` (bf16 unless it says float16); ``kw`` sets the handle's capacities
    (max_seq, max_prefix, streams, rows_per_stream)."""
    from .decode import ModelConfig
    c = (cfg.get("thinker_config") or {}).get("text_config") or cfg.get("text_config") or cfg
    q = cfg.get("quantization") or cfg.get("quantization_config") or c.get("quantization")
    if q:
        if int(q.get("group_size", 64)) != 64:
            raise ValueError(f"quantized checkpoint with group size {q.get('group_size')} (the kernels use 64)")
        if bits is not None and bits != int(q["bits"]):
            raise ValueError("the checkpoint is already quantized")
        bits = int(q["bits"])
    if dtype is None:
        dtype = _lib.F16 if str(c.get("torch_dtype", cfg.get("torch_dtype", ""))) == "float16" else _lib.BF16
    d, H = c["hidden_size"], c["num_attention_heads"]
    return ModelConfig(n_layers=c["num_hidden_layers"], d_model=d, n_heads=H,
                       n_kv_heads=c.get("num_key_value_heads", H), head_dim=c.get("head_dim") or d // H,
                       ffn=c["intermediate_size"], vocab=c["vocab_size"], bits=int(bits or 0), dtype=dtype,
                       qk_norm=qk_norm, rms_eps=float(c.get("rms_norm_eps", 1e-6)),
                       rope_theta=float(c.get("rope_theta", 1e6)), **kw)


def check_model_checkpoint(st: SafeTensors, cfg) -> None:
    c = cfg.c()
    _lib.check(_lib.lib().vella_model_check_checkpoint(st.h, ctypes.byref(c)))


def load_model(model_dir, bits: Optional[int] = None, dtype: Optional[int] = None, device: int = 0, **kw):
    """A decoder model handle with the directory's weights; q/k RMSNorm when the checkpoint
    has them."""
    from .decode import Model
    model_dir = Path(model_dir)
    raw = json.loads((model_dir / "config.json").read_text())
    with SafeTensors([str(p) for p in safetensors_files(model_dir)]) as st:
        qk = any(st.index(pre + "model.layers.0.self_attn.q_norm.weight") >= 0 for pre in ("", "thinker."))
        cfg = model_config(raw, bits, dtype, qk_norm=qk, **kw)
        check_model_checkpoint(st, cfg)
        m = Model(cfg, device)
        try:
            _lib.check(_lib.lib().vella_model_load(m.handle, st.h))
        except Exception:
            m.close()
            raise
    return m



# ---------------------------------------------------------------------------------------
# Nemotron-H (NeMo or MLX layout)
# ---------------------------------------------------------------------------------------

def check_nh_checkpoint(st: SafeTensors, cfg) -> None:
    """Raises VellaError naming the first missing or mis-shaped tensor of a Nemotron-H checkpoint."""
    c = cfg.c()
    _lib.check(_lib.lib().vella_nh_check_checkpoint(st.h, ctypes.byref(c)))


def load_nh(paths, cfg, device: int = 0):
    """A Nemotron-H backbone handle (``vella_b200.nemotron.NHModel``) with the weights of the
    safetensors files (in the order given)."""
    from .nemotron import NHModel
    with SafeTensors([str(p) for p in paths]) as st:
        check_nh_checkpoint(st, cfg)
        m = NHModel(cfg, device)
        try:
            _lib.check(_lib.lib().vella_nh_load(m.h, st.h))
        except Exception:
            m.close()
            raise
    return m
