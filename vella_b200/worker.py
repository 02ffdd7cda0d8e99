"""The dictation helper's stdio protocol (one JSON object per line), as a drop-in for the
reference's `VellaWorker` (Worker/Sources/VellaWorker/WorkerMain.swift:99-123,
DictationService.swift:446-547): the app writes requests with an `id`, the helper answers
each with a reply carrying that `id`, and pushes a `{"status": ...}` line before every reply
that changes (or reports) its state.

Run as ``python -m vella_b200.worker``.  Requests:

* ``{"id", "op": "status"}`` / ``"trim"`` / ``"unload"`` -- the status line, then ``ok`` /
  ``unloaded``;
* ``{"id", "op": "load", "model": "/abs/dir"}`` -- load (or report the loaded model), then
  ``{"loaded": true, "metrics": ...}`` or ``{"error": {"code": "load", ...}}``;
* ``{"id", "model", "audio"[, "options"]}`` -- transcribe a 16 kHz mono 16-bit WAV file,
  loading the model first when it is not the loaded one;
* anything else -- ``{"error": {"code": "invalid", ...}, "id": <id or null>}``.

Lines are written with sorted keys, unescaped slashes, every non-ASCII UTF-16 unit as
``\\uXXXX`` and doubles with 17 significant digits (Transport.swift:4-17), so the bytes match
the reference helper's (tests/test_worker_wire.py against its wire fixtures).  Metric and
status field names keep the reference's (``peakMLXBytes`` ...): the app and scripts read
them; on this machine they report the CUDA allocator and the process.

Runtimes: ``whisper`` checkpoints run on the B200 Whisper path (vella_b200.whisper, loaded by
vella_b200.checkpoint; text through the checkpoint's own tokenizer files), and the ``stub``
test model (``VELLA_STUB_MODELS=1``: a folder whose config.json says ``"model_type": "stub"``)
answers ``stub:<folder> <seconds>s`` without the GPU.  The other architectures the reference
admits (parakeet, qwen3_asr, nemotron_transcribe) pass admission and then fail their load as
the reference does for an architecture without a runtime.
"""
import json
import math
import os
import resource
import signal
import sys
import time
from typing import Any, Dict, Optional

GATE_VERSION = "native-kernels-10"          # the gate version the app's status readers expect
MAX_LINE = 16 * 1024                        # request line limit (Validation.swift:7)
CACHE_BYTES = 64 * 1024 * 1024              # allocator cache limit reported per request (Validation.swift:8)
INVALID = {"code": "invalid", "message": "Invalid local transcription request."}

# Environment switches reported in the status `test_hooks` when set (the worker-reported
# entries of the reference's registry, EnvironmentSwitch.swift:29-90), and the prefix family.
REPORTED_SWITCHES = (
    "VELLA_PARAKEET_FAST", "VELLA_PARAKEET_NAX", "VELLA_PARAKEET_INT8", "VELLA_PARAKEET_INT4",
    "VELLA_PARAKEET_TAILBLOCK", "VELLA_TEST_TOLERANT_FAULT", "VELLA_NEMO_KEEPCACHE", "VELLA_NEMO_JOINTBATCH",
    "VELLA_FORCE_STOCK", "VELLA_PARAKEET_FORCE_STOCK", "VELLA_MLX_DEVICE", "VELLA_KERNEL_DEBUG_LOG",
    "VELLA_KERNEL_DIAGNOSTIC_COMPONENT", "VELLA_KERNEL_DIAGNOSTIC_CLIP", "VELLA_PARAKEET_PROFILE",
    "VELLA_DICTATION_KEEP_CACHE", "VELLA_NEMOTRON_TRANSCRIBE_MTP", "VELLA_NEMOTRON_TRANSCRIBE_DRAFTS",
    "VELLA_NEMOTRON_TRANSCRIBE_PROFILE", "VELLA_QWEN_PROFILE", "VELLA_WHISPER_PROFILE", "VELLA_STREAM_PROFILE",
    "VELLA_WHISPER_SEED", "VELLA_SUPPORT_DIR", "VELLA_WORKER_DATA_DIR", "VELLA_STUB_MODELS",
    "VELLA_TEST_LOAD_FAULT", "VELLA_TEST_OPTIMIZED_FAULT", "VELLA_TEST_STOCK_FAULT",
    "VELLA_TEST_STUB_FOOTPRINT_MB", "VELLA_TEST_SELFTEST_FAULT", "VELLA_TEST_DECODER_NONFINITE",
    "VELLA_TEST_ENCODER_NONFINITE", "VELLA_SELFTEST_RESULT")
REPORTED_PREFIXES = ("VELLA_NEMO_",)
ARCHITECTURES = ("parakeet", "qwen3_asr", "whisper", "nemotron_transcribe")


class RequestError(Exception):
    """A request the helper refuses (answered with code "invalid")."""


class LoadFault(Exception):
    """The injected load failure of VELLA_TEST_LOAD_FAULT."""


# ---- the wire format ----------------------------------------------------------------------

def _string(s: str) -> str:
    out = ['"']
    for ch in s:
        o = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif ch == "\n":
            out.append("\\n")
        elif ch == "\r":
            out.append("\\r")
        elif ch == "\t":
            out.append("\\t")
        elif ch == "\b":
            out.append("\\b")
        elif ch == "\f":
            out.append("\\f")
        elif o < 0x20:
            out.append("\\u%04x" % o)
        elif o < 0x80:
            out.append(ch)
        elif o < 0x10000:
            out.append("\\u%04x" % o)
        else:  # UTF-16 surrogate pair
            v = o - 0x10000
            out.append("\\u%04x\\u%04x" % (0xD800 + (v >> 10), 0xDC00 + (v & 0x3FF)))
    out.append('"')
    return "".join(out)


def _value(v: Any) -> str:
    if v is None:
        return "null"
    if v is True:
        return "true"
    if v is False:
        return "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        if not math.isfinite(v):
            raise ValueError("non-finite number")
        if v == int(v) and abs(v) < 2 ** 53:
            return str(int(v))
        return "%.17g" % v
    if isinstance(v, str):
        return _string(v)
    if isinstance(v, dict):
        return "{" + ",".join(_string(k) + ":" + _value(v[k]) for k in sorted(v)) + "}"
    if isinstance(v, (list, tuple)):
        return "[" + ",".join(_value(x) for x in v) + "]"
    raise TypeError(f"not a JSON value: {type(v).__name__}")


def wire_line(obj: Dict[str, Any]) -> bytes:
    """One protocol line: sorted keys, unescaped slashes, non-ASCII as \\uXXXX, a newline."""
    return (_value(obj) + "\n").encode("ascii")


def decode_request(data: bytes) -> Any:
    """JSON of a request line; NaN / Infinity / -Infinity outside strings read as 1 (a truthy
    number no field accepts), as the reference's decoder does (RequestValidation.swift:30-46)."""
    out = bytearray()
    i, quoted, escaped = 0, False, False
    tokens = (b"-Infinity", b"Infinity", b"NaN")
    while i < len(data):
        b = data[i]
        if quoted:
            out.append(b)
            if escaped:
                escaped = False
            elif b == 0x5C:
                escaped = True
            elif b == 0x22:
                quoted = False
            i += 1
        elif b == 0x22:
            quoted = True
            out.append(b)
            i += 1
        else:
            for t in tokens:
                if data.startswith(t, i):
                    out.append(0x31)
                    i += len(t)
                    break
            else:
                out.append(b)
                i += 1
    return json.loads(out.decode("utf-8"))


def request_identifier(v: Any) -> Optional[str]:
    """The id as a UUID in any of the forms Python's uuid.UUID accepts (the text is echoed)."""
    if not isinstance(v, str):
        return None
    s = v.replace("urn:", "").replace("uuid:", "").strip("{}").replace("-", "")
    if len(s.encode()) != 32 or any(c not in "0123456789abcdefABCDEF" for c in s):
        return None
    return v


def local_path(v: Any) -> str:
    """An absolute path that exists, resolved."""
    if not isinstance(v, str) or not v.startswith("/") or "\0" in v or not os.path.exists(v):
        raise RequestError()
    return os.path.realpath(v)


def read_wav(v: Any):
    """The samples of a 16 kHz mono 16-bit PCM WAV file (at most 2 MiB, 30 s), as float32 in
    [-1, 1); the reference's checks (RequestValidation.swift:63-101)."""
    import numpy as np
    path = local_path(v)
    if not os.path.isfile(path):
        raise RequestError()
    size = os.path.getsize(path)
    if not 44 <= size <= 2 * 1024 * 1024:
        raise RequestError()
    with open(path, "rb") as f:
        d = f.read(2 * 1024 * 1024 + 1)
    if not 44 <= len(d) <= 2 * 1024 * 1024:
        raise RequestError()
    u16 = lambda i: d[i] | d[i + 1] << 8  # noqa: E731
    u32 = lambda i: u16(i) | u16(i + 2) << 16  # noqa: E731
    if d[0:4] != b"RIFF" or d[8:12] != b"WAVE":
        raise RequestError()
    cursor, fmt, pcm = 12, False, None
    end = min(len(d), 8 + u32(4))
    while cursor + 8 <= end:
        name, length = d[cursor:cursor + 4], u32(cursor + 4)
        cursor += 8
        if name == b"fmt ":
            if length < 16 or cursor + length > end:
                raise RequestError()
            code = u16(cursor)
            if u16(cursor + 2) != 1 or u32(cursor + 4) != 16000 or u16(cursor + 14) != 16:
                raise RequestError()
            if code == 0xFFFE:  # WAVE_FORMAT_EXTENSIBLE with the PCM sub-format GUID
                if length < 40 or list(d[cursor + 24:cursor + 40]) != [1, 0, 0, 0, 0, 0, 16, 0, 128, 0, 0, 170, 0, 56,
                                                                       155, 113]:
                    raise RequestError()
            elif code != 1:
                raise RequestError()
            fmt = True
        elif name == b"data":
            frames = length // 2
            if not fmt or frames <= 0 or frames > 480000 or cursor + frames * 2 > end:
                raise RequestError()
            pcm = np.frombuffer(d[cursor:cursor + frames * 2], dtype="<i2").astype(np.float32) / 32768.0
            break
        cursor += length + length % 2
    if pcm is None:
        raise RequestError()
    return pcm


def _truthy(v: Any) -> bool:
    if v is None:
        return False
    if isinstance(v, (bool, int, float)):
        return v != 0
    if isinstance(v, (str, list, dict)):
        return len(v) > 0
    return True


def _json_file(path: str) -> Dict[str, Any]:
    try:
        with open(path, "rb") as f:
            obj = decode_request(f.read())
    except (OSError, ValueError):
        raise RequestError()
    if not isinstance(obj, dict):
        raise RequestError()
    return obj


def admit(path: str) -> str:
    """The architecture of a checkpoint directory the helper may load, else RequestError: a
    known model_type (NeMo transducers and the Nemotron SpeechLM release by their own fields),
    4- or 8-bit quantization when quantized, no remote code, at least one .safetensors file
    (Validation.swift:20-59)."""
    config = _json_file(os.path.join(path, "config.json"))
    mt = config.get("model_type")
    if mt is not None and not isinstance(mt, str):
        raise RequestError()
    arch = mt
    if arch is None and config.get("target") == "nemo.collections.asr.models.rnnt_bpe_models.EncDecRNNTBPEModel":
        arch = "parakeet"
    if arch == "nemo_speechlm" and "Nemotron3_5TranscribeForConditionalGeneration" in (config.get("architectures") or []):
        arch = "nemotron_transcribe"
    if arch == "nemotron_transcribe":
        llm = config.get("llm_config")
        if not isinstance(llm, dict) or llm.get("model_type") != "nemotron_h" or \
                config.get("prompt_format", "nemotron3p5") != "nemotron3p5":
            raise RequestError()
    stub = os.environ.get("VELLA_STUB_MODELS") == "1" and arch == "stub"
    if arch is None or not (stub or arch in ARCHITECTURES):
        raise RequestError()
    quant = config["quantization"] if _truthy(config.get("quantization")) else (
        config["quantization_config"] if _truthy(config.get("quantization_config")) else {})
    if not isinstance(quant, dict):
        raise RequestError()
    bits = quant.get("bits")
    if bits is not None and (isinstance(bits, bool) or not isinstance(bits, (int, float)) or bits not in (4, 8)):
        raise RequestError()
    for name in ("config.json", "tokenizer_config.json"):
        p = os.path.join(path, name)
        if os.path.exists(p) and _truthy(_json_file(p).get("auto_map")):
            raise RequestError()
    for root, _, files in os.walk(path):
        if any(f.endswith(".py") for f in files):
            raise RequestError()
    if not any(f.endswith(".safetensors") for f in os.listdir(path)):
        raise RequestError()
    return arch


class RequestOptions:
    """A transcription request's `options`: language (1-16 characters), prompt (<= 16 KiB),
    vocabulary (bool), words (<= 64 letter-only words) (DictationService.swift:15-47)."""

    def __init__(self, value: Any = None):
        self.language: Optional[str] = None
        self.prompt: Optional[str] = None
        self.vocabulary = True
        self.words: list = []
        if value is None:
            return
        if not isinstance(value, dict) or not set(value) <= {"language", "prompt", "vocabulary", "words"}:
            raise RequestError()
        if "language" in value:
            code = value["language"]
            if not isinstance(code, str) or not 1 <= len(code) <= 16:
                raise RequestError()
            self.language = code
        if "prompt" in value:
            text = value["prompt"]
            if not isinstance(text, str) or len(text.encode()) > 16 * 1024:
                raise RequestError()
            self.prompt = text if text.strip() else None
        if "vocabulary" in value:
            if not isinstance(value["vocabulary"], bool):
                raise RequestError()
            self.vocabulary = value["vocabulary"]
        if "words" in value:
            words = value["words"]
            if not isinstance(words, list) or len(words) > 64 or not all(
                    isinstance(w, str) and 0 < len(w) <= 64 and w.isalpha() for w in words):
                raise RequestError()
            self.words = words

    def unsupported(self, arch: Optional[str]) -> Optional[str]:
        """The setting an architecture cannot apply (the request is then refused)."""
        language, prompt = {"whisper": (True, False), "qwen3_asr": (True, False),
                            "nemotron_transcribe": (True, True), "stub": (True, True)}.get(arch, (False, False))
        if self.language is not None and not language:
            return "language"
        if self.prompt is not None and not prompt:
            return "prompt"
        if self.words and arch not in ("parakeet", "nemotron_transcribe", "stub"):
            return "words"
        if self.words and self.prompt is not None:
            return "words with prompt"
        return None


# ---- runtimes ------------------------------------------------------------------------------

class StubRuntime:
    """The test model (VELLA_STUB_MODELS=1): no weights; text `stub:<folder> <seconds>s`."""
    components = {"stub": True}

    def __init__(self, path: str):
        self.name = os.path.basename(path)

    def transcribe(self, samples, options: RequestOptions) -> str:
        return "stub:%s %.1fs" % (self.name, len(samples) / 16000.0)

    def close(self):
        pass


class WhisperRuntime:
    """A Whisper checkpoint on the B200 path: log-mel, encoder and greedy decoder with the
    reference's token rules and temperature fallback (vella_b200.whisper.WhisperSTT); the text
    through the checkpoint's own tokenizer files."""
    components = {"whisper_decoder": True, "whisper_encoder": True}

    def __init__(self, path: str):
        import torch  # noqa: F401  (device memory figures in the status and metrics)
        from vella_b200 import checkpoint as C
        from vella_b200 import whisper as VW
        try:
            from transformers import AutoTokenizer
            tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        except Exception as e:  # no usable tokenizer files: the text cannot be produced
            raise LoadFault(f"tokenizer: {e}")
        tokens = C.whisper_tokens(path)
        self.model = C.load_whisper(path)
        try:
            self.model.set_rules(**tokens.rules())
        except Exception:
            self.model.close()
            raise
        self.stt = VW.WhisperSTT(self.model, tokens, lambda ids: tok.decode(ids, skip_special_tokens=True))

    def transcribe(self, samples, options: RequestOptions) -> str:
        language = options.language.lower().replace("_", "-").split("-")[0] if options.language else None
        return self.stt.generate(samples, language=language).text

    def close(self):
        self.model.close()


RUNTIMES = {"stub": StubRuntime, "whisper": WhisperRuntime}


def _process_memory() -> Dict[str, int]:
    """Resident and peak resident bytes of this process (the footprint fields report the
    same resident size: Linux has no separate physical-footprint counter)."""
    peak = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * 1024
    rss = peak
    try:
        with open("/proc/self/statm") as f:
            rss = int(f.read().split()[1]) * os.sysconf("SC_PAGE_SIZE")
    except (OSError, ValueError, IndexError):
        pass
    return {"processPeakRSSBytes": peak, "processRSSBytes": rss, "processFootprintBytes": rss,
            "processPeakFootprintBytes": peak}


_PEAK = [0]


def _device_memory(reset: bool = False) -> Dict[str, int]:
    """Device bytes in use (the library allocates through the CUDA runtime, outside torch's
    allocator, so this is the device's used memory: total minus free), the part torch's
    allocator holds cached, and the running maximum of the samples since the last reset.
    Zero until a GPU runtime has imported torch (the stub model never does)."""
    if reset:
        _PEAK[0] = 0
    t = sys.modules.get("torch")
    if t is None or not t.cuda.is_available():
        return {"active": 0, "cache": 0, "peak": 0}
    free, total = t.cuda.mem_get_info()
    cache = t.cuda.memory_reserved() - t.cuda.memory_allocated() if t.cuda.is_initialized() else 0
    active = max(0, total - free - cache)
    _PEAK[0] = max(_PEAK[0], active)
    return {"active": active, "cache": cache, "peak": _PEAK[0]}


def _gpu() -> Dict[str, Optional[str]]:
    t = sys.modules.get("torch")
    if t is not None and t.cuda.is_available():
        p = t.cuda.get_device_properties(0)
        return {"chip": p.name, "family": "sm_%d%d" % (p.major, p.minor)}
    return {"chip": "unavailable", "family": "unsupported"}


def reported_environment(env=None) -> Dict[str, str]:
    env = os.environ if env is None else env
    return {k: v for k, v in env.items()
            if v and (k in REPORTED_SWITCHES or any(k.startswith(p) for p in REPORTED_PREFIXES))}


# ---- the helper ----------------------------------------------------------------------------

class Worker:
    """One model at a time; every state change pushes one status line before its reply
    (DictationService.swift:97-99, 177-256, 446-547)."""

    def __init__(self, push):
        self.push = push
        self.runtime = None
        self.path: Optional[str] = None
        self.arch: Optional[str] = None
        self.load_s: Optional[float] = None
        self.stock_reason: Optional[str] = "No model loaded."
        self.optimizations: Dict[str, bool] = {}
        self.applied: Dict[str, Any] = {}

    # -- state ---------------------------------------------------------------------------------
    def push_status(self, event: str):
        self.push({"status": self.status(event)})

    def status(self, event: str) -> Dict[str, Any]:
        pm, dm = _process_memory(), _device_memory()
        footprint = pm["processFootprintBytes"] / 1e6
        stub_mb = os.environ.get("VELLA_TEST_STUB_FOOTPRINT_MB")
        if isinstance(self.runtime, StubRuntime) and stub_mb:
            try:
                footprint = float(stub_mb)
            except ValueError:
                pass
        loaded = self.runtime is not None
        out = {"worker": "dictation", "pid": os.getpid(), "version": GATE_VERSION, "event": event, "model": self.path,
               "architecture": self.arch, "engine": ("optimized" if self.stock_reason is None else "stock") if loaded
               else None, "engine_reason": self.stock_reason if loaded else None,
               "optimizations": dict(self.optimizations), "load_s": self.load_s,
               "memory": {"footprint_mb": footprint, "mlx_active_mb": dm["active"] / 1e6,
                          "mlx_cache_mb": dm["cache"] / 1e6},
               "gpu": _gpu(), "recipe": os.environ.get("VELLA_RECIPE") or "optimized_fast"}
        hooks = reported_environment()
        if hooks:
            out["test_hooks"] = hooks
        return out

    def cleanup(self, keep_cache: bool = False):
        t = sys.modules.get("torch")
        if not keep_cache and t is not None and t.cuda.is_available() and t.cuda.is_initialized():
            t.cuda.synchronize()
            t.cuda.empty_cache()

    def release(self):
        if self.runtime is not None:
            self.runtime.close()
        self.runtime = None
        self.path = self.arch = self.load_s = None
        self.stock_reason = "No model loaded."
        self.optimizations = {}
        self.cleanup()

    def _load(self, path: str, arch: str):
        fault = os.environ.get("VELLA_TEST_LOAD_FAULT")
        if fault and fault in path:
            raise LoadFault("injected")
        cls = RUNTIMES.get(arch)
        if cls is None:  # an architecture without a runtime here
            raise RequestError()
        runtime = cls(path)
        self.arch = arch
        self.stock_reason = None
        self.optimizations = dict(cls.components)
        return runtime

    def load_if_needed(self, path: str, arch: str, metrics: Dict[str, Any]):
        if path == self.path:
            return
        self.release()
        _device_memory(reset=True)
        t0 = time.monotonic()
        try:
            self.runtime = self._load(path, arch)
            self.path = path
        except Exception:
            self.release()
            self.push_status("load-failed")
            raise
        self.load_s = time.monotonic() - t0
        metrics["loadSeconds"] = self.load_s
        metrics["loadPeakMLXBytes"] = _device_memory()["peak"]
        self.push_status("load")

    @staticmethod
    def failure(e: BaseException) -> Dict[str, str]:
        if isinstance(e, RequestError):
            return dict(INVALID)
        text = str(e).lower()
        if any(s in text for s in ("out of memory", "memory allocation", "insufficient memory")):
            return {"code": "memory", "message": "Insufficient memory for transcription."}
        return {"code": "inference", "message": "Local transcription failed."}

    # -- requests ------------------------------------------------------------------------------
    def handle(self, request: Any) -> Dict[str, Any]:
        ident = request_identifier(request.get("id")) if isinstance(request, dict) else None
        if ident is None:
            return {"id": None, "error": dict(INVALID)}
        if "op" not in request:
            return self.transcribe(request, ident)
        keys, op = set(request), request["op"]
        if op == "load" and keys == {"id", "op", "model"}:
            try:
                path = local_path(request["model"])
                arch = (self.arch or admit(path)) if path == self.path else admit(path)
            except RequestError:
                return {"id": ident, "error": dict(INVALID)}
            metrics: Dict[str, Any] = {}
            try:
                if path == self.path:
                    self.push_status("load")
                else:
                    self.load_if_needed(path, arch, metrics)
                self.cleanup()
                return {"id": ident, "loaded": True, "metrics": metrics}
            except Exception as e:
                f = self.failure(e)
                if f["code"] == "inference":
                    f = {"code": "load", "message": "The model failed to load."}
                return {"id": ident, "error": f}
        if op == "unload" and keys == {"id", "op"}:
            self.release()
            self.push_status("unload")
            return {"id": ident, "unloaded": True}
        if op == "status" and keys == {"id", "op"}:
            self.push_status("status")
            return {"id": ident, "ok": True}
        if op == "trim" and keys == {"id", "op"}:
            self.cleanup()
            self.push_status("trim")
            return {"id": ident, "ok": True}
        return {"id": ident, "error": dict(INVALID)}

    def transcribe(self, request: Dict[str, Any], ident: str) -> Dict[str, Any]:
        start = time.monotonic()
        response: Dict[str, Any] = {"id": ident}
        metrics: Dict[str, Any] = {}
        try:
            try:
                keys = set(request)
                if keys != {"id", "model", "audio"} and keys != {"id", "model", "audio", "options"}:
                    raise RequestError()
                path = local_path(request["model"])
                samples = read_wav(request["audio"])
                options = RequestOptions(request.get("options"))
                arch = admit(path) if path != self.path else None
                reason = options.unsupported(arch or self.arch)
                if reason is not None:
                    response["error"] = {"code": "unsupported", "message": f"This model cannot apply {reason}."}
                    return response
            except RequestError:
                raise
            except Exception:
                raise RequestError()
            cold = path != self.path
            metrics = {"audioSeconds": len(samples) / 16000.0, "modelLoaded": cold, "loadSeconds": 0.0,
                       "mlxPeakPhase": "load_and_first_request" if cold else "warm_request",
                       "allocatorCacheLimitBytes": CACHE_BYTES}
            if cold:
                self.load_if_needed(path, arch, metrics)
            if self.runtime is None:
                raise RequestError()
            t0 = time.monotonic()
            if not cold:
                _device_memory(reset=True)
            response["text"] = self.runtime.transcribe(samples, options)
            self.applied = {"language": options.language, "vocabulary": options.vocabulary}
            response["applied"] = dict(self.applied)
            metrics["inferenceSeconds"] = time.monotonic() - t0
            metrics["peakMLXBytes"] = _device_memory()["peak"]
        except Exception as e:
            f = self.failure(e)
            response["error"] = f
            if f["code"] != "invalid" and self.runtime is not None:
                self.release()
                self.push_status("unload")
        t0 = time.monotonic()
        try:
            self.cleanup(keep_cache="text" in response and os.environ.get("VELLA_DICTATION_KEEP_CACHE") != "0")
        except Exception:
            self.runtime = None
            self.path = None
            return {"id": ident, "error": {"code": "memory", "message": "Insufficient memory for transcription."}}
        if "text" in response:
            dm = _device_memory()
            metrics["cleanupSeconds"] = time.monotonic() - t0
            metrics["requestSeconds"] = time.monotonic() - start
            metrics["activeMLXBytes"] = dm["active"]
            metrics["cacheMLXBytes"] = dm["cache"]
            metrics.update(_process_memory())
            response["metrics"] = metrics
        return response


def read_line(stream, on_overlong=None) -> Optional[bytes]:
    """One request line with its newline, at most MAX_LINE + 1 bytes kept; an overlong line is
    drained to its newline (the request is then answered "invalid").  None at end of input."""
    data = stream.readline(MAX_LINE + 1)
    if not data:
        return None
    if len(data) > MAX_LINE and not data.endswith(b"\n"):
        if on_overlong:
            on_overlong()
        while True:
            rest = stream.readline(1 << 16)
            if not rest or rest.endswith(b"\n"):
                break
    return data


def main(stdin=None, out_fd: Optional[int] = None) -> int:
    """The stdio loop: replies (and pushed status lines) on the original stdout; stdout and
    stderr themselves point at /dev/null so that no library output can corrupt the protocol."""
    if out_fd is None:
        out_fd = os.dup(1)
        sink = os.open(os.devnull, os.O_WRONLY)
        os.dup2(sink, 1)
        os.dup2(sink, 2)
        os.close(sink)
    stdin = stdin if stdin is not None else sys.stdin.buffer

    def write(obj):
        data = wire_line(obj)
        while data:
            n = os.write(out_fd, data)
            data = data[n:]

    worker = Worker(write)
    while True:
        line = read_line(stdin, on_overlong=lambda: signal.alarm(120))
        if line is None:
            break
        ok = len(line) <= MAX_LINE
        if ok:
            signal.alarm(120)  # a request that hangs ends the helper
        request = None
        if ok:
            try:
                request = decode_request(line)
            except (ValueError, UnicodeDecodeError):
                request = None
        write(worker.handle(request))
        signal.alarm(0)
    worker.release()
    os.close(out_fd)
    return 0


if __name__ == "__main__":
    sys.exit(main())
