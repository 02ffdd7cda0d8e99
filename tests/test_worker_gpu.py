"""The dictation helper's Whisper runtime on the GPU: a written int4 Whisper-tiny checkpoint
(random weights) with offline tokenizer files, transcribed through `python -m
vella_b200.worker` (load, then a transcription request), gives the text of the same checkpoint
run directly through vella_b200.whisper.WhisperSTT with the same tokenizer and seed, and the
reply carries the reference's metric keys."""
import json
import os
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from tests.test_checkpoint import _hf_config, _write_dir, export_hf
from vella_b200 import worker as W

ROOT = Path(__file__).resolve().parents[1]
ID = "6f1c2a4e-8d3b-4c1a-9e7f-2b5d8c0a1e34"


def _checkpoint(tmp_path):
    from vella_b200 import whisper as VW
    cfg = VW.TINY
    src = VW.Whisper(cfg)
    src.init_random(21, 0.05)
    d = tmp_path / "whisper-tiny"
    _write_dir(d, export_hf(src, cfg), {**_hf_config(cfg, quant=cfg.bits), "model_type": "whisper"})
    src.close()
    (d / "vocab.json").write_text(json.dumps({f"t{i}": i for i in range(cfg.vocab)}))
    (d / "merges.txt").write_text("#version: 0.2\n")
    (d / "tokenizer_config.json").write_text(json.dumps({"tokenizer_class": "GPT2Tokenizer"}))
    return Path(os.path.realpath(d))


def _wav(path, seconds=1.5):
    pcm = (np.random.default_rng(4).standard_normal(int(16000 * seconds)) * 3000).astype("<i2").tobytes()
    path.write_bytes(b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE" + b"fmt " +
                     struct.pack("<IHHIIHH", 16, 1, 1, 16000, 32000, 2, 16) + b"data" + struct.pack("<I", len(pcm)) +
                     pcm)
    return path


@pytest.mark.gpu
def test_whisper_transcription_through_the_helper(tmp_path):
    model = _checkpoint(tmp_path)
    audio = _wav(tmp_path / "clip.wav")
    lines = [json.dumps({"id": ID, "op": "load", "model": str(model)}),
             json.dumps({"id": ID, "model": str(model), "audio": str(audio), "options": {"language": "en"}}),
             json.dumps({"id": ID, "op": "unload"})]
    env = {**os.environ, "PYTHONPATH": str(ROOT)}
    p = subprocess.run([sys.executable, "-m", "vella_b200.worker"], input="".join(l + "\n" for l in lines).encode(),
                       stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, env=env, cwd=str(ROOT), timeout=600)
    assert p.returncode == 0
    out = [json.loads(l) for l in p.stdout.decode().splitlines()]
    assert out[0]["status"]["event"] == "load" and out[0]["status"]["architecture"] == "whisper"
    assert out[0]["status"]["engine"] == "optimized" and out[0]["status"]["gpu"]["family"] == "sm_100"
    assert out[1]["loaded"] is True and out[1]["metrics"]["loadSeconds"] > 0
    reply = out[2]
    assert "error" not in reply, reply
    assert reply["applied"] == {"language": "en", "vocabulary": True}
    m = reply["metrics"]
    assert m["modelLoaded"] is False and m["mlxPeakPhase"] == "warm_request" and m["audioSeconds"] == 1.5
    assert m["peakMLXBytes"] > 0 and m["inferenceSeconds"] > 0
    assert out[3]["status"]["event"] == "unload" and out[4] == {"id": ID, "unloaded": True}

    # the same checkpoint, tokenizer and seed directly
    rt = W.WhisperRuntime(str(model))
    try:
        samples = W.read_wav(str(audio))
        want = rt.transcribe(samples, W.RequestOptions({"language": "en"}))
    finally:
        rt.close()
    assert reply["text"] == want


@pytest.mark.gpu
def test_cold_transcription_loads_first(tmp_path):
    model = _checkpoint(tmp_path)
    audio = _wav(tmp_path / "clip.wav", 0.5)
    sent = []
    w = W.Worker(sent.append)
    try:
        reply = w.handle({"id": ID, "model": str(model), "audio": str(audio)})
        assert "text" in reply, reply
        assert reply["metrics"]["modelLoaded"] is True
        assert reply["metrics"]["mlxPeakPhase"] == "load_and_first_request"
        assert [s["status"]["event"] for s in sent] == ["load"]
        # a prompt is not applicable to Whisper: refused, the model stays loaded
        r2 = w.handle({"id": ID, "model": str(model), "audio": str(audio), "options": {"prompt": "hello"}})
        assert r2["error"]["code"] == "unsupported" and w.runtime is not None
    finally:
        w.release()
