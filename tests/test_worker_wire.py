"""The dictation helper's stdio bytes against the reference helper's wire fixtures
(tests/golden/wire, copied from Tests/Fixtures/wire by tests/golden/make_wire.py), driven the
way the reference's WireSnapshotTests.swift:82-140 drives its helper: a stub model folder, a
0.1 s 16 kHz WAV, the same request lines, stdin closed after them.  Volatile values (pid,
timings, memory, GPU name, the scratch path) are normalised as that test does; everything
else is compared byte for byte.  CPU only: the stub model runs no GPU work."""
import json
import os
import re
import struct
import subprocess
import sys
from pathlib import Path

import pytest

from vella_b200 import worker as W

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden" / "wire"
ID = "6f1c2a4e-8d3b-4c1a-9e7f-2b5d8c0a1e34"
VOLATILE = ("pid", "load_s", "footprint_mb", "mlx_active_mb", "mlx_cache_mb", "loadSeconds", "loadPeakMLXBytes",
            "cleanupSeconds", "inferenceSeconds", "requestSeconds", "processFootprintBytes",
            "processPeakFootprintBytes", "processPeakRSSBytes", "processRSSBytes", "peakMLXBytes", "activeMLXBytes",
            "cacheMLXBytes")


def scratch(tmp_path):
    d = Path(os.path.realpath(tmp_path))
    model, data = d / "stub-model", d / "data"
    model.mkdir()
    data.mkdir()
    (model / "config.json").write_text('{"model_type": "stub"}\n')
    (model / "model.safetensors").write_text("stub weights\n")
    pcm = b"".join(struct.pack("<H", 1000 if i % 2 == 0 else 0xFC18) for i in range(1600))
    wav = (b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE" + b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, 16000,
           32000, 2, 16) + b"data" + struct.pack("<I", len(pcm)) + pcm)
    (d / "clip.wav").write_bytes(wav)
    return d, model, d / "clip.wav"


def exchange(lines, env):
    full = {"HOME": os.environ.get("HOME", "/root"), "PATH": "/usr/bin:/bin", "PYTHONPATH": str(ROOT), **env}
    p = subprocess.run([sys.executable, "-m", "vella_b200.worker"], input="".join(l + "\n" for l in lines).encode(),
                       stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, env=full, cwd=str(ROOT), timeout=120)
    assert p.returncode == 0
    return p.stdout.decode()


def normalized(text, d):
    text = text.replace(str(d), "$SCRATCH")
    for key in VOLATILE:
        text = re.sub('"%s":-?[0-9][0-9.eE+-]*' % key, '"%s":0' % key, text)
    return re.sub(r'"gpu":\{"chip":"[^"]*","family":"[^"]*"\}', '"gpu":{"chip":"CHIP","family":"FAMILY"}', text)


def test_dictation_wire_matches_fixture(tmp_path):
    d, model, audio = scratch(tmp_path)
    lines = [
        json.dumps({"id": ID, "op": "status"}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "load", "model": str(model)}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "load", "model": str(model)}, separators=(",", ":")),
        json.dumps({"id": ID, "model": str(model), "audio": str(audio)}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "trim"}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "unload"}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "bogus"}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "load", "model": str(d) + "/missing"}, separators=(",", ":")),
        json.dumps({"id": ID, "op": "status", "extra": 1}, separators=(",", ":")),
        json.dumps({"id": "not-a-uuid", "op": "status"}, separators=(",", ":")),
        "not json",
    ]
    out = exchange(lines, {"VELLA_STUB_MODELS": "1", "VELLA_WORKER_DATA_DIR": str(d / "data")})
    assert normalized(out, d) == (GOLDEN / "dictation.txt").read_text()


def test_dictation_load_failure_matches_fixture(tmp_path):
    d, model, audio = scratch(tmp_path)
    lines = [json.dumps({"id": ID, "op": "load", "model": str(model)}, separators=(",", ":")),
             json.dumps({"id": ID, "model": str(model), "audio": str(audio)}, separators=(",", ":"))]
    out = exchange(lines, {"VELLA_STUB_MODELS": "1", "VELLA_WORKER_DATA_DIR": str(d / "data"),
                           "VELLA_TEST_LOAD_FAULT": "stub-model"})
    assert normalized(out, d) == (GOLDEN / "dictation-load-failed.txt").read_text()


@pytest.mark.parametrize("obj,text", [
    ({"b": 1, "a": "x/y"}, '{"a":"x/y","b":1}\n'),
    ({"t": "café \U0001F600"}, '{"t":"caf\\u00e9 \\ud83d\\ude00"}\n'),
    ({"v": 0.1}, '{"v":0.10000000000000001}\n'),
    ({"v": 2.0, "n": None, "f": False}, '{"f":false,"n":null,"v":2}\n'),
    ({"s": "a\"b\\c\n\x01"}, '{"s":"a\\"b\\\\c\\n\\u0001"}\n'),
])
def test_wire_line_format(obj, text):
    assert W.wire_line(obj) == text.encode()


def test_request_validation():
    assert W.request_identifier(ID) == ID
    assert W.request_identifier("not-a-uuid") is None
    assert W.request_identifier(ID.upper()) is not None
    with pytest.raises(ValueError):
        W.decode_request(b"not json")
    assert W.decode_request(b'{"id":"x","n":NaN}') == {"id": "x", "n": 1}
    assert W.decode_request(b'{"id":"NaN"}') == {"id": "NaN"}


def test_overlong_line_is_drained(tmp_path):
    d, model, _ = scratch(tmp_path)
    lines = ['{"id":"%s","op":"status","pad":"%s"}' % (ID, "x" * (W.MAX_LINE + 10)),
             json.dumps({"id": ID, "op": "unload"}, separators=(",", ":"))]
    out = exchange(lines, {"VELLA_STUB_MODELS": "1"}).splitlines()
    assert json.loads(out[0]) == {"error": W.INVALID, "id": None}
    assert json.loads(out[1])["status"]["event"] == "unload"
    assert json.loads(out[2]) == {"id": ID, "unloaded": True}
