"""Checkpoints: the safetensors reader, the Whisper key mapping and shape checks, config.json
and the tokenizer's special ids (CPU), and loading a written checkpoint into a Whisper handle
(B200: every tensor bit-equal to the handle it was written from, in the Hugging Face and
mlx-whisper layouts, and the derived int4 precision bit-equal to the oracle's quantizer).

The files are written here by ``write_safetensors`` (8-byte little-endian header length,
JSON header of dtype / shape / data_offsets per tensor, then the data)."""
import json
import struct

import numpy as np
import pytest

from oracle import affine as A

_ST = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32",
       np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.int64): "I64", np.dtype(np.float64): "F64"}


def write_safetensors(path, tensors: dict, metadata=None, dtypes=None):
    """tensors: name -> numpy array; dtypes: name -> safetensors dtype overriding the array's
    (e.g. "BF16" for uint16 words)."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, a in tensors.items():
        a = np.asarray(a, order="C")  # keeps 0-d arrays 0-d
        b = a.tobytes()
        dt = (dtypes or {}).get(name) or _ST[a.dtype]
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _st(paths):
    from vella_b200 import checkpoint as C
    return C.SafeTensors([str(p) for p in paths])


def test_reader_round_trips_dtypes_shapes_and_metadata(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a.f16": rng.standard_normal((3, 5)).astype(np.float16),
         "b.f32": rng.standard_normal(7).astype(np.float32),
         "c.u32": rng.integers(0, 2**32, (2, 2, 2), dtype=np.uint64).astype(np.uint32),
         "d.bf16": rng.integers(0, 2**16, (4,), dtype=np.uint64).astype(np.uint16),
         "e.scalar": np.array(3.5, np.float32), "f.empty": np.zeros((0, 4), np.float16),
         "g.unié": np.arange(3, dtype=np.int64)}
    p = tmp_path / "m.safetensors"
    write_safetensors(p, t, metadata={"format": "pt"}, dtypes={"d.bf16": "BF16"})
    with _st([p]) as st:
        assert sorted(st.keys()) == sorted(t)
        assert st.info("d.bf16") == ("BF16", (4,))
        assert st.info("e.scalar") == ("F32", ())
        for k, a in t.items():
            got = st.array(k)
            assert got.shape == a.shape and np.array_equal(got.view(a.dtype), a), k
        assert st.index("missing") == -1
        with pytest.raises(KeyError):
            st.info("missing")


def test_later_shards_replace_earlier_keys(tmp_path):
    a, b = tmp_path / "model-00001.safetensors", tmp_path / "model-00002.safetensors"
    write_safetensors(a, {"x": np.ones(2, np.float32), "y": np.zeros(3, np.float16)})
    write_safetensors(b, {"x": np.full(4, 2.0, np.float32)})
    with _st([a, b]) as st:
        assert len(st) == 2
        assert np.array_equal(st.array("x"), np.full(4, 2.0, np.float32))
        assert st.array("y").shape == (3,)


@pytest.mark.parametrize("case", ["truncated", "bad_json", "offsets", "dtype", "short_data", "missing", "overflow"])
def test_malformed_files_are_rejected(tmp_path, case):
    from vella_b200 import _lib
    p = tmp_path / "bad.safetensors"
    if case == "missing":
        p = tmp_path / "absent.safetensors"
    elif case == "truncated":
        p.write_bytes(b"\x10\x00\x00")
    elif case == "bad_json":
        h = b'{"x": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]'
        p.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 4)
    else:
        shape, offs, dt = [2], [0, 8], "F32"
        if case == "offsets":
            offs = [0, 12]
        if case == "dtype":
            dt = "Q7"
        if case == "overflow":  # 2**62 elements * 4 bytes wraps to 0 bytes in 64 bits
            shape, offs = [2**62], [0, 0]
        body = 8 if case != "short_data" else 4
        h = json.dumps({"x": {"dtype": dt, "shape": shape, "data_offsets": offs}}).encode()
        p.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * body)
    with pytest.raises(_lib.VellaError) as e:
        _st([p])
    assert e.value.code == _lib.E_INVALID


# ---- a small Whisper checkpoint (shapes only; the values are random) -------------------

def small_cfg(bits=4):
    from vella_b200.whisper import WhisperConfig
    return WhisperConfig(n_mels=8, d_model=64, heads=1, enc_layers=1, dec_layers=1, ffn=128, vocab=96, n_audio=16,
                         max_target=8, bits=bits)


def hf_tensors(cfg, quant_bits=0, rng=None):
    """Hugging Face key layout with random float values (fp16); decoder Linears and the token
    embedding MLX-affine packed when quant_bits is set."""
    rng = rng or np.random.default_rng(1)
    d, F, V = cfg.d_model, cfg.ffn, cfg.vocab
    f = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float16)  # noqa: E731
    t = {"model.encoder.conv1.weight": f(d, cfg.n_mels, 3), "model.encoder.conv1.bias": f(d),
         "model.encoder.conv2.weight": f(d, d, 3), "model.encoder.conv2.bias": f(d),
         "model.encoder.layer_norm.weight": f(d), "model.encoder.layer_norm.bias": f(d),
         "model.decoder.layer_norm.weight": f(d), "model.decoder.layer_norm.bias": f(d),
         "model.decoder.embed_positions.weight": f(cfg.max_target, d),
         "proj_out.weight": f(V, d)}

    def lin(prefix, n, k, bias=True, quant=False):
        w = f(n, k)
        if quant:
            q, s, b = A.quantize(w.astype(np.float32), quant_bits, "f16")
            t[prefix + ".weight"], t[prefix + ".scales"], t[prefix + ".biases"] = q, s, b
        else:
            t[prefix + ".weight"] = w
        if bias:
            t[prefix + ".bias"] = f(n)

    lin("model.decoder.embed_tokens", V, d, bias=False, quant=bool(quant_bits))
    for l in range(cfg.enc_layers):
        p = f"model.encoder.layers.{l}."
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            t[p + ln + ".weight"], t[p + ln + ".bias"] = f(d), f(d)
        for pr in ("q", "k", "v", "out"):
            lin(p + f"self_attn.{pr}_proj", d, d, bias=pr != "k")
        lin(p + "fc1", F, d)
        lin(p + "fc2", d, F)
    for l in range(cfg.dec_layers):
        p = f"model.decoder.layers.{l}."
        for ln in ("self_attn_layer_norm", "encoder_attn_layer_norm", "final_layer_norm"):
            t[p + ln + ".weight"], t[p + ln + ".bias"] = f(d), f(d)
        for att in ("self_attn", "encoder_attn"):
            for pr in ("q", "k", "v", "out"):
                lin(p + f"{att}.{pr}_proj", d, d, bias=pr != "k", quant=bool(quant_bits))
        lin(p + "fc1", F, d, quant=bool(quant_bits))
        lin(p + "fc2", d, F, quant=bool(quant_bits))
    return t


_MLX_ATTN = {"q_proj": "query", "k_proj": "key", "v_proj": "value", "out_proj": "out"}
_MLX_LN = {"self_attn_layer_norm": "attn_ln", "encoder_attn_layer_norm": "cross_attn_ln", "final_layer_norm": "mlp_ln"}


def to_mlx_names(t: dict) -> dict:
    """The same tensors under OpenAI/mlx-whisper names, conv weights as [out, 3, in]."""
    out = {}
    for k, v in t.items():
        if k == "proj_out.weight":
            continue
        if k.endswith("conv1.weight") or k.endswith("conv2.weight"):
            v = np.ascontiguousarray(v.transpose(0, 2, 1))
        n = k[len("model."):]
        n = n.replace("encoder.embed_positions.weight", "encoder.positional_embedding")
        n = n.replace("decoder.embed_positions.weight", "decoder.positional_embedding")
        n = n.replace("decoder.embed_tokens.", "decoder.token_embedding.")
        n = n.replace("encoder.layer_norm.", "encoder.ln_post.").replace("decoder.layer_norm.", "decoder.ln.")
        if ".layers." in n:
            stem, rest = n.split(".layers.", 1)
            idx, suf = rest.split(".", 1)
            for a, b in _MLX_LN.items():
                suf = suf.replace(a + ".", b + ".")
            suf = suf.replace("self_attn.", "attn.").replace("encoder_attn.", "cross_attn.")
            for a, b in _MLX_ATTN.items():
                suf = suf.replace(a + ".", b + ".")
            suf = suf.replace("fc1.", "mlp1.").replace("fc2.", "mlp2.")
            n = f"{stem}.blocks.{idx}.{suf}"
        out[n] = v
    out["alignment_heads"] = np.zeros((2, 2), np.uint8)
    return out


def _check(tmp_path, tensors, cfg, name="model.safetensors"):
    from vella_b200 import checkpoint as C
    p = tmp_path / name
    write_safetensors(p, tensors)
    with _st([p]) as st:
        C.check_whisper_checkpoint(st, cfg)


@pytest.mark.parametrize("quant", [0, 4])
def test_whisper_checkpoint_layouts_pass_the_check(tmp_path, quant):
    cfg = small_cfg(bits=4)
    t = hf_tensors(cfg, quant_bits=quant)
    _check(tmp_path, t, cfg, "hf.safetensors")
    _check(tmp_path, to_mlx_names(t), cfg, "mlx.safetensors")
    # a re-export without the top-level "model." prefix
    _check(tmp_path, {k[6:] if k.startswith("model.") else k: v for k, v in t.items()}, cfg, "bare.safetensors")


def test_whisper_checkpoint_problems_are_named(tmp_path):
    from vella_b200 import _lib
    cfg = small_cfg(bits=4)
    t = hf_tensors(cfg)
    gone = dict(t)
    del gone["model.decoder.layers.0.encoder_attn.v_proj.bias"]
    with pytest.raises(_lib.VellaError, match="encoder_attn.v_proj.bias"):
        _check(tmp_path, gone, cfg)
    bad = dict(t)
    bad["model.encoder.layers.0.fc1.weight"] = np.zeros((cfg.ffn, cfg.d_model + 64), np.float16)
    with pytest.raises(_lib.VellaError, match="fc1.weight"):
        _check(tmp_path, bad, cfg)
    short = dict(t)
    short["model.decoder.embed_positions.weight"] = np.zeros((cfg.max_target - 1, cfg.d_model), np.float16)
    with pytest.raises(_lib.VellaError, match="embed_positions"):
        _check(tmp_path, short, cfg)
    q8 = hf_tensors(cfg, quant_bits=8)
    with pytest.raises(_lib.VellaError) as e:
        _check(tmp_path, q8, cfg)  # an 8-bit checkpoint for a 4-bit handle
    assert e.value.code == _lib.E_UNSUPPORTED


def test_whisper_config_from_both_key_sets():
    from vella_b200 import _lib
    from vella_b200 import checkpoint as C
    hf = {"num_mel_bins": 128, "d_model": 1280, "encoder_attention_heads": 20, "encoder_layers": 32,
          "decoder_layers": 4, "encoder_ffn_dim": 5120, "vocab_size": 51866, "max_source_positions": 1500,
          "max_target_positions": 448}
    c = C.whisper_config(hf)
    assert (c.n_mels, c.d_model, c.heads, c.enc_layers, c.dec_layers, c.ffn, c.vocab, c.bits, c.dtype) == \
        (128, 1280, 20, 32, 4, 5120, 51866, 0, _lib.F16)
    mlx = {"n_mels": 80, "n_audio_ctx": 1500, "n_audio_state": 384, "n_audio_head": 6, "n_audio_layer": 4,
           "n_vocab": 51865, "n_text_ctx": 448, "n_text_state": 384, "n_text_head": 6, "n_text_layer": 4,
           "quantization": {"group_size": 64, "bits": 4}}
    c = C.whisper_config(mlx)
    assert (c.n_mels, c.d_model, c.heads, c.ffn, c.vocab, c.bits) == (80, 384, 6, 1536, 51865, 4)
    assert C.whisper_config(hf, bits=8).bits == 8  # derived precision
    with pytest.raises(ValueError):
        C.whisper_config(mlx, bits=8)
    with pytest.raises(ValueError):
        C.whisper_config({**mlx, "quantization": {"group_size": 32, "bits": 4}})


def test_whisper_token_ids_and_suppress_lists(tmp_path):
    from vella_b200 import checkpoint as C
    (tmp_path / "config.json").write_text(json.dumps({"vocab_size": 51866, "decoder_start_token_id": 50258}))
    (tmp_path / "generation_config.json").write_text(json.dumps({
        "eos_token_id": 50257, "no_timestamps_token_id": 50364, "suppress_tokens": [1, 2, 7],
        "begin_suppress_tokens": [220, 50257], "lang_to_id": {"<|en|>": 50259, "<|de|>": 50261},
        "task_to_id": {"transcribe": 50360, "translate": 50359}, "is_multilingual": True}))
    (tmp_path / "tokenizer_config.json").write_text(json.dumps({"added_tokens_decoder": {
        "50258": {"content": "<|startoftranscript|>"}, "50361": {"content": "<|startoflm|>"},
        "50362": {"content": "<|startofprev|>"}, "50363": {"content": "<|nospeech|>"},
        "50260": {"content": "<|zh|>"}}}))
    t = C.whisper_tokens(tmp_path)
    assert (t.sot, t.eot, t.no_timestamps, t.timestamp_begin) == (50258, 50257, 50364, 50365)
    assert t.suppress == [1, 2, 7, 50258, 50359, 50360, 50361, 50362, 50363]
    assert t.begin_suppress == [220, 50257]
    assert t.prompt("en") == [50258, 50259, 50360]
    assert t.prompt("<|zh|>", task="translate") == [50258, 50260, 50359]
    assert t.prompt(None, without_timestamps=True) == [50258, 50360, 50364]
    assert t.rules()["timestamp_begin"] == 50365
    # without generation or tokenizer files: the config's ids (WhisperTokenizer.swift:53)
    bare = tmp_path / "bare"
    bare.mkdir()
    (bare / "config.json").write_text(json.dumps({"vocab_size": 51865}))
    t = C.whisper_tokens(bare)
    assert (t.sot, t.eot, t.no_timestamps, t.multilingual) == (50258, 50257, 50363, False)
    assert t.begin_suppress == [220, 50257] and t.suppress == [50258]
    (bare / "config.json").write_text(json.dumps({"vocab_size": 51864, "decoder_start_token_id": 50257}))
    assert C.whisper_tokens(bare).no_timestamps == 50361  # English-only vocabulary: start + 104


# ---- B200: loading into a handle ------------------------------------------------------

def _download(model, name, layer=-1):
    import torch

    class _Dev:
        def __init__(self, ptr, nbytes):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3}
    ptr, nbytes = model.tensor(name, layer)
    return torch.as_tensor(_Dev(ptr, nbytes), device="cuda").cpu().numpy()


def _handle_tensors(cfg):
    out = [("conv1.w", -1), ("conv1.bias", -1), ("conv2.w", -1), ("conv2.bias", -1), ("enc_pos", -1),
           ("dec_pos", -1), ("enc_ln.weight", -1), ("enc_ln.bias", -1), ("dec_ln.weight", -1), ("dec_ln.bias", -1),
           ("embed.w", -1)]
    if cfg.bits:
        out += [("embed.s", -1), ("embed.b", -1)]
    for l in range(cfg.enc_layers):
        for n in ("ln1", "ln2"):
            out += [(f"enc.{n}.weight", l), (f"enc.{n}.bias", l)]
        for n in ("qkv", "o", "fc1", "fc2"):
            out += [(f"enc.{n}.w", l), (f"enc.{n}.bias", l)]
    for l in range(cfg.dec_layers):
        for n in ("ln1", "ln2", "ln3"):
            out += [(f"dec.{n}.weight", l), (f"dec.{n}.bias", l)]
        for n in ("qkv", "o", "cq", "ckv", "co", "fc1", "fc2"):
            out += [(f"dec.{n}.w", l), (f"dec.{n}.bias", l)]
            if cfg.bits:
                out += [(f"dec.{n}.s", l), (f"dec.{n}.b", l)]
    return out


def export_hf(model, cfg):
    """The handle's tensors as a Hugging Face checkpoint (decoder MLX-affine when bits)."""
    d, F, V, C = cfg.d_model, cfg.ffn, cfg.vocab, cfg.n_mels
    f16 = lambda name, layer=-1: _download(model, name, layer).view(np.float16)  # noqa: E731
    u32 = lambda name, layer=-1: _download(model, name, layer).view(np.uint32)  # noqa: E731
    kp1 = (3 * C + 63) // 64 * 64
    t = {"model.encoder.conv1.weight": f16("conv1.w").reshape(d, kp1)[:, :3 * C].reshape(d, 3, C).transpose(0, 2, 1),
         "model.encoder.conv1.bias": f16("conv1.bias"),
         "model.encoder.conv2.weight": f16("conv2.w").reshape(d, 3, d).transpose(0, 2, 1),
         "model.encoder.conv2.bias": f16("conv2.bias"),
         "model.encoder.embed_positions.weight": f16("enc_pos").reshape(cfg.n_audio, d),
         "model.decoder.embed_positions.weight": f16("dec_pos").reshape(cfg.max_target, d),
         "model.encoder.layer_norm.weight": f16("enc_ln.weight"), "model.encoder.layer_norm.bias": f16("enc_ln.bias"),
         "model.decoder.layer_norm.weight": f16("dec_ln.weight"), "model.decoder.layer_norm.bias": f16("dec_ln.bias")}

    def lin(dst, rows, name, layer, k, bits, bias=True):
        """Split the handle's Linear `name` by rows into the checkpoint Linears `dst`."""
        if bits:
            w = u32(f"{name}.w", layer).reshape(-1, k * bits // 32)
            s = f16(f"{name}.s", layer).reshape(-1, k // 64)
            b = f16(f"{name}.b", layer).reshape(-1, k // 64)
        else:
            w = f16(f"{name}.w", layer).reshape(-1, k)
        bb = f16(f"{name}.bias", layer) if bias else None
        r0 = 0
        for prefix, n in zip(dst, rows):
            t[prefix + ".weight"] = w[r0:r0 + n]
            if bits:
                t[prefix + ".scales"], t[prefix + ".biases"] = s[r0:r0 + n], b[r0:r0 + n]
            if bb is not None and not prefix.endswith("k_proj"):
                t[prefix + ".bias"] = bb[r0:r0 + n]
            r0 += n

    lin(["model.decoder.embed_tokens"], [V], "embed", -1, d, cfg.bits, bias=False)
    for l in range(cfg.enc_layers):
        p = f"model.encoder.layers.{l}."
        for n, hf in (("ln1", "self_attn_layer_norm"), ("ln2", "final_layer_norm")):
            t[p + hf + ".weight"], t[p + hf + ".bias"] = f16(f"enc.{n}.weight", l), f16(f"enc.{n}.bias", l)
        lin([p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"], [d] * 3, "enc.qkv", l, d, 0)
        lin([p + "self_attn.out_proj"], [d], "enc.o", l, d, 0)
        lin([p + "fc1"], [F], "enc.fc1", l, d, 0)
        lin([p + "fc2"], [d], "enc.fc2", l, F, 0)
    b = cfg.bits
    for l in range(cfg.dec_layers):
        p = f"model.decoder.layers.{l}."
        for n, hf in (("ln1", "self_attn_layer_norm"), ("ln2", "encoder_attn_layer_norm"), ("ln3", "final_layer_norm")):
            t[p + hf + ".weight"], t[p + hf + ".bias"] = f16(f"dec.{n}.weight", l), f16(f"dec.{n}.bias", l)
        lin([p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"], [d] * 3, "dec.qkv", l, d, b)
        lin([p + "self_attn.out_proj"], [d], "dec.o", l, d, b)
        lin([p + "encoder_attn.q_proj"], [d], "dec.cq", l, d, b)
        lin([p + "encoder_attn.k_proj", p + "encoder_attn.v_proj"], [d, d], "dec.ckv", l, d, b)
        lin([p + "encoder_attn.out_proj"], [d], "dec.co", l, d, b)
        lin([p + "fc1"], [F], "dec.fc1", l, d, b)
        lin([p + "fc2"], [d], "dec.fc2", l, F, b)
    return {k: np.ascontiguousarray(v) for k, v in t.items()}


def _write_dir(path, tensors, cfg_json, shards=1):
    path.mkdir()
    (path / "config.json").write_text(json.dumps(cfg_json))
    keys = sorted(tensors)
    for i in range(shards):
        write_safetensors(path / f"model-{i + 1:05d}-of-{shards:05d}.safetensors",
                          {k: tensors[k] for k in keys[i::shards]})


def _hf_config(cfg, quant=None):
    j = {"num_mel_bins": cfg.n_mels, "d_model": cfg.d_model, "encoder_attention_heads": cfg.heads,
         "encoder_layers": cfg.enc_layers, "decoder_layers": cfg.dec_layers, "encoder_ffn_dim": cfg.ffn,
         "vocab_size": cfg.vocab, "max_source_positions": cfg.n_audio, "max_target_positions": cfg.max_target}
    if quant:
        j["quantization"] = {"group_size": 64, "bits": quant}
    return j


@pytest.mark.gpu
def test_loaded_handles_equal_their_source(tmp_path):
    """Hugging Face (two shards) and mlx-whisper layouts of an int4 Whisper-tiny handle load into
    handles whose every tensor is bit-equal to the source's, and which decode the same tokens."""
    from vella_b200 import checkpoint as C
    from vella_b200 import whisper as VW
    cfg = VW.TINY
    src = VW.Whisper(cfg)
    src.init_random(11, 0.05)
    t = export_hf(src, cfg)
    mel = np.random.default_rng(3).standard_normal((cfg.n_mels, 2 * cfg.n_audio)).astype(np.float32)
    src.encode(mel)
    prompt = [50258, 50259, 50359, 50363]
    want = src.decode(prompt, 12).tokens
    names = _handle_tensors(cfg)
    ref = {n: _download(src, *n) for n in names}
    for tag, tensors, shards in (("hf", t, 2), ("mlx", to_mlx_names(t), 1)):
        d = tmp_path / tag
        _write_dir(d, tensors, _hf_config(cfg, quant=cfg.bits), shards)
        m = C.load_whisper(d)
        for n in names:
            assert np.array_equal(_download(m, *n), ref[n]), (tag, n)
        m.encode(mel)
        assert m.decode(prompt, 12).tokens == want, tag
        m.close()
    src.close()


@pytest.mark.gpu
def test_derived_int4_matches_the_oracle_quantizer(tmp_path):
    """A float (fp16) checkpoint loaded into an int4 handle: every decoder Linear and the token
    embedding are the oracle's MLX-affine quantization of the float rows, bit for bit; the
    dense encoder Linears hold those codes dequantized (the reference's derived precision
    quantizes every Linear), the convolutions their float values."""
    from vella_b200 import checkpoint as C
    from vella_b200 import whisper as VW
    from dataclasses import replace
    cfg = replace(VW.TINY, bits=0)
    src = VW.Whisper(cfg)
    src.init_random(12, 0.05)
    t = export_hf(src, cfg)
    d = tmp_path / "float"
    _write_dir(d, t, _hf_config(cfg))
    m = C.load_whisper(d, bits=4)
    D = cfg.d_model
    for name, layer, parts, k in (("embed", -1, ["model.decoder.embed_tokens"], D),
                                  ("dec.qkv", 0, [f"model.decoder.layers.0.self_attn.{p}_proj" for p in "qkv"], D),
                                  ("dec.ckv", 1, [f"model.decoder.layers.1.encoder_attn.{p}_proj" for p in "kv"], D),
                                  ("dec.fc2", 3, ["model.decoder.layers.3.fc2"], cfg.ffn)):
        w = np.concatenate([t[p + ".weight"] for p in parts]).astype(np.float32)
        q, s, b = A.quantize(w, 4, "f16")
        assert np.array_equal(_download(m, f"{name}.w", layer).view(np.uint32).reshape(q.shape), q), name
        assert np.array_equal(_download(m, f"{name}.s", layer).view(np.float16).reshape(s.shape), s), name
        assert np.array_equal(_download(m, f"{name}.b", layer).view(np.float16).reshape(b.shape), b), name
    for l in (0, 2):
        w = t[f"model.encoder.layers.{l}.fc1.weight"].astype(np.float32)
        deq = A.dequantize(*A.quantize(w, 4, "f16"), 4, "f16").astype(np.float16)
        assert np.array_equal(_download(m, "enc.fc1.w", l).view(np.float16).reshape(deq.shape), deq), l
    assert np.array_equal(_download(m, "conv2.w"), _download(src, "conv2.w"))
    m.close()
    src.close()


# ---- Qwen3-style decoder models ---------------------------------------------------------

def small_model_cfg(bits=4, qk_norm=True):
    from vella_b200.decode import ModelConfig
    return ModelConfig(2, 256, 4, 2, 64, 512, 1000, bits=bits, qk_norm=qk_norm, max_seq=128, max_prefix=64)


def qwen3_tensors(cfg, quant_bits=0, tied=False, prefix="", rng=None):
    rng = rng or np.random.default_rng(2)
    d, F, V, H, KV, hd = cfg.d_model, cfg.ffn, cfg.vocab, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    f = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float16)  # noqa: E731
    t = {}

    def lin(name, n, k, quant=bool(quant_bits)):
        w = f(n, k)
        if quant:
            q, s, b = A.quantize(w.astype(np.float32), quant_bits, "f16")
            t[name + ".weight"], t[name + ".scales"], t[name + ".biases"] = q, s, b
        else:
            t[name + ".weight"] = w

    lin("model.embed_tokens", V, d)
    t["model.norm.weight"] = f(d)
    if not tied:
        lin("lm_head", V, d)
    for l in range(cfg.n_layers):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"], t[p + "post_attention_layernorm.weight"] = f(d), f(d)
        if cfg.qk_norm:
            t[p + "self_attn.q_norm.weight"], t[p + "self_attn.k_norm.weight"] = f(hd), f(hd)
        lin(p + "self_attn.q_proj", H * hd, d)
        lin(p + "self_attn.k_proj", KV * hd, d)
        lin(p + "self_attn.v_proj", KV * hd, d)
        lin(p + "self_attn.o_proj", d, H * hd)
        lin(p + "mlp.gate_proj", F, d)
        lin(p + "mlp.up_proj", F, d)
        lin(p + "mlp.down_proj", d, F)
    return {prefix + k: v for k, v in t.items()}


def _check_model(tmp_path, tensors, cfg, name="model.safetensors"):
    from vella_b200 import checkpoint as C
    p = tmp_path / name
    write_safetensors(p, tensors)
    with _st([p]) as st:
        C.check_model_checkpoint(st, cfg)


@pytest.mark.parametrize("quant,tied,prefix", [(0, False, ""), (4, False, ""), (4, True, "thinker."), (0, True, "")])
def test_qwen3_checkpoints_pass_the_check(tmp_path, quant, tied, prefix):
    cfg = small_model_cfg(bits=4)
    _check_model(tmp_path, qwen3_tensors(cfg, quant, tied, prefix), cfg)


def test_qwen3_checkpoint_problems_are_named(tmp_path):
    from vella_b200 import _lib
    cfg = small_model_cfg(bits=4)
    t = qwen3_tensors(cfg)
    del t["model.layers.1.self_attn.k_norm.weight"]
    with pytest.raises(_lib.VellaError, match="k_norm"):
        _check_model(tmp_path, t, cfg)
    _check_model(tmp_path, t, small_model_cfg(bits=4, qk_norm=False), "noqk.safetensors")  # not needed then
    t = qwen3_tensors(cfg)
    t["model.layers.0.self_attn.o_proj.weight"] = t["model.layers.0.self_attn.o_proj.weight"][:, :128].copy()
    with pytest.raises(_lib.VellaError, match="o_proj"):
        _check_model(tmp_path, t, cfg, "bad.safetensors")


def test_qwen3_config():
    from vella_b200 import _lib
    from vella_b200 import checkpoint as C
    j = {"num_hidden_layers": 28, "hidden_size": 2048, "num_attention_heads": 16, "num_key_value_heads": 8,
         "head_dim": 128, "intermediate_size": 6144, "vocab_size": 151936, "rms_norm_eps": 1e-6,
         "rope_theta": 1000000, "torch_dtype": "bfloat16"}
    c = C.model_config(j, max_seq=1280)
    assert (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab, c.bits, c.dtype,
            c.max_seq) == (28, 2048, 16, 8, 128, 6144, 151936, 0, _lib.BF16, 1280)
    asr = {"thinker_config": {"text_config": {**j, "torch_dtype": "float16"}},
           "quantization": {"group_size": 64, "bits": 4}}
    c = C.model_config(asr)
    assert (c.bits, c.dtype, c.vocab) == (4, _lib.F16, 151936)


def export_qwen3(model, cfg):
    """The model handle's tensors as a Qwen3 checkpoint (MLX-affine when bits)."""
    d, F, V, H, KV, hd = cfg.d_model, cfg.ffn, cfg.vocab, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    raw = lambda n, l=-1: _download(model, n, l)  # noqa: E731
    t = {"model.embed_tokens.weight": raw("embed").view(np.float16).reshape(V, d),
         "model.norm.weight": raw("final_norm").view(np.float16)}
    b = cfg.bits

    def lin(dst, rows, name, layer, k):
        if b:
            w = raw(f"{name}.w", layer).view(np.uint32).reshape(-1, k * b // 32)
            s = raw(f"{name}.s", layer).view(np.float16).reshape(-1, k // 64)
            bb = raw(f"{name}.b", layer).view(np.float16).reshape(-1, k // 64)
        else:
            w = raw(f"{name}.w", layer).view(np.float16).reshape(-1, k)
        r0 = 0
        for prefix, n in zip(dst, rows):
            t[prefix + ".weight"] = w[r0:r0 + n]
            if b:
                t[prefix + ".scales"], t[prefix + ".biases"] = s[r0:r0 + n], bb[r0:r0 + n]
            r0 += n

    lin(["lm_head"], [V], "lm_head", -1, d)
    for l in range(cfg.n_layers):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = raw("attn_norm", l).view(np.float16)
        t[p + "post_attention_layernorm.weight"] = raw("mlp_norm", l).view(np.float16)
        if cfg.qk_norm:
            t[p + "self_attn.q_norm.weight"] = raw("q_norm", l).view(np.float16)
            t[p + "self_attn.k_norm.weight"] = raw("k_norm", l).view(np.float16)
        lin([p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"], [H * hd, KV * hd, KV * hd],
            "qkv", l, d)
        lin([p + "self_attn.o_proj"], [d], "o", l, H * hd)
        lin([p + "mlp.gate_proj"], [F], "gate", l, d)
        lin([p + "mlp.up_proj"], [F], "up", l, d)
        lin([p + "mlp.down_proj"], [d], "down", l, F)
    return {k: np.ascontiguousarray(v) for k, v in t.items()}


def _model_tensors(cfg):
    out = [("embed", -1), ("final_norm", -1), ("lm_head.w", -1)] + ([("lm_head.s", -1), ("lm_head.b", -1)] if cfg.bits else [])
    for l in range(cfg.n_layers):
        out += [("attn_norm", l), ("mlp_norm", l)] + ([("q_norm", l), ("k_norm", l)] if cfg.qk_norm else [])
        for n in ("qkv", "o", "gate", "up", "down"):
            out += [(f"{n}.w", l)] + ([(f"{n}.s", l), (f"{n}.b", l)] if cfg.bits else [])
    return out


def _qwen3_json(cfg, quant=None):
    j = {"num_hidden_layers": cfg.n_layers, "hidden_size": cfg.d_model, "num_attention_heads": cfg.n_heads,
         "num_key_value_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn,
         "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta, "torch_dtype": "float16"}
    if quant:
        j["quantization"] = {"group_size": 64, "bits": quant}
    return j


@pytest.mark.gpu
def test_loaded_models_equal_their_source_and_derive_int4(tmp_path):
    """An int4 Qwen3-style model written as an MLX-quantized checkpoint (two shards, "thinker."
    prefix) loads bit-equal, tensor by tensor; a float checkpoint with a tied
    embedding loads into an int4 model whose lm_head and Linears are the oracle quantizer's
    codes of the float rows."""
    from dataclasses import replace

    from vella_b200 import _lib
    from vella_b200 import checkpoint as C
    from vella_b200 import decode as VD
    cfg = replace(small_model_cfg(bits=4), dtype=_lib.F16)
    src = VD.Model(cfg)
    src.init_random(21, 0.05)
    t = export_qwen3(src, cfg)
    d = tmp_path / "q4"
    _write_dir(d, {"thinker." + k: v for k, v in t.items()}, _qwen3_json(cfg, quant=4), shards=2)
    m = C.load_model(d, max_seq=cfg.max_seq, max_prefix=cfg.max_prefix)
    assert m.cfg.bits == 4 and m.cfg.qk_norm and m.cfg.dtype == _lib.F16
    for n in _model_tensors(cfg):
        assert np.array_equal(_download(m, *n), _download(src, *n)), n
    m.close()
    # float source, tied embedding, derived int4
    fcfg = replace(cfg, bits=0)
    fsrc = VD.Model(fcfg)
    fsrc.init_random(22, 0.05)
    ft = export_qwen3(fsrc, fcfg)
    del ft["lm_head.weight"]
    d = tmp_path / "tied"
    _write_dir(d, ft, _qwen3_json(fcfg))
    m = C.load_model(d, bits=4, max_seq=cfg.max_seq, max_prefix=cfg.max_prefix)
    emb = ft["model.embed_tokens.weight"]
    assert np.array_equal(_download(m, "embed").view(np.float16).reshape(emb.shape), emb)
    for name, layer, w in (("lm_head", -1, emb),
                           ("qkv", 1, np.concatenate([ft[f"model.layers.1.self_attn.{p}_proj.weight"] for p in "qkv"])),
                           ("down", 0, ft["model.layers.0.mlp.down_proj.weight"])):
        q, s, b = A.quantize(w.astype(np.float32), 4, "f16")
        assert np.array_equal(_download(m, f"{name}.w", layer).view(np.uint32).reshape(q.shape), q), name
        assert np.array_equal(_download(m, f"{name}.s", layer).view(np.float16).reshape(s.shape), s), name
        assert np.array_equal(_download(m, f"{name}.b", layer).view(np.float16).reshape(b.shape), b), name
    m.close()
    fsrc.close()
    src.close()


def test_corrupted_files_are_rejected_without_crashing(tmp_path):
    """Random byte flips, truncations and header rewrites of a valid file, opened in a child
    process: each open either succeeds or raises VellaError (no crash, no hang)."""
    import subprocess
    import sys
    rng = np.random.default_rng(11)
    good = tmp_path / "good.safetensors"
    write_safetensors(good, {"a": np.arange(12, dtype=np.float32).reshape(3, 4), "b": np.ones(5, np.float16),
                             "c": np.zeros((2, 2), np.uint32)}, metadata={"k": "v"})
    raw = good.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    cases = []
    for i in range(60):
        b = bytearray(raw)
        kind = i % 4
        if kind == 0:  # flip bytes inside the JSON header
            for _ in range(rng.integers(1, 6)):
                j = int(rng.integers(8, 8 + hlen))
                b[j] = int(rng.integers(0, 256))
        elif kind == 1:  # truncate anywhere
            b = b[:int(rng.integers(0, len(b)))]
        elif kind == 2:  # a wrong header length
            b[:8] = struct.pack("<Q", int(rng.integers(0, 2 * len(b))))
        else:  # a header with extreme or negative numbers
            h = json.dumps({"x": {"dtype": "F32", "shape": [int(rng.integers(-5, 2**62))],
                                  "data_offsets": [int(rng.integers(-10, 100)), int(rng.integers(-10, 2**62))]}})
            hb = h.encode()
            b = bytearray(struct.pack("<Q", len(hb)) + hb + bytes(16))
        p = tmp_path / f"case{i}.safetensors"
        p.write_bytes(bytes(b))
        cases.append(str(p))
    code = (
        "import sys\n"
        "from vella_b200 import _lib, checkpoint as C\n"
        "ok = bad = 0\n"
        "for p in sys.argv[1:]:\n"
        "    try:\n"
        "        st = C.SafeTensors([p]); [st.array(k) for k in st.keys()]; st.close(); ok += 1\n"
        "    except _lib.VellaError:\n"
        "        bad += 1\n"
        "print(ok, bad)\n")
    import os
    root = str(__import__("pathlib").Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", code, *cases], capture_output=True, text=True, timeout=120,
                       cwd=root, env={**os.environ, "PYTHONPATH": root})
    assert r.returncode == 0, r.stderr[-2000:]
    ok, bad = map(int, r.stdout.split())
    assert ok + bad == len(cases) and bad > 0


# ---- Nemotron-H ---------------------------------------------------------------------------

def small_nh_cfg(bits=0, mtp=True):
    from vella_b200.nemotron import NHConfig
    return NHConfig(vocab=96, hidden=64, heads=2, kv_heads=1, head_dim=64, m_heads=4, m_head_dim=16, state_dim=32,
                    groups=2, moe_inter=128, shared_inter=64, experts=4, top_k=2, pattern="M*E", bits=bits, mtp=mtp,
                    max_seq=32, max_rows=8)


def nemo_tensors(c, quant_bits=0, rng=None):
    """NVIDIA NeMo key layout (llm.model.*, experts [E][in][out], llm.mtp.*) with random values."""
    rng = rng or np.random.default_rng(6)
    f = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float16)  # noqa: E731
    d, I = c.hidden, c.m_heads * c.m_head_dim
    conv = I + 2 * c.groups * c.state_dim
    t = {"llm.model.embed_tokens.weight": f(c.vocab, d), "llm.model.norm.weight": f(d), "llm.lm_head.weight": f(c.vocab, d)}

    def attn(p):
        t[p + "q_proj.weight"] = f(c.heads * c.head_dim, d)
        t[p + "k_proj.weight"] = f(c.kv_heads * c.head_dim, d)
        t[p + "v_proj.weight"] = f(c.kv_heads * c.head_dim, d)
        t[p + "o_proj.weight"] = f(d, c.heads * c.head_dim)

    def moe(p):
        t[p + "gate.weight"] = f(c.experts, d)
        t[p + "gate.e_score_correction_bias"] = np.zeros(c.experts, np.float32)
        t[p + "experts.gate_and_up_projs"] = f(c.experts, d, c.moe_inter)      # [E][in][out]
        t[p + "experts.down_projs"] = f(c.experts, c.moe_inter, d)
        t[p + "shared_experts.up_proj.weight"] = f(c.shared_inter, d)
        t[p + "shared_experts.down_proj.weight"] = f(d, c.shared_inter)

    for l, kind in enumerate(c.pattern):
        p = f"llm.model.layers.{l}."
        t[p + "norm.weight"] = f(d)
        if kind == "M":
            t[p + "mixer.in_proj.weight"] = f(I + conv + c.m_heads, d)
            t[p + "mixer.out_proj.weight"] = f(d, I)
            t[p + "mixer.conv1d.weight"] = f(conv, 1, c.conv_kernel)
            t[p + "mixer.conv1d.bias"] = f(conv)
            t[p + "mixer.norm.weight"] = f(I)
            for n in ("A_log", "dt_bias", "D"):
                t[p + "mixer." + n] = rng.standard_normal(c.m_heads).astype(np.float32)
        elif kind == "*":
            attn(p + "mixer.")
        else:
            moe(p + "mixer.")
    if c.mtp:
        m = "llm.mtp.layers."
        t[m + "0.eh_proj.weight"] = f(d, 2 * d)
        for n in ("enorm", "hnorm"):
            t[m + f"0.{n}.weight"] = f(d)
        t[m + "0.norm.weight"] = f(d)
        attn(m + "0.mixer.")
        t[m + "1.norm.weight"] = f(d)
        moe(m + "1.mixer.")
        t[m + "1.final_layernorm.weight"] = f(d)
    t["llm.model.layers.0.mixer._extra_state"] = np.zeros(4, np.uint8)  # skipped like the reference
    return t


def test_nemotron_checkpoint_layout_passes_the_check(tmp_path):
    from vella_b200 import checkpoint as C
    c = small_nh_cfg()
    p = tmp_path / "nh.safetensors"
    write_safetensors(p, nemo_tensors(c))
    with _st([p]) as st:
        C.check_nh_checkpoint(st, c)
        C.check_nh_checkpoint(st, small_nh_cfg(bits=4))  # float experts: derived at load


def test_nemotron_checkpoint_problems_are_named(tmp_path):
    from vella_b200 import _lib
    from vella_b200 import checkpoint as C
    c = small_nh_cfg()
    t = nemo_tensors(c)
    del t["llm.mtp.layers.1.final_layernorm.weight"]
    p = tmp_path / "a.safetensors"
    write_safetensors(p, t)
    with _st([p]) as st:
        with pytest.raises(_lib.VellaError, match="mtp.final_norm"):
            C.check_nh_checkpoint(st, c)
        C.check_nh_checkpoint(st, small_nh_cfg(mtp=False))  # no MTP head wanted: fine
    t = nemo_tensors(c)
    t["llm.model.layers.2.mixer.experts.down_projs"] = np.zeros((c.experts, c.hidden, c.moe_inter), np.float16)
    p = tmp_path / "b.safetensors"
    write_safetensors(p, t)
    with _st([p]) as st:
        with pytest.raises(_lib.VellaError, match="switch_mlp.fc2"):
            C.check_nh_checkpoint(st, c)  # [E][out][in] where NeMo stores [E][in][out]
