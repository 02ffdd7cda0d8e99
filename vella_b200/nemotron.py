"""ctypes binding of the Nemotron-H Mamba-2 mixer core (``vella_mamba_*`` in
``include/vella_cuda.h``), over torch tensors on the device.

Names follow the reference's ``NTMamba`` (``Worker/Sources/MLXAudioSTT/NemotronTranscribe/
NemotronTranscribeDecoder.swift:318-360``): ``conv`` is the cached causal conv with SiLU,
``ssm`` the selective scan with its fp32 state, ``gated_norm`` NTGatedRMSNorm.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib


class MambaDesc(ctypes.Structure):
    _fields_ = [("streams", ctypes.c_int32), ("tokens", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("groups", ctypes.c_int32), ("state_dim", ctypes.c_int32),
                ("conv_kernel", ctypes.c_int32), ("dtype", ctypes.c_int32), ("in_stride", ctypes.c_int32),
                ("dt_min", ctypes.c_float), ("dt_max", ctypes.c_float), ("eps", ctypes.c_float)]


_vp = ctypes.c_void_p
for _name, _args in [
    ("vella_mamba_conv", [ctypes.POINTER(MambaDesc), _vp, _vp, _vp, _vp, _vp, _vp]),
    ("vella_mamba_ssm", [ctypes.POINTER(MambaDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("vella_mamba_gated_norm", [ctypes.POINTER(MambaDesc), _vp, _vp, _vp, _vp, _vp]),
]:
    _lib.declare(_name, ctypes.c_int, _args)


@dataclass
class MambaShape:
    heads: int
    head_dim: int
    groups: int
    state_dim: int
    conv_kernel: int = 4
    dt_min: float = 0.0
    dt_max: float = float("inf")
    eps: float = 1e-5
    dtype: int = _lib.BF16

    @property
    def inner(self) -> int:
        return self.heads * self.head_dim

    @property
    def conv_dim(self) -> int:
        return self.inner + 2 * self.groups * self.state_dim

    @property
    def in_width(self) -> int:
        return self.inner + self.conv_dim + self.heads

    def desc(self, streams: int, tokens: int, in_stride: int = 0) -> MambaDesc:
        return MambaDesc(streams, tokens, self.heads, self.head_dim, self.groups, self.state_dim, self.conv_kernel,
                         self.dtype, in_stride or self.in_width, self.dt_min, self.dt_max, self.eps)


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def conv(shape: MambaShape, zxbcdt, conv_w, conv_b, conv_state, xbc, streams: int, tokens: int):
    d = shape.desc(streams, tokens, zxbcdt.stride(0))
    _lib.check(_lib.lib().vella_mamba_conv(ctypes.byref(d), _p(zxbcdt), _p(conv_w), _p(conv_b), _p(conv_state),
                                           _p(xbc), _stream()))


def ssm(shape: MambaShape, xbc, zxbcdt, a_log, dt_bias, D, state, y, streams: int, tokens: int):
    d = shape.desc(streams, tokens, zxbcdt.stride(0))
    _lib.check(_lib.lib().vella_mamba_ssm(ctypes.byref(d), _p(xbc), _p(zxbcdt), _p(a_log), _p(dt_bias), _p(D),
                                          _p(state), _p(y), _stream()))


def gated_norm(shape: MambaShape, y, zxbcdt, norm_w, out, streams: int, tokens: int):
    d = shape.desc(streams, tokens, zxbcdt.stride(0))
    _lib.check(_lib.lib().vella_mamba_gated_norm(ctypes.byref(d), _p(y), _p(zxbcdt), _p(norm_w), _p(out),
                                                 _stream()))


class MoeRouteDesc(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int32), ("hidden", ctypes.c_int32), ("experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("norm_topk", ctypes.c_int32), ("scaling", ctypes.c_float),
                ("dtype", ctypes.c_int32)]


_lib.declare("vella_moe_route", ctypes.c_int, [ctypes.POINTER(MoeRouteDesc), _vp, _vp, _vp, _vp, _vp, _vp])


def moe_route(x, router_w, bias, top_k: int, norm_topk: bool, scaling: float):
    """``NTMoE`` routing of the rows of x [rows, hidden] (bf16 or fp16 on the device): expert
    indices [rows, top_k] int32 and weights [rows, top_k] fp32."""
    import torch
    M, hidden = x.shape
    d = MoeRouteDesc(M, hidden, router_w.shape[0], top_k, int(norm_topk), scaling,
                     _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F16)
    idx = torch.empty(M, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(M, top_k, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().vella_moe_route(ctypes.byref(d), _p(x), _p(router_w), _p(bias), _p(idx), _p(w), _stream()))
    return idx, w


class MoeExpertsDesc(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("experts", ctypes.c_int32), ("top_k", ctypes.c_int32), ("bits", ctypes.c_int32),
                ("dtype", ctypes.c_int32)]


_lib.declare("vella_moe_experts_workspace_size", ctypes.c_size_t, [ctypes.POINTER(MoeExpertsDesc)])
# desc, x, expert_idx, expert_w, fc1 (w, scales, biases), fc2 (w, scales, biases), out; accumulate, workspace,
# workspace_bytes, stream
_lib.declare("vella_moe_experts", ctypes.c_int, [ctypes.POINTER(MoeExpertsDesc)] + [_vp] * 10 + [ctypes.c_int32, _vp,
                                                                                               ctypes.c_size_t, _vp])


def moe_experts(x, expert_idx, expert_w, fc1, fc2, inter: int, bits: int, out=None, accumulate: bool = False):
    """Routed relu^2 experts of the rows of x [rows, hidden] (device tensors): fc1 and fc2 are
    (w, scales, biases) triples (scales/biases None for dense weights)."""
    import torch
    M, hidden = x.shape
    E = fc1[0].shape[0]
    d = MoeExpertsDesc(M, hidden, inter, E, expert_idx.shape[1], bits,
                       _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F16)
    nbytes = int(_lib.lib().vella_moe_experts_workspace_size(ctypes.byref(d)))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty_like(x)
    _lib.check(_lib.lib().vella_moe_experts(ctypes.byref(d), _p(x), _p(expert_idx), _p(expert_w), _p(fc1[0]),
                                            _p(fc1[1]), _p(fc1[2]), _p(fc2[0]), _p(fc2[1]), _p(fc2[2]), _p(out),
                                            int(accumulate), _p(ws), ws.numel(), _stream()))
    return out


# ---------------------------------------------------------------------------------------
# The Nemotron-H backbone handle
# ---------------------------------------------------------------------------------------

class NHCfg(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int32), ("hidden", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("m_heads", ctypes.c_int32),
                ("m_head_dim", ctypes.c_int32), ("state_dim", ctypes.c_int32), ("conv_kernel", ctypes.c_int32),
                ("groups", ctypes.c_int32), ("moe_inter", ctypes.c_int32), ("shared_inter", ctypes.c_int32),
                ("experts", ctypes.c_int32), ("top_k", ctypes.c_int32), ("norm_topk", ctypes.c_int32),
                ("routed_scaling", ctypes.c_float), ("dt_min", ctypes.c_float), ("dt_max", ctypes.c_float),
                ("eps", ctypes.c_float), ("bits", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("max_rows", ctypes.c_int32), ("mtp", ctypes.c_int32),
                ("pattern", ctypes.c_char * 128)]


for _name, _res, _args in [
    ("vella_nh_create", ctypes.c_int, [ctypes.POINTER(NHCfg), ctypes.c_int32, ctypes.POINTER(_vp)]),
    ("vella_nh_destroy", ctypes.c_int, [_vp]),
    ("vella_nh_tensor", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int32, ctypes.POINTER(_vp),
                                       ctypes.POINTER(ctypes.c_size_t)]),
    ("vella_nh_forward", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int32), _vp, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), _vp, _vp]),
    ("vella_nh_mtp_forward", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int32), _vp, _vp, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), _vp]),
]:
    _lib.declare(_name, _res, _args)


@dataclass
class NHConfig:
    """Shapes of a Nemotron-H backbone (the reference's NTDecoderConfig, NemotronTranscribeDecoder.swift:11-36)."""
    vocab: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    m_heads: int
    m_head_dim: int
    state_dim: int
    groups: int
    moe_inter: int
    shared_inter: int
    experts: int
    top_k: int
    pattern: str
    conv_kernel: int = 4
    norm_topk: bool = True
    routed_scaling: float = 1.0
    dt_min: float = 0.0
    dt_max: float = float("inf")
    eps: float = 1e-5
    bits: int = 0
    dtype: int = _lib.BF16
    max_seq: int = 2048
    max_rows: int = 16
    mtp: bool = False

    def c(self) -> NHCfg:
        return NHCfg(self.vocab, self.hidden, self.heads, self.kv_heads, self.head_dim, self.m_heads, self.m_head_dim,
                     self.state_dim, self.conv_kernel, self.groups, self.moe_inter, self.shared_inter, self.experts,
                     self.top_k, int(self.norm_topk), self.routed_scaling, self.dt_min, self.dt_max, self.eps, self.bits,
                     self.dtype, self.max_seq, self.max_rows, int(self.mtp), self.pattern.encode())


class _DevBytes:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class NHModel:
    """A Nemotron-H backbone on one GPU (weights, Mamba states, attention caches)."""

    def __init__(self, cfg: NHConfig, device: int = 0):
        self.cfg = cfg
        self.h = _vp()
        c = cfg.c()
        _lib.check(_lib.lib().vella_nh_create(ctypes.byref(c), device, ctypes.byref(self.h)))

    def close(self):
        if self.h:
            _lib.lib().vella_nh_destroy(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor(self, name: str, layer: int = -1):
        p, n = _vp(), ctypes.c_size_t()
        _lib.check(_lib.lib().vella_nh_tensor(self.h, name.encode(), layer, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def forward(self, tokens=None, embeds=None, pos: int = 0, logits_rows: int = 1, logits_out=None,
                hidden_out=None):
        """Runs the rows (host token ids, or a device tensor of embeddings [rows, hidden]) at
        positions pos..; returns the argmax of the last logits_rows rows."""
        out = (ctypes.c_int32 * max(logits_rows, 1))()
        if tokens is not None:
            tk = (ctypes.c_int32 * len(tokens))(*tokens)
            rows = len(tokens)
            _lib.check(_lib.lib().vella_nh_forward(self.h, tk, None, rows, pos, logits_rows, out, _p(logits_out),
                                                   _p(hidden_out)))
        else:
            import torch
            torch.cuda.current_stream(embeds.device).synchronize()  # the handle's stream does not wait for torch's
            _lib.check(_lib.lib().vella_nh_forward(self.h, None, _p(embeds), embeds.shape[0], pos, logits_rows, out,
                                                   _p(logits_out), _p(hidden_out)))
        return list(out[:logits_rows])

    def mtp_forward(self, hidden, pos: int, next_tokens=None, next_embeds=None, logits_rows: int = 1, x_out=None):
        """The MTP head over (next token or embedding row, hidden row) pairs at MTP-cache
        positions pos..; returns the argmax of the last logits_rows rows."""
        import torch
        torch.cuda.current_stream(hidden.device).synchronize()
        out = (ctypes.c_int32 * max(logits_rows, 1))()
        tk = None if next_tokens is None else (ctypes.c_int32 * len(next_tokens))(*next_tokens)
        _lib.check(_lib.lib().vella_nh_mtp_forward(self.h, tk, _p(next_embeds), _p(hidden), hidden.shape[0], pos,
                                                   logits_rows, out, _p(x_out)))
        return list(out[:logits_rows])

    def embedding_rows(self, tokens):
        """Rows of the token embedding table (a device view, [len(tokens), hidden])."""
        import torch
        ptr, nbytes = self.tensor("embed")
        dt = torch.bfloat16 if self.cfg.dtype == _lib.BF16 else torch.float16
        table = torch.as_tensor(_DevBytes(ptr, nbytes), device="cuda").view(dt).view(-1, self.cfg.hidden)
        return table[list(tokens)]

    def reset(self):
        """A fresh sequence: the Mamba states zeroed (the reference makes a new cache per decode;
        attention and MTP cache rows are overwritten from position 0)."""
        for v in self.mamba_states():
            v.zero_()

    def mamba_states(self):
        """Device views of every Mamba layer's conv and SSM states (for snapshot / restore)."""
        import torch
        views = []
        for layer, kind in enumerate(self.cfg.pattern):
            if kind == "M":
                for name in ("conv_state", "ssm_state"):
                    ptr, nbytes = self.tensor(name, layer)
                    views.append(torch.as_tensor(_DevBytes(ptr, nbytes), device="cuda"))
        return views


_lib.declare("vella_loop_cut", ctypes.c_int, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_int32)])


def ends_in_loop(out: list) -> bool:
    """endsInLoop (NemotronTranscribeModel.swift:296-302) through the library's repetition guard
    (vella_loop_cut): once there are at least 20 tokens and their count is a multiple of 4, a tail
    of one block of at most 64 tokens repeated 20 times is cut to its first copy, in place, and
    True is returned."""
    n = len(out)
    arr = (ctypes.c_int32 * max(n, 1))(*out)
    kept = ctypes.c_int32(n)
    rc = _lib.lib().vella_loop_cut(arr, n, 1, ctypes.byref(kept))
    if rc < 0:
        _lib.check(rc)
    if rc == 1:
        del out[kept.value:]
        return True
    return False


def decode_greedy(model: NHModel, embeddings, max_tokens: int, eos=()):
    """decodeGreedy (NemotronTranscribeModel.swift:266-290) on the device: the prefix in chunks
    of max_rows, then one token per forward.  Like the reference, the decode stops at a
    repetition loop (ends_in_loop after every token), keeps one copy of the repeated block and
    sets ``model.decode_looped`` (the reference's ``decodeLooped``)."""
    R, T = model.cfg.max_rows, embeddings.shape[0]
    model.decode_looped = False
    model.reset()
    t = None
    for s0 in range(0, T, R):
        t = model.forward(embeds=embeddings[s0:s0 + R].contiguous(), pos=s0)[0]
    out, pos = [], T
    while len(out) < max_tokens and t not in eos:
        out.append(t)
        if ends_in_loop(out):
            model.decode_looped = True
            break
        t = model.forward(tokens=[t], pos=pos)[0]
        pos += 1
    return out


def decode_mtp(model: NHModel, embeddings, max_tokens: int, depth: int, eos=()):
    """decodeMTP (NemotronTranscribeModel.swift:306-396) on the device: depth chained MTP drafts
    verified in one forward; on a partial acceptance the Mamba states are restored from the
    pass's snapshot and the accepted prefix is fed again (the attention rows are overwritten);
    the MTP cache drops its depth - 1 chain rows every pass.  Returns (tokens, accepted counts).

    Two points where the device handle differs from MLX, which takes a feed of any length:
    vella_nh_forward takes at most max_rows rows, so once the re-fed prefix plus the next drafts
    would pass max_rows, the accepted prefix is committed instead (forwarded again after the
    restore, in chunks of at most max_rows, which leaves the Mamba states and attention rows
    where the reference's next verify pass would leave them) and only the bonus token stays
    pending; and, as in the reference, the decode stops at a repetition loop (ends_in_loop after
    every emitted token) and sets ``model.decode_looped``."""
    import torch
    R, T, d = model.cfg.max_rows, embeddings.shape[0], model.cfg.hidden
    if depth + 1 > R:
        raise ValueError(f"decode_mtp: depth {depth} needs max_rows >= {depth + 1} (max_rows {R})")
    dev = embeddings.device
    hs = torch.empty(T, d, dtype=embeddings.dtype, device=dev)
    model.decode_looped = False
    model.reset()
    t = None
    for s0 in range(0, T, R):
        t = model.forward(embeds=embeddings[s0:s0 + R].contiguous(), pos=s0, hidden_out=hs[s0:s0 + R])[0]
    out, hist = [], []
    if t in eos or max_tokens == 0:
        return out, hist
    out.append(t)
    mlen = 0
    x = torch.empty(R, d, dtype=embeddings.dtype, device=dev)

    def chain(x0, first):
        nonlocal mlen
        drafts, token, cur = [first], first, x0
        for _ in range(depth - 1):
            nx = torch.empty(1, d, dtype=embeddings.dtype, device=dev)
            token = model.mtp_forward(cur, mlen, next_tokens=[token], x_out=nx)[0]
            mlen += 1
            cur = nx
            drafts.append(token)
        return drafts

    nxt = torch.cat([embeddings[1:], model.embedding_rows([t]).to(embeddings.dtype)])
    first = None
    for s0 in range(0, T, R):
        n = min(R, T - s0)
        first = model.mtp_forward(hs[s0:s0 + n].contiguous(), mlen, next_embeds=nxt[s0:s0 + n].contiguous(),
                                  x_out=x[:n])[0]
        mlen += n
    drafts = chain(x[n - 1:n].clone(), first)
    pending, mtp_done, blen = [t], 0, T
    while len(out) < max_tokens:
        snapshot = [v.clone() for v in model.mamba_states()]
        fed = pending + drafts
        verified = torch.empty(len(fed), d, dtype=embeddings.dtype, device=dev)
        ys = model.forward(tokens=fed, pos=blen, logits_rows=len(fed), hidden_out=verified)
        k, a = len(pending), 0
        while a < len(drafts) and ys[k - 1 + a] == drafts[a]:
            a += 1
        bonus = ys[k - 1 + a]
        new = drafts[:a] + [bonus]
        hist.append(a)
        mlen -= depth - 1
        upto = k + a
        e_next = (fed[1:upto] + [bonus])[mtp_done:]
        nx = torch.empty(len(e_next), d, dtype=embeddings.dtype, device=dev)
        head = model.mtp_forward(verified[mtp_done:upto].contiguous(), mlen, next_tokens=e_next, x_out=nx)[0]
        mlen += len(e_next)
        drafts = chain(nx[-1:].clone(), head)
        if upto == len(fed):  # every draft accepted
            pending, mtp_done, blen = [bonus], 0, blen + len(fed)
        else:
            for v, s in zip(model.mamba_states(), snapshot):
                v.copy_(s)
            if upto + 1 + depth > R:
                # commit the accepted prefix: the next feed would not fit in max_rows rows
                for c0 in range(0, upto, R):
                    model.forward(tokens=fed[c0:min(upto, c0 + R)], pos=blen + c0, logits_rows=0)
                pending, mtp_done, blen = [bonus], 0, blen + upto
            else:
                pending, mtp_done = fed[:upto] + [bonus], upto
        for tok in new:
            if tok in eos:
                return out, hist
            out.append(tok)
            if len(out) >= max_tokens:
                return out, hist
            if ends_in_loop(out):
                model.decode_looped = True
                return out, hist
    return out, hist
