"""Parity of the Mamba-2 mixer kernels (vella_mamba_* through the C ABI) with the oracle,
each stage fed the device's own output of the stage before, so errors do not compound.

Bars: conv output and gated norm within 2e-2 absolute (bf16 storage of O(1) values); the scan's
output within 2e-2 of the oracle's and its fp32 state within 1e-4 relative; a 5-token chunk
gives, bit for bit, the outputs and states of 5 one-token calls.
"""
import numpy as np
import pytest

from oracle import decoder as D
from oracle import nemotron as N

pytestmark = pytest.mark.gpu


def _bf16(t):
    return t.float().cpu().numpy().astype(np.float64)


def _setup(S, T, seed=0):
    import torch

    from vella_b200 import nemotron as VN
    sh = VN.MambaShape(heads=8, head_dim=64, groups=2, state_dim=128, conv_kernel=4, dt_min=1e-3, dt_max=10.0)
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = "cuda"
    zx = (torch.randn(S * T, sh.in_width, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    conv_w = (torch.randn(sh.conv_dim, sh.conv_kernel, generator=g, device=dev) * 0.4).to(torch.bfloat16)
    conv_b = (torch.randn(sh.conv_dim, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    cstate = (torch.randn(S, sh.conv_kernel - 1, sh.conv_dim, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(sh.heads, generator=g, device=dev) * 0.5
    dt_bias = torch.randn(sh.heads, generator=g, device=dev) * 0.5
    D = torch.randn(sh.heads, generator=g, device=dev)
    state = torch.randn(S, sh.heads, sh.head_dim, sh.state_dim, generator=g, device=dev) * 0.1
    norm_w = (1.0 + 0.1 * torch.randn(sh.inner, generator=g, device=dev)).to(torch.bfloat16)
    return sh, zx, conv_w, conv_b, cstate, a_log, dt_bias, D, state, norm_w


@pytest.mark.parametrize("S,T", [(1, 1), (2, 5), (3, 9)])
def test_mixer_stages_match_the_oracle(S, T):
    import torch

    from vella_b200 import nemotron as VN
    sh, zx, conv_w, conv_b, cstate, a_log, dt_bias, D, state, norm_w = _setup(S, T)
    I, H, Dh, G, Ds = sh.inner, sh.heads, sh.head_dim, sh.groups, sh.state_dim
    cs0, st0 = _bf16(cstate), state.double().cpu().numpy()
    xbc = torch.empty(S * T, sh.conv_dim, dtype=torch.bfloat16, device="cuda")
    VN.conv(sh, zx, conv_w, conv_b, cstate, xbc, S, T)
    y = torch.empty(S * T, I, dtype=torch.bfloat16, device="cuda")
    VN.ssm(sh, xbc, zx, a_log, dt_bias, D, state, y, S, T)
    out = torch.empty_like(y)
    VN.gated_norm(sh, y, zx, norm_w, out, S, T)
    torch.cuda.synchronize()
    z = _bf16(zx).reshape(S, T, -1)
    xg, yg = _bf16(xbc).reshape(S, T, -1), _bf16(y).reshape(S, T, -1)
    for s in range(S):
        ref_x, ref_cs = N.conv_step(z[s][:, I:I + sh.conv_dim], _bf16(conv_w), _bf16(conv_b), cs0[s])
        assert np.abs(xg[s] - ref_x).max() <= 2e-2
        assert np.array_equal(_bf16(cstate)[s], ref_cs.astype(np.float32).astype(np.float64))
        x, B, C = N.split_xbc(xg[s], H, Dh, G, Ds)
        dt = N.compute_dt(z[s][:, I + sh.conv_dim:], dt_bias.cpu().numpy(), 1e-3, 10.0)
        ref_y, ref_st = N.ssm_scan(x, B, C, dt, a_log.cpu().numpy(), D.cpu().numpy(), st0[s])
        assert np.abs(yg[s] - ref_y.reshape(T, -1)).max() <= 2e-2 * max(1.0, np.abs(ref_y).max())
        st = state[s].double().cpu().numpy()
        assert np.abs(st - ref_st).max() <= 1e-4 * max(1.0, np.abs(ref_st).max())
        ref_o = N.gated_rmsnorm(yg[s], z[s][:, :I], _bf16(norm_w), G, sh.eps)
        assert np.abs(_bf16(out).reshape(S, T, -1)[s] - ref_o).max() <= 2e-2 * max(1.0, np.abs(ref_o).max())


def test_a_chunk_equals_one_token_steps():
    import torch

    from vella_b200 import nemotron as VN
    S, T = 2, 5
    sh, zx, conv_w, conv_b, cstate, a_log, dt_bias, D, state, norm_w = _setup(S, T, seed=3)
    cs_a, st_a = cstate.clone(), state.clone()
    xbc = torch.empty(S * T, sh.conv_dim, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(S * T, sh.inner, dtype=torch.bfloat16, device="cuda")
    VN.conv(sh, zx, conv_w, conv_b, cs_a, xbc, S, T)
    VN.ssm(sh, xbc, zx, a_log, dt_bias, D, st_a, y, S, T)
    cs_b, st_b = cstate.clone(), state.clone()
    zr = zx.view(S, T, -1)
    for t in range(T):
        z1 = zr[:, t].contiguous()
        x1 = torch.empty(S, sh.conv_dim, dtype=torch.bfloat16, device="cuda")
        y1 = torch.empty(S, sh.inner, dtype=torch.bfloat16, device="cuda")
        VN.conv(sh, z1, conv_w, conv_b, cs_b, x1, S, 1)
        VN.ssm(sh, x1, z1, a_log, dt_bias, D, st_b, y1, S, 1)
        assert torch.equal(x1, xbc.view(S, T, -1)[:, t]) and torch.equal(y1, y.view(S, T, -1)[:, t]), t
    assert torch.equal(cs_a, cs_b) and torch.equal(st_a, st_b)


def test_bad_descriptors_are_rejected():
    import torch

    from vella_b200 import _lib
    from vella_b200 import nemotron as VN
    sh = VN.MambaShape(heads=8, head_dim=64, groups=3, state_dim=100)
    t = torch.zeros(4, 4096, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.VellaError):
        VN.conv(sh, t, t, None, t, t, 1, 1)


def test_moe_route_matches_the_oracle():
    """The chosen experts equal the oracle's wherever the k-th and (k+1)-th biased scores are
    apart by more than the fp32 dot-product error, and each expert's weight is within 1e-5."""
    import torch

    from vella_b200 import nemotron as VN
    g = torch.Generator(device="cuda").manual_seed(7)
    M, hidden, E, k = 9, 2688, 128, 6
    x = torch.randn(M, hidden, generator=g, device="cuda").to(torch.bfloat16)
    W = torch.randn(E, hidden, generator=g, device="cuda") * 0.02
    b = torch.randn(E, generator=g, device="cuda") * 0.05
    idx, w = VN.moe_route(x, W, b, k, True, 2.5)
    ridx, rw, biased = N.moe_route(_bf16(x), W.double().cpu().numpy(), b.double().cpu().numpy(), k, True, 2.5)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    for m in range(M):
        srt = np.sort(biased[m])[::-1]
        if srt[k - 1] - srt[k] > 1e-5:
            assert set(idx[m]) == set(ridx[m]), m
            got = dict(zip(idx[m].tolist(), w[m].tolist()))
            assert max(abs(got[e] - v) for e, v in zip(ridx[m].tolist(), rw[m].tolist())) <= 1e-5, m


@pytest.mark.parametrize("bits", [4, 0])
def test_moe_experts_match_the_oracle(bits):
    """Routed experts (int4 MLX-affine or dense bf16) and the shared expert as a one-expert call
    accumulated into the same output, against the oracle on the dequantized weights; relative
    error 2e-2 of the output's scale."""
    import torch

    from oracle import affine as A
    from vella_b200 import nemotron as VN
    rng = np.random.default_rng(5)
    M, hidden, inter, E, k, shared = 9, 256, 192, 8, 3, 128
    x = torch.tensor(rng.standard_normal((M, hidden)), dtype=torch.bfloat16, device="cuda")
    idx = torch.tensor(np.stack([rng.choice(E, k, replace=False) for _ in range(M)]), dtype=torch.int32, device="cuda")
    wts = torch.tensor(rng.random((M, k)), dtype=torch.float32, device="cuda")

    def weights(n_e, n_out, n_in):
        w = (rng.standard_normal((n_e, n_out, n_in)) * 0.05).astype(np.float32)
        if bits == 0:
            wb = torch.tensor(w, dtype=torch.bfloat16)
            return (wb.cuda(), None, None), wb.float().numpy().astype(np.float64)
        qs = [A.quantize(w[e], bits, "bf16") for e in range(n_e)]
        deq = np.stack([A.dequantize(*q, bits, "bf16") for q in qs]).astype(np.float64)
        # raw words as int32 / int16 tensors (torch has few uint32 / uint16 operations), viewed as needed
        t = lambda i, src, dst: torch.tensor(np.stack([q[i] for q in qs]).astype(src).view(dst)).cuda()  # noqa: E731
        return (t(0, np.uint32, np.int32), t(1, np.uint16, np.int16).view(torch.bfloat16),
                t(2, np.uint16, np.int16).view(torch.bfloat16)), deq

    f1, d1 = weights(E, inter, hidden)
    f2, d2 = weights(E, hidden, inter)
    s1, e1 = weights(1, shared, hidden)
    s2, e2 = weights(1, hidden, shared)
    out = VN.moe_experts(x, idx, wts, f1, f2, inter, bits)
    ones_i = torch.zeros(M, 1, dtype=torch.int32, device="cuda")
    ones_w = torch.ones(M, 1, dtype=torch.float32, device="cuda")
    VN.moe_experts(x, ones_i, ones_w, s1, s2, shared, bits, out=out, accumulate=True)
    torch.cuda.synchronize()
    xs = x.float().cpu().numpy().astype(np.float64)
    ref = N.moe_experts(xs, idx.cpu().numpy(), wts.cpu().numpy().astype(np.float64), d1, d2)
    ref += N.moe_experts(xs, np.zeros((M, 1), np.int64), np.ones((M, 1)), e1, e2)
    got = out.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()


def _hybrid_params(c, seed):
    """Oracle parameters (float64) scaled by 1/sqrt(fan-in), rounded to bf16 as the device holds them."""
    import torch
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.tensor(a, dtype=torch.float32).to(torch.bfloat16).float().double().numpy()  # noqa: E731
    r = lambda *s, sc=1.0: bf(rng.standard_normal(s) * sc)  # noqa: E731
    lin = lambda n, k: r(n, k, sc=1.0 / np.sqrt(k))  # noqa: E731
    d = c.hidden
    layers = []
    for kind in c.pattern:
        L = {"kind": kind, "norm": 1.0 + r(d, sc=0.1)}
        if kind == "M":
            L.update(in_proj=lin(c.m_inner + c.conv_dim + c.m_heads, d), out_proj=lin(d, c.m_inner),
                     conv_w=r(c.conv_dim, c.conv_k, sc=0.4), conv_b=r(c.conv_dim, sc=0.1),
                     a_log=rng.standard_normal(c.m_heads) * 0.5, dt_bias=rng.standard_normal(c.m_heads) * 0.5,
                     D=rng.standard_normal(c.m_heads), norm_w=1.0 + r(c.m_inner, sc=0.1))
        elif kind == "*":
            L.update(q=lin(c.heads * c.head_dim, d), k=lin(c.kv_heads * c.head_dim, d),
                     v=lin(c.kv_heads * c.head_dim, d), o=lin(d, c.heads * c.head_dim))
        else:
            L.update(router=rng.standard_normal((c.experts, d)) / np.sqrt(d), bias=rng.standard_normal(c.experts) * 0.1,
                     fc1=r(c.experts, c.moe_inter, d, sc=1.0 / np.sqrt(d)),
                     fc2=r(c.experts, d, c.moe_inter, sc=1.0 / np.sqrt(c.moe_inter)),
                     up=lin(c.shared_inter, d), down=lin(d, c.shared_inter))
        layers.append(L)
    mtp = {"eh": lin(d, 2 * d), "enorm": 1.0 + r(d, sc=0.1), "hnorm": 1.0 + r(d, sc=0.1),
           "attn_norm": 1.0 + r(d, sc=0.1), "moe_norm": 1.0 + r(d, sc=0.1), "final_norm": 1.0 + r(d, sc=0.1),
           "attn": {"q": lin(c.heads * c.head_dim, d), "k": lin(c.kv_heads * c.head_dim, d),
                    "v": lin(c.kv_heads * c.head_dim, d), "o": lin(d, c.heads * c.head_dim)},
           "moe": {"router": rng.standard_normal((c.experts, d)) / np.sqrt(d),
                   "bias": rng.standard_normal(c.experts) * 0.1,
                   "fc1": r(c.experts, c.moe_inter, d, sc=1.0 / np.sqrt(d)),
                   "fc2": r(c.experts, d, c.moe_inter, sc=1.0 / np.sqrt(c.moe_inter)),
                   "up": lin(c.shared_inter, d), "down": lin(d, c.shared_inter)}}
    return {"embed": r(c.vocab, d), "layers": layers, "norm_f": 1.0 + r(d, sc=0.1), "lm_head": lin(c.vocab, d),
            "mtp": mtp}


def _upload(model, P, c):
    import torch

    class _Dev:
        def __init__(self, ptr, nbytes):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3}

    def put(name, layer, arr, dtype=torch.bfloat16):
        ptr, nbytes = model.tensor(name, layer)
        t = torch.tensor(np.ascontiguousarray(arr), dtype=torch.float32).to(dtype).cuda().view(torch.uint8).reshape(-1)
        assert t.numel() == nbytes, (name, layer, t.numel(), nbytes)
        torch.as_tensor(_Dev(ptr, nbytes), device="cuda").copy_(t)

    put("embed", -1, P["embed"]); put("norm_f", -1, P["norm_f"]); put("lm_head.w", -1, P["lm_head"])
    for l, L in enumerate(P["layers"]):
        put("norm", l, L["norm"])
        if L["kind"] == "M":
            put("in_proj.w", l, L["in_proj"]); put("out_proj.w", l, L["out_proj"])
            put("conv_w", l, L["conv_w"]); put("conv_b", l, L["conv_b"]); put("gnorm", l, L["norm_w"])
            for n, key in (("a_log", "a_log"), ("dt_bias", "dt_bias"), ("D", "D")):
                put(n, l, L[key], torch.float32)
        elif L["kind"] == "*":
            put("qkv.w", l, np.concatenate([L["q"], L["k"], L["v"]])); put("o.w", l, L["o"])
        else:
            put("router", l, L["router"], torch.float32); put("router_bias", l, L["bias"], torch.float32)
            put("fc1.w", l, L["fc1"]); put("fc2.w", l, L["fc2"])
            put("shared_up.w", l, L["up"]); put("shared_down.w", l, L["down"])
    if getattr(model.cfg, "mtp", False):
        T = P["mtp"]
        for n, key in (("enorm", "enorm"), ("hnorm", "hnorm"), ("attn_norm", "attn_norm"), ("moe_norm", "moe_norm"),
                       ("final_norm", "final_norm")):
            put("mtp." + n, -1, T[key])
        put("mtp.eh_proj.w", -1, T["eh"])
        put("mtp.qkv.w", -1, np.concatenate([T["attn"]["q"], T["attn"]["k"], T["attn"]["v"]]))
        put("mtp.o.w", -1, T["attn"]["o"])
        put("mtp.router", -1, T["moe"]["router"], torch.float32)
        put("mtp.router_bias", -1, T["moe"]["bias"], torch.float32)
        put("mtp.fc1.w", -1, T["moe"]["fc1"]); put("mtp.fc2.w", -1, T["moe"]["fc2"])
        put("mtp.shared_up.w", -1, T["moe"]["up"]); put("mtp.shared_down.w", -1, T["moe"]["down"])
    torch.cuda.synchronize()


def test_backbone_matches_the_oracle_and_rolls_back():
    """A dense bf16 Nemotron-H backbone ("M*EM*E") on the device against the oracle's float64
    hybrid model: prefix logits within 3e-2 of the logit scale; every greedy token within that
    margin of the oracle's argmax along the device's own sequence; and a verify pass undone by
    restoring the Mamba states then run again gives the same tokens and logits, bit for bit."""
    import torch

    from vella_b200 import nemotron as VN
    cfg = VN.NHConfig(vocab=512, hidden=256, heads=4, kv_heads=2, head_dim=64, m_heads=8, m_head_dim=32,
                      state_dim=64, groups=2, moe_inter=128, shared_inter=128, experts=8, top_k=2,
                      pattern="M*EM*E", routed_scaling=1.5, max_seq=64, max_rows=16)
    oc = N.HybridConfig(vocab=512, hidden=256, heads=4, kv_heads=2, head_dim=64, m_heads=8, m_head_dim=32, state=64,
                        conv_k=4, groups=2, moe_inter=128, shared_inter=128, experts=8, top_k=2, norm_topk=True,
                        scaling=1.5, pattern="M*EM*E")
    P = _hybrid_params(oc, 0)
    m = VN.NHModel(cfg)
    _upload(m, P, oc)
    emb = torch.tensor(np.random.default_rng(1).standard_normal((8, 256)), dtype=torch.bfloat16, device="cuda")
    logits = torch.empty(1, 512, dtype=torch.bfloat16, device="cuda")
    first = m.forward(embeds=emb, pos=0, logits_rows=1, logits_out=logits)[0]
    cache = N.make_cache(oc)
    post = N.backbone(oc, P, emb.float().cpu().numpy().astype(np.float64), cache)
    ref = post[-1] @ P["lm_head"].T
    got = logits.float().cpu().numpy()[0]
    tol = 3e-2 * np.abs(ref).max()
    assert np.abs(got - ref).max() <= tol
    toks = [first]
    for t in range(1, 10):
        toks.append(m.forward(tokens=[toks[-1]], pos=7 + t, logits_rows=1)[0])
    # the oracle along the device's sequence
    row = ref
    for t in range(10):
        assert row[toks[t]] >= row.max() - tol, t
        if t < 9:
            row = N.backbone(oc, P, P["embed"][[toks[t]]], cache)[-1] @ P["lm_head"].T
    # a verify pass of 3 rows, rolled back (Mamba states restored), then run again
    class _Dev:
        def __init__(self, ptr, nbytes):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3}

    states = [m.tensor(n, l) for l, k in enumerate(oc.pattern) if k == "M" for n in ("conv_state", "ssm_state")]
    saved = [torch.as_tensor(_Dev(ptr, nb), device="cuda").clone() for ptr, nb in states]
    lg1 = torch.empty(3, 512, dtype=torch.bfloat16, device="cuda")
    a1 = m.forward(tokens=[5, 6, 7], pos=17, logits_rows=3, logits_out=lg1)
    for (ptr, nb), buf in zip(states, saved):
        torch.as_tensor(_Dev(ptr, nb), device="cuda").copy_(buf)
    torch.cuda.synchronize()
    lg2 = torch.empty(3, 512, dtype=torch.bfloat16, device="cuda")
    a2 = m.forward(tokens=[5, 6, 7], pos=17, logits_rows=3, logits_out=lg2)
    assert a1 == a2 and torch.equal(lg1, lg2)
    m.close()


def test_mtp_head_and_draft_and_verify_on_the_device():
    """The MTP head's output x matches the oracle's NTMTP within 3e-2 of its scale, and the
    device decodeMTP loop (snapshot / restore of the Mamba states, attention rows overwritten,
    the MTP cache trimmed) emits exactly the device's greedy tokens, with both the
    full-acceptance and the rollback branch taken."""
    import torch

    from vella_b200 import nemotron as VN
    # a 4-token vocabulary and parameter seed 8: on the oracle these decodes accept every draft
    # in 18 passes, reject in the others, and one of them stops at a repetition loop
    kw = dict(vocab=4, hidden=256, heads=4, kv_heads=2, head_dim=64, m_heads=8, m_head_dim=32, groups=2,
              moe_inter=128, shared_inter=128, experts=8, top_k=2)
    cfg = VN.NHConfig(state_dim=64, pattern="M*EM*E", routed_scaling=1.5, max_seq=160, max_rows=16, mtp=True, **kw)
    oc = N.HybridConfig(state=64, conv_k=4, norm_topk=True, scaling=1.5, pattern="M*EM*E", **kw)
    P = _hybrid_params(oc, 8)
    m = VN.NHModel(cfg)
    _upload(m, P, oc)
    # the head alone on 4 (next embedding, hidden) pairs
    rng = np.random.default_rng(4)
    e = torch.tensor(rng.standard_normal((4, 256)), dtype=torch.bfloat16, device="cuda")
    h = torch.tensor(rng.standard_normal((4, 256)), dtype=torch.bfloat16, device="cuda")
    x = torch.empty(4, 256, dtype=torch.bfloat16, device="cuda")
    m.mtp_forward(h, 0, next_embeds=e, x_out=x)
    ref, _ = N.mtp_forward(oc, P, e.float().cpu().numpy().astype(np.float64),
                           h.float().cpu().numpy().astype(np.float64), N.KV())
    assert np.abs(x.float().cpu().numpy() - ref).max() <= 3e-2 * np.abs(ref).max()
    seen = set()
    for seed in range(3):
        emb = torch.tensor(np.random.default_rng(10 + seed).standard_normal((20, 256)), dtype=torch.bfloat16,
                           device="cuda")
        want = VN.decode_greedy(m, emb, 40)
        looped = m.decode_looped
        for depth in (2, 3):
            got, hist = VN.decode_mtp(m, emb, 40, depth)
            if looped and len(got) == 40 and len(want) < 40:
                # the reference's decodeMTP returns at maxTokens before its loop check
                # (NemotronTranscribeModel.swift:389-390), decodeGreedy checks every token (:285):
                # a loop completed by the 40th token is cut by greedy only
                assert D.loop_cut(got) == (want, True) and not m.decode_looped, (seed, depth)
            else:
                assert got == want and m.decode_looped == looped, (seed, depth)
            seen |= {a == depth for a in hist}
    assert seen == {True, False}
    m.close()


def test_nemo_checkpoint_loads_into_the_backbone(tmp_path):
    """A NeMo-layout checkpoint loaded into a dense bf16 handle: the experts transposed from
    [E][in][out], q|k|v stacked, the conv weight and router as stored (bf16 / fp32); a forward
    runs; an int4 handle derives its codes from the same float checkpoint."""
    import torch

    from tests.test_checkpoint import nemo_tensors, small_nh_cfg, write_safetensors
    from vella_b200 import checkpoint as C
    c = small_nh_cfg()
    t = nemo_tensors(c)
    p = tmp_path / "nh.safetensors"
    write_safetensors(p, t)
    m = C.load_nh([p], c)

    class _Dev:
        def __init__(self, ptr, nbytes):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3}

    def get(name, layer, dt=torch.bfloat16):
        ptr, nb = m.tensor(name, layer)
        return torch.as_tensor(_Dev(ptr, nb), device="cuda").view(dt).float().cpu().numpy()

    bf = lambda a: torch.tensor(np.asarray(a, np.float32)).to(torch.bfloat16).float().numpy()  # noqa: E731
    up = t["llm.model.layers.2.mixer.experts.gate_and_up_projs"]
    assert np.array_equal(get("fc1.w", 2).reshape(c.experts, c.moe_inter, c.hidden), bf(up.transpose(0, 2, 1)))
    qkv = np.concatenate([t[f"llm.model.layers.1.mixer.{n}_proj.weight"] for n in "qkv"])
    assert np.array_equal(get("qkv.w", 1).reshape(qkv.shape), bf(qkv))
    conv = t["llm.model.layers.0.mixer.conv1d.weight"]
    assert np.array_equal(get("conv_w", 0).reshape(conv.shape[0], -1), bf(conv.reshape(conv.shape[0], -1)))
    assert np.array_equal(get("router", 2, torch.float32), t["llm.model.layers.2.mixer.gate.weight"].astype(np.float32).reshape(-1))
    assert np.array_equal(get("mtp.final_norm", -1), bf(t["llm.mtp.layers.1.final_layernorm.weight"]))
    assert len(m.forward(tokens=[1, 2, 3], pos=0, logits_rows=3)) == 3
    m.close()
    m4 = C.load_nh([p], small_nh_cfg(bits=4))
    assert len(m4.forward(tokens=[1, 2, 3], pos=0, logits_rows=1)) == 1
    m4.close()
