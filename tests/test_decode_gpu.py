"""Parity of the resident decoder and the draft-and-verify loop (through the C ABI) with
the CPU oracle, on small seeded models.

Bars: logits max |error| <= 2e-2 against the oracle (teacher forced); greedy tokens equal
the oracle's argmax wherever its top-2 margin exceeds that tolerance; draft-and-verify
emits exactly the greedy tokens (bit-exact, any K, any acceptance rate); the accepted-
length histogram equals the oracle's simulation with the same Philox proposals.
"""
import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle import decoder as D

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


class _Dev:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def download(model, name, layer=-1):
    ptr, nbytes = model.tensor(name, layer)
    return torch.as_tensor(_Dev(ptr, nbytes), device="cuda").cpu().numpy()


def upload(model, name, arr, layer=-1):
    ptr, nbytes = model.tensor(name, layer)
    raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    assert raw.nbytes <= nbytes
    torch.as_tensor(_Dev(ptr, raw.nbytes), device="cuda").copy_(torch.from_numpy(raw.copy()))


def oracle_weights(model, cfg: D.Config):
    d, V = cfg.d_model, cfg.vocab
    f = lambda a: A.bf16_from_bits(a.view(np.uint16))  # noqa: E731

    def lin(name, layer, n, k):
        w = download(model, f"{name}.w", layer)
        if cfg.bits:
            return {"w": w.view(np.uint32).reshape(n, k * cfg.bits // 32),
                    "s": download(model, f"{name}.s", layer).view(np.uint16).reshape(n, k // 64),
                    "b": download(model, f"{name}.b", layer).view(np.uint16).reshape(n, k // 64)}
        return {"w": w.view(np.uint16).reshape(n, k)}

    H, KV, hd, F = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn
    W = {"embed": f(download(model, "embed")).reshape(V, d),
         "final_norm": f(download(model, "final_norm")),
         "lm_head": lin("lm_head", -1, V, d), "layers": []}
    for l in range(cfg.n_layers):
        L = {"attn_norm": f(download(model, "attn_norm", l)), "mlp_norm": f(download(model, "mlp_norm", l)),
             "qkv": lin("qkv", l, (H + 2 * KV) * hd, d), "o": lin("o", l, d, H * hd),
             "gate": lin("gate", l, F, d), "up": lin("up", l, F, d), "down": lin("down", l, d, F)}
        if cfg.qk_norm:
            L["q_norm"] = f(download(model, "q_norm", l))
            L["k_norm"] = f(download(model, "k_norm", l))
        W["layers"].append(L)
    return W


def make(n_layers=2, d=256, H=4, KV=2, hd=64, ffn=512, V=1000, bits=4, qk_norm=False, seed=1, max_seq=512,
         max_prefix=128):
    from vella_b200 import decode as VD
    mc = VD.ModelConfig(n_layers, d, H, KV, hd, ffn, V, bits=bits, qk_norm=qk_norm, max_seq=max_seq,
                        max_prefix=max_prefix)
    m = VD.Model(mc)
    m.init_random(seed, 0.02 if d > 128 else 0.05)
    oc = D.Config(n_layers, d, H, KV, hd, ffn, V, bits=bits, qk_norm=qk_norm)
    return m, oc


def prefix_of(P, d, seed):
    x = np.random.default_rng(seed).standard_normal((P, d)).astype(np.float32)
    return A.bf16_bits(x)


@pytest.fixture(scope="module")
def pair():
    """Target (int4, 2 layers) and draft (dense bf16, 1 layer), same vocabulary."""
    t, tc = make(bits=4, seed=1)
    d, dc = make(n_layers=1, d=128, H=2, KV=1, ffn=256, bits=0, seed=2)
    return t, tc, d, dc


@pytest.mark.parametrize("bits,qk", [(4, False), (8, False), (0, False), (4, True)])
def test_score_matches_oracle(bits, qk):
    m, oc = make(bits=bits, qk_norm=qk, seed=3 + bits)
    W = oracle_weights(m, oc)
    table = D.rope_table(64, oc.head_dim, oc.rope_theta)
    P = 20
    pre = prefix_of(P, oc.d_model, 5)
    toks = list(np.random.default_rng(6).integers(0, oc.vocab, 30))
    got = A.bf16_from_bits(m.score(pre, toks))
    ref = D.score(oc, W, A.bf16_from_bits(pre), toks, table)
    assert got.shape == ref.shape == (30, oc.vocab)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= LOGIT_TOL, err


@pytest.mark.parametrize("H,KV,hd", [(4, 2, 64), (8, 1, 64), (4, 1, 128)])
def test_long_context_score_matches_oracle(H, KV, hd):
    """700 positions: every CTA of an attention cluster owns several 64-key chunks."""
    m, oc = make(bits=4, H=H, KV=KV, hd=hd, seed=9, max_seq=1024)
    W = oracle_weights(m, oc)
    P, T = 100, 600
    pre = prefix_of(P, oc.d_model, 7)
    toks = list(np.random.default_rng(8).integers(0, oc.vocab, T))
    got = A.bf16_from_bits(m.score(pre, toks))
    ref = D.score(oc, W, A.bf16_from_bits(pre), toks, D.rope_table(P + T, oc.head_dim, oc.rope_theta))
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= LOGIT_TOL, err
    m.close()


def test_long_context_draft_and_verify_is_bit_exact_greedy():
    """A 600-position prefix: the verify rows' attention spans 10+ chunks per kv head."""
    from vella_b200 import decode as VD
    t, tc = make(bits=4, seed=21, max_seq=1024, max_prefix=640)
    d, dc = make(n_layers=1, d=128, H=2, KV=1, ffn=256, bits=0, seed=22, max_seq=1024, max_prefix=640)
    P = 600
    pre_t, pre_d = prefix_of(P, tc.d_model, 23), prefix_of(P, dc.d_model, 24)
    ref, sd = greedy_tokens(t, d, P, pre_t, pre_d, 40)
    sd.close()
    sd = VD.SpecDecoder(t, d, k=4, mode=VD.DRAFT_ORACLE, oracle_p=0.5, seed=3)
    sd.set_prefix(pre_t, pre_d, P)
    sd.set_reference(ref)
    assert sd.decode_mtp(40).tokens == ref
    sd.close()
    for x in (t, d):
        x.close()


def greedy_tokens(t, d, P, pre_t, pre_d, n, **kw):
    from vella_b200 import decode as VD
    sd = VD.SpecDecoder(t, d, **kw)
    sd.set_prefix(pre_t, pre_d, P)
    return sd.decode_greedy(n).tokens, sd


def test_greedy_matches_oracle_teacher_forced(pair):
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    toks, _ = greedy_tokens(t, d, P, pre_t, pre_d, 48)
    assert len(toks) == 48
    W = oracle_weights(t, tc)
    logits = D.score(tc, W, A.bf16_from_bits(pre_t), toks, D.rope_table(P + 64, tc.head_dim, tc.rope_theta))
    for j, tok in enumerate(toks):
        row = logits[j]
        best = int(np.argmax(row))
        assert tok == best or row[best] - row[tok] <= LOGIT_TOL, (j, tok, best, row[best] - row[tok])


@pytest.mark.parametrize("k", [1, 2, 4, 8])
@pytest.mark.parametrize("p", [0.0, 0.5, 0.9, 1.0])
def test_draft_and_verify_is_bit_exact_greedy(pair, k, p):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P, N = 24, 64
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    ref, _ = greedy_tokens(t, d, P, pre_t, pre_d, N + 16)
    sd = VD.SpecDecoder(t, d, k=k, mode=VD.DRAFT_ORACLE, oracle_p=p, seed=99)
    sd.set_prefix(pre_t, pre_d, P)
    sd.set_reference(ref)
    res = sd.decode_mtp(N)
    assert res.tokens == ref[:N]
    # pass-by-pass acceptance replayed by the oracle with the same Philox proposals
    def propose(out, pi):
        return [D.oracle_proposal(99, pi, i, ref[len(out) + i] if len(out) + i < len(ref) else None, p, tc.vocab)
                for i in range(k)]

    def verify(out, drafts):
        return [ref[len(out) + j] for j in range(k + 1)]

    toks, _, hist = D.draft_and_verify(verify, propose, ref[0], N, k)
    assert toks == ref[:N]
    expect = np.bincount(np.asarray(hist, dtype=np.int64), minlength=16)[:16]
    got = np.asarray(res.stats["accepted"])  # passes by number of accepted drafts
    assert np.array_equal(got[: k + 1], expect[: k + 1]), (got, expect)
    assert res.stats["passes"] == len(hist)


def test_model_draft_and_self_speculation(pair):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    ref, _ = greedy_tokens(t, d, P, pre_t, pre_d, 40)
    # a real (random) draft: output still equals greedy
    sd = VD.SpecDecoder(t, d, k=4, mode=VD.DRAFT_MODEL)
    sd.set_prefix(pre_t, pre_d, P)
    assert sd.decode_mtp(40).tokens == ref
    # draft = a second copy of the target: every draft is accepted
    t2, _ = make(bits=4, seed=1)
    sd2 = VD.SpecDecoder(t, t2, k=4, mode=VD.DRAFT_MODEL)
    sd2.set_prefix(pre_t, pre_t, P)
    res = sd2.decode_mtp(40)
    assert res.tokens == ref
    assert res.stats["accepted"][4] == res.stats["passes"] > 0


def test_graph_replay_equals_eager(pair):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 13), prefix_of(P, dc.d_model, 14)
    outs = []
    for graphs in (False, True):
        sd = VD.SpecDecoder(t, d, k=3, mode=VD.DRAFT_ORACLE, oracle_p=0.6, seed=5, use_graphs=graphs)
        sd.set_prefix(pre_t, pre_d, P)
        g = sd.decode_greedy(50).tokens
        sd.set_reference(g)
        outs.append((g, sd.decode_mtp(50).tokens))
    assert outs[0] == outs[1] and outs[0][0] == outs[0][1]


@pytest.mark.parametrize("fault", [1, 2])  # FAULT_THROW, FAULT_NONFINITE
def test_runtime_failure_falls_back_to_greedy_sticky(pair, fault):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    ref, _ = greedy_tokens(t, d, P, pre_t, pre_d, 30)
    sd = VD.SpecDecoder(t, d, k=4, mode=VD.DRAFT_MODEL)
    sd.set_prefix(pre_t, pre_d, P)
    sd.set_fault(fault)
    res = sd.decode(30)
    assert res.tokens == ref and res.flags & VD.FLAG_FELL_BACK
    st = sd.stats()
    assert st["fallbacks"] == 1 and st["draft_disabled"]
    sd.set_fault(VD.FAULT_NONE)
    res2 = sd.decode(30)  # sticky: plain greedy until reset, no second fallback
    assert res2.tokens == ref and not res2.flags & VD.FLAG_FELL_BACK and sd.stats()["fallbacks"] == 1
    sd.reset()
    res3 = sd.decode(29)
    assert res3.tokens == ref[:29] and sd.stats()["passes"] > 0 and not sd.stats()["draft_disabled"]


def test_eos_stops_and_is_not_emitted(pair):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    ref, _ = greedy_tokens(t, d, P, pre_t, pre_d, 40)
    stop = ref[17]
    first = ref.index(stop)
    for mode in (VD.DECODE_GREEDY, VD.DECODE_SPEC):
        sd = VD.SpecDecoder(t, d, k=4, mode=VD.DRAFT_MODEL, eos=[stop])
        sd.set_prefix(pre_t, pre_d, P)
        assert sd.decode(40, mode).tokens == ref[:first]


def test_runaway_retry_when_max_tokens_reached(pair):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    sd = VD.SpecDecoder(t, d, k=2, mode=VD.DRAFT_MODEL)
    sd.set_prefix(pre_t, pre_d, P)
    res = sd.decode(16)  # AUTO: reaching max_tokens counts as a runaway -> greedy retry
    assert res.flags & VD.FLAG_RUNAWAY_RETRY and sd.stats()["runaway_retries"] == 1 and len(res.tokens) == 16


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_device_quantizer_matches_oracle_bitwise(bits, dtype):
    import ctypes
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD  # noqa: F401  (declares vella_quantize)
    rng = np.random.default_rng(bits)
    n, k = 300, 1024
    w = (rng.standard_normal((n, k)) * np.float32(0.02) * (1 + 10 * rng.random((n, 1)))).astype(np.float32)
    w[0, :64] = 0.0          # all-zero group
    w[1, :64] = -0.5         # constant negative group
    wd = torch.from_numpy(w).cuda()
    packed = torch.zeros(n, k * bits // 32, dtype=torch.int32, device="cuda")
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    sc = torch.zeros(n, k // 64, dtype=tdt, device="cuda")
    bi = torch.zeros(n, k // 64, dtype=tdt, device="cuda")
    desc = L.QgemmDesc(0, n, k, bits, 64, L.BF16 if dtype == "bf16" else L.F16, 0)
    L.check(L.lib().vella_quantize(ctypes.byref(desc), 2, wd.data_ptr(), packed.data_ptr(), sc.data_ptr(),
                                   bi.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    p, s, b = A.quantize(w, bits, dtype)
    assert np.array_equal(packed.cpu().numpy().view(np.uint32), p)
    if dtype == "bf16":
        assert np.array_equal(sc.cpu().view(torch.int16).numpy().view(np.uint16), s)
        assert np.array_equal(bi.cpu().view(torch.int16).numpy().view(np.uint16), b)
    else:
        assert np.array_equal(sc.cpu().numpy(), s) and np.array_equal(bi.cpu().numpy(), b)


def _batch_models(S, max_seq=160):
    t, tc = make(bits=4, seed=31, max_seq=max_seq)
    d, dc = make(n_layers=1, d=128, H=2, KV=1, ffn=256, bits=0, seed=32, max_seq=max_seq)
    from vella_b200 import decode as VD
    tb = VD.Model(VD.ModelConfig(2, 256, 4, 2, 64, 512, 1000, bits=4, max_seq=max_seq, max_prefix=128, streams=S))
    tb.init_random(31, 0.02)
    db = VD.Model(VD.ModelConfig(1, 128, 2, 1, 64, 256, 1000, bits=0, max_seq=max_seq, max_prefix=128, streams=S))
    db.init_random(32, 0.05)
    return t, d, tb, db


def test_batched_greedy_equals_single_stream_greedy():
    """Three streams decoded as one batch (3 rows, small-M kernels) give each stream exactly
    the tokens of its own single-stream greedy decode."""
    from vella_b200 import decode as VD
    S, P, n = 3, 24, 32
    t, d, tb, db = _batch_models(S)
    pre_t = np.stack([prefix_of(P, 256, 40 + j) for j in range(S)])
    pre_d = np.stack([prefix_of(P, 128, 50 + j) for j in range(S)])
    sb = VD.SpecDecoder(tb, db, k=4)
    sb.set_prefix(pre_t, pre_d)
    batch = sb.decode_batch(n, VD.DECODE_GREEDY)
    for j in range(S):
        single, sd = greedy_tokens(t, d, P, pre_t[j], pre_d[j], n)
        sd.close()
        assert list(batch[j]) == single, j
    sb.close()
    for m in (t, d, tb, db):
        m.close()


@pytest.mark.parametrize("S,k", [(3, 4), (20, 3), (32, 4)])
def test_batched_spec_equals_batched_greedy(S, k):
    """Draft-and-verify over S streams in one batch emits each stream's greedy tokens bit for
    bit; S=3, K=4 keeps every GEMM on the small-M kernels (15 verify rows), S=20 puts the
    greedy step (20 rows) and the verify (80 rows) on the tensor cores; S=32 verifies 160 rows
    (two token tiles, argmax rows past 128 after 32-row draft launches on the same scratch)."""
    from vella_b200 import decode as VD
    P, n = 20, 40
    _, _, tb, db = _batch_models(S)
    pre_t = np.stack([prefix_of(P, 256, 60 + j) for j in range(S)])
    pre_d = np.stack([prefix_of(P, 128, 70 + j) for j in range(S)])
    sb = VD.SpecDecoder(tb, db, k=k)
    sb.set_prefix(pre_t, pre_d)
    greedy = sb.decode_batch(n, VD.DECODE_GREEDY)
    spec = sb.decode_batch(n, VD.DECODE_SPEC)
    assert np.array_equal(spec, greedy)
    # oracle draft over the batch: same tokens, acceptance follows the oracle rate
    so = VD.SpecDecoder(tb, db, k=k, mode=VD.DRAFT_ORACLE, oracle_p=0.9, seed=5)
    so.set_prefix(pre_t, pre_d)
    so.set_reference(greedy)
    assert np.array_equal(so.decode_batch(n, VD.DECODE_SPEC), greedy)
    st = so.stats()
    assert st["passes"] > 0 and sum(st["accepted"][1:]) > sum(st["accepted"][:1])
    for x in (sb, so, tb, db):
        x.close()


def _chi2(counts, probs, n):
    """Chi-square statistic over cells merged so every expected count is at least 5."""
    order = np.argsort(-probs)
    stat, obs, exp = 0.0, 0.0, 0.0
    cells = 0
    for i in order:
        obs += counts[i]
        exp += probs[i] * n
        if exp >= 5:
            stat += (obs - exp) ** 2 / exp
            obs, exp = 0.0, 0.0
            cells += 1
    if exp > 0:
        stat += (obs - exp) ** 2 / max(exp, 1e-9)
        cells += 1
    return stat, cells


def _softmax(row, T):
    z = (row - row.max()) / T
    e = np.exp(z)
    return e / e.sum()


@pytest.mark.parametrize("spec", [True, False])
def test_sampled_tokens_follow_the_target_distribution(spec):
    """Stochastic acceptance (temperature 1): over 1024 streams with one prefix, the first
    token (drawn after the prefill) and the second (drawn by draft-and-verify with rejections
    against the residual, or by a plain sampling step) follow the target's softmax."""
    from vella_b200 import decode as VD
    S, P, V, T = 1024, 4, 16, 1.0
    cfg = dict(n_layers=1, d_model=64, n_heads=1, n_kv_heads=1, head_dim=64, ffn=64, vocab=V, bits=0,
               max_seq=32, max_prefix=8)
    tb = VD.Model(VD.ModelConfig(**cfg, streams=S))
    tb.init_random(41, 0.5)
    db = VD.Model(VD.ModelConfig(**cfg, streams=S))
    db.init_random(42, 0.5)
    single = VD.Model(VD.ModelConfig(**cfg))
    single.init_random(41, 0.5)
    pre = prefix_of(P, 64, 43)
    sb = VD.SpecDecoder(tb, db, k=2, seed=123, temperature=T)
    sb.set_prefix(np.stack([pre] * S), np.stack([prefix_of(P, 64, 44)] * S))
    toks = sb.decode_batch(3, VD.DECODE_SPEC if spec else VD.DECODE_GREEDY)
    assert toks.min() >= 0 and toks.max() < V
    # exact probabilities from the target's own logits (teacher forced, bf16)
    p1 = _softmax(A.bf16_from_bits(single.score(pre, [0]))[0].astype(np.float64), T)
    p2 = np.zeros(V)
    for t1 in range(V):
        row = A.bf16_from_bits(single.score(pre, [t1, 0]))[1].astype(np.float64)
        p2 += p1[t1] * _softmax(row, T)
    for col, probs in ((0, p1), (1, p2)):
        counts = np.bincount(toks[:, col], minlength=V).astype(np.float64)
        stat, cells = _chi2(counts, probs, S)
        assert stat < 3.0 * cells + 20, (col, stat, cells, counts, probs * S)
    if spec:
        st = sb.stats()
        assert st["passes"] > 0 and st["accepted"][0] > 0  # rejections happened (residual draws)
    # same seed, same tokens; another seed, other tokens
    again = sb.decode_batch(3, VD.DECODE_SPEC if spec else VD.DECODE_GREEDY)
    assert np.array_equal(again, toks)
    sb.close()
    for m in (tb, db, single):
        m.close()


def test_sampled_oracle_draft_runs_and_is_reproducible(pair):
    from vella_b200 import decode as VD
    t, tc, d, dc = pair
    P = 24
    pre_t, pre_d = prefix_of(P, tc.d_model, 11), prefix_of(P, dc.d_model, 12)
    ref, _ = greedy_tokens(t, d, P, pre_t, pre_d, 40)
    outs = []
    for seed in (5, 5, 6):
        sd = VD.SpecDecoder(t, d, k=4, mode=VD.DRAFT_ORACLE, oracle_p=0.7, seed=seed, temperature=0.7)
        sd.set_prefix(pre_t, pre_d, P)
        sd.set_reference(ref)
        outs.append(sd.decode_mtp(40).tokens)
        assert sd.stats()["passes"] > 0
        sd.close()
    assert outs[0] == outs[1] and len(outs[0]) == 40
    assert outs[0] != outs[2]


def _argmax_consistent(single, pre, toks):
    """Each token is the target's argmax (teacher forced) or within the logits tolerance of it."""
    logits = A.bf16_from_bits(single.score(pre, list(toks))).astype(np.float64)
    for j, t in enumerate(toks):
        row = logits[j]
        best = int(np.argmax(row))
        assert t == best or row[best] - row[t] <= LOGIT_TOL, (j, t, best, row[best] - row[t])


@pytest.mark.parametrize("mode", ["oracle", "self"])
def test_tree_greedy_follows_target_argmax(mode):
    """Tree verification (branching 3, 2, 2, 1: 33 draft nodes) with greedy acceptance over 4
    streams: every emitted token is the target's argmax along the emitted sequence, and the
    accepted paths are long (oracle p = 1 or a draft identical to the target)."""
    from vella_b200 import decode as VD
    S, P, n = 4, 20, 40
    cfg_t = dict(n_layers=2, d_model=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=1000, bits=4,
                 max_seq=160, max_prefix=128)
    tb = VD.Model(VD.ModelConfig(**cfg_t, streams=S, rows_per_stream=64))
    tb.init_random(31, 0.02)
    if mode == "self":
        db = VD.Model(VD.ModelConfig(**cfg_t, streams=S))
        db.init_random(31, 0.02)
        dd = 256
    else:
        db = VD.Model(VD.ModelConfig(1, 128, 2, 1, 64, 256, 1000, bits=0, max_seq=160, max_prefix=128, streams=S))
        db.init_random(32, 0.05)
        dd = 128
    single = VD.Model(VD.ModelConfig(**cfg_t))
    single.init_random(31, 0.02)
    pre_t = np.stack([prefix_of(P, 256, 80 + j) for j in range(S)])
    pre_d = np.stack([prefix_of(P, dd, 90 + j) for j in range(S)]) if mode == "oracle" else pre_t
    greedy = VD.SpecDecoder(tb, db, k=4)
    greedy.set_prefix(pre_t, pre_d)
    ref = greedy.decode_batch(n, VD.DECODE_GREEDY)
    greedy.close()
    kw = dict(mode=VD.DRAFT_ORACLE, oracle_p=1.0, seed=3) if mode == "oracle" else dict(mode=VD.DRAFT_MODEL)
    sd = VD.SpecDecoder(tb, db, k=4, tree=(3, 2, 2, 1), **kw)
    sd.set_prefix(pre_t, pre_d)
    if mode == "oracle":
        sd.set_reference(ref)
    toks = sd.decode_batch(n, VD.DECODE_SPEC)
    st = sd.stats()
    for j in range(S):
        _argmax_consistent(single, pre_t[j], toks[j])
    mean_new = sum((i + 1) * c for i, c in enumerate(st["accepted"])) / max(sum(st["accepted"]), 1)
    assert mean_new > 3.0, st["accepted"]  # tree depth 4: up to 5 tokens per pass
    sd.close()
    for m in (tb, db, single):
        m.close()


def test_tree_sampled_tokens_follow_the_target_distribution():
    """Stochastic tree acceptance (branching 3, 2): over 1024 streams with one prefix, the
    second token follows the target's softmax (children tried in order against the running
    residual)."""
    from vella_b200 import decode as VD
    S, P, V, T = 1024, 4, 16, 1.0
    cfg = dict(n_layers=1, d_model=64, n_heads=1, n_kv_heads=1, head_dim=64, ffn=64, vocab=V, bits=0,
               max_seq=32, max_prefix=8)
    tb = VD.Model(VD.ModelConfig(**cfg, streams=S, rows_per_stream=16))
    tb.init_random(41, 0.5)
    db = VD.Model(VD.ModelConfig(**cfg, streams=S))
    db.init_random(42, 0.5)
    single = VD.Model(VD.ModelConfig(**cfg))
    single.init_random(41, 0.5)
    pre = prefix_of(P, 64, 43)
    sb = VD.SpecDecoder(tb, db, k=2, seed=321, temperature=T, tree=(3, 2))
    sb.set_prefix(np.stack([pre] * S), np.stack([prefix_of(P, 64, 44)] * S))
    toks = sb.decode_batch(3, VD.DECODE_SPEC)
    assert toks.min() >= 0 and toks.max() < V
    p1 = _softmax(A.bf16_from_bits(single.score(pre, [0]))[0].astype(np.float64), T)
    p2 = np.zeros(V)
    for t1 in range(V):
        row = A.bf16_from_bits(single.score(pre, [t1, 0]))[1].astype(np.float64)
        p2 += p1[t1] * _softmax(row, T)
    for col, probs in ((0, p1), (1, p2)):
        counts = np.bincount(toks[:, col], minlength=V).astype(np.float64)
        stat, cells = _chi2(counts, probs, S)
        assert stat < 3.0 * cells + 20, (col, stat, cells, counts, probs * S)
    st = sb.stats()
    assert st["passes"] > 0 and st["accepted"][0] > 0
    sb.close()
    for m in (tb, db, single):
        m.close()
