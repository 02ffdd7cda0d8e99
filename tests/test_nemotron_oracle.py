"""The Mamba-2 mixer oracle against itself and the reference's forms (CPU only): the chunked
causal conv equals token-by-token steps, the sequential scan equals the reference's SSD chunk
form with a carried state, one-token steps equal a chunk, and the gated norm normalises
per group."""
import numpy as np

from oracle import nemotron as N


def _rand(rng, *shape, scale=1.0):
    return rng.standard_normal(shape) * scale


def test_conv_chunk_equals_steps():
    rng = np.random.default_rng(0)
    C, K, T = 24, 4, 7
    w, b = _rand(rng, C, K), _rand(rng, C)
    x, st = _rand(rng, T, C), _rand(rng, K - 1, C)
    out, st_chunk = N.conv_step(x, w, b, st)
    s = st.copy()
    for t in range(T):
        o, s = N.conv_step(x[t:t + 1], w, b, s)
        assert np.allclose(o[0], out[t])
    assert np.allclose(s, st_chunk) and np.allclose(st_chunk, x[-(K - 1):])


def test_scan_equals_ssd_with_a_carried_state():
    rng = np.random.default_rng(1)
    T, H, Dh, G, Ds = 9, 8, 6, 2, 16
    x = _rand(rng, T, H, Dh)
    B, Cm = _rand(rng, T, G, Ds), _rand(rng, T, G, Ds)
    dt = N.compute_dt(_rand(rng, T, H), _rand(rng, H), 1e-3, 10.0)
    a_log, D = _rand(rng, H, scale=0.5), _rand(rng, H)
    st0 = _rand(rng, H, Dh, Ds)
    y1, s1 = N.ssm_scan(x, B, Cm, dt, a_log, D, st0)
    y2, s2 = N.ssm_ssd(x, B, Cm, dt, a_log, D, st0)
    assert np.allclose(y1, y2, rtol=1e-10, atol=1e-10) and np.allclose(s1, s2, rtol=1e-10, atol=1e-10)
    # one token at a time (the step kernel) gives the same as the chunk
    s = st0
    for t in range(T):
        y, s = N.ssm_scan(x[t:t + 1], B[t:t + 1], Cm[t:t + 1], dt[t:t + 1], a_log, D, s)
        assert np.allclose(y[0], y1[t])
    assert np.allclose(s, s1)


def test_dt_is_clipped_softplus():
    dt = N.compute_dt(np.array([[-50.0, 0.0, 50.0]]), np.zeros(3), 0.01, 5.0)
    assert np.allclose(dt, [[0.01, np.log(2.0), 5.0]])


def test_gated_norm_normalises_each_group():
    rng = np.random.default_rng(2)
    y, g = _rand(rng, 3, 32), _rand(rng, 3, 32)
    out = N.gated_rmsnorm(y, g, np.ones(32), groups=4, eps=1e-12).reshape(3, 4, 8)
    assert np.allclose((out * out).mean(axis=-1), 1.0)


def test_mixer_state_carries_across_calls():
    rng = np.random.default_rng(3)
    H, Dh, G, Ds, K = 4, 8, 2, 32, 4
    I = H * Dh
    conv_dim = I + 2 * G * Ds
    args = dict(H=H, Dh=Dh, G=G, Ds=Ds, lo=0.0, hi=float("inf"), eps=1e-5)
    params = (_rand(rng, conv_dim, K, scale=0.3), _rand(rng, conv_dim, scale=0.1), _rand(rng, H, scale=0.3),
              _rand(rng, H, scale=0.3), _rand(rng, H), 1.0 + _rand(rng, I, scale=0.1))
    z = _rand(rng, 6, I + conv_dim + H)
    cs0, ss0 = np.zeros((K - 1, conv_dim)), np.zeros((H, Dh, Ds))
    full, cs_f, ss_f = N.mixer(z, *params, cs0, ss0, **args)
    a, cs, ss = N.mixer(z[:4], *params, cs0, ss0, **args)
    b, cs, ss = N.mixer(z[4:], *params, cs, ss, **args)
    assert np.allclose(np.concatenate([a, b]), full) and np.allclose(ss, ss_f) and np.allclose(cs, cs_f)


def test_moe_route_properties():
    rng = np.random.default_rng(4)
    M, E, hd, k = 5, 16, 32, 4
    x, W, b = _rand(rng, M, hd), _rand(rng, E, hd, scale=0.2), _rand(rng, E, scale=0.3)
    idx, w, biased = N.moe_route(x, W, b, k, True, 2.5)
    assert idx.shape == (M, k) and np.allclose(w.sum(axis=1), 2.5)
    for m in range(M):
        assert set(idx[m]) == set(np.argsort(-biased[m], kind="stable")[:k])
        assert all(biased[m, idx[m, j]] >= biased[m, idx[m, j + 1]] for j in range(k - 1))
    # the weights are the unbiased sigmoid scores
    idx, w, _ = N.moe_route(x, W, b, k, False, 1.0)
    p = 1.0 / (1.0 + np.exp(-(x @ W.T)))
    assert np.allclose(w, np.take_along_axis(p, idx, axis=1))


def test_mtp_draft_and_verify_equals_greedy():
    """The reference's MTP loop with Mamba snapshot/restore and attention trims emits exactly
    the greedy tokens; both the full-acceptance and the rollback branches run."""
    c = N.HybridConfig()
    seen = set()
    for seed in range(4):
        P = N.random_hybrid(c, seed)
        emb = np.random.default_rng(100 + seed).standard_normal((7, c.hidden))
        want = N.decode_greedy(c, P, emb, 24)
        for depth in (2, 3):
            got, hist = N.decode_mtp(c, P, emb, 24, depth)
            assert got == want, (seed, depth)
            seen |= {a == depth for a in hist}
    assert seen == {True, False}


class _OracleNH:
    """The device handle's interface (forward / mtp_forward with positional caches, Mamba state
    views, embedding rows) over the float64 oracle, to run the library's host decode loops on
    the CPU."""

    class _State:
        def __init__(self, owner, layer, key):
            self.owner, self.layer, self.key = owner, layer, key

        def clone(self):
            return self.owner.cache[self.layer][self.key].copy()

        def copy_(self, arr):
            self.owner.cache[self.layer][self.key] = arr.copy()

        def zero_(self):
            self.owner.cache[self.layer][self.key] = np.zeros_like(self.owner.cache[self.layer][self.key])

    def __init__(self, c, P, max_rows=16):
        import types
        self.c, self.P = c, P
        self.cfg = types.SimpleNamespace(max_rows=max_rows, hidden=c.hidden, pattern=c.pattern)
        self.reset()

    def reset(self):
        self.cache, self.mkv = N.make_cache(self.c), N.KV()

    def mamba_states(self):
        return [self._State(self, l, k) for l, kind in enumerate(self.c.pattern) if kind == "M"
                for k in ("conv", "state")]

    def embedding_rows(self, tokens):
        import torch
        return torch.tensor(self.P["embed"][list(tokens)])

    @staticmethod
    def _at(kv, pos):  # a positional cache: rows from `pos` on are overwritten
        if kv.k is not None:
            kv.trim(kv.k.shape[0] - pos)

    def _rows(self, n, what):  # the device handle's row limit (vella_nh_forward / vella_nh_mtp_forward)
        if not 1 <= n <= self.cfg.max_rows:
            raise ValueError(f"{what}: {n} rows (max_rows {self.cfg.max_rows})")

    def forward(self, tokens=None, embeds=None, pos=0, logits_rows=1, logits_out=None, hidden_out=None):
        x = self.P["embed"][list(tokens)] if tokens is not None else embeds.numpy().astype(np.float64)
        self._rows(x.shape[0], "forward")
        for lc in self.cache:
            if isinstance(lc, N.KV):
                self._at(lc, pos)
        post = N.backbone(self.c, self.P, x, self.cache)
        if hidden_out is not None:
            hidden_out.copy_(__import__("torch").tensor(post))
        return list(N.head(self.P, post[post.shape[0] - logits_rows:]))

    def mtp_forward(self, hidden, pos, next_tokens=None, next_embeds=None, logits_rows=1, x_out=None):
        e = self.P["embed"][list(next_tokens)] if next_tokens is not None else next_embeds.numpy().astype(np.float64)
        self._rows(e.shape[0], "mtp_forward")
        self._at(self.mkv, pos)
        x, xo = N.mtp_forward(self.c, self.P, e, hidden.numpy().astype(np.float64), self.mkv)
        if x_out is not None:
            x_out.copy_(__import__("torch").tensor(x))
        return list(N.head(self.P, xo[xo.shape[0] - logits_rows:]))


def test_device_decode_loops_follow_the_reference_on_the_oracle():
    """The library's host loops (vella_b200.nemotron decode_greedy / decode_mtp: prefix chunks of
    max_rows, positional caches, the MTP cache trimmed each pass, Mamba states restored from a
    snapshot) over an oracle-backed handle give the oracle's own greedy tokens."""
    import torch

    from vella_b200 import nemotron as VN
    c = N.HybridConfig()
    for seed in range(3):
        P = N.random_hybrid(c, seed)
        emb = np.random.default_rng(200 + seed).standard_normal((21, c.hidden))
        want = N.decode_greedy(c, P, emb, 24)
        fake = _OracleNH(c, P, max_rows=8)
        assert VN.decode_greedy(fake, torch.tensor(emb), 24) == want
        for depth in (2, 3):
            got, hist = VN.decode_mtp(fake, torch.tensor(emb), 24, depth)
            assert got == want, (seed, depth)


def test_mtp_loop_commits_the_prefix_when_the_feed_would_pass_max_rows():
    """With a large vocabulary the random MTP head's drafts almost never match, so the re-fed
    prefix grows by one token every pass; with max_rows 8 the loop must commit it (forward it
    again after the Mamba restore) long before 40 tokens, and still emit the oracle's greedy
    tokens.  The oracle-backed handle rejects feeds above max_rows, as the device does."""
    import dataclasses

    import torch

    from vella_b200 import nemotron as VN
    c = dataclasses.replace(N.HybridConfig(), vocab=4000)
    P = N.random_hybrid(c, 7)
    emb = np.random.default_rng(7).standard_normal((11, c.hidden))
    want = N.decode_greedy(c, P, emb, 44)
    assert len(want) == 44
    for depth in (2, 3):
        fake = _OracleNH(c, P, max_rows=8)
        got, hist = VN.decode_mtp(fake, torch.tensor(emb), 44, depth)
        assert got == want, depth
        assert sum(1 for a in hist if a < depth) >= 8 - depth  # enough rejections to need the commit
        assert not fake.decode_looped


class _ScriptedNH(_OracleNH):
    """A handle whose greedy token at every absolute position comes from a script (the model
    ignores its inputs), so repetition loops can be planted.  Hidden rows carry their absolute
    position; the MTP head predicts the script's token two positions on with probability 1/2,
    else a wrong token, so both acceptance branches run."""

    def __init__(self, script, T, max_rows=8, seed=0):
        import types
        self.script, self.T, self.rng = list(script), T, np.random.default_rng(seed)
        self.cfg = types.SimpleNamespace(max_rows=max_rows, hidden=4, pattern="M")
        self.state = [np.zeros(1), np.zeros(1)]

    def reset(self):
        pass

    def mamba_states(self):
        owner = self

        class _S:
            def __init__(self, i):
                self.i = i

            def clone(self):
                return owner.state[self.i].copy()

            def copy_(self, a):
                owner.state[self.i] = a.copy()

            def zero_(self):
                owner.state[self.i] = np.zeros(1)
        return [_S(0), _S(1)]

    def embedding_rows(self, tokens):
        import torch
        return torch.zeros(len(tokens), 4, dtype=torch.float64)

    def _tok(self, p):  # the token at absolute position p (p >= T)
        return self.script[p - self.T] if 0 <= p - self.T < len(self.script) else 0

    def forward(self, tokens=None, embeds=None, pos=0, logits_rows=1, logits_out=None, hidden_out=None):
        import torch
        n = len(tokens) if tokens is not None else embeds.shape[0]
        self._rows(n, "forward")
        if hidden_out is not None:
            h = torch.zeros(n, 4, dtype=hidden_out.dtype)
            h[:, 0] = torch.arange(pos, pos + n, dtype=hidden_out.dtype)
            hidden_out.copy_(h)
        return [self._tok(p + 1) for p in range(pos + n - logits_rows, pos + n)]

    def mtp_forward(self, hidden, pos, next_tokens=None, next_embeds=None, logits_rows=1, x_out=None):
        import torch
        n = hidden.shape[0]
        self._rows(n, "mtp_forward")
        p = [int(v) for v in hidden[:, 0].tolist()]
        if x_out is not None:
            x = torch.zeros(n, 4, dtype=x_out.dtype)
            x[:, 0] = torch.tensor([q + 1 for q in p], dtype=x_out.dtype)
            x_out.copy_(x)
        good = [self._tok(q + 2) for q in p[n - logits_rows:]]
        return [g if self.rng.random() < 0.5 else g + 1 for g in good]


def test_decode_loops_stop_at_a_planted_repetition_loop():
    """A block repeated 30 times after a few distinct tokens: greedy and MTP decoding stop where
    the reference's endsInLoop stops (checked every 4 tokens once there are 20), keep one copy
    of the block and set decode_looped; a script without a loop runs to max_tokens."""
    import torch

    from oracle import decoder as D
    from vella_b200 import nemotron as VN
    T = 6
    emb = torch.zeros(T, 4, dtype=torch.float64)
    for script in ([5, 6, 7, 8, 9] + [21, 22, 23] * 30, [3, 4] + [11] * 40, list(range(100, 190))):
        want, looped = [], False
        for tok in script[:80]:
            want.append(tok)
            if D.ends_in_loop(want):
                looped = True
                break
        h = _ScriptedNH(script, T)
        assert VN.decode_greedy(h, emb, 80) == want and h.decode_looped == looped, script[:8]
        for depth in (2, 3):
            h = _ScriptedNH(script, T, seed=depth)
            got, _ = VN.decode_mtp(h, emb, 80, depth)
            assert got == want and h.decode_looped == looped, (script[:8], depth)
    # the oracle's own loops stop the same way
    c = N.HybridConfig()
    P = N.random_hybrid(c, 1)
    P["lm_head"] = np.zeros_like(P["lm_head"])  # every argmax is token 0: a loop of one token
    emb2 = np.random.default_rng(1).standard_normal((5, c.hidden))
    info = {}
    assert N.decode_greedy(c, P, emb2, 64, info=info) == [0] and info["looped"]
    got, _ = N.decode_mtp(c, P, emb2, 64, 2, info=info)
    assert got == [0] and info["looped"]
