"""Sampled acceptance and tree verification are token-exact against the oracle, given the same
logits rows and the same Philox uniforms.

The decoder runs one pass at a time (vella_spec_step).  After each pass the test reads the
rows the device sampled from -- the target's verify logits (the model's "logits" buffer) and
the draft's kept rows (vella_spec_tensor "draft_rows") -- and replays the pass in the oracle
(oracle/decoder.py: sample_drafts / sampled_accept for a linear draft, tree_children /
tree_accept for a tree), which draws its uniforms from the same Philox counters (pass,
position or node, purpose, stream).  The emitted tokens must be identical; the oracle works in
float64 and the device in float32, so a pass is only excused when one of its decisions sits
within 1e-5 (relative) of its threshold, and such passes must be rare.  This catches what a
distribution test cannot: a wrong counter assignment, a wrong node order, a residual that is
not renormalised, a bonus drawn from the wrong row.
"""
import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle import decoder as D
from tests.test_decode_gpu import prefix_of

pytestmark = pytest.mark.gpu

T, SEED, TIE = 0.7, 0x1234ABCD5678, 1e-5


class _Dev:
    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def _read(ptr_bytes, dtype):
    ptr, nbytes = ptr_bytes
    raw = torch.as_tensor(_Dev(ptr, nbytes), device="cuda").cpu().numpy()
    if dtype == "bf16":
        return A.bf16_from_bits(raw.view(np.uint16)).astype(np.float64)
    return raw.view(dtype)


def _models(target_rows=16, draft_rows=16):
    """Target: 2 int4 layers, d 256, vocab 1000; draft: 1 bf16 layer, d 128.  Larger init scales
    than the other tests give peaked softmaxes, so most draws are far from a bin edge."""
    from vella_b200 import decode as VD
    t = VD.Model(VD.ModelConfig(2, 256, 4, 2, 64, 512, 1000, bits=4, max_seq=256, max_prefix=32,
                                rows_per_stream=target_rows))
    t.init_random(61, 0.08)
    d = VD.Model(VD.ModelConfig(1, 128, 2, 1, 64, 256, 1000, bits=0, max_seq=256, max_prefix=32,
                                rows_per_stream=draft_rows))
    d.init_random(62, 0.1)
    return t, d


@pytest.mark.parametrize("mode", ["model", "oracle", "self"])
def test_linear_sampled_acceptance_is_token_exact(mode):
    """model: the random bf16 draft (rejections, residual draws); oracle: the oracle draft's
    mixture q; self: a draft identical to the target, so every draft is accepted and the bonus
    is drawn from the last verify row."""
    from vella_b200 import decode as VD
    K, P, V, passes = 4, 16, 1000, 30
    t, d = _models()
    pre_t, pre_d = prefix_of(P, 256, 63), prefix_of(P, 128, 64)
    ref = None
    if mode == "self":
        d.close()
        d = VD.Model(VD.ModelConfig(2, 256, 4, 2, 64, 512, 1000, bits=4, max_seq=256, max_prefix=32,
                                    rows_per_stream=16))
        d.init_random(61, 0.08)
        pre_d = pre_t
    if mode == "oracle":
        g = VD.SpecDecoder(t, d, k=K)
        g.set_prefix(pre_t, pre_d, P)
        ref = g.decode_greedy(200).tokens
        g.close()
        sd = VD.SpecDecoder(t, d, k=K, mode=VD.DRAFT_ORACLE, oracle_p=0.6, seed=SEED, temperature=T)
        sd.set_prefix(pre_t, pre_d, P)
        sd.set_reference(ref)
    else:
        sd = VD.SpecDecoder(t, d, k=K, mode=VD.DRAFT_MODEL, seed=SEED, temperature=T)
        sd.set_prefix(pre_t, pre_d, P)
    sd.prefill()
    L = P + 1
    exact = ties = rejections = 0
    for pi in range(passes):
        new = sd.step()
        p_rows = _read(t.tensor("logits"), "bf16").reshape(-1, V)[:K + 1]
        dev_tok = _read(sd.tensor("tokens"), np.int32)
        if mode != "oracle":
            q_rows = _read(sd.tensor("draft_rows"), "bf16").reshape(K, V)
            drafts, m1 = D.sample_drafts(q_rows, T, SEED, pi)
            qs = [D.softmax_t(r, T) for r in q_rows]
        else:
            m1 = np.inf
            ref_at = [ref[L + i - P] if 0 <= L + i - P < len(ref) else None for i in range(K)]
            drafts = [D.oracle_proposal(SEED, pi, i, ref_at[i], 0.6, V) for i in range(K)]
            qs = [D.oracle_draft_q(V, r, 0.6) for r in ref_at]
        a, bonus, m2 = D.sampled_accept(p_rows, qs, drafts, T, SEED, pi)
        want = drafts[:a] + [bonus]
        # the device keeps the rejected drafts after the bonus in its token buffer
        seen = [int(v) for v in dev_tok[L:L + K]]
        if new == want and seen[a + 1:] == drafts[a + 1:]:
            exact += 1
        else:
            assert min(m1, m2) < TIE, (pi, new, want, seen, drafts, min(m1, m2))
            ties += 1
        rejections += a < K
        L += len(new)
    assert exact >= passes - 2 and ties <= 2, (exact, ties)
    if mode == "self":
        assert rejections <= 2, rejections  # q == p: the bonus comes from the last verify row
    else:
        assert rejections > 0  # the residual draw ran
    sd.close()
    t.close()
    d.close()


def test_tree_sampled_acceptance_is_token_exact():
    from vella_b200 import decode as VD
    branching = (3, 2, 2, 1)
    dep, first, nch = D.tree_topology(branching)
    N, P, V, passes = len(dep), 16, 1000, 20
    t, d = _models(target_rows=N, draft_rows=16)
    pre_t, pre_d = prefix_of(P, 256, 65), prefix_of(P, 128, 66)
    sd = VD.SpecDecoder(t, d, k=len(branching), mode=VD.DRAFT_MODEL, seed=SEED, temperature=T, tree=branching)
    sd.set_prefix(pre_t, pre_d, P)
    sd.prefill()
    topo = _read(sd.tensor("tree_topology"), np.int32).reshape(3, N)
    assert np.array_equal(topo[0], dep) and np.array_equal(topo[1][nch > 0], first[nch > 0])
    assert np.array_equal(topo[2], nch)
    exact = ties = 0
    depth_hist = np.zeros(len(branching) + 1, np.int64)
    for pi in range(passes):
        new = sd.step()
        p_rows = _read(t.tensor("logits"), "bf16").reshape(-1, V)[:N]
        q_all = _read(sd.tensor("draft_rows"), "bf16").reshape(N, V)
        q_rows = {u: q_all[u] for u in range(N) if nch[u]}
        ttok = _read(sd.tensor("tree_tokens"), np.int32)[:N]
        toks, m1 = D.tree_children(q_rows, branching, T, SEED, pi)
        path, bonus, m2 = D.tree_accept(p_rows, lambda u: D.softmax_t(q_rows[u], T), ttok, branching, T, SEED, pi)
        want = [int(ttok[c]) for c in path] + [bonus]
        if new == want and np.array_equal(toks[1:], ttok[1:]):
            exact += 1
        else:
            assert min(m1, m2) < TIE, (pi, new, want, min(m1, m2))
            ties += 1
        depth_hist[len(path)] += 1
    assert exact >= passes - 2 and ties <= 2, (exact, ties)
    assert depth_hist[0] > 0 and depth_hist[1:].sum() > 0, depth_hist  # rejections and acceptances
    sd.close()
    t.close()
    d.close()
