"""The oracle's stochastic acceptance and tree verification against their defining property
(CPU only): whatever the draft distribution, the first emitted token of a pass is
distributed exactly as the target's softmax at temperature T (speculative sampling,
Leviathan et al. 2023; multi-candidate tree acceptance, SpecInfer, Miao et al. 2023).  The
reference's own draft-and-verify is greedy only, so these algorithms have no reference
fixtures: the property is the pin.  Also: the inverse-CDF draw, the Philox uniforms, and the
breadth-first tree numbering."""
import numpy as np

from oracle import decoder as D

T = 0.7


def _chi2_ok(counts, probs, n):
    """Pearson chi-square over the cells with expected count >= 5, below the 99.9% point."""
    from scipy.stats import chi2
    exp = probs * n
    keep = exp >= 5
    stat = (((counts[keep] - exp[keep]) ** 2) / exp[keep]).sum()
    return stat < chi2.ppf(0.999, max(int(keep.sum()) - 1, 1)), stat


def test_icdf_draws_follow_the_weights_and_report_margins():
    w = np.array([0.0, 1.0, 3.0, 0.0, 4.0])
    assert D.icdf(w, 0.0)[0] == 1
    assert D.icdf(w, 0.124)[0] == 1 and D.icdf(w, 0.126)[0] == 2
    assert D.icdf(w, 0.999)[0] == 4
    idx, margin = D.icdf(w, 0.5)  # target 4.0 sits on the edge between bins 2 and 4
    assert idx == 4 and margin == 0.0
    assert D.icdf(np.zeros(4), 0.3)[0] == -1


def test_uniforms_are_philox_words_and_distinct_per_counter():
    u = D.uniform(7, 3, 2, D.PURPOSE_ACCEPT, 1)
    r = D.philox4x32_10((3, 2, D.PURPOSE_ACCEPT, 1), (7, 0))
    assert u == D.u01(r[0]) and 0.0 <= u < 1.0
    draws = {D.uniform(7, a, b, p, s) for a in range(3) for b in range(3)
             for p in (D.PURPOSE_ACCEPT, D.PURPOSE_RESIDUAL, D.PURPOSE_DRAFT) for s in range(2)}
    assert len(draws) == 54


def test_tree_topology_is_breadth_first():
    dep, first, nch = D.tree_topology((3, 2, 2, 1))
    assert len(dep) == 34 and list(nch[:4]) == [3, 2, 2, 2] and list(first[:4]) == [1, 4, 6, 8]
    assert all(dep[first[u] + i] == dep[u] + 1 for u in range(34) for i in range(nch[u]))
    assert list(dep) == sorted(dep)


def test_speculative_sampling_emits_the_target_distribution():
    rng = np.random.default_rng(0)
    V, K, n = 6, 3, 12000
    p_rows = rng.standard_normal((K + 1, V)) * 1.5
    q_rows = rng.standard_normal((K, V)) * 1.5
    qs = [D.softmax_t(r, T) for r in q_rows]
    first = np.zeros(V)
    accepted = np.zeros(K + 1)
    for it in range(n):
        drafts, _ = D.sample_drafts(q_rows, T, seed=5, pass_index=it)
        a, bonus, _ = D.sampled_accept(p_rows, qs, drafts, T, seed=5, pass_index=it)
        emitted = drafts[:a] + [bonus]
        first[emitted[0]] += 1
        accepted[a] += 1
    ok, stat = _chi2_ok(first, D.softmax_t(p_rows[0], T), n)
    assert ok, stat
    # the first draft is accepted with probability sum_x min(p(x), q(x))
    p0 = D.softmax_t(p_rows[0], T)
    want = np.minimum(p0, qs[0]).sum()
    got = 1.0 - accepted[0] / n
    assert abs(got - want) < 4 * np.sqrt(want * (1 - want) / n), (got, want)


def test_oracle_draft_sampling_emits_the_target_distribution():
    rng = np.random.default_rng(1)
    V, K, n = 5, 2, 12000
    p_rows = rng.standard_normal((K + 1, V)) * 1.5
    qs = [D.oracle_draft_q(V, 2, 0.6), D.oracle_draft_q(V, None, 0.6)]
    first = np.zeros(V)
    for it in range(n):
        drafts = [D.icdf(q, D.uniform(9, it, i, D.PURPOSE_DRAFT, 0))[0] for i, q in enumerate(qs)]
        a, bonus, _ = D.sampled_accept(p_rows, qs, drafts, T, seed=9, pass_index=it)
        first[(drafts[:a] + [bonus])[0]] += 1
    ok, stat = _chi2_ok(first, D.softmax_t(p_rows[0], T), n)
    assert ok, stat


def test_tree_acceptance_emits_the_target_distribution():
    """Branching (3, 2): the first emitted token (the accepted depth-1 child, else the bonus)
    follows p at the root, and the token after an accepted node follows p at that node."""
    rng = np.random.default_rng(2)
    V, n = 6, 12000
    branching = (3, 2)
    dep, first, nch = D.tree_topology(branching)
    N = len(dep)
    q_rows = {u: rng.standard_normal(V) * 1.5 for u in range(N) if nch[u]}
    p_rows = rng.standard_normal((N, V)) * 1.5
    c1 = np.zeros(V)
    c2 = {}
    for it in range(n):
        toks, _ = D.tree_children(q_rows, branching, T, seed=3, pass_index=it)
        path, bonus, _ = D.tree_accept(p_rows, lambda u: D.softmax_t(q_rows[u], T), toks, branching, T, seed=3,
                                       pass_index=it)
        emitted = [int(toks[c]) for c in path] + [bonus]
        c1[emitted[0]] += 1
        if path:
            c2.setdefault(path[0], np.zeros(V))[emitted[1]] += 1
    ok, stat = _chi2_ok(c1, D.softmax_t(p_rows[0], T), n)
    assert ok, stat
    for node, counts in c2.items():
        ok, stat = _chi2_ok(counts, D.softmax_t(p_rows[node], T), counts.sum())
        assert ok, (node, stat)
