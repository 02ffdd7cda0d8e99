"""The persistent decode forward (one cooperative launch per forward of at most 16 rows) against
the per-op kernels and the oracle, on small models with head_dim 128 (the shapes it serves).

Bars: logits within 2e-2 of the per-op path (the GEMMs' arithmetic is shared; the large int4
GEMMs' split-K boundaries differ from the per-op path's two CTAs per SM, and the attention
takes its keys in chunks of 32 instead of 64, so the online softmax rounds differently); dense
weights -> within 2e-2 of the oracle; int4 weights -> within 2e-2 of the oracle's fp32 logits
plus half a bf16 ulp, widened to twice the oracle's own rounding-order spread; draft-and-verify
with the persistent forward emits exactly its greedy tokens, single stream and three streams;
a 5:1 query-head grouping; switching it on is refused where the shapes do not suit it.
"""
import numpy as np
import pytest

from oracle import affine as A
from oracle import decoder as D
from tests.test_baseline_shapes_gpu import _bf16_ulp
from tests.test_decode_gpu import LOGIT_TOL, oracle_weights, prefix_of

pytestmark = pytest.mark.gpu


def _model(bits, d=256, H=2, KV=1, ffn=512, V=1000, layers=2, seed=1, std=0.05, **kw):
    from vella_b200 import decode as VD
    mc = VD.ModelConfig(layers, d, H, KV, 128, ffn, V, bits=bits, max_seq=256, max_prefix=64, **kw)
    m = VD.Model(mc)
    m.init_random(seed, std)
    m.set_persistent(True)
    return m, D.Config(layers, d, H, KV, 128, ffn, V, bits=bits)


def _score(m, pre, toks, persistent):
    m.set_persistent(persistent)
    return A.bf16_from_bits(m.score(pre, toks))


def test_dense_logits_match_per_op_path_and_oracle():
    m, oc = _model(0, seed=3)
    pre = prefix_of(20, oc.d_model, 4)
    toks = [int(t) for t in np.random.default_rng(5).integers(0, oc.vocab, 30)]
    on, off = _score(m, pre, toks, True), _score(m, pre, toks, False)
    assert np.isfinite(on).all()
    assert np.abs(on - off).max() <= LOGIT_TOL
    ref = D.score(oc, oracle_weights(m, oc), A.bf16_from_bits(pre), toks, D.rope_table(64, 128, oc.rope_theta))
    assert np.abs(on - ref).max() <= LOGIT_TOL
    m.close()


def test_int4_logits_match_per_op_path_and_oracle():
    m, oc = _model(4, d=512, H=4, KV=2, ffn=1024, seed=7)
    pre = prefix_of(24, oc.d_model, 8)
    toks = [int(t) for t in np.random.default_rng(9).integers(0, oc.vocab, 20)]
    on, off = _score(m, pre, toks, True), _score(m, pre, toks, False)
    assert np.isfinite(on).all()
    assert np.abs(on - off).max() <= LOGIT_TOL
    # against the oracle's fp32 logits before their bf16 rounding, half an ulp of the device's
    # bf16 output allowed on top (logits of magnitude 2..4 have an ulp of 1.6e-2), and the bar
    # widened to twice the oracle's own rounding-order spread (its K sums ascending vs
    # descending) where that exceeds 2e-2
    W, table = oracle_weights(m, oc), D.rope_table(64, 128, oc.rope_theta)
    with A.c_accumulation():
        ref = D.score(oc, W, A.bf16_from_bits(pre), toks, table, raw_logits=True)
    with A.c_accumulation(reverse=True):
        ref_rev = D.score(oc, W, A.bf16_from_bits(pre), toks, table, raw_logits=True)
    spread = float(np.abs(ref - ref_rev).max())
    err = float((np.abs(on - ref) - 0.5 * _bf16_ulp(on)).max())
    assert err <= max(LOGIT_TOL, 2.0 * spread), (err, spread)
    assert A.relative_rms(on, ref) <= 1e-2
    m.close()


@pytest.mark.parametrize("H,KV", [(4, 2), (20, 4)])  # 2:1 and the 30B target's 5:1 grouping
def test_draft_and_verify_equals_greedy_on_the_persistent_forward(H, KV):
    from vella_b200 import decode as VD
    t, tc = _model(4, d=512, H=H, KV=KV, ffn=1024, seed=11)
    d, dc = _model(0, seed=12)
    pre_t, pre_d = prefix_of(24, 512, 13), prefix_of(24, 256, 14)
    g = VD.SpecDecoder(t, d, k=4)
    g.set_prefix(pre_t, pre_d, 24)
    ref = g.decode_greedy(60).tokens
    assert len(ref) == 60
    for mode, kw in ((VD.DRAFT_MODEL, {}), (VD.DRAFT_ORACLE, dict(oracle_p=0.7, seed=3))):
        sd = VD.SpecDecoder(t, d, k=4, mode=mode, **kw)
        sd.set_prefix(pre_t, pre_d, 24)
        sd.set_reference(ref)
        assert sd.decode_mtp(48).tokens == ref[:48]
        sd.close()
    # the greedy tokens follow the oracle by the margin rule
    logits = D.score(tc, oracle_weights(t, tc), A.bf16_from_bits(pre_t), ref[:24], D.rope_table(64, 128, tc.rope_theta))
    for j, tok in enumerate(ref[:24]):
        row = logits[j]
        best = int(np.argmax(row))
        assert tok == best or row[best] - row[tok] <= LOGIT_TOL, (j, tok, best)
    for x in (g, t, d):
        x.close()


def test_three_streams_verify_in_one_persistent_forward():
    """3 streams x (K + 1 = 5) rows = 15 rows per verify forward: batched draft-and-verify equals
    batched greedy, and each stream equals its single-stream decode."""
    from vella_b200 import decode as VD
    S = 3
    t, tc = _model(4, d=512, H=4, KV=2, ffn=1024, seed=21, streams=S)
    d, dc = _model(0, seed=22, streams=S)
    pre_t = np.stack([prefix_of(16, 512, 30 + j) for j in range(S)])
    pre_d = np.stack([prefix_of(16, 256, 40 + j) for j in range(S)])
    sb = VD.SpecDecoder(t, d, k=4)
    sb.set_prefix(pre_t, pre_d)
    greedy = sb.decode_batch(32, VD.DECODE_GREEDY)
    spec = sb.decode_batch(32, VD.DECODE_SPEC)
    assert np.array_equal(spec, greedy)
    sb.close()
    t1, _ = _model(4, d=512, H=4, KV=2, ffn=1024, seed=21)
    d1, _ = _model(0, seed=22)
    for j in range(S):
        g = VD.SpecDecoder(t1, d1, k=4)
        g.set_prefix(pre_t[j], pre_d[j], 16)
        assert g.decode_greedy(32).tokens == list(greedy[j]), j
        g.close()
    for x in (t, d, t1, d1):
        x.close()


def test_switch_is_refused_where_the_shapes_do_not_suit():
    from vella_b200 import _lib as L
    from vella_b200 import decode as VD
    m = VD.Model(VD.ModelConfig(1, 256, 4, 2, 64, 512, 1000, bits=4, max_seq=64, max_prefix=16))  # head_dim 64
    m.set_persistent(False)
    with pytest.raises(L.VellaError):
        m.set_persistent(True)
    m.close()
