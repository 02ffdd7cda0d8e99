"""Known-answer pins of the decode-loop oracle (integer logic), restated from the
reference's tests, plus Philox-4x32-10 known-answer vectors and the decode-loop
properties the library's design relies on."""
import numpy as np
import pytest

from oracle import decoder as D


def test_token_loop_is_detected_and_cut():
    # NemotronTranscribeTests.swift:157-177 (tokenLoopIsDetectedAndCut)
    prefix = [5, 6, 7, 8, 9]
    block = [21, 22, 23]
    tokens = prefix + block * 20
    assert D.loop_tail(tokens) == (len(prefix), 3)
    cut, looped = D.loop_cut(tokens)
    assert cut == prefix + block and looped
    short = prefix + block * 19  # 19 repeats is speech, not a loop
    assert D.loop_tail(short) is None
    assert D.loop_cut(short) == (short, False)
    assert D.loop_tail(list(range(200))) is None
    out = tokens + [21]
    while len(out) % 4 != 0:
        out.append(out[-3])
    assert D.ends_in_loop(out)
    assert out == prefix + block


def test_ends_in_loop_checks_every_fourth_token_only():
    out = [1] * 21  # a loop, but 21 is not a multiple of 4
    assert not D.ends_in_loop(out) and len(out) == 21
    out = [1] * 19 + [1]  # 20 tokens: checked
    assert D.ends_in_loop(out) and out == [1]


def test_runaway_draft_and_verify_is_decoded_again_greedy():
    # NemotronTranscribeTests.swift:278-298 (runawayDraftAndVerifyIsDecodedAgainGreedy)
    toks, looped, retried = D.retrying_runaway(8, lambda: ([7] * 8, False), lambda: ([1, 2, 3], False))
    assert toks == [1, 2, 3] and not looped and retried
    toks, looped, retried = D.retrying_runaway(1024, lambda: ([7, 7], True), lambda: ([9], True))
    assert toks == [9] and looped and retried
    ran = []
    toks, looped, retried = D.retrying_runaway(8, lambda: ([4, 5, 6, 7, 8, 9, 10], False),
                                               lambda: ran.append(1) or ([], False))
    assert toks == [4, 5, 6, 7, 8, 9, 10] and not retried and not ran


@pytest.mark.parametrize("ctr,key,expected", [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
])
def test_philox_known_answers(ctr, key, expected):
    # Random123 known-answer vectors for philox4x32 with 10 rounds
    assert D.philox4x32_10(ctr, key) == expected


def test_acceptance_rule():
    # NemotronTranscribeModel.swift:365-369: longest prefix ys[i] == drafts[i], bonus ys[a]
    assert D.accept([5, 6, 7, 8], [5, 6, 9]) == (2, 7)
    assert D.accept([5, 6, 7, 8], [5, 6, 7]) == (3, 8)
    assert D.accept([4, 6, 7, 8], [5, 6, 7]) == (0, 4)


def test_draft_and_verify_emits_exactly_the_greedy_sequence():
    """With a deterministic target, draft-and-verify returns the greedy tokens whatever the
    drafts are (the property the bit-exact GPU test relies on)."""
    rng = np.random.default_rng(0)
    V = 50
    table = rng.integers(0, V, size=(V, V))

    def nxt(seq):
        return int(table[seq[-1], seq[-2] if len(seq) > 1 else 0])

    first = 3
    ref, _ = D.greedy(nxt, first, 60)
    for k in (1, 2, 4, 8):
        for p in (0.0, 0.5, 0.9, 1.0):
            def propose(out, pi, k=k, p=p):
                drafts, seq = [], list(out)
                for i in range(k):
                    t = D.oracle_proposal(7, pi, i, ref[len(seq)] if len(seq) < len(ref) else None, p, V)
                    drafts.append(t)
                    seq.append(t)
                return drafts

            def verify(out, drafts):
                seq, ys = list(out), []
                for d in drafts + [None]:
                    ys.append(nxt(seq))
                    if d is not None:
                        seq.append(d)
                return ys

            toks, looped, hist = D.draft_and_verify(verify, propose, first, 60, k)
            assert toks == ref, (k, p)
            if p == 1.0:
                assert all(a == k for a in hist[:-1])


def test_oracle_proposal_rate():
    hits = sum(D.oracle_proposal(1, i, 0, 5, 0.7, 1000) == 5 for i in range(4000))
    assert abs(hits / 4000 - 0.7) < 0.03


def test_library_rope_table_matches_the_oracle():
    """The RoPE table the model handles upload (host code), bit for bit against the oracle's."""
    import ctypes

    import numpy as np

    from oracle import decoder as D
    from vella_b200 import _lib
    _lib.declare("vella_rope_table", ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                                    ctypes.POINTER(ctypes.c_float)])
    for S, hd, theta in ((1280, 128, 1e6), (64, 64, 1e4)):
        out = np.zeros((S, hd // 2, 2), np.float32)
        _lib.check(_lib.lib().vella_rope_table(S, hd, theta, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        assert np.array_equal(out, D.rope_table(S, hd, theta).astype(np.float32))


def _lib_cut(tokens, every_fourth=False):
    import ctypes

    import numpy as np

    from vella_b200 import _lib
    _lib.declare("vella_loop_cut", ctypes.c_int, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_int32)])
    arr = np.ascontiguousarray(np.asarray(tokens, np.int32))
    kept = ctypes.c_int32()
    rc = _lib.lib().vella_loop_cut(arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(tokens),
                                   int(every_fourth), ctypes.byref(kept))
    assert rc in (0, 1)
    return list(tokens[:kept.value]), bool(rc)


def test_library_loop_guard_matches_the_known_answers_and_the_oracle():
    """The library's host-side loop guard (the one the decode loop runs) on the reference's
    known answers (NemotronTranscribeTests.swift:145-206) and on random sequences with and
    without planted loops, against the oracle."""
    import random
    prefix, block = [5, 6, 7, 8, 9], [21, 22, 23]  # NemotronTranscribeTests.swift:157-177
    tokens = prefix + block * 20
    assert _lib_cut(tokens) == (prefix + block, True)
    short = prefix + block * 19
    assert _lib_cut(short) == (short, False)
    assert _lib_cut(list(range(200))) == (list(range(200)), False)
    assert _lib_cut([1] * 21, every_fourth=True) == ([1] * 21, False)  # 21 is not a multiple of 4
    assert _lib_cut([1] * 20, every_fourth=True) == ([1], True)
    rng = random.Random(3)
    for _ in range(300):
        head = [rng.randrange(6) for _ in range(rng.randrange(0, 40))]
        blk = [rng.randrange(6) for _ in range(rng.randrange(1, 70))]
        seq = head + blk * rng.randrange(1, 26) + [rng.randrange(6) for _ in range(rng.randrange(0, 3))]
        assert _lib_cut(seq) == D.loop_cut(seq), seq
        out = list(seq)
        looped = D.ends_in_loop(out)
        assert _lib_cut(seq, every_fourth=True) == (out, looped), seq
