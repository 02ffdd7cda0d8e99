"""Token-by-token Whisper decoding (vella_whisper_begin / vella_whisper_step) against the
whole-loop decode."""
import pytest

from tests.test_whisper_gpu import mel_of

pytestmark = pytest.mark.gpu


def test_token_by_token_equals_the_loop():
    """begin + step give the tokens and log-probability sum of one decode call, with and
    without the token rules; a step before begin or after a new window is rejected."""
    from vella_b200 import _lib
    from vella_b200 import whisper as VW
    m = VW.Whisper(VW.TINY)
    m.init_random(5, 0.1)
    mel = mel_of(VW.TINY, 21)
    m.encode(mel)
    prompt = [50258, 50259, 50359, 50363]
    with pytest.raises(_lib.VellaError):
        m.step()
    V = VW.TINY.vocab
    for rules in (None, dict(eot=50257, no_timestamps=V - 3, timestamp_begin=V - 2, suppress=[220],
                             begin_suppress=[50257, 220])):
        m.set_rules(**rules) if rules else m.set_rules(None)
        want = m.decode(prompt, 12).tokens
        lp = m.stats()["sum_logprob"]
        got = [m.begin(prompt)] + [m.step() for _ in range(11)]
        assert got == want
        assert m.logprobs()[0] == lp
    m.encode(mel)
    with pytest.raises(_lib.VellaError):
        m.step()
    m.close()
