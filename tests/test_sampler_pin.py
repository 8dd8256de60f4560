"""Pin the oracle's sampler (orc_sample) to the reference's own ember_sample
(oracle/_ref/libember_ref_det.so, built from its sources): on random logits of a
small and of the Qwen vocabulary, every setting of tests/sampler_helpers.py, a
run of draws that feeds each token back into the sampler's history -- the same
tokens and the same random stream."""
import numpy as np
import pytest

from . import helpers as H
from . import sampler_helpers as S


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    return H.Oracle()


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("vocab", [640, 151936])
@pytest.mark.parametrize("k", range(len(S.SETTINGS)))
def test_oracle_sampler_matches_reference(orc, vocab, k):
    ref = S.ref_lib()
    setting = S.SETTINGS[k]
    rng = np.random.default_rng(100 + k)
    s = S.new_ref_sampler(ref, setting, seed=1234 + k)
    for step in range(6):
        logits = (rng.standard_normal(vocab) * (1.0 + step)).astype(np.float32)
        logits[rng.integers(0, vocab, 8)] = logits.max()          # ties at the top
        hist, hl = S.history_of(s)
        want_rng = s.rng_state
        tok_o, rng_o = S.oracle_sample(orc, logits, setting, want_rng, hist, hl)
        lg = logits.copy()
        tok_r = ref.ember_sample(s, lg.ctypes.data_as(S.ctypes.POINTER(S.ctypes.c_float)), vocab)
        assert tok_o == tok_r, (setting, step)
        assert rng_o == s.rng_state
    ref.ember_sampler_free(s)
