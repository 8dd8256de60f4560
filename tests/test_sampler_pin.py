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


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("last_n,rp,pres,freq", [(0, 1.1, 0.0, 0.0), (4, 1.0, 0.0, 0.0), (5, 1.2, 0.3, 0.0),
                                                  (3, 1.0, 0.0, 0.2), (16, 1.1, 0.5, 0.3)])
def test_python_sampler_mirrors_the_reference_state(last_n, rp, pres, freq):
    """emberllm_b200.Sampler (the host half of ember_sample_device) keeps the
    reference's EmberSampler state: seed handling, a history ring only when a
    penalty is active, and accept / reset moving hist_len and hist_pos alike"""
    from emberllm_b200 import Sampler
    ref = S.ref_lib()
    for seed in (0, 12345):
        r = S.RefSampler()
        ref.ember_sampler_init(S.ctypes.byref(r), 0.7, 0.9, 40, seed)
        ref.ember_sampler_set_penalties(S.ctypes.byref(r), rp, last_n, pres, freq, 0.05)
        d = Sampler(0.7, 0.9, 40, seed)
        d.set_penalties(rp, last_n, pres, freq, 0.05)
        assert d.rng_state.value == r.rng_state
        assert (d.history is None) == (not r.history)
        for step, tok in enumerate([5, 9, 5, 2, 7, 7, 1, 3, 9, 4, 8, 6, 0, 11, 5, 12, 13, 14, 2, 5]):
            ref.ember_sampler_accept(S.ctypes.byref(r), tok)
            d.accept(tok)
            assert (d.hist_len, d.hist_pos) == (r.hist_len, r.hist_pos), step
            if d.history is not None:
                assert list(d.history)[:d.hist_len] == [r.history[i] for i in range(r.hist_len)]
            if step == 9:
                ref.ember_sampler_reset(S.ctypes.byref(r))
                d.reset()
        ref.ember_sampler_free(S.ctypes.byref(r))
