"""The device sampler (ember_sample_device, Ember.sample) against the reference's
own ember_sample (oracle/_ref/libember_ref_det.so, built from its sources) on the
same logits: the same token, the same random stream and the same history, step
after step of a sampled run, for every setting of tests/sampler_helpers.py, on a
small vocabulary and on Qwen's 151,936; then planted logits with the cases the
order and the truncation turn on (ties, a flat vocabulary, -inf, top_k beyond the
vocabulary, top_p met by the first candidate, min_p near 1)."""
import ctypes

import numpy as np
import pytest

from emberllm_b200 import Ember, Sampler, synth

from . import helpers as H
from . import sampler_helpers as S

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")]


def _pair(setting, seed):
    ref = S.ref_lib()
    r = S.new_ref_sampler(ref, setting, seed)
    temp, top_p, top_k, min_p, rp, last_n, pres, freq = setting
    d = Sampler(temp, top_p, top_k, seed)
    d.set_penalties(rp, last_n, pres, freq, min_p)
    return ref, r, d


def _ref_draw(ref, r, logits):
    lg = np.ascontiguousarray(logits, np.float32).copy()
    return ref.ember_sample(ctypes.byref(r), lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(lg))


def _same_state(r, d):
    assert r.rng_state == d.rng_state.value
    assert r.hist_len == d.hist_len and r.hist_pos == d.hist_pos
    for i in range(r.hist_len):
        assert r.history[i] == d.history[i]


@pytest.mark.parametrize("name,steps", [("tiny-llama", 24), ("qwen3-0.6b", 12)])
@pytest.mark.parametrize("k", range(len(S.SETTINGS)))
def test_sampled_run_matches_reference(name, steps, k):
    """prefill, then `steps` rounds of draw-and-forward: every draw the reference's"""
    H.ensure_built()
    e = Ember(synth.ensure_model(name), ctx=64)
    ref, r, d = _pair(S.SETTINGS[k], seed=77 + k)
    prompt = [int(t) for t in np.random.default_rng(k).integers(0, e.vocab, 9)]
    logits = np.ctypeslib.as_array(e.prefill(prompt), (e.vocab,)).copy()
    pos = len(prompt)
    for i in range(steps):
        want = _ref_draw(ref, r, logits)
        got = e.sample(d)
        assert got == want, (name, S.SETTINGS[k], i)
        _same_state(r, d)
        logits = np.ctypeslib.as_array(e.forward(got, pos), (e.vocab,)).copy()
        pos += 1
    ref.ember_sampler_free(ctypes.byref(r))
    e.close()


def _planted_cases(vocab):
    g = np.random.default_rng(5)
    base = g.standard_normal(vocab).astype(np.float32)
    ties = base.copy()
    ties[g.choice(vocab, 64, replace=False)] = base.max() + 1.0           # 64-way tie at the top
    ties[g.choice(vocab, 300, replace=False)] = np.float32(0.5)           # a tie band inside
    flat = np.zeros(vocab, np.float32)                                    # every p equal
    neg = base.copy()
    neg[g.choice(vocab, vocab // 3, replace=False)] = -np.inf             # masked entries
    peak = base.copy()
    peak[17] = 60.0                                                       # one candidate holds all mass
    wide = (g.standard_normal(vocab) * 30).astype(np.float32)             # many p underflow to 0
    return {"ties": ties, "flat": flat, "neg_inf": neg, "peak": peak, "wide": wide}


PLANT_SETTINGS = S.SETTINGS + [
    (1.0, 1.0, 10 ** 9, 0.0, 1.0, 0, 0.0, 0.0),     # top_k beyond the vocabulary
    (1.0, 1e-6, 0, 0.0, 1.0, 0, 0.0, 0.0),          # top_p met by the first candidate
    (1.0, 1.0, 0, 0.999, 1.0, 0, 0.0, 0.0),         # min_p near 1
    (0.05, 0.5, 5, 0.1, 1.0, 0, 0.0, 0.0),          # cold, every truncation
]


@pytest.mark.parametrize("name", ["tiny-llama", "qwen3-0.6b"])
def test_planted_logits_match_reference(name):
    H.ensure_built()
    hooks = H.testhooks()
    e = Ember(synth.ensure_model(name), ctx=16)
    e.prefill([1, 2, 3])
    dev = e.lib.ember_cuda_state_logits_dev(e.lib.ember_state_cuda(e.st))
    for case, logits in _planted_cases(e.vocab).items():
        assert hooks.ember_testhook_copy_to_device(dev, logits.ctypes.data, logits.nbytes) == 0
        for k, setting in enumerate(PLANT_SETTINGS):
            ref, r, d = _pair(setting, seed=1000 + k)
            for i in range(3):
                want = _ref_draw(ref, r, logits)
                got = e.sample(d)
                assert got == want, (name, case, setting, i)
                _same_state(r, d)
            ref.ember_sampler_free(ctypes.byref(r))
    e.close()


def test_sampler_leaves_logits_and_rejects_bad_settings():
    """the state's logits are unchanged by a draw (a greedy draw afterwards is
    the argmax of the step's logits); a NaN temperature or a negative history
    length is an error status with the context usable afterwards"""
    H.ensure_built()
    e = Ember(synth.ensure_model("tiny-llama"), ctx=16)
    lg = np.ctypeslib.as_array(e.prefill([5, 6, 7]), (e.vocab,)).copy()
    hot = Sampler(1.5, 0.9, 50, seed=3)
    hot.set_penalties(1.2, 4, 0.3, 0.2, 0.0)
    for _ in range(4):
        e.sample(hot)
    assert e.sample(Sampler(0.0)) == H.first_argmax(lg)
    cs = e.lib.ember_state_cuda(e.st)
    out = ctypes.c_int(-1)
    bad = Sampler(float("nan")).params()
    assert e.lib.ember_cuda_sample(cs, ctypes.byref(bad), 0.5, None, 0, ctypes.byref(out)) != 0
    assert b"NaN" in e.lib.ember_cuda_error()
    ok = Sampler(0.0).params()
    assert e.lib.ember_cuda_sample(cs, ctypes.byref(ok), 0.0, None, -1, ctypes.byref(out)) != 0
    assert e.lib.ember_cuda_sample(cs, ctypes.byref(ok), 0.0, None, 0, ctypes.byref(out)) == 0
    assert out.value == H.first_argmax(lg)
    e.close()
