"""Pin the oracle (oracle/ember_oracle.c) before trusting it as the GPU checker.

1. Against the committed golden vectors, produced by the unmodified reference
   (tests/golden/make_golden.py): works anywhere, including the GPU box.
2. Against the reference itself, compiled from its own sources into
   oracle/_ref/libember_ref_det.so, on fresh inputs: where that build exists.
Both comparisons are bit-for-bit.
"""
import hashlib
import os

import numpy as np
import pytest

from emberllm_b200 import synth

from . import helpers as H

NAMES = ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-smol-q4", "tiny-f32"]
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    return H.Oracle()


def _sha(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read())
    return h.hexdigest()


@pytest.mark.parametrize("name", NAMES)
def test_synthetic_model_bytes_match_golden(name):
    """the synthetic writer + quantizer still produce the exact files the goldens were made from"""
    H.ensure_built()
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    assert _sha(synth.ensure_model(name)) == bytes(g["sha256"]).decode()


@pytest.mark.parametrize("kv", ["kv32", "kv16"])
@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_goldens(orc, name, kv):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    path = synth.ensure_model(name)
    s = orc.session(path, 0, 1 if kv == "kv16" else 0)
    assert np.array_equal(H.bits(s.prefill(g[kv + "_prompt"])), H.bits(g[kv + "_prefill"]))
    for i, t in enumerate(g[kv + "_forced_ids"]):
        assert np.array_equal(H.bits(s.forward(int(t), 16 + i)), H.bits(g[kv + "_forced"][i]))
    s.close()
    s = orc.session(path, 0, 1 if kv == "kv16" else 0)
    got = H.greedy_run(s, [int(t) for t in g[kv + "_prompt"]], 24)
    s.close()
    assert got == [int(t) for t in g[kv + "_greedy"]]


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("kv16", [0, 1])
@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_live_reference(orc, name, kv16):
    ref = H.ApiLib(H.REF_DET)
    path = synth.ensure_model(name)
    a, b = ref.session(path, 0, kv16), orc.session(path, 0, kv16)
    rng = np.random.default_rng(99)
    ids = rng.integers(0, a.vocab, 40)
    assert np.array_equal(H.bits(a.prefill(ids)), H.bits(b.prefill(ids)))
    for pos in range(40, 100):
        t = int(rng.integers(0, a.vocab))
        assert np.array_equal(H.bits(a.forward(t, pos)), H.bits(b.forward(t, pos)))
    a.close()
    b.close()


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
def test_oracle_prefill_chunks_equal_reference_batched_prefill(orc):
    """the reference's batched prefill (ref src/model.c:283-360) split into chunks
    at different starts equals the oracle's (sequential) prefill"""
    ref = H.ApiLib(H.REF_DET)
    path = synth.ensure_model("tiny-qwen3")
    a, b = ref.session(path, 0, 0), orc.session(path, 0, 0)
    rng = np.random.default_rng(5)
    ids = [int(t) for t in rng.integers(0, a.vocab, 70)]
    for lo, hi in [(0, 1), (1, 33), (33, 70)]:
        assert np.array_equal(H.bits(a.prefill(ids[lo:hi], lo)), H.bits(b.prefill(ids[lo:hi], lo)))
    a.close()
    b.close()


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
def test_oracle_stories110m_first_steps_match_reference(orc):
    """one full-size architecture through both, a few steps (CPU-cheap)"""
    ref = H.ApiLib(H.REF_DET)
    path = synth.ensure_model("stories110m")
    a, b = ref.session(path, 64, 0), orc.session(path, 64, 0)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, a.vocab, 6)
    assert np.array_equal(H.bits(a.prefill(ids)), H.bits(b.prefill(ids)))
    a.close()
    b.close()


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
def test_oracle_long_prefill_chunks_match_reference(orc):
    """a 600-token prompt: the oracle's batched prefill goes through it in chunks
    of 256 tokens, the reference's in one batch; logits and the following steps
    agree bit for bit"""
    ref = H.ApiLib(H.REF_DET)
    path = synth.ensure_model("tiny-long")
    a, b = ref.session(path, 700, 0), orc.session(path, 700, 0)
    rng = np.random.default_rng(11)
    ids = rng.integers(0, a.vocab, 600)
    assert np.array_equal(H.bits(a.prefill(ids)), H.bits(b.prefill(ids)))
    for pos in range(600, 604):
        t = int(rng.integers(0, a.vocab))
        assert np.array_equal(H.bits(a.forward(t, pos)), H.bits(b.forward(t, pos)))
    a.close()
    b.close()


_REF_THREADS = []


def _ref_threads(ref):
    """start the reference's thread pool once per process (its rows split over
    threads give the same results; a second ember_threads_init would restart
    the pool under the running workers)"""
    if not _REF_THREADS:
        ref.lib.ember_threads_init(min(16, os.cpu_count() or 1))
        _REF_THREADS.append(1)


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("name", ["qwen3-0.6b", "qwen2.5-0.5b", "smollm2-135m"])
def test_oracle_fullsize_qwen_steps_match_reference(orc, name):
    """the full-size BASELINE shapes -- head_dim 128 with QK-norm (Qwen3), q/k/v
    biases (Qwen2.5), Q4_0 layers (SmolLM2), a 151,936 or 49,152-entry vocab --
    through the reference and the oracle: a 20-token prefill, then teacher-forced
    steps, logits bit for bit"""
    ref = H.ApiLib(H.REF_DET)
    _ref_threads(ref)
    path = synth.ensure_model(name)
    a, b = ref.session(path, 64, 0), orc.session(path, 64, 0)
    rng = np.random.default_rng(21)
    ids = rng.integers(0, a.vocab, 20)
    assert np.array_equal(H.bits(a.prefill(ids)), H.bits(b.prefill(ids)))
    for pos in range(20, 23):
        t = int(rng.integers(0, a.vocab))
        assert np.array_equal(H.bits(a.forward(t, pos)), H.bits(b.forward(t, pos)))
    a.close()
    b.close()
