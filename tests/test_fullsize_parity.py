"""GPU parity on the BASELINE configurations at their stated sizes, bit for bit
against the oracle (oracle/liboracle.so, pinned to the reference build).

  configs[3] Qwen3-0.6B  the bench workload itself: a 128-token prompt (seed 1),
                         then 128 greedy tokens at depth 128; and the cache
                         prefilled to 1024 and 4096 positions, then greedy steps
                         (the split decode attention at head_dim 128)
  configs[2] Qwen2.5-0.5B  512-token prefill, then 128 decode steps at depth 512
  configs[1] SmolLM2-135M  512-token prefill (Q4_0), then 256 greedy tokens

Every step compares the full vocab logits through ember_forward (tolerance 0;
the 1e-3 rel-L2 bound of the north star is asserted too), and the device greedy
loop (ember_forward_greedy, the bench's timed path) must pick the oracle's tokens.
"""
import numpy as np
import pytest

from emberllm_b200 import Ember, synth

from . import helpers as H
from .test_gpu_parity import assert_same

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def prod():
    H.ensure_built()
    return H.ApiLib(H.LIB)


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    return H.Oracle()


def _run(prod, orc, name, ctx, kv16, prompt, steps):
    """prefill `prompt`, then `steps` greedy forwards on both sides, comparing
    every step's logits; returns the oracle's greedy tokens"""
    path = synth.ensure_model(name)
    a = prod.session(path, ctx, kv16)
    b = orc.session(path, ctx, kv16)
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert_same(la, lb, f"{name} prefill {len(prompt)}")
    toks = []
    pos = len(prompt)
    for i in range(steps):
        ta, tb = H.first_argmax(la), H.first_argmax(lb)
        assert ta == tb, f"{name}: greedy diverged at token {i}"
        toks.append(tb)
        la, lb = a.forward(ta, pos), b.forward(tb, pos)
        assert_same(la, lb, f"{name} step {i} (pos {pos})")
        pos += 1
    a.close()
    b.close()
    return toks


def _device_greedy(name, ctx, kv16, prompt, steps):
    """the bench's path: prefill, then ember_forward_greedy from the first pick"""
    e = Ember(synth.ensure_model(name), ctx=ctx, kv_fp16=bool(kv16))
    logits = np.ctypeslib.as_array(e.prefill(prompt), (e.vocab,)).copy()
    first = H.first_argmax(logits)
    got = [first] + e.greedy(first, len(prompt), steps - 1)
    e.close()
    return got


def _prompt(vocab, n, seed=1):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


@pytest.mark.parametrize("persist", ["0", "1"])
def test_qwen3_bench_workload_128_greedy(prod, orc, persist, monkeypatch):
    """configs[3] exactly as bench.py times it: depth 128, 128 greedy tokens,
    context depth + tokens + 8, on the graph step and on the persistent kernel"""
    monkeypatch.setenv("EMBER_PERSIST", persist)
    depth, ntok = 128, 128
    ctx = depth + ntok + 8
    prompt = _prompt(151936, depth)
    want = _run(prod, orc, "qwen3-0.6b", ctx, 0, prompt, ntok)
    assert _device_greedy("qwen3-0.6b", ctx, 0, prompt, ntok) == want


@pytest.mark.parametrize("depth,kv16", [(1024, 0), (1024, 1), (4096, 0)])
def test_qwen3_deep_cache_greedy(prod, orc, depth, kv16):
    """configs[3] at depths 1024 and 4096: the cache prefilled with `depth`
    random tokens, then 16 greedy steps (the split attention: keys scored over
    many 128-position CTAs, head_dim 128, QK-norm)"""
    steps = 16
    ctx = depth + steps + 8
    prompt = _prompt(151936, depth)
    want = _run(prod, orc, "qwen3-0.6b", ctx, kv16, prompt, steps)
    assert _device_greedy("qwen3-0.6b", ctx, kv16, prompt, steps) == want


def test_qwen25_prefill512_decode128(prod, orc):
    """512-token prefill (q/k/v biases), then 128 decode steps at depth 512"""
    prompt = _prompt(151936, 512)
    want = _run(prod, orc, "qwen2.5-0.5b", 512 + 128 + 8, 0, prompt, 128)
    assert _device_greedy("qwen2.5-0.5b", 512 + 128 + 8, 0, prompt, 128) == want


def test_smollm2_q4_prefill512_greedy256(prod, orc):
    """512-token prefill with Q4_0 layers, then 256 greedy tokens"""
    prompt = _prompt(49152, 512)
    want = _run(prod, orc, "smollm2-135m", 512 + 256 + 8, 0, prompt, 256)
    assert _device_greedy("smollm2-135m", 512 + 256 + 8, 0, prompt, 256) == want


@pytest.mark.parametrize("name,ctx,want", [("qwen3-0.6b", 264, 1), ("qwen2.5-0.5b", 648, 1),
                                           ("smollm2-135m", 776, 1), ("stories110m", 264, 1),
                                           ("qwen3-0.6b", 1048, 0)])
def test_which_decode_path_serves_each_config(prod, name, ctx, want, monkeypatch):
    """with the persistent step requested (EMBER_PERSIST=1), the BASELINE decode
    configurations run as the persistent kernel (the bench workload included);
    contexts whose keys exceed shared memory keep the graph step"""
    from .test_gpu_parity import is_persistent
    monkeypatch.setenv("EMBER_PERSIST", "1")
    a = prod.session(synth.ensure_model(name), ctx, 0)
    got, why = is_persistent(prod.lib, a)
    a.close()
    assert got == want, why
