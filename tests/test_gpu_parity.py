"""GPU parity: the B200 token loop against the CPU checkers, through the C-ABI.

Bar: int8 block sums bit-exact, logits within 1e-3 relative
L2, greedy-identical tokens. This implementation reproduces the reference's
deterministic fp32 operation order, so the tests demand more: logits are
compared BIT FOR BIT (tolerance 0), and the 1e-3 rel-L2 bound is asserted too so
a failure report shows how far off it is.
"""
import ctypes
import os

import numpy as np
import pytest

from emberllm_b200 import synth

from . import helpers as H

pytestmark = pytest.mark.gpu

TINY = ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-smol-q4", "tiny-f32", "tiny-mqa"]
REL_L2 = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_same(got, want, what):
    err = rel_l2(got, want)
    assert err <= REL_L2, f"{what}: rel-L2 {err:.3e}"
    nd = int(np.count_nonzero(H.bits(got) != H.bits(want)))
    assert nd == 0, f"{what}: {nd} of {len(want)} logits differ in their bits (rel-L2 {err:.3e})"


@pytest.fixture(scope="module")
def prod():
    H.ensure_built()
    return H.ApiLib(H.LIB)


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    return H.Oracle()


def is_persistent(lib, sess):
    """whether a product session's decode runs as the persistent kernel"""
    lib.ember_state_cuda.restype = ctypes.c_void_p
    lib.ember_state_cuda.argtypes = [ctypes.c_void_p]
    lib.ember_cuda_state_persistent.restype = ctypes.c_int
    lib.ember_cuda_state_persistent.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p)]
    why = ctypes.c_char_p()
    return lib.ember_cuda_state_persistent(lib.ember_state_cuda(sess.s), ctypes.byref(why)) == 1, why.value


@pytest.mark.parametrize("attn", ["fused", "split", "persistent"])
@pytest.mark.parametrize("kv16", [0, 1])
@pytest.mark.parametrize("name", TINY)
def test_tiny_teacher_forced_bitexact(prod, orc, name, kv16, attn, monkeypatch):
    """prefill 24 random ids, then 40 forced forwards: every step's logits equal,
    on each decode path: the captured graphs with one attention kernel per head
    or with the cache split over CTAs, and the persistent kernel (quantized
    models)"""
    if attn == "persistent":
        if name == "tiny-f32":
            pytest.skip("the persistent step serves quantized models")
        monkeypatch.setenv("EMBER_PERSIST", "1")
    else:
        monkeypatch.setenv("EMBER_PERSIST", "0")
        monkeypatch.setenv("EMBER_ATTN", attn)
    path = synth.ensure_model(name)
    a = prod.session(path, 0, kv16)
    assert is_persistent(prod.lib, a)[0] == (attn == "persistent"), is_persistent(prod.lib, a)
    b = orc.session(path, 0, kv16)
    rng = np.random.default_rng(7)
    ids = rng.integers(0, a.vocab, 24)
    assert_same(a.prefill(ids), b.prefill(ids), f"{name} prefill")
    for pos in range(24, 64):
        t = int(rng.integers(0, a.vocab))
        assert_same(a.forward(t, pos), b.forward(t, pos), f"{name} pos {pos}")
    a.close()
    b.close()


@pytest.mark.parametrize("persist", ["0", "1"])
@pytest.mark.parametrize("name", TINY)
def test_tiny_device_greedy_matches_oracle(prod, orc, name, persist, monkeypatch):
    """device-side greedy loop (ember_forward_greedy) = oracle's greedy, on the
    graph step and on the persistent kernel (one launch for the whole run)"""
    monkeypatch.setenv("EMBER_PERSIST", persist)
    from emberllm_b200 import Ember
    path = synth.ensure_model(name)
    rng = np.random.default_rng(3)
    b = orc.session(path)
    prompt = [int(t) for t in rng.integers(0, b.vocab, 16)]
    want = H.greedy_run(b, prompt, 48)
    b.close()
    e = Ember(path)
    got = e.generate_ids(prompt, 48)
    e.close()
    assert got == want


@pytest.mark.parametrize("name,fused", [("tiny-llama", 1), ("tiny-smol-q4", 1), ("tiny-f32", 0),
                                        ("qwen3-0.6b", 1)])
def test_greedy_token_runs_the_fused_head(prod, name, fused, monkeypatch):
    """a quantized lm_head streams through the head kernel whose epilogue picks
    the token (no separate argmax launch); an fp32 head keeps the tiled GEMV and
    the argmax kernel"""
    monkeypatch.setenv("EMBER_PERSIST", "0")
    from emberllm_b200 import Ember
    e = Ember(synth.ensure_model(name), ctx=32)
    e.generate_ids([1, 2, 3], 3)
    e.forward(4, 6)
    cs = e.lib.ember_state_cuda(e.st)
    per_step = e.lib.ember_cuda_state_launches_per_step(cs)
    per_token = e.lib.ember_cuda_state_launches_per_token(cs)
    e.close()
    assert per_token == per_step + (1 - fused)


def _random_matrix(rng, rows, cols, dtype, orc):
    w = (rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    if dtype == 0:
        return w.tobytes()
    nb = cols // 32
    blk = 34 if dtype == 1 else 18
    out = np.empty(rows * nb * blk, np.uint8)
    fn = orc.lib.orc_quantize_q8_0 if dtype == 1 else orc.lib.orc_quantize_q4_0
    fn(w.ctypes.data, out.ctypes.data, rows * cols)
    return out.tobytes()


@pytest.mark.parametrize("dtype", [0, 1, 2])
@pytest.mark.parametrize("shape", [(96, 64), (1024, 1024), (3072, 1024), (1024, 3072), (4864, 896)])
def test_op_matmul_matches_reference_op(prod, orc, dtype, shape):
    """ember_matmul on the GPU vs the CPU matmul (oracle op, pinned to the
    reference's ember_matmul): outputs and the quantized activation bit-exact"""
    rows, cols = shape
    rng = np.random.default_rng(rows * 7 + cols + dtype)
    w = _random_matrix(rng, rows, cols, dtype, orc)
    x = rng.standard_normal(cols).astype(np.float32) * 0.5
    x[::17] = 0.0
    out_g = np.zeros(rows, np.float32)
    out_c = np.zeros(rows, np.float32)
    xq_g = np.zeros((cols // 32 + 1) * 34, np.uint8)
    xq_c = np.zeros_like(xq_g)
    wb = ctypes.create_string_buffer(w, len(w))
    prod.lib.ember_matmul(out_g.ctypes.data, x.ctypes.data, wb, dtype, cols, rows, xq_g.ctypes.data)
    orc.lib.orc_matmul(out_c.ctypes.data, x.ctypes.data, wb, dtype, cols, rows, xq_c.ctypes.data)
    assert np.array_equal(H.bits(out_g), H.bits(out_c))
    if dtype != 0:
        assert np.array_equal(xq_g, xq_c)


def test_op_matmul_batch(prod, orc):
    rng = np.random.default_rng(11)
    rows, cols, B = 256, 512, 5
    w = _random_matrix(rng, rows, cols, 1, orc)
    x = rng.standard_normal((B, cols)).astype(np.float32)
    out_g = np.zeros((B, rows), np.float32)
    xq_g = np.zeros(B * (cols // 32) * 34, np.uint8)
    wb = ctypes.create_string_buffer(w, len(w))
    prod.lib.ember_matmul_batch(out_g.ctypes.data, x.ctypes.data, wb, 1, cols, rows, B, xq_g.ctypes.data)
    for b in range(B):
        want = np.zeros(rows, np.float32)
        xq = np.zeros((cols // 32) * 34, np.uint8)
        xb = np.ascontiguousarray(x[b])
        orc.lib.orc_matmul(want.ctypes.data, xb.ctypes.data, wb, 1, cols, rows, xq.ctypes.data)
        assert np.array_equal(H.bits(out_g[b]), H.bits(want))
        assert np.array_equal(xq_g[b * len(xq):(b + 1) * len(xq)], xq)


@pytest.mark.slow
def test_stories110m_greedy_128(prod, orc):
    """BASELINE gate: 128 greedy tokens identical on the stories110M shape
    (prompt 128 uniform random ids), plus the logits of every step bit-exact"""
    path = synth.ensure_model("stories110m")
    rng = np.random.default_rng(1)
    a = prod.session(path, 0, 0)
    b = orc.session(path, 0, 0)
    prompt = [int(t) for t in rng.integers(0, a.vocab, 128)]
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert_same(la, lb, "stories110m prefill")
    pos = 128
    for i in range(128):
        ta, tb = H.first_argmax(la), H.first_argmax(lb)
        assert ta == tb, f"greedy diverged at token {i}"
        la, lb = a.forward(ta, pos), b.forward(tb, pos)
        assert_same(la, lb, f"stories110m step {i}")
        pos += 1
    a.close()
    b.close()


@pytest.mark.slow
@pytest.mark.parametrize("name,prompt_len,steps", [("qwen3-0.6b", 24, 8), ("qwen2.5-0.5b", 24, 8),
                                                   ("smollm2-135m", 64, 32)])
def test_full_size_configs(prod, orc, name, prompt_len, steps):
    """the other BASELINE architectures at full size: prefill + greedy, bit-exact"""
    path = synth.ensure_model(name)
    rng = np.random.default_rng(2)
    a = prod.session(path, 4096, 0)
    b = orc.session(path, 4096, 0)
    prompt = [int(t) for t in rng.integers(0, a.vocab, prompt_len)]
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert_same(la, lb, f"{name} prefill")
    pos = prompt_len
    for i in range(steps):
        ta, tb = H.first_argmax(la), H.first_argmax(lb)
        assert ta == tb, f"{name}: greedy diverged at token {i}"
        la, lb = a.forward(ta, pos), b.forward(tb, pos)
        assert_same(la, lb, f"{name} step {i}")
        pos += 1
    a.close()
    b.close()
