"""GPU parity of the batched prefill (tensor-core GEMM, per-token norms, tiled
attention) against the CPU checkers, through the C ABI.

The reference's ember_prefill (src/model.c:283-360) gives the same bits as n
single-token forwards; the oracle restates it that way. Every comparison here is
bit for bit: logits after the prefill, the cache it leaves (checked through the
logits of later forwards), and the op-level ember_matmul_batch outputs.
"""
import ctypes

import numpy as np
import pytest

from emberllm_b200 import synth

from . import helpers as H
from .test_gpu_parity import _random_matrix, assert_same

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prod():
    H.ensure_built()
    return H.ApiLib(H.LIB)


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    o = H.Oracle()
    o.lib.orc_matmul_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return o


# (rows, cols, columns): rows and K below one tile, ragged tiles, K of every
# BASELINE model (576, 896, 1024, 3072, 4864), column counts that pick each
# token-tile width and leave partial tiles
GEMM_SHAPES = [(96, 96, 2), (300, 576, 33), (1024, 1024, 130), (257, 4864, 64),
               (1152, 896, 512), (1024, 3072, 77), (6144, 1024, 300)]


@pytest.mark.parametrize("dtype", [1, 2])
@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_gemm_matches_reference_batch_matmul(prod, orc, dtype, shape):
    """ember_matmul_batch (tcgen05 int8 GEMM + fp32 block chain) vs the CPU
    ember_matmul_batch: every output bit-exact"""
    rows, cols, B = shape
    rng = np.random.default_rng(rows * 13 + cols * 7 + B + dtype)
    w = _random_matrix(rng, rows, cols, dtype, orc)
    x = (rng.standard_normal((B, cols)) * 0.7).astype(np.float32)
    x[:, ::19] = 0.0
    x[B // 2, :] = 0.0                      # an all-zero column: scale 0, codes 0
    wb = ctypes.create_string_buffer(w, len(w))
    got = np.zeros((B, rows), np.float32)
    want = np.zeros((B, rows), np.float32)
    xq = np.zeros(B * (cols // 32 + 1) * 34, np.uint8)
    prod.lib.ember_matmul_batch(got.ctypes.data, x.ctypes.data, wb, dtype, cols, rows, B, xq.ctypes.data)
    orc.lib.orc_matmul_batch(want.ctypes.data, x.ctypes.data, wb, dtype, cols, rows, B, xq.ctypes.data)
    nd = int(np.count_nonzero(H.bits(got) != H.bits(want)))
    assert nd == 0, f"{nd} of {got.size} outputs differ"


QUANT_TINY = ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-smol-q4", "tiny-mqa"]


@pytest.mark.parametrize("kv16", [0, 1])
@pytest.mark.parametrize("name", QUANT_TINY)
def test_tiny_prefill_lengths_and_continuation(prod, orc, name, kv16):
    """prefills of 2, 17 and 100 tokens, a second prefill continuing at the end
    of the first, then forced forwards over the cache both left"""
    path = synth.ensure_model(name)
    rng = np.random.default_rng(21 + kv16)
    for n in (2, 17, 100):
        a = prod.session(path, 0, kv16)
        b = orc.session(path, 0, kv16)
        ids = [int(t) for t in rng.integers(0, a.vocab, n + 13)]
        assert_same(a.prefill(ids[:n]), b.prefill(ids[:n]), f"{name} prefill {n}")
        assert_same(a.prefill(ids[n:], n), b.prefill(ids[n:], n), f"{name} continued prefill at {n}")
        pos = n + 13
        for i in range(4):
            t = int(rng.integers(0, a.vocab))
            assert_same(a.forward(t, pos + i), b.forward(t, pos + i), f"{name} forward {pos + i}")
        a.close()
        b.close()


@pytest.mark.parametrize("kv16", [0, 1])
def test_long_prefill_chunks(prod, orc, kv16):
    """2100 tokens: five 512-token chunks, softmax denominators past 2048 terms
    (the CTA-parallel exact sum), then forced forwards"""
    path = synth.ensure_model("tiny-long")
    rng = np.random.default_rng(5 + kv16)
    a = prod.session(path, 2200, kv16)
    b = orc.session(path, 2200, kv16)
    ids = [int(t) for t in rng.integers(0, a.vocab, 2100)]
    assert_same(a.prefill(ids), b.prefill(ids), "tiny-long prefill 2100")
    for i in range(3):
        t = int(rng.integers(0, a.vocab))
        assert_same(a.forward(t, 2100 + i), b.forward(t, 2100 + i), f"tiny-long forward {2100 + i}")
    a.close()
    b.close()


@pytest.mark.slow
@pytest.mark.parametrize("name,n", [("smollm2-135m", 512), ("qwen2.5-0.5b", 512), ("qwen3-0.6b", 256)])
def test_full_size_prefill(prod, orc, name, n):
    """the BASELINE prefill workloads (512-token prompts) at full size: logits
    after the prefill and four greedy steps over its cache, bit-exact"""
    path = synth.ensure_model(name)
    rng = np.random.default_rng(1)
    a = prod.session(path, 1024, 0)
    b = orc.session(path, 1024, 0)
    prompt = [int(t) for t in rng.integers(0, a.vocab, n)]
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert_same(la, lb, f"{name} prefill {n}")
    pos = n
    for i in range(4):
        ta, tb = H.first_argmax(la), H.first_argmax(lb)
        assert ta == tb, f"{name}: greedy diverged at token {i}"
        la, lb = a.forward(ta, pos), b.forward(tb, pos)
        assert_same(la, lb, f"{name} step {i}")
        pos += 1
    a.close()
    b.close()


@pytest.mark.parametrize("kv16", [0, 1])
def test_long_context_decode(prod, orc, kv16):
    """decode past 3000 cached positions: the split attention's many position
    splits and the exact parallel softmax denominator, bit-exact"""
    path = synth.ensure_model("tiny-long")
    rng = np.random.default_rng(9 + kv16)
    a = prod.session(path, 4096, kv16)
    b = orc.session(path, 4096, kv16)
    ids = [int(t) for t in rng.integers(0, a.vocab, 3000)]
    assert_same(a.prefill(ids), b.prefill(ids), "tiny-long prefill 3000")
    for i in range(6):
        t = int(rng.integers(0, a.vocab))
        assert_same(a.forward(t, 3000 + i), b.forward(t, 3000 + i), f"tiny-long forward {3000 + i}")
    a.close()
    b.close()
