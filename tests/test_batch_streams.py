"""GPU parity of the batched decode of independent streams (ember_batch_*).

BASELINE's many-sequence workload runs 8 x N independent streams, each with its
own prompt and greedy continuation. The library decodes up to 8 streams as
concurrent single-stream states (their step graphs on separate CUDA streams) and
more streams together (one tensor-core GEMM per weight matrix per step, each
stream at its own position in its own cache). Either way the arithmetic per
stream is the single-sequence step's, so every stream must produce exactly the
tokens of its own greedy run, and the last step's logits must equal the oracle's
bit for bit.
"""
import numpy as np
import pytest

from emberllm_b200 import Ember, EmberBatch, synth

from . import helpers as H
from .test_gpu_parity import assert_same

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def orc():
    H.ensure_built()
    return H.Oracle()


def oracle_stream(orc, path, prompt, n_steps, kv16, ctx):
    """the oracle's greedy continuation of one stream: (first token, the next
    n_steps tokens, the logits after the last fed token)"""
    s = orc.session(path, ctx, kv16)
    logits = s.prefill(prompt)
    first = H.first_argmax(logits)
    toks, t, pos = [], first, len(prompt)
    for _ in range(n_steps):
        logits = s.forward(t, pos)
        t = H.first_argmax(logits)
        toks.append(t)
        pos += 1
    s.close()
    return first, toks, logits


def run_batch(path, prompts, n_steps, kv16, ctx):
    e = Ember(path)
    b = EmberBatch(e, len(prompts), ctx=ctx, kv_fp16=kv16, max_steps=n_steps)
    firsts = [b.prefill(i, p) for i, p in enumerate(prompts)]
    toks, lg = b.greedy(firsts, [len(p) for p in prompts], n_steps, logits=True)
    logits = np.ctypeslib.as_array(lg).reshape(len(prompts), e.vocab).copy()
    b.close()
    e.close()
    return firsts, toks, logits


@pytest.mark.parametrize("mode", ["replicas", "gemm", "gemm-head", "gemm-tile", "gemm-swap"])
@pytest.mark.parametrize("kv16", [0, 1])
@pytest.mark.parametrize("name", ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-smol-q4", "tiny-mqa"])
def test_tiny_streams_match_single_sequence_runs(orc, name, kv16, mode, monkeypatch):
    """five streams with prompts of 1..30 tokens, 12 steps together; up to 8
    streams run as concurrent single-stream states unless EMBER_BATCH=gemm
    forces the batched GEMM path, whose attention runs per (kv head, stream)
    (attn_batch_kernel), per (query head, stream) with EMBER_BATCH_ATTN=head
    (attn_decode_kernel) or, with =tile, as the prefill's token-tile kernel, and
    whose GEMMs may swap operands (EMBER_PF_SWAP=1)"""
    if mode.startswith("gemm"):
        monkeypatch.setenv("EMBER_BATCH", "gemm")
    else:
        monkeypatch.delenv("EMBER_BATCH", raising=False)
    if mode in ("gemm-tile", "gemm-head"):
        monkeypatch.setenv("EMBER_BATCH_ATTN", mode[5:])
    else:
        monkeypatch.delenv("EMBER_BATCH_ATTN", raising=False)
    if mode == "gemm-swap":   # the opt-in swapped-operand GEMM
        monkeypatch.setenv("EMBER_PF_SWAP", "1")
    else:
        monkeypatch.delenv("EMBER_PF_SWAP", raising=False)
    path = synth.ensure_model(name)
    vocab = H.header_of(path)["vocab_size"]
    rng = np.random.default_rng(31 + kv16)
    prompts = [[int(t) for t in rng.integers(0, vocab, n)] for n in (3, 9, 17, 1, 30)]
    n_steps, ctx = 12, 64
    firsts, toks, logits = run_batch(path, prompts, n_steps, kv16, ctx)
    for i, p in enumerate(prompts):
        f, want, want_logits = oracle_stream(orc, path, p, n_steps, kv16, ctx)
        assert firsts[i] == f, f"{name} stream {i}: first token"
        assert [toks[s][i] for s in range(n_steps)] == want, f"{name} stream {i}: greedy tokens"
        assert_same(logits[i], want_logits, f"{name} stream {i} last logits")


@pytest.mark.slow
@pytest.mark.parametrize("mode", ["replicas", "gemm"])
def test_qwen3_eight_streams(orc, mode, monkeypatch):
    """the BASELINE streams architecture at full size: 8 streams (configs[4],
    N = 1), 32-token prompts, 16 steps, on both batch paths"""
    if mode == "gemm":
        monkeypatch.setenv("EMBER_BATCH", "gemm")
    else:
        monkeypatch.delenv("EMBER_BATCH", raising=False)
    path = synth.ensure_model("qwen3-0.6b")
    rng = np.random.default_rng(4)
    vocab = H.header_of(path)["vocab_size"]
    prompts = [[int(t) for t in rng.integers(0, vocab, 32)] for _ in range(8)]
    n_steps, ctx = 16, 64
    firsts, toks, logits = run_batch(path, prompts, n_steps, 0, ctx)
    for i, p in enumerate(prompts):
        f, want, want_logits = oracle_stream(orc, path, p, n_steps, 0, ctx)
        assert firsts[i] == f and [toks[s][i] for s in range(n_steps)] == want, f"stream {i}"
        assert_same(logits[i], want_logits, f"qwen3 stream {i} last logits")


def _single_stream_run(e, prompt, n_steps):
    """the single-sequence device path (pinned to the oracle elsewhere): prefill,
    first pick, then ember_forward_greedy; returns (first, tokens, last logits)"""
    import ctypes
    lg = np.ctypeslib.as_array(e.prefill(prompt), (e.vocab,)).copy()
    first = H.first_argmax(lg)
    out = (ctypes.c_int * n_steps)()
    p = e.lib.ember_forward_greedy(e.m, e.st, first, len(prompt), n_steps, out)
    return first, list(out), np.ctypeslib.as_array(p, (e.vocab,)).copy()


@pytest.mark.slow
@pytest.mark.parametrize("kv16", [0, 1])
@pytest.mark.parametrize("n", [16, 64])
def test_qwen3_many_streams(orc, n, kv16, monkeypatch):
    """configs[4] at the per-GPU sizes of 8 x 16 and 8 x 64 streams over 8 GPUs:
    n Qwen3-0.6B streams (prompts of 8..47 tokens) decoded together for 8 steps
    on the batched path; every stream equals its own single-sequence run (tokens
    and last logits, bit for bit), two of them also the oracle's"""
    monkeypatch.delenv("EMBER_BATCH", raising=False)
    monkeypatch.delenv("EMBER_BATCH_ATTN", raising=False)
    path = synth.ensure_model("qwen3-0.6b")
    vocab = H.header_of(path)["vocab_size"]
    rng = np.random.default_rng(100 + n)
    prompts = [[int(t) for t in rng.integers(0, vocab, 8 + (7 * i) % 40)] for i in range(n)]
    n_steps, ctx = 8, 64
    firsts, toks, logits = run_batch(path, prompts, n_steps, kv16, ctx)
    e = Ember(path, ctx=ctx, kv_fp16=bool(kv16))
    for i, p in enumerate(prompts):
        f, want, want_logits = _single_stream_run(e, p, n_steps)
        assert firsts[i] == f and [toks[s][i] for s in range(n_steps)] == want, f"stream {i}"
        assert_same(logits[i], want_logits, f"qwen3 stream {i} of {n} last logits")
    e.close()
    for i in (0, n - 1):
        f, want, _ = oracle_stream(orc, path, prompts[i], n_steps, kv16, ctx)
        assert firsts[i] == f and [toks[s][i] for s in range(n_steps)] == want, f"stream {i} vs oracle"
