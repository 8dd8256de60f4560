"""The allocation-free greedy pick, ember_cuda_argmax_static.

It exists for programs that cannot let this library allocate device memory (a
host that owns the GPU through its own memory pool, or a per-token path that
must not risk cudaMalloc's synchronisation). It works only on buffers the
caller owns -- device logits in, one device int out -- and keeps its scratch in
a fixed array inside the library.

The test calls it through the C ABI on the logits the existing entry point
left on the device (ember_forward_greedy, whose argmax uses scratch allocated
in the run state) and requires the same token, on two calls in a row (the
shared scratch keeps the previous call's contents). Integer indices: the
comparison is exact. This file sorts last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from emberllm_b200 import _lib, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from . import helpers as H
    H.ensure_built()
    lib = _lib.load()
    lib.ember_cuda_argmax_static.restype = ctypes.c_int
    lib.ember_cuda_argmax_static.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                             ctypes.c_void_p]
    return lib


def test_matches_existing_greedy_on_two_calls(lib):
    import torch
    path = synth.ensure_model("tiny-qwen3")
    m = lib.ember_model_load(path.encode())
    s = lib.ember_state_new_ex(m, 0, 0)
    cs = lib.ember_state_cuda(s)
    vocab = lib.ember_model_header(m).contents.vocab_size
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    picks = []
    for tok, pos in [(5, 0), (17, 1)]:
        # existing entry point: one device greedy step at (tok, pos)
        chosen = (ctypes.c_int * 1)()
        host = lib.ember_forward_greedy(m, s, tok, pos, 1, chosen)
        want = chosen[0]
        host_logits = np.ctypeslib.as_array(host, (vocab,)).copy()
        assert want == int(np.argmax(host_logits))          # first index of the max
        # the new entry point, on the same logits still on the device
        rc = lib.ember_cuda_argmax_static(lib.ember_cuda_state_logits_dev(cs), vocab,
                                          out.data_ptr(), lib.ember_cuda_state_stream(cs))
        assert rc == 0
        torch.cuda.synchronize()
        got = int(out.item())
        assert got == want, (got, want)
        picks.append(got)
        out.fill_(-1)
    lib.ember_state_free(s)
    lib.ember_model_free(m)
    assert len(picks) == 2


def test_rejects_sizes_beyond_the_limit(lib, capfd):
    import torch
    buf = torch.zeros(4, dtype=torch.float32, device="cuda:0")
    idx = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    assert lib.ember_cuda_argmax_static(buf.data_ptr(), (1 << 26) + 1, idx.data_ptr(), None) == 1
    assert lib.ember_cuda_argmax_static(buf.data_ptr(), 0, idx.data_ptr(), None) == 1
    err = capfd.readouterr().err
    assert "outside the supported range" in err
    # a valid call after the rejected ones still works
    buf[2] = 3.0
    assert lib.ember_cuda_argmax_static(buf.data_ptr(), 4, idx.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert int(idx.item()) == 2
