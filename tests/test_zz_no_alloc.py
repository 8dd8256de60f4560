"""The allocation-free greedy pick, ember_cuda_argmax_static.

It exists for programs that cannot let this library allocate device memory (a
host that owns the GPU through its own memory pool, or a per-token path that
must not risk cudaMalloc's synchronisation). It works only on buffers the
caller owns -- device logits in, one device int out -- and keeps its scratch in
a fixed array inside the library.

The first test calls it through the C ABI on the logits the existing entry point
left on the device (ember_forward_greedy, whose argmax uses scratch allocated
in the run state) and requires the same token, on two calls in a row (the
shared scratch keeps the previous call's contents). Integer indices: the
comparison is exact. Further tests spread the pick over many blocks (the
partials are merged through the shared scratch) and compare it with the
reference's loop, including its NaN and -inf cases. This file sorts last so that
a run stopping at the first failure has already run every other test.
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


def _ref_pick(v):
    """the reference's loop (src/sample.c:114-118), through the oracle's copy"""
    from . import helpers as H
    o = H.Oracle()
    a = np.ascontiguousarray(v, np.float32)
    return int(o.lib.orc_argmax(a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(a)))


def _cases(n, rng):
    """(name, vector): the maximum in the last block, a tie across two blocks,
    runs of -inf and NaN, a NaN at index 0, all -inf"""
    base = rng.standard_normal(n).astype(np.float32)
    out = []
    v = base.copy(); v[n - 1] = 50.0
    out.append(("max at the end", v))
    v = base.copy(); v[n // 3] = 40.0; v[n - 5] = 40.0; v[n // 3 + 1024 * 7 + 3] = 40.0
    out.append(("tie across blocks", v))
    v = base.copy(); v[: n // 2] = -np.inf; v[n // 2: n // 2 + 4096] = np.nan; v[n - 2] = 7.0
    out.append(("-inf and NaN runs", v))
    v = base.copy(); v[0] = np.nan; v[n // 2] = 60.0
    out.append(("NaN at index 0", v))
    v = np.full(n, -np.inf, np.float32)
    out.append(("all -inf", v))
    return out


@pytest.mark.parametrize("n", [151936, 1 << 26])
def test_multi_block_merge_matches_reference_rule(lib, n):
    """sizes that spread over many blocks, so the partials in the shared scratch
    are merged by the last block; each case runs twice in a row (the scratch and
    its ticket carry the previous call's contents)"""
    import torch
    rng = np.random.default_rng(n % 1000)
    idx = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    for name, v in _cases(n, rng):
        want = _ref_pick(v)
        dev = torch.from_numpy(v).to("cuda:0")
        for rep in range(2):
            idx.fill_(-1)
            assert lib.ember_cuda_argmax_static(dev.data_ptr(), n, idx.data_ptr(), None) == 0
            torch.cuda.synchronize()
            assert int(idx.item()) == want, (name, rep, int(idx.item()), want)
        del dev


def test_keeps_the_callers_current_device_and_checks_the_output(lib, capfd):
    import torch
    buf = torch.zeros(8, dtype=torch.float32, device="cuda:0")
    host_out = (ctypes.c_int * 1)()
    # a host pointer as the output is refused, not written through
    assert lib.ember_cuda_argmax_static(buf.data_ptr(), 8, ctypes.addressof(host_out), None) == 2
    assert "out_index" in capfd.readouterr().err
    idx = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    assert lib.ember_cuda_argmax_static(buf.data_ptr(), 8, idx.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert torch.cuda.current_device() == 0
