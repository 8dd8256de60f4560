"""Failure detection, in the forms that fault no GPU.

1. Invalid input dies on the host before any launch, with the reference's fatal
   convention and message (ref src/model.c:368-371, src/util.c:8-16): a token id
   or a position out of range ends the process with status 1 and
   `ember: token id T out of range [0,V)` / `ember: position P out of range
   [0,C)` on stderr. Each case runs in a child process against this library
   and against the reference's own build, and the two must agree.
2. A bounded device wait that runs out: the wait helper of the kernels (a flag
   that nothing sets, a short limit) gives up, records its code in the error
   word and returns; the host reads the status and the context stays usable.
"""
import os
import subprocess
import sys

import pytest

from emberllm_b200 import synth

from . import helpers as H

ROOT = H.ROOT

CHILD = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
lib.ember_model_load.restype = ctypes.c_void_p
lib.ember_model_load.argtypes = [ctypes.c_char_p]
lib.ember_state_new_ex.restype = ctypes.c_void_p
lib.ember_state_new_ex.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
lib.ember_forward.restype = ctypes.c_void_p
lib.ember_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
m = lib.ember_model_load(sys.argv[2].encode())
s = lib.ember_state_new_ex(m, int(sys.argv[3]), 0)
print("state ok", flush=True)
lib.ember_forward(m, s, int(sys.argv[4]), int(sys.argv[5]))
print("returned", flush=True)
"""


def _run(lib_path, model, ctx, tok, pos):
    r = subprocess.run([sys.executable, "-c", CHILD, lib_path, model, str(ctx), str(tok), str(pos)],
                       capture_output=True, text=True, timeout=300)
    return r.returncode, r.stdout, r.stderr.strip().splitlines()[-1] if r.stderr.strip() else ""


CASES = [(-1, 3), (640, 3), (100000, 0), (5, -1), (5, 48), (5, 4096)]


@pytest.mark.gpu
@pytest.mark.parametrize("tok,pos", CASES)
def test_out_of_range_token_or_position_dies_like_the_reference(tok, pos):
    H.ensure_built()
    model = synth.ensure_model("tiny-qwen3")
    rc, out, err = _run(H.LIB, model, 48, tok, pos)
    assert "state ok" in out and "returned" not in out
    assert rc == 1, (rc, err)
    kind = "token id %d out of range [0,640)" % tok if not 0 <= tok < 640 else \
        "position %d out of range [0,48)" % pos
    assert err == "ember: " + kind, err
    if H.have_reference():
        rrc, rout, rerr = _run(H.REF_DET, model, 48, tok, pos)
        assert (rrc, rerr) == (rc, err), (rrc, rerr)


@pytest.mark.gpu
@pytest.mark.parametrize("mode,code", [(0, 1), (1, 11)])
def test_device_wait_runs_out_reports_and_the_context_stays_usable(mode, code):
    """mode 0: the copies' mbarrier wait on a barrier nothing completes; mode 1:
    the persistent step's tagged hand-off wait on a word nothing writes. Each,
    bounded to a few thousand tries, returns failure and records its code
    (ERR_GEMV_WAIT = 1, ERR_P_HANDOFF = 11) in the error word; the GPU then
    runs the next work normally (a greedy run equal to the oracle's)."""
    import ctypes
    import numpy as np
    from emberllm_b200 import Ember
    hooks = H.testhooks()
    ok, err, ms = ctypes.c_int(-1), ctypes.c_int(-1), ctypes.c_float(-1)
    assert hooks.ember_testhook_wait_timeout(mode, 4000, ctypes.byref(ok), ctypes.byref(err), ctypes.byref(ms)) == 0
    assert ok.value == 0, "the wait reported success on a barrier nothing completes"
    assert err.value == code
    assert 0.0 <= ms.value < 5000.0
    path = synth.ensure_model("tiny-llama")
    prompt = [int(t) for t in np.random.default_rng(9).integers(0, 512, 10)]
    o = H.Oracle().session(path)
    want = H.greedy_run(o, prompt, 8)
    o.close()
    e = Ember(path)
    assert e.generate_ids(prompt, 8) == want
    e.close()
