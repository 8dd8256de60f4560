"""The greedy pick when logit 0 is NaN, on every device picker.

The reference's argmax (src/sample.c:114-118) starts from best = 0 and moves only
when v[i] > v[best]; nothing compares greater than NaN, so a NaN at index 0 keeps
index 0 whatever follows. A model whose lm_head row 0 has a NaN scale gives NaN
as logit 0 at every step: the oracle then picks 0 every step, and so must the
device greedy loop (argmax_advance) and the batched streams (batch_argmax).
"""
import os
import shutil
import struct

import numpy as np
import pytest

from emberllm_b200 import Ember, EmberBatch, synth

from . import helpers as H

pytestmark = pytest.mark.gpu


def _nan_head_model(tmp_path):
    """tiny-llama (untied lm_head) with the fp16 scale of lm_head row 0, block 0 set to NaN"""
    src = synth.ensure_model("tiny-llama")
    dst = os.path.join(str(tmp_path), "tiny-llama-nan-head.ember")
    shutil.copyfile(src, dst)
    with open(dst, "r+b") as f:
        raw = f.read(256)
        n_tensors = struct.unpack_from("<i", raw, 76)[0]
        table_off = struct.unpack_from("<Q", raw, 112)[0]
        f.seek(table_off)
        table = f.read(n_tensors * 88)
        for i in range(n_tensors):
            name = table[i * 88:i * 88 + 48].split(b"\0")[0].decode()
            if name == "lm_head":
                dtype = struct.unpack_from("<i", table, i * 88 + 48)[0]
                off = struct.unpack_from("<Q", table, i * 88 + 72)[0]
                assert dtype == synth.DT_Q8_0
                f.seek(off)
                f.write(struct.pack("<H", 0x7E00))   # quiet NaN in fp16
                break
        else:
            raise AssertionError("no lm_head tensor")
    return dst


def test_nan_at_index_zero_picks_zero(tmp_path):
    H.ensure_built()
    path = _nan_head_model(tmp_path)
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, 512, 12)]
    o = H.Oracle().session(path)
    lo = o.prefill(prompt)
    assert np.isnan(lo[0])
    want = []
    pos = len(prompt)
    for _ in range(6):
        t = int(o.lib.orc_argmax(lo.ctypes.data_as(H._FP), len(lo)))
        want.append(t)
        lo = o.forward(t, pos)
        pos += 1
    o.close()
    assert want == [0] * 6
    # device greedy: argmax_advance after the lm_head GEMV
    e = Ember(path)
    lg = np.ctypeslib.as_array(e.prefill(prompt), (e.vocab,)).copy()
    assert np.isnan(lg[0])
    got = e.greedy(0, len(prompt), 5)
    assert got == want[1:]
    # batched streams on the tensor-core path: batch_argmax per stream
    os.environ["EMBER_BATCH"] = "gemm"
    try:
        b = EmberBatch(e, 2, ctx=64, max_steps=8)
        for i in range(2):
            b.prefill(i, prompt)
        toks = b.greedy([0, 0], [len(prompt)] * 2, 4)
        b.close()
    finally:
        del os.environ["EMBER_BATCH"]
    assert toks == [[0, 0]] * 4
    e.close()
