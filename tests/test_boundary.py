"""The C-ABI boundary on the CPU: the library loads, exports every symbol the
headers declare, keeps the reference's struct layouts and loader behaviour,
and refuses to run the token loop without a GPU (no CPU fallback)."""
import ctypes
import os
import re
import struct
import subprocess
import sys

import numpy as np
import pytest

from emberllm_b200 import _lib, synth

from . import helpers as H

ROOT = H.ROOT
HEADERS = [os.path.join(ROOT, "include", h) for h in ("ember.h", "ember_ops.h", "ember_cuda.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(ember_\w+)\s*\(", text):
            # a declaration is a name followed by '(' at statement level
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    H.ensure_built()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 40
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    listed = set(_lib.PUBLIC_SYMBOLS + _lib.OPS_SYMBOLS + _lib.CUDA_SYMBOLS)
    assert names <= listed | {"ember_cuda_error"}, sorted(names - listed)


def test_struct_layouts():
    assert ctypes.sizeof(_lib.EmberHeader) == 256
    assert _lib.EmberHeader.vocab_size.offset == 40
    assert _lib.EmberHeader.tokenizer_offset.offset == 96
    assert _lib.EmberHeader.reserved.offset == 128


def test_loader_reads_synthetic_model(lib):
    path = synth.ensure_model("tiny-qwen3")
    m = lib.ember_model_load(path.encode())
    assert m
    h = lib.ember_model_header(m).contents
    assert (h.dim, h.n_layers, h.n_heads, h.n_kv_heads, h.head_dim) == (128, 2, 4, 2, 64)
    t = lib.ember_model_tensor(m, b"layers.1.wq")
    assert t
    assert lib.ember_model_data(m, t)
    assert not lib.ember_model_tensor(m, b"layers.9.wq")
    lib.ember_model_free(m)


@pytest.mark.parametrize("blob", ["random", "truncated", "version", "table"])
def test_malformed_files_return_null(lib, tmp_path, blob):
    """reference test 5 (tests/run_tests.sh:75-86): a bad file is refused, not a crash"""
    good = open(synth.ensure_model("tiny-llama"), "rb").read()
    if blob == "random":
        data = np.random.default_rng(0).integers(0, 256, 4096, dtype=np.uint8).tobytes()
    elif blob == "truncated":
        data = good[:200]
    elif blob == "version":
        data = good[:4] + struct.pack("<I", 2) + good[8:]
    else:
        data = good[:112] + struct.pack("<Q", len(good) + 8) + good[120:]
    p = tmp_path / "bad.ember"
    p.write_bytes(data)
    assert not lib.ember_model_load(str(p).encode())


def test_thread_pool_api_is_a_callable_noop(lib):
    lib.ember_threads_init(6)
    assert lib.ember_nthreads() == 6
    lib.ember_threads_shutdown()
    assert lib.ember_nthreads() == 1


def test_fp16_helpers_match_reference_all_halves(lib):
    if not H.have_reference():
        pytest.skip("reference build not present")
    ref = H.ApiLib(H.REF_DET).lib
    for h in range(0, 65536, 1):
        a, b = lib.ember_f16_to_f32(h), ref.ember_f16_to_f32(h)
        if a != a:
            assert b != b
        else:
            assert struct.pack("<f", a) == struct.pack("<f", b), h
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                           for s in (1e-9, 1e-6, 1e-4, 1.0, 1e4, 7e4)])
    vals = np.concatenate([vals, np.array([0.0, -0.0, 65504.0, 65520.0, 2.0 ** -25, 2.0 ** -24,
                                           3 * 2.0 ** -26, np.inf, -np.inf], np.float32)])
    for v in vals:
        assert lib.ember_f32_to_f16(float(v)) == ref.ember_f32_to_f16(float(v)), v


CPU_ONLY = """
import sys
sys.path.insert(0, {root!r})
from emberllm_b200 import _lib, synth
lib = _lib.load()
m = lib.ember_model_load(synth.ensure_model("tiny-llama").encode())
s = lib.ember_state_new_ex(m, 0, 0)
print("state created", bool(s))
"""


def test_no_cpu_fallback_without_gpu(lib):
    """without a usable device the token loop ends the process with the
    reference's fatal-error convention; it never computes on the CPU"""
    if lib.ember_cuda_available():
        pytest.skip("a GPU is present")
    r = subprocess.run([sys.executable, "-c", CPU_ONLY.format(root=ROOT)], capture_output=True,
                       text=True, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 1, r.stdout + r.stderr
    assert "ember: cuda:" in r.stderr
    assert "state created" not in r.stdout
