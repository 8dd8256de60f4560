"""The loader is a drop-in for the reference's (ref src/io.c:30-96): the same
files load, the same malformed files are refused, in the same order of checks
and with the same message on stderr. Each case loads one file through this
library and through the reference's own build (oracle/_ref), each in a fresh
process, and compares what they print."""
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from emberllm_b200 import synth
from emberllm_b200._lib import EmberHeader

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OURS = os.path.join(ROOT, "emberllm_b200", "libember_b200.so")
REF = os.path.join(ROOT, "oracle", "_ref", "libember_ref_det.so")

pytestmark = pytest.mark.skipif(not os.path.exists(REF), reason="the reference's build (oracle/_ref) is absent")

# load the file, then (if it loaded) look a tensor up and ask for its data
SNIPPET = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
lib.ember_model_load.restype = ctypes.c_void_p
lib.ember_model_tensor.restype = ctypes.c_void_p
lib.ember_model_tensor.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
lib.ember_model_data.restype = ctypes.c_void_p
lib.ember_model_data.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
m = lib.ember_model_load(sys.argv[2].encode())
print("loaded", bool(m))
if m:
    t = lib.ember_model_tensor(m, sys.argv[3].encode())
    print("tensor", bool(t))
    if t:
        print("data", bool(lib.ember_model_data(m, t)))
"""


def field(name):
    """(offset, struct format) of a header field"""
    f = getattr(EmberHeader, name)
    fmt = {1: "<B", 4: "<i", 8: "<Q"}[f.size]
    if name in ("version", "flags"):
        fmt = "<I"
    return f.offset, fmt


def patched(data, name, value):
    off, fmt = field(name)
    return data[:off] + struct.pack(fmt, value) + data[off + struct.calcsize(fmt):]


def table_entry_offset(data, name):
    """byte offset of tensor `name`'s entry in the tensor table"""
    h = EmberHeader.from_buffer_copy(data[:256])
    for i in range(h.n_tensors):
        at = h.tensor_table_offset + 88 * i
        if data[at:at + 48].rstrip(b"\0") == name.encode():
            return at
    raise KeyError(name)


def cases():
    good = open(synth.ensure_model("tiny-llama"), "rb").read()
    h = EmberHeader.from_buffer_copy(good[:256])
    size = len(good)
    ent = table_entry_offset(good, "layers.0.wq")
    # entry: name[48], dtype, ndim, shape[4], offset (byte 72), nbytes (byte 80)
    data_out = good[:ent + 72] + struct.pack("<Q", size - 16) + good[ent + 80:]
    return {
        "valid": good,
        "empty": b"",
        "truncated": good[:200],
        "random": np.random.default_rng(0).integers(0, 256, 4096, dtype=np.uint8).tobytes(),
        "magic": b"EMBX" + good[4:],
        "version": patched(good, "version", 2),
        "dim": patched(good, "dim", 0),
        "layers": patched(good, "n_layers", -1),
        "vocab": patched(good, "vocab_size", 0),
        "ntensors": patched(good, "n_tensors", -1),
        "table_offset": patched(good, "tensor_table_offset", size + 8),
        "table_size": patched(good, "tensor_table_size", size - h.tensor_table_offset + 1),
        "table_short": patched(good, "tensor_table_size", 88 * h.n_tensors - 1),
        "tok_offset": patched(good, "tokenizer_offset", size + 1),
        "tok_size": patched(good, "tokenizer_size", size - h.tokenizer_offset + 1),
        "data_out": data_out,
    }


def run(lib, path, tensor="layers.0.wq"):
    r = subprocess.run([sys.executable, "-c", SNIPPET, lib, path, tensor], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout, r.stderr


@pytest.mark.parametrize("case", ["valid", "empty", "truncated", "random", "magic", "version", "dim", "layers",
                                  "vocab", "ntensors", "table_offset", "table_size", "table_short",
                                  "tok_offset", "tok_size", "data_out"])
def test_same_verdict_and_message_as_the_reference(tmp_path, case):
    p = tmp_path / (case + ".ember")
    p.write_bytes(cases()[case])
    ours, ref = run(OURS, str(p)), run(REF, str(p))
    assert ours == ref, (case, ours, ref)
    if case == "valid":
        assert ours[0] == "loaded True\ntensor True\ndata True\n"
    elif case == "data_out":
        assert ours[0] == "loaded True\ntensor True\ndata False\n" and "tensor data out of bounds" in ours[1]
    else:
        assert ours[0] == "loaded False\n" and ours[1].startswith("ember: ")


def test_missing_file_and_unknown_tensor(tmp_path):
    assert run(OURS, str(tmp_path / "none.ember")) == run(REF, str(tmp_path / "none.ember"))
    path = synth.ensure_model("tiny-llama")
    ours = run(OURS, path, "layers.7.wq")
    assert ours == run(REF, path, "layers.7.wq")
    assert ours[0] == "loaded True\ntensor False\n"


STATE_SNIPPET = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
lib.ember_model_load.restype = ctypes.c_void_p
lib.ember_state_new.restype = ctypes.c_void_p
lib.ember_state_new.argtypes = [ctypes.c_void_p, ctypes.c_int]
m = lib.ember_model_load(sys.argv[2].encode())
print("loaded", bool(m), flush=True)
lib.ember_state_new(m, 64)
"""


@pytest.mark.parametrize("model,tensor", [("tiny-llama", "layers.1.wq"), ("tiny-llama", "final_norm"),
                                          ("tiny-llama", "tok_embeddings"), ("tiny-qwen3", "layers.0.attn_norm"),
                                          ("tiny-qwen3", "layers.1.w2")])
def test_missing_tensor_dies_like_the_reference(tmp_path, model, tensor):
    """ref src/model.c:161-171: state creation resolves every tensor and dies with
    the reference's message on the first one missing (here before any device work)"""
    good = open(synth.ensure_model(model), "rb").read()
    at = table_entry_offset(good, tensor)
    bad = good[:at] + b"missing_" + good[at + 8:]     # rename the entry
    p = tmp_path / "missing.ember"
    p.write_bytes(bad)
    got = {}
    for lib in (OURS, REF):
        r = subprocess.run([sys.executable, "-c", STATE_SNIPPET, lib, str(p)], capture_output=True, text=True,
                           timeout=120)
        got[lib] = (r.returncode, r.stdout, r.stderr)
    assert got[OURS] == got[REF], got
    assert got[OURS][0] == 1 and got[OURS][2].startswith("ember: ")
