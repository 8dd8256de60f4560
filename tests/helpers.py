"""Test helpers: build-on-demand and ctypes access to the three libraries.

  product   emberllm_b200/libember_b200.so      (the thing under test)
  hooks     emberllm_b200/libember_testhooks.so (device helpers run alone, test-only)
  oracle    oracle/liboracle.so                 (our C restatement, test-only)
  reference oracle/_ref/libember_ref_det.so     (emberllm compiled from its own
                                                 sources with its deterministic
                                                 flags; present where it was built)
"""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "emberllm_b200", "libember_b200.so")
HOOKS = os.path.join(ROOT, "emberllm_b200", "libember_testhooks.so")
ORACLE = os.path.join(ROOT, "oracle", "liboracle.so")
REF_DET = os.path.join(ROOT, "oracle", "_ref", "libember_ref_det.so")

_P = ctypes.c_void_p
_FP = ctypes.POINTER(ctypes.c_float)
_IP = ctypes.POINTER(ctypes.c_int)


def ensure_built():
    if not os.path.exists(LIB) or not os.path.exists(HOOKS):
        subprocess.run(["make", "-C", os.path.join(ROOT, "emberllm_b200"), "-j8"], check=True,
                       stdout=subprocess.DEVNULL)
    if not os.path.exists(ORACLE):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True,
                       stdout=subprocess.DEVNULL)


def reference_dir():
    """the reference source tree's location: oracle/Makefile's REF variable"""
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "print-ref"], capture_output=True,
                       text=True)
    return r.stdout.strip() if r.returncode == 0 else ""


def have_reference():
    return os.path.exists(REF_DET)


class ApiLib:
    """The emberllm C API as exported by either the product or the reference."""

    def __init__(self, path):
        self.path = path
        lib = ctypes.CDLL(path)
        lib.ember_model_load.restype = _P
        lib.ember_model_load.argtypes = [ctypes.c_char_p]
        lib.ember_model_free.argtypes = [_P]
        lib.ember_state_new_ex.restype = _P
        lib.ember_state_new_ex.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.ember_state_free.argtypes = [_P]
        lib.ember_forward.restype = _FP
        lib.ember_forward.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
        lib.ember_prefill.restype = _FP
        lib.ember_prefill.argtypes = [_P, _P, _IP, ctypes.c_int, ctypes.c_int]
        lib.ember_matmul.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        lib.ember_matmul_batch.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, _P]
        lib.ember_quantize_q8_0.argtypes = [_P, _P, ctypes.c_int]
        lib.ember_quantize_q4_0.argtypes = [_P, _P, ctypes.c_int]
        lib.ember_quantize_file.restype = ctypes.c_int
        lib.ember_quantize_file.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        lib.ember_f32_to_f16.restype = ctypes.c_uint16
        lib.ember_f32_to_f16.argtypes = [ctypes.c_float]
        lib.ember_f16_to_f32.restype = ctypes.c_float
        lib.ember_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.ember_threads_init.argtypes = [ctypes.c_int]
        self.lib = lib

    def session(self, path, ctx=0, kv_fp16=0):
        return Session(self, path, ctx, kv_fp16)


class Session:
    def __init__(self, api, path, ctx, kv_fp16):
        self.api = api
        self.m = api.lib.ember_model_load(path.encode())
        assert self.m, "model failed to load: " + path
        self.s = api.lib.ember_state_new_ex(self.m, ctx, kv_fp16)
        self.vocab = header_of(path)["vocab_size"]

    def forward(self, tok, pos):
        p = self.api.lib.ember_forward(self.m, self.s, int(tok), int(pos))
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def prefill(self, ids, start=0):
        arr = (ctypes.c_int * len(ids))(*[int(i) for i in ids])
        p = self.api.lib.ember_prefill(self.m, self.s, arr, len(ids), int(start))
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def close(self):
        if self.s:
            self.api.lib.ember_state_free(self.s)
            self.s = None
        if self.m:
            self.api.lib.ember_model_free(self.m)
            self.m = None


class Oracle:
    """oracle/liboracle.so: the C restatement (test infrastructure)."""

    def __init__(self, threads=None):
        lib = ctypes.CDLL(ORACLE)
        lib.orc_load.restype = _P
        lib.orc_load.argtypes = [ctypes.c_char_p]
        lib.orc_free.argtypes = [_P]
        lib.orc_state_new.restype = _P
        lib.orc_state_new.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.orc_state_free.argtypes = [_P]
        lib.orc_forward.restype = _FP
        lib.orc_forward.argtypes = [_P, ctypes.c_int, ctypes.c_int]
        lib.orc_prefill.restype = _FP
        lib.orc_prefill.argtypes = [_P, _IP, ctypes.c_int, ctypes.c_int]
        lib.orc_argmax.restype = ctypes.c_int
        lib.orc_argmax.argtypes = [_FP, ctypes.c_int]
        lib.orc_matmul.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        lib.orc_quantize_q8_0.argtypes = [_P, _P, ctypes.c_int]
        lib.orc_quantize_q4_0.argtypes = [_P, _P, ctypes.c_int]
        lib.orc_f32_to_f16.restype = ctypes.c_uint16
        lib.orc_f32_to_f16.argtypes = [ctypes.c_float]
        lib.orc_expf.restype = ctypes.c_float
        lib.orc_expf.argtypes = [ctypes.c_float]
        lib.orc_set_threads.argtypes = [ctypes.c_int]
        lib.orc_set_threads(threads or min(32, os.cpu_count() or 1))
        self.lib = lib

    def session(self, path, ctx=0, kv_fp16=0):
        return OracleSession(self, path, ctx, kv_fp16)


class OracleSession:
    def __init__(self, orc, path, ctx, kv_fp16):
        self.lib = orc.lib
        self.m = self.lib.orc_load(path.encode())
        assert self.m
        self.s = self.lib.orc_state_new(self.m, ctx, kv_fp16)
        self.vocab = header_of(path)["vocab_size"]

    def forward(self, tok, pos):
        p = self.lib.orc_forward(self.s, int(tok), int(pos))
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def prefill(self, ids, start=0):
        arr = (ctypes.c_int * len(ids))(*[int(i) for i in ids])
        p = self.lib.orc_prefill(self.s, arr, len(ids), int(start))
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def close(self):
        if self.s:
            self.lib.orc_state_free(self.s)
            self.s = None
        if self.m:
            self.lib.orc_free(self.m)
            self.m = None


def header_of(path):
    import struct
    with open(path, "rb") as f:
        raw = f.read(256)
    names = ["dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
             "vocab_size", "max_seq_len"]
    vals = struct.unpack_from("<8i", raw, 16)
    return dict(zip(names, vals))


def first_argmax(v):
    """first index of the strict maximum, as emberllm's greedy sampler picks"""
    return int(np.argmax(v))   # numpy returns the first occurrence of the max


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def greedy_run(sess, prompt, n):
    """prefill the prompt, then n greedy forwards; returns the n chosen tokens"""
    logits = sess.prefill(prompt)
    out = []
    pos = len(prompt)
    for _ in range(n):
        t = first_argmax(logits)
        out.append(t)
        logits = sess.forward(t, pos)
        pos += 1
    return out


def testhooks():
    """libember_testhooks.so with its prototypes (test infrastructure)"""
    ensure_built()
    lib = ctypes.CDLL(HOOKS)
    lib.ember_cuda_split_sum_batch.restype = ctypes.c_int
    lib.ember_cuda_split_sum_batch.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P]
    lib.ember_cuda_psum_batch.restype = ctypes.c_int
    lib.ember_cuda_psum_batch.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P]
    lib.ember_testhook_wait_timeout.restype = ctypes.c_int
    lib.ember_testhook_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_uint, _P, _P, _P]
    lib.ember_testhook_copy_to_device.restype = ctypes.c_int
    lib.ember_testhook_copy_to_device.argtypes = [_P, _P, ctypes.c_ulonglong]
    return lib
