"""The device expf recipe (csrc/expf_core.h), evaluated on the host with the same
bits, must equal this machine's C library expf for every float input. The
exception table is built by a full scan; here it is checked on the table's own
entries, on neighbourhoods of them, on random inputs and on the range ends."""
import ctypes

import numpy as np
import pytest

from emberllm_b200 import _lib

from . import helpers as H


class Params(ctypes.Structure):
    """EmberExpfParams (include/ember_cuda.h)"""
    _fields_ = [("coef", ctypes.c_double * 6), ("inv_step", ctypes.c_double),
                ("step_hi", ctypes.c_double), ("step_lo", ctypes.c_double),
                ("shifter", ctypes.c_double), ("window", ctypes.c_uint32),
                ("lo", ctypes.c_float), ("hi", ctypes.c_float),
                ("n_slots", ctypes.c_uint32), ("n_entries", ctypes.c_uint32),
                ("tab", ctypes.POINTER(ctypes.c_double)),
                ("slots", ctypes.POINTER(ctypes.c_uint32))]


@pytest.fixture(scope="module")
def params():
    H.ensure_built()
    lib = _lib.load()
    p = Params()
    assert lib.ember_host_expf_params(ctypes.byref(p)) == 0
    lib.ember_host_expf_emulated.restype = ctypes.c_float
    lib.ember_host_expf_emulated.argtypes = [ctypes.POINTER(Params), ctypes.c_float]
    return lib, p


def _glibc():
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    return libm.expf


def _check(lib, p, xs):
    expf = _glibc()
    bad = []
    for x in xs:
        a = lib.ember_host_expf_emulated(ctypes.byref(p), float(x))
        b = expf(float(x))
        if np.float32(a).view(np.uint32) != np.float32(b).view(np.uint32):
            bad.append(float(x))
    return bad


def test_table_is_nontrivial(params):
    _, p = params
    assert p.n_entries > 1000               # the library's expf is not correctly rounded
    assert p.n_slots >= 2 * p.n_entries     # at most half full
    assert 0 < p.window < (1 << 29) // 100  # a small fraction of an ulp


def test_listed_inputs_and_neighbours(params):
    lib, p = params
    keys = np.array([p.slots[2 * i] for i in range(p.n_slots)], np.uint32)
    keys = keys[keys != 0xFFFFFFFF]
    rng = np.random.default_rng(0)
    pick = rng.choice(keys, 3000, replace=False)
    xs = np.concatenate([pick, pick + 1, pick - 1]).astype(np.uint32).view(np.float32)
    assert _check(lib, p, xs) == []


def test_random_inputs_over_the_used_range(params):
    lib, p = params
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.uniform(-110, 95, 60000), rng.standard_normal(20000) * 3,
                         rng.standard_normal(5000) * 1e-3]).astype(np.float32)
    assert _check(lib, p, xs) == []


def test_range_ends_and_specials(params):
    lib, p = params
    f = np.float32
    xs = [f(-105.0), np.nextafter(f(-105.0), f(0)), f(-103.97), f(-103.28), f(-87.3),
          f(88.72), f(88.7228), np.nextafter(f(90.0), f(0)), f(90.0), f(0.0), f(-0.0),
          f(1e-30), f(-1e-30), f(np.inf), f(-np.inf)]
    assert _check(lib, p, xs) == []
