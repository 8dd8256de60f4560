"""The RoPE table the host builds for the device (ember_host_rope_table) holds,
bit for bit, the cos/sin values the reference evaluates inside rope() (ref
src/model.c:66-80): freq = 1/powf(theta, (2i)/hd) and val = pos*freq in float,
then cosf/sinf of this machine's C library. Restated here with numpy float32
arithmetic and the C library's own powf/cosf/sinf."""
import ctypes

import numpy as np
import pytest

from emberllm_b200 import _lib

from . import helpers as H


@pytest.fixture(scope="module")
def lib():
    H.ensure_built()
    return _lib.load()


def libm():
    m = ctypes.CDLL("libm.so.6")
    for f in ("powf", "cosf", "sinf"):
        getattr(m, f).restype = ctypes.c_float
    m.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    m.cosf.argtypes = m.sinf.argtypes = [ctypes.c_float]
    return m


@pytest.mark.parametrize("ctx,hd,theta", [(1024, 64, 10000.0), (2048, 128, 1e6), (700, 64, 100000.0),
                                          (64, 32, 10000.0)])
def test_rope_table_equals_the_reference_expressions(lib, ctx, hd, theta):
    m = libm()
    half = hd // 2
    out = np.zeros((ctx, half, 2), np.float32)
    lib.ember_host_rope_table(out.ctypes.data, ctx, hd, theta)
    f32 = np.float32
    freq = [f32(1.0) / f32(m.powf(theta, float(f32(2 * i) / f32(hd)))) for i in range(half)]
    for pos in range(ctx):
        for i in range(half):
            val = f32(pos) * freq[i]
            want = (f32(m.cosf(float(val))), f32(m.sinf(float(val))))
            got = out[pos, i]
            assert got[0].view(np.uint32) == want[0].view(np.uint32) and \
                got[1].view(np.uint32) == want[1].view(np.uint32), (pos, i, got, want)
