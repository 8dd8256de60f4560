"""The offline format producer: this library's quantizers and ember_quantize_file
against the reference's (ref src/kernels.c:73-115, src/quant.c:59-125), byte for
byte, and against the oracle restatement where the reference build is absent."""
import os

import numpy as np
import pytest

from emberllm_b200 import _lib, synth

from . import helpers as H


@pytest.fixture(scope="module")
def libs():
    H.ensure_built()
    prod = _lib.load()
    ref = H.ApiLib(H.REF_DET).lib if H.have_reference() else None
    return prod, ref


def _edge_rows(n_blocks=64):
    rng = np.random.default_rng(4)
    rows = [rng.standard_normal(32 * n_blocks).astype(np.float32) * s for s in (0.02, 1.0, 300.0)]
    z = np.zeros(32 * 4, np.float32)
    z[40] = -1.0
    z[70] = 1.0
    z[71] = -1.0                               # tie on |max|: the first one sets Q4's sign
    half = np.full(32, 0.5, np.float32) * np.float32(1 / 127.0) * 127  # exact halves after scaling
    rows += [z, half, np.linspace(-1, 1, 32 * 8, dtype=np.float32)]
    return rows


@pytest.mark.parametrize("kind", ["q8", "q4"])
def test_block_quantizers_bitexact(libs, kind):
    prod, ref = libs
    orc = H.Oracle().lib
    for x in _edge_rows():
        n = len(x)
        blk = 34 if kind == "q8" else 18
        a = np.zeros(n // 32 * blk, np.uint8)
        c = np.zeros_like(a)
        getattr(prod, "ember_quantize_%s_0" % kind)(x.ctypes.data, a.ctypes.data, n)
        getattr(orc, "orc_quantize_%s_0" % kind)(x.ctypes.data, c.ctypes.data, n)
        assert np.array_equal(a, c)
        if ref is not None:
            b = np.zeros_like(a)
            getattr(ref, "ember_quantize_%s_0" % kind)(x.ctypes.data, b.ctypes.data, n)
            assert np.array_equal(a, b)


@pytest.mark.skipif(not H.have_reference(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("target", [1, 2])
def test_quantize_file_byte_identical_to_reference(libs, tmp_path, target):
    prod, ref = libs
    src = str(tmp_path / "f32.ember")
    synth.write_model(src, synth.CONFIGS["tiny-qwen2"], seed=3, quant="f32")
    a, b = str(tmp_path / "ours.ember"), str(tmp_path / "ref.ember")
    assert prod.ember_quantize_file(src.encode(), a.encode(), target) == 0
    assert ref.ember_quantize_file(src.encode(), b.encode(), target) == 0
    assert open(a, "rb").read() == open(b, "rb").read()


def test_synthetic_writer_equals_quantize_file_of_f32(libs, tmp_path):
    """writing a quantized model directly = writing fp32 then `ember quantize`"""
    prod, _ = libs
    cfg = synth.CONFIGS["tiny-smol-q4"]
    f32 = str(tmp_path / "f.ember")
    synth.write_model(f32, cfg, seed=0, quant="f32")
    q = str(tmp_path / "q.ember")
    assert prod.ember_quantize_file(f32.encode(), q.encode(), 2) == 0
    direct = str(tmp_path / "d.ember")
    synth.write_model(direct, cfg, seed=0, quant="q4_0")
    assert open(q, "rb").read() == open(direct, "rb").read()


def test_weight_bytes_per_token_matches_the_stated_figures():
    # algorithmic weight bytes per decoded token: stories110M 116.4 MB, Qwen3 633.5 MB
    s = synth.weight_bytes_per_token(synth.CONFIGS["stories110m"]) / 1e6
    q = synth.weight_bytes_per_token(synth.CONFIGS["qwen3-0.6b"]) / 1e6
    assert abs(s - 116.4) < 0.5 and abs(q - 633.5) < 1.5, (s, q)
