"""The drop-in recipes for emberllm's callers, checked on CPU. emberllm's own front-end
sources (tokenizer, sampler, JSON, server) link against this library into a
`libember.so`, and emberllm's unmodified Python binding (bindings/python/
emberllm.py) loads it through EMBER_LIB: model header and tokenizer round trip
equal the same binding over the reference's own build. emberllm's CLI
(main.c + the same front ends) links against this library too: `info`,
`tokenize` and `quantize` print and write what the reference's CLI does. (State
creation and the token loop need the GPU; the GPU tests cover them.)"""
import json
import os
import subprocess
import sys

import pytest

from emberllm_b200 import synth

from . import helpers as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = H.reference_dir()   # oracle/Makefile's REF
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libember_ref_det.so")
B200 = os.path.join(ROOT, "emberllm_b200")

pytestmark = pytest.mark.skipif(
    not (os.path.exists(os.path.join(REF_SRC, "bindings", "python", "emberllm.py")) and os.path.exists(REF_LIB)),
    reason="emberllm's sources and its build (oracle/_ref) are needed")

# the reference's binding module, pointed at EMBER_LIB by the environment
PROBE = r"""
import ctypes, importlib.util, json, sys
spec = importlib.util.spec_from_file_location("emberllm", sys.argv[1])
em = importlib.util.module_from_spec(spec)
spec.loader.exec_module(em)
lib = em._lib
m = lib.ember_model_load(sys.argv[2].encode())
h = lib.ember_model_header(m).contents
tok = lib.ember_tokenizer_new(m)
ids = ctypes.POINTER(ctypes.c_int)()
n = lib.ember_encode(tok, sys.argv[3].encode(), 1, ctypes.byref(ids))
got = [ids[i] for i in range(n)]
text = b"".join(lib.ember_decode(tok, got[i - 1] if i else -1, got[i]) or b"" for i in range(n))
print(json.dumps({"header": [h.dim, h.hidden_dim, h.n_layers, h.n_heads, h.n_kv_heads, h.head_dim,
                             h.vocab_size, h.n_tensors], "ids": got, "text": text.decode("latin-1")}))
"""


@pytest.fixture(scope="module")
def dropin(tmp_path_factory):
    out = tmp_path_factory.mktemp("dropin") / "libember.so"
    src = [os.path.join(REF_SRC, "src", f) for f in ("tokenizer.c", "sample.c", "json.c", "server.c")]
    r = subprocess.run(["gcc", "-std=c11", "-D_DEFAULT_SOURCE", "-O2", "-fPIC", "-shared", "-o", str(out), *src,
                        "-L" + B200, "-lember_b200", "-Wl,-rpath," + B200], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return str(out)


def probe(lib, model, text):
    env = dict(os.environ, EMBER_LIB=lib)
    r = subprocess.run([sys.executable, "-c", PROBE, os.path.join(REF_SRC, "bindings", "python", "emberllm.py"),
                        model, text], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-llama"])
def test_reference_binding_runs_on_the_dropin_library(dropin, name):
    model = synth.ensure_model(name)
    text = "hello world, the quick brown fox"
    ours, ref = probe(dropin, model, text), probe(REF_LIB, model, text)
    assert ours == ref
    assert len(ours["ids"]) > 1


@pytest.fixture(scope="module")
def cli(tmp_path_factory):
    """emberllm's CLI linked against this library: its front-end sources
    (main.c, tokenizer, sampler, JSON, server) and libember_b200"""
    out = tmp_path_factory.mktemp("cli") / "ember"
    src = [os.path.join(REF_SRC, "src", f) for f in ("main.c", "tokenizer.c", "sample.c", "json.c", "server.c")]
    r = subprocess.run(["gcc", "-std=c11", "-D_DEFAULT_SOURCE", "-O2", "-o", str(out), *src, "-L" + B200,
                        "-lember_b200", "-Wl,-rpath," + B200, "-lm", "-lpthread"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return str(out)


def ref_cli():
    path = os.path.join(ROOT, "oracle", "_ref", "ember_ref_v3")
    if not os.path.exists(path):
        pytest.skip("the reference CLI (oracle/_ref) was not built")
    return path


def run_cli(binary, *args):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=300)
    return r.returncode, r.stdout


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-smol-q4"])
def test_cli_info_and_tokenize_on_the_dropin_library(cli, name):
    model = synth.ensure_model(name)
    ref = ref_cli()
    assert run_cli(cli, "info", model) == run_cli(ref, "info", model)
    text = "Once upon a time, 42 foxes"
    got = run_cli(cli, "tokenize", model, text)
    assert got == run_cli(ref, "tokenize", model, text) and got[0] == 0 and got[1].strip()


@pytest.mark.parametrize("target", ["q8_0", "q4_0"])
def test_cli_quantize_on_the_dropin_library(cli, tmp_path, target):
    """`ember quantize` runs this library's ember_quantize_file; the file equals the
    reference CLI's byte for byte"""
    src = str(tmp_path / "f32.ember")
    synth.write_model(src, synth.CONFIGS["tiny-qwen2"], seed=5, quant="f32")
    ours, refs = str(tmp_path / "ours.ember"), str(tmp_path / "ref.ember")
    assert run_cli(cli, "quantize", src, ours, target)[0] == 0
    assert run_cli(ref_cli(), "quantize", src, refs, target)[0] == 0
    assert open(ours, "rb").read() == open(refs, "rb").read()
