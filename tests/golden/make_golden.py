"""Generate the golden vectors in this directory from the UNMODIFIED reference.

emberllm's own tests pin the token loop only with a transcript of real
stories15M weights that is bit-exact on macOS arm64 alone
(tests/run_tests.sh:153-169, .github/workflows/ci.yml:41-44); no checkpoint is
available offline. The goldens here are therefore produced by running emberllm
itself -- compiled from its own sources with its deterministic `make debug`
flags into oracle/_ref/libember_ref_det.so by oracle/Makefile -- on the small
synthetic models of emberllm_b200/synth.py, through its public C API
(ember_prefill / ember_forward, ref src/ember.h:127-129).

For each model the fixture records the model file's sha256 (so a change in the
synthetic writer is caught), the last-token logits of a 16-token prefill, the
logits of 8 teacher-forced forward steps after it, 24 greedy tokens, and the
same with the fp16 KV cache. Run from the repository root:

    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from emberllm_b200 import synth  # noqa: E402
from tests import helpers as H  # noqa: E402

NAMES = ["tiny-llama", "tiny-qwen3", "tiny-qwen2", "tiny-smol-q4", "tiny-f32"]


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def record(api, path, kv16):
    rng = np.random.default_rng(12345)
    s = api.session(path, 0, kv16)
    prompt = rng.integers(0, s.vocab, 16).astype(np.int32)
    prefill = s.prefill(prompt)
    forced_ids = rng.integers(0, s.vocab, 8).astype(np.int32)
    forced = np.stack([s.forward(int(t), 16 + i) for i, t in enumerate(forced_ids)])
    s.close()
    s = api.session(path, 0, kv16)
    greedy = np.array(H.greedy_run(s, [int(t) for t in prompt], 24), np.int32)
    s.close()
    return dict(prompt=prompt, prefill=prefill, forced_ids=forced_ids, forced=forced, greedy=greedy)


def main():
    if not H.have_reference():
        sys.exit("oracle/_ref/libember_ref_det.so is missing: run `make -C oracle ref` first")
    H.ensure_built()
    ref = H.ApiLib(H.REF_DET)
    out_dir = os.path.dirname(os.path.abspath(__file__))
    for name in NAMES:
        path = synth.ensure_model(name)
        arrays = {"sha256": np.frombuffer(sha256(path).encode(), np.uint8)}
        for kv16 in (0, 1):
            for k, v in record(ref, path, kv16).items():
                arrays["kv%d_%s" % (kv16 * 16 or 32, k)] = v
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **arrays)
        print("wrote", name)


if __name__ == "__main__":
    main()
