"""Host check of the parallel evaluation of sequential non-negative fp32 sums
(emberllm_b200/csrc/exact_sum_core.h): the CTA algorithm emulated thread by
thread must equal the plain sequential sum bit for bit on adversarial inputs
(tests/exact_sum_check.c). The device kernels that use it are covered by the
bit-exact GPU parity tests."""
import os
import subprocess

from . import helpers as H


def test_parallel_exact_sum_matches_sequential(tmp_path):
    exe = str(tmp_path / "xs_check")
    src = os.path.join(H.ROOT, "tests", "exact_sum_check.c")
    inc = os.path.join(H.ROOT, "emberllm_b200", "csrc")
    subprocess.run(["gcc", "-O2", "-fno-fast-math", "-ffp-contract=off", "-I" + inc, src, "-o", exe,
                    "-lm"], check=True)
    r = subprocess.run([exe, "44000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
