"""The decode GEMVs' RMSNorm sum of squares (split_chain_sum, csrc/cuda/common.cuh)
must equal the reference's sequential loop (ref src/model.c:50-55) bit for bit:
each later quarter of the terms is added from the 64 floats around an estimate of
the sum before it, and the chains that started from the sums actually reached
are taken. Checked against a float32 left-to-right sum on activation-like,
heavy-tailed, sparse, tiny, huge, tie-prone, outlier and softmax-like terms (an
outlier swallows the small terms after it, so its sums may leave the windows and
take the sequential fallback); on activation-like data the split evaluation must
answer."""
import numpy as np
import pytest

from . import helpers as H

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return H.testhooks()


def seq_sum(terms):
    """the reference's loop: float32 additions in index order from 0"""
    with np.errstate(over="ignore"):   # the huge-term cases overflow to inf, as the loop does
        return np.cumsum(terms.astype(np.float32), dtype=np.float32)[-1]


def squares(rng, n):
    """(name, squares) cases"""
    cases = [
        ("normal", rng.standard_normal(n)),
        ("scaled", rng.standard_normal(n) * 37.0),
        ("t2", rng.standard_t(2, n)),
        ("sparse", np.where(rng.random(n) < 0.9, 0.0, rng.standard_normal(n))),
        ("tiny", rng.standard_normal(n) * 1e-18),
        ("huge", rng.standard_normal(n) * 1e18),
        ("lognormal", np.exp(rng.standard_normal(n) * 4.0)),
        ("ints", rng.integers(-64, 64, n).astype(np.float64)),
        ("const", np.full(n, 0.75)),
        ("zeros", np.zeros(n)),
    ]
    x = rng.standard_normal(n)
    x[rng.integers(0, n)] = 1e4
    cases.append(("outlier", x))
    x = rng.standard_normal(n)
    x[: n // 2] *= 1e-3
    cases.append(("small-then-large", x))
    out = []
    for name, v in cases:
        v = v.astype(np.float32)
        out.append((name, (v * v).astype(np.float32)))
    return out


def run(lib, vecs, n):
    v = np.ascontiguousarray(np.stack(vecs), dtype=np.float32)
    out = np.zeros(len(vecs), np.float32)
    hit = np.zeros(len(vecs), np.int32)
    assert lib.ember_cuda_split_sum_batch(v.ctypes.data, n, len(vecs), out.ctypes.data, hit.ctypes.data) == 0
    return out, hit


@pytest.mark.parametrize("n", [32, 64, 100, 128, 576, 896, 1024, 2048, 4096])
def test_split_sum_matches_the_loop(lib, n):
    rng = np.random.default_rng(7 + n)
    names, vecs = [], []
    for rep in range(8):
        for name, t in squares(rng, n):
            names.append(name)
            vecs.append(t)
        x = (rng.standard_normal(n) * (2.0 + 3 * rep)).astype(np.float32)
        names.append("softmax")
        vecs.append(np.exp((x - x.max()).astype(np.float64)).astype(np.float32))
    out, hit = run(lib, vecs, n)
    for i, t in enumerate(vecs):
        want = seq_sum(t)
        assert out[i].view(np.uint32) == want.view(np.uint32), (n, names[i], out[i], want, hit[i])
    if n % 64 == 0 and 128 <= n <= 1024:
        typical = ("normal", "scaled", "sparse", "zeros", "const", "ints", "softmax")
        misses = [names[i] for i in range(len(vecs)) if not hit[i] and names[i] in typical]
        assert not misses, (n, misses)


def test_split_sum_random_sweep(lib):
    """exact on every vector; the split evaluation answers on all but a few of
    the mild ones (heavy tails may take the fallback)"""
    rng = np.random.default_rng(99)
    for n in (128, 256, 576, 896, 1024):
        vecs, mild = [], []
        for k in range(200):
            scale = np.exp(rng.uniform(-20, 20))
            x = (rng.standard_normal(n) * scale * np.exp(rng.standard_normal(n) * (k % 5))).astype(np.float32)
            vecs.append((x * x).astype(np.float32))
            mild.append(k % 5 < 2)
        out, hit = run(lib, vecs, n)
        for i, t in enumerate(vecs):
            assert out[i].view(np.uint32) == seq_sum(t).view(np.uint32), (n, i)
        assert hit[np.array(mild)].mean() > 0.97, (n, hit[np.array(mild)].mean())


@pytest.mark.parametrize("n", [64, 128, 256, 576, 768, 896, 1024, 2048, 4096])
def test_persistent_step_sum_matches_the_loop(lib, n):
    """the persistent step's 512-thread variant (psum: 16, 8 or 4 segments by n,
    float tree estimates) equals the sequential float loop bit for bit on every
    case above, including the outliers that send it to its sequential fallback"""
    rng = np.random.default_rng(n + 7)
    vecs = []
    for rep in range(4):
        vecs += [t for _, t in squares(rng, n)]
        x = (rng.standard_normal(n) * (2.0 + 3 * rep)).astype(np.float32)
        vecs.append(np.exp((x - x.max()).astype(np.float64)).astype(np.float32))
    for k in range(100):
        x = (rng.standard_normal(n) * np.exp(rng.uniform(-20, 20)) * np.exp(rng.standard_normal(n) * (k % 5))).astype(np.float32)
        vecs.append((x * x).astype(np.float32))
    v = np.ascontiguousarray(np.stack(vecs), dtype=np.float32)
    out = np.zeros(len(vecs), np.float32)
    assert lib.ember_cuda_psum_batch(v.ctypes.data, n, len(vecs), out.ctypes.data) == 0
    for i, t in enumerate(vecs):
        assert out[i].view(np.uint32) == seq_sum(t).view(np.uint32), (n, i)
