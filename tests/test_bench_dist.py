"""The multi-rank host path of bench.py on CPU: two gloo ranks (the GPU box runs
the same code with NCCL, one rank per GPU). Replicas and stream partitions share
no data; only barriers and the max-over-ranks of the step timer cross ranks."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)
    import bench
    w, r, local, dist = bench.dist_setup(backend="gloo", timeout_s=60)
    try:
        bench.barrier(dist)
        # every rank sees the slowest rank's time
        t = bench.max_over_ranks(dist, 1.0 + 0.5 * r)
        lo, hi = bench.stream_range(8 * 16, w, r)
        # the reference arm: rank 0 alone runs and prints; the others do no work
        class A:
            pass
        ref = bench.run_reference(A(), w, r) if r != 0 else "rank0"
        out[r] = (w, r, t, lo, hi, ref)
        bench.barrier(dist)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_only_the_timer():
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert set(res) == {0, 1}
    for r, (w, rr, t, lo, hi, ref) in res.items():
        assert w == 2 and rr == r
        assert t == pytest.approx(1.5)                  # max over ranks
    # the two partitions tile the 128 streams without overlap
    assert res[0][3:5] == (0, 64) and res[1][3:5] == (64, 128)
    assert res[1][5] is None                            # non-zero ranks of the reference arm exit empty


def test_stream_partition_covers_every_stream():
    sys.path.insert(0, ROOT)
    import bench
    for total in (8, 128, 512):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                lo, hi = bench.stream_range(total, world, r)
                seen.extend(range(lo, hi))
            assert seen == list(range(total))
