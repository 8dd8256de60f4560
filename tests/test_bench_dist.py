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


def test_streams_summary_reports_the_contract_keys():
    """the streams aggregate's figures from one measurement: device-timed value,
    wall-clock e2e with the host copies' bytes, per-stream rate, step time"""
    sys.path.insert(0, ROOT)
    import bench
    m = {"S": 64, "t_wall": 2.0, "t_dev": 1.6, "clk": {}, "gemm": True, "tokens": 512 * 64 * 2}
    sm = bench.streams_summary(m, 512, 8, 64, 2)
    assert sm["value"] == round(512 * 64 * 2 / 1.6, 1)
    assert sm["e2e"]["value"] == round(512 * 64 * 2 / 2.0, 1)
    assert sm["per_stream_tok_s"] == round(sm["value"] / 512, 2)
    assert sm["streams"] == 512 and sm["streams_per_gpu"] == 64 and sm["n_gpus"] == 8
    assert sm["e2e"]["h2d_bytes_per_step"] == 64 * 8 and sm["e2e"]["d2h_bytes_per_step"] == 64 * 64 * 4
    assert sm["ms_per_step"] == round(1.6 / 2 * 1e3, 3)
    assert sm["path"] == "batched GEMMs" and "events" in sm["timing"]
    # without device events (concurrent single-stream states), wall time is the figure
    m2 = dict(m, t_dev=None, gemm=False)
    sm2 = bench.streams_summary(m2, 512, 8, 64, 2)
    assert sm2["value"] == sm2["e2e"]["value"] and sm2["timing"] == "wall clock"


def test_streams_partition_has_no_gaps_at_every_scale():
    """8 x 16, 8 x 64 split over 1..8 GPUs and 64 per GPU: every stream exactly once"""
    sys.path.insert(0, ROOT)
    import bench
    for total_fn in (lambda w: 128, lambda w: 512, lambda w: 64 * w):
        for world in range(1, 9):
            total = total_fn(world)
            seen = []
            for r in range(world):
                lo, hi = bench.stream_range(total, world, r)
                assert hi - lo in (total // world, total // world + 1)
                seen.extend(range(lo, hi))
            assert seen == list(range(total))
