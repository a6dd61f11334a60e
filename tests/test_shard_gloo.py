"""Multi-GPU host logic on CPU.  One process per rank, as on the GPUs, over
gloo at world size 2.  Each rank takes a contiguous range of whole streams
(q3s.shard.stream_range) and samples it with the oracle; the union must
equal the single-process result, since rows are independent.  The timing
reduction must return the slowest rank's time.
"""
import json
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from q3s import shard, workloads  # noqa: E402

STREAMS = 7  # uneven over 2 ranks on purpose
ROWS_PER_STREAM = 16


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sample_rows(w, rows):
    import oracle
    return oracle.sample_rows(*w.oracle_layout(rows), nthreads=1)


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w = workloads.hetero("cpu", streams=STREAMS)
        b, e = shard.stream_range(STREAMS, ROWS_PER_STREAM, world, rank)
        ref = _sample_rows(w, np.arange(b, e))
        parts = [None] * world
        dist.all_gather_object(parts, {"begin": b, "end": e,
                                       "tokens": ref["tokens"].tolist(),
                                       "status": ref["status"].tolist()})
        slowest = shard.max_over_ranks(10.0 * (rank + 1))
        rate = shard.whole_job_rate(e - b, world, 4, slowest)
        if rank == 0:
            with open(out_path, "w") as f:
                json.dump({"parts": parts, "slowest": slowest, "rate": rate}, f)
    finally:
        dist.destroy_process_group()


def test_row_range_partitions_exactly():
    for total in (0, 1, 7, 64, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard.row_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
            sizes = [e - b for b, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def test_stream_range_keeps_streams_whole():
    for world in (1, 2, 4, 8):
        prev = 0
        for r in range(world):
            b, e = shard.stream_range(4096, 16, world, r)
            assert b == prev and b % 16 == 0 and e % 16 == 0
            prev = e
        assert prev == 4096 * 16


def test_two_gloo_ranks_reproduce_single_process(tmp_path):
    out = tmp_path / "rank0.json"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(out)), nprocs=2, join=True,
                       start_method="spawn")
    got = json.loads(out.read_text())
    parts = got["parts"]
    assert [p["begin"] for p in parts] == [0, 4 * ROWS_PER_STREAM]
    assert parts[-1]["end"] == STREAMS * ROWS_PER_STREAM
    tokens = np.concatenate([np.asarray(p["tokens"], np.uint32) for p in parts])
    status = np.concatenate([np.asarray(p["status"], np.uint8) for p in parts])
    w = workloads.hetero("cpu", streams=STREAMS)
    ref = _sample_rows(w, np.arange(STREAMS * ROWS_PER_STREAM))
    np.testing.assert_array_equal(status, ref["status"])
    np.testing.assert_array_equal(tokens, ref["tokens"])
    assert got["slowest"] == 20.0
    assert got["rate"] == pytest.approx(2 * 4 * ROWS_PER_STREAM * 4 / 0.020)
