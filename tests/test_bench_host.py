"""Host-side logic of bench.py that needs no GPU: the cross-rank timing reduction (two
gloo ranks on CPU), the whole-job rate, the launch count and the reference arm's
rank handling."""

import io
import os
import socket
import sys
from contextlib import redirect_stdout

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    local_ms = [120.0, 80.0][rank]  # rank 0 is the slow one
    ms = bench.max_over_ranks(local_ms, dist, "cpu")
    out[rank] = (ms, bench.whole_job_rate(10, world, ms))
    dist.barrier()
    dist.destroy_process_group()


def test_max_over_ranks_and_weak_scaling_rate_gloo():
    world = 2
    out = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    assert out[0] == out[1]
    ms, rate = out[0]
    assert ms == 120.0
    assert rate == pytest.approx(2 * 10 / 0.120)


def test_single_process_reduction_is_identity():
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.whole_job_rate(80, 1, 400.0) == pytest.approx(200.0)


def test_gpu_launch_count_per_step():
    # 7 embedding launches + 1 adaLN GEMM + 7 per sub-block x 32 + 2 final + 1 sampler
    # 7 head kernels, first QKV, 32 x (attention + chained launch), final GEMM, sampler
    assert bench.gpu_launches_per_step(16) == 7 + 1 + 64 + 1 + 1
    assert bench.gpu_launches_per_step(2, chained=False, sampler=False) == 7 + 20 + 1


def test_reference_arm_nonzero_rank_prints_nothing():
    class A:
        steps, warmup = 1, 0
    buf = io.StringIO()
    with redirect_stdout(buf):
        assert bench.run_reference(A(), rank=1, world=2) == 0
    assert buf.getvalue() == ""
