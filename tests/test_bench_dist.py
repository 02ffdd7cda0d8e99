"""The benchmark's multi-GPU host logic (one process per GPU, barrier, max over ranks,
weak-scaling aggregate) on CPU ranks over gloo, world size 2."""
import os
import socket

import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import bench
    dist = bench.dist_setup(world, backend="gloo")
    seconds = [1.5, 2.0][rank]          # each rank decoded 100 tokens of its own stream
    dist.barrier()
    slowest = bench.dist_max(dist, seconds, "cpu")
    out[rank] = (slowest, bench.weak_scaling_value(100, world, slowest))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_max_and_weak_scaling():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank, args=(2, _free_port(), out), nprocs=2, start_method="spawn", join=True)
        assert out[0] == out[1] == (2.0, 100.0)


def test_reference_arm_prints_one_line_on_rank0_only(tmp_path):
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip() == ""
