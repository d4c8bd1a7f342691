"""The N>1 bench path on CPU ranks (gloo, world_size 2): each rank owns a
distinct seeded request shard (no data exchange), and the whole-job figure
is the token sum over ranks divided by the slowest rank's time."""
import os
import socket
import sys

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "marian-edge_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench
    import argparse
    args = argparse.Namespace(model="tiny_self", requests=8, workload="stream", docs=3)
    shard = bench.step_batches(args, rank, 1, 1000, world)[0]
    tokens = int(shard.force_len.sum())            # this rank's work
    dev_ms = 100.0 * (rank + 1)                    # rank 1 is the slowest
    total, max_ms, max_wall = bench.reduce_job(tokens, dev_ms, 1.0 + rank, world, "cpu")
    args.workload = "longtext"
    lt = bench.step_batches(args, rank, 1, 1000, world)[0]
    out[rank] = (shard.tokens.tobytes(), tokens, total, max_ms, max_wall,
                 [int(x) for x in (lt.offsets[1:] - lt.offsets[:-1])])
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    world, port = 2, _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    (t0, n0, total0, ms0, w0, lt0), (t1, n1, total1, ms1, w1, lt1) = out[0], out[1]
    assert t0 != t1                       # request-sharded streams differ per rank
    assert total0 == total1 == n0 + n1    # tokens summed over ranks
    assert ms0 == ms1 == 200.0            # slowest rank's device time
    assert w0 == w1 == 2.0
    # long-text stream: the two replicas' segments partition the global set
    sys.path.insert(0, os.path.join(ROOT, "marian-edge_b200"))
    from marian_cuda import workloads as W
    full = W.longtext_batch(3 * world, vocab=512, seed=1000)
    assert sorted(lt0 + lt1) == sorted(int(x) for x in (full.offsets[1:] - full.offsets[:-1]))
    assert abs(len(lt0) - len(lt1)) <= 1
