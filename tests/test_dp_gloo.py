"""Data-parallel host logic on CPU: two gloo ranks (world_size 2).

- BucketAllReduce averages a flat grad arena span by span, with the spans
  arriving in backward order as ptcg_set_grad_hook delivers them, and
  reports whether they tiled the arena exactly once.
- weights_agree (min/max of a per-rank checksum) tells identical weights
  from diverged ones.
- A rank that leaves before a collective makes its peer's collective end
  with an error instead of hanging (short process-group timeout).
"""
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _bucket_worker(rank, world, port):
    _init(rank, world, port)
    from ptcg_b200.dp import BucketAllReduce
    n = 1000
    grads = torch.arange(n, dtype=torch.float32) * (rank + 1)
    red = BucketAllReduce(grads)
    # spans in backward order: last parameters first, like the model's hook
    bounds = [0, 90, 300, 301, 700, n]
    for a, b in reversed(list(zip(bounds[:-1], bounds[1:]))):
        red(a, b - a, None)
    red.wait()
    assert red.covered(n)
    expect = torch.arange(n, dtype=torch.float32) * sum(r + 1 for r in range(world)) / world
    torch.testing.assert_close(grads, expect)
    # a gap or a repeated span is reported
    red.reset()
    red(0, 10, None)
    red(20, n - 20, None)
    assert not red.covered(n)
    red.reset()
    red(0, n, None)
    red(0, 10, None)
    assert not red.covered(n)
    dist.destroy_process_group()


def _agree_worker(rank, world, port):
    _init(rank, world, port)
    from ptcg_b200.dp import checksum_u64, weights_agree
    same = checksum_u64(torch.tensor([123456789, 42], dtype=torch.int32))
    mn, mx = weights_agree(same)
    assert int(mn) == int(mx) == (42 << 32 | 123456789)
    diff = checksum_u64(torch.tensor([7 + rank, -1], dtype=torch.int32))
    mn, mx = weights_agree(diff)
    assert int(mn) != int(mx)
    dist.destroy_process_group()


def _leaver_worker(rank, world, port, flag):
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)                       # both ranks take part once
    if rank == 1:
        os._exit(0)                          # leaves between steps, nothing in flight
    try:
        dist.all_reduce(t)
    except Exception:                        # noqa: BLE001 -- peer gone: error, not a hang
        with open(flag, "w") as f:
            f.write("error")
        os._exit(0)
    os._exit(3)


def _run(fn, *args):
    mp.start_processes(fn, args=(2, _port()) + args, nprocs=2, join=True, start_method="spawn")


def test_bucket_allreduce_averages_and_tiles():
    _run(_bucket_worker)


def test_weights_agree_detects_divergence():
    _run(_agree_worker)


@pytest.mark.timeout(120)
def test_rank_leaving_fails_peer_collective(tmp_path):
    flag = str(tmp_path / "flag")
    ctx = mp.start_processes(_leaver_worker, args=(2, _port(), flag), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(90)
    codes = [p.exitcode for p in ctx.processes]
    assert codes == [0, 0], codes
    assert open(flag).read() == "error"
