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


def _torch_adam(p, m, v, g, t, lr=1e-2, b1=0.9, b2=0.999, eps=1e-8):
    """The update formula of the fused Adam kernels, in torch."""
    m.mul_(b1).add_((1 - b1) * g)
    v.mul_(b2).add_((1 - b2) * g * g)
    p.sub_(lr / (1 - b1 ** t) * m / (v.sqrt() / (1 - b2 ** t) ** 0.5 + eps))


def _sharded_worker(rank, world, port):
    _init(rank, world, port)
    from ptcg_b200.dp import ShardedAdam
    n, max_norm = 1000, 1.0
    torch.manual_seed(0)
    p0 = torch.randn(n)                                   # identical start on every rank
    params, m, v = p0.clone(), torch.zeros(n), torch.zeros(n)
    step = [0]

    def update(shard, seg, nseg, ss, stats):
        norm = float(ss[0].sqrt())
        coef = min(1.0, max_norm / (norm + 1e-6))
        t = step[0] + 1
        for k in range(nseg):
            a, so, ln = [int(x) for x in seg[3 * k:3 * k + 3]]
            _torch_adam(params[a:a + ln], m[a:a + ln], v[a:a + ln], shard[so:so + ln] * coef, t)
        step[0] += 1
        stats[0], stats[1] = norm, 1.0

    grads = torch.zeros(n)
    red = ShardedAdam(grads, params, update,
                      sumsq=lambda x, out: out.copy_((x.double() ** 2).sum().view(1)),
                      refresh=lambda: None)
    bounds = [0, 92, 300, 304, 700, 1000]                # spans in backward order
    ref_p, ref_m, ref_v = p0.clone(), torch.zeros(n), torch.zeros(n)
    for it in range(3):
        g_all = [torch.randn(n, generator=torch.Generator().manual_seed(100 * it + r))
                 for r in range(world)]
        grads.copy_(g_all[rank])
        red.reset()
        for a, b in reversed(list(zip(bounds[:-1], bounds[1:]))):
            red(a, b - a, None)
        assert red.covered(n)
        stats = torch.zeros(2)
        red.step(stats)
        # reference: the averaged gradient, clipped, full Adam on every rank
        g = torch.stack(g_all).mean(0)
        norm = float(g.double().norm())
        assert abs(float(stats[0]) - norm) <= 1e-5 * norm
        _torch_adam(ref_p, ref_m, ref_v, g * min(1.0, max_norm / (norm + 1e-6)), it + 1)
        torch.testing.assert_close(params, ref_p, rtol=1e-5, atol=1e-6)
    # this rank's segments: disjoint pieces that, over all ranks, tile the arena
    seg = red.segments().view(-1, 3)
    mine = torch.zeros(n, dtype=torch.int32)
    for a, _, ln in seg.tolist():
        mine[a:a + ln] += 1
    dist.all_reduce(mine)
    assert torch.equal(mine, torch.ones(n, dtype=torch.int32))
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


def test_sharded_adam_matches_allreduce_adam():
    """Reduce-scatter per bucket + Adam on each rank's shard + all-gather ==
    all-reduce + Adam over the whole arena, on every rank."""
    _run(_sharded_worker)


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
