"""Data-parallel plumbing for the PPO step: one process per GPU, the
gradient average as the only exchange per optimizer step.

Replaces the single post-backward ``ncclAllReduce(avg)`` of the reference's
trainer (native/src/muon.cu:212-213) with bucketed reductions that start as
soon as backward finalises each span of the flat fp32 grad arena
(``ptcg_set_grad_hook``: spans arrive in backward order), overlapping the
rest of backward.  Also the cross-rank "weights identical" check
(min == max of a 64-bit checksum of the master weights).

Works on any ``torch.distributed`` backend: with NCCL on CUDA tensors the
reductions run on a side stream ordered after the compute stream; on CPU
(gloo) they run inline, which is what the host-logic tests use.
"""
import torch
import torch.distributed as dist


class BucketAllReduce:
    """Callable grad hook: ``hook(offset, count, stream_ptr)`` averages
    ``grads[offset:offset+count]`` across the group.  Call ``wait()`` before
    the optimizer reads the grads."""

    def __init__(self, grads, group=None):
        self.grads = grads
        self.group = group
        self.world = dist.get_world_size(group)
        self.avg = dist.get_backend(group) == "nccl"       # gloo has no AVG
        self.cuda = grads.is_cuda
        self.comm = torch.cuda.Stream(device=grads.device) if self.cuda else None
        self.spans = []

    def __call__(self, offset, count, stream_ptr=None):
        self.spans.append((offset, count))
        view = self.grads[offset:offset + count]
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.grads.device))
            self.comm.wait_event(ev)
            with torch.cuda.stream(self.comm):
                self._reduce(view)
        else:
            self._reduce(view)

    def _reduce(self, view):
        if self.avg:
            dist.all_reduce(view, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group)
            view.div_(self.world)

    def wait(self):
        """Order the caller's current stream after every reduction issued."""
        if self.cuda:
            torch.cuda.current_stream(self.grads.device).wait_stream(self.comm)

    def covered(self, n):
        """True when the spans issued since the last reset tile [0, n)
        exactly once (every grad averaged, none twice)."""
        cur = 0
        for off, cnt in sorted(self.spans):
            if off != cur:
                return False
            cur += cnt
        return cur == n

    def reset(self):
        self.spans = []


class ShardedAdam:
    """Data-parallel gradient exchange fused with a sharded optimizer step.

    As a grad hook, each final gradient span (bucket) is reduce-scattered on a
    side stream while the rest of backward runs: rank r receives the average
    of piece r of the bucket (pieces of ceil(count / world) floats, rounded up
    to 4).  ``step()`` then takes the global gradient norm (each rank's shard
    sum of squares, summed over ranks), runs the Adam update on this rank's
    pieces only, and all-gathers the updated weights bucket by bucket before
    refreshing the bf16 compute copies.  Together the reduce-scatter and the
    all-gather move what one all-reduce moves; the optimizer pass reads and
    writes 1/world of the arena on each rank.  The reference instead
    all-reduces the whole arena and every rank updates all of it
    (native/src/muon.cu:209-214).

    ``update(grad_shard, seg, nseg, sumsq, stats)``, ``sumsq(x, out)`` and
    ``refresh()`` are the device calls (PTCGPolicy.adam_segments / .sumsq /
    .refresh_copies); tests on CPU pass torch stand-ins.
    """

    def __init__(self, grads, params, update, sumsq, refresh, group=None, max_buckets=64):
        self.grads, self.params = grads, params
        self.update, self.sumsq_fn, self.refresh = update, sumsq, refresh
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.avg = dist.get_backend(group) == "nccl"
        self.cuda = grads.is_cuda
        self.comm = torch.cuda.Stream(device=grads.device) if self.cuda else None
        n = grads.numel()
        cap = n // self.world + 4 * max_buckets + 4
        self.shard = torch.zeros(cap, dtype=torch.float32, device=grads.device)
        self.used = 0
        self.plans = {}                  # bucket offset -> plan
        self.spans = []                  # spans seen since reset()
        self.ss = torch.zeros(1, dtype=torch.float64, device=grads.device)
        self.seg = None

    def _plan(self, offset, count):
        p = self.plans.get(offset)
        if p is not None:
            assert p["count"] == count, "bucket spans must not change between steps"
            return p
        c = ((count + self.world - 1) // self.world + 3) // 4 * 4
        if self.used + c > self.shard.numel():
            raise RuntimeError("ShardedAdam: more buckets than max_buckets")
        dev = self.grads.device
        p = {"offset": offset, "count": count, "c": c, "soff": self.used,
             "send": torch.zeros(self.world * c, dtype=torch.float32, device=dev),
             "piece": torch.zeros(c, dtype=torch.float32, device=dev),
             "gather": torch.zeros(self.world * c, dtype=torch.float32, device=dev)}
        self.used += c
        self.plans[offset] = p
        self.seg = None                  # the segment table changes
        return p

    def _shard_of(self, p):
        return self.shard[p["soff"]:p["soff"] + p["c"]]

    def __call__(self, offset, count, stream_ptr=None):
        self.spans.append((offset, count))
        p = self._plan(offset, count)
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.grads.device))
            self.comm.wait_event(ev)
            with torch.cuda.stream(self.comm):
                self._reduce_scatter(p)
        else:
            self._reduce_scatter(p)

    def _reduce_scatter(self, p):
        send = p["send"]
        send[:p["count"]].copy_(self.grads[p["offset"]:p["offset"] + p["count"]])
        out = self._shard_of(p)
        if self.avg:
            dist.reduce_scatter_tensor(out, send, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.reduce_scatter_tensor(out, send, group=self.group)
            out.div_(self.world)

    def segments(self):
        """{arena offset, shard offset, length} of this rank's pieces."""
        if self.seg is None:
            rows = []
            for p in sorted(self.plans.values(), key=lambda q: q["offset"]):
                start = self.rank * p["c"]
                length = max(0, min(p["count"] - start, p["c"]))
                if length > 0:
                    rows.append((p["offset"] + start, p["soff"], length))
            self.seg = torch.tensor(rows, dtype=torch.int64, device=self.grads.device).view(-1)
        return self.seg

    def covered(self, n):
        """True when the spans since the last reset tile [0, n) exactly once."""
        cur = 0
        for off, cnt in sorted(self.spans):
            if off != cur:
                return False
            cur += cnt
        return cur == n

    def reset(self):
        self.spans = []

    def step(self, stats):
        """Global-norm clip + Adam on this rank's shard, then the all-gather
        of the updated weights and the bf16 copy refresh.  `stats` (2 floats)
        receives {grad norm, applied}."""
        if self.cuda:
            torch.cuda.current_stream(self.grads.device).wait_stream(self.comm)
        self.sumsq_fn(self.shard[:self.used], self.ss)
        dist.all_reduce(self.ss, op=dist.ReduceOp.SUM, group=self.group)
        seg = self.segments()
        self.update(self.shard, seg, seg.numel() // 3, self.ss, stats)
        for p in sorted(self.plans.values(), key=lambda q: q["offset"]):
            start = self.rank * p["c"]
            length = max(0, min(p["count"] - start, p["c"]))
            piece = p["piece"]
            if length > 0:
                piece[:length].copy_(self.params[p["offset"] + start:p["offset"] + start + length])
            dist.all_gather_into_tensor(p["gather"], piece, group=self.group)
            self.params[p["offset"]:p["offset"] + p["count"]].copy_(p["gather"][:p["count"]])
        self.refresh()


def checksum_u64(pair):
    """Two uint32 halves (as int32/int64 tensor) -> one int64 value tensor."""
    c = pair.to(torch.int64) & 0xFFFFFFFF
    return c[0] | (c[1] << 32)


def weights_agree(value, group=None):
    """(min, max) over ranks of a per-rank int64 scalar tensor, in ONE
    collective: a MAX all-reduce of [v, ~v] (bitwise not reverses the
    order of two's-complement integers without overflow, so min = ~max(~v)).
    Equal on every rank iff all ranks hold the same weights."""
    both = torch.stack([value, torch.bitwise_not(value)])
    dist.all_reduce(both, op=dist.ReduceOp.MAX, group=group)
    return torch.bitwise_not(both[1]), both[0]
