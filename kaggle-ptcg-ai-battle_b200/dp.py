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


def checksum_u64(pair):
    """Two uint32 halves (as int32/int64 tensor) -> one int64 value tensor."""
    c = pair.to(torch.int64) & 0xFFFFFFFF
    return c[0] | (c[1] << 32)


def weights_agree(value, group=None):
    """(min, max) over ranks of a per-rank int64 scalar tensor: equal on
    every rank iff all ranks hold the same weights."""
    mn, mx = value.clone(), value.clone()
    dist.all_reduce(mn, op=dist.ReduceOp.MIN, group=group)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    return mn, mx
