"""Pinned-host -> device input feed with the copies on their own stream.

The reference moves each rollout buffer's observations host -> device with a
cudaMemcpyAsync on that buffer's stream, so one buffer's transfer overlaps
another buffer's forward pass (native/src/vecenv.h:310-345, one stream per
buffer at :292).  ``HostFeed`` gives the train step the same overlap: the
inputs of step i+1 cross PCIe on a dedicated copy stream while step i
computes, into a ring of ``depth`` device slots.  Every step still copies its
own inputs from pinned host memory; only the wait moves off the compute
stream.

Ordering is by CUDA events, never by host synchronisation:
  * ``put(host)`` makes the copy stream wait until the slot's previous
    consumer has finished (the event ``release()`` recorded), enqueues one
    non-blocking copy per tensor and records the slot's ready event;
  * ``get()`` makes the caller's current stream wait on the ready event of
    the oldest filled slot and returns its device tensors;
  * ``release()`` records, on the current stream, that the work reading the
    slot returned by the last ``get()`` has been enqueued.
"""
import torch


class HostFeed:
    def __init__(self, like, device, depth=2):
        """``like``: dict name -> tensor giving the shape / dtype of each
        input (host or device).  ``depth`` device slots are allocated once."""
        if depth < 1:
            raise ValueError("HostFeed depth must be >= 1")
        self.device = torch.device(device) if not isinstance(device, torch.device) else device
        if self.device.type != "cuda":
            raise ValueError("HostFeed copies into CUDA memory; got device %s" % self.device)
        self.names = list(like)
        self.depth = depth
        self.slots = [{k: torch.empty(like[k].shape, dtype=like[k].dtype, device=self.device)
                       for k in self.names} for _ in range(depth)]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.free = [torch.cuda.Event() for _ in range(depth)]
        self.n_put = 0
        self.n_get = 0
        self.bytes_per_put = sum(like[k].numel() * like[k].element_size() for k in self.names)

    def start(self):
        """Order the copy stream after the work already on the current
        stream (for example a timing event recorded just before)."""
        self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))

    def put(self, host):
        if self.n_put - self.n_get >= self.depth:
            raise RuntimeError("HostFeed: all %d slots are filled; get() one first" % self.depth)
        if set(host) != set(self.names):
            raise KeyError("HostFeed.put: expected inputs %s, got %s"
                           % (sorted(self.names), sorted(host)))
        i = self.n_put % self.depth
        slot = self.slots[i]
        for k in self.names:
            v = host[k]
            if v.device.type != "cpu" or not v.is_pinned():
                raise ValueError("HostFeed.put: input %r must be a pinned host tensor" % k)
            if v.shape != slot[k].shape or v.dtype != slot[k].dtype:
                raise ValueError("HostFeed.put: input %r is %s %s, the slot is %s %s"
                                 % (k, tuple(v.shape), v.dtype, tuple(slot[k].shape),
                                    slot[k].dtype))
        cs = self.copy_stream
        cs.wait_event(self.free[i])
        with torch.cuda.stream(cs):
            for k in self.names:
                slot[k].copy_(host[k], non_blocking=True)
            self.ready[i].record(cs)
        self.n_put += 1

    def get(self):
        if self.n_get >= self.n_put:
            raise RuntimeError("HostFeed.get: no filled slot; put() first")
        i = self.n_get % self.depth
        torch.cuda.current_stream(self.device).wait_event(self.ready[i])
        self.n_get += 1
        return self.slots[i]

    def release(self):
        if self.n_get == 0:
            raise RuntimeError("HostFeed.release: nothing was taken with get()")
        i = (self.n_get - 1) % self.depth
        self.free[i].record(torch.cuda.current_stream(self.device))
