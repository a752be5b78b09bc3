"""HostFeed: pinned-host -> device inputs on a copy stream (a ring of device
slots ordered by CUDA events)."""
import pytest
import torch


def test_feed_rejects_a_host_device(pkg):
    from ptcg_b200.feed import HostFeed
    with pytest.raises(ValueError):
        HostFeed({"obs": torch.zeros(4, 8)}, "cpu")


@pytest.mark.gpu
def test_feed_delivers_each_step_in_order(pkg):
    from ptcg_b200.feed import HostFeed
    dev = torch.device("cuda", 0)
    n = 1 << 20
    hosts = [dict(obs=torch.full((n,), float(i)).pin_memory(),
                  act=torch.full((64,), i, dtype=torch.int32).pin_memory()) for i in range(6)]
    feed = HostFeed(hosts[0], dev, depth=2)
    assert feed.bytes_per_put == n * 4 + 64 * 4
    seen = []
    feed.start()
    feed.put(hosts[0])
    for i in range(6):
        b = feed.get()
        if i + 1 < 6:
            feed.put(hosts[i + 1])          # overwrites the other slot only after its release
        torch.cuda._sleep(2_000_000)        # a long consumer on the compute stream
        seen.append((b["obs"].sum() / n, b["act"].float().mean()))
        feed.release()
    torch.cuda.synchronize()
    for i, (o, a) in enumerate(seen):
        assert o.item() == float(i) and a.item() == float(i)


@pytest.mark.gpu
def test_feed_checks_its_inputs(pkg):
    from ptcg_b200.feed import HostFeed
    dev = torch.device("cuda", 0)
    like = dict(obs=torch.zeros(16).pin_memory())
    feed = HostFeed(like, dev, depth=1)
    with pytest.raises(RuntimeError):
        feed.get()
    with pytest.raises(ValueError):
        feed.put(dict(obs=torch.zeros(16)))             # not pinned
    with pytest.raises(ValueError):
        feed.put(dict(obs=torch.zeros(8).pin_memory()))  # wrong shape
    with pytest.raises(KeyError):
        feed.put(dict(x=torch.zeros(16).pin_memory()))
    feed.put(like)
    with pytest.raises(RuntimeError):
        feed.put(like)                                   # the only slot is still filled
    feed.get()
    feed.release()
    torch.cuda.synchronize()
