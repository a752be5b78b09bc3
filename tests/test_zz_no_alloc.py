"""ptcg_ppo_loss_noalloc (scratch in a static device array inside the
library) against ptcg_ppo_loss (caller-supplied scratch), both through the
C-ABI on the same seeded inputs: two calls in a row must each match the
caller-scratch results.  Named to be collected last, so it also runs after
every other test has used the library in the same process."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PTCG_ERANGE = 4
MAX_ROWS = 65536            # PTCG_PPO_NOALLOC_MAX_ROWS in include/ptcg_b200.h


def _p(t):
    return C.c_void_p(t.data_ptr())


def _inputs(n_seg, horizon, nopt, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    nt = n_seg * horizon
    dec = torch.randn(nt, nopt + 1, generator=g)
    mask = (torch.rand(nt, nopt, generator=g) < 0.4).float()
    mask[torch.arange(nt), torch.randint(0, nopt, (nt,), generator=g)] = 1.0
    act = torch.multinomial(mask, 1, generator=g)[:, 0].float()
    old = -torch.rand(nt, generator=g) * 3
    adv = torch.randn(nt, generator=g)
    val = torch.randn(nt, generator=g)
    ret = torch.randn(nt, generator=g)
    prio = torch.rand(n_seg, generator=g) + 0.5
    return [t.cuda().contiguous() for t in (dec, mask, act, old, adv, val, ret, prio)]


def _outputs(nt, nopt):
    return (torch.empty(nt, nopt + 1, device="cuda"), torch.empty(nt, device="cuda"),
            torch.empty(nt, device="cuda"), torch.zeros(8, device="cuda"))


HYPER = (0.2, 0.2, 0.5, 0.01)


def test_ppo_loss_noalloc_matches_caller_scratch(pkg):
    import ptcg_b200.native as n
    lib = n.lib()
    n_seg, horizon, nopt = 96, 64, 64
    nt = n_seg * horizon
    dec, mask, act, old, adv, val, ret, prio = _inputs(n_seg, horizon, nopt, 2024)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ins = [_p(t) for t in (act, old, adv, val, ret, prio)]

    grad_r, nlp_r, ratio_r, st_r = _outputs(nt, nopt)
    scratch = torch.empty(16 + 7 * ((nt + 7) // 8), device="cuda")
    rc = lib.ptcg_ppo_loss(_p(dec), nopt, _p(mask), *ins, n_seg, horizon, *HYPER,
                           _p(grad_r), _p(nlp_r), _p(ratio_r), _p(st_r), _p(scratch), stream)
    assert rc == 0, lib.ptcg_last_error()

    for call in range(2):
        grad, nlp, ratio, st = _outputs(nt, nopt)
        rc = lib.ptcg_ppo_loss_noalloc(_p(dec), nopt, _p(mask), *ins, n_seg, horizon, *HYPER,
                                       _p(grad), _p(nlp), _p(ratio), _p(st), stream)
        assert rc == 0, lib.ptcg_last_error()
        torch.cuda.synchronize()
        for a, b in ((grad, grad_r), (nlp, nlp_r), (ratio, ratio_r), (st, st_r)):
            np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=1e-6, atol=1e-7,
                                       err_msg=f"call {call}")
    assert np.isfinite(st_r.cpu().numpy()).all()


def test_ppo_loss_noalloc_rejects_oversize(pkg):
    """more rows than the static scratch holds: PTCG_ERANGE before any launch"""
    import ptcg_b200.native as n
    lib = n.lib()
    nopt, horizon = 64, 64
    n_seg = MAX_ROWS // horizon + 1
    t = torch.zeros(1, device="cuda")
    rc = lib.ptcg_ppo_loss_noalloc(_p(t), nopt, _p(t), _p(t), _p(t), _p(t), _p(t), _p(t), _p(t),
                                   n_seg, horizon, *HYPER, _p(t), _p(t), _p(t), _p(t),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == PTCG_ERANGE
    assert b"static scratch limit" in lib.ptcg_last_error()
