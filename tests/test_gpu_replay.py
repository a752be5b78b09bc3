"""Minibatch selection around the train step against the CPU oracle:
prioritised segment replay (ptcg_prio_replay), the segment gather
(ptcg_select_copy) and the write-back (ptcg_index_copy)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pol(pkg):
    s = pkg.config.PRESETS["tiny"]
    return pkg.PTCGPolicy(s, precision="fp32", tables=pkg.synth.make_tables(s, 11),
                          weights=pkg.synth.make_weights(s, 21))


@pytest.mark.parametrize("case", ["normal", "zeros", "nan_rows", "one_segment", "alpha0"])
def test_prio_replay_matches_oracle(pkg, oracle, case):
    rng = np.random.default_rng(5)
    B, T, n = (512, 64, 256) if case != "one_segment" else (1, 64, 16)
    adv = rng.standard_normal((B, T)).astype(np.float32) * rng.random((B, 1)).astype(np.float32)
    alpha, beta = (0.0 if case == "alpha0" else 0.6), 0.4
    if case == "zeros":
        adv[:] = 0
    if case == "nan_rows":
        adv[3, 5] = np.nan
        adv[7, :] = np.inf
    u = rng.random(n).astype(np.float32)
    pol = _pol(pkg)
    idx, mb_prio, probs = pol.prio_replay(adv, alpha, beta, B, u)
    oidx, omb, oprobs, margin = oracle.prio_replay(adv, alpha, beta, B, u)
    np.testing.assert_allclose(probs.cpu().numpy(), oprobs, rtol=2e-5, atol=1e-9)
    ok = margin > 1e-5                      # ties at a cdf boundary are rounding-dependent
    assert ok.mean() > 0.9
    np.testing.assert_array_equal(idx.cpu().numpy()[ok], oidx[ok])
    np.testing.assert_allclose(mb_prio.cpu().numpy()[ok], omb[ok], rtol=1e-4)
    assert (idx.cpu().numpy() >= 0).all() and (idx.cpu().numpy() < B).all()


@pytest.mark.parametrize("with_mask", [True, False])
def test_select_copy_and_index_copy(pkg, oracle, with_mask):
    rng = np.random.default_rng(9)
    B, T, W, nopt, n = 96, 16, 40, 8, 70
    obs = rng.standard_normal((B, T, W)).astype(np.float32)
    act, lp, val, adv = (rng.standard_normal((B, T)).astype(np.float32) for _ in range(4))
    mask = (rng.random((B, T, nopt)) < 0.5).astype(np.float32) if with_mask else None
    idx = rng.integers(0, B, n).astype(np.int32)          # with repeats, like sampling
    pol = _pol(pkg)
    out = pol.select_copy(torch.from_numpy(idx), obs, act, lp, val, adv, mask)
    ref = oracle.select_copy(idx, obs, act, lp, val, adv, mask)
    for k in ("obs", "actions", "logprobs", "values", "advantages", "returns"):
        np.testing.assert_array_equal(out[k].cpu().numpy(), ref[k], err_msg=k)
    if with_mask:
        np.testing.assert_array_equal(out["mask"].cpu().numpy(), ref["mask"])
    # write-back of per-segment results (unique rows, as the trainer's ratio / value)
    uniq = rng.permutation(B)[:n].astype(np.int32)
    dst = torch.from_numpy(val.copy()).cuda()
    src = torch.from_numpy(rng.standard_normal((n, T)).astype(np.float32)).cuda()
    pol.index_copy(dst, torch.from_numpy(uniq), src)
    expect = val.copy()
    expect[uniq] = src.cpu().numpy()
    np.testing.assert_array_equal(dst.cpu().numpy(), expect)
