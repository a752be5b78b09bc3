"""Parity at the size bench.py runs: c0, bf16, 16384-row micro-batches.

At this size the trunk GEMMs have M = 2.1 M rows, the FFN1 output holds
more than 2^31 elements and the weight-gradient GEMMs split K over about
2 M rows, so 64-bit indexing and the split-K planner are exercised where the
small parity tests cannot reach them.

- forward_train on 16384 rows: sampled rows (first, middle, last) against
  the CPU oracle, bf16 tolerance.
- ptcg_train_step on one 32768-row minibatch (512 segments x 64) in
  16384-row micro-batches against the same step in 4096-row micro-batches:
  gradients within 5e-3, loss stats within 1e-3.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MICRO = 16384
SEGMENTS, HORIZON = 512, 64


def rel(a, b):
    a = np.asarray(a, np.float64).ravel(); b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def c0_case(pkg):
    torch.cuda.empty_cache()
    s = pkg.config.PRESETS["c0"]
    nt = SEGMENTS * HORIZON
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    obs = pkg.synth.make_obs_batch(s, nt, 77)
    a, b = s.offsets["opt_mask"]
    act = pkg.synth.sample_legal(obs[:, a:b], 3)
    rng = np.random.default_rng(12)
    old = rng.normal(-2.0, 0.5, nt).astype(np.float32)
    adv = rng.standard_normal(nt).astype(np.float32)
    ret = rng.standard_normal(nt).astype(np.float32)
    val = (0.1 * rng.standard_normal(nt)).astype(np.float32)
    prio = np.ones(SEGMENTS, np.float32)
    return s, tabs, blob, obs, (act, old, adv, val, ret, prio)


def test_forward_16384_rows_vs_oracle(pkg, oracle, c0_case):
    torch.set_float32_matmul_precision("highest")
    s, tabs, blob, obs, _ = c0_case
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=blob, train_rows=MICRO)
    out = pol.forward_train(obs[:MICRO]).cpu().numpy()
    pol.close()
    del pol
    torch.cuda.empty_cache()
    assert np.isfinite(out).all()
    rows = np.r_[0:96, MICRO // 2 - 48:MICRO // 2 + 48, MICRO - 96:MICRO]
    P = oracle.params_from_blob(blob, s)
    T = oracle.tables_to_torch(tabs)
    with torch.no_grad():
        sc, _, v = oracle.forward_eval(P, T, torch.from_numpy(obs[rows]), s)
    a, b = s.offsets["opt_mask"]
    legal = obs[rows, a:b] != 0
    got = out[rows]
    assert rel(got[:, :-1][legal], sc.numpy()[legal]) <= 2e-2
    assert rel(got[:, -1], v.numpy()) <= 2e-2


def test_train_step_micro_16384_vs_4096(pkg, c0_case):
    s, tabs, blob, obs, (act, old, adv, val, ret, prio) = c0_case
    res = []
    for micro in (MICRO, 4096):
        pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=blob, train_rows=micro)
        st = pol.train_step(obs, act, old, adv, val, ret, prio, SEGMENTS, HORIZON,
                            skip_adam=True).cpu().numpy()
        res.append((st, pol.grads_packed()))
        pol.close()
        del pol
        torch.cuda.empty_cache()
    (s1, g1), (s2, g2) = res
    assert np.isfinite(g1).all() and np.isfinite(s1[:8]).all()
    assert rel(g1, g2) <= 5e-3, rel(g1, g2)
    np.testing.assert_allclose(s1[:8], s2[:8], rtol=1e-3, atol=1e-5)
