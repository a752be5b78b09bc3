"""Pin the CPU oracle (and this library's kernels) against the reference's own
CUDA kernels, run on the GPU from oracle/_ref/libptcg_ref.so
(oracle/build_ref.py compiles it from the reference checkout):

- PPO loss: ppo_loss_fwd_bwd (native/src/pufferlib.cu:1368-1449) against
  oracle.ppo_loss and ptcg_ppo_loss: the seven loss sums, the logit and
  value gradients, the ratio;
- sampler: sample_logits (pufferlib.cu:584-718) on curand Philox states
  against oracle.sample_logits and ptcg_sample_logits, fed the uniform the
  reference kernel draws (read from a copy of each state);
- negamax advantage: ptcg_puff_advantage (native/model/ptcg_model2.cu:
  288-321, compiled for the reference default shape) against
  oracle.negamax_advantage and ptcg_negamax_advantage.

These parts have no torch implementation in the reference, so the kernels
themselves are the reference.  Skipped when the harness was not built.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libptcg_ref.so")
P, I, F = C.c_void_p, C.c_int, C.c_float


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libptcg_ref.so not built (python oracle/build_ref.py --ref ...)")
    # the trainer code around the kernels references the C env, which is not
    # linked and never called: bind lazily
    h = C.CDLL(REF_LIB, mode=os.RTLD_LAZY)
    sig = {
        "ref_rng_state_bytes": (C.c_long, []),
        "ref_rng_init": (I, [P, C.c_ulonglong, I, P]),
        "ref_draw_uniforms": (I, [P, P, I, P]),
        "ref_sample_logits": (I, [P, I, I, P, I, P, P, P, P, P, P]),
        "ref_ppo_loss": (I, [P, I, I, I, P, P, P, P, P, P, P, F, F, F, P, P, P, P, P, P, P,
                             P, P, P]),
        "ref_puff_advantage": (I, [P, P, P, P, P, P, I, I, F, F, F, F, P]),
        "ref_obs_size": (C.c_long, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(h, name)
        fn.restype, fn.argtypes = res, args
    return h


def _p(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _ppo_inputs(n_seg, horizon, nopt, seed):
    rng = np.random.default_rng(seed)
    nt = n_seg * horizon
    scores = (rng.standard_normal((nt, nopt)) * 1.5).astype(np.float32)
    mask = (rng.random((nt, nopt)) < 0.3).astype(np.float32)
    mask[np.arange(nt), rng.integers(0, nopt, nt)] = 1.0
    mask[0] = 0.0
    mask[0, 7] = 1.0                                   # a single legal option
    act = np.array([rng.choice(np.nonzero(m)[0]) for m in mask], np.float32)
    vpred = rng.standard_normal(nt).astype(np.float32)
    old = rng.normal(-1.5, 0.6, nt).astype(np.float32)
    adv = rng.standard_normal(nt).astype(np.float32)
    val = (vpred + rng.normal(0, 0.4, nt)).astype(np.float32)     # both vf-clip branches
    ret = rng.standard_normal(nt).astype(np.float32)
    prio = rng.uniform(0.5, 2.0, n_seg).astype(np.float32)
    return scores, mask, act, vpred, old, adv, val, ret, prio


@pytest.mark.parametrize("nopt", [64, 128])
def test_ppo_loss_pinned_to_reference_kernel(pkg, oracle, ref, nopt):
    n_seg, horizon = 24, 32
    nt = n_seg * horizon
    scores, mask, act, vpred, old, adv, val, ret, prio = _ppo_inputs(n_seg, horizon, nopt, 7)
    hyper = dict(clip=0.2, vf_clip=0.2, vf_coef=0.5, ent_coef=0.01)
    dec = _cuda(np.concatenate([scores, vpred[:, None]], 1))
    d_act, d_old, d_adv, d_val, d_ret, d_prio, d_mask = [
        _cuda(x) for x in (act, old, adv, val, ret, prio, mask)]
    ent = torch.tensor([hyper["ent_coef"]], device="cuda")
    size = torch.tensor([nopt], dtype=torch.int32, device="cuda")
    gl = torch.zeros(nt, nopt, device="cuda")
    gv = torch.zeros(nt, device="cuda")
    ratio = torch.zeros(nt, device="cuda")
    newv = torch.zeros(nt, device="cuda")
    losses = torch.zeros(8, device="cuda")
    lout = torch.zeros(1, device="cuda")
    scratch = torch.zeros(4, device="cuda")
    rc = ref.ref_ppo_loss(_p(dec), n_seg, horizon, nopt, _p(d_act), _p(d_old), _p(d_adv),
                          _p(d_val), _p(d_ret), _p(d_prio), _p(d_mask), hyper["clip"],
                          hyper["vf_clip"], hyper["vf_coef"], _p(ent), _p(size), _p(gl), _p(gv),
                          _p(ratio), _p(newv), _p(losses), _p(lout), _p(scratch), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    r_loss = losses.cpu().numpy()
    r_gl, r_gv = gl.cpu().numpy(), gv.cpu().numpy()
    # reference loss order: pg, vf, ent, total, old_approx_kl, approx_kl, clipfrac
    keys = ["pg", "vf", "ent", "total", "old_approx_kl", "approx_kl", "clipfrac"]
    assert r_loss[7] == 1.0 and abs(lout.item() - r_loss[3]) <= 1e-6 * max(1, abs(r_loss[3]))
    np.testing.assert_array_equal(newv.cpu().numpy(), vpred)

    # CPU oracle against the reference kernel
    st, d_scores, d_values, _, o_ratio = oracle.ppo_loss(scores, mask, vpred, act, old, adv, val,
                                                         ret, prio, n_seg, horizon, **hyper)
    for k, key in enumerate(keys):
        assert abs(st[key] - r_loss[k]) <= 2e-5 * max(1.0, abs(r_loss[k])), (key, st[key], r_loss[k])
    legal = mask != 0
    np.testing.assert_allclose(d_scores[legal], r_gl[legal], rtol=1e-4, atol=2e-8)
    assert np.abs(r_gl[~legal]).max() <= 1e-30
    np.testing.assert_allclose(d_values, r_gv, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(o_ratio, ratio.cpu().numpy(), rtol=1e-5)

    # this library's fused kernel against the reference kernel
    pol = pkg.PTCGPolicy(pkg.config.PRESETS["tiny"].with_(nopt=nopt), precision="fp32")
    grad, nlp, my_ratio, stats = pol.ppo_loss(dec, mask, act, old, adv, val, ret, prio, n_seg,
                                              horizon, **hyper)
    torch.cuda.synchronize()
    mine = stats.cpu().numpy()
    for k, key in enumerate(keys):
        j = ["total", "pg", "vf", "ent", "old_approx_kl", "approx_kl", "clipfrac"].index(key)
        assert abs(mine[j] - r_loss[k]) <= 2e-5 * max(1.0, abs(r_loss[k])), (key, mine[j], r_loss[k])
    g = grad.cpu().numpy()
    np.testing.assert_allclose(g[:, :nopt][legal], r_gl[legal], rtol=1e-4, atol=2e-8)
    np.testing.assert_allclose(g[:, nopt], r_gv, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(my_ratio.cpu().numpy(), ratio.cpu().numpy(), rtol=1e-5)


@pytest.mark.parametrize("nopt", [64, 128])
def test_sampler_pinned_to_reference_kernel(pkg, oracle, ref, nopt):
    n = 4096
    rng = np.random.default_rng(3)
    scores = (rng.standard_normal((n, nopt)) * 2).astype(np.float32)
    mask = (rng.random((n, nopt)) < 0.3).astype(np.float32)
    mask[np.arange(n), rng.integers(0, nopt, n)] = 1.0
    dec = _cuda(np.concatenate([scores, rng.standard_normal((n, 1)).astype(np.float32)], 1))
    d_mask = _cuda(mask)
    states = torch.zeros(n * ref.ref_rng_state_bytes(), dtype=torch.uint8, device="cuda")
    assert ref.ref_rng_init(_p(states), 1234, n, _stream()) == 0
    u = torch.zeros(n, device="cuda")
    assert ref.ref_draw_uniforms(_p(states), _p(u), n, _stream()) == 0
    size = torch.tensor([nopt], dtype=torch.int32, device="cuda")
    act, logp, val = (torch.zeros(n, device="cuda") for _ in range(3))
    assert ref.ref_sample_logits(_p(dec), n, nopt, _p(d_mask), nopt, _p(size), _p(act), _p(logp),
                                 _p(val), _p(states), _stream()) == 0
    torch.cuda.synchronize()
    r_act, r_logp = act.cpu().numpy().astype(np.int64), logp.cpu().numpy()
    uu = u.cpu().numpy()
    np.testing.assert_array_equal(val.cpu().numpy(), dec[:, -1].cpu().numpy())
    assert np.all(mask[np.arange(n), r_act] == 1)
    # oracle inverse CDF on the same uniforms; rows within 1e-5 of a CDF
    # boundary may round either way and are excluded
    o_act, o_logp, margin = oracle.sample_logits(scores, mask, uu)
    ok = margin > 1e-5
    assert ok.mean() > 0.99
    np.testing.assert_array_equal(o_act[ok], r_act[ok])
    np.testing.assert_allclose(o_logp[ok], r_logp[ok], atol=1e-5)
    # this library's sampler on the same uniforms
    pol = pkg.PTCGPolicy(pkg.config.PRESETS["tiny"].with_(nopt=nopt), precision="fp32")
    m_act, m_logp, m_val = pol.sample(dec, d_mask, u)
    m_act = m_act.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(m_act[ok], r_act[ok])
    np.testing.assert_allclose(m_logp.cpu().numpy()[ok], r_logp[ok], atol=1e-5)


def test_advantage_pinned_to_reference_kernel(pkg, oracle, ref):
    s = pkg.config.PRESETS["default"]
    assert ref.ref_obs_size() == s.obs_size
    B, T = 7, 24
    rng = np.random.default_rng(9)
    obs = pkg.synth.make_obs(s, B * T, 2).reshape(B, T, -1)
    vals = rng.standard_normal((B, T)).astype(np.float32)
    rew = rng.standard_normal((B, T)).astype(np.float32)
    dones = (rng.random((B, T)) < 0.1).astype(np.float32)
    imp = rng.uniform(0.5, 1.5, (B, T)).astype(np.float32)
    args = [_cuda(x) for x in (vals, rew, dones, imp, obs)]
    adv = torch.zeros(B, T, device="cuda")
    assert ref.ref_puff_advantage(*[_p(a) for a in args], _p(adv), B, T, 0.99, 0.95, 1.0, 1.0,
                                  _stream()) == 0
    torch.cuda.synchronize()
    r = adv.cpu().numpy()
    o = oracle.negamax_advantage(vals, rew, dones, imp, obs[:, :, s.seat_col], 0.99, 0.95, 1.0, 1.0)
    np.testing.assert_allclose(o, r, rtol=1e-6, atol=1e-6)
    pol = pkg.PTCGPolicy(s, precision="fp32")
    mine = pol.advantage(*args, 0.99, 0.95, 1.0, 1.0).cpu().numpy()
    np.testing.assert_array_equal(mine, r)
