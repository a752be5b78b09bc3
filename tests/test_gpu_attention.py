"""Attention kernels (fp32 SIMT and bf16 tensor-core flash attention) against
torch scaled_dot_product_attention with a boolean key-padding mask."""
import ctypes as C

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


IMPL = {"mma": 0, "tc": 1, "tc_bwd": 2}


@pytest.fixture(params=["mma", "tc", "tc_bwd"])
def attn_impl(request, pkg):
    """bf16 attention kernels under test: mma.sync, tcgen05 / TMEM for both
    passes, or the tcgen05 backward after the mma.sync forward."""
    import ptcg_b200.native as n
    lib = n.lib()
    old = lib.ptcg_get_attention_impl()
    assert lib.ptcg_set_attention_impl(IMPL[request.param]) == 0
    yield request.param
    lib.ptcg_set_attention_impl(old)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("L,H", [(129, 8), (186, 8), (17, 2), (257, 16), (314, 16), (33, 4)])
def test_attention_matches_sdpa(pkg, dtype, L, H, attn_impl):
    import ptcg_b200.native as n
    lib = n.lib()
    if dtype == "fp32" and attn_impl != "mma":
        pytest.skip("the tcgen05 kernels take bf16 operands")
    torch.manual_seed(L * 10 + H)
    nseq, D = 5, H * 32
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    qkv = torch.randn(nseq * L, 3 * D, device="cuda").to(tdt)
    keep = torch.rand(nseq, L, device="cuda") < 0.7
    keep[:, 0] = True
    keep[1, L // 2:] = False                       # long masked tail
    keep_u8 = keep.to(torch.uint8).contiguous()
    out = torch.zeros(nseq * L, D, device="cuda", dtype=tdt)
    lse = torch.zeros(nseq, H, L, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    dt = 1 if dtype == "bf16" else 0
    assert lib.ptcg_attention_fwd(dt, _p(qkv), 3 * D, _p(keep_u8), _p(out), D, _p(lse), nseq, L, H, s) == 0
    assert lib.ptcg_device_error() == 0
    q, k, v = qkv.float().view(nseq, L, 3, H, 32).permute(2, 0, 3, 1, 4).unbind(0)
    q.requires_grad_(True); k.requires_grad_(True); v.requires_grad_(True)
    ref = F.scaled_dot_product_attention(q, k, v, attn_mask=keep.view(nseq, 1, 1, L))
    ref_o = ref.transpose(1, 2).reshape(nseq * L, D)
    tol = 2e-2 if dtype == "bf16" else 1e-5
    err = (out.float() - ref_o).abs().max().item() / ref_o.abs().max().item()
    assert err < tol, err
    sc = (q @ k.transpose(-1, -2)) / 32 ** 0.5
    sc = sc.masked_fill(~keep.view(nseq, 1, 1, L), float("-inf"))
    ref_lse = torch.logsumexp(sc, -1)
    assert (lse - ref_lse).abs().max().item() < (2e-2 if dtype == "bf16" else 1e-4)
    # backward
    dout = torch.randn(nseq * L, D, device="cuda").to(tdt)
    ref_o.backward(dout.float())
    dqkv = torch.zeros_like(qkv)
    dbias = torch.zeros(3 * D, device="cuda")
    assert lib.ptcg_attention_bwd(dt, _p(qkv), 3 * D, _p(keep_u8), _p(out), D, _p(dout), D,
                                  _p(lse), _p(dqkv), 3 * D, _p(dbias), nseq, L, H, s) == 0
    torch.cuda.synchronize()
    refd = torch.stack([q.grad, k.grad, v.grad], 2).permute(0, 3, 2, 1, 4).reshape(nseq * L, 3 * D)
    for part in range(3):
        a = dqkv.float()[:, part * D:(part + 1) * D]
        b = refd[:, part * D:(part + 1) * D]
        e = (a - b).norm().item() / b.norm().item()
        assert e < (3e-2 if dtype == "bf16" else 1e-4), (part, e)
        # fp32 column sums (bias grads); judged against the sum of |values|
        # since the K part is analytically zero (softmax shift invariance)
        cs = dbias[part * D:(part + 1) * D]
        scale = b.abs().sum(0).norm().item()
        assert (cs - b.sum(0)).norm().item() <= (3e-2 if dtype == "bf16" else 1e-4) * scale, part


@pytest.mark.parametrize("L,H", [(129, 8), (186, 8), (33, 4)])
def test_attention_bwd_zero_dout_blocks(pkg, L, H):
    """Query blocks whose dO rows are all zero (unread rows such as padding)
    are skipped by the bf16 backward: the result must equal the dense one,
    with exactly zero dQ on those rows."""
    import ptcg_b200.native as n
    lib = n.lib()
    torch.manual_seed(L + H)
    nseq, D = 4, H * 32
    qkv = torch.randn(nseq * L, 3 * D, device="cuda").to(torch.bfloat16)
    keep = torch.rand(nseq, L, device="cuda") < 0.8
    keep[:, 0] = True
    nvalid = [L, L // 2, L - 17, 5]
    for i, nv in enumerate(nvalid):
        keep[i, nv:] = False                          # padded suffix
    keep_u8 = keep.to(torch.uint8).contiguous()
    out = torch.zeros(nseq * L, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(nseq, H, L, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.ptcg_attention_fwd(1, _p(qkv), 3 * D, _p(keep_u8), _p(out), D, _p(lse), nseq, L, H, s) == 0
    dout = torch.randn(nseq * L, D, device="cuda")
    rowmask = torch.ones(nseq, L, device="cuda")
    for i, nv in enumerate(nvalid):
        rowmask[i, nv:] = 0                           # nothing reads the padded rows
    rowmask[0, 16:48] = 0                             # and two whole blocks in the middle
    dout = (dout * rowmask.view(-1, 1)).to(torch.bfloat16)
    dout[rowmask.view(-1) == 0] = -0.0                # negative zero counts as zero
    q, k, v = qkv.float().view(nseq, L, 3, H, 32).permute(2, 0, 3, 1, 4).unbind(0)
    q.requires_grad_(True); k.requires_grad_(True); v.requires_grad_(True)
    ref = F.scaled_dot_product_attention(q, k, v, attn_mask=keep.view(nseq, 1, 1, L))
    ref.transpose(1, 2).reshape(nseq * L, D).backward(dout.float())
    dqkv = torch.full_like(qkv, 7.0)                  # every element must be written
    dbias = torch.zeros(3 * D, device="cuda")
    assert lib.ptcg_attention_bwd(1, _p(qkv), 3 * D, _p(keep_u8), _p(out), D, _p(dout), D,
                                  _p(lse), _p(dqkv), 3 * D, _p(dbias), nseq, L, H, s) == 0
    torch.cuda.synchronize()
    refd = torch.stack([q.grad, k.grad, v.grad], 2).permute(0, 3, 2, 1, 4).reshape(nseq * L, 3 * D)
    for part in range(3):
        a = dqkv.float()[:, part * D:(part + 1) * D]
        b = refd[:, part * D:(part + 1) * D]
        assert (a - b).norm().item() / b.norm().item() < 3e-2, part
    zero_rows = rowmask.view(-1) == 0
    assert (dqkv.float()[zero_rows, :D] == 0).all()


@pytest.mark.parametrize("preset", ["c0", "c4", "default"])
def test_model_forward_with_tc_attention(pkg, oracle, preset):
    """The whole bf16 forward with the tcgen05 attention kernels (row
    extents, multi-chunk keys at c4) against the CPU oracle."""
    import numpy as np
    import ptcg_b200.native as n
    lib = n.lib()
    torch.set_float32_matmul_precision("highest")
    s = pkg.config.PRESETS[preset]
    nrows = 6
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    obs = pkg.synth.make_obs(s, nrows, 3, edge=True)
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=blob, rollout_rows=nrows)
    old = lib.ptcg_get_attention_impl()
    assert lib.ptcg_set_attention_impl(1) == 0
    try:
        out = pol.forward(obs).cpu().numpy()
        assert lib.ptcg_device_error() == 0
    finally:
        lib.ptcg_set_attention_impl(old)
    P = oracle.params_from_blob(blob, s)
    T = oracle.tables_to_torch(tabs)
    with torch.no_grad():
        sc, _, v = oracle.forward_eval(P, T, torch.from_numpy(obs), s)
    a, b = s.offsets["opt_mask"]
    legal = obs[:, a:b] != 0
    rel = lambda x, y: float(np.linalg.norm(x - y) / np.linalg.norm(y))
    assert rel(out[:, :-1][legal], sc.numpy()[legal]) <= 2e-2
    assert rel(out[:, -1], v.numpy()) <= 2e-2


@pytest.mark.parametrize("preset", ["small", "c0", "default", "c4"])
def test_train_grads_with_tc_backward(pkg, oracle, preset):
    """bf16 gradients of forward_train -> PPO loss -> backward with the
    tcgen05 attention backward (sequences whose extent fits one 128-row tile;
    longer ones, e.g. the edge rows, through the mma.sync backward) against
    the CPU oracle, and against the same step with the mma.sync backward."""
    import numpy as np
    import ptcg_b200.native as n
    from test_gpu_parity import ROWS, TOL, _rollout_tensors, make, oracle_fwd, rel
    lib = n.lib()
    torch.set_float32_matmul_precision("highest")
    rows = ROWS[preset]
    s, tabs, blob, obs, pol = make(pkg, preset, "bf16", rows)
    sc, v = oracle_fwd(oracle, s, tabs, blob, obs)
    mask, act, old_lp, adv, ret, val = _rollout_tensors(pkg, oracle, s, obs, sc, 5)
    prio = np.ones(1, np.float32)
    old = lib.ptcg_get_attention_impl()
    grads = {}
    try:
        for impl in (0, 2):
            assert lib.ptcg_set_attention_impl(impl) == 0
            out = pol.forward_train(obs)
            grad, _, _, _ = pol.ppo_loss(out, mask, act, old_lp, adv, val, ret, prio, 1, rows)
            pol.backward(grad, ret)
            grads[impl] = pol.grads_packed()
            assert lib.ptcg_device_error() == 0
    finally:
        lib.ptcg_set_attention_impl(old)
    P = oracle.params_from_blob(blob, s, requires_grad=True)
    T = oracle.tables_to_torch(tabs)
    _, _, og = oracle.train_grads(P, T, obs, s, act, old_lp, adv, val, ret, prio, 1, rows)
    ref = np.concatenate([og[name].detach().numpy().ravel() for name, _ in pkg.config.param_table(s)])
    g2 = grads[2][:ref.size]
    assert np.isfinite(g2).all()
    assert rel(g2, ref) <= TOL["bf16"], rel(g2, ref)
    assert rel(g2, grads[0][:ref.size]) <= TOL["bf16"], rel(g2, grads[0][:ref.size])


def test_tc_backward_matches_mma_backward_many_rows(pkg):
    """The PPO step's gradients at c0 over 512 synthetic rows (every extent
    the generator draws, padded and full sequences) with the tcgen05
    backward against the mma.sync backward, same forward."""
    import numpy as np
    import ptcg_b200.native as n
    from test_gpu_parity import rel
    lib = n.lib()
    s = pkg.config.PRESETS["c0"]
    n_seg, horizon = 8, 64
    nt = n_seg * horizon
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    obs = pkg.synth.make_obs_batch(s, nt, 5)
    a, b = s.offsets["opt_mask"]
    act = pkg.synth.sample_legal(obs[:, a:b], 3)
    rng = np.random.default_rng(4)
    old_lp = rng.normal(-2.0, 0.5, nt).astype(np.float32)
    adv = rng.standard_normal(nt).astype(np.float32)
    ret = rng.standard_normal(nt).astype(np.float32)
    val = (0.1 * rng.standard_normal(nt)).astype(np.float32)
    prio = np.ones(n_seg, np.float32)
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=blob, train_rows=256)
    old = lib.ptcg_get_attention_impl()
    res = {}
    try:
        for impl in (0, 2):
            assert lib.ptcg_set_attention_impl(impl) == 0
            st = pol.train_step(obs, act, old_lp, adv, val, ret, prio, n_seg, horizon,
                                skip_adam=True).cpu().numpy()
            res[impl] = (st, pol.grads_packed())
            assert lib.ptcg_device_error() == 0
    finally:
        lib.ptcg_set_attention_impl(old)
    (s0, g0), (s2, g2) = res[0], res[2]
    assert np.isfinite(g2).all()
    assert rel(g2, g0) <= 1e-2, rel(g2, g0)
    np.testing.assert_allclose(s2[:8], s0[:8], rtol=1e-3, atol=1e-5)
