"""The rollout forward's fused MLP kernel (FFN1 -> GELU -> FFN2 + bias +
residual in one tcgen05 kernel, the hidden activation kept on chip) against
the two-GEMM path it replaces, and the fused forward against the CPU oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = np.asarray(a, np.float64).ravel(); b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("preset,rows", [("small", 7), ("c0", 300), ("default", 130)])
def test_fused_mlp_matches_two_gemms(pkg, preset, rows):
    import ptcg_b200.native as n
    lib = n.lib()
    s = pkg.config.PRESETS[preset]
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=pkg.synth.make_tables(s, 11),
                         weights=pkg.synth.make_weights(s, 21), rollout_rows=rows)
    obs = pkg.synth.make_obs_batch(s, rows, 5)
    try:
        assert lib.ptcg_set_fused_mlp(0) == 0
        ref = pol.forward(obs).cpu().numpy()
        assert lib.ptcg_set_fused_mlp(1) == 0
        out = pol.forward(obs).cpu().numpy()
        assert lib.ptcg_device_error() == 0
    finally:
        lib.ptcg_set_fused_mlp(0)
    a, b = s.offsets["opt_mask"]
    legal = obs[:, a:b] != 0
    assert np.isfinite(out[:, :-1][legal]).all() and np.isfinite(out[:, -1]).all()
    # same GELU and bf16 rounding of the hidden units, same K order; only the
    # final bias + residual additions may round differently
    assert _rel(out[:, :-1][legal], ref[:, :-1][legal]) <= 1e-3
    assert _rel(out[:, -1], ref[:, -1]) <= 1e-3


def test_fused_mlp_forward_vs_oracle(pkg, oracle):
    torch.set_float32_matmul_precision("highest")
    s = pkg.config.PRESETS["c0"]
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    obs = pkg.synth.make_obs(s, 6, 3, edge=True)
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=blob, rollout_rows=6)
    import ptcg_b200.native as n
    lib = n.lib()
    try:
        assert lib.ptcg_set_fused_mlp(1) == 0
        out = pol.forward(obs).cpu().numpy()
        assert lib.ptcg_device_error() == 0
    finally:
        lib.ptcg_set_fused_mlp(0)
    P = oracle.params_from_blob(blob, s)
    T = oracle.tables_to_torch(tabs)
    with torch.no_grad():
        sc, _, v = oracle.forward_eval(P, T, torch.from_numpy(obs), s)
    a, b = s.offsets["opt_mask"]
    legal = obs[:, a:b] != 0
    assert _rel(out[:, :-1][legal], sc.numpy()[legal]) <= 2e-2
    assert _rel(out[:, -1], v.numpy()) <= 2e-2
