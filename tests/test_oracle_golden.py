"""Pin the CPU oracle against fixtures produced by the reference's own torch
model (tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

GOLD = os.path.join(ROOT, "tests", "golden")
PRESETS = ["tiny", "small", "c0", "default", "c4"]


def _close(a, b, rtol=2e-4, atol=2e-5):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    scale = max(np.abs(b).max(), 1e-12)
    err = np.abs(a - b).max()
    assert err <= atol + rtol * scale, f"max|d|={err:.3e} scale={scale:.3e}"


@pytest.mark.parametrize("preset", PRESETS)
def test_oracle_matches_reference(preset, oracle, pkg):
    z = np.load(os.path.join(GOLD, f"ref_{preset}.npz"))
    s = pkg.config.PRESETS[preset]
    wseed, tseed, _, _ = [int(x) for x in z["seeds"]]
    blob = pkg.synth.make_weights(s, wseed)
    assert abs(blob.astype(np.float64).sum() - float(z["blob_sum"])) < 1e-6 * max(1, abs(float(z["blob_sum"])))
    assert abs((blob.astype(np.float64) ** 2).sum() - float(z["blob_sq"])) < 1e-6 * float(z["blob_sq"])
    T = oracle.tables_to_torch(pkg.synth.make_tables(s, tseed))
    P = oracle.params_from_blob(blob, s, requires_grad=True)
    obs = torch.from_numpy(z["obs"])
    torch.set_float32_matmul_precision("highest")

    with torch.no_grad():
        scores, logits, value = oracle.forward_eval(P, T, obs, s)
    mask = z["logits"] > -1e8
    _close(logits.numpy()[mask], z["logits"][mask])
    assert np.all((logits.numpy() <= -1e8) == ~mask)
    _close(value.numpy(), z["value"])

    out = oracle.forward_train(P, T, obs, s)
    _close(out["blind_v"].detach().numpy(), z["blind_v"])
    _close(torch.nn.functional.softplus(out["hand_lin"]).detach().numpy(), z["hand_pred"])
    _close(out["prize_logits"].detach().numpy(), z["prize_logits"])

    l_aux, parts = oracle.aux_loss(out, obs, torch.from_numpy(z["returns"]), s)
    for k in ("blind", "hand", "prize"):
        assert abs(float(parts[k]) - float(z["aux_" + k])) <= 1e-5 * max(1e-3, abs(float(z["aux_" + k])))

    sur = (out["scores"] * torch.from_numpy(z["d_scores"])).sum() \
        + (out["oracle_v"] * torch.from_numpy(z["d_value"])).sum() + l_aux
    sur.backward()
    for name, shp in pkg.config.param_table(s):
        g = P[name].grad
        g = np.zeros(shp) if g is None else g.numpy().astype(np.float64).ravel()
        norm = float(z[f"g_{name}_norm"])
        tol = 1e-4 * max(norm, 1e-9) + 1e-9
        assert abs(np.sqrt((g ** 2).sum()) - norm) <= tol, name
        idx = z[f"g_{name}_idx"]
        vals = z[f"g_{name}_val"].astype(np.float64)
        assert np.abs(g[idx] - vals).max() <= tol, name
        rng = np.random.default_rng(5000 + [n for n, _ in pkg.config.param_table(s)].index(name))
        rng.choice(g.size, min(256, g.size), replace=False)
        proj = rng.standard_normal((4, g.size)) @ g
        assert np.abs(proj - z[f"g_{name}_proj"]).max() <= 1e-4 * max(np.abs(z[f"g_{name}_proj"]).max(), 1e-9) * 10 + 1e-9, name


def test_param_counts(pkg):
    c = pkg.config
    assert c.param_count(c.PRESETS["default"]) == 4465812     # docs/model.md:190
    assert c.param_count(c.PRESETS["c0"]) == 7035536
    assert c.param_count(c.PRESETS["c4"]) == 33626000
    assert c.PRESETS["default"].obs_size == 10944
    assert c.PRESETS["c0"].obs_size == 5920
    assert c.PRESETS["c4"].obs_size == 11616
