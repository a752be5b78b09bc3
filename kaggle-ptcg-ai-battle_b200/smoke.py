"""One small forward + PPO train step on cuda:0 through the C-ABI, checked
against the CPU oracle (used by __graft_entry__.smoke)."""
import numpy as np
import torch

from .config import PRESETS
from . import synth
from .policy import PTCGPolicy


def run(preset="small", n=8, precision="bf16"):
    import ptcg_oracle as oracle          # test infrastructure: the checker only
    assert torch.cuda.is_available(), "smoke() needs a CUDA device"
    s = PRESETS[preset]
    tabs = synth.make_tables(s, 11)
    blob = synth.make_weights(s, 21)
    obs = synth.make_obs(s, n, 5, edge=True)
    pol = PTCGPolicy(s, precision=precision, tables=tabs, weights=blob,
                     rollout_rows=n, train_rows=n)
    out = pol.forward(obs).cpu().numpy()
    P = oracle.params_from_blob(blob, s)
    with torch.no_grad():
        sc, _, v = oracle.forward_eval(P, oracle.tables_to_torch(tabs), torch.from_numpy(obs), s)
    a, b = s.offsets["opt_mask"]
    legal = obs[:, a:b] != 0
    err_s = np.linalg.norm(out[:, :-1][legal] - sc.numpy()[legal]) / np.linalg.norm(sc.numpy()[legal])
    err_v = np.linalg.norm(out[:, -1] - v.numpy()) / np.linalg.norm(v.numpy())
    tol = 2e-2 if precision == "bf16" else 1e-4
    assert err_s <= tol and err_v <= tol, (err_s, err_v)
    rng = np.random.default_rng(0)
    act = np.array([rng.choice(np.nonzero(m)[0]) for m in obs[:, a:b]], np.float32)
    st = pol.train_step(obs, act, np.full(n, -2.0, np.float32),
                        rng.standard_normal(n).astype(np.float32),
                        np.zeros(n, np.float32), rng.standard_normal(n).astype(np.float32),
                        np.ones(1, np.float32), 1, n).cpu().numpy()
    assert np.isfinite(st).all() and st[9] == 1.0, st
    w = pol.save_weights()
    assert np.isfinite(w).all() and not np.array_equal(w, blob)
    print(f"smoke ok: {preset} {precision} n={n} rel err scores {err_s:.2e} value {err_v:.2e}, "
          f"loss {st[0]:.4f} grad-norm {st[8]:.4f}")
