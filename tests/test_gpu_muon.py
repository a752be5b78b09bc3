"""ptcg_muon_step (the reference trainer's optimizer) against the CPU
oracle's restatement of muon_step (native/src/muon.cu:209-297): two steps with
fresh gradients, exact fp32 (SIMT) and TF32 (bf16 mode) Newton-Schulz GEMMs,
and the gate veto."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-4, "bf16": 1e-2}


def _unpack(pkg, s, flat, offs):
    return {name: torch.from_numpy(flat[o:o + int(np.prod(shp))].astype(np.float64))
            for (name, shp), o in zip(pkg.config.param_table(s), offs)}


@pytest.mark.parametrize("prec", ["fp32", "bf16"])
@pytest.mark.parametrize("preset", ["tiny", "small"])
def test_muon_matches_oracle(pkg, oracle, preset, prec):
    s = pkg.config.PRESETS[preset]
    blob = pkg.synth.make_weights(s, 21)
    pol = pkg.PTCGPolicy(s, precision=prec, tables=pkg.synth.make_tables(s, 11), weights=blob)
    offs = pol.param_offsets()
    table = pkg.config.param_table(s)
    shapes = {name: (shp[0], shp[1] if len(shp) > 1 else 0) for name, shp in table}
    P = _unpack(pkg, s, pol.arena(0).cpu().numpy(), offs)
    Mo = {k: torch.zeros_like(v) for k, v in P.items()}
    hyper = dict(lr=0.02, momentum=0.95, weight_decay=0.01, wd_1d=0.05, max_norm=1.5)
    rng = np.random.default_rng(17)
    for step in range(2):
        # gradients in the parameter slices; the 16-byte alignment gaps stay 0
        g = torch.zeros(pol.arena(1).numel())
        for (name, shp), o in zip(table, offs):
            k = int(np.prod(shp))
            g[o:o + k] = torch.from_numpy(rng.standard_normal(k).astype(np.float32) * 0.05)
        pol.arena(1).copy_(g.cuda())
        G = _unpack(pkg, s, g.numpy(), offs)
        stats = pol.muon_step(**hyper)
        norm = oracle.muon_step(P, G, Mo, shapes, hyper["lr"], hyper["momentum"],
                                hyper["weight_decay"], hyper["wd_1d"], hyper["max_norm"])
        torch.cuda.synchronize()
        assert abs(stats[0].item() - norm) <= 1e-5 * norm and stats[1].item() == 1.0
    w = _unpack(pkg, s, pol.arena(0).cpu().numpy(), offs)
    m = _unpack(pkg, s, pol.arena(2).cpu().numpy(), offs)
    w0 = _unpack(pkg, s, np.frombuffer(np.asarray(blob, np.float32).tobytes(), np.float32).copy(),
                 [sum(int(np.prod(sh)) for _, sh in table[:i]) for i in range(len(table))])
    worst = []
    for name in P:
        d_gpu, d_ref = w[name] - w0[name], P[name] - w0[name]
        worst.append(((d_gpu - d_ref).norm().item() / max(d_ref.norm().item(), 1e-12), name))
        mr = (m[name] - Mo[name]).norm().item() / max(Mo[name].norm().item(), 1e-12)
        assert mr <= TOL[prec], (name, mr)
    worst.sort(reverse=True)
    assert worst[0][0] <= TOL[prec], worst[:4]


def test_muon_gate_vetoes_the_step(pkg, oracle):
    s = pkg.config.PRESETS["tiny"]
    pol = pkg.PTCGPolicy(s, precision="fp32", tables=pkg.synth.make_tables(s, 11),
                         weights=pkg.synth.make_weights(s, 21))
    pol.arena(1).copy_(torch.randn(pol.arena(1).numel(), device="cuda") * 0.05)
    w_before = pol.arena(0).clone()
    m_before = pol.arena(2).clone()
    gate = torch.zeros(1, device="cuda")
    stats = pol.muon_step(gate=gate)
    torch.cuda.synchronize()
    assert stats[1].item() == 0.0
    assert torch.equal(pol.arena(0), w_before) and torch.equal(pol.arena(2), m_before)
