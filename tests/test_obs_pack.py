"""Compact transfer form of observation rows (ptcg_obs_pack /
ptcg_obs_unpack): int16 id fields + fp32 float fields.

CPU: the host encoder against a numpy decoder of the documented layout
(exact round trip, sizes), and its refusal of ids that int16 cannot hold.
GPU: the device decoder restores the rows bit for bit, and the forward on
decoded rows equals the forward on the originals."""
import numpy as np
import pytest
import torch

from conftest import ROOT  # noqa: F401


def _runs(s):
    """(int runs, float runs) as (dst, count, stride) of the fp32 row."""
    o = s.offsets
    orc = o["oracle"][0]
    ints = [(o["tok_int"][0], s.ltok * 5, 1), (o["opt_int"][0], s.nopt * 6, 1),
            (o["opt_mask"][0], s.nopt, 1), (o["dec_int"][0], 8, 1),
            (orc, 24, 2), (orc + 48, 24, 3), (orc + 120, 8, 2)]
    floats = [(o["tok_float"][0], s.ltok * s.tok_f, 1), (o["opt_float"][0], s.nopt * 8, 1),
              (o["global_f"][0], 64, 1), (o["dec_float"][0], 16, 1),
              (orc + 1, 24, 2), (orc + 49, 24, 3), (orc + 50, 24, 3), (orc + 121, 8, 2)]
    return ints, floats


def _decode(s, packed):
    ints, floats = _runs(s)
    ni = sum(c for _, c, _ in ints)
    nf = sum(c for _, c, _ in floats)
    foff = (ni * 2 + 15) // 16 * 16
    n = packed.shape[0]
    iv = packed[:, :ni * 2].copy().view(np.int16)
    fv = packed[:, foff:foff + nf * 4].copy().view(np.float32)
    out = np.zeros((n, s.obs_size), np.float32)
    b = 0
    for d, c, st in ints:
        out[:, d + st * np.arange(c)] = iv[:, b:b + c]
        b += c
    b = 0
    for d, c, st in floats:
        out[:, d + st * np.arange(c)] = fv[:, b:b + c]
        b += c
    return out


@pytest.mark.parametrize("preset", ["c0", "c4", "default"])
def test_pack_roundtrip_host(pkg, preset):
    import ptcg_b200.native as n
    s = pkg.config.PRESETS[preset]
    obs = pkg.synth.make_obs(s, 7, 3)
    ti, oi = s.offsets["tok_int"][0], s.offsets["opt_int"][0]
    obs[0, ti] = -3                                        # ids the kernels clamp:
    obs[1, ti + 5] = s.n_cards + 5                         # negative, beyond the vocabulary,
    obs[2, oi + 1] = s.ltok + 3                            # pointers out of range
    obs[3, s.offsets["oracle"][0]] = 32767
    packed = n.obs_pack(s, obs)
    nb = n.lib().ptcg_obs_packed_bytes(n.C.byref(n.PtcgShape.from_shape(s)))
    assert packed.shape == (7, nb) and nb % 16 == 0 and nb < s.obs_size * 4
    ints, floats = _runs(s)
    assert sum(c for _, c, _ in ints) + sum(c for _, c, _ in floats) == s.obs_size
    cover = np.zeros(s.obs_size, np.int32)
    for d, c, st in ints + floats:
        cover[d + st * np.arange(c)] += 1
    assert (cover == 1).all()                              # every column exactly once
    ref = obs.copy()
    ref[ref == 0] = 0.0                                    # -0.0 ids come back as +0.0
    assert np.array_equal(_decode(s, packed), ref)


def test_pack_refuses_lossy_ids(pkg):
    import ptcg_b200.native as n
    s = pkg.config.PRESETS["c0"]
    obs = pkg.synth.make_obs(s, 3, 1)
    for col, val in ((s.offsets["tok_int"][0] + 5, 7.5), (s.offsets["opt_int"][0], 40000.0),
                     (s.offsets["oracle"][0], float("nan"))):
        bad = obs.copy()
        bad[2, col] = val
        with pytest.raises(n.PtcgError, match="int16"):
            n.obs_pack(s, bad)
    # float fields are carried as they are
    ok = obs.copy()
    ok[1, s.offsets["tok_float"][0]] = 7.5
    assert np.array_equal(_decode(s, n.obs_pack(s, ok))[1], ok[1])


@pytest.mark.gpu
@pytest.mark.parametrize("preset", ["c0", "c4"])
def test_unpack_on_device(pkg, preset):
    import ptcg_b200.native as n
    s = pkg.config.PRESETS[preset]
    obs = pkg.synth.make_obs_batch(s, 64, 9)
    tabs = pkg.synth.make_tables(s, 11)
    pol = pkg.PTCGPolicy(s, precision="bf16", tables=tabs, weights=pkg.synth.make_weights(s, 21),
                         rollout_rows=64)
    packed = torch.from_numpy(n.obs_pack(s, obs)).cuda()
    rows = pol.obs_unpack(packed)
    assert torch.equal(rows.cpu(), torch.from_numpy(obs))
    assert torch.equal(pol.forward(rows), pol.forward(obs))
