"""On-disk formats through the C-ABI: packed fp32 weight files, the
reference trainer's PTCGSTA1 state file (native/src/bindings.cu:252-341)
and the PTCGADM1 Adam state file, each checked against a Python reading /
writing of the same byte layout."""
import struct

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pol(pkg, seed=21):
    s = pkg.config.PRESETS["tiny"]
    return pkg.PTCGPolicy(s, precision="fp32", tables=pkg.synth.make_tables(s, 11),
                          weights=pkg.synth.make_weights(s, seed), train_rows=8)


def _step(pkg, pol):
    """one Adam step so that the moments are non-zero"""
    g = pol.arena(1)
    g.copy_(torch.randn_like(g) * 1e-2)
    pol.adam_step(lr=1e-3)
    torch.cuda.synchronize()


def test_weight_file_roundtrip(pkg, tmp_path):
    pol = _pol(pkg)
    p = tmp_path / "w.bin"
    pol.save_weights_file(p)
    blob = np.fromfile(p, np.float32)
    np.testing.assert_array_equal(blob, pol.save_weights())
    other = _pol(pkg, seed=5)
    other.load_weights_file(p)
    np.testing.assert_array_equal(other.save_weights(), blob)
    (tmp_path / "short.bin").write_bytes(blob[:-1].tobytes())
    with pytest.raises(Exception, match="size mismatch"):
        other.load_weights_file(tmp_path / "short.bin")


def test_ptcgsta1_layout_and_roundtrip(pkg, tmp_path):
    pol = _pol(pkg)
    _step(pkg, pol)
    p = tmp_path / "s.state"
    pol.save_state(p, global_step=1234, epoch=7, fmt="PTCGSTA1")
    raw = p.read_bytes()
    magic, gs, ep, n = struct.unpack("<8sqqq", raw[:32])
    assert (magic, gs, ep, n) == (b"PTCGSTA1", 1234, 7, pol.n_params)
    body = np.frombuffer(raw[32:], np.float32)
    assert body.size == 2 * n
    np.testing.assert_array_equal(body[:n], pol.save_weights())
    np.testing.assert_array_equal(body[n:], pol.packed(2))
    other = _pol(pkg, seed=5)
    assert other.load_state(p) == (1234, 7)
    np.testing.assert_array_equal(other.save_weights(), body[:n])
    np.testing.assert_array_equal(other.packed(2), body[n:])


def test_ptcgsta1_written_like_the_reference_loads(pkg, tmp_path):
    """a file laid out as bindings.cu:save_state writes it"""
    pol = _pol(pkg)
    rng = np.random.default_rng(3)
    w = rng.standard_normal(pol.n_params).astype(np.float32)
    mom = rng.standard_normal(pol.n_params).astype(np.float32)
    p = tmp_path / "ref.state"
    p.write_bytes(struct.pack("<8sqqq", b"PTCGSTA1", 99, 3, pol.n_params) + w.tobytes() + mom.tobytes())
    assert pol.load_state(p) == (99, 3)
    np.testing.assert_array_equal(pol.save_weights(), w)
    np.testing.assert_array_equal(pol.packed(2), mom)
    bad = tmp_path / "bad.state"
    bad.write_bytes(b"NOTSTATE" + bytes(64))
    with pytest.raises(Exception, match="not a PTCGSTA1"):
        pol.load_state(bad)


def test_ptcgadm1_roundtrip(pkg, tmp_path):
    pol = _pol(pkg)
    _step(pkg, pol)
    _step(pkg, pol)
    p = tmp_path / "a.state"
    pol.save_state(p, global_step=50, epoch=2, fmt="PTCGADM1")
    raw = p.read_bytes()
    magic, gs, ep, n, astep = struct.unpack("<8sqqqq", raw[:40])
    assert (magic, gs, ep, n, astep) == (b"PTCGADM1", 50, 2, pol.n_params, pol.step)
    body = np.frombuffer(raw[40:], np.float32)
    np.testing.assert_array_equal(body[2 * n:], pol.packed(3))
    other = _pol(pkg, seed=5)
    assert other.load_state(p) == (50, 2)
    assert other.step == pol.step
    for k in (2, 3):
        np.testing.assert_array_equal(other.packed(k), pol.packed(k))
    np.testing.assert_array_equal(other.save_weights(), pol.save_weights())
