"""CPU-only checks of the C-ABI library: it loads, exports every symbol that
include/ptcg_b200.h declares, and its layout functions agree with the
Python shape config (no compute calls without a GPU)."""
import ctypes as C

import pytest


def test_library_exports_header_symbols(pkg):
    import ptcg_b200.native as n
    h = n.lib()
    syms = n.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(h, s), s
    assert h.ptcg_abi_version() == 1


@pytest.mark.parametrize("preset", ["default", "c0", "c4", "tiny", "small"])
def test_layout_matches_config(pkg, preset):
    import ptcg_b200.native as n
    from ptcg_b200.config import PRESETS, param_table, param_count
    s = PRESETS[preset]
    h = n.lib()
    cs = n.PtcgShape.from_shape(s)
    assert h.ptcg_obs_size(C.byref(cs)) == s.obs_size
    assert h.ptcg_param_total(C.byref(cs)) == param_count(s)
    tab = param_table(s)
    assert h.ptcg_num_params(C.byref(cs)) == len(tab)
    for i, (name, shp) in enumerate(tab):
        nm = C.c_char_p(); r = C.c_long(); c = C.c_long()
        assert h.ptcg_param_info(C.byref(cs), i, C.byref(nm), C.byref(r), C.byref(c)) == 0
        assert nm.value.decode() == name
        assert (r.value, c.value) == (shp[0], shp[1] if len(shp) > 1 else 0)


def test_shape_validation(pkg):
    import ptcg_b200.native as n
    from ptcg_b200.config import PRESETS
    h = n.lib()
    bad = n.PtcgShape.from_shape(PRESETS["c0"].with_(heads=4))   # head width 64
    assert h.ptcg_obs_size(C.byref(bad)) == -1
    assert b"head width" in h.ptcg_last_error()
