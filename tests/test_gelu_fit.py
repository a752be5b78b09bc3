"""The epilogue GELU's constants (csrc/common.cuh) against their generator
(csrc/fit_gelu.py) and the exact erf form, on the CPU: the same float32
operations in the same order as gelu1 / gelu2, with ex2 evaluated exactly
(the device's ex2.approx is bounded on the GPU in test_gpu_gemm.py)."""
import importlib.util
import os
import re

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "kaggle-ptcg-ai-battle_b200", "csrc")


def _constants():
    src = open(os.path.join(CSRC, "common.cuh")).read()
    c = {m.group(1): np.float32(float(m.group(2).rstrip("f")))
         for m in re.finditer(r"#define PTCG_GELU_(\w+)\s+([-0-9.eE+]+f)", src)}
    return [c[f"PN{k}"] for k in range(7, -1, -1)], c["UMAX"], c["S2"], c["S0"]


def _gelu_f32(x, pn, umax, s2, s0):
    f = np.float32
    u = np.minimum(np.abs(x), umax)
    p = np.full_like(x, pn[0])
    for k in pn[1:]:
        p = (p * u + k).astype(f)
    e = np.exp2((x * x * s2 + s0).astype(f)).astype(f)            # pdf(x)
    cdf = (f(0.5) + np.copysign((e * p + f(0.5)).astype(f), x)).astype(f)
    return (x * cdf).astype(f), (x * e + cdf).astype(f)


def test_gelu_constants_error_bound():
    erf = pytest.importorskip("scipy.special").erf
    pn, umax, s2, s0 = _constants()
    x = np.linspace(-12, 12, 2_000_001).astype(np.float32)
    g, dg = _gelu_f32(x, pn, umax, s2, s0)
    xd = x.astype(np.float64)
    cdf = 0.5 * (1 + erf(xd / np.sqrt(2)))
    pdf = np.exp(-0.5 * xd * xd) / np.sqrt(2 * np.pi)
    eg = (np.abs(g - xd * cdf) / np.maximum(np.abs(xd), 1)).max()
    edg = np.abs(dg - (cdf + xd * pdf)).max()
    assert eg < 4.5e-6, eg
    assert edg < 4.5e-6, edg


def test_gelu_constants_match_fit():
    pytest.importorskip("scipy")
    spec = importlib.util.spec_from_file_location("fit_gelu", os.path.join(CSRC, "fit_gelu.py"))
    fit = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fit)
    coef, err = fit.fit(7, n=40001, iters=80)
    pn, umax, _, _ = _constants()
    assert abs(float(umax) - fit.UMAX) < 1e-6
    # highest degree first in the header, lowest first from the fit
    np.testing.assert_allclose(np.array(pn, np.float64), coef[::-1].astype(np.float64),
                               rtol=2e-3, atol=1e-6)
    assert err < 4.5e-6
