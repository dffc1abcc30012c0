"""CPU checks of the ECDL oracle (oracle/ecdl.py): the random stream against
the Random123 known-answer vectors, the sampler's limits and distribution,
and the proxy-gradient coefficients against finite differences."""

import numpy as np
import pytest

from oracle import ecdl as E


@pytest.mark.parametrize("ctr,key,want", [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
])
def test_philox_known_answers(ctr, key, want):
    got = E.philox4x32(*[np.array([c]) for c in ctr], *key)
    assert [int(g[0]) for g in got] == list(want)


def test_uniform_range_and_mean():
    u = E.uniform(7, np.arange(200000, dtype=np.uint64))
    assert u.min() >= 0.0 and u.max() < 1.0
    assert abs(float(u.mean()) - 0.5) < 5e-3


@pytest.mark.parametrize("fmt", [E.NVFP4, E.MXFP8])
def test_tables(fmt):
    f = E.Format(fmt)
    assert np.all(np.diff(f.level) >= 0) and np.all(f.gap > 0)
    if fmt == E.NVFP4:
        assert f.tn == 16 and f.qn == 126 and f.f_max == 2688.0 and f.emax == 2
    else:
        assert f.tn == 254 and f.level[0] == -448.0 and f.level[-1] == 448.0 and f.emax == 8


@pytest.mark.parametrize("fmt,topk", [(E.NVFP4, 4), (E.NVFP4, 16), (E.MXFP8, 8)])
def test_large_kappa_samples_the_nearest_level(fmt, topk):
    f = E.Format(fmt)
    rng = np.random.RandomState(0)
    v = (rng.randn(5000) * (2.0 if fmt == E.NVFP4 else 60.0)).astype(np.float32)
    u = rng.rand(5000).astype(np.float32)
    idx = E.sample(f, v, 1e6, u, topk)
    c, start, _ = E._window(f, v, topk)
    near = np.clip(np.floor(c + np.float32(0.5)), start, start + topk - 1).astype(np.int64)
    assert np.array_equal(idx, near)


def test_sampler_follows_its_probabilities():
    f = E.Format(E.NVFP4)
    v = np.full(200000, 1.3, dtype=np.float32)
    u = E.uniform(3, np.arange(v.size, dtype=np.uint64))
    idx = E.sample(f, v, 2.0, u, 8)
    start, p = E.probabilities(f, v[:1], 2.0, 8)
    freq = np.bincount(idx - start[0], minlength=8) / v.size
    assert np.max(np.abs(freq - p[0])) < 5 * np.sqrt(0.25 / v.size) + 1e-4


@pytest.mark.parametrize("kappa", [0.5, 3.0])
def test_proxy_coefficient_is_the_derivative_of_the_expected_level(kappa):
    """dth = d E[level] / dv (per unit of v, the chain rule through x = v s
    lives in the caller)."""
    f = E.Format(E.NVFP4)
    v = np.array([-2.7, -0.9, 0.1, 0.62, 1.1, 2.2, 3.3, 4.8], dtype=np.float64)
    dth, _, _ = E.proxy_coeffs(f, v.astype(np.float32), kappa, 16)

    def expect(x):
        start, p = E.probabilities(f, x.astype(np.float32), kappa, 16)
        lev = np.stack([f.level[start + j] for j in range(16)], -1)
        return (p * lev).sum(-1)

    h = 1e-3
    num = (expect(v + h) - expect(v - h)) / (2 * h)
    assert np.allclose(dth, num, rtol=2e-2, atol=2e-3), (dth, num)


def test_ecdl_workspace_bytes_on_host():
    from cdl_b200 import _lib

    lib = _lib.lib()
    assert lib.cdlb200_ecdl_bwd_workspace_bytes(0, 4, 0) == 0
    assert lib.cdlb200_ecdl_bwd_workspace_bytes(64, 4, 0) > 0
    assert lib.cdlb200_ecdl_bwd_workspace_bytes(64, 4, 7) == 0  # unknown format


def test_ccdl_truncated_sampler_limits():
    """The scale-side (truncated) sampler picks the nearest scale level for a
    sharp window, on both scale grids."""
    for fmt in (E.NVFP4, E.MXFP4):
        fq = E.QFormat(fmt)
        rng = np.random.RandomState(fmt)
        v = np.exp(rng.uniform(-6, 5, 4000)).astype(np.float32)
        u = rng.rand(4000).astype(np.float32)
        idx = E.sample_truncated(fq, v, 1e6, u, 5)
        c, start, _ = E._window(fq, v, 5)
        near = np.clip(np.floor(c + np.float32(0.5)), start, start + 4).astype(np.int64)
        assert np.array_equal(idx, near)


def test_ccdl_oracle_shapes_and_shared_q():
    th = np.random.RandomState(0).randn(4, 8, 16).astype(np.float32)
    q = np.full((1, 8), 64.0, dtype=np.float32)
    p, s = E.ccdl_forward(E.NVFP4, th, q, 3.0, 2.0, 0.01, 5, 5, 5)
    assert p.shape == (4, 64) and s.shape == (1, 8)
    dth, dq, sc = E.ccdl_backward(E.NVFP4, np.ones_like(th), th, q, s, 3.0, 2.0, 0.01, 5, 5)
    assert dth.shape == th.shape and dq.shape == (4, 8) and len(sc) == 3 and np.all(np.isfinite(sc))


def _ccdl_round_cases():
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ccdl_round.npz"))
    return [{k.split("_", 1)[1]: z[k] for k in z.files if k.startswith(f"c{i}_")} for i in range(int(z["count"]))]


def test_ccdl_round_oracle_matches_reference_golden():
    """The eval-mode round restated in the oracle reproduces the reference's
    cascaded_nearest_round on every committed case (all formats, bf16 / fp32
    theta and levels, per-row and shared scales)."""
    cases = _ccdl_round_cases()
    assert len(cases) == 24
    for c in cases:
        fmt = int(c["fmt"])
        tpb = 16 if fmt == E.NVFP4 else 32
        theta = c["theta"]
        packed, scale = E.ccdl_round(fmt, theta.reshape(theta.shape[0], -1, tpb), c["q"], float(c["alpha"]),
                                     bool(c["theta_bf16"]), bool(c["levels_bf16"]))
        np.testing.assert_array_equal(packed, c["packed"])
        np.testing.assert_array_equal(scale, c["scale"])


def _cdl_window_cases():
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "cdl_window.npz"))
    return [{k.split("_", 1)[1]: z[k] for k in z.files if k.startswith(f"c{i}_")} for i in range(int(z["count"]))]


def test_window_probabilities_and_proxy_match_reference_formulae():
    """The oracle's CDL window, sampling distribution, expected level and
    proxy derivatives against the reference's own torch formulae
    (topk_cpmf_companded / topk_q_d and their autograd gradients, fp32;
    tests/golden/cdl_window.npz): window starts equal, probabilities within
    3e-7, the expected level within 2e-6 relative, the derivatives within
    fp32 rounding of the sums they are formed from (terms of size
    max|level| * kappa * dmax / gap for d/dx, max|level| * dmax^2 for
    d/dkappa, dmax the farthest window level)."""
    cases = [c for c in _cdl_window_cases() if str(c["fmt"]) in ("e2m1", "e4m3")]
    assert len(cases) == 18
    for i, c in enumerate(cases):
        f = E.Format(E.NVFP4 if str(c["fmt"]) == "e2m1" else E.MXFP8)
        v, kappa, topk = c["v"], float(c["kappa"]), int(c["topk"])
        start, p = E.probabilities(f, v, kappa, topk)
        assert np.array_equal(start, c["start"])
        assert float(np.abs(p - c["pmf"]).max()) < 3e-7
        lv = np.stack([f.level[start + j] for j in range(topk)], -1)
        ev = (p * lv).sum(-1)
        assert float(np.max(np.abs(ev - c["ev"]) / np.maximum(np.abs(c["ev"]), 1e-3))) < 2e-6
        dth, _, dk = E.proxy_coeffs(f, v, kappa, topk)
        cpos, _, kgap = E._window(f, v, topk)
        dmax = np.max(np.abs(cpos[:, None] - (start[:, None] + np.arange(topk))), -1) + 1.0
        top = float(np.abs(f.level).max())
        assert np.all(np.abs(dth - c["dv"]) <= 1e-5 * top * kappa * dmax / kgap + 1e-7), i
        assert np.all(np.abs(dk - c["dk"]) <= 1e-5 * top * dmax ** 2 + 1e-7), i


def test_truncated_scale_window_matches_reference_formulae():
    """The CCDL scale sampler's truncated window (UE4M3 without zero, E8M0)
    against the reference's full-window torch formulae: window starts equal;
    where the truncated window covers the whole top-k window, the expected
    level and its derivatives agree to fp32 rounding of their terms (scaled by
    the window's largest level); where it leaves out far levels, by at most
    their weight, exp(-kappa (hq - 1/2)^2) each (the truncation the reference's
    Triton primitive makes)."""
    cases = [c for c in _cdl_window_cases() if str(c["fmt"]) in ("ue4m3", "e8m0")]
    assert len(cases) == 12
    for i, c in enumerate(cases):
        f = E.QFormat(E.NVFP4 if str(c["fmt"]) == "ue4m3" else E.MXFP4)
        v, kappa, topk = c["v"], float(c["kappa"]), int(c["topk"])
        cpos, start, kgap = E._window(f, v, topk)
        assert np.array_equal(start, c["start"]), i
        dth, ds, dk = E.proxy_coeffs_truncated(f, v, kappa, topk)
        ev = ds + v * dth
        lmax = np.abs(np.stack([f.level[start + j] for j in range(topk)], -1)).max(-1)
        dmax = np.max(np.abs(cpos[:, None] - (start[:, None] + np.arange(topk))), -1) + 1.0
        hq = E._half_window(topk, kappa)
        t_near, _ = E._near(cpos, start, topk, np.float32(kappa))
        cut = np.maximum(start, t_near - hq) > start  # levels left out of the truncated window
        tail = np.where(cut, topk * np.exp(-kappa * (hq - 0.5) ** 2), 0.0)
        assert np.all(np.abs(ev - c["ev"]) <= lmax * (2e-6 + tail)), i
        assert np.all(np.abs(dth - c["dv"]) <= lmax * kappa * dmax / kgap * (1e-5 + tail * dmax)), i
        assert np.all(np.abs(dk - c["dk"]) <= lmax * dmax ** 2 * (1e-5 + tail)), i
