"""Kernel-density-integral preprocessing worker: limits (quantile transform for a small
bandwidth factor, min-max scaling for a large one), monotonicity, NaN handling and the
reference's worker tags."""

import math

import torch

from synthefy_nori_b200.inference.preprocess import KernelDensityIntegral, RebalanceFeatureDistribution


def _data(n=400, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(n, generator=g).exp()  # skewed
    b = torch.rand(n, generator=g) * 10 - 3
    return torch.stack([a, b], 1).double()


def test_kdi_limits_and_monotone():
    x = _data()
    wide = KernelDensityIntegral(alpha=1000.0).fit(x).transform(x)
    minmax = (x - x.min(0).values) / (x.max(0).values - x.min(0).values)
    torch.testing.assert_close(wide, minmax, atol=2e-3, rtol=0)
    narrow = KernelDensityIntegral(alpha=1e-3, n_grid=8192).fit(x).transform(x)
    ranks = (x.argsort(0).argsort(0).double()) / (x.shape[0] - 1)
    assert (narrow - ranks).abs().max() < 0.02  # close to the empirical CDF (quantile transform)
    mid = KernelDensityIntegral(alpha=1.0).fit(x).transform(x)
    assert mid.min() >= 0 and mid.max() <= 1
    for j in range(2):
        order = x[:, j].argsort()
        assert (mid[order, j].diff() >= -1e-12).all()


def test_kdi_nan_normal_output_and_tags():
    x = _data(200, seed=1)
    x[::17, 0] = float("nan")
    t = KernelDensityIntegral(alpha=0.5, output="normal").fit(x)
    out = t.transform(x)
    assert torch.isfinite(out).all()
    assert out.abs().max() <= -torch.special.ndtri(torch.tensor(1e-7, dtype=torch.float64)) + 1e-9
    for tag, width in (("kdi_uni", 2), ("kdi_norm", 2), ("kdi_uni_alpha_0.3", 2), ("kdi_norm_alpha_3.0", 2),
                       ("norm_and_kdi", 4)):
        step = RebalanceFeatureDistribution(worker_tags=[tag])
        step.fit(x.float(), [], seed=0)
        y = step.transform(x.float())
        assert y.shape == (200, width)
        assert math.isfinite(float(y[~torch.isnan(y)].abs().max()))
