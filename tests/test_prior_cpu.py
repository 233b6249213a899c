"""Host-side pieces of the SCM prior: meta-distributions, block-wise dropout weights,
roots, the tree SCM tensor program, stabilisation, and the plain-tensor statement of the
benchmark prior (CPU)."""

import numpy as np
import torch

from synthefy_nori_b200.training import scm_prior as sp


def test_hyperparameter_ranges():
    rng = np.random.default_rng(0)
    hps = [sp.sample_hyperparams(rng) for _ in range(2000)]
    assert 0.62 < np.mean([h.scm_type == "mlp" for h in hps]) < 0.78
    assert min(h.num_layers for h in hps) >= 2 and min(h.hidden_dim for h in hps) >= 4
    assert min(h.num_causes for h in hps) >= 1
    assert all(h.init_std > 0 and h.noise_std > 0 for h in hps)  # truncated draws: no atom at zero
    assert all(0 <= h.dropout_prob <= 0.9 for h in hps)
    assert {h.sampling for h in hps} == {"normal", "mixed", "uniform"}
    assert all(0 <= h.act_factory < sp.N_FACTORIES for h in hps)


def test_block_dropout_weight_structure():
    rng = np.random.default_rng(1)
    g = torch.Generator().manual_seed(1)
    for out_dim, in_dim, p in [(40, 30, 0.8), (7, 50, 0.5), (64, 64, 0.0)]:
        w = sp.block_dropout_weight(rng, out_dim, in_dim, 1.0, p, g, "cpu")
        nz = w != 0
        assert bool(nz.any(1).all()) and bool(nz.any(0).all())  # no disconnected neuron


def test_tree_scm_and_stabilize():
    rng = np.random.default_rng(2)
    hps = [sp.sample_hyperparams(rng, mlp_prob=0.0) for _ in range(3)]
    X, y = sp.tree_scm_batch(hps, [4, 6, 3], 200, 150, seed=3, device="cpu", rng=rng)
    assert X.shape == (3, 200, 6) and torch.isfinite(X).all() and torch.isfinite(y).all()
    Xs, ys = sp.stabilize(X, y, [4, 6, 3], 150)
    assert float(Xs.abs().max()) <= 50.0
    assert bool((Xs[0, :, 4:] == 0).all())
    torch.testing.assert_close(ys[:, :150].mean(1), torch.zeros(3), atol=1e-5, rtol=0)


def test_roots_mixed_sampling():
    rng = np.random.default_rng(4)
    g = torch.Generator().manual_seed(4)
    hp = sp.sample_hyperparams(rng)
    hp.sampling = "mixed"
    r = sp.sample_roots(rng, hp, 12, 500, 400, g, "cpu")
    assert r.shape == (500, 12) and torch.isfinite(r).all()
    p = sp._zipf_table(2.5)
    assert abs(p.sum() - 1) < 1e-9 and p[0] > p[1] > p[2]


def test_benchmark_prior_on_cpu():
    from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch

    b = scm_prior_batch(PriorConfig(max_features=10, pad_features=10), 3, 120, 80, seed=0, device=torch.device("cpu"))
    assert b.x.shape == (3, 120, 10) and torch.isfinite(b.x).all()
    torch.testing.assert_close(b.y[:, :80].mean(1), torch.zeros(3), atol=1e-5, rtol=0)


def test_scm_tables_and_mixture_on_cpu():
    from synthefy_nori_b200.training.generators import FAMILIES, generate_batch

    X, y, meta = sp.scm_prior_tables(6, 160, [3, 8, 5, 12, 2, 7], 120, seed=1, device="cpu", pad_features=12)
    assert X.shape == (6, 160, 12) and torch.isfinite(X).all() and torch.isfinite(y).all()
    for fam in FAMILIES:
        Xb, yb, nf, fams = generate_batch(3, 150, 100, seed=2, device="cpu", min_features=4, max_features=20,
                                          pad_features=20, family_probs={fam: 1.0})
        assert fams == [fam] * 3
        assert Xb.shape == (3, 150, 20) and torch.isfinite(yb).all()
        assert not torch.isinf(Xb).any()
        std = yb[:, :100].std(1, unbiased=False)
        assert bool((std > 0.99).all() & (std < 1.01).all()), (fam, std)
        for b in range(3):  # padded columns stay zero
            assert bool((Xb[b, :, int(nf[b]):] == 0).all())
