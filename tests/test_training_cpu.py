"""CPU tests for the training extras: Muon (vs torch.optim.Muon), regression losses
(vs the reference's loss functions where installed), masks."""

import copy

import pytest
import torch

from synthefy_nori_b200.training.loss import (bar_distribution_loss, feature_reconstruction_loss,
                                              normal_quantile_borders, regression_objective)
from synthefy_nori_b200.training.masking import apply_query_masks, batch_masks, create_masks
from synthefy_nori_b200.training.muon import HybridMuonAdamW, newton_schulz, split_muon_adamw_params


def test_newton_schulz_orthogonalises():
    G = torch.randn(4, 96, 48)
    s = torch.linalg.svdvals(newton_schulz(G).float())
    assert s.min() > 0.5 and s.max() < 1.3  # quintic iteration lands in ~[0.7, 1.2]


@pytest.mark.skipif(not hasattr(torch.optim, "Muon"), reason="torch.optim.Muon not available")
def test_hybrid_muon_matches_torch_muon_plus_adamw():
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.GELU(), torch.nn.Linear(32, 8))
    ref = copy.deepcopy(net)
    ours = HybridMuonAdamW(net, "cpu", lr=0.01, weight_decay=0.1, ema_decay=None, max_grad_norm=0.0)
    mu = [p for p in ref.parameters() if p.ndim == 2]
    ad = [p for p in ref.parameters() if p.ndim != 2]
    o1 = torch.optim.Muon(mu, lr=0.01, weight_decay=0.1, momentum=0.95, nesterov=True, adjust_lr_fn="match_rms_adamw")
    o2 = torch.optim.AdamW(ad, lr=0.01, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8)
    for _ in range(3):
        x = torch.randn(64, 16)
        ours.zero_grad()
        net(x).pow(2).mean().backward()
        ours.step()
        o1.zero_grad()
        o2.zero_grad()
        ref(x).pow(2).mean().backward()
        o1.step()
        o2.step()
    for a, b in zip(net.parameters(), ref.parameters()):
        torch.testing.assert_close(a, b, atol=2e-3, rtol=0)


def test_muon_split_policy_and_clip():
    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.feature_positional_embedding = torch.nn.Linear(4, 8)
            self.proj = torch.nn.Linear(8, 8)
            self.qkv = torch.nn.Parameter(torch.randn(3, 2, 4, 8))

    m = M()
    mu, ad = split_muon_adamw_params(m.named_parameters())
    assert [n for n, _ in mu] == ["proj.weight"]
    mu, _ = split_muon_adamw_params(m.named_parameters(), include_nd=True, include_embeddings=True)
    assert {n for n, _ in mu} == {"feature_positional_embedding.weight", "proj.weight", "qkv"}
    opt = HybridMuonAdamW(m, "cpu", lr=1e-3, include_nd=True, max_grad_norm=1.0)
    (m.proj.weight.sum() * 1e6 + m.qkv.sum()).backward()
    before = m.proj.bias.detach().clone()
    opt.step()
    assert torch.isfinite(opt.flat.data).all() and not torch.equal(before, m.proj.bias.detach())
    sd = opt.state_dict()
    opt2 = HybridMuonAdamW(copy.deepcopy(m), "cpu", lr=1e-3, include_nd=True)
    opt2.load_state_dict(sd)
    assert opt2.step_count == 1


def test_point_losses_and_bar(reference_pkg):
    import importlib

    rl = importlib.import_module("synthefy_nori.training.loss")
    torch.manual_seed(0)
    b = normal_quantile_borders(64)
    logits, t = torch.randn(3, 7, 64), torch.randn(3, 7) * 2
    torch.testing.assert_close(bar_distribution_loss(logits, t, b), rl._bar_distribution_loss(logits, t, b))
    torch.testing.assert_close(bar_distribution_loss(logits, t, b, 0.12),
                               rl._bar_distribution_soft_loss(logits, t, b, 0.12))


def test_regression_objectives_definitions():
    torch.manual_seed(1)
    p, t = torch.randn(2, 5, 1), torch.randn(2, 5)
    var = t.var(1, unbiased=False).clamp(min=0.01)
    want = (((p[..., 0] - t) ** 2).mean(1) / var).mean()
    torch.testing.assert_close(regression_objective("mse", p, t), want)
    with pytest.raises(ValueError):
        regression_objective("nope", p, t)
    fp, x = torch.randn(2, 5, 3), torch.randn(2, 5, 3)
    m = torch.zeros(2, 5, 3, dtype=torch.bool)
    m[0, 1, 2] = True
    torch.testing.assert_close(feature_reconstruction_loss(fp, x, m), (fp[0, 1, 2] - x[0, 1, 2]) ** 2)


def test_masks():
    g = torch.Generator().manual_seed(0)
    c = create_masks(40, 10, 0.3, "column", g)
    assert c.all(0).sum() == 3 and (c.any(0) == c.all(0)).all()
    b = create_masks(40, 10, 0.25, "block", g)
    assert 0 < b.float().mean() <= 0.6
    bm = batch_masks(3, 20, 6, seed=2)
    x = torch.randn(3, 30, 6)
    xm = apply_query_masks(x, 10, bm)
    assert torch.isnan(xm[:, 10:]).sum() == bm.sum() and not torch.isnan(xm[:, :10]).any()
    with pytest.raises(ValueError):
        create_masks(4, 4, 0.2, "diag")


def test_shape_sampler_budget_buckets_and_palette():
    from synthefy_nori_b200.training.shapes import FEATURE_BUCKETS, SAMPLE_BUCKETS, ShapeConfig, ShapeSampler

    cfg = ShapeConfig(min_samples=256, max_samples=8192, min_features=4, max_features=512, features_per_group=2,
                      max_budget=500_000, dim_bias_samples=2.2, dim_bias_features=1.5, bucketed=True)
    s = ShapeSampler(cfg, 0)
    seen = [s.sample() for _ in range(400)]
    for n, f, r in seen:
        assert n in SAMPLE_BUCKETS and f in FEATURE_BUCKETS and n * f <= 500_000 and f % 2 == 0
        assert r in (0.3, 0.4, 0.5, 0.6, 0.7, 0.8)
    # the same seed gives the same stream (shared across ranks); biasing pushes draws up
    s2 = ShapeSampler(cfg, 0)
    assert [s2.sample() for _ in range(400)] == seen
    plain = ShapeSampler(ShapeConfig(min_samples=256, max_samples=8192, bucketed=False), 1)
    biased = ShapeSampler(ShapeConfig(min_samples=256, max_samples=8192, bucketed=False, dim_bias_samples=3.0), 1)
    assert sum(biased.sample()[0] for _ in range(300)) > sum(plain.sample()[0] for _ in range(300))
    pal = ShapeSampler(ShapeConfig(shape_palette=[(512, 10, 1.0), (1024, 20, 3.0)], context_ratio_palette=[0.7]), 2)
    draws = [pal.sample() for _ in range(200)]
    assert {(n, f) for n, f, _ in draws} == {(512, 10), (1024, 20)} and {r for *_, r in draws} == {0.7}


def test_icl_health_mask():
    from synthefy_nori_b200.training.icl_filter import health_mask

    X = torch.randn(4, 50, 3)
    y = torch.randn(4, 50)
    y[1, 10] = float("nan")  # non-finite target
    y[2, :30] = 1.0  # constant context target
    X[3, :30] = 0.0  # no varying context feature
    assert health_mask(X, y, 30).tolist() == [True, False, False, False]


def test_curriculum_tier_args():
    from synthefy_nori_b200.training.cli import parse_args
    from synthefy_nori_b200.training.curriculum import TIERS, tier_args

    for t in TIERS:
        a = parse_args(tier_args(t) + ["--checkpoint-dir", "/tmp/x"])
        assert a.max_budget == TIERS[t]["budget"] and a.gradient_accumulation == TIERS[t]["accum"]
        assert a.prior == "mixture" and a.optimizer == "muon"


def test_tree_learnability_and_scaling_filters(monkeypatch):
    """Learnable tables pass the tree-ensemble gate, pure-noise tables are rejected and
    regenerated until every slot passes; the context-scaling gate keeps a table only when the
    score at the full context beats the smallest prefix by the required margin."""
    import torch

    from synthefy_nori_b200.training.icl_filter import TreeLearnabilityFilter

    g = torch.Generator().manual_seed(0)

    def tables(B, learnable):
        X = torch.randn(B, 400, 6, generator=g)
        X[:, :, 5] = 0.0  # a padded column
        y = (X[:, :, 0] * 2 + torch.sin(3 * X[:, :, 1])) if learnable else torch.randn(B, 400, generator=g)
        return X, y + 0.05 * torch.randn(B, 400, generator=g)

    f = TreeLearnabilityFilter(min_score=0.10)
    Xg, yg = tables(2, True)
    Xn, yn = tables(2, False)
    assert f.score(Xg, yg, 300).tolist() == [1.0, 1.0]
    assert f.score(Xn, yn, 300).tolist() == [0.0, 0.0]
    X = torch.cat((Xg[:1], Xn[:1]))
    y = torch.cat((yg[:1], yn[:1]))
    calls = []

    def regenerate(slots, rnd):
        calls.append((slots, rnd))
        return tables(len(slots), True)

    X2, y2 = f.filter(X, y, 300, regenerate)
    assert calls == [([1], 1)] and bool((f.score(X2, y2, 300) == 1).all())
    assert f.stats["first_round_rejects"] == 1
    # constant context targets are unhealthy: rejected without fitting
    yc = yg.clone()
    yc[:, :300] = 1.0
    assert f.score(Xg, yc, 300).tolist() == [0.0, 0.0]
    # the scaling rule, with the ensemble's scores fixed per context size
    seen = []

    def fake(rising):
        def fit_score(Xf, yf, Xt, yt, trees, depth):
            seen.append((len(Xf), trees, depth))
            return 0.2 + (0.001 * len(Xf) if rising else 0.0)
        return staticmethod(fit_score)

    sc = TreeLearnabilityFilter(min_score=0.10, scaling=True, learnability=False)
    monkeypatch.setattr(TreeLearnabilityFilter, "_fit_score", fake(True))
    assert sc.score(Xg[:1], yg[:1], 300).tolist() == [1.0]
    assert [k for k, _, _ in seen] == [75, 119, 188, 300] and seen[0][1:] == (10, 5)
    monkeypatch.setattr(TreeLearnabilityFilter, "_fit_score", fake(False))
    assert sc.score(Xg[:1], yg[:1], 300).tolist() == [0.0]


def test_memory_plan_arithmetic(monkeypatch):
    """The training step's memory plan (host arithmetic, with the device queries faked): the
    attention stash needs all layers' outputs within a quarter of the available memory, and
    the trailing layers that skip checkpointing fit next to the checkpointed ones."""
    import torch

    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.ops import fused_layer
    from synthefy_nori_b200.ops.fused_layer import Geometry, _layer_bytes, memory_plan
    from synthefy_nori_b200.utils.loading import build_model

    model = build_model(preset_config("nori-100m"))
    GiB = 2 ** 30

    class Props:
        total_memory = 180 * GiB

    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: Props())
    dev = torch.device("cuda", 0)

    def plan(avail_gib, rows):
        monkeypatch.setattr(fused_layer, "_available_bytes", lambda d: int(avail_gib * GiB))
        g = Geometry(B=16, ep=rows * 2 // 3, nq=rows - rows * 2 // 3, T=51, E=448, H=8)
        return memory_plan(model, g, dev), _layer_bytes(model, g)

    (stash, plain), (x_b, stash_b, full_b) = plan(170, 1200)
    assert stash and 0 < plain < 26 and x_b < stash_b < full_b
    (stash_big, plain_big), _ = plan(170, 2048)
    assert plain_big < plain  # bigger tables keep fewer layers un-checkpointed
    (stash_low, plain_low), _ = plan(20, 1200)
    assert not stash_low and plain_low == 0  # little memory: full checkpointing, no stash
    monkeypatch.setenv("NORI_PLAIN_LAYERS", "3")
    assert plan(170, 1200)[0][1] == 3
    assert memory_plan(model, Geometry(B=1, ep=8, nq=4, T=3, E=448, H=8), torch.device("cpu")) == (False, 0)
