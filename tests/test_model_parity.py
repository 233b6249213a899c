"""The PyTorch model reproduces the reference FeaturesTransformer exactly (CPU, fp32).

State dicts are exchanged in both directions, so a released checkpoint loads strictly.
"""

import pytest
import torch

from synthefy_nori_b200.models.config import preset_config
from synthefy_nori_b200.utils.loading import build_model


def _pair(reference_pkg, name):
    from synthefy_nori.utils.loading import build_model as ref_build

    cfg = preset_config(name)
    torch.manual_seed(0)
    ref = ref_build(dict(cfg)).eval()
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for _, p in ref.named_parameters():
            if p.abs().sum() == 0:  # zero-initialised gates: make them matter
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    ours = build_model(dict(cfg)).eval()
    ours.load_state_dict(ref.state_dict(), strict=True)
    return ref, ours


@pytest.mark.parametrize("name", ["nori-tiny", "nori-6m"])
def test_forward_matches_reference(reference_pkg, name):
    ref, ours = _pair(reference_pkg, name)
    assert sum(p.numel() for p in ref.parameters()) == sum(p.numel() for p in ours.parameters())
    torch.manual_seed(2)
    B, S, F, ep = 2, 80, 7, 56
    x = torch.randn(B, S, F)
    x[torch.rand(B, S, F) < 0.05] = float("nan")
    y = torch.randn(B, S)
    with torch.no_grad():
        r = ref(x, y[:, :ep], ep, task_type="reg")
        o = ours(x, y[:, :ep], ep, task_type="reg")
    assert o.shape == r.shape == (B, S - ep, 999)
    torch.testing.assert_close(o, r, atol=1e-5, rtol=1e-5)


def test_context_cache_matches_full_forward(reference_pkg):
    ref, ours = _pair(reference_pkg, "nori-tiny")
    torch.manual_seed(3)
    x = torch.randn(1, 70, 5)
    y = torch.randn(1, 50)
    with torch.no_grad():
        full = ours(x, y, 50, task_type="reg")
        for dtype, tol in (("bf16", 1e-5), ("int8", 5e-2)):
            cache = ours.build_context_cache(x[:, :50], y, cache_dtype=dtype)
            out = ours.apply_context_cache(x[:, 50:], cache, row_chunk_size=7)
            torch.testing.assert_close(out, full, atol=tol, rtol=tol)


def test_state_dict_round_trip_into_reference(reference_pkg):
    from synthefy_nori.utils.loading import build_model as ref_build

    cfg = preset_config("nori-tiny")
    ours = build_model(dict(cfg))
    ref = ref_build(dict(cfg))
    ref.load_state_dict(ours.state_dict(), strict=True)


def test_two_phase_v3_matches_reference(reference_pkg):
    """Model v3 (nori-1-5 architecture family): two-phase encoder parity."""
    from synthefy_nori.utils.loading import build_model as ref_build

    from synthefy_nori_b200.models.config import preset_config

    cfg = preset_config("nori-tiny")
    cfg["two_phase_config"] = {"target_tokens": 2, "row_layers": 1, "row_heads": 2, "row_hidden_dim": 96}
    torch.manual_seed(0)
    ref = ref_build(dict(cfg)).eval()
    ours = build_model(dict(cfg)).eval()
    ours.load_state_dict(ref.state_dict(), strict=True)
    torch.manual_seed(5)
    x = torch.randn(2, 60, 5)
    y = torch.randn(2, 40)
    with torch.no_grad():
        r = ref(x, y, 40, task_type="reg")
        o = ours(x, y, 40, task_type="reg")
    torch.testing.assert_close(o, r, atol=1e-5, rtol=1e-5)
