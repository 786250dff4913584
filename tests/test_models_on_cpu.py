"""Model families on CPU: shapes, gradients, parameter counts of the full-size presets (meta device)."""

import pytest
import torch

from verl_omni_b200.models.registry import ARCHS, get_arch


@pytest.mark.parametrize("name", ["tiny_dit", "sd35_tiny", "flux_tiny", "wan_tiny"])
def test_tiny_forward_backward(name):
    from verl_omni_b200.pipelines.model_base import DiffusionModelBase

    spec = get_arch(name)
    torch.manual_seed(0)
    m = spec.build()
    ad = DiffusionModelBase.get(spec.adapter, "flow_grpo")
    B = 2
    x = torch.randn(B, *spec.latent_shape)
    t = torch.tensor([700.0, 100.0])
    if spec.text_encoder is not None:
        cond = {"prompt_embeds": torch.randn(B, 16, 256)}
    else:
        cond = {k: torch.randn(B, *s) for k, s in spec.cond_shapes.items()}
    out = ad.forward(m, x, t, cond)
    assert out.shape == x.shape and out.dtype == torch.float32
    out.square().mean().backward()
    assert all(p.grad is not None for p in m.parameters() if p.requires_grad)


@pytest.mark.parametrize("name,lo,hi", [("sd35_medium", 2.0e9, 2.6e9), ("flux1_dev", 11.0e9, 12.6e9),
                                        ("wan21_14b", 13.0e9, 15.5e9)])
def test_full_size_param_counts(name, lo, hi):
    with torch.device("meta"):
        m = get_arch(name).build()
    n = sum(p.numel() for p in m.parameters())
    assert lo < n < hi, n
