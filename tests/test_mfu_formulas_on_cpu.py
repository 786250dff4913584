"""The per-family forward FLOPs formulas behind ``perf/mfu/*`` agree with the FLOPs torch counts when the
family's tiny model actually runs (matmuls, attention), within 7 %."""

import pytest
import torch
from torch.utils.flop_counter import FlopCounterMode

from verl_omni_b200.models.registry import get_arch
from verl_omni_b200.pipelines.model_base import DiffusionModelBase
from verl_omni_b200.utils.mfu import DiffusionFlopsCounter, token_counts


@pytest.mark.parametrize("name", ["sd35_tiny", "flux_tiny", "wan_tiny", "qwen_image_tiny", "qwen_image_edit_tiny",
                                  "ltx2_tiny", "minimax_h3_tiny", "bagel_tiny"])
def test_forward_flops_formula_matches_counted(name):
    spec = get_arch(name)
    torch.manual_seed(0)
    m = spec.build().eval()
    ad = DiffusionModelBase.get(spec.adapter, "flow_grpo")
    x = torch.randn(1, *spec.latent_shape)
    cond = {k: (torch.randint(0, spec.vocab, (1, *s)) if k.endswith("_ids") else torch.randn(1, *s))
            for k, s in spec.cond_shapes.items()}
    with torch.no_grad(), FlopCounterMode(display=False) as fc:
        ad.forward(m, x, torch.tensor([700.0]), cond)
    image, text = token_counts(spec)
    ratio = DiffusionFlopsCounter(m, m.family).forward_flops(image, text) / fc.get_total_flops()
    assert 0.93 <= ratio <= 1.07, ratio


def test_moe_llm_flops_formula_matches_counted():
    from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM
    from verl_omni_b200.utils.mfu import moe_llm_forward_flops, omni_step_mfu_metrics

    cfg = MoEConfig.tiny()
    torch.manual_seed(0)
    m = MoELLM(cfg).eval()
    with torch.no_grad(), FlopCounterMode(display=False) as fc:
        m(torch.randint(0, 500, (2, 40)))
    assert 0.93 <= moe_llm_forward_flops(cfg, 2, 40) / fc.get_total_flops() <= 1.07
    mfu = omni_step_mfu_metrics(cfg, batch=8, seq=40, timing={"gen": 1.0, "update_actor": 2.0}, n_gpus=2)
    assert set(mfu) == {"perf/mfu/rollout", "perf/mfu/actor"} and mfu["perf/mfu/actor"] == pytest.approx(
        1.5 * mfu["perf/mfu/rollout"])
