"""Model families on CPU: shapes, gradients, parameter counts of the full-size presets (meta device)."""

import pytest
import torch

from verl_omni_b200.models.registry import ARCHS, get_arch


@pytest.mark.parametrize("name", ["tiny_dit", "sd35_tiny", "flux_tiny", "wan_tiny", "qwen_image_tiny",
                                  "qwen_image_edit_tiny", "ltx2_tiny", "bagel_tiny", "minimax_h3_tiny"])
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
        cond = {k: (torch.randint(0, spec.vocab, (B, *s)) if k.endswith("_ids") else torch.randn(B, *s))
                for k, s in spec.cond_shapes.items()}
    out = ad.forward(m, x, t, cond)
    assert out.shape == x.shape and out.dtype == torch.float32
    out.square().mean().backward()
    missing = [n for n, p in m.named_parameters() if p.requires_grad and p.grad is None]
    if spec.adapter == "Bagel":  # the prompt stream's last-layer outputs are discarded
        last = f"layers.{len(m.layers) - 1}.und."
        missing = [n for n in missing if not (n.startswith(last) and (".o." in n or ".gate_up." in n or ".down." in n
                                                                     or n.endswith("ln2") or n.endswith("q_norm")))]
        missing = [n for n in missing if n != "norm_und"]
    if spec.adapter.startswith("QwenImage"):
        # the last block's text stream output is discarded (as in the original model)
        last = f"transformer_blocks.{len(m.transformer_blocks) - 1}."
        missing = [n for n in missing if not (n.startswith(last) and (".txt_out" in n or ".txt_mlp" in n))]
    assert not missing, missing


@pytest.mark.parametrize("name,lo,hi", [("sd35_medium", 2.0e9, 2.6e9), ("flux1_dev", 11.0e9, 12.6e9),
                                        ("wan21_14b", 13.0e9, 15.5e9), ("qwen_image", 19.0e9, 21.5e9),
                                        ("ltx2", 17.0e9, 21.0e9), ("bagel_7b_mot", 13.0e9, 16.5e9),
                                        ("minimax_h3", 5.0e9, 7.0e9)])
def test_full_size_param_counts(name, lo, hi):
    with torch.device("meta"):
        m = get_arch(name).build()
    n = sum(p.numel() for p in m.parameters())
    assert lo < n < hi, n


def _one_step(rank, world, arch):
    import math

    from tests.test_e2e_tiny_on_cpu import OVR
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    ovr = [o for o in OVR if not o.startswith("actor_rollout_ref.model.architecture")]
    cfg = load_config("diffusion_trainer", ovr + [f"actor_rollout_ref.model.architecture={arch}",
                                                  "data.train_batch_size=2", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
                                                  "trainer.total_training_steps=1", "trainer.resume_mode=disable"])
    m = PolicyGradientTrainer(cfg).step()
    assert math.isfinite(m["actor/grad_norm"]) and math.isfinite(m["actor/pg_loss"])


@pytest.mark.parametrize("arch", ["qwen_image_tiny", "qwen_image_edit_tiny", "ltx2_tiny", "bagel_tiny"])
def test_flowgrpo_step_new_families(arch):
    from tests._dist_util import run_ranks

    run_ranks(_one_step, 1, (arch,))


def test_sd3_diffusers_export_import_round_trip(tmp_path):
    """The fused MMDiT exports diffusers SD3Transformer2DModel names (to_qkv split into to_q/k/v, the patch
    linear as a [D, C, p, p] convolution) and a fresh model loaded from that directory computes the same
    output."""
    import json

    from safetensors.torch import load_file

    from verl_omni_b200.models import hf_io
    from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig

    torch.manual_seed(0)
    m = MMDiT(MMDiTConfig.tiny())
    named = dict(m.named_parameters())
    hf_io.save_diffusers(named, m, str(tmp_path))
    sd = load_file(str(tmp_path / "diffusion_pytorch_model.safetensors"))
    assert "transformer_blocks.0.attn.to_q.weight" in sd and "transformer_blocks.0.attn2.to_k.weight" in sd
    assert sd["pos_embed.proj.weight"].shape == (64, 4, 2, 2)
    assert "transformer_blocks.1.ff_context.net.2.weight" not in sd  # context-pre-only last block
    assert json.load(open(tmp_path / "config.json"))["num_layers"] == 2
    torch.manual_seed(1)
    m2 = MMDiT(MMDiTConfig.tiny())
    assert hf_io.load_diffusers(m2, str(tmp_path)) == len(named)
    x = torch.randn(2, 4, 8, 8)
    t = torch.tensor([100.0, 700.0])
    ctx, pooled = torch.randn(2, 12, 48), torch.randn(2, 32)
    torch.testing.assert_close(m2(x, t, ctx, pooled), m.to(torch.bfloat16).float()(x, t, ctx, pooled), rtol=2e-2, atol=2e-2)


def test_reference_family_scorers_through_multi_manager():
    """PickScore / HPSv3 / OCR judge / UnifiedReward / CLAP / ImageBind-shaped scorers (tiny sizes) and the
    MMK12 / choice rules, combined by the multi reward manager."""
    import numpy as np

    from verl_omni_b200.models.scorers import choice_reward, mmk12_reward
    from verl_omni_b200.utils.dataproto import DataProto
    from verl_omni_b200.workers.reward.reward_manager import (MultiVisualRewardManager, VisualRewardManager,
                                                              build_model_scorer)

    torch.manual_seed(0)
    dev = torch.device("cpu")
    vit = dict(image_size=32, patch=8, vision_dim=32, vision_depth=1, vision_heads=2)
    vlm = dict(vit, lm_dim=32, lm_depth=1, lm_heads=2, vocab=300, text_len=8)
    subs = [("pickscore", build_model_scorer("pickscore", dev, torch.float32, **vit, text_dim=32, text_depth=1,
                                             text_heads=2, embed_dim=16, vocab=300, text_len=8)),
            ("hpsv3", build_model_scorer("hpsv3", dev, torch.float32, **vlm)),
            ("ocr", build_model_scorer("ocr", dev, torch.float32, new_tokens=3, **vlm)),
            ("unified_reward", build_model_scorer("unified_reward", dev, torch.float32, new_tokens=3, **vlm)),
            ("clap", build_model_scorer("clap", dev, torch.float32, n_mels=8, audio_dim=32, audio_depth=1,
                                        audio_heads=2, text_dim=32, text_depth=1, text_heads=2, embed_dim=16,
                                        vocab=300, text_len=8)),
            ("imagebind", build_model_scorer("imagebind", dev, torch.float32, image_size=32, patch=8, dim=32,
                                             depth=2, heads=2, n_mels=8, embed_dim=16, vocab=300, text_len=8))]
    batch = DataProto({"images": torch.rand(3, 3, 64, 64) * 2 - 1, "audio_mels": torch.randn(3, 10, 8)},
                      {"raw_prompt": np.array(["a red cat", "SALE", "two dogs"], dtype=object),
                       "ground_truth": np.array([None, "SALE", None], dtype=object)})
    mgr = MultiVisualRewardManager([(n, VisualRewardManager(s, name=n), 1.0, True) for n, s in subs])
    total, metrics = mgr(batch)
    assert total.shape == (3,) and torch.isfinite(total).all()
    assert all(f"reward/{n}_mean" in metrics for n, _ in subs)
    assert mmk12_reward(["so x = \\boxed{42}", "41"], ["42", "42"]).tolist() == [1.0, 0.0]
    assert choice_reward(["I pick (B)", "answer: C"], ["B", "D"]).tolist() == [1.0, 0.0]


def test_trainer_multi_reward_config():
    """reward.sub_rewards builds the weighted multi-reward manager inside the trainer (default scorer + a
    tiny PickScore-shaped model)."""
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=2",
        "actor_rollout_ref.actor.ppo_mini_batch_size=2", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=1"])
    cfg.reward.sub_rewards = [{"name": "latent", "scorer": "default", "weight": 0.5},
                              {"name": "hps", "scorer": "hpsv3", "weight": 1.0, "required": False,
                               "sizes": {"image_size": 32, "patch": 8, "vision_dim": 32, "vision_depth": 1,
                                         "vision_heads": 2, "lm_dim": 32, "lm_depth": 1, "lm_heads": 2,
                                         "vocab": 300, "text_len": 8}}]
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    m = t.step()
    assert "reward/latent_mean" in m and ("reward/hps_mean" in m or "reward/hps_failed" in m)
