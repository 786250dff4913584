"""Qwen-Image-shaped MMDiT (and the Edit variant) on CPU: shapes, masking, adapter registry, rope layout."""

import torch

from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT
from verl_omni_b200.pipelines.model_base import DiffusionModelBase


def _inputs(B=2, St=12, C=4, H=8, W=8):
    g = torch.Generator().manual_seed(0)
    lat = torch.randn(B, C, H, W, generator=g)
    emb = torch.randn(B, St, 48, generator=g)
    t = torch.tensor([900.0, 300.0])[:B]
    return lat, t, emb


def test_forward_shapes_and_backward():
    torch.manual_seed(0)
    m = QwenImageDiT(QwenImageConfig.tiny())
    lat, t, emb = _inputs()
    out = m(lat, t, emb)
    assert out.shape == lat.shape and torch.isfinite(out).all()
    out.square().mean().backward()
    assert m.transformer_blocks[0].img_qkv.weight.grad is not None
    assert m.txt_norm_weight.grad is not None


def test_padded_prompt_tokens_do_not_change_the_output():
    """Masked (right-padded) prompt positions are excluded from attention: changing their embeddings
    leaves the prediction unchanged, changing a valid position does not."""
    torch.manual_seed(0)
    m = QwenImageDiT(QwenImageConfig.tiny()).eval()
    lat, t, emb = _inputs()
    mask = torch.ones(2, 12)
    mask[0, 7:] = 0
    mask[1, 10:] = 0
    with torch.no_grad():
        a = m(lat, t, emb, mask)
        emb2 = emb.clone()
        emb2[0, 9] += 5.0
        emb2[1, 11] -= 3.0
        b = m(lat, t, emb2, mask)
        emb3 = emb.clone()
        emb3[0, 2] += 5.0
        c = m(lat, t, emb3, mask)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    assert (a - c).abs().max() > 1e-4


def test_edit_variant_appends_reference_tokens():
    torch.manual_seed(0)
    m = QwenImageDiT(QwenImageConfig.tiny()).eval()
    lat, t, emb = _inputs()
    ref = torch.randn_like(lat)
    with torch.no_grad():
        a = m(lat, t, emb, image_latents=ref)
        b = m(lat, t, emb, image_latents=ref + 1.0)
    assert a.shape == lat.shape
    assert (a - b).abs().max() > 1e-4  # the reference image conditions the prediction
    c, s = m._rope(4, 4, 1, 12, "cpu")
    assert c.shape[0] == 2 * 16 + 12  # generated tokens, reference tokens, text


def test_adapters_registered():
    a = DiffusionModelBase.get("QwenImage", "flow_grpo")
    assert a.true_cfg_renorm and a.scheduler_kind == "qwen_image"
    assert DiffusionModelBase.get("QwenImage", "dpo") is a
    e = DiffusionModelBase.get("QwenImageEdit", "flow_grpo")
    assert "image_latents" in e.cond_keys()
    # the reference's pipeline-class keys select the same adapters
    assert DiffusionModelBase.get("QwenImagePipeline", "flow_grpo") is a
    assert DiffusionModelBase.get("QwenImageEditPlusPipeline", "flow_grpo") is e
    for cls_name, algo in (("StableDiffusion3Pipeline", "flow_grpo"), ("StableDiffusion3Pipeline", "dpo"),
                           ("WanPipeline", "dance_grpo"), ("LTX2Pipeline", "flow_grpo"),
                           ("MiniMaxH3Pipeline", "diffusion_nft"), ("OmniBagelForConditionalGeneration", "flow_grpo"),
                           ("QwenImagePipeline", "mix_grpo"), ("QwenImagePipeline", "diffusion_nft")):
        assert DiffusionModelBase.get(cls_name, algo) is not None
    m = QwenImageDiT(QwenImageConfig.tiny()).eval()
    lat, t, emb = _inputs()
    cond = {"prompt_embeds": emb, "prompt_embeds_mask": torch.ones(2, 12)}
    with torch.no_grad():
        v = a.predict(m, lat, t, cond, {"prompt_embeds": torch.zeros_like(emb),
                                        "prompt_embeds_mask": torch.ones(2, 12)}, 4.0)
    assert v.shape == lat.shape


def test_dual_grpo_rollout_and_loss():
    """Dual-GRPO: the text-encoder LM samples a response whose hidden states condition the Qwen-Image DiT
    rollout; recomputed LM token log-probs equal the sampling ones, and the joint loss back-propagates into
    both the text encoder and the DiT."""
    import torch

    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.pipelines.dual_grpo import DualGRPORollout, TextEncoderLM, dual_grpo_loss
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=qwen_image_tiny", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=1", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
        "trainer.resume_mode=disable", "trainer.logger=[]"])
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    torch.manual_seed(0)
    lm = TextEncoderLM(vocab=64, dim=48, depth=2, heads=2, max_len=64)
    roll = DualGRPORollout(lm, t.rollout, max_new_tokens=5)
    prompt = torch.randint(0, 64, (3, 7))
    out = roll.generate(prompt, seed=3)
    assert out.batch["llm_response_ids"].shape == (3, 5) and out.batch["rollout_log_probs"].shape == (3, 3)
    P = out.meta_info["llm_prompt_len"]
    lp = lm.token_logprobs(out.batch["llm_input_ids"], P)
    torch.testing.assert_close(lp, out.batch["llm_log_probs"], rtol=1e-4, atol=1e-4)
    # one DiT step recomputed with the conditioning the rollout used
    cond = {"prompt_embeds": lm.hidden(out.batch["llm_input_ids"]), "prompt_embeds_mask": out.batch["prompt_embeds_mask"]}
    so = t.adapter.forward_and_sample_previous_step(
        t.actor.module, t.scheduler, latents=out.batch["latents"][:, 0], prev_latents=out.batch["latents"][:, 1],
        step_index=out.batch["step_index"][:, 0], cond=cond, neg_cond=None, guidance_scale=None, noise_level=1.0,
        sde_type="sde")
    loss, m = dual_grpo_loss(so["log_probs"], out.batch["rollout_log_probs"][:, 0], lp, out.batch["llm_log_probs"],
                             torch.tensor([1.0, -0.5, -0.5]))
    loss.backward()
    assert lm.embed.weight.grad is not None and lm.embed.weight.grad.abs().sum() > 0
    assert float(t.actor.engine.flat.main_grad.abs().sum()) > 0  # the DiT gradients land in the fp32 main grads
