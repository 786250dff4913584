"""Qwen3-Omni thinker weights in the Hugging Face layout: the language model of transformers'
``Qwen3OmniMoeThinkerTextModel`` (random tiny config) loads into ``MoELLM`` and gives the same hidden
states; the hub layout (one tensor per expert) round-trips through export and ``load_thinker``; expert-parallel
ranks and pipeline stages take only their own slices."""

from types import SimpleNamespace

import pytest
import torch

from verl_omni_b200.models import hf_omni_io as H
from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM, MoEStage

tr = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")


def _hf_state(cfg: MoEConfig, seed: int = 0):
    from transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe import Qwen3OmniMoeTextConfig

    torch.manual_seed(seed)
    tc = Qwen3OmniMoeTextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=64, num_hidden_layers=cfg.layers,
        num_attention_heads=cfg.q_heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        num_experts=cfg.experts, num_experts_per_tok=cfg.top_k, moe_intermediate_size=cfg.expert_ffn,
        rms_norm_eps=cfg.eps, max_position_embeddings=256,
        rope_parameters={"rope_theta": cfg.rope_theta, "rope_type": "default", "mrope_section": [2, 3, 3]})
    tc._attn_implementation = "eager"
    hf = tr.Qwen3OmniMoeThinkerTextModel(tc).eval()
    with torch.no_grad():
        for p in hf.parameters():
            p.normal_(0, 0.05)
    sd = {"thinker.model." + k: v.clone() for k, v in hf.state_dict().items()}
    sd["thinker.lm_head.weight"] = torch.randn(cfg.vocab, cfg.hidden) * 0.05
    return hf, sd


def _load(m, ours):
    params = dict(m.named_parameters())
    with torch.no_grad():
        for n, t in ours.items():
            params[n].copy_(t)


def test_thinker_matches_transformers_text_model():
    cfg = MoEConfig.tiny()
    hf, sd = _hf_state(cfg)
    m = MoELLM(cfg).eval()
    ours = H.thinker_from_hf(sd, m)
    text = [n for n, _ in m.named_parameters() if not n.startswith(("audio_tower.", "visual."))]
    assert sorted(ours) == sorted(text)
    _load(m, ours)
    ids = torch.randint(0, cfg.vocab - 2, (2, 13))
    with torch.no_grad():
        ref = hf(input_ids=ids).last_hidden_state
        got = m(ids, return_hidden=True)
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
        logits = m(ids)
    torch.testing.assert_close(logits, ref @ sd["thinker.lm_head.weight"].t(), rtol=1e-4, atol=1e-5)


def test_hub_layout_round_trip_and_load_from_directory(tmp_path):
    cfg = MoEConfig.tiny()
    _, sd = _hf_state(cfg, seed=1)
    a = MoELLM(cfg).eval()
    _load(a, H.thinker_from_hf(sd, a))
    hub = H.thinker_to_hf(dict(a.named_parameters()), a)
    assert "thinker.model.layers.1.mlp.experts.7.up_proj.weight" in hub
    assert "thinker.model.layers.0.self_attn.v_proj.weight" in hub
    assert not any(k.startswith(("thinker.audio_tower", "thinker.visual")) for k in hub)
    from safetensors.torch import save_file

    save_file({k: v.detach().contiguous() for k, v in hub.items()}, str(tmp_path / "model-00001.safetensors"))
    b = MoELLM(cfg).eval()
    n = H.load_thinker(b, str(tmp_path))
    assert n == len(H.thinker_from_hf(sd, a))
    ids = torch.randint(0, cfg.vocab - 2, (2, 9))
    with torch.no_grad():
        torch.testing.assert_close(b(ids), a(ids))


def test_expert_parallel_rank_and_pipeline_stage_take_their_slices():
    cfg = MoEConfig.tiny()
    _, sd = _hf_state(cfg, seed=2)
    full = MoELLM(cfg).eval()
    _load(full, H.thinker_from_hf(sd, full))
    ep = SimpleNamespace(ep=2, rank=1, per_rank=cfg.experts // 2)
    part = MoELLM(cfg, ep).eval()
    got = H.thinker_from_hf(sd, part)
    torch.testing.assert_close(got["layers.0.w_gate_up"], full.layers[0].w_gate_up[cfg.experts // 2:])
    torch.testing.assert_close(got["layers.1.w_down"], full.layers[1].w_down[cfg.experts // 2:])
    # per-expert hub layout, EP slice
    hub = H.thinker_to_hf(dict(full.named_parameters()), full)
    got2 = H.thinker_from_hf(hub, part)
    torch.testing.assert_close(got2["layers.1.w_gate_up"], full.layers[1].w_gate_up[cfg.experts // 2:])
    # second pipeline stage: global layer 1 as its layer 0, the head, no embedding
    st = MoEStage(MoELLM(cfg), 1, 2, False, True)
    gs = H.thinker_from_hf(sd, st, layer_offset=1)
    assert "embed" not in gs and "lm_head.weight" in gs
    torch.testing.assert_close(gs["layers.0.q_proj.weight"], full.layers[1].q_proj.weight)


def test_omni_trainer_starts_from_hf_checkpoint(tmp_path):
    """``OmniGRPOTrainer(model_path=...)`` (``actor_rollout_ref.model.path``) starts from the checkpoint's
    language-model weights; a step runs from there."""
    from safetensors.torch import save_file

    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    cfg = MoEConfig.tiny()
    _, sd = _hf_state(cfg, seed=3)
    save_file({k: v.contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    t = OmniGRPOTrainer(cfg, DiffusionActorConfig(), device=torch.device("cpu"), n=2, model_path=str(tmp_path))
    torch.testing.assert_close(t.model.layers[1].router.weight, sd["thinker.model.layers.1.mlp.gate.weight"])
    torch.testing.assert_close(t.model.embed, sd["thinker.model.embed_tokens.weight"])
    m = t.step(num_prompts=1)
    assert m["actor/grad_norm"] == m["actor/grad_norm"]
