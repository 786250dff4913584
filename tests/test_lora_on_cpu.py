"""LoRA adapters: injection, reference (disabled) path, copy/EMA, PEFT export/import, trainer step."""

import json

import torch

from verl_omni_b200.models.dit import DiT, DiTConfig
from verl_omni_b200.models import lora as LR


def test_inject_ema_export(tmp_path):
    torch.manual_seed(0)
    m = DiT(DiTConfig.tiny_plumbing())
    x, t, c = torch.randn(2, 4, 16, 16), torch.tensor([500.0, 20.0]), torch.randn(2, 7, 256)
    base_out = m(x, t, c)
    names = LR.inject_lora(m, rank=8, alpha=16, target_modules=["qkv", "o"], adapters=("default", "old"))
    assert names and all(n.endswith(("qkv", "o")) for n in names)
    trainable = [n for n, p in m.named_parameters() if p.requires_grad]
    assert trainable and all("lora_" in n and ".default" in n for n in trainable)
    # B initialised to zero -> identical output; disabled adapters -> base model
    torch.testing.assert_close(m(x, t, c), base_out)
    for _, l in LR.lora_layers(m):
        torch.nn.init.normal_(l.lora_B["default"], std=0.1)
    out = m(x, t, c)
    assert not torch.allclose(out, base_out)
    with LR.use_adapter(m, None):
        torch.testing.assert_close(m(x, t, c), base_out)
    LR.copy_adapter(m, "default", "old")
    with LR.use_adapter(m, "old"):
        torch.testing.assert_close(m(x, t, c), out)
    l0 = next(iter(LR.lora_layers(m)))[1]
    before = l0.lora_B["old"].detach().clone()
    with torch.no_grad():
        l0.lora_B["default"].add_(1.0)
    LR.ema_update_adapter(m, "default", "old", decay=0.75)
    torch.testing.assert_close(l0.lora_B["old"], 0.75 * before + 0.25 * l0.lora_B["default"])
    LR.export_peft_adapter(m, str(tmp_path / "adapter"))
    cfg = json.loads((tmp_path / "adapter" / "adapter_config.json").read_text())
    assert cfg["r"] == 8 and cfg["peft_type"] == "LORA"
    m2 = DiT(DiTConfig.tiny_plumbing())
    LR.inject_lora(m2, rank=8, alpha=16, target_modules=["qkv", "o"])
    assert LR.load_peft_adapter(m2, str(tmp_path / "adapter")) == len(names)
    assert abs(LR.lora_checksum(m2) - LR.lora_checksum(m)) < 1e-3


def _lora_ckpt(rank, world, outdir):
    from verl_omni_b200.models.lora import export_peft_adapter
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=2",
        "actor_rollout_ref.actor.ppo_mini_batch_size=2", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=1",
        "actor_rollout_ref.model.lora_rank=4", "actor_rollout_ref.model.lora_alpha=8",
        "actor_rollout_ref.actor.optim.lr=1e-2", f"trainer.default_local_dir={outdir}"])
    t = PolicyGradientTrainer(cfg)
    t.step()
    t.save_checkpoint()
    if rank == 0:
        export_peft_adapter(t.actor.module, f"{outdir}/live")


def test_peft_export_from_sharded_checkpoint(tmp_path):
    """Two gloo ranks write a LoRA run's sharded checkpoint; the PEFT adapter re-assembled from the shard files
    equals the one exported from the live module."""
    import json

    from safetensors.torch import load_file

    from tests._dist_util import run_ranks
    from verl_omni_b200.models.lora import export_peft_from_checkpoint

    run_ranks(_lora_ckpt, 2, (str(tmp_path),))
    n = export_peft_from_checkpoint(str(tmp_path / "global_step_1" / "actor"), str(tmp_path / "from_ckpt"),
                                    lora_alpha=8)
    a = load_file(str(tmp_path / "from_ckpt" / "adapter_model.safetensors"))
    b = load_file(str(tmp_path / "live" / "adapter_model.safetensors"))
    assert n > 0 and set(a) == set(b)
    for k in a:
        torch.testing.assert_close(a[k], b[k].float(), rtol=1e-2, atol=1e-3)  # fp32 master vs bf16 copy
    assert json.load(open(tmp_path / "from_ckpt" / "adapter_config.json"))["r"] == 4
