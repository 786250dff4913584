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
