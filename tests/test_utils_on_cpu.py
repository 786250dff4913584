"""CPU tests: config overrides/interpolation, MFU counter, tracking, profiler, attention policy, CLI."""

import json

import pytest
import torch

from verl_omni_b200.utils.config import load_config


def test_config_overrides_and_errors():
    c = load_config("diffusion_trainer", ["actor_rollout_ref.rollout.n=3", "+custom.key=[1,2]",
                                          "~trainer.v1.warmup_batches"])
    assert c.actor_rollout_ref.actor.rollout_n == 3 and c.custom.key == [1, 2]
    assert "warmup_batches" not in c.trainer.v1
    with pytest.raises(KeyError):
        load_config("diffusion_trainer", ["no.such.key=1"])
    assert c.algorithm.adv_estimator == "flow_grpo"


def test_mfu_counter_matches_manual_count():
    from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig
    from verl_omni_b200.utils.mfu import DiffusionFlopsCounter

    cfg = MMDiTConfig.tiny()
    m = MMDiT(cfg)
    c = DiffusionFlopsCounter(m, "sd3")
    f1 = c.forward_flops(16, 12)
    assert f1 > 0 and c.forward_flops(32, 12) > f1
    assert c.estimate_flops(2, 3, 16, 12) == pytest.approx(f1 * 2 * 3 * 3)
    assert 0 < c.mfu(1e15, 1.0) < 10


def test_tracking_and_dump(tmp_path):
    from verl_omni_b200.utils.tracking import Tracking, dump_generations

    t = Tracking("p", "e", ["jsonl"], log_dir=str(tmp_path))
    t.log({"a": 1.0, "b": 2}, step=3)
    t.finish()
    line = json.loads((tmp_path / "p" / "e" / "metrics.jsonl").read_text().splitlines()[0])
    assert line["step"] == 3 and line["a"] == 1.0
    fn = dump_generations(str(tmp_path / "gen"), 1, torch.zeros(2, 3, 8, 8), ["x", "y"], [0.1, 0.2])
    assert len(open(fn).read().splitlines()) == 2


def test_profiler_torch_trace(tmp_path):
    from verl_omni_b200.utils.profiler import StepProfiler, mark

    p = StepProfiler({"tool": "torch", "steps": [2], "save_path": str(tmp_path)})
    p.start(1)
    assert p.stop(1) is None
    p.start(2)
    with mark("phase"):
        torch.ones(4) + 1
    out = p.stop(2)
    assert out and (tmp_path / out.split("/")[-1]).exists()


def test_attention_policy():
    from verl_omni_b200.utils import attention_backend as ab

    assert ab.resolve_backend("native") == "sdpa"
    assert ab.validate_attention_consistency("TORCH_SDPA", "sdpa") == "sdpa"
    if not torch.cuda.is_available():
        assert ab.resolve_backend("_flash_3_varlen_hub") == "sdpa"


def test_cli_entrypoints(capsys):
    from verl_omni_b200.cli import diagnose, print_cfg

    assert "torch" in diagnose.collect()
    print_cfg.main(["actor_rollout_ref.rollout.n=5"])
    assert "n: 5" in capsys.readouterr().out


def test_non_diffusers_model_base_roundtrip(tmp_path):
    from dataclasses import dataclass

    import torch.nn as nn

    from verl_omni_b200.pipelines.non_diffusers_model_base import NonDiffusersModelBase

    @dataclass
    class Cfg:
        dim: int = 8
        layers: int = 2

    class Block(nn.Module):
        def __init__(self, d):
            super().__init__()
            self.lin = nn.Linear(d, d)

        def forward(self, x):
            return torch.relu(self.lin(x))

    class Toy(NonDiffusersModelBase):
        config_class = Cfg
        _no_split_modules = ("Block",)
        supports_gradient_checkpointing = True

        def __init__(self, config):
            super().__init__(config)
            self.blocks = nn.ModuleList([Block(config.dim) for _ in range(config.layers)])

        def forward(self, x):
            for b in self.blocks:
                x = self.maybe_checkpoint(b, x)
            return x

    torch.manual_seed(0)
    m = Toy(Cfg())
    m.save_pretrained(str(tmp_path))
    m2 = Toy.from_pretrained(str(tmp_path))
    x = torch.randn(3, 8, requires_grad=True)
    torch.testing.assert_close(m(x), m2(x))
    assert len(m.no_split_module_instances()) == 2
    m2.enable_gradient_checkpointing()
    m2(x).sum().backward()
    assert x.grad is not None
