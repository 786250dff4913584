"""CPU tests: config overrides/interpolation, MFU counter, tracking, profiler, attention policy, CLI."""

import json

import numpy as np

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


def test_parquet_datasets(tmp_path):
    """Prompt / offline-DPO / MLLM-DPO parquet datasets: tensors and prompts round-trip through pyarrow."""
    import pandas as pd

    from verl_omni_b200.utils.datasets_parquet import (ParquetMLLMDPODataset, ParquetOfflineDPODataset,
                                                       ParquetPromptDataset)

    rng = np.random.default_rng(0)
    emb = [rng.standard_normal((5, 8)).astype("float32") for _ in range(3)]
    msgs = lambda t: [{"role": "user", "content": t}]  # noqa: E731  (chat-message prompts, verl's format)
    pd.DataFrame({"prompt": [msgs("a cat"), msgs("a dog"), msgs("hi")],
                  "negative_prompt": ["", "blurry", ""], "data_source": ["ocr"] * 3,
                  "reward_model": [{"ground_truth": "CAT"}, {"ground_truth": "DOG"}, {"ground_truth": None}],
                  "prompt_embeds": [e.reshape(-1).tolist() for e in emb], "prompt_embeds_shape": [[5, 8]] * 3}
                 ).to_parquet(tmp_path / "p.parquet")
    ds = ParquetPromptDataset(str(tmp_path / "p.parquet"), cond_keys=("prompt_embeds",), token_len=6, vocab=100)
    b = ds.get_batch([2, 0])
    assert b.batch["input_ids"].shape == (2, 6) and b.batch["prompt_embeds"].shape == (2, 5, 8)
    assert torch.allclose(b.batch["prompt_embeds"][1], torch.tensor(emb[0]))
    assert list(b.non_tensor_batch["ground_truth"]) == [None, "CAT"] and b.non_tensor_batch["raw_prompt"][0] == "hi"
    lat = rng.standard_normal((2, 4, 4, 4)).astype("float32")
    pd.DataFrame({"img_win_latents": [lat[0].reshape(-1).tolist()], "img_win_latents_shape": [[4, 4, 4]],
                  "img_lose_latents": [lat[1].reshape(-1).tolist()], "img_lose_latents_shape": [[4, 4, 4]],
                  "prompt_embeds": [emb[0].reshape(-1).tolist()], "prompt_embeds_shape": [[5, 8]],
                  "win_score": [0.9], "lose_score": [0.1]}).to_parquet(tmp_path / "d.parquet")
    d = ParquetOfflineDPODataset(str(tmp_path / "d.parquet"), cond_keys=("prompt_embeds",)).get_batch([0])
    assert d.batch["latents_clean"].shape == (2, 4, 4, 4)
    torch.testing.assert_close(d.batch["rm_scores"], torch.tensor([0.9, 0.1]))
    pd.DataFrame({"prompt_ids": [[5, 6, 7], [8]], "chosen_ids": [[1, 2], [3]], "rejected_ids": [[4], [5, 6, 7]]}
                 ).to_parquet(tmp_path / "m.parquet")
    ch, rj = ParquetMLLMDPODataset(str(tmp_path / "m.parquet")).get_pairs([0, 1])
    assert ch.batch["input_ids"].shape == (2, 5) and rj.batch["response_mask"].sum().item() == 4


def test_trainer_reads_parquet_prompts(tmp_path):
    """data.train_files pointing at a parquet file feeds the trainer's prompts (text-encoder model)."""
    import pandas as pd

    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

    pd.DataFrame({"prompt": [[{"role": "user", "content": f"prompt number {i}"}] for i in range(6)],
                  "data_source": ["toy"] * 6}).to_parquet(tmp_path / "train.parquet")
    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        f"data.train_files={tmp_path / 'train.parquet'}", "actor_rollout_ref.rollout.n=2",
        "actor_rollout_ref.rollout.pipeline.num_inference_steps=2", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4", "trainer.resume_mode=disable", "trainer.logger=[]",
        "trainer.total_training_steps=1"])
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    assert len(t.dataset) == 6
    m = t.step()
    assert m["actor/grad_norm"] == m["actor/grad_norm"]


def test_media_dump_video_and_wav(tmp_path):
    """Video frames (mp4 when an ffmpeg writer exists, else an animated gif) and 16-bit WAV audio are written
    beside the JSONL record."""
    import wave

    from verl_omni_b200.utils.tracking import dump_media_generations

    vids = torch.rand(2, 3, 4, 16, 16) * 2 - 1
    aud = [torch.sin(torch.linspace(0, 100, 800)), None]
    fn = dump_media_generations(str(tmp_path), 3, ["a", "b"], [0.1, 0.2], videos=vids, audios=aud,
                                sample_rates=[8000, 8000])
    rows = [json.loads(ln) for ln in open(fn)]
    assert rows[0]["video"].split(".")[-1] in ("mp4", "gif", "npy") and "audio" not in rows[1]
    with wave.open(rows[0]["audio"]) as w:
        assert w.getframerate() == 8000 and w.getnframes() == 800 and w.getsampwidth() == 2
