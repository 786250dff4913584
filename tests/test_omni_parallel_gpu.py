"""The omni thinker's parallel rollout / training paths on 2 B200s over NCCL: tensor-parallel decode (heads and
KV caches split, one all-reduce per layer) against the replicated decode, and a GRPO step with the model split
into 2 pipeline stages (pipelined decode, forward-only old log-probs, 1F1B update)."""

import math

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _cfg():
    from verl_omni_b200.models.moe_llm import MoEConfig

    return MoEConfig(vocab=2048, hidden=512, layers=2, q_heads=16, kv_heads=2, head_dim=128, experts=8, top_k=2,
                     expert_ffn=256, audio_layers=1, audio_dim=128, audio_mel=16, vision_layers=1, vision_dim=128,
                     vision_patch_dim=48, audio_token=2046, image_token=2047)


def _tp_decode(rank, world):
    import torch.distributed as dist

    import verl_omni_b200.workers.rollout.llm_rollout as LR
    from verl_omni_b200.models.moe_llm import MoELLM
    from verl_omni_b200.parallel.tensor_parallel import TPContext
    from verl_omni_b200.utils.dataproto import DataProto

    torch.manual_seed(0)
    m = MoELLM(_cfg()).to("cuda", torch.bfloat16).eval()
    g = torch.Generator().manual_seed(10 + rank)
    batch = DataProto({"input_ids": torch.randint(0, 2000, (4, 40), generator=g)}, {})
    dev = torch.device("cuda", rank)
    tp = LR.LLMRolloutEngine(m, max_new_tokens=6, temperature=0.0, device=dev, tp=TPContext(dist.group.WORLD))
    ref = LR.LLMRolloutEngine(m, max_new_tokens=6, temperature=0.0, device=dev)
    a, b = tp.generate(batch, seed=1), ref.generate(batch, seed=1)
    # bf16 partial sums + all-reduce vs one GEMM: the first greedy token agrees except at near-ties
    agree = (a.batch["responses"][:, 0] == b.batch["responses"][:, 0]).float().mean().item()
    assert agree >= 0.75, agree
    assert torch.isfinite(a.batch["rollout_log_probs"]).all()
    # sampled decode: both ranks draw the same tokens for the group's batch
    drawn, orig = [], LR.sample_tokens

    def rec(*args, **kw):
        out = orig(*args, **kw)
        drawn.append(out[0].clone())
        return out

    LR.sample_tokens = rec
    try:
        tp.temperature = 1.0
        tp.generate(batch, seed=3)
    finally:
        LR.sample_tokens = orig
    mine = torch.stack(drawn)
    both = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(both, mine)
    assert torch.equal(both[0], both[1])


def test_tensor_parallel_rollout_decode_nccl():
    run_ranks(_tp_decode, 2, device="cuda")


def _pp_step(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    ac = DiffusionActorConfig()
    ac.optim.lr = 1e-4
    cfg = _cfg()
    cfg.layers = 3
    t = OmniGRPOTrainer(cfg, ac, device=torch.device("cuda", rank), n=4, prompt_text=24, audio_tokens=4,
                        image_tokens=4, response_len=6, micro_batch_size=3, pp_size=2)
    assert len(t.model.layers) == (2 if rank == 0 else 1)
    for _ in range(2):
        m = t.step(num_prompts=2)
        vals = torch.tensor([m["actor/pg_loss"], m["actor/grad_norm"], m["rollout_corr/logprob_abs_diff_mean"]],
                            device="cuda", dtype=torch.float64)
        assert all(math.isfinite(v) for v in vals.tolist())
        both = [torch.empty_like(vals) for _ in range(world)]
        dist.all_gather(both, vals)
        assert torch.equal(both[0], both[1])
        # rollout (pipelined decode) and recompute (pipelined forward) agree on the sampled tokens' log-probs
        assert m["rollout_corr/logprob_abs_diff_mean"] < 5e-2


def test_pipeline_parallel_omni_step_nccl():
    run_ranks(_pp_step, 2, device="cuda")
