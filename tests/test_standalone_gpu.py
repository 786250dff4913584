"""Standalone-rollout topology on GPUs: trainer ranks + rollout ranks of one job, batches sent rollout ->
trainer, weights pushed trainer 0 -> rollout ranks by the peer-store kernel into their symmetric buffers.
Checks that every rollout rank ends up holding exactly trainer 0's last pushed flat buffer and that the
trainers report one-step staleness.  Needs 2 GPUs (1 + 1) and runs 2 + 2 when 4 are present."""

import json

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _run(rank, world, outdir):
    from verl_omni_b200.trainer.diffusion.v1.standalone import RolloutRank
    from verl_omni_b200.trainer.diffusion.v1.trainer import build_v1_trainer
    from verl_omni_b200.utils.config import load_config

    R = world // 2
    cfg = load_config("diffusion_trainer", [
        "trainer.device=cuda", "actor_rollout_ref.model.architecture=sd35_small", f"data.train_batch_size={2 * R}",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
        f"actor_rollout_ref.actor.ppo_mini_batch_size={2 * R}", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=8",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=4", "trainer.use_v1=true",
        "trainer.v1.trainer_mode=separate_async", f"trainer.v1.standalone_rollout_ranks={R}",
        "actor_rollout_ref.actor.optim.lr=1e-3", "actor_rollout_ref.nccl_timeout=120"])
    role = build_v1_trainer(cfg)
    hist = role.fit()
    torch.cuda.synchronize()
    if isinstance(role, RolloutRank):
        torch.save({"buf": role.channel.buf.cpu(), "symm": role.channel.symm is not None},
                   f"{outdir}/rollout_{rank}.pt")
    else:
        with open(f"{outdir}/trainer_{rank}.json", "w") as f:
            json.dump([{k: v for k, v in m.items() if isinstance(v, (int, float))} for m in hist], f)
        if rank == 0:
            torch.save(role.last_pushed.cpu(), f"{outdir}/pushed.pt")


def test_standalone_rollout_ranks_cuda(tmp_path):
    n = torch.cuda.device_count()
    world = 4 if n >= 4 else 2
    run_ranks(_run, world, (str(tmp_path),), device="cuda")
    pushed = torch.load(tmp_path / "pushed.pt")
    for r in range(world // 2, world):
        got = torch.load(tmp_path / f"rollout_{r}.pt")
        assert got["symm"], "the push should run over peer memory on one node"
        assert torch.equal(got["buf"], pushed)
    h0 = json.load(open(tmp_path / "trainer_0.json"))
    assert [m["training/staleness/mean"] for m in h0] == [0.0, 1.0, 1.0, 1.0]
