"""v1 trainers on CPU: replay-buffer sync mode, separate-async mode with weight pushes, retry + refill."""

import numpy as np
import pytest
import torch

from verl_omni_b200.trainer.diffusion.v1.replay_buffer import ReplayBuffer
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.rollout.retry_client import WholeSampleRetryClient

OVR = ["trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
       "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
       "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
       "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4", "trainer.logger=[]", "trainer.use_v1=true",
       "trainer.resume_mode=disable"]


def _row(i):
    return DataProto({"x": torch.tensor([float(i)])})


def test_replay_buffer_refill_and_staleness():
    buf = ReplayBuffer(max_off_policy_threshold=2, strategy="fifo", max_refill_rounds=2)
    for g in ("a", "b"):
        buf.register(g, 2, submit_step=0)
    buf.put("a", _row(0), min_global_steps=0, max_global_steps=0)
    buf.put("a", _row(1), min_global_steps=0, max_global_steps=0)
    buf.put("b", None, status="failure")
    calls = []

    def refill(n):
        calls.append(n)
        buf.register("c", 2, submit_step=1)
        buf.put("c", _row(2), min_global_steps=1, max_global_steps=1)
        buf.put("c", _row(3), min_global_steps=1, max_global_steps=1)
        return n

    batch, m = buf.sample(global_steps=1, batch_size=2, refill_fn=refill)
    assert calls == [1] and len(batch) == 4
    assert m["training/rollout_failure/evicted_groups"] == 1
    assert m["training/staleness/max"] == 1
    # stale group dropped (3 steps old > threshold 2)
    buf.register("d", 1, submit_step=0)
    buf.put("d", _row(4), min_global_steps=0, max_global_steps=0)
    buf.register("e", 1, submit_step=5)
    buf.put("e", _row(5), min_global_steps=4, max_global_steps=4)
    batch, m = buf.sample(global_steps=5, batch_size=1)
    assert float(batch.batch["x"][0]) == 5.0 and buf.dropped_stale == 1


def test_retry_client_retries_aborted_then_fails():
    calls = {"n": 0}

    def gen(b):
        calls["n"] += 1
        out = DataProto({"x": torch.arange(len(b)).float()})
        out.meta_info["aborted"] = np.array([True] + [False] * (len(b) - 1))  # first row always aborted
        return out

    c = WholeSampleRetryClient(gen, lambda: 7, max_attempts=3, wait_s=0.0)
    out, status, vmin, vmax = c.generate(DataProto({"x": torch.zeros(3)}))
    assert list(status) == ["failure", "finished", "finished"]
    assert calls["n"] == 3 and len(out) == 2 and vmin[1] == 7


@pytest.mark.parametrize("mode,extra", [("sync", []), ("separate_async",
                                                     ["trainer.v1.parameter_sync_step=2", "trainer.v1.warmup_batches=1"])])
def test_v1_trainer_modes(mode, extra):
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.v1.trainer import build_v1_trainer
    from verl_omni_b200.utils.config import load_config

    D.init_distributed(device="cpu")
    cfg = load_config("diffusion_trainer", OVR + [f"trainer.v1.trainer_mode={mode}", "trainer.total_training_steps=2",
                                                  "trainer.v1.max_off_policy_threshold=4"] + extra)
    t = build_v1_trainer(cfg)
    hist = t.fit()
    assert t.global_steps == 2
    for m in hist:
        assert np.isfinite(m["actor/grad_norm"])
        assert "training/staleness/mean" in m
    if mode == "separate_async":
        assert t.weight_version == 2
        # the replica received the trainer's weights
        for (n1, p1), (n2, p2) in zip(t.core.actor.module.named_parameters(), t.rollout.module.named_parameters()):
            assert torch.equal(p1.detach(), p2.detach()), n1


def _standalone(rank, world, outdir):
    import json

    from verl_omni_b200.trainer.diffusion.v1.trainer import build_v1_trainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=4",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=2",
        "actor_rollout_ref.actor.ppo_mini_batch_size=4", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=4", "trainer.use_v1=true",
        "trainer.v1.trainer_mode=separate_async", "trainer.v1.standalone_rollout_ranks=2",
        "trainer.v1.parameter_sync_step=1", "actor_rollout_ref.actor.optim.lr=1e-3"])
    role = build_v1_trainer(cfg)
    hist = role.fit()
    from verl_omni_b200.trainer.diffusion.v1.standalone import RolloutRank

    if isinstance(role, RolloutRank):
        # after the run the rollout's weights are a pushed version: compare with the trainer's final push
        torch.save(role.channel.buf.clone(), f"{outdir}/rollout_{rank}.pt")
    else:
        json.dump([{k: v for k, v in m.items() if isinstance(v, (int, float))} for m in hist],
                  open(f"{outdir}/trainer_{rank}.json", "w"))
        if rank == 0:
            torch.save(role.last_pushed.clone(), f"{outdir}/pushed.pt")


def test_standalone_rollout_ranks_gloo(tmp_path):
    """4 gloo ranks: 2 trainers + 2 standalone rollout ranks.  Batches travel rollout -> trainer, weights
    trainer 0 -> both rollout ranks after every step (one-step off-policy): each rollout rank ends up holding
    exactly the last pushed flat buffer, and the trainers see samples one version behind their policy."""
    import json

    from tests._dist_util import run_ranks

    run_ranks(_standalone, 4, (str(tmp_path),))
    pushed = torch.load(tmp_path / "pushed.pt")
    for r in (2, 3):
        assert torch.equal(torch.load(tmp_path / f"rollout_{r}.pt"), pushed)
    h0 = json.load(open(tmp_path / "trainer_0.json"))
    assert [m["training/global_step"] for m in h0] == [1, 2, 3, 4]
    assert h0[0]["training/staleness/mean"] == 0.0 and h0[2]["training/staleness/mean"] == 1.0
    assert all(m["actor/grad_norm"] == m["actor/grad_norm"] for m in h0)
