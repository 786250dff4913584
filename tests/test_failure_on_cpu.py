"""Failure detection without any GPU: a rank that stops (host-side), capacity-expiration checkpoints."""

import os
import time

import pytest
import torch
import torch.multiprocessing as mp

from tests._dist_util import free_port
from verl_omni_b200.utils.failure import HeartbeatMonitor, RankFailure, should_save_ckpt_esi


def test_esi_expiration_rule(monkeypatch):
    now = 1_700_000_000.0
    monkeypatch.delenv("MLP_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP", raising=False)
    monkeypatch.delenv("SAGEMAKER_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP", raising=False)
    assert not should_save_ckpt_esi(60, 0, now=now)
    monkeypatch.setenv("MLP_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP", str(now + 100))
    assert not should_save_ckpt_esi(60, 10, now=now)
    assert should_save_ckpt_esi(60, 50, now=now)
    monkeypatch.setenv("MLP_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP", str((now + 30) * 1000))  # ms form
    assert should_save_ckpt_esi(60, 0, now=now)


def _rank(rank, world, port, q):
    mon = HeartbeatMonitor(rank, world, "127.0.0.1", port, interval_s=0.1, timeout_s=1.0)
    if rank == world - 1:  # this rank dies between steps: its heartbeat thread stops with it
        time.sleep(0.5)
        mon.stop()
        q.put((rank, "exited"))
        q.close()
        q.join_thread()  # flush before the hard exit
        os._exit(0)
    t0 = time.time()
    detected = None
    while time.time() - t0 < 20:
        try:
            mon.check()
        except RankFailure as e:
            detected = e.ranks
            break
        time.sleep(0.2)
    q.put((rank, detected))
    time.sleep(1.0)  # keep rank 0's store alive until the others have read


def test_heartbeat_reports_stopped_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    world = 3
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    assert res[2] == "exited"
    assert res[0] == [2] and res[1] == [2]


def _esi_train(rank, world, outdir):
    from tests.test_e2e_tiny_on_cpu import OVR
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    # capacity block ends in 1 h, redundancy 2 h: every step forces a checkpoint although save_freq=100
    os.environ["MLP_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP"] = str(time.time() + 3600)
    cfg = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={outdir}",
                                                  "trainer.total_training_steps=5", "trainer.save_freq=100",
                                                  "trainer.esi_redundant_time=7200", "trainer.resume_mode=disable",
                                                  "trainer.heartbeat_timeout_s=30"])
    t = PolicyGradientTrainer(cfg)
    t.step()
    assert t.max_steps_duration > 0
    t._heartbeat.stop()


def test_esi_forces_checkpoint_gloo_world2(tmp_path):
    from tests._dist_util import run_ranks

    run_ranks(_esi_train, 2, (str(tmp_path),))
    assert (tmp_path / "latest_checkpointed_iteration.txt").read_text() == "1"
    assert (tmp_path / "global_step_1" / "actor" / "fsdp_config.json").exists()


def test_rollout_server_drain_then_abort():
    """A stuck engine call is aborted after the drain timeout; queued requests get aborted outputs."""
    import asyncio
    import threading
    from types import SimpleNamespace

    import torch

    from verl_omni_b200.pipelines.request_batch import DiffusionRequest, RolloutOutput
    from verl_omni_b200.workers.rollout.server import DiffusionRolloutServer

    stop = threading.Event()

    class _Engine:
        cfg = SimpleNamespace(max_num_seqs=1)

        def abort(self):
            stop.set()

    class _Srv(DiffusionRolloutServer):
        def _window(self, req):
            return (0, 1)

        def _run(self, reqs):
            stop.wait(30)  # stands for a long engine call that only an abort ends
            return [RolloutOutput({"x": torch.zeros(1)}, {"aborted": stop.is_set(), "request_id": r.request_id})
                    for r in reqs]

    async def main():
        srv = _Srv(_Engine(), max_num_seqs=1, batch_wait_s=0.0)
        reqs = [DiffusionRequest(request_id=f"r{i}", cond={"p": torch.zeros(4)}, sampling={}, seed=i)
                for i in range(3)]
        tasks = [asyncio.create_task(srv.generate(r)) for r in reqs]
        await asyncio.sleep(0.2)  # first request is in the engine, the other two queued
        t0 = time.monotonic()
        n = await srv.abort_all_requests(drain_timeout_s=0.3)
        outs = await asyncio.gather(*tasks)
        dt = time.monotonic() - t0
        await srv.stop()
        return n, outs, dt

    n, outs, dt = asyncio.run(main())
    assert n == 2 and dt < 10
    assert all(o.aborted for o in outs)
    assert sorted(o.metadata["request_id"] for o in outs) == ["r0", "r1", "r2"]


def _retention(rank, world, outdir):
    from tests.test_e2e_tiny_on_cpu import OVR
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=3",
                                                  "trainer.save_freq=1", "trainer.resume_mode=disable",
                                                  "trainer.max_actor_ckpt_to_keep=2",
                                                  "global_profiler.tool=torch", "global_profiler.steps=[2]",
                                                  f"global_profiler.save_path={outdir}/prof"])
    PolicyGradientTrainer(cfg).fit()


def test_checkpoint_retention_and_step_profiler(tmp_path):
    from tests._dist_util import run_ranks

    run_ranks(_retention, 1, (str(tmp_path),))
    kept = sorted(d for d in os.listdir(tmp_path) if d.startswith("global_step_"))
    assert kept == ["global_step_2", "global_step_3"]
    assert (tmp_path / "prof" / "trace_step2_rank0.json").exists()


def _det(rank, world, outdir, tag):
    from tests.test_e2e_tiny_on_cpu import OVR
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", OVR + ["trainer.total_training_steps=2", "trainer.resume_mode=disable"])
    t = PolicyGradientTrainer(cfg)
    t.fit()
    if rank == 0:
        torch.save(t.actor.engine.flat.flat.clone(), f"{outdir}/{tag}.pt")


def test_two_identical_runs_are_bitwise_equal(tmp_path):
    """Deterministic mode: the same seeds and config give bit-identical weights (two gloo world-2 runs)."""
    import torch

    from tests._dist_util import run_ranks

    run_ranks(_det, 2, (str(tmp_path), "a"))
    run_ranks(_det, 2, (str(tmp_path), "b"))
    assert torch.equal(torch.load(tmp_path / "a.pt"), torch.load(tmp_path / "b.pt"))
