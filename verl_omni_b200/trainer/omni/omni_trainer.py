"""Omni (Qwen3-Omni-thinker-shaped MoE) GRPO / GSPO trainer and offline DPO.

Counterpart of ``main_omni`` / ``OmniPPOTrainerSync`` / ``OmniDirectPreferenceRayTrainer``
(``verl_omni/trainer/main_omni.py:57-360``, ``verl_omni/trainer/omni/ray_omni_trainer.py:66-728``):
one step = multimodal prompts (text ids + audio log-mel frames + image patches) -> ``n`` sampled
responses per prompt -> rule reward (seeded hash of the response tokens) -> GRPO group advantage ->
recomputed old log-probs -> token-level GRPO or sequence-level GSPO update.  Expert weights can be
sharded over an EP group (all-to-all dispatch/combine).
"""

from __future__ import annotations

import time
from typing import Optional

import numpy as np
import torch

from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM
from verl_omni_b200.parallel import dist as D
from verl_omni_b200.trainer.diffusion.diffusion_algos import group_normalize
from verl_omni_b200.trainer.omni.omni_algos import get_omni_loss_fn, omni_dpo_loss, sequence_logps
from verl_omni_b200.utils import metrics as M
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig
from verl_omni_b200.workers.engine.base import ShardedEngine
from verl_omni_b200.workers.reward.reward_manager import hash_token_reward
from verl_omni_b200.workers.rollout.llm_rollout import LLMRolloutEngine


class OmniGRPOTrainer:
    def __init__(self, cfg: MoEConfig, actor_cfg: DiffusionActorConfig, *, device, n: int = 8,
                 prompt_text: int = 16, audio_tokens: int = 4, image_tokens: int = 4, response_len: int = 8,
                 loss_mode: str = "grpo", ep_group=None, tp_group=None, seed: int = 0,
                 micro_batch_size: Optional[int] = None, temperature: float = 1.0, kv_block_size: int = 0,
                 total_steps: int = 1000, pp_size: int = 1, rollout_tp_group=None, model_path: Optional[str] = None):
        """``pp_size > 1``: pipeline parallelism over ``pp_size`` stages (rank r is stage r // (world / pp) of
        data-parallel rank r % (world / pp)); each stage holds a contiguous slice of the layers, the rollout
        decodes through the stages and the update runs the 1F1B schedule over the micro-batches."""
        torch.manual_seed(seed)
        self.pp_size = int(pp_size)
        if self.pp_size > 1 and tp_group is not None and D.world_size(tp_group) > 1:
            raise ValueError("pipeline parallelism is combined with data and expert parallelism (no TP groups)")
        self.micro_batch_size = micro_batch_size  # sequences per forward/backward (None: the whole batch)
        self.cfg, self.actor_cfg, self.device, self.n = cfg, actor_cfg, device, n
        self.prompt_text, self.audio_tokens, self.image_tokens = prompt_text, audio_tokens, image_tokens
        ep = None
        self.expert_dp_group = None
        if ep_group is not None and D.world_size(ep_group) > 1:
            from verl_omni_b200.parallel.expert_parallel import FusedExpertParallel

            # expert parallelism over consecutive blocks of ranks: each rank holds experts / ep of every layer
            # (weights, fp32 main grads and optimizer state); the ranks holding the same experts form the
            # expert data-parallel group.  Peer-memory dispatch / combine where it applies (CUDA, one node),
            # NCCL all-to-all otherwise.
            ep_size = D.world_size(ep_group)
            ep_group, self.expert_dp_group = D.make_hsdp_groups(ep_size)
            if self.pp_size > 1:
                # EP groups of consecutive ranks lie inside one stage (ep divides the ranks per stage); the
                # ranks holding the same experts are those of the same EP position within the same stage
                W = D.world_size()
                dpn = W // self.pp_size
                if dpn % ep_size:
                    raise ValueError(f"expert_model_parallel_size={ep_size} must divide the {dpn} ranks per stage")
                self.expert_dp_group = D.make_partition_groups(
                    [[s * dpn + j + k * ep_size for k in range(dpn // ep_size)]
                     for s in range(self.pp_size) for j in range(ep_size)])
            ep = FusedExpertParallel(cfg.experts, ep_group)
        with torch.device(device):
            self.model = MoELLM(cfg, ep)
        if model_path:
            # HF checkpoint of the thinker (hub or fused expert layout): the language model's weights; each EP
            # rank reads its own experts (the towers keep their initialisation)
            from verl_omni_b200.models.hf_omni_io import load_thinker

            load_thinker(self.model, model_path)
        # tensor + sequence parallelism (Megatron layout): ranks of a TP group share their samples and split each
        # sequence and the attention heads; weights stay replicated, so every rank's gradient is its share and
        # the loss is scaled by tp for the world-averaged gradient (groups of consecutive ranks)
        self.tp_size = D.world_size(tp_group) if tp_group is not None else 1
        if self.tp_size > 1:
            from verl_omni_b200.parallel.tensor_parallel import TPContext

            self.model.tp = TPContext(tp_group)
        self.pp = None
        dp_group = None
        if self.pp_size > 1:
            from verl_omni_b200.models.moe_llm import MoEStage
            from verl_omni_b200.parallel.pipeline import PipeLink, stage_layers

            W = D.world_size()
            if W % self.pp_size or cfg.layers < self.pp_size:
                raise ValueError(f"pipeline_model_parallel_size={self.pp_size} must divide the world size {W} "
                                 f"and not exceed the layer count {cfg.layers}")
            dpn = W // self.pp_size
            dp_group, pp_group = D.make_hsdp_groups(dpn)  # same-stage ranks, and the ranks of one pipeline
            s_idx = D.rank() // dpn
            lo, hi = stage_layers(cfg.layers, self.pp_size, s_idx)
            self.model = MoEStage(self.model, lo, hi, s_idx == 0, s_idx == self.pp_size - 1)
            self.pp = PipeLink(s_idx, self.pp_size, [D.rank() % dpn + k * dpn for k in range(self.pp_size)],
                               pp_group, device)
        self.engine = ShardedEngine(self.model, actor_cfg, device=device, total_steps=total_steps,
                                    expert_group=self.expert_dp_group, group=dp_group, pp_size=self.pp_size)
        rtp = None
        if rollout_tp_group is not None and D.world_size(rollout_tp_group) > 1:
            from verl_omni_b200.parallel.tensor_parallel import TPContext

            if self.pp is not None:
                raise ValueError("a tensor-parallel rollout is not combined with pipeline stages")
            rtp = self.model.tp if (self.model.tp is not None and self.model.tp.group is rollout_tp_group) \
                else TPContext(rollout_tp_group)
        self.rollout = LLMRolloutEngine(self.model, max_new_tokens=response_len, device=device,
                                        temperature=temperature, kv_block_size=kv_block_size, pp=self.pp,
                                        tp=rtp)
        self.temperature = temperature
        self.loss_fn = get_omni_loss_fn(loss_mode)
        self.loss_mode = loss_mode
        self.step_count = 0
        self.rank = D.rank()
        self.dp_rank, self.dp = self.rank // self.tp_size, D.world_size() // self.tp_size
        if self.pp is not None:
            self.dp = D.world_size() // self.pp_size
            self.dp_rank = self.rank % self.dp

    dataset = None  # a ParquetOmniRLDataset: prompts come from it instead of the synthetic generator

    def make_prompts(self, num: int, seed: int) -> DataProto:
        if self.dataset is not None:
            # step s, data-parallel rank r: rows [((s - 1) dp + r) num, ... + num) of the dataset, cycling
            start = ((self.step_count - 1) * self.dp + self.dp_rank) * num
            return self.dataset.get_batch(list(range(start, start + num)), uid_prefix=f"{self.step_count}-")
        g = torch.Generator().manual_seed(seed)
        cfg = self.cfg
        text = torch.randint(0, cfg.vocab - 2, (num, self.prompt_text), generator=g)
        ids = torch.cat([text, torch.full((num, self.audio_tokens), cfg.audio_token),
                         torch.full((num, self.image_tokens), cfg.image_token)], 1)
        return DataProto({"input_ids": ids,
                          "audio_feats": torch.randn(num, self.audio_tokens, cfg.audio_mel, generator=g),
                          "image_patches": torch.randn(num, self.image_tokens, cfg.vision_patch_dim, generator=g)},
                         {"uid": np.array([f"{seed}-{i}" for i in range(num)], dtype=object)})

    def _resp_logprobs(self, data: DataProto) -> torch.Tensor:
        ids = data.batch["input_ids"].to(self.device)
        P = data.batch["prompts"].shape[1]
        # the vocabulary projection and log-softmax run chunked inside the model (no [B, S, V] logits)
        tgt = torch.zeros_like(ids[:, :-1])
        tgt[:, P - 1:] = ids[:, P:]
        af, ip = self._feats(data)
        lp = self.model(ids[:, :-1], audio_feats=af, image_patches=ip, targets=tgt,
                        temperature=self.temperature)
        return lp[:, P - 1:]

    def _feats(self, data: DataProto):
        """The prompt's audio frames / image patches on the device (None when the batch has none)."""
        return tuple(data.batch[k].to(self.device) if k in data.batch else None
                     for k in ("audio_feats", "image_patches"))

    def _micro(self, data: DataProto) -> list[slice]:
        n = len(data)
        mb = self.micro_batch_size or n
        return [slice(i, min(n, i + mb)) for i in range(0, n, mb)]

    def step(self, num_prompts: int = 2) -> dict:
        """One GRPO / GSPO step on ``num_prompts`` prompts x ``n`` responses of this data-parallel rank:
        rollout -> rule reward -> group advantage -> old log-probs -> micro-batched update -> optimizer."""
        if self.pp is not None:
            return self._step_pp(num_prompts)
        self.step_count += 1
        t0 = time.perf_counter()
        timing = {}
        prompts = self.make_prompts(num_prompts, seed=1000 * self.step_count + self.dp_rank).repeat(self.n)
        tg = time.perf_counter()
        out = self.rollout.generate(prompts, seed=self.step_count)
        rewards = hash_token_reward(out, seed=7).to(self.device)
        adv = group_normalize(rewards, out.non_tensor_batch["uid"], global_std=False)
        mask = out.batch["response_mask"].to(self.device)
        self._sync()
        timing["gen"] = time.perf_counter() - tg
        tg = time.perf_counter()
        slices = self._micro(out)
        with torch.no_grad():
            old = torch.cat([self._resp_logprobs(out.select_idxs(sl)) for sl in slices], 0)
        self._sync()
        timing["old_log_prob"] = time.perf_counter() - tg
        tg = time.perf_counter()
        self.engine.train_mode()
        self.engine.zero_grad()
        # each micro-batch's token-mean (sequence-mean for GSPO) is weighted by its share of the batch, so the
        # accumulated gradient is that of the whole batch's mean
        seq_level = self.loss_mode == "gspo"
        total = float(mask.shape[0]) if seq_level else float(mask.sum().clamp_min(1))
        losses, ms = [], []
        for sl in slices:
            logp = self._resp_logprobs(out.select_idxs(sl))
            mk = mask[sl]
            loss, m = self.loss_fn(logp, old[sl], adv[sl], mk)
            w = (mk.shape[0] if seq_level else float(mk.sum().clamp_min(1))) / total
            (loss * (w * self.tp_size)).backward()
            losses.append(loss.detach() * w)
            ms.append(m)
        norm = self.engine.optimizer_step()
        self._sync()
        timing["update_actor"] = time.perf_counter() - tg
        m = {k: float(np.mean([x[k] for x in ms])) for k in ms[0]}
        m.update({"actor/pg_loss": float(torch.stack(losses).sum()), "actor/grad_norm": float(norm.reshape(())),
                  "actor/lr": self.engine.lr(), "critic/rewards/mean": float(rewards.mean()),
                  "training/global_step": self.step_count,
                  "response_length/mean": float(mask.sum(-1).mean()),
                  "rollout_corr/logprob_abs_diff_mean": float(((old - out.batch["rollout_log_probs"].to(self.device))
                                                               .abs() * mask).sum() / mask.sum())})
        m.update(M.compute_timing_metrics_diffusion(timing, len(out)))
        m.update(M.compute_throughput_metrics_diffusion(time.perf_counter() - t0, len(out) * self.dp,
                                                         D.world_size()))
        m.update(self._mfu(out, timing))
        return m

    # ------------------------------------------------------------------ pipeline parallel step
    def _stage_fn(self, data: DataProto, slices, with_loss: bool, old=None, adv=None, mask=None, total=None,
                  store=None):
        """This stage's computation of micro-batch ``i``: the first stage embeds the prompt + response ids
        (and the multimodal features), every stage runs its layers, the last computes the response
        log-probs (and, ``with_loss``, the weighted policy loss)."""
        st = self.model
        ids = data.batch["input_ids"].to(self.device)
        P = data.batch["prompts"].shape[1]
        af, ip = self._feats(data)
        seq_level = self.loss_mode == "gspo"

        def fn(x, i):
            sl = slices[i]
            tgt = None
            if st.last:
                tgt = torch.zeros_like(ids[sl, :-1])
                tgt[:, P - 1:] = ids[sl, P:]
            if st.first:
                x = ids[sl, :-1]
            y = st(x, audio_feats=af[sl] if (st.first and af is not None) else None,
                   image_patches=ip[sl] if (st.first and ip is not None) else None,
                   targets=tgt, temperature=self.temperature)
            if not st.last:
                return y
            lp = y[:, P - 1:]
            if not with_loss:
                return lp
            mk = mask[sl]
            loss, m = self.loss_fn(lp, old[i], adv[sl], mk)
            w = (mk.shape[0] if seq_level else float(mk.sum().clamp_min(1))) / total
            store.append(m)
            return loss * w

        return fn

    def _step_pp(self, num_prompts: int) -> dict:
        """The GRPO / GSPO step with the model split into pipeline stages: pipelined decode, forward-only
        old log-probs over the stages, 1F1B update, one optimizer step per stage with the gradient norm of the
        whole model; the last stage's metrics are broadcast to the pipeline."""
        from verl_omni_b200.parallel.pipeline import PipelineStage

        self.step_count += 1
        t0 = time.perf_counter()
        timing = {}
        link = self.pp
        prompts = self.make_prompts(num_prompts, seed=1000 * self.step_count + self.dp_rank).repeat(self.n)
        tg = time.perf_counter()
        out = self.rollout.generate(prompts, seed=self.step_count)
        rewards = hash_token_reward(out, seed=7).to(self.device)
        adv = group_normalize(rewards, out.non_tensor_batch["uid"], global_std=False)
        mask = out.batch["response_mask"].to(self.device)
        self._sync()
        timing["gen"] = time.perf_counter() - tg
        slices = self._micro(out)
        Lm1 = out.batch["input_ids"].shape[1] - 1
        shape = lambda i: (slices[i].stop - slices[i].start, Lm1, self.cfg.hidden)
        stage = PipelineStage(None, link.s, link.S, link.ranks, shape, shape, self.engine.dtype, self.device)
        tg = time.perf_counter()
        old = stage.forward_only(len(slices), self._stage_fn(out, slices, False))
        self._sync()
        timing["old_log_prob"] = time.perf_counter() - tg
        tg = time.perf_counter()
        self.engine.train_mode()
        self.engine.zero_grad()
        seq_level = self.loss_mode == "gspo"
        total = float(mask.shape[0]) if seq_level else float(mask.sum().clamp_min(1))
        ms: list = []
        stage.fn = self._stage_fn(out, slices, True, old, adv, mask, total, ms)
        losses = stage.run(len(slices))
        norm = self.engine.optimizer_step()
        self._sync()
        timing["update_actor"] = time.perf_counter() - tg
        m = {}
        if link.last:
            m = {k: float(np.mean([x[k] for x in ms])) for k in ms[0]}
            oldc = torch.cat(old, 0)
            m.update({"actor/pg_loss": float(torch.stack(losses).sum()),
                      "rollout_corr/logprob_abs_diff_mean": float(
                          ((oldc - out.batch["rollout_log_probs"].to(self.device)).abs() * mask).sum() / mask.sum())})
        m = D.broadcast_object(m, src=link.ranks[-1], group=link.group)
        m.update({"actor/grad_norm": float(norm.reshape(())), "actor/lr": self.engine.lr(),
                  "critic/rewards/mean": float(rewards.mean()), "training/global_step": self.step_count,
                  "response_length/mean": float(mask.sum(-1).mean())})
        m.update(M.compute_timing_metrics_diffusion(timing, len(out)))
        m.update(M.compute_throughput_metrics_diffusion(time.perf_counter() - t0, len(out) * self.dp,
                                                         D.world_size()))
        m.update(self._mfu(out, timing))
        return m

    def _mfu(self, out: DataProto, timing: dict) -> dict:
        """``perf/mfu/*`` of the step: the language model's FLOPs over every data-parallel rank's sequences."""
        from verl_omni_b200.utils.mfu import omni_step_mfu_metrics

        return omni_step_mfu_metrics(self.cfg, batch=len(out) * self.dp, seq=int(out.batch["input_ids"].shape[1]),
                                     timing=timing, n_gpus=D.world_size())

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ checkpoint / resume
    def save_checkpoint(self, root_dir: str) -> str:
        """``{root_dir}/global_step_{N}/actor`` (engine shards, expert slices) + ``data.pt`` +
        ``latest_checkpointed_iteration.txt`` -- the diffusion trainers' layout."""
        import os

        root = os.path.join(root_dir, f"global_step_{self.step_count}")
        contents = tuple(self.actor_cfg.checkpoint.save_contents)
        self.engine.save_checkpoint(self._actor_dir(root), self.step_count,
                                    tuple(c for c in contents if c != "hf_model"))
        if "hf_model" in contents:
            self.export_hf(os.path.join(root, "actor", "huggingface"))
        if D.rank() == 0:
            torch.save({"global_step": self.step_count}, os.path.join(root, "data.pt"))
            with open(os.path.join(root_dir, "latest_checkpointed_iteration.txt"), "w") as f:
                f.write(str(self.step_count))
        D.barrier()
        return root

    def export_hf(self, directory: str) -> None:
        """The thinker's language model in the HF hub layout (bf16 safetensors, ``thinker.`` names, one tensor
        per expert).  Ranks write disjoint files: the first rank of each pipeline stage its dense tensors,
        the first rank of each expert data-parallel group its experts; together they form one checkpoint."""
        import os

        from safetensors.torch import save_file

        from verl_omni_b200.models.hf_omni_io import thinker_to_hf

        os.makedirs(directory, exist_ok=True)
        stage = self.pp.s if self.pp is not None else 0
        off = self.model.lo if self.pp is not None else 0
        first_of_stage = D.rank() % self.dp == 0 if self.pp is not None else D.rank() == 0
        first_expert_holder = self.expert_dp_group is None and first_of_stage or (
            self.expert_dp_group is not None and D.rank(self.expert_dp_group) == 0)
        named = {}
        for n, p in self.model.named_parameters():
            is_expert = n.endswith(("w_gate_up", "w_down"))
            if (first_expert_holder if is_expert else first_of_stage):
                named[n] = p
        state = {k: v.detach().to(torch.bfloat16).cpu().contiguous()
                 for k, v in thinker_to_hf(named, self.model, off).items()}
        if state:
            save_file(state, os.path.join(directory, f"model-stage{stage:02d}-rank{D.rank():05d}.safetensors"))
        D.barrier()

    def _actor_dir(self, root: str) -> str:
        """``actor`` (``actor/pp_rank_{s:02d}`` per stage under pipeline parallelism: each stage's shards)."""
        import os

        d = os.path.join(root, "actor")
        return d if self.pp is None else os.path.join(d, f"pp_rank_{self.pp.s:02d}")

    def load_checkpoint(self, root_dir: str) -> bool:
        import os

        marker = os.path.join(root_dir, "latest_checkpointed_iteration.txt")
        if not os.path.exists(marker):
            return False
        with open(marker) as f:
            root = os.path.join(root_dir, f"global_step_{int(f.read().strip())}")
        self.engine.load_checkpoint(self._actor_dir(root))
        self.step_count = int(torch.load(os.path.join(root, "data.pt"))["global_step"])
        return True

    def dpo_step(self, chosen: DataProto, rejected: DataProto, ref_model: MoELLM, beta: float = 0.1) -> dict:
        """Offline omni DPO on (chosen, rejected) response pairs against a frozen reference."""
        def seqlp(model, d):
            ids = d.batch["input_ids"].to(self.device)
            P = d.batch["prompts"].shape[1]
            tgt = torch.zeros_like(ids[:, :-1])
            tgt[:, P - 1:] = ids[:, P:]
            af, ip = self._feats(d)
            lp = model(ids[:, :-1], audio_feats=af, image_patches=ip, targets=tgt)[:, P - 1:]
            return sequence_logps(lp, d.batch["response_mask"].to(self.device))

        with torch.no_grad():
            rc, rr = seqlp(ref_model, chosen), seqlp(ref_model, rejected)
        self.engine.zero_grad()
        loss, m = omni_dpo_loss(seqlp(self.model, chosen), seqlp(self.model, rejected), rc, rr, beta=beta)
        loss.backward()
        self.engine.optimizer_step()
        return m
