"""Trainer: one process per GPU, flat fp32-master AdamW, fused loss.

A training step is: H2D of the micro-batch (pinned, non-blocking) -> forward
through the sm_100a kernels -> fused linear cross-entropy -> backward ->
data-parallel gradient reduction over the flat gradient buffers (all-reduce
for ``ddp``, reduce-scatter + sharded update + all-gather for ``fsdp``) ->
device-side grad-norm clip -> one fused AdamW launch per parameter group.

Public surface follows complexity/training/trainer.py:42-774 (``Trainer``,
``train``, ``evaluate``, checkpoint save/resume, the canary parameter-update
check after the first step) with a flat-buffer optimizer in place of
per-parameter loops.
"""
from __future__ import annotations

import logging
import time
from typing import Callable, Iterable, List, Optional

import torch
import torch.distributed as dist

from ..utils.checkpointing import CheckpointManager
from .config import TrainingConfig
from .optim import FusedAdamW, default_param_groups
from .scheduler import build_scheduler

logger = logging.getLogger(__name__)


def _singleton_group(group):
    """A process group holding only this rank (collective: every rank of ``group`` calls it)."""
    mine = None
    me = dist.get_rank()
    for r in dist.get_process_group_ranks(group):
        g = dist.new_group([r])
        if r == me:
            mine = g
    return mine


class Trainer:
    def __init__(self, model: torch.nn.Module, config: Optional[TrainingConfig] = None, *,
                 device: Optional[torch.device] = None, process_group=None,
                 callbacks: Optional[List] = None, compute_loss: Optional[Callable] = None):
        self.config = config or TrainingConfig()
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(process_group) if on else 1
        self.rank = dist.get_rank(process_group) if on else 0
        self.is_main = self.rank == 0
        if device is None:
            device = (torch.device("cuda", torch.cuda.current_device())
                      if torch.cuda.is_available() else torch.device("cpu"))
        self.device = torch.device(device)
        dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[
            self.config.precision]
        if self.device.type == "cpu":
            dtype = torch.float32
        self.model = model.to(device=self.device, dtype=dtype)
        mode = self.config.distributed_mode
        if mode == "auto":
            tagged = getattr(self.model, "dp_mode", None)  # set by wrap_model_fsdp / simple_ddp
            mode = ((tagged or ("fsdp" if self.config.use_fsdp else "ddp"))
                    if self.world > 1 else "none")
        self.distributed_mode = mode
        self.sp_ws = getattr(self.model, "sp_ws", None)
        if self.sp_ws is not None:
            # fused sequence-parallel TP: every rank of the group owns different
            # parameter shards; only replicated parameters are reduced (below),
            # so the optimizer works rank-locally
            process_group = _singleton_group(self.sp_ws.group)
            self.world, self.rank = 1, 0
            mode = "none"
        if self.world > 1:
            self._broadcast_parameters(process_group)
        self.zero3 = None
        if mode == "zero3":
            # parameters, gradients' owners and optimizer state sharded per block
            from ..parallel.fsdp import ShardedModel

            if self.world == 1:
                mode = "none"
            else:
                self.zero3 = ShardedModel(self.model, process_group)
        self.distributed_mode = mode
        self.optimizer = self._build_optimizer(process_group, mode)
        sched_opt = getattr(self.optimizer, "optimizer", self.optimizer)
        self.scheduler = build_scheduler(sched_opt, kind=self.config.lr_scheduler,
                                         warmup_steps=self.config.warmup_steps,
                                         total_steps=self.config.max_steps,
                                         min_lr_ratio=self.config.min_lr_ratio,
                                         wsd_decay_ratio=self.config.wsd_decay_ratio)
        self.ckpt = CheckpointManager(self.config.checkpoint_dir, self.config.save_total_limit)
        self.callbacks = list(callbacks or [])
        self.global_step = 0
        self.epoch = 0
        self.total_tokens = 0
        self.best_loss = float("inf")
        self._compute_loss = compute_loss
        self._graphed = None
        self._canary = None
        self.should_stop = False

    # ----------------------------------------------------------------- setup
    def _build_optimizer(self, process_group, mode: str):
        """``adamw`` -> the flat fused AdamW (ZeRO-2 sharded under fsdp); any other
        ``optimizer_type`` (muon, muon_tr, adam_tr, lion, sophia, adam8bit, came,
        adalomo, musgd, adam, sgd) -> that optimizer behind a bucketed all-reduce."""
        cfg = self.config
        kind = cfg.optimizer_type.lower()
        if mode == "zero3":
            from ..parallel.fsdp import Zero3AdamW

            if kind != "adamw":
                raise ValueError("zero3 sharding supports the adamw optimizer")
            return Zero3AdamW(self.zero3, lr=cfg.learning_rate, betas=(0.9, 0.95),
                              weight_decay=cfg.weight_decay)
        if kind == "adamw":
            groups = default_param_groups(self.model, cfg.weight_decay)
            return FusedAdamW(groups, lr=cfg.learning_rate, betas=(0.9, 0.95),
                              weight_decay=cfg.weight_decay, process_group=process_group,
                              shard_state=(mode == "fsdp"))
        from .optimizers import DistributedOptimizer, get_optimizer

        kw = {}
        if kind in ("muon", "muon_tr"):
            kw["muon_lr"] = cfg.muon_lr
        if kind in ("muon_tr", "adam_tr"):
            mc = getattr(self.model, "config", None)
            kw["num_experts"] = int(getattr(mc, "num_experts", 4) or 4)
        if kind == "adam_tr":
            kw["expert_lr_scale"] = cfg.expert_lr_scale
            kw["expert_weight_decay"] = cfg.expert_weight_decay
        if kind == "muon_tr":
            kw["adaptive_ns"] = cfg.adaptive_ns
        opt = get_optimizer(self.model, kind, lr=cfg.learning_rate,
                            weight_decay=cfg.weight_decay, **kw)
        return DistributedOptimizer(opt, process_group)

    @torch.no_grad()
    def _broadcast_parameters(self, pg) -> None:
        src = dist.get_global_rank(pg, 0) if pg is not None else 0
        for p in self.model.parameters():
            if getattr(p, "_ep_local", False):
                continue  # expert-parallel shard: each rank owns different experts
            dist.broadcast(p.data, src=src, group=pg)
        for b in self.model.buffers():
            if b.is_floating_point():
                dist.broadcast(b, src=src, group=pg)

    # ------------------------------------------------------------------ step
    def compute_loss(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None):
        if self._compute_loss is not None:
            return self._compute_loss(self.model, input_ids, labels)
        return self.model.loss(input_ids, labels)

    def train_step(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None, *,
                   sync: bool = True):
        """One optimizer step on one micro-batch.

        ``input_ids`` may live on the host (pinned memory is copied
        asynchronously).  Returns the loss as a Python float when ``sync``
        (one device-to-host read), else the detached device scalar.  With
        ``config.cuda_graph`` the step is replayed from a captured CUDA graph
        after the warm-up steps (``training/graph_step.py``); the returned
        device scalar is then overwritten by the next step.
        """
        if self.config.cuda_graph and not isinstance(input_ids, dict):
            if self._graphed is None:
                from .graph_step import GraphedTrainStep

                self._graphed = GraphedTrainStep(self)
            out = self._graphed(input_ids, labels)
            return float(out) if sync else out
        return self._train_step_eager(input_ids, labels, sync=sync)

    def _train_step_eager(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None, *,
                          sync: bool = True):
        self.model.train()
        if isinstance(input_ids, dict):
            # structured batch (e.g. contrastive pairs): tensors moved as a whole,
            # the loss callable receives the dict
            ids = {k: (v.to(self.device, non_blocking=True) if torch.is_tensor(v) else v)
                   for k, v in input_ids.items()}
            n_tok = sum(int(v.numel()) for k, v in ids.items()
                        if k.endswith("input_ids") and torch.is_tensor(v))
            lab = None
        else:
            ids = input_ids.to(self.device, non_blocking=True)
            lab = labels.to(self.device, non_blocking=True) if labels is not None else None
            n_tok = ids.numel()
        loss = self.compute_loss(ids, lab)
        loss.backward()
        self._finish_step()
        self.total_tokens += n_tok * self.world
        out = loss.detach()
        if self.sp_ws is not None:
            # each TP rank returned its share of the global mean loss
            out = out.float().clone()
            dist.all_reduce(out, group=self.sp_ws.group)
        return float(out) if sync else out

    def accumulate_step(self, micro_batches: Iterable[torch.Tensor], *, sync: bool = True):
        """Gradient accumulation over micro-batches, one optimizer step at the end."""
        self.model.train()
        batches = list(micro_batches)
        total = None
        n = 0
        for mb in batches:
            ids = mb.to(self.device, non_blocking=True)
            loss = self.compute_loss(ids) / len(batches)
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
            n += ids.numel()
        self._finish_step()
        self.total_tokens += n * self.world
        return float(total) if sync else total

    def _finish_step(self) -> None:
        opt = self.optimizer
        check = (self.global_step == 0 and not self.config.skip_param_update_check)
        if check:
            self._canary = self._snapshot()
        if self.sp_ws is not None:
            from ..parallel.tp_fused import allreduce_replicated_grads

            if hasattr(opt, "_gather_grads"):
                opt._gather_grads()  # bind the fresh gradients to the flat buffers first
            allreduce_replicated_grads(self.model)
        opt.reduce_gradients()
        clip = self.config.grad_clip > 0
        if clip:
            opt.clip_grad_norm_(self.config.grad_clip)
        opt.step(clip=clip)
        self.scheduler.step()
        opt.zero_grad()
        self.global_step += 1
        if check:
            self._verify_canary()

    # ------------------------------------------------- canary update check
    def _snapshot(self):
        if self.zero3 is not None:  # parameters live in per-rank shards between steps
            us = self.zero3.all_units()
            return [(u.shard_buf, u.shard_buf.reshape(-1)[:64].clone())
                    for u in (us[0], us[len(us) // 2], us[-1])]
        ps = [p for p in self.model.parameters() if p.requires_grad]
        picks = [ps[0], ps[len(ps) // 2], ps[-1]]
        return [(p, p.detach().reshape(-1)[:64].clone()) for p in picks]

    def _verify_canary(self) -> None:
        """After the first step at least one sampled parameter must have moved."""
        moved = any(not torch.equal(p.detach().reshape(-1)[:64], before)
                    for p, before in self._canary)
        self._canary = None
        if self.is_main:
            logger.info("canary param-update check: %s", "ok" if moved else "NO UPDATE")
        if not moved:
            raise RuntimeError("parameters did not change after the first optimizer step")

    # ------------------------------------------------------------------ loop
    @staticmethod
    def _split_batch(batch):
        if isinstance(batch, dict):
            if "input_ids" not in batch:
                return batch, None  # structured batch for a custom compute_loss
            return batch["input_ids"], batch.get("labels")
        if isinstance(batch, (tuple, list)):
            return batch[0], (batch[1] if len(batch) > 1 else None)
        return batch, None

    def _emit(self, hook: str, *args) -> None:
        for cb in self.callbacks:
            fn = getattr(cb, hook, None)
            if fn is not None:
                fn(self, *args)

    def train(self, batches: Iterable, max_steps: Optional[int] = None,
              eval_batches: Optional[Callable[[], Iterable]] = None) -> dict:
        """Run optimizer steps over an iterable of batches (``[B, S]`` token
        tensors, ``(input_ids, labels)`` pairs or dicts with those keys).

        ``eval_batches`` is a factory of evaluation iterables, used every
        ``eval_steps`` steps.  A callback may stop training early by setting
        ``trainer.should_stop``.
        """
        max_steps = max_steps or self.config.max_steps
        t0 = time.perf_counter()
        last = None
        self.should_stop = False
        self._emit("on_train_begin")
        try:
            for batch in batches:
                if self.global_step >= max_steps or self.should_stop:
                    break
                ids, labels = self._split_batch(batch)
                sync = (self.global_step % self.config.log_steps == 0)
                out = self.train_step(ids, labels, sync=sync)
                last_val = out if sync else None
                if last_val is not None:
                    last = last_val
                    self.best_loss = min(self.best_loss, last_val)
                self._emit("on_step_end", self.global_step, last_val)
                if (eval_batches is not None and self.config.eval_steps
                        and self.global_step % self.config.eval_steps == 0):
                    ev = self.evaluate(eval_batches())
                    self._emit("on_evaluate", self.global_step, ev)
                if self.global_step % self.config.save_steps == 0:
                    self.save_checkpoint()
        except KeyboardInterrupt:
            self.save_checkpoint(tag="interrupted")
            raise
        summary = {"steps": self.global_step, "tokens": self.total_tokens,
                   "seconds": time.perf_counter() - t0, "last_loss": last}
        self._emit("on_train_end", summary)
        return summary

    @torch.no_grad()
    def evaluate(self, batches: Iterable[torch.Tensor]) -> float:
        self.model.eval()
        tot = torch.zeros(2, device=self.device, dtype=torch.float64)
        for b in batches:
            ids, labels = self._split_batch(b)
            ids = ids.to(self.device, non_blocking=True)
            lab = labels.to(self.device, non_blocking=True) if labels is not None else None
            loss = self.compute_loss(ids, lab)
            tot[0] += loss.double() * ids.numel()
            tot[1] += ids.numel()
        if self.world > 1:
            dist.all_reduce(tot)
        self.model.train()
        return float(tot[0] / tot[1].clamp_min(1))

    # ----------------------------------------------------------- checkpoints
    def save_checkpoint(self, tag: str = "step"):
        return self.ckpt.save(self.model, self.optimizer, step=self.global_step,
                              scheduler=self.scheduler, epoch=self.epoch,
                              best_loss=self.best_loss, total_tokens=self.total_tokens, tag=tag)

    def resume(self, path: Optional[str] = "auto") -> bool:
        """Restore model/optimizer/scheduler/step from ``path`` or the newest checkpoint."""
        target = self.ckpt.latest() if path in (None, "auto") else path
        if target is None:
            return False
        state = self.ckpt.load(target, self.model, self.optimizer, self.scheduler)
        self.global_step = int(state["step"])
        self.epoch = int(state.get("epoch", 0))
        self.best_loss = float(state.get("best_loss", float("inf")))
        self.total_tokens = int(state.get("total_tokens", 0))
        return True
