"""One training step as a replayed CUDA graph.

The reference trainer launches every kernel of a step from Python
(complexity/training/trainer.py:196-334); with ~750 launches per 200M step
that host work is a measurable share of the step.  ``GraphedTrainStep``
runs the first ``cuda_graph_warmup`` steps eagerly (the last ones on a side
stream, so library handles and workspaces exist before capture), then
captures forward, backward, gradient gather, norm clipping, the fused AdamW
update and ``zero_grad`` in one CUDA graph and replays it for every later
step.  Per step the host only refreshes the static input, writes the
optimizer's device hyper-parameters (learning rate and bias corrections of
the upcoming step, see ``FusedAdamW.enable_device_hyper``), replays, and does
the Python bookkeeping (step counters, lr scheduler).

Eligibility: the flat fused AdamW on CUDA and fixed input shapes, in one
process or data-parallel on the fused NVLink reduce + AdamW kernels (their
barrier epochs and hyper-parameters live on the device, so every replay
advances them on all ranks alike).  Tensor/expert-parallel steps and the NCCL
data-parallel path run eagerly.
"""
from __future__ import annotations

from typing import Optional

import torch


class GraphedTrainStep:
    def __init__(self, trainer):
        self.tr = trainer
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.calls = 0
        self.ids = None
        self.labels = None
        self.loss = None
        self.shape = None
        self._side = None

    # ------------------------------------------------------------ eligibility
    def reason_ineligible(self) -> Optional[str]:
        from .optim import FusedAdamW

        tr = self.tr
        if not torch.cuda.is_available():
            return "no CUDA device"
        opt = tr.optimizer
        if not isinstance(opt, FusedAdamW) or not opt._use_kernels():
            return "needs the fused AdamW kernels"
        if tr.sp_ws is not None or getattr(tr.model, "ep", None) is not None:
            return "tensor/expert-parallel step (their barriers count epochs on the host)"
        if tr.world > 1 and opt._fused is None:
            return "multi-process step on NCCL collectives (only the fused NVLink path replays)"
        return None

    # ----------------------------------------------------------------- body
    def _body(self, ids: torch.Tensor, labels: Optional[torch.Tensor]) -> torch.Tensor:
        tr = self.tr
        opt = tr.optimizer
        loss = tr.compute_loss(ids, labels)
        loss.backward()
        opt.reduce_gradients()
        clip = tr.config.grad_clip > 0
        if clip:
            opt.clip_grad_norm_(tr.config.grad_clip)
        opt.step(clip=clip)
        opt.zero_grad()
        return loss.detach()

    def _eager(self, input_ids, labels, side: bool):
        tr = self.tr
        if not side:
            return tr._train_step_eager(input_ids, labels, sync=False)
        if self._side is None:
            self._side = torch.cuda.Stream()
        cur = torch.cuda.current_stream()
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            out = tr._train_step_eager(input_ids, labels, sync=False)
        cur.wait_stream(self._side)
        return out

    def _capture(self, input_ids, labels) -> None:
        tr = self.tr
        opt = tr.optimizer
        dev = next(tr.model.parameters()).device
        self.shape = tuple(input_ids.shape)
        self.ids = torch.empty(self.shape, dtype=input_ids.dtype, device=dev)
        self.ids.copy_(input_ids, non_blocking=True)
        if labels is not None:
            self.labels = torch.empty(tuple(labels.shape), dtype=labels.dtype, device=dev)
            self.labels.copy_(labels, non_blocking=True)
        opt.enable_device_hyper()
        opt.write_hyper(opt._step_count + 1)
        tr.model.train()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            # Python side effects of this pass (optimizer step count, state
            # "step" entries) are this step's bookkeeping; the kernels run at
            # the replay below
            self.loss = self._body(self.ids, self.labels)
        self.graph = g
        g.replay()

    # ------------------------------------------------------------------ call
    def __call__(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None):
        tr = self.tr
        warm = max(1, int(tr.config.cuda_graph_warmup))
        if self.graph is None and (self.calls < warm or self.reason_ineligible() is not None):
            self.calls += 1
            return self._eager(input_ids, labels, side=self.calls > 1 and
                               self.reason_ineligible() is None)
        if self.graph is None:
            self._capture(input_ids, labels)
        else:
            if tuple(input_ids.shape) != self.shape:
                raise ValueError(f"CUDA-graph step captured for input shape {self.shape}, "
                                 f"got {tuple(input_ids.shape)}")
            if (labels is None) != (self.labels is None):
                raise ValueError("CUDA-graph step: labels must be given on every step or never")
            opt = tr.optimizer
            t = opt._step_count + 1
            self.ids.copy_(input_ids, non_blocking=True)
            if labels is not None:
                self.labels.copy_(labels, non_blocking=True)
            opt.write_hyper(t)
            self.graph.replay()
            opt.finish_replayed_step(t)
        tr.scheduler.step()
        tr.global_step += 1
        tr.total_tokens += input_ids.numel() * tr.world
        self.calls += 1
        return self.loss
