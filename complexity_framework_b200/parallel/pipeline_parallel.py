"""Pipeline parallelism with a working 1F1B (or GPipe) schedule.

Each rank of the pipeline group keeps a contiguous slice of decoder layers;
the first stage owns the token embedding, the last stage the final norm, the
(tied) output projection and the loss.  Activations ``[mb, S, H]`` and their
gradients move between neighbouring stages with point-to-point send/recv
(NCCL on GPUs, gloo on CPU), posted as batched isend/irecv pairs so adjacent
stages never deadlock.  With tied embeddings the last stage holds a copy of
the embedding matrix and the two copies' gradients are summed over an
embedding group after backward, so both stay identical.

The reference's hand-written schedules never communicate and run backward
on the last stage only (complexity/parallel/pipeline_parallel.py:176-365); the names ``PipelineStage``, ``PipelineModel``,
``split_model_for_pipeline`` and ``PipelineScheduler`` are kept.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn


def split_model_for_pipeline(num_layers: int, num_stages: int) -> List[Tuple[int, int]]:
    """Contiguous [start, end) layer ranges, earlier stages get the extra layers."""
    if num_stages < 1 or num_stages > num_layers:
        raise ValueError("need 1 <= num_stages <= num_layers")
    base, extra = divmod(num_layers, num_stages)
    out, s = [], 0
    for i in range(num_stages):
        n = base + (1 if i < extra else 0)
        out.append((s, s + n))
        s += n
    return out


class PipelineStage(nn.Module):
    """One stage: optional embedding, a slice of blocks, optional norm + LM head."""

    def __init__(self, model, start: int, end: int, first: bool, last: bool):
        super().__init__()
        self.config = model.config
        self.first, self.last = first, last
        self.start, self.end = start, end
        self.layers = nn.ModuleList(list(model.layers)[start:end])
        self.embed_tokens = model.embed_tokens if first else None
        self.norm = model.norm if last else None
        self.lm_head = None
        self.head_weight = None
        if last:
            if model.lm_head is not None:
                self.lm_head = model.lm_head
            elif not first:
                # tied output projection: a copy kept in sync through the embedding group
                self.head_weight = nn.Parameter(model.embed_tokens.weight.detach().clone())
        self._model = [model]  # for embed()/logits helpers, not registered as a child

    def output_weight(self):
        if self.lm_head is not None:
            return self.lm_head.weight
        if self.head_weight is not None:
            return self.head_weight
        return self.embed_tokens.weight

    def forward(self, x: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
        if self.first:
            x = self._model[0].embed(token_ids)
        for layer in self.layers:
            x, _, _ = layer(x, token_ids=token_ids)
        if self.last:
            x = self.norm(x)
        return x

    def loss(self, hidden: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
        from ..core.losses import causal_lm_loss_from_hidden

        labels = torch.roll(token_ids, -1, dims=1)
        labels[:, -1] = -100
        return causal_lm_loss_from_hidden(hidden, self.output_weight(), labels)


class PipelineModel(nn.Module):
    """The stage of ``model`` owned by this rank of ``group`` plus its schedule."""

    def __init__(self, model, group=None, num_stages: Optional[int] = None,
                 schedule: str = "1f1b"):
        super().__init__()
        self.group = group
        self.num_stages = num_stages or dist.get_world_size(group)
        self.stage_id = dist.get_rank(group)
        ranges = split_model_for_pipeline(model.config.num_hidden_layers, self.num_stages)
        s, e = ranges[self.stage_id]
        self.first = self.stage_id == 0
        self.last = self.stage_id == self.num_stages - 1
        self.stage = PipelineStage(model, s, e, self.first, self.last)
        self.schedule = schedule
        ranks = [dist.get_global_rank(group, i) if group is not None else i
                 for i in range(self.num_stages)]
        self.prev = ranks[self.stage_id - 1] if not self.first else None
        self.next = ranks[self.stage_id + 1] if not self.last else None
        self.tied = model.lm_head is None and self.num_stages > 1
        self.embedding_group = None
        if self.tied:
            # every rank must create the group, members or not
            self.embedding_group = dist.new_group([ranks[0], ranks[-1]])
        self.config = model.config

    # ---------------------------------------------------------------- p2p
    def _p2p(self, send: Optional[Tuple[torch.Tensor, int]], recv: Optional[Tuple[torch.Tensor, int]]):
        ops = []
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send[0].contiguous(), send[1]))
        if recv is not None:
            ops.append(dist.P2POp(dist.irecv, recv[0], recv[1]))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()

    # ------------------------------------------------------------ schedule
    def train_step(self, micro_batches: Sequence[torch.Tensor]) -> Optional[torch.Tensor]:
        """Forward + backward over micro-batches; returns the mean loss on the last stage."""
        M = len(micro_batches)
        P, s = self.num_stages, self.stage_id
        H = self.config.hidden_size
        dtype = next(self.stage.parameters()).dtype
        mb_shape = (*micro_batches[0].shape, H)
        dev = micro_batches[0].device
        inputs: List[Optional[torch.Tensor]] = [None] * M
        outputs: List[Optional[torch.Tensor]] = [None] * M
        losses: List[torch.Tensor] = []
        first, last = self.first, self.last

        def buf():
            return torch.empty(mb_shape, device=dev, dtype=dtype)

        def run_fwd(i: int, x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
            ids = micro_batches[i]
            if x is not None:
                x.requires_grad_(True)
            y = self.stage(x, ids)
            inputs[i] = x
            if last:
                loss = self.stage.loss(y, ids) / M
                outputs[i] = loss
                losses.append(loss.detach())
                return None
            outputs[i] = y
            return y.detach()

        def run_bwd(i: int, g: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
            if last:
                outputs[i].backward()
            else:
                outputs[i].backward(g)
            gin = None if first else inputs[i].grad
            inputs[i] = outputs[i] = None
            return gin

        def recv_fwd():
            if first:
                return None
            x = buf()
            self._p2p(None, (x, self.prev))
            return x

        def send_fwd(y):
            if not last:
                self._p2p((y, self.next), None)

        def send_fwd_recv_bwd(y):
            if last:
                return None
            g = buf()
            self._p2p((y, self.next), (g, self.next))
            return g

        def send_bwd_recv_fwd(gin):
            if first:
                return None
            x = buf()
            self._p2p((gin, self.prev), (x, self.prev))
            return x

        def send_bwd(gin):
            if not first:
                self._p2p((gin, self.prev), None)

        def recv_bwd():
            if last:
                return None
            g = buf()
            self._p2p(None, (g, self.next))
            return g

        if self.schedule == "gpipe":
            for i in range(M):
                send_fwd(run_fwd(i, recv_fwd()))
            for i in range(M):
                send_bwd(run_bwd(i, recv_bwd()))
        else:
            # 1F1B: neighbouring stages exchange the next activation and the
            # pending gradient in one batched send/recv, so no pair of blocking
            # sends can wait on each other.
            warm = min(P - s - 1, M)
            for i in range(warm):
                send_fwd(run_fwd(i, recv_fwd()))
            remaining = M - warm
            x = recv_fwd() if remaining > 0 else None
            for i in range(remaining):
                y = run_fwd(i + warm, x)
                g = send_fwd_recv_bwd(y)
                gin = run_bwd(i, g)
                if i == remaining - 1:
                    send_bwd(gin)
                else:
                    x = send_bwd_recv_fwd(gin)
            for i in range(remaining, M):
                send_bwd(run_bwd(i, recv_bwd()))
        self.sync_tied_embedding_grads()
        return torch.stack(losses).sum() if losses else None

    def sync_tied_embedding_grads(self) -> None:
        if not self.tied or not (self.first or self.last):
            return
        w = self.stage.embed_tokens.weight if self.first else self.stage.head_weight
        if w.grad is None:
            w.grad = torch.zeros_like(w)
        dist.all_reduce(w.grad, group=self.embedding_group)


class PipelineScheduler:
    """Name kept from the reference: runs ``PipelineModel.train_step``."""

    def __init__(self, pipeline: PipelineModel, schedule: str = "1f1b"):
        self.pipeline = pipeline
        pipeline.schedule = schedule

    def run(self, micro_batches):
        return self.pipeline.train_step(micro_batches)


# --------------------------------------------------- reference helper names
from dataclasses import dataclass as _dataclass  # noqa: E402
from enum import Enum as _Enum  # noqa: E402


class PipelineSchedule(_Enum):
    GPIPE = "gpipe"
    ONE_F_ONE_B = "1f1b"
    INTERLEAVED = "interleaved"


@_dataclass
class PipelineConfig:
    """Stages, micro-batches per step and schedule (complexity/parallel/
    pipeline_parallel.py:26-38).  ``INTERLEAVED`` (virtual stages) is not built:
    the export-based pipeline (``parallel/pipeline_export.py``) is the
    alternative for finer stage splits."""
    num_stages: int
    num_micro_batches: int = 4
    schedule: PipelineSchedule = PipelineSchedule.ONE_F_ONE_B

    def __post_init__(self):
        self.schedule = PipelineSchedule(self.schedule)
        if self.schedule is PipelineSchedule.INTERLEAVED:
            raise ValueError("interleaved (virtual-stage) schedules are not built; use gpipe "
                             "or 1f1b")


def get_pipeline_parallel_rank(group=None) -> int:
    return dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0


def get_pipeline_parallel_world_size(group=None) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def send_forward(tensor: torch.Tensor, next_rank: int, group=None) -> None:
    """Activation to the next stage (NCCL / gloo point-to-point)."""
    if dist.is_available() and dist.is_initialized():
        dist.send(tensor.contiguous(), next_rank, group=group)


def recv_forward(tensor_shape, dtype: torch.dtype, prev_rank: int, device,
                 group=None) -> torch.Tensor:
    t = torch.zeros(tuple(tensor_shape), dtype=dtype, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.recv(t, prev_rank, group=group)
    return t


def send_backward(tensor: torch.Tensor, prev_rank: int, group=None) -> None:
    """Activation gradient to the previous stage."""
    if dist.is_available() and dist.is_initialized():
        dist.send(tensor.contiguous(), prev_rank, group=group)


def recv_backward(tensor_shape, dtype: torch.dtype, next_rank: int, device,
                  group=None) -> torch.Tensor:
    t = torch.zeros(tuple(tensor_shape), dtype=dtype, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.recv(t, next_rank, group=group)
    return t
