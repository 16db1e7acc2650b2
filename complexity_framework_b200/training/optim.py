"""Flat-buffer AdamW with fp32 master weights.

Each param group is laid out in one contiguous buffer: the model parameters
become views into a flat compute buffer (bf16 on GPU), their ``.grad`` views
into a flat gradient buffer, and the optimizer keeps flat fp32 master weights
and moments.  A step is one sm_100a kernel launch per group (plus two tiny
launches for the gradient norm when clipping), never a per-parameter loop, and
needs no host synchronisation: the clip coefficient stays on the device.

Semantics are those of ``torch.optim.AdamW`` (decoupled weight decay applied
as ``p *= 1 - lr*wd``, bias-corrected moments, ``eps`` added to
``sqrt(v_hat)``), which the reference trainer uses with betas (0.9, 0.95)
(complexity/training/trainer.py:196-334).  Unlike the reference FSDP path
(parallel/data_parallel.py:105-108) the master weights and moments are fp32.

Sharded mode (``shard_state=True`` with a process group of W > 1 ranks) is
ZeRO-2: gradients are reduce-scattered into a per-rank shard, each rank
updates the fp32 master/moments of its shard only, and the bf16 compute
buffer is all-gathered.
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional

import torch


def default_param_groups(model: torch.nn.Module, weight_decay: float) -> List[dict]:
    """Decay / no-decay split by name, as the reference trainer does."""
    decay, no_decay, local = [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if getattr(p, "_ep_local", False):
            local.append(p)
        elif "bias" in name or "norm" in name or ".mu" in name:
            no_decay.append(p)
        else:
            decay.append(p)
    groups = [{"params": decay, "weight_decay": weight_decay}]
    if no_decay:
        groups.append({"params": no_decay, "weight_decay": 0.0})
    if local:
        # expert-parallel shards: owned by one rank, not averaged over data parallel
        groups.append({"params": local, "weight_decay": weight_decay, "dp_reduce": False})
    return groups


class _FlatGroup:
    """Flat storage of one parameter group (optionally with sharded optimizer state)."""

    def __init__(self, params: List[torch.nn.Parameter], compute_dtype: torch.dtype,
                 pad_to: int = 128, world: int = 1, rank: int = 0):
        self.params = params
        dev = params[0].device
        self.sizes = [p.numel() for p in params]
        self.offsets = []
        off = 0
        for n in self.sizes:
            self.offsets.append(off)
            off += (n + pad_to - 1) // pad_to * pad_to  # 256-byte aligned starts
        unit = pad_to * world
        off = (off + unit - 1) // unit * unit
        self.numel = off
        self.world, self.rank = world, rank
        self.shard = off // world
        self.lo = rank * self.shard
        self.compute = torch.zeros(off, device=dev, dtype=compute_dtype)
        self.grad = torch.zeros(off, device=dev, dtype=compute_dtype)
        with torch.no_grad():
            for p, o, n in zip(params, self.offsets, self.sizes):
                self.compute[o:o + n].copy_(p.detach().reshape(-1))
                # gradients that already exist (optimizer built after a backward)
                # move into the flat buffer instead of being dropped by rebind()
                if p.grad is not None:
                    self.grad[o:o + n].copy_(p.grad.reshape(-1))
            masters = torch.zeros(off, device=dev, dtype=torch.float32)
            for p, o, n in zip(params, self.offsets, self.sizes):
                masters[o:o + n].copy_(p.detach().reshape(-1).float())
        self.master = masters[self.lo:self.lo + self.shard].clone()
        del masters
        self.exp_avg = torch.zeros(self.shard, device=dev, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(self.shard, device=dev, dtype=torch.float32)
        self.grad_shard = (self.grad[self.lo:self.lo + self.shard] if world == 1 else
                           torch.zeros(self.shard, device=dev, dtype=compute_dtype))
        self.rebind()

    @property
    def compute_shard(self) -> torch.Tensor:
        return self.compute[self.lo:self.lo + self.shard]

    def rebind(self) -> None:
        """Point every parameter's data and grad at its slice of the flat buffers."""
        for p, o, n in zip(self.params, self.offsets, self.sizes):
            p.data = self.compute[o:o + n].view(p.shape)
            p.grad = self.grad[o:o + n].view(p.shape)

    def rebind_grads(self) -> None:
        for p, o, n in zip(self.params, self.offsets, self.sizes):
            p.grad = self.grad[o:o + n].view(p.shape)

    def view(self, flat: torch.Tensor, i: int) -> Optional[torch.Tensor]:
        """View of parameter i inside a full-length flat buffer, or inside a
        shard-length buffer when the parameter lies entirely in this shard."""
        o, n = self.offsets[i], self.sizes[i]
        if flat.numel() == self.numel:
            return flat[o:o + n].view(self.params[i].shape)
        if o >= self.lo and o + n <= self.lo + self.shard:
            return flat[o - self.lo:o - self.lo + n].view(self.params[i].shape)
        return None


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, compute_dtype: Optional[torch.dtype] = None,
                 process_group=None, shard_state: bool = False,
                 fused_collectives: Optional[bool] = None):
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        import torch.distributed as dist

        self.process_group = process_group
        self.world, self.rank = 1, 0
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(process_group)
            self.rank = dist.get_rank(process_group)
        self.sharded = bool(shard_state) and self.world > 1
        self._flat: List[Optional[_FlatGroup]] = []
        self._step_count = 0
        # gradients set on the parameters before the first zero_grad (assigned
        # tensors rather than the flat views) are gathered too
        self._gathered = False
        for group in self.param_groups:
            ps = [p for p in group["params"] if p.requires_grad]
            if not ps:
                self._flat.append(None)
                continue
            shard = self.sharded and group.get("dp_reduce", True)
            fg = _FlatGroup(ps, compute_dtype or ps[0].dtype,
                            world=self.world if shard else 1, rank=self.rank if shard else 0)
            fg.dp_reduce = group.get("dp_reduce", True)
            self._flat.append(fg)
            for i, p in enumerate(ps):
                st = {"step": torch.zeros((), dtype=torch.float32)}
                for key, buf in (("exp_avg", fg.exp_avg), ("exp_avg_sq", fg.exp_avg_sq),
                                 ("master", fg.master)):
                    v = fg.view(buf, i)
                    if v is not None:
                        st[key] = v
                self.state[p] = st
        dev = next((fg.master.device for fg in self._flat if fg is not None), torch.device("cpu"))
        self._sumsq = torch.zeros(1, device=dev, dtype=torch.float32)
        self._clip = torch.ones(1, device=dev, dtype=torch.float32)
        self._norm = torch.zeros(1, device=dev, dtype=torch.float32)
        self._sq_distinct = None
        self._max_norm = 0.0
        self._hyper = None  # device (lr, bc1, bc2) per flat group; see enable_device_hyper
        self._fused = None
        if fused_collectives is None:
            fused_collectives = os.environ.get("CFB_FUSED_DP", "1") != "0"
        if fused_collectives and self._fused_eligible():
            self._fused = _FusedDP(self)

    # ----------------------------------------------------------- flat access
    @property
    def flat_groups(self) -> List[_FlatGroup]:
        return [fg for fg in self._flat if fg is not None]

    def group_flat_grads(self) -> List[torch.Tensor]:
        return [fg.grad for fg in self.flat_groups]

    def zero_grad(self, set_to_none: bool = False) -> None:
        """Drop the gradient views: the next backward hands each parameter a fresh
        gradient tensor (no accumulate-add kernel per parameter), and
        ``_gather_grads`` copies them into the flat buffer with a few
        multi-tensor launches."""
        for fg in self.flat_groups:
            for p in fg.params:
                p.grad = None
        self._gathered = False

    @torch.no_grad()
    def _gather_grads(self) -> None:
        if self._gathered:
            return
        for fg in self.flat_groups:
            dst, src, missing = [], [], []
            for p, o, n in zip(fg.params, fg.offsets, fg.sizes):
                view = fg.grad[o:o + n].view(p.shape)
                g = p.grad
                if g is None:
                    missing.append(view)
                elif g.data_ptr() != view.data_ptr():
                    dst.append(view)
                    src.append(g)
            if dst:
                torch._foreach_copy_(dst, src)
            if missing:
                torch._foreach_zero_(missing)
            fg.rebind_grads()
        self._gathered = True

    @torch.no_grad()
    def reduce_gradients(self) -> None:
        """Average gradients over the data-parallel group (one collective per group)."""
        self._gather_grads()
        if self.world == 1 or self._fused is not None:
            return
        import torch.distributed as dist

        avg = dist.get_backend(self.process_group) == "nccl"
        op = dist.ReduceOp.AVG if avg else dist.ReduceOp.SUM
        for fg in self.flat_groups:
            if not fg.dp_reduce:
                # rank-local parameters (expert-parallel shards): loss is a mean
                # over this rank's tokens, the global loss a mean over ranks
                fg.grad.div_(self.world)
                continue
            if fg.world > 1:
                dist.reduce_scatter_tensor(fg.grad_shard, fg.grad, op=op, group=self.process_group)
                out = fg.grad_shard
            else:
                dist.all_reduce(fg.grad, op=op, group=self.process_group)
                out = fg.grad
            if not avg:
                out.div_(self.world)

    def _fused_eligible(self) -> bool:
        """NVLink-fused reduce + AdamW: sharded, NCCL, one GPU per rank, <= 8 ranks."""
        import torch.distributed as dist

        if not (self.sharded and 1 < self.world <= 8 and self._use_kernels()):
            return False
        if any(not (fg.dp_reduce and fg.world > 1) for fg in self.flat_groups):
            return False  # mixed replicated / rank-local groups use the NCCL path
        if dist.get_backend(self.process_group) != "nccl":
            return False
        from ..ops import require

        return hasattr(require(), "dp_reduce_shard")

    def _use_kernels(self) -> bool:
        fg = self.flat_groups[0] if self.flat_groups else None
        if fg is None or not fg.master.is_cuda or fg.compute.dtype != torch.bfloat16:
            return False
        from ..ops import available

        return available()

    # ------------------------------------------------------------- clipping
    def _allreduce_sumsq(self) -> None:
        """Sum the squared-norm partials of rank-distinct gradient pieces over ranks.

        Sharded groups and expert-parallel groups hold different elements on
        each rank; replicated groups (plain data parallel) hold identical
        gradients and are counted once.
        """
        if self.world == 1:
            return
        import torch.distributed as dist

        if self._sq_distinct is not None:
            dist.all_reduce(self._sq_distinct, op=dist.ReduceOp.SUM, group=self.process_group)
            self._sumsq.add_(self._sq_distinct)

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        """Compute the global grad norm on the device; the next ``step(clip=True)``
        scales by ``min(1, max_norm / (norm + 1e-6))``.  Returns the norm (no sync)."""
        self._max_norm = float(max_norm)
        self._gather_grads()
        if self._fused is not None:
            return self._norm[0]  # computed inside the fused reduce kernels during step()
        if self._use_kernels():
            from ..ops import require

            C = require()
            self._sumsq.zero_()
            self._sq_distinct = None if self.world == 1 else torch.zeros_like(self._sumsq)
            for fg in self.flat_groups:
                distinct = self.world > 1 and (fg.world > 1 or not fg.dp_reduce)
                C.sumsq_bf16(fg.grad_shard, self._sq_distinct if distinct else self._sumsq)
            self._allreduce_sumsq()
            C.clip_coef(self._sumsq, float(max_norm), self._clip, self._norm)
        else:
            self._sumsq.zero_()
            self._sq_distinct = None if self.world == 1 else torch.zeros_like(self._sumsq)
            for fg in self.flat_groups:
                distinct = self.world > 1 and (fg.world > 1 or not fg.dp_reduce)
                target = self._sq_distinct if distinct else self._sumsq
                target.add_((fg.grad_shard.float() ** 2).sum())
            self._allreduce_sumsq()
            self._norm.copy_(torch.sqrt(self._sumsq))
            if max_norm > 0:
                self._clip.copy_(torch.clamp(max_norm / (self._norm + 1e-6), max=1.0))
            else:
                self._clip.fill_(1.0)
        return self._norm[0]

    # ------------------------------------------------ device hyper-parameters
    def enable_device_hyper(self) -> None:
        """Make the AdamW kernels read (lr, bias corrections) from a device
        buffer, filled by ``write_hyper`` before each step, instead of launch
        arguments: a CUDA graph that captured ``step`` then follows the
        learning-rate schedule and the step count across replays."""
        if not self._use_kernels():
            raise RuntimeError("device hyper-parameters need the fused AdamW kernels")
        dev = self.flat_groups[0].master.device
        self._hyper = torch.zeros(len(self.param_groups), 3, device=dev, dtype=torch.float32)

    def write_hyper(self, t: int) -> None:
        """Fill the device buffer for step ``t`` from each group's current lr."""
        vals = []
        for group in self.param_groups:
            b1, b2 = group["betas"]
            vals.append([group["lr"], 1.0 - b1 ** t, 1.0 - b2 ** t])
        # pageable source: the copy is staged before this call returns, so the
        # host list may be rebuilt next step while earlier work is still queued
        self._hyper.copy_(torch.tensor(vals, dtype=torch.float32), non_blocking=True)

    def finish_replayed_step(self, t: int) -> None:
        """Host bookkeeping of a step whose kernels ran from a replayed graph."""
        self._step_count = t
        for fg in self.flat_groups:
            for p in fg.params:
                self.state[p]["step"].fill_(t)

    # ----------------------------------------------------------------- step
    @torch.no_grad()
    def step(self, closure=None, clip: bool = False):
        loss = closure() if closure is not None else None
        self._gather_grads()
        self._step_count += 1
        t = self._step_count
        if self._fused is not None:
            self._fused.step(t, self._max_norm if clip else 0.0)
            return loss
        kernels = self._use_kernels()
        if kernels:
            from ..ops import require

            C = require()
        for gi, (group, fg) in enumerate(zip(self.param_groups, self._flat)):
            if fg is None:
                continue
            b1, b2 = group["betas"]
            bc1 = 1.0 - b1 ** t
            bc2 = 1.0 - b2 ** t
            lr, wd, eps = group["lr"], group["weight_decay"], group["eps"]
            if kernels:
                C.adamw_flat(fg.master, fg.exp_avg, fg.exp_avg_sq, fg.grad_shard, fg.compute_shard,
                             lr, b1, b2, eps, wd, bc1, bc2, self._clip if clip else None,
                             None if self._hyper is None else self._hyper[gi])
            else:
                g = fg.grad_shard.float() * (self._clip if clip else 1.0)
                fg.exp_avg.mul_(b1).add_(g, alpha=1 - b1)
                fg.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
                fg.master.mul_(1 - lr * wd)
                denom = (fg.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
                fg.master.addcdiv_(fg.exp_avg, denom, value=-lr / bc1)
                fg.compute_shard.copy_(fg.master)
            if fg.world > 1:
                import torch.distributed as dist

                dist.all_gather_into_tensor(fg.compute, fg.compute_shard,
                                            group=self.process_group)
            for p in fg.params:
                self.state[p]["step"].fill_(t)
        return loss

    # ------------------------------------------------------------ state dict
    def state_dict(self) -> Dict:
        sd = super().state_dict()
        sd["flat_step"] = self._step_count
        return sd

    def load_state_dict(self, state_dict: Dict) -> None:
        """Copy saved moments/master weights into the existing flat views."""
        saved_groups = state_dict["param_groups"]
        if len(saved_groups) != len(self.param_groups):
            raise ValueError("optimizer state has a different number of param groups")
        id_map = {}
        for group, sg in zip(self.param_groups, saved_groups):
            if len(group["params"]) != len(sg["params"]):
                raise ValueError("optimizer param group sizes differ")
            for p, sid in zip(group["params"], sg["params"]):
                id_map[sid] = p
            for k, v in sg.items():
                if k != "params":
                    group[k] = v
        for sid, st in state_dict["state"].items():
            p = id_map.get(sid)
            if p is None:
                continue
            mine = self.state[p]
            for key in ("exp_avg", "exp_avg_sq", "master"):
                if key in st and key in mine:
                    mine[key].copy_(st[key].to(mine[key].device, mine[key].dtype))
            if "step" in st:
                mine["step"].fill_(float(st["step"]))
        self._step_count = int(state_dict.get("flat_step", self._step_count))
        with torch.no_grad():
            for fg in self.flat_groups:
                fg.compute_shard.copy_(fg.master)
                if fg.world > 1:
                    import torch.distributed as dist

                    dist.all_gather_into_tensor(fg.compute, fg.compute_shard,
                                                group=self.process_group)
                fg.rebind()


class _FusedDP:
    """Symmetric-memory buffers and epochs for the fused NVLink reduce + AdamW kernels.

    The flat bf16 gradient and parameter buffers of every group are moved into
    symmetric memory (torch's symmetric-memory allocator is used only to map
    the peers' buffers); the kernels are ``csrc/dist_fused.cu``.
    """

    def __init__(self, opt: "FusedAdamW"):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.opt = opt
        pg = opt.process_group or dist.group.WORLD
        self.rank = dist.get_rank(pg)
        self.groups = []
        for fg in opt.flat_groups:
            if not (fg.dp_reduce and fg.world > 1):
                continue
            grad = symm.empty(fg.numel, dtype=fg.grad.dtype, device=fg.grad.device)
            param = symm.empty(fg.numel, dtype=fg.compute.dtype, device=fg.compute.device)
            grad.zero_()
            param.copy_(fg.compute)
            fg.grad, fg.compute = grad, param
            fg.rebind()
            hg = symm.rendezvous(grad, pg)
            hp = symm.rendezvous(param, pg)
            ctrl = symm.empty(64, dtype=torch.int32, device=fg.grad.device)
            ctrl.zero_()
            hc = symm.rendezvous(ctrl, pg)
            torch.cuda.synchronize()
            dist.barrier(group=pg)

            def peer(h, t):
                off = t.data_ptr() - h.buffer_ptrs[h.rank]
                return [int(b) + off for b in h.buffer_ptrs]

            pads = peer(hc, ctrl)
            slots = [p + 3 * 8 * 4 for p in pads]  # floats after 3 rounds x 8 ranks of ints
            self.groups.append(dict(
                fg=fg, grad=peer(hg, grad), param=peer(hp, param), pad=pads, slots=slots,
                gs=grad[fg.lo:fg.lo + fg.shard],
                handles=(hg, hp, hc), ctrl=ctrl))
        dev = opt.flat_groups[0].compute.device
        self.sumsq = torch.zeros(1, device=dev, dtype=torch.float32)
        self.ticket = torch.zeros(2, device=dev, dtype=torch.int32)
        # barrier epochs live on the device (bumped by a kernel each step), so a
        # captured step keeps every rank's barriers in lockstep across replays
        self.epoch_dev = torch.zeros(1, device=dev, dtype=torch.int32)

    def step(self, t: int, max_norm: float) -> None:
        from ..ops import require

        C = require()
        opt = self.opt
        C.dp_epoch_bump(self.epoch_dev)
        # reduce every group first: the partial norms of all groups accumulate in
        # one counter; the last group's last block publishes the total
        for i, g in enumerate(self.groups):
            fg = g["fg"]
            C.dp_reduce_shard(g["grad"], g["param"], g["pad"], g["slots"], self.rank, fg.lo,
                              fg.shard, g["gs"], self.sumsq, self.ticket[0:1], i + 1,
                              i == len(self.groups) - 1, self.epoch_dev)
        for i, g in enumerate(self.groups):
            fg = g["fg"]
            gi, group = next((k, gr) for k, (gr, f) in enumerate(zip(opt.param_groups, opt._flat))
                             if f is fg)
            b1, b2 = group["betas"]
            C.dp_adamw_shard(g["grad"], g["param"], g["pad"], g["slots"], self.rank, fg.lo,
                             fg.shard, fg.master, fg.exp_avg, fg.exp_avg_sq, g["gs"],
                             group["lr"], b1, b2, group["eps"], group["weight_decay"],
                             1.0 - b1 ** t, 1.0 - b2 ** t, max_norm, opt._norm,
                             self.ticket[1:2], i + 1, self.epoch_dev,
                             None if opt._hyper is None else opt._hyper[gi])
        for p_group, fg in zip(opt.param_groups, opt._flat):
            if fg is None:
                continue
            for p in fg.params:
                opt.state[p]["step"].fill_(t)
