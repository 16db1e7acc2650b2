"""Fully sharded data parallelism (ZeRO-3) for ``ComplexityModel``.

Each transformer block is one *unit*; everything else (embedding, final norm,
LM head) forms a root unit.  A unit's parameters live in one flat bf16
buffer split into ``world`` contiguous shards; rank r keeps only its shard
(in symmetric memory, readable by every peer) and the fp32 master weights
and Adam moments of that shard.  The unit's full bf16 buffer exists only
while the unit runs:

* forward: a pre-hook makes the unit's parameters views of its gathered
  buffer and starts the gather of the NEXT unit on a side stream
  (``C.fsdp_gather``: bounded barrier, then NVLink pulls of every shard), so
  weight transfers overlap the current unit's compute; a post-hook frees the
  buffer's storage (autograd keeps the views; they are refilled before use);
* backward: a hook on the unit's output gathers the unit again (and starts
  the previous unit's gather); when the unit's parameter gradients are
  complete (multi-grad hook), they are copied into the unit's symmetric
  bf16 gradient buffer and its reduce-scatter (``C.dp_reduce_shard``: every
  rank sums its slice of all peers' gradients over NVLink, with the squared
  norm) is launched on the side stream -- it overlaps the remaining backward;
* step: global norm (one all-reduce of a scalar), clip, and AdamW on each
  shard (``adamw_flat``) writing the new bf16 shard in place.

On CPU (gloo) the gather and reduce-scatter fall back to the process group's
collectives, so the same code runs in the CPU tests.

Reference counterpart: ``wrap_model_fsdp`` / ``fully_shard`` per block in
complexity/parallel/data_parallel.py:102-129 (FSDP2, NCCL all-gather and
reduce-scatter, bf16 optimizer state); here the optimizer keeps fp32
master weights and the collectives are this framework's own kernels.
Activation checkpointing inside a unit (a second forward) is not supported.
"""
from __future__ import annotations

import contextlib
from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

_PAD = 128  # element alignment of every parameter inside a unit (256 bytes)


def _no_decay(name: str, p: torch.Tensor) -> bool:
    return p.dim() < 2 or "norm" in name or name.endswith(".bias")


class _Unit:
    """Flat sharded storage of one unit's parameters."""

    def __init__(self, owner: "ShardedModel", name: str, named: Sequence, idx: int):
        self.owner, self.name, self.idx = owner, name, idx
        world, rank, dev = owner.world, owner.rank, owner.device
        decay = [(n, p) for n, p in named if not _no_decay(n, p)]
        nodecay = [(n, p) for n, p in named if _no_decay(n, p)]
        self.params = [p for _, p in decay + nodecay]
        self.names = [n for n, _ in decay + nodecay]
        self.shapes = [p.shape for p in self.params]
        self.offsets, off = [], 0
        for p in self.params:
            self.offsets.append(off)
            off += (p.numel() + _PAD - 1) // _PAD * _PAD
        self.decay_end = self.offsets[len(decay)] if nodecay else off
        unit = _PAD * world
        self.numel = (off + unit - 1) // unit * unit
        self.shard = self.numel // world
        self.lo = rank * self.shard
        dt = owner.dtype
        full = torch.zeros(self.numel, device=dev, dtype=dt)
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                full[o:o + p.numel()].copy_(p.detach().reshape(-1))
        self.master = full[self.lo:self.lo + self.shard].float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        if owner.fused:
            symm = owner.symm
            self.shard_buf = symm.empty(self.shard, dtype=torch.bfloat16, device=dev)
            self.grad_full = symm.empty(self.numel, dtype=torch.bfloat16, device=dev)
            self.pad = symm.empty(64, dtype=torch.int32, device=dev)
            self.pad.zero_()
            self.grad_full.zero_()
            self._handles = [symm.rendezvous(t, owner.group)
                             for t in (self.shard_buf, self.grad_full, self.pad)]
            self.shard_ptrs = owner.peer_ptrs(self._handles[0], self.shard_buf)
            self.grad_ptrs = owner.peer_ptrs(self._handles[1], self.grad_full)
            self.pad_ptrs = owner.peer_ptrs(self._handles[2], self.pad)
            self.slot_ptrs = [p + 24 * 4 for p in self.pad_ptrs]  # unused (no publish)
        else:
            self.shard_buf = torch.empty(self.shard, device=dev, dtype=dt)
            self.grad_full = torch.zeros(self.numel, device=dev, dtype=dt)
        self.shard_buf.copy_(full[self.lo:self.lo + self.shard])
        self.full = full  # resident after construction; freed by reshard()
        self.resident = True
        self.ready: Optional[torch.cuda.Event] = None
        self.epochs = [0, 0, 0, 0]  # per round: reduce, forward gather, backward gather, summon
        self.grad_done = False
        self._bind()

    # -------------------------------------------------------------- storage
    def _bind(self) -> None:
        for p, o, shp in zip(self.params, self.offsets, self.shapes):
            p.data = self.full[o:o + shp.numel()].view(shp)

    def _alloc(self) -> None:
        st = self.full.untyped_storage()
        if st.size() == 0:
            st.resize_(self.numel * self.full.element_size())

    def reshard(self) -> None:
        """Free the full buffer (parameter views stay; refilled by the next gather)."""
        if self.resident and not self.owner.keep_resident:
            self.full.untyped_storage().resize_(0)
            self.resident = False
            self.ready = None

    def gather(self, rnd: int, async_: bool) -> None:
        """Fill the full buffer from every rank's shard (round 1 forward, 2
        backward, 3 summon).  With ``async_`` the copy runs on the side stream."""
        o = self.owner
        if self.resident:
            return
        self._alloc()
        self.epochs[rnd] += 1
        if not o.fused:
            parts = [torch.empty_like(self.shard_buf) for _ in range(o.world)]
            dist.all_gather(parts, self.shard_buf, group=o.group)
            self.full.copy_(torch.cat(parts))
            self.resident = True
            return
        C = o.C
        if async_:
            o.comm.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(o.comm):
                C.fsdp_gather(self.shard_ptrs, self.pad_ptrs, o.rank, self.full, self.shard, rnd,
                              self.epochs[rnd])
                self.ready = torch.cuda.Event()
                self.ready.record(o.comm)
        else:
            C.fsdp_gather(self.shard_ptrs, self.pad_ptrs, o.rank, self.full, self.shard, rnd,
                          self.epochs[rnd])
            self.ready = None
        self.resident = True

    def wait(self) -> None:
        if self.ready is not None:
            torch.cuda.current_stream().wait_event(self.ready)
            self.ready = None

    # ------------------------------------------------------------ gradients
    @torch.no_grad()
    def reduce_grads(self, grads: Optional[Sequence[Optional[torch.Tensor]]] = None) -> None:
        """Move this unit's gradients (the hook's ``grads``, else ``p.grad``) into
        its flat buffer and reduce-scatter them (the side stream overlaps the
        reduction with the rest of backward)."""
        o = self.owner
        if self.grad_done:
            return
        self.grad_done = True
        dst, src, missing = [], [], []
        for i, (p, off, shp) in enumerate(zip(self.params, self.offsets, self.shapes)):
            view = self.grad_full[off:off + shp.numel()].view(shp)
            g = grads[i] if grads is not None else p.grad
            if g is None:
                missing.append(view)
            else:
                dst.append(view)
                src.append(g)
            p.grad = None
        if dst:
            torch._foreach_copy_(dst, src)
        if missing:
            torch._foreach_zero_(missing)
        self.epochs[0] += 1
        if not o.fused:
            g = self.grad_full.float()
            dist.all_reduce(g, group=o.group)
            self.grad_full[self.lo:self.lo + self.shard].copy_(
                (g[self.lo:self.lo + self.shard] / o.world).to(self.grad_full.dtype))
            self.reshard()
            return
        done = torch.cuda.Event()
        done.record()
        with torch.cuda.stream(o.comm):
            o.comm.wait_event(done)
            o.C.dp_reduce_shard(self.grad_ptrs, self.shard_ptrs, self.pad_ptrs, self.slot_ptrs,
                                o.rank, self.lo, self.shard,
                                self.grad_full[self.lo:self.lo + self.shard], o.sumsq, o.ticket,
                                self.epochs[0], False)
        self.reshard()

    @property
    def grad_shard(self) -> torch.Tensor:
        return self.grad_full[self.lo:self.lo + self.shard]


class ShardedModel:
    """ZeRO-3 sharding of ``model`` over ``group`` (installed in place; the
    model object is returned by ``shard_model``)."""

    def __init__(self, model: nn.Module, group=None, *, prefetch: bool = True,
                 fused: Optional[bool] = None):
        self.model = model
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        p0 = next(model.parameters())
        self.device, self.dtype = p0.device, p0.dtype
        if fused is None:
            fused = (self.device.type == "cuda" and 1 < self.world <= 8
                     and dist.get_backend(self.group) == "nccl")
        self.fused = bool(fused)
        if self.fused and self.dtype != torch.bfloat16:
            raise ValueError("the NVLink ZeRO-3 path keeps bf16 parameters; cast the model first")
        self.keep_resident = False
        self.prefetch = prefetch
        if self.fused:
            import torch.distributed._symmetric_memory as symm

            from ..ops import require

            self.symm, self.C = symm, require()
            self.comm = torch.cuda.Stream(self.device)
            self.sumsq = torch.zeros(1, device=self.device, dtype=torch.float32)
            self.ticket = torch.zeros(1, device=self.device, dtype=torch.int32)
        blocks = list(model.layers)
        in_block = set()
        self.units: List[_Unit] = []
        for i, blk in enumerate(blocks):
            named = [(f"layers.{i}.{n}", p) for n, p in blk.named_parameters()
                     if p.requires_grad]
            in_block.update(id(p) for _, p in named)
            self.units.append(_Unit(self, f"layers.{i}", named, i))
        seen, root = set(), []
        for n, p in model.named_parameters():
            if p.requires_grad and id(p) not in in_block and id(p) not in seen:
                seen.add(id(p))
                root.append((n, p))
        self.root = _Unit(self, "root", root, len(blocks))
        if self.fused:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        for u in self.units:
            u.reshard()
        self._hooks = []
        for i, blk in enumerate(blocks):
            self._hooks.append(blk.register_forward_pre_hook(self._pre_forward(i)))
            self._hooks.append(blk.register_forward_hook(self._post_forward(i)))
            self._hooks.append(torch.autograd.graph.register_multi_grad_hook(
                tuple(self.units[i].params), self._post_backward(i), mode="all"))
        self._hooks.append(model.register_forward_pre_hook(self._root_pre_forward))
        model.zero3 = self

    @staticmethod
    def peer_ptrs(h, t) -> List[int]:
        off = t.data_ptr() - int(h.buffer_ptrs[h.rank])
        return [int(p) + off for p in h.buffer_ptrs]

    # ---------------------------------------------------------------- hooks
    def _root_pre_forward(self, module, args):
        self.root.gather(1, async_=False)
        self.root.wait()
        if self.prefetch and self.units:
            self.units[0].gather(1, async_=True)

    def _pre_forward(self, i: int):
        def hook(module, args):
            u = self.units[i]
            u.gather(1, async_=False)
            u.wait()
            u.grad_done = False
            if self.prefetch and i + 1 < len(self.units):
                self.units[i + 1].gather(1, async_=True)
        return hook

    def _post_forward(self, i: int):
        def hook(module, args, out):
            t = out[0] if isinstance(out, (tuple, list)) else out
            if torch.is_grad_enabled() and isinstance(t, torch.Tensor) and t.requires_grad:
                t.register_hook(self._pre_backward(i))
            if not (torch.is_grad_enabled() and i == len(self.units) - 1):
                self.units[i].reshard()  # the last unit stays for the backward
            return None
        return hook

    def _pre_backward(self, i: int):
        def hook(grad):
            u = self.units[i]
            u.gather(2, async_=False)
            u.wait()
            if self.prefetch and i > 0:
                self.units[i - 1].gather(2, async_=True)
            return grad
        return hook

    def _post_backward(self, i: int):
        def hook(grads):
            self.units[i].reduce_grads(grads)
        return hook

    # ------------------------------------------------------------- optimizer
    def finish_backward(self) -> None:
        """After ``loss.backward()``: reduce whatever the hooks did not (units
        without gradients, the root) and wait for the side stream."""
        for u in self.units:
            u.reduce_grads()
        self.root.reduce_grads()
        if self.fused:
            torch.cuda.current_stream().wait_stream(self.comm)

    def all_units(self) -> List[_Unit]:
        return self.units + [self.root]

    @contextlib.contextmanager
    def summon_full_params(self):
        """Every unit gathered and resident (checkpointing, evaluation by hand)."""
        for u in self.all_units():
            u.gather(3, async_=False)
        prev, self.keep_resident = self.keep_resident, True
        try:
            yield
        finally:
            self.keep_resident = prev
            for u in self.units:
                u.reshard()

    @torch.no_grad()
    def load_full_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        """Load full weights into every unit's shard (and fp32 master)."""
        with self.summon_full_params():
            self.model.load_state_dict(sd, strict=False)
            for u in self.all_units():
                u.shard_buf.copy_(u.full[u.lo:u.lo + u.shard])
                u.master.copy_(u.shard_buf.float())

    def full_state_dict(self) -> Dict[str, torch.Tensor]:
        with self.summon_full_params():
            return {k: v.detach().clone() for k, v in self.model.state_dict().items()}


class Zero3AdamW(torch.optim.Optimizer):
    """AdamW on the ZeRO-3 shards: fp32 master weights and moments of this
    rank's shard of every unit, global-norm clipping, bf16 shard written in
    place (the next forward gathers it)."""

    def __init__(self, sharded: ShardedModel, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1):
        params = [p for u in sharded.all_units() for p in u.params]
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps,
                                      weight_decay=weight_decay))
        self.sh = sharded
        self._step = 0
        dev = sharded.device
        self._sumsq = torch.zeros(1, device=dev, dtype=torch.float32)
        self._clip = torch.ones(1, device=dev, dtype=torch.float32)
        self._norm = torch.zeros(1, device=dev, dtype=torch.float32)
        self._max_norm = 0.0

    def zero_grad(self, set_to_none: bool = True) -> None:
        # the hooks consumed every gradient; AccumulateGrad's copies are dropped here
        for u in self.sh.all_units():
            for p in u.params:
                p.grad = None
            u.grad_done = False
        if self.sh.fused:
            self.sh.sumsq.zero_()

    @torch.no_grad()
    def reduce_gradients(self) -> None:
        self.sh.finish_backward()

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        sh = self.sh
        if sh.fused:  # the reduce kernels summed squares of the shards they wrote
            self._sumsq.copy_(sh.sumsq)
            # the root's and gradient-less units' shards were reduced too: count all
        else:
            self._sumsq.zero_()
            for u in sh.all_units():
                self._sumsq += u.grad_shard.float().pow(2).sum()
        if sh.world > 1:
            dist.all_reduce(self._sumsq, group=sh.group)
        self._norm.copy_(self._sumsq.sqrt())
        self._clip.copy_(torch.clamp(max_norm / (self._norm + 1e-6), max=1.0))
        self._max_norm = max_norm
        return self._norm

    @torch.no_grad()
    def step(self, closure=None, clip: bool = False) -> None:
        self._step += 1
        grp = self.param_groups[0]
        lr, (b1, b2), eps, wd = grp["lr"], grp["betas"], grp["eps"], grp["weight_decay"]
        bc1, bc2 = 1 - b1 ** self._step, 1 - b2 ** self._step
        use_kernel = self.sh.device.type == "cuda" and self.sh.dtype == torch.bfloat16
        if use_kernel:
            from ..ops import require

            C = require()
        for u in self.sh.all_units():
            lo, hi = u.lo, u.lo + u.shard
            for a, b, w in ((lo, min(hi, u.decay_end), wd), (max(lo, u.decay_end), hi, 0.0)):
                if a >= b:
                    continue
                s = slice(a - lo, b - lo)
                if use_kernel:
                    C.adamw_flat(u.master[s], u.exp_avg[s], u.exp_avg_sq[s], u.grad_shard[s],
                                 u.shard_buf[s], lr, b1, b2, eps, w, bc1, bc2,
                                 self._clip if clip else None)
                else:
                    g = u.grad_shard[s].float() * (self._clip if clip else 1.0)
                    m, v, p = u.exp_avg[s], u.exp_avg_sq[s], u.master[s]
                    p.mul_(1 - lr * w)
                    m.mul_(b1).add_(g, alpha=1 - b1)
                    v.mul_(b2).addcmul_(g, g, value=1 - b2)
                    p.addcdiv_(m / bc1, (v / bc2).sqrt_().add_(eps), value=-lr)
                    u.shard_buf[s].copy_(p.to(u.shard_buf.dtype))
        for u in self.sh.all_units():  # every unit is gathered afresh by the next forward
            u.reshard()

    def state_dict(self):
        return {"step": self._step,
                "units": [{"master": u.master, "exp_avg": u.exp_avg, "exp_avg_sq": u.exp_avg_sq}
                          for u in self.sh.all_units()],
                "param_groups": [{k: v for k, v in g.items() if k != "params"}
                                 for g in self.param_groups]}

    def load_state_dict(self, sd) -> None:
        self._step = int(sd["step"])
        for u, st in zip(self.sh.all_units(), sd["units"]):
            u.master.copy_(st["master"])
            u.exp_avg.copy_(st["exp_avg"])
            u.exp_avg_sq.copy_(st["exp_avg_sq"])
            u.shard_buf.copy_(u.master.to(u.shard_buf.dtype))
        for g, s in zip(self.param_groups, sd.get("param_groups", [])):
            g.update({k: v for k, v in s.items() if k in ("lr", "betas", "eps", "weight_decay")})


def shard_model(model: nn.Module, group=None, **kw) -> nn.Module:
    """Install ZeRO-3 sharding on ``model`` (bf16) over ``group``; returns the model
    (its ``zero3`` attribute is the :class:`ShardedModel`)."""
    ShardedModel(model, group, **kw)
    return model
