"""TR-Hash execution engine: shared SwiGLU plus deterministic top-k experts.

    y = shared_scale * SwiGLU_shared(x) + routed_scale * sum_j a_j * SwiGLU_{R[j, id]}(x)

Parameters, buffers and their names/shapes are the reference's checkpoint
contract (complexity/tr_hash/engine.py:107-189): ``route_table`` [k, V] int64,
``fused_route_codes`` uint8 [V], ``fused_expert_pairs`` int32 [P, 2],
``expert_gate``/``expert_up`` [E, H, W], ``expert_down`` [E, W, H] and the
``shared_gate``/``shared_up``/``shared_down`` Linears.

Execution paths (``select_backend``):
  * fused_cuda: the whole layer FFN is two tcgen05 GEMMs (see ops.fused.TRHashMLPFn).
  * cggr: planner + per-expert contiguous execution for wide experts (ops.grouped).
  * pytorch: ``reference_topk_swiglu``, the authoritative math.
  * cuda_graph: inference-only captured replay, one graph per shape bucket.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Callable, Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .buckets import GraphBucketPlanner
from .capabilities import BackendDecision, has_pair_metadata, select_backend, supports_fused_cuda
from .config import (SUPPORTED_EXPERT_COUNTS, GraphBucket, TRHashBackend, TRHashEngineConfig,
                     TRHashPhase)
from .routing import build_route_table, compile_top2_pair_metadata


def _silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


def reference_topk_swiglu(flat_x: torch.Tensor, routes: torch.Tensor, gate_weights: torch.Tensor,
                          up_weights: torch.Tensor, down_weights: torch.Tensor,
                          route_weights: torch.Tensor, *,
                          activation: Callable = _silu_mul,
                          intermediate_transform: Optional[Callable] = None) -> torch.Tensor:
    """Routed-expert output for ``flat_x [T, H]`` given ``routes [k, T]``.

    For each expert e the per-token weight is sum_j [routes[j] == e] * w[j];
    tokens with zero weight contribute nothing (their input is masked).
    """
    if flat_x.ndim != 2:
        raise ValueError("flat_x must be [tokens, hidden]")
    if routes.ndim != 2 or routes.size(1) != flat_x.size(0):
        raise ValueError("routes must be [top_k, tokens]")
    if route_weights.shape != routes.shape:
        raise ValueError("route_weights must match routes")
    if gate_weights.shape != up_weights.shape:
        raise ValueError("gate and up expert weights must have the same shape")
    if gate_weights.ndim != 3 or down_weights.ndim != 3:
        raise ValueError("expert weights must be rank-3 tensors")
    if gate_weights.size(0) != down_weights.size(0):
        raise ValueError("expert weight tensors must have the same expert count")
    out = torch.zeros_like(flat_x)
    for e in range(gate_weights.size(0)):
        weight = ((routes == e).to(flat_x.dtype) * route_weights).sum(0)
        xe = flat_x * (weight != 0).to(flat_x.dtype)[:, None]
        inter = activation(xe @ gate_weights[e], xe @ up_weights[e])
        if intermediate_transform is not None:
            inter = intermediate_transform(inter, e)
        out = out + (inter @ down_weights[e]).to(out.dtype) * weight[:, None]
    return out


class TRHashEngine(nn.Module):
    def __init__(self, config: TRHashEngineConfig):
        super().__init__()
        self.config = config
        self.register_buffer("route_table", build_route_table(config))
        self.register_buffer("_route_weights",
                             torch.tensor(config.route_weights, dtype=torch.float32),
                             persistent=False)
        codes, pairs = self._pair_metadata(self.route_table)
        self.register_buffer("fused_route_codes", codes)
        self.register_buffer("fused_expert_pairs", pairs)
        E, H, W = config.num_experts, config.hidden_size, config.expert_width
        self.expert_gate = nn.Parameter(torch.empty(E, H, W))
        self.expert_up = nn.Parameter(torch.empty(E, H, W))
        self.expert_down = nn.Parameter(torch.empty(E, W, H))
        if config.shared_width:
            self.shared_gate = nn.Linear(H, config.shared_width, bias=False)
            self.shared_up = nn.Linear(H, config.shared_width, bias=False)
            self.shared_down = nn.Linear(config.shared_width, H, bias=False)
        else:
            self.shared_gate = self.shared_up = self.shared_down = None
        self.reset_parameters()
        self.last_backend: Optional[BackendDecision] = None
        self._graph_pool: Dict[GraphBucket, "_CapturedTRHashGraph"] = {}
        self._bucket_planner = (GraphBucketPlanner(config.graph_buckets)
                                if config.graph_buckets else None)
        self._active_num_experts = E
        self._active_expert_width = W
        self._active_route_table = self.route_table
        self._fused_shared_gate_up_weight: Optional[torch.Tensor] = None
        # inference-only packed (gate|up, down) weights: (key, w_gu, w_down)
        self._packed_cache: Optional[tuple] = None

    # ------------------------------------------------------------ housekeeping
    def train(self, mode: bool = True):
        self._packed_cache = None
        return super().train(mode)

    def invalidate_packed_cache(self) -> None:
        """Drop the inference copy of the packed weights (call after updating
        weights in place while in eval mode)."""
        self._packed_cache = None

    def _packed_for_inference(self):
        """Packed (w_gu, w_down) reused across eval-mode, no-grad forwards.

        Decoding runs a few tokens per forward, so re-packing the whole FFN
        (the shared SwiGLU and every expert) each call would cost more than the
        GEMMs.  The copy is keyed on each weight's storage and version counter
        and dropped by ``train()``; CUDA graphs captured over it keep reading the
        same tensors.
        """
        from ..ops import fused

        sg, su, sd = self._shared_weights()
        ws = (sg, su, self.expert_gate, self.expert_up, sd, self.expert_down)
        key = tuple((w.data_ptr(), w._version) for w in ws if w is not None)
        got = self._packed_cache
        if got is None or got[0] != key:
            with torch.no_grad():
                w_gu, w_down = fused.pack_trhash_weights(*ws)
            got = self._packed_cache = (key, w_gu, w_down)
        return got[1], got[2]

    INFER_DENSE_ROWS = 1024  # eval-mode rows up to which dense-masked experts are used

    def _inference_dense_ready(self, x: torch.Tensor) -> bool:
        """Eval-mode FFN on the fused dense-masked kernels (decoding reads every
        expert's weights anyway, so the masked columns cost no extra bytes)."""
        from ..ops import fused

        sg = self.shared_gate.weight if self.shared_gate is not None else None
        return (not (self.training or torch.is_grad_enabled()) and x.is_cuda
                and x.dtype == torch.bfloat16 and self.expert_gate.dtype == torch.bfloat16
                and not self.is_reduced_capacity and fused.packable(sg, self.expert_gate)
                and self.config.expert_width % 32 == 0 and self.config.num_experts <= 16
                and not any(getattr(m, "is_lora_adapter", False)
                            for m in (self.shared_gate, self.shared_up, self.shared_down)
                            if m is not None))

    def _fused_partial(self, hidden: torch.Tensor, token_ids: torch.Tensor,
                       out: Optional[torch.Tensor],
                       residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """FFN output (this rank's partial under tensor parallelism) plus
        ``residual`` when given, into ``out`` when given."""
        from ..ops import fused

        cfg = self.config
        scales = fused.route_scales(token_ids, self._active_route_table, self._route_weights,
                                    cfg.num_experts, cfg.routed_output_scale)
        w_gu, w_down = self._packed_for_inference()
        return fused.trhash_mlp_infer(hidden, w_gu, w_down, scales, cfg.shared_width,
                                      cfg.expert_width, cfg.num_experts,
                                      cfg.shared_output_scale, out, residual)

    def _apply(self, fn, recurse: bool = True):
        self._packed_cache = None
        aliased = self._active_route_table is self.route_table
        super()._apply(fn, recurse=recurse)
        self._active_route_table = self.route_table if aliased else fn(self._active_route_table)
        if self._fused_shared_gate_up_weight is not None:
            self._fused_shared_gate_up_weight = fn(self._fused_shared_gate_up_weight)
        return self

    def _pair_metadata(self, table: torch.Tensor):
        with torch.device("cpu"):  # host-side metadata, also under a meta default device
            if has_pair_metadata(self.config):
                return compile_top2_pair_metadata(table.cpu(), num_experts=self.config.num_experts)
            return torch.empty(0, dtype=torch.uint8), torch.empty((0, 2), dtype=torch.int32)

    @property
    def active_num_experts(self) -> int:
        return self._active_num_experts

    @property
    def active_expert_width(self) -> int:
        return self._active_expert_width

    @property
    def is_reduced_capacity(self) -> bool:
        return (self._active_num_experts != self.config.num_experts
                or self._active_expert_width != self.config.expert_width)

    def set_active_capacity(self, *, num_experts: Optional[int] = None,
                            expert_width: Optional[int] = None) -> None:
        """Run a deterministic prefix sub-network (fewer experts and/or narrower experts).

        Routes for a reduced expert count are rebuilt with the same builder, so
        routing stays a pure function of token id.
        """
        if num_experts is not None:
            if num_experts not in SUPPORTED_EXPERT_COUNTS:
                raise ValueError(f"num_experts must be one of {SUPPORTED_EXPERT_COUNTS}, "
                                 f"got {num_experts}")
            if num_experts > self.config.num_experts:
                raise ValueError(f"active num_experts ({num_experts}) cannot exceed the "
                                 f"allocated capacity ({self.config.num_experts})")
            if num_experts == self.config.num_experts:
                self._active_route_table = self.route_table
            else:
                sub = replace(self.config, num_experts=num_experts)
                self._active_route_table = build_route_table(sub).to(self.route_table.device)
            self._active_num_experts = num_experts
        if expert_width is not None:
            if not 0 < expert_width <= self.config.expert_width:
                raise ValueError(f"active expert_width must be in (0, {self.config.expert_width}]"
                                 f", got {expert_width}")
            self._active_expert_width = expert_width
        if num_experts is not None or expert_width is not None:
            self._graph_pool.clear()

    def load_route_table(self, route_table: torch.Tensor) -> None:
        """Install an exact externally supplied table (e.g. from a converted checkpoint)."""
        if tuple(route_table.shape) != tuple(self.route_table.shape):
            raise ValueError(f"route_table shape {tuple(route_table.shape)} does not match the "
                             f"engine's {tuple(self.route_table.shape)} ([top_k, vocab_size])")
        if int(route_table.min()) < 0 or int(route_table.max()) >= self.config.num_experts:
            raise ValueError("route_table contains an out-of-range expert index")
        self.route_table.copy_(route_table.to(self.route_table.device))
        codes, pairs = self._pair_metadata(self.route_table)
        self.fused_route_codes = codes.to(self.fused_route_codes.device)
        self.fused_expert_pairs = pairs.to(self.fused_expert_pairs.device)
        if self._active_num_experts == self.config.num_experts:
            self._active_route_table = self.route_table
        else:
            sub = replace(self.config, num_experts=self._active_num_experts)
            self._active_route_table = build_route_table(sub).to(self.route_table.device)
        self._graph_pool.clear()

    def set_route_weights(self, weights) -> None:
        """Change the per-slot blend weights; every backend reads the same values."""
        self.config = replace(self.config, route_weights=tuple(float(w) for w in weights))
        self._route_weights.copy_(torch.tensor(self.config.route_weights, dtype=torch.float32))
        self._graph_pool.clear()

    def reset_parameters(self) -> None:
        std = self.config.initializer_range
        for p in (self.expert_gate, self.expert_up, self.expert_down):
            nn.init.normal_(p, mean=0.0, std=std)
        for m in (self.shared_gate, self.shared_up, self.shared_down):
            if m is not None:
                nn.init.normal_(m.weight, mean=0.0, std=std)

    # ------------------------------------------------------------------ pieces
    def _routes(self, token_ids: torch.Tensor) -> torch.Tensor:
        ids = token_ids.clamp(0, self.config.vocab_size - 1)
        return self._active_route_table[:, ids]

    def _active_expert_weights(self):
        E, W = self._active_num_experts, self._active_expert_width
        if not self.is_reduced_capacity:
            return self.expert_gate, self.expert_up, self.expert_down
        return (self.expert_gate[:E, :, :W].contiguous(), self.expert_up[:E, :, :W].contiguous(),
                self.expert_down[:E, :W, :].contiguous())

    def _shared(self, flat_x: torch.Tensor) -> torch.Tensor:
        if self.shared_gate is None:
            return torch.zeros_like(flat_x)
        fused = self._fused_shared_gate_up_weight
        if (fused is not None and getattr(self.shared_gate, "is_lora_adapter", False)
                and getattr(self.shared_up, "is_lora_adapter", False)):
            width = int(self.shared_gate.base.out_features)
            g, u = F.linear(flat_x, fused).split([width, width], -1)
            g = g + self.shared_gate.lora_residual(flat_x)
            u = u + self.shared_up.lora_residual(flat_x)
        else:
            g, u = self.shared_gate(flat_x), self.shared_up(flat_x)
        return self.shared_down(_silu_mul(g, u))

    def _shared_ep(self, flat_x: torch.Tensor) -> torch.Tensor:
        """shared_scale * shared SwiGLU; one fused gate|up + down GEMM pair on CUDA bf16."""
        cfg = self.config
        if self.shared_gate is None:
            return torch.zeros_like(flat_x)
        if (flat_x.is_cuda and flat_x.dtype == torch.bfloat16 and cfg.shared_width % 128 == 0
                and self.shared_gate.weight.dtype == torch.bfloat16):
            from ..ops import fused

            w_gu = fused.pack_shared_gate_up(self.shared_gate.weight, self.shared_up.weight)
            dummy = flat_x.new_zeros(1, dtype=torch.float32)
            return fused.trhash_mlp(flat_x, w_gu, self.shared_down.weight, dummy, None,
                                    cfg.shared_width, 32, 0, cfg.shared_output_scale)
        return cfg.shared_output_scale * self._shared(flat_x)

    def refresh_fused_shared_lora_weight(self) -> bool:
        if not (getattr(self.shared_gate, "is_lora_adapter", False)
                and getattr(self.shared_up, "is_lora_adapter", False)):
            self._fused_shared_gate_up_weight = None
            return False
        self._fused_shared_gate_up_weight = torch.cat(
            [self.shared_gate.base.weight, self.shared_up.base.weight], 0).detach()
        return True

    def _reference_routed(self, flat_x: torch.Tensor, routes: torch.Tensor) -> torch.Tensor:
        w = self._route_weights.to(flat_x.dtype)[:, None].expand_as(routes)
        g, u, d = self._active_expert_weights()
        return reference_topk_swiglu(flat_x, routes, g, u, d, w)

    def packed_weights(self):
        """(gate|up interleaved [2A, H], down [H, A]) for the fused path (autograd-tracked)."""
        from ..ops import fused
        from ..ops.fused import pack_down, pack_gate_up

        if any(getattr(m, "is_lora_adapter", False)
               for m in (self.shared_gate, self.shared_up, self.shared_down) if m is not None):
            raise RuntimeError("fused path does not execute LoRA-adapted shared projections")
        wg, wu, wd = self._shared_weights()
        if fused.packable(wg, self.expert_gate):
            return fused.PackTRHashFn.apply(wg, wu, self.expert_gate, self.expert_up, wd,
                                            self.expert_down)
        return (pack_gate_up(wg, wu, self.expert_gate, self.expert_up),
                pack_down(wd, self.expert_down))

    def _shared_weights(self):
        if self.shared_gate is None:
            return None, None, None
        return self.shared_gate.weight, self.shared_up.weight, self.shared_down.weight

    def _fused_forward(self, hidden: torch.Tensor, token_ids: torch.Tensor,
                       residual: Optional[torch.Tensor]) -> torch.Tensor:
        from ..ops import fused

        if self.is_reduced_capacity:
            raise RuntimeError(
                "FUSED_CUDA requires the full allocated capacity "
                f"(active={self._active_num_experts}/{self.config.num_experts} experts, "
                f"{self._active_expert_width}/{self.config.expert_width} width); use the "
                "pytorch backend while capacity is reduced")
        cfg = self.config
        scales = fused.route_scales(token_ids, self._active_route_table,
                                    self._route_weights, cfg.num_experts,
                                    cfg.routed_output_scale)
        wg, wu, wd = self._shared_weights()
        if (fused.packable(wg, self.expert_gate) and not any(
                getattr(m, "is_lora_adapter", False)
                for m in (self.shared_gate, self.shared_up, self.shared_down) if m is not None)):
            if not (self.training or torch.is_grad_enabled()):
                w_gu, w_down = self._packed_for_inference()
                return fused.trhash_mlp(hidden, w_gu, w_down, scales, residual,
                                        cfg.shared_width, cfg.expert_width, cfg.num_experts,
                                        cfg.shared_output_scale)
            # packing and gradient unpacking fused into the MLP's own autograd node
            return fused.trhash_mlp_params(hidden, wg, wu, self.expert_gate, self.expert_up, wd,
                                           self.expert_down, scales, residual, cfg.shared_width,
                                           cfg.expert_width, cfg.num_experts,
                                           cfg.shared_output_scale)
        w_gu, w_down = self.packed_weights()
        return fused.trhash_mlp(hidden, w_gu, w_down, scales, residual, cfg.shared_width,
                                cfg.expert_width, cfg.num_experts, cfg.shared_output_scale)

    def _grouped_forward(self, flat_x: torch.Tensor, flat_ids: torch.Tensor) -> torch.Tensor:
        from ..ops import grouped

        routes = self._routes(flat_ids).reshape(self.config.top_k, -1)
        g, u, d = self._active_expert_weights()
        return grouped.routed_experts(flat_x, routes, self._route_weights, g, u, d)

    def _forward_eager(self, hidden_states: torch.Tensor, token_ids: torch.Tensor,
                       backend: TRHashBackend, residual: Optional[torch.Tensor] = None
                       ) -> torch.Tensor:
        if hidden_states.ndim != 3:
            raise ValueError("hidden_states must be [batch, sequence, hidden]")
        if token_ids.shape != hidden_states.shape[:2]:
            raise ValueError("token_ids must match hidden batch/sequence dimensions")
        if hidden_states.size(-1) != self.config.hidden_size:
            raise ValueError(f"expected hidden size {self.config.hidden_size}, "
                             f"got {hidden_states.size(-1)}")
        B, S, H = hidden_states.shape
        ep = getattr(self, "ep", None)
        if backend is TRHashBackend.FUSED_CUDA and ep is None:
            return self._fused_forward(hidden_states, token_ids, residual)
        flat = hidden_states.reshape(-1, H)
        if ep is not None:
            # expert parallel: shared SwiGLU locally, routed experts via all-to-all
            routes = self._routes(token_ids).reshape(self.config.top_k, -1)
            routed = ep(flat, routes, self._route_weights, token_ids=token_ids,
                        route_fn=self._routes)
            out = (self._shared_ep(flat) + self.config.routed_output_scale * routed).view(B, S, H)
            return out if residual is None else residual + out
        if backend is TRHashBackend.CGGR:
            # shared SwiGLU as one fused gate|up + down GEMM pair on CUDA bf16,
            # routed experts on the grouped kernels
            shared_term = self._shared_ep(flat)
            routed = self._grouped_forward(flat, token_ids.reshape(-1))
        else:
            shared_term = self.config.shared_output_scale * self._shared(flat)
            routes = self._routes(token_ids).reshape(self.config.top_k, -1)
            routed = self._reference_routed(flat, routes)
        out = shared_term + self.config.routed_output_scale * routed
        out = out.view(B, S, H)
        return out if residual is None else residual + out

    def decide(self, device_type: str) -> BackendDecision:
        decision = select_backend(self.config, device_type=device_type)
        if (decision.selected is TRHashBackend.FUSED_CUDA and self.config.backend
                is TRHashBackend.AUTO and self.is_reduced_capacity):
            decision = BackendDecision(decision.requested, TRHashBackend.PYTORCH,
                                       ("reduced capacity runs on the reference path",), False,
                                       False)
        return decision

    def forward(self, hidden_states: torch.Tensor, token_ids: torch.Tensor,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """FFN output; when ``residual`` is given returns ``residual + FFN`` (fused on CUDA)."""
        decision = self.decide(hidden_states.device.type)
        if (decision.selected is TRHashBackend.FUSED_CUDA
                and hidden_states.dtype != torch.bfloat16):
            decision = BackendDecision(decision.requested, TRHashBackend.PYTORCH,
                                       ("fused path computes in bf16; input is "
                                        f"{hidden_states.dtype}",), False, False)
        self.last_backend = decision
        tp = getattr(self, "tp_group", None)
        H = hidden_states.shape[-1]
        kernels = decision.selected in (TRHashBackend.FUSED_CUDA, TRHashBackend.CGGR)
        if (tp is None and kernels and hidden_states.numel() // H <= self.INFER_DENSE_ROWS
                and self._inference_dense_ready(hidden_states)):
            # decoding: few rows read every expert's weights anyway, so the
            # dense-masked fused kernels are the bandwidth-optimal choice
            return self._fused_partial(hidden_states, token_ids, None,
                                       residual).view_as(hidden_states)
        if (tp is not None and kernels and hasattr(self, "tp_site")
                and self._inference_dense_ready(hidden_states)):
            # tensor-parallel inference: partial FFN into the symmetric buffer of
            # this call site, then one fused all-reduce + residual
            from ..parallel.tp_inference import tp_reduce_add

            rows = hidden_states.numel() // H
            y = tp_reduce_add(getattr(self, "tp_decode", None), self.tp_site,
                              lambda out: self._fused_partial(hidden_states, token_ids, out),
                              rows, residual, tp)
            return y.view_as(hidden_states)
        if tp is not None:
            # tensor parallel: this rank holds a slice of every width; sum the slices
            from ..parallel.tensor_parallel import copy_to_tp, reduce_from_tp

            x = copy_to_tp(hidden_states, tp)
            out = reduce_from_tp(self._forward_eager(x, token_ids, decision.selected), tp)
            return out if residual is None else residual + out
        if decision.selected is TRHashBackend.CUDA_GRAPH:
            out = self._forward_cuda_graph(hidden_states, token_ids)
            return out if residual is None else residual + out
        return self._forward_eager(hidden_states, token_ids, decision.selected, residual)

    def _forward_cuda_graph(self, hidden_states: torch.Tensor, token_ids: torch.Tensor):
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("CUDA Graph TR-Hash requires eval mode and torch.no_grad()")
        if hidden_states.device.type != "cuda":
            raise RuntimeError("CUDA Graph TR-Hash requires CUDA tensors")
        if self._bucket_planner is None:
            raise RuntimeError("CUDA Graph backend has no configured buckets")
        B, S, _ = hidden_states.shape
        bucket = self._bucket_planner.select(B, S)
        runner = self._graph_pool.get(bucket)
        if runner is None:
            runner = _CapturedTRHashGraph(self, bucket, hidden_states)
            self._graph_pool[bucket] = runner
        return runner.replay(hidden_states, token_ids)

    def capability_summary(self, device_type: str = "cpu") -> dict:
        """Stable, serialisable metadata for logs and manifests (same keys as the reference)."""
        d = self.decide(device_type)
        cfg = self.config
        return {
            "experts": cfg.num_experts,
            "top_k": cfg.top_k,
            "shared_width": cfg.shared_width,
            "expert_width": cfg.expert_width,
            "stored_width": cfg.stored_mlp_width,
            "active_width": cfg.active_mlp_width,
            "active_width_fraction": cfg.active_width_fraction,
            "active_num_experts": self._active_num_experts,
            "active_expert_width": self._active_expert_width,
            "is_reduced_capacity": self.is_reduced_capacity,
            "attention": cfg.attention_backbone.value,
            "routing": cfg.routing_strategy.value,
            "phase": cfg.phase.value,
            "precision": cfg.precision.value,
            "world_size": cfg.world_size,
            "parallelism": "replicated_ddp" if cfg.world_size > 1 else "single_device",
            "requested_backend": d.requested.value,
            "selected_backend": d.selected.value,
            "backend_reasons": list(d.reasons),
            "fused_cuda_eligible": supports_fused_cuda(cfg),
            "cuda_graph_buckets": [[b.batch_size, b.sequence_length] for b in cfg.graph_buckets],
        }


class _CapturedTRHashGraph:
    """A lazily captured inference graph with persistent padded input buffers."""

    def __init__(self, engine: TRHashEngine, bucket: GraphBucket, sample: torch.Tensor):
        if engine.config.phase is not TRHashPhase.INFERENCE:
            raise RuntimeError("only inference graphs can be captured")
        self.engine = engine
        self.bucket = bucket
        shape = (bucket.batch_size, bucket.sequence_length, engine.config.hidden_size)
        self.hidden = torch.zeros(shape, dtype=sample.dtype, device=sample.device)
        self.token_ids = torch.zeros(shape[:2], dtype=torch.long, device=sample.device)
        inner = (TRHashBackend.FUSED_CUDA
                 if sample.dtype == torch.bfloat16 and select_backend(
                     replace(engine.config, backend=TRHashBackend.AUTO),
                     device_type="cuda").selected is TRHashBackend.FUSED_CUDA
                 else TRHashBackend.PYTORCH)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                self.output = engine._forward_eager(self.hidden, self.token_ids, inner)
        side.synchronize()
        with torch.cuda.graph(self.graph):
            self.output = engine._forward_eager(self.hidden, self.token_ids, inner)

    def replay(self, hidden_states: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
        B, S, _ = hidden_states.shape
        self.hidden.zero_()
        self.token_ids.zero_()
        self.hidden[:B, :S].copy_(hidden_states)
        self.token_ids[:B, :S].copy_(token_ids)
        self.graph.replay()
        return self.output[:B, :S].clone()
