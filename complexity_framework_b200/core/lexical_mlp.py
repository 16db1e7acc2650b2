"""Lexical MLPs: a dense SwiGLU whose output or channels are modulated by a
per-token-id table, with no expert dispatch.

* ``lexical_modulated`` / ``lexical_object``: shared SwiGLU plus a low-rank
  object residual ``gate * down(silu(up(x)) * (1 + scale[id]))``, where
  ``scale`` is a ``[vocab, rank]`` table initialised to zero.
* ``lexical_channel_modulated`` / ``lexical_channel_object``: the SwiGLU
  channels are multiplied by ``1 + gate * scale[id]`` with each of the rank
  values covering a contiguous block of ceil(width / rank) channels.
* ``lexical_object_micro_expert``: the object residual plus a top-1 micro
  expert picked by ``(id + layer) % n`` from small per-expert SwiGLUs.

Parameter names, shapes and the optional model-level shared table
(``tie_lexical_object_embeddings``: one ``lexical_token_scale`` for all
layers) follow complexity/core/mlp/lexical_modulated.py,
lexical_channel_modulated.py and lexical_object_micro_expert.py so checkpoints
load in either framework.  On CUDA bf16 the shared SwiGLU runs on the fused
gate|up + down kernel pair; the lexical branches are small and stay in PyTorch.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import use_fused
from .registry import register_mlp

LEXICAL_MLP_TYPES = ("lexical_modulated", "lexical_object", "lexical_channel_modulated",
                     "lexical_channel_object", "lexical_object_micro_expert")


def _check_ids(hidden_states: torch.Tensor, token_ids: Optional[torch.Tensor], kind: str):
    if token_ids is None:
        raise ValueError(f"token_ids are required for the {kind} MLP")
    if token_ids.shape != hidden_states.shape[:-1]:
        raise ValueError(f"token_ids shape {tuple(token_ids.shape)} must match hidden state "
                         f"prefix shape {tuple(hidden_states.shape[:-1])}")


class _LexicalBase(nn.Module):
    def __init__(self, config):
        super().__init__()
        H = config.hidden_size
        self.hidden_size = H
        self.intermediate_size = int(config.intermediate_size)
        self.object_rank = int(config.lexical_object_rank)
        bias = bool(getattr(config, "bias", False))
        self.shared_gate = nn.Linear(H, self.intermediate_size, bias=bias)
        self.shared_up = nn.Linear(H, self.intermediate_size, bias=bias)
        self.shared_down = nn.Linear(self.intermediate_size, H, bias=bias)
        self.token_scale = nn.Embedding(config.vocab_size, self.object_rank)
        nn.init.zeros_(self.token_scale.weight)
        self.object_output_gate = nn.Parameter(torch.tensor(float(config.lexical_object_gate_init)))
        self._tied_scale = None  # model-level shared table (not a submodule of this layer)

    def tie_token_scale(self, table: nn.Embedding) -> None:
        """Use the model's shared ``lexical_token_scale`` instead of a per-layer table."""
        if hasattr(self, "token_scale"):
            del self.token_scale
        self._tied_scale = [table]

    def scale_values(self, token_ids: torch.Tensor, values: Optional[torch.Tensor]):
        if values is not None:
            return values
        table = self._tied_scale[0] if self._tied_scale is not None else self.token_scale
        return table(token_ids)

    def shared_swiglu(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> torch.Tensor:
        """residual + down(silu(gate x) * up x); fused kernels on CUDA bf16."""
        if (use_fused(x) and x.dtype == torch.bfloat16 and self.intermediate_size % 256 == 0
                and self.shared_gate.bias is None):
            from ..ops.fused import pack_shared_gate_up, trhash_mlp

            w_gu = pack_shared_gate_up(self.shared_gate.weight, self.shared_up.weight)
            return trhash_mlp(x, w_gu, self.shared_down.weight, None, residual,
                              self.intermediate_size, 1, 0, 1.0)
        out = self.shared_down(F.silu(self.shared_gate(x)) * self.shared_up(x))
        return out if residual is None else residual + out

    def training_control_capabilities(self) -> frozenset:
        return frozenset({"lexical_object_gate"})

    def training_telemetry(self) -> dict:
        return {"object_gate": float(self.object_output_gate.detach().float().item())}


@register_mlp("lexical_modulated")
@register_mlp("lexical_object")
class LexicalModulatedMLP(_LexicalBase):
    def __init__(self, config):
        super().__init__(config)
        self.object_up = nn.Linear(self.hidden_size, self.object_rank, bias=False)
        self.object_down = nn.Linear(self.object_rank, self.hidden_size, bias=False)

    def object_residual(self, x, token_ids, values):
        scale = 1.0 + self.scale_values(token_ids, values)
        return self.object_output_gate * self.object_down(F.silu(self.object_up(x)) * scale)

    def forward(self, hidden_states, token_ids=None, residual=None,
                lexical_token_scale_values=None, **kw):
        _check_ids(hidden_states, token_ids, "lexical_modulated")
        out = self.shared_swiglu(hidden_states, residual)
        return out + self.object_residual(hidden_states, token_ids,
                                          lexical_token_scale_values).to(out.dtype)


@register_mlp("lexical_channel_modulated")
@register_mlp("lexical_channel_object")
class LexicalChannelModulatedMLP(_LexicalBase):
    def forward(self, hidden_states, token_ids=None, residual=None,
                lexical_token_scale_values=None, **kw):
        _check_ids(hidden_states, token_ids, "lexical_channel_modulated")
        x = hidden_states
        channels = F.silu(self.shared_gate(x)) * self.shared_up(x)
        block = math.ceil(self.intermediate_size / self.object_rank)
        per_rank = self.scale_values(token_ids, lexical_token_scale_values)
        mod = per_rank.repeat_interleave(block, dim=-1)[..., :self.intermediate_size]
        out = self.shared_down(channels * (1.0 + self.object_output_gate * mod).to(channels.dtype))
        return out if residual is None else residual + out


@register_mlp("lexical_object_micro_expert")
class LexicalObjectMicroExpertMLP(LexicalModulatedMLP):
    def __init__(self, config):
        super().__init__(config)
        self.micro_num_experts = int(config.micro_num_experts)
        self.micro_expert_width = int(config.micro_expert_width)
        width = self.micro_num_experts * self.micro_expert_width
        self.micro_gate = nn.Linear(self.hidden_size, width, bias=False)
        self.micro_up = nn.Linear(self.hidden_size, width, bias=False)
        self.micro_down = nn.Parameter(torch.empty(self.micro_num_experts,
                                                   self.micro_expert_width, self.hidden_size))
        nn.init.kaiming_uniform_(self.micro_down, a=math.sqrt(5))
        self.micro_output_gate = nn.Parameter(torch.tensor(float(config.micro_expert_gate_init)))
        ids = torch.arange(config.vocab_size, dtype=torch.long)
        self.register_buffer("token_to_micro_expert",
                             (ids + int(config.layer_idx)) % self.micro_num_experts)

    def forward(self, hidden_states, token_ids=None, residual=None,
                lexical_token_scale_values=None, **kw):
        out = super().forward(hidden_states, token_ids, residual, lexical_token_scale_values)
        x = hidden_states
        E, W = self.micro_num_experts, self.micro_expert_width
        h = (F.silu(self.micro_gate(x)) * self.micro_up(x)).view(*x.shape[:-1], E, W)
        e = self.token_to_micro_expert[token_ids]
        # one [.., W] x [W, H] product per micro expert, kept for its own tokens
        sel = None
        for j in range(E):
            part = (h[..., j, :] @ self.micro_down[j]) * (e == j).unsqueeze(-1).to(h.dtype)
            sel = part if sel is None else sel + part
        return out + (self.micro_output_gate * sel).to(out.dtype)

    def training_control_capabilities(self) -> frozenset:
        return super().training_control_capabilities() | {"micro_expert_gate"}

    def training_telemetry(self) -> dict:
        t = super().training_telemetry()
        t["micro_gate"] = float(self.micro_output_gate.detach().float().item())
        return t
