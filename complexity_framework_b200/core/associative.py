"""Fast-weight associative memory: a token-addressed [rank, rank] state that
causal mixers read and write along the sequence.

Counterparts: complexity/core/context/associative.py:14-126
(``SharedAssociativeContext``: fixed lexical addresses) and
complexity/experiments/shared_associative_attention.py:14-104 and 142-300
(``SharedAssociativeAttention`` with learned contextual addresses,
``StableDeltaAssociativeAttention`` with error-correcting writes).

Model, per sequence (b omitted):
  address a_t = normalize(lex(id_t) + tanh(mix) * normalize(W_a h_t))
  value   v_t = W_v h_t                                  [rank]
  write key k_t = a_{t-1} (the previous token's address: the memory learns
  "what followed this context"), read query q_t = a_t
  state   S_{t+1} = d S_t + w k_t e_t^T,   read r_t = q_t^T S_t
  e_t = v_t                        (mode "decay")
  e_t = v_t - S_t^T k_t            (mode "delta": write only what the memory
                                    does not already predict)
with d = sigmoid(decay_logit), w = sigmoid(write_logit).  ``lex(id)`` is the
fixed unit vector normalize(sin(id * pi * sqrt(j))), j = 1..rank.

Chunked evaluation (C positions at a time, exact): with P = diag(d^i) and the
causal decay matrix D_ij = d^(i-1-j) for j < i (else 0), the scaled write
terms E = w e solve the unit lower-triangular system
  (I + w (K K^T o D)) E = w (V - P K S_0)       (delta; E = w V for decay),
reads are R = P Q S_0 + (Q K^T o D) E, and the state leaving the chunk is
d^C S_0 + K^T (d^(C-1-j) o E).  Everything is batched matmuls plus one
triangular solve per chunk; fp32 throughout.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def lexical_addresses(token_ids: torch.Tensor, rank: int) -> torch.Tensor:
    j = torch.arange(1, rank + 1, device=token_ids.device, dtype=torch.float64)
    ph = token_ids.double()[..., None] * math.pi * j.sqrt()
    return F.normalize(ph.sin().float(), dim=-1)


def associative_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: torch.Tensor,
                     decay: torch.Tensor, write: torch.Tensor, delta: bool,
                     chunk: int = 256) -> Tuple[torch.Tensor, torch.Tensor]:
    """Reads [B, S, r] and the final state [B, r, r] of the recurrence above."""
    q, k, v, S = q.float(), k.float(), v.float(), state.float()
    d, w = decay.float(), write.float()
    reads = []
    for c0 in range(0, q.shape[1], chunk):
        qc, kc, vc = q[:, c0:c0 + chunk], k[:, c0:c0 + chunk], v[:, c0:c0 + chunk]
        C = qc.shape[1]
        t = torch.arange(C, device=q.device, dtype=torch.float32)
        dist = t[:, None] - t[None, :] - 1
        D = torch.where(dist >= 0, d ** dist.clamp_min(0), torch.zeros_like(dist))
        P = (d ** t)[None, :, None]
        if delta:
            A = torch.eye(C, device=q.device) + w * (kc @ kc.transpose(1, 2)) * D
            rhs = w * (vc - P * (kc @ S))
            E = torch.linalg.solve_triangular(A, rhs, upper=False, unitriangular=True)
        else:
            E = w * vc
        reads.append(P * (qc @ S) + ((qc @ kc.transpose(1, 2)) * D) @ E)
        tail = (d ** (C - 1 - t))[None, :, None]
        S = d ** C * S + kc.transpose(1, 2) @ (E * tail)
    return torch.cat(reads, 1), S


class AssociativeMemory(nn.Module):
    """Reads from / writes to the fast-weight state; returns (residual, state)."""

    def __init__(self, hidden_size: int, rank: int, *, delta: bool = False,
                 contextual_mix_init: float = 0.0, output_gate_init: float = 1.0,
                 chunk_size: int = 256):
        super().__init__()
        self.rank, self.delta, self.chunk = int(rank), bool(delta), int(chunk_size)
        self.value_proj = nn.Linear(hidden_size, rank, bias=False)
        self.output_proj = nn.Linear(rank, hidden_size, bias=False)
        self.address_proj = nn.Linear(hidden_size, rank, bias=False)
        self.contextual_mix = nn.Parameter(torch.tensor(float(contextual_mix_init)))
        self.output_gate = nn.Parameter(torch.tensor(float(output_gate_init)))
        # write rate 0.9 and decay 0.999 at init
        self.write_logit = nn.Parameter(torch.tensor(math.log(9.0)))
        self.decay_logit = nn.Parameter(torch.tensor(math.log(999.0)))

    def initial_state(self, batch: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        return (torch.zeros(batch, self.rank, self.rank, device=device),
                torch.zeros(batch, self.rank, device=device))

    def forward(self, h: torch.Tensor, token_ids: torch.Tensor,
                state: Optional[Tuple[torch.Tensor, torch.Tensor]] = None):
        B = h.shape[0]
        S0, prev = state if state is not None else self.initial_state(B, h.device)
        a = lexical_addresses(token_ids, self.rank)
        ctx = F.normalize(self.address_proj(h).float(), dim=-1)
        a = F.normalize(a + torch.tanh(self.contextual_mix.float()) * ctx, dim=-1)
        k = torch.cat((prev.float()[:, None], a[:, :-1]), 1)
        v = self.value_proj(h)
        reads, S = associative_scan(a, k, v, S0, torch.sigmoid(self.decay_logit),
                                    torch.sigmoid(self.write_logit), self.delta, self.chunk)
        out = self.output_gate * self.output_proj(reads.to(self.output_proj.weight.dtype))
        return out, (S, a[:, -1])
