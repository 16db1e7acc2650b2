"""Research fast-weight memories: token-addressed associative attention variants.

Counterparts of complexity/experiments/shared_associative_attention.py
(``SharedAssociativeAttention`` :14-103, ``SharedContextFusion`` :105-140,
``StableDeltaAssociativeAttention`` :142-299, ``MultiOrderLexicalDeltaAttention``
:301-432, ``MultiTimescaleDeltaAttention`` :434-553,
``CollisionNormalizedDeltaAttention`` :555-669, ``LexicalValueDeltaAttention``
:671-755, ``LexicalForgeDeltaAttention`` :757-852,
``CollisionNormalizedLexicalForgeDeltaAttention`` :860-922 and
``PositionAwareCollisionForgeDeltaAttention`` :924-1001).  The class names,
constructor arguments, parameter names (so state dicts load across) and the
caller-owned state tuples are kept; the implementation is one configurable
module, ``FastWeightMemory``, whose options each variant switches on.

Every variant runs the same recurrence per sequence, on a [rank, rank] state S:

  write key k_t = w_{t-1} (the previous position's write code), query q_t
  S_{t+1} = d S_t + rate k_t e_t^T,   read r_t = q_t^T S_t
  e_t = v_t                    (mode "decay": plain decayed outer products)
  e_t = v_t - S_t^T k_t        (mode "delta": only what S does not predict)

evaluated chunk by chunk, exactly: with D_ij = d^(i-1-j) (j < i) and
P = diag(d^i), the scaled writes E of a chunk solve one unit lower-triangular
system (I + rate (K K^T o D)) E = rate (V - P K S_0) (E = rate V in decay
mode), reads are P Q S_0 + (Q K^T o D) E and S leaves as d^C S_0 + K^T
(d^(C-1-j) o E).  ``d`` and ``rate`` may differ per batch row, which is how
value-channel groups with their own timescale run in one batched solve.

Options layered on the addresses:
  * lexical codes normalize(sin(id * pi * sqrt(j))), j = 1..rank, mixed with a
    contextual direction (projected hidden state, or a low-rank "signature")
    by tanh(contextual_mix), and optionally a position signature;
  * a "forge": separate read and write codes from per-dimension log-scales
    (clamped to [-2, 2]) and an optional token-embedding modulation;
  * collision normalisation: a decayed running load sum_j d^(t-1-j) k_j^2 per
    state dimension rescales keys and queries by rsqrt(load + 1e-4), so
    dimensions that many tokens write to stop dominating;
  * lexical values normalize(cos((id + 1/2) pi sqrt(j))), j = rank+1..2 rank,
    instead of projected hidden states;
  * n-gram addresses (sum of rotated lexical codes of the last n ids).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

_LOAD_EPS = 1e-4


# ------------------------------------------------------------------ codes
def sin_codes(ids: torch.Tensor, rank: int) -> torch.Tensor:
    """Unit lexical codes normalize(sin(id * pi * sqrt(j))), j = 1..rank (fp64 phases)."""
    j = torch.arange(1, rank + 1, device=ids.device, dtype=torch.float64)
    return F.normalize((ids.double()[..., None] * math.pi * j.sqrt()).sin().float(), dim=-1)


def cos_value_codes(ids: torch.Tensor, rank: int) -> torch.Tensor:
    """Unit lexical value codes normalize(cos((id + 0.5) pi sqrt(j))), j = rank+1..2 rank."""
    j = torch.arange(rank + 1, 2 * rank + 1, device=ids.device, dtype=torch.float64)
    return F.normalize(((ids.double()[..., None] + 0.5) * math.pi * j.sqrt()).cos().float(),
                       dim=-1)


def position_codes(pos: torch.Tensor, rank: int) -> torch.Tensor:
    """Unit position signatures normalize(sin(pi (p + 1) sqrt(j))) (fp32 phases)."""
    j = torch.arange(1, rank + 1, device=pos.device, dtype=torch.float32)
    return F.normalize(torch.sin(math.pi * (pos.float()[..., None] + 1.0) * j.sqrt()), dim=-1)


# ------------------------------------------------------------------- scan
def _causal_decay(d: torch.Tensor, C: int) -> torch.Tensor:
    """[B, C, C] with d^(i-1-j) below the diagonal, 0 elsewhere (d: [B])."""
    t = torch.arange(C, device=d.device, dtype=torch.float32)
    dist = t[:, None] - t[None, :] - 1
    return torch.where(dist >= 0, d[:, None, None] ** dist.clamp_min(0), torch.zeros_like(dist))


def chunk_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, S: torch.Tensor,
               d: torch.Tensor, rate: torch.Tensor, delta: bool
               ) -> Tuple[torch.Tensor, torch.Tensor]:
    """One chunk of the recurrence: (reads [B, C, n], S_next [B, r, n]).

    q, k: [B, C, r]; v: [B, C, n]; S: [B, r, n]; d, rate: [B] (fp32).
    """
    B, C, _ = k.shape
    D = _causal_decay(d, C)
    t = torch.arange(C, device=k.device, dtype=torch.float32)
    P = (d[:, None] ** t[None])[..., None]
    r3 = rate[:, None, None]
    if delta:
        A = torch.eye(C, device=k.device) + r3 * (k @ k.transpose(1, 2)) * D
        E = torch.linalg.solve_triangular(A, r3 * (v - P * (k @ S)), upper=False,
                                          unitriangular=True)
    else:
        E = r3 * v
    reads = P * (q @ S) + ((q @ k.transpose(1, 2)) * D) @ E
    tail = (d[:, None] ** (C - 1 - t)[None])[..., None]
    S = d[:, None, None] ** C * S + k.transpose(1, 2) @ (E * tail)
    return reads, S


def collision_normalise(k: torch.Tensor, q: torch.Tensor, load: torch.Tensor, d: torch.Tensor,
                        rate: torch.Tensor):
    """Rescale one chunk's keys/queries by the decayed per-dimension write load.

    load_t = d^t load_0 + rate sum_{j<t} d^(t-1-j) k_j^2 (raw keys) is the load
    before position t; keys and queries become normalize(x * rsqrt(load_t +
    1e-4)); the load leaving the chunk is d^C load_0 + rate sum_j d^(C-1-j) k_j^2.
    """
    B, C, _ = k.shape
    D = _causal_decay(d, C)
    t = torch.arange(C, device=k.device, dtype=torch.float32)
    k2 = k.square()
    before = (d[:, None] ** t[None])[..., None] * load[:, None] + rate[:, None, None] * (D @ k2)
    scale = torch.rsqrt(before + _LOAD_EPS)
    tail = (d[:, None] ** (C - 1 - t)[None])[..., None]
    nxt = d[:, None] ** C * load + rate[:, None] * (k2 * tail).sum(1)
    return F.normalize(k * scale, dim=-1), F.normalize(q * scale, dim=-1), nxt


# ----------------------------------------------------------------- module
class FastWeightMemory(nn.Module):
    """Configurable token-addressed fast-weight memory; ``forward(h, ids, state)``
    returns ``(residual, next_state)``.  The variants below are presets."""

    def __init__(self, hidden_size: int, rank: int, vocab_size: Optional[int] = None, *,
                 delta: bool = True, contextual_mix_init: float = 0.1,
                 output: str = "residual", output_gate_init: float = 1.0,
                 residual_scale: float = 0.1, chunk_size: int = 512,
                 address: str = "projection", context_signature_rank: int = 8,
                 position: bool = False, forge: bool = False, lexical_object_rank: int = 16,
                 forge_bottleneck: int = 4, collision: bool = False,
                 lexical_values: bool = False, timescales: int = 0,
                 fusion_size: int = 0, fusion_scale: float = 0.1):
        super().__init__()
        self.hidden_size, self.rank = int(hidden_size), int(rank)
        self.delta, self.chunk = bool(delta), int(chunk_size)
        self.output_mode, self.address_mode = output, address
        self.position, self.forge, self.collision = position, forge, collision
        self.lexical_values = lexical_values
        self.residual_scale = float(residual_scale)
        self.state_rank = self.rank
        if not lexical_values:
            self.value_proj = nn.Linear(hidden_size, rank, bias=False)
        if output == "fusion":
            self.fusion_gate = nn.Linear(hidden_size, fusion_size, bias=False)
            self.fusion_value = nn.Linear(rank, fusion_size, bias=False)
            self.fusion_out = nn.Linear(fusion_size, hidden_size, bias=False)
            self.fusion_scale = float(fusion_scale)
        else:
            self.output_proj = nn.Linear(rank, hidden_size, bias=False)
        if output == "gate":
            self.output_gate = nn.Parameter(torch.tensor(float(output_gate_init)))
        if address == "projection":
            self.address_proj = nn.Linear(hidden_size, rank, bias=False)
        elif address == "signature":
            self.context_down = nn.Linear(hidden_size, context_signature_rank, bias=False)
            self.context_up = nn.Linear(context_signature_rank, rank, bias=False)
        if address != "none":
            self.contextual_mix = nn.Parameter(torch.tensor(float(contextual_mix_init)))
        if position:
            self.position_gate = nn.Parameter(torch.tensor(0.0))
        if forge:
            self.read_log_scale = nn.Parameter(torch.zeros(rank))
            self.write_log_scale = nn.Parameter(torch.zeros(rank))
            self.forge_down = nn.Linear(lexical_object_rank, forge_bottleneck, bias=False)
            self.forge_up = nn.Linear(forge_bottleneck, rank, bias=False)
            self.lexical_token_scale: Optional[nn.Embedding] = None
        self.timescales = int(timescales)
        if timescales:
            if rank % timescales:
                raise ValueError("state_rank must be divisible by num_timescales")
            self.num_timescales, self.group_size = int(timescales), rank // timescales
            self.decay_logits = nn.Parameter(torch.logit(torch.linspace(0.95, 0.9995,
                                                                        timescales)))
            self.write_logits = nn.Parameter(torch.full((timescales,), math.log(4.0)))
        else:
            # write rate 0.9 and decay 0.999 at init (logits log 9, log 999)
            self.write_logit = nn.Parameter(torch.tensor(2.197225))
            self.decay_logit = nn.Parameter(torch.tensor(6.906755))
        table = sin_codes(torch.arange(vocab_size), rank) if vocab_size else torch.empty(0, rank)
        self.register_buffer("address_table", table, persistent=False)
        if lexical_values:
            vt = (cos_value_codes(torch.arange(vocab_size), rank) if vocab_size
                  else torch.empty(0, rank))
            self.register_buffer("value_table", vt, persistent=False)

    # ----------------------------------------------------------- pieces
    def attach_token_scale(self, token_scale: nn.Embedding) -> None:
        """Modulate the forged codes by a (shared) per-token embedding."""
        if not self.forge:
            raise RuntimeError("this memory has no lexical forge")
        if token_scale.embedding_dim != self.forge_down.in_features:
            raise ValueError(f"token_scale rank {token_scale.embedding_dim} does not match "
                             f"forge rank {self.forge_down.in_features}")
        self.lexical_token_scale = token_scale

    def _lex(self, ids: torch.Tensor) -> torch.Tensor:
        t = self.address_table
        return F.embedding(ids, t) if t.numel() else sin_codes(ids, self.rank)

    def _values(self, h: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        if self.lexical_values:
            t = self.value_table
            return F.embedding(ids, t) if t.numel() else cos_value_codes(ids, self.rank)
        return self.value_proj(h).float()

    def _rates(self, B: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        if self.timescales:
            d = torch.sigmoid(self.decay_logits.float()).repeat(B)
            w = torch.sigmoid(self.write_logits.float()).repeat(B)
        else:
            d = torch.sigmoid(self.decay_logit.float()).expand(B)
            w = torch.sigmoid(self.write_logit.float()).expand(B)
        return d, w

    def _contextual(self, h: torch.Tensor) -> Optional[torch.Tensor]:
        if self.address_mode == "projection":
            return F.normalize(self.address_proj(h).float(), dim=-1)
        if self.address_mode == "signature":
            return F.normalize(self.context_up(F.silu(self.context_down(h))).float(), dim=-1)
        return None

    def codes(self, h: torch.Tensor, ids: torch.Tensor, start: Optional[torch.Tensor] = None
              ) -> Tuple[torch.Tensor, torch.Tensor]:
        """(read codes, write codes) [B, S, rank] in fp32."""
        lex = self._lex(ids).float()
        if self.forge:
            if self.lexical_token_scale is not None:
                mod = self.forge_up(F.silu(self.forge_down(self.lexical_token_scale(ids))))
                lex = F.normalize(lex + mod.float(), dim=-1)
            rd = F.normalize(lex * torch.exp(self.read_log_scale.float().clamp(-2, 2)), dim=-1)
            wr = F.normalize(lex * torch.exp(self.write_log_scale.float().clamp(-2, 2)), dim=-1)
        else:
            rd = wr = lex
        extra = None
        ctx = self._contextual(h)
        if ctx is not None:
            extra = torch.tanh(self.contextual_mix.float()) * ctx
        if self.position:
            pos = start[:, None] + torch.arange(ids.shape[1], device=ids.device)[None]
            p = torch.tanh(self.position_gate.float()) * position_codes(pos, self.rank)
            extra = p if extra is None else extra + p
        if extra is not None:
            rd = F.normalize(rd + extra, dim=-1)
            wr = rd if not self.forge else F.normalize(wr + extra, dim=-1)
        return rd, wr

    def _output(self, h: torch.Tensor, reads: torch.Tensor) -> torch.Tensor:
        if self.output_mode == "fusion":
            fused = F.silu(self.fusion_gate(h)) * self.fusion_value(reads.to(h.dtype))
            return self.fusion_scale * self.fusion_out(fused)
        out = self.output_proj(reads.to(self.output_proj.weight.dtype))
        return self.output_gate * out if self.output_mode == "gate" else self.residual_scale * out

    # ----------------------------------------------------------- state
    def initial_state(self, batch_size: int, *, device=None, dtype=None) -> Tuple:
        S = torch.zeros(batch_size, self.rank, self.rank, device=device)
        prev = torch.zeros(batch_size, self.rank, device=device)
        st = [S, prev]
        if self.collision:
            st.append(torch.zeros(batch_size, self.rank, device=device))
        if self.position:
            st.append(torch.zeros(batch_size, device=device, dtype=torch.int64))
        return tuple(st)

    def forward(self, hidden_states: torch.Tensor, token_ids: torch.Tensor, state: Tuple
                ) -> Tuple[torch.Tensor, Tuple]:
        S, prev = state[0].float(), state[1].float()
        load = state[2].float() if self.collision else None
        start = state[-1] if self.position else None
        B, L = token_ids.shape
        rd, wr = self.codes(hidden_states, token_ids, start)
        v = self._values(hidden_states, token_ids)
        d, w = self._rates(B, token_ids.device)
        G = self.timescales or 1
        reads = []
        for c0 in range(0, L, self.chunk):
            qc, wc, vc = rd[:, c0:c0 + self.chunk], wr[:, c0:c0 + self.chunk], v[:, c0:c0 + self.chunk]
            kc = torch.cat((prev[:, None], wc[:, :-1]), 1)
            prev = wc[:, -1]
            if self.collision:
                dd, ww = (d, w) if G == 1 else (d[::G], w[::G])
                kc, qc, load = collision_normalise(kc, qc, load, dd, ww)
            if G == 1:
                rc, S = chunk_scan(qc, kc, vc, S, d, w, self.delta)
            else:
                # value channel groups as batch rows, each with its own timescale
                C, g = kc.shape[1], self.group_size
                rep = lambda x: x[:, None].expand(-1, G, -1, -1).reshape(B * G, C, -1)  # noqa: E731
                vg = vc.reshape(B, C, G, g).transpose(1, 2).reshape(B * G, C, g)
                Sg = S.reshape(B, self.rank, G, g).transpose(1, 2).reshape(B * G, self.rank, g)
                rg, Sg = chunk_scan(rep(qc), rep(kc), vg, Sg, d, w, self.delta)
                S = Sg.reshape(B, G, self.rank, g).transpose(1, 2).reshape(B, self.rank,
                                                                           self.rank)
                rc = rg.reshape(B, G, C, g).transpose(1, 2).reshape(B, C, self.rank)
            reads.append(rc)
        out = self._output(hidden_states, torch.cat(reads, 1))
        nxt = [S, prev]
        if self.collision:
            nxt.append(load)
        if self.position:
            nxt.append(start + L)
        return out, tuple(nxt)


# ----------------------------------------------------------------- presets
class SharedAssociativeAttention(FastWeightMemory):
    """Decayed outer-product memory (no delta), scalar output gate, 256-position
    chunks.  A zero ``contextual_mix_init`` fixes lexical-only addresses (the
    contextual branch then never runs, as in the reference)."""

    def __init__(self, hidden_size: int, rank: int, vocab_size: Optional[int] = None,
                 output_gate_init: float = 1.0, contextual_mix_init: float = 0.0):
        super().__init__(hidden_size, rank, vocab_size, delta=False,
                         contextual_mix_init=contextual_mix_init, output="gate",
                         output_gate_init=output_gate_init, chunk_size=256)
        self.contextual_enabled = contextual_mix_init != 0.0

    def _contextual(self, h):
        return super()._contextual(h) if self.contextual_enabled else None


class SharedContextFusion(FastWeightMemory):
    """Decayed memory whose reads are fused token by token:
    fusion_scale * W_out(silu(W_gate h) * W_val reads)."""

    def __init__(self, hidden_size: int, rank: int, fusion_size: int,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 fusion_scale: float = 0.1):
        super().__init__(hidden_size, rank, vocab_size, delta=False,
                         contextual_mix_init=contextual_mix_init, output="fusion",
                         chunk_size=256, fusion_size=fusion_size, fusion_scale=fusion_scale)


class StableDeltaAssociativeAttention(FastWeightMemory):
    """Error-correcting (delta) writes, residual_scale * W_out reads."""

    def __init__(self, hidden_size: int, rank: int, vocab_size: Optional[int] = None,
                 contextual_mix_init: float = 0.1, residual_scale: float = 0.1,
                 delta_chunk_size: int = 512):
        super().__init__(hidden_size, rank, vocab_size, contextual_mix_init=contextual_mix_init,
                         residual_scale=residual_scale, chunk_size=delta_chunk_size)


class MultiTimescaleDeltaAttention(FastWeightMemory):
    """Delta memory whose value channels form ``num_timescales`` groups, each with
    its own learned decay (initialised 0.95 .. 0.9995) and write rate."""

    def __init__(self, hidden_size: int, state_rank: int = 128, num_timescales: int = 4,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, timescales=num_timescales)


class CollisionNormalizedDeltaAttention(FastWeightMemory):
    """Delta memory with keys and queries rescaled by the decayed write load of
    each state dimension (state: matrix, previous write code, load)."""

    def __init__(self, hidden_size: int, state_rank: int = 128,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, collision=True)


class LexicalValueDeltaAttention(FastWeightMemory):
    """Delta memory that writes deterministic token value codes (no value projection)."""

    def __init__(self, hidden_size: int, state_rank: int = 128,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, lexical_values=True)
        self.lexical_value_rank = int(state_rank)


class LexicalForgeDeltaAttention(FastWeightMemory):
    """Delta memory with forged read / write codes (per-dimension log-scales and an
    optional token-embedding modulation) mixed with the contextual direction."""

    def __init__(self, hidden_size: int, state_rank: int = 128,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 lexical_object_rank: int = 16, forge_bottleneck: int = 4,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, forge=True,
                         lexical_object_rank=lexical_object_rank,
                         forge_bottleneck=forge_bottleneck)


class CollisionNormalizedLexicalForgeDeltaAttention(FastWeightMemory):
    """Forged codes plus collision normalisation."""

    def __init__(self, hidden_size: int, state_rank: int = 128,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 lexical_object_rank: int = 16, forge_bottleneck: int = 4,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, forge=True, collision=True,
                         lexical_object_rank=lexical_object_rank,
                         forge_bottleneck=forge_bottleneck)


class PositionAwareCollisionForgeDeltaAttention(FastWeightMemory):
    """Forged, collision-normalised codes whose "occurrence" term mixes a compact
    context signature (hidden -> rank ``context_signature_rank`` -> state rank)
    with a position signature gated by tanh(position_gate); the state carries
    the absolute position of the next token."""

    def __init__(self, hidden_size: int, state_rank: int = 128,
                 vocab_size: Optional[int] = None, contextual_mix_init: float = 0.1,
                 lexical_object_rank: int = 16, forge_bottleneck: int = 4,
                 residual_scale: float = 0.1, delta_chunk_size: int = 512,
                 context_signature_rank: int = 8):
        super().__init__(hidden_size, state_rank, vocab_size,
                         contextual_mix_init=contextual_mix_init, residual_scale=residual_scale,
                         chunk_size=delta_chunk_size, forge=True, collision=True,
                         lexical_object_rank=lexical_object_rank,
                         forge_bottleneck=forge_bottleneck, address="signature",
                         context_signature_rank=context_signature_rank, position=True)


class _OrderHead(FastWeightMemory):
    def __init__(self, hidden_size: int, rank: int, chunk: int):
        super().__init__(hidden_size, rank, None, address="none", residual_scale=1.0,
                         chunk_size=chunk)


class MultiOrderLexicalDeltaAttention(nn.Module):
    """One delta memory per n-gram order; order n addresses position t by
    normalize(sum_{lag < n} roll(lex(id_{t-lag}), 7 lag mod rank)) over the ids
    seen so far (a history of the last max_order - 1 ids crosses calls).
    residual = residual_scale / sqrt(#orders) * sum of the heads' outputs."""

    def __init__(self, hidden_size: int, head_rank: int = 32,
                 orders: Sequence[int] = (1, 2, 4, 8), vocab_size: Optional[int] = None,
                 delta_chunk_size: int = 512, residual_scale: float = 0.1):
        super().__init__()
        del vocab_size
        self.hidden_size, self.head_rank = int(hidden_size), int(head_rank)
        self.orders = tuple(int(o) for o in orders)
        self.max_order = max(self.orders)
        self.delta_chunk_size = int(delta_chunk_size)
        self.residual_scale = float(residual_scale)
        self.heads = nn.ModuleList(_OrderHead(hidden_size, head_rank, delta_chunk_size)
                                   for _ in self.orders)

    def initial_state(self, batch_size: int, *, device=None, dtype=None):
        n = len(self.orders)
        return (torch.zeros(batch_size, n, self.head_rank, self.head_rank, device=device),
                torch.zeros(batch_size, n, self.head_rank, device=device),
                torch.full((batch_size, self.max_order - 1), -1, device=device,
                           dtype=torch.int64))

    def ngram_codes(self, token_ids: torch.Tensor, history: torch.Tensor, order: int):
        ids = torch.cat((history, token_ids), 1)
        L, h = token_ids.shape[1], self.max_order - 1
        acc = torch.zeros(*token_ids.shape, self.head_rank, device=token_ids.device)
        for lag in range(order):
            lagged = ids[:, h - lag:h - lag + L]
            code = sin_codes(lagged.clamp_min(0), self.head_rank)
            acc = acc + code.roll((lag * 7) % self.head_rank, -1) * (lagged >= 0)[..., None]
        return F.normalize(acc, dim=-1)

    def forward(self, hidden_states: torch.Tensor, token_ids: torch.Tensor, state):
        mats, prevs, history = state
        total, nm, npv = 0.0, [], []
        for i, (order, head) in enumerate(zip(self.orders, self.heads)):
            a = self.ngram_codes(token_ids, history, order)
            B = token_ids.shape[0]
            S, prev = mats[:, i].float(), prevs[:, i].float()
            v = head.value_proj(hidden_states).float()
            d, w = head._rates(B, token_ids.device)
            reads = []
            for c0 in range(0, token_ids.shape[1], self.delta_chunk_size):
                qc = a[:, c0:c0 + self.delta_chunk_size]
                kc = torch.cat((prev[:, None], qc[:, :-1]), 1)
                prev = qc[:, -1]
                rc, S = chunk_scan(qc, kc, v[:, c0:c0 + self.delta_chunk_size], S, d, w, True)
                reads.append(rc)
            total = total + head.output_proj(torch.cat(reads, 1).to(head.output_proj.weight.dtype))
            nm.append(S)
            npv.append(prev)
        hist = torch.cat((history, token_ids), 1)[:, history.shape[1] + token_ids.shape[1]
                                                  - (self.max_order - 1):]
        res = self.residual_scale / math.sqrt(len(self.orders)) * total
        return res, (torch.stack(nm, 1), torch.stack(npv, 1), hist)
