"""``ComplexityModel``: embedding -> N decoder blocks -> final norm -> (tied) LM head.

Public surface as complexity/models/builder.py:51-743: the constructor
initialisation (N(0, 0.02) for Linear/Embedding, residual projections o_proj,
expert_down and shared_down at 0.02/sqrt(2N), optional muP scaling), the
forward signature and returned dict, activation checkpointing,
``save_pretrained``/``from_pretrained`` (config.json + model.safetensors,
collective gather when sharded), ``from_preset`` and ``num_parameters``.

Differences by design: on CUDA bf16 the forward runs the sm_100a kernels;
``generate`` works (through the paged-KV inference engine) instead of raising;
``loss`` fuses the LM head with the cross-entropy.
"""
from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Any, Dict, List, Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as activation_checkpoint

from ..config.model_config import ModelConfig, get_preset
from ..core.layers import use_fused
from ..core.registry import NORMALIZATION_REGISTRY
from .block import TransformerBlock

_DETERMINISTIC_BUFFER = re.compile(
    r"\.(inv_freq|token_to_expert|pair_hash_route_codes|pair_hash_expert_pairs)$")


def build_lexical_zipf_weights(counts: torch.Tensor, *, mode: str, alpha: float, floor: float,
                               permutation_seed: int) -> torch.Tensor:
    """Per-token weights (rank / V)^alpha over descending-frequency ranks (ties
    keep vocabulary order), floored at ``floor``, scaled to unit RMS; ``permuted``
    shuffles them with a seeded permutation (a frequency-blind control).
    Mirrors complexity/models/builder.py:22-48."""
    if counts.ndim != 1:
        raise ValueError("Zipf counts must be a 1D tensor")
    if mode not in ("ordered", "permuted"):
        raise ValueError(f"Unsupported Zipf mode: {mode}")
    if alpha <= 0.0:
        raise ValueError("lexical_zipf_alpha must be positive")
    if not 0.0 <= floor <= 1.0:
        raise ValueError("lexical_zipf_floor must lie in [0, 1]")
    V = counts.numel()
    order = torch.argsort(counts.double(), descending=True, stable=True)
    rank = torch.empty(V, dtype=torch.float32)
    rank[order] = torch.arange(1, V + 1, dtype=torch.float32)
    w = (rank / V).pow(float(alpha)).clamp_min(float(floor))
    w = w / w.square().mean().sqrt().clamp_min(1e-12)
    if mode == "permuted":
        w = w[torch.randperm(V, generator=torch.Generator().manual_seed(int(permutation_seed)))]
    return w


class ComplexityModel(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(
            [TransformerBlock(config, layer_idx=i) for i in range(config.num_hidden_layers)])
        self.norm = NORMALIZATION_REGISTRY.build(config.norm_type, config.hidden_size,
                                                 eps=config.norm_eps)
        self.lm_head = (None if config.tie_word_embeddings
                        else nn.Linear(config.hidden_size, config.vocab_size, bias=False))
        if str(config.rope_type).lower() == "learned":
            from ..core.positions import LearnedPositionalEmbedding

            self.embed_positions = LearnedPositionalEmbedding(config.max_position_embeddings,
                                                              config.hidden_size)
        from ..core.lexical_mlp import LEXICAL_MLP_TYPES

        lexical = config.mlp_type in LEXICAL_MLP_TYPES
        if lexical and config.tie_lexical_object_embeddings:
            # one [vocab, rank] table shared by every layer, owned by the model
            self.lexical_token_scale = self.layers[0].mlp.token_scale
            for layer in self.layers:
                layer.mlp.tie_token_scale(self.lexical_token_scale)
        zipf = str(getattr(config, "lexical_zipf_mode", "uniform"))
        if zipf != "uniform":
            # persistent per-token weights from corpus frequency ranks (part of
            # the checkpoint contract of lexical configurations)
            if not config.lexical_zipf_path:
                raise ValueError("lexical_zipf_path is required for non-uniform Zipf")
            art = torch.load(config.lexical_zipf_path, map_location="cpu", weights_only=True)
            counts = art["counts"] if isinstance(art, dict) else art
            if counts.numel() != config.vocab_size:
                raise ValueError(f"Zipf counts have vocab {counts.numel()}, expected "
                                 f"{config.vocab_size}")
            self.register_buffer("lexical_zipf_weights", build_lexical_zipf_weights(
                counts, mode=zipf, alpha=float(config.lexical_zipf_alpha),
                floor=float(config.lexical_zipf_floor),
                permutation_seed=int(config.lexical_zipf_permutation_seed)), persistent=True)
        self._gradient_checkpointing = False
        self.apply(self._init_weights)
        if lexical:  # as in the reference: the first (or shared) table starts at zero
            table = (self.lexical_token_scale if hasattr(self, "lexical_token_scale")
                     else self.layers[0].mlp.token_scale)
            nn.init.zeros_(table.weight)
        self._init_residual_scaling()
        self._apply_mup_init_scaling()

    # ------------------------------------------------------------------ init
    def _init_weights(self, module: nn.Module) -> None:
        std = self.config.initializer_range
        if getattr(module, "_deterministic_init", False):
            return  # initialised from its own seeded generator
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=std)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=std)

    def _init_residual_scaling(self) -> None:
        std = self.config.initializer_range / (2 * self.config.num_hidden_layers) ** 0.5
        for layer in self.layers:
            o_proj = getattr(layer.self_attn, "o_proj", None)
            if isinstance(o_proj, nn.Linear):  # routed experts keep their zero init
                nn.init.normal_(o_proj.weight, mean=0.0, std=std)
            engine = getattr(layer.mlp, "engine", None)
            if engine is not None:
                nn.init.normal_(engine.expert_down, mean=0.0, std=std)
                if engine.shared_down is not None:
                    nn.init.normal_(engine.shared_down.weight, mean=0.0, std=std)

    def _apply_mup_init_scaling(self) -> None:
        if not self.config.use_mup_init:
            return
        mult = self.config.hidden_size / self.config.mup_base_width
        if mult <= 1.0:
            return
        s = 1.0 / mult ** 0.5
        with torch.no_grad():
            for name, module in self.named_modules():
                if isinstance(module, nn.Linear) and "embed_tokens" not in name:
                    module.weight.mul_(s)

    # --------------------------------------------------------------- helpers
    @classmethod
    def from_preset(cls, name: str) -> "ComplexityModel":
        return cls(get_preset(name))

    @classmethod
    def from_config(cls, config_path: str) -> "ComplexityModel":
        return cls(ModelConfig.load(config_path))

    def num_parameters(self, trainable_only: bool = True) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad or not trainable_only)

    def gradient_checkpointing_enable(self) -> None:
        self._gradient_checkpointing = True

    def gradient_checkpointing_disable(self) -> None:
        self._gradient_checkpointing = False

    def get_input_embeddings(self) -> nn.Embedding:
        return self.embed_tokens

    def output_weight(self) -> torch.Tensor:
        return self.lm_head.weight if self.lm_head is not None else self.embed_tokens.weight

    def set_tokenizer(self, tokenizer) -> None:
        self.tokenizer = tokenizer

    # --------------------------------------------------------------- forward
    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        w = self.embed_tokens.weight
        if input_ids.is_cuda and w.dtype == torch.bfloat16 and w.shape[1] % 8 == 0:
            from ..ops.fused import embedding

            return embedding(input_ids, w)
        return self.embed_tokens(input_ids)

    def forward(self, input_ids: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                past_key_values: Optional[List[Any]] = None, use_cache: bool = False,
                return_hidden_states: bool = False, return_logits: bool = True,
                inputs_embeds: Optional[torch.Tensor] = None,
                routing_ids: Optional[torch.Tensor] = None) -> Dict[str, Any]:
        if inputs_embeds is None:
            if input_ids is None:
                raise ValueError("input_ids or inputs_embeds must be provided")
            hidden = self.embed(input_ids)
        else:
            if inputs_embeds.ndim != 3:
                raise ValueError("inputs_embeds must have shape [batch, seq, hidden]")
            if inputs_embeds.size(-1) != self.config.hidden_size:
                raise ValueError("inputs_embeds hidden size does not match the model configuration")
            hidden = inputs_embeds
        B, S = hidden.shape[:2]
        if hasattr(self, "embed_positions"):
            past_len = 0
            if past_key_values is not None and past_key_values[0] is not None:
                past_len = past_key_values[0][0].shape[2]
            hidden = self.embed_positions(hidden, offset=past_len)
        token_ids = routing_ids if routing_ids is not None else input_ids
        if token_ids is None:
            token_ids = torch.zeros(B, S, dtype=torch.long, device=hidden.device)
        if token_ids.shape != (B, S):
            raise ValueError("routing_ids must match the embedded sequence shape")
        all_hidden = [hidden] if return_hidden_states else None
        new_kv = [] if use_cache else None
        for i, layer in enumerate(self.layers):
            past = past_key_values[i] if past_key_values is not None else None
            if self._gradient_checkpointing and self.training:
                hidden, kv, _ = activation_checkpoint(layer, hidden, attention_mask, past,
                                                      use_cache, token_ids, use_reentrant=False)
            else:
                hidden, kv, _ = layer(hidden, attention_mask=attention_mask, past_key_value=past,
                                      use_cache=use_cache, token_ids=token_ids)
            if use_cache:
                new_kv.append(kv)
            if return_hidden_states:
                all_hidden.append(hidden)
        hidden = self.norm(hidden)
        out = {"logits": None, "past_key_values": new_kv, "hidden_states": all_hidden,
               "last_hidden_state": hidden}
        if return_logits:
            out["logits"] = self.logits(hidden)
        return out

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        w = self.output_weight()
        if use_fused(hidden) and w.dtype == torch.bfloat16 and w.shape[0] % 32 == 0:
            from ..ops.fused import linear

            logits = linear(hidden, w)
        else:
            logits = F.linear(hidden, w)
        if self.config.use_mup_output_mult:
            mult = self.config.hidden_size / self.config.mup_base_width
            if mult > 1.0:
                logits = logits / mult
        return logits

    def loss(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
             ignore_index: int = -100) -> torch.Tensor:
        """Mean next-token cross-entropy; the LM head is fused with the loss on CUDA.

        ``labels`` default to ``input_ids`` shifted left by one with the last
        position of every sequence ignored, i.e. the same rows as
        ``hidden[:, :-1]`` against ``ids[:, 1:]``.
        """
        from ..core.losses import causal_lm_loss_from_hidden

        if getattr(self, "sp_ws", None) is not None and input_ids.is_cuda:
            return self._loss_sp(input_ids, labels, ignore_index)
        hidden = self(input_ids, return_logits=False)["last_hidden_state"]
        if labels is None:
            labels = torch.roll(input_ids, -1, dims=1)
            labels[:, -1] = ignore_index
        scale = 1.0
        if self.config.use_mup_output_mult:
            scale = 1.0 / max(1.0, self.config.hidden_size / self.config.mup_base_width)
        return causal_lm_loss_from_hidden(hidden, self.output_weight(), labels,
                                          ignore_index=ignore_index, logit_scale=scale)

    def _loss_sp(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor],
                 ignore_index: int) -> torch.Tensor:
        """Fused sequence-parallel TP loss: this rank embeds, normalises and scores
        its T/P token rows; attention / MLP communicate inside their GEMMs.
        Returns this rank's share of the global mean loss (shares sum to the
        loss; replicated-parameter gradients are summed over the TP group by
        ``parallel.tp_fused.allreduce_replicated_grads``)."""
        from ..core.losses import causal_lm_loss_from_hidden

        ws = self.sp_ws
        P, r = ws.world, ws.rank
        B, S = input_ids.shape
        T = B * S
        rows = T // P
        if labels is None:
            labels = torch.roll(input_ids, -1, dims=1)
            labels[:, -1] = ignore_index
        if self.training and torch.is_grad_enabled():
            ws.begin_step()
        flat = input_ids.reshape(-1)
        x = self.embed(flat[r * rows:(r + 1) * rows].view(1, rows)).view(rows, -1)
        for layer in self.layers:
            x = layer.forward_sp(x, input_ids, B, S, ws)
        x = self.norm(x)
        lab = labels.reshape(-1)[r * rows:(r + 1) * rows]
        n_local = (lab != ignore_index).sum()
        n_total = (labels != ignore_index).sum().clamp_min(1)
        loss = causal_lm_loss_from_hidden(x.view(1, rows, -1), self.output_weight(),
                                          lab.view(1, rows), ignore_index=ignore_index)
        return loss * (n_local / n_total)

    # ------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, input_ids: Optional[torch.Tensor] = None, max_new_tokens: int = 100,
                 temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                 do_sample: bool = False, eos_token_id: Optional[int] = None, **kwargs):
        """Decode with the paged-KV engine; returns prompt + generated ids per row."""
        from ..inference.engine import GenerationConfig, InferenceEngine

        if input_ids is None:
            raise ValueError("generate needs input_ids")
        eng = InferenceEngine(self)
        gen = GenerationConfig(max_new_tokens=max_new_tokens, temperature=temperature,
                               top_k=top_k, top_p=top_p, do_sample=do_sample,
                               eos_token_id=eos_token_id)
        rows = [r.tolist() for r in input_ids.cpu()]
        outs = eng.generate_tokens(rows, gen)
        return [r + o for r, o in zip(rows, outs)]

    # -------------------------------------------------------------- save/load
    def save_pretrained(self, save_directory: Union[str, Path], safe_serialization: bool = True):
        """Write config.json + model.safetensors; collective when distributed."""
        from ..utils.checkpointing import gather_full_state_dict

        save_directory = Path(save_directory)
        sd, is_main = gather_full_state_dict(self)
        if not is_main:
            return
        save_directory.mkdir(parents=True, exist_ok=True)
        with open(save_directory / "config.json", "w") as fh:
            json.dump(self.config.to_dict(), fh, indent=2)
        if safe_serialization:
            from safetensors.torch import save_file

            save_file(sd, str(save_directory / "model.safetensors"))
        else:
            torch.save(sd, save_directory / "pytorch_model.bin")

    @classmethod
    def from_pretrained(cls, path: Union[str, Path], device: Optional[str] = None,
                        dtype: Optional[torch.dtype] = None) -> "ComplexityModel":
        path = Path(path)
        cfg_path = path / "config.json"
        if not cfg_path.exists():
            raise ValueError(f"Config not found at {cfg_path}")
        with open(cfg_path) as fh:
            config = ModelConfig.from_dict(json.load(fh))
        model = cls(config)
        st, pt = path / "model.safetensors", path / "pytorch_model.bin"
        if st.exists():
            from safetensors.torch import load_file

            sd = load_file(str(st))
        elif pt.exists():
            sd = torch.load(pt, map_location="cpu", weights_only=True)
        else:
            raise ValueError(f"No model weights found. Expected {st} or {pt}")
        missing, unexpected = model.load_state_dict(sd, strict=False)
        bad = [k for k in missing if not _DETERMINISTIC_BUFFER.search(k)]
        if bad or unexpected:
            raise RuntimeError("Error(s) in loading state_dict for ComplexityModel: "
                               f"missing={bad}, unexpected={list(unexpected)}")
        if dtype is not None:
            model = model.to(dtype=dtype)
        if device is not None:
            model = model.to(device)
        return model
