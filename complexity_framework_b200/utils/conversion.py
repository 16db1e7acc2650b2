"""Checkpoint converters.

Counterparts: complexity/utils/token_routed_conversion.py:63-191
(token_routed -> tr_hash_engine with the exact trained route tables),
multi_hash_conversion.py:25-115 (upgrade to 4-expert top-2 multi-hash routing,
route buffers regenerated) and expert_expansion.py:35-172 (clone 4 experts
into 8, function preserving through hierarchical route expansion).

The tensor rename table and the dropped-buffer list are the ones of the
historical ``TokenRoutedMLP`` checkpoints (they must match those files).
"""
from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Any, Dict, Mapping, Tuple, Union

import torch

from ..config.model_config import ModelConfig

_MLP_KEY = re.compile(r"^(?P<prefix>layers\.(?P<layer>\d+)\.mlp)\.(?P<rest>.+)$")
_ENGINE_ROUTE_KEY = re.compile(r"^layers\.(?P<layer>\d+)\.mlp\.engine\.route_table$")
_TOKEN_ROUTED_RENAME = {
    "gate_proj_w": "engine.expert_gate",
    "up_proj_w": "engine.expert_up",
    "down_proj_w": "engine.expert_down",
    "shared_gate.weight": "engine.shared_gate.weight",
    "shared_up.weight": "engine.shared_up.weight",
    "shared_down.weight": "engine.shared_down.weight",
}
_TOKEN_ROUTED_TABLE = "topk_token_to_expert"
_TOKEN_ROUTED_DROPPED = ("token_to_expert", "pair_hash_route_codes", "pair_hash_expert_pairs",
                         "lsh_planes", "lsh_bucket_to_expert", "lsh_threshold",
                         "last_shared_rms", "last_routed_rms")
CONVERTIBLE_MLP_TYPES = ("token_routed", "sort_split", "sort_split_moe")
ROUTE_BUFFER_SUFFIXES = (".engine.route_table", ".engine.fused_route_codes",
                         ".engine.fused_expert_pairs")
EXPERT_PARAM_SUFFIXES = (".engine.expert_gate", ".engine.expert_up", ".engine.expert_down")
_TOLERATED_MISSING = ROUTE_BUFFER_SUFFIXES + (".rotary_emb.inv_freq",)


def _read_dir(path: Union[str, Path]) -> Tuple[Dict[str, torch.Tensor], Dict[str, Any]]:
    path = Path(path)
    cfg = json.loads((path / "config.json").read_text())
    st = path / "model.safetensors"
    if st.exists():
        from safetensors.torch import load_file

        return load_file(str(st)), cfg
    return torch.load(path / "pytorch_model.bin", map_location="cpu", weights_only=True), cfg


def _load_checked(model, state: Dict[str, torch.Tensor], what: str) -> None:
    missing, unexpected = model.load_state_dict(state, strict=False)
    bad = [k for k in missing if not k.endswith(_TOLERATED_MISSING)]
    if bad or unexpected:
        raise RuntimeError(f"{what} left mismatched tensors: missing={bad}, "
                           f"unexpected={list(unexpected)}")


def _float_dtype(state: Mapping[str, torch.Tensor]) -> torch.dtype:
    return next((v.dtype for v in state.values() if v.is_floating_point()), torch.float32)


# ------------------------------------------------------ token_routed -> tr_hash
def convert_token_routed_state_dict(state_dict: Mapping[str, torch.Tensor]
                                    ) -> Tuple[Dict[str, torch.Tensor], Dict[int, torch.Tensor]]:
    """Renamed state dict plus ``{layer: trained [top_k, vocab] route table}``."""
    out: Dict[str, torch.Tensor] = {}
    tables: Dict[int, torch.Tensor] = {}
    for key, val in state_dict.items():
        m = _MLP_KEY.match(key)
        if not m:
            out[key] = val
            continue
        rest = m.group("rest")
        if rest == _TOKEN_ROUTED_TABLE:
            tables[int(m.group("layer"))] = val
        elif any(rest == s or rest.endswith("." + s) for s in _TOKEN_ROUTED_DROPPED):
            continue
        elif rest in _TOKEN_ROUTED_RENAME:
            out[f"{m.group('prefix')}.{_TOKEN_ROUTED_RENAME[rest]}"] = val
        else:
            raise ValueError(f"no tr_hash_engine equivalent for token_routed tensor {key!r}")
    return out, tables


def convert_token_routed_config(config: Mapping[str, Any]) -> ModelConfig:
    if config.get("mlp_type") not in CONVERTIBLE_MLP_TYPES:
        raise ValueError(f"expected mlp_type in {CONVERTIBLE_MLP_TYPES}, got "
                         f"{config.get('mlp_type')!r}")
    return ModelConfig.from_dict(dict(config, mlp_type="tr_hash_engine"))


def convert_token_routed_checkpoint(state_dict, config):
    from ..models.builder import ComplexityModel

    model = ComplexityModel(convert_token_routed_config(config))
    state, tables = convert_token_routed_state_dict(state_dict)
    _load_checked(model, state, "token_routed -> tr_hash_engine conversion")
    for layer, table in tables.items():
        model.layers[layer].mlp.engine.load_route_table(table)
    return model


def convert_token_routed_checkpoint_dir(path):
    return convert_token_routed_checkpoint(*_read_dir(path))


# ---------------------------------------------------------------- multi-hash
def multi_hash_config(raw_config: Mapping[str, Any], *, route_hash_count: int = 2) -> ModelConfig:
    cfg = dict(raw_config)
    if cfg.get("mlp_type") in CONVERTIBLE_MLP_TYPES:
        cfg["mlp_type"] = "tr_hash_engine"
    if cfg.get("mlp_type", "tr_hash_engine") not in ("tr_hash_engine", "tr_hash_moe"):
        raise ValueError("multi-hash conversion requires a TR-Hash MLP checkpoint")
    if int(cfg.get("num_experts", 1)) != 4 or int(cfg.get("top_k", 1)) != 2:
        raise ValueError("multi-hash conversion requires 4 experts with top_k=2")
    cfg["routing_strategy"] = "token_id_multi_hash"
    cfg["route_hash_count"] = int(route_hash_count)
    return ModelConfig.from_dict(cfg)


def convert_checkpoint_to_multi_hash(state_dict, raw_config, *, route_hash_count: int = 2):
    """Expert weights transfer exactly; route buffers are regenerated for the new
    routing (continued pretraining lets the experts adapt)."""
    from ..models.builder import ComplexityModel

    cfg = multi_hash_config(raw_config, route_hash_count=route_hash_count)
    state = (convert_token_routed_state_dict(state_dict)[0]
             if raw_config.get("mlp_type") in CONVERTIBLE_MLP_TYPES else dict(state_dict))
    state = {k: v for k, v in state.items() if not k.endswith(ROUTE_BUFFER_SUFFIXES)}
    model = ComplexityModel(cfg).to(dtype=_float_dtype(state))
    _load_checked(model, state, "multi-hash conversion")
    return model


def convert_checkpoint_dir_to_multi_hash(path, *, route_hash_count: int = 2):
    sd, cfg = _read_dir(path)
    return convert_checkpoint_to_multi_hash(sd, cfg, route_hash_count=route_hash_count)


# ----------------------------------------------------------- expert expansion
def expanded_expert_config(raw_config: Mapping[str, Any], *, target_num_experts: int = 8
                           ) -> ModelConfig:
    cfg = dict(raw_config)
    src = int(cfg.get("num_experts", 1))
    if src != 4 or target_num_experts != 8 or int(cfg.get("top_k", 1)) != 2:
        raise ValueError("expert expansion supports 4 -> 8 experts with top_k=2")
    if cfg.get("mlp_type") in CONVERTIBLE_MLP_TYPES:
        cfg["mlp_type"] = "tr_hash_engine"
    elif cfg.get("mlp_type", "tr_hash_engine") not in ("tr_hash_engine", "tr_hash_moe"):
        raise ValueError("expert expansion requires a TR-Hash MLP checkpoint")
    routed = int(cfg["intermediate_size"])
    if routed % src:
        raise ValueError("routed width must divide by the expert count")
    cfg.update(intermediate_size=routed // src * target_num_experts,
               num_experts=target_num_experts, routing_strategy="token_id_hierarchical_hash",
               route_hash_count=2, active_num_experts=None, active_expert_width=None)
    return ModelConfig.from_dict(cfg)


def convert_checkpoint_to_expanded_experts(state_dict, raw_config, *,
                                           target_num_experts: int = 8):
    """Each trained expert is cloned; the old route picks the parent family and a
    second token hash picks the clone, so outputs are unchanged until the clones
    diverge in continued training."""
    from ..models.builder import ComplexityModel
    from ..tr_hash.routing import expand_route_table_hierarchically

    src = int(raw_config.get("num_experts", 1))
    cfg = expanded_expert_config(raw_config, target_num_experts=target_num_experts)
    if raw_config.get("mlp_type") in CONVERTIBLE_MLP_TYPES:
        state, routes = convert_token_routed_state_dict(state_dict)
    else:
        state, routes = dict(state_dict), {}
        for k in list(state):
            m = _ENGINE_ROUTE_KEY.match(k)
            if m:
                routes[int(m.group("layer"))] = state.pop(k)
            elif k.endswith(ROUTE_BUFFER_SUFFIXES[1:]):
                state.pop(k)
    if set(routes) != set(range(cfg.num_hidden_layers)):
        raise ValueError("source checkpoint lacks route tables for some layers")
    clones = target_num_experts // src
    out = {}
    for k, v in state.items():
        if k.endswith(EXPERT_PARAM_SUFFIXES):
            if v.ndim != 3 or v.shape[0] != src:
                raise ValueError(f"bad expert tensor {k}: {tuple(v.shape)}")
            v = torch.cat([v.clone() for _ in range(clones)], 0)
        out[k] = v
    model = ComplexityModel(cfg).to(dtype=_float_dtype(out))
    _load_checked(model, out, "expert expansion")
    for layer, table in routes.items():
        model.layers[layer].mlp.engine.load_route_table(expand_route_table_hierarchically(
            table, source_num_experts=src, target_num_experts=target_num_experts,
            layer_index=layer))
    return model


def convert_checkpoint_dir_to_expanded_experts(path, *, target_num_experts: int = 8):
    sd, cfg = _read_dir(path)
    return convert_checkpoint_to_expanded_experts(sd, cfg, target_num_experts=target_num_experts)


# ------------------------------------------------------------ HF (Llama-style)
_HF_LLAMA = {
    "model.embed_tokens.weight": "embed_tokens.weight",
    "model.norm.weight": "norm.weight",
    "lm_head.weight": "lm_head.weight",
    "model.layers.{i}.input_layernorm.weight": "layers.{i}.input_layernorm.weight",
    "model.layers.{i}.post_attention_layernorm.weight": "layers.{i}.post_attention_layernorm.weight",
    "model.layers.{i}.self_attn.q_proj.weight": "layers.{i}.self_attn.q_proj.weight",
    "model.layers.{i}.self_attn.k_proj.weight": "layers.{i}.self_attn.k_proj.weight",
    "model.layers.{i}.self_attn.v_proj.weight": "layers.{i}.self_attn.v_proj.weight",
    "model.layers.{i}.self_attn.o_proj.weight": "layers.{i}.self_attn.o_proj.weight",
    "model.layers.{i}.mlp.gate_proj.weight": "layers.{i}.mlp.engine.shared_gate.weight",
    "model.layers.{i}.mlp.up_proj.weight": "layers.{i}.mlp.engine.shared_up.weight",
    "model.layers.{i}.mlp.down_proj.weight": "layers.{i}.mlp.engine.shared_down.weight",
}


def get_weight_mapping(model_type: str = "llama") -> Dict[str, str]:
    if model_type not in ("llama", "mistral", "qwen2"):
        raise ValueError(f"unsupported HF model type {model_type!r}")
    return dict(_HF_LLAMA)


def _map_keys(sd: Mapping[str, torch.Tensor], mapping: Dict[str, str]) -> Dict[str, torch.Tensor]:
    pats = [(re.compile("^" + re.escape(a).replace(r"\{i\}", r"(\d+)") + "$"), b)
            for a, b in mapping.items()]
    out = {}
    for k, v in sd.items():
        for pat, dst in pats:
            m = pat.match(k)
            if m:
                out[dst.replace("{i}", m.group(1)) if m.groups() else dst] = v
                break
    return out


def convert_hf_state_dict(hf_sd: Mapping[str, torch.Tensor], model_type: str = "llama"):
    """HF Llama-family dense weights -> this framework's names (the dense MLP
    becomes the shared SwiGLU of the TR-Hash engine; experts start fresh)."""
    return _map_keys(hf_sd, get_weight_mapping(model_type))


def convert_to_hf_state_dict(sd: Mapping[str, torch.Tensor], model_type: str = "llama"):
    inv = {b: a for a, b in get_weight_mapping(model_type).items()}
    return _map_keys(sd, inv)


def create_hf_config(config: ModelConfig, model_type: str = "llama") -> Dict[str, Any]:
    return {"model_type": model_type, "architectures": ["LlamaForCausalLM"],
            "hidden_size": config.hidden_size, "num_hidden_layers": config.num_hidden_layers,
            "num_attention_heads": config.num_attention_heads,
            "num_key_value_heads": config.num_key_value_heads,
            "intermediate_size": config.shared_intermediate_size or config.intermediate_size,
            "vocab_size": config.vocab_size, "rms_norm_eps": config.norm_eps,
            "rope_theta": config.rope_theta,
            "max_position_embeddings": config.max_position_embeddings,
            "tie_word_embeddings": config.tie_word_embeddings, "torch_dtype": "bfloat16"}


def load_from_huggingface(model_name_or_path: str, model, model_type: str = "llama",
                          device: str = "cpu"):
    """Load a local Hugging Face Llama-family checkpoint directory (safetensors
    or a PyTorch bin) into ``model`` through ``convert_hf_state_dict``; keys the
    HF model lacks (TR-Hash experts, route tables) keep their initial values.
    Hub downloads are not available offline: pass a directory."""
    p = Path(model_name_or_path)
    if not p.is_dir():
        raise FileNotFoundError(f"{p} is not a local checkpoint directory (no network access "
                                "to download from the Hub)")
    sd: Dict[str, torch.Tensor] = {}
    files = sorted(p.glob("*.safetensors"))
    if files:
        from safetensors.torch import load_file

        for f in files:
            sd.update(load_file(str(f), device=device))
    else:
        for f in sorted(p.glob("pytorch_model*.bin")):
            sd.update(torch.load(f, map_location=device, weights_only=True))
    if not sd:
        raise FileNotFoundError(f"no weights (*.safetensors / pytorch_model*.bin) in {p}")
    mapped = convert_hf_state_dict(sd, model_type)
    missing, unexpected = model.load_state_dict(mapped, strict=False)
    if unexpected:
        raise ValueError(f"unmapped Hugging Face keys: {unexpected[:5]}")
    return model


def save_to_huggingface(model, save_path: str, model_type: str = "llama", config=None) -> str:
    """Write ``config.json`` + ``model.safetensors`` in Llama-family layout (the
    shared SwiGLU is the dense MLP; routed experts have no HF counterpart and
    are left out)."""
    from safetensors.torch import save_file

    out = Path(save_path)
    out.mkdir(parents=True, exist_ok=True)
    cfg = config or model.config
    sd = {k: v.detach().contiguous().cpu() for k, v in
          convert_to_hf_state_dict(model.state_dict(), model_type).items()
          if not any(k.endswith(s) for s in ROUTE_BUFFER_SUFFIXES + EXPERT_PARAM_SUFFIXES)
          and ".engine." not in k}
    save_file(sd, str(out / "model.safetensors"))
    (out / "config.json").write_text(json.dumps(create_hf_config(cfg, model_type), indent=2))
    return str(out)


def push_to_hub(*args, **kwargs):
    raise RuntimeError("push_to_hub needs network access, which this environment does not "
                       "have; use save_to_huggingface and upload the directory separately")
