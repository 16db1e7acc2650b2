"""HF Transformers adapter: ``TRHashConfig`` / ``TRHashForCausalLM``.

Counterpart of integrations/transformers/tr_hash_moe/ (configuration 114 LoC,
modeling_tr_hash_moe.py:34-548).  The adapter keeps this framework's native
tensor names (``embed_tokens.*``, ``layers.N.*``, ``norm.*``) so a checkpoint
directory written by ``ComplexityModel.save_pretrained`` loads with
``TRHashForCausalLM.from_pretrained`` and vice versa; routes come from the
persisted ``route_table`` buffers.  Forward runs the framework's own model
(fused sm_100a kernels on CUDA); ``generate`` runs the paged-KV engine.
"""
from __future__ import annotations

from typing import Optional

import torch

try:
    from transformers import PretrainedConfig, PreTrainedModel
    from transformers.modeling_outputs import CausalLMOutputWithPast
    HAVE_TRANSFORMERS = True
except ImportError:  # pragma: no cover - optional dependency
    HAVE_TRANSFORMERS = False
    PretrainedConfig = object
    PreTrainedModel = torch.nn.Module

from ..config.model_config import ModelConfig

MODEL_TYPE = "tr_hash_moe"


class TRHashConfig(PretrainedConfig):
    model_type = MODEL_TYPE

    def __init__(self, **kwargs):
        # ModelConfig fields live flat in config.json, so the same file also
        # loads with ComplexityModel.from_pretrained
        mc_fields = set(ModelConfig.__dataclass_fields__)
        mine = {k: kwargs.pop(k) for k in list(kwargs) if k in mc_fields}
        mc = ModelConfig.from_dict(mine)
        super().__init__(**kwargs)
        for k, v in mc.to_dict().items():
            setattr(self, k, v)
        self._mc_keys = sorted(mc.to_dict())

    def to_model_config(self) -> ModelConfig:
        keys = getattr(self, "_mc_keys", None) or list(ModelConfig.__dataclass_fields__)
        return ModelConfig.from_dict({k: getattr(self, k) for k in keys if hasattr(self, k)})

    @classmethod
    def from_model_config(cls, mc: ModelConfig) -> "TRHashConfig":
        return cls(**mc.to_dict())


class TRHashForCausalLM(PreTrainedModel):
    config_class = TRHashConfig
    base_model_prefix = ""
    _no_split_modules = ["TransformerBlock"]
    _tied_weights_keys = {}

    def __init__(self, config: TRHashConfig):
        super().__init__(config)
        from ..models.builder import ComplexityModel

        inner = ComplexityModel(config.to_model_config())
        # adopt the submodules so state-dict keys are the native ones
        for name, mod in inner.named_children():
            self.add_module(name, mod)
        object.__setattr__(self, "_inner", inner)
        self.post_init()

    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        model = super().from_pretrained(*args, **kwargs)
        model._restore_runtime_state()
        return model

    @torch.no_grad()
    def _restore_runtime_state(self) -> None:
        """Rebuild non-checkpoint state after deferred (meta-device) loading:
        route blend weights, pair metadata from the loaded route tables, RoPE
        frequencies."""
        for m in self.modules():
            if type(m).__name__ == "TRHashEngine":
                m.set_route_weights(m.config.route_weights)
                m.load_route_table(m.route_table.clone())
            if hasattr(m, "set_inv_freq") and hasattr(m, "_inv32"):
                m.set_inv_freq(m._inv32)

    def _init_weights(self, module):
        """Weights are initialised by the framework's model constructor."""

    def get_input_embeddings(self):
        return self.embed_tokens

    def forward(self, input_ids: Optional[torch.LongTensor] = None,
                attention_mask: Optional[torch.Tensor] = None, labels=None, **kwargs):
        out = self._inner(input_ids)
        logits = out["logits"]
        loss = None
        if labels is not None:
            loss = torch.nn.functional.cross_entropy(
                logits[:, :-1].float().reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1),
                ignore_index=-100)
        return CausalLMOutputWithPast(loss=loss, logits=logits)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 32, do_sample: bool = False,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 0,
                 eos_token_id: Optional[int] = None, attention_mask=None, **kwargs):
        from ..inference.engine import GenerationConfig, InferenceEngine

        eng = InferenceEngine(self._inner)
        gen = GenerationConfig(max_new_tokens=max_new_tokens, do_sample=do_sample,
                               temperature=temperature, top_p=top_p, top_k=top_k,
                               eos_token_id=eos_token_id)
        res = eng.generate(input_ids, gen, attention_mask=attention_mask)
        width = max(len(s) for s in res["sequences"])
        pad = eos_token_id if eos_token_id is not None else 0
        return torch.tensor([s + [pad] * (width - len(s)) for s in res["sequences"]],
                            device=input_ids.device)


def register_auto_classes() -> None:
    """Make ``AutoConfig`` / ``AutoModelForCausalLM`` resolve ``model_type: tr_hash_moe``."""
    from transformers import AutoConfig, AutoModelForCausalLM

    try:
        AutoConfig.register(MODEL_TYPE, TRHashConfig)
    except ValueError:
        pass
    try:
        AutoModelForCausalLM.register(TRHashConfig, TRHashForCausalLM)
    except ValueError:
        pass


def export_hf(model, directory) -> None:
    """Write an HF-loadable directory (config.json with ``model_type`` + safetensors)."""
    cfg = TRHashConfig.from_model_config(model.config)
    hf = TRHashForCausalLM(cfg)
    hf.load_state_dict(model.state_dict(), strict=False)
    hf.save_pretrained(directory)
