"""High-level facade for quick use: load or build a model, generate, chat,
train on text, save.

Counterpart of complexity/api/ (``Model``, ``Generate``, ``Trainer`` /
``TrainerConfig`` facades).  Everything delegates to the framework's own
components (paged-KV engine, Trainer, token shards, ByteTokenizer by default).
"""
from __future__ import annotations

import tempfile
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence, Union

import torch

from ..config.model_config import ModelConfig, get_preset
from ..data.tokenization import ChatTemplate, Message, Tokenizer, get_tokenizer
from ..inference.engine import GenerationConfig, InferenceEngine
from ..models.builder import ComplexityModel


class Model:
    def __init__(self, model: ComplexityModel, tokenizer: Optional[Tokenizer] = None):
        self.model = model
        self.tokenizer = tokenizer or get_tokenizer("byte")
        self._engine: Optional[InferenceEngine] = None

    # -------------------------------------------------------------- creation
    @classmethod
    def from_preset(cls, name: str = "tiny", tokenizer: Optional[Tokenizer] = None,
                    device: Optional[str] = None, **overrides) -> "Model":
        tok = tokenizer or get_tokenizer("byte")
        cfg = get_preset(name)
        d = cfg.to_dict()
        d.update(overrides)
        d.setdefault("vocab_size", tok.vocab_size)
        if "vocab_size" not in overrides:
            d["vocab_size"] = tok.vocab_size
        m = ComplexityModel(ModelConfig.from_dict(d))
        return cls(_place(m, device), tok)

    @classmethod
    def load(cls, path: Union[str, Path], tokenizer: Optional[Tokenizer] = None,
             device: Optional[str] = None) -> "Model":
        return cls(_place(ComplexityModel.from_pretrained(path), device), tokenizer)

    def save(self, path: Union[str, Path]) -> None:
        self.model.save_pretrained(path)

    # ------------------------------------------------------------ generation
    @property
    def engine(self) -> InferenceEngine:
        if self._engine is None:
            self._engine = InferenceEngine(self.model)
        return self._engine

    def generate(self, prompt: Union[str, Sequence[str]], max_new_tokens: int = 64,
                 temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0,
                 seed: Optional[int] = None) -> Union[str, List[str]]:
        single = isinstance(prompt, str)
        prompts = [prompt] if single else list(prompt)
        gen = GenerationConfig(max_new_tokens=max_new_tokens, do_sample=temperature > 0,
                               temperature=temperature if temperature > 0 else 1.0, top_p=top_p,
                               top_k=top_k, eos_token_id=self.tokenizer.eos_token_id, seed=seed)
        outs = self.engine.generate_tokens([self.tokenizer.encode(p) for p in prompts], gen)
        texts = [self.tokenizer.decode(o) for o in outs]
        return texts[0] if single else texts

    def chat(self, messages: Sequence[Union[Message, Dict]], max_new_tokens: int = 128,
             chat_format: str = "complexity", **kw) -> str:
        text = ChatTemplate(chat_format).apply(list(messages), add_generation_prompt=True)
        return self.generate(text, max_new_tokens=max_new_tokens, **kw)

    # --------------------------------------------------------------- training
    def train(self, texts: Union[Iterable[str], str, Path], steps: int = 100, batch_size: int = 8,
              seq_len: int = 256, lr: float = 3e-4, **cfg_kw) -> Dict:
        """Tokenise ``texts`` (strings, or a .txt/.jsonl path) into a temporary token
        shard and train on it with the framework Trainer."""
        from ..data.loader import TokenBatchLoader
        from ..data.streaming import iter_texts
        from ..data.token_shards import write_token_shard
        from ..training import Trainer, TrainingConfig

        if isinstance(texts, (str, Path)) and Path(texts).exists():
            texts = iter_texts([str(texts)])
        tok = self.tokenizer
        eos = [tok.eos_token_id] if tok.eos_token_id is not None else []
        tmp = tempfile.mkdtemp(prefix="cfb_api_")
        write_token_shard(tmp, (tok.encode(t) + eos for t in texts), vocab_size=tok.vocab_size)
        dev = next(self.model.parameters()).device
        cfg = TrainingConfig(max_steps=steps, learning_rate=lr, warmup_steps=max(1, steps // 20),
                             precision="bf16" if dev.type == "cuda" else "fp32",
                             checkpoint_dir=str(Path(tmp) / "ck"), save_steps=steps + 1,
                             skip_param_update_check=True, **cfg_kw)
        trainer = Trainer(self.model, cfg, device=dev)
        loader = TokenBatchLoader(tmp, batch_size, seq_len, eval_ratio=0.0,
                                  pin_memory=dev.type == "cuda")
        try:
            out = trainer.train(loader, steps)
        finally:
            loader.close()
        self._engine = None
        return out

    def num_parameters(self) -> int:
        return self.model.num_parameters()


def _place(m: ComplexityModel, device: Optional[str]) -> ComplexityModel:
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    return m.to(device=dev, dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32)


def load(path_or_preset: str, **kw) -> Model:
    p = Path(path_or_preset)
    return Model.load(p, **kw) if p.exists() else Model.from_preset(path_or_preset, **kw)
