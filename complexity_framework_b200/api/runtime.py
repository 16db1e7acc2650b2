"""Tokenizer, data, trainer and generation facades.

Facade names follow complexity/api/{tokenizer,dataset,trainer,inference}.py
(``Tokenizer`` / ``TokenizerConfig``, ``Dataset`` / ``DataConfig`` /
``StreamingDataset`` / ``DataPipeline``, ``Trainer`` / ``TrainerConfig``,
``Generate`` / ``create_engine``); each wraps this framework's components
(byte / BPE / sentencepiece tokenizers, token shards + the C++ batch loader,
the fused ``training.Trainer``, the paged-KV ``InferenceEngine``).
"""
from __future__ import annotations

import tempfile
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Iterable, Iterator, List, Optional, Sequence, Union

import torch

from ..data.streaming import StreamingDataset, iter_texts
from ..data.tokenization import Tokenizer as _TokenizerBase, get_tokenizer
from ..inference.engine import (DecodingStrategy, GenerationConfig, InferenceConfig,
                                InferenceEngine)


# ---------------------------------------------------------------- tokenizer
@dataclass
class TokenizerConfig:
    kind: str = "byte"                 # byte | bpe | sentencepiece | hf path
    path: Optional[str] = None
    vocab_size: Optional[int] = None


class Tokenizer:
    """``Tokenizer.load("byte")`` / ``Tokenizer.from_config(cfg)``; ``encode`` /
    ``decode`` / ``batch_encode`` over the framework tokenizers."""

    def __init__(self, inner: _TokenizerBase):
        self.inner = inner

    @classmethod
    def load(cls, name_or_path: str = "byte", **kw) -> "Tokenizer":
        """A kind ("byte", "tiktoken") or a path: ``*.model`` loads sentencepiece,
        any other path a Hugging Face tokenizer directory."""
        if name_or_path in ("byte", "tiktoken"):
            return cls(get_tokenizer(name_or_path, **kw))
        kind = "sentencepiece" if str(name_or_path).endswith(".model") else "hf"
        return cls(get_tokenizer(kind, model_path=str(name_or_path), **kw))

    @classmethod
    def from_config(cls, config: TokenizerConfig) -> "Tokenizer":
        if config.path is None:
            return cls.load(config.kind)
        if config.kind in ("sentencepiece", "hf", "huggingface"):
            return cls(get_tokenizer(config.kind, model_path=config.path))
        return cls.load(config.path)

    @property
    def vocab_size(self) -> int:
        return self.inner.vocab_size

    @property
    def eos_token_id(self) -> Optional[int]:
        return self.inner.eos_token_id

    def encode(self, text: str) -> List[int]:
        return self.inner.encode(text)

    def decode(self, ids: Sequence[int]) -> str:
        return self.inner.decode(list(ids))

    def batch_encode(self, texts: Sequence[str]) -> List[List[int]]:
        return [self.encode(t) for t in texts]

    def __getattr__(self, name):
        return getattr(self.inner, name)


# --------------------------------------------------------------------- data
@dataclass
class DataConfig:
    seq_len: int = 2048
    batch_size: int = 8
    text_key: str = "text"
    add_eos: bool = True
    shuffle: bool = True
    seed: int = 0


class Dataset:
    """Texts (strings or .txt / .jsonl paths) tokenised into a token shard and
    served as ``(input_ids, labels)`` batches by the C++ loader."""

    def __init__(self, shard_dir: Union[str, Path], config: Optional[DataConfig] = None):
        self.shard_dir = str(shard_dir)
        self.config = config or DataConfig()

    @classmethod
    def from_texts(cls, texts: Union[Iterable[str], str, Path], tokenizer: Tokenizer,
                   config: Optional[DataConfig] = None,
                   out_dir: Optional[Union[str, Path]] = None) -> "Dataset":
        from ..data.token_shards import write_token_shard

        cfg = config or DataConfig()
        if isinstance(texts, (str, Path)) and Path(texts).exists():
            texts = iter_texts([str(texts)], text_key=cfg.text_key)
        eos = [tokenizer.eos_token_id] if cfg.add_eos and tokenizer.eos_token_id is not None else []
        out = str(out_dir or tempfile.mkdtemp(prefix="cfb_ds_"))
        write_token_shard(out, (tokenizer.encode(t) + eos for t in texts),
                          vocab_size=tokenizer.vocab_size)
        return cls(out, cfg)

    def loader(self, rank: int = 0, world_size: int = 1, pin_memory: Optional[bool] = None):
        from ..data.loader import TokenBatchLoader

        c = self.config
        return TokenBatchLoader(self.shard_dir, c.batch_size, c.seq_len, rank=rank,
                                world_size=world_size, seed=c.seed,
                                order="random" if c.shuffle else "sequential", eval_ratio=0.0,
                                pin_memory=torch.cuda.is_available() if pin_memory is None
                                else pin_memory)

    def __iter__(self):
        return iter(self.loader())


class DataPipeline:
    """Chain of text transforms followed by tokenisation into a ``Dataset``."""

    def __init__(self, tokenizer: Tokenizer, config: Optional[DataConfig] = None):
        self.tokenizer = tokenizer
        self.config = config or DataConfig()
        self.steps = []

    def map(self, fn) -> "DataPipeline":
        self.steps.append(("map", fn))
        return self

    def filter(self, fn) -> "DataPipeline":
        self.steps.append(("filter", fn))
        return self

    def _apply(self, texts: Iterable[str]) -> Iterator[str]:
        for t in texts:
            keep = True
            for kind, fn in self.steps:
                if kind == "map":
                    t = fn(t)
                elif not fn(t):
                    keep = False
                    break
            if keep:
                yield t

    def build(self, texts: Union[Iterable[str], str, Path],
              out_dir: Optional[Union[str, Path]] = None) -> Dataset:
        if isinstance(texts, (str, Path)) and Path(texts).exists():
            texts = iter_texts([str(texts)], text_key=self.config.text_key)
        return Dataset.from_texts(self._apply(texts), self.tokenizer, self.config, out_dir)


# ------------------------------------------------------------------ trainer
@dataclass
class TrainerConfig:
    learning_rate: float = 3e-4
    max_steps: int = 1000
    batch_size: int = 8
    seq_len: int = 2048
    warmup_steps: int = 100
    weight_decay: float = 0.1
    grad_clip: float = 1.0
    precision: str = "bf16"
    output_dir: str = "checkpoints"
    save_steps: int = 1000
    log_steps: int = 10
    lr_scheduler: str = "cosine"
    distributed_mode: str = "auto"
    extra: Dict[str, Any] = field(default_factory=dict)

    def to_training_config(self):
        from ..training.config import TrainingConfig

        return TrainingConfig(learning_rate=self.learning_rate, max_steps=self.max_steps,
                              batch_size=self.batch_size, warmup_steps=self.warmup_steps,
                              weight_decay=self.weight_decay, grad_clip=self.grad_clip,
                              precision=self.precision, checkpoint_dir=self.output_dir,
                              save_steps=self.save_steps, log_steps=self.log_steps,
                              lr_scheduler=self.lr_scheduler,
                              distributed_mode=self.distributed_mode, **self.extra)


class Trainer:
    """``Trainer(model, TrainerConfig(...)).train(dataset)``."""

    def __init__(self, model, config: Optional[TrainerConfig] = None, **kwargs):
        from ..training.trainer import Trainer as _Trainer

        self.model = getattr(model, "model", model)  # api.Model or ComplexityModel
        self.config = config or TrainerConfig(**kwargs)
        self.inner = _Trainer(self.model, self.config.to_training_config())

    def train(self, train_data, val_data=None, **kwargs) -> Dict:
        batches = train_data.loader() if isinstance(train_data, Dataset) else train_data
        evals = None
        if val_data is not None:
            evals = (lambda: val_data.loader()) if isinstance(val_data, Dataset) else (
                lambda: val_data)
        try:
            return self.inner.train(batches, self.config.max_steps, eval_batches=evals)
        finally:
            if hasattr(batches, "close"):
                batches.close()

    def save(self, path: str) -> None:
        self.model.save_pretrained(path)


# --------------------------------------------------------------- generation
def create_engine(model, cache_type: str = "paged", max_cache_length: int = 4096,
                  max_batch_size: int = 64, **kwargs) -> InferenceEngine:
    if cache_type != "paged":
        raise ValueError("the serving engine uses the paged KV cache; contiguous and "
                         "sliding-window caches are available through ComplexityModel.generate")
    model = getattr(model, "model", model)
    return InferenceEngine(model, InferenceConfig(max_cache_length=max_cache_length,
                                                  max_batch_size=max_batch_size, **kwargs))


class Generate:
    """One-call generation helpers over the paged-KV engine."""

    _engines: Dict[int, InferenceEngine] = {}

    @classmethod
    def engine(cls, model, **kwargs) -> InferenceEngine:
        key = id(getattr(model, "model", model))
        if key not in cls._engines or kwargs:
            cls._engines[key] = create_engine(model, **kwargs)
        return cls._engines[key]

    @classmethod
    def tokens(cls, model, prompts: Sequence[Sequence[int]],
               config: Optional[GenerationConfig] = None, **kw) -> List[List[int]]:
        return cls.engine(model).generate_tokens([list(p) for p in prompts],
                                                 config or GenerationConfig(**kw))

    @classmethod
    def text(cls, model, prompt: Union[str, Sequence[str]], tokenizer: Optional[Tokenizer] = None,
             max_new_tokens: int = 64, **kw) -> Union[str, List[str]]:
        tok = tokenizer or Tokenizer.load("byte")
        single = isinstance(prompt, str)
        prompts = [prompt] if single else list(prompt)
        kw.setdefault("eos_token_id", tok.eos_token_id)
        outs = cls.tokens(model, [tok.encode(p) for p in prompts],
                          GenerationConfig(max_new_tokens=max_new_tokens, **kw))
        texts = [tok.decode(o) for o in outs]
        return texts[0] if single else texts

    @classmethod
    def stream(cls, model, prompt: str, tokenizer: Optional[Tokenizer] = None,
               max_new_tokens: int = 64, **kw) -> Iterator[str]:
        """Yields the decoded text of each new token as the engine produces it."""
        tok = tokenizer or Tokenizer.load("byte")
        eng = cls.engine(model)
        kw.setdefault("eos_token_id", tok.eos_token_id)
        rid = eng.add_request(tok.encode(prompt), GenerationConfig(max_new_tokens=max_new_tokens,
                                                                   **kw))
        seen = 0
        while not eng.requests[rid].done:
            eng.step()
            out = eng.requests[rid].output
            for t in out[seen:]:
                yield tok.decode([t])
            seen = len(out)
        eng.requests.pop(rid, None)

    @classmethod
    def chat(cls, model, messages, tokenizer: Optional[Tokenizer] = None,
             chat_format: str = "complexity", max_new_tokens: int = 128, **kw) -> str:
        from ..data.tokenization import ChatTemplate

        text = ChatTemplate(chat_format).apply(list(messages), add_generation_prompt=True)
        return cls.text(model, text, tokenizer, max_new_tokens, **kw)


__all__ = ["Tokenizer", "TokenizerConfig", "Dataset", "DataConfig", "DataPipeline",
           "StreamingDataset", "Trainer", "TrainerConfig", "Generate", "GenerationConfig",
           "InferenceConfig", "InferenceEngine", "DecodingStrategy", "create_engine"]
