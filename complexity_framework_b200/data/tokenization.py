"""Tokenizers and chat templates.

API of complexity/data/tokenization.py:33-410 (``Tokenizer`` ABC,
SentencePiece / HuggingFace / tiktoken wrappers, ``get_tokenizer``) and of the
chat formats of :412-1100 (``Message``, ``ChatTemplate`` with the
``complexity`` / ``chatml`` / ``llama`` renderings).  The special-token
strings of the ``complexity`` format are the reference's own, kept so that
prompts rendered here match what its checkpoints were trained on.

``ByteTokenizer`` (UTF-8 bytes + special tokens) needs no model file and is
the default for tests and synthetic runs.  ``encode_chat`` returns token ids
plus assistant-only labels for SFT.
"""
from __future__ import annotations

import json
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

IGNORE_INDEX = -100


class Tokenizer(ABC):
    @abstractmethod
    def encode(self, text: str) -> List[int]: ...

    @abstractmethod
    def decode(self, tokens: Sequence[int]) -> str: ...

    @property
    @abstractmethod
    def vocab_size(self) -> int: ...

    @property
    def bos_token_id(self) -> Optional[int]:
        return None

    @property
    def eos_token_id(self) -> Optional[int]:
        return None

    @property
    def pad_token_id(self) -> Optional[int]:
        return None

    def encode_batch(self, texts: Sequence[str]) -> List[List[int]]:
        return [self.encode(t) for t in texts]

    def decode_batch(self, seqs: Sequence[Sequence[int]]) -> List[str]:
        return [self.decode(s) for s in seqs]


# Special tokens of the "complexity" chat format (strings only).
COMPLEXITY_SPECIALS = {
    "bos": "<|begin|>", "eos": "<|end|>", "pad": "<|pad|>", "unk": "<|unk|>",
    "turn": "<|turn|>", "turn_end": "<|/turn|>",
    "system": "<|system|>", "system_end": "<|/system|>",
    "user": "<|user|>", "user_end": "<|/user|>",
    "assistant": "<|assistant|>", "assistant_end": "<|/assistant|>",
    "reason": "<|reason|>", "reason_end": "<|/reason|>",
    "step": "<|step|>", "step_end": "<|/step|>",
    "conclude": "<|conclude|>", "conclude_end": "<|/conclude|>",
    "call": "<|call|>", "call_end": "<|/call|>", "args": "<|args|>", "args_end": "<|/args|>",
    "result": "<|result|>", "result_end": "<|/result|>",
    "tools": "<|tools|>", "tools_end": "<|/tools|>",
}


class ByteTokenizer(Tokenizer):
    """UTF-8 bytes as ids ``n_special .. n_special+255``; specials first."""

    def __init__(self, specials: Optional[Sequence[str]] = None):
        self.specials = list(specials if specials is not None else COMPLEXITY_SPECIALS.values())
        self._sid = {s: i for i, s in enumerate(self.specials)}
        self.offset = len(self.specials)

    @property
    def vocab_size(self) -> int:
        return self.offset + 256

    @property
    def bos_token_id(self):
        return self._sid.get(COMPLEXITY_SPECIALS["bos"])

    @property
    def eos_token_id(self):
        return self._sid.get(COMPLEXITY_SPECIALS["eos"])

    @property
    def pad_token_id(self):
        return self._sid.get(COMPLEXITY_SPECIALS["pad"])

    def token_to_id(self, tok: str) -> Optional[int]:
        return self._sid.get(tok)

    def encode(self, text: str) -> List[int]:
        out: List[int] = []
        i = 0
        while i < len(text):
            if text.startswith("<|", i):
                j = text.find("|>", i)
                if j > 0 and text[i:j + 2] in self._sid:
                    out.append(self._sid[text[i:j + 2]])
                    i = j + 2
                    continue
            k = text.find("<|", i + 1)
            seg = text[i:k if k > 0 else len(text)]
            out.extend(b + self.offset for b in seg.encode("utf-8"))
            i += len(seg)
        return out

    def decode(self, tokens: Sequence[int]) -> str:
        parts, buf = [], bytearray()
        for t in tokens:
            t = int(t)
            if t < self.offset:
                if buf:
                    parts.append(buf.decode("utf-8", errors="replace"))
                    buf = bytearray()
                parts.append(self.specials[t])
            elif t < self.offset + 256:
                buf.append(t - self.offset)
        if buf:
            parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)


class SentencePieceTokenizer(Tokenizer):
    def __init__(self, model_path: str):
        import sentencepiece as spm

        self.sp = spm.SentencePieceProcessor(model_file=model_path)

    @property
    def vocab_size(self) -> int:
        return self.sp.get_piece_size()

    @property
    def bos_token_id(self):
        v = self.sp.bos_id()
        return v if v >= 0 else None

    @property
    def eos_token_id(self):
        v = self.sp.eos_id()
        return v if v >= 0 else None

    @property
    def pad_token_id(self):
        v = self.sp.pad_id()
        return v if v >= 0 else None

    def encode(self, text: str) -> List[int]:
        return list(self.sp.encode(text))

    def decode(self, tokens: Sequence[int]) -> str:
        return self.sp.decode([int(t) for t in tokens])


class HuggingFaceTokenizer(Tokenizer):
    """Wraps a local ``tokenizer.json`` / HF tokenizer directory (no downloads)."""

    def __init__(self, path: str, **kwargs):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True, **kwargs)

    @property
    def vocab_size(self) -> int:
        return len(self.tok)

    @property
    def bos_token_id(self):
        return self.tok.bos_token_id

    @property
    def eos_token_id(self):
        return self.tok.eos_token_id

    @property
    def pad_token_id(self):
        return self.tok.pad_token_id

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, tokens: Sequence[int]) -> str:
        return self.tok.decode([int(t) for t in tokens])


class TiktokenWrapper(Tokenizer):
    def __init__(self, encoding_name: str = "cl100k_base"):
        try:
            import tiktoken
        except ImportError as e:  # not in every image
            raise ImportError("tiktoken is not installed") from e
        self.enc = tiktoken.get_encoding(encoding_name)

    @property
    def vocab_size(self) -> int:
        return self.enc.n_vocab

    @property
    def eos_token_id(self):
        return self.enc.eot_token

    def encode(self, text: str) -> List[int]:
        return self.enc.encode(text, allowed_special="all")

    def decode(self, tokens: Sequence[int]) -> str:
        return self.enc.decode([int(t) for t in tokens])


def get_tokenizer(tokenizer_type: str = "byte", model_path: Optional[str] = None,
                  **kwargs) -> Tokenizer:
    kind = tokenizer_type.lower()
    if kind == "byte":
        return ByteTokenizer()
    if kind == "tiktoken":
        return TiktokenWrapper(kwargs.get("encoding_name", "cl100k_base"))
    if kind in ("sentencepiece", "huggingface", "hf") and model_path is None:
        raise ValueError(f"model_path required for {tokenizer_type}")
    if kind == "sentencepiece":
        return SentencePieceTokenizer(model_path)
    if kind in ("huggingface", "hf"):
        return HuggingFaceTokenizer(model_path, **kwargs)
    raise ValueError(f"unknown tokenizer type {tokenizer_type!r}")


# -------------------------------------------------------------- chat format
@dataclass
class Message:
    role: str  # system | user | assistant | tool
    content: str = ""
    name: Optional[str] = None
    tool_calls: Optional[List[Dict[str, Any]]] = None
    reasoning: Optional[str] = None
    steps: Optional[List[str]] = None
    conclusion: Optional[str] = None

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "Message":
        return cls(**{k: d[k] for k in ("role", "content", "name", "tool_calls", "reasoning",
                                         "steps", "conclusion") if k in d})


@dataclass
class ToolDefinition:
    name: str
    description: str = ""
    parameters: Dict[str, Any] = field(default_factory=dict)

    def to_json(self) -> str:
        return json.dumps({"name": self.name, "description": self.description,
                           "parameters": self.parameters}, sort_keys=True)


@dataclass
class ChatTemplate:
    """Renders a conversation as text; each rendered piece is tagged as
    trainable (assistant output) or not, which ``encode_chat`` turns into
    labels."""

    format: str = "complexity"  # complexity | chatml | llama

    def segments(self, messages: Sequence[Message], add_generation_prompt: bool = False,
                 tools: Optional[Sequence[ToolDefinition]] = None) -> List[Tuple[str, bool]]:
        msgs = [m if isinstance(m, Message) else Message.from_dict(m) for m in messages]
        if self.format == "complexity":
            return self._complexity(msgs, add_generation_prompt, tools)
        if self.format == "chatml":
            return self._chatml(msgs, add_generation_prompt)
        if self.format == "llama":
            return self._llama(msgs, add_generation_prompt)
        raise ValueError(f"unknown chat format {self.format!r}")

    def apply(self, messages, add_generation_prompt: bool = True, tools=None) -> str:
        return "".join(s for s, _ in self.segments(messages, add_generation_prompt, tools))

    def _complexity(self, msgs, gen, tools):
        t = COMPLEXITY_SPECIALS
        out = [(t["bos"] + "\n", False)]
        if tools:
            body = "\n".join(td.to_json() for td in tools)
            out.append((f"{t['tools']}\n{body}\n{t['tools_end']}\n", False))
        for m in msgs:
            if m.role == "system":
                out.append((f"{t['system']}\n{m.content}\n{t['system_end']}\n", False))
        for m in msgs:
            if m.role == "system":
                continue
            out.append((f"{t['turn']}\n", False))
            if m.role == "user":
                out.append((f"{t['user']}\n{m.content}\n{t['user_end']}\n", False))
            elif m.role == "assistant":
                out.append((f"{t['assistant']}\n", False))
                body = []
                if m.reasoning or m.steps:
                    body.append(f"{t['reason']}\n")
                    for s in m.steps or []:
                        body.append(f"{t['step']}{s}{t['step_end']}\n")
                    if m.reasoning:
                        body.append(m.reasoning + "\n")
                    if m.conclusion:
                        body.append(f"{t['conclude']}{m.conclusion}{t['conclude_end']}\n")
                    body.append(f"{t['reason_end']}\n")
                for tc in m.tool_calls or []:
                    body.append(f"{t['call']}\n{t['args']}\n{json.dumps(tc)}\n{t['args_end']}\n"
                                f"{t['call_end']}\n")
                if m.content:
                    body.append(m.content + "\n")
                body.append(f"{t['assistant_end']}\n")
                out.append(("".join(body), True))
            elif m.role == "tool":
                out.append((f"{t['result']}\n{m.content}\n{t['result_end']}\n", False))
            out.append((f"{t['turn_end']}\n", False))
        if gen:
            out.append((f"{t['turn']}\n{t['assistant']}\n", False))
        else:
            out.append((t["eos"], True))
        return out

    @staticmethod
    def _chatml(msgs, gen):
        out = []
        for m in msgs:
            head = f"<|im_start|>{m.role}\n"
            if m.role == "assistant":
                out.append((head, False))
                out.append((f"{m.content}<|im_end|>\n", True))
            else:
                out.append((f"{head}{m.content}<|im_end|>\n", False))
        if gen:
            out.append(("<|im_start|>assistant\n", False))
        return out

    @staticmethod
    def _llama(msgs, gen):
        out, sys_txt = [], ""
        for m in msgs:
            if m.role == "system":
                sys_txt = f"<<SYS>>\n{m.content}\n<</SYS>>\n\n"
            elif m.role == "user":
                out.append((f"<s>[INST] {sys_txt}{m.content} [/INST]", False))
                sys_txt = ""
            elif m.role == "assistant":
                out.append((f" {m.content} </s>", True))
        return out


def encode_chat(tokenizer: Tokenizer, messages, template: Optional[ChatTemplate] = None,
                max_len: Optional[int] = None, tools=None) -> Tuple[List[int], List[int]]:
    """Token ids and assistant-only labels (``IGNORE_INDEX`` elsewhere)."""
    tpl = template or ChatTemplate()
    ids: List[int] = []
    labels: List[int] = []
    for text, train in tpl.segments(messages, add_generation_prompt=False, tools=tools):
        toks = tokenizer.encode(text)
        ids.extend(toks)
        labels.extend(toks if train else [IGNORE_INDEX] * len(toks))
    if max_len is not None:
        ids, labels = ids[:max_len], labels[:max_len]
    return ids, labels
