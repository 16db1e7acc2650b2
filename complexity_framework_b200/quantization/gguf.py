"""GGUF (llama.cpp) file writer.

Counterpart of complexity/quantization/gguf_export.py:26-400.  Writes GGUF v3:
header (magic, version, tensor count, metadata count), typed key/value
metadata, tensor infos (name, dims innermost first, type, offset) and the
32-byte-aligned tensor data.  Supported tensor types: F32, F16 and Q8_0
(blocks of 32 int8 values with one fp16 scale).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from enum import IntEnum
from pathlib import Path
from typing import Any, Dict, List, Tuple

import numpy as np
import torch

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
GGUF_VERSION = 3
ALIGN = 32


class GGUFQuantType(IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q8_0 = 8


class _VT(IntEnum):  # metadata value types
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10


def _s(b: bytearray, text: str) -> None:
    raw = text.encode("utf-8")
    b += struct.pack("<Q", len(raw)) + raw


def _kv(b: bytearray, key: str, val: Any) -> None:
    _s(b, key)
    if isinstance(val, bool):
        b += struct.pack("<IB", _VT.BOOL, int(val))
    elif isinstance(val, int):
        b += struct.pack("<Iq", 11, val) if val < 0 else struct.pack("<IQ", _VT.UINT64, val)
    elif isinstance(val, float):
        b += struct.pack("<If", _VT.FLOAT32, val)
    elif isinstance(val, str):
        b += struct.pack("<I", _VT.STRING)
        _s(b, val)
    elif isinstance(val, (list, tuple)):
        b += struct.pack("<II", _VT.ARRAY, _VT.STRING if val and isinstance(val[0], str) else
                         _VT.INT32)
        b += struct.pack("<Q", len(val))
        for v in val:
            if isinstance(v, str):
                _s(b, v)
            else:
                b += struct.pack("<i", int(v))
    else:
        raise TypeError(f"unsupported metadata type for {key}: {type(val)}")


def quantize_q8_0(x: np.ndarray) -> bytes:
    """Blocks of 32: fp16 scale d = max|x|/127, then 32 int8 codes round(x/d)."""
    flat = x.astype(np.float32).reshape(-1)
    if flat.size % 32:
        raise ValueError("Q8_0 needs a multiple of 32 elements")
    blk = flat.reshape(-1, 32)
    d = np.abs(blk).max(1) / 127.0
    q = np.where(d[:, None] > 0, np.round(blk / np.where(d[:, None] > 0, d[:, None], 1)), 0)
    out = np.empty(blk.shape[0], dtype=[("d", "<f2"), ("q", "i1", 32)])
    out["d"] = d.astype(np.float16)
    out["q"] = q.astype(np.int8)
    return out.tobytes()


def dequantize_q8_0(raw: bytes, n: int) -> np.ndarray:
    arr = np.frombuffer(raw, dtype=[("d", "<f2"), ("q", "i1", 32)])
    return (arr["q"].astype(np.float32) * arr["d"].astype(np.float32)[:, None]).reshape(-1)[:n]


@dataclass
class GGUFTensorInfo:
    """One tensor-info record: name, dims (innermost first), type, and byte
    offset inside the aligned data section."""
    name: str
    dims: List[int]
    dtype: GGUFQuantType
    offset: int


class GGUFWriter:
    def __init__(self, path, arch: str = "tr_hash"):
        self.path = Path(path)
        self.arch = arch
        self.meta: Dict[str, Any] = {"general.architecture": arch}
        self.tensors: List[Tuple[str, List[int], GGUFQuantType, bytes]] = []

    def add_metadata(self, key: str, value: Any) -> None:
        self.meta[key] = value

    def add_tensor(self, name: str, t: torch.Tensor, qtype: GGUFQuantType = GGUFQuantType.F16):
        a = t.detach().float().cpu().numpy()
        if qtype == GGUFQuantType.F32:
            raw = a.astype("<f4").tobytes()
        elif qtype == GGUFQuantType.F16:
            raw = a.astype("<f2").tobytes()
        elif qtype == GGUFQuantType.Q8_0:
            if a.shape[-1] % 32:
                qtype, raw = GGUFQuantType.F16, a.astype("<f2").tobytes()
            else:
                raw = quantize_q8_0(a)
        else:
            raise ValueError(f"unsupported tensor type {qtype}")
        self.tensors.append((name, list(reversed(a.shape)), qtype, raw))

    def tensor_infos(self) -> List[GGUFTensorInfo]:
        """The tensor-info records ``write`` emits, with their data offsets."""
        out, off = [], 0
        for name, dims, qt, raw in self.tensors:
            out.append(GGUFTensorInfo(name, list(dims), qt, off))
            off += (len(raw) + ALIGN - 1) // ALIGN * ALIGN
        return out

    def write(self) -> Path:
        head = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self.tensors),
                                     len(self.meta)))
        for k, v in self.meta.items():
            _kv(head, k, v)
        for info in self.tensor_infos():
            _s(head, info.name)
            head += struct.pack("<I", len(info.dims))
            for d in info.dims:
                head += struct.pack("<Q", d)
            head += struct.pack("<IQ", int(info.dtype), info.offset)
        head += b"\0" * ((-len(head)) % ALIGN)
        with self.path.open("wb") as f:
            f.write(head)
            for (_, _, _, raw) in self.tensors:
                f.write(raw)
                f.write(b"\0" * ((-len(raw)) % ALIGN))
        return self.path


def _gguf_name(name: str) -> str:
    table = [("embed_tokens.weight", "token_embd.weight"), ("norm.weight", "output_norm.weight"),
             ("lm_head.weight", "output.weight")]
    for a, b in table:
        if name == a:
            return b
    n = name.replace("layers.", "blk.")
    for a, b in (("self_attn.q_proj", "attn_q"), ("self_attn.k_proj", "attn_k"),
                 ("self_attn.v_proj", "attn_v"), ("self_attn.o_proj", "attn_output"),
                 ("self_attn.q_norm", "attn_q_norm"), ("self_attn.k_norm", "attn_k_norm"),
                 ("input_layernorm", "attn_norm"), ("post_attention_layernorm", "ffn_norm"),
                 ("mlp.engine.shared_gate", "ffn_gate_shexp"),
                 ("mlp.engine.shared_up", "ffn_up_shexp"),
                 ("mlp.engine.shared_down", "ffn_down_shexp"),
                 ("mlp.engine.expert_gate", "ffn_gate_exps.weight"),
                 ("mlp.engine.expert_up", "ffn_up_exps.weight"),
                 ("mlp.engine.expert_down", "ffn_down_exps.weight"),
                 ("mlp.engine.route_table", "ffn_route_table")):
        n = n.replace(a, b)
    return n


def export_gguf(model, path, qtype: GGUFQuantType = GGUFQuantType.Q8_0) -> Path:
    cfg = model.config
    w = GGUFWriter(path)
    a = w.arch
    for k, v in (("context_length", cfg.max_position_embeddings),
                 ("embedding_length", cfg.hidden_size), ("block_count", cfg.num_hidden_layers),
                 ("attention.head_count", cfg.num_attention_heads),
                 ("attention.head_count_kv", cfg.num_key_value_heads),
                 ("expert_count", cfg.num_experts), ("expert_used_count", cfg.top_k),
                 ("rope.freq_base", float(cfg.rope_theta)),
                 ("attention.layer_norm_rms_epsilon", float(cfg.norm_eps))):
        w.add_metadata(f"{a}.{k}", v)
    w.add_metadata("general.name", "complexity_framework_b200 TR-Hash")
    for name, t in model.state_dict().items():
        if "fused_" in name or "inv_freq" in name:
            continue
        if not t.is_floating_point():
            w.add_tensor(_gguf_name(name), t.float(), GGUFQuantType.F32)
        elif t.ndim >= 2:
            w.add_tensor(_gguf_name(name), t, qtype)
        else:
            w.add_tensor(_gguf_name(name), t, GGUFQuantType.F32)
    return w.write()


def read_gguf_header(path) -> Dict[str, Any]:
    """Minimal reader (header + tensor infos) used to validate written files."""
    data = Path(path).read_bytes()
    magic, ver, nt, nkv = struct.unpack_from("<IIQQ", data, 0)
    return {"magic": magic, "version": ver, "n_tensors": nt, "n_kv": nkv}
