"""Safe checkpoint loading, hashes and manifests, input validation, audit log.

Counterpart of complexity/utils/security.py:37-470: ``safe_torch_load``
(``weights_only`` loading with an allow-list, size limit and optional hash
check), safetensors helpers, model hashes, ``ModelManifest``, distributed
environment / input-id validation, config sanitising and ``AuditLogger``.
"""
from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Union

import torch
import torch.nn as nn


class UnsafeCheckpointError(Exception):
    pass


def file_sha256(path: Union[str, Path], chunk: int = 8 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(chunk), b""):
            h.update(b)
    return h.hexdigest()


def safe_torch_load(path: Union[str, Path], map_location="cpu", *, max_size_gb: float = 100.0,
                    expected_sha256: Optional[str] = None, allow_pickle: bool = False):
    """``torch.load`` restricted to tensors and plain containers (no arbitrary
    unpickling) unless ``allow_pickle``; rejects oversized files and hash mismatches."""
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(path)
    size_gb = path.stat().st_size / 1e9
    if size_gb > max_size_gb:
        raise UnsafeCheckpointError(f"{path} is {size_gb:.1f} GB > limit {max_size_gb} GB")
    if expected_sha256 is not None and file_sha256(path) != expected_sha256:
        raise UnsafeCheckpointError(f"sha256 mismatch for {path}")
    if path.suffix == ".safetensors":
        return load_safetensors(path)
    try:
        return torch.load(path, map_location=map_location, weights_only=not allow_pickle)
    except Exception as e:  # noqa: BLE001 - surfaced as a security error
        if allow_pickle:
            raise
        raise UnsafeCheckpointError(f"{path} needs unpickling of non-tensor objects: {e}") from e


def load_safetensors(path) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    return load_file(str(path))


def save_safetensors(state_dict: Dict[str, torch.Tensor], path, metadata=None) -> None:
    from safetensors.torch import save_file

    save_file({k: v.detach().contiguous().cpu() for k, v in state_dict.items()}, str(path),
              metadata=metadata)


def compute_model_hash(model: nn.Module, algorithm: str = "sha256") -> str:
    """Hash over parameter/buffer names, shapes, dtypes and bytes (order-independent of devices)."""
    h = hashlib.new(algorithm)
    for k, v in sorted(model.state_dict().items()):
        t = v.detach().contiguous().cpu()
        h.update(k.encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()


def verify_model_hash(model: nn.Module, expected: str, algorithm: str = "sha256") -> bool:
    return compute_model_hash(model, algorithm) == expected


@dataclass
class ModelManifest:
    model_hash: str
    num_parameters: int
    config: Dict[str, Any]
    files: Dict[str, str] = field(default_factory=dict)
    created: float = field(default_factory=time.time)
    framework: str = "complexity_framework_b200"

    def save(self, path) -> None:
        Path(path).write_text(json.dumps(asdict(self), indent=2, sort_keys=True))

    @classmethod
    def load(cls, path) -> "ModelManifest":
        return cls(**json.loads(Path(path).read_text()))

    def verify_files(self, root) -> List[str]:
        """Names of files whose sha256 no longer matches."""
        return [f for f, h in self.files.items() if file_sha256(Path(root) / f) != h]


def create_model_manifest(model: nn.Module, directory=None) -> ModelManifest:
    cfg = getattr(model, "config", None)
    files = {}
    if directory is not None:
        for p in sorted(Path(directory).iterdir()):
            if p.is_file() and p.name != "manifest.json":
                files[p.name] = file_sha256(p)
    return ModelManifest(compute_model_hash(model), sum(p.numel() for p in model.parameters()),
                         cfg.to_dict() if hasattr(cfg, "to_dict") else {}, files)


def validate_distributed_env() -> Dict[str, Any]:
    """Checks the torchrun variables are coherent; returns them."""
    env = {k: os.environ.get(k) for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR",
                                          "MASTER_PORT")}
    if env["WORLD_SIZE"] is not None:
        w, r = int(env["WORLD_SIZE"]), int(env["RANK"] or 0)
        if not 0 <= r < w:
            raise ValueError(f"RANK {r} outside WORLD_SIZE {w}")
        if env["MASTER_PORT"] is not None and not 0 < int(env["MASTER_PORT"]) < 65536:
            raise ValueError("MASTER_PORT out of range")
    return env


def validate_input_ids(input_ids: torch.Tensor, vocab_size: int, max_len: Optional[int] = None) -> None:
    if input_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("input_ids must be an integer tensor")
    if input_ids.numel() and (int(input_ids.min()) < 0 or int(input_ids.max()) >= vocab_size):
        raise ValueError(f"token ids must lie in [0, {vocab_size})")
    if max_len is not None and input_ids.shape[-1] > max_len:
        raise ValueError(f"sequence length {input_ids.shape[-1]} > {max_len}")


_SECRET_KEYS = ("token", "key", "secret", "password", "credential")


def sanitize_config(config: Dict[str, Any]) -> Dict[str, Any]:
    """Copy with secret-looking values masked (for logs and manifests)."""
    out = {}
    for k, v in config.items():
        if isinstance(v, dict):
            out[k] = sanitize_config(v)
        elif any(s in k.lower() for s in _SECRET_KEYS) and v:
            out[k] = "***"
        else:
            out[k] = v
    return out


class AuditLogger:
    """Append-only JSONL audit trail (training start/end, checkpoint saves/loads)."""

    def __init__(self, path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)

    def log(self, event: str, **details) -> None:
        rec = {"time": time.time(), "event": event, "pid": os.getpid(),
               "rank": int(os.environ.get("RANK", "0")), **sanitize_config(details)}
        with self.path.open("a") as f:
            f.write(json.dumps(rec, default=str) + "\n")

    def events(self) -> List[Dict[str, Any]]:
        if not self.path.exists():
            return []
        return [json.loads(l) for l in self.path.read_text().splitlines() if l.strip()]


class SecureTrainingContext:
    """Context that validates the environment and audits start/end of a run."""

    def __init__(self, audit_path, config: Optional[Dict[str, Any]] = None):
        self.audit = AuditLogger(audit_path)
        self.config = config or {}

    def __enter__(self):
        validate_distributed_env()
        self.audit.log("training_start", config=self.config)
        return self

    def __exit__(self, et, ev, tb):
        self.audit.log("training_end", ok=et is None, error=repr(ev) if ev else None)
        return False
