"""Training hyper-parameters (field names/validation as complexity/training/config.py:8-168)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass
class TrainingConfig:
    max_steps: int = 100000
    max_epochs: Optional[int] = None
    batch_size: int = 32
    gradient_accumulation_steps: int = 1
    optimizer_type: str = "adamw"
    learning_rate: float = 1e-4
    weight_decay: float = 0.1
    muon_lr: float = 0.02
    mup_base_width: int = 256
    expert_lr_scale: float = 1.5
    expert_weight_decay: float = 0.005
    expert_lr_pack: bool = False
    adaptive_ns: bool = True
    warmup_steps: int = 1000
    lr_scheduler: str = "auto"
    min_lr_ratio: float = 0.1
    wsd_decay_ratio: float = 0.2
    precision: str = "bf16"
    grad_clip: float = 1.0
    skip_param_update_check: bool = False
    # capture forward + backward + optimizer of a step in one CUDA graph after
    # `cuda_graph_warmup` eager steps (single GPU, fused AdamW); replays skip
    # the per-kernel launch overhead
    cuda_graph: bool = False
    cuda_graph_warmup: int = 3
    use_fsdp: bool = True
    sharding_mode: str = "full_shard"
    checkpoint_dir: str = "checkpoints"
    save_steps: int = 1000
    save_total_limit: int = 3
    resume_from: Optional[str] = None
    init_checkpoint: Optional[str] = None
    log_steps: int = 10
    eval_steps: int = 500
    log_dir: str = "logs"
    num_workers: int = 4
    pin_memory: bool = True
    distributed_mode: str = "auto"  # auto | none | ddp | fsdp (ZeRO-2) | zero3

    def __post_init__(self) -> None:
        checks = (
            (self.max_steps > 0, "max_steps must be positive"),
            (self.max_epochs is None or self.max_epochs > 0, "max_epochs must be positive when set"),
            (self.batch_size > 0, "batch_size must be positive"),
            (self.gradient_accumulation_steps > 0, "gradient_accumulation_steps must be positive"),
            (self.learning_rate > 0, "learning_rate must be positive"),
            (self.weight_decay >= 0, "weight_decay must be non-negative"),
            (self.warmup_steps >= 0, "warmup_steps must be non-negative"),
            (0.0 <= self.min_lr_ratio <= 1.0, "min_lr_ratio must be in [0, 1]"),
            (0.0 <= self.wsd_decay_ratio <= 1.0, "wsd_decay_ratio must be in [0, 1]"),
            (self.precision in ("fp32", "fp16", "bf16"), "precision must be one of: fp32, fp16, bf16"),
            (self.grad_clip >= 0, "grad_clip must be non-negative"),
            (self.save_steps > 0, "save_steps must be positive"),
            (self.log_steps > 0, "log_steps must be positive"),
            (self.eval_steps >= 0, "eval_steps must be non-negative"),
            (self.num_workers >= 0, "num_workers must be non-negative"),
            (self.distributed_mode in ("auto", "none", "ddp", "fsdp", "zero3"),
             "distributed_mode must be auto, none, ddp, fsdp or zero3"),
        )
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)

    @property
    def eval_every_n_steps(self) -> int:
        return self.eval_steps

    @eval_every_n_steps.setter
    def eval_every_n_steps(self, v: int) -> None:
        self.eval_steps = v

    @property
    def save_every_n_steps(self) -> int:
        return self.save_steps

    @save_every_n_steps.setter
    def save_every_n_steps(self, v: int) -> None:
        self.save_steps = v

    @property
    def log_every_n_steps(self) -> int:
        return self.log_steps

    @log_every_n_steps.setter
    def log_every_n_steps(self, v: int) -> None:
        self.log_steps = v

    @property
    def max_grad_norm(self) -> float:
        return self.grad_clip

    @max_grad_norm.setter
    def max_grad_norm(self, v: float) -> None:
        self.grad_clip = v

    @property
    def output_dir(self) -> str:
        return self.checkpoint_dir

    @output_dir.setter
    def output_dir(self, v: str) -> None:
        self.checkpoint_dir = v
