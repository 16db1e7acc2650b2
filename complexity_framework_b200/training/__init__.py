"""Training stack: config, flat fp32-master AdamW, schedulers, Trainer."""
from .config import TrainingConfig
from .optim import FusedAdamW, default_param_groups
from .scheduler import build_scheduler, lr_multiplier
from .trainer import Trainer

__all__ = ["FusedAdamW", "Trainer", "TrainingConfig", "build_scheduler", "default_param_groups",
           "lr_multiplier"]
