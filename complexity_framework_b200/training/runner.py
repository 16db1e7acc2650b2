"""Standard training pipeline behind the command-line entry points.

Counterpart of complexity/training/runner.py:161-567 (``TrainRunner``): the
same flags (``--target-tokens``, ``--batch-size``, ``--seq-len``,
``--gradient-accumulation``, ``--lr``, ``--warmup-steps|--warmup-tokens``,
``--lr-scheduler``, ``--max-steps``, ``--save-steps``, ``--token-packs``,
``--log-steps``, ``--checkpoint-dir``, ``--resume [auto|DIR]``,
``--init-checkpoint``, ``--distributed-mode``, ``--precision``,
``--optimizer``, ``--top-k``, ``--use-custom-kernels``, ``--wandb``), YAML run
configs (``--config``), SIGTERM -> "interrupted" checkpoint, per-step
``training_log.csv`` + ``metrics.jsonl`` and a final HF-style export in
``<checkpoint-dir>/final``.

Input data: ``--data DIR`` (a token shard, read by the native loader) or
``--synthetic`` (Zipf token ids, for smoke runs and benchmarks).
"""
from __future__ import annotations

import argparse
import logging
import math
import os
import signal
from pathlib import Path
from typing import Callable, Optional

import torch

from ..config.model_config import ModelConfig, get_preset
from ..parallel.distributed import cleanup_distributed, init_distributed
from .callbacks import CSVLoggerCallback, MetricsJsonlCallback, TqdmCallback, WandBCallback
from .config import TrainingConfig
from .run_config import (args_to_run_config, parse_args_with_yaml_config, token_shard_fingerprint,
                         write_or_validate_run_config)
from .trainer import Trainer

logger = logging.getLogger(__name__)


def _raise_interrupt(signum, frame):  # noqa: ARG001
    raise KeyboardInterrupt(f"signal {signum}")


class TrainRunner:
    """Subclass (or pass ``make_config``) to define a run; ``main()`` does the rest."""

    run_name = "complexity"
    default_target_tokens = 1_000_000_000
    default_batch_size = 8
    default_seq_len = 1024
    default_gradient_accumulation = 1
    default_lr = 3e-4
    default_save_steps = 1000
    default_distributed_mode = "ddp"
    optimizer_type = "adamw"
    checkpoint_dir = "checkpoints"

    def __init__(self, make_config: Optional[Callable[[argparse.Namespace], ModelConfig]] = None):
        self._make_config = make_config

    # ------------------------------------------------------------- arguments
    def add_args(self, p: argparse.ArgumentParser) -> None:
        """Hook for run-specific flags."""

    def build_parser(self) -> argparse.ArgumentParser:
        p = argparse.ArgumentParser(description=f"Train {self.run_name}")
        p.add_argument("--model", type=str, default=None, help="preset name or config.json/yaml")
        p.add_argument("--data", type=str, default=None, help="token shard directory")
        p.add_argument("--synthetic", action="store_true", help="Zipf synthetic token ids")
        p.add_argument("--token-mixture", type=str, default=None,
                       help="pretokenized corpus mixture directory (mixture_manifest.json)")
        p.add_argument("--replay-plan", type=str, default=None,
                       help="token replay plan for --token-mixture")
        p.add_argument("--tokenizer", type=str, default=None)
        p.add_argument("--target-tokens", type=str, default=str(self.default_target_tokens))
        p.add_argument("--batch-size", type=int, default=self.default_batch_size)
        p.add_argument("--seq-len", type=int, default=self.default_seq_len)
        p.add_argument("--gradient-accumulation", type=int,
                       default=self.default_gradient_accumulation)
        p.add_argument("--lr", type=float, default=self.default_lr)
        p.add_argument("--warmup-steps", type=int, default=None)
        p.add_argument("--warmup-tokens", type=str, default=None)
        p.add_argument("--lr-scheduler", default="auto",
                       choices=["auto", "cosine", "linear", "constant", "wsd"])
        p.add_argument("--max-steps", type=int, default=None)
        p.add_argument("--save-steps", type=int, default=self.default_save_steps)
        p.add_argument("--token-packs", type=int, default=1)
        p.add_argument("--log-steps", type=int, default=10)
        p.add_argument("--eval-steps", type=int, default=0)
        p.add_argument("--checkpoint-dir", type=str, default=self.checkpoint_dir)
        p.add_argument("--resume", type=str, default=None)
        p.add_argument("--init-checkpoint", type=str, default=None)
        p.add_argument("--num-workers", type=int, default=4)
        p.add_argument("--distributed-mode", choices=["fsdp", "ddp"],
                       default=self.default_distributed_mode)
        p.add_argument("--wandb", type=str, default=None)
        p.add_argument("--precision", default="bf16", choices=["fp32", "fp16", "bf16"])
        p.add_argument("--optimizer", default=self.optimizer_type,
                       choices=["adamw", "adamw_mup", "muon", "muon_tr", "adam_tr", "lion",
                                "sophia", "adam8bit", "came", "adalomo", "musgd"])
        p.add_argument("--weight-decay", type=float, default=0.1)
        p.add_argument("--grad-clip", type=float, default=1.0)
        p.add_argument("--top-k", type=int, default=None)
        p.add_argument("--use-custom-kernels", default="auto", choices=["auto", "true", "false"])
        p.add_argument("--seed", type=int, default=42)
        p.add_argument("--no-progress", action="store_true")
        self.add_args(p)
        return p

    # ----------------------------------------------------------------- model
    def make_config(self, args: argparse.Namespace) -> ModelConfig:
        if self._make_config is not None:
            return self._make_config(args)
        if args.model is None:
            return get_preset("tr-hash-200m")
        if os.path.exists(args.model):
            return ModelConfig.load(args.model)
        return get_preset(args.model)

    def build_model(self, cfg: ModelConfig):
        from ..models.builder import ComplexityModel

        return ComplexityModel(cfg)

    # ------------------------------------------------------------------ data
    def build_batches(self, args, rank: int, world: int, start_batch: int):
        if args.token_mixture:
            from ..data.corpus_mixture import PretokenizedCorpusMixtureDataset

            # every optimizer step consumes one batch of batch_size rows on each
            # rank: a resumed run skips exactly the rows it already trained on
            skip = start_batch * args.batch_size
            ds = PretokenizedCorpusMixtureDataset(args.token_mixture, rank=rank,
                                                  world_size=world,
                                                  replay_plan=args.replay_plan,
                                                  resume_skip_rows=skip)
            if ds.seq_len != args.seq_len:
                raise SystemExit(f"--seq-len {args.seq_len} but the mixture has rows of "
                                 f"{ds.seq_len} tokens")

            def rows():
                buf_x, buf_y = [], []
                for item in ds:
                    buf_x.append(item["input_ids"])
                    buf_y.append(item["labels"])
                    if len(buf_x) == args.batch_size:
                        yield torch.stack(buf_x), torch.stack(buf_y)
                        buf_x, buf_y = [], []

            return rows()
        if args.data:
            from ..data.loader import TokenBatchLoader

            return TokenBatchLoader(args.data, args.batch_size, args.seq_len, rank=rank,
                                    world_size=world, seed=args.seed, order="sequential"
                                    if args.token_packs > 1 else "random",
                                    start_batch=start_batch)
        if not args.synthetic:
            raise SystemExit("pass --data <token shard>, --token-mixture <dir> or --synthetic")
        g = torch.Generator().manual_seed(args.seed + 7919 * rank)
        vocab = self.cfg.vocab_size

        def gen():
            while True:
                # Zipf-like ids: floor(V^u) - 1 with u uniform is heavy-tailed
                u = torch.rand(args.batch_size, args.seq_len + 1, generator=g)
                ids = (torch.pow(float(vocab), u).long() - 1).clamp_(0, vocab - 1)
                yield ids[:, :-1], ids[:, 1:]

        return gen()

    # ------------------------------------------------------------------- run
    def main(self, argv=None) -> dict:
        args = parse_args_with_yaml_config(self.build_parser(), argv)
        logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
        rank, world, local, device = init_distributed()
        torch.manual_seed(args.seed)
        prev = signal.signal(signal.SIGTERM, _raise_interrupt)
        try:
            return self._run(args, rank, world, device)
        finally:
            signal.signal(signal.SIGTERM, prev)
            cleanup_distributed()

    def _run(self, args, rank, world, device) -> dict:
        from ..parallel.distributed import barrier
        from ..utils.checkpointing import load_weights_only, peek_latest_checkpoint_step
        from .cluster_plan import parse_tokens

        self.cfg = cfg = self.make_config(args)
        if args.top_k is not None:
            cfg.top_k = args.top_k
        if args.use_custom_kernels != "auto":
            cfg.use_custom_kernels = args.use_custom_kernels == "true"
        tokens_per_step = args.batch_size * args.seq_len * args.gradient_accumulation * world
        target = parse_tokens(args.target_tokens)
        max_steps = args.max_steps or max(1, math.ceil(target / tokens_per_step))
        if args.warmup_steps is not None:
            warmup = args.warmup_steps
        elif args.warmup_tokens is not None:
            warmup = math.ceil(parse_tokens(args.warmup_tokens) / tokens_per_step)
        else:
            warmup = min(2000, max(1, max_steps // 100))
        save_steps = args.save_steps
        if args.token_packs > 1:
            save_steps = max(1, math.ceil(max_steps / args.token_packs))
        tcfg = TrainingConfig(max_steps=max_steps, batch_size=args.batch_size,
                              gradient_accumulation_steps=args.gradient_accumulation,
                              optimizer_type=("adamw" if args.optimizer == "adamw_mup"
                                              else args.optimizer),
                              learning_rate=args.lr, weight_decay=args.weight_decay,
                              warmup_steps=warmup, lr_scheduler=args.lr_scheduler,
                              precision=args.precision, grad_clip=args.grad_clip,
                              checkpoint_dir=args.checkpoint_dir, save_steps=save_steps,
                              log_steps=args.log_steps, eval_steps=args.eval_steps,
                              num_workers=args.num_workers,
                              distributed_mode=args.distributed_mode if world > 1 else "none")
        model = self.build_model(cfg)
        if args.init_checkpoint:
            load_weights_only(model, args.init_checkpoint)
        ckdir = Path(args.checkpoint_dir)
        logs = ckdir / "logs"
        callbacks = [CSVLoggerCallback(str(logs / "training_log.csv")),
                     MetricsJsonlCallback(str(logs / "metrics.jsonl"), {"run": self.run_name})]
        if not args.no_progress:
            callbacks.append(TqdmCallback(max_steps))
        if args.wandb:
            callbacks.append(WandBCallback(args.wandb, vars(args)))
        trainer = Trainer(model, tcfg, device=device, callbacks=callbacks)
        run_cfg = args_to_run_config(args, {"world_size": world, "max_steps": max_steps,
                                            "model_config": cfg.to_dict(),
                                            "data": token_shard_fingerprint(args.data)})
        if rank == 0:
            for k, a, b in write_or_validate_run_config(ckdir, run_cfg):
                logger.warning("run config changed on resume: %s: %r -> %r", k, a, b)
        if args.resume:
            if args.resume == "auto" and peek_latest_checkpoint_step(str(ckdir)) is None:
                logger.info("no checkpoint under %s; starting fresh", ckdir)
            else:
                trainer.resume(args.resume)
                logger.info("resumed at step %d", trainer.global_step)
        if rank == 0:
            logger.info("TRAINING CONFIG: %s params, %d steps x %d tokens/step, %s, world %d",
                        f"{sum(p.numel() for p in model.parameters()):,}", max_steps,
                        tokens_per_step, args.optimizer, world)
        batches = self.build_batches(args, rank, world, trainer.global_step)
        try:
            summary = trainer.train(batches, max_steps)
        finally:
            if hasattr(batches, "close"):
                batches.close()
        trainer.save_checkpoint()
        barrier()
        if rank == 0:
            model.save_pretrained(ckdir / "final")
        return summary


def main(argv=None) -> dict:
    return TrainRunner().main(argv)


if __name__ == "__main__":
    main()
