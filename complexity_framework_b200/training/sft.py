"""Supervised fine-tuning on chat data (full-parameter or LoRA).

Counterpart of scripts/sft_tr.py -> scripts/sft_500m_32k_tr.py (JSONL chat
datasets with assistant-only labels, packing, LoRA or full-parameter
training, evaluation, per-epoch checkpoints): data-parallel over ranks (each
epoch's global order padded and strided by rank, equal steps everywhere),
resumable per-epoch checkpoints that carry every rank's RNG state and the
position inside the epoch, evaluation with best-checkpoint selection and
early stopping (patience, minimum delta, minimum epochs), and curriculum
stages (training/sft_curriculum.py) whose task weights become per-token
loss weights.  Rows are JSON objects with a
``messages`` list (``role`` / ``content``); labels are the assistant tokens
only.  Batches go through the same Trainer (and fused kernels) as
pretraining; labels are shifted to next-token targets.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path
from typing import Dict, Iterator, List, Optional, Sequence

import torch

from ..data.tokenization import IGNORE_INDEX, ChatTemplate, encode_chat, get_tokenizer


class SFTDataset:
    def __init__(self, path: str, tokenizer, max_len: int = 2048, chat_format: str = "complexity"):
        self.rows = [json.loads(l) for l in Path(path).read_text().splitlines() if l.strip()]
        self.tok, self.max_len = tokenizer, max_len
        self.tpl = ChatTemplate(chat_format)

    def __len__(self) -> int:
        return len(self.rows)

    def __getitem__(self, i):
        row = self.rows[i]
        if "messages" not in row and "prompt" in row and "completion" in row:
            return encode_prompt_completion(self.tok, row["prompt"], row["completion"],
                                            self.max_len)
        ids, labels = encode_chat(self.tok, row["messages"], self.tpl, self.max_len)
        return ids, labels


def encode_prompt_completion(tok, prompt: str, completion: str, max_len: Optional[int] = None):
    """Raw prompt/completion record: labels on the completion (and EOS) only."""
    p, c = list(tok.encode(prompt)), list(tok.encode(completion))
    eos = getattr(tok, "eos_token_id", None)
    if eos is not None:
        c.append(int(eos))
    ids, labels = p + c, [IGNORE_INDEX] * len(p) + c
    if max_len is not None:
        ids, labels = ids[:max_len], labels[:max_len]
    return ids, labels


def shift_labels(labels: torch.Tensor) -> torch.Tensor:
    """Aligned labels (label[t] = token t if trainable) -> next-token targets."""
    out = torch.full_like(labels, IGNORE_INDEX)
    out[:, :-1] = labels[:, 1:]
    return out


def collate(batch: Sequence, pad_id: int, seq_len: Optional[int] = None):
    L = seq_len or max(len(ids) for ids, _ in batch)
    ids = torch.full((len(batch), L), pad_id, dtype=torch.long)
    lab = torch.full((len(batch), L), IGNORE_INDEX, dtype=torch.long)
    for i, (x, y) in enumerate(batch):
        n = min(L, len(x))
        ids[i, :n] = torch.tensor(x[:n])
        lab[i, :n] = torch.tensor(y[:n])
    return ids, shift_labels(lab)


def pack_examples(ds: SFTDataset, seq_len: int, pad_id: int) -> List:
    """Greedy packing of whole conversations into rows of ``seq_len`` tokens."""
    rows, cur_x, cur_y = [], [], []
    for i in range(len(ds)):
        x, y = ds[i]
        if cur_x and len(cur_x) + len(x) > seq_len:
            rows.append((cur_x, cur_y))
            cur_x, cur_y = [], []
        cur_x, cur_y = cur_x + x[:seq_len], cur_y + y[:seq_len]
    if cur_x:
        rows.append((cur_x, cur_y))
    return rows


def batches(examples: List, batch_size: int, pad_id: int, seq_len: Optional[int], seed: int,
            epochs: int) -> Iterator:
    g = torch.Generator().manual_seed(seed)
    for _ in range(epochs):
        order = torch.randperm(len(examples), generator=g).tolist()
        for s in range(0, len(order), batch_size):
            yield collate([examples[j] for j in order[s:s + batch_size]], pad_id, seq_len)


# ------------------------------------------------------------------ epochs
def epoch_order(n_items: int, epoch: int, seed: int) -> List[int]:
    """The global example order of one epoch (same on every rank)."""
    g = torch.Generator().manual_seed(seed * 1000003 + epoch)
    return torch.randperm(n_items, generator=g).tolist()


def rank_epoch_items(order: Sequence[int], rank: int, world: int, batch_size: int) -> List[int]:
    """This rank's examples of an epoch: the order padded (by wrapping around) to
    a multiple of world * batch_size, then strided by rank, so every rank runs
    the same number of steps."""
    unit = world * batch_size
    n = max(unit, -(-len(order) // unit) * unit)
    padded = [order[i % len(order)] for i in range(n)]
    return padded[rank::world]


def weighted_sft_loss(model, input_ids, packed_labels):
    """Per-token weighted next-token CE: ``packed_labels [..., 2]`` holds (label,
    weight); the loss is sum(w * ce) / sum(w) over supervised tokens."""
    labels = packed_labels[..., 0].long()
    weights = packed_labels[..., 1].float()
    hidden = model(input_ids, return_logits=False)["last_hidden_state"]
    W = model.output_weight()
    h = hidden.reshape(-1, hidden.shape[-1])
    y = labels.reshape(-1)
    w = weights.reshape(-1)
    valid = y != IGNORE_INDEX
    total = h.new_zeros((), dtype=torch.float32)
    for s in range(0, h.shape[0], 4096):
        logits = (h[s:s + 4096] @ W.t()).float()
        ce = torch.nn.functional.cross_entropy(logits, y[s:s + 4096].clamp_min(0),
                                               reduction="none")
        total = total + (ce * w[s:s + 4096] * valid[s:s + 4096]).sum()
    return total / (w * valid).sum().clamp_min(1e-6)


def update_early_stopping(best: float, bad_evals: int, current: float, *, min_delta: float):
    """(improved, best, evaluations without improvement) after one evaluation."""
    if current < best - min_delta:
        return True, current, 0
    return False, best, bad_evals + 1


def capture_rng_state() -> Dict:
    import random

    import numpy as np

    st = {"python": random.getstate(), "numpy": np.random.get_state(),
          "torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        st["cuda"] = torch.cuda.get_rng_state()
    return st


def restore_rng_state(st: Dict) -> None:
    import random

    import numpy as np

    random.setstate(st["python"])
    np.random.set_state(st["numpy"])
    torch.set_rng_state(st["torch"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state(st["cuda"])


def _save_sft_state(trainer, tag: str, sft_state: Dict) -> Path:
    """Trainer checkpoint + SFT position + every rank's RNG state."""
    import torch.distributed as dist

    path = trainer.save_checkpoint(tag=tag)
    states = [capture_rng_state()]
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        states = [None] * dist.get_world_size()
        dist.all_gather_object(states, capture_rng_state())
    if trainer.is_main:
        torch.save(states, path / "rng_states.pt")
        (path / "sft_state.json").write_text(json.dumps(sft_state, indent=2))
    return path


def main(argv=None) -> Dict:
    import torch.distributed as dist

    from ..models.builder import ComplexityModel
    from ..parallel.distributed import cleanup_distributed, init_distributed
    from .config import TrainingConfig
    from .lora import LoRAConfig, apply_lora, lora_state_dict
    from .sft_curriculum import load_curriculum, select_examples
    from .trainer import Trainer

    ap = argparse.ArgumentParser(description="Supervised fine-tuning")
    ap.add_argument("--model", required=True, help="checkpoint directory")
    ap.add_argument("--data", required=True, help="JSONL with a messages list per row")
    ap.add_argument("--eval-data", default=None)
    ap.add_argument("--tokenizer", default="byte")
    ap.add_argument("--output", default="sft_out")
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--batch-size", type=int, default=8, help="per rank")
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--lr", type=float, default=2e-5)
    ap.add_argument("--lora-rank", type=int, default=0, help="0 = full-parameter SFT")
    ap.add_argument("--lora-alpha", type=float, default=16.0)
    ap.add_argument("--pack", action="store_true")
    ap.add_argument("--chat-format", default="complexity")
    ap.add_argument("--precision", default="bf16")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--curriculum", default=None, help="curriculum YAML")
    ap.add_argument("--curriculum-stage", default=None)
    ap.add_argument("--eval-steps", type=int, default=0, help="0 = evaluate at epoch ends")
    ap.add_argument("--early-stopping-patience", type=int, default=0, help="0 = off")
    ap.add_argument("--early-stopping-min-delta", type=float, default=0.0)
    ap.add_argument("--early-stopping-min-epochs", type=int, default=1)
    ap.add_argument("--save-best", action="store_true")
    ap.add_argument("--resume", default=None, help="'auto' or a checkpoint directory")
    ap.add_argument("--max-steps", type=int, default=0,
                    help="stop after this many optimizer steps (0 = run the epochs)")
    ap.add_argument("--lora-targets", default=None,
                    help="comma-separated module names for LoRA (default: the standard set)")
    ap.add_argument("--merge-lora", action="store_true",
                    help="merge the trained LoRA deltas and save a full checkpoint in final/")
    a = ap.parse_args(argv)
    if (a.curriculum is None) != (a.curriculum_stage is None):
        raise SystemExit("--curriculum and --curriculum-stage go together")
    rank, world, _, device = init_distributed()
    try:
        return _run(a, rank, world, device, ComplexityModel, TrainingConfig, LoRAConfig,
                    apply_lora, lora_state_dict, load_curriculum, select_examples, Trainer)
    finally:
        if world > 1:
            dist.barrier()
        cleanup_distributed()


def _run(a, rank, world, device, ComplexityModel, TrainingConfig, LoRAConfig, apply_lora,
         lora_state_dict, load_curriculum, select_examples, Trainer) -> Dict:
    import torch.distributed as dist

    tok = get_tokenizer(a.tokenizer) if a.tokenizer == "byte" else get_tokenizer(
        "sentencepiece" if a.tokenizer.endswith(".model") else "huggingface", a.tokenizer)
    torch.manual_seed(a.seed)
    model = ComplexityModel.from_pretrained(a.model)
    if a.lora_rank > 0:
        lcfg = LoRAConfig(r=a.lora_rank, alpha=a.lora_alpha)
        if a.lora_targets:
            lcfg.target_modules = [t.strip() for t in a.lora_targets.split(",") if t.strip()]
        apply_lora(model, lcfg)
    if Path(a.data).is_dir():  # pre-tokenised SFT shards (input_ids.bin / labels.bin)
        from ..data.sft_shards import SFTTokenShardDataset

        ds = SFTTokenShardDataset(a.data, a.seq_len)
        ds.rows = [{} for _ in range(len(ds))]
    else:
        ds = SFTDataset(a.data, tok, a.seq_len, a.chat_format)
    pad = tok.pad_token_id or 0
    keep = list(range(len(ds)))
    stage = None
    if a.curriculum:
        cur = load_curriculum(a.curriculum)
        stage = cur.stage(a.curriculum_stage)
        counts = []
        for i in range(len(ds)):
            x, y = ds[i]
            counts.append((len(x), sum(1 for t in y if t != IGNORE_INDEX)))
        keep = select_examples(ds.rows, stage, seed=cur.seed, token_counts=counts)
        if not keep:
            raise SystemExit(f"curriculum stage {stage.name!r} selects no examples")
    weighted = stage is not None and any(w != 1.0 for _, w in stage.task_weights)
    items = []
    for i in keep:
        x, y = ds[i]
        w = stage.task_weight(ds.rows[i].get("task")) if stage is not None else 1.0
        items.append((x, y, w))
    if a.pack:
        packed = pack_examples(_ListDS([(x, y) for x, y, _ in items]), a.seq_len, pad)
        items = [(x, y, 1.0) for x, y in packed]
        weighted = False
    steps_per_epoch = len(rank_epoch_items(list(range(len(items))), rank, world,
                                           a.batch_size)) // a.batch_size
    if a.max_steps > 0 and steps_per_epoch > 0:
        a.epochs = max(a.epochs, -(-a.max_steps // steps_per_epoch))
    total_steps = steps_per_epoch * a.epochs
    if a.max_steps > 0:
        total_steps = min(total_steps, a.max_steps)
    cfg = TrainingConfig(max_steps=total_steps, learning_rate=a.lr,
                         warmup_steps=max(1, total_steps // 20), lr_scheduler="cosine",
                         precision=a.precision, weight_decay=0.0, checkpoint_dir=a.output,
                         save_steps=10 ** 12, log_steps=1, skip_param_update_check=True,
                         distributed_mode="ddp" if world > 1 else "none")
    tr = Trainer(model, cfg, device=device,
                 compute_loss=weighted_sft_loss if weighted else None)
    sft = {"epoch": 0, "step_in_epoch": 0, "best_eval_loss": float("inf"),
           "evals_without_improvement": 0, "stopped_early": False}
    if a.resume:
        if tr.resume(a.resume):
            target = Path(tr.ckpt.latest() if a.resume == "auto" else a.resume)
            sft.update(json.loads((target / "sft_state.json").read_text()))
            states = torch.load(target / "rng_states.pt", weights_only=False)
            restore_rng_state(states[rank if rank < len(states) else 0])

    evaluator = None
    if a.eval_data:
        ev = SFTDataset(a.eval_data, tok, a.seq_len, a.chat_format)
        ev_items = [ev[i] for i in range(len(ev))]

        def evaluator():
            mine = ev_items[rank::world] or ev_items[:1]
            loss = tr.evaluate(batches(mine, min(a.batch_size, len(mine)), pad, None, 0, 1))
            if world > 1:
                t = torch.tensor([loss], device=tr.device, dtype=torch.float64)
                dist.all_reduce(t)
                loss = float(t.item()) / world
            return loss

    def evaluate_and_select(epoch_done: float) -> bool:
        """Evaluate; update best/early stopping; returns True to stop."""
        if evaluator is None:
            return False
        loss = evaluator()
        eligible = epoch_done >= a.early_stopping_min_epochs
        history.append({"step": tr.global_step, "eval_loss": loss})
        if not eligible:
            return False
        improved, sft["best_eval_loss"], sft["evals_without_improvement"] = update_early_stopping(
            sft["best_eval_loss"], sft["evals_without_improvement"], loss,
            min_delta=a.early_stopping_min_delta)
        if improved and a.save_best:
            path = _save_sft_state(tr, "best", dict(sft))
            if tr.is_main:
                (Path(a.output) / "best.json").write_text(json.dumps(
                    {"step": tr.global_step, "eval_loss": loss, "checkpoint": str(path)}, indent=2))
        return (a.early_stopping_patience > 0
                and sft["evals_without_improvement"] >= a.early_stopping_patience)

    history: List[Dict] = []
    last = None
    stop = False
    for epoch in range(sft["epoch"], a.epochs):
        mine = rank_epoch_items(epoch_order(len(items), epoch, a.seed), rank, world, a.batch_size)
        start = sft["step_in_epoch"] if epoch == sft["epoch"] else 0
        for s in range(start, steps_per_epoch):
            chunk = [items[j] for j in mine[s * a.batch_size:(s + 1) * a.batch_size]]
            ids, lab = collate([(x, y) for x, y, _ in chunk], pad, None)
            if weighted:
                w = torch.tensor([cw for _, _, cw in chunk], dtype=torch.float64)[:, None]
                lab = torch.stack([lab.double(), w.expand_as(lab)], -1)
            last = tr.train_step(ids, lab)
            tr._emit("on_step_end", tr.global_step, {"loss": last})
            sft["step_in_epoch"] = s + 1
            if a.max_steps > 0 and tr.global_step >= total_steps:
                stop = True
                break
            if a.eval_steps > 0 and tr.global_step % a.eval_steps == 0:
                if evaluate_and_select(epoch + (s + 1) / steps_per_epoch):
                    stop = True
                    break
        if stop:
            sft["stopped_early"] = tr.global_step < total_steps
            if not sft["stopped_early"]:
                _save_sft_state(tr, "epoch", dict(sft))
            break
        sft["epoch"], sft["step_in_epoch"] = epoch + 1, 0
        if a.eval_steps <= 0 and evaluate_and_select(epoch + 1):
            sft["stopped_early"] = True
            _save_sft_state(tr, "epoch", dict(sft))
            break
        _save_sft_state(tr, "epoch", dict(sft))           # resumable per-epoch checkpoint

    summary = {"steps": tr.global_step, "last_loss": last, "epochs_done": sft["epoch"],
               "stopped_early": sft["stopped_early"], "eval_history": history,
               "best_eval_loss": sft["best_eval_loss"], "examples": len(items),
               "curriculum_stage": stage.name if stage is not None else None}
    if history:
        summary["eval_loss"] = history[-1]["eval_loss"]
        summary["eval_ppl"] = math.exp(min(50.0, history[-1]["eval_loss"]))
    out = Path(a.output)
    if tr.is_main:
        out.mkdir(parents=True, exist_ok=True)
        if a.lora_rank > 0:
            torch.save(lora_state_dict(model), out / "adapter.pt")
        (out / "sft_summary.json").write_text(json.dumps(summary, indent=2, default=float))
    if a.lora_rank > 0 and a.merge_lora:
        from .lora import merge_lora

        merge_lora(model)
    if a.lora_rank <= 0 or a.merge_lora:
        model.save_pretrained(out / "final")
    return summary


class _ListDS:
    def __init__(self, items):
        self.items = items

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        return self.items[i]


if __name__ == "__main__":
    main()
