"""Supervised fine-tuning on chat data (full-parameter or LoRA).

Counterpart of scripts/sft_tr.py -> scripts/sft_500m_32k_tr.py (JSONL chat
datasets with assistant-only labels, packing, LoRA or full-parameter
training, evaluation, per-epoch checkpoints).  Rows are JSON objects with a
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
        ids, labels = encode_chat(self.tok, self.rows[i]["messages"], self.tpl, self.max_len)
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


def main(argv=None) -> Dict:
    from ..models.builder import ComplexityModel
    from .config import TrainingConfig
    from .lora import LoRAConfig, apply_lora, lora_state_dict
    from .trainer import Trainer

    ap = argparse.ArgumentParser(description="Supervised fine-tuning")
    ap.add_argument("--model", required=True, help="checkpoint directory")
    ap.add_argument("--data", required=True, help="JSONL with a messages list per row")
    ap.add_argument("--eval-data", default=None)
    ap.add_argument("--tokenizer", default="byte")
    ap.add_argument("--output", default="sft_out")
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--lr", type=float, default=2e-5)
    ap.add_argument("--lora-rank", type=int, default=0, help="0 = full-parameter SFT")
    ap.add_argument("--lora-alpha", type=float, default=16.0)
    ap.add_argument("--pack", action="store_true")
    ap.add_argument("--chat-format", default="complexity")
    ap.add_argument("--precision", default="bf16")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    tok = get_tokenizer(a.tokenizer) if a.tokenizer == "byte" else get_tokenizer(
        "sentencepiece" if a.tokenizer.endswith(".model") else "huggingface", a.tokenizer)
    model = ComplexityModel.from_pretrained(a.model)
    if a.lora_rank > 0:
        apply_lora(model, LoRAConfig(r=a.lora_rank, alpha=a.lora_alpha))
    ds = SFTDataset(a.data, tok, a.seq_len, a.chat_format)
    pad = tok.pad_token_id or 0
    examples = pack_examples(ds, a.seq_len, pad) if a.pack else [ds[i] for i in range(len(ds))]
    steps = -(-len(examples) // a.batch_size) * a.epochs
    cfg = TrainingConfig(max_steps=steps, learning_rate=a.lr, warmup_steps=max(1, steps // 20),
                         lr_scheduler="cosine", precision=a.precision, weight_decay=0.0,
                         checkpoint_dir=a.output, save_steps=max(1, steps), log_steps=1,
                         skip_param_update_check=True)
    tr = Trainer(model, cfg)
    summary = tr.train(batches(examples, a.batch_size, pad, None, a.seed, a.epochs))
    if a.eval_data:
        ev = SFTDataset(a.eval_data, tok, a.seq_len, a.chat_format)
        summary["eval_loss"] = tr.evaluate(batches([ev[i] for i in range(len(ev))],
                                                   min(a.batch_size, len(ev)), pad, None, 0, 1))
        summary["eval_ppl"] = math.exp(min(50.0, summary["eval_loss"]))
    out = Path(a.output)
    out.mkdir(parents=True, exist_ok=True)
    if a.lora_rank > 0:
        torch.save(lora_state_dict(model), out / "adapter.pt")
    else:
        model.save_pretrained(out / "final")
    (out / "sft_summary.json").write_text(json.dumps(summary, indent=2, default=float))
    return summary


if __name__ == "__main__":
    main()
