"""GRPO / DAPO training driver and its helpers.

    python -m complexity_framework_b200.rl.train_grpo --model ckpt/ --data mmlu.jsonl \
        --task mmlu --steps 100 --output runs/grpo

Counterpart of complexity/RL/grpo/train_grpo.py:63-700: MMLU prompts in the
reference's layout (system line, "Question (subject):", lettered choices,
"Answer:"), FineWeb-Edu continuation prompts, left-truncating prompt
encoding, group sampling (here through the framework's paged engine, or an
OpenAI-compatible server in place of in-process vLLM), completion
log-probabilities with and without gradients, and the training loop on
``GRPOTrainer`` (group advantages, DAPO clipped objective, optional k3 KL).
Datasets are local files (no network): MMLU as JSONL rows ``{question,
choices, answer, subject}`` (answer an index or a letter), FineWeb-Edu as
JSONL rows ``{text}``.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import torch

from .grpo import GRPOConfig, GRPOTrainer, sequence_log_probs

CHOICES = "ABCD"
SYSTEM_PROMPT = ("Answer the following multiple choice question. Reply with the letter of the "
                 "correct option.")


def format_mmlu_prompt(question: str, choices: List[str], subject: str = "") -> str:
    opts = "\n".join(f"{CHOICES[i]}. {c}" for i, c in enumerate(choices))
    subj = f" ({subject})" if subject else ""
    return f"{SYSTEM_PROMPT}\n\nQuestion{subj}:\n{question}\n\n{opts}\n\nAnswer:"


def _jsonl(path) -> List[dict]:
    return [json.loads(x) for x in Path(path).read_text(encoding="utf-8").splitlines() if x.strip()]


def load_mmlu_dataset(path: str, subset: str = "all", max_samples: int = 0) -> List[Dict]:
    out = []
    for row in _jsonl(path):
        if subset != "all" and row.get("subject") != subset:
            continue
        a = row["answer"]
        ans = CHOICES[a] if isinstance(a, int) else str(a).strip().upper()
        out.append({"prompt": format_mmlu_prompt(row["question"], row["choices"],
                                                 row.get("subject", "")), "answer": ans})
        if max_samples and len(out) >= max_samples:
            break
    return out


def load_fineweb_edu_dataset(path: str, max_samples: int = 10000,
                             prompt_words: int = 50) -> List[Dict]:
    """The first ``prompt_words`` words of each long-enough document."""
    out = []
    for row in _jsonl(path):
        words = row.get("text", "").split()
        if len(words) < prompt_words + 20:
            continue
        out.append({"prompt": " ".join(words[:prompt_words]), "answer": ""})
        if len(out) >= max_samples:
            break
    return out


def encode_prompt(tokenizer, prompt: str, max_len: int) -> torch.Tensor:
    """Token ids (with BOS when the tokenizer has one), keeping the last ``max_len``."""
    ids = list(tokenizer.encode(prompt))
    bos = getattr(tokenizer, "bos_token_id", None)
    if bos is not None and (not ids or ids[0] != bos):
        ids = [int(bos)] + ids
    return torch.tensor(ids[-max_len:], dtype=torch.long)


def decode_tokens(tokenizer, token_ids) -> str:
    ids = token_ids.tolist() if torch.is_tensor(token_ids) else list(token_ids)
    return tokenizer.decode(ids)


@torch.no_grad()
def generate_group(model, prompt_ids: torch.Tensor, group_size: int, max_new_tokens: int,
                   temperature: float = 1.0, top_p: float = 0.9,
                   eos_token_id: Optional[int] = None, seed: Optional[int] = None) -> torch.Tensor:
    """``group_size`` sampled continuations of one prompt through the paged
    engine; returns [G, prompt + new] ids right-padded with 0."""
    from ..inference.engine import GenerationConfig, InferenceEngine

    was = model.training
    eng = InferenceEngine(model)
    gen = GenerationConfig(max_new_tokens=max_new_tokens, do_sample=True,
                           temperature=temperature, top_p=top_p, eos_token_id=eos_token_id,
                           seed=seed)
    p = prompt_ids.tolist()
    outs = eng.generate_tokens([p] * group_size, gen)
    model.train(was)
    L = len(p) + max(len(o) for o in outs)
    ids = torch.zeros(group_size, L, dtype=torch.long)
    for i, o in enumerate(outs):
        ids[i, :len(p) + len(o)] = torch.tensor(p + list(o))
    return ids


def generate_group_vllm(backend, prompt: str, group_size: int, max_new_tokens: int,
                        temperature: float = 1.0, top_p: float = 0.9) -> List[str]:
    """Group sampling through an OpenAI-compatible server (vLLM / SGLang /
    this framework's server) given as ``inference.external.OpenAICompatibleBackend``."""
    from ..inference.external import ExternalGenerationConfig

    cfg = ExternalGenerationConfig(max_tokens=max_new_tokens, temperature=temperature, top_p=top_p)
    return [backend.complete(prompt, cfg) for _ in range(group_size)]


def _completion_logp(model, input_ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
    prompts = [input_ids[i, :prompt_len].tolist() for i in range(input_ids.shape[0])]
    comps = []
    for i in range(input_ids.shape[0]):
        c = input_ids[i, prompt_len:].tolist()
        while c and c[-1] == 0:      # right padding
            c.pop()
        comps.append(c)
    lp, mask = sequence_log_probs(model, prompts, comps)
    return (lp * mask).sum(-1)


@torch.no_grad()
def compute_log_probs(model, input_ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
    """Summed log p(completion | prompt) per row (no gradient)."""
    was = model.training
    model.eval()
    out = _completion_logp(model, input_ids, prompt_len)
    model.train(was)
    return out


def compute_log_probs_trainable(model, input_ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
    model.train()
    return _completion_logp(model, input_ids, prompt_len)


def mmlu_reward(completions: Sequence[str], answer: str) -> List[float]:
    """Reward of the MMLU task: 1 when the first option letter in a completion is the answer, else 0."""
    out = []
    for c in completions:
        letter = next((ch for ch in c.strip().upper() if ch in CHOICES), None)
        out.append(1.0 if letter == answer else 0.0)
    return out


def train_grpo(model, tokenizer, examples: Sequence[Dict], *, steps: int,
               batch_prompts: int = 4, config: Optional[GRPOConfig] = None, reward_fn=None,
               output: Optional[str] = None) -> List[Dict]:
    """``steps`` GRPO updates over ``examples`` (cycled, ``batch_prompts`` per
    step); returns the per-step statistics and saves the policy to ``output``."""
    cfg = config or GRPOConfig()
    rf = reward_fn or mmlu_reward
    tr = GRPOTrainer(model, tokenizer, cfg, reward_fn=rf)
    hist = []
    for s in range(steps):
        batch = [examples[(s * batch_prompts + i) % len(examples)] for i in range(batch_prompts)]
        answers = [b["answer"] for b in batch] if any(b["answer"] for b in batch) else None
        st = tr.step([b["prompt"] for b in batch], answers)
        st["step"] = s + 1
        hist.append(st)
    if output:
        Path(output).mkdir(parents=True, exist_ok=True)
        model.save_pretrained(Path(output) / "final")
        (Path(output) / "history.json").write_text(json.dumps(hist, indent=2, default=float))
    return hist


def main(argv=None) -> List[Dict]:
    from ..data.tokenization import get_tokenizer
    from ..models.builder import ComplexityModel

    ap = argparse.ArgumentParser(description="GRPO / DAPO on MMLU or FineWeb-Edu prompts")
    ap.add_argument("--model", required=True)
    ap.add_argument("--data", required=True, help="local JSONL")
    ap.add_argument("--task", choices=("mmlu", "fineweb"), default="mmlu")
    ap.add_argument("--tokenizer", default="byte")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch-prompts", type=int, default=4)
    ap.add_argument("--group-size", type=int, default=8)
    ap.add_argument("--max-new-tokens", type=int, default=32)
    ap.add_argument("--lr", type=float, default=1e-5)
    ap.add_argument("--kl-coef", type=float, default=0.0)
    ap.add_argument("--max-samples", type=int, default=0)
    ap.add_argument("--output", default="grpo_out")
    a = ap.parse_args(argv)
    tok = get_tokenizer(a.tokenizer) if a.tokenizer == "byte" else get_tokenizer(
        "huggingface", a.tokenizer)
    model = ComplexityModel.from_pretrained(a.model)
    if torch.cuda.is_available():
        model = model.cuda().to(torch.bfloat16)
    data = (load_mmlu_dataset(a.data, max_samples=a.max_samples) if a.task == "mmlu"
            else load_fineweb_edu_dataset(a.data, max_samples=a.max_samples or 10000))
    reward = mmlu_reward
    if a.task == "fineweb":
        from .rewards import language_quality_reward

        reward = language_quality_reward
    cfg = GRPOConfig(group_size=a.group_size, max_new_tokens=a.max_new_tokens, lr=a.lr,
                     kl_coef=a.kl_coef)
    return train_grpo(model, tok, data, steps=a.steps, batch_prompts=a.batch_prompts, config=cfg,
                      reward_fn=reward, output=a.output)


if __name__ == "__main__":
    main()
