"""GRPO / DAPO training.

Counterpart of complexity/RL/grpo/train_grpo.py:178-640: for every prompt a
group of G completions is sampled (here through the paged-KV continuous
batching engine, all groups in one batch), rewards are normalised within the
group into advantages, and the policy is updated with the DAPO objective:
token-level mean over all completion tokens of
min(r * A, clip(r, 1 - eps_low, 1 + eps_high) * A) with r the probability
ratio to the sampling policy, plus an optional KL penalty to a frozen
reference model.  Groups whose rewards are all equal carry no signal and are
dropped (dynamic sampling).
"""
from __future__ import annotations

import copy
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.nn.functional as F


@dataclass
class GRPOConfig:
    group_size: int = 8
    max_new_tokens: int = 64
    temperature: float = 1.0
    top_p: float = 1.0
    lr: float = 1e-5
    eps_low: float = 0.2
    eps_high: float = 0.28
    kl_coef: float = 0.0
    updates_per_batch: int = 1
    max_grad_norm: float = 1.0
    drop_uniform_groups: bool = True
    seed: int = 0


def group_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-6) -> torch.Tensor:
    """(r - mean_group) / (std_group + eps) for rewards laid out group after group."""
    r = rewards.view(-1, group_size)
    return ((r - r.mean(1, keepdim=True)) / (r.std(1, keepdim=True) + eps)).view(-1)


def sequence_log_probs(model, prompt_ids: Sequence[Sequence[int]],
                       completion_ids: Sequence[Sequence[int]], pad_id: int = 0):
    """Per-token log p(completion | prompt) as a padded [N, Lc] tensor + mask."""
    dev = next(model.parameters()).device
    seqs = [list(p) + list(c) for p, c in zip(prompt_ids, completion_ids)]
    L = max(len(s) for s in seqs)
    Lc = max(1, max(len(c) for c in completion_ids))
    ids = torch.full((len(seqs), L), pad_id, dtype=torch.long)
    for i, s in enumerate(seqs):
        ids[i, :len(s)] = torch.tensor(s)
    ids = ids.to(dev)
    logits = model(ids)["logits"].float()
    lp = torch.log_softmax(logits, -1)
    out = torch.zeros(len(seqs), Lc, device=dev)
    mask = torch.zeros(len(seqs), Lc, device=dev)
    for i, (p, c) in enumerate(zip(prompt_ids, completion_ids)):
        if not c:
            continue
        pos = torch.arange(len(p) - 1, len(p) - 1 + len(c), device=dev)
        tgt = torch.tensor(list(c), device=dev)
        out[i, :len(c)] = lp[i, pos, tgt]
        mask[i, :len(c)] = 1.0
    return out, mask


def dapo_loss(logp: torch.Tensor, old_logp: torch.Tensor, adv: torch.Tensor, mask: torch.Tensor,
              eps_low: float, eps_high: float, ref_logp: Optional[torch.Tensor] = None,
              kl_coef: float = 0.0) -> torch.Tensor:
    ratio = torch.exp(logp - old_logp)
    a = adv[:, None]
    obj = torch.minimum(ratio * a, ratio.clamp(1 - eps_low, 1 + eps_high) * a)
    loss = -obj
    if ref_logp is not None and kl_coef > 0:
        # k3 estimator of KL(policy || reference), non-negative
        d = ref_logp - logp
        loss = loss + kl_coef * (torch.exp(d) - d - 1)
    return (loss * mask).sum() / mask.sum().clamp_min(1)


class GRPOTrainer:
    def __init__(self, model, tokenizer, config: Optional[GRPOConfig] = None,
                 reward_fn: Optional[Callable] = None):
        self.model = model
        self.tok = tokenizer
        self.cfg = config or GRPOConfig()
        self.reward_fn = reward_fn
        self.opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad],
                                     lr=self.cfg.lr, betas=(0.9, 0.95), weight_decay=0.0)
        self.ref = None
        if self.cfg.kl_coef > 0:
            self.ref = copy.deepcopy(model).eval()
            for p in self.ref.parameters():
                p.requires_grad_(False)
        self.step_count = 0

    def sample(self, prompts: Sequence[str]):
        from ..inference.engine import GenerationConfig, InferenceEngine

        G = self.cfg.group_size
        was_training = self.model.training
        eng = InferenceEngine(self.model)
        gen = GenerationConfig(max_new_tokens=self.cfg.max_new_tokens, do_sample=True,
                               temperature=self.cfg.temperature, top_p=self.cfg.top_p,
                               eos_token_id=self.tok.eos_token_id,
                               seed=self.cfg.seed + self.step_count * 7919)
        prompt_ids = [self.tok.encode(p) for p in prompts for _ in range(G)]
        completions = eng.generate_tokens(prompt_ids, gen)
        self.model.train(was_training)
        return prompt_ids, completions

    def step(self, prompts: Sequence[str], answers: Optional[Sequence[str]] = None) -> Dict:
        cfg = self.cfg
        G = cfg.group_size
        prompt_ids, comp_ids = self.sample(prompts)
        texts = [self.tok.decode(c) for c in comp_ids]
        rewards = []
        for i, p in enumerate(prompts):
            group = texts[i * G:(i + 1) * G]
            if answers is not None:
                rewards.extend(self.reward_fn(group, answers[i]))
            else:
                rewards.extend(self.reward_fn([p] * G, group))
        r = torch.tensor(rewards, dtype=torch.float32)
        adv = group_advantages(r, G)
        keep = torch.ones(len(prompts), dtype=torch.bool)
        if cfg.drop_uniform_groups:
            keep = r.view(-1, G).std(1) > 1e-6
        idx = [i for i in range(len(prompt_ids)) if keep[i // G]]
        stats = {"reward_mean": float(r.mean()), "groups_kept": int(keep.sum()),
                 "completion_len": sum(len(c) for c in comp_ids) / max(1, len(comp_ids))}
        if not idx:
            self.step_count += 1
            stats["loss"] = 0.0
            return stats
        p_ids = [prompt_ids[i] for i in idx]
        c_ids = [comp_ids[i] for i in idx]
        a = adv[idx].to(next(self.model.parameters()).device)
        with torch.no_grad():
            old, mask = sequence_log_probs(self.model, p_ids, c_ids)
            ref_lp = sequence_log_probs(self.ref, p_ids, c_ids)[0] if self.ref is not None else None
        self.model.train()
        for _ in range(cfg.updates_per_batch):
            logp, mask = sequence_log_probs(self.model, p_ids, c_ids)
            loss = dapo_loss(logp, old, a, mask, cfg.eps_low, cfg.eps_high, ref_lp, cfg.kl_coef)
            self.opt.zero_grad()
            loss.backward()
            torch.nn.utils.clip_grad_norm_(self.model.parameters(), cfg.max_grad_norm)
            self.opt.step()
        self.step_count += 1
        stats["loss"] = float(loss.detach())
        return stats
