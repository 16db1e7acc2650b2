"""Shared online RL while serving: monitor, batch one update, one checkpoint.

Counterpart: complexity/inference/shared_online_rl.py:34-430
(``SharedRLEvent``, ``SharedOnlineRLConfig``, ``SharedOnlineRLLoop``).
Requests keep being served; a response whose user feedback is non-empty, whose
mean next-token entropy is high or whose mean chosen-token probability is low
becomes a compact event (appended to a JSONL monitor log).  When enough
events are pending, ONE policy-gradient update runs over all of them and ONE
checkpoint is written (with a pointer file naming the current one), instead
of a checkpoint per request.

Differences of construction: the update scores every event in one padded
forward (``grpo.sequence_log_probs``) instead of one forward per event;
questions a deterministic tool can answer get a verified target transcript
and reward 1 automatically (``tool_rewards.build_verified_tool_episode``),
trained as supervised positives with weight ``verified_target_weight``; other
events use REINFORCE with an exponential-moving-average reward baseline.
"""
from __future__ import annotations

import json
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from .grpo import sequence_log_probs
from .tool_rewards import build_verified_tool_episode

NEGATIVE_WORDS = ("wrong", "false", "bad", "non", "faux", "incorrect")
POSITIVE_WORDS = ("correct", "good", "yes", "oui", "exact")


@dataclass
class SharedRLEvent:
    prompt: str
    response: str
    target_response: Optional[str] = None
    feedback: Optional[str] = None
    reward: Optional[float] = None
    mean_entropy: Optional[float] = None
    mean_confidence: Optional[float] = None
    tool_calls: List[Dict[str, Any]] = field(default_factory=list)
    tool_results: List[Dict[str, Any]] = field(default_factory=list)
    created_at_unix: float = field(default_factory=time.time)
    metadata: Dict[str, Any] = field(default_factory=dict)


@dataclass
class SharedOnlineRLConfig:
    output_dir: str = "checkpoints/online_rl"
    min_events_before_update: int = 16
    max_pending_events: int = 128
    max_new_tokens: int = 128
    temperature: float = 0.8
    top_k: int = 50
    entropy_trigger: float = 5.0
    confidence_trigger: float = 0.20
    positive_reward: float = 1.0
    negative_reward: float = -1.0
    uncertainty_reward: float = -0.2
    baseline_beta: float = 0.95
    learning_rate: float = 1e-7
    rl_epochs: int = 1
    max_grad_norm: float = 1.0
    checkpoint_prefix: str = "checkpoint_online_rl"
    monitor_log_name: str = "shared_rl_events.jsonl"
    current_pointer_name: str = "current_online_rl_checkpoint.txt"
    save_optimizer: bool = True
    reload_after_save: bool = False
    prefer_target_response: bool = True
    verified_target_weight: float = 1.0
    keep_last_n_checkpoints: int = 5   # 0 keeps all
    verify_tools: bool = True


class SharedOnlineRLLoop:
    def __init__(self, model: torch.nn.Module, tokenizer, optimizer=None,
                 config: Optional[SharedOnlineRLConfig] = None, device=None,
                 extra_state_fn: Optional[Callable[[], Dict[str, Any]]] = None,
                 reload_fn: Optional[Callable[[Path], None]] = None):
        self.model, self.tokenizer = model, tokenizer
        self.config = c = config or SharedOnlineRLConfig()
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.optimizer = optimizer or torch.optim.AdamW(model.parameters(), lr=c.learning_rate)
        self.extra_state_fn, self.reload_fn = extra_state_fn, reload_fn
        self.output_dir = Path(c.output_dir)
        self.output_dir.mkdir(parents=True, exist_ok=True)
        self.monitor_log = self.output_dir / c.monitor_log_name
        self.pending_events: List[SharedRLEvent] = []
        self.baseline = 0.0
        existing = self._checkpoints()
        self.rl_step = (int(existing[-1].name.rsplit("_", 1)[-1]) + 1) if existing else 1

    # ------------------------------------------------------------- serving
    @torch.no_grad()
    def generate_with_stats(self, prompt: str, **over) -> Tuple[str, float, float]:
        """Sampled response, mean next-token entropy, mean chosen-token probability."""
        c = self.config
        n_new = int(over.get("max_new_tokens", c.max_new_tokens))
        temp = float(over.get("temperature", c.temperature))
        top_k = int(over.get("top_k", c.top_k))
        was = self.model.training
        self.model.eval()
        ids = torch.tensor([self.tokenizer.encode(prompt)], device=self.device)
        out, ent, conf = [], [], []
        eos = getattr(self.tokenizer, "eos_token_id", None)
        for _ in range(n_new):
            logits = self.model(ids)["logits"][0, -1].float()
            p = torch.softmax(logits, -1)
            ent.append(float(-(p * torch.log(p.clamp_min(1e-12))).sum()))
            scaled = logits / max(temp, 1e-5)
            if 0 < top_k < scaled.numel():
                kth = scaled.topk(top_k).values[-1]
                scaled = scaled.masked_fill(scaled < kth, float("-inf"))
            tok = int(torch.multinomial(torch.softmax(scaled, -1), 1)) if temp > 0 \
                else int(scaled.argmax())
            conf.append(float(p[tok]))
            if eos is not None and tok == eos:
                break
            out.append(tok)
            ids = torch.cat((ids, torch.tensor([[tok]], device=self.device)), 1)
        self.model.train(was)
        n = max(1, len(ent))
        return self.tokenizer.decode(out), sum(ent) / n, sum(conf) / n

    def compute_reward(self, feedback: Optional[str], entropy: Optional[float],
                       confidence: Optional[float]) -> float:
        c = self.config
        if feedback:
            t = feedback.lower()
            if any(w in t for w in NEGATIVE_WORDS):   # before the positives: "incorrect"
                return c.negative_reward
            if any(w in t for w in POSITIVE_WORDS):
                return c.positive_reward
        if (entropy is not None and entropy >= c.entropy_trigger) or \
                (confidence is not None and confidence <= c.confidence_trigger):
            return c.uncertainty_reward
        return 0.0

    def should_monitor(self, e: SharedRLEvent) -> bool:
        c = self.config
        return bool((e.feedback and e.feedback.strip())
                    or (e.mean_entropy is not None and e.mean_entropy >= c.entropy_trigger)
                    or (e.mean_confidence is not None and e.mean_confidence <= c.confidence_trigger)
                    or e.target_response is not None)

    def infer(self, prompt: str, user_feedback: Optional[str] = None,
              target_response: Optional[str] = None, reward: Optional[float] = None,
              tool_calls=None, tool_results=None, metadata=None, force_monitor: bool = False,
              force_update: bool = False, question: Optional[str] = None, **gen):
        """Serve one request; returns (response, update stats or None, checkpoint or None)."""
        response, ent, conf = self.generate_with_stats(prompt, **gen)
        meta = dict(metadata or {})
        if self.config.verify_tools and target_response is None:
            ep = build_verified_tool_episode(prompt, question if question is not None else prompt)
            if ep is not None:
                target_response, reward = ep.target_response, ep.reward
                tool_calls, tool_results = [ep.tool_call], [ep.tool_result]
                meta.update(ep.metadata)
        ev = SharedRLEvent(prompt, response, target_response, user_feedback,
                           reward if reward is not None else
                           self.compute_reward(user_feedback, ent, conf),
                           ent, conf, list(tool_calls or []), list(tool_results or []),
                           metadata=meta)
        if force_monitor or self.should_monitor(ev):
            self._append(ev)
        stats = ckpt = None
        if force_update or len(self.pending_events) >= self.config.min_events_before_update:
            stats = self.update()
            ckpt = self.save_checkpoint(stats)
            self.pending_events.clear()
            if self.config.reload_after_save:
                if self.reload_fn is None:
                    raise RuntimeError("reload_after_save=True requires a reload_fn")
                self.reload_fn(ckpt)
        return response, stats, ckpt

    # -------------------------------------------------------------- update
    def _verified(self, e: SharedRLEvent) -> bool:
        return bool(self.config.prefer_target_response and e.target_response is not None
                    and e.reward is not None and e.reward > 0)

    def update(self) -> Dict[str, float]:
        c = self.config
        events = self.pending_events[-c.max_pending_events:]
        if not events:
            return {"num_events": 0.0, "loss": 0.0}
        enc = self.tokenizer.encode
        prompts = [enc(e.prompt) for e in events]
        comps = [enc(e.target_response if self._verified(e) else e.response) for e in events]
        rewards = [float(e.reward or 0.0) for e in events]
        self.model.train()
        loss = gn = torch.zeros(())
        for _ in range(max(1, int(c.rl_epochs))):
            coefs = []
            for e, r in zip(events, rewards):
                if self._verified(e):
                    coefs.append(c.verified_target_weight * r)
                else:
                    self.baseline = c.baseline_beta * self.baseline + (1 - c.baseline_beta) * r
                    coefs.append(r - self.baseline)
            lp, mask = sequence_log_probs(self.model, prompts, comps)
            mean_lp = (lp * mask).sum(1) / mask.sum(1).clamp_min(1.0)
            loss = -(torch.tensor(coefs, device=mean_lp.device) * mean_lp).mean()
            self.optimizer.zero_grad(set_to_none=True)
            loss.backward()
            gn = torch.nn.utils.clip_grad_norm_(self.model.parameters(), c.max_grad_norm)
            self.optimizer.step()
        self.model.eval()
        return {"num_events": float(len(events)), "rl_epochs": float(max(1, int(c.rl_epochs))),
                "mean_reward": sum(rewards) / len(rewards), "baseline": float(self.baseline),
                "loss": float(loss.detach()), "grad_norm": float(gn)}

    # --------------------------------------------------------- persistence
    def _append(self, e: SharedRLEvent) -> None:
        self.pending_events.append(e)
        del self.pending_events[:-self.config.max_pending_events]
        with self.monitor_log.open("a", encoding="utf-8") as f:
            f.write(json.dumps(asdict(e), ensure_ascii=False, sort_keys=True) + "\n")

    def _checkpoints(self) -> List[Path]:
        pre = self.config.checkpoint_prefix + "_"
        found = [p for p in self.output_dir.glob(pre + "*")
                 if p.is_dir() and p.name[len(pre):].isdigit()]
        return sorted(found, key=lambda p: int(p.name[len(pre):]))

    def save_checkpoint(self, stats: Dict[str, float]) -> Path:
        c = self.config
        path = self.output_dir / f"{c.checkpoint_prefix}_{self.rl_step:06d}"
        path.mkdir(parents=True, exist_ok=True)
        torch.save(self.model.state_dict(), path / "model.pt")
        if c.save_optimizer:
            torch.save(self.optimizer.state_dict(), path / "optimizer.pt")
        state = {"rl_step": self.rl_step, "baseline": self.baseline, "stats": stats}
        if self.extra_state_fn is not None:
            state["extra"] = self.extra_state_fn()
        (path / "online_rl_state.json").write_text(json.dumps(state, indent=1))
        (self.output_dir / c.current_pointer_name).write_text(str(path))
        self.rl_step += 1
        if c.keep_last_n_checkpoints > 0:
            for old in self._checkpoints()[:-c.keep_last_n_checkpoints]:
                for f in old.iterdir():
                    f.unlink()
                old.rmdir()
        return path
