"""Reward functions for GRPO.

Counterpart of complexity/RL/grpo/rewards.py:13-260: multiple-choice answer
extraction and exact match, a format reward, and a language-quality reward
(repetition, length window, coherence heuristics) for open continuation.
"""
from __future__ import annotations

import re
from typing import List, Optional

_ANSWER_PATTERNS = [
    r"answer\s*(?:is|:)\s*\(?([A-D])\)?",
    r"^\s*\(?([A-D])\)?[\s\.\):]",
    r"\b([A-D])\b",
]


def extract_answer(text: str) -> Optional[str]:
    """First A-D choice found by increasingly loose patterns."""
    for pat in _ANSWER_PATTERNS:
        m = re.search(pat, text, flags=re.IGNORECASE | re.MULTILINE)
        if m:
            return m.group(1).upper()
    return None


def mcq_exact_match_reward(completions: List[str], answer: str) -> List[float]:
    return [1.0 if extract_answer(c) == answer.upper() else 0.0 for c in completions]


def format_reward(completions: List[str]) -> List[float]:
    """0.2 when a single clear choice letter leads the completion."""
    return [0.2 if re.match(r"^\s*\(?[A-D]\)?([\s\.\):]|$)", c) else 0.0 for c in completions]


def combined_reward(completions: List[str], answer: str, format_weight: float = 1.0) -> List[float]:
    return [a + format_weight * b for a, b in zip(mcq_exact_match_reward(completions, answer),
                                                   format_reward(completions))]


def _repetition_score(text: str) -> float:
    words = text.split()
    if len(words) < 4:
        return 0.0
    trigrams = [tuple(words[i:i + 3]) for i in range(len(words) - 2)]
    return len(set(trigrams)) / len(trigrams)


def _length_score(text: str, target_min: int = 20, target_max: int = 200) -> float:
    n = len(text.split())
    if n < target_min:
        return n / target_min
    if n > target_max:
        return max(0.0, 1.0 - (n - target_max) / target_max)
    return 1.0


def _coherence_score(text: str) -> float:
    sentences = [s for s in re.split(r"[.!?]+", text) if s.strip()]
    if not sentences:
        return 0.0
    avg = sum(len(s.split()) for s in sentences) / len(sentences)
    return 1.0 if 5 <= avg <= 35 else 0.5


def language_quality_reward(prompts: List[str], completions: List[str]) -> List[float]:
    return [(_repetition_score(c) + _length_score(c) + _coherence_score(c)) / 3.0
            for _, c in zip(prompts, completions)]
