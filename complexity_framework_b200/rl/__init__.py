"""Reinforcement learning: GRPO / DAPO with group sampling on the paged-KV engine."""
from .grpo import (GRPOConfig, GRPOTrainer, dapo_loss, group_advantages, sequence_log_probs)
from .rewards import (combined_reward, extract_answer, format_reward, language_quality_reward,
                      mcq_exact_match_reward)
