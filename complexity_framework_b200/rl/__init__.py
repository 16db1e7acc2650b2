"""Reinforcement learning: GRPO / DAPO with group sampling on the paged-KV engine."""
from .grpo import (GRPOConfig, GRPOTrainer, dapo_loss, group_advantages, sequence_log_probs)
from .rewards import (combined_reward, extract_answer, format_reward, language_quality_reward,
                      mcq_exact_match_reward)
from .online import SharedOnlineRLConfig, SharedOnlineRLLoop, SharedRLEvent
from .tool_rewards import (VerifiedToolEpisode, build_verified_tool_episode, parse_tool_call,
                           batch_tool_rewards, safe_calculator, safe_datetime, tool_call_reward)
