"""Run launching and supervision: torchrun launch of a training run, a
supervisor that restarts a stalled or crashed run from its last checkpoint,
replay-plan building and token-data verification.

Counterparts of the reference's operational scripts
(scripts/watch_and_restart_stalled_process.py, the launch_*.sh and
vast_*_supervisor wrappers, build_corrective_replay_plan.py,
verify_token_shards.py).
"""
from .launcher import build_torchrun_command, launch
from .replay import build_replay_plan, verify_token_data
from .supervisor import (RunSupervisor, SupervisorConfig, restart_program, seconds_since_last_write,
                         watch_once, watch_supervisord)

__all__ = ["build_torchrun_command", "launch", "build_replay_plan", "verify_token_data",
           "RunSupervisor", "SupervisorConfig", "seconds_since_last_write", "restart_program",
           "watch_once", "watch_supervisord"]
