"""torchrun launch of a training run on one node (or one node of several).

``cfb launch --gpus 8 -- --model tr-hash-200m --token-mixture DIR ...`` runs
``python -m torch.distributed.run --nnodes N --nproc-per-node G
--master-addr A --master-port P -m complexity_framework_b200.training.runner
<runner flags>``; ``--supervise`` wraps it in the restart supervisor.
Counterpart of the reference's launch_*.sh wrappers.
"""
from __future__ import annotations

import os
import subprocess
import sys
from typing import List, Optional, Sequence


def build_torchrun_command(runner_args: Sequence[str], gpus: int = 1, nodes: int = 1,
                           node_rank: int = 0, master_addr: str = "127.0.0.1",
                           master_port: int = 29500,
                           module: str = "complexity_framework_b200.training.runner"
                           ) -> List[str]:
    if gpus < 1 or nodes < 1 or not 0 <= node_rank < nodes:
        raise ValueError("gpus and nodes must be positive and node_rank in [0, nodes)")
    return [sys.executable, "-m", "torch.distributed.run", f"--nnodes={nodes}",
            f"--node-rank={node_rank}", f"--nproc-per-node={gpus}",
            f"--master-addr={master_addr}", f"--master-port={master_port}",
            "-m", module, *runner_args]


def launch(runner_args: Sequence[str], gpus: int = 1, nodes: int = 1, node_rank: int = 0,
           master_addr: str = "127.0.0.1", master_port: int = 29500, dry_run: bool = False,
           supervise: bool = False, progress_file: Optional[str] = None,
           stall_seconds: float = 900.0, max_restarts: int = 3) -> int:
    cmd = build_torchrun_command(runner_args, gpus, nodes, node_rank, master_addr, master_port)
    if dry_run:
        print(" ".join(cmd))
        return 0
    if supervise:
        from .supervisor import RunSupervisor, SupervisorConfig

        return RunSupervisor(SupervisorConfig(cmd, progress_file=progress_file,
                                              stall_seconds=stall_seconds,
                                              max_restarts=max_restarts)).run()
    return subprocess.call(cmd, env=dict(os.environ))
