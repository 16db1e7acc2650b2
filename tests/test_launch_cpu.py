"""Run supervision (crash and stall restarts with resume), torchrun command
building, replay plans and token-data verification, on CPU."""
import json
import sys

import numpy as np
import pytest

from complexity_framework_b200.data.corpus_mixture import (PretokenizedCorpusMixtureDataset,
                                                           write_token_mixture)
from complexity_framework_b200.launch import (RunSupervisor, SupervisorConfig,
                                              build_replay_plan, build_torchrun_command,
                                              verify_token_data)


def _script(tmp_path, body):
    p = tmp_path / "job.py"
    p.write_text(body)
    return [sys.executable, str(p)]


def test_supervisor_restarts_crash_with_resume(tmp_path):
    # fails until it is started with --resume, then succeeds
    cmd = _script(tmp_path, "import sys\nsys.exit(0 if '--resume' in sys.argv else 3)\n")
    cfg = SupervisorConfig(cmd, poll_seconds=0.05, max_restarts=2)
    assert RunSupervisor(cfg).run() == 0
    kinds = [e["event"] for e in cfg.events]
    assert kinds == ["start", "restart", "start", "finished"]
    assert cfg.events[1]["reason"] == "exit 3" and cfg.events[2]["resume"]


def test_supervisor_restarts_stalled_run(tmp_path):
    prog = tmp_path / "progress.log"
    # first attempt writes once then hangs without exiting; the resumed one finishes
    cmd = _script(tmp_path, f"""
import sys, time, pathlib
p = pathlib.Path({str(prog)!r})
p.write_text("step 1")
if '--resume' in sys.argv:
    sys.exit(0)
time.sleep(60)
""")
    cfg = SupervisorConfig(cmd, progress_file=str(prog), stall_seconds=0.5,
                           startup_grace_seconds=5, poll_seconds=0.1, max_restarts=1,
                           term_grace_seconds=2)
    assert RunSupervisor(cfg).run() == 0
    assert [e["event"] for e in cfg.events].count("restart") == 1
    assert cfg.events[1]["reason"] == "stalled"


def test_supervisor_gives_up(tmp_path):
    cmd = _script(tmp_path, "import sys\nsys.exit(5)\n")
    cfg = SupervisorConfig(cmd, poll_seconds=0.05, max_restarts=1)
    assert RunSupervisor(cfg).run() == 5
    assert cfg.events[-1]["event"] == "giving_up"


def test_torchrun_command():
    cmd = build_torchrun_command(["--model", "tiny"], gpus=8)
    assert "--nproc-per-node=8" in cmd and "--master-addr=127.0.0.1" in cmd
    assert cmd[-2:] == ["--model", "tiny"]
    with pytest.raises(ValueError):
        build_torchrun_command([], gpus=0)


def test_replay_plan_and_verify(tmp_path):
    rng = np.random.default_rng(0)
    write_token_mixture(tmp_path, {"web": (0.5, rng.integers(0, 500, 8 * 64 + 1)),
                                   "code": (0.5, rng.integers(0, 500, 8 * 32 + 1))}, 8, 16)
    plan = build_replay_plan(tmp_path, [{"name": "a", "passes": 2,
                                         "fractions": {"web": 0.5, "code": 1.0}}],
                             row_alignment=8)
    ds = PretokenizedCorpusMixtureDataset(tmp_path, replay_plan=plan)
    assert ds.trained_tokens == plan["trained_tokens"] == (32 + 32) * 2 * 8
    assert len(list(ds)) == 128
    assert verify_token_data(tmp_path)["ok"]
    shard = tmp_path / "corpora" / "web" / "shard-00000.bin"
    b = bytearray(shard.read_bytes())
    b[0] ^= 1
    shard.write_bytes(bytes(b))
    r = verify_token_data(tmp_path)
    assert not r["ok"] and r["bad"][0]["problem"] == "sha256"
