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


def test_supervisord_watchdog(tmp_path):
    import os
    from types import SimpleNamespace

    from complexity_framework_b200.launch import (restart_program, seconds_since_last_write,
                                                  watch_once, watch_supervisord)

    log = tmp_path / "train.log"
    assert seconds_since_last_write(log) is None
    calls = []
    assert not watch_once(log, "train", 60, restart=calls.append)       # not written yet
    log.write_text("step 1\n")
    os.utime(log, (1000.0, 1000.0))
    assert seconds_since_last_write(log, now=1030.0) == 30.0
    assert not watch_once(log, "train", 60, now=1030.0, restart=calls.append)
    assert watch_once(log, "train", 60, now=1100.0, restart=calls.append) and calls == ["train"]

    ran = []
    ok = restart_program("train", runner=lambda cmd, **kw: ran.append(cmd) or
                         SimpleNamespace(returncode=0, stdout="", stderr=""))
    assert ok and ran == [["supervisorctl", "restart", "train"]]
    assert not restart_program("train", runner=lambda cmd, **kw:
                               SimpleNamespace(returncode=1, stdout="", stderr="no such"))

    # stale the whole time: restarts respect the cooldown (every 3rd poll here)
    t = iter(range(2000, 2000 + 60 * 10, 60))
    restarted = []
    n = watch_supervisord(log, "train", stall_seconds=100, poll_seconds=60,
                          cooldown_seconds=150, max_checks=9, sleep=lambda s: None,
                          clock=lambda: float(next(t)), restart=restarted.append)
    assert n == 3 and restarted == ["train"] * 3


def test_collect_run_artifacts(tmp_path):
    import hashlib
    import json

    import pytest
    import torch
    from safetensors.torch import load_file

    from complexity_framework_b200.launch.artifacts import collect_run_artifacts

    ck = tmp_path / "ck" / "step_000010"
    ck.mkdir(parents=True)
    tied = torch.randn(8, 4)
    torch.save({"step": 10, "model": {"embed.weight": tied, "lm_head.weight": tied},
                "config": {"hidden_size": 4}, "optimizer": {"huge": 1}}, ck / "checkpoint.pt")
    run = tmp_path / "run"
    run.mkdir()
    (run / "metrics.csv").write_text("step,loss\n10,2.0\n")
    (run / "train.log").write_text("ok\n")
    (run / "notes.bin").write_bytes(b"skip")
    data = tmp_path / "data" / "train"
    data.mkdir(parents=True)
    (data / "tokens.idx.json").write_text("{}")
    (data / "tokens.bin").write_bytes(b"\0" * 64)
    tok = tmp_path / "tok"
    tok.mkdir()
    (tok / "tokenizer.json").write_text("{}")
    out = tmp_path / "out"
    man = collect_run_artifacts("r", str(ck), str(run), str(out), str(tmp_path / "data"), str(tok))
    w = load_file(str(out / "model.safetensors"))
    assert torch.equal(w["embed.weight"], tied) and torch.equal(w["lm_head.weight"], tied)
    cfg = json.loads((out / "model_config.json").read_text())
    assert cfg["checkpoint_step"] == 10 and cfg["model"]["hidden_size"] == 4
    assert man["checkpoint"]["sha256"] == hashlib.sha256((ck / "checkpoint.pt").read_bytes()
                                                         ).hexdigest()
    paths = {f["path"] for f in man["files"]}
    assert {"model.safetensors", "metrics.csv", "train.log", "dataset/train/tokens.idx.json",
            "tokenizer/tokenizer.json"} <= paths
    assert "notes.bin" not in paths and "dataset/train/tokens.bin" not in paths
    with pytest.raises(FileExistsError):
        collect_run_artifacts("r", str(ck), str(run), str(out))
