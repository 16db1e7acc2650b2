"""Failure handling on the host, without any GPU fault.

* A rank that raises inside ``safe_main`` aborts the process group, so a peer
  blocked in a collective gets an error quickly instead of hanging until the
  process-group timeout (gloo ranks on CPU).
* SIGTERM during a ``TrainRunner`` run leaves an ``interrupted-<step>``
  checkpoint that resumes.
* A crash in the middle of writing a checkpoint leaves the previous checkpoint
  as the newest complete one, and it loads.

Counterparts: complexity/gpu/distributed_cleanup.py:23-68 (safe_main,
cleanup_distributed(abort=True)) and the crash-mid-save regression of
tests/test_fsdp.py:210-245 in the reference.
"""
import datetime
import json
import os
import signal
import socket
import subprocess
import sys
import textwrap
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _safe_main_rank(rank, world, port, out_dir):
    from complexity_framework_b200.parallel.distributed import safe_main

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    # a long process-group timeout: only the abort can end the peer's wait early
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    dist.barrier()

    @safe_main
    def body():
        if rank == 1:
            raise RuntimeError("rank 1 failed between steps")
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(4))
            outcome = "completed"
        except Exception as exc:  # the aborted peer surfaces as an error
            outcome = f"raised {type(exc).__name__}"
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
            json.dump({"outcome": outcome, "seconds": time.monotonic() - t0}, fh)

    try:
        body()
    except RuntimeError:
        os._exit(3)  # the failing rank exits non-zero after safe_main's abort


def test_safe_main_peer_failure_aborts_instead_of_hanging(tmp_path):
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_safe_main_rank, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung after its peer failed")
    assert procs[1].exitcode == 3
    rec = json.loads((tmp_path / "rank0.json").read_text())
    assert rec["outcome"].startswith("raised"), rec
    assert rec["seconds"] < 60, rec                     # well before the 120 s timeout


_RUNNER_SCRIPT = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    from complexity_framework_b200 import ModelConfig
    from complexity_framework_b200.training.runner import TrainRunner
    cfg = dict(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
               num_key_value_heads=2, vocab_size=256, intermediate_size=64,
               shared_intermediate_size=128, num_experts=4, top_k=2,
               routing_strategy="modulo_cyclic", max_position_embeddings=64)
    TrainRunner(make_config=lambda a: ModelConfig(**cfg)).main(sys.argv[1:])
""")


def test_sigterm_writes_interrupted_checkpoint_that_resumes(tmp_path):
    ck = tmp_path / "ck"
    script = tmp_path / "run.py"
    script.write_text(_RUNNER_SCRIPT.format(root=ROOT))
    args = ["--synthetic", "--max-steps", "100000", "--batch-size", "2", "--seq-len", "16",
            "--checkpoint-dir", str(ck), "--log-steps", "1", "--save-steps", "100000",
            "--precision", "fp32", "--no-progress"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    proc = subprocess.Popen([sys.executable, str(script)] + args, env=env,
                            stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
    log = ck / "logs" / "training_log.csv"
    deadline = time.monotonic() + 120
    while time.monotonic() < deadline:            # wait until a few steps have run
        if log.exists() and len(log.read_text().splitlines()) > 3:
            break
        time.sleep(0.2)
    proc.send_signal(signal.SIGTERM)
    try:
        proc.wait(60)
    except subprocess.TimeoutExpired:
        proc.kill()
        pytest.fail("the run did not stop on SIGTERM")
    assert proc.returncode != 0                   # the interrupt propagates after the save
    saved = [p for p in ck.iterdir() if p.name.startswith("interrupted-")]
    assert saved, sorted(p.name for p in ck.iterdir())
    step = json.loads((saved[0] / "training_state.json").read_text())["step"]
    assert step >= 3

    from complexity_framework_b200.utils.checkpointing import peek_latest_checkpoint_step

    assert peek_latest_checkpoint_step(str(ck)) == step


def test_crash_mid_save_keeps_previous_checkpoint_loadable(tmp_path, monkeypatch):
    import safetensors.torch

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.utils.checkpointing import CheckpointManager

    torch.manual_seed(0)
    cfg = ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=256, intermediate_size=64,
                      shared_intermediate_size=128, num_experts=4, top_k=2,
                      routing_strategy="modulo_cyclic", max_position_embeddings=64)
    model = ComplexityModel(cfg)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    mgr = CheckpointManager(str(tmp_path))
    mgr.save(model, opt, step=1)
    good = {k: v.clone() for k, v in model.state_dict().items()}

    with torch.no_grad():
        for p in model.parameters():
            p.add_(1.0)

    def crash(*a, **kw):
        raise OSError("disk full while writing the weights")

    monkeypatch.setattr(safetensors.torch, "save_file", crash)
    with pytest.raises(OSError):
        mgr.save(model, opt, step=2)
    monkeypatch.undo()

    latest = mgr.latest()
    assert latest is not None and latest.name == "step-1"
    fresh = ComplexityModel(cfg)
    state = mgr.load(latest, fresh, torch.optim.AdamW(fresh.parameters(), lr=1e-3))
    assert state["step"] == 1
    for k, v in fresh.state_dict().items():
        assert torch.equal(v, good[k]), k
