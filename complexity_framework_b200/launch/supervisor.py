"""Supervise a training run: restart it when it crashes or stalls.

A rank stuck outside a collective (a hung data loader, a wedged filesystem)
raises nothing and never exits, so exit-code based restarts never fire; the
run's own progress file is the liveness signal instead.  The supervisor
starts the command in its own process group, polls the mtime of a progress
file (``metrics.jsonl`` / the training log), and when it has not been written
for ``stall_seconds`` -- or the process exits non-zero -- it stops the whole
group (SIGTERM, then SIGKILL after a grace period: the TrainRunner turns
SIGTERM into an "interrupted" checkpoint) and starts the command again with
``--resume auto`` appended, up to ``max_restarts`` times.  SIGTERM / SIGINT to
the supervisor are forwarded to the run.

Reference counterpart: scripts/watch_and_restart_stalled_process.py (stale-log
detection driving ``supervisorctl restart``); here the supervisor owns the
process directly and needs no supervisord.
"""
from __future__ import annotations

import logging
import os
import signal
import subprocess
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Sequence

logger = logging.getLogger(__name__)


def seconds_since_last_write(path: Path, now: Optional[float] = None) -> Optional[float]:
    """Seconds since ``path`` was last written, or None when it does not exist."""
    path = Path(path)
    if not path.exists():
        return None
    return (time.time() if now is None else now) - path.stat().st_mtime


@dataclass
class SupervisorConfig:
    command: Sequence[str]
    progress_file: Optional[str] = None    # liveness signal (None: exit codes only)
    stall_seconds: float = 900.0
    startup_grace_seconds: float = 600.0   # time allowed before the first write
    poll_seconds: float = 30.0
    max_restarts: int = 3
    term_grace_seconds: float = 60.0
    resume_args: Sequence[str] = ("--resume", "auto")
    env: Optional[dict] = None
    events: List[dict] = field(default_factory=list)


class RunSupervisor:
    def __init__(self, config: SupervisorConfig):
        self.cfg = config
        self.proc: Optional[subprocess.Popen] = None
        self.restarts = 0
        self._stop = False

    # ------------------------------------------------------------- process
    def _start(self, resume: bool) -> None:
        cmd = list(self.cfg.command)
        if resume:
            cmd += [a for a in self.cfg.resume_args if a not in cmd]
        env = dict(os.environ, **(self.cfg.env or {}))
        self.proc = subprocess.Popen(cmd, env=env, start_new_session=True)
        self.started = time.time()
        self._event("start", pid=self.proc.pid, resume=resume)

    def _kill_group(self) -> None:
        """SIGTERM to the run's process group, SIGKILL after the grace period."""
        p = self.proc
        if p is None or p.poll() is not None:
            return
        pgid = os.getpgid(p.pid)
        os.killpg(pgid, signal.SIGTERM)
        try:
            p.wait(timeout=self.cfg.term_grace_seconds)
        except subprocess.TimeoutExpired:
            os.killpg(pgid, signal.SIGKILL)
            p.wait()

    def _event(self, kind: str, **kw) -> None:
        rec = {"event": kind, "time": time.time(), **kw}
        self.cfg.events.append(rec)
        logger.info("supervisor: %s", rec)

    def _stalled(self) -> bool:
        if self.cfg.progress_file is None:
            return False
        idle = seconds_since_last_write(Path(self.cfg.progress_file))
        if idle is None:  # nothing written yet: startup grace
            return time.time() - self.started > self.cfg.startup_grace_seconds
        # a progress file older than this attempt counts from the attempt's start
        idle = min(idle, time.time() - self.started)
        return idle > self.cfg.stall_seconds

    # ---------------------------------------------------------------- loop
    def run(self) -> int:
        """Supervise until the run exits 0, restarts are exhausted, or the
        supervisor is signalled; returns the final exit code."""
        prev = {s: signal.signal(s, self._on_signal) for s in (signal.SIGTERM, signal.SIGINT)}
        try:
            self._start(resume=False)
            while True:
                code = self.proc.poll()
                if self._stop:
                    self._kill_group()
                    self._event("stopped")
                    return self.proc.returncode if self.proc.returncode is not None else 1
                if code == 0:
                    self._event("finished")
                    return 0
                reason = None
                if code is not None:
                    reason = f"exit {code}"
                elif self._stalled():
                    reason = "stalled"
                    self._kill_group()
                if reason is not None:
                    if self.restarts >= self.cfg.max_restarts:
                        self._event("giving_up", reason=reason)
                        return code if code not in (None, 0) else 1
                    self.restarts += 1
                    self._event("restart", reason=reason, attempt=self.restarts)
                    self._start(resume=True)
                time.sleep(self.cfg.poll_seconds)
        finally:
            for s, h in prev.items():
                signal.signal(s, h)

    def _on_signal(self, signum, frame):  # noqa: ARG002
        self._stop = True


# ------------------------------------------- external watchdog (supervisord)
def restart_program(program: str, runner=subprocess.run) -> bool:
    """``supervisorctl restart <program>``; True when it exits 0.  For runs
    that supervisord owns (the process cannot be a child of this one)."""
    logger.error("%s: progress file stale, restarting through supervisorctl", program)
    res = runner(["supervisorctl", "restart", program], capture_output=True, text=True)
    if res.returncode != 0:
        logger.error("restart of %s failed: %s %s", program, (res.stdout or "").strip(),
                     (res.stderr or "").strip())
        return False
    return True


def watch_once(log_file: Path, program: str, stall_seconds: float,
               now: Optional[float] = None, restart=restart_program) -> bool:
    """One staleness check: restart ``program`` (and return True) when
    ``log_file`` exists and has not been written for over ``stall_seconds``;
    a file that does not exist yet means the run is still starting."""
    idle = seconds_since_last_write(log_file, now=now)
    if idle is None or idle <= stall_seconds:
        return False
    restart(program)
    return True


def watch_supervisord(log_file: Path, program: str, stall_seconds: float = 900.0,
                      poll_seconds: float = 60.0, cooldown_seconds: Optional[float] = None,
                      max_checks: Optional[int] = None, sleep=time.sleep, clock=time.time,
                      restart=restart_program) -> int:
    """Poll forever (or ``max_checks`` times); restarts are at least
    ``cooldown_seconds`` apart (default ``stall_seconds``, so a run that is
    broken is not restarted faster than it could write a fresh line).  Keep
    ``stall_seconds`` above the collective timeout so a hung collective
    errors out before the watchdog fires.  Returns the number of restarts."""
    cooldown = stall_seconds if cooldown_seconds is None else cooldown_seconds
    last, restarts, checks = float("-inf"), 0, 0
    while max_checks is None or checks < max_checks:
        now = clock()
        if now - last >= cooldown and watch_once(Path(log_file), program, stall_seconds, now,
                                                 restart=restart):
            last, restarts = now, restarts + 1
        checks += 1
        if max_checks is None or checks < max_checks:
            sleep(poll_seconds)
    return restarts
