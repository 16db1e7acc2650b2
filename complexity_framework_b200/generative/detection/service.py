"""Local HTTP API for detector inference and isolated training jobs.

    python -m complexity_framework_b200.generative.detection.service \
        --checkpoint runs/det/best --jobs-root runs/jobs --port 8090 [--api-key KEY]

Counterpart of complexity/generative/detection/service.py:26-598:
  * ``ModelRuntime``: a detector checkpoint (``config.json`` + weights) loaded
    once, warmed up, and hot-swappable under a lock (``promote`` of a finished
    job's best checkpoint replaces the serving model atomically);
  * ``TrainingJobManager``: each training request runs
    ``generative.detection.train`` in its own subprocess and directory; job
    records persist as JSON (they survive a restart: jobs that were running
    are marked ``interrupted``), with status, cancel, log tail and the run's
    metrics;
  * ``create_app``: FastAPI routes ``/health``, ``/model``, ``/predict`` (raw
    image bytes in the body, detections in original image pixels and
    normalised coordinates), ``/train``, ``/train/{id}``, ``/train/{id}/logs``,
    ``/train/{id}/cancel``, ``/train/{id}/promote``; an ``X-API-Key`` header
    is required when a key is configured.
"""

import argparse
import io
import json
import os
import subprocess
import sys
import threading
import time
import uuid
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch

from .config import TRHashDetectorConfig
from .data import preprocess_detector_image, restore_detector_boxes
from .model import TRHashObjectDetector


def resolve_device(override: Optional[str]) -> torch.device:
    if override:
        return torch.device(override)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def decode_image(data: bytes) -> torch.Tensor:
    """Image file bytes -> float [3, H, W] in [0, 1]."""
    from PIL import Image

    img = Image.open(io.BytesIO(data)).convert("RGB")
    import numpy as np

    arr = torch.from_numpy(np.asarray(img, dtype=np.uint8).copy())
    return arr.permute(2, 0, 1).float() / 255.0


class ModelRuntime:
    """A served detector; ``load`` swaps in another checkpoint atomically."""

    def __init__(self, checkpoint, device: torch.device):
        self.device = device
        self.lock = threading.RLock()
        self.model: Optional[TRHashObjectDetector] = None
        self.config: Optional[TRHashDetectorConfig] = None
        self.validation: Dict[str, Any] = {}
        self.checkpoint = Path()
        self.loaded_at = 0.0
        self.load(checkpoint)

    def load(self, checkpoint) -> None:
        ck = Path(checkpoint).resolve()
        cfg = TRHashDetectorConfig.from_dict(json.loads((ck / "config.json").read_text()))
        model = TRHashObjectDetector(cfg)
        model.load_state_dict(torch.load(ck / "model.pt", map_location="cpu"))
        model.to(self.device).eval()
        with torch.inference_mode():  # warm-up before the swap
            model(torch.zeros(1, cfg.num_channels, cfg.image_size, cfg.image_size,
                              device=self.device))
        metrics = ck / "metrics.json"
        with self.lock:
            self.model, self.config = model, cfg
            self.validation = json.loads(metrics.read_text()) if metrics.exists() else {}
            self.checkpoint, self.loaded_at = ck, time.time()

    @torch.inference_mode()
    def predict(self, image: torch.Tensor, *, confidence: float = 0.25,
                iou_threshold: Optional[float] = None) -> List[Dict[str, Any]]:
        with self.lock:
            if self.model is None:
                raise RuntimeError("model is not loaded")
            c = self.config
            pixels, meta = preprocess_detector_image(image, c.image_size)
            kw = {"score_threshold": confidence}
            if iou_threshold is not None:
                kw["iou_threshold"] = iou_threshold
            det = self.model.predict(pixels[None].to(self.device), **kw)[0]
            boxes = restore_detector_boxes(det["boxes"].float().cpu(), meta)
            H, W = meta.original_size
            return [{"box_xyxy": [float(v) for v in b],
                     "box_normalized": [float(b[0]) / W, float(b[1]) / H, float(b[2]) / W,
                                        float(b[3]) / H],
                     "score": float(s), "label": int(lab),
                     "name": (c.class_names[int(lab)] if int(lab) < len(c.class_names) else None)}
                    for b, s, lab in zip(boxes, det["scores"].cpu(), det["labels"].cpu())]

    def info(self) -> Dict[str, Any]:
        with self.lock:
            c = self.config
            return {"checkpoint": str(self.checkpoint), "loaded_at": self.loaded_at,
                    "device": str(self.device), "image_size": c.image_size,
                    "num_classes": c.num_classes, "class_names": list(c.class_names),
                    "parameters": sum(p.numel() for p in self.model.parameters()),
                    "validation": self.validation}


@dataclass
class JobRecord:
    job_id: str
    status: str                 # queued | running | succeeded | failed | cancelled | interrupted
    created_at: float
    output_dir: str
    log_path: str
    arguments: List[str] = field(default_factory=list)
    return_code: Optional[int] = None
    finished_at: Optional[float] = None
    pid: Optional[int] = None


class TrainingJobManager:
    """Training runs as subprocesses with persisted records."""

    def __init__(self, root, python_executable: str = sys.executable):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.python = python_executable
        self.lock = threading.Lock()
        self.jobs: Dict[str, JobRecord] = {}
        self.procs: Dict[str, subprocess.Popen] = {}
        self._restore()

    def _restore(self) -> None:
        for f in sorted(self.root.glob("*/job.json")):
            rec = JobRecord(**json.loads(f.read_text()))
            if rec.status in ("queued", "running"):
                rec.status = "interrupted"  # the process did not survive the restart
                self._persist(rec)
            self.jobs[rec.job_id] = rec

    def _persist(self, rec: JobRecord) -> None:
        d = self.root / rec.job_id
        d.mkdir(parents=True, exist_ok=True)
        tmp = d / ".job.json.tmp"
        tmp.write_text(json.dumps(asdict(rec), indent=2))
        tmp.replace(d / "job.json")

    def start(self, options: Dict[str, Any], device: Optional[str] = None) -> JobRecord:
        jid = uuid.uuid4().hex[:12]
        d = self.root / jid
        d.mkdir(parents=True)
        args = ["-m", "complexity_framework_b200.generative.detection.train",
                "--output", str(d / "run")]
        for k, v in options.items():
            if k in ("output", "resume"):
                continue
            flag = f"--{k.replace('_', '-')}"
            if isinstance(v, bool):
                if v:
                    args.append(flag)
            elif isinstance(v, dict):
                args += [flag, json.dumps(v)]
            elif v is not None:
                args += [flag, str(v)]
        if device:
            args += ["--device", device]
        rec = JobRecord(job_id=jid, status="queued", created_at=time.time(),
                        output_dir=str(d / "run"), log_path=str(d / "train.log"), arguments=args)
        log = open(rec.log_path, "w")
        env = dict(os.environ)
        root = str(Path(__file__).resolve().parents[3])
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        proc = subprocess.Popen([self.python] + args, stdout=log, stderr=subprocess.STDOUT,
                                env=env, start_new_session=True)
        rec.status, rec.pid = "running", proc.pid
        with self.lock:
            self.jobs[jid], self.procs[jid] = rec, proc
            self._persist(rec)
        threading.Thread(target=self._wait, args=(jid, proc, log), daemon=True).start()
        return rec

    def _wait(self, jid: str, proc: subprocess.Popen, log) -> None:
        rc = proc.wait()
        log.close()
        with self.lock:
            rec = self.jobs[jid]
            rec.return_code, rec.finished_at = rc, time.time()
            if rec.status != "cancelled":
                rec.status = "succeeded" if rc == 0 else "failed"
            self._persist(rec)
            self.procs.pop(jid, None)

    def get(self, jid: str) -> JobRecord:
        if jid not in self.jobs:
            raise KeyError(jid)
        return self.jobs[jid]

    def wait(self, jid: str, timeout: Optional[float] = None) -> JobRecord:
        proc = self.procs.get(jid)
        if proc is not None:
            proc.wait(timeout)
            deadline = time.time() + 5
            while self.get(jid).status == "running" and time.time() < deadline:
                time.sleep(0.01)
        return self.get(jid)

    def cancel(self, jid: str) -> JobRecord:
        with self.lock:
            rec = self.get(jid)
            proc = self.procs.get(jid)
            if proc is not None and proc.poll() is None:
                rec.status = "cancelled"
                proc.terminate()  # only the job's own process
                self._persist(rec)
        return rec

    def metrics(self, jid: str) -> Optional[Dict[str, Any]]:
        out = Path(self.get(jid).output_dir)
        if (out / "summary.json").exists():
            return json.loads((out / "summary.json").read_text())
        hist = out / "history.jsonl"
        if hist.exists():
            lines = [json.loads(x) for x in hist.read_text().splitlines() if x.strip()]
            return {"history": lines}
        return None

    def log_tail(self, jid: str, lines: int = 100) -> str:
        p = Path(self.get(jid).log_path)
        return "\n".join(p.read_text(errors="replace").splitlines()[-lines:]) if p.exists() else ""

    def best_checkpoint(self, jid: str) -> Path:
        rec = self.get(jid)
        if rec.status != "succeeded":
            raise ValueError(f"job {jid} has not succeeded (status {rec.status})")
        best = Path(rec.output_dir) / "best"
        if not (best / "config.json").exists():
            raise ValueError(f"job {jid} produced no best checkpoint")
        return best


def create_app(runtime: Optional[ModelRuntime], jobs: Optional[TrainingJobManager] = None,
               api_key: Optional[str] = None, train_device: Optional[str] = None):
    from fastapi import Depends, FastAPI, Header, HTTPException, Request
    from pydantic import BaseModel

    class TrainingRequest(BaseModel):
        options: Dict[str, Any] = {}

    app = FastAPI(title="TR-Hash detector service")

    def authenticate(x_api_key: Optional[str] = Header(default=None)) -> None:
        if api_key is not None and x_api_key != api_key:
            raise HTTPException(status_code=401, detail="invalid or missing API key")

    def need_runtime() -> ModelRuntime:
        if runtime is None:
            raise HTTPException(status_code=503, detail="no model loaded")
        return runtime

    def need_jobs() -> TrainingJobManager:
        if jobs is None:
            raise HTTPException(status_code=503, detail="training jobs are disabled")
        return jobs

    def job_or_404(jid: str) -> JobRecord:
        try:
            return need_jobs().get(jid)
        except KeyError:
            raise HTTPException(status_code=404, detail=f"unknown job {jid}")

    @app.get("/health")
    def health():
        return {"status": "ok", "model_loaded": runtime is not None}

    @app.get("/model", dependencies=[Depends(authenticate)])
    def model_info():
        return need_runtime().info()

    @app.post("/predict", dependencies=[Depends(authenticate)])
    async def predict(request: Request, confidence: float = 0.25,
                      iou_threshold: Optional[float] = None):
        data = await request.body()
        if not data:
            raise HTTPException(status_code=400, detail="empty body: send the image bytes")
        try:
            image = decode_image(data)
        except Exception as exc:
            raise HTTPException(status_code=400, detail=f"cannot decode image: {exc}")
        dets = need_runtime().predict(image, confidence=confidence, iou_threshold=iou_threshold)
        return {"detections": dets, "count": len(dets)}

    @app.post("/train", dependencies=[Depends(authenticate)])
    def start_training(req: TrainingRequest):
        return asdict(need_jobs().start(req.options, train_device))

    @app.get("/train/{jid}", dependencies=[Depends(authenticate)])
    def training_status(jid: str):
        rec = job_or_404(jid)
        return {**asdict(rec), "metrics": need_jobs().metrics(jid)}

    @app.get("/train/{jid}/logs", dependencies=[Depends(authenticate)])
    def training_logs(jid: str, lines: int = 100):
        job_or_404(jid)
        return {"job_id": jid, "log": need_jobs().log_tail(jid, lines)}

    @app.post("/train/{jid}/cancel", dependencies=[Depends(authenticate)])
    def cancel_training(jid: str):
        job_or_404(jid)
        return asdict(need_jobs().cancel(jid))

    @app.post("/train/{jid}/promote", dependencies=[Depends(authenticate)])
    def promote(jid: str):
        job_or_404(jid)
        try:
            best = need_jobs().best_checkpoint(jid)
        except ValueError as exc:
            raise HTTPException(status_code=409, detail=str(exc))
        need_runtime().load(best)
        return {"promoted": str(best), "model": runtime.info()}

    return app


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="TR-Hash detector inference / training service")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--jobs-root", default="detector_jobs")
    ap.add_argument("--device", default=None)
    ap.add_argument("--train-device", default=None)
    ap.add_argument("--api-key", default=os.environ.get("DETECTOR_API_KEY"))
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8090)
    a = ap.parse_args(argv)
    import uvicorn

    rt = ModelRuntime(a.checkpoint, resolve_device(a.device)) if a.checkpoint else None
    app = create_app(rt, TrainingJobManager(a.jobs_root), a.api_key, a.train_device)
    uvicorn.run(app, host=a.host, port=a.port)


if __name__ == "__main__":
    main()
