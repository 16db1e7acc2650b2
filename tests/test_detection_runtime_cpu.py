"""Detector runtime: COCO-style metrics (against the reference accumulator on
identical inputs), schedules, exact-resume training state, a training run with
accumulation / Mosaic closing / validation / resume, gloo data parallel, and
the HTTP service (inference, job lifecycle, promotion)."""
import io
import json
import os
import socket
import sys
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from complexity_framework_b200.generative.detection import schedule as S
from complexity_framework_b200.generative.detection.metrics import DetectionMetricsAccumulator
from complexity_framework_b200.generative.detection.train import DetectorRunConfig, train_detector

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

TINY = dict(hidden_size=32, num_layers=1, num_heads=2, shared_width=64, expert_width=32,
            neck_channels=32, patch_size=8)


def _rand_case(g, n_img=6, C=3):
    imgs = []
    for _ in range(n_img):
        n = int(torch.randint(1, 6, (1,), generator=g))
        cxcy = torch.rand(n, 2, generator=g) * 0.8 + 0.1
        wh = torch.rand(n, 2, generator=g) * 0.3 + 0.02
        lab = torch.randint(0, C, (n,), generator=g).float()
        targets = torch.cat((cxcy, wh, lab[:, None]), 1)
        gt = torch.cat((cxcy - wh / 2, cxcy + wh / 2), 1)
        m = int(torch.randint(0, 9, (1,), generator=g))
        pick = torch.randint(0, n, (m,), generator=g)
        boxes = (gt[pick] + 0.03 * torch.randn(m, 4, generator=g)).clamp(0, 1)
        scores = torch.rand(m, generator=g)
        labels = torch.where(torch.rand(m, generator=g) < 0.8, lab[pick].long(),
                             torch.randint(0, C, (m,), generator=g))
        imgs.append((boxes, scores, labels, targets))
    return imgs


def test_metrics_match_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.generative.detection.metrics import DetectionMetricsAccumulator as Ref
    finally:
        sys.path.remove(REF)
    g = torch.Generator().manual_seed(0)
    case = _rand_case(g)
    a, b = DetectionMetricsAccumulator(3, 320), Ref(3, 320)
    for x in case:
        a.update(*x)
        b.update(*x)
    ra, rb = a.compute(0.3), b.compute(0.3)
    assert set(ra) == set(rb)
    for k in ra:
        assert abs(ra[k] - rb[k]) < 1e-6, (k, ra[k], rb[k])
    # merging two halves equals one pass
    h1, h2 = DetectionMetricsAccumulator(3, 320), DetectionMetricsAccumulator(3, 320)
    for i, x in enumerate(case):
        (h1 if i % 2 else h2).update(*x)
    h1.merge_state_dict(h2.state_dict())
    for k, v in h1.compute(0.3).items():
        assert abs(v - ra[k]) < 1e-6, k


def test_perfect_predictions_score_one():
    acc = DetectionMetricsAccumulator(2)
    gt = torch.tensor([[10.0, 10, 50, 50], [60, 60, 200, 200]])
    acc.update_xyxy(gt, torch.tensor([0.9, 0.8]), torch.tensor([0, 1]), gt, torch.tensor([0, 1]))
    r = acc.compute(0.5)
    assert r["map50"] == pytest.approx(1.0) and r["map50_95"] == pytest.approx(1.0)
    assert r["precision"] == 1.0 and r["recall"] == 1.0


def test_schedules():
    assert S.cosine_schedule(0, warmup_steps=10, total_steps=100, min_ratio=0.1) == 0.1
    assert S.cosine_schedule(100, warmup_steps=10, total_steps=100, min_ratio=0.1) == pytest.approx(0.1)
    assert S.cosine_schedule(10, warmup_steps=10, total_steps=100, min_ratio=0.1) == pytest.approx(1.0)
    assert [S.should_validate_epoch(e, 5, 2) for e in range(5)] == [False, True, False, True, True]
    assert S.validation_selection_score({"map50": 0.3}) == ("map50", 0.3)
    assert S.validation_selection_score({"official_coco": True, "coco_map50_95": 0.2,
                                         "map50": 0.5}) == ("coco_map50_95", 0.2)
    assert S.mosaic_source_images_per_sample(0.5) == 2.5
    act = [S.mosaic_is_active_epoch(e, total_epochs=10, close_mosaic_epochs=3,
                                    mosaic_probability=1.0) for e in range(10)]
    assert act == [True] * 7 + [False] * 3
    assert S.detector_step_schedule(10, total_epochs=4, mosaic_probability=1.0,
                                    close_mosaic_epochs=1, mosaic_packed_epoch=True,
                                    packed_epochs=4) == (3, 3, 3, 10)
    assert S.resolve_accumulation_steps(per_device_batch_size=8, world_size=2,
                                        nominal_batch_size=64) == 4
    assert S.optimizer_step_schedule((10, 7), 4) == (3, 2)
    assert [S.accumulation_group(i, epoch_batches=7, accumulation_steps=3) for i in range(7)] == [
        (3, False), (3, False), (3, True), (3, False), (3, False), (3, True), (1, True)]
    assert S.normalized_weight_decay(0.05, global_batch_size=16, accumulation_steps=4,
                                     nominal_batch_size=64) == pytest.approx(0.05)
    assert S.resolve_warmup_steps(requested_steps=100, warmup_epochs=0.5, steps_in_first_epoch=40,
                                  total_steps=400) == 20
    assert S.resolve_warmup_steps(requested_steps=100, warmup_epochs=None, steps_in_first_epoch=40,
                                  total_steps=200, unpacked_total_steps=400) == 50
    m = S.format_loss_metrics_for_logging({"loss": 2.0, "monitor_loss": 1.5})
    assert m == {"optimization_loss": 2.0, "loss": 1.5}


def _cfg(tmp, **kw):
    base = dict(dataset="synthetic", synthetic_train=16, synthetic_val=8, image_size=64,
                num_classes=2, model_overrides=TINY, epochs=3, batch_size=4,
                nominal_batch_size=8, warmup_steps=2, close_mosaic_epochs=1, amp_bf16=False,
                output=str(tmp), device="cpu")
    base.update(kw)
    return DetectorRunConfig(**base)


def test_training_run_validates_checkpoints_and_resumes(tmp_path):
    s = train_detector(_cfg(tmp_path / "a"))
    assert s["accumulation_steps"] == 2 and s["steps"] == 3 * 2
    assert [h["mosaic"] for h in s["history"]] == [True, True, False]
    assert all("val_map50" in h for h in s["history"])
    for d in ("best", "last"):
        assert (tmp_path / "a" / d / "config.json").exists()
    assert (tmp_path / "a" / "last" / "training_state.pt").exists()
    # interrupted after 2 epochs, then resumed: same final weights as one run
    s2 = train_detector(_cfg(tmp_path / "b", epochs=3, eval_every=10))
    part = _cfg(tmp_path / "c", epochs=3, eval_every=10)
    # stop the run after its third epoch's training, before that epoch is saved
    import complexity_framework_b200.generative.detection.train as mod

    calls = {"n": 0}
    real = mod.should_validate_epoch

    def stop_after_two(epoch, total, every):
        calls["n"] += 1
        if epoch == 2:
            raise KeyboardInterrupt
        return real(epoch, total, every)

    mod.should_validate_epoch = stop_after_two
    try:
        with pytest.raises(KeyboardInterrupt):
            train_detector(part)
    finally:
        mod.should_validate_epoch = real
    resumed = train_detector(_cfg(tmp_path / "c", epochs=3, eval_every=10, resume=True))
    assert resumed["steps"] == s2["steps"]
    a = torch.load(tmp_path / "b" / "last" / "train_model.pt")
    b = torch.load(tmp_path / "c" / "last" / "train_model.pt")
    assert all(torch.allclose(a[k], b[k], atol=1e-6) for k in a)
    with pytest.raises(ValueError, match="mismatched"):
        train_detector(_cfg(tmp_path / "c", epochs=3, eval_every=10, resume=True,
                            learning_rate=5e-4))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ddp_body(rank, world, port, out, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = train_detector(_cfg(out, epochs=2, batch_size=2, nominal_batch_size=8,
                                synthetic_train=8))
        q.put((rank, s["steps"], s["accumulation_steps"], s["history"][-1]["val_map50"]))
    finally:
        dist.destroy_process_group()


def test_data_parallel_training_gloo(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ddp_body, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert [p.exitcode for p in ps] == [0, 0]
    res = sorted(q.get() for _ in range(2))
    # 8 images / (2 per rank x 2 ranks) = 2 microbatches per epoch; nominal 8 -> accumulate 2
    assert res[0][1:3] == (2, 2) and res[0][1:] == res[1][1:]


def test_service_predict_jobs_and_promote(tmp_path):
    from fastapi.testclient import TestClient
    from PIL import Image

    from complexity_framework_b200.generative.detection.service import (ModelRuntime,
                                                                        TrainingJobManager,
                                                                        create_app)

    train_detector(_cfg(tmp_path / "seed", epochs=1))
    rt = ModelRuntime(tmp_path / "seed" / "best", torch.device("cpu"))
    jobs = TrainingJobManager(tmp_path / "jobs")
    client = TestClient(create_app(rt, jobs, api_key="k"))
    assert client.get("/health").json()["model_loaded"]
    assert client.get("/model").status_code == 401
    info = client.get("/model", headers={"X-API-Key": "k"}).json()
    assert info["image_size"] == 64
    buf = io.BytesIO()
    Image.new("RGB", (96, 48), (200, 30, 30)).save(buf, format="PNG")
    r = client.post("/predict?confidence=0.0", content=buf.getvalue(), headers={"X-API-Key": "k"})
    assert r.status_code == 200
    for d in r.json()["detections"]:
        assert 0 <= d["box_xyxy"][0] <= 96 and 0 <= d["box_normalized"][3] <= 1
    assert client.post("/predict", content=b"x", headers={"X-API-Key": "k"}).status_code == 400
    opts = {k: v for k, v in vars(_cfg(tmp_path / "unused", epochs=1)).items()
            if k not in ("output", "device", "resume")}
    job = client.post("/train", json={"options": opts}, headers={"X-API-Key": "k"}).json()
    rec = jobs.wait(job["job_id"], timeout=600)
    assert rec.status == "succeeded", jobs.log_tail(job["job_id"])
    st = client.get(f"/train/{job['job_id']}", headers={"X-API-Key": "k"}).json()
    assert st["metrics"]["epochs"] == 1
    pr = client.post(f"/train/{job['job_id']}/promote", headers={"X-API-Key": "k"}).json()
    assert pr["promoted"].endswith("best")
    # records survive a restart
    assert TrainingJobManager(tmp_path / "jobs").get(job["job_id"]).status == "succeeded"
