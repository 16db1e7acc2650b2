"""TR-Hash detector: box ops, losses, letterboxing, COCO-style metric, training,
checkpoint and TorchScript export (CPU)."""
import torch

from complexity_framework_b200.generative.detection import (
    DetectorTrainer, DetectorTrainingConfig, SyntheticShapesDataset, TRHashDetectorConfig,
    TRHashObjectDetector, box_iou, class_aware_nms, collate_detection, complete_iou,
    distribution_focal_loss, evaluate_detections, export_detector_torchscript, greedy_nms,
    load_detector_checkpoint, preprocess_detector_image, quality_focal_loss,
    restore_detector_boxes, save_detector_checkpoint)


def _brute_nms(boxes, scores, t):
    order = scores.argsort(descending=True).tolist()
    keep = []
    for i in order:
        if all(box_iou(boxes[i:i + 1], boxes[j:j + 1])[0, 0] <= t for j in keep):
            keep.append(i)
    return keep


def test_nms_matches_sequential_definition():
    g = torch.Generator().manual_seed(0)
    xy = torch.rand(60, 2, generator=g) * 50
    wh = torch.rand(60, 2, generator=g) * 30 + 5
    boxes = torch.cat([xy, xy + wh], 1)
    scores = torch.rand(60, generator=g)
    assert greedy_nms(boxes, scores, 0.5).tolist() == _brute_nms(boxes, scores, 0.5)
    cls = torch.randint(0, 3, (60,), generator=g)
    keep = class_aware_nms(boxes, scores, cls, 0.5)
    for c in range(3):  # per class it is plain NMS
        idx = (cls == c).nonzero().squeeze(1)
        ref = idx[torch.tensor(_brute_nms(boxes[idx], scores[idx], 0.5), dtype=torch.long)]
        assert sorted(keep[cls[keep] == c].tolist()) == sorted(ref.tolist())


def test_iou_and_ciou():
    a = torch.tensor([[0., 0., 10., 10.]])
    b = torch.tensor([[5., 0., 15., 10.]])
    assert abs(float(box_iou(a, b)) - 50 / 150) < 1e-6
    assert abs(float(complete_iou(a[0], a[0])) - 1.0) < 1e-5
    # same IoU, farther centres -> lower CIoU
    assert float(complete_iou(a[0], b[0])) < float(box_iou(a, b))


def test_focal_losses():
    x = torch.tensor([[2.0, -3.0]])
    assert float(quality_focal_loss(x, torch.sigmoid(x))) < 1e-6
    d = torch.full((1, 16), -10.0)
    d[0, 3] = 10.0
    assert float(distribution_focal_loss(d, torch.tensor([3.0]))) < 1e-3
    assert float(distribution_focal_loss(d, torch.tensor([3.5]))) > 1.0


def test_letterbox_round_trip():
    img = torch.rand(3, 60, 100)
    out, meta = preprocess_detector_image(img, 128)
    assert out.shape == (3, 128, 128)
    b = torch.tensor([[10., 5., 50., 40.]])
    lb = b.clone()
    lb[:, [0, 2]] = lb[:, [0, 2]] * meta.scale + meta.pad_x
    lb[:, [1, 3]] = lb[:, [1, 3]] * meta.scale + meta.pad_y
    assert torch.allclose(restore_detector_boxes(lb, meta), b, atol=1e-4)


def test_coco_metric_known_cases():
    gt = [{"boxes": torch.tensor([[0., 0., 10., 10.], [20., 20., 30., 30.]]),
           "labels": torch.tensor([0, 1])}]
    perfect = [{"boxes": gt[0]["boxes"], "scores": torch.tensor([0.9, 0.8]),
                "labels": torch.tensor([0, 1])}]
    assert abs(evaluate_detections(perfect, gt, 2)["mAP"] - 1.0) < 1e-9
    half = [{"boxes": torch.tensor([[0., 0., 10., 10.]]), "scores": torch.tensor([0.9]),
             "labels": torch.tensor([0])}]
    r = evaluate_detections(half, gt, 2)
    assert abs(r["AP50"] - 0.5) < 1e-9  # class 0 found, class 1 missed


def _small():
    return TRHashDetectorConfig(image_size=64, patch_size=16, hidden_size=64, num_layers=1,
                                num_heads=4, shared_width=128, expert_width=32, num_classes=2,
                                neck_channels=32)


def test_detector_trains_and_predicts(tmp_path):
    torch.manual_seed(0)
    m = TRHashObjectDetector(_small())
    dl = torch.utils.data.DataLoader(SyntheticShapesDataset(32, 64, 2, 2), batch_size=8,
                                     collate_fn=collate_detection)
    tr = DetectorTrainer(m, DetectorTrainingConfig(learning_rate=2e-3, warmup_steps=4,
                                                   max_steps=40, ema_tau=5))
    ev = torch.utils.data.DataLoader(SyntheticShapesDataset(16, 64, 2, 2, seed=7), batch_size=8,
                                     collate_fn=collate_detection)
    before = tr.evaluate(ev, use_ema=False)["AP50"]
    for _ in range(10):
        for im, tg in dl:
            tr.train_step(im, tg)
    after = tr.evaluate(ev, use_ema=False)["AP50"]
    # the loss is IoU-weighted (it grows as boxes start to overlap), so measure progress by AP
    assert after > max(0.2, before), (before, after)
    out = m.predict(torch.rand(2, 3, 64, 64))
    assert len(out) == 2 and set(out[0]) == {"boxes", "scores", "labels"}
    save_detector_checkpoint(m, str(tmp_path / "det"))
    m2 = load_detector_checkpoint(str(tmp_path / "det"))
    x = torch.rand(1, 3, 64, 64)
    m.eval()
    assert torch.allclose(m(x)["boxes"], m2(x)["boxes"], atol=1e-5)
    path = export_detector_torchscript(m, str(tmp_path / "det.pt"))
    scores, boxes = torch.jit.load(path)(x)
    assert torch.allclose(boxes, m(x)["boxes"], atol=1e-4)
    assert scores.shape[-1] == 2


def test_hierarchical_tower_and_detector(tmp_path):
    from complexity_framework_b200.generative.hierarchical import (
        HierarchicalTowerConfig, HierarchicalTRHashVisionClassifier, HierarchicalTRHashVisionTower)

    torch.manual_seed(0)
    hc = HierarchicalTowerConfig(image_size=64, dims=(32, 64, 64, 96), depths=(2, 1, 2, 1),
                                 heads=(2, 2, 4, 4), window_size=4)
    maps = HierarchicalTRHashVisionTower(hc)(torch.rand(2, 3, 64, 64))
    assert [tuple(m.shape[1:]) for m in maps] == [(32, 16, 16), (64, 8, 8), (64, 4, 4), (96, 2, 2)]
    # other resolutions: positions are interpolated
    maps = HierarchicalTRHashVisionTower(hc)(torch.rand(1, 3, 96, 64))
    assert tuple(maps[0].shape[-2:]) == (24, 16)
    clf = HierarchicalTRHashVisionClassifier(hc, 3)
    clf(torch.rand(2, 3, 64, 64), torch.tensor([0, 1]))["loss"].backward()
    cfg = TRHashDetectorConfig(image_size=64, backbone="hierarchical", hier_dims=(32, 64, 64, 96),
                               hier_depths=(1, 1, 1, 1), hier_heads=(2, 2, 4, 4), hier_window=4,
                               num_classes=2, neck_channels=32)
    det = TRHashObjectDetector(cfg)
    dl = torch.utils.data.DataLoader(SyntheticShapesDataset(16, 64, 2, 2), batch_size=8,
                                     collate_fn=collate_detection)
    tr = DetectorTrainer(det, DetectorTrainingConfig(warmup_steps=2, max_steps=10))
    for im, tg in dl:
        assert all(torch.isfinite(torch.tensor(v)) for v in tr.train_step(im, tg).values())
    save_detector_checkpoint(det, str(tmp_path / "h"))
    back = load_detector_checkpoint(str(tmp_path / "h"))
    det.eval()
    x = torch.rand(1, 3, 64, 64)
    assert torch.allclose(det(x)["boxes"], back(x)["boxes"], atol=1e-5)


def test_window_padding_is_masked():
    """A 3x3 grid in one 4x4 window (7 padded slots) attends exactly like the
    same attention over the 9 real tokens."""
    import torch.nn.functional as F

    from complexity_framework_b200.generative.hierarchical import (HierarchicalBlock,
                                                                   HierarchicalTowerConfig)

    torch.manual_seed(0)
    blk = HierarchicalBlock(16, 2, 4, False, HierarchicalTowerConfig(), 64, 0)
    x = torch.randn(2, 9, 16)
    win, mask, Hp, Wp = blk._windows(blk.n1(x), 3, 3)
    got = blk._unwindows(blk.attn(win, mask), 2, 3, 3, Hp, Wp)
    a = blk.attn
    q, k, v = a.qkv(blk.n1(x)).view(2, 9, 3, 2, 8).permute(2, 0, 3, 1, 4)
    rel = a.bias[:, a.rel].view(2, 4, 4, 4, 4)[:, :3, :3, :3, :3].reshape(2, 9, 9)
    ref = F.scaled_dot_product_attention(q, k, v, attn_mask=rel[None])
    ref = a.proj(ref.transpose(1, 2).reshape(2, 9, 16))
    assert torch.allclose(got, ref, atol=1e-5)


def test_augmentations_keep_boxes_on_objects():
    import random

    from complexity_framework_b200.generative.detection import (AugmentedDataset,
                                                                DetectionAugment, horizontal_flip,
                                                                mosaic, random_scale)

    ds = SyntheticShapesDataset(8, 64, 2, 1)  # class 0: filled rectangles

    def covered(img, t):
        # every box still encloses mostly object pixels (bright in some channel)
        for b in t["boxes"].round().long().tolist():
            patch = img[:, b[1]:b[3], b[0]:b[2]]
            if patch.numel() and float((patch.max(0).values > 0.5).float().mean()) < 0.6:
                return False
        return True

    img, t = ds[0]
    assert covered(*horizontal_flip(img, t))
    rng = random.Random(3)
    for _ in range(5):
        assert covered(*random_scale(img, t, 0.7, 1.3, rng=rng))
    m_img, m_t = mosaic([ds[i] for i in range(4)], rng)
    assert m_img.shape == img.shape and len(m_t["boxes"]) >= 1 and covered(m_img, m_t)
    aug = AugmentedDataset(ds, DetectionAugment(p_mosaic=1.0, color=0.0, seed=1))
    a_img, a_t = aug[0]
    assert a_img.shape == img.shape and a_t["boxes"].shape[1] == 4


def _ddp_worker(rank, world, port, q):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    torch.manual_seed(0)  # same initial weights on every rank
    m = TRHashObjectDetector(_small())
    tr = DetectorTrainer(m, DetectorTrainingConfig(warmup_steps=1, max_steps=4))
    ds = SyntheticShapesDataset(8, 64, 2, 2, seed=rank)  # different data per rank
    for i in range(2):
        tr.train_step(*collate_detection([ds[2 * i], ds[2 * i + 1]]))
    flat = torch.cat([p.detach().reshape(-1) for p in m.parameters()])
    ev = [collate_detection([ds[4], ds[5]])]
    res = tr.evaluate(ev, use_ema=False)
    gathered = [None] * world
    dist.all_gather_object(gathered, (float(flat.sum()), float(flat.abs().sum()), res["AP50"]))
    if rank == 0:
        q.put(gathered)
    dist.destroy_process_group()


def test_detector_trainer_data_parallel_gloo():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    g = q.get(timeout=240)
    for p in ps:
        p.join(timeout=60)
    (s0, a0, ap0), (s1, a1, ap1) = g
    assert abs(s0 - s1) < 1e-4 and abs(a0 - a1) < 1e-4  # replicas stayed in sync
    assert ap0 == ap1                                     # both scored the union


def test_cli_train_detector_and_detect(tmp_path, capsys):
    import json

    from torchvision.io import write_png

    from complexity_framework_b200.cli.app import main

    out = str(tmp_path / "det")
    main(["train-detector", "--data", "synthetic", "--image-size", "64", "--synthetic-images",
          "16", "--batch", "8", "--steps", "3", "--log-every", "1", "--output", out])
    lines = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines()]
    assert lines[0]["step"] == 1 and "mAP" in lines[-2]["eval"] and lines[-1]["saved"] == out
    img_path = str(tmp_path / "x.png")
    write_png((torch.rand(3, 48, 80) * 255).to(torch.uint8), img_path)
    main(["detect", "--checkpoint", out, "--score", "0.0", img_path])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["image"] == img_path
    for d in res["detections"]:
        x0, y0, x1, y1 = d["box"]
        assert 0 <= x0 <= x1 <= 80 and 0 <= y0 <= y1 <= 48  # original-image coordinates


def test_release_evaluation_branches_and_timing():
    import pytest

    from complexity_framework_b200.generative.detection.release_eval import (
        BRANCHES, branches_to_run, evaluate_release, percentile, timing_summary)

    with pytest.raises(ValueError, match="NMS-free"):
        branches_to_run("both", has_nms_free=False)
    assert branches_to_run("o2m-nms", has_nms_free=False) == ("o2m-nms",)
    assert branches_to_run("both", has_nms_free=True) == BRANCHES
    s = timing_summary([0.1, 0.3, 0.2], image_count=12)
    assert s["mean_batch_ms"] == pytest.approx(200.0) and s["p50_batch_ms"] == pytest.approx(200.0)
    assert s["p95_batch_ms"] == pytest.approx(300.0) and s["images_per_second"] == pytest.approx(20.0)
    assert s["measured_seconds"] == pytest.approx(0.6) and percentile([], 0.95) == 0.0
    torch.manual_seed(0)
    m = TRHashObjectDetector(_small())
    ds = SyntheticShapesDataset(6, 64, 2, 2, seed=3)
    ims, tgs = collate_detection([ds[i] for i in range(6)])
    r = evaluate_release(m, ims, tgs, batch_size=4, warmup=1)
    assert set(r) == {"o2m-nms"} and {"mAP", "AP50"} <= set(r["o2m-nms"]["metrics"])
    assert r["o2m-nms"]["timing"]["images_per_second"] > 0
