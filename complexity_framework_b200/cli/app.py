"""``cfb`` command-line tool.

Counterpart of the typer app of complexity/cli (app.py + commands/train.py,
inference.py, serve.py, convert.py, tokenize.py, profile.py, info.py):

    cfb train [TrainRunner flags]            pretraining run
    cfb generate --model DIR --prompt TEXT   text generation (paged-KV engine)
    cfb chat --model DIR                     interactive chat
    cfb bench-infer --model DIR              decode throughput / TTFT
    cfb serve --model DIR --port 8000        OpenAI-compatible server
    cfb convert {to-gguf,to-safetensors,to-hf,from-hf,quantize,token-routed,
                 multi-hash,expand-experts} SRC DST
    cfb tokenize --input FILES --output DIR  build a token shard
    cfb profile {model,kernels,throughput}
    cfb plan [cluster plan flags]
    cfb info

Grouped form (``cli/groups.py``): ``cfb train {run,resume,validate,create-config}``,
``cfb inference {generate,chat,batch,benchmark}``, ``cfb tokenize {train,
train-sentencepiece,extend,merge,encode,decode,count,preprocess,info,special-tokens,
benchmark}``, ``cfb profile {model,gpu,throughput,attention,kernels}``,
``cfb convert {...}``, ``cfb serve {start,benchmark-server,openai-proxy}``,
``cfb info {version,model,config,tokens,benchmark-env}``, ``cfb quickstart``,
``cfb shell``.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path
from typing import List, Optional

import torch


def _device(arg: Optional[str]) -> torch.device:
    if arg:
        return torch.device(arg)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def _load_model(path: str, device: torch.device):
    from ..config.model_config import get_preset
    from ..models.builder import ComplexityModel

    p = Path(path)
    if p.exists():
        m = ComplexityModel.from_pretrained(p)
    else:
        m = ComplexityModel(get_preset(path))
    dt = torch.bfloat16 if device.type == "cuda" else torch.float32
    return m.to(device=device, dtype=dt).eval()


def _tokenizer(spec: Optional[str]):
    from ..data.tokenization import get_tokenizer

    if not spec or spec == "byte":
        return get_tokenizer("byte")
    p = Path(spec)
    if p.suffix == ".model":
        return get_tokenizer("sentencepiece", str(p))
    return get_tokenizer("huggingface", str(p))


# ------------------------------------------------------------------ commands
def cmd_train(argv: List[str]) -> None:
    from ..training.runner import TrainRunner

    TrainRunner().main(argv)


def cmd_generate(a) -> None:
    from ..inference.engine import GenerationConfig, InferenceEngine

    dev = _device(a.device)
    model, tok = _load_model(a.model, dev), _tokenizer(a.tokenizer)
    eng = InferenceEngine(model)
    gen = GenerationConfig(max_new_tokens=a.max_new_tokens, do_sample=a.temperature > 0,
                           temperature=a.temperature or 1.0, top_p=a.top_p, top_k=a.top_k,
                           eos_token_id=tok.eos_token_id, seed=a.seed)
    ids = tok.encode(a.prompt)
    if a.stream:
        for t in eng.generate_stream(ids, gen):
            print(tok.decode([t]), end="", flush=True)
        print()
    else:
        print(tok.decode(eng.generate_tokens([ids], gen)[0]))


def cmd_chat(a) -> None:
    from ..data.tokenization import ChatTemplate, Message
    from ..inference.engine import GenerationConfig, InferenceEngine

    dev = _device(a.device)
    model, tok = _load_model(a.model, dev), _tokenizer(a.tokenizer)
    eng, tpl = InferenceEngine(model), ChatTemplate(a.format)
    msgs = [Message("system", a.system)] if a.system else []
    for line in sys.stdin:
        msgs.append(Message("user", line.strip()))
        ids = tok.encode(tpl.apply(msgs, add_generation_prompt=True))
        out = eng.generate_tokens([ids], GenerationConfig(max_new_tokens=a.max_new_tokens,
                                                          eos_token_id=tok.eos_token_id))[0]
        reply = tok.decode(out)
        print(reply, flush=True)
        msgs.append(Message("assistant", reply))


def cmd_bench_infer(a) -> None:
    from ..inference.engine import GenerationConfig, InferenceEngine

    dev = _device(a.device)
    model = _load_model(a.model, dev)
    V = model.config.vocab_size
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, V, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    eng = InferenceEngine(model)
    gen = GenerationConfig(max_new_tokens=a.new_tokens)
    eng.generate_tokens(prompts[:1], GenerationConfig(max_new_tokens=2))  # warm-up
    if dev.type == "cuda":
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    rids = [eng.add_request(p, gen) for p in prompts]
    ttft = None
    while eng.has_pending():
        eng.step()
        if ttft is None and all(eng.requests[r].output for r in rids):
            ttft = time.perf_counter() - t0
    if dev.type == "cuda":
        torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    print(json.dumps({"batch": a.batch, "prompt_len": a.prompt_len, "new_tokens": a.new_tokens,
                      "decode_tok_s": a.batch * a.new_tokens / dt, "ttft_s": ttft,
                      "seconds": dt}))


def cmd_serve(a) -> None:
    from ..inference.server import serve

    dev = _device(a.device)
    serve(_load_model(a.model, dev), _tokenizer(a.tokenizer), host=a.host, port=a.port,
          model_name=Path(a.model).name)


def cmd_convert(a) -> None:
    from ..models.builder import ComplexityModel
    from ..utils import conversion as cv

    kind, src, dst = a.kind, a.src, Path(a.dst)
    if kind == "to-gguf":
        from ..quantization.gguf import GGUFQuantType, export_gguf

        export_gguf(ComplexityModel.from_pretrained(src), dst, GGUFQuantType[a.qtype])
    elif kind == "to-safetensors":
        from ..utils.security import safe_torch_load, save_safetensors

        sd = safe_torch_load(src)
        sd = sd.get("model", sd) if isinstance(sd, dict) else sd
        save_safetensors(sd, dst)
    elif kind == "to-hf":
        from ..integrations.hf import export_hf

        export_hf(ComplexityModel.from_pretrained(src), dst)
    elif kind == "from-hf":
        from safetensors.torch import load_file

        from ..config.model_config import ModelConfig

        cfg = json.loads((Path(src) / "config.json").read_text())
        mc = ModelConfig(hidden_size=cfg["hidden_size"], num_hidden_layers=cfg["num_hidden_layers"],
                         num_attention_heads=cfg["num_attention_heads"],
                         num_key_value_heads=cfg.get("num_key_value_heads"),
                         vocab_size=cfg["vocab_size"],
                         shared_intermediate_size=cfg["intermediate_size"],
                         max_position_embeddings=cfg.get("max_position_embeddings", 2048))
        m = ComplexityModel(mc)
        sd = cv.convert_hf_state_dict(load_file(str(Path(src) / "model.safetensors")))
        m.load_state_dict(sd, strict=False)
        m.save_pretrained(dst)
    elif kind == "quantize":
        from ..quantization import quantize_model

        m = quantize_model(ComplexityModel.from_pretrained(src), bits=a.bits,
                           method=a.method)
        dst.mkdir(parents=True, exist_ok=True)
        torch.save(m.state_dict(), dst / "quantized.pt")
    elif kind == "token-routed":
        cv.convert_token_routed_checkpoint_dir(src).save_pretrained(dst)
    elif kind == "multi-hash":
        cv.convert_checkpoint_dir_to_multi_hash(src).save_pretrained(dst)
    elif kind == "expand-experts":
        cv.convert_checkpoint_dir_to_expanded_experts(src).save_pretrained(dst)
    print(f"wrote {dst}")


def cmd_tokenize(a) -> None:
    from ..data.streaming import iter_texts
    from ..data.token_shards import write_token_shard

    tok = _tokenizer(a.tokenizer)

    def stream():
        for text in iter_texts(a.input, a.text_key):
            yield tok.encode(text) + ([tok.eos_token_id] if tok.eos_token_id is not None else [])

    idx = write_token_shard(a.output, stream(), vocab_size=tok.vocab_size,
                            tokenizer=a.tokenizer or "byte")
    print(json.dumps(json.loads(Path(idx).read_text())))


def cmd_profile(a) -> None:
    if a.what == "kernels":
        from ..profiling.kernel_cases import main as kc

        kc([a.case])
        return
    from ..profiling import FLOPSCounter, count_parameters, model_flops_per_token

    dev = _device(a.device)
    model = _load_model(a.model, dev)
    cfg = model.config
    if a.what == "model":
        f = model_flops_per_token(cfg, a.seq_len)
        print(json.dumps({"params": count_parameters(model),
                          "train_flops_per_token": f["total"],
                          "forward_flops_per_token": f["forward"]}))
        ids = torch.randint(0, cfg.vocab_size, (1, min(a.seq_len, 256)), device=dev)
        c = FLOPSCounter()
        print(c.count(model, ids))
    elif a.what == "throughput":
        from ..profiling import ThroughputBenchmark

        ids = torch.randint(0, cfg.vocab_size, (a.batch, a.seq_len), device=dev)
        with torch.no_grad():
            r = ThroughputBenchmark(lambda: model(ids), a.batch * a.seq_len).run()
        print(json.dumps(r))


def cmd_info(a) -> None:
    from .. import __version__
    from ..ops._ext import available

    info = {"framework": "complexity_framework_b200", "version": __version__,
            "torch": torch.__version__, "cuda_available": torch.cuda.is_available(),
            "extension_loaded": available()}
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        info.update(gpu=p.name, sm=f"{p.major}.{p.minor}", sms=p.multi_processor_count,
                    memory_gb=round(p.total_memory / 1e9, 1))
    print(json.dumps(info, indent=2))


# --------------------------------------------------------------- detection
def cmd_train_detector(a) -> None:
    """Train a TR-Hash detector on COCO-format data, YOLO labels, or synthetic
    shapes; evaluates the EMA model and writes a checkpoint directory."""
    from ..generative.detection import (AugmentedDataset, CocoDetectionDataset,
                                        DetectionAugment, DetectorTrainer,
                                        DetectorTrainingConfig, SyntheticShapesDataset,
                                        TRHashDetectorConfig, TRHashObjectDetector,
                                        YoloDetectionDataset, collate_detection,
                                        save_detector_checkpoint)

    if a.data == "synthetic":
        train = SyntheticShapesDataset(a.synthetic_images, a.image_size, 4, a.num_classes)
        val = SyntheticShapesDataset(max(16, a.synthetic_images // 8), a.image_size, 4,
                                     a.num_classes, seed=1)
    elif a.data == "coco":
        train = CocoDetectionDataset(a.annotations, a.images, a.image_size)
        val = CocoDetectionDataset(a.val_annotations or a.annotations,
                                   a.val_images or a.images, a.image_size)
    else:
        train = YoloDetectionDataset(a.images, a.labels, a.image_size)
        val = YoloDetectionDataset(a.val_images or a.images, a.val_labels or a.labels,
                                   a.image_size)
    if a.augment:
        train = AugmentedDataset(train, DetectionAugment(seed=a.seed))
    cfg = TRHashDetectorConfig(image_size=a.image_size, num_classes=a.num_classes,
                               backbone=a.backbone)
    dev = torch.device(a.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = TRHashObjectDetector(cfg).to(dev)
    trainer = DetectorTrainer(model, DetectorTrainingConfig(
        learning_rate=a.lr, max_steps=a.steps, warmup_steps=min(100, a.steps // 10)))
    dl = torch.utils.data.DataLoader(train, batch_size=a.batch, shuffle=True, drop_last=True,
                                     collate_fn=collate_detection, num_workers=a.workers)
    done = False
    while not done:
        for images, targets in dl:
            losses = trainer.train_step(images, targets)
            if trainer.step % a.log_every == 0:
                print(json.dumps({"step": trainer.step, **{k: round(v, 4) for k, v in losses.items()}}))
            if trainer.step >= a.steps:
                done = True
                break
    vl = torch.utils.data.DataLoader(val, batch_size=a.batch, collate_fn=collate_detection)
    print(json.dumps({"eval": trainer.evaluate(vl)}))
    save_detector_checkpoint(model, a.output, ema=trainer.ema)
    print(json.dumps({"saved": a.output}))


def cmd_detect(a) -> None:
    """Run a saved detector on image files; prints boxes in original-image pixels."""
    from torchvision.io import read_image

    from ..generative.detection import (load_detector_checkpoint, preprocess_detector_image,
                                        restore_detector_boxes)

    dev = torch.device(a.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = load_detector_checkpoint(a.checkpoint).to(dev)
    names = model.config.class_names
    for path in a.images:
        img = read_image(path).float()[:3] / 255.0
        x, meta = preprocess_detector_image(img, model.config.image_size)
        r = model.predict(x[None].to(dev), score_threshold=a.score)[0]
        boxes = restore_detector_boxes(r["boxes"].cpu(), meta)
        dets = [{"box": [round(float(v), 1) for v in b], "score": round(float(s), 4),
                 "label": (names[int(l)] if int(l) < len(names) else int(l))}
                for b, s, l in zip(boxes, r["scores"].cpu(), r["labels"].cpu())]
        print(json.dumps({"image": path, "detections": dets}))


# ------------------------------------------------------------------- parser
def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="cfb", description="complexity_framework_b200 CLI")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("train", help="pretraining run (TrainRunner flags follow)", add_help=False)

    def model_args(p):
        p.add_argument("--model", required=True, help="checkpoint dir or preset name")
        p.add_argument("--tokenizer", default=None)
        p.add_argument("--device", default=None)

    g = sub.add_parser("generate")
    model_args(g)
    g.add_argument("--prompt", required=True)
    g.add_argument("--max-new-tokens", type=int, default=64)
    g.add_argument("--temperature", type=float, default=0.0)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--top-k", type=int, default=0)
    g.add_argument("--seed", type=int, default=None)
    g.add_argument("--stream", action="store_true")
    c = sub.add_parser("chat")
    model_args(c)
    c.add_argument("--system", default=None)
    c.add_argument("--format", default="complexity", choices=["complexity", "chatml", "llama"])
    c.add_argument("--max-new-tokens", type=int, default=256)
    b = sub.add_parser("bench-infer")
    model_args(b)
    b.add_argument("--batch", type=int, default=32)
    b.add_argument("--prompt-len", type=int, default=512)
    b.add_argument("--new-tokens", type=int, default=128)
    s = sub.add_parser("serve")
    model_args(s)
    s.add_argument("--host", default="127.0.0.1")
    s.add_argument("--port", type=int, default=8000)
    cv = sub.add_parser("convert")
    cv.add_argument("kind", choices=["to-gguf", "to-safetensors", "to-hf", "from-hf", "quantize",
                                     "token-routed", "multi-hash", "expand-experts"])
    cv.add_argument("src")
    cv.add_argument("dst")
    cv.add_argument("--qtype", default="Q8_0", choices=["F32", "F16", "Q8_0"])
    cv.add_argument("--bits", type=int, default=8)
    cv.add_argument("--method", default="dynamic", choices=["dynamic", "fp8"])
    t = sub.add_parser("tokenize")
    t.add_argument("--input", nargs="+", required=True)
    t.add_argument("--output", required=True)
    t.add_argument("--tokenizer", default=None)
    t.add_argument("--text-key", default="text")
    pr = sub.add_parser("profile")
    pr.add_argument("what", choices=["model", "kernels", "throughput"])
    pr.add_argument("--model", default="tr-hash-200m")
    pr.add_argument("--case", default="gemm", choices=["gemm", "gemm_bn", "flash", "norms"])
    pr.add_argument("--seq-len", type=int, default=2048)
    pr.add_argument("--batch", type=int, default=1)
    pr.add_argument("--device", default=None)
    sub.add_parser("plan", help="cluster run plan (cluster_plan flags follow)", add_help=False)
    sub.add_parser("info")
    td = sub.add_parser("train-detector", help="train a TR-Hash object detector")
    td.add_argument("--data", choices=["synthetic", "coco", "yolo"], default="synthetic")
    td.add_argument("--images", default=None)
    td.add_argument("--annotations", default=None, help="COCO instances json")
    td.add_argument("--labels", default=None, help="YOLO label directory")
    td.add_argument("--val-images", default=None)
    td.add_argument("--val-annotations", default=None)
    td.add_argument("--val-labels", default=None)
    td.add_argument("--num-classes", type=int, default=2)
    td.add_argument("--image-size", type=int, default=320)
    td.add_argument("--backbone", choices=["plain", "hierarchical"], default="plain")
    td.add_argument("--synthetic-images", type=int, default=512)
    td.add_argument("--augment", action="store_true")
    td.add_argument("--batch", type=int, default=16)
    td.add_argument("--steps", type=int, default=1000)
    td.add_argument("--lr", type=float, default=1e-3)
    td.add_argument("--workers", type=int, default=0)
    td.add_argument("--log-every", type=int, default=50)
    td.add_argument("--seed", type=int, default=0)
    td.add_argument("--device", default=None)
    td.add_argument("--output", required=True)
    dt = sub.add_parser("detect", help="run a saved detector on images")
    dt.add_argument("--checkpoint", required=True)
    dt.add_argument("--score", type=float, default=0.25)
    dt.add_argument("--device", default=None)
    dt.add_argument("images", nargs="+")
    return ap


def main(argv: Optional[List[str]] = None) -> None:
    argv = list(sys.argv[1:] if argv is None else argv)
    from .groups import dispatch

    if dispatch(argv):  # cfb <group> <command> ... (train run, tokenize count, info env, ...)
        return
    run_flat(argv)


def run_flat(argv: List[str]) -> None:
    """Run one of the flat commands (``cfb convert to-gguf ...``); grouped
    commands that share a name with a flat one end here without re-dispatch."""
    if argv and argv[0] == "train":
        return cmd_train(argv[1:])
    if argv and argv[0] == "plan":
        from ..training.cluster_plan import main as plan

        return plan(argv[1:])
    a = build_parser().parse_args(argv)
    {"generate": cmd_generate, "chat": cmd_chat, "bench-infer": cmd_bench_infer,
     "serve": cmd_serve, "convert": cmd_convert, "tokenize": cmd_tokenize,
     "profile": cmd_profile, "info": cmd_info, "train-detector": cmd_train_detector,
     "detect": cmd_detect}[a.cmd](a)


if __name__ == "__main__":
    main()
