"""Grouped ``cfb`` subcommands: ``cfb <group> <command> [flags]``.

The group / command names follow the reference's typer tree
(complexity/cli/commands/{train,inference,tokenize,profile,convert,serve,
info}.py plus ``quickstart`` and ``shell``); the flat commands of ``app.py``
stay as aliases.  Every command runs this framework's components.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path
from typing import Callable, Dict, List, Optional

import torch

from . import app as flat


def _emit(obj) -> None:
    print(json.dumps(obj, indent=2, default=str))


# ------------------------------------------------------------------- train
def _train_run(argv: List[str]) -> None:
    flat.cmd_train(argv)


def _train_resume(argv: List[str]) -> None:
    if "--resume" not in argv:
        argv = argv + ["--resume", "auto"]
    flat.cmd_train(argv)


def _train_validate(argv: List[str]) -> None:
    """Check a run config (YAML/JSON) or model config: parse, build the model on
    the meta device, report parameter count and tokens per step."""
    p = argparse.ArgumentParser(prog="cfb train validate")
    p.add_argument("config")
    a = p.parse_args(argv)
    import yaml

    from ..config.model_config import ModelConfig
    from ..models.builder import ComplexityModel

    path = Path(a.config)
    text = path.read_text()
    data = yaml.safe_load(text) if path.suffix in (".yaml", ".yml") else json.loads(text)
    mc = data.get("model_config", data)
    cfg = ModelConfig.from_dict(mc) if "hidden_size" in mc else None
    out = {"config": str(path), "valid": True}
    if cfg is not None:
        with torch.device("meta"):
            m = ComplexityModel(cfg)
        out["parameters"] = sum(p.numel() for p in m.parameters())
    for k in ("batch_size", "seq_len", "gradient_accumulation", "world_size"):
        if k in data:
            out[k] = data[k]
    _emit(out)


def _train_create_config(argv: List[str]) -> None:
    """Write a YAML run config with the TrainRunner defaults (edit, then
    ``cfb train run --config FILE``)."""
    p = argparse.ArgumentParser(prog="cfb train create-config")
    p.add_argument("output")
    p.add_argument("--model", default="tr-hash-200m")
    a = p.parse_args(argv)
    import yaml

    from ..training.runner import TrainRunner

    parser = TrainRunner().build_parser()
    defaults = {act.dest: act.default for act in parser._actions
                if act.dest not in ("help", "config") and act.default is not argparse.SUPPRESS}
    defaults["model"] = a.model
    Path(a.output).write_text(yaml.safe_dump(defaults, sort_keys=True))
    _emit({"written": a.output, "keys": len(defaults)})


# --------------------------------------------------------------- inference
def _model_parser(prog: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog=prog)
    p.add_argument("--model", required=True, help="checkpoint dir or preset name")
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--device", default=None)
    return p


def _inference_batch(argv: List[str]) -> None:
    """Prompts from a text file (one per line) or JSONL (``prompt`` field) ->
    JSONL of completions, all requests in one continuous batch."""
    p = _model_parser("cfb inference batch")
    p.add_argument("--input", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--max-new-tokens", type=int, default=64)
    p.add_argument("--temperature", type=float, default=0.0)
    a = p.parse_args(argv)
    from ..inference.engine import GenerationConfig, InferenceEngine

    dev = flat._device(a.device)
    model, tok = flat._load_model(a.model, dev), flat._tokenizer(a.tokenizer)
    lines = [l for l in Path(a.input).read_text().splitlines() if l.strip()]
    prompts = [json.loads(l)["prompt"] if a.input.endswith(".jsonl") else l for l in lines]
    gen = GenerationConfig(max_new_tokens=a.max_new_tokens, do_sample=a.temperature > 0,
                           temperature=a.temperature if a.temperature > 0 else 1.0,
                           eos_token_id=tok.eos_token_id)
    t0 = time.perf_counter()
    outs = InferenceEngine(model).generate_tokens([tok.encode(x) for x in prompts], gen)
    dt = time.perf_counter() - t0
    with open(a.output, "w") as fh:
        for pr, o in zip(prompts, outs):
            fh.write(json.dumps({"prompt": pr, "completion": tok.decode(o)}) + "\n")
    _emit({"requests": len(prompts), "seconds": round(dt, 3),
           "tokens_per_s": round(sum(map(len, outs)) / max(dt, 1e-9), 1)})


# ---------------------------------------------------------------- tokenize
def _tok_from(argv_tok: Optional[str]):
    return flat._tokenizer(argv_tok)


def _tokenize_encode(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize encode")
    p.add_argument("text")
    p.add_argument("--tokenizer", default=None)
    a = p.parse_args(argv)
    _emit({"ids": _tok_from(a.tokenizer).encode(a.text)})


def _tokenize_decode(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize decode")
    p.add_argument("ids", nargs="+", type=int)
    p.add_argument("--tokenizer", default=None)
    a = p.parse_args(argv)
    _emit({"text": _tok_from(a.tokenizer).decode(a.ids)})


def _tokenize_count(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize count")
    p.add_argument("input", nargs="+")
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--text-key", default="text")
    a = p.parse_args(argv)
    from ..data.streaming import iter_texts

    tok = _tok_from(a.tokenizer)
    docs = toks = chars = 0
    for t in iter_texts(a.input, a.text_key):
        docs += 1
        chars += len(t)
        toks += len(tok.encode(t))
    _emit({"documents": docs, "tokens": toks, "characters": chars,
           "chars_per_token": round(chars / max(toks, 1), 3)})


def _tokenize_info(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize info")
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--shard", default=None, help="token shard directory")
    a = p.parse_args(argv)
    tok = _tok_from(a.tokenizer)
    out = {"tokenizer": type(tok).__name__, "vocab_size": tok.vocab_size,
           "eos_token_id": tok.eos_token_id,
           "bos_token_id": getattr(tok, "bos_token_id", None),
           "pad_token_id": getattr(tok, "pad_token_id", None)}
    if a.shard:
        from ..data.token_shards import read_token_shard_metadata

        out["shard"] = read_token_shard_metadata(a.shard)
    _emit(out)


def _tokenize_special_tokens(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize special-tokens")
    p.add_argument("--tokenizer", default=None)
    a = p.parse_args(argv)
    from ..data.tokenization import ChatTemplate

    tok = _tok_from(a.tokenizer)
    names = {k: getattr(tok, k) for k in dir(tok) if k.endswith("_token_id")
             and not callable(getattr(tok, k))}
    tmpl = ChatTemplate("complexity")
    _emit({"ids": names, "chat_markers": getattr(tmpl, "special_tokens", None)})


def _tokenize_preprocess(argv: List[str]) -> None:
    """Texts (txt / jsonl) -> a token shard (``tokens.bin`` + index)."""
    p = argparse.ArgumentParser(prog="cfb tokenize preprocess")
    p.add_argument("--input", nargs="+", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--text-key", default="text")
    flat.cmd_tokenize(p.parse_args(argv))


def _tokenize_train(argv: List[str], kind: str = "bpe") -> None:
    """Train a byte-level BPE (``tokenizers``) or a sentencepiece model on texts."""
    p = argparse.ArgumentParser(prog=f"cfb tokenize train{'-sentencepiece' if kind == 'sp' else ''}")
    p.add_argument("--input", nargs="+", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--vocab-size", type=int, default=32000)
    p.add_argument("--text-key", default="text")
    p.add_argument("--special", nargs="*", default=["<|endoftext|>", "<|pad|>"])
    a = p.parse_args(argv)
    from ..data.streaming import iter_texts

    out = Path(a.output)
    out.mkdir(parents=True, exist_ok=True)
    if kind == "sp":
        import sentencepiece as spm

        corpus = out / "corpus.txt"
        with open(corpus, "w") as fh:
            for t in iter_texts(a.input, a.text_key):
                fh.write(t.replace("\n", " ") + "\n")
        spm.SentencePieceTrainer.train(input=str(corpus), model_prefix=str(out / "tokenizer"),
                                       vocab_size=a.vocab_size, character_coverage=1.0,
                                       user_defined_symbols=a.special)
        _emit({"model": str(out / "tokenizer.model"), "vocab_size": a.vocab_size})
        return
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    t = Tokenizer(models.BPE())
    t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    t.decoder = decoders.ByteLevel()
    tr = trainers.BpeTrainer(vocab_size=a.vocab_size, special_tokens=a.special,
                             initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    t.train_from_iterator(iter_texts(a.input, a.text_key), tr)
    t.save(str(out / "tokenizer.json"))
    _emit({"tokenizer": str(out / "tokenizer.json"), "vocab_size": t.get_vocab_size()})


def _tokenize_extend(argv: List[str]) -> None:
    """Add tokens to a ``tokenizers`` JSON tokenizer (e.g. chat markers)."""
    p = argparse.ArgumentParser(prog="cfb tokenize extend")
    p.add_argument("tokenizer_json")
    p.add_argument("--tokens", nargs="+", required=True)
    p.add_argument("--special", action="store_true")
    p.add_argument("--output", default=None)
    a = p.parse_args(argv)
    from tokenizers import AddedToken, Tokenizer

    t = Tokenizer.from_file(a.tokenizer_json)
    before = t.get_vocab_size()
    toks = [AddedToken(x, special=a.special) for x in a.tokens]
    (t.add_special_tokens if a.special else t.add_tokens)(toks)
    t.save(a.output or a.tokenizer_json)
    _emit({"before": before, "after": t.get_vocab_size()})


def _tokenize_merge(argv: List[str]) -> None:
    """Concatenate token shards into one (same dtype)."""
    p = argparse.ArgumentParser(prog="cfb tokenize merge")
    p.add_argument("shards", nargs="+")
    p.add_argument("--output", required=True)
    a = p.parse_args(argv)
    from ..data.token_shards import load_token_shard, write_token_shard

    vocab = None

    def stream():
        nonlocal vocab
        for s in a.shards:
            arr, meta = load_token_shard(s)
            vocab = max(vocab or 0, int(meta.get("vocab_size") or 0)) or None
            step = 1 << 22
            for i in range(0, arr.size, step):
                yield arr[i:i + step]

    chunks = list(stream())
    idx = write_token_shard(a.output, iter(chunks), vocab_size=vocab)
    _emit(json.loads(Path(idx).read_text()))


def _tokenize_benchmark(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb tokenize benchmark")
    p.add_argument("input", nargs="+")
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--text-key", default="text")
    a = p.parse_args(argv)
    from ..data.streaming import iter_texts

    tok = _tok_from(a.tokenizer)
    texts = list(iter_texts(a.input, a.text_key))
    t0 = time.perf_counter()
    n = sum(len(tok.encode(t)) for t in texts)
    dt = time.perf_counter() - t0
    _emit({"documents": len(texts), "tokens": n, "tokens_per_s": round(n / max(dt, 1e-9))})


# ----------------------------------------------------------------- profile
def _profile_gpu(argv: List[str]) -> None:
    """Device properties, the extension, and the measured peaks used as roofline
    denominators."""
    from ..ops._ext import available
    from ..profiling.timing import load_measured_peaks

    out = {"cuda_available": torch.cuda.is_available(), "extension_loaded": available(),
           "measured_peaks": load_measured_peaks()}
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            pr = torch.cuda.get_device_properties(i)
            out[f"gpu{i}"] = {"name": pr.name, "sm": f"{pr.major}.{pr.minor}",
                              "sms": pr.multi_processor_count,
                              "memory_gb": round(pr.total_memory / 1e9, 1)}
    _emit(out)


def _profile_attention(argv: List[str]) -> None:
    from ..profiling.kernel_cases import main as kc

    kc(["flash"] + argv)


# -------------------------------------------------------------------- serve
def _serve_benchmark(argv: List[str]) -> None:
    """Concurrent completions against a running OpenAI-compatible server."""
    p = argparse.ArgumentParser(prog="cfb serve benchmark-server")
    p.add_argument("--url", default="http://127.0.0.1:8000")
    p.add_argument("--requests", type=int, default=32)
    p.add_argument("--concurrency", type=int, default=8)
    p.add_argument("--max-tokens", type=int, default=32)
    p.add_argument("--prompt", default="Hello")
    a = p.parse_args(argv)
    from concurrent.futures import ThreadPoolExecutor

    import requests

    def one(i):
        t0 = time.perf_counter()
        r = requests.post(f"{a.url}/v1/completions", json={
            "prompt": f"{a.prompt} {i}", "max_tokens": a.max_tokens}, timeout=300)
        r.raise_for_status()
        usage = r.json().get("usage", {})
        return time.perf_counter() - t0, usage.get("completion_tokens", a.max_tokens)

    t0 = time.perf_counter()
    with ThreadPoolExecutor(a.concurrency) as ex:
        res = list(ex.map(one, range(a.requests)))
    wall = time.perf_counter() - t0
    lat = sorted(r[0] for r in res)
    _emit({"requests": a.requests, "wall_s": round(wall, 3),
           "completion_tokens_per_s": round(sum(r[1] for r in res) / wall, 1),
           "latency_p50_s": round(lat[len(lat) // 2], 4),
           "latency_p90_s": round(lat[int(len(lat) * 0.9) - 1], 4)})


def _serve_proxy(argv: List[str]) -> None:
    """OpenAI-compatible endpoint that forwards to an external backend
    (another server of this framework, vLLM, ...)."""
    p = argparse.ArgumentParser(prog="cfb serve openai-proxy")
    p.add_argument("--backend", required=True, help="base URL of the upstream server")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8001)
    a = p.parse_args(argv)
    import uvicorn
    from fastapi import FastAPI, Request

    from ..inference.server import ExternalBackend

    up = ExternalBackend(a.backend)
    api = FastAPI()

    def _extra(body, skip):
        return {k: v for k, v in body.items() if k not in (skip, "model", "stream")}

    @api.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        text = up.complete(body.get("prompt", ""), **_extra(body, "prompt"))
        return {"object": "text_completion", "model": body.get("model", "proxy"),
                "choices": [{"index": 0, "text": text, "finish_reason": "stop"}]}

    @api.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        text = up.chat(body.get("messages", []), **_extra(body, "messages"))
        return {"object": "chat.completion", "model": body.get("model", "proxy"),
                "choices": [{"index": 0, "finish_reason": "stop",
                             "message": {"role": "assistant", "content": text}}]}

    uvicorn.run(api, host=a.host, port=a.port)


# --------------------------------------------------------------------- info
def _info_version(argv: List[str]) -> None:
    from .. import __version__

    _emit({"complexity_framework_b200": __version__, "torch": torch.__version__,
           "cuda": torch.version.cuda})


def _info_model(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb info model")
    p.add_argument("model", help="checkpoint dir or preset name")
    a = p.parse_args(argv)
    from ..config.model_config import ModelConfig, get_preset
    from ..models.builder import ComplexityModel

    path = Path(a.model)
    cfg = (ModelConfig.from_dict(json.loads((path / "config.json").read_text()))
           if path.exists() else get_preset(a.model))
    with torch.device("meta"):
        m = ComplexityModel(cfg)
    n = sum(p.numel() for p in m.parameters())
    _emit({"parameters": n, "layers": cfg.num_hidden_layers, "hidden": cfg.hidden_size,
           "heads": [cfg.num_attention_heads, cfg.num_key_value_heads],
           "experts": cfg.num_experts, "top_k": cfg.top_k, "vocab": cfg.vocab_size,
           "bf16_gb": round(2 * n / 1e9, 2)})


def _info_config(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb info config")
    p.add_argument("model", help="checkpoint dir, config.json or preset name")
    a = p.parse_args(argv)
    from ..config.model_config import get_preset

    path = Path(a.model)
    if path.is_dir():
        path = path / "config.json"
    _emit(json.loads(path.read_text()) if path.exists() else get_preset(a.model).to_dict())


def _info_tokens(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb info tokens")
    p.add_argument("shard")
    a = p.parse_args(argv)
    from ..data.token_shards import read_token_shard_metadata

    _emit(read_token_shard_metadata(a.shard))


def _info_env(argv: List[str]) -> None:
    import platform

    from ..ops._ext import available

    out = {"python": platform.python_version(), "torch": torch.__version__,
           "cuda": torch.version.cuda, "cuda_available": torch.cuda.is_available(),
           "extension_loaded": available(),
           "nccl": (".".join(map(str, torch.cuda.nccl.version()))
                    if torch.cuda.is_available() else None),
           "gpus": torch.cuda.device_count()}
    _emit(out)


# ---------------------------------------------------------- quickstart/shell
def _quickstart(argv: List[str]) -> None:
    """Tiny model, a few training steps on built-in text, then generation."""
    p = argparse.ArgumentParser(prog="cfb quickstart")
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--output", default=None)
    a = p.parse_args(argv)
    from ..api import Model

    m = Model.from_preset("tiny", hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                          num_key_value_heads=2, intermediate_size=128,
                          shared_intermediate_size=256)
    texts = ["The quick brown fox jumps over the lazy dog."] * 64
    out = m.train(texts, steps=a.steps, batch_size=4, seq_len=64)
    sample = m.generate("The quick", max_new_tokens=16)
    if a.output:
        m.save(a.output)
    _emit({"trained_steps": out.get("steps"), "sample": sample, "saved": a.output})


def _shell(argv: List[str]) -> None:
    """Interactive prompt -> completion loop (empty line exits)."""
    p = _model_parser("cfb shell")
    p.add_argument("--max-new-tokens", type=int, default=64)
    a = p.parse_args(argv)
    from ..inference.engine import GenerationConfig, InferenceEngine

    dev = flat._device(a.device)
    model, tok = flat._load_model(a.model, dev), flat._tokenizer(a.tokenizer)
    eng = InferenceEngine(model)
    gen = GenerationConfig(max_new_tokens=a.max_new_tokens, eos_token_id=tok.eos_token_id)
    for line in sys.stdin:
        line = line.rstrip("\n")
        if not line:
            break
        print(tok.decode(eng.generate_tokens([tok.encode(line)], gen)[0]), flush=True)


def _flat(name: str) -> Callable[[List[str]], None]:
    def run(argv: List[str]) -> None:
        flat.run_flat([name] + argv)
    return run


def _flat_kind(name: str, kind: str) -> Callable[[List[str]], None]:
    def run(argv: List[str]) -> None:
        flat.run_flat([name, kind] + argv)
    return run


GROUPS: Dict[str, Dict[str, Callable[[List[str]], None]]] = {
    "train": {"run": _train_run, "resume": _train_resume, "validate": _train_validate,
              "create-config": _train_create_config},
    "inference": {"generate": _flat("generate"), "chat": _flat("chat"),
                  "batch": _inference_batch, "benchmark": _flat("bench-infer")},
    "tokenize": {"train": _tokenize_train,
                 "train-sentencepiece": lambda argv: _tokenize_train(argv, "sp"),
                 "extend": _tokenize_extend, "merge": _tokenize_merge,
                 "encode": _tokenize_encode, "decode": _tokenize_decode,
                 "count": _tokenize_count, "preprocess": _tokenize_preprocess,
                 "info": _tokenize_info, "special-tokens": _tokenize_special_tokens,
                 "benchmark": _tokenize_benchmark},
    "profile": {"model": _flat_kind("profile", "model"), "gpu": _profile_gpu,
                "throughput": _flat_kind("profile", "throughput"),
                "attention": _profile_attention, "kernels": _flat_kind("profile", "kernels")},
    "convert": {k: _flat_kind("convert", k) for k in
                ("to-gguf", "to-safetensors", "from-hf", "to-hf", "quantize", "token-routed",
                 "multi-hash", "expand-experts")},
    "serve": {"start": _flat("serve"), "benchmark-server": _serve_benchmark,
              "openai-proxy": _serve_proxy},
    "info": {"version": _info_version, "model": _info_model, "config": _info_config,
             "tokens": _info_tokens, "benchmark-env": _info_env},
}
def _launch(argv: List[str]) -> None:
    """``cfb launch --gpus N [--nodes M ...] [--supervise ...] -- <TrainRunner flags>``."""
    if "--" in argv:
        i = argv.index("--")
        own, runner = argv[:i], argv[i + 1:]
    else:
        own, runner = argv, []
    p = argparse.ArgumentParser(prog="cfb launch")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--nodes", type=int, default=1)
    p.add_argument("--node-rank", type=int, default=0)
    p.add_argument("--master-addr", default="127.0.0.1")
    p.add_argument("--master-port", type=int, default=29500)
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--supervise", action="store_true")
    p.add_argument("--progress-file", default=None)
    p.add_argument("--stall-seconds", type=float, default=900.0)
    p.add_argument("--max-restarts", type=int, default=3)
    a = p.parse_args(own)
    from ..launch import launch

    code = launch(runner, a.gpus, a.nodes, a.node_rank, a.master_addr, a.master_port,
                  a.dry_run, a.supervise, a.progress_file, a.stall_seconds, a.max_restarts)
    if code:
        raise SystemExit(code)


def _supervise(argv: List[str]) -> None:
    """``cfb supervise --progress-file F [--stall-seconds S] -- <command>``."""
    i = argv.index("--") if "--" in argv else len(argv)
    p = argparse.ArgumentParser(prog="cfb supervise")
    p.add_argument("--progress-file", default=None)
    p.add_argument("--stall-seconds", type=float, default=900.0)
    p.add_argument("--startup-grace", type=float, default=600.0)
    p.add_argument("--poll", type=float, default=30.0)
    p.add_argument("--max-restarts", type=int, default=3)
    a = p.parse_args(argv[:i])
    from ..launch import RunSupervisor, SupervisorConfig

    cfg = SupervisorConfig(argv[i + 1:], progress_file=a.progress_file,
                           stall_seconds=a.stall_seconds, startup_grace_seconds=a.startup_grace,
                           poll_seconds=a.poll, max_restarts=a.max_restarts)
    code = RunSupervisor(cfg).run()
    _emit({"exit_code": code, "events": cfg.events})
    if code:
        raise SystemExit(code)


def _data_replay_plan(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb data build-replay-plan")
    p.add_argument("mixture")
    p.add_argument("--phases", required=True,
                   help='JSON list: [{"name": .., "passes": 2, "fractions": {"web": 0.5}}]')
    p.add_argument("--row-alignment", type=int, default=512)
    p.add_argument("--output", required=True)
    a = p.parse_args(argv)
    from ..launch import build_replay_plan

    plan = build_replay_plan(a.mixture, json.loads(a.phases), a.row_alignment)
    Path(a.output).write_text(json.dumps(plan, indent=1))
    _emit({k: plan[k] for k in ("unique_tokens", "trained_tokens")})


def _data_verify(argv: List[str]) -> None:
    p = argparse.ArgumentParser(prog="cfb data verify")
    p.add_argument("path")
    a = p.parse_args(argv)
    from ..launch import verify_token_data

    r = verify_token_data(a.path)
    _emit(r)
    if not r["ok"]:
        raise SystemExit(1)


GROUPS["data"] = {"build-replay-plan": _data_replay_plan, "verify": _data_verify}
TOP = {"quickstart": _quickstart, "shell": _shell, "launch": _launch, "supervise": _supervise}


def dispatch(argv: List[str]) -> bool:
    """Run a grouped command; False when ``argv`` is not one (flat command)."""
    if argv and argv[0] in TOP:
        TOP[argv[0]](argv[1:])
        return True
    if len(argv) >= 2 and argv[0] in GROUPS and argv[1] in GROUPS[argv[0]]:
        GROUPS[argv[0]][argv[1]](argv[2:])
        return True
    if len(argv) == 2 and argv[0] in GROUPS and argv[1] in ("-h", "--help"):
        print(f"cfb {argv[0]} {{{','.join(GROUPS[argv[0]])}}} ...")
        return True
    return False
