"""The high-level API namespaces (counterparts of the reference's complexity.api):
building blocks, helpers, small-budget tools, runtime facades, multimodal."""
import torch

from complexity_framework_b200 import api

TINY = dict(vocab_size=256, intermediate_size=128, shared_intermediate_size=128)


def test_block_factories_and_registry():
    x = torch.randn(2, 8, 64)
    for attn in (api.GQA(64, 4, 2), api.MHA(64, 4), api.MQA(64, 4),
                 api.Attention.create("sliding_window", hidden_size=64, num_heads=4,
                                      sliding_window=4),
                 api.CUDA.flash(64, 4)):
        assert attn(x).shape == x.shape
    ids = torch.randint(0, 256, (2, 8))
    moe = api.MLP.moe(64, num_experts=4, **TINY)
    assert moe(x, token_ids=ids).shape == x.shape
    assert api.Norm.rms(64)(x).shape == x.shape and api.Norm.layer(64)(x).shape == x.shape
    cos, sin = api.Position.rope(16, max_seq_len=32)(8)
    assert cos.shape == (8, 16)
    assert api.Position.alibi(4).bias(3, 5, "cpu", torch.float32).shape == (1, 4, 3, 5)
    blk = api.Block.moe(64, 4, num_experts=4, **TINY)
    out = blk(x, token_ids=ids)
    assert (out[0] if isinstance(out, tuple) else out).shape == x.shape

    @api.register("mlp", "my_test_mlp")
    class Mine(torch.nn.Module):
        def __init__(self, cfg):
            super().__init__()

    assert "my_test_mlp" in api.MLP_REGISTRY
    assert "gqa" in api.Attention.available()


def test_helpers():
    m = api.Mask.causal(4)
    assert m[0, 1] == float("-inf") and m[1, 0] == 0
    assert api.Mask.sliding_window(6, 2)[5, 3] == float("-inf")
    p = api.Mask.padding(torch.tensor([[1, 1, 0]]))
    assert p.shape == (1, 1, 1, 3) and p[0, 0, 0, 2] < -1e30
    c = api.KVCache.create(2)
    k = torch.randn(1, 2, 3, 4)
    c.update(0, k, k)
    c.update(0, k, k)
    assert c.seq_length == 6
    sw = api.SlidingWindowCache.create(1, window=4)
    sw.update(0, k, k)
    sw.update(0, k, k)
    assert sw.seq_length == 4
    logits = torch.tensor([[0.0, 5.0, 1.0]])
    assert api.Sampling.greedy(logits).item() == 1
    assert api.Sampling.top_k(logits, 1)[0, 0] == float("-inf")
    g = torch.Generator().manual_seed(0)
    assert api.Sampling.sample(logits, temperature=0.5, top_p=0.5, generator=g).item() == 1
    assert api.Tensors.repeat_kv(k, 2).shape == (1, 4, 3, 4)
    model = api.SmallModels.nano(256)
    api.Init.apply(model, "normal", std=0.01)
    assert "ComplexityModel" in api.Debug.model_summary(model, 1)
    assert api.Debug.count_params(model)["total"] == model.num_parameters()


def test_efficient_quantize_and_presets():
    lin = torch.nn.Linear(64, 32)
    q = api.Quantize.linear(lin, bits=8)
    x = torch.randn(4, 64)
    assert (q(x) - lin(x)).abs().max() < 0.1
    model = api.SmallModels.nano(256)
    ids = torch.randint(0, 256, (1, 16))
    before = model(ids)["logits"]
    api.Quantize.dynamic(model, bits=8)
    after = model(ids)["logits"]
    assert (before - after).abs().max() < 0.5
    s = api.Efficient.estimate_savings(api.SmallModels.nano(256), bits=4)
    assert s["ratio"].endswith("x")


def test_runtime_facades(tmp_path):
    tok = api.Tokenizer.load("byte")
    texts = [f"line number {i} of the corpus" for i in range(200)]
    ds = api.DataPipeline(tok, api.DataConfig(seq_len=32, batch_size=2)).filter(
        lambda t: "1" in t).map(str.upper).build(texts, tmp_path / "ds")
    model = api.SmallModels.nano(tok.vocab_size)
    tr = api.Trainer(model, api.TrainerConfig(max_steps=2, precision="fp32", warmup_steps=1,
                                              output_dir=str(tmp_path / "ck"), save_steps=100,
                                              extra={"skip_param_update_check": True}))
    out = tr.train(ds)
    assert out["steps"] == 2
    text = api.Generate.text(model, "hello", tok, max_new_tokens=4)
    assert isinstance(text, str)
    pieces = list(api.Generate.stream(model, "hi", tok, max_new_tokens=3))
    assert len(pieces) == 3


def test_multimodal_factories():
    v = api.Vision.encoder(image_size=32, patch_size=8, hidden_size=64, num_layers=1, num_heads=4)
    assert v(torch.randn(1, 3, 32, 32)).shape == (1, 17, 64)
    a = api.Audio.encoder(n_mels=16, hidden_size=64, num_layers=1, num_heads=4, max_frames=64)
    assert a(torch.randn(1, 8000)).shape[-1] == 64  # raw 16 kHz audio -> log-mel -> encoder
    f = api.Fusion.gated(64)
    assert isinstance(f, torch.nn.Module)
    r = api.Robot.model(num_classes=5)
    assert isinstance(r, torch.nn.Module)
