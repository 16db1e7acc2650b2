"""Quantization on CPU: layer round trips, GPTQ beats round-to-nearest, AWQ, GGUF file."""
import copy

import numpy as np
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.quantization import (AWQConfig, GGUFQuantType, GPTQConfig,
                                                    Linear4bit, Linear8bit, LinearFP8,
                                                    awq_quantize, compare_outputs, export_gguf,
                                                    gptq_quantize_model, quantize_model,
                                                    read_gguf_header)
from complexity_framework_b200.quantization.gguf import dequantize_q8_0, quantize_q8_0


def test_linear_layers_roundtrip():
    torch.manual_seed(0)
    lin = torch.nn.Linear(256, 64)
    x = torch.randn(8, 256)
    y = lin(x)
    for mod, tol in ((Linear8bit.from_linear(lin), 0.02), (Linear4bit.from_linear(lin, 64), 0.2),
                     (LinearFP8.from_linear(lin), 0.1)):
        err = (mod(x) - y).abs().max() / y.abs().max()
        assert float(err) < tol, (type(mod).__name__, float(err))


def _mlp():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(128, 256), torch.nn.GELU(), torch.nn.Linear(256, 64))


def test_gptq_better_than_rtn():
    """GPTQ minimises the layer-output error on its calibration distribution."""
    torch.manual_seed(0)
    lin = torch.nn.Linear(128, 64)
    mix = torch.randn(128, 128) / 8 + torch.eye(128)
    calib = [torch.randn(128, 128) @ mix * torch.linspace(0.1, 3, 128) for _ in range(4)]
    test = torch.randn(512, 128) @ mix * torch.linspace(0.1, 3, 128)
    ref = torch.nn.Sequential(lin)
    rtn = quantize_model(copy.deepcopy(ref), bits=4, group_size=32, exclude_layers=["none"])
    gq = gptq_quantize_model(copy.deepcopy(ref), calib, GPTQConfig(bits=4, group_size=32),
                             exclude=())
    e_rtn = compare_outputs(ref, rtn, test)["mse"]
    e_gq = compare_outputs(ref, gq, test)["mse"]
    assert e_gq < 0.95 * e_rtn, (e_gq, e_rtn)


def test_awq_runs_and_is_close():
    m = _mlp()
    calib = [torch.randn(64, 128) * torch.linspace(0.1, 3, 128)]
    q = awq_quantize(copy.deepcopy(m), calib, AWQConfig(bits=4, group_size=32), exclude=())
    assert compare_outputs(m, q, calib[0])["cosine"] > 0.98


def test_gguf_export(tmp_path):
    a = np.random.randn(4, 64).astype(np.float32)
    back = dequantize_q8_0(quantize_q8_0(a), a.size).reshape(a.shape)
    assert np.abs(back - a).max() < np.abs(a).max() / 100
    model = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                        num_key_value_heads=2, vocab_size=256,
                                        intermediate_size=64, shared_intermediate_size=128,
                                        num_experts=4, top_k=2, routing_strategy="modulo_cyclic"))
    p = export_gguf(model, tmp_path / "m.gguf", GGUFQuantType.Q8_0)
    h = read_gguf_header(p)
    assert h["magic"] == 0x46554747 and h["version"] == 3 and h["n_tensors"] > 10


def test_gguf_tensor_infos_match_written_header(tmp_path):
    import struct

    from complexity_framework_b200.quantization import GGUFQuantType, GGUFTensorInfo, GGUFWriter

    w = GGUFWriter(tmp_path / "m.gguf")
    w.add_tensor("a", torch.randn(3, 5), GGUFQuantType.F32)     # 60 bytes -> 64
    w.add_tensor("b", torch.randn(2, 64), GGUFQuantType.Q8_0)
    infos = w.tensor_infos()
    assert infos[0] == GGUFTensorInfo("a", [5, 3], GGUFQuantType.F32, 0)
    assert infos[1].offset == 64 and infos[1].dims == [64, 2]
    raw = w.write().read_bytes()
    # the "a" tensor info in the header: name, ndims, dims, type, offset
    i = raw.index(struct.pack("<Q", 1) + b"a")
    nd, d0, d1, t, off = struct.unpack_from("<IQQIQ", raw, i + 9)
    assert (nd, d0, d1, t, off) == (2, 5, 3, 0, 0)
