"""Multimodal encoders and the vision-language model on CPU."""
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.multimodal.encoders import (AudioEncoder, EncoderConfig, VideoEncoder,
                                                           VisionEncoder)
from complexity_framework_b200.multimodal.fusion import VisionLanguageModel


def test_encoders_shapes():
    cfg = EncoderConfig(hidden_size=64, num_layers=2, num_heads=4, num_experts=2)
    v = VisionEncoder(cfg, image_size=32, patch_size=8)
    assert v(torch.randn(2, 3, 32, 32)).shape == (2, 17, 64)
    a = AudioEncoder(cfg, n_mels=16, max_frames=200)
    assert a(torch.randn(2, 16000 // 2)).shape[0] == 2
    vid = VideoEncoder(cfg, frames=4, image_size=32, patch_size=8, tubelet=2)
    assert vid(torch.randn(1, 3, 4, 32, 32)).shape == (1, 32, 64)


def test_vlm_trains():
    torch.manual_seed(0)
    lm = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                     num_key_value_heads=2, vocab_size=128, intermediate_size=64,
                                     shared_intermediate_size=128, num_experts=4, top_k=2,
                                     routing_strategy="modulo_cyclic", max_position_embeddings=64))
    vlm = VisionLanguageModel(lm, VisionEncoder(EncoderConfig(hidden_size=32, num_layers=1,
                                                              num_heads=4), 16, 8),
                              resampler_latents=4)
    ids = torch.randint(0, 128, (2, 10))
    img = torch.randn(2, 3, 16, 16)
    opt = torch.optim.AdamW(vlm.parameters(), lr=3e-3)
    l0 = None
    for _ in range(5):
        loss = vlm.loss(ids, img)
        opt.zero_grad()
        loss.backward()
        opt.step()
        l0 = l0 or float(loss)
    assert float(loss) < l0
