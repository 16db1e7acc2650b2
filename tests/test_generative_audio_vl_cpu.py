"""Audio front end / speech-to-text / text-to-speech and image-text-to-text (CPU)."""
import io
import tarfile

import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.generative.audio import (
    AudioEncoderConfig, LogMelSpectrogram, TRHashAudioConfig, TRHashSpeechToText,
    TRHashTextToSpeech, build_mel_filterbank)
from complexity_framework_b200.generative.towers import TRHashVisionTowerConfig
from complexity_framework_b200.generative.vision_language import (
    TRHashImageTextToText, TRHashVisionLanguageConfig, VisionLanguageTarDataset,
    collate_vision_language)


def _decoder():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2,
                                       vocab_size=256, intermediate_size=64,
                                       shared_intermediate_size=128, num_experts=4,
                                       max_position_embeddings=512))


def _enc():
    return AudioEncoderConfig(n_mels=32, max_frames=400, hidden_size=64, num_layers=1,
                              num_heads=4, shared_width=128, expert_width=32)


def test_mel_filterbank_and_tone_peak():
    fb = build_mel_filterbank(40, 512, 16000)
    assert fb.shape == (40, 257) and float(fb.min()) >= 0
    assert (fb.sum(1) > 0).all()  # every filter covers some bins
    t = torch.arange(16000) / 16000
    lo = LogMelSpectrogram(16000, 512, 160, 40)(torch.sin(2 * torch.pi * 300 * t)[None])
    hi = LogMelSpectrogram(16000, 512, 160, 40)(torch.sin(2 * torch.pi * 4000 * t)[None])
    assert int(lo.mean(-1).argmax()) < int(hi.mean(-1).argmax())


def _fit(model, step_fn, steps=25):
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], 3e-3)
    first = None
    for _ in range(steps):
        loss = step_fn()
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss)
    return first, float(loss)


def test_speech_to_text_fits_and_decodes():
    cfg = TRHashAudioConfig(n_fft=256, hop_length=128, encoder=_enc(), num_audio_tokens=8)
    m = TRHashSpeechToText(cfg, _decoder())
    audio = torch.randn(2, 8000)
    ids = torch.randint(1, 256, (2, 12))
    first, last = _fit(m, lambda: m(ids, audio=audio)["loss"])
    assert last < 0.5 * first
    out = m.transcribe(audio, bos_id=int(ids[0, 0]), max_new_tokens=4)
    assert out.shape == (2, 5)


def test_text_to_speech_fits():
    cfg = TRHashAudioConfig(encoder=_enc(), frames_per_token=3)
    m = TRHashTextToSpeech(cfg, _decoder())
    ids = torch.randint(0, 256, (2, 10))
    mel = torch.randn(2, 32, 30)
    first, last = _fit(m, lambda: m(ids, mel)["loss"])
    assert m(ids)["mel"].shape == (2, 32, 30)
    assert last < first


def test_image_text_to_text_and_tar_dataset(tmp_path):
    from PIL import Image

    vcfg = TRHashVisionTowerConfig(image_size=32, patch_size=8, hidden_size=64, num_layers=1,
                                   num_heads=4, shared_width=128, expert_width=32)
    m = TRHashImageTextToText(TRHashVisionLanguageConfig(vision=vcfg, num_visual_tokens=8),
                              _decoder())
    tar = tmp_path / "shard.tar"
    with tarfile.open(tar, "w") as tf:
        for k, colour in enumerate([(255, 0, 0), (0, 0, 255)]):
            buf = io.BytesIO()
            Image.new("RGB", (40, 40), colour).save(buf, format="PNG")
            for name, data in ((f"{k:04d}.png", buf.getvalue()),
                               (f"{k:04d}.txt", ("red" if k == 0 else "blue").encode())):
                info = tarfile.TarInfo(name)
                info.size = len(data)
                tf.addfile(info, io.BytesIO(data))

    class Bytes:
        def encode(self, s):
            return [1] + list(s.encode())

    ds = VisionLanguageTarDataset(str(tar), Bytes(), image_size=32)
    assert len(ds) == 2
    images, ids, labels = collate_vision_language([ds[0], ds[1]])
    assert images.shape == (2, 3, 32, 32) and (labels[0, 4:] == -100).all()
    first, last = _fit(m, lambda: m(images, ids, labels)["loss"], steps=40)
    assert last < 0.3 * first
    # the caption is decoded from the image
    out = m.generate(images[1:], torch.tensor([[1]]), max_new_tokens=4)
    assert bytes(out[0, 1:].tolist()) == b"blue"


def test_prefix_lm_cached_generation_matches_recompute():
    from complexity_framework_b200.generative.prefix_lm import PrefixLM

    torch.manual_seed(0)
    lm = PrefixLM(_decoder()).eval()
    prefix = torch.randn(2, 5, 64)
    bos = torch.tensor([[3], [7]])
    a = lm.generate(prefix, bos, max_new_tokens=6, use_cache=True)
    b = lm.generate(prefix, bos, max_new_tokens=6, use_cache=False)
    assert torch.equal(a, b)
