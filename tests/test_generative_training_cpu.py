"""Vision-tower pretraining and image-text-to-text training drivers on CPU."""
import io
import json
import tarfile

import pytest
import torch

from complexity_framework_b200.generative.vision_pretraining import (ResumableBatchSampler,
                                                                     VisionPretrainConfig,
                                                                     pretrain_vision_tower)
from complexity_framework_b200.generative.vlm_training import (PromptResponseTarDataset,
                                                               VLMTrainConfig,
                                                               collate_prompt_response,
                                                               prune_checkpoints, stage_is_sft,
                                                               tokenize_prompt_response,
                                                               train_vlm)

TOWER = dict(image_size=32, patch_size=8, hidden_size=32, num_layers=1, num_heads=2,
             shared_width=64, expert_width=32)


def test_resumable_batch_sampler_skips_by_index():
    s = ResumableBatchSampler(20, 4, seed=3, rank=1, world=2)
    s.set_epoch(2)
    full = list(s)
    s.set_epoch(2, skip=1)
    assert list(s) == full[1:] and len(s) == len(full) - 1
    s0 = ResumableBatchSampler(20, 4, seed=3, rank=0, world=2)
    s0.set_epoch(2)
    mine = {i for b in full for i in b}
    other = {i for b in s0 for i in b}
    assert not mine & other


def _vcfg(tmp, **kw):
    base = dict(synthetic=True, synthetic_train=64, synthetic_val=32, num_classes=4,
                tower=TOWER, epochs=3, batch_size=16, learning_rate=3e-3, warmup_steps=2,
                bf16=False, num_workers=0, output=str(tmp), device="cpu")
    base.update(kw)
    return VisionPretrainConfig(**base)


def test_vision_pretraining_learns_and_resumes(tmp_path):
    s = pretrain_vision_tower(_vcfg(tmp_path / "a"))
    assert s["steps"] == 3 * 4
    assert s["history"][-1]["train_loss"] < s["history"][0]["train_loss"]
    assert (tmp_path / "a" / "best" / "tower.pt").exists()
    # two epochs, then resume to three: same weights as the straight run
    pretrain_vision_tower(_vcfg(tmp_path / "b", epochs=3))
    import complexity_framework_b200.generative.vision_pretraining as mod

    real = mod.validate
    calls = {"n": 0}

    def stop(model, loader, ctx):
        calls["n"] += 1
        if calls["n"] == 3:
            raise KeyboardInterrupt
        return real(model, loader, ctx)

    mod.validate = stop
    try:
        with pytest.raises(KeyboardInterrupt):
            pretrain_vision_tower(_vcfg(tmp_path / "c", epochs=3))
    finally:
        mod.validate = real
    pretrain_vision_tower(_vcfg(tmp_path / "c", epochs=3, resume=True))
    a = torch.load(tmp_path / "b" / "last" / "classifier.pt")
    b = torch.load(tmp_path / "c" / "last" / "classifier.pt")
    assert all(torch.allclose(a[k], b[k], atol=1e-6) for k in a)


class ByteTok:
    pad_token_id = 0
    eos_token_id = 1

    def encode(self, text):
        return [2 + (b % 200) for b in text.encode()]


def test_prompt_response_labels_and_stages():
    ids, lab = tokenize_prompt_response(ByteTok(), ["ab", "abcd"], ["xy", "z"], 16)
    assert ids.shape == (2, 6)
    assert lab[0].tolist()[:2] == [-100, -100] and lab[0, 2:5].tolist() == ids[0, 2:5].tolist()
    assert lab[0, 4] == 1 and lab[0, 5:].tolist() == [-100]   # EOS learned, pad masked
    assert lab[1, :4].tolist() == [-100] * 4 and lab[1, 5] == 1
    assert [stage_is_sft(s, total_steps=10, sft_steps=3) for s in (6, 7, 9)] == [False, True, True]


def _vlm():
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.generative.towers import TRHashVisionTowerConfig
    from complexity_framework_b200.generative.vision_language import (TRHashImageTextToText,
                                                                      TRHashVisionLanguageConfig)

    torch.manual_seed(0)
    dec = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                      num_key_value_heads=2, vocab_size=256, intermediate_size=64,
                                      shared_intermediate_size=128, num_experts=2, top_k=2,
                                      max_position_embeddings=64))
    return TRHashImageTextToText(TRHashVisionLanguageConfig(
        vision=TRHashVisionTowerConfig(**TOWER), num_visual_tokens=4), dec)


def _shard(path, n=6):
    from PIL import Image

    with tarfile.open(path, "w") as tf:
        for i in range(n):
            for name, data in ((f"s{i}.png", None), (f"s{i}.txt", f"colour {i % 3}".encode()),
                               (f"s{i}.prompt", b"what colour?") if i % 2 else (None, None)):
                if name is None:
                    continue
                if data is None:
                    buf = io.BytesIO()
                    Image.new("RGB", (40, 40), (80 * (i % 3), 40, 200)).save(buf, format="PNG")
                    data = buf.getvalue()
                info = tarfile.TarInfo(name)
                info.size = len(data)
                tf.addfile(info, io.BytesIO(data))


def test_vlm_training_stages_checkpoints_and_resume(tmp_path):
    _shard(tmp_path / "a.tar")
    ds = PromptResponseTarDataset(str(tmp_path / "a.tar"), image_size=32)
    assert len(ds) == 6 and ds[0][1] == "Describe the image." and ds[1][1] == "what colour?"
    batches = list(torch.utils.data.DataLoader(ds, batch_size=3,
                                               collate_fn=collate_prompt_response))
    m = _vlm()
    dec_before = m.lm.decoder.embed_tokens.weight.detach().clone()
    cfg = VLMTrainConfig(max_steps=6, sft_steps=2, save_steps=2, keep_checkpoints=2,
                         log_steps=1, bf16=False, learning_rate=3e-3, warmup_steps=1,
                         output=str(tmp_path / "run"))
    s = train_vlm(m, ByteTok(), batches, cfg)
    assert s["steps"] == 6 and s["frozen"]["frozen"] > 0
    assert [e["stage"] for e in s["log"]] == ["alignment"] * 4 + ["sft"] * 2
    assert s["log"][-1]["loss"] < s["log"][0]["loss"]
    assert sorted(p.name for p in (tmp_path / "run").glob("step_*")) == ["step_0000004",
                                                                         "step_0000006"]
    assert not torch.equal(dec_before, m.lm.decoder.embed_tokens.weight)
    # resume continues from the newest checkpoint
    cfg2 = VLMTrainConfig(**{**cfg.__dict__, "max_steps": 8, "resume": True})
    s2 = train_vlm(_vlm(), ByteTok(), batches, cfg2)
    assert s2["steps"] == 8 and s2["log"][0]["step"] == 7
    with pytest.raises(ValueError):
        prune_checkpoints(tmp_path / "run", 0)


# ------------------------------------------------------------ image models
def _img_cfg(cls, **kw):
    base = dict(image_size=32, hidden_size=32, num_layers=1, num_heads=2, shared_width=64,
                expert_width=32, text_vocab_size=256, text_dim=32, cond_drop_prob=0.2)
    base.update(kw)
    return cls(**base)


def test_edit_condition_dropout_is_joint():
    from complexity_framework_b200.generative.image import sample_edit_condition_dropout

    g = torch.Generator().manual_seed(0)
    dt, ds = sample_edit_condition_dropout(4000, caption_dropout=0.1, source_dropout=0.2,
                                           device="cpu", generator=g)
    assert bool((dt | ~ds).all())                 # a dropped source always drops the text
    assert 0.25 < float(dt.float().mean()) < 0.31   # 1 - 0.9 * 0.8 = 0.28


def test_image_and_edit_training_drivers(tmp_path):
    from complexity_framework_b200.generative.image import (FrozenAutoencoderKL,
                                                            TRHashImageEditConfig,
                                                            TRHashImageEditor, TRHashImageConfig,
                                                            TRHashTextToImage)
    from complexity_framework_b200.generative.image_training import (ImageTrainConfig,
                                                                     tokenize_captions,
                                                                     train_image_model)

    ids, mask = tokenize_captions(ByteTok(), ["ab", ""], 8)
    assert ids.shape == (2, 2) and mask.tolist() == [[True, True], [True, False]]
    torch.manual_seed(0)
    m = TRHashTextToImage(_img_cfg(TRHashImageConfig), FrozenAutoencoderKL(channels=16))
    imgs = torch.rand(6, 3, 32, 32) * 2 - 1
    batches = [(imgs[:3], ["red", "blue", "red"]), (imgs[3:], ["blue", "red", "blue"])]
    cfg = ImageTrainConfig(max_steps=5, sft_steps=2, sft_lr_scale=0.5, save_steps=2,
                           keep_checkpoints=2, log_steps=1, bf16=False, warmup_steps=1,
                           learning_rate=1e-3, output=str(tmp_path / "t2i"))
    s = train_image_model(m, ByteTok(), batches, cfg, sft_batches=batches[:1])
    assert [e["stage"] for e in s["log"]] == ["pretrain"] * 3 + ["sft"] * 2
    assert s["log"][3]["lr"] < s["log"][2]["lr"]      # SFT runs at a scaled learning rate
    assert sorted(p.name for p in (tmp_path / "t2i").glob("step_*")) == ["step_0000004",
                                                                         "step_0000005"]
    s2 = train_image_model(TRHashTextToImage(_img_cfg(TRHashImageConfig),
                                             FrozenAutoencoderKL(channels=16)),
                           ByteTok(), batches, ImageTrainConfig(**{**cfg.__dict__,
                                                                   "max_steps": 6,
                                                                   "resume": True}))
    assert s2["steps"] == 6 and s2["log"][0]["step"] == 6
    ed = TRHashImageEditor(_img_cfg(TRHashImageEditConfig, source_drop_prob=0.3),
                           FrozenAutoencoderKL(channels=16))
    eb = [(imgs[:3], imgs[3:], ["make it red", "blue", "flip"])]
    s3 = train_image_model(ed, ByteTok(), eb, ImageTrainConfig(
        max_steps=2, bf16=False, warmup_steps=1, save_steps=10, log_steps=1,
        output=str(tmp_path / "edit")), edit=True)
    assert s3["steps"] == 2 and all(torch.isfinite(torch.tensor(e["loss"])) for e in s3["log"])
