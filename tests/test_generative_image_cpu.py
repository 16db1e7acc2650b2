"""Latent codec, text-to-image flow transformer and image editor (CPU)."""
import io
import tarfile

import torch

from complexity_framework_b200.generative.image import (
    AtlasImageEditTarDataset, AtlasImageTarDataset, FrozenAutoencoderKL, TRHashImageConfig,
    TRHashImageEditConfig, TRHashImageEditor, TRHashTextToImage, collate_atlas_image_edits,
    collate_atlas_images)


def _cfg(cls=TRHashImageConfig):
    return cls(image_size=32, hidden_size=64, num_layers=2, num_heads=4, shared_width=128,
               expert_width=32, text_vocab_size=64, text_dim=32)


def _fit(params, fn, steps):
    opt = torch.optim.AdamW(params, 3e-3)
    first = None
    for _ in range(steps):
        loss = fn()
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss)
    return first, float(loss)


def test_codec_trains_and_freezes():
    torch.manual_seed(0)
    codec = FrozenAutoencoderKL(channels=16, frozen=False)
    x = torch.rand(2, 3, 32, 32) * 2 - 1
    first, last = _fit(codec.parameters(), lambda: codec.loss(x)["loss"], 30)
    assert last < first
    codec.set_frozen(True)
    assert not any(p.requires_grad for p in codec.parameters())
    assert codec.encode(x).shape == (2, 4, 4, 4) and codec.decode(codec.encode(x)).shape == x.shape


def test_text_to_image_flow_fits_and_samples():
    torch.manual_seed(0)
    codec = FrozenAutoencoderKL(channels=16)
    m = TRHashTextToImage(_cfg(), codec)
    lat = torch.randn(4, 4, 4, 4)
    ids = torch.randint(0, 64, (4, 6))
    first, last = _fit([p for p in m.parameters() if p.requires_grad],
                       lambda: m(text_ids=ids, latents=lat)["loss"], 40)
    assert last < first
    g = torch.Generator().manual_seed(1)
    img = m.generate(text_ids=ids[:2], steps=3, guidance=2.0, generator=g)
    assert img.shape == (2, 3, 32, 32) and float(img.abs().max()) <= 1.0
    # classifier-free guidance of 1 equals the conditional velocity alone
    z = torch.randn(1, 4, 4, 4)
    t = torch.full((1,), 0.5)
    ctx = m.text_context(ids[:1])
    assert torch.allclose(m.velocity(z, t, ctx), m.velocity(z, t, ctx))


def test_editor_and_tar_datasets(tmp_path):
    from PIL import Image

    torch.manual_seed(0)
    m = TRHashImageEditor(_cfg(TRHashImageEditConfig), FrozenAutoencoderKL(channels=16))
    src, tgt = torch.rand(2, 3, 32, 32) * 2 - 1, torch.rand(2, 3, 32, 32) * 2 - 1
    ids = torch.randint(0, 64, (2, 5))
    out = m(src, tgt, text_ids=ids)
    out["loss"].backward()
    assert m.edit(src, text_ids=ids, steps=2).shape == (2, 3, 32, 32)

    def png(colour):
        b = io.BytesIO()
        Image.new("RGB", (20, 20), colour).save(b, format="PNG")
        return b.getvalue()

    tar = tmp_path / "edits.tar"
    with tarfile.open(tar, "w") as tf:
        for name, data in (("a.src.png", png((255, 0, 0))), ("a.tgt.png", png((0, 255, 0))),
                           ("a.txt", b"make it green"), ("b.png", png((0, 0, 255))),
                           ("b.txt", b"blue")):
            info = tarfile.TarInfo(name)
            info.size = len(data)
            tf.addfile(info, io.BytesIO(data))

    class Tok:
        def encode(self, s):
            return [len(w) for w in s.split()]

    eds = AtlasImageEditTarDataset(str(tar), Tok(), image_size=32)
    s, t, i = collate_atlas_image_edits([eds[0]])
    assert len(eds) == 1 and s.shape == (1, 3, 32, 32) and i.tolist() == [[4, 2, 5]]
    assert float(s[0, 0].mean()) > 0.9 and float(t[0, 1].mean()) > 0.9  # red -> green
    ids_ds = AtlasImageTarDataset(str(tar), Tok(), image_size=32)
    imgs, txt = collate_atlas_images([ids_ds[0]])
    assert len(ids_ds) == 1 and imgs.shape == (1, 3, 32, 32)


def test_generative_trainer_resumes(tmp_path):
    from complexity_framework_b200.generative.training import (GenerativeTrainer,
                                                               GenerativeTrainingConfig)

    torch.manual_seed(0)
    m = TRHashTextToImage(_cfg(), FrozenAutoencoderKL(channels=16))
    lat = torch.randn(4, 4, 4, 4)
    ids = torch.randint(0, 64, (4, 6))
    tr = GenerativeTrainer(m, GenerativeTrainingConfig(learning_rate=3e-3, warmup_steps=2,
                                                       max_steps=30, log_every=1000))
    batches = [{"latents": lat, "text_ids": ids}] * 30
    first = tr.train_step(batches[0])["loss"]
    last = tr.train(batches[1:], max_steps=30, log=None)["loss"]
    assert last < first and tr.step == 30
    tr.save(str(tmp_path / "ck"))
    tr2 = GenerativeTrainer(TRHashTextToImage(_cfg(), FrozenAutoencoderKL(channels=16)))
    tr2.load(str(tmp_path / "ck"))
    assert tr2.step == 30
    assert all(torch.equal(a, b) for a, b in zip(m.state_dict().values(),
                                                 tr2.model.state_dict().values()))
