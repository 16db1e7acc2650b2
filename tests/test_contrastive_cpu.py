"""Contrastive embedding training: InfoNCE contract, the bidirectional encoder,
weighted pair mixtures (order, hard negatives, token-target replay, sharding)
and a short chained training run; parity with the reference where it exists."""
import json
import os
import sys

import pytest
import torch
import torch.nn.functional as F

from complexity_framework_b200.training.contrastive import (WeightedPairMixtureDataset,
                                                             compute_pair_loss, info_nce_loss,
                                                             sqrt_normalized_weights,
                                                             train_embedding_stage)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


class WordTok:
    """Whitespace tokenizer with a fixed vocabulary (pad id 0)."""
    pad_token_id = 0

    def __init__(self):
        self.vocab = {}

    def encode(self, text):
        return [self.vocab.setdefault(w, 1 + len(self.vocab) % 250) for w in text.split()]


def test_info_nce_contract():
    torch.manual_seed(0)
    a = F.normalize(torch.randn(8, 16), dim=-1)
    assert info_nce_loss(a, a.clone()).item() < 0.05
    assert info_nce_loss(a, a[torch.randperm(8)]) > info_nce_loss(a, a.clone())
    with pytest.raises(ValueError, match="batch_size"):
        info_nce_loss(a[:1], a[:1])
    with pytest.raises(ValueError, match="shape mismatch"):
        info_nce_loss(a, a[:, :8])
    p = F.normalize(torch.randn(8, 16), dim=-1)
    sim = a @ p.T / 0.1
    lab = torch.arange(8)
    want = 0.5 * (F.cross_entropy(sim, lab) + F.cross_entropy(sim.T, lab))
    assert torch.allclose(info_nce_loss(a, p, temperature=0.1, symmetric=True), want)
    hn = F.normalize(torch.randn(8, 3, 16), dim=-1)
    logits = torch.cat((sim, torch.einsum("bd,bkd->bk", a, hn) / 0.1), 1)
    assert torch.allclose(info_nce_loss(a, p, temperature=0.1, hard_negative_embeddings=hn),
                          F.cross_entropy(logits, lab))
    with pytest.raises(ValueError, match="hard_negative_embeddings"):
        info_nce_loss(a, p, hard_negative_embeddings=hn[:4])


def test_info_nce_matches_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.training.info_nce import info_nce_loss as ref_loss
    finally:
        sys.path.remove(REF)
    g = torch.Generator().manual_seed(2)
    a, p = (F.normalize(torch.randn(6, 8, generator=g), dim=-1) for _ in range(2))
    hn = F.normalize(torch.randn(6, 2, 8, generator=g), dim=-1)
    for kw in ({}, {"symmetric": True}, {"hard_negative_embeddings": hn, "temperature": 0.2}):
        assert torch.allclose(info_nce_loss(a, p, **kw), ref_loss(a, p, **kw), atol=1e-6)


def _tiny_encoder():
    from complexity_framework_b200 import ModelConfig
    from complexity_framework_b200.models.embedding import BidirectionalEmbeddingModel

    cfg = ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=256, intermediate_size=64,
                      shared_intermediate_size=128, num_experts=2, top_k=2,
                      max_position_embeddings=32, is_causal=False)
    torch.manual_seed(0)
    return BidirectionalEmbeddingModel(cfg)


def test_encoder_pooling_and_padding():
    from complexity_framework_b200 import ModelConfig
    from complexity_framework_b200.models.embedding import BidirectionalEmbeddingModel

    with pytest.raises(ValueError, match="is_causal"):
        BidirectionalEmbeddingModel(ModelConfig(hidden_size=64, num_hidden_layers=1,
                                                num_attention_heads=4, vocab_size=64))
    m = _tiny_encoder().eval()
    ids = torch.randint(1, 256, (2, 12))
    mask = torch.ones(2, 12)
    mask[1, 7:] = 0
    e = m(ids, mask)
    assert torch.allclose(e.norm(dim=-1), torch.ones(2), atol=1e-5)
    # padding positions change nothing; bidirectional: a late token changes early states
    ids2 = ids.clone()
    ids2[1, 9] = (ids2[1, 9] + 1) % 256
    assert torch.allclose(m(ids2, mask)[1], e[1], atol=1e-5)
    ids3 = ids.clone()
    ids3[0, 11] = (ids3[0, 11] + 1) % 256
    assert not torch.allclose(m(ids3, mask)[0], e[0], atol=1e-4)


def test_encoder_matches_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        import complexity
        from complexity.models.embedding import BidirectionalEmbeddingModel as RefEnc
    finally:
        sys.path.remove(REF)
    mm = _tiny_encoder().eval()
    kw = {k: getattr(mm.config, k) for k in ("hidden_size", "num_hidden_layers",
                                             "num_attention_heads", "num_key_value_heads",
                                             "vocab_size", "intermediate_size",
                                             "shared_intermediate_size", "num_experts", "top_k",
                                             "max_position_embeddings", "is_causal")}
    rm = RefEnc(complexity.ModelConfig(**kw)).eval()
    rm.load_state_dict(mm.state_dict())
    ids = torch.randint(1, 256, (3, 16), generator=torch.Generator().manual_seed(4))
    mask = torch.ones(3, 16)
    mask[2, 10:] = 0
    assert torch.allclose(mm(ids, mask), rm(ids, mask), atol=1e-5)


def _rows(tag, n, negs=True):
    return [{"query": f"{tag} q {i}", "document": f"{tag} d {i} text",
             **({"negative": [f"{tag} n {i} a", f"{tag} n {i} b"]} if negs else {})}
            for i in range(n)]


def test_mixture_order_negatives_replay_and_sharding(tmp_path):
    assert sqrt_normalized_weights({"a": 100, "b": 25}) == pytest.approx({"a": 2 / 3, "b": 1 / 3})
    tok = WordTok()
    streams = {"a": _rows("a", 6), "b": _rows("b", 3)}
    ds = WeightedPairMixtureDataset(tok, split_weights={"a": 2.0, "b": 1.0}, max_seq_len=8,
                                    streams=streams)
    out = list(ds)
    assert len(out) == 9  # one full pass over both sources
    assert out[0]["anchor_input_ids"].shape == (8,)
    # weighted fair queuing: a, b, a, a, b, a, a, b, a  (smallest emitted/weight, first on ties)
    firsts = [tok_id for tok_id in (int(e["anchor_input_ids"][0]) for e in out)]
    a_id, b_id = tok.vocab["a"], tok.vocab["b"]
    assert firsts == [a_id, b_id, a_id, a_id, b_id, a_id, a_id, b_id, a_id]
    hard = list(WeightedPairMixtureDataset(tok, split_weights={"a": 1.0}, max_seq_len=8,
                                           num_hard_negatives=3, streams=streams))
    assert hard[0]["negative_input_ids"].shape == (3, 8)
    # token target above one pass: sources restart until the target is met
    one_pass = sum(int(e["anchor_attention_mask"].sum() + e["positive_attention_mask"].sum())
                   for e in out)
    rep = list(WeightedPairMixtureDataset(tok, split_weights={"a": 2.0, "b": 1.0},
                                          max_seq_len=8, streams=streams,
                                          target_tokens=2 * one_pass))
    assert len(rep) > len(out)
    # files + rank sharding: two ranks see disjoint rows that cover the source
    f = tmp_path / "a.jsonl"
    f.write_text("\n".join(json.dumps(r) for r in _rows("a", 6)))
    seen = []
    for r in range(2):
        seen += [tuple(e["positive_input_ids"].tolist()) for e in WeightedPairMixtureDataset(
            tok, split_weights={"a": 1.0}, max_seq_len=8, files={"a": str(f)}, rank=r,
            world_size=2)]
    assert len(seen) == 6 and len(set(seen)) == 6


def test_embedding_stages_train_and_chain(tmp_path):
    from torch.utils.data import DataLoader

    from complexity_framework_b200.training import TrainingConfig

    tok = WordTok()
    rows = _rows("x", 64)
    ds = WeightedPairMixtureDataset(tok, split_weights={"x": 1.0}, max_seq_len=8,
                                    num_hard_negatives=2, streams={"x": rows})
    batches = list(DataLoader(ds, batch_size=8))
    m = _tiny_encoder()
    with torch.no_grad():
        before = float(compute_pair_loss(m, batches[0]))
    cfg = TrainingConfig(learning_rate=3e-3, warmup_steps=0, lr_scheduler="constant",
                         precision="fp32", max_steps=16, checkpoint_dir=str(tmp_path / "ck"),
                         save_steps=10 ** 6, log_steps=1)
    summary = train_embedding_stage(m, batches * 2, cfg)
    assert summary["steps"] == 16
    with torch.no_grad():
        after = float(compute_pair_loss(m, batches[0]))
    assert after < before
    m.save_pretrained(tmp_path / "stage1")
    m2 = _tiny_encoder()
    cfg2 = TrainingConfig(learning_rate=1e-9, warmup_steps=0, lr_scheduler="constant",
                          precision="fp32", max_steps=1, checkpoint_dir=str(tmp_path / "ck2"),
                          save_steps=10 ** 6, log_steps=1, skip_param_update_check=True)
    train_embedding_stage(m2, batches[:1], cfg2, init_checkpoint=str(tmp_path / "stage1"))
    with torch.no_grad():
        assert abs(float(compute_pair_loss(m2, batches[0])) - after) < 1e-3
