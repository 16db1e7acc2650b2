"""Pretokenized corpus mixtures: manifest validation, weighted interleaving,
rank sharding, replay plans and resume-skip."""
import json

import numpy as np
import pytest
import torch

from complexity_framework_b200.data.corpus_mixture import (
    PretokenizedCorpusMixtureDataset, TextCorpusSource, WeightedStreamingTextDataset,
    allocate_weighted_counts, validate_corpus_mixture, write_token_mixture)

S = 8


def _mixture(tmp_path, rows=(12, 6), rps=4):
    toks = {}
    for i, (name, r) in enumerate(zip(("web", "code"), rows)):
        toks[name] = (2 / 3 if i == 0 else 1 / 3,
                      np.arange(r * S + 1, dtype=np.int64) + 1000 * (i + 1))
    write_token_mixture(tmp_path, toks, S, rps)
    return toks


def _rows(ds):
    return [tuple(x["input_ids"].tolist()) for x in ds]


def test_validation_and_allocation():
    a = TextCorpusSource("a", 0.5, data_files="x")
    b = TextCorpusSource("b", 0.5, data_files="y")
    validate_corpus_mixture([a, b])
    with pytest.raises(ValueError, match="sum to 1.0"):
        validate_corpus_mixture([a])
    with pytest.raises(ValueError, match="unique"):
        validate_corpus_mixture([a, a])
    with pytest.raises(ValueError, match="exactly one"):
        TextCorpusSource("c", 1.0).validate()
    c = [TextCorpusSource("a", 0.7, data_files="x"), TextCorpusSource("b", 0.3, data_files="y")]
    assert allocate_weighted_counts(11, c) == {"a": 8, "b": 3}
    assert sum(allocate_weighted_counts(7, c).values()) == 7


def test_rows_labels_and_weighted_order(tmp_path):
    _mixture(tmp_path)
    ds = PretokenizedCorpusMixtureDataset(tmp_path)
    items = list(ds)
    assert len(items) == 18 and ds.unique_tokens == 18 * S
    x = items[0]
    assert torch.equal(x["labels"][:-1], x["input_ids"][1:])
    # 2:1 weights: the pattern web, code, web repeats (fair queuing, first on ties)
    src = ["web" if int(i["input_ids"][0]) < 2000 else "code" for i in items]
    assert src[:6] == ["web", "code", "web", "web", "code", "web"]
    # rows of a source come in order and cross shard boundaries seamlessly
    web = [int(i["input_ids"][0]) for i in items if int(i["input_ids"][0]) < 2000]
    assert web == [1000 + r * S for r in range(12)]


def test_rank_sharding_and_resume_skip(tmp_path):
    _mixture(tmp_path)
    full = set(_rows(PretokenizedCorpusMixtureDataset(tmp_path)))
    r0 = _rows(PretokenizedCorpusMixtureDataset(tmp_path, rank=0, world_size=2))
    r1 = _rows(PretokenizedCorpusMixtureDataset(tmp_path, rank=1, world_size=2))
    assert set(r0) | set(r1) == full and not set(r0) & set(r1)
    resumed = _rows(PretokenizedCorpusMixtureDataset(tmp_path, rank=1, world_size=2,
                                                     resume_skip_rows=4))
    assert resumed == r1[4:]
    with pytest.raises(ValueError, match="divisible"):
        list(PretokenizedCorpusMixtureDataset(tmp_path, rank=0, world_size=4))


def test_replay_plan(tmp_path):
    _mixture(tmp_path)
    plan = {"format": "tr-hash-token-replay-v1", "seq_len": S,
            "phases": [{"name": "warm", "passes": 2,
                        "sources": {"web": [{"file": "shard-00000.bin", "rows": 2}],
                                    "code": [{"file": "shard-00000.bin"}]}},
                       {"name": "main", "sources": {"web": [{"file": "shard-00001.bin"}]}}]}
    plan["unique_tokens"] = (2 + 4 + 4) * S
    plan["trained_tokens"] = ((2 + 4) * 2 + 4) * S
    ds = PretokenizedCorpusMixtureDataset(tmp_path, replay_plan=plan)
    rows = _rows(ds)
    assert len(rows) == 16 and rows[:6] == rows[6:12]
    skip = _rows(PretokenizedCorpusMixtureDataset(tmp_path, replay_plan=plan,
                                                  resume_skip_rows=5))
    assert skip == rows[5:]
    bad = dict(plan, trained_tokens=1)
    with pytest.raises(ValueError, match="trained_tokens mismatch"):
        PretokenizedCorpusMixtureDataset(tmp_path, replay_plan=bad)
    (tmp_path / "plan.json").write_text(json.dumps(plan))
    assert _rows(PretokenizedCorpusMixtureDataset(tmp_path, replay_plan="plan.json")) == rows


def test_manifest_corruption_detected(tmp_path):
    _mixture(tmp_path)
    shard = tmp_path / "corpora" / "code" / "shard-00000.bin"
    shard.write_bytes(shard.read_bytes()[:-2])
    with pytest.raises(ValueError, match="corrupt"):
        PretokenizedCorpusMixtureDataset(tmp_path)


def test_weighted_text_streams():
    class Tok:
        eos_token_id = 0

        def encode(self, text, add_special_tokens=False):
            return [ord(c) for c in text]

    srcs = [TextCorpusSource("a", 0.5, data_files="-"), TextCorpusSource("b", 0.5, data_files="-")]
    streams = {"a": [{"text": "aaaaaaaaaa"}] * 20, "b": [{"text": "bbbbbbbbbb"}] * 20}
    ds = WeightedStreamingTextDataset(tokenizer=Tok(), seq_len=4, sources=srcs, streams=streams)
    it = iter(ds)
    first = [next(it)["input_ids"] for _ in range(6)]
    kinds = [int(x[0]) for x in first]
    assert kinds[0] in (97, 0) and sum(1 for x in first if 98 in x.tolist()) >= 2
    # documents never cross sources
    assert all(not ({97, 98} <= set(x.tolist())) for x in first)
