"""Data library: token shards through the native reader, loaders, packing, chat labels."""
import json

import numpy as np
import torch

from complexity_framework_b200.data import (ByteTokenizer, ChatTemplate, Message,
                                            PackedSequenceCollator, TokenBatchLoader,
                                            TokenShardDataset, TokenShardMixture, encode_chat,
                                            load_token_shard, pack_documents,
                                            token_shard_frequencies, write_token_shard)
from complexity_framework_b200.data.tokenization import IGNORE_INDEX


def _shard(tmp_path, n=10000, vocab=1000, name="s"):
    toks = np.arange(n) % vocab
    write_token_shard(tmp_path / name, toks, vocab_size=vocab)
    return tmp_path / name, toks


def test_write_load_format(tmp_path):
    p, toks = _shard(tmp_path)
    meta = json.loads((p / "tokens.idx.json").read_text())
    assert meta["format"] == "complexity-token-shard-v1" and meta["dtype"] == "<u2"
    arr, m = load_token_shard(p)
    assert np.array_equal(np.asarray(arr), toks) and m["num_tokens"] == len(toks)
    f = token_shard_frequencies(p, 1000)
    assert int(f.sum()) == len(toks) and int(f[5]) == 10


def test_sequential_dataset_partitions_ranks(tmp_path):
    p, toks = _shard(tmp_path, vocab=10000)
    seen = []
    for r in range(2):
        ds = TokenShardDataset(p, 64, rank=r, world_size=2, order="sequential", eval_ratio=0)
        for item in ds:
            assert torch.equal(item["labels"][:-1], item["input_ids"][1:])
            seen.append(int(item["input_ids"][0]))
    starts = sorted(seen)
    assert len(starts) == len(set(starts))
    assert len(starts) == (10000 - 1) // 64


def test_batch_loader_matches_shard(tmp_path):
    p, toks = _shard(tmp_path, n=50000, vocab=30000)
    ld = TokenBatchLoader(p, 4, 128, pin_memory=False, seed=3)
    x, y = next(iter(ld))
    assert x.shape == (4, 128)
    for row in range(4):
        s = int(x[row, 0])
        # positions are start offsets into arange % vocab
        idx = np.where(toks == s)[0]
        assert any(np.array_equal(toks[i:i + 129], torch.cat([x[row], y[row, -1:]]).numpy())
                   for i in idx)
    ld.close()
    seq = TokenBatchLoader(p, 4, 128, order="sequential", pin_memory=False, eval_ratio=0)
    n = 0
    for _ in seq:
        n += 1
    assert n == (50000 - 1) // 512


def test_mixture_counts_and_replay(tmp_path):
    a, _ = _shard(tmp_path, name="a")
    b, _ = _shard(tmp_path, name="b")
    mx = TokenShardMixture([a, b], [3, 1], batch_size=8, seq_len=32, eval_ratio=0)
    assert list(mx.counts()) == [6, 2]
    b1 = mx.batch(5)
    assert torch.equal(b1, mx.batch(5)) and b1.shape == (8, 33)


def test_packing_labels_never_cross_documents():
    docs = [[1, 2, 3], [4, 5, 6, 7, 8], [9, 10]]
    t, d = pack_documents(docs, 6, pad_id=0)
    assert t.shape[1] == 6
    assert sorted(x for x in t.flatten().tolist() if x) == list(range(1, 11))
    out = PackedSequenceCollator(6)(docs)
    lab, ids, pos = out["labels"], out["input_ids"], out["position_ids"]
    for r in range(ids.shape[0]):
        for i in range(5):
            if lab[r, i] != IGNORE_INDEX:
                assert out["doc_ids"][r, i] == out["doc_ids"][r, i + 1]
    assert pos[0, 0] == 0


def test_byte_tokenizer_and_chat_labels():
    tok = ByteTokenizer()
    s = "héllo <|user|> x"
    assert tok.decode(tok.encode(s)) == s
    msgs = [Message("system", "be brief"), Message("user", "hi"), Message("assistant", "hello")]
    ids, labels = encode_chat(tok, msgs, ChatTemplate("complexity"))
    assert len(ids) == len(labels)
    trained = tok.decode([i for i, l in zip(ids, labels) if l != IGNORE_INDEX])
    assert "hello" in trained and "hi" not in trained.replace("hello", "")
    text = ChatTemplate("chatml").apply(msgs, add_generation_prompt=True)
    assert text.endswith("<|im_start|>assistant\n")


def test_sequence_packing_plan_and_epoch_schedule():
    import pytest

    from complexity_framework_b200.data.packing import pack_example_lengths, resolve_epoch_schedule

    plan = pack_example_lengths([3, 4, 2, 8, 1, 1], sequence_length=8, separator_tokens=1)
    assert plan.packs == ((0, 1), (2,), (3,), (4, 5))
    assert plan.source_tokens == 19 and plan.separator_count == 2
    assert plan.compression_ratio == 1.5
    assert abs(plan.occupied_utilization - 21 / 32) < 1e-12
    with pytest.raises(ValueError, match="within the sequence window"):
        pack_example_lengths([9], sequence_length=8)
    s = resolve_epoch_schedule(items=10, world_size=3, batch_size_per_rank=2, epochs=3)
    assert s.steps_per_epoch == 2 and s.total_steps == 6 and s.epoch_steps() == (2, 4, 6)


def test_preprocessing_augmentation_and_text_shards(tmp_path):
    import json

    import torch

    from complexity_framework_b200.data.preprocessing import (DataAugmenter, DataPipeline,
                                                              MixupCollator, TextPreprocessor)
    from complexity_framework_b200.data.token_shards import (build_token_shard_from_texts,
                                                             iter_texts_from_files,
                                                             load_token_shard)
    from complexity_framework_b200.data.tokenization import get_tokenizer

    p = TextPreprocessor(lowercase=True)
    assert p("<b>Visit</b> https://x.io now,  mail a@b.com   PLEASE") == "visit now, mail please"
    assert p("short") is None
    assert DataPipeline.create_default()("   tiny  ") is None
    aug = DataAugmenter(delete_prob=0.3, swap_prob=0.2, insert_prob=0.2)
    assert aug.augment_tokens(list(range(50)), seed=1) == aug.augment_tokens(list(range(50)), seed=1)
    b = MixupCollator(0.4)([{"input_ids": torch.arange(4), "labels": torch.tensor(0)},
                            {"input_ids": torch.arange(4) + 4, "labels": torch.tensor(1)}])
    assert b["input_ids_mixed"].shape == (2, 4) and 0 <= float(b["mixup_lambda"]) <= 1
    f = tmp_path / "a.jsonl"
    f.write_text("\n".join(json.dumps({"text": t}) for t in ("ab", "", "cde")) + "\n")
    assert list(iter_texts_from_files([f])) == ["ab", "cde"]
    assert list(iter_texts_from_files([f], limit=1)) == ["ab"]
    tok = get_tokenizer("byte")
    build_token_shard_from_texts(iter_texts_from_files([f]), tok, tmp_path / "shard")
    arr, meta = load_token_shard(tmp_path / "shard")
    assert meta["num_tokens"] == len(arr) == len(tok.encode("ab")) + len(tok.encode("cde")) + 2
