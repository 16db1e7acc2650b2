"""SFT token shards: write / read round trip, supervision contract, relabeling
(parity with the reference's relabel_example), and SFT training on shards."""
import json
import os
import sys

import numpy as np
import pytest

from complexity_framework_b200.data import sft_shards as S

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
MARK, EOS = [50, 51], 2


def _example():
    # User: 10 11 | Assistant: 12 13 EOS | User: 14 | Assistant: 15 16 (EOS only as label)
    ids = [7, 10, 11, *MARK, 12, 13, EOS, 8, 14, *MARK, 15, 16]
    # only the final response is supervised (causal: label[t] = ids[t + 1]); the
    # marker's last token predicts the first content token, the EOS is a target only
    lab = [-100] * len(ids)
    last_marker = len(ids) - 3          # index of MARK[-1] of the final marker
    lab[last_marker], lab[last_marker + 1], lab[last_marker + 2] = 15, 16, EOS
    return ids, lab


def test_relabel_example_supervises_every_turn():
    ids, lab = _example()
    new, n = S.relabel_example(ids, lab, assistant_marker=MARK, eos_token_id=EOS)
    first = 4  # MARK[-1] of the first marker
    assert new[first:first + 3].tolist() == [12, 13, EOS]
    assert n == 6
    with pytest.raises(ValueError, match="no Assistant marker"):
        S.relabel_example([1, 2, 3], [-100] * 3, assistant_marker=MARK, eos_token_id=EOS)
    bad = list(lab)
    bad[0] = 10
    with pytest.raises(ValueError, match="outside"):
        S.relabel_example(ids, bad, assistant_marker=MARK, eos_token_id=EOS)


def test_relabel_matches_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.training.sft_relabel import relabel_example as ref_relabel
    finally:
        sys.path.remove(REF)
    ids, lab = _example()
    a, na = S.relabel_example(ids, lab, assistant_marker=MARK, eos_token_id=EOS)
    b, nb = ref_relabel(np.array(ids), np.array(lab), assistant_marker=MARK, eos_token_id=EOS)
    assert na == nb and a.tolist() == b.tolist()


def test_contract():
    S.validate_shard_supervision({"format": "other"})
    S.validate_shard_supervision({"format": S.SHARD_FORMAT_V2,
                                  "assistant_supervision": "all_assistant_turns"})
    S.validate_shard_supervision({"format": S.SHARD_FORMAT_V2,
                                  "assistant_supervision": "final_assistant_only",
                                  "history_assistant_turns": "masked_context"})
    with pytest.raises(ValueError, match="masked assistant history"):
        S.validate_shard_supervision({"format": S.SHARD_FORMAT_V2,
                                      "assistant_supervision": "final_assistant_only"})
    with pytest.raises(ValueError, match="requires"):
        S.validate_shard_supervision({"format": S.SHARD_FORMAT_V2})


def test_write_read_relabel_dataset(tmp_path):
    ids, lab = _example()
    meta = {"assistant_supervision": "final_assistant_only",
            "history_assistant_turns": "masked_context"}
    for part in ("p0", "p1"):
        S.write_sft_shard(tmp_path / "src" / part, [(ids, lab), (ids[:5] + [12, EOS], [-100] * 4
                                                                   + [12, EOS, -100])], meta)
    (tmp_path / "src" / "chat_template.json").write_text(json.dumps({"name": "x"}))
    ds = S.SFTTokenShardDataset(tmp_path / "src")
    assert len(ds) == 4
    x, y = ds[0]
    assert x == ids and y[1:] == [v for v in lab[:-1]] and y[0] == -100
    src_labels = (tmp_path / "src" / "p0" / "labels.bin").read_bytes()
    res = S.relabel_dataset(tmp_path / "src", tmp_path / "out", assistant_marker=MARK,
                            eos_token_id=EOS)
    assert res["p0"]["changed_labels"] == 3 and res["p1"]["examples"] == 2
    assert (tmp_path / "src" / "p0" / "labels.bin").read_bytes() == src_labels  # untouched
    meta2 = json.loads((tmp_path / "out" / "p0" / "sft.idx.json").read_text())
    assert meta2["assistant_supervision"] == "all_assistant_turns"
    assert meta2["content_verification"] == "sha256"
    tpl = json.loads((tmp_path / "out" / "chat_template.json").read_text())
    assert tpl["training_projection"] == S.ALL_ASSISTANT_PROJECTION
    with pytest.raises(FileExistsError):
        S.relabel_dataset(tmp_path / "src", tmp_path / "out", assistant_marker=MARK,
                          eos_token_id=EOS)


def test_sft_trains_on_shards(tmp_path):
    import torch

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.training import sft

    ids, lab = _example()
    S.write_sft_shard(tmp_path / "data", [(ids, lab)] * 8,
                      {"assistant_supervision": "final_assistant_only",
                       "history_assistant_turns": "masked_context"})
    torch.manual_seed(0)
    ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                num_key_value_heads=2, vocab_size=260, intermediate_size=64,
                                shared_intermediate_size=128, num_experts=2, top_k=2,
                                max_position_embeddings=64)).save_pretrained(tmp_path / "m")
    s = sft.main(["--model", str(tmp_path / "m"), "--data", str(tmp_path / "data"),
                  "--output", str(tmp_path / "out"), "--batch-size", "4", "--epochs", "2",
                  "--precision", "fp32", "--lr", "1e-3"])
    assert s["steps"] == 4 and s["examples"] == 8
