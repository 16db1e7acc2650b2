"""Training-stage policy: transitions, refinement corpus proof, full-parameter gating."""
import copy

import pytest

from complexity_framework_b200.training import finetuning as P

PLAN = {"format": "tr-hash-token-replay-v1", "dataset": "d", "revision": "r", "seq_len": 2048,
        "selection_mode": "rows", "row_alignment": 1, "unique_tokens": 100,
        "trained_tokens": 100, "source_unique_tokens": {"a": 60, "b": 40},
        "source_passes": {"a": 1, "b": 1},
        "phases": [{"name": "unique_core", "passes": 1, "sources": {"a": [0, 3], "b": [0, 2]}}]}


def test_transitions():
    P.validate_training_stage_transition("text", "pretraining", "refinement", same_corpus=True,
                                         fresh_optimizer=True)
    P.validate_training_stage_transition("text", "refinement", "supervised-finetuning")
    P.validate_training_stage_transition("text", "supervised-finetuning", "supervised-finetuning")
    P.validate_training_stage_transition("vision", "pretraining", "supervised-finetuning")
    for args, kw, msg in [
        (("text", "pretraining", "supervised-finetuning"), {}, "direct"),
        (("text", "refinement", "refinement"), {"same_corpus": True, "fresh_optimizer": True},
         "pretraining checkpoint"),
        (("text", "pretraining", "refinement"), {"fresh_optimizer": True}, "exact pretraining"),
        (("text", "pretraining", "refinement"), {"same_corpus": True}, "fresh optimizer"),
        (("text", "refinement", "pretraining"), {}, "lineage root"),
        (("text", "warmup", "refinement"), {}, "unknown source"),
        (("vision", "supervised-finetuning", "supervised-finetuning"), {}, "Vision SFT"),
    ]:
        with pytest.raises(ValueError, match=msg):
            P.validate_training_stage_transition(*args, **kw)


def test_refinement_plan_proof():
    pre = copy.deepcopy(PLAN)
    pre["phases"].append({"name": "replay", "passes": 2, "sources": {"a": [0, 1]}})
    pre["trained_tokens"] = 160
    fp = P.validate_refinement_plan(PLAN, pre)
    assert fp == P.refinement_corpus_fingerprint(pre) and len(fp) == 64
    bad = copy.deepcopy(PLAN)
    bad["phases"][0]["sources"]["b"] = [0, 1]
    with pytest.raises(ValueError, match="does not exactly match"):
        P.validate_refinement_plan(bad, pre)
    rep = copy.deepcopy(PLAN)
    rep["trained_tokens"] = 120
    with pytest.raises(ValueError, match="exactly once"):
        P.validate_refinement_plan(rep, pre)
    two = copy.deepcopy(PLAN)
    two["source_passes"]["a"] = 2
    with pytest.raises(ValueError, match="one pass per source"):
        P.validate_refinement_plan(two, pre)
    with pytest.raises(ValueError, match="only the unique_core"):
        P.validate_refinement_plan(pre, pre)


def test_full_parameter_gating():
    P.validate_full_parameter_finetuning("vision-supervised-finetuning")
    P.validate_full_parameter_finetuning("supervised-finetuning", source_stage="refinement")
    P.validate_full_parameter_finetuning("text-refinement", unique_tokens=5,
                                         pretrain_unique_tokens=5)
    with pytest.raises(ValueError, match="restricted"):
        P.validate_full_parameter_finetuning("lora-everything")
    with pytest.raises(ValueError, match="direct"):
        P.validate_full_parameter_finetuning("supervised-finetuning")
    with pytest.raises(ValueError, match="exactly match"):
        P.validate_full_parameter_finetuning("text-refinement", unique_tokens=5,
                                             pretrain_unique_tokens=6)
    assert P.TEXT_CONTINUED_PRETRAINING == P.TEXT_REFINEMENT
