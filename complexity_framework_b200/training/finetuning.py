"""Training-stage policy: which stage may follow which, what a refinement must
prove, and which pipelines may fine-tune every parameter.

Counterpart of complexity/training/finetuning.py:1-244.  The stage and
pipeline names are the reference's strings (run metadata and launchers match
on them).  Rules:
  * a lineage is ``pretraining -> refinement -> supervised-finetuning``; more
    SFT stages may follow SFT; pretraining is a root, never a target;
  * a refinement starts from pretraining weights, on the exact pretraining
    corpus, with a fresh optimizer and scheduler; a replay plan proves the
    corpus by a SHA-256 fingerprint of its single-pass ``unique_core`` phase
    (format, dataset, revision, sequence length, selection and row alignment,
    token totals and the per-source selections), and the refinement plan must
    train each unique token exactly once;
  * vision lineages fold refinement into pretraining (augmentation anneal), so
    vision SFT may start from pretraining;
  * full-parameter fine-tuning is allowed only for the listed pipelines, and
    non-vision SFT must name its source stage (no direct pretraining -> SFT).
"""
from __future__ import annotations

import hashlib
import json
from typing import Any, Mapping, Optional

PRETRAINING_STAGE = "pretraining"
REFINEMENT_STAGE = "refinement"
SUPERVISED_FINETUNING_STAGE = "supervised-finetuning"
STAGES = frozenset({PRETRAINING_STAGE, REFINEMENT_STAGE, SUPERVISED_FINETUNING_STAGE})

TEXT_MODEL_FAMILY = "text"
VISION_MODEL_FAMILY = "vision"
IMAGE_GENERATION_MODEL_FAMILY = "image-generation"
IMAGE_EDITING_MODEL_FAMILY = "image-editing"
IMAGE_TEXT_TO_TEXT_MODEL_FAMILY = "image-text-to-text"

TEXT_SUPERVISED_FINETUNING = "supervised-finetuning"
VISION_SUPERVISED_FINETUNING = "vision-supervised-finetuning"
IMAGE_GENERATION_SUPERVISED_FINETUNING = "image-generation-supervised-finetuning"
IMAGE_EDITING_SUPERVISED_FINETUNING = "image-editing-supervised-finetuning"
IMAGE_TEXT_TO_TEXT_SUPERVISED_FINETUNING = "image-text-to-text-supervised-finetuning"
TEXT_REFINEMENT = "text-refinement"
TEXT_CONTINUED_PRETRAINING = TEXT_REFINEMENT   # older name of the same stage

INTEGRATED_REFINEMENT_MODEL_FAMILIES = frozenset({VISION_MODEL_FAMILY})
PIPELINE_FAMILY = {
    TEXT_SUPERVISED_FINETUNING: TEXT_MODEL_FAMILY,
    VISION_SUPERVISED_FINETUNING: VISION_MODEL_FAMILY,
    IMAGE_GENERATION_SUPERVISED_FINETUNING: IMAGE_GENERATION_MODEL_FAMILY,
    IMAGE_EDITING_SUPERVISED_FINETUNING: IMAGE_EDITING_MODEL_FAMILY,
    IMAGE_TEXT_TO_TEXT_SUPERVISED_FINETUNING: IMAGE_TEXT_TO_TEXT_MODEL_FAMILY,
}
FULL_PARAMETER_FINETUNING_PIPELINES = frozenset(set(PIPELINE_FAMILY) | {TEXT_REFINEMENT})


def validate_training_stage_transition(model_family: str, source_stage: str, target_stage: str,
                                       *, same_corpus: Optional[bool] = None,
                                       fresh_optimizer: Optional[bool] = None) -> None:
    for what, st in (("source", source_stage), ("target", target_stage)):
        if st not in STAGES:
            raise ValueError(f"unknown {what} training stage: {st!r}")
    if target_stage == PRETRAINING_STAGE:
        raise ValueError("pretraining is a lineage root, not a transition target")
    if target_stage == REFINEMENT_STAGE:
        if source_stage != PRETRAINING_STAGE:
            raise ValueError("refinement must start from a pretraining checkpoint")
        if same_corpus is not True:
            raise ValueError("refinement must reuse the exact pretraining corpus")
        if fresh_optimizer is not True:
            raise ValueError("refinement must start with a fresh optimizer and scheduler")
        return
    # supervised fine-tuning
    if model_family in INTEGRATED_REFINEMENT_MODEL_FAMILIES:
        if source_stage not in (PRETRAINING_STAGE, REFINEMENT_STAGE):
            raise ValueError("Vision SFT must start from its pretraining lineage or an "
                             "explicit refinement checkpoint")
        return
    if source_stage not in (REFINEMENT_STAGE, SUPERVISED_FINETUNING_STAGE):
        raise ValueError(f"{model_family} SFT requires a refinement checkpoint; direct "
                         "pretraining -> SFT is forbidden")


def _unique_core(plan: Mapping[str, Any]) -> Mapping[str, Any]:
    phases = plan.get("phases")
    if not isinstance(phases, list):
        raise ValueError("replay plan must contain a phases list")
    core = [p for p in phases if p.get("name") == "unique_core"]
    if len(core) != 1:
        raise ValueError("replay plan must contain exactly one unique_core phase")
    ph = core[0]
    if ph.get("passes") != 1:
        raise ValueError("unique_core must contain exactly one pass")
    if not isinstance(ph.get("sources"), Mapping) or not ph["sources"]:
        raise ValueError("unique_core must contain non-empty source selections")
    return ph


def refinement_corpus_fingerprint(plan: Mapping[str, Any]) -> str:
    """SHA-256 of the canonical JSON of the unique-corpus contract (replay
    phases excluded), so two plans with the same single-pass selection agree."""
    keys = ("format", "dataset", "revision", "seq_len", "selection_mode", "row_alignment",
            "unique_tokens", "source_unique_tokens")
    contract = {k: plan.get(k) for k in keys}
    contract["sources"] = _unique_core(plan)["sources"]
    blob = json.dumps(contract, sort_keys=True, separators=(",", ":"), ensure_ascii=True)
    return hashlib.sha256(blob.encode("utf-8")).hexdigest()


def validate_refinement_plan(refinement_plan: Mapping[str, Any],
                             pretrain_plan: Mapping[str, Any]) -> str:
    """Check that ``refinement_plan`` is exactly one pass over the pretraining
    corpus; returns the corpus fingerprint for audit metadata."""
    validate_training_stage_transition(TEXT_MODEL_FAMILY, PRETRAINING_STAGE, REFINEMENT_STAGE,
                                       same_corpus=True, fresh_optimizer=True)
    core = _unique_core(refinement_plan)
    _unique_core(pretrain_plan)
    if len(refinement_plan["phases"]) != 1:
        raise ValueError("refinement plan must contain only the unique_core phase")
    if int(refinement_plan.get("trained_tokens", -1)) != int(refinement_plan.get("unique_tokens",
                                                                                 -2)):
        raise ValueError("refinement plan must train each unique token exactly once")
    sp = refinement_plan.get("source_passes")
    if (not isinstance(sp, Mapping) or not sp or set(sp) != set(core["sources"])
            or any(int(v) != 1 for v in sp.values())):
        raise ValueError("refinement plan must use exactly one pass per source")
    want, got = refinement_corpus_fingerprint(pretrain_plan), refinement_corpus_fingerprint(
        refinement_plan)
    if want != got:
        raise ValueError("refinement corpus does not exactly match the pretraining unique_core "
                         f"(expected {want}, got {got})")
    return got


def validate_full_parameter_finetuning(pipeline: str, *, unique_tokens: Optional[int] = None,
                                       pretrain_unique_tokens: Optional[int] = None,
                                       source_stage: Optional[str] = None,
                                       model_family: Optional[str] = None) -> None:
    if pipeline not in FULL_PARAMETER_FINETUNING_PIPELINES:
        allowed = ", ".join(repr(p) for p in sorted(FULL_PARAMETER_FINETUNING_PIPELINES))
        raise ValueError(f"full-parameter SFT is restricted to {allowed}; got {pipeline!r}")
    if pipeline == TEXT_REFINEMENT:
        if unique_tokens is None or pretrain_unique_tokens is None:
            raise ValueError("text-refinement requires unique_tokens and pretrain_unique_tokens")
        if unique_tokens != pretrain_unique_tokens:
            raise ValueError(f"text-refinement requires unique_tokens ({unique_tokens:,}) to "
                             "exactly match the completed pretrain's unique_tokens "
                             f"({pretrain_unique_tokens:,})")
        return
    family = model_family or PIPELINE_FAMILY[pipeline]
    if source_stage is not None:
        validate_training_stage_transition(family, source_stage, SUPERVISED_FINETUNING_STAGE)
    elif family != VISION_MODEL_FAMILY:
        raise ValueError(f"{pipeline} requires source_stage={REFINEMENT_STAGE!r}; direct "
                         "pretraining -> SFT is forbidden")
