"""Multimodal sensor fusion classifier (robot / activity perception).

Counterpart: complexity/generative/sensor_fusion/ (config.py
``SENSOR_MODALITIES`` / ``TRHashSensorFusionConfig``, model.py
``TRHashSensorFusionBlock`` / ``TRHashSensorFusionClassifier``, folds.py
``CrossSubjectFold`` / ``resolve_cross_subject_fold``, cuhkx_records.py
``subject_disjoint_records`` and the dataset / manifest helpers).

Six streams: depth, infrared and thermal clips share one TR-Hash vision
tower (each frame -> patch features -> pooled to a small token grid, averaged
over time, or pooled to a (time, height, width) token lattice; clips come as
[B, T, C, H, W] or, with ``visual_layout="bcthw"``, the reference's
[B, C, T, H, W]); IMU, radar and skeleton sequences are projected and pooled to a
fixed number of tokens.  Tokens of all present streams (missing ones are
simply absent) get modality embeddings and pass through TR-Hash blocks routed
by ``(modality, local token position)``; the prediction mixes the fused head
with the mean of per-modality heads (``late_fusion_weight``).
"""
from __future__ import annotations

import json
import random
from dataclasses import asdict, dataclass, field
from typing import Dict, Iterable, List, Mapping, Optional, Sequence, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .towers import TRHashVisionBlock, TRHashVisionTower, TRHashVisionTowerConfig

SENSOR_MODALITIES: Tuple[str, ...] = ("depth", "ir", "thermal", "imu", "radar", "skeleton")
VISUAL_MODALITIES = ("depth", "ir", "thermal")


@dataclass
class TRHashSensorFusionConfig:
    num_classes: int = 40
    hidden_size: int = 256
    num_hidden_layers: int = 4
    num_attention_heads: int = 8
    num_experts: int = 8
    top_k: int = 2
    shared_width: int = 256
    expert_width: int = 128
    route_seed: int = 0x71D5A17
    dropout: float = 0.0
    classifier_dropout: float = 0.1
    visual_channels: Tuple[int, int, int] = (3, 1, 3)   # depth, ir, thermal
    # int g: g x g spatial tokens per clip, averaged over time; (t, h, w):
    # a 3-D lattice of t*h*w tokens over time and space
    visual_token_grid: Union[int, Tuple[int, int, int]] = 4
    # clip layout: "btchw" ([B, T, C, H, W]) or "bcthw" ([B, C, T, H, W], the
    # reference's; the ``Robot`` facade defaults to it)
    visual_layout: str = "btchw"
    vision_image_size: int = 64
    vision_patch_size: int = 8
    vision_hidden_size: int = 128
    vision_layers: int = 2
    vision_heads: int = 4
    vision_num_experts: int = 4
    vision_top_k: int = 2
    vision_shared_width: int = 0     # 0: 2 x vision_hidden_size
    vision_expert_width: int = 0     # 0: max(16, vision_hidden_size // 4)
    # The reference's hierarchical tower splits vision_layers into windowed
    # stages; this tower is one flat stage with global attention over the
    # (small) patch grid, so the split is validated and otherwise unused.
    vision_stage_depths: Tuple[int, ...] = ()
    vision_window_size: int = 0
    precision: str = "bf16"          # fp32 | bf16 | fp16: dtype ``Robot.from_config`` casts to
    layer_norm_eps: float = 1e-5
    late_fusion_weight: float = 0.5
    imu_features: int = 45
    radar_features: int = 16
    skeleton_joints: int = 17
    skeleton_coordinates: int = 3
    sequence_tokens: int = 32
    modality_gate: bool = False   # learned per-sample gate over the stream heads
    structured_encoders: bool = False  # graph encoders for skeleton / 45-channel IMU
    num_subjects: int = 0         # > 0: subject head behind gradient reversal

    def __post_init__(self):
        if not isinstance(self.visual_token_grid, int):
            self.visual_token_grid = tuple(int(v) for v in self.visual_token_grid)
            if len(self.visual_token_grid) != 3 or min(self.visual_token_grid) <= 0:
                raise ValueError("visual_token_grid must be an int or (time, height, width)")
        self.visual_channels = tuple(self.visual_channels)
        self.vision_stage_depths = tuple(self.vision_stage_depths)
        if self.visual_layout not in ("btchw", "bcthw"):
            raise ValueError("visual_layout must be 'btchw' or 'bcthw'")
        if self.precision not in ("fp32", "bf16", "fp16"):
            raise ValueError("precision must be fp32, bf16 or fp16")
        if self.vision_stage_depths and sum(self.vision_stage_depths) != self.vision_layers:
            raise ValueError("vision_layers must equal sum(vision_stage_depths)")
        if not 0 < self.vision_top_k <= self.vision_num_experts:
            raise ValueError("invalid vision expert routing configuration")
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden_size must be divisible by num_attention_heads")

    @property
    def visual_tokens(self) -> int:
        g = self.visual_token_grid
        return g * g if isinstance(g, int) else g[0] * g[1] * g[2]

    @property
    def tokens_per_stream(self) -> int:
        return max(self.visual_tokens, self.sequence_tokens)

    @property
    def route_vocab_size(self) -> int:
        return len(SENSOR_MODALITIES) * self.tokens_per_stream

    # TRHashVisionBlock reads these names
    @property
    def num_heads(self) -> int:
        return self.num_attention_heads

    def to_dict(self) -> dict:
        return asdict(self)


class TRHashSensorFusionBlock(TRHashVisionBlock):
    """Attention over all streams' tokens, then the routed FFN (route id =
    modality index * tokens_per_stream + local position)."""

    def __init__(self, config: TRHashSensorFusionConfig, layer_index: int):
        super().__init__(config, layer_index)


class TRHashSensorFusionClassifier(nn.Module):
    def __init__(self, config: TRHashSensorFusionConfig):
        super().__init__()
        self.config = c = config
        H = c.hidden_size
        # the visual streams share one tower; each stream's channels map to 3
        self.vision = TRHashVisionTower(TRHashVisionTowerConfig(
            image_size=c.vision_image_size, patch_size=c.vision_patch_size, num_channels=3,
            hidden_size=c.vision_hidden_size, num_layers=c.vision_layers,
            num_heads=c.vision_heads, num_experts=c.vision_num_experts, top_k=c.vision_top_k,
            shared_width=c.vision_shared_width or 2 * c.vision_hidden_size,
            expert_width=c.vision_expert_width or max(16, c.vision_hidden_size // 4),
            use_cls_token=False))
        self.visual_in = nn.ModuleDict({m: nn.Conv2d(ch, 3, 1)
                                        for m, ch in zip(VISUAL_MODALITIES, c.visual_channels)})
        self.visual_proj = nn.Linear(c.vision_hidden_size, H)
        self.seq_in = nn.ModuleDict({
            "imu": nn.Linear(c.imu_features, H),
            "radar": nn.Linear(c.radar_features, H),
            "skeleton": nn.Linear(c.skeleton_joints * c.skeleton_coordinates, H)})
        if c.structured_encoders:
            from .sensor_structured import IMUDeviceGraphTokenizer, SkeletonGraphTokenizer

            self.structured = nn.ModuleDict()
            if (c.skeleton_joints, c.skeleton_coordinates) == (17, 3):
                self.structured["skeleton"] = SkeletonGraphTokenizer(17, 3, H, c.sequence_tokens)
            if c.imu_features == 45:
                self.structured["imu"] = IMUDeviceGraphTokenizer(45, H, c.sequence_tokens)
        if c.num_subjects > 0:
            self.subject_head = nn.Linear(H, c.num_subjects)
        self.modality = nn.Embedding(len(SENSOR_MODALITIES), H)
        self.pos = nn.Parameter(torch.randn(1, c.tokens_per_stream, H) * 0.02)
        self.blocks = nn.ModuleList(TRHashSensorFusionBlock(c, i) for i in range(c.num_hidden_layers))
        self.norm = nn.LayerNorm(H, eps=c.layer_norm_eps)
        self.drop = nn.Dropout(c.classifier_dropout)
        self.head = nn.Linear(H, c.num_classes)
        self.stream_heads = nn.ModuleDict({m: nn.Linear(H, c.num_classes) for m in SENSOR_MODALITIES})
        if c.modality_gate:
            self.gate = nn.Linear(H, 1)

    def _visual_tokens(self, m: str, clip: torch.Tensor) -> torch.Tensor:
        """A clip ([B, T, C, H, W], or [B, C, T, H, W] with the "bcthw"
        layout) -> [B, visual_tokens, hidden]."""
        if self.config.visual_layout == "bcthw":
            clip = clip.transpose(1, 2)
        B, T = clip.shape[:2]
        frames = self.visual_in[m](clip.flatten(0, 1).to(self.visual_proj.weight.dtype))
        if frames.shape[-1] != self.config.vision_image_size:
            frames = F.interpolate(frames, size=(self.config.vision_image_size,) * 2,
                                   mode="bilinear", align_corners=False)
        f = self.vision.patch_features(frames)                      # [B*T, D, g, g]
        g = self.config.visual_token_grid
        if isinstance(g, int):
            f = F.adaptive_avg_pool2d(f, g).view(B, T, -1, g * g).mean(1)
        else:   # (time, height, width) lattice
            f = f.view(B, T, *f.shape[1:]).transpose(1, 2)          # [B, D, T, g, g]
            f = F.adaptive_avg_pool3d(f, g).flatten(2)              # [B, D, t*h*w]
        return self.visual_proj(f.transpose(1, 2))

    def _sequence_tokens(self, m: str, seq: torch.Tensor) -> torch.Tensor:
        """[B, T, F] (skeleton [B, T, J, 3]) -> [B, sequence_tokens, hidden]."""
        enc = getattr(self, "structured", None)
        if enc is not None and m in enc:
            return enc[m](seq.to(self.visual_proj.weight.dtype))
        if seq.dim() == 4:
            seq = seq.flatten(2)
        x = self.seq_in[m](seq.to(self.visual_proj.weight.dtype))
        return F.adaptive_avg_pool1d(x.transpose(1, 2), self.config.sequence_tokens).transpose(1, 2)

    def forward(self, inputs: Mapping[str, torch.Tensor],
                labels: Optional[torch.Tensor] = None,
                masks: Optional[Mapping[str, torch.Tensor]] = None,
                subject_adversarial_scale: float = 0.0) -> Dict[str, torch.Tensor]:
        """``inputs``: the streams present in the batch; ``masks`` (optional):
        per-stream [B] bools marking the samples that really have that stream
        (absent samples carry zeros and are masked out of attention, pooling
        and the stream heads).  Every sample needs at least one stream.  With
        ``num_subjects`` > 0, ``subject_logits`` come from the pooled features
        through gradient reversal scaled by ``subject_adversarial_scale``."""
        c = self.config
        toks, ids, spans = [], [], []
        for mi, m in enumerate(SENSOR_MODALITIES):
            x = inputs.get(m)
            if x is None:
                continue
            t = self._visual_tokens(m, x) if m in VISUAL_MODALITIES else self._sequence_tokens(m, x)
            n = t.shape[1]
            t = t + self.modality.weight[mi].to(t.dtype) + self.pos[:, :n].to(t.dtype)
            spans.append((m, sum(s.shape[1] for s in toks), n))
            toks.append(t)
            ids.append(torch.arange(n, device=t.device) + mi * c.tokens_per_stream)
        if not toks:
            raise ValueError(f"no sensor stream given; expected some of {SENSOR_MODALITIES}")
        x = torch.cat(toks, 1)
        B = x.shape[0]
        present = torch.stack([
            (masks[m].to(x.device).bool() if masks is not None and m in masks
             else torch.ones(B, dtype=torch.bool, device=x.device)) for m, _, _ in spans], 1)
        if not bool(present.any(1).all()):
            raise ValueError("every sample must expose at least one sensor stream")
        tok_keep = torch.cat([present[:, i:i + 1].expand(-1, n)
                              for i, (_, _, n) in enumerate(spans)], 1)
        attn = None
        if not bool(tok_keep.all()):
            attn = torch.zeros(B, 1, 1, x.shape[1], device=x.device, dtype=x.dtype)
            attn = attn.masked_fill(~tok_keep[:, None, None, :], float("-inf"))
        route = torch.cat(ids).unsqueeze(0).expand(B, -1)
        for blk in self.blocks:
            x = blk(x, route, attn)
        x = self.norm(x)
        kf = tok_keep.to(x.dtype)[..., None]
        fused = self.head(self.drop((x * kf).sum(1) / kf.sum(1).clamp_min(1)))
        pooled = torch.stack([x[:, s:s + n].mean(1) for _, s, n in spans], 1)   # [B, S, H]
        stream = torch.stack([self.stream_heads[m](pooled[:, i])
                              for i, (m, _, _) in enumerate(spans)], 1)     # [B, S, C]
        if c.modality_gate:
            score = self.gate(pooled).squeeze(-1).float().masked_fill(~present, float("-inf"))
            weights = score.softmax(1)
        else:
            weights = present.float() / present.float().sum(1, keepdim=True)
        per = (stream.float() * weights[..., None]).sum(1).to(fused.dtype)
        w = c.late_fusion_weight
        logits = (1 - w) * fused + w * per
        full = torch.zeros(B, len(SENSOR_MODALITIES), c.num_classes, device=x.device,
                           dtype=stream.dtype)
        full_w = torch.zeros(B, len(SENSOR_MODALITIES), device=x.device)
        full_mask = torch.zeros(B, len(SENSOR_MODALITIES), dtype=torch.bool, device=x.device)
        for i, (m, _, _) in enumerate(spans):
            j = SENSOR_MODALITIES.index(m)
            full[:, j], full_w[:, j], full_mask[:, j] = stream[:, i], weights[:, i], present[:, i]
        out = {"logits": logits, "fused_logits": fused, "stream_logits": per,
               "modality_logits": full, "modality_weights": full_w, "modality_mask": full_mask,
               "features": (x * kf).sum(1) / kf.sum(1).clamp_min(1)}
        if c.num_subjects > 0:
            from .sensor_structured import gradient_reverse

            out["subject_logits"] = self.subject_head(
                gradient_reverse(out["features"], subject_adversarial_scale))
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels)
        return out


def load_pretrained_visual_tower(model: TRHashSensorFusionClassifier,
                                 tower_state: Mapping[str, torch.Tensor], strict: bool = False):
    """Initialise the shared visual tower from a vision checkpoint's tower weights
    (keys with or without a ``tower.`` prefix); returns the load result."""
    sd = {k[len("tower."):] if k.startswith("tower.") else k: v for k, v in tower_state.items()}
    own = model.vision.state_dict()
    sd = {k: v for k, v in sd.items() if k in own and own[k].shape == v.shape}
    return model.vision.load_state_dict(sd, strict=strict)


# ------------------------------------------------------------- data splits
@dataclass(frozen=True)
class CrossSubjectFold:
    name: str
    train_subjects: Tuple[int, ...]
    val_subjects: Tuple[int, ...]


def make_cross_subject_folds(subjects: Sequence[int], k: int) -> List[CrossSubjectFold]:
    """``k`` folds over sorted subjects; fold i validates on every k-th subject
    starting at i, so each subject is validated exactly once."""
    s = sorted(set(subjects))
    out = []
    for i in range(k):
        val = tuple(s[i::k])
        out.append(CrossSubjectFold(f"fold{i}", tuple(x for x in s if x not in val), val))
    return out


def validate_cross_subject_folds(folds: Sequence[CrossSubjectFold]) -> None:
    seen = set()
    for f in folds:
        if set(f.train_subjects) & set(f.val_subjects):
            raise ValueError(f"{f.name}: a subject is in both train and validation")
        if set(f.val_subjects) & seen:
            raise ValueError(f"{f.name}: a subject is validated by two folds")
        seen |= set(f.val_subjects)


def resolve_cross_subject_fold(name: str, folds: Sequence[CrossSubjectFold]) -> CrossSubjectFold:
    for f in folds:
        if f.name == name:
            return f
    raise KeyError(f"unknown fold {name!r}; known: {[f.name for f in folds]}")


@dataclass
class SensorRecord:
    """One labelled sample: per-modality tensor files (``.pt``), label, subject."""
    files: Dict[str, str]
    label: int
    subject: int
    meta: Dict[str, str] = field(default_factory=dict)


def save_sensor_manifest(records: Iterable[SensorRecord], path: str) -> None:
    with open(path, "w") as f:
        json.dump([asdict(r) for r in records], f, indent=1)


def load_sensor_manifest(path: str) -> List[SensorRecord]:
    with open(path) as f:
        return [SensorRecord(**d) for d in json.load(f)]


def subject_disjoint_records(records: Sequence[SensorRecord], val_fraction: float = 0.2,
                             seed: int = 0) -> Tuple[List[SensorRecord], List[SensorRecord]]:
    """Split so that no subject appears on both sides."""
    subjects = sorted({r.subject for r in records})
    rng = random.Random(seed)
    rng.shuffle(subjects)
    n_val = max(1, round(len(subjects) * val_fraction)) if len(subjects) > 1 else 0
    val = set(subjects[:n_val])
    return [r for r in records if r.subject not in val], [r for r in records if r.subject in val]


class SensorDataset(torch.utils.data.Dataset):
    def __init__(self, records: Sequence[SensorRecord]):
        self.records = list(records)

    def __len__(self):
        return len(self.records)

    def __getitem__(self, i):
        r = self.records[i]
        x = {m: torch.load(p, weights_only=True) for m, p in r.files.items()}
        return x, r.label


def collate_sensors_masked(samples: Sequence):
    """-> (inputs, masks, labels): every stream present in ANY sample is stacked,
    zero-filled where a sample lacks it, with a per-sample presence mask."""
    names = [m for m in SENSOR_MODALITIES if any(m in s[0] for s in samples)]
    inputs, masks = {}, {}
    for m in names:
        ref = next(s[0][m] for s in samples if m in s[0])
        inputs[m] = torch.stack([s[0][m] if m in s[0] else torch.zeros_like(ref)
                                 for s in samples])
        masks[m] = torch.tensor([m in s[0] for s in samples])
    return inputs, masks, torch.tensor([s[1] for s in samples], dtype=torch.long)


def collate_sensors(samples: Sequence) -> Tuple[Dict[str, torch.Tensor], torch.Tensor]:
    """Stacks each modality present in every sample of the batch."""
    common = set.intersection(*(set(s[0]) for s in samples))
    batch = {m: torch.stack([s[0][m] for s in samples]) for m in sorted(common)}
    return batch, torch.tensor([s[1] for s in samples], dtype=torch.long)
