"""Graph-structured sequence encoders for the sensor-fusion classifier, and
gradient reversal for subject-adversarial training.

Counterpart of complexity/generative/sensor_fusion/structured_encoders.py:12-187
(``SkeletonGraphTokenizer``, ``IMUDeviceGraphTokenizer``) and
complexity/generative/sensor_fusion/model.py:28-42 (``gradient_reverse``).

A flat linear projection of a skeleton ([T, 17 joints, 3]) or of 45 IMU
channels (5 devices x 9) throws away which values belong together.  These
encoders keep one feature vector per node (joint or device) through the
stack: each block mixes neighbouring nodes over the fixed sensor graph
(symmetrically normalised adjacency with self loops), then filters every
node's trajectory along time with a dilated depthwise convolution; both
residual branches start near zero (learned scales of 1e-3) so a fresh
encoder passes its input projection through.  A learned score per node
pools nodes, and adaptive average pooling over time gives ``token_count``
tokens of ``hidden_size``.

Inputs carry motion explicitly: skeleton positions plus per-frame velocity,
IMU raw readings plus per-clip centred readings plus velocity.
"""
from __future__ import annotations

from typing import Iterable, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class _GradReverse(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale):
        ctx.scale = float(scale)
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return g * -ctx.scale, None


def gradient_reverse(values: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """Identity forward; the backward multiplies the gradient by ``-scale``
    (a head trained through it pushes the encoder to remove what it predicts)."""
    return _GradReverse.apply(values, scale)


def graph_adjacency(nodes: int, edges: Iterable[Tuple[int, int]]) -> torch.Tensor:
    """D^-1/2 (A + I) D^-1/2 of an undirected graph."""
    a = torch.eye(nodes)
    for i, j in edges:
        a[i, j] = a[j, i] = 1.0
    d = a.sum(1).rsqrt()
    return d[:, None] * a * d[None, :]


class _GraphTemporalBlock(nn.Module):
    def __init__(self, width: int, dilation: int, kernel: int = 5):
        super().__init__()
        self.mix_norm = nn.LayerNorm(width)
        self.mix = nn.Linear(width, width, bias=False)
        self.mix_scale = nn.Parameter(torch.tensor(1e-3))
        self.time_norm = nn.LayerNorm(width)
        self.time_dw = nn.Conv1d(width, width, kernel, padding=dilation * (kernel // 2),
                                 dilation=dilation, groups=width, bias=False)
        self.time_mlp = nn.Sequential(nn.Linear(width, 2 * width), nn.GELU(),
                                      nn.Linear(2 * width, width))
        self.time_scale = nn.Parameter(torch.tensor(1e-3))

    def forward(self, x: torch.Tensor, adj: torch.Tensor) -> torch.Tensor:
        # x [B, T, N, C]
        nb = torch.matmul(adj.to(x.dtype), self.mix_norm(x))          # neighbours, per frame
        x = x + self.mix_scale * self.mix(nb)
        B, T, N, C = x.shape
        h = self.time_norm(x).permute(0, 2, 3, 1).reshape(B * N, C, T)  # node trajectories
        h = self.time_dw(h).reshape(B, N, C, T).permute(0, 3, 1, 2)
        return x + self.time_scale * self.time_mlp(h)


class _GraphSequenceEncoder(nn.Module):
    """[B, T, nodes, node_features] -> [B, token_count, hidden_size]."""

    def __init__(self, nodes: int, node_features: int, hidden_size: int, token_count: int,
                 edges: Sequence[Tuple[int, int]], dilations: Sequence[int] = (1, 2, 4, 8)):
        super().__init__()
        width = max(64, hidden_size // 2)
        self.nodes, self.node_features, self.token_count = nodes, node_features, token_count
        self.input_projection = nn.Linear(node_features, width)
        self.node_embedding = nn.Parameter(torch.randn(nodes, width) * 0.02)
        self.blocks = nn.ModuleList(_GraphTemporalBlock(width, d) for d in dilations)
        self.node_score = nn.Linear(width, 1)
        self.output_projection = nn.Linear(width, hidden_size)
        self.register_buffer("adjacency", graph_adjacency(nodes, edges))

    def encode_nodes(self, feats: torch.Tensor) -> torch.Tensor:
        if feats.dim() != 4 or tuple(feats.shape[-2:]) != (self.nodes, self.node_features):
            raise ValueError(f"expected [batch, time, {self.nodes}, {self.node_features}], "
                             f"got {tuple(feats.shape)}")
        x = self.input_projection(feats) + self.node_embedding
        for blk in self.blocks:
            x = blk(x, self.adjacency)
        w = self.node_score(x).softmax(2)                                # pool nodes
        x = (x * w).sum(2)                                               # [B, T, C]
        x = F.adaptive_avg_pool1d(x.transpose(1, 2), self.token_count).transpose(1, 2)
        return self.output_projection(x)


def _velocity(x: torch.Tensor) -> torch.Tensor:
    """Frame-to-frame difference along dim 1 (zero at the first frame)."""
    return torch.cat([torch.zeros_like(x[:, :1]), x[:, 1:] - x[:, :-1]], 1)


class SkeletonGraphTokenizer(_GraphSequenceEncoder):
    """17-joint skeletons on the Human3.6M kinematic tree (pelvis 0; right
    leg 1-3; left leg 4-6; spine 7, thorax 8, neck 9, head 10; left arm
    11-13; right arm 14-16); joint features = position and velocity."""

    EDGES = ((0, 1), (1, 2), (2, 3), (0, 4), (4, 5), (5, 6), (0, 7), (7, 8), (8, 9), (9, 10),
             (8, 11), (11, 12), (12, 13), (8, 14), (14, 15), (15, 16))

    def __init__(self, num_joints: int, coordinates: int, hidden_size: int, token_count: int):
        if (num_joints, coordinates) != (17, 3):
            raise ValueError("the skeleton graph encoder takes 17 joints in 3-D")
        super().__init__(num_joints, 2 * coordinates, hidden_size, token_count, self.EDGES)
        self.coordinates = coordinates

    def forward(self, joints: torch.Tensor) -> torch.Tensor:
        if joints.dim() != 4 or tuple(joints.shape[-2:]) != (self.nodes, self.coordinates):
            raise ValueError(f"skeleton must be [batch, time, {self.nodes}, {self.coordinates}]")
        return self.encode_nodes(torch.cat([joints, _velocity(joints)], -1))


class IMUDeviceGraphTokenizer(_GraphSequenceEncoder):
    """Five wearable IMUs of nine channels each (45 inputs), device 2 the hub
    joined to the other four; device features = raw, clip-centred, velocity."""

    DEVICES = 5
    FEATURES_PER_DEVICE = 9
    EDGES = ((2, 0), (2, 1), (2, 3), (2, 4))

    def __init__(self, input_features: int, hidden_size: int, token_count: int):
        if input_features != self.DEVICES * self.FEATURES_PER_DEVICE:
            raise ValueError("the IMU graph encoder takes 5 devices x 9 features = 45 inputs")
        super().__init__(self.DEVICES, 3 * self.FEATURES_PER_DEVICE, hidden_size, token_count,
                         self.EDGES)

    def forward(self, imu: torch.Tensor) -> torch.Tensor:
        if imu.dim() != 3 or imu.shape[-1] != self.DEVICES * self.FEATURES_PER_DEVICE:
            raise ValueError("IMU must be [batch, time, 45]")
        d = imu.reshape(imu.shape[0], imu.shape[1], self.DEVICES, self.FEATURES_PER_DEVICE)
        return self.encode_nodes(torch.cat([d, d - d.mean(1, keepdim=True), _velocity(d)], -1))


__all__ = ["IMUDeviceGraphTokenizer", "SkeletonGraphTokenizer", "gradient_reverse",
           "graph_adjacency"]
