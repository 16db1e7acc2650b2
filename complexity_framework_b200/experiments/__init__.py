"""Research modules outside the TR-GQA / TR-MHA models (counterpart of
complexity/experiments): token-addressed fast-weight memories."""
from .associative import (CollisionNormalizedDeltaAttention,
                          CollisionNormalizedLexicalForgeDeltaAttention, FastWeightMemory,
                          LexicalForgeDeltaAttention, LexicalValueDeltaAttention,
                          MultiOrderLexicalDeltaAttention, MultiTimescaleDeltaAttention,
                          PositionAwareCollisionForgeDeltaAttention, SharedAssociativeAttention,
                          SharedContextFusion, StableDeltaAssociativeAttention, chunk_scan)

__all__ = ["FastWeightMemory", "chunk_scan", "SharedAssociativeAttention", "SharedContextFusion",
           "StableDeltaAssociativeAttention", "MultiOrderLexicalDeltaAttention",
           "MultiTimescaleDeltaAttention", "CollisionNormalizedDeltaAttention",
           "LexicalValueDeltaAttention", "LexicalForgeDeltaAttention",
           "CollisionNormalizedLexicalForgeDeltaAttention",
           "PositionAwareCollisionForgeDeltaAttention"]
