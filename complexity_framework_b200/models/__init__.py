from .block import TransformerBlock
from .builder import ComplexityModel

__all__ = ["ComplexityModel", "TransformerBlock"]
