"""Command-line interface (``python -m complexity_framework_b200.cli`` / ``cfb``)."""
from .app import main

__all__ = ["main"]
