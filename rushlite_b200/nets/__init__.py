from . import layers
from .Module import Module

__all__ = ["Module", "layers"]
