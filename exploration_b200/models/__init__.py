"""Model families: the Stack LM and the dense Transformer baseline."""
from .baseline import BaselineBlock, BaselineModel
from .blocks import FeedForward, HaloMemoryBlock, KVProjection, RotaryEmbedding
from .stack import GlobalReadBlock, StackModel, parse_arch

__all__ = ["BaselineBlock", "BaselineModel", "FeedForward", "HaloMemoryBlock", "KVProjection",
           "RotaryEmbedding", "GlobalReadBlock", "StackModel", "parse_arch"]
