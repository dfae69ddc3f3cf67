"""nn.Module wrappers (mirrors the reference's Ops/ package)."""
from .sparse_conv2d import SparseConv2d
from .sparse_fused_conv_lif import FusedSparseConvLIF
from .lif_node import LIFNode

__all__ = ["SparseConv2d", "FusedSparseConvLIF", "LIFNode"]
