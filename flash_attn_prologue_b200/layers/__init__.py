from .FusedQKV import FusedQKV
from .RMSNorm import RMSNormRoPEScale

__all__ = ["FusedQKV", "RMSNormRoPEScale"]
