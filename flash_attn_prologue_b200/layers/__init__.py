from .RMSNorm import RMSNormRoPEScale

__all__ = ["RMSNormRoPEScale"]
