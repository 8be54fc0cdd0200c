"""Model-agnostic drafter losses (reference: losses/__init__.py:10-12).

    from losses import dpace_loss, fused_dpace_loss
"""
from losses.dpace import dpace_loss, fused_dpace_loss

__all__ = ["dpace_loss", "fused_dpace_loss"]
