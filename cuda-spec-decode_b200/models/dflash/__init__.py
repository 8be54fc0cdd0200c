"""DFlash block drafter and its fused objective (reference: models/dflash/__init__.py:5-15).

    from models.dflash import DFlashSpeculator, dflash_loss
"""
from models.dflash.loss import dflash_loss, dflash_objective, fused_dflash_loss
from models.dflash.model import DFlashAttention, DFlashSpeculator, DFlashTransformerLayer

__all__ = [
    "DFlashSpeculator",
    "DFlashAttention",
    "DFlashTransformerLayer",
    "dflash_loss",
    "dflash_objective",
    "fused_dflash_loss",
]
