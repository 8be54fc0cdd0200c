"""B200 runtime for the fused drafter losses.

    specdec._lib   ctypes binding of libspecdec.so (include/specdec.h)
    specdec.ops    tensor-level calls into the C ABI
    specdec.dist   N-sharded losses over torch.distributed (NCCL / gloo)
    specdec.drafter  the DFlash drafter's RMSNorm and attention kernels
    specdec.graphs   a whole training step captured as one CUDA graph

The reference-facing API lives beside this package, under the reference's own
module names: ``losses.dpace`` (dpace_loss, fused_dpace_loss) and
``models.dflash`` (dflash_loss, fused_dflash_loss, dflash_objective,
DFlashSpeculator.compute_loss).
"""
from . import _lib, ops  # noqa: F401
from .ops import set_target_validation  # noqa: F401

__all__ = ["ops", "set_target_validation"]
