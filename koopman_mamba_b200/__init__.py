"""koopman_mamba_b200: the Spectral Koopman Attention (SKA) core of Koopman_Mamba
as hand-written sm_100a CUDA kernels behind a C ABI (``include/ska_b200.h``),
with a drop-in ``SKAModule`` for the reference's ``koopman_lm.ska.SKAModule``.
"""
from .ska import SKAModule, SkaCoreFunction, ska_core  # noqa: F401

__all__ = ["SKAModule", "SkaCoreFunction", "ska_core"]
