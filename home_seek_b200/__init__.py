"""home_seek_b200 — the MTP speculative-decode MoE step of home-seek on B200.

Host layer (Python/PyTorch) over libhs_ext.so, a C-ABI library of hand-written
sm_100a CUDA kernels: router + hash routing, the routed FP4 expert FFN with the
FP8 shared expert fused in, permute/unpermute, and speculative acceptance.
The operator surface mirrors the reference (FusedMoEFFN.forward, the router,
_load_expert_weights, acceptance, the MTP draft/verify step); there is no CPU
or Triton fallback.
"""
from ._lib import HsError  # noqa: F401

__version__ = "0.1.0"
