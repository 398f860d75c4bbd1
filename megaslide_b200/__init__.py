"""megaslide_b200 — B200-native (sm_100a) 3D Deformable Slide Attention for MegaSlide-DiT.

``DeformableSlideAttention3D`` is a drop-in for ``infinity.video.attention.DeformableSlideAttention3D``
(same constructor, forward signature and parameter names) whose forward and backward run on the
hand-written kernels of ``libmegaslide_b200.so`` (C ABI in ``include/megaslide_b200.h``).
"""

from . import ops
from .ops import check_status
from ._lib import MslError, launch_count, library_path
from .attention import DeformableSlideAttention3D, DSA3DFunction

__all__ = ["DeformableSlideAttention3D", "DSA3DFunction", "MslError", "ops", "launch_count", "library_path",
           "check_status"]
__version__ = "0.1.0"
