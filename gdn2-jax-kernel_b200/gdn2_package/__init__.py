"""gdn2_package — Gated DeltaNet-2 chunked forward and fused backward on B200.

Drop-in for the package of Akseleu-J/gdn2-jax-kernel: the same entry points
(``gdn2_pallas_forward``, ``gdn2_pallas_forward_trainable``), the same module
constants (``gdn2_fwd.BT``/``BC``/``CLIP``) and the same (B, T, H, D) tensor
conventions, executed by hand-written sm_100a kernels in libgdn2.so.
"""
__version__ = "0.2.0"

from .gdn2_fwd import gdn2_pallas_forward, gdn2_pallas_forward_with_residuals  # noqa: E402,F401
from .gdn2_pipeline import gdn2_pallas_forward_trainable  # noqa: E402,F401
from .gdn2_bwd import gdn2_backward  # noqa: E402,F401
from . import gdn2_fwd, gdn2_bwd, gdn2_pipeline  # noqa: E402,F401
from . import sequence_parallel  # noqa: E402,F401
from .gdn2_decode import gdn2_decode  # noqa: E402,F401
from .streaming import gdn2_fwd_bwd  # noqa: E402,F401
from .segmented import gdn2_segmented_forward_trainable  # noqa: E402,F401
