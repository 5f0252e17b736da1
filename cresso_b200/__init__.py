"""B200-native CRESSO5 optimizer step.

``cresso_b200.CRESSO5`` is a drop-in for ``cresso_v5.CRESSO5`` whose step runs
as hand-written sm_100a CUDA kernels behind a C ABI (``include/cresso_b200.h``).
"""

from .optim import CRESSO, CRESSO5, count_optimizer_state_elements, theoretical_state_elements

__all__ = ["CRESSO5", "CRESSO", "count_optimizer_state_elements", "theoretical_state_elements"]
__version__ = "0.1.0"
