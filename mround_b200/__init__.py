"""mround_b200: a B200-native SignRound v2 block-tuning path.

A drop-in for MRound's hot path (fbaldassarri/mround 0.1.0a6): the public
objects keep their names and meaning (``QuantScheme``, ``TuningConfig``,
``api.quantize``), while the arithmetic runs in hand-written sm_100a kernels
of ``libmround_b200.so`` behind a C ABI (``include/mround_b200.h``).
"""

from mround_b200.exceptions import MRoundError, SchemeError
from mround_b200.schemes import QuantScheme, ScaleInit, Symmetry, TuningConfig

__version__ = "0.1.0"

__all__ = ["MRoundError", "QuantScheme", "ScaleInit", "SchemeError", "Symmetry", "TuningConfig",
           "__version__"]
