"""B200-native tensor/sequence-parallel GPT training and GemmRS overlap framework.

Capabilities follow TempName-5090 (four GemmRS arms, TACO FP8 codec, arrival
plans, TP/SP GPT with its sharded state_dict layout), re-designed for sm_100a:
tcgen05/TMEM GEMMs fed by TMA, epilogues that push tiles to their owner GPU
over NVLink with per-tile readiness flags, and hand-written kernels for every
hot op.  Importing this package never requires a GPU; CUDA entry points fail
loudly when the native extension is missing on a CUDA machine.
"""
__version__ = "0.1.0"

from . import config  # noqa: F401

__all__ = ["config", "__version__"]
