"""motoria_b200: B200 (sm_100a) MoE FFN block for the motorIa engine.

The product is libmiag.so (C ABI, include/miag/miag.h) built from csrc/ by
``python -m motoria_b200.build``; this package is its host-side mirror of the
reference interface (engine.py) plus seeded synthetic inputs (synth.py).
"""

from . import synth  # noqa: F401
from .engine import (MIA_F32, MIA_Q8_0, PREFILL_MMA, PREFILL_TCGEN05, MoEEngine,  # noqa: F401
                     blob_bytes, matvec, quantize_row_q8)

__all__ = ["MoEEngine", "blob_bytes", "matvec", "quantize_row_q8", "MIA_F32", "MIA_Q8_0",
           "PREFILL_MMA", "PREFILL_TCGEN05", "synth"]
