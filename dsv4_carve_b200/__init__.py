"""B200-native (sm_100a) EXL3 decode hot path: trellis dequant, dense EXL3
linear (GEMV form) and the routed-MoE decode layer, behind the reference's
``vllm_exl3_c`` entry points.  See include/exl3_b200.h for the C ABI."""
from . import _lib  # noqa: F401

__all__ = ["vllm_exl3_c", "linear", "moe", "synth"]
