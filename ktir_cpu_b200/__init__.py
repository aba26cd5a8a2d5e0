"""B200 execution backend for KTIR (Kernel Tile IR) kernels.

Drop-in for the ktir-cpu interpreter's execution path: same
``KTIRInterpreter`` API, execution lowered onto hand-written sm_100a kernels
through the C ABI in include/ktir_b200.h (libktir_b200.so).
"""

from .interpreter import KTIRInterpreter
from .latency import HardwareConfig, LatencyCategory, LatencyReport
from .parser import KTIRParser, KTIRParserBase

__all__ = ["KTIRInterpreter", "KTIRParser", "KTIRParserBase", "HardwareConfig",
           "LatencyCategory", "LatencyReport"]
