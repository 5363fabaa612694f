"""B200-native (sm_100a) sparse-MoE layer forward for Noor's noor-core path.

The compute lives in libnoor_moe.so (csrc/, C ABI in include/noor_moe.h);
`api` binds it with ctypes and mirrors the reference's layer classes;
`workloads` draws the seeded synthetic layers the tests and bench use.
"""
from . import workloads  # noqa: F401
from . import api  # noqa: F401
from . import gguf  # noqa: F401
from . import stack  # noqa: F401
from .api import (ExpertUtilization, GeGLUFFN, Handle, MoELayer, MoERouter, NoorMoEError,  # noqa: F401
                  ParallelFFN, RMSNorm, RouteResult, SandwichNorm, SMEBU, SwiGLUFFN, ffn_sublayer_forward,
                  matmul_f32)
