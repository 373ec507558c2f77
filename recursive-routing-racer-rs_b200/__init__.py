"""B200 (sm_100a) weight path of Recursive Routing Racer (Peterc3-dev/recursive-routing-racer-rs):
raw-block Q4_K/Q5_K/Q6_K GEMV, batched tensor-core GEMM, RMSNorm and F32 logits kernels
behind the C ABI of include/rrr_cuda.h, with host mirrors of the reference's dispatch API
(engine.py), GGUF loader (gguf.py) and decode step (phi4.py).

The directory name is not a Python identifier; import it with
`importlib.import_module("recursive-routing-racer-rs_b200")`.
"""
from . import ffi  # noqa: F401
from .engine import ComputeEngine, GpuBuffer, QType, gpu_matmul_f32, gpu_matmul_kquant, \
    gpu_rmsnorm, kquant_dispatch, push_u32  # noqa: F401
from .ffi import Context, RRRError  # noqa: F401
from .gguf import GGUFModel, TensorInfo  # noqa: F401
from .phi4 import ModelConfig, Phi4Decoder, SyntheticPhi4  # noqa: F401


def build(verbose: bool = False) -> str:
    from .build import build as _b
    return _b(verbose)
