"""nexus_b200 -- B200 (sm_100a) CUDA backend for the Nexus quantized decode path.

The product is ``libnexus_cuda.so`` (C ABI in ``include/nexus_cuda.h``); this
package is its Python binding and the reference-shaped engine surface.
"""
from . import _lib
from ._lib import (BF16, F16, F32, FORMAT_IDS, FORMAT_NAMES, Q2_K, Q4_0, Q4_K, Q8_0, NexusError)
from .engine import (BackendCapabilities, CudaBackend, InferenceEngine, MemoryInfo, QWeight,
                     cuda_capabilities, quantize_host, tp_plan, tp_unique_id, write_synthetic_model)
from .configs import CONFIGS, model_path
from .scheduler import ContinuousBatcher, KvPageAllocation, ScheduledDecode, Scheduler, ServeEvent

__all__ = ["_lib", "F32", "F16", "BF16", "Q4_0", "Q8_0", "Q2_K", "Q4_K", "FORMAT_IDS", "FORMAT_NAMES",
           "NexusError", "BackendCapabilities", "CudaBackend", "InferenceEngine", "MemoryInfo", "QWeight",
           "cuda_capabilities", "quantize_host", "tp_plan", "tp_unique_id", "write_synthetic_model", "CONFIGS",
           "model_path", "Scheduler", "ScheduledDecode", "KvPageAllocation", "ContinuousBatcher", "ServeEvent"]
