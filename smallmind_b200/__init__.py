"""SmallMind.Cuda — B200-native (sm_100a) quantized decode/prefill path for SmallMind.

The product is ``libsmallmind_cuda.so`` (C-ABI: include/smallmind_cuda.h).  This
package is its host-side mirror of the reference operator API; it has no CPU
compute path.
"""
from ._lib import (LAYOUT_INTENDED, LAYOUT_REFERENCE, PTR_DEVICE, PTR_HOST, ShapeError, SmallMindCudaError,
                   last_error, lib)
from .api import (ChatSession, CudaContext, CudaModel, CudaWeightTensor, DeterministicRng, InferenceSession, KVCache,
                  QuantScheme, SamplingOptions, attention, longest_common_prefix, rmsnorm, rope, sample, silu_mul)

__all__ = [
    "ChatSession", "longest_common_prefix", "DeterministicRng", "SamplingOptions", "sample", "CudaContext", "CudaModel", "CudaWeightTensor", "InferenceSession", "KVCache", "QuantScheme", "attention",
    "rmsnorm", "rope", "silu_mul", "LAYOUT_INTENDED", "LAYOUT_REFERENCE", "PTR_HOST", "PTR_DEVICE", "ShapeError",
    "SmallMindCudaError", "last_error", "lib",
]
