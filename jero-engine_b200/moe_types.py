"""Plain-Python types shared by the binding (jeromoe.py) and the synthetic
layer builder (synth.py): status codes and the exceptions named after the
K3Error variants they map to, GGUF quant ids, and the tensor containers that
play the role of jero_core::TensorView / ModelWeights.

Importing this module loads no native library.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import numpy as np

# status codes (include/jeromoe.h moe_status)
MOE_OK = 0
MOE_ERR_INVALID_ARGS = 2
MOE_ERR_CAPABILITY_MISMATCH = 10
MOE_ERR_INSUFFICIENT_MEMORY = 11
MOE_ERR_RESOURCE_EXHAUSTED = 12
MOE_ERR_TENSOR_BOUNDS = 14
MOE_ERR_CONTEXT_LENGTH = 15
MOE_ERR_NOT_UPLOADED = 16
MOE_ERR_CUDA = 20
MOE_ERR_NCCL = 21
MOE_ERR_TIMEOUT = 22

F32, Q8_0, Q4_K = 0, 8, 12
QUANT_NAMES = {F32: "F32", Q8_0: "Q8_0", Q4_K: "Q4_K"}
ROUTE_SOFTMAX_TOPK, ROUTE_GROUP_LIMITED = 0, 1


class MoeError(RuntimeError):
    code = -1

    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class InvalidArguments(MoeError): pass
class CapabilityMismatch(MoeError): pass
class InsufficientLockableMemory(MoeError): pass
class ResourceExhausted(MoeError): pass
class TensorBoundsError(MoeError): pass
class ContextLengthExceeded(MoeError): pass
class NotUploaded(MoeError): pass
class CudaError(MoeError): pass
class NcclError(MoeError): pass
class DeviceTimeout(MoeError): pass


ERRORS = {
    MOE_ERR_INVALID_ARGS: InvalidArguments,
    MOE_ERR_CAPABILITY_MISMATCH: CapabilityMismatch,
    MOE_ERR_INSUFFICIENT_MEMORY: InsufficientLockableMemory,
    MOE_ERR_RESOURCE_EXHAUSTED: ResourceExhausted,
    MOE_ERR_TENSOR_BOUNDS: TensorBoundsError,
    MOE_ERR_CONTEXT_LENGTH: ContextLengthExceeded,
    MOE_ERR_NOT_UPLOADED: NotUploaded,
    MOE_ERR_CUDA: CudaError,
    MOE_ERR_NCCL: NcclError,
    MOE_ERR_TIMEOUT: DeviceTimeout,
}


def gguf_row_bytes(quant: int, cols: int) -> int:
    """GGUF bytes of one row of cols values (0 if cols is not whole blocks)."""
    if cols <= 0:
        return 0
    if quant == F32:
        return cols * 4
    if quant == Q8_0:
        return 0 if cols % 32 else cols // 32 * 34
    if quant == Q4_K:
        return 0 if cols % 256 else cols // 256 * 144
    return 0


@dataclass
class Tensor:
    """A GGUF tensor: raw bytes + quant + GGUF shape (jero_core::TensorView)."""
    quant: int
    shape: Sequence[int]
    data: np.ndarray  # uint8 (or float32 for F32) C-contiguous


def f32_tensor(values: np.ndarray, shape: Sequence[int]) -> Tensor:
    return Tensor(F32, list(shape), np.ascontiguousarray(values, dtype=np.float32))


class ModelWeights:
    """Name -> Tensor map, the role of jero_core::ModelWeights in the reference."""

    def __init__(self, tensors: Optional[Dict[str, Tensor]] = None):
        self.tensors: Dict[str, Tensor] = dict(tensors or {})

    def contains_tensor(self, name: str) -> bool:
        return name in self.tensors

    def tensor(self, name: str) -> Tensor:
        if name not in self.tensors:
            raise TensorBoundsError(MOE_ERR_TENSOR_BOUNDS, f"tensor '{name}' not present")
        return self.tensors[name]

    def tensor_count(self) -> int:
        return len(self.tensors)

    def total_weight_bytes(self) -> int:
        return sum(t.data.nbytes for t in self.tensors.values())

    def insert(self, name: str, t: Tensor):
        self.tensors[name] = t


@dataclass
class RouteSpec:
    mode: int = ROUTE_SOFTMAX_TOPK
    normalize: bool = True
    n_groups: int = 0
    topk_groups: int = 0
    routed_scale: float = 1.0
