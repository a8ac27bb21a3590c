"""Python binding of libjeromoe.so (include/jeromoe.h) over ctypes.

The library is the product; this module only marshals arguments. Every call
goes to the CUDA path, and a missing or unloadable library raises at import
(there is no CPU fallback).

Names follow the reference: tensors are addressed by their GGUF names
(blk.{L}.ffn_gate_inp.weight, blk.{L}.ffn_{gate,up,down}_exps.weight, ...) with
GGUF shapes [in, out(, experts)], and failures raise MoeError subclasses named
after the K3Error variants of jero-core that the status codes map to.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjeromoe.so")

# ---------------------------------------------------------------- constants
# status codes, quant ids, the K3Error-named exceptions and the GGUF tensor
# containers are plain Python (moe_types); re-exported here
from moe_types import (  # noqa: F401,E402
    MOE_OK, MOE_ERR_INVALID_ARGS, MOE_ERR_CAPABILITY_MISMATCH, MOE_ERR_INSUFFICIENT_MEMORY,
    MOE_ERR_RESOURCE_EXHAUSTED, MOE_ERR_TENSOR_BOUNDS, MOE_ERR_CONTEXT_LENGTH, MOE_ERR_NOT_UPLOADED, MOE_ERR_CUDA,
    MOE_ERR_NCCL, MOE_ERR_TIMEOUT, F32, Q8_0, Q4_K, QUANT_NAMES, ROUTE_SOFTMAX_TOPK, ROUTE_GROUP_LIMITED, MoeError,
    InvalidArguments, CapabilityMismatch, InsufficientLockableMemory, ResourceExhausted, TensorBoundsError,
    ContextLengthExceeded, NotUploaded, CudaError, NcclError, DeviceTimeout, Tensor, f32_tensor, ModelWeights,
    RouteSpec, ERRORS as _ERRORS)

PTR_HOST, PTR_DEVICE = 0, 1
FLAG_TENSOR_CORES_ALWAYS, FLAG_TENSOR_CORES_NEVER = 1, 2
FLAG_EP_NCCL_ONLY = 4   # expert parallelism: NCCL exchange for every batch size
# small batches: int8 weight-streaming kernels only / int8 tensor cores for every size below the f16 path
FLAG_INT8_TENSOR_CORES_NEVER, FLAG_INT8_TENSOR_CORES_ALWAYS = 8, 16
FLAG_FUSED_TC_NEVER = 32   # small batches: no fused tensor-core expert launch
FLAG_FUSED_I8_NEVER, FLAG_FUSED_I8_ALWAYS = 64, 128   # the fused launch's f16 / int8 form
TENSOR_CORE_MIN_TOKENS = 256

# ------------------------------------------------------------------- structs


class moe_tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("nbytes", C.c_uint64), ("quant", C.c_int32),
                ("n_dims", C.c_int32), ("shape", C.c_int64 * 4)]


class moe_layer_desc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
                ("expert_ffn_dim", C.c_int32), ("use_shared_expert", C.c_int32),
                ("route_mode", C.c_int32), ("normalize", C.c_int32), ("n_groups", C.c_int32),
                ("topk_groups", C.c_int32), ("routed_scale", C.c_float),
                ("router", moe_tensor), ("exp_probs_b", moe_tensor), ("logit_bias", moe_tensor),
                ("gate_exps", moe_tensor), ("up_exps", moe_tensor), ("down_exps", moe_tensor),
                ("gate_shexp", moe_tensor), ("up_shexp", moe_tensor), ("down_shexp", moe_tensor)]


class moe_device_spec(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_tokens", C.c_int32), ("max_layers", C.c_int32),
                ("flags", C.c_int32), ("reserve_bytes", C.c_uint64)]


class moe_mem_inspector(C.Structure):
    _fields_ = [("free_bytes", C.c_uint64), ("total_bytes", C.c_uint64)]


class moe_footprint(C.Structure):
    _fields_ = [("weight_bytes", C.c_uint64), ("scratch_bytes", C.c_uint64),
                ("total_required_bytes", C.c_uint64), ("budget_bytes", C.c_uint64),
                ("prefill_arena_bytes", C.c_uint64), ("prefill_enabled", C.c_int32),
                ("_pad", C.c_int32)]


class moe_residency(C.Structure):
    _fields_ = [("layers_resident", C.c_int32), ("upload_count", C.c_int32),
                ("resident_bytes", C.c_uint64), ("gguf_bytes", C.c_uint64),
                ("scratch_bytes", C.c_uint64)]


class moe_kernel_time(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("total_ms", C.c_double), ("launches", C.c_int64)]


# ------------------------------------------------------------------- library

EXPORTS = {
    "moe_ctx_create": (C.c_int, [C.POINTER(moe_device_spec), C.POINTER(C.c_void_p)]),
    "moe_ctx_destroy": (C.c_int, [C.c_void_p]),
    "moe_ctx_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "moe_admission_check": (C.c_int, [C.POINTER(moe_device_spec), C.POINTER(moe_layer_desc), C.c_int32,
                                      C.POINTER(moe_mem_inspector), C.POINTER(moe_footprint)]),
    "moe_layer_upload": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(moe_layer_desc)]),
    "moe_forward": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                              C.c_void_p, C.c_int32]),
    "moe_layer_set_ffn_norm": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_float]),
    "moe_forward_block": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_int32]),
    "moe_prefill_ffn_layers": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32]),
    "moe_lm_head_upload": (C.c_int, [C.c_void_p, C.POINTER(moe_tensor), C.POINTER(moe_tensor), C.c_int32]),
    "moe_lm_head": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32]),
    "moe_residency_summary": (C.c_int, [C.c_void_p, C.POINTER(moe_residency)]),
    "moe_device_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "moe_ctx_set_profiling": (C.c_int, [C.c_void_p, C.c_int32]),
    "moe_profile_read": (C.c_int, [C.c_void_p, C.POINTER(moe_kernel_time), C.c_int32, C.POINTER(C.c_int32),
                                   C.POINTER(C.c_int32)]),
    "moe_last_error_message": (C.c_char_p, [C.c_void_p]),
    "moe_debug_permutation": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int32)]),
    "moe_debug_capture_block_sums": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "moe_debug_block_dots": (C.c_int, [C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32,
                                       C.c_void_p, C.c_void_p, C.c_void_p]),
    "moe_route_noalloc": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                    C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_float, C.c_int32, C.c_int32,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "moe_probe_tensor": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_int32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "moe_ep_unique_id": (C.c_int, [C.c_void_p]),
    "moe_ep_init": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "moe_ep_reset": (C.c_int, [C.c_void_p]),
    "moe_debug_ep_fault": (C.c_int, [C.c_void_p, C.c_uint32, C.c_int64]),
    "moe_forward_ep": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_int32]),
    "moe_ep_plan": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                              C.c_void_p, C.c_void_p, C.POINTER(C.c_int32), C.c_void_p, C.POINTER(C.c_int32)]),
    "moe_row_bytes": (C.c_uint64, [C.c_int32, C.c_int32]),
    "moe_quantize_rows": (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_int32]),
    "moe_gen_normal": (C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_int32]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python jero-engine_b200/build.py`")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _check(rc, ctx=None):
    if rc != MOE_OK:
        msg = lib.moe_last_error_message(ctx)
        raise _ERRORS.get(rc, MoeError)(rc, msg.decode() if msg else "")


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to libjeromoe must be C-contiguous"
    return a.ctypes.data


def threads_default():
    return max(1, min(32, os.cpu_count() or 1))


# --------------------------------------------------------------- host utils


def row_bytes(quant: int, cols: int) -> int:
    return int(lib.moe_row_bytes(quant, cols))


def quantize_rows(quant: int, src: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """f32 [rows, cols] -> GGUF bytes [rows, row_bytes] with the repository quantiser."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    rows, cols = src.reshape(-1, src.shape[-1]).shape
    rb = row_bytes(quant, cols)
    if rb == 0:
        raise CapabilityMismatch(MOE_ERR_CAPABILITY_MISMATCH, f"{cols} columns are not whole {QUANT_NAMES.get(quant)} blocks")
    out = np.empty((rows, rb), dtype=np.uint8)
    _check(lib.moe_quantize_rows(quant, _ptr(src), rows, cols, _ptr(out), n_threads or threads_default()))
    return out


def gen_normal(seed: int, stream: int, n: int, sigma: float, n_threads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _check(lib.moe_gen_normal(seed, stream, n, sigma, _ptr(out), n_threads or threads_default()))
    return out


# ------------------------------------------------------------------ tensors


def tensor_c(t: Tensor) -> moe_tensor:
    """moe_tensor view of a GGUF tensor (the caller keeps t alive)."""
    c = moe_tensor()
    raw = t.data
    c.data = raw.ctypes.data
    c.nbytes = raw.nbytes
    c.quant = t.quant
    c.n_dims = len(t.shape)
    for i, dim in enumerate(t.shape):
        c.shape[i] = int(dim)
    return c


def layer_desc(weights: ModelWeights, layer: int, num_experts: int, top_k: int, expert_ffn_dim: int,
               use_shared_expert: bool, route: Optional[RouteSpec] = None, hidden: Optional[int] = None):
    """Builds moe_layer_desc from the GGUF tensor names dispatch_qwen3_moe_ffn reads
    (src/qwen_deepseek.rs:860-932). Returns (desc, keepalive)."""
    route = route or RouteSpec()
    d = moe_layer_desc()
    router_name = f"blk.{layer}.ffn_gate_inp.weight"
    d.hidden = hidden if hidden is not None else (
        weights.tensor(router_name).shape[0] if weights.contains_tensor(router_name) else 0)
    d.num_experts = num_experts
    d.top_k = top_k
    d.expert_ffn_dim = expert_ffn_dim
    d.use_shared_expert = int(bool(use_shared_expert))
    d.route_mode = route.mode
    d.normalize = int(bool(route.normalize))
    d.n_groups = route.n_groups
    d.topk_groups = route.topk_groups
    d.routed_scale = route.routed_scale
    names = {
        "router": router_name,
        "exp_probs_b": f"blk.{layer}.exp_probs_b.bias",
        "logit_bias": f"blk.{layer}.ffn_gate_inp.logit_bias",
        "gate_exps": f"blk.{layer}.ffn_gate_exps.weight",
        "up_exps": f"blk.{layer}.ffn_up_exps.weight",
        "down_exps": f"blk.{layer}.ffn_down_exps.weight",
        "gate_shexp": f"blk.{layer}.ffn_gate_shexp.weight",
        "up_shexp": f"blk.{layer}.ffn_up_shexp.weight",
        "down_shexp": f"blk.{layer}.ffn_down_shexp.weight",
    }
    keep = []
    for field_name, tname in names.items():
        if weights.contains_tensor(tname):
            t = weights.tensor(tname)
            keep.append(t)
            setattr(d, field_name, tensor_c(t))
    return d, keep


# ------------------------------------------------------------------ context


class Context:
    """One device context (moe_ctx): device-resident layers + forward scratch."""

    def __init__(self, device: int = 0, max_tokens: int = 64, max_layers: int = 1, reserve_bytes: int = 0,
                 flags: int = 0):
        spec = moe_device_spec(device, max_tokens, max_layers, flags, reserve_bytes)
        h = C.c_void_p()
        _check(lib.moe_ctx_create(C.byref(spec), C.byref(h)))
        self.h = h
        self.device = device
        self.max_tokens = max_tokens
        self.layers = {}

    def close(self):
        if self.h:
            lib.moe_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def set_stream(self, stream_ptr: int):
        _check(lib.moe_ctx_set_stream(self.h, C.c_void_p(stream_ptr)), self.h)

    def upload(self, layer: int, desc: moe_layer_desc, meta=None):
        _check(lib.moe_layer_upload(self.h, layer, C.byref(desc)), self.h)
        self.layers[layer] = meta or {"H": desc.hidden, "k": desc.top_k, "E": desc.num_experts}

    def forward(self, layer: int, x: np.ndarray, want_selection: bool = True):
        """Host arrays in and out: x [T, H] f32 -> (out [T, H], sel_idx [T, k], sel_w [T, k])."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, H = x.shape
        k = self.layers.get(layer, {"k": 1})["k"]   # unknown layers are rejected by the library
        out = np.empty((T, H), dtype=np.float32)
        si = np.empty((T, k), dtype=np.int32) if want_selection else None
        sw = np.empty((T, k), dtype=np.float32) if want_selection else None
        _check(lib.moe_forward(self.h, layer, T, _ptr(x), _ptr(out), _ptr(si), _ptr(sw), PTR_HOST), self.h)
        return out, si, sw

    def forward_ptrs(self, layer: int, T: int, x_ptr: int, out_ptr: int, sel_idx_ptr: int = 0, sel_w_ptr: int = 0,
                     ptr_kind: int = PTR_DEVICE):
        _check(lib.moe_forward(self.h, layer, T, C.c_void_p(x_ptr), C.c_void_p(out_ptr),
                               C.c_void_p(sel_idx_ptr or None), C.c_void_p(sel_w_ptr or None), ptr_kind), self.h)

    # ---- the FFN sublayer (moe_layer_set_ffn_norm / moe_forward_block)

    def set_ffn_norm(self, layer: int, weight, eps: float):
        """RMSNorm weight [H] (None: ones) and eps of the layer's FFN pre-norm."""
        w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        _check(lib.moe_layer_set_ffn_norm(self.h, layer, _ptr(w) if w is not None else None, C.c_float(eps)), self.h)
        self._keep_norm = w

    def forward_block(self, layer: int, hidden: np.ndarray, want_selection: bool = True):
        """hidden [T, H] -> (hidden + MoE(rmsnorm(hidden)), sel_idx, sel_w), host arrays."""
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        T, H = hidden.shape
        k = self.layers.get(layer, {"k": 1})["k"]
        out = np.empty((T, H), dtype=np.float32)
        si = np.empty((T, k), dtype=np.int32) if want_selection else None
        sw = np.empty((T, k), dtype=np.float32) if want_selection else None
        _check(lib.moe_forward_block(self.h, layer, T, _ptr(hidden), _ptr(out), _ptr(si), _ptr(sw), PTR_HOST),
               self.h)
        return out, si, sw

    def forward_block_ptrs(self, layer: int, T: int, hidden_ptr: int, out_ptr: int, sel_idx_ptr: int = 0,
                           sel_w_ptr: int = 0, ptr_kind: int = PTR_DEVICE):
        _check(lib.moe_forward_block(self.h, layer, T, C.c_void_p(hidden_ptr), C.c_void_p(out_ptr),
                                     C.c_void_p(sel_idx_ptr or None), C.c_void_p(sel_w_ptr or None), ptr_kind),
               self.h)

    def lm_head_upload(self, output_weight: Optional["Tensor"], token_embd: Optional["Tensor"], hidden: int):
        """The LM head: output.weight, or the tied token_embd.weight when it is
        absent (moe_lm_head_upload); both None: the synthetic logits."""
        o = tensor_c(output_weight) if output_weight is not None else None
        e = tensor_c(token_embd) if token_embd is not None else None
        _check(lib.moe_lm_head_upload(self.h, C.byref(o) if o is not None else None,
                                      C.byref(e) if e is not None else None, hidden), self.h)
        self._keep_head = (output_weight, token_embd)

    def lm_head(self, normed: np.ndarray, n_logits: int) -> np.ndarray:
        """logits [T, n_logits] of final-normed rows [T, hidden] (moe_lm_head)."""
        x = np.ascontiguousarray(normed, dtype=np.float32)
        out = np.empty((x.shape[0], n_logits), dtype=np.float32)
        _check(lib.moe_lm_head(self.h, x.shape[0], _ptr(x), _ptr(out), n_logits, PTR_HOST), self.h)
        return out

    def lm_head_ptrs(self, T: int, normed_ptr: int, logits_ptr: int, n_logits: int, ptr_kind: int = PTR_DEVICE):
        _check(lib.moe_lm_head(self.h, T, C.c_void_p(normed_ptr), C.c_void_p(logits_ptr), n_logits, ptr_kind), self.h)

    def prefill_ffn_layers(self, first_layer: int, n_layers: int, hidden: np.ndarray) -> np.ndarray:
        """Layer-major prefill of FFN sublayers first_layer .. + n_layers - 1 over all
        rows of hidden [T, H] at once (moe_prefill_ffn_layers); returns the new rows."""
        rows = np.array(hidden, dtype=np.float32, order="C", copy=True)
        T = rows.shape[0]
        _check(lib.moe_prefill_ffn_layers(self.h, first_layer, n_layers, T, _ptr(rows), PTR_HOST), self.h)
        return rows

    # ---- expert parallelism (moe_ep_init / moe_forward_ep)

    def ep_init(self, rank: int, world: int, uid: bytes):
        """Joins an expert-parallel world (collective); call before any upload."""
        buf = (C.c_uint8 * EP_ID_BYTES).from_buffer_copy(uid)
        _check(lib.moe_ep_init(self.h, rank, world, buf), self.h)
        self.ep = (rank, world)

    def forward_ep(self, layer: int, x: np.ndarray, want_selection: bool = True):
        """moe_forward_ep with host arrays; every rank of the world calls it (T may be 0)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, H = x.shape
        k = self.layers.get(layer, {"k": 1})["k"]
        out = np.empty((T, H), dtype=np.float32)
        si = np.empty((T, k), dtype=np.int32) if want_selection else None
        sw = np.empty((T, k), dtype=np.float32) if want_selection else None
        _check(lib.moe_forward_ep(self.h, layer, T, _ptr(x) if T else None, _ptr(out) if T else None,
                                  _ptr(si) if T else None, _ptr(sw) if T else None, PTR_HOST), self.h)
        return out, si, sw

    def forward_ep_ptrs(self, layer: int, T: int, x_ptr: int, out_ptr: int, ptr_kind: int = PTR_DEVICE):
        _check(lib.moe_forward_ep(self.h, layer, T, C.c_void_p(x_ptr or None), C.c_void_p(out_ptr or None), None,
                                  None, ptr_kind), self.h)

    def ep_reset(self):
        """Collective recovery of the peer exchange after a peer-rank timeout."""
        _check(lib.moe_ep_reset(self.h), self.h)

    def debug_ep_fault(self, epoch_skew: int, wait_cycles: int = 0):
        """Test hook: the next expert-parallel forward waits for a flag nothing
        raises (epoch_skew), and flag waits are bounded by wait_cycles."""
        _check(lib.moe_debug_ep_fault(self.h, epoch_skew, wait_cycles), self.h)

    def device_status(self) -> int:
        st = C.c_int32()
        _check(lib.moe_device_status(self.h, C.byref(st)), self.h)
        return st.value

    def set_profiling(self, on: bool):
        _check(lib.moe_ctx_set_profiling(self.h, int(bool(on))), self.h)

    def profile_read(self):
        """{kernel: (total_ms, launches)}, forwards timed since the last read."""
        cap = 32
        arr = (moe_kernel_time * cap)()
        nk, nf = C.c_int32(), C.c_int32()
        _check(lib.moe_profile_read(self.h, arr, cap, C.byref(nk), C.byref(nf)), self.h)
        return {arr[i].name.decode(): (arr[i].total_ms, arr[i].launches) for i in range(min(nk.value, cap))}, nf.value

    def residency(self) -> moe_residency:
        r = moe_residency()
        _check(lib.moe_residency_summary(self.h, C.byref(r)), self.h)
        return r

    def debug_capture_block_sums(self, device_ptr: int, n_ints: int):
        """Raw int32 block sums of the int8 tensor-core gate/up launch go to this
        device buffer (0, 0: off); layout [slot][gate/up][row of I][block]."""
        _check(lib.moe_debug_capture_block_sums(self.h, C.c_void_p(device_ptr or None), n_ints), self.h)

    def debug_permutation(self, E: int, k: int):
        T = C.c_int32()
        offs = np.empty(E + 1, dtype=np.int32)
        perm = np.empty(self.max_tokens * k, dtype=np.int32)
        _check(lib.moe_debug_permutation(self.h, _ptr(offs), _ptr(perm), C.byref(T)), self.h)
        return offs, perm[: T.value * k]


EP_ID_BYTES = 128


def ep_unique_id() -> bytes:
    """NCCL unique id bytes for moe_ep_init (made on one rank, shared out of band)."""
    buf = (C.c_uint8 * EP_ID_BYTES)()
    _check(lib.moe_ep_unique_id(buf))
    return bytes(buf)


@dataclass
class EpPlan:
    send_cnt: np.ndarray
    send_off: np.ndarray
    recv_cnt: np.ndarray
    recv_off: np.ndarray
    problems: np.ndarray   # [n, 3] (local expert, first slot, slots)
    segments: np.ndarray   # [n, 3] (first slot, first received row, rows)


def ep_plan(rank: int, world: int, E: int, all_offsets: np.ndarray) -> EpPlan:
    """The exchange plan moe_forward_ep derives from all ranks' slot offsets [world, E+1] (host only)."""
    offs = np.ascontiguousarray(all_offsets, dtype=np.int32).reshape(world, E + 1)
    v = [np.empty(world, dtype=np.int32) for _ in range(4)]
    El = max(1, E // max(world, 1))
    probs = np.empty((El, 3), dtype=np.int32)
    segs = np.empty((world * El, 3), dtype=np.int32)
    npb, nsg = C.c_int32(), C.c_int32()
    _check(lib.moe_ep_plan(rank, world, E, _ptr(offs), _ptr(v[0]), _ptr(v[1]), _ptr(v[2]), _ptr(v[3]), _ptr(probs),
                           C.byref(npb), _ptr(segs), C.byref(nsg)))
    return EpPlan(v[0], v[1], v[2], v[3], probs[: npb.value].copy(), segs[: nsg.value].copy())


def admission_check(device: int, max_tokens: int, descs: Sequence[moe_layer_desc],
                    free_bytes: Optional[int] = None, total_bytes: Optional[int] = None,
                    reserve_bytes: int = 0) -> moe_footprint:
    spec = moe_device_spec(device, max_tokens, max(1, len(descs)), 0, reserve_bytes)
    arr = (moe_layer_desc * max(1, len(descs)))(*descs)
    fp = moe_footprint()
    insp = None
    if free_bytes is not None:
        insp = C.byref(moe_mem_inspector(free_bytes, total_bytes or free_bytes))
    _check(lib.moe_admission_check(C.byref(spec), arr, len(descs), insp, C.byref(fp)))
    return fp


def probe_tensor(device: int, kind: int, m: int, n: int, a_tmem: bool = False, n_acc: int = 1, ctas_per_sm: int = 1,
                 n_mma: int = 4096):
    """Tensor-core throughput probe: (dense TOPS, cycles per MMA) of n_mma
    back-to-back MMAs of one shape on every SM (kind 0 f16, 1 int8) over
    n_acc independent accumulators, from ctas_per_sm issuing CTAs per SM."""
    tops, cyc = C.c_double(), C.c_double()
    _check(lib.moe_probe_tensor(device, kind, m, n, int(bool(a_tmem)), n_acc, ctas_per_sm, n_mma, C.byref(tops),
                                C.byref(cyc)))
    return tops.value, cyc.value


def debug_block_dots(device: int, quant: int, w_rows: np.ndarray, x: np.ndarray):
    """Integer block sums of GGUF rows w against the activation quantiser of the
    forward path: returns (isum [n, cols/32], xq [n, cols], xd [n, cols/32])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, cols = x.shape
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    isum = np.empty((n, cols // 32), dtype=np.int32)
    xq = np.empty((n, cols), dtype=np.int8)
    xd = np.empty((n, cols // 32), dtype=np.float32)
    _check(lib.moe_debug_block_dots(device, quant, _ptr(w_rows), _ptr(x), n, cols, _ptr(isum), _ptr(xq), _ptr(xd)))
    return isum, xq, xd
