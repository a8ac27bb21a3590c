"""ctypes wrapper of liboracle.so, the CPU restatement of the reference MoE path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker (or the timed CPU
baseline), never as part of the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, Q8_0, Q4_K = 0, 8, 12


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class orc_matrix(C.Structure):
    _fields_ = [("type", C.c_int32), ("rows", C.c_int32), ("cols", C.c_int32), ("_pad", C.c_int32),
                ("data", C.c_void_p), ("expert_stride", C.c_uint64)]


class orc_layer(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32), ("normalize", C.c_int32),
                ("scale", C.c_float), ("n_groups", C.c_int32), ("topk_groups", C.c_int32), ("_pad", C.c_int32),
                ("router", C.c_void_p), ("sel_bias", C.c_void_p), ("logit_bias", C.c_void_p),
                ("gate", orc_matrix), ("up", orc_matrix), ("down", orc_matrix),
                ("sh_gate", orc_matrix), ("sh_up", orc_matrix), ("sh_down", orc_matrix)]


def _load():
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "moe_oracle.c")):
        build()
    lib = C.CDLL(LIB_PATH)
    sig = {
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_row_bytes": (C.c_size_t, [C.c_int, C.c_int]),
        "orc_dequantize_row": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
        "orc_quantize_act": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
        "orc_block_dots": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
        "orc_row_dot_q": (C.c_float, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
        "orc_router_logits": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
        "orc_rmsnorm": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p]),
        "orc_select": (C.c_int, [C.POINTER(orc_layer), C.c_void_p, C.c_void_p, C.c_void_p]),
        "orc_moe_forward": (C.c_int, [C.POINTER(orc_layer), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int]),
        "orc_permutation": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
        "orc_lm_head": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                  C.c_void_p]),
        "orc_moe_forward_ex": (C.c_int, [C.POINTER(orc_layer), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_int, C.c_int]),
        "orc_gen_normal": (C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_int]),
        "orc_quantize_rows": (C.c_int, [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_int]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _p(a):
    return None if a is None else a.ctypes.data


def f16_to_f32(h: int) -> float:
    return lib.orc_f16_to_f32(h)


def row_bytes(quant, cols):
    return lib.orc_row_bytes(quant, cols)


def dequantize_row(quant, row: np.ndarray, cols: int) -> np.ndarray:
    out = np.empty(cols, dtype=np.float32)
    row = np.ascontiguousarray(row, dtype=np.uint8)
    assert lib.orc_dequantize_row(quant, _p(row), cols, _p(out)) == 0
    return out


def quantize_act(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.shape[-1], dtype=np.int8)
    d = np.empty(x.shape[-1] // 32, dtype=np.float32)
    assert lib.orc_quantize_act(_p(x), x.shape[-1], _p(q), _p(d)) == 0
    return q, d


def block_dots(quant, wrow: np.ndarray, xq: np.ndarray, cols: int):
    isum = np.empty(cols // 32, dtype=np.int32)
    xsum = np.empty(cols // 32, dtype=np.int32)
    wrow = np.ascontiguousarray(wrow, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    assert lib.orc_block_dots(quant, _p(wrow), _p(xq), cols, _p(isum), _p(xsum)) == 0
    return isum, xsum


def router_logits(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    E, H = w.shape
    out = np.empty(E, dtype=np.float32)
    lib.orc_router_logits(_p(w), _p(x), E, H, _p(out))
    return out


def rmsnorm(x: np.ndarray, w, eps: float) -> np.ndarray:
    """Rows of x [T, H] through orc_rmsnorm (w None: ones)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, H = x.shape
    wv = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    for t in range(T):
        lib.orc_rmsnorm(_p(x[t]), _p(wv) if wv is not None else None, H, C.c_float(eps), _p(out[t]))
    return out


def lm_head(head, hidden: int, normed: np.ndarray, n_logits: int) -> np.ndarray:
    """project_lm_head (orc_lm_head) of normed rows [T, hidden]; head: a
    jeromoe Tensor (output.weight or the tied token_embd.weight) or None."""
    x = np.ascontiguousarray(normed, dtype=np.float32)
    T = x.shape[0]
    out = np.zeros((T, n_logits), dtype=np.float32)
    if head is None:
        rc = lib.orc_lm_head(0, None, 0, 0, hidden, T, _p(x), n_logits, _p(out))
    else:
        shape = list(head.shape)
        shaped = len(shape) == 2 and shape[0] == hidden and shape[1] > 0
        n = int(np.prod(shape))
        rows = shape[1] if shaped else (n // hidden if n % hidden == 0 else 0)
        data = np.ascontiguousarray(head.data)
        rc = lib.orc_lm_head(int(head.quant), _p(data), int(shaped), rows, hidden, T, _p(x), n_logits, _p(out))
    assert rc == 0, rc
    return out


def _mat(t, experts):
    m = orc_matrix()
    if t is None:
        return m
    m.type = t.quant
    m.cols = int(t.shape[0])
    m.rows = int(t.shape[1])
    m.data = t.data.ctypes.data
    m.expert_stride = t.data.nbytes // experts
    return m


class Layer:
    """orc_layer over the same GGUF tensors the product consumes (jeromoe.ModelWeights)."""

    def __init__(self, weights, layer, num_experts, top_k, use_shared, route=None, hidden=None):
        g = lambda n: weights.tensor(n) if weights.contains_tensor(n) else None
        router = g(f"blk.{layer}.ffn_gate_inp.weight")
        self.keep = []
        L = orc_layer()
        L.hidden = hidden if hidden is not None else int(router.shape[0])
        L.n_experts = num_experts
        L.top_k = top_k
        L.normalize = 1 if route is None else int(bool(route.normalize))
        L.scale = 1.0 if route is None else route.routed_scale
        L.n_groups = 0 if route is None or route.mode != 1 else route.n_groups
        L.topk_groups = 0 if route is None or route.mode != 1 else route.topk_groups
        L.router = router.data.ctypes.data
        sb, lb = g(f"blk.{layer}.exp_probs_b.bias"), g(f"blk.{layer}.ffn_gate_inp.logit_bias")
        L.sel_bias = sb.data.ctypes.data if sb is not None else None
        L.logit_bias = lb.data.ctypes.data if lb is not None else None
        L.gate = _mat(g(f"blk.{layer}.ffn_gate_exps.weight"), num_experts)
        L.up = _mat(g(f"blk.{layer}.ffn_up_exps.weight"), num_experts)
        L.down = _mat(g(f"blk.{layer}.ffn_down_exps.weight"), num_experts)
        sh = [g(f"blk.{layer}.ffn_{m}_shexp.weight") for m in ("gate", "up", "down")]
        if use_shared and all(t is not None for t in sh):
            L.sh_gate, L.sh_up, L.sh_down = (_mat(t, 1) for t in sh)
        self.c = L
        self.k = top_k
        self.H = L.hidden
        self.E = num_experts

    def forward(self, x: np.ndarray, n_threads: int = 1, act_f32: bool = False):
        """The block over the rows of x. act_f32: the other reading of the
        reference's quantised dots (dequantised weights . f32 activations)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.empty((T, self.H), dtype=np.float32)
        si = np.empty((T, self.k), dtype=np.int32)
        sw = np.empty((T, self.k), dtype=np.float32)
        rc = lib.orc_moe_forward_ex(C.byref(self.c), T, _p(x), _p(out), _p(si), _p(sw), n_threads, int(act_f32))
        if rc != 0:
            raise ValueError(f"oracle rejected the layer (code {rc})")
        return out, si, sw

    def select(self, logits: np.ndarray):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        idx = np.empty(self.k, dtype=np.int32)
        w = np.empty(self.k, dtype=np.float32)
        n = lib.orc_select(C.byref(self.c), _p(logits), _p(idx), _p(w))
        return idx[:n], w[:n]


def permutation(sel_idx: np.ndarray, E: int):
    sel_idx = np.ascontiguousarray(sel_idx, dtype=np.int32)
    T, k = sel_idx.shape
    offs = np.empty(E + 1, dtype=np.int32)
    perm = np.empty(T * k, dtype=np.int32)
    assert lib.orc_permutation(_p(sel_idx), T, k, E, _p(offs), _p(perm)) == 0
    return offs, perm


# ---------------------------------------------------- synthetic inputs
# The same bytes as the product library's moe_gen_normal / moe_quantize_rows,
# restated here so the benchmark's reference arm builds its layers without
# loading the product library.

def _threads(n):
    return n or max(1, min(32, os.cpu_count() or 1))


def gen_normal(seed: int, stream: int, n: int, sigma: float, n_threads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    assert lib.orc_gen_normal(seed, stream, n, sigma, _p(out), _threads(n_threads)) == 0
    return out


def quantize_rows(quant: int, src: np.ndarray, n_threads: int = 0) -> np.ndarray:
    src = np.ascontiguousarray(src, dtype=np.float32)
    rows, cols = src.reshape(-1, src.shape[-1]).shape
    rb = row_bytes(quant, cols)
    if rb == 0:
        raise ValueError(f"{cols} columns are not whole blocks of quant {quant}")
    out = np.empty((rows, rb), dtype=np.uint8)
    assert lib.orc_quantize_rows(quant, _p(src), rows, cols, _p(out), _threads(n_threads)) == 0
    return out

