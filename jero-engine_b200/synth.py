"""Seeded synthetic MoE layers with the shapes of the five benchmark configs.

Inputs are generated, never read from a dataset: activations ~N(0, 1), weights
~N(0, 0.02) drawn in f32 and quantised by the repository quantiser; the
router stays f32. Each tensor has its own counter-based stream, so a smaller T
is a prefix of a larger one and experts can be generated independently:

    x = 1, router = 2, logit bias = 3, shared gate/up/down = 8/9/10,
    expert e gate/up/down = 16 + 3e, 17 + 3e, 18 + 3e.

Rows whose length is not a whole number of Q4_K super-blocks (the routed down
projection of config 3 has 1408 columns) use Q8_0, as GGUF quantisers fall
back to another block type for such tensors.

The generator and the quantiser come from the product library (jeromoe) by
default; use_backend(module) swaps in any module with the same gen_normal /
quantize_rows functions (the CPU oracle's restatement, which produces the same
bytes, lets the benchmark's reference arm build its layers without loading
the product library).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import moe_types as jm

_backend = None


def use_backend(module) -> None:
    """Module providing gen_normal(seed, stream, n, sigma, n_threads) and
    quantize_rows(quant, src, n_threads); None: the product library."""
    global _backend
    _backend = module


def _be():
    global _backend
    if _backend is None:
        import jeromoe
        _backend = jeromoe
    return _backend

WEIGHT_SIGMA = 0.02


@dataclass
class MoeConfig:
    name: str
    H: int
    E: int
    k: int
    I: int
    S: int = 0
    quant: int = jm.Q4_K
    normalize: bool = True
    routed_scale: float = 1.0
    n_groups: int = 0
    topk_groups: int = 0
    logit_bias_sigma: float = 0.0
    seed: int = 0
    tokens: tuple = (32,)

    @property
    def route(self) -> jm.RouteSpec:
        mode = jm.ROUTE_GROUP_LIMITED if self.n_groups else jm.ROUTE_SOFTMAX_TOPK
        return jm.RouteSpec(mode, self.normalize, self.n_groups, self.topk_groups, self.routed_scale)

    def scaled(self, **kw) -> "MoeConfig":
        d = dict(self.__dict__)
        d.update(kw)
        return MoeConfig(**d)


CONFIGS = {
    1: MoeConfig("cfg1-qwen3moe-q8_0", H=2048, E=128, k=8, I=768, quant=jm.Q8_0, seed=0, tokens=(32,)),
    2: MoeConfig("cfg2-qwen3moe-q4_k-decode", H=2048, E=128, k=8, I=768, quant=jm.Q4_K, seed=1,
                 tokens=(1, 2, 4, 8, 16, 32, 64)),
    3: MoeConfig("cfg3-deepseek-v2-lite", H=2048, E=64, k=6, I=1408, S=2816, quant=jm.Q4_K, normalize=False,
                 routed_scale=1.0, seed=2, tokens=(2048,)),
    4: MoeConfig("cfg4-qwen3moe-large-skewed", H=4096, E=128, k=8, I=1536, quant=jm.Q4_K, logit_bias_sigma=1.5,
                 seed=3, tokens=(512, 4096)),
    5: MoeConfig("cfg5-deepseek-v2-ep", H=5120, E=160, k=6, I=1536, S=3072, quant=jm.Q4_K, normalize=False,
                 routed_scale=1.0, n_groups=8, topk_groups=3, seed=4, tokens=(8192,)),
}

STREAM_X, STREAM_ROUTER, STREAM_LOGIT_BIAS = 1, 2, 3
STREAM_SH = (8, 9, 10)


def expert_stream(e: int, which: int) -> int:
    return 16 + 3 * e + which


def pick_quant(quant: int, cols: int) -> int:
    return quant if jm.gguf_row_bytes(quant, cols) else jm.Q8_0


def gen_x(cfg: MoeConfig, T: int, n_threads: int = 0) -> np.ndarray:
    return _be().gen_normal(cfg.seed, STREAM_X, T * cfg.H, 1.0, n_threads).reshape(T, cfg.H)


def _stack(cfg: MoeConfig, rows: int, cols: int, which: int, n_threads: int):
    q = pick_quant(cfg.quant, cols)
    rb = jm.gguf_row_bytes(q, cols)
    out = np.empty((cfg.E, rows * rb), dtype=np.uint8)
    for e in range(cfg.E):
        w = _be().gen_normal(cfg.seed, expert_stream(e, which), rows * cols, WEIGHT_SIGMA, n_threads)
        out[e] = _be().quantize_rows(q, w.reshape(rows, cols), n_threads).reshape(-1)
    return jm.Tensor(q, [cols, rows, cfg.E], out.reshape(-1))


def _matrix(cfg: MoeConfig, rows: int, cols: int, stream: int, n_threads: int):
    q = pick_quant(cfg.quant, cols)
    w = _be().gen_normal(cfg.seed, stream, rows * cols, WEIGHT_SIGMA, n_threads)
    return jm.Tensor(q, [cols, rows], _be().quantize_rows(q, w.reshape(rows, cols), n_threads).reshape(-1))


def build_weights(cfg: MoeConfig, layer: int = 0, n_threads: int = 0) -> jm.ModelWeights:
    """GGUF-named tensors of one MoE layer for cfg."""
    w = jm.ModelWeights()
    H, E, I, S = cfg.H, cfg.E, cfg.I, cfg.S
    router = _be().gen_normal(cfg.seed, STREAM_ROUTER, E * H, WEIGHT_SIGMA, n_threads)
    w.insert(f"blk.{layer}.ffn_gate_inp.weight", jm.f32_tensor(router, [H, E]))
    if cfg.logit_bias_sigma:
        lb = _be().gen_normal(cfg.seed, STREAM_LOGIT_BIAS, E, cfg.logit_bias_sigma, n_threads)
        w.insert(f"blk.{layer}.ffn_gate_inp.logit_bias", jm.f32_tensor(lb, [E]))
    w.insert(f"blk.{layer}.ffn_gate_exps.weight", _stack(cfg, I, H, 0, n_threads))
    w.insert(f"blk.{layer}.ffn_up_exps.weight", _stack(cfg, I, H, 1, n_threads))
    w.insert(f"blk.{layer}.ffn_down_exps.weight", _stack(cfg, H, I, 2, n_threads))
    if S:
        w.insert(f"blk.{layer}.ffn_gate_shexp.weight", _matrix(cfg, S, H, STREAM_SH[0], n_threads))
        w.insert(f"blk.{layer}.ffn_up_shexp.weight", _matrix(cfg, S, H, STREAM_SH[1], n_threads))
        w.insert(f"blk.{layer}.ffn_down_shexp.weight", _matrix(cfg, H, S, STREAM_SH[2], n_threads))
    return w


def desc_for(cfg: MoeConfig, weights: jm.ModelWeights, layer: int = 0):
    import jeromoe
    return jeromoe.layer_desc(weights, layer, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, hidden=cfg.H)


def algorithmic_bytes(cfg: MoeConfig, weights: jm.ModelWeights, sel_idx: np.ndarray, T: int, layer: int = 0) -> int:
    """Bytes one layer call must move at least: the weights of every expert that
    received a token (read once), the shared expert, the router, x in and out."""
    U = len(np.unique(sel_idx[sel_idx >= 0]))
    per_expert = sum(weights.tensor(f"blk.{layer}.ffn_{m}_exps.weight").data.nbytes // cfg.E
                     for m in ("gate", "up", "down"))
    shared = sum(weights.tensor(f"blk.{layer}.ffn_{m}_shexp.weight").data.nbytes
                 for m in ("gate", "up", "down")) if cfg.S else 0
    return U * per_expert + shared + cfg.E * cfg.H * 4 + 2 * T * cfg.H * 4 + T * cfg.k * 8


def algorithmic_ops(cfg: MoeConfig, T: int) -> int:
    return 2 * T * cfg.k * 3 * cfg.H * cfg.I + 2 * T * 3 * cfg.H * cfg.S + 2 * T * cfg.E * cfg.H
