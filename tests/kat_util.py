"""Helpers shared by the test files: golden fixture loading and error metrics."""
import json
import os

import numpy as np

import jeromoe as jm

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


# Small seeded layers of the five benchmark configs whose oracle outputs are
# committed in golden/seeded_small.npz: name -> (config id, overrides, T).
SEEDED_CASES = {
    "cfg1_small": (1, dict(E=16, I=256, H=512), 6),
    "cfg2_small": (2, dict(E=16, I=256, H=512), 5),
    "cfg3_small": (3, dict(E=16, k=4, I=352, S=512, H=512), 7),
    "cfg4_small": (4, dict(E=32, I=256, H=512), 9),
    "cfg5_small": (5, dict(E=32, k=6, I=256, S=512, H=512, n_groups=8, topk_groups=3), 8),
}


def seeded_case(name):
    import synth
    cid, over, T = SEEDED_CASES[name]
    return synth.CONFIGS[cid].scaled(**over), T


def load_kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


def load_seeded():
    return np.load(os.path.join(GOLDEN, "seeded_small.npz"))


def _values(spec):
    shape = spec["shape"]
    n = int(np.prod(shape))
    if "fill" in spec:
        return np.full(n, spec["fill"], dtype=np.float32)
    if "values" in spec:
        return np.array([np.nan if v is None else v for v in spec["values"]], dtype=np.float32)
    if "row_fill" in spec:   # [in, out]: one value per output row
        return np.repeat(np.array(spec["row_fill"], dtype=np.float32), shape[0])
    if "expert_fill" in spec:  # [in, out, E]: one value per expert slab
        return np.repeat(np.array(spec["expert_fill"], dtype=np.float32), shape[0] * shape[1])
    raise ValueError(spec)


def kat_weights(case):
    w = jm.ModelWeights()
    for name, spec in case["tensors"].items():
        assert spec["quant"] == "F32"
        w.insert(name, jm.f32_tensor(_values(spec), spec["shape"]))
    return w


def check_dispatch_expect(case, out, sel_idx, sel_w):
    """The assertions of the reference test the case restates."""
    ex = case["expect"]
    sel = [int(i) for i in sel_idx if i >= 0]
    assert len(sel) == ex["n_selected"]
    if "weight_sum" in ex:
        assert abs(float(np.sum(sel_w[: len(sel)])) - ex["weight_sum"]) < ex["weight_sum_tol"]
    if "first" in ex:
        assert sel[0] == ex["first"] and sel[-1] == ex["last"]
    if "winners_in_rank_order" in ex:
        assert sel == ex["winners_in_rank_order"]
    if "contains" in ex:
        assert all(c in sel for c in ex["contains"])
    if ex.get("out_finite"):
        assert np.all(np.isfinite(out))
    if "out_any_abs_gt" in ex:
        assert np.any(np.abs(out) > ex["out_any_abs_gt"])
    if "out_all_gt" in ex:
        assert np.all(out > ex["out_all_gt"])


def row_rel_err(y, ref):
    """max_i |y - ref| / max_i |ref| per token row (the parity metric)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    num = np.max(np.abs(y - ref), axis=-1)
    den = np.maximum(np.max(np.abs(ref), axis=-1), 1e-30)
    return num / den


def tied_embedding_fixture():
    """The token embedding of the reference's tied-embedding test
    (build_qwen_dense_weights, src/qwen_deepseek.rs:2465-2479): GGUF shape
    [hidden 8, vocab 16], element i = ((i mod 19) - 9) * 0.04; with no
    output.weight the head is this tensor (test at :2501-2546)."""
    hidden, vocab = 8, 16
    i = np.arange(vocab * hidden)
    emb = (((i % 19).astype(np.float32) - np.float32(9.0)) * np.float32(0.04)).astype(np.float32)
    return hidden, vocab, jm.f32_tensor(emb, [hidden, vocab])
