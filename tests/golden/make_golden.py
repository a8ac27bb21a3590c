"""Regenerates the committed golden fixtures in this directory.

reference_kats.json -- the known-answer tests that jero-engine's own test suite
    holds for the MoE path, restated as data: how each test builds its inputs
    and what it asserts (file:line of the jero-engine source tree in "source").
    Inputs are written out in full so the fixture does not depend on this script.

seeded_small.npz -- oracle outputs for small seeded layers of the benchmark
    configurations (selection, weights, permutation, output rows). They pin the
    oracle against drift; the GPU parity tests compare against the same arrays.

Run from the repository root: python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "jero-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def qwen3moe_dispatch_kat(num_experts, expert_ffn, winners, source):
    """build_qwen3_moe_weights + test_qwen3moe_128_top8_dispatch
    (src/qwen_deepseek.rs:2646-2721): router rows of the winners hold
    3 + (8 - rank) * 0.25, all others -1; expert e gate = ((e % 7) + 1) * 0.02,
    up = 0.1, down = 0.05, all F32; x = 0.4."""
    hidden = 8
    router = np.full((num_experts, hidden), -1.0, dtype=np.float32)
    for idx, e in enumerate(winners):
        router[e, :] = np.float32(3.0) + np.float32(len(winners) - idx) * np.float32(0.25)
    gate = np.stack([np.full((expert_ffn, hidden), ((e % 7) + 1.0) * 0.02, dtype=np.float32)
                     for e in range(num_experts)])
    return {
        "name": f"qwen3moe_top8_dispatch_E{num_experts}",
        "source": source,
        "hidden": hidden, "num_experts": num_experts, "top_k": 8, "expert_ffn_dim": expert_ffn,
        "use_shared_expert": False,
        "x": [0.4] * hidden,
        "tensors": {
            "blk.0.ffn_gate_inp.weight": {"quant": "F32", "shape": [hidden, num_experts],
                                          "row_fill": router[:, 0].tolist()},
            "blk.0.ffn_gate_exps.weight": {"quant": "F32", "shape": [hidden, expert_ffn, num_experts],
                                           "expert_fill": gate[:, 0, 0].tolist()},
            "blk.0.ffn_up_exps.weight": {"quant": "F32", "shape": [hidden, expert_ffn, num_experts],
                                         "fill": 0.1},
            "blk.0.ffn_down_exps.weight": {"quant": "F32", "shape": [expert_ffn, hidden, num_experts],
                                           "fill": 0.05},
        },
        "expect": {"n_selected": 8, "weight_sum": 1.0, "weight_sum_tol": 1e-4,
                   "first": winners[0], "last": winners[7], "winners_in_rank_order": list(winners),
                   "out_finite": True, "out_any_abs_gt": 1e-6},
    }


def deepseek2_bias_kat():
    """build_deepseek2_test_recipe_and_weights + test_deepseek2_mla_and_shared_moe_recipe
    (src/qwen_deepseek.rs:2868-2929): every tensor filled with a constant,
    exp_probs_b = [0,2,0,0,0,3,0,0], x = 0.5, k = 2, shared expert on."""
    h = 8
    return {
        "name": "deepseek2_bias_and_shared",
        "source": "src/qwen_deepseek.rs:2868-2929",
        "hidden": h, "num_experts": 8, "top_k": 2, "expert_ffn_dim": 8, "use_shared_expert": True,
        "x": [0.5] * h,
        "tensors": {
            "blk.0.ffn_gate_shexp.weight": {"quant": "F32", "shape": [8, 8], "fill": 0.08},
            "blk.0.ffn_up_shexp.weight": {"quant": "F32", "shape": [8, 8], "fill": 0.05},
            "blk.0.ffn_down_shexp.weight": {"quant": "F32", "shape": [8, 8], "fill": 0.04},
            "blk.0.ffn_gate_inp.weight": {"quant": "F32", "shape": [8, 8], "fill": 0.1},
            "blk.0.exp_probs_b.bias": {"quant": "F32", "shape": [8],
                                       "values": [0.0, 2.0, 0.0, 0.0, 0.0, 3.0, 0.0, 0.0]},
            "blk.0.ffn_gate_exps.weight": {"quant": "F32", "shape": [8, 8, 8], "fill": 0.03},
            "blk.0.ffn_up_exps.weight": {"quant": "F32", "shape": [8, 8, 8], "fill": 0.02},
            "blk.0.ffn_down_exps.weight": {"quant": "F32", "shape": [8, 8, 8], "fill": 0.03},
        },
        "expect": {"n_selected": 2, "contains": [5, 1], "out_finite": True, "out_any_abs_gt": 1e-6},
    }


def untouched_experts_kat():
    """The property of test_gemma4_26b_a4b_moe_routing (src/gemma.rs:1742-1798):
    experts the router does not pick are never read. The reference gives them
    1x1 tensors that would fail bounds; a stacked layout has one shape for all
    experts, so here they hold NaN and the output must stay finite. Router rows:
    expert 0 -> 5, 2 -> 7, 1 and 3 -> -9 (first column), hidden = [1, .5, .5, .5]."""
    h, ffn, E = 4, 2, 4
    router = np.zeros((E, h), dtype=np.float32)
    router[0, 0], router[1, 0], router[2, 0], router[3, 0] = 5.0, -9.0, 7.0, -9.0
    def stack(val_by_expert, rows, cols):
        return np.stack([np.full((rows, cols), v, dtype=np.float32) for v in val_by_expert]).reshape(-1)
    vals = [1.0, float("nan"), 2.0, float("nan")]
    return {
        "name": "unselected_experts_never_read",
        "source": "src/gemma.rs:1742-1798",
        "hidden": h, "num_experts": E, "top_k": 2, "expert_ffn_dim": ffn, "use_shared_expert": False,
        "x": [1.0, 0.5, 0.5, 0.5],
        "tensors": {
            "blk.0.ffn_gate_inp.weight": {"quant": "F32", "shape": [h, E], "values": router.reshape(-1).tolist()},
            "blk.0.ffn_gate_exps.weight": {"quant": "F32", "shape": [h, ffn, E],
                                           "values": [None if np.isnan(v) else float(v) for v in stack(vals, ffn, h)]},
            "blk.0.ffn_up_exps.weight": {"quant": "F32", "shape": [h, ffn, E],
                                         "values": [None if np.isnan(v) else float(v) for v in stack(vals, ffn, h)]},
            "blk.0.ffn_down_exps.weight": {"quant": "F32", "shape": [ffn, h, E],
                                           "values": [None if np.isnan(v) else float(v) for v in stack(vals, h, ffn)]},
        },
        "expect": {"n_selected": 2, "winners_in_rank_order": [2, 0], "out_finite": True, "out_all_gt": 0.0},
    }


def routing_kats():
    """test_select_top_k_experts_deterministic (src/gemma.rs:1722-1740)."""
    return [{
        "name": "select_top_k_ties_to_lower_index",
        "source": "src/gemma.rs:1722-1740",
        "logits": [0.1, 3.0, 0.5, 1.0, 3.0, 2.0],
        "top_k": 2,
        "normalize": {"indices": [1, 4], "weights": [0.5, 0.5], "tol": 1e-6},
        "raw": {"weight_sum_lt": 0.99},
        "empty_logits_gives_empty": True,
        "k0_gives_empty": True,
    }]


def format_kats():
    """Block decoding known answers (src/gemma.rs:1628-1662; src/weights.rs:1204-1208;
    f16 constants of tests/wave1_engine_regression_test.rs:116-117)."""
    return {
        "f16": [{"bits": 0x3C00, "value": 1.0}, {"bits": 0x3800, "value": 0.5},
                {"bits": 0x2C00, "value": 0.0625}, {"bits": 0x2400, "value": 0.015625}],
        "q8_0_dequant": [
            {"q": 1, "d_bits": 0x3C00, "blocks": 2, "value": 1.0, "source": "src/gemma.rs:1630-1646"},
            {"q": 2, "d_bits": 0x3C00, "blocks": 2, "value": 2.0, "source": "src/gemma.rs:1630-1646"},
        ],
        "q8_0_block_bytes": 34,
        "q4_k_tensor_bytes": [{"elements": 512, "bytes": 288, "source": "src/weights.rs:1204-1208"}],
    }


def write_kats():
    kats = {
        "dispatch": [
            qwen3moe_dispatch_kat(128, 12, [5, 19, 31, 47, 63, 79, 95, 111], "src/qwen_deepseek.rs:2702-2721"),
            qwen3moe_dispatch_kat(16, 4, [1, 3, 5, 7, 9, 11, 13, 15], "src/qwen_deepseek.rs:2704-2708 (miri shape)"),
            deepseek2_bias_kat(),
            untouched_experts_kat(),
        ],
        "routing": routing_kats(),
        "formats": format_kats(),
    }
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(kats, f, indent=1)


def write_seeded():
    from kat_util import SEEDED_CASES, seeded_case
    import oracle as orc
    import synth
    arrays = {}
    for name in SEEDED_CASES:
        cfg, T = seeded_case(name)
        w = synth.build_weights(cfg, n_threads=1)
        x = synth.gen_x(cfg, T, n_threads=1)
        L = orc.Layer(w, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)
        out, si, sw = L.forward(x, 1)
        offs, perm = orc.permutation(si, cfg.E)
        arrays[f"{name}/x_head"] = x[:, :8].copy()
        arrays[f"{name}/sel_idx"] = si
        arrays[f"{name}/sel_w"] = sw
        arrays[f"{name}/offsets"] = offs
        arrays[f"{name}/perm_token"] = perm
        arrays[f"{name}/out"] = out
    np.savez_compressed(os.path.join(HERE, "seeded_small.npz"), **arrays)


if __name__ == "__main__":
    write_kats()
    write_seeded()
    print("wrote", os.listdir(HERE))
