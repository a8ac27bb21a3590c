"""The CPU oracle against the reference's own known-answer tests
(tests/golden/reference_kats.json) and the committed seeded fixtures."""
import numpy as np
import pytest

import jeromoe as jm
import oracle as orc
import synth
from kat_util import check_dispatch_expect, kat_weights, load_kats, load_seeded, seeded_case

KATS = load_kats()


@pytest.mark.parametrize("case", KATS["dispatch"], ids=lambda c: c["name"])
def test_oracle_dispatch_kats(case):
    w = kat_weights(case)
    L = orc.Layer(w, 0, case["num_experts"], case["top_k"], case["use_shared_expert"], hidden=case["hidden"])
    out, si, sw = L.forward(np.array([case["x"]], dtype=np.float32))
    check_dispatch_expect(case, out[0], si[0], sw[0])


@pytest.mark.parametrize("case", KATS["routing"], ids=lambda c: c["name"])
def test_oracle_select_top_k(case):
    logits = np.array(case["logits"], dtype=np.float32)
    w = jm.ModelWeights({"blk.0.ffn_gate_inp.weight": jm.f32_tensor(np.zeros(len(logits)), [1, len(logits)])})
    L = orc.Layer(w, 0, len(logits), case["top_k"], False, hidden=1)
    idx, wts = L.select(logits)
    assert idx.tolist() == case["normalize"]["indices"]
    np.testing.assert_allclose(wts, case["normalize"]["weights"], atol=case["normalize"]["tol"])
    raw = orc.Layer(w, 0, len(logits), case["top_k"], False, route=jm.RouteSpec(normalize=False), hidden=1)
    _, rw = raw.select(logits)
    assert float(rw.sum()) < case["raw"]["weight_sum_lt"]
    k0 = orc.Layer(w, 0, len(logits), 0, False, hidden=1)
    assert len(k0.select(logits)[0]) == 0


def test_oracle_format_kats():
    f = KATS["formats"]
    for kat in f["f16"]:
        assert orc.f16_to_f32(kat["bits"]) == kat["value"]
    for kat in f["q8_0_dequant"]:
        blk = bytes([kat["d_bits"] & 0xFF, kat["d_bits"] >> 8]) + bytes([kat["q"] & 0xFF]) * 32
        row = np.frombuffer(blk * kat["blocks"], dtype=np.uint8)
        vals = orc.dequantize_row(orc.Q8_0, row, 32 * kat["blocks"])
        assert np.all(np.abs(vals - kat["value"]) < 1e-5)
    assert orc.row_bytes(orc.Q8_0, 32) == f["q8_0_block_bytes"]
    for kat in f["q4_k_tensor_bytes"]:
        assert orc.row_bytes(orc.Q4_K, kat["elements"]) == kat["bytes"]
        assert jm.row_bytes(jm.Q4_K, kat["elements"]) == kat["bytes"]


@pytest.mark.parametrize("name", ["cfg1_small", "cfg2_small", "cfg3_small", "cfg4_small", "cfg5_small"])
def test_oracle_matches_committed_fixture(name):
    """The oracle (and the generator + quantiser feeding it) reproduce the
    committed fixture bit for bit on this host."""
    g = load_seeded()
    cfg, T = seeded_case(name)
    w = synth.build_weights(cfg, n_threads=2)
    x = synth.gen_x(cfg, T)
    np.testing.assert_array_equal(x[:, :8], g[f"{name}/x_head"])
    L = orc.Layer(w, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)
    out, si, sw = L.forward(x, 2)
    np.testing.assert_array_equal(si, g[f"{name}/sel_idx"])
    np.testing.assert_array_equal(sw, g[f"{name}/sel_w"])
    np.testing.assert_array_equal(out, g[f"{name}/out"])
    offs, perm = orc.permutation(si, cfg.E)
    np.testing.assert_array_equal(offs, g[f"{name}/offsets"])
    np.testing.assert_array_equal(perm, g[f"{name}/perm_token"])


def test_oracle_threads_do_not_change_results():
    cfg = synth.CONFIGS[2].scaled(E=16, I=256, H=512)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, 3)
    L = orc.Layer(w, 0, cfg.E, cfg.k, False, cfg.route, hidden=cfg.H)
    a = L.forward(x, 1)
    b = L.forward(x, 5)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)


def test_oracle_rmsnorm_matches_float64_and_defaults():
    """orc_rmsnorm (the fixed-order restatement of rmsnorm_standard) against a
    float64 RMSNorm, a NULL weight as all ones, and a zero row staying zero."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((4, 2048)).astype(np.float32) * np.array([[1.0], [1e-3], [1e3], [0.0]], np.float32)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    eps = 1e-6
    y = orc.rmsnorm(x, w, eps)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + eps) * w
    for t in range(3):
        assert np.abs(y[t] - ref[t]).max() <= 1e-6 * np.abs(ref[t]).max()
    assert np.all(y[3] == 0.0)
    np.testing.assert_array_equal(orc.rmsnorm(x, None, eps), orc.rmsnorm(x, np.ones(2048, np.float32), eps))
