"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Gates: router top-k indices and the dispatch permutation bit-exact; integer
block sums of the quantised dots bit-exact; selection weights within 1e-5
relative (the softmax sum is reduced in a different order); layer outputs
within 1e-2 max relative error per token row, max|y - y_ref| / max|y_ref|.
"""
import numpy as np
import pytest

import jeromoe as jm
import oracle as orc
import synth
from kat_util import (SEEDED_CASES, check_dispatch_expect, kat_weights, load_kats, load_seeded,
                      row_rel_err, seeded_case)

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2
W_RTOL = 1e-5
KATS = load_kats()


def gpu_layer(weights, E, k, I, use_shared, route, hidden, max_tokens, layer=0, flags=0):
    ctx = jm.Context(0, max_tokens, layer + 1, flags=flags)
    d, keep = jm.layer_desc(weights, layer, E, k, I, use_shared, route, hidden)
    ctx.upload(layer, d)
    return ctx


def oracle_layer(weights, cfg):
    return orc.Layer(weights, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)


def assert_parity(out, si, sw, ref_out, ref_si, ref_sw, tol=OUT_TOL):
    np.testing.assert_array_equal(si, ref_si)
    np.testing.assert_allclose(sw, ref_sw, rtol=W_RTOL, atol=1e-7)
    err = row_rel_err(out, ref_out)
    assert np.all(np.isfinite(out))
    assert err.max() <= tol, f"max row rel err {err.max():.3e}"
    return err.max()


# ------------------------------------------------------------ reference KATs

@pytest.mark.parametrize("case", KATS["dispatch"], ids=lambda c: c["name"])
def test_gpu_reference_dispatch_kats(case):
    w = kat_weights(case)
    with gpu_layer(w, case["num_experts"], case["top_k"], case["expert_ffn_dim"], case["use_shared_expert"],
                   None, case["hidden"], 4) as ctx:
        x = np.array([case["x"]], dtype=np.float32)
        out, si, sw = ctx.forward(0, x)
    check_dispatch_expect(case, out[0], si[0], sw[0])
    L = orc.Layer(w, 0, case["num_experts"], case["top_k"], case["use_shared_expert"], hidden=case["hidden"])
    ro, rsi, rsw = L.forward(x)
    assert_parity(out, si, sw, ro, rsi, rsw, tol=1e-5)


@pytest.mark.parametrize("case", KATS["routing"], ids=lambda c: c["name"])
def test_gpu_reference_select_top_k(case):
    """Router logits equal to the KAT logits: hidden 1, x = [1], router row e = logit e."""
    logits = np.array(case["logits"], dtype=np.float32)
    E = len(logits)
    w = jm.ModelWeights({
        "blk.0.ffn_gate_inp.weight": jm.f32_tensor(logits, [1, E]),
        "blk.0.ffn_gate_exps.weight": jm.f32_tensor(np.full(4 * E, 0.1), [1, 4, E]),
        "blk.0.ffn_up_exps.weight": jm.f32_tensor(np.full(4 * E, 0.2), [1, 4, E]),
        "blk.0.ffn_down_exps.weight": jm.f32_tensor(np.full(4 * E, 0.3), [4, 1, E]),
    })
    x = np.ones((1, 1), dtype=np.float32)
    with gpu_layer(w, E, case["top_k"], 4, False, None, 1, 1) as ctx:
        _, si, sw = ctx.forward(0, x)
    assert si[0].tolist() == case["normalize"]["indices"]
    np.testing.assert_allclose(sw[0], case["normalize"]["weights"], atol=case["normalize"]["tol"])
    with gpu_layer(w, E, case["top_k"], 4, False, jm.RouteSpec(normalize=False), 1, 1) as ctx:
        _, si2, sw2 = ctx.forward(0, x)
    assert si2[0].tolist() == case["normalize"]["indices"]
    assert float(sw2[0].sum()) < case["raw"]["weight_sum_lt"]


# ------------------------------------------------------- committed fixtures

@pytest.mark.parametrize("name", list(SEEDED_CASES))
def test_gpu_matches_committed_fixture(name):
    g = load_seeded()
    cfg, T = seeded_case(name)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T) as ctx:
        out, si, sw = ctx.forward(0, x)
        offs, perm = ctx.debug_permutation(cfg.E, cfg.k)
    assert_parity(out, si, sw, g[f"{name}/out"], g[f"{name}/sel_idx"], g[f"{name}/sel_w"])
    np.testing.assert_array_equal(offs, g[f"{name}/offsets"])
    np.testing.assert_array_equal(perm, g[f"{name}/perm_token"])


# ------------------------------------------------------- integer block sums

@pytest.mark.parametrize("quant", [jm.Q8_0, jm.Q4_K])
def test_gpu_block_sums_bit_exact(quant):
    n, cols = 24, 2048
    wf = jm.gen_normal(11, 1, n * cols, 0.02).reshape(n, cols)
    wq = jm.quantize_rows(quant, wf)
    x = jm.gen_normal(11, 2, n * cols, 1.0).reshape(n, cols)
    x[3, :64] = 0.0                      # an all-zero block
    x[5, 100] = 1e30                     # a block dominated by one value
    isum, xq, xd = jm.debug_block_dots(0, quant, wq, x)
    for r in range(n):
        oq, od = orc.quantize_act(x[r])
        np.testing.assert_array_equal(xq[r], oq)
        np.testing.assert_array_equal(xd[r], od)
        ref, _ = orc.block_dots(quant, wq[r], oq, cols)
        np.testing.assert_array_equal(isum[r], ref)


# ------------------------------------------------------- full-size configs

def _full_size_parity(cid, T, sample=16, seed=0):
    cfg = synth.CONFIGS[cid]
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T) as ctx:
        out, si, sw = ctx.forward(0, x)
        offs, perm = ctx.debug_permutation(cfg.E, cfg.k)
    L = oracle_layer(w, cfg)
    # routing of every token, bit-exact
    router = w.tensor("blk.0.ffn_gate_inp.weight").data.reshape(cfg.E, cfg.H)
    ref_si = np.empty_like(si)
    ref_sw = np.empty_like(sw)
    for t in range(T):
        idx, wt = L.select(orc.router_logits(router, x[t]))
        ref_si[t, : len(idx)] = idx
        ref_sw[t, : len(idx)] = wt
    np.testing.assert_array_equal(si, ref_si)
    np.testing.assert_allclose(sw, ref_sw, rtol=W_RTOL, atol=1e-7)
    # the dispatch permutation, bit-exact
    ro, rp = orc.permutation(ref_si, cfg.E)
    np.testing.assert_array_equal(offs, ro)
    np.testing.assert_array_equal(perm, rp)
    # output rows: all of them for small T, a seeded sample otherwise
    rows = np.arange(T) if T <= sample else np.sort(np.random.default_rng(seed).choice(T, sample, replace=False))
    r_out, r_si, r_sw = L.forward(x[rows], 8)
    return assert_parity(out[rows], si[rows], sw[rows], r_out, r_si, r_sw)


@pytest.mark.parametrize("T", [1, 2, 4, 8, 16, 32, 64])
def test_gpu_cfg2_decode_sweep(T):
    _full_size_parity(2, T, sample=64)


def test_gpu_cfg1_q8_0():
    _full_size_parity(1, 32, sample=32)


def test_gpu_cfg3_deepseek_lite_shared():
    _full_size_parity(3, 2048)


@pytest.mark.parametrize("T", [512, 4096])
def test_gpu_cfg4_skewed(T):
    _full_size_parity(4, T)


def test_gpu_cfg5_group_limited():
    _full_size_parity(5, 8192, sample=12)


# ------------------------------------------------- tensor-core expert path

# Small layers whose matrices are whole 128-row tiles, forced onto the
# tensor-core path (f16 operands, f32 accumulation) for every T.
TC_CASES = {
    "cfg2_q4k": (2, dict(E=16, I=256, H=512)),
    "cfg1_q8_0": (1, dict(E=16, I=256, H=512)),
    "cfg3_shared_q8_down": (3, dict(E=16, k=4, I=384, S=512, H=512)),
    "cfg5_groups_shared": (5, dict(E=32, k=6, I=256, S=512, H=512, n_groups=8, topk_groups=3)),
}


@pytest.mark.parametrize("name", list(TC_CASES))
@pytest.mark.parametrize("T", [1, 37, 300])
def test_gpu_tensor_core_path(name, T):
    cid, over = TC_CASES[name]
    cfg = synth.CONFIGS[cid].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T, flags=jm.FLAG_TENSOR_CORES_ALWAYS) as ctx:
        out, si, sw = ctx.forward(0, x)
        prof_ok = ctx.device_status() == 0
    assert prof_ok
    ref = oracle_layer(w, cfg).forward(x, 8)
    # f16 operands move the SwiGLU output by ~1e-3 relative; its int8 block
    # re-quantisation can then differ from the oracle's by one step in a few
    # values, so this path is held to the contract tolerance (1e-2), not 1e-5.
    assert_parity(out, si, sw, *ref)


def test_gpu_tensor_core_matches_streaming_path():
    """Both expert paths on the same layer and tokens: same routing, outputs
    within the tolerance (the tensor-core path rounds operands to f16)."""
    cfg = synth.CONFIGS[2].scaled(E=32, I=256, H=512)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, 200)
    outs = []
    for flags in (jm.FLAG_TENSOR_CORES_ALWAYS, jm.FLAG_TENSOR_CORES_NEVER | jm.FLAG_INT8_TENSOR_CORES_NEVER):
        with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 200, flags=flags) as ctx:
            outs.append(ctx.forward(0, x))
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    assert row_rel_err(outs[0][0], outs[1][0]).max() <= OUT_TOL


# ------------------------- fused f16 tensor-core expert launch (small batches)

@pytest.mark.parametrize("name", list(TC_CASES))
@pytest.mark.parametrize("T", [1, 5, 33, 100, 255])
def test_gpu_fused_tensor_core_path(name, T):
    """The default path below 256 tokens: gate/up, SwiGLU and down in one
    tensor-core launch (f16 weights expanded from the GGUF blocks, f32
    accumulation over the whole K). Same routing as the oracle, outputs within
    the contract tolerance of it and of the int8 streaming path, and the fused
    launch is the one that ran. Run twice to cover the chunk counters' reset."""
    cid, over = TC_CASES[name]
    cfg = synth.CONFIGS[cid].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    ref = oracle_layer(w, cfg).forward(x, 8)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T, flags=jm.FLAG_FUSED_I8_NEVER) as ctx:
        ctx.set_profiling(True)
        first = ctx.forward(0, x)
        second = ctx.forward(0, x)
        prof, _ = ctx.profile_read()
        assert ctx.device_status() == 0
    assert "experts_tc" in prof, sorted(prof)
    assert_parity(*first, *ref)
    np.testing.assert_array_equal(first[0], second[0])
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T,
                   flags=jm.FLAG_INT8_TENSOR_CORES_NEVER) as ctx:
        stream = ctx.forward(0, x)
    np.testing.assert_array_equal(first[1], stream[1])
    assert row_rel_err(first[0], stream[0]).max() <= OUT_TOL


@pytest.mark.parametrize("name", list(TC_CASES))
@pytest.mark.parametrize("T", [1, 5, 33, 100, 255])
def test_gpu_fused_int8_path(name, T):
    """The fused launch with integer operands (exact int32 block sums from
    tcgen05 kind::i8, f32 block scaling in the epilogue), forced for every T:
    same routing as the oracle and the streaming path, outputs within the
    contract tolerance of the oracle, identical on a second call, and the
    launch is the one that ran."""
    cid, over = TC_CASES[name]
    cfg = synth.CONFIGS[cid].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    ref = oracle_layer(w, cfg).forward(x, 8)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T, flags=jm.FLAG_FUSED_I8_ALWAYS) as ctx:
        ctx.set_profiling(True)
        first = ctx.forward(0, x)
        second = ctx.forward(0, x)
        prof, _ = ctx.profile_read()
        assert ctx.device_status() == 0
    assert "experts_i8" in prof, sorted(prof)
    assert_parity(*first, *ref)
    np.testing.assert_array_equal(first[0], second[0])


# ---------------------------------- int8 tensor-core path (small batches)

INT8_PATHS = {"streaming_tc": ("gate_up_i8", jm.FLAG_INT8_TENSOR_CORES_ALWAYS),
              "fused": ("experts_i8", jm.FLAG_FUSED_I8_ALWAYS)}


@pytest.mark.parametrize("path", list(INT8_PATHS))
@pytest.mark.parametrize("name", ["cfg2_q4k", "cfg1_q8_0"])
@pytest.mark.parametrize("T", [5, 33])
def test_gpu_int8_tensor_core_block_sums_bit_exact(name, T, path):
    """The tcgen05 kind::i8 MMAs produce the int32 sum of every 32-value block
    of every routed gate/up product -- per block accumulator (the per-launch
    path) or four blocks of four slots in one accumulator off block-diagonal
    activation tiles (the fused launch); captured before any scaling, each
    equals the oracle's integer block dot (orc_block_dots) of the GGUF row and
    the token's int8 activation block, bit for bit."""
    stage, flags = INT8_PATHS[path]
    import torch
    cid, over = TC_CASES[name]
    cfg = synth.CONFIGS[cid].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    nb = cfg.H // 32
    slots = T * cfg.k
    buf = torch.zeros(slots * 2 * cfg.I * nb, dtype=torch.int32, device="cuda")
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, T, flags=flags) as ctx:
        ctx.debug_capture_block_sums(buf.data_ptr(), buf.numel())
        ctx.set_profiling(True)
        ctx.forward(0, x)
        prof, _ = ctx.profile_read()
        offs, perm = ctx.debug_permutation(cfg.E, cfg.k)
        ctx.debug_capture_block_sums(0, 0)
    assert stage in prof, sorted(prof)
    got = buf.cpu().numpy().reshape(slots, 2, cfg.I, nb)
    xq = [orc.quantize_act(x[t])[0] for t in range(T)]
    for m, name_m in enumerate(("gate", "up")):
        t = w.tensor(f"blk.0.ffn_{name_m}_exps.weight")
        rows = t.data.reshape(cfg.E, cfg.I, -1)
        for e in range(cfg.E):
            for s in range(offs[e], offs[e + 1]):
                tok = perm[s]
                for f in range(0, cfg.I, 7):   # a spread of rows of every tile
                    ref, _ = orc.block_dots(t.quant, rows[e, f], xq[tok], cfg.H)
                    np.testing.assert_array_equal(got[s, m, f], ref, err_msg=f"slot {s} {name_m} row {f}")


@pytest.mark.parametrize("cid,T", [(1, 16), (2, 16)])
def test_gpu_output_between_the_two_readings(cid, T):
    """Full-size layers on the default path against both readings of the
    reference's quantised dot: within the contract tolerance (1e-2) of the
    int8-activation reading the oracle defines, and within 3e-2 of the
    dequantised-weights x f32-activations reading (the two readings are about
    1.2% apart themselves; see test_oracle_two_readings_of_the_quantised_dot)."""
    cfg = synth.CONFIGS[cid]
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T) as ctx:
        out, si, sw = ctx.forward(0, x)
    L = oracle_layer(w, cfg)
    assert_parity(out, si, sw, *L.forward(x, 8))
    of, sif, swf = L.forward(x, 8, act_f32=True)
    np.testing.assert_array_equal(si, sif)
    assert row_rel_err(out, of).max() <= 3e-2

@pytest.mark.parametrize("name", list(TC_CASES))
@pytest.mark.parametrize("T", [1, 5, 33, 100])
def test_gpu_int8_tensor_core_path(name, T):
    """The same small layers forced onto the int8 tensor-core path (exact
    int32 block sums from tcgen05 kind::i8, f32 block scaling) and onto the
    dp4a streaming path: same routing, both within the contract tolerance of
    the oracle, and the int8 path is the one that ran."""
    cid, over = TC_CASES[name]
    cfg = synth.CONFIGS[cid].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    ref = oracle_layer(w, cfg).forward(x, 8)
    outs = []
    for flags in (jm.FLAG_INT8_TENSOR_CORES_ALWAYS, jm.FLAG_INT8_TENSOR_CORES_NEVER):
        with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T, flags=flags) as ctx:
            ctx.set_profiling(True)
            outs.append(ctx.forward(0, x))
            prof, _ = ctx.profile_read()
            assert ctx.device_status() == 0
        assert ("gate_up_i8" in prof) == (flags == jm.FLAG_INT8_TENSOR_CORES_ALWAYS), sorted(prof)
        assert_parity(*outs[-1], *ref)
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    assert row_rel_err(outs[0][0], outs[1][0]).max() <= OUT_TOL


@pytest.mark.parametrize("cid,T", [(3, 64), (5, 64), (1, 17)])
def test_gpu_int8_tensor_core_full_size(cid, T):
    """Full-size layers at decode batch sizes on the default path (the int8
    tensor cores from MOE_INT8_TENSOR_CORE_MIN_TOKENS tokens): shared experts,
    group-limited routing and Q8_0 weights."""
    _full_size_parity(cid, T, sample=16)


# ------------------------------------------------ FFN sublayer (pre-norm + residual)

@pytest.mark.parametrize("cid,over,T", [(2, dict(E=32, I=256, H=512), 5),
                                        (3, dict(E=16, k=4, I=384, S=512, H=512), 40),
                                        (2, {}, 64)])
def test_gpu_forward_block_is_norm_block_residual(cid, over, T):
    """moe_forward_block(hidden) == hidden + moe_forward(rmsnorm(hidden)) bit for
    bit, with the norm taken by the oracle's fixed-order restatement (so the
    device norm equals it bit for bit too); and within the contract tolerance of
    the oracle's whole sublayer. Non-finite norm weights read as 1.0. Host and
    device pointers, the device call in place (out = hidden)."""
    import torch
    cfg = synth.CONFIGS[cid].scaled(**over) if over else synth.CONFIGS[cid]
    w = synth.build_weights(cfg)
    rng = np.random.default_rng(7)
    hidden = (synth.gen_x(cfg, T) * 3.0).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, cfg.H).astype(np.float32)
    nw[3] = np.nan
    nw[7] = np.inf
    nw_eff = nw.copy()
    nw_eff[[3, 7]] = 1.0
    eps = 1e-6
    xn = orc.rmsnorm(hidden, nw_eff, eps)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H, T) as ctx:
        ctx.set_ffn_norm(0, nw, eps)
        out_b, si_b, sw_b = ctx.forward_block(0, hidden)
        out_f, si_f, sw_f = ctx.forward(0, xn)
        dev = torch.from_numpy(hidden.copy()).cuda()
        ctx.forward_block_ptrs(0, T, dev.data_ptr(), dev.data_ptr())
        torch.cuda.synchronize()
        out_d = dev.cpu().numpy()
        assert ctx.device_status() == 0
    np.testing.assert_array_equal(si_b, si_f)
    np.testing.assert_array_equal(sw_b, sw_f)
    np.testing.assert_array_equal(out_b, hidden + out_f)
    np.testing.assert_array_equal(out_d, out_b)
    rows = np.arange(T) if T <= 16 else np.arange(0, T, T // 16)
    r_out, r_si, r_sw = oracle_layer(w, cfg).forward(xn[rows], 8)
    assert_parity(out_b[rows], si_b[rows], sw_b[rows], hidden[rows] + r_out, r_si, r_sw)


@pytest.mark.parametrize("cid,over,T", [(2, dict(E=32, I=256, H=512), 40),
                                        (3, dict(E=16, k=4, I=384, S=512, H=512), 300)])
def test_gpu_layer_major_prefill_of_a_stack(cid, over, T):
    """moe_prefill_ffn_layers over three FFN sublayers (different weights and
    norms): bit for bit the layer-by-layer moe_forward_block calls, and within
    the contract tolerance of the oracle run token-major as the reference's
    prefill loop does it (each token through every layer in turn)."""
    n_layers = 3
    cfgs = [synth.CONFIGS[cid].scaled(**over, seed=synth.CONFIGS[cid].seed + 10 * l) for l in range(n_layers)]
    rng = np.random.default_rng(11)
    hidden = (synth.gen_x(cfgs[0], T) * 3.0).astype(np.float32)
    norms = [rng.uniform(0.5, 1.5, cfgs[0].H).astype(np.float32) for _ in range(n_layers)]
    eps = 1e-6
    ws = [synth.build_weights(cfgs[l], layer=l) for l in range(n_layers)]
    with jm.Context(0, T, n_layers) as ctx:
        keep = []
        for l, c in enumerate(cfgs):
            d, k = jm.layer_desc(ws[l], l, c.E, c.k, c.I, c.S > 0, c.route, c.H)
            keep.append(k)
            ctx.upload(l, d)
            ctx.set_ffn_norm(l, norms[l], eps)
        got = ctx.prefill_ffn_layers(0, n_layers, hidden)
        ref = hidden
        for l in range(n_layers):
            ref, _, _ = ctx.forward_block(l, ref)
        assert ctx.device_status() == 0
    np.testing.assert_array_equal(got, ref)
    layers = [orc.Layer(ws[l], l, c.E, c.k, c.S > 0, c.route, hidden=c.H) for l, c in enumerate(cfgs)]
    rows = np.arange(0, T, max(1, T // 8))
    for t in rows:   # token-major, as run_prefill_with_hidden
        h = hidden[t:t + 1].copy()
        for l in range(n_layers):
            o, _, _ = layers[l].forward(orc.rmsnorm(h, norms[l], eps), 1)
            h = h + o
        assert row_rel_err(got[t:t + 1], h).max() <= OUT_TOL, f"token {t}"


def test_gpu_forward_block_needs_norm():
    cfg = synth.CONFIGS[2].scaled(E=32, I=256, H=512)
    w = synth.build_weights(cfg)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 4) as ctx:
        with pytest.raises(jm.MoeError):
            ctx.forward_block(0, synth.gen_x(cfg, 2))
        with pytest.raises(jm.MoeError):
            ctx.set_ffn_norm(0, None, float("nan"))


# ------------------------------------------------------------- edge cases

def _small_cfg(**kw):
    return synth.CONFIGS[2].scaled(E=32, I=256, H=512, **kw)


def test_gpu_edge_token_counts_and_errors():
    cfg = _small_cfg()
    w = synth.build_weights(cfg)
    L = oracle_layer(w, cfg)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 70) as ctx:
        for T in (0, 1, 31, 33, 70):
            x = synth.gen_x(cfg, max(T, 1))[:T]
            out, si, sw = ctx.forward(0, x)
            assert out.shape == (T, cfg.H)
            if T:
                assert_parity(out, si, sw, *L.forward(x, 4))
        with pytest.raises(jm.ContextLengthExceeded):
            ctx.forward(0, synth.gen_x(cfg, 71))
        with pytest.raises(jm.InvalidArguments):
            ctx.forward(3, synth.gen_x(cfg, 1))
        r = ctx.residency()
        assert r.layers_resident == 1 and r.upload_count == 1 and r.resident_bytes > 0
    ctx = jm.Context(0, 8, 2)
    with pytest.raises(jm.NotUploaded):
        ctx.forward(1, synth.gen_x(cfg, 1))
    ctx.close()


def test_gpu_skewed_routing_many_tokens_per_expert():
    """Every token picks the same experts (large logit bias): one problem holds
    all T tokens, several token tiles per CTA."""
    cfg = _small_cfg(logit_bias_sigma=0.0)
    w = synth.build_weights(cfg)
    bias = np.zeros(cfg.E, dtype=np.float32)
    bias[[3, 7, 11, 12, 20, 25, 30, 31]] = 50.0
    w.insert("blk.0.ffn_gate_inp.logit_bias", jm.f32_tensor(bias, [cfg.E]))
    x = synth.gen_x(cfg, 100)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 100) as ctx:
        out, si, sw = ctx.forward(0, x)
        offs, perm = ctx.debug_permutation(cfg.E, cfg.k)
    assert sorted(set(si.reshape(-1).tolist())) == [3, 7, 11, 12, 20, 25, 30, 31]
    assert_parity(out, si, sw, *oracle_layer(w, cfg).forward(x, 4))
    ro, rp = orc.permutation(si, cfg.E)
    np.testing.assert_array_equal(offs, ro)
    np.testing.assert_array_equal(perm, rp)


def test_gpu_ties_signed_zero_and_non_finite_logits():
    """Identical router rows tie -> lower index; zero rows give +0.0 logits
    that tie with each other; an infinite or NaN logit ranks as -inf with
    probability 0 (select_top_k_experts, src/gemma.rs:371-417)."""
    cfg = _small_cfg()
    w = synth.build_weights(cfg)
    router = w.tensor("blk.0.ffn_gate_inp.weight").data.reshape(cfg.E, cfg.H).copy()
    router[9] = router[4]            # exact tie between experts 4 and 9
    router[14] = 0.0                 # logit +0.0
    router[15] = -0.0                # the fma chain starts at +0.0, so this logit is +0.0 too
    router[16, 0] = np.inf           # +inf or NaN logit
    router[17, :] = np.nan
    w.insert("blk.0.ffn_gate_inp.weight", jm.f32_tensor(router.reshape(-1), [cfg.H, cfg.E]))
    x = synth.gen_x(cfg, 40)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 40) as ctx:
        out, si, sw = ctx.forward(0, x)
    ro, rsi, rsw = oracle_layer(w, cfg).forward(x, 4)
    assert_parity(out, si, sw, ro, rsi, rsw)
    pos4 = np.argwhere(si == 4)
    for t, r in pos4:
        if 9 in si[t]:
            assert r < list(si[t]).index(9)


def test_gpu_sel_bias_and_group_modes_small():
    cfg = synth.CONFIGS[5].scaled(E=64, I=256, S=256, H=512)
    w = synth.build_weights(cfg)
    bias = jm.gen_normal(99, 1, cfg.E, 0.05)
    w.insert("blk.0.exp_probs_b.bias", jm.f32_tensor(bias, [cfg.E]))
    x = synth.gen_x(cfg, 50)
    for route in (cfg.route, jm.RouteSpec(), jm.RouteSpec(normalize=False, routed_scale=2.5)):
        c2 = cfg.scaled(n_groups=route.n_groups, topk_groups=route.topk_groups, normalize=route.normalize,
                        routed_scale=route.routed_scale)
        with gpu_layer(w, c2.E, c2.k, c2.I, True, route, c2.H, 50) as ctx:
            out, si, sw = ctx.forward(0, x)
        assert_parity(out, si, sw, *oracle_layer(w, c2).forward(x, 4))


def test_gpu_device_pointers_and_determinism():
    import torch
    cfg = _small_cfg()
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, 20)
    with gpu_layer(w, cfg.E, cfg.k, cfg.I, False, cfg.route, cfg.H, 20) as ctx:
        out_h, si_h, sw_h = ctx.forward(0, x)
        out_h2, _, _ = ctx.forward(0, x)
        np.testing.assert_array_equal(out_h, out_h2)
        xd = torch.from_numpy(x).cuda()
        od = torch.empty_like(xd)
        sid = torch.empty((20, cfg.k), dtype=torch.int32, device="cuda")
        swd = torch.empty((20, cfg.k), dtype=torch.float32, device="cuda")
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        ctx.set_stream(stream.cuda_stream)
        ctx.forward_ptrs(0, 20, xd.data_ptr(), od.data_ptr(), sid.data_ptr(), swd.data_ptr())
        torch.cuda.synchronize()
        ctx.set_stream(0)
    np.testing.assert_array_equal(od.cpu().numpy(), out_h)
    np.testing.assert_array_equal(sid.cpu().numpy(), si_h)
    np.testing.assert_array_equal(swd.cpu().numpy(), sw_h)


def test_gpu_reupload_replaces_layer():
    cfg = _small_cfg()
    w1 = synth.build_weights(cfg)
    w2 = synth.build_weights(cfg.scaled(seed=77))
    x = synth.gen_x(cfg, 5)
    ctx = jm.Context(0, 5, 1)
    d1, k1 = synth.desc_for(cfg, w1)
    ctx.upload(0, d1)
    a = ctx.forward(0, x)[0]
    d2, k2 = synth.desc_for(cfg, w2)
    ctx.upload(0, d2)
    b = ctx.forward(0, x)[0]
    assert ctx.residency().upload_count == 2 and ctx.residency().layers_resident == 1
    ctx.close()
    assert not np.allclose(a, b)
    ref = oracle_layer(w2, cfg).forward(x, 2)[0]
    assert row_rel_err(b, ref).max() <= OUT_TOL


# ------------------------------------------------------------------ LM head

def _lm_head_case(quant, hidden, rows, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((rows, hidden)) * 0.05).astype(np.float32)
    if quant == jm.F32:
        return jm.f32_tensor(W, [hidden, rows])
    return jm.Tensor(quant, [hidden, rows], orc.quantize_rows(quant, W).reshape(-1))


@pytest.mark.parametrize("quant", [jm.F32, jm.Q8_0, jm.Q4_K])
@pytest.mark.parametrize("T", [1, 7, 8, 64])
@pytest.mark.parametrize("rows", [10000, 10240])
def test_gpu_lm_head(quant, T, rows):
    """moe_lm_head against the oracle's project_lm_head: fewer logits than
    head rows (the first rows), more (the rows past the head are
    normed * 0.05, bit for bit), and the tied token_embd head when
    output.weight is absent. Rows within 1e-2 max relative error. 10240 rows
    (whole 128-row tiles) take the int8 tensor-core launch from 8 tokens and
    the f16 tensor-core GEMM from 16."""
    hidden = 1024
    head = _lm_head_case(quant, hidden, rows, 3)
    x = np.random.default_rng(T).standard_normal((T, hidden)).astype(np.float32)
    with jm.Context(0, 64, 1) as ctx:
        ctx.lm_head_upload(head, None, hidden)
        for n in (9000, rows + 50):
            got = ctx.lm_head(x, n)
            ref = orc.lm_head(head, hidden, x, n)
            assert np.all(np.isfinite(got))
            tgt = min(n, rows)
            assert row_rel_err(got[:, :tgt], ref[:, :tgt]).max() <= OUT_TOL
            np.testing.assert_array_equal(got[:, tgt:], ref[:, tgt:])
        ctx.lm_head_upload(None, head, hidden)   # tied embeddings
        got = ctx.lm_head(x, rows)
        assert row_rel_err(got, orc.lm_head(head, hidden, x, rows)).max() <= OUT_TOL
        # device pointers with every logit a head row: the product writes the
        # caller's buffer directly; bit for bit the host call
        import torch
        xd = torch.from_numpy(x).cuda()
        od = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()   # the fill runs on torch's stream, the head on the context's
        ctx.lm_head_ptrs(T, xd.data_ptr(), od.data_ptr(), rows)
        assert ctx.device_status() == 0
        np.testing.assert_array_equal(od.cpu().numpy(), got)


def test_gpu_lm_head_flat_synthetic_device_pointers_and_errors():
    """A flat head of n_logits * hidden elements, the synthetic logits (no
    head, or one that fits no branch), device pointers (bit for bit the host
    call), T = 0, and the errors: no upload, T above max_tokens, an
    unsupported quantisation, a byte count that does not match the shape."""
    import torch
    hidden, T, n = 512, 5, 777
    rng = np.random.default_rng(1)
    x = rng.standard_normal((T, hidden)).astype(np.float32)
    flat = jm.Tensor(jm.Q8_0, [n * hidden],
                     orc.quantize_rows(jm.Q8_0, rng.standard_normal((n, hidden)).astype(np.float32)).reshape(-1))
    with jm.Context(0, 8, 1) as ctx:
        with pytest.raises(jm.NotUploaded):
            ctx.lm_head(x, n)
        ctx.lm_head_upload(flat, None, hidden)
        got = ctx.lm_head(x, n)
        assert row_rel_err(got, orc.lm_head(flat, hidden, x, n)).max() <= OUT_TOL
        syn = ctx.lm_head(x, n + 1)   # the flat head no longer fits: synthetic logits
        np.testing.assert_allclose(syn, orc.lm_head(None, hidden, x, n + 1), rtol=0, atol=2e-6)
        xd = torch.from_numpy(x).cuda()
        for m in (n, n + 1):
            od = torch.empty((T, m), dtype=torch.float32, device="cuda")
            ctx.lm_head_ptrs(T, xd.data_ptr(), od.data_ptr(), m)
            assert ctx.device_status() == 0
            np.testing.assert_array_equal(od.cpu().numpy(), ctx.lm_head(x, m))
        ctx.lm_head_upload(None, None, hidden)
        np.testing.assert_allclose(ctx.lm_head(x, 300), orc.lm_head(None, hidden, x, 300), rtol=0, atol=2e-6)
        assert ctx.lm_head(x[:0], 300).shape == (0, 300)
        with pytest.raises(jm.ContextLengthExceeded):
            ctx.lm_head(np.zeros((9, hidden), np.float32), 300)
        with pytest.raises(jm.CapabilityMismatch):
            ctx.lm_head_upload(jm.Tensor(14, [hidden, 4],
                                         np.zeros(4 * 420, np.uint8)), None, hidden)
        with pytest.raises(jm.TensorBoundsError):
            ctx.lm_head_upload(jm.Tensor(jm.Q8_0, [hidden, 4], np.zeros(10, np.uint8)), None, hidden)


@pytest.mark.parametrize("quant", [jm.Q8_0, jm.Q4_K])
def test_gpu_lm_head_tensor_cores_match_streaming(quant):
    """The int8 tensor-core product and the streaming one over the same head
    and rows: the same integer block sums, f32 sums in another order."""
    hidden, rows, T = 2048, 4096, 24
    head = _lm_head_case(quant, hidden, rows, 8)
    x = np.random.default_rng(2).standard_normal((T, hidden)).astype(np.float32)
    outs = []
    for flags in (jm.FLAG_INT8_TENSOR_CORES_NEVER, jm.FLAG_INT8_TENSOR_CORES_ALWAYS):
        with jm.Context(0, T, 1, flags=flags) as ctx:
            ctx.lm_head_upload(head, None, hidden)
            outs.append(ctx.lm_head(x, 3000))
    assert row_rel_err(outs[1], outs[0]).max() <= 1e-5
    assert row_rel_err(outs[1], orc.lm_head(head, hidden, x, 3000)).max() <= OUT_TOL


def test_gpu_lm_head_tied_embedding_fixture():
    """The tied token embedding of the reference's own test model (f32,
    [hidden 8, vocab 16]) as the head when output.weight is absent: finite,
    not all zero, and the oracle's logits within 1e-5."""
    from kat_util import tied_embedding_fixture
    hidden, vocab, emb = tied_embedding_fixture()
    x = np.random.default_rng(3).standard_normal((2, hidden)).astype(np.float32)
    with jm.Context(0, 4, 1) as ctx:
        ctx.lm_head_upload(None, emb, hidden)
        got = ctx.lm_head(x, vocab)
    assert np.all(np.isfinite(got)) and np.any(np.abs(got) > 1e-6)
    np.testing.assert_allclose(got, orc.lm_head(emb, hidden, x, vocab), rtol=1e-5, atol=1e-6)
