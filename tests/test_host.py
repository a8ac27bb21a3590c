"""Host-side logic of libjeromoe.so that needs no GPU: the exported C ABI,
the quantiser and generator, descriptor validation and the HBM admission check
(run against a fixed inspector, as the reference's MockMemoryInspector tests do)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import jeromoe as jm
import oracle as orc
import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^[a-z_][\w \*]*?\b(moe_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 13
    lib = C.CDLL(jm.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(jm.EXPORTS), set(names) - set(jm.EXPORTS)


def test_row_bytes_match_gguf_blocks():
    assert jm.row_bytes(jm.Q8_0, 2048) == 64 * 34
    assert jm.row_bytes(jm.Q4_K, 2048) == 8 * 144
    assert jm.row_bytes(jm.Q4_K, 1408) == 0
    assert jm.row_bytes(jm.F32, 7) == 28
    for q in (jm.Q8_0, jm.Q4_K):
        for cols in (256, 512, 5120):
            assert jm.row_bytes(q, cols) == orc.row_bytes(q, cols)


@pytest.mark.parametrize("quant,tol", [(jm.Q8_0, 0.006), (jm.Q4_K, 0.09)])
def test_quantiser_round_trip_through_oracle_decoder(quant, tol):
    x = jm.gen_normal(7, 5, 64 * 512, 0.02).reshape(64, 512)
    q = jm.quantize_rows(quant, x)
    deq = np.stack([orc.dequantize_row(quant, q[r], 512) for r in range(64)])
    rel = np.sqrt(np.mean((deq - x) ** 2)) / 0.02
    assert rel < tol, rel
    if quant == jm.Q8_0:
        # every block: |err| <= d/2 (plus f16 rounding of d)
        d = np.array([orc.f16_to_f32(int(q[r, 34 * b]) | (int(q[r, 34 * b + 1]) << 8))
                      for r in range(64) for b in range(16)]).reshape(64, 16)
        err = np.abs(deq - x).reshape(64, 16, 32).max(-1)
        assert np.all(err <= d * 0.5 * 1.01 + 1e-9)


def test_generator_is_counter_based_and_normal():
    a = jm.gen_normal(3, 11, 100001, 1.0, n_threads=1)
    b = jm.gen_normal(3, 11, 100001, 1.0, n_threads=7)
    np.testing.assert_array_equal(a, b)
    c = jm.gen_normal(3, 11, 1000, 1.0)
    np.testing.assert_array_equal(a[:1000], c)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02
    assert not np.array_equal(a[:1000], jm.gen_normal(3, 12, 1000, 1.0))


def _fake_desc(cfg, data_holder):
    """A descriptor with real shapes/sizes and a dummy data pointer: admission
    reads shapes, quant ids and byte counts only."""
    ptr = data_holder.ctypes.data
    d = jm.moe_layer_desc()
    d.hidden, d.num_experts, d.top_k, d.expert_ffn_dim = cfg.H, cfg.E, cfg.k, cfg.I
    d.use_shared_expert = int(cfg.S > 0)
    d.route_mode = cfg.route.mode
    d.normalize = int(cfg.normalize)
    d.n_groups, d.topk_groups, d.routed_scale = cfg.n_groups, cfg.topk_groups, cfg.routed_scale

    def t(quant, shape):
        m = jm.moe_tensor()
        m.data = ptr
        rows = int(np.prod(shape[1:]))
        m.nbytes = jm.row_bytes(quant, shape[0]) * rows
        m.quant, m.n_dims = quant, len(shape)
        for i, s in enumerate(shape):
            m.shape[i] = s
        return m
    q = cfg.quant
    d.router = t(jm.F32, [cfg.H, cfg.E])
    d.gate_exps = t(q, [cfg.H, cfg.I, cfg.E])
    d.up_exps = t(q, [cfg.H, cfg.I, cfg.E])
    d.down_exps = t(synth.pick_quant(q, cfg.I), [cfg.I, cfg.H, cfg.E])
    if cfg.S:
        d.gate_shexp = t(q, [cfg.H, cfg.S])
        d.up_shexp = t(q, [cfg.H, cfg.S])
        d.down_shexp = t(synth.pick_quant(q, cfg.S), [cfg.S, cfg.H])
    return d


def test_admission_qwen3_30b_a3b_moe_layers():
    """The structure of test_qwen3_30b_a3b_admission (tests/residency_admission_test.rs:183-233):
    the 48 Qwen3-30B-A3B MoE layers (Q4_K) are admitted under a 28 GiB budget and
    rejected fail-closed under a smaller one."""
    holder = np.zeros(16, dtype=np.uint8)
    cfg = synth.CONFIGS[2]
    descs = [_fake_desc(cfg, holder) for _ in range(48)]
    gib = 1 << 30
    fp = jm.admission_check(0, 64, descs, free_bytes=28 * gib)
    per_layer = 128 * 2654208 + 128 * 2048 * 4
    assert fp.weight_bytes >= 48 * per_layer
    assert fp.weight_bytes < 48 * per_layer * 1.01
    assert fp.total_required_bytes == fp.weight_bytes + fp.scratch_bytes
    assert fp.total_required_bytes <= 28 * gib
    with pytest.raises(jm.InsufficientLockableMemory):
        jm.admission_check(0, 64, descs, free_bytes=8 * gib)
    # the reserve is subtracted from the free bytes
    with pytest.raises(jm.InsufficientLockableMemory):
        jm.admission_check(0, 64, descs, free_bytes=28 * gib, reserve_bytes=20 * gib)


def test_admission_downgrades_optional_prefill_arena():
    """Base footprint fits, the optional large-T arena does not -> admitted with
    the arena dropped (check_footprint_against_inspector, src/memory.rs:1599-1602)."""
    holder = np.zeros(16, dtype=np.uint8)
    cfg = synth.CONFIGS[2]
    d = [_fake_desc(cfg, holder)]
    big = jm.admission_check(0, 8192, d, free_bytes=1 << 40)
    assert big.prefill_enabled == 1 and big.prefill_arena_bytes > 0
    tight = big.total_required_bytes + big.prefill_arena_bytes // 2
    fp = jm.admission_check(0, 8192, d, free_bytes=tight)
    assert fp.prefill_enabled == 0 and fp.prefill_arena_bytes == 0
    assert fp.total_required_bytes == big.total_required_bytes


def test_descriptor_validation_errors():
    holder = np.zeros(16, dtype=np.uint8)
    cfg = synth.CONFIGS[2]
    d = _fake_desc(cfg, holder)
    d.gate_exps.quant = 14  # Q6_K: not supported by this path
    with pytest.raises(jm.CapabilityMismatch):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)
    d = _fake_desc(cfg, holder)
    d.down_exps.nbytes -= 1
    with pytest.raises(jm.TensorBoundsError):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)
    d = _fake_desc(cfg, holder)
    d.router.data = None
    with pytest.raises(jm.CapabilityMismatch):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)
    d = _fake_desc(cfg, holder)
    d.top_k = 17
    with pytest.raises(jm.CapabilityMismatch):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)
    d = _fake_desc(synth.CONFIGS[5], holder)
    d.topk_groups = 8
    with pytest.raises(jm.CapabilityMismatch):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)
    d = _fake_desc(cfg, holder)
    d.gate_exps.shape[2] = 127
    with pytest.raises(jm.TensorBoundsError):
        jm.admission_check(0, 64, [d], free_bytes=1 << 40)


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device error path")
def test_context_without_device_fails_closed():
    with pytest.raises(jm.MoeError) as ei:
        jm.Context(0, 64, 1)
    assert ei.value.code in (jm.MOE_ERR_RESOURCE_EXHAUSTED, jm.MOE_ERR_CUDA)
    assert "device" in jm.lib.moe_last_error_message(None).decode().lower()


def test_invalid_arguments_without_context():
    assert jm.lib.moe_forward(None, 0, 1, None, None, None, None, 0) == jm.MOE_ERR_INVALID_ARGS
    assert jm.lib.moe_layer_upload(None, 0, None) == jm.MOE_ERR_INVALID_ARGS
    assert jm.lib.moe_ctx_destroy(None) == jm.MOE_OK
