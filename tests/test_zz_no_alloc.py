"""moe_route_noalloc: routing and dispatch permutation without any allocation.

Some callers cannot allocate device memory themselves or let a library do it:
a runtime that owns all device memory through its own pool, or a decode loop
held to zero allocations once it runs (jero-engine's decode step allocates
nothing). For them the library routes tokens with its working memory in one
fixed static device array; the caller passes device inputs and outputs only.

This file runs last (pytest collects it after the other test files), so a run
that stops at the first failure has already run everything else. It checks,
through the C ABI, that two calls in a row give the same routing as the
context-based moe_forward entry point: indices and permutation bit for bit,
weights within the parity tolerance of the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import jeromoe as jm
import synth

pytestmark = pytest.mark.gpu

W_RTOL = 1e-5


def _route_noalloc(x_dev, router_dev, T, H, E, k, route, lbias_dev=None, sbias_dev=None):
    import torch
    si = torch.empty((max(T, 1), k), dtype=torch.int32, device="cuda")
    sw = torch.empty((max(T, 1), k), dtype=torch.float32, device="cuda")
    offs = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(max(T, 1) * k, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = jm.lib.moe_route_noalloc(
        0, C.c_void_p(x_dev.data_ptr()), C.c_void_p(router_dev.data_ptr()),
        C.c_void_p(lbias_dev.data_ptr() if lbias_dev is not None else None),
        C.c_void_p(sbias_dev.data_ptr() if sbias_dev is not None else None),
        T, H, E, k, int(route.normalize), route.routed_scale,
        route.n_groups if route.mode == jm.ROUTE_GROUP_LIMITED else 0, route.topk_groups,
        C.c_void_p(si.data_ptr()), C.c_void_p(sw.data_ptr()), C.c_void_p(offs.data_ptr()),
        C.c_void_p(perm.data_ptr()), C.c_void_p(stream))
    torch.cuda.synchronize()
    return rc, si.cpu().numpy()[:T], sw.cpu().numpy()[:T], offs.cpu().numpy(), perm.cpu().numpy()[: T * k]


@pytest.mark.parametrize("cid", [2, 5])
def test_route_noalloc_matches_forward_twice(cid):
    import torch
    cfg = synth.CONFIGS[cid].scaled(E=64, I=256, S=256 if cid == 5 else 0, H=512)
    w = synth.build_weights(cfg)
    router = torch.from_numpy(w.tensor("blk.0.ffn_gate_inp.weight").data.reshape(cfg.E, cfg.H).copy()).cuda()
    ctx = jm.Context(0, 300, 1)
    d, keep = synth.desc_for(cfg, w)
    ctx.upload(0, d)
    # calls in a row with different token counts: the small-batch kernel after
    # the tiled one relies on the routing tickets being back at zero
    for T in (37, 300, 37):
        x = synth.gen_x(cfg.scaled(seed=cfg.seed + T), T)
        _, ref_si, ref_sw = ctx.forward(0, x)
        ref_offs, ref_perm = ctx.debug_permutation(cfg.E, cfg.k)
        rc, si, sw, offs, perm = _route_noalloc(torch.from_numpy(x).cuda(), router, T, cfg.H, cfg.E, cfg.k,
                                                cfg.route)
        assert rc == jm.MOE_OK, jm.lib.moe_last_error_message(None)
        np.testing.assert_array_equal(si, ref_si)
        np.testing.assert_allclose(sw, ref_sw, rtol=W_RTOL, atol=1e-7)
        np.testing.assert_array_equal(offs, ref_offs)
        np.testing.assert_array_equal(perm, ref_perm)
    ctx.close()


def test_route_noalloc_hidden_not_a_multiple_of_four():
    """H = 510 takes the scalar router and the ticketed selection kernel (no
    memset): routing and permutation equal the CPU oracle's, twice in a row,
    and the caller's current device is left as it was."""
    import torch
    import oracle as orc
    H, E, k = 510, 32, 4
    rng = np.random.default_rng(3)
    router_h = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    wts = jm.ModelWeights({"blk.0.ffn_gate_inp.weight": jm.f32_tensor(router_h, [H, E])})
    L = orc.Layer(wts, 0, E, k, False, hidden=H)
    router = torch.from_numpy(router_h).cuda()
    for T in (19, 19):
        x = rng.standard_normal((T, H)).astype(np.float32)
        dev_before = torch.cuda.current_device()
        rc, si, sw, offs, perm = _route_noalloc(torch.from_numpy(x).cuda(), router, T, H, E, k, jm.RouteSpec())
        assert rc == jm.MOE_OK, jm.lib.moe_last_error_message(None)
        assert torch.cuda.current_device() == dev_before
        ref_si = np.stack([L.select(orc.router_logits(router_h, x[t]))[0] for t in range(T)])
        ref_sw = np.stack([L.select(orc.router_logits(router_h, x[t]))[1] for t in range(T)])
        np.testing.assert_array_equal(si, ref_si)
        np.testing.assert_allclose(sw, ref_sw, rtol=W_RTOL, atol=1e-7)
        ro, rp = orc.permutation(ref_si, E)
        np.testing.assert_array_equal(offs, ro)
        np.testing.assert_array_equal(perm, rp)


def test_route_noalloc_rejects_oversized_calls():
    import torch
    x = torch.zeros((1025, 64), dtype=torch.float32, device="cuda")
    router = torch.zeros((8, 64), dtype=torch.float32, device="cuda")
    rc, *_ = _route_noalloc(x, router, 1025, 64, 8, 2, jm.RouteSpec())
    assert rc == jm.MOE_ERR_CONTEXT_LENGTH
    assert "1024" in jm.lib.moe_last_error_message(None).decode()
    router = torch.zeros((300, 64), dtype=torch.float32, device="cuda")
    rc, *_ = _route_noalloc(x[:4], router, 4, 64, 300, 2, jm.RouteSpec())
    assert rc == jm.MOE_ERR_CONTEXT_LENGTH
