"""Expert parallelism: the exchange plan (host logic, CPU ranks over gloo)
and moe_forward_ep against moe_forward (GPU)."""
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import jeromoe as jm
import synth
from ep_util import gpu_worker, plan_worker


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_plan_two_ranks_by_hand():
    # rank 0 slots per expert (1, 2, 0, 2), rank 1 (0, 2, 2, 0); 4 experts over 2 ranks
    offs = np.array([[0, 1, 3, 3, 5], [0, 0, 2, 4, 4]], dtype=np.int32)
    p0 = jm.ep_plan(0, 2, 4, offs)
    assert p0.send_cnt.tolist() == [3, 2] and p0.send_off.tolist() == [0, 3]
    assert p0.recv_cnt.tolist() == [3, 2] and p0.recv_off.tolist() == [0, 3]
    assert p0.problems.tolist() == [[0, 0, 1], [1, 1, 4]]
    assert p0.segments.tolist() == [[0, 0, 1], [1, 1, 2], [3, 3, 2]]
    p1 = jm.ep_plan(1, 2, 4, offs)
    assert p1.send_cnt.tolist() == [2, 2] and p1.recv_cnt.tolist() == [2, 2]
    assert p1.problems.tolist() == [[0, 0, 2], [1, 2, 2]]
    assert p1.segments.tolist() == [[0, 2, 2], [2, 0, 2]]


def test_ep_plan_rejects_bad_input():
    offs = np.zeros((2, 6), dtype=np.int32)
    with pytest.raises(jm.MoeError):
        jm.ep_plan(0, 2, 5, offs)   # 5 experts do not split over 2 ranks
    bad = np.array([[0, 2, 1, 3, 3]], dtype=np.int32)
    with pytest.raises(jm.MoeError):
        jm.ep_plan(0, 1, 4, bad)    # offsets must be monotone


@pytest.mark.parametrize("world,E,k,T_total", [(2, 8, 2, 37), (2, 16, 4, 64), (3, 6, 2, 2), (4, 8, 3, 19)])
def test_ep_exchange_over_gloo(world, E, k, T_total):
    """Both exchanges of the plan with gloo ranks on CPU (a rank may have no tokens)."""
    mp.spawn(plan_worker, args=(world, free_port(), E, k, T_total, 7), nprocs=world, join=True)


# ------------------------------------------------------------------ GPU

def _ep_layer(cfg_id, over, flags, T):
    cfg = synth.CONFIGS[cfg_id].scaled(**over)
    w = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    d, keep = jm.layer_desc(w, 0, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H)
    return cfg, d, keep, x


# max_tokens <= 256 uses the exchange over peer memory, larger the NCCL one;
# FLAG_EP_NCCL_ONLY keeps the NCCL exchange covered for small batches too.
# STREAM / INT8 pin the expert path of small batches (streaming kernels or
# int8 tensor cores); both are deterministic, so EP equals moe_forward bit
# for bit on them.
STREAM = jm.FLAG_TENSOR_CORES_NEVER | jm.FLAG_INT8_TENSOR_CORES_NEVER
INT8 = jm.FLAG_TENSOR_CORES_NEVER | jm.FLAG_INT8_TENSOR_CORES_ALWAYS
EP1_CASES = {
    "cfg2_stream": (2, dict(E=16, I=256, H=512), STREAM, 40, True),
    "cfg2_stream_nccl": (2, dict(E=16, I=256, H=512), STREAM | jm.FLAG_EP_NCCL_ONLY, 40, True),
    "cfg3_shared_stream": (3, dict(E=16, k=4, I=384, S=512, H=512), STREAM, 33, True),
    "cfg2_int8": (2, dict(E=16, I=256, H=512), INT8, 40, True),
    # default flags: the local experts of the peer-memory exchange run the fused
    # f16 launch over the received rows, the single-GPU forward the fused int8
    # one -- two arithmetics, compared within the contract tolerance
    "cfg2_fused": (2, dict(E=16, I=256, H=512), 0, 40, False),
    "cfg3_shared_int8_nccl": (3, dict(E=16, k=4, I=384, S=512, H=512), INT8 | jm.FLAG_EP_NCCL_ONLY, 33, True),
    "cfg5_groups_shared_int8": (5, dict(E=32, k=6, I=256, S=512, H=512, n_groups=8, topk_groups=3), INT8, 64, True),
    "cfg2_tensor_cores": (2, dict(E=16, I=256, H=512), jm.FLAG_TENSOR_CORES_ALWAYS, 300, False),
    "cfg5_groups_shared_tc": (5, dict(E=32, k=6, I=256, S=512, H=512, n_groups=8, topk_groups=3),
                              jm.FLAG_TENSOR_CORES_ALWAYS, 260, False),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(EP1_CASES))
def test_gpu_ep_world_of_one_matches_forward(name):
    """A world of one rank runs every step of the expert-parallel forward (the
    peer-memory exchange with itself, or NCCL send/recv to itself): same
    routing and output as moe_forward, also on a second call."""
    cid, over, flags, T, exact = EP1_CASES[name]
    cfg, d, keep, x = _ep_layer(cid, over, flags, T)
    uid = jm.ep_unique_id()
    with jm.Context(0, T, 1, flags=flags) as ep, jm.Context(0, T, 1, flags=flags) as ref:
        ep.ep_init(0, 1, uid)
        ep.upload(0, d)
        ref.upload(0, d)
        out, si, sw = ep.forward_ep(0, x)
        out2, _, _ = ep.forward_ep(0, x)
        r_out, r_si, r_sw = ref.forward(0, x)
        empty, _, _ = ep.forward_ep(0, x[:0])
        assert empty.shape == (0, cfg.H)
        assert ep.device_status() == 0
    np.testing.assert_array_equal(si, r_si)
    np.testing.assert_array_equal(sw, r_sw)
    np.testing.assert_array_equal(out, out2)
    if exact:
        np.testing.assert_array_equal(out, r_out)
    else:
        from kat_util import row_rel_err
        assert row_rel_err(out, r_out).max() <= 1e-2


@pytest.mark.gpu
def test_gpu_ep_requires_init_and_split():
    cfg, d, keep, x = _ep_layer(2, dict(E=16, I=256, H=512), 0, 4)
    with jm.Context(0, 4, 1) as ctx:
        ctx.upload(0, d)
        with pytest.raises(jm.MoeError):
            ctx.forward_ep(0, x)   # no moe_ep_init
        with pytest.raises(jm.MoeError):
            ctx.ep_init(0, 1, jm.ep_unique_id())   # after an upload


@pytest.mark.gpu
@pytest.mark.parametrize("flags,exact,T", [(STREAM, True, 40),
                                           (STREAM | jm.FLAG_EP_NCCL_ONLY, True, 40),
                                           (INT8, True, 40),
                                           (0, False, 40),
                                           (0, False, 1),   # one token per rank: the streaming local stage
                                           (jm.FLAG_TENSOR_CORES_ALWAYS, False, 300)])
def test_gpu_ep_two_ranks(flags, exact, T):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    over = dict(E=16, k=4, I=384, S=512, H=512)
    mp.spawn(gpu_worker, args=(2, free_port(), 3, over, T, flags, exact), nprocs=2, join=True)


@pytest.mark.gpu
def test_gpu_ep_peer_wait_times_out_and_recovers():
    """Failure detection without a device fault: a world of one on the
    peer-memory exchange is made to wait for a flag epoch that nothing raises,
    with the flag waits bounded to about a millisecond. The forward returns
    MOE_ERR_TIMEOUT naming the peer-rank wait, within a short host-side limit;
    later forwards refuse until moe_ep_reset; after it the context is usable
    and matches moe_forward again."""
    import time
    cfg, d, keep, x = _ep_layer(2, dict(E=16, I=256, H=512), STREAM, 40)
    uid = jm.ep_unique_id()
    with jm.Context(0, 40, 1, flags=STREAM) as ep, jm.Context(0, 40, 1, flags=STREAM) as ref:
        ep.ep_init(0, 1, uid)
        ep.upload(0, d)
        ref.upload(0, d)
        r_out, r_si, _ = ref.forward(0, x)
        out0, _, _ = ep.forward_ep(0, x)
        np.testing.assert_array_equal(out0, r_out)
        ep.debug_ep_fault(5, 2_000_000)   # ~1 ms per wait at 2 GHz
        t0 = time.time()
        with pytest.raises(jm.DeviceTimeout) as ei:
            ep.forward_ep(0, x)
        assert time.time() - t0 < 5.0
        assert "peer-rank" in ei.value.msg
        with pytest.raises(jm.DeviceTimeout) as ei2:
            ep.forward_ep(0, x)   # refused until the world resets
        assert "moe_ep_reset" in ei2.value.msg
        ep.ep_reset()
        ep.debug_ep_fault(0, 0)
        out, si, _ = ep.forward_ep(0, x)
        assert ep.device_status() == 0
    np.testing.assert_array_equal(si, r_si)
    np.testing.assert_array_equal(out, r_out)
