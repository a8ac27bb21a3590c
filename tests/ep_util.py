"""Workers of the expert-parallel tests, one process per rank (spawned).

plan_worker: CPU-only (gloo). Routes a synthetic token batch, shards the
tokens contiguously, derives each rank's exchange plan with moe_ep_plan from
the all-gathered slot offsets and runs both exchanges over gloo with token
tags as payload: the received slots must be the global canonical permutation
(expert ascending, token ascending) restricted to the rank's experts, and the
returned rows must arrive in the sender's own slot order.

gpu_worker: one GPU per rank. moe_forward_ep of the rank's token shard
against moe_forward of the same tokens on a context that holds all experts.
"""
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

import jeromoe as jm


def _init(rank, world, port, backend="gloo"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60))


def _shard(T_total, world, rank):
    return np.array_split(np.arange(T_total), world)[rank]


def plan_worker(rank, world, port, E, k, T_total, seed):
    _init(rank, world, port)
    try:
        rng = np.random.default_rng(seed)   # the same global routing on every rank
        sel = np.stack([rng.choice(E, k, replace=False) for _ in range(T_total)]) if T_total else np.zeros((0, k), int)
        mine = _shard(T_total, world, rank)
        El, e0 = E // world, rank * (E // world)
        # this rank's slots in its canonical order
        pairs = sorted((int(e), int(t)) for t in range(len(mine)) for e in sel[mine[t]])
        counts = np.bincount([e for e, _ in pairs], minlength=E)
        offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        gathered = [torch.zeros(E + 1, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(offsets))
        all_off = torch.stack(gathered).numpy()
        plan = jm.ep_plan(rank, world, E, all_off)
        assert plan.send_cnt.sum() == len(pairs)
        # dispatch: each slot row carries its global token id
        send = torch.tensor([int(mine[t]) for _, t in pairs], dtype=torch.int64)
        n_recv = int(plan.recv_cnt.sum())
        recv = torch.empty(n_recv, dtype=torch.int64)
        dist.all_to_all_single(recv, send, output_split_sizes=plan.recv_cnt.tolist(),
                               input_split_sizes=plan.send_cnt.tolist())
        recv = recv.numpy()
        slot_tok = np.full(n_recv, -1, dtype=np.int64)
        slot_row = np.full(n_recv, -1, dtype=np.int64)
        slot_exp = np.full(n_recv, -1, dtype=np.int64)
        for sb, rb, c in plan.segments:
            slot_tok[sb:sb + c] = recv[rb:rb + c]
            slot_row[sb:sb + c] = np.arange(rb, rb + c)
        for el, s0, c in plan.problems:
            slot_exp[s0:s0 + c] = e0 + el
        expected = sorted((int(e), t) for t in range(T_total) for e in sel[t] if e0 <= e < e0 + El)
        got = list(zip(slot_exp.tolist(), slot_tok.tolist()))
        assert got == expected, f"rank {rank}: received slots are not the canonical order"
        assert sorted(slot_row.tolist()) == list(range(n_recv)), "segments must cover every received row once"
        # return: outputs written at their received row, tagged (expert, token)
        back_rows = np.zeros((n_recv, 2), dtype=np.int64)
        back_rows[slot_row] = np.stack([slot_exp, slot_tok], axis=1)
        back = torch.empty((len(pairs), 2), dtype=torch.int64)
        dist.all_to_all_single(back, torch.from_numpy(back_rows), output_split_sizes=plan.send_cnt.tolist(),
                               input_split_sizes=plan.recv_cnt.tolist())
        want = [(e, int(mine[t])) for e, t in pairs]
        assert [tuple(r) for r in back.numpy().tolist()] == want, f"rank {rank}: returned rows out of order"
    finally:
        dist.destroy_process_group()


def gpu_worker(rank, world, port, cfg_id, over, T_per_rank, flags, exact):
    import synth
    from kat_util import row_rel_err
    _init(rank, world, port)
    try:
        ids = [jm.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        cfg = synth.CONFIGS[cfg_id].scaled(**over)
        w = synth.build_weights(cfg)
        x_all = synth.gen_x(cfg, T_per_rank * world)
        x = np.ascontiguousarray(x_all[rank * T_per_rank:(rank + 1) * T_per_rank])
        max_tokens = max(T_per_rank, 1)
        ep = jm.Context(rank, max_tokens, 1, flags=flags)
        ep.ep_init(rank, world, ids[0])
        d, keep = jm.layer_desc(w, 0, cfg.E, cfg.k, cfg.I, cfg.S > 0, cfg.route, cfg.H)
        ep.upload(0, d)
        out, si, sw = ep.forward_ep(0, x)
        out2, _, _ = ep.forward_ep(0, x)   # a second call reuses the arena
        ref = jm.Context(rank, max_tokens, 1, flags=flags)
        ref.upload(0, d)
        r_out, r_si, r_sw = ref.forward(0, x)
        np.testing.assert_array_equal(si, r_si)
        np.testing.assert_array_equal(sw, r_sw)
        np.testing.assert_array_equal(out, out2)
        if exact:
            np.testing.assert_array_equal(out, r_out)
        else:
            assert row_rel_err(out, r_out).max() <= 1e-2
        assert ep.device_status() == 0
        ep.close()
        ref.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
