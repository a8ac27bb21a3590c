// ep_p2p.h -- expert-parallel exchange over peer memory (small batches).
//
// Every rank owns one arena with the same layout; the ranks map each other's
// arenas (CUDA IPC) once, so kernels write straight into a peer's inbox over
// NVLink. Two phases per forward, each announced by raising a per-source
// epoch flag in every peer's arena (system-scope release store) and awaited
// with a bounded spin (system-scope acquire load):
//   rows   : my slot offsets by expert -> every rank's offset inbox, and my
//            routed rows (int8 blocks + scales, or the f16 rows of the fused
//            expert launch) -> the owner's row inbox;
//            the receiver's plan waits for every source's rows flag;
//   outputs: expert outputs of received rows -> the source's output inbox
//            (stored by the fused expert launch itself, or by a return pass).
// Reuse across forwards is ordered by the phases themselves. A rank writes a
// peer's offset and row inboxes for forward n only after its own forward n-1
// has finished, which waited for that peer's outputs of n-1; the peer raises
// them only after its expert stage of n-1, the last reader of those inboxes.
// A peer writes my output inbox for forward n only after its expert stage of
// n, which needs my rows of n, sent after my combine of n-1 (its reader). So
// a flag never runs ahead of the forward that waits for it: a rank waits for
// exactly its own epoch, and a later epoch is reported as a desync. When the
// rows wait fails (a peer missing or out of step), the rank stores no outputs
// into any peer's arena and raises no outputs flag; its peers' waits then run
// out as well, and every rank must reset the exchange (moe_ep_reset) before
// the next forward, which restores the ordering above.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "moe_device.h"

namespace jmoe {

constexpr int kEpMaxRanks = 8;
constexpr int kEpP2PMaxTokens = 256;   // per rank; larger batches use the NCCL exchange
constexpr int kErrEpTimeout = 2;       // device status: a peer's flag did not arrive in time
constexpr int kErrEpDesync = 3;        // device status: a peer's flag was already past this forward
constexpr int kEpPhaseRows = 0, kEpPhaseOut = 1, kEpPhases = 2;

struct EpP2PLayout {
    int world = 0, E = 0, El = 0, H = 0, W = 0, cap = 0, slots_y = 0;
    size_t rb = 0;          // bytes of one packed row: H int8 + H/32 d + H/32 s
    // regions other ranks write
    size_t o_flags = 0;     // [kEpPhases][kEpMaxRanks] uint32 epoch flags (phase, source)
    size_t o_off = 0;       // [world][E+1] int32 slot offsets of each source
    size_t o_xin = 0;       // [world][cap][rb] rows received from each source
    size_t o_yin = 0;       // [slots_y][H] f32 outputs of my own slots (routed, then shared)
    // regions only this rank touches
    size_t o_peers = 0;     // [kEpMaxRanks] arena bases of the ranks (device copy)
    size_t o_misc = 0;      // tickets [2], n_active, total, a zero word, ok (16 B each)
    size_t o_prob = 0;      // [El] Problem
    size_t o_perm = 0;      // [world*cap] received row of each local slot
    size_t o_ret = 0;       // [world*cap] int2 (source rank, source slot) of each local slot
    size_t o_aq = 0, o_ad = 0, o_as = 0;   // SwiGLU blocks of the local slots [world*cap][W]
    size_t o_y = 0;         // [world*cap][H] f32 expert outputs of the local slots
    size_t o_x16 = 0;       // [world*cap][H] f16 rows received from each source, written by the
                            // sources when the fused f16 expert launch takes them
    size_t o_a16dn = 0;     // [world*cap][W] f16 down operand of the local slots (same launch)
    size_t bytes = 0;
};

inline size_t ep_align(size_t v) { return (v + 255) / 256 * 256; }

// cap: rows one source may send to one rank (its max_tokens * k); slots_y: my
// routed slots plus shared rows (max_tokens * k + max_tokens).
inline EpP2PLayout ep_p2p_layout(int world, int E, int H, int W, int cap, int slots_y)
{
    EpP2PLayout l;
    l.world = world; l.E = E; l.El = E / world; l.H = H; l.W = W < 32 ? 32 : W; l.cap = cap; l.slots_y = slots_y;
    l.rb = (size_t)H + 8 * (size_t)(H / 32);
    const size_t R = (size_t)world * cap;
    size_t o = 0;
    auto take = [&](size_t b) { size_t r = o; o += ep_align(b ? b : 1); return r; };
    l.o_flags = take(kEpPhases * kEpMaxRanks * 4);
    l.o_off = take((size_t)world * (E + 1) * 4);
    l.o_xin = take(R * l.rb);
    l.o_yin = take((size_t)slots_y * H * 4);
    l.o_peers = take(kEpMaxRanks * sizeof(void *));
    l.o_misc = take(128);
    l.o_prob = take((size_t)l.El * sizeof(Problem));
    l.o_perm = take(R * 4);
    l.o_ret = take(R * 8);
    l.o_aq = take(R * l.W);
    l.o_ad = take(R * (l.W / 32) * 4);
    l.o_as = take(R * (l.W / 32) * 4);
    l.o_y = take(R * H * 4);
    l.o_x16 = take(R * H * 2);
    l.o_a16dn = take(R * l.W * 2);
    l.bytes = o;
    return l;
}

// Kernel arguments of one forward's exchange.
struct EpP2PArgs {
    uint8_t *const *peers;      // [world] arena bases (device array; peers[rank] = own)
    uint8_t *own;
    int rank, world, E, El, e0, H, cap;
    size_t rb, o_flags, o_off, o_xin, o_yin;
    size_t o_x16;               // 0: rows go out as packed int8 rows into o_xin; else as f16
                                // token rows (the receiver's fused f16 launch) at this offset
    uint32_t epoch;             // this forward's epoch, raised in this rank's flags
    uint32_t wait_epoch;        // the epoch the waits expect (epoch, unless a test skews it)
    long long wait_cycles;      // bound of each flag wait (clock cycles)
    int *err;                   // the context's device status word
    int *ok;                    // own arena: 1 once every source's rows of this forward were seen
    int *ticket;                // [2] in the own arena (dispatch, return)
    int32_t *n_active, *total;  // local problems of the received rows
    Problem *problems;
    int32_t *perm;
    int2 *ret;
    const int32_t *offsets;     // this rank's slot offsets [E+1]
    const int32_t *perm_token;  // this rank's slot -> token
    const int8_t *xq;           // this rank's activation blocks [T][H]
    const float *xd, *xs;       // [T][H/32]
    int n_slots;                // T * k of this rank
    const float *y;             // expert outputs of the received rows, by local slot [*][H]
};

cudaError_t launch_ep_p2p_plan(const EpP2PArgs &a, cudaStream_t st);
cudaError_t launch_ep_p2p_dispatch(const EpP2PArgs &a, int num_sms, cudaStream_t st);
cudaError_t launch_ep_p2p_return(const EpP2PArgs &a, int num_sms, cudaStream_t st);
cudaError_t launch_ep_p2p_wait(const EpP2PArgs &a, int phase, cudaStream_t st);

}  // namespace jmoe
