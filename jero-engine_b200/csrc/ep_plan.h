// ep_plan.h -- host-side plan of one expert-parallel exchange.
//
// World of G ranks; rank g owns the experts [g*E/G, (g+1)*E/G) and routes its
// own token shard. After routing, each rank's slots are in its canonical order
// (expert ascending, then token ascending), so the slots bound for rank r are
// one contiguous run: the experts of r. Every rank knows every rank's slot
// offsets (all-gathered), which fixes:
//   send:  rows [send_off[r], send_off[r] + send_cnt[r]) of my slots go to r;
//   recv:  rank s's rows for my experts land at recv_off[s] (source order);
//   local problems: my experts with tokens, slots in (expert, source, token)
//          order -- the global canonical order restricted to my experts;
//   segments: slot_base .. slot_base + count of a (local expert, source) pair
//          read the received rows row_base .. row_base + count.
// Expert outputs are written back at their received row, so the return
// exchange (the same runs with send and receive swapped) hands each source
// its rows in its own slot order.
#pragma once

#include <cstdint>
#include <vector>

namespace jmoe {

struct EpProblem {
    int32_t expert;   // local expert index (0 .. E/G - 1)
    int32_t slot0, count;
};

struct EpSegment {
    int32_t slot_base, row_base, count;
};

struct EpPlan {
    std::vector<int32_t> send_cnt, send_off, recv_cnt, recv_off;   // rows, per peer rank
    std::vector<EpProblem> problems;
    std::vector<EpSegment> segs;
    int32_t n_recv = 0;
};

// all_off: [world][E + 1] slot offsets by expert of every rank (offsets[e] =
// slots of experts below e). Returns false if E is not a multiple of world or
// an offset table is not monotone.
inline bool ep_plan(int rank, int world, int E, const int32_t *all_off, EpPlan &out)
{
    if (world <= 0 || rank < 0 || rank >= world || E <= 0 || E % world) return false;
    const int El = E / world, e0 = rank * El;
    auto off = [&](int s, int e) { return all_off[(size_t)s * (E + 1) + e]; };
    for (int s = 0; s < world; s++)
        for (int e = 0; e < E; e++)
            if (off(s, e + 1) < off(s, e) || off(s, 0) != 0) return false;
    out = EpPlan{};
    out.send_cnt.resize(world);
    out.send_off.resize(world);
    out.recv_cnt.resize(world);
    out.recv_off.resize(world);
    for (int r = 0; r < world; r++) {
        out.send_off[r] = off(rank, r * El);
        out.send_cnt[r] = off(rank, (r + 1) * El) - off(rank, r * El);
    }
    int32_t acc = 0;
    for (int s = 0; s < world; s++) {
        out.recv_off[s] = acc;
        out.recv_cnt[s] = off(s, e0 + El) - off(s, e0);
        acc += out.recv_cnt[s];
    }
    out.n_recv = acc;
    int32_t slot = 0;
    for (int el = 0; el < El; el++) {
        const int e = e0 + el;
        int32_t cnt = 0;
        for (int s = 0; s < world; s++) cnt += off(s, e + 1) - off(s, e);
        if (!cnt) continue;
        out.problems.push_back({el, slot, cnt});
        int32_t within = 0;
        for (int s = 0; s < world; s++) {
            const int32_t c = off(s, e + 1) - off(s, e);
            if (!c) continue;
            out.segs.push_back({slot + within, out.recv_off[s] + (off(s, e) - off(s, e0)), c});
            within += c;
        }
        slot += cnt;
    }
    return true;
}

}  // namespace jmoe
