// fused_common.cuh -- pieces shared by the fused small-batch expert launches
// (experts_tc.cu: f16 operands; experts_i8.cu: int8 operands): the work-item
// table of gate/up and down items and the Q4_K scale decode.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "moe_device.h"
#include "tc_common.cuh"

namespace jmoe {

struct XItem {
    int phase;       // 0 gate/up, 1 down
    int expert, slot, n, tile, chunk;
    bool shared;
};

// Item `it` of the launch, problems cut into chunks of at most `cap` slots.
// Table: s_prob[q] = (expert, slot0, count, shared), s_o0[q] / s_o1[q] the
// first gate/up / down item of problem q (s_o0[nq] = the number of gate/up
// items), s_cb[q] the first slot chunk of q. Chunks of a tile are adjacent
// items, so CTAs that share a weight tile read it together.
__device__ __forceinline__ XItem x_item(const int *s_o0, const int *s_o1, const int *s_cb, const int4 *s_prob,
                                        int nq, int it, int cap = 32)
{
    XItem x;
    const int total0 = s_o0[nq];
    x.phase = it >= total0 ? 1 : 0;
    const int *off = x.phase ? s_o1 : s_o0;
    const int local_it = x.phase ? it - total0 : it;
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= local_it) lo = mid;
        else hi = mid - 1;
    }
    const int4 pr = s_prob[lo];
    // chunks of equal size rounded up to 16 slots (the MMA's N granularity),
    // or to the cap when it is below 16
    const int gran = cap < 16 ? cap : 16, nch = chunk_count(pr.z, cap);
    const int base = ((pr.z + nch - 1) / nch + gran - 1) / gran * gran;
    const int local = local_it - off[lo];
    const int ch = local % nch;
    x.tile = local / nch;
    x.expert = pr.x;
    x.slot = pr.y + ch * base;
    x.n = min(base, pr.z - ch * base);
    x.chunk = s_cb[lo] + ch;
    x.shared = pr.w != 0;
    return x;
}

__device__ __forceinline__ const DevMatrix &x_mat(const LayerDev &L, const XItem &x)
{
    return x.phase == 0 ? (x.shared ? L.sh_gate : L.gate) : (x.shared ? L.sh_down : L.down);
}

// Q4_K scales of the eight sub-blocks of a super-block from the device meta
// row (f16 d, f16 dmin, eight 12-bit fields sc | m << 6 from bit 32).
__device__ __forceinline__ void q4_scales_all(const uint4 &m, float (&sc)[8], float (&mn)[8])
{
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&m.x));
    const uint64_t lo = (uint64_t)m.y | ((uint64_t)m.z << 32);
    const uint32_t w2 = m.w;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int bit = 12 * j;
        const uint32_t f = bit + 12 <= 64 ? (uint32_t)(lo >> bit) & 0xFFFu
                                          : (bit >= 64 ? (w2 >> (bit - 64)) & 0xFFFu
                                                       : ((uint32_t)(lo >> bit) | (w2 << (64 - bit))) & 0xFFFu);
        sc[j] = dd.x * (float)(f & 63u);
        mn[j] = dd.y * (float)(f >> 6);
    }
}

}  // namespace jmoe
