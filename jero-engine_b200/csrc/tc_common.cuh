// tc_common.cuh -- pieces shared by the tensor-core expert kernels
// (prefill.cu: f16 operands; decode_tc.cu: int8 operands): bounded mbarrier
// waits and the work-item table of (problem, 128-row weight tile, slot chunk).
#pragma once

#include <stdint.h>

#include "ptx.cuh"

namespace jmoe {

constexpr long long kWaitCycles = 4000000000LL;
constexpr int kErrTimeout = 1;

// Waiting warps sleep in try_wait (suspend hint) instead of spinning, so they
// leave the issue slots to the dequant and epilogue warps; the abort flag and
// the clock are checked only when a try_wait times out.
constexpr uint32_t kSleepNs = 20000;

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity, kSleepNs)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicExch(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

// The same bounded wait without the suspend hint: try_wait in a loop (the
// hardware still parks the warp briefly inside each try_wait). For pipelines
// with several hand-offs per K step, where a sleeping waiter's wake-up
// latency would add up on every step.
__device__ __forceinline__ bool tc_spin_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t n = 1;; n++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitCycles) {
                *abort_flag = 1;
                atomicExch(err, kErrTimeout);
                return false;
            }
        }
    }
}

// Bounded wait used while draining after an abort (no error recorded).
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity)
{
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity, kSleepNs) && clock64() - t0 < kWaitCycles) {}
}

struct TcItem {
    int expert, slot, n, nt;   // n: slots of this item (1..cap)
    bool shared;
};

// Slot chunks of a problem: ceil(count / cap) chunks of equal size rounded up
// to 16 (the MMA's N granularity); the last one takes the remainder.
__device__ __forceinline__ int chunk_count(int count, int cap) { return (count + cap - 1) / cap; }
__device__ __forceinline__ int chunk_size(int count, int nch) { return (((count + nch - 1) / nch) + 15) & ~15; }

// The item table lives in shared memory: s_off[0..nq] is the first item of
// each problem of the launch (routed problems in list order, then the shared
// expert), s_prob[q] = (expert, slot0, count, is_shared).
__device__ __forceinline__ TcItem tc_item(const int *s_off, const int4 *s_prob, int nq, int cap, int it)
{
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= it) lo = mid;
        else hi = mid - 1;
    }
    const int4 pr = s_prob[lo];
    const int nch = chunk_count(pr.z, cap), base = chunk_size(pr.z, nch);
    const int local = it - s_off[lo];
    const int ch = local % nch;
    TcItem x;
    x.nt = local / nch;
    x.expert = pr.x;
    x.slot = pr.y + ch * base;
    x.n = min(base, pr.z - ch * base);
    x.shared = pr.w != 0;
    return x;
}

__device__ __forceinline__ void sts128(uint32_t a, uint4 v)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

}  // namespace jmoe
