// ep_p2p.cu -- kernels of the expert-parallel exchange over peer memory.
// Peer arenas are written with plain stores from this GPU; nothing reads a
// peer's memory. Every wait on a peer's flag is bounded (about 2 s at 2 GHz
// unless a test shortens it) and records kErrEpTimeout (or kErrEpDesync for a
// flag already past this forward) in the status word instead of waiting on.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "ep_p2p.h"
#include "kernels.h"
#include "ptx.cuh"

namespace jmoe {
namespace {

__device__ __forceinline__ uint32_t *ep_flag(uint8_t *arena, size_t o_flags, int phase, int src)
{
    return reinterpret_cast<uint32_t *>(arena + o_flags) + phase * kEpMaxRanks + src;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until flag == epoch. Returns 0, or kErrEpDesync at once when the flag
// is already past it (wrap-safe), or kErrEpTimeout after `cycles`.
__device__ __forceinline__ int wait_epoch(const uint32_t *flag, uint32_t epoch, long long cycles)
{
    const long long t0 = clock64();
    for (;;) {
        const int32_t d = (int32_t)(ld_acquire_sys(flag) - epoch);
        if (d == 0) return 0;
        if (d > 0) return kErrEpDesync;
        if (clock64() - t0 > cycles) return kErrEpTimeout;
        __nanosleep(256);
    }
}

// Raises this rank's flag of `phase` in every rank's arena once every CTA of
// the grid has finished its stores: a CTA barrier, then one system-scope fence
// and one ticket per CTA (the fence is cumulative over the barrier); the last
// CTA raises the flags.
__device__ __forceinline__ void signal_when_done(const EpP2PArgs &a, int *ticket, int phase)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(ticket, 1) == (int)gridDim.x - 1) {
            atomicExch(ticket, 0);   // ready for the next forward
            __threadfence_system();
            for (int g = 0; g < a.world; g++) st_release_sys(ep_flag(a.peers[g], a.o_flags, phase, a.rank), a.epoch);
        }
    }
}

// One CTA, after the dispatch: wait for every source's rows (and with them
// its slot offsets), then the plan of the rows I receive: my experts in order,
// each with its rows in (source rank, source slot) order -- the global
// canonical order restricted to my experts. perm[slot] = received row,
// ret[slot] = (source, source slot).
__global__ void __launch_bounds__(256) ep_p2p_plan_kernel(EpP2PArgs a)
{
    __shared__ int s_off[kEpMaxRanks * (kMaxRouteExperts + 1)];
    __shared__ int s_cnt[kMaxRouteExperts], s_slot0[kMaxRouteExperts];
    __shared__ int s_ok;
    pdl_wait();   // launched as a dependent: the routing is complete
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int E = a.E, G = a.world, El = a.El;
    if (tid == 0) s_ok = 1;
    __syncthreads();
    if (tid < G) {
        const int r = wait_epoch(ep_flag(a.own, a.o_flags, kEpPhaseRows, tid), a.wait_epoch, a.wait_cycles);
        if (r) {
            s_ok = 0;
            atomicExch(a.err, r);
        }
    }
    __syncthreads();
    if (tid == 0) *a.ok = s_ok;   // read by this forward's expert launch, return and waits
    if (!s_ok) {
        if (tid == 0) { *a.n_active = 0; *a.total = 0; }
        return;
    }
    const int32_t *off = reinterpret_cast<const int32_t *>(a.own + a.o_off);
    for (int i = tid; i < G * (E + 1); i += blockDim.x) s_off[i] = off[i];
    __syncthreads();
    for (int el = tid; el < El; el += blockDim.x) {
        const int e = a.e0 + el;
        int c = 0;
        for (int s = 0; s < G; s++) c += s_off[s * (E + 1) + e + 1] - s_off[s * (E + 1) + e];
        s_cnt[el] = c;
    }
    __syncthreads();
    if (warp == 0) {
        const int chunk = (El + 31) / 32, b = lane * chunk;
        int local = 0;
        for (int i = 0; i < chunk; i++)
            if (b + i < El) local += s_cnt[b + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < chunk; i++)
            if (b + i < El) { s_slot0[b + i] = run; run += s_cnt[b + i]; }
        if (lane == 31) *a.total = incl;
        int nact = 0;
        for (int c0 = 0; c0 < El; c0 += 32) {
            const int el = c0 + lane;
            const bool act = el < El && s_cnt[el] > 0;
            const uint32_t bal = __ballot_sync(0xffffffffu, act);
            __syncwarp();
            const int pos = nact + __popc(bal & ((1u << lane) - 1u));
            if (act) a.problems[pos] = Problem{el, s_slot0[el], s_cnt[el], 0};
            nact += __popc(bal);
        }
        if (lane == 0) *a.n_active = nact;
    }
    __syncthreads();
    for (int it = warp; it < El * G; it += nw) {
        const int el = it / G, s = it - el * G, e = a.e0 + el;
        const int *os = s_off + s * (E + 1);
        const int c = os[e + 1] - os[e];
        if (!c) continue;
        int base = s_slot0[el];
        for (int s2 = 0; s2 < s; s2++) base += s_off[s2 * (E + 1) + e + 1] - s_off[s2 * (E + 1) + e];
        const int row = s * a.cap + (os[e] - os[a.e0]);
        for (int i = lane; i < c; i += 32) {
            a.perm[base + i] = row + i;
            a.ret[base + i] = make_int2(s, os[e] + i);
        }
    }
}

// The first step of a forward's exchange: my slot offsets into every rank's
// offset inbox, and my routed rows, packed [H int8 | H/32 d | H/32 s], into
// the row inbox of the rank that owns each row's expert, at (my rank,
// position among my rows for that rank). One warp per row; the rows flag
// follows once every CTA's stores are fenced.
__global__ void __launch_bounds__(256) ep_p2p_dispatch_kernel(EpP2PArgs a)
{
    __shared__ int s_off[kMaxRouteExperts + 1];
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    const int H = a.H, chunks = H >> 4, nd = H >> 5;
    if (blockIdx.x == 0)
        for (int g = 0; g < a.world; g++) {
            int32_t *dst = reinterpret_cast<int32_t *>(a.peers[g] + a.o_off) + (size_t)a.rank * (a.E + 1);
            for (int i = threadIdx.x; i <= a.E; i += blockDim.x) dst[i] = a.offsets[i];
        }
    for (int i = threadIdx.x; i <= a.E; i += blockDim.x) s_off[i] = a.offsets[i];
    __syncthreads();
    for (int s = warp; s < a.n_slots; s += nwarps) {
        int lo = 0, hi = a.E - 1;   // the expert of slot s: last e with offsets[e] <= s
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_off[mid] <= s) lo = mid;
            else hi = mid - 1;
        }
        const int dest = lo / a.El;
        const int r = s - s_off[dest * a.El];
        const size_t tok = (size_t)a.perm_token[s];
        if (a.o_x16) {
            // f16(q * d), groups of four as (0, 2, 1, 3): the token row operand of
            // the receiver's fused f16 expert launch (quantize_tile's arithmetic)
            uint2 *row16 = reinterpret_cast<uint2 *>(a.peers[dest] + a.o_x16 +
                                                     ((size_t)a.rank * a.cap + r) * (size_t)H * 2);
            const uint32_t *q4 = reinterpret_cast<const uint32_t *>(a.xq + tok * H);
            const float *dv = a.xd + tok * nd;
#pragma unroll 4
            for (int g = lane; g < (H >> 2); g += 32) {
                const uint32_t q = q4[g];
                const float d = dv[g >> 3];
                const float q0 = (float)(int8_t)(q & 0xFF), q1 = (float)(int8_t)((q >> 8) & 0xFF);
                const float q2 = (float)(int8_t)((q >> 16) & 0xFF), q3 = (float)(int8_t)(q >> 24);
                const __half2 lo = __floats2half2_rn(q0 * d, q2 * d), hi = __floats2half2_rn(q1 * d, q3 * d);
                row16[g] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
            }
            continue;
        }
        uint8_t *row = a.peers[dest] + a.o_xin + ((size_t)a.rank * a.cap + r) * a.rb;
        const int4 *q = reinterpret_cast<const int4 *>(a.xq + tok * H);
        for (int c = lane; c < chunks; c += 32) reinterpret_cast<int4 *>(row)[c] = q[c];
        float *rd = reinterpret_cast<float *>(row + H);
        for (int c = lane; c < nd; c += 32) {
            rd[c] = a.xd[tok * nd + c];
            rd[nd + c] = a.xs[tok * nd + c];
        }
    }
    signal_when_done(a, a.ticket, kEpPhaseRows);
}

// Expert outputs of the rows I received, by local slot, into each source's
// output inbox at the source's own slot. One warp per row.
__global__ void __launch_bounds__(256) ep_p2p_return_kernel(EpP2PArgs a)
{
    pdl_wait();   // the down projection's outputs are complete
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    const int H = a.H, chunks = H >> 2;
    if (!*a.ok) return;   // no stores into any peer's arena, no flags (uniform over the grid)
    const int total = *a.total;
    for (int s = warp; s < total; s += nwarps) {
        const int2 rr = a.ret[s];
        float4 *dst = reinterpret_cast<float4 *>(a.peers[rr.x] + a.o_yin + (size_t)rr.y * H * 4);
        const float4 *src = reinterpret_cast<const float4 *>(a.y + (size_t)s * H);
        for (int c = lane; c < chunks; c += 32) dst[c] = src[c];
    }
    signal_when_done(a, a.ticket + 1, kEpPhaseOut);
}

// Waits for every rank's flag of `phase` in this rank's arena.
__global__ void ep_p2p_wait_kernel(EpP2PArgs a, int phase)
{
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x;
    if (!*a.ok) return;   // the forward has already failed: nobody raises these flags
    if (lane < a.world) {
        const int r = wait_epoch(ep_flag(a.own, a.o_flags, phase, lane), a.wait_epoch, a.wait_cycles);
        if (r) atomicExch(a.err, r);
    }
}

int rows_grid(long long rows, int num_sms)
{
    const long long blocks = (rows + 7) / 8;   // 8 warps per block
    const long long cap = 4LL * num_sms;
    return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

cudaError_t launch_ep_p2p_plan(const EpP2PArgs &a, cudaStream_t st)
{
    return launch_dependent(ep_p2p_plan_kernel, dim3(1), dim3(256), 0, st, a);
}

cudaError_t launch_ep_p2p_dispatch(const EpP2PArgs &a, int num_sms, cudaStream_t st)
{
    return launch_dependent(ep_p2p_dispatch_kernel, dim3(rows_grid(a.n_slots, num_sms)), dim3(256), 0, st, a);
}

cudaError_t launch_ep_p2p_return(const EpP2PArgs &a, int num_sms, cudaStream_t st)
{
    // the received rows are counted on the device: one CTA per SM covers them
    // with a grid-stride loop (capacity world * cap would mostly idle)
    const int g = rows_grid((long long)a.world * a.cap, num_sms);
    return launch_dependent(ep_p2p_return_kernel, dim3(g < num_sms ? g : num_sms), dim3(256), 0, st, a);
}

cudaError_t launch_ep_p2p_wait(const EpP2PArgs &a, int phase, cudaStream_t st)
{
    return launch_dependent(ep_p2p_wait_kernel, dim3(1), dim3(32), 0, st, a, phase);
}

}  // namespace jmoe
