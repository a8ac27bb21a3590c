// experts.cu -- grouped SwiGLU experts over quantised weights and the combine.
//
// Quantised experts run as weight-streaming kernels: the HBM traffic of a
// decode-sized MoE layer is the weight rows of the routed experts, read once.
// A work item is (problem, 32-row tile); each CTA owns a contiguous range of
// items. A producer warp streams each item's rows, one K-slice at a time, into
// a shared-memory ring with bulk async copies (cp.async.bulk, one per row and
// matrix, completing on an mbarrier), while eight consumer warps dot them
// against the problem's int8 activation blocks held in shared memory. The copy
// stream does not stop between items.
//
// Consumer mapping: warp w owns rows 4w..4w+3 of the tile, 8 lanes per row;
// lane l8 takes the 32-value units l8, l8+8, ... of the slice, so a lane always
// sees the same Q4_K sub-block index (l8) and the 8 lanes of a row read 128
// contiguous bytes. Activation loads are broadcast to the 4 rows of a warp.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace jmoe {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kStreamThreads = kConsumers + 32;
constexpr int kRows = 32;                           // rows per work item and per chunk
constexpr long long kWaitCycles = 4000000000LL;     // ~2 s: a wait that long means a fault
constexpr int kRingBudget = 80 * 1024;
constexpr int kErrTimeout = 1;

// Bounded mbarrier wait: gives up (and flags the CTA and the forward) after
// kWaitCycles or when another thread of the CTA gave up. A waiting warp sleeps
// in try_wait (suspend hint) rather than spinning, leaving the issue slots to
// the warps with work; the flag and the clock are read only on a timeout.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity, 20000)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicExch(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

struct Item {
    Problem pr;
    bool shared;
    int rt;
};

// Shared memory: ring [stages][stage_bytes] | xq int4 [kTT][2][act_k/32] |
// xds float2 [kTT][act_k/32] | g, u [kTT][32] f32 | problem table int4 [max_q] |
// cost prefix int64 [max_q + 1] | full[stages], empty[stages] | abort.
struct Smem {
    uint8_t *ring;
    int4 *xq;
    float2 *xds;
    float *g, *u;
    int4 *prob;            // (expert, slot0, count, is_shared) of the launch's problems
    long long *cpre;       // cost of all items of the problems before q
    uint64_t *full, *empty;
    volatile int *abort_flag;
};

// Staged activation blocks, unit-major: block u of token t, half h (16 bytes)
// at u * kUnitStride + t * 32 + h * 16; its (d, d*sum q) pair at
// u * kDsStride + t * 8. The 16- and 8-byte pads put the eight lanes of a row
// (eight consecutive units) on distinct banks, and every token offset is a
// compile-time immediate in the dot loop.
constexpr int kUnitStride = kTT * 32 + 16;
constexpr int kDsStride = kTT * 8 + 8;

// Bytes of the (d, d*sum q) region, rounded up to 16 so that the int4 problem
// table after the g/u buffers stays 16-byte aligned for any block count.
__host__ __device__ inline size_t ds_region_bytes(size_t nu) { return (nu * kDsStride + 15) / 16 * 16; }

__host__ __device__ inline size_t smem_bytes(const StreamCfg &c)
{
    const size_t nu = (size_t)c.act_k / 32;
    return (size_t)c.stages * c.stage_bytes + nu * kUnitStride + ds_region_bytes(nu) + 2 * (size_t)kTT * 32 * 4 +
           16 * (size_t)c.max_q + 8 * ((size_t)c.max_q + 1) + 16 * (size_t)c.stages + 16;
}

__device__ __forceinline__ Item item_at(const Smem &s, const StreamCfg &c, int nr, int it)
{
    Item x;
    const bool sh = it >= nr * c.rt_routed;
    const int q = sh ? nr : it / c.rt_routed;
    const int4 v = s.prob[q];
    x.pr.expert = v.x;
    x.pr.slot0 = v.y;
    x.pr.count = v.z;
    x.pr.is_shared = v.w;
    x.rt = sh ? it - nr * c.rt_routed : it - q * c.rt_routed;
    x.shared = sh;
    return x;
}

// Estimated cost of one row-tile item of a problem with `count` tokens: the
// weight stream and block decode once per token tile, the dots per token.
__device__ __forceinline__ long long item_cost(int count)
{
    return 7LL * ((count + kTT - 1) / kTT) + 5LL * count;
}

// First item whose cost-prefix start is at or after X (items are ordered by
// problem, then row tile, each problem's items all costing item_cost(count)).
__device__ __forceinline__ int first_item_from(const Smem &s, const StreamCfg &c, int nq, int nr, long long X)
{
    if (X >= s.cpre[nq]) return nr * c.rt_routed + (nq > nr ? c.rt_shared : 0);
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s.cpre[mid] <= X) lo = mid;
        else hi = mid - 1;
    }
    const long long cq = item_cost(s.prob[lo].z);
    const int rt = lo < nr ? c.rt_routed : c.rt_shared;
    const long long r = (X - s.cpre[lo] + cq - 1) / cq;
    const int base = lo * c.rt_routed;   // the shared problem (lo == nr) starts at nr * rt_routed too
    return r >= rt ? base + rt : base + (int)r;
}

__device__ __forceinline__ Smem carve(uint8_t *base, const StreamCfg &c)
{
    const int nu = c.act_k / 32;
    Smem s;
    s.ring = base;
    s.xq = reinterpret_cast<int4 *>(base + (size_t)c.stages * c.stage_bytes);
    s.xds = reinterpret_cast<float2 *>(reinterpret_cast<uint8_t *>(s.xq) + (size_t)nu * kUnitStride);
    s.g = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(s.xds) + ds_region_bytes(nu));
    s.u = s.g + kTT * 32;
    s.prob = reinterpret_cast<int4 *>(s.u + kTT * 32);
    s.cpre = reinterpret_cast<long long *>(s.prob + c.max_q);
    s.full = reinterpret_cast<uint64_t *>(s.cpre + c.max_q + 1);
    s.empty = s.full + c.stages;
    s.abort_flag = reinterpret_cast<volatile int *>(s.empty + c.stages);
    return s;
}

__device__ __forceinline__ void init_ring(const Smem &s, int stages)
{
    if (threadIdx.x == 0) {
        for (int i = 0; i < stages; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kConsumerWarps);
        }
        *s.abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
}

// After a failed wait the producer still owns the copies it issued: wait for
// each of the last min(g, stages) uses to land (bounded) before returning.
__device__ __forceinline__ void drain(const Smem &s, int stages, uint32_t g)
{
    for (uint32_t k = g > (uint32_t)stages ? g - stages : 0; k < g; k++) {
        const long long t0 = clock64();
        while (!mbar_try_wait_sleep(&s.full[k % stages], (k / stages) & 1, 20000))
            if (clock64() - t0 > kWaitCycles) break;
    }
}

// Stages the activation blocks of nt rows in the unit-major layout above.
// Rows are token ids from perm, or consecutive slots from row0 when perm is null.
__device__ __forceinline__ void stage_act(const Smem &s, const int8_t *gq, const float *gd, const float *gs,
                                          size_t q_stride, size_t d_stride, const int32_t *perm, int row0, int nt,
                                          int K)
{
    const int nu = K >> 5;
    uint8_t *xq = reinterpret_cast<uint8_t *>(s.xq);
    uint8_t *xds = reinterpret_cast<uint8_t *>(s.xds);
    for (int v = threadIdx.x; v < nt * nu * 2; v += kConsumers) {
        const int i = v / (2 * nu), rem = v - i * 2 * nu, u = rem >> 1, h = rem & 1;
        const size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        *reinterpret_cast<int4 *>(xq + (size_t)u * kUnitStride + i * 32 + h * 16) =
            __ldg(reinterpret_cast<const int4 *>(gq + row * q_stride) + 2 * u + h);
    }
    for (int v = threadIdx.x; v < nt * nu; v += kConsumers) {
        const int i = v / nu, u = v - i * nu;
        const size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        *reinterpret_cast<float2 *>(xds + (size_t)u * kDsStride + i * 8) =
            make_float2(__ldg(gd + row * d_stride + u), __ldg(gs + row * d_stride + u));
    }
}

// Producer: one chunk (item, token tile, K-slice) = for each matrix two 2-D
// TMA boxes of 32 rows (quants and scales) landing back to back in the stage.
// Boxes past the end of a row read zeros and still count full box bytes.
__device__ __forceinline__ void produce_chunk(const Smem &s, const StreamCfg &c, int st, const MatMaps *const *mm,
                                              int nmat, int y, int sl)
{
    mbar_arrive_expect_tx(&s.full[st], (uint32_t)nmat * kRows * (c.qs_row + c.meta_row));
    uint8_t *stage = s.ring + (size_t)st * c.stage_bytes;
    for (int m = 0; m < nmat; m++) {
        uint8_t *dq = stage + (size_t)m * kRows * (c.qs_row + c.meta_row);
        uint8_t *dm = dq + (size_t)kRows * c.qs_row;
        tma_load_2d(dq, &mm[m]->qs, sl * (c.qs_row / 8), y, &s.full[st]);
        tma_load_2d(dm, &mm[m]->meta, sl * (c.meta_row / 8), y, &s.full[st]);
    }
}

// Dots of one chunk: NMAT matrices (gate/up or down), NT tokens. acc[m][t]
// accumulates the lane's partial sums over the units it owns.
template <int FMT, int NMAT, int NT>
__device__ __forceinline__ void consume_chunk(const Smem &s, const StreamCfg &c, const uint8_t *stage, int rw, int l8,
                                              int nu_slice, int ubase, int nu_s, float (&acc)[NMAT][NT])
{
    // 32-bit shared addresses, advanced by constants each iteration
    const uint32_t st = smem_addr(stage);
    const uint32_t mat_stride = (uint32_t)kRows * (c.qs_row + c.meta_row);
    const uint32_t q0a = st + (uint32_t)rw * c.qs_row;
    const uint32_t m0a = st + (uint32_t)kRows * c.qs_row + (uint32_t)rw * c.meta_row;
    uint32_t qa[NMAT], ma[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        qa[m] = q0a + m * mat_stride + (FMT == FMT_Q4_K ? 16 : 32) * l8;
        ma[m] = m0a + m * mat_stride + (FMT == FMT_Q4_K ? 0 : 2 * l8);
    }
    uint32_t xu = smem_addr(s.xq) + (uint32_t)(ubase + l8) * kUnitStride;
    uint32_t du = smem_addr(s.xds) + (uint32_t)(ubase + l8) * kDsStride;
#pragma unroll 1
    for (int u = l8; u < nu_slice; u += 8) {
        if (FMT == FMT_Q4_K) {
            Q4Nib nb[NMAT];
            float2 sc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                nb[m] = q4_nibbles(lds128(qa[m]));
                sc[m] = q4_scales(lds128(ma[m]), l8);   // super-block u / 8 (u % 8 == l8)
                qa[m] += 128;
                ma[m] += 16;
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const int4 a = lds128i(xu + t * 32);
                const int4 b = lds128i(xu + t * 32 + 16);
                const float2 ds = lds64f(du + t * 8);
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const float f = i2f_small(q4_isum16(nb[m], a, b));
                    acc[m][t] = fmaf(f, ds.x * sc[m].x, acc[m][t]);
                    acc[m][t] = fmaf(-ds.y, sc[m].y, acc[m][t]);
                }
            }
        } else {
            uint4 q0[NMAT], q1[NMAT];
            float d[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                q0[m] = lds128(qa[m]);
                q1[m] = lds128(qa[m] + 16);
                d[m] = __half2float(__ushort_as_half((unsigned short)lds16(ma[m])));
                qa[m] += 256;
                ma[m] += 16;
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const int4 a = lds128i(xu + t * 32);
                const int4 b = lds128i(xu + t * 32 + 16);
                const float xd = lds64f(du + t * 8).x;
#pragma unroll
                for (int m = 0; m < NMAT; m++)
                    acc[m][t] = fmaf(i2f_small(q8_isum(q0[m], q1[m], a, b)), d[m] * xd, acc[m][t]);
            }
        }
        xu += 8 * kUnitStride;
        du += 8 * kDsStride;
    }
}

// Consumer side of one (item, token tile) with NT tokens: all K-slices of the
// 32-row tile, then the 8-lane reduction. Returns false when a wait gave up.
template <int FMT, int NMAT, int NT>
__device__ __forceinline__ bool consume_tile(const Smem &s, const StreamCfg &c, RingPos &g, int K, int nu_s,
                                             int *err, float (&out)[NMAT][NT], int rw,
                                             int l8)
{
    float acc[NMAT][NT];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[m][t] = 0.0f;
    const int ns = (K + c.ks - 1) / c.ks;
    for (int sl = 0; sl < ns; sl++) {
        const int st = g.slot;
        if (!wait_bar(&s.full[st], g.phase, s.abort_flag, err)) return false;
        const int ks_cur = min(c.ks, K - sl * c.ks);
        consume_chunk<FMT, NMAT, NT>(s, c, s.ring + (size_t)st * c.stage_bytes, rw, l8, ks_cur >> 5, sl * (c.ks >> 5),
                                     nu_s, acc);
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.empty[st]);
        g.advance(c.stages);
    }
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float v = acc[m][t];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            out[m][t] = v;
        }
    return true;
}

// Gate/up epilogue for NT tokens: the row-group leaders publish g and u.
template <int NT>
__device__ __forceinline__ void publish_gu(const Smem &s, const float (&o)[2][NT], int nt, int row, int l8)
{
    if (l8 == 0) {
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < nt) {
                s.g[t * 32 + row] = o[0][t];
                s.u[t * 32 + row] = o[1][t];
            }
    }
}

template <int NT>
__device__ __forceinline__ void publish_y(const FwdParams &p, const float (&o)[1][NT], int nt, size_t slot0, int row,
                                          int l8)
{
    if (l8 == 0) {
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < nt) p.y[(size_t)y_row(p, slot0 + t) * p.H + row] = o[0][t];
    }
}

// ---------------------------------------------------------- the kernels

// NMAT == 2: gate and up (rows of I or S, K = H), epilogue a = silu(g) * u
// quantised per 32 rows. NMAT == 1: down (rows of H, K = I or S), y written.
template <int FMT, int NMAT>
__global__ void __launch_bounds__(kStreamThreads, 2)
    expert_stream_kernel(FwdParams p, LayerDev L, StreamCfg c, const __grid_constant__ LayerMaps maps)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, c);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();      // launched as a dependent: routing / gate_up output is complete
    pdl_trigger();
    // the launch's problems (routed, then the shared expert) and their cost prefix
    const int with_sh = (c.mode != 0 && p.S > 0) ? 1 : 0;
    const int nr = min(c.mode == 1 ? 0 : *p.n_active, c.max_q - with_sh);
    const int nq = nr + with_sh;
    for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        const Problem pr = i < nr ? p.problems[i] : p.problems[p.max_problems - 1];
        s.prob[i] = make_int4(pr.expert, pr.slot0, pr.count, i < nr ? 0 : 1);
    }
    __syncthreads();
    if (warp == 0) {
        const int per = (nq + 31) / 32, b = lane * per;
        long long local = 0;
        for (int i = b; i < min(b + per, nq); i++) local += item_cost(s.prob[i].z) * (i < nr ? c.rt_routed : c.rt_shared);
        long long incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        long long run = incl - local;
        for (int i = b; i < min(b + per, nq); i++) {
            s.cpre[i] = run;
            run += item_cost(s.prob[i].z) * (i < nr ? c.rt_routed : c.rt_shared);
        }
        if (lane == 31) s.cpre[nq] = incl;
    }
    init_ring(s, c.stages);   // also publishes the tables (__syncthreads)
    // contiguous item range of this CTA, balanced by estimated cost
    const long long ctot = s.cpre[nq];
    const int it0 = first_item_from(s, c, nq, nr, ctot * blockIdx.x / gridDim.x);
    const int it1 = first_item_from(s, c, nq, nr, ctot * (blockIdx.x + 1) / gridDim.x);

    if (warp == kConsumerWarps) {   // producer: one thread issues the TMA boxes
        if (lane != 0) return;
        RingPos r;
        uint32_t g = 0;   // uses issued, for the drain after an abort
        for (int it = it0; it < it1; it++) {
            const Item x = item_at(s, c, nr, it);
            const MatMaps *mm[NMAT];
            int K, rows;
            if (NMAT == 2) {
                mm[0] = x.shared ? &maps.sh_gate : &maps.gate;
                mm[NMAT - 1] = x.shared ? &maps.sh_up : &maps.up;
                K = x.shared ? L.sh_gate.cols : L.gate.cols;
                rows = x.shared ? L.sh_gate.rows : L.gate.rows;
            } else {
                mm[0] = x.shared ? &maps.sh_down : &maps.down;
                K = x.shared ? L.sh_down.cols : L.down.cols;
                rows = x.shared ? L.sh_down.rows : L.down.rows;
            }
            const int y = x.pr.expert * rows + x.rt * kRows;
            const int tiles = (x.pr.count + kTT - 1) / kTT, ns = (K + c.ks - 1) / c.ks;
            for (int tt = 0; tt < tiles; tt++) {
                for (int sl = 0; sl < ns; sl++) {
                    if (!wait_bar(&s.empty[r.slot], r.phase ^ 1u, s.abort_flag, p.err)) {
                        drain(s, c.stages, g);
                        return;
                    }
                    produce_chunk(s, c, r.slot, mm, NMAT, y, sl);
                    r.advance(c.stages);
                    g++;
                }
            }
        }
        return;
    }

    // consumers
    RingPos g;
    int staged_slot = -1, staged_tile = -1;
    const int rw = warp * 4 + (lane >> 3), l8 = lane & 7;
    const int nu_s = c.act_k >> 5;
    for (int it = it0; it < it1; it++) {
        const Item x = item_at(s, c, nr, it);
        int K, rows;
        if (NMAT == 2) {
            const DevMatrix &G = x.shared ? L.sh_gate : L.gate;
            K = G.cols;
            rows = G.rows;
        } else {
            const DevMatrix &D = x.shared ? L.sh_down : L.down;
            K = D.cols;
            rows = D.rows;
        }
        const int r0 = x.rt * kRows, nrow = min(kRows, rows - r0);
        const int tiles = (x.pr.count + kTT - 1) / kTT;
        for (int tt = 0; tt < tiles; tt++) {
            const int t0 = tt * kTT, nt = min(kTT, x.pr.count - t0);
            if (staged_slot != x.pr.slot0 || staged_tile != tt) {
                named_bar(1, kConsumers);
                if (NMAT == 2)
                    stage_act(s, p.xq, p.xd, p.xs, (size_t)(p.x_qstride ? p.x_qstride : p.H),
                              (size_t)(p.x_dstride ? p.x_dstride : (p.H >> 5)), p.perm_token,
                              x.pr.slot0 + t0, nt, K);
                else
                    stage_act(s, p.aq, p.ad, p.as, (size_t)p.W, (size_t)(p.W >> 5), nullptr, x.pr.slot0 + t0, nt,
                              K);
                named_bar(1, kConsumers);
                staged_slot = x.pr.slot0;
                staged_tile = tt;
            }
            const bool row_ok = rw < nrow;
            bool ok = true;
            const size_t slot0 = (size_t)x.pr.slot0 + t0;
#define JMOE_TILE(NTV)                                                                                   \
    {                                                                                                    \
        float o[NMAT][NTV];                                                                              \
        ok = consume_tile<FMT, NMAT, NTV>(s, c, g, K, nu_s, p.err, o, rw, l8);                           \
        if (ok && row_ok) {                                                                              \
            if constexpr (NMAT == 2) publish_gu<NTV>(s, o, nt, rw, l8);                                  \
            else publish_y<NTV>(p, o, nt, slot0, r0 + rw, l8);                                           \
        }                                                                                                \
    }
            switch (nt) {
            case 1: JMOE_TILE(1) break;
            case 2: JMOE_TILE(2) break;
            case 3: JMOE_TILE(3) break;
            case 4: JMOE_TILE(4) break;
            case 5: JMOE_TILE(5) break;
            case 6: JMOE_TILE(6) break;
            case 7: JMOE_TILE(7) break;
            default: JMOE_TILE(8) break;
            }
#undef JMOE_TILE
            if (!ok) return;
            if (NMAT == 2) {
                named_bar(1, kConsumers);
                if (warp < nt) {
                    const size_t slot = slot0 + warp;
                    const float a = lane < nrow ? swiglu(s.g[warp * 32 + lane], s.u[warp * 32 + lane]) : 0.0f;
                    if (c.down_f32) {
                        if (lane < nrow) p.af[slot * p.W + r0 + lane] = a;
                    } else {
                        quant_block32(a, p.aq + slot * p.W + r0, p.ad + slot * (p.W >> 5) + (r0 >> 5),
                                      p.as + slot * (p.W >> 5) + (r0 >> 5), lane);
                    }
                }
                named_bar(1, kConsumers);
            }
        }
    }
}

// ---------------------------------------------------------- F32 experts

struct ProblemSel {
    Problem pr;
    bool shared;
    bool ok;
};

// shared_mode: 0 routed problems only, 1 the shared problem only (grid.y == 1),
// 2 routed problems plus the shared one in the last grid row.
__device__ __forceinline__ ProblemSel pick_problem(const FwdParams &p, int shared_mode)
{
    ProblemSel s;
    const int y = blockIdx.y;
    s.shared = (shared_mode == 1) || (shared_mode == 2 && y == (int)gridDim.y - 1);
    if (s.shared) {
        s.pr = p.problems[p.max_problems - 1];
        s.ok = true;
    } else {
        s.ok = y < *p.n_active;
        if (s.ok) s.pr = p.problems[y];
    }
    return s;
}

// F32 expert matrices (the reference's own unit tests use F32 stacks): one
// token at a time, activations read from global memory, any shape.
__global__ void __launch_bounds__(256) gate_up_f32_kernel(FwdParams p, LayerDev L, int shared_mode)
{
    const ProblemSel ps = pick_problem(p, shared_mode);
    if (!ps.ok) return;
    const DevMatrix &G = ps.shared ? L.sh_gate : L.gate;
    const DevMatrix &U = ps.shared ? L.sh_up : L.up;
    const int rows = G.rows, K = G.cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane >> 3, l8 = lane & 7;
    const int row = blockIdx.x * 32 + warp * 4 + sub;
    const int e = ps.pr.expert;
    const float *gw = reinterpret_cast<const float *>(G.qs + (size_t)e * G.qs_estride + (size_t)row * G.qs_rstride);
    const float *uw = reinterpret_cast<const float *>(U.qs + (size_t)e * U.qs_estride + (size_t)row * U.qs_rstride);
    for (int t = 0; t < ps.pr.count; t++) {
        const size_t slot = (size_t)ps.pr.slot0 + t;
        const float *x = p.x + (size_t)p.perm_token[slot] * p.H;
        float g = 0.0f, u = 0.0f;
        if (row < rows)
            for (int c = l8; c < K; c += 8) {
                g = __fmaf_rn(gw[c], x[c], g);
                u = __fmaf_rn(uw[c], x[c], u);
            }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            g += __shfl_xor_sync(0xffffffffu, g, o);
            u += __shfl_xor_sync(0xffffffffu, u, o);
        }
        if (l8 == 0 && row < rows) p.af[slot * p.W + row] = swiglu(g, u);
    }
}

__global__ void __launch_bounds__(256) down_f32_kernel(FwdParams p, LayerDev L, int shared_mode)
{
    const ProblemSel ps = pick_problem(p, shared_mode);
    if (!ps.ok) return;
    const DevMatrix &D = ps.shared ? L.sh_down : L.down;
    const int rows = D.rows, K = D.cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane >> 3, l8 = lane & 7;
    const int row = blockIdx.x * 32 + warp * 4 + sub;
    const int e = ps.pr.expert;
    const float *dw = reinterpret_cast<const float *>(D.qs + (size_t)e * D.qs_estride + (size_t)row * D.qs_rstride);
    for (int t = 0; t < ps.pr.count; t++) {
        const size_t slot = (size_t)ps.pr.slot0 + t;
        const float *a = p.af + slot * p.W;
        float v = 0.0f;
        if (row < rows)
            for (int c = l8; c < K; c += 8) v = __fmaf_rn(dw[c], a[c], v);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (l8 == 0 && row < rows) p.y[(size_t)y_row(p, slot) * p.H + row] = v;
    }
}

// ---------------------------------------------------------------- combine

// out[t] = 0 + shared(x_t), then += w_r * y_r in rank order, each step a
// separately rounded multiply and add (src/qwen_deepseek.rs:858-938).
__global__ void __launch_bounds__(256) combine_kernel(FwdParams p)
{
    __shared__ long long s_pos[kMaxK];
    __shared__ float s_w[kMaxK];
    pdl_wait();
    pdl_trigger();
    const int k = p.k, H = p.H, mw = p.mask_words;
    for (int t = blockIdx.y; t < p.T; t += gridDim.y) {
        if (threadIdx.x < k) {
            const int r = threadIdx.x;
            long long pos;
            if (p.T <= kFusedRoutingMaxT) {   // the routing kernel wrote the slot of each choice
                pos = p.slot_of[(size_t)t * k + r];
            } else {                          // slot from the expert masks
                const int e = p.sel_idx[(size_t)t * k + r];
                pos = -1;
                if (e >= 0) {
                    const uint32_t m = p.mask[(size_t)e * mw + (t >> 5)];
                    pos = p.offsets[e] + p.wprefix[(size_t)e * mw + (t >> 5)] + __popc(m & ((1u << (t & 31)) - 1u));
                }
            }
            s_pos[r] = pos;
            s_w[r] = p.sel_w[(size_t)t * k + r];
        }
        __syncthreads();
        const size_t shared_row = (size_t)p.T * k + t;
        if ((H & 3) == 0) {   // four values per thread, same operation order per value
            const int H4 = H >> 2;
            for (int h4 = blockIdx.x * blockDim.x + threadIdx.x; h4 < H4; h4 += gridDim.x * blockDim.x) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (p.S > 0) {
                    const float4 s = reinterpret_cast<const float4 *>(p.y + shared_row * H)[h4];
                    v = make_float4(__fadd_rn(v.x, s.x), __fadd_rn(v.y, s.y), __fadd_rn(v.z, s.z), __fadd_rn(v.w, s.w));
                }
                // all rows' loads in flight first (8 at a time), then the adds in rank order
                for (int r0 = 0; r0 < k; r0 += 8) {
                    float4 yv[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int r = r0 + i;
                        yv[i] = (r < k && s_pos[r] >= 0)
                                    ? reinterpret_cast<const float4 *>(p.y + (size_t)s_pos[r] * H)[h4]
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int r = r0 + i;
                        if (r < k && s_pos[r] >= 0) {
                            const float w = s_w[r];
                            v.x = __fadd_rn(v.x, __fmul_rn(w, yv[i].x));
                            v.y = __fadd_rn(v.y, __fmul_rn(w, yv[i].y));
                            v.z = __fadd_rn(v.z, __fmul_rn(w, yv[i].z));
                            v.w = __fadd_rn(v.w, __fmul_rn(w, yv[i].w));
                        }
                    }
                }
                if (p.residual) {   // hidden += ffn_out (src/qwen_deepseek.rs:1304-1306)
                    const float4 r = reinterpret_cast<const float4 *>(p.residual + (size_t)t * H)[h4];
                    v = make_float4(__fadd_rn(r.x, v.x), __fadd_rn(r.y, v.y), __fadd_rn(r.z, v.z), __fadd_rn(r.w, v.w));
                }
                reinterpret_cast<float4 *>(p.out + (size_t)t * H)[h4] = v;
            }
        } else {
            for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x) {
                float v = 0.0f;
                if (p.S > 0) v = __fadd_rn(v, p.y[shared_row * H + h]);
                for (int r = 0; r < k; r++)
                    if (s_pos[r] >= 0) v = __fadd_rn(v, __fmul_rn(s_w[r], p.y[(size_t)s_pos[r] * H + h]));
                if (p.residual) v = __fadd_rn(p.residual[(size_t)t * H + h], v);
                p.out[(size_t)t * H + h] = v;
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------ launchers

template <typename Kern>
cudaError_t set_smem(Kern k, size_t bytes)
{
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <typename Kern>
cudaError_t launch_stream(Kern kern, const FwdParams &p, const LayerDev &L, const LayerMaps &maps, StreamCfg c,
                          int upper, int num_sms, cudaStream_t st)
{
    if (upper <= 0) return cudaSuccess;
    const size_t sm = smem_bytes(c);
    cudaError_t err = set_smem(kern, sm);
    if (err != cudaSuccess) return err;
    int per_sm = 0;
    if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStreamThreads, sm)) != cudaSuccess)
        return err;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = upper < num_sms * per_sm ? upper : num_sms * per_sm;
    return launch_dependent(kern, dim3(grid), dim3(kStreamThreads), sm, st, p, L, c, maps);
}

// Ring geometry from the slice plan of the matrices the launch streams (the
// routed and shared matrices of one launch share a plan; see stream_plans_match).
void plan_stream(StreamCfg &c, const DevMatrix &m, int nmat)
{
    c.ks = m.ks;
    c.qs_row = m.qs_box;
    c.meta_row = m.meta_box;
    const size_t stage = (size_t)nmat * kRows * (c.qs_row + c.meta_row);
    c.stage_bytes = (int)((stage + 127) / 128 * 128);
    int stg = kRingBudget / c.stage_bytes;
    c.stages = stg < 2 ? 2 : (stg > 16 ? 16 : stg);
}

}  // namespace

bool stream_plans_match(const DevMatrix &a, const DevMatrix &b)
{
    return a.type == b.type && a.ks == b.ks && a.qs_box == b.qs_box && a.meta_box == b.meta_box;
}

cudaError_t launch_gate_up(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                           cudaStream_t st)
{
    const DevMatrix &G0 = mode == 1 ? L.sh_gate : L.gate;
    if (G0.type == FMT_F32) {
        int rows = mode == 1 ? L.sh_gate.rows : L.gate.rows;
        if (mode == 2 && L.sh_gate.rows > rows) rows = L.sh_gate.rows;
        const int ny = mode == 1 ? 1 : (mode == 2 ? p.max_problems : p.max_problems - (p.S > 0 ? 1 : 0));
        gate_up_f32_kernel<<<dim3((rows + 31) / 32, ny), 256, 0, st>>>(p, L, mode);
        return cudaGetLastError();
    }
    StreamCfg c{};
    c.mode = mode;
    c.rt_routed = mode == 1 ? 0 : (L.gate.rows + kRows - 1) / kRows;
    c.rt_shared = (mode != 0 && p.S > 0) ? (L.sh_gate.rows + kRows - 1) / kRows : 0;
    c.down_f32 = (mode == 1 ? L.sh_down.type : L.down.type) == FMT_F32;
    c.act_k = p.H;
    c.max_q = p.max_problems;
    plan_stream(c, G0, 2);
    const int upper = (mode == 1 ? 0 : (p.max_problems - (p.S > 0 ? 1 : 0)) * c.rt_routed) + c.rt_shared;
    if (G0.type == FMT_Q4_K)
        return launch_stream(expert_stream_kernel<FMT_Q4_K, 2>, p, L, maps, c, upper, num_sms, st);
    return launch_stream(expert_stream_kernel<FMT_Q8_0, 2>, p, L, maps, c, upper, num_sms, st);
}

cudaError_t launch_down(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                        cudaStream_t st)
{
    const DevMatrix &D0 = mode == 1 ? L.sh_down : L.down;
    if (D0.type == FMT_F32) {
        const int ny = mode == 1 ? 1 : (mode == 2 ? p.max_problems : p.max_problems - (p.S > 0 ? 1 : 0));
        down_f32_kernel<<<dim3((p.H + 31) / 32, ny), 256, 0, st>>>(p, L, mode);
        return cudaGetLastError();
    }
    StreamCfg c{};
    c.mode = mode;
    c.rt_routed = mode == 1 ? 0 : (p.H + kRows - 1) / kRows;
    c.rt_shared = (mode != 0 && p.S > 0) ? (p.H + kRows - 1) / kRows : 0;
    int kmax = D0.cols;
    if (mode == 2 && L.sh_down.cols > kmax) kmax = L.sh_down.cols;
    c.act_k = kmax;
    c.max_q = p.max_problems;
    plan_stream(c, D0, 1);
    const int upper = (mode == 1 ? 0 : (p.max_problems - (p.S > 0 ? 1 : 0)) * c.rt_routed) + c.rt_shared;
    if (D0.type == FMT_Q4_K)
        return launch_stream(expert_stream_kernel<FMT_Q4_K, 1>, p, L, maps, c, upper, num_sms, st);
    return launch_stream(expert_stream_kernel<FMT_Q8_0, 1>, p, L, maps, c, upper, num_sms, st);
}

cudaError_t launch_combine(const FwdParams &p, cudaStream_t st)
{
    const int per = (p.H & 3) == 0 ? p.H / 4 : p.H;
    dim3 grid((per + 255) / 256 < 8 ? (per + 255) / 256 : 8, p.T < 65535 ? p.T : 65535);
    cudaError_t e = launch_dependent(combine_kernel, grid, dim3(256), 0, st, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace jmoe
