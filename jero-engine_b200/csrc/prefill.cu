// prefill.cu -- grouped expert GEMMs on the 5th-generation tensor cores for
// large token counts (tcgen05.mma kind::f16, fp32 accumulators in TMEM).
//
// Tile: 128 slots (M, TMEM lanes) x 128 weight rows (N) of one expert, K in
// steps of 64. Operands are K-major in the 128-byte swizzle layout:
//   A = the problem's activations in f16, rows in slot order, loaded by TMA;
//   B = the expert's weight rows, TMA-loaded as GGUF blocks (Q4_K / Q8_0) per
//       256-value super-step and expanded to f16 by eight dequant warps.
// gate/up tiles carry two accumulators (gate, up); their epilogue applies
// SwiGLU and the int8 block quantiser of the decode path (so both paths feed
// the down projection the same values) and stores the down operand in f16.
// down tiles store y in f32. Work items (problem, n-tile, m-tile) are spread
// over a persistent grid, m-tiles innermost so neighbouring CTAs share a
// weight tile in L2. Every wait is bounded.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace jmoe {
namespace {

constexpr int kTM = 128, kTN = 128, kKS = 64, kSuper = 256;
constexpr int kWarpTma = 0, kWarpMma = 1, kDeqWarp0 = 2, kDeqWarps = 8, kEpiWarp0 = 10, kEpiWarps = 4;
constexpr int kTcThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kAStages = 4, kBStages = 2, kQStages = 2;
constexpr long long kWaitCycles = 4000000000LL;
constexpr int kErrTimeout = 1;
constexpr int kATileBytes = kTM * kKS * 2;    // 16 KB
constexpr int kBTileBytes = kTN * kKS * 2;    // 16 KB per matrix

struct TcCfg {
    int nmat;        // 2: gate + up, 1: down
    int mode;        // 0 routed problems, 1 shared only, 2 both
    int qs_box;      // bytes of one row's quants per 256-value super-step
    int q_bytes;     // bytes of one quantized stage per matrix (quants + scales, 128 rows)
    int qstages;     // quantized stages in flight (1 or 2, by shared-memory room)
    int smem_a, smem_b, smem_q, smem_bar;   // region offsets
};

struct TcMaps {
    CUtensorMap a;                        // activations f16 [slots][K], box 64 x 128, swizzle 128B
    CUtensorMap wq[2], wm[2];             // routed weights: quants, scales (box 128 rows)
    CUtensorMap sq[2], sm[2];             // shared expert weights
};

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicExch(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

struct TcItem {
    Problem pr;
    bool shared;
    int mt, nt;
};

// tile_off[0..nq]: first item of each problem of the launch (routed problems in
// list order, then the shared expert); binary search for the item's problem.
__device__ __forceinline__ TcItem tc_item(const FwdParams &p, const int32_t *tile_off, int nq, int n_routed, int it)
{
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tile_off[mid] <= it) lo = mid;
        else hi = mid - 1;
    }
    TcItem x;
    x.shared = lo >= n_routed;
    x.pr = x.shared ? p.problems[p.max_problems - 1] : p.problems[lo];
    const int mtiles = (x.pr.count + kTM - 1) / kTM;
    const int local = it - tile_off[lo];
    x.mt = local % mtiles;
    x.nt = local / mtiles;
    return x;
}

// Four f16 pairs of one 8-value chunk of a Q4_K sub-block: nibbles from the
// 8 bytes (w0, w1), high nibbles when hi; w = q * dsc - dmn in one HFMA2.
__device__ __forceinline__ uint4 q4_chunk_f16(uint32_t w0, uint32_t w1, bool hi, __half2 dsc, __half2 ndmn)
{
    const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
    uint32_t src[4] = {__byte_perm(w0, 0, 0x4140), __byte_perm(w0, 0, 0x4342), __byte_perm(w1, 0, 0x4140),
                       __byte_perm(w1, 0, 0x4342)};
    uint4 out;
    uint32_t *o = &out.x;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t v = hi ? (src[i] >> 4) : src[i];
        v = (v & 0x000F000Fu) | 0x64006400u;               // f16 (1024 + q) in each half
        __half2 q = __hsub2(*reinterpret_cast<__half2 *>(&v), k1024);
        __half2 w = __hfma2(q, dsc, ndmn);
        o[i] = *reinterpret_cast<uint32_t *>(&w);
    }
    return out;
}

// Eight f16 values of a Q8_0 block: signed bytes (w0, w1) times the f16 scale.
__device__ __forceinline__ uint4 q8_chunk_f16(uint32_t w0, uint32_t w1, __half2 d)
{
    const __half2 k1152 = __half2half2(__ushort_as_half(0x6480));   // 1024 + 128
    uint32_t src[4] = {__byte_perm(w0, 0, 0x4140), __byte_perm(w0, 0, 0x4342), __byte_perm(w1, 0, 0x4140),
                       __byte_perm(w1, 0, 0x4342)};
    uint4 out;
    uint32_t *o = &out.x;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t v = (src[i] ^ 0x00800080u) | 0x64006400u;   // f16 (1024 + q + 128)
        __half2 q = __hsub2(*reinterpret_cast<__half2 *>(&v), k1152);
        __half2 w = __hmul2(q, d);
        o[i] = *reinterpret_cast<uint32_t *>(&w);
    }
    return out;
}

template <int FMT, int NMAT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_expert_kernel(FwdParams p, LayerDev L, TcCfg c, const __grid_constant__ TcMaps maps)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment of the operand tiles (swizzle atoms)
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sa = base + c.smem_a, *sb = base + c.smem_b, *sq = base + c.smem_q;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + c.smem_bar);
    uint64_t *a_full = bars, *a_empty = a_full + kAStages;
    uint64_t *b_full = a_empty + kAStages, *b_empty = b_full + kBStages;
    uint64_t *q_full = b_empty + kBStages, *q_empty = q_full + kQStages;
    uint64_t *acc_full = q_empty + kQStages, *acc_empty = acc_full + 2, *drain_bar = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kAStages; i++) { mbar_init(&a_full[i], 1); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < kBStages; i++) { mbar_init(&b_full[i], kDeqWarps); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < kQStages; i++) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], kDeqWarps); }
        for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], kEpiWarps); }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) tmem_alloc(tmem_slot, NMAT == 2 ? 512 : 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the launch's problems: routed ones, then the shared expert
    const int n_routed = c.mode == 1 ? 0 : *p.n_active;
    const bool with_shared = c.mode != 0 && p.S > 0;
    const int nq = n_routed + (with_shared ? 1 : 0);
    const int32_t *tile_off = p.tile_off + (NMAT == 2 ? 0 : 2 * kTileOffStride) + (c.mode == 1 ? kTileOffStride : 0);
    const int total = nq > 0 ? tile_off[nq] : 0;

    if (warp == kWarpTma) {
        if (lane == 0) {
            uint32_t ga = 0, gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(p, tile_off, nq, n_routed, it);
                const DevMatrix &M0 = NMAT == 2 ? (x.shared ? L.sh_gate : L.gate) : (x.shared ? L.sh_down : L.down);
                const int K = M0.cols, nk = (K + kKS - 1) / kKS;
                const int ay = x.pr.slot0 + x.mt * kTM, wy = x.pr.expert * M0.rows + x.nt * kTN;
                for (int kk = 0; kk < nk && ok; kk++) {
                    if ((kk & 3) == 0) {
                        const int s = gq % c.qstages;
                        if (gq >= (uint32_t)c.qstages && !tc_wait(&q_empty[s], ((gq / c.qstages) - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                        mbar_arrive_expect_tx(&q_full[s], (uint32_t)(NMAT * c.q_bytes));
                        for (int m = 0; m < NMAT; m++) {
                            uint8_t *dst = sq + (size_t)(s * NMAT + m) * c.q_bytes;
                            const CUtensorMap *mq = x.shared ? &maps.sq[m] : &maps.wq[m];
                            const CUtensorMap *mm = x.shared ? &maps.sm[m] : &maps.wm[m];
                            tma_load_2d(dst, mq, (kk >> 2) * (c.qs_box / 8), wy, &q_full[s]);
                            tma_load_2d(dst + kTN * c.qs_box, mm, (kk >> 2) * 2, wy, &q_full[s]);
                        }
                        gq++;
                    }
                    const int s = ga % kAStages;
                    if (ga >= (uint32_t)kAStages && !tc_wait(&a_empty[s], ((ga / kAStages) - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&a_full[s], (uint32_t)kATileBytes);
                    tma_load_2d(sa + (size_t)s * kATileBytes, &maps.a, kk * kKS, ay, &a_full[s]);
                    ga++;
                }
            }
            if (!ok) {   // wait (bounded) for the copies still in flight
                for (uint32_t g = ga > (uint32_t)kAStages ? ga - kAStages : 0; g < ga; g++) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&a_full[g % kAStages], (g / kAStages) & 1) && clock64() - t0 < kWaitCycles) {}
                }
                for (uint32_t g = gq > (uint32_t)c.qstages ? gq - c.qstages : 0; g < gq; g++) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&q_full[g % c.qstages], (g / c.qstages) & 1) && clock64() - t0 < kWaitCycles) {}
                }
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            // instruction descriptor: f32 accumulate, f16 A and B, both K-major, N = 128, M = 128
            const uint32_t idesc = (1u << 4) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
            uint32_t ga = 0, gb = 0, gt = 0;
            bool ok = true, issued = false;
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(p, tile_off, nq, n_routed, it);
                const int K = NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                        : (x.shared ? L.sh_down.cols : L.down.cols);
                const int nk = (K + kKS - 1) / kKS;
                const int buf = gt & 1;
                if (gt >= 2 && !tc_wait(&acc_empty[buf], ((gt >> 1) - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                for (int kk = 0; kk < nk; kk++) {
                    const int s_a = ga % kAStages, s_b = gb % kBStages;
                    if (!tc_wait(&a_full[s_a], (ga / kAStages) & 1, abort_flag, p.err) ||
                        !tc_wait(&b_full[s_b], (gb / kBStages) & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(sa + (size_t)s_a * kATileBytes);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const uint32_t b_addr = smem_addr(sb + (size_t)(s_b * NMAT + m) * kBTileBytes);
                        const uint32_t d = tmem + (uint32_t)(buf * NMAT * kTN + m * kTN);
#pragma unroll
                        for (int k16 = 0; k16 < kKS / 16; k16++)
                            tc_mma_f16(d, umma_desc_sw128(a_addr + 32 * k16), umma_desc_sw128(b_addr + 32 * k16), idesc,
                                       (kk | k16) != 0);
                    }
                    issued = true;
                    tc_commit(&a_empty[s_a]);
                    tc_commit(&b_empty[s_b]);
                    ga++;
                    gb++;
                }
                if (!ok) break;
                tc_commit(&acc_full[buf]);
                gt++;
            }
            if (issued) {   // every MMA has completed before the CTA may release TMEM
                tc_commit(drain_bar);
                const long long t0 = clock64();
                while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < kWaitCycles) {}
            }
        }
    } else if (warp < kEpiWarp0) {
        // dequant warps: thread d owns weight row d >> 1 and one 32-value sub-block of each 64-value step
        const int d = threadIdx.x - kDeqWarp0 * 32, r = d >> 1, hf = d & 1;
        uint32_t gb = 0, gq = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const TcItem x = tc_item(p, tile_off, nq, n_routed, it);
            const int K = NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                    : (x.shared ? L.sh_down.cols : L.down.cols);
            const int nk = (K + kKS - 1) / kKS;
            for (int kk = 0; kk < nk; kk++) {
                const int s_q = gq % c.qstages;
                if ((kk & 3) == 0 && !tc_wait(&q_full[s_q], (gq / c.qstages) & 1, abort_flag, p.err)) { ok = false; break; }
                const int s_b = gb % kBStages;
                if (gb >= (uint32_t)kBStages && !tc_wait(&b_empty[s_b], ((gb / kBStages) - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                const int j = 2 * (kk & 3) + hf;   // sub-block of the super-step
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const uint8_t *qrow = sq + (size_t)(s_q * NMAT + m) * c.q_bytes + (size_t)r * c.qs_box;
                    const uint8_t *mrow = sq + (size_t)(s_q * NMAT + m) * c.q_bytes + (size_t)kTN * c.qs_box + (size_t)r * 16;
                    uint8_t *brow = sb + (size_t)(s_b * NMAT + m) * kBTileBytes + (size_t)r * 128;
                    uint4 out[4];
                    if (FMT == FMT_Q4_K) {
                        const uint4 q = *reinterpret_cast<const uint4 *>(qrow + 16 * j);
                        const float2 sc = q4_scales(*reinterpret_cast<const uint4 *>(mrow), j);   // (d*sc/16, dmin*m)
                        const __half2 dsc = __float2half2_rn(sc.x * 16.0f), ndmn = __float2half2_rn(-sc.y);
                        out[0] = q4_chunk_f16(q.x, q.y, false, dsc, ndmn);
                        out[1] = q4_chunk_f16(q.z, q.w, false, dsc, ndmn);
                        out[2] = q4_chunk_f16(q.x, q.y, true, dsc, ndmn);
                        out[3] = q4_chunk_f16(q.z, q.w, true, dsc, ndmn);
                    } else {
                        const uint4 q0 = *reinterpret_cast<const uint4 *>(qrow + 32 * j);
                        const uint4 q1 = *reinterpret_cast<const uint4 *>(qrow + 32 * j + 16);
                        const __half2 dd = __half2half2(*reinterpret_cast<const __half *>(mrow + 2 * j));
                        out[0] = q8_chunk_f16(q0.x, q0.y, dd);
                        out[1] = q8_chunk_f16(q0.z, q0.w, dd);
                        out[2] = q8_chunk_f16(q1.x, q1.y, dd);
                        out[3] = q8_chunk_f16(q1.z, q1.w, dd);
                    }
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) {
                        const int chunk = 4 * hf + cc;   // 16-byte chunk of the 128-byte row
                        *reinterpret_cast<uint4 *>(brow + 16 * (chunk ^ (r & 7))) = out[cc];
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[s_b]);
                gb++;
                if ((kk & 3) == 3 || kk == nk - 1) {
                    if (lane == 0) mbar_arrive(&q_empty[s_q]);
                    gq++;
                }
            }
        }
    } else {
        // epilogue warps: thread = one TMEM lane = one slot row of the tile
        const int qw = warp & 3, row = 32 * qw + lane;
        uint32_t gt = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const TcItem x = tc_item(p, tile_off, nq, n_routed, it);
            const int buf = gt & 1;
            if (!tc_wait(&acc_full[buf], (gt >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            const int ri = x.mt * kTM + row;
            const bool valid = ri < x.pr.count;
            const size_t slot = (size_t)x.pr.slot0 + ri;
            const uint32_t tbase = tmem + ((uint32_t)(32 * qw) << 16) + (uint32_t)(buf * NMAT * kTN);
#pragma unroll 1
            for (int cc = 0; cc < kTN / 32; cc++) {
                uint32_t g[32];
                tmem_ld32(tbase + 32 * cc, g);
                if (NMAT == 2) {
                    uint32_t u[32];
                    tmem_ld32(tbase + kTN + 32 * cc, u);
                    tmem_ld_wait();
                    float a[32];
                    float amax = 0.0f;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        a[i] = swiglu(__uint_as_float(g[i]), __uint_as_float(u[i]));
                        amax = fmaxf(amax, fabsf(a[i]));
                    }
                    // the decode path's block quantiser, then f16 of q * d for the down operand
                    const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                    const float dq = __fdiv_rn(amax, 127.0f);
                    uint32_t h[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        float q0 = fminf(fmaxf(roundf(__fmul_rn(a[2 * i], id)), -127.0f), 127.0f);
                        float q1 = fminf(fmaxf(roundf(__fmul_rn(a[2 * i + 1], id)), -127.0f), 127.0f);
                        __half2 hv = __floats2half2_rn(q0 * dq, q1 * dq);
                        h[i] = *reinterpret_cast<uint32_t *>(&hv);
                    }
                    if (valid) {
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.a16dn) + slot * p.a16dn_stride +
                                                               x.nt * kTN + 32 * cc);
#pragma unroll
                        for (int v = 0; v < 4; v++) dst[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
                    }
                } else {
                    tmem_ld_wait();
                    if (valid) {
                        float4 *dst = reinterpret_cast<float4 *>(p.y + slot * p.H + x.nt * kTN + 32 * cc);
#pragma unroll
                        for (int v = 0; v < 8; v++)
                            dst[v] = make_float4(__uint_as_float(g[4 * v]), __uint_as_float(g[4 * v + 1]),
                                                 __uint_as_float(g[4 * v + 2]), __uint_as_float(g[4 * v + 3]));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
            gt++;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, NMAT == 2 ? 512 : 256);
    }
}

// A operand of the gate/up GEMM: slot s holds f16(xq * d) of its token (the
// activation blocks the decode path uses), 8 values per thread.
__global__ void gather_act_f16_kernel(FwdParams p, int n_slots)
{
    const int per_row = p.H >> 3;
    const long long total = (long long)n_slots * per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int s = (int)(i / per_row), c = (int)(i % per_row);
        const int tok = p.perm_token[s];
        const uint2 q = *reinterpret_cast<const uint2 *>(p.xq + (size_t)tok * p.H + 8 * c);
        const float d = p.xd[(size_t)tok * (p.H >> 5) + (c >> 2)];
        const int8_t *qb = reinterpret_cast<const int8_t *>(&q);
        uint32_t h[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            __half2 v = __floats2half2_rn((float)qb[2 * k] * d, (float)qb[2 * k + 1] * d);
            h[k] = *reinterpret_cast<uint32_t *>(&v);
        }
        *reinterpret_cast<uint4 *>(static_cast<__half *>(p.a16) + (size_t)s * p.a16_stride + 8 * c) =
            make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// Item offsets of the tensor-core launches (one warp): for each launch
// layout (gate/up routed+shared, gate/up shared only, down routed+shared, down
// shared only) the prefix over problems of m_tiles * n_tiles.
__global__ void tile_plan_kernel(FwdParams p, int rows_gu, int rows_gu_sh, int rows_dn)
{
    if (threadIdx.x != 0) return;
    const int nr = *p.n_active;
    const int mtile_sh = p.S > 0 ? (p.T + kTM - 1) / kTM : 0;
    int32_t *gu = p.tile_off, *gu_sh = p.tile_off + kTileOffStride;
    int32_t *dn = p.tile_off + 2 * kTileOffStride, *dn_sh = p.tile_off + 3 * kTileOffStride;
    int a = 0, b = 0;
    for (int q = 0; q < nr; q++) {
        gu[q] = a;
        dn[q] = b;
        const int mt = (p.problems[q].count + kTM - 1) / kTM;
        a += mt * (rows_gu / kTN);
        b += mt * (rows_dn / kTN);
    }
    gu[nr] = a;
    dn[nr] = b;
    gu[nr + 1] = a + mtile_sh * (rows_gu_sh / kTN);
    dn[nr + 1] = b + mtile_sh * (rows_dn / kTN);
    gu_sh[0] = 0;
    dn_sh[0] = 0;
    gu_sh[1] = mtile_sh * (rows_gu_sh / kTN);
    dn_sh[1] = mtile_sh * (rows_dn / kTN);
}

// f16 activation operand [rows][cols] with row stride stride_elems: box 64 x 128, 128-byte swizzle.
cudaError_t encode_f16_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint64_t stride_elems)
{
    return encode_tiled(m, 0, base, rows, cols, stride_elems * 2, kKS, kTM, 1) == 0 ? cudaSuccess
                                                                                    : cudaErrorInvalidValue;
}

template <int FMT, int NMAT>
cudaError_t launch_tc(const FwdParams &p, const LayerDev &L, const LayerMaps &lm, int mode, int num_sms,
                      cudaStream_t st)
{
    TcMaps maps;
    const DevMatrix &A0 = NMAT == 2 ? (mode == 1 ? L.sh_gate : L.gate) : (mode == 1 ? L.sh_down : L.down);
    const int K = A0.cols;
    cudaError_t e;
    if (NMAT == 2) e = encode_f16_map(&maps.a, p.a16, p.slots_cap, (uint64_t)p.H, p.a16_stride);
    else e = encode_f16_map(&maps.a, p.a16dn, p.slots_cap, (uint64_t)(mode == 2 ? p.W : K), p.a16dn_stride);
    if (e != cudaSuccess) return e;
    if (NMAT == 2) {
        maps.wq[0] = lm.gate_tc.qs; maps.wm[0] = lm.gate_tc.meta; maps.wq[1] = lm.up_tc.qs; maps.wm[1] = lm.up_tc.meta;
        maps.sq[0] = lm.sh_gate_tc.qs; maps.sm[0] = lm.sh_gate_tc.meta;
        maps.sq[1] = lm.sh_up_tc.qs; maps.sm[1] = lm.sh_up_tc.meta;
    } else {
        maps.wq[0] = maps.wq[1] = lm.down_tc.qs; maps.wm[0] = maps.wm[1] = lm.down_tc.meta;
        maps.sq[0] = maps.sq[1] = lm.sh_down_tc.qs; maps.sm[0] = maps.sm[1] = lm.sh_down_tc.meta;
    }
    TcCfg c{};
    c.nmat = NMAT;
    c.mode = mode;
    c.qs_box = FMT == FMT_Q4_K ? kSuper / 2 : kSuper;
    c.q_bytes = kTN * c.qs_box + kTN * 16;
    c.qstages = (FMT == FMT_Q8_0 && NMAT == 2) ? 1 : kQStages;   // Q8_0 gate+up stages are 68 KB each
    c.smem_a = 0;
    c.smem_b = c.smem_a + kAStages * kATileBytes;
    c.smem_q = c.smem_b + kBStages * NMAT * kBTileBytes;
    c.smem_bar = c.smem_q + c.qstages * NMAT * c.q_bytes;
    const size_t smem = (size_t)c.smem_bar + 256 + 1024;   // barriers + alignment slack
    if ((e = cudaFuncSetAttribute(tc_expert_kernel<FMT, NMAT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)) != cudaSuccess)
        return e;
    tc_expert_kernel<FMT, NMAT><<<num_sms, kTcThreads, smem, st>>>(p, L, c, maps);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                           const Marker &mk, cudaStream_t st)
{
    cudaError_t e;
    const int n_slots = p.T * p.k + (p.S > 0 ? p.T : 0);
    gather_act_f16_kernel<<<num_sms * 4, 256, 0, st>>>(p, n_slots);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    tile_plan_kernel<<<1, 32, 0, st>>>(p, L.gate.rows, p.S > 0 ? L.sh_gate.rows : 0, p.H);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    mk.mark("prefill_prep");
    const bool has_sh = p.S > 0;
    const bool same_gu = has_sh && L.sh_gate.type == L.gate.type;
    const bool same_dn = has_sh && L.sh_down.type == L.down.type;
    auto gu = [&](int mode) {
        const int fmt = mode == 1 ? L.sh_gate.type : L.gate.type;
        return fmt == FMT_Q4_K ? launch_tc<FMT_Q4_K, 2>(p, L, maps, mode, num_sms, st)
                               : launch_tc<FMT_Q8_0, 2>(p, L, maps, mode, num_sms, st);
    };
    auto dn = [&](int mode) {
        const int fmt = mode == 1 ? L.sh_down.type : L.down.type;
        return fmt == FMT_Q4_K ? launch_tc<FMT_Q4_K, 1>(p, L, maps, mode, num_sms, st)
                               : launch_tc<FMT_Q8_0, 1>(p, L, maps, mode, num_sms, st);
    };
    if ((e = gu(same_gu ? 2 : 0)) != cudaSuccess) return e;
    if (has_sh && !same_gu && (e = gu(1)) != cudaSuccess) return e;
    mk.mark("gate_up_tc");
    if ((e = dn(same_dn ? 2 : 0)) != cudaSuccess) return e;
    if (has_sh && !same_dn && (e = dn(1)) != cudaSuccess) return e;
    mk.mark("down_tc");
    return cudaSuccess;
}

}  // namespace jmoe
