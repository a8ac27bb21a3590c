// experts_i8.cu -- the expert FFN of a small batch (decode) as ONE persistent
// launch on the 5th-generation tensor cores with integer operands: gate/up
// with SwiGLU and down, the int32 sum of every 32-value block from one
// tcgen05.mma kind::i8, scaled and accumulated in f32 by the epilogue.
//
// A decode batch uses each weight value for a handful of tokens, so the launch
// is bound by streaming the weights from HBM, and the work per weight value
// must stay small. Here a Q4_K nibble becomes its u8 operand with about 0.4
// instructions per value (two masks per 32-bit word of 8 nibbles) and a Q8_0
// quant is the operand as loaded; the per-block scales are applied once per
// (row, block, slot) by the epilogue:
//     Q4_K: acc[row][slot] += (d sc)[row][blk] (dx[slot][blk] S) - (dmin m)[row][blk] sx[slot][blk]
//     Q8_0: acc[row][slot] += d[row][blk] (dx[slot][blk] S)
// with S the exact int32 block sum, dx the activation block scale and sx =
// dx * sum(q) -- the arithmetic of the int8 paths, so the integer sums equal
// the oracle's orc_block_dots. One thread cannot issue more than about one
// tcgen05 instruction (MMA or commit) per 130 cycles whatever N is, and lanes
// of one warp share that rate, so four warps issue (matrix x half of the
// blocks of each K step) with one commit each per step; the B stages are
// released by the epilogue, which sees every step's completion anyway.
//
// Work items (as the f16 fused launch, experts_tc.cu): gate/up = (problem, 128
// rows of the intermediate dim, chunk of up to 8 slots), matrix 0 = gate,
// 1 = up, K = H; down = (problem, 256 output rows, chunk), matrix 0/1 = the
// two 128-row halves, K = I (or S). A K step is 128 values (four blocks). The
// gate/up epilogue applies SwiGLU and the int8 block quantiser and stores the
// down operand rows (aq / ad / as); the down items of a chunk start once all
// of its gate/up tiles have counted themselves done (bounded wait; all gate/up
// items precede all down items and each CTA takes its items in order).
//
// Operands: A = Q8_0 quants straight from the TMA quant tile (128 rows x 128
// bytes, 128-byte swizzle), or Q4_K nibbles unpacked to u8 by the unpack warps
// into TMEM (one weight row per lane, four values per column in K order).
// B = the item's slot rows of int8 activation blocks, one TMA box (128 bytes,
// 128-byte swizzle) per row and K step. Block scales of the slots: copied per
// item into shared memory by the act warp. Weight scales: read by the epilogue
// from the quant stage's 16-byte scale rows.
// Warp roles (448 threads, one CTA per SM):
//   0       TMA producer of the quant ring
//   1       act: B operand loads, the item's activation block scales, the down
//           items' dependency waits
//   2..5    MMA issue, lane 0 of warp 2 + i: matrix i & 1, blocks 2 (i >> 1),
//           2 (i >> 1) + 1 of every step, one commit; warp 2 owns the TMEM
//   6..9    unpack (Q4_K) of the warp's TMEM lane quarter, thread = weight
//           row, both matrices
//   10..13  epilogue, thread = weight row = TMEM lane
// Rings: quant stages (TMA -> unpack / MMA / epilogue), A stages in TMEM
// (unpack -> MMA; reused once the block sums two steps back are complete), B
// stages (TMA -> MMA -> released by the epilogue), block sums in TMEM (MMA ->
// epilogue), item scales (act -> epilogue). Every wait is bounded; a timeout
// sets the status word and the CTA drains.
//
// Semantics followed: the per-token expert FFN of dispatch_qwen3_moe_ffn
// (src/qwen_deepseek.rs:847-951, run_single_swiglu_expert :748-771) over GGUF
// Q4_K / Q8_0 weights, with the activation blocks of the oracle's
// orc_quantize_act.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "fused_common.cuh"
#include "kernels.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace jmoe {
namespace {

constexpr int kYM = 128;                          // rows of a matrix tile (MMA M, TMEM lanes)
constexpr int kYKS = 128;                         // K values per step (four 32-value blocks)
constexpr int kYCap = 8;                          // slots per item (MMA N = 16, rows 8..15 unused)
constexpr int kYTma = 0, kYAct = 1, kYMma0 = 2, kYMmas = 4, kYUnp0 = 6, kYUnps = 4, kYEpi0 = 10, kYEpis = 4;
constexpr int kYThreads = (kYEpi0 + kYEpis) * 32;
constexpr int kYQuantBox = kYM * 128;             // quants of one matrix tile per quant stage (16 KB)
constexpr int kYQBytes = kYQuantBox + kYM * 16;   // + one 16-byte scale row per weight row
constexpr int kYStage = 2 * kYQBytes;             // both matrices (36 KB)
constexpr int kYBTile = 16 * 128;                 // B operand of one K step (N = 16 rows x 128 bytes)
constexpr int kYBst = 8;                          // B ring depth
constexpr int kYMaxQst = 4;
constexpr int kYAccS = 3;                         // block-sum stages in TMEM
constexpr int kYAccCols = 128;                    // a stage: [matrix][block][16 slots] int32
constexpr int kYA0 = kYAccS * kYAccCols;          // then the A stages (Q4_K)
constexpr int kYAs = 2;                           // A stages: 64 columns = [matrix][32 columns of u8 x 4]
constexpr long long kYDepWaitCycles = 4000000000LL;
static_assert(kYA0 + kYAs * 64 <= 512, "TMEM");

struct YCfg {
    int mode;                // 0 routed problems, 1 shared only, 2 both
    int qst;                 // quant ring depth
    int max_q;               // capacity of the problem table
    int kb_max;              // largest K / 32 of the launch's matrices (item scale rows)
    int smem_q, smem_b, smem_sc, smem_tab, smem_bar;
};

struct YMaps {
    CUtensorMap gq[2], gm[2];   // routed gate/up: quants (128 x 128 B, swizzle 128B), scales (128 x 16 B)
    CUtensorMap dq, dm;         // routed down
    CUtensorMap sq[2], sm[2];   // shared gate/up
    CUtensorMap sdq, sdm;       // shared down
    CUtensorMap bx, ba;         // B rows: xq token rows, aq slot rows (box 128 bytes x 1 row, swizzle 128B)
};

__device__ __forceinline__ bool ywait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    return tc_wait(bar, parity, abort_flag, err);
}

// The same wait by all 32 lanes of a warp, with one verdict for the warp (the
// warp-wide tcgen05 loads and stores that follow need every lane).
__device__ __forceinline__ bool ywait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    return __all_sync(0xffffffffu, tc_wait(bar, parity, abort_flag, err)) != 0;
}

// One item of the epilogue for NT (compile time, >= n) slots: consumes the
// item's K steps from the block-sum ring and returns the f32 sums of matrix 0
// and 1 for its row and the slots < n. The weight scales come from the quant
// stage (waited for, then released), the slot scales from the item's scale
// buffer sc: [slot][kb] dx, then [slot][kb] sx.
struct YEpi {
    uint64_t *q_full, *q_empty, *acc_full, *acc_empty, *b_empty, *a_empty;
    uint32_t sq;
    uint32_t sc;             // shared address of the item's scale buffer
    int kb;                  // K / 32 of the item (scale row length)
    int qst;
    volatile int *abort_flag;
};

// (d sc, dmin m) of sub-blocks 4 h .. 4 h + 3 from a Q4_K meta row (f16 d,
// f16 dmin, eight 12-bit fields sc | m << 6 from bit 32).
__device__ __forceinline__ void q4_scales4(const uint4 &m, int h, float (&sc)[4], float (&mn)[4])
{
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&m.x));
    // fields 4 h .. 4 h + 3 sit at bits 48 h .. 48 h + 47 of the 96 bits (y, z, w)
    const uint64_t lo = (uint64_t)m.y | ((uint64_t)m.z << 32);
    const uint64_t f48 = h ? ((uint64_t)(m.z >> 16) | ((uint64_t)m.w << 16)) : (lo & 0xFFFFFFFFFFFFull);
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const uint32_t f = (uint32_t)(f48 >> (12 * b)) & 0xFFFu;
        sc[b] = dd.x * (float)(f & 63u);
        mn[b] = dd.y * (float)(f >> 6);
    }
}

// d of the four blocks of half hf of a 256-value Q8_0 scale row (eight f16).
__device__ __forceinline__ void q8_scales4(const uint4 &m, int hf, float (&d)[4])
{
    const uint32_t w0 = hf ? m.z : m.x, w1 = hf ? m.w : m.y;
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&w0));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&w1));
    d[0] = a.x; d[1] = a.y; d[2] = b.x; d[3] = b.y;
}

template <int NT>
__device__ __forceinline__ bool epi_steps(const FwdParams &p, const YEpi &e, bool q4, int nk, int n, uint32_t tb0,
                                          int r, RingPos &qr, RingPos &cr, RingPos &br, RingPos &ar,
                                          float (&a0)[NT], float (&a1)[NT])
{
#pragma unroll
    for (int j = 0; j < NT; j++) { a0[j] = 0.0f; a1[j] = 0.0f; }
    const int spq = q4 ? 2 : 1;   // K steps per quant stage
    uint4 meta0 = make_uint4(0u, 0u, 0u, 0u), meta1 = meta0;
    for (int kk = 0; kk < nk; kk++) {
        const int h = q4 ? (kk & 1) : 0;
        if (h == 0) {
            if (!ywait_warp(&e.q_full[qr.slot], qr.phase, e.abort_flag, p.err)) return false;
            const uint32_t mrow = e.sq + (uint32_t)(qr.slot * kYStage + kYQuantBox + r * 16);
            meta0 = lds128(mrow);
            meta1 = lds128(mrow + kYQBytes);
        }
        // weight scales of this step's four blocks
        float s0[4], m0[4], s1[4], m1[4];
        if (q4) {
            q4_scales4(meta0, h, s0, m0);
            q4_scales4(meta1, h, s1, m1);
        } else {
            // a Q8_0 stage is 128 values: half (kk & 1) of the 256-value scale row
            q8_scales4(meta0, kk & 1, s0);
            q8_scales4(meta1, kk & 1, s1);
#pragma unroll
            for (int b = 0; b < 4; b++) { m0[b] = 0.0f; m1[b] = 0.0f; }
        }
        if (!ywait_warp(&e.acc_full[cr.slot], cr.phase, e.abort_flag, p.err)) return false;
        tc_fence_after();
        // the step's MMAs are complete: its A and B stages may be refilled
        if (threadIdx.x == kYEpi0 * 32) {
            mbar_arrive(&e.b_empty[br.slot]);
            mbar_arrive(&e.a_empty[ar.slot]);
        }
        br.advance(kYBst);
        ar.advance(kYAs);
        const uint32_t tb = tb0 + (uint32_t)(cr.slot * kYAccCols);
        // the step's four blocks are 16 contiguous bytes of every slot's scale rows
        const uint32_t scs = e.sc + 16u * (uint32_t)kk;
        // slots four at a time: the four slots' dx (and sx) rows of the step,
        // then per matrix its four blocks' sums of the four slots in flight
        // together
#pragma unroll
        for (int j0 = 0; j0 < NT; j0 += 4) {
            if (j0 < n) {
                uint4 dx[4], sx[4];
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    uint32_t S[4][4];
#pragma unroll
                    for (int b = 0; b < 4; b++) tmem_ld_small<4>(tb + (uint32_t)((4 * m + b) * 16 + j0), S[b]);
                    if (m == 0) {
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) {
                            dx[jj] = lds128(scs + 4u * (uint32_t)((j0 + jj) * e.kb));
                            sx[jj] = q4 ? lds128(scs + 4u * (uint32_t)((kYCap + j0 + jj) * e.kb))
                                        : make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                    tmem_ld_wait();
                    const float(&w)[4] = m ? s1 : s0;
                    const float(&mn)[4] = m ? m1 : m0;
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) {
                        const float dxv[4] = {__uint_as_float(dx[jj].x), __uint_as_float(dx[jj].y),
                                              __uint_as_float(dx[jj].z), __uint_as_float(dx[jj].w)};
                        const float sxv[4] = {__uint_as_float(sx[jj].x), __uint_as_float(sx[jj].y),
                                              __uint_as_float(sx[jj].z), __uint_as_float(sx[jj].w)};
                        float acc = m ? a1[j0 + jj] : a0[j0 + jj];
#pragma unroll
                        for (int b = 0; b < 4; b++) {
                            acc = __fmaf_rn(w[b], __fmul_rn(dxv[b], i2f_small((int)S[b][jj])), acc);
                            if (q4) acc = __fmaf_rn(-mn[b], sxv[b], acc);
                        }
                        if (m) a1[j0 + jj] = acc;
                        else a0[j0 + jj] = acc;
                    }
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&e.acc_empty[cr.slot]);
        cr.advance(kYAccS);
        if (h == spq - 1) {
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(&e.q_empty[qr.slot]);
            qr.advance(e.qst);
        }
    }
    return true;
}

// SwiGLU of one slot's gate and up sums and the int8 block quantiser of the
// down operand (the warp's 32 lanes are one 32-row block starting at row r0).
__device__ __forceinline__ void swiglu_quant_slot(const FwdParams &p, int slot, int r0, float g, float u, int lane)
{
    const size_t W = (size_t)p.W, s = (size_t)slot;
    quant_block32(swiglu(g, u), p.aq + s * W + r0, p.ad + s * (W >> 5) + (r0 >> 5), p.as + s * (W >> 5) + (r0 >> 5),
                  lane);
}

// One item of the epilogue: the f32 sums of its K steps, then SwiGLU and the
// int8 block quantiser of the down operand (gate/up) or the output rows (down).
template <int NT>
__device__ __forceinline__ bool epi_item(const FwdParams &p, const YEpi &e, const XItem &x, bool q4, int nk,
                                         uint32_t tb0, int wq, int lane, RingPos &qr, RingPos &cr, RingPos &br,
                                         RingPos &ar)
{
    float a0[NT], a1[NT];
    const int r = 32 * wq + lane;
    if (!epi_steps<NT>(p, e, q4, nk, x.n, tb0, r, qr, cr, br, ar, a0, a1)) return false;
    if (x.phase == 0) {
        // the warp's 32 lanes are one 32-row block of the intermediate dimension
        const int r0 = x.tile * kYM + 32 * wq;
#pragma unroll
        for (int j = 0; j < NT; j++)
            if (j < x.n) swiglu_quant_slot(p, x.slot + j, r0, a0[j], a1[j], lane);
    } else {
        const int f0 = x.tile * 2 * kYM + r;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            if (j < x.n) {
                float *yr = p.y + y_row(p, (size_t)x.slot + j) * p.H;
                yr[f0] = a0[j];
                yr[f0 + kYM] = a1[j];
            }
        }
    }
    return true;
}

// 14 warps: up to four per SM sub-partition, whose 16K registers cap a thread at 128
__global__ void __launch_bounds__(kYThreads, 1)
    fused_i8_kernel(FwdParams p, LayerDev L, YCfg c, const __grid_constant__ YMaps maps)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sq = base + c.smem_q, *sb = base + c.smem_b;
    float *ssc = reinterpret_cast<float *>(base + c.smem_sc);
    const int tab_n = (c.max_q + 4) & ~3;
    int *s_o0 = reinterpret_cast<int *>(base + c.smem_tab);
    int *s_o1 = s_o0 + tab_n, *s_cb = s_o1 + tab_n;
    int4 *s_prob = reinterpret_cast<int4 *>(s_cb + tab_n);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + c.smem_bar);
    uint64_t *q_full = bars, *q_empty = q_full + kYMaxQst;
    uint64_t *a_full = q_empty + kYMaxQst, *a_empty = a_full + kYAs;
    uint64_t *b_full = a_empty + kYAs, *b_empty = b_full + kYBst;
    uint64_t *acc_full = b_empty + kYBst, *acc_empty = acc_full + kYAccS;
    uint64_t *sc_full = acc_empty + kYAccS, *sc_empty = sc_full + 2, *drain_bar = sc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + kYMmas);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *s_last = reinterpret_cast<int *>(tmem_slot + 2);
    const int sc_stride = 2 * kYCap * c.kb_max;   // floats per item-scale buffer

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    pdl_wait();   // launched as a dependent: the routing output is complete
    pdl_trigger();

    const int n_routed = c.mode == 1 ? 0 : *p.n_active;
    const bool with_shared = c.mode != 0 && p.S > 0;
    const int nq = min(n_routed + (with_shared ? 1 : 0), c.max_q);
    for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        const bool sh = i >= n_routed;
        const Problem pr = sh ? p.problems[p.max_problems - 1] : p.problems[i];
        s_prob[i] = make_int4(pr.expert, pr.slot0, pr.count, sh ? 1 : 0);
    }
    __syncthreads();
    if (warp == 0) {
        int run0 = 0, run1 = 0, runc = 0;
        for (int b0 = 0; b0 < nq; b0 += 32) {
            const int i = b0 + lane;
            int v0 = 0, v1 = 0, vc = 0;
            if (i < nq) {
                const int4 pr = s_prob[i];
                vc = chunk_count(pr.z, kYCap);
                v0 = vc * ((pr.w ? L.sh_gate.rows : L.gate.rows) / kYM);
                v1 = vc * (p.H / (2 * kYM));
            }
            int i0 = v0, i1 = v1, ic = vc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u0 = __shfl_up_sync(0xffffffffu, i0, o);
                const int u1 = __shfl_up_sync(0xffffffffu, i1, o);
                const int uc = __shfl_up_sync(0xffffffffu, ic, o);
                if (lane >= o) { i0 += u0; i1 += u1; ic += uc; }
            }
            if (i < nq) {
                s_o0[i] = run0 + i0 - v0;
                s_o1[i] = run1 + i1 - v1;
                s_cb[i] = runc + ic - vc;
            }
            run0 += __shfl_sync(0xffffffffu, i0, 31);
            run1 += __shfl_sync(0xffffffffu, i1, 31);
            runc += __shfl_sync(0xffffffffu, ic, 31);
        }
        if (lane == 0) {
            s_o0[nq] = run0;
            s_o1[nq] = run1;
            s_cb[nq] = runc;
            // a quant stage is released by the unpack warps and the epilogue
            // (the epilogue's release of a stage follows the completion of the
            // MMAs that read it); the A and B stages of a step by the first
            // epilogue warp once the block sums of the step are complete
            for (int i = 0; i < c.qst; i++) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], kYUnps + kYEpis); }
            for (int i = 0; i < kYAs; i++) { mbar_init(&a_full[i], kYUnps); mbar_init(&a_empty[i], 1); }
            for (int i = 0; i < kYBst; i++) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
            for (int i = 0; i < kYAccS; i++) { mbar_init(&acc_full[i], kYMmas); mbar_init(&acc_empty[i], kYEpis); }
            for (int i = 0; i < 2; i++) { mbar_init(&sc_full[i], 1); mbar_init(&sc_empty[i], kYEpis); }
            for (int i = 0; i < kYMmas; i++) mbar_init(&drain_bar[i], 1);
            *abort_flag = 0;
            fence_barrier_init();
        }
    }
    if (warp == kYMma0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = nq > 0 ? s_o0[nq] + s_o1[nq] : 0;
    const bool fits = nq == 0 || s_cb[nq] <= p.dep_cap;
    const int n_items = fits ? total : 0;
    if (!fits && threadIdx.x == 0) atomicExch(p.err, kErrTimeout + 1);

    if (warp == kYTma) {
        if (lane == 0) {
            RingPos qr;
            uint32_t gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
                const DevMatrix &M = x_mat(L, x);
                const bool q4 = M.type == FMT_Q4_K;
                const int nqs = M.cols / (q4 ? 256 : 128);
                const CUtensorMap *mq0, *mm0, *mq1, *mm1;
                int y0, y1;
                if (x.phase == 0) {
                    mq0 = x.shared ? &maps.sq[0] : &maps.gq[0];
                    mm0 = x.shared ? &maps.sm[0] : &maps.gm[0];
                    mq1 = x.shared ? &maps.sq[1] : &maps.gq[1];
                    mm1 = x.shared ? &maps.sm[1] : &maps.gm[1];
                    y0 = y1 = x.expert * M.rows + x.tile * kYM;
                } else {
                    mq0 = mq1 = x.shared ? &maps.sdq : &maps.dq;
                    mm0 = mm1 = x.shared ? &maps.sdm : &maps.dm;
                    y0 = x.expert * M.rows + x.tile * 2 * kYM;
                    y1 = y0 + kYM;
                }
                for (int qs = 0; qs < nqs; qs++) {
                    if (!ywait(&q_empty[qr.slot], qr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint64_t *bar = &q_full[qr.slot];
                    mbar_arrive_expect_tx(bar, (uint32_t)kYStage);
                    uint8_t *dst = sq + (size_t)qr.slot * kYStage;
                    const int mx = q4 ? 2 * qs : 2 * (qs >> 1);   // 16-byte scale row of the 256-value group
                    tma_load_2d(dst, mq0, 16 * qs, y0, bar);
                    tma_load_2d(dst + kYQuantBox, mm0, mx, y0, bar);
                    tma_load_2d(dst + kYQBytes, mq1, 16 * qs, y1, bar);
                    tma_load_2d(dst + kYQBytes + kYQuantBox, mm1, mx, y1, bar);
                    qr.advance(c.qst);
                    gq++;
                }
            }
            if (!ok)   // wait (bounded) for the copies still in flight
                for (uint32_t g = gq > (uint32_t)c.qst ? gq - c.qst : 0; g < gq; g++)
                    drain_wait(&q_full[g % c.qst], (g / c.qst) & 1);
        }
    } else if (warp == kYAct) {
        const int tiles_gu_r = L.gate.rows / kYM, tiles_gu_s = p.S > 0 ? L.sh_gate.rows / kYM : 0;
        RingPos br, sr;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const int K = x_mat(L, x).cols, nk = K / kYKS, kb = K >> 5;
            if (x.phase == 1) {
                const int need = kYEpis * (x.shared ? tiles_gu_s : tiles_gu_r);
                const long long t0 = clock64();
                while (ld_acquire_gpu(p.dep + x.chunk) < need) {
                    if (*abort_flag) { ok = false; break; }
                    if (clock64() - t0 > kYDepWaitCycles) {
                        *abort_flag = 1;
                        atomicExch(p.err, kErrTimeout);
                        ok = false;
                        break;
                    }
                    __nanosleep(256);
                }
                ok = __all_sync(0xffffffffu, ok) != 0;
                if (!ok) break;
                fence_proxy_async_global();   // the generic stores seen above -> the TMA reads below
            }
            // the item's activation block scales: [slot][kb] dx, then [16 + slot][kb] sx
            if (!ywait_warp(&sc_empty[sr.slot], sr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
            float *dst = ssc + (size_t)sr.slot * sc_stride;
            const int kb4 = kb >> 2, units = x.n * kb4;
            for (int u = lane; u < 2 * units; u += 32) {
                const int which = u >= units, v = which ? u - units : u;
                const int j = v / kb4, c4 = v - j * kb4;
                const float *src;
                if (x.phase == 0) {
                    const size_t tok = (size_t)p.perm_token[x.slot + j];
                    src = (which ? p.xs : p.xd) + tok * (size_t)(p.H >> 5);
                } else {
                    src = (which ? p.as : p.ad) + ((size_t)x.slot + j) * (size_t)(p.W >> 5);
                }
                const float4 val = __ldcg(reinterpret_cast<const float4 *>(src) + c4);
                *reinterpret_cast<float4 *>(dst + (size_t)(which * kYCap + j) * kb + 4 * c4) = val;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sc_full[sr.slot]);
            sr.advance(2);
            // B operand: one TMA box per slot row and K step
            const CUtensorMap *map = x.phase == 0 ? &maps.bx : &maps.ba;
            const int row = lane < x.n ? (x.phase == 0 ? p.perm_token[x.slot + lane] : x.slot + lane) : 0;
            for (int kk = 0; kk < nk; kk++) {
                if (!ywait_warp(&b_empty[br.slot], br.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                if (lane == 0) mbar_arrive_expect_tx(&b_full[br.slot], (uint32_t)(x.n * 128));
                __syncwarp();
                if (lane < x.n)
                    tma_load_2d(sb + (size_t)br.slot * kYBTile + lane * 128, map, kk * (kYKS / 8), row, &b_full[br.slot]);
                br.advance(kYBst);
            }
        }
        if (!ok && lane == 0) {   // wait (bounded) for the loads still in flight
            for (int i = 0; i < kYBst; i++) {
                drain_wait(&b_full[br.slot], br.phase ^ 1u);
                br.advance(kYBst);
            }
        }
    } else if (warp < kYUnp0) {
        // MMA issue: lane 0 of warp kYMma0 + i issues matrix i & 1, blocks
        // 2 (i >> 1) and 2 (i >> 1) + 1 of every K step, and one commit per
        // step. Separate warps issue in parallel; one thread completes about
        // one tcgen05 instruction per 130 cycles.
        if (lane == 0) {
            const int iss = warp - kYMma0, m_i = iss & 1, hb = iss >> 1;
            const uint64_t q_desc0 = umma_desc_sw128(smem_addr(sq)), b_desc0 = umma_desc_sw128(smem_addr(sb));
            RingPos qr, br;
            uint32_t ks = 0;   // K steps of the launch so far (acc stage ks % kYAccS, A stage ks % kYAs)
            bool ok = true, issued = false;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
                const DevMatrix &M = x_mat(L, x);
                const bool q4 = M.type == FMT_Q4_K;
                const int nk = M.cols / kYKS, spq = q4 ? 2 : 1;
                // s32 accumulate; A u8 (Q4_K nibbles) or s8 (Q8_0), B s8; K-major; N = 16, M = 128
                const uint32_t idesc = (2u << 4) | ((q4 ? 0u : 1u) << 7) | (1u << 10) | ((16u >> 3) << 17) |
                                       ((uint32_t)(kYM >> 4) << 24);
                for (int kk = 0; kk < nk; kk++, ks++) {
                    const int h = q4 ? (kk & 1) : 0;
                    const uint32_t as = ks % kYAs, acs = ks % kYAccS;
                    if ((!q4 && !ywait(&q_full[qr.slot], qr.phase, abort_flag, p.err)) ||
                        !ywait(&acc_empty[acs], ((ks / kYAccS) & 1u) ^ 1u, abort_flag, p.err) ||
                        !ywait(&b_full[br.slot], br.phase, abort_flag, p.err) ||
                        !ywait(&a_full[as], (ks / kYAs) & 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bd = b_desc0 + (uint64_t)((br.slot * kYBTile) >> 4);
#pragma unroll
                    for (int bb = 0; bb < 2; bb++) {   // blocks 2 hb, 2 hb + 1: their own block-sum columns
                        const int b = 2 * hb + bb;
                        const uint32_t d = tmem + acs * (uint32_t)kYAccCols + (uint32_t)((m_i * 4 + b) * 16);
                        if (q4) {
                            tc_mma_i8_ts(d, tmem + (uint32_t)kYA0 + as * 64u + (uint32_t)(32 * m_i + 8 * b),
                                         bd + 2 * b, idesc, 0u);
                        } else {
                            const uint64_t ad = q_desc0 + (uint64_t)((qr.slot * kYStage + m_i * kYQBytes) >> 4);
                            tc_mma_i8(d, ad + 2 * b, bd + 2 * b, idesc, 0u);
                        }
                    }
                    issued = true;
                    tc_commit(&acc_full[acs]);
                    br.advance(kYBst);
                    if (h == spq - 1) qr.advance(c.qst);
                }
            }
            if (issued) {   // every MMA has completed before the CTA may release TMEM
                tc_commit(&drain_bar[iss]);
                drain_wait(&drain_bar[iss], 0);
            }
        }
    } else if (warp < kYEpi0) {
        // unpack: the warp's TMEM lane quarter of the A operand, thread =
        // weight row, Q4_K nibbles of both matrices to u8 (four values per
        // 32-bit column in K order). Every step completes a phase of its A
        // stage (Q8_0 steps without data, once their quant stage is in).
        const int quarter = warp & 3;
        const int r = 32 * quarter + lane;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t q_row = smem_addr(sq) + (uint32_t)(r * 128);
        const uint32_t arow = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)kYA0;
        RingPos qr;
        uint32_t ks = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const DevMatrix &M = x_mat(L, x);
            const bool q4 = M.type == FMT_Q4_K;
            const int nk = M.cols / kYKS, spq = q4 ? 2 : 1;
            for (int kk = 0; kk < nk; kk++, ks++) {
                const int h = q4 ? (kk & 1) : 0;
                const uint32_t as = ks % kYAs;
                if (h == 0 && !ywait_warp(&q_full[qr.slot], qr.phase, abort_flag, p.err)) { ok = false; break; }
                uint4 qv[2][4];
                if (q4) {
#pragma unroll
                    for (int m = 0; m < 2; m++)
#pragma unroll
                        for (int i = 0; i < 4; i++)   // sub-block 4 h + i of the 256-value quant row
                            qv[m][i] = lds128(q_row + (uint32_t)(qr.slot * kYStage + m * kYQBytes) +
                                              16u * ((uint32_t)(4 * h + i) ^ swz));
                }
                // the A stage is free once the MMAs that read it last (step ks -
                // kYAs) are complete. Waited for on every step, Q8_0 ones too, so
                // that the A stage phases never run a lap ahead of the MMA issuers
                // that wait for them.
                if (!ywait_warp(&a_empty[as], ((ks / kYAs) & 1u) ^ 1u, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                if (q4) {
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        uint32_t v[32];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint4 q = qv[m][i];
                            // values 0..15 (low nibbles), then 16..31 (high nibbles), four per column
                            v[8 * i + 0] = q.x & 0x0F0F0F0Fu;
                            v[8 * i + 1] = q.y & 0x0F0F0F0Fu;
                            v[8 * i + 2] = q.z & 0x0F0F0F0Fu;
                            v[8 * i + 3] = q.w & 0x0F0F0F0Fu;
                            v[8 * i + 4] = (q.x >> 4) & 0x0F0F0F0Fu;
                            v[8 * i + 5] = (q.y >> 4) & 0x0F0F0F0Fu;
                            v[8 * i + 6] = (q.z >> 4) & 0x0F0F0F0Fu;
                            v[8 * i + 7] = (q.w >> 4) & 0x0F0F0F0Fu;
                        }
                        tmem_st32(arow + as * 64u + 32u * (uint32_t)m, v);
                    }
                    tmem_st_wait();
                    tc_fence_before();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[as]);
                if (h == spq - 1) {
                    if (lane == 0) mbar_arrive(&q_empty[qr.slot]);
                    qr.advance(c.qst);
                }
            }
        }
    } else {
        const int wq = warp & 3;
        const YEpi e{q_full, q_empty, acc_full, acc_empty, b_empty, a_empty, smem_addr(sq), 0u, 0, c.qst, abort_flag};
        const uint32_t tb0 = tmem + ((uint32_t)(32 * wq) << 16);
        RingPos qr, cr, sr, br, ar;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const DevMatrix &M = x_mat(L, x);
            const bool q4 = M.type == FMT_Q4_K;
            const int nk = M.cols / kYKS;
            if (!ywait_warp(&sc_full[sr.slot], sr.phase, abort_flag, p.err)) break;
            YEpi ei = e;
            ei.sc = smem_addr(ssc + (size_t)sr.slot * sc_stride);
            ei.kb = M.cols >> 5;
            bool ok;
            if (x.n <= 4) ok = epi_item<4>(p, ei, x, q4, nk, tb0, wq, lane, qr, cr, br, ar);
            else ok = epi_item<8>(p, ei, x, q4, nk, tb0, wq, lane, qr, cr, br, ar);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sc_empty[sr.slot]);
            sr.advance(2);
            if (!ok) break;
            if (x.phase == 0) {
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(p.dep + x.chunk, 1);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kYMma0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    // the last CTA returns the chunk counters and the ticket to zero
    if (threadIdx.x == 0) {
        __threadfence();
        *s_last = atomicAdd(p.dep_done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (*s_last) {
        __threadfence();
        const int n = min(nq > 0 ? s_cb[nq] : 0, p.dep_cap);
        for (int i = threadIdx.x; i < n; i += blockDim.x) p.dep[i] = 0;
        if (threadIdx.x == 0) *p.dep_done = 0;
    }
}

bool y_matrix_ok(const DevMatrix &m, int row_tile)
{
    return (m.type == FMT_Q4_K || m.type == FMT_Q8_0) && m.rows % row_tile == 0 &&
           m.cols % (m.type == FMT_Q4_K ? 256 : 128) == 0 && m.cols >= 128 && m.cols % 128 == 0;
}

bool y_aligned(const void *ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace
}  // namespace jmoe

namespace jmoe {

bool fused_i8_ok(const FwdParams &p, const LayerDev &L)
{
    if (!y_matrix_ok(L.gate, kYM) || !y_matrix_ok(L.up, kYM) || !y_matrix_ok(L.down, 2 * kYM)) return false;
    if (L.gate.type != L.up.type || L.gate.rows != L.up.rows) return false;
    if (p.S > 0 && (!y_matrix_ok(L.sh_gate, kYM) || !y_matrix_ok(L.sh_up, kYM) || !y_matrix_ok(L.sh_down, 2 * kYM) ||
                    L.sh_gate.type != L.sh_up.type))
        return false;
    if (!p.dep || !p.dep_done || p.dep_cap <= 0) return false;
    // B rows: xq token rows and aq slot rows in 128-byte boxes; block scales as float4 rows
    if (p.x_qstride != 0 || p.x_dstride != 0 || p.y_rows) return false;
    if (p.H % 128 != 0 || p.W % 128 != 0) return false;
    if (!y_aligned(p.xq, 16) || !y_aligned(p.aq, 16) || !y_aligned(p.xd, 16) || !y_aligned(p.xs, 16) ||
        !y_aligned(p.ad, 16) || !y_aligned(p.as, 16))
        return false;
    return true;
}

cudaError_t launch_fused_i8(const FwdParams &p, const LayerDev &L, const LayerMaps &lm, int mode, int num_sms,
                            cudaStream_t st)
{
    YMaps maps;
    maps.gq[0] = lm.gate_tc.qs; maps.gm[0] = lm.gate_tc.meta;
    maps.gq[1] = lm.up_tc.qs; maps.gm[1] = lm.up_tc.meta;
    maps.dq = lm.down_tc.qs; maps.dm = lm.down_tc.meta;
    maps.sq[0] = lm.sh_gate_tc.qs; maps.sm[0] = lm.sh_gate_tc.meta;
    maps.sq[1] = lm.sh_up_tc.qs; maps.sm[1] = lm.sh_up_tc.meta;
    maps.sdq = lm.sh_down_tc.qs; maps.sdm = lm.sh_down_tc.meta;
    const int sx = p.T * p.k + (p.S > 0 ? p.T : 0);
    // int8 rows as u64 elements: 128 bytes = 16 elements per box
    if (encode_tiled(&maps.bx, 1, p.xq, (uint64_t)p.T, (uint64_t)p.H / 8, (uint64_t)p.H, kYKS / 8, 1, 1) != 0 ||
        encode_tiled(&maps.ba, 1, p.aq, (uint64_t)sx, (uint64_t)p.W / 8, (uint64_t)p.W, kYKS / 8, 1, 1) != 0)
        return cudaErrorInvalidValue;
    YCfg c{};
    c.mode = mode;
    c.max_q = p.max_problems;
    c.kb_max = (p.H > p.W ? p.H : p.W) / 32;
    const int tab = (((c.max_q + 4) & ~3) * 3 * 4 + c.max_q * 16 + 15) / 16 * 16;
    const int bar_bytes = (2 * kYMaxQst + 2 * kYAs + 2 * kYBst + 2 * kYAccS + 4 + kYMmas) * 8 + 16;
    const int sc_bytes = 2 * 2 * kYCap * c.kb_max * 4;
    const int fixed = kYBst * kYBTile + sc_bytes + tab + bar_bytes + 1024;   // + alignment slack
    c.qst = kYMaxQst;
    while (c.qst > 2 && (size_t)c.qst * kYStage + fixed > 232448) c.qst--;
    c.smem_q = 0;
    c.smem_b = c.smem_q + c.qst * kYStage;
    c.smem_sc = c.smem_b + kYBst * kYBTile;
    c.smem_tab = c.smem_sc + sc_bytes;
    c.smem_bar = c.smem_tab + tab;
    const size_t smem = (size_t)c.smem_bar + bar_bytes + 1024;
    if (smem > 232448) return cudaErrorInvalidValue;
    static int opted[64];
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || opted[dev] < (int)smem) {
        e = cudaFuncSetAttribute(fused_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) opted[dev] = (int)smem;
    }
    return launch_dependent(fused_i8_kernel, dim3(num_sms), dim3(kYThreads), smem, st, p, L, c, maps);
}

}  // namespace jmoe

