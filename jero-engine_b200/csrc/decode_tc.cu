// decode_tc.cu -- expert GEMMs of small batches on the 5th-generation tensor
// cores with integer operands (tcgen05.mma kind::i8, s32 results in TMEM).
//
// The streaming kernels compute each weight row . activation row as integer
// block sums (the 32 int8 activation values of a block times the block's 4-bit
// or 8-bit weight quants) scaled in f32. Here the tensor cores produce those
// block sums: one MMA per 32-value block (K = 32) writes the int32 sums of 128
// weight rows x N slots into the block's own TMEM columns, and the epilogue
// warps scale and accumulate them in f32, block by block in increasing K:
//     Q4_K: acc[row][slot] += (d*sc)[row][blk] * (dx[slot][blk] * S) - (dmin*m)[row][blk] * sx[slot][blk]
//     Q8_0: acc[row][slot] += d[row][blk] * (dx[slot][blk] * S)
// with dx the activation block scale and sx = dx * sum(q). The integer sums
// are exact and equal the dp4a ones (Q4_K nibbles as u8, activations s8).
//
// Operands: B = the item's activation rows in shared memory (128-byte
// swizzle). A = Q8_0 quants straight from the TMA tile in shared memory;
// Q4_K nibbles unpacked to u8 by the helper warps into TMEM (tcgen05.st, one
// weight row per lane), which keeps the unpacked tile out of shared memory.
//
// Work item: (problem, 128 weight rows, up to CAP slots); a K step is 128
// values (four blocks). Warp roles (448 threads, one CTA per SM):
//   0       TMA: quant tiles (128 rows x 128 bytes, 128-byte swizzle) and the
//           16-byte scale rows of each row
//   1       MMA issue (one thread); owns the 512 TMEM columns
//   2..5    helpers, thread = weight row (its TMEM lane): Q4_K nibbles -> u8
//           A operand, block scales decoded to f32, and chunks of the slot
//           rows of the activation operand (cp.async, six K steps ahead)
//   6..13   epilogue, thread = TMEM lane = weight row, in two warpgroups:
//           gate/up: one matrix each, the up sums handed to the gate group
//           for SwiGLU; down: two blocks of each K step each, the partial
//           sums of the second group added by the first
// Rings: quant stages (TMA -> helpers, and for Q8_0 the MMA operand itself),
// A stages in TMEM (helpers -> MMA, Q4_K), activation rows + their scales
// (helpers -> MMA and epilogue), weight scales (helpers -> epilogue), both
// freed by the epilogue, accumulator stages in TMEM (MMA -> epilogue). Every
// wait is bounded; a timeout sets the context's error word and the CTA drains.
//
// Semantics followed: the per-token expert FFN of dispatch_qwen3_moe_ffn
// (src/qwen_deepseek.rs:847-951) over GGUF Q4_K / Q8_0 weights, with the
// activation blocks of the streaming path (the oracle's orc_quantize_act).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace jmoe {
namespace {

constexpr int kDM = 128;                   // weight rows per item (MMA M, TMEM lanes)
constexpr int kDTma = 0, kDMma = 1, kDHelp0 = 2, kDHelpers = 4, kDEpi0 = kDHelp0 + kDHelpers, kDEpis = 8;
constexpr int kDThreads = (kDEpi0 + kDEpis) * 32;
constexpr int kDHT = kDHelpers * 32;       // helper threads (one per weight row)
constexpr int kDPf = 6;                    // K steps the activation copies run ahead
constexpr int kDMaxRing = 12;
constexpr int kDWst = 4;                   // weight-scale slots (written per step, freed by the epilogue)
constexpr int kDQuantBox = kDM * 128;      // quants of one matrix per quant stage
constexpr int kDQBytes = kDQuantBox + kDM * 16;   // + one 16-byte scale row per weight row
constexpr int kDWsc = kDM * 32;            // per matrix: [rows] float4 weight scale, then [rows] float4 min
constexpr int kDTmemCols = 512;
static_assert(kDHT == kDM, "one helper thread per weight row");

// Layout of one instantiation. gate/up items take up to 16 slots so that two
// matrices' accumulators (and for Q4_K the A stages) fit TMEM with room for
// three stages; down items take 32.
template <int FMT, int NMAT>
struct DtL {
    static constexpr bool Q4 = FMT == FMT_Q4_K;
    static constexpr int CAP = NMAT == 2 ? 16 : 32;                  // slots per item (MMA N <= CAP)
    static constexpr int BTILE = CAP * 128;                           // activation operand per K step
    static constexpr int DXS = CAP * 32;                              // per slot: d of four blocks, then d * sum(q)
    static constexpr int WSB = NMAT * kDWsc;                          // weight-scale slot
    static constexpr int STAGE = 4 * NMAT * CAP;                      // TMEM columns of an accumulator stage
    static constexpr int AS = Q4 ? 3 : 0;                             // A stages in TMEM (Q4_K)
    static constexpr int ACOLS = 32 * NMAT;                           // TMEM columns of an A stage
    static constexpr int TS0 = (kDTmemCols - AS * ACOLS) / STAGE;
    static constexpr int TS = TS0 < 4 ? TS0 : 4;                      // accumulator stages
    static constexpr int A0 = TS * STAGE;                             // first A column
    static constexpr int CH = CAP * 8 / kDHT;                         // activation chunks per helper thread
    static constexpr int XCH = CAP * kDM * 4;                         // epilogue exchange: [slot][row] f32
    static_assert(TS >= 2 && A0 + AS * ACOLS <= kDTmemCols && CH >= 1, "TMEM / helper layout");
};

struct DtCfg {
    int mode;                // 0 routed problems, 1 shared only, 2 both
    int qst, bst;            // ring depths: quant stages, activation slots
    int max_q;               // capacity of the item table
    int smem_q, smem_b, smem_d, smem_w, smem_x, smem_tab, smem_bar;
};

struct DtMaps {
    CUtensorMap wq[2], wm[2];   // routed: quants (128 rows x 128 bytes, swizzle 128B), scales (128 rows x 16 bytes)
    CUtensorMap sq[2], sm[2];   // shared expert
};

__device__ __forceinline__ float f4_at(const float4 &v, int i)
{
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Activation operand of one K step: the item's slot rows (128 values each,
// 128-byte swizzle: 16-byte chunk c of row n at position c ^ (n & 7)) and their
// block scales. Helper thread h copies chunk h & 7 of rows (h + i kDHT) >> 3,
// and half h & 1 of the scales of row h >> 1 (h < 2 CAP).
template <int CH>
struct ActSrc {
    const int8_t *q[CH];     // operand row bases (null: past the item's slots)
    const float *ds;         // scale row base (d or d * sum(q)), null when none
};

template <int NMAT, int CH>
__device__ __forceinline__ ActSrc<CH> act_src(const FwdParams &p, const TcItem &x, int h)
{
    ActSrc<CH> a{};
    const int nd = h >> 1, half = h & 1;
    const bool dsok = nd < x.n;   // nd < n <= CAP
    if (NMAT == 2) {
        const size_t qs = (size_t)(p.x_qstride ? p.x_qstride : p.H);
        const size_t dst = (size_t)(p.x_dstride ? p.x_dstride : (p.H >> 5));
#pragma unroll
        for (int i = 0; i < CH; i++) {
            const int na = (h + i * kDHT) >> 3;
            a.q[i] = na < x.n ? p.xq + (size_t)p.perm_token[x.slot + na] * qs : nullptr;
        }
        a.ds = dsok ? (half ? p.xs : p.xd) + (size_t)p.perm_token[x.slot + nd] * dst : nullptr;
    } else {
        const size_t W = (size_t)p.W;
#pragma unroll
        for (int i = 0; i < CH; i++) {
            const int na = (h + i * kDHT) >> 3;
            a.q[i] = na < x.n ? p.aq + (size_t)(x.slot + na) * W : nullptr;
        }
        a.ds = dsok ? (half ? p.as : p.ad) + (size_t)(x.slot + nd) * (W >> 5) : nullptr;
    }
    return a;
}

template <int CH>
__device__ __forceinline__ void issue_act(const ActSrc<CH> &a, uint32_t dst, uint32_t dst_ds, int h, int k0)
{
    const int c = h & 7;
#pragma unroll
    for (int i = 0; i < CH; i++) {
        const int na = (h + i * kDHT) >> 3;
        if (a.q[i]) cp_async16_s(dst + na * 128 + ((c ^ (na & 7)) << 4), a.q[i] + k0 + 16 * c);
    }
    if (a.ds) cp_async16_s(dst_ds + (h >> 1) * 32 + 16 * (h & 1), a.ds + (k0 >> 5));
}

// TMEM columns [col, col + NL) of this warp's 32 lanes.
template <int NL>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[NL])
{
    if constexpr (NL == 32) tmem_ld32(taddr, r);
    else if constexpr (NL == 16) tmem_ld16(taddr, r);
    else tmem_ld_small<NL>(taddr, r);
}

// Epilogue of one item by one warpgroup (wg): consumes its nk TMEM stages and
// stores the result. gate/up: warpgroup wg accumulates matrix wg over all four
// blocks of a K step; down: blocks 2 wg and 2 wg + 1. The second warpgroup
// then hands its sums for the item to the first through xch (bounded
// mbarriers, one pair per 32-row quarter), which finishes the item.
// NT (compile time) slots are computed for the item's n <= NT; columns past n
// hold sums of stale operand rows, are computed like the others (no branch
// per slot, so the chains of all slots interleave) and never stored.
struct EpiSync {
    uint64_t *t_full, *t_empty, *b_full, *b_empty, *w_empty, *x_full, *x_empty;
    const uint8_t *dxs, *wsc;   // activation scale slots, weight-scale slots
    float *xch;
    int bst;
    volatile int *abort_flag;
};

template <int FMT, int NMAT, int NT>
__device__ __forceinline__ bool epi_item(const FwdParams &p, const TcItem &x, int nk, uint32_t tmem,
                                         const EpiSync &es, RingPos &tr, RingPos &br, RingPos &wr, RingPos &xr,
                                         int wg, int wq, int lane)
{
    using Lt = DtL<FMT, NMAT>;
    constexpr bool Q4 = Lt::Q4;
    constexpr int NL = NT <= 1 ? 1 : NT <= 2 ? 2 : NT <= 4 ? 4 : NT <= 8 ? 8 : NT <= 16 ? 16 : 32;   // load width
    constexpr int NB = NMAT == 2 ? 4 : 2;        // blocks of a K step per warpgroup
    constexpr int BG = NL * NB <= 32 ? NB : (NL * 2 <= 32 ? 2 : 1);   // blocks per TMEM load group
    const int m = NMAT == 2 ? wg : 0, b0 = NMAT == 2 ? 0 : 2 * wg;
    const int r = 32 * wq + lane;
    const uint32_t npad = x.n <= 16 ? 16u : 32u;   // column stride of the MMA's blocks
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    for (int kk = 0; kk < nk; kk++) {
        // the epilogue and TMA warps wait sleeping (they have slack; spinning
        // would take issue slots from the helpers); the MMA and helpers spin
        if (!tc_wait(&es.t_full[tr.slot], tr.phase, es.abort_flag, p.err) ||
            !tc_wait(&es.b_full[br.slot], br.phase, es.abort_flag, p.err))
            return false;
        tc_fence_after();
        const float *dxs = reinterpret_cast<const float *>(es.dxs + (size_t)br.slot * Lt::DXS);   // [slot][d0..d3, s0..s3]
        const float4 *wsc = reinterpret_cast<const float4 *>(es.wsc + (size_t)wr.slot * Lt::WSB);
        const float4 sw = wsc[m * (kDWsc / 16) + r];
        const float4 mw = Q4 ? wsc[m * (kDWsc / 16) + kDM + r] : make_float4(0.f, 0.f, 0.f, 0.f);
        const uint32_t tb = tmem + ((uint32_t)(32 * wq) << 16) + (uint32_t)(tr.slot * Lt::STAGE);
#pragma unroll
        for (int g = 0; g < NB; g += BG) {
            uint32_t S[BG][NL];
#pragma unroll
            for (int bb = 0; bb < BG; bb++) tmem_ld_cols<NL>(tb + (uint32_t)((b0 + g + bb) * NMAT + m) * npad, S[bb]);
            tmem_ld_wait();
            if (g + BG == NB) {   // this warp's columns of the stage are in registers
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&es.t_empty[tr.slot]);
            }
            if (NMAT == 2 && p.dbg_isum && !x.shared) {   // parity probe: the raw int32 block sums
                const size_t f = (size_t)x.nt * kDM + r, nb = (size_t)(p.H >> 5);
#pragma unroll
                for (int t = 0; t < NT; t++)
#pragma unroll
                    for (int bb = 0; bb < BG; bb++)
                        if (t < x.n)
                            p.dbg_isum[(((size_t)(x.slot + t) * 2 + m) * p.I + f) * nb + 4 * kk + b0 + g + bb] =
                                (int32_t)S[bb][t];
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
#pragma unroll
                for (int bb = 0; bb < BG; bb++) {
                    const int b = b0 + g + bb;
                    const float v = __fmul_rn(dxs[t * 8 + b], i2f_small((int)S[bb][t]));
                    acc[t] = __fmaf_rn(f4_at(sw, b), v, acc[t]);
                    if (Q4) acc[t] = __fmaf_rn(-f4_at(mw, b), dxs[t * 8 + 4 + b], acc[t]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&es.b_empty[br.slot]);
            mbar_arrive(&es.w_empty[wr.slot]);
        }
        tr.advance(Lt::TS);
        br.advance(es.bst);
        wr.advance(kDWst);
    }
    // hand-off between the warpgroups
    float *xrow = es.xch + r;
    if (wg == 1) {
        if (!tc_wait(&es.x_empty[wq], xr.phase ^ 1u, es.abort_flag, p.err)) return false;
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < x.n) xrow[t * kDM] = acc[t];
        __syncwarp();
        if (lane == 0) mbar_arrive(&es.x_full[wq]);
        xr.advance(1);
        return true;
    }
    if (!tc_wait(&es.x_full[wq], xr.phase, es.abort_flag, p.err)) return false;
    float other[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) other[t] = t < x.n ? xrow[t * kDM] : 0.0f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&es.x_empty[wq]);
    xr.advance(1);
    if (NMAT == 2) {
        // SwiGLU, then the activation block quantiser of the down operand: the
        // warp's 32 lanes are one 32-row block of the intermediate dimension
        const int r0 = x.nt * kDM + 32 * wq;
        const size_t W = (size_t)p.W;
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < x.n) {
                const size_t slot = (size_t)x.slot + t;
                const float a = swiglu(acc[t], other[t]);
                quant_block32(a, p.aq + slot * W + r0, p.ad + slot * (W >> 5) + (r0 >> 5),
                              p.as + slot * (W >> 5) + (r0 >> 5), lane);
            }
        }
    } else {
        const int f = x.nt * kDM + r;
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < x.n) p.y[y_row(p, (size_t)x.slot + t) * p.H + f] = __fadd_rn(acc[t], other[t]);
    }
    return true;
}

// Q4_K scales of the eight sub-blocks of a super-block (device meta: f16 d,
// f16 dmin, eight 12-bit fields sc | m << 6 from bit 32): (d * sc, dmin * m).
__device__ __forceinline__ void q4_scales8(const uint4 &m, float (&sc)[8], float (&mn)[8])
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

template <int FMT, int NMAT>
__global__ void __launch_bounds__(kDThreads, 1)
    dtc_expert_kernel(FwdParams p, LayerDev L, DtCfg c, const __grid_constant__ DtMaps maps)
{
    using Lt = DtL<FMT, NMAT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sq = base + c.smem_q, *sb = base + c.smem_b, *sd = base + c.smem_d, *sw = base + c.smem_w;
    float *xch = reinterpret_cast<float *>(base + c.smem_x);
    int *s_off = reinterpret_cast<int *>(base + c.smem_tab);
    int4 *s_prob = reinterpret_cast<int4 *>(s_off + ((c.max_q + 4) & ~3));
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + c.smem_bar);
    uint64_t *q_full = bars, *q_empty = q_full + kDMaxRing, *a_full = q_empty + kDMaxRing;
    uint64_t *a_empty = a_full + kDMaxRing, *b_full = a_empty + kDMaxRing, *b_empty = b_full + kDMaxRing;
    uint64_t *w_empty = b_empty + kDMaxRing;
    uint64_t *t_full = w_empty + kDWst, *t_empty = t_full + 4, *x_full = t_empty + 4, *x_empty = x_full + 4;
    uint64_t *drain_bar = x_empty + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    constexpr bool Q4 = Lt::Q4;
    constexpr int QK = Q4 ? 2 : 1;   // K steps per quant stage (256 / 128 values)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    pdl_wait();   // launched as a dependent: routing / gate_up output is complete
    pdl_trigger();

    // the launch's problems (routed ones, then the shared expert) and the
    // first item of each: slot chunks x 128-row weight tiles
    const int n_routed = c.mode == 1 ? 0 : *p.n_active;
    const bool with_shared = c.mode != 0 && p.S > 0;
    const int nq = min(n_routed + (with_shared ? 1 : 0), c.max_q);
    const int rows_r = NMAT == 2 ? L.gate.rows : L.down.rows;
    const int rows_s = NMAT == 2 ? L.sh_gate.rows : L.sh_down.rows;
    for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        const bool sh = i >= n_routed;
        const Problem pr = sh ? p.problems[p.max_problems - 1] : p.problems[i];
        s_prob[i] = make_int4(pr.expert, pr.slot0, pr.count, sh ? 1 : 0);
    }
    __syncthreads();
    if (warp == 0) {
        int run = 0;
        for (int b0 = 0; b0 < nq; b0 += 32) {
            const int i = b0 + lane;
            int v = 0;
            if (i < nq) {
                const int4 pr = s_prob[i];
                v = chunk_count(pr.z, Lt::CAP) * ((pr.w ? rows_s : rows_r) / kDM);
            }
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            if (i < nq) s_off[i] = run + incl - v;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            s_off[nq] = run;
            for (int i = 0; i < c.qst; i++) {
                mbar_init(&q_full[i], 1);
                mbar_init(&q_empty[i], kDHelpers + (Q4 ? 0 : 1));
            }
            for (int i = 0; i < Lt::AS; i++) { mbar_init(&a_full[i], kDHelpers); mbar_init(&a_empty[i], 1); }
            for (int i = 0; i < c.bst; i++) { mbar_init(&b_full[i], kDHelpers); mbar_init(&b_empty[i], kDEpis); }
            for (int i = 0; i < kDWst; i++) mbar_init(&w_empty[i], kDEpis);
            for (int i = 0; i < Lt::TS; i++) { mbar_init(&t_full[i], 1); mbar_init(&t_empty[i], kDEpis); }
            for (int i = 0; i < 4; i++) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
            mbar_init(drain_bar, 1);
            *abort_flag = 0;
            fence_barrier_init();
        }
    }
    if (warp == kDMma) tmem_alloc(tmem_slot, kDTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = nq > 0 ? s_off[nq] : 0;

    if (warp == kDTma) {
        if (lane == 0) {
            RingPos qr;
            uint32_t gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(s_off, s_prob, nq, Lt::CAP, it);
                const DevMatrix &M0 = NMAT == 2 ? (x.shared ? L.sh_gate : L.gate) : (x.shared ? L.sh_down : L.down);
                const int nqs = M0.cols / (128 * QK);
                const int wy = x.expert * M0.rows + x.nt * kDM;
                const CUtensorMap *mq0 = x.shared ? &maps.sq[0] : &maps.wq[0], *mm0 = x.shared ? &maps.sm[0] : &maps.wm[0];
                const CUtensorMap *mq1 = x.shared ? &maps.sq[1] : &maps.wq[1], *mm1 = x.shared ? &maps.sm[1] : &maps.wm[1];
                for (int qs = 0; qs < nqs; qs++) {
                    if (!tc_wait(&q_empty[qr.slot], qr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint64_t *bar = &q_full[qr.slot];
                    mbar_arrive_expect_tx(bar, (uint32_t)(NMAT * kDQBytes));
                    uint8_t *dst = sq + (size_t)qr.slot * NMAT * kDQBytes;
                    const int mx = Q4 ? 2 * qs : 2 * (qs >> 1);   // 16-byte scale row of the 256-value group
                    tma_load_2d(dst, mq0, 16 * qs, wy, bar);
                    tma_load_2d(dst + kDQuantBox, mm0, mx, wy, bar);
                    if (NMAT == 2) {
                        tma_load_2d(dst + kDQBytes, mq1, 16 * qs, wy, bar);
                        tma_load_2d(dst + kDQBytes + kDQuantBox, mm1, mx, wy, bar);
                    }
                    qr.advance(c.qst);
                    gq++;
                }
            }
            if (!ok)   // wait (bounded) for the copies still in flight
                for (uint32_t g = gq > (uint32_t)c.qst ? gq - c.qst : 0; g < gq; g++)
                    drain_wait(&q_full[g % c.qst], (g / c.qst) & 1);
        }
    } else if (warp == kDMma) {
        if (lane == 0) {
            RingPos qr, ar, br, tr;
            bool ok = true, issued = false;
            const uint64_t q_desc0 = umma_desc_sw128(smem_addr(sq)), b_desc0 = umma_desc_sw128(smem_addr(sb));
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(s_off, s_prob, nq, Lt::CAP, it);
                const int K = NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                        : (x.shared ? L.sh_down.cols : L.down.cols);
                const int nk = K >> 7;
                const uint32_t npad = x.n <= 16 ? 16u : 32u;
                // s32 accumulate; A u8 (Q4_K nibbles) or s8 (Q8_0), B s8; both K-major; N = npad, M = 128
                const uint32_t idesc = (2u << 4) | ((Q4 ? 0u : 1u) << 7) | (1u << 10) | ((npad >> 3) << 17) |
                                       ((uint32_t)(kDM >> 4) << 24);
                for (int kk = 0; kk < nk; kk++) {
                    const bool w_ok = Q4 ? tc_spin_wait(&a_full[ar.slot], ar.phase, abort_flag, p.err)
                                         : tc_spin_wait(&q_full[qr.slot], qr.phase, abort_flag, p.err);
                    if (!w_ok || !tc_spin_wait(&b_full[br.slot], br.phase, abort_flag, p.err) ||
                        !tc_spin_wait(&t_empty[tr.slot], tr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t dbase = tmem + (uint32_t)(tr.slot * Lt::STAGE);
                    const uint64_t bd = b_desc0 + (uint64_t)((br.slot * Lt::BTILE) >> 4);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
#pragma unroll
                        for (int b = 0; b < 4; b++) {   // one block (K = 32 bytes) per MMA, its own columns
                            const uint32_t d = dbase + (uint32_t)(b * NMAT + m) * npad;
                            if (Q4) {
                                const uint32_t a = tmem + (uint32_t)(Lt::A0 + (ar.slot * NMAT + m) * 32 + 8 * b);
                                tc_mma_i8_ts(d, a, bd + 2 * b, idesc, 0u);
                            } else {
                                const uint64_t ad = q_desc0 + (uint64_t)(((qr.slot * NMAT + m) * kDQBytes) >> 4);
                                tc_mma_i8(d, ad + 2 * b, bd + 2 * b, idesc, 0u);
                            }
                        }
                    }
                    issued = true;
                    if (Q4) {
                        tc_commit(&a_empty[ar.slot]);
                        ar.advance(Lt::AS);
                    } else {
                        tc_commit(&q_empty[qr.slot]);
                        qr.advance(c.qst);
                    }
                    tc_commit(&t_full[tr.slot]);
                    tr.advance(Lt::TS);
                    br.advance(c.bst);
                }
            }
            if (issued) {   // every MMA has completed before the CTA may release TMEM
                tc_commit(drain_bar);
                drain_wait(drain_bar, 0);
            }
        }
    } else if (warp < kDEpi0) {
        // helpers: thread = weight row r = this warp's TMEM lane window + lane
        const int h = threadIdx.x - kDHelp0 * 32, r = 32 * (warp & 3) + lane;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t sq_a = smem_addr(sq), sb_a = smem_addr(sb), sd_a = smem_addr(sd), sw_a = smem_addr(sw);
        const uint32_t arow = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)Lt::A0;
        RingPos qr, ar, bc, bp, wc;
        bool ok = true;
        // the activation copies run kDPf K steps ahead of the current step: a
        // second cursor (item, K step) over the same item sequence
        int it_p = blockIdx.x, kk_p = 0, nk_p = 0;
        TcItem x_p{};
        ActSrc<Lt::CH> src_p{};
        auto load_item = [&](int it) {
            x_p = tc_item(s_off, s_prob, nq, Lt::CAP, it);
            nk_p = (NMAT == 2 ? (x_p.shared ? L.sh_gate.cols : L.gate.cols)
                              : (x_p.shared ? L.sh_down.cols : L.down.cols)) >> 7;
            src_p = act_src<NMAT, Lt::CH>(p, x_p, h);
        };
        if (it_p < total) load_item(it_p);
        auto prefetch = [&]() -> bool {
            if (it_p < total) {
                if (!tc_spin_wait(&b_empty[bp.slot], bp.phase ^ 1u, abort_flag, p.err)) return false;
                issue_act<Lt::CH>(src_p, sb_a + (uint32_t)(bp.slot * Lt::BTILE), sd_a + (uint32_t)(bp.slot * Lt::DXS), h,
                                  kk_p * 128);
                bp.advance(c.bst);
                if (++kk_p == nk_p) {
                    kk_p = 0;
                    it_p += gridDim.x;
                    if (it_p < total) load_item(it_p);
                }
            }
            cp_async_commit();   // one group per step, empty past the end
            return true;
        };
        float s8v[NMAT][8], m8v[NMAT][8];   // Q4_K: decoded scales of the current super-block
        for (int i = 0; i < kDPf && ok; i++) ok = prefetch();
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const TcItem x = tc_item(s_off, s_prob, nq, Lt::CAP, it);
            const int nk = (NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                      : (x.shared ? L.sh_down.cols : L.down.cols)) >> 7;
            for (int kk = 0; kk < nk; kk++) {
                if (!prefetch()) { ok = false; break; }
                const int qi = Q4 ? (kk & 1) : 0;
                if (qi == 0 && !tc_spin_wait(&q_full[qr.slot], qr.phase, abort_flag, p.err)) { ok = false; break; }
                if (Q4 && !tc_spin_wait(&a_empty[ar.slot], ar.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                if (!tc_spin_wait(&w_empty[wc.slot], wc.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                const uint32_t wsc = sw_a + (uint32_t)(wc.slot * Lt::WSB);
                if (Q4) {
                    tc_fence_after();   // the MMA that read this A stage has completed
                    uint4 qv[NMAT][4];
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const uint32_t qm = sq_a + (uint32_t)((qr.slot * NMAT + m) * kDQBytes);
                        if (qi == 0) q4_scales8(lds128(qm + kDQuantBox + (uint32_t)r * 16), s8v[m], m8v[m]);
#pragma unroll
                        for (int i = 0; i < 4; i++)   // sub-block 4 qi + i of the 256-value quant row
                            qv[m][i] = lds128(qm + (uint32_t)r * 128 + 16u * ((uint32_t)(4 * qi + i) ^ swz));
                    }
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const uint32_t acol = arow + (uint32_t)((ar.slot * NMAT + m) * 32);
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint4 q = qv[m][i];
                            // values 0..15 (low nibbles), then 16..31 (high nibbles), four per column
                            const uint32_t v[8] = {q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q.z & 0x0F0F0F0Fu,
                                                   q.w & 0x0F0F0F0Fu, (q.x >> 4) & 0x0F0F0F0Fu,
                                                   (q.y >> 4) & 0x0F0F0F0Fu, (q.z >> 4) & 0x0F0F0F0Fu,
                                                   (q.w >> 4) & 0x0F0F0F0Fu};
                            tmem_st8(acol + 8 * i, v);
                        }
                        const uint32_t wrow = wsc + (uint32_t)(m * kDWsc) + (uint32_t)r * 16;
                        float s4[4], m4[4];   // blocks 4 qi .. 4 qi + 3 (selects keep the arrays in registers)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            s4[i] = qi ? s8v[m][4 + i] : s8v[m][i];
                            m4[i] = qi ? m8v[m][4 + i] : m8v[m][i];
                        }
                        sts128(wrow, make_uint4(__float_as_uint(s4[0]), __float_as_uint(s4[1]),
                                                __float_as_uint(s4[2]), __float_as_uint(s4[3])));
                        sts128(wrow + kDM * 16, make_uint4(__float_as_uint(m4[0]), __float_as_uint(m4[1]),
                                                           __float_as_uint(m4[2]), __float_as_uint(m4[3])));
                    }
                    tmem_st_wait();
                    tc_fence_before();
                } else {
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        // f16 d of blocks 4 (kk & 1) .. + 3 of the 256-value scale row
                        const uint4 meta = lds128(sq_a + (uint32_t)((qr.slot * NMAT + m) * kDQBytes) + kDQuantBox +
                                                  (uint32_t)r * 16);
                        const uint32_t w0 = (kk & 1) ? meta.z : meta.x, w1 = (kk & 1) ? meta.w : meta.y;
                        const float2 d01 = __half22float2(*reinterpret_cast<const __half2 *>(&w0));
                        const float2 d23 = __half22float2(*reinterpret_cast<const __half2 *>(&w1));
                        sts128(wsc + (uint32_t)(m * kDWsc) + (uint32_t)r * 16,
                               make_uint4(__float_as_uint(d01.x), __float_as_uint(d01.y), __float_as_uint(d23.x),
                                          __float_as_uint(d23.y)));
                    }
                }
                cp_async_wait<kDPf>();   // this step's activation rows have landed
                fence_async_smem();      // operand writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&b_full[bc.slot]);
                    if (Q4) mbar_arrive(&a_full[ar.slot]);
                }
                bc.advance(c.bst);
                wc.advance(kDWst);
                if (Q4) ar.advance(Lt::AS);
                if (qi == QK - 1 || kk == nk - 1) {
                    if (lane == 0) mbar_arrive(&q_empty[qr.slot]);
                    qr.advance(c.qst);
                }
            }
        }
        cp_async_wait<0>();
    } else {
        const int wq = warp & 3;   // TMEM lane window of this warp
        const int wg = (warp - kDEpi0) >> 2;
        const EpiSync es{t_full, t_empty, b_full, b_empty, w_empty, x_full, x_empty, sd, sw, xch, c.bst, abort_flag};
        RingPos tr, br, wr, xr;
        for (int it = blockIdx.x; it < total; it += gridDim.x) {
            const TcItem x = tc_item(s_off, s_prob, nq, Lt::CAP, it);
            const int nk = (NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                      : (x.shared ? L.sh_down.cols : L.down.cols)) >> 7;
            bool ok;
#define JMOE_EPI(NTV) ok = epi_item<FMT, NMAT, NTV>(p, x, nk, tmem, es, tr, br, wr, xr, wg, wq, lane)
            switch (x.n) {
            case 1: JMOE_EPI(1); break;
            case 2: JMOE_EPI(2); break;
            case 3: JMOE_EPI(3); break;
            case 4: JMOE_EPI(4); break;
            case 5: JMOE_EPI(5); break;
            case 6: JMOE_EPI(6); break;
            case 7: JMOE_EPI(7); break;
            case 8: JMOE_EPI(8); break;
            default:
                if (x.n <= 12) JMOE_EPI(12);
                else if (Lt::CAP <= 16 || x.n <= 16) JMOE_EPI(16);
                else if (x.n <= 24) JMOE_EPI(24);
                else JMOE_EPI(32);
            }
#undef JMOE_EPI
            if (!ok) break;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kDMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kDTmemCols);
    }
}

template <int FMT, int NMAT>
cudaError_t launch_dtc(const FwdParams &p, const LayerDev &L, const LayerMaps &lm, int mode, int num_sms,
                       cudaStream_t st)
{
    using Lt = DtL<FMT, NMAT>;
    DtMaps maps;
    if (NMAT == 2) {
        maps.wq[0] = lm.gate_tc.qs; maps.wm[0] = lm.gate_tc.meta; maps.wq[1] = lm.up_tc.qs; maps.wm[1] = lm.up_tc.meta;
        maps.sq[0] = lm.sh_gate_tc.qs; maps.sm[0] = lm.sh_gate_tc.meta;
        maps.sq[1] = lm.sh_up_tc.qs; maps.sm[1] = lm.sh_up_tc.meta;
    } else {
        maps.wq[0] = maps.wq[1] = lm.down_tc.qs; maps.wm[0] = maps.wm[1] = lm.down_tc.meta;
        maps.sq[0] = maps.sq[1] = lm.sh_down_tc.qs; maps.sm[0] = maps.sm[1] = lm.sh_down_tc.meta;
    }
    DtCfg c{};
    c.mode = mode;
    c.max_q = p.max_problems;
    // ring depths by shared-memory room: a quant stage is 18 KB per matrix, an
    // activation slot 2.5 KB (gate/up) or 5 KB (down), a weight-scale slot 4 KB
    // per matrix, the exchange 8 / 16 KB
    c.qst = NMAT == 2 ? 4 : 7;
    c.bst = 10;
    c.smem_q = 0;
    c.smem_b = c.smem_q + c.qst * NMAT * kDQBytes;
    c.smem_d = c.smem_b + c.bst * Lt::BTILE;
    c.smem_w = c.smem_d + c.bst * Lt::DXS;
    c.smem_x = c.smem_w + kDWst * Lt::WSB;
    c.smem_tab = c.smem_x + Lt::XCH;
    c.smem_bar = c.smem_tab + (((c.max_q + 4) & ~3) * 4 + c.max_q * 16 + 15) / 16 * 16;
    const size_t smem = (size_t)c.smem_bar + (6 * kDMaxRing + kDWst + 17) * 8 + 16 + 1024;   // barriers + alignment slack
    if (smem > 232448) return cudaErrorInvalidValue;
    static int opted[64];
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || opted[dev] < (int)smem) {
        e = cudaFuncSetAttribute(dtc_expert_kernel<FMT, NMAT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) opted[dev] = (int)smem;
    }
    return launch_dependent(dtc_expert_kernel<FMT, NMAT>, dim3(num_sms), dim3(kDThreads), smem, st, p, L, c, maps);
}

bool dtc_matrix_ok(const DevMatrix &m)
{
    return (m.type == FMT_Q4_K || m.type == FMT_Q8_0) && m.rows % kDM == 0 &&
           m.cols % (m.type == FMT_Q4_K ? 256 : 128) == 0;
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace

bool decode_tc_ok(const FwdParams &p, const LayerDev &L)
{
    if (!dtc_matrix_ok(L.gate) || !dtc_matrix_ok(L.up) || !dtc_matrix_ok(L.down) || L.gate.type != L.up.type)
        return false;
    if (p.S > 0 && (!dtc_matrix_ok(L.sh_gate) || !dtc_matrix_ok(L.sh_up) || !dtc_matrix_ok(L.sh_down) ||
                    L.sh_gate.type != L.sh_up.type))
        return false;
    // 16-byte activation copies: rows and scale rows on 16-byte boundaries
    if (p.H % 128 != 0 || p.W % 128 != 0) return false;
    if (p.x_qstride % 16 != 0 || p.x_dstride % 4 != 0) return false;
    if (!aligned16(p.xq) || !aligned16(p.xd) || !aligned16(p.xs) || !aligned16(p.aq) || !aligned16(p.ad) ||
        !aligned16(p.as))
        return false;
    return true;
}

bool decode_tc_down_ok(const FwdParams &p, const LayerDev &L)
{
    return dtc_matrix_ok(L.down) && p.H % 128 == 0 && p.W % 128 == 0 && aligned16(p.aq) && aligned16(p.ad) &&
           aligned16(p.as);
}

cudaError_t launch_decode_tc_down(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                                  cudaStream_t st)
{
    if (!decode_tc_down_ok(p, L)) return cudaErrorInvalidValue;
    return L.down.type == FMT_Q4_K ? launch_dtc<FMT_Q4_K, 1>(p, L, maps, 0, num_sms, st)
                                   : launch_dtc<FMT_Q8_0, 1>(p, L, maps, 0, num_sms, st);
}

cudaError_t launch_decode_tc(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                             const Marker &mk, cudaStream_t st, bool shared_only)
{
    cudaError_t e;
    const bool has_sh = p.S > 0;
    if (shared_only) {
        if (!has_sh) return cudaSuccess;
        if ((e = (L.sh_gate.type == FMT_Q4_K ? launch_dtc<FMT_Q4_K, 2>(p, L, maps, 1, num_sms, st)
                                             : launch_dtc<FMT_Q8_0, 2>(p, L, maps, 1, num_sms, st))) != cudaSuccess)
            return e;
        mk.mark("gate_up_i8_shared");
        if ((e = (L.sh_down.type == FMT_Q4_K ? launch_dtc<FMT_Q4_K, 1>(p, L, maps, 1, num_sms, st)
                                             : launch_dtc<FMT_Q8_0, 1>(p, L, maps, 1, num_sms, st))) != cudaSuccess)
            return e;
        mk.mark("down_i8_shared");
        return cudaSuccess;
    }
    const bool same_gu = has_sh && L.sh_gate.type == L.gate.type;
    const bool same_dn = has_sh && L.sh_down.type == L.down.type;
    auto gu = [&](int mode) {
        const int fmt = mode == 1 ? L.sh_gate.type : L.gate.type;
        return fmt == FMT_Q4_K ? launch_dtc<FMT_Q4_K, 2>(p, L, maps, mode, num_sms, st)
                               : launch_dtc<FMT_Q8_0, 2>(p, L, maps, mode, num_sms, st);
    };
    auto dn = [&](int mode) {
        const int fmt = mode == 1 ? L.sh_down.type : L.down.type;
        return fmt == FMT_Q4_K ? launch_dtc<FMT_Q4_K, 1>(p, L, maps, mode, num_sms, st)
                               : launch_dtc<FMT_Q8_0, 1>(p, L, maps, mode, num_sms, st);
    };
    if ((e = gu(same_gu ? 2 : 0)) != cudaSuccess) return e;
    mk.mark("gate_up_i8");
    if (has_sh && !same_gu) {
        if ((e = gu(1)) != cudaSuccess) return e;
        mk.mark("gate_up_i8_shared");
    }
    if ((e = dn(same_dn ? 2 : 0)) != cudaSuccess) return e;
    mk.mark("down_i8");
    if (has_sh && !same_dn) {
        if ((e = dn(1)) != cudaSuccess) return e;
        mk.mark("down_i8_shared");
    }
    return cudaSuccess;
}

}  // namespace jmoe
