// experts_i8.cu -- the expert FFN of a small batch (decode) as ONE persistent
// launch on the 5th-generation tensor cores with integer operands: gate/up
// with SwiGLU and down, the int32 sum of every 32-value block from tcgen05.mma
// kind::i8, scaled and accumulated in f32 by the epilogue.
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
// the oracle's orc_block_dots.
//
// Issue cost, not tensor throughput, bounds such small MMAs: one thread
// completes about one tcgen05 instruction per 130-250 cycles whatever N is,
// and the lanes of one warp share that rate. So the work per weight value is
// packed into few instructions: a K step is 256 values (a Q4_K super-block),
// and the B operand of a step is block-diagonal -- row (block b, slot j) holds
// slot j's 32 activation bytes of block b and zeros in the other blocks -- so
// the four MMAs (K = 32 each) of a half step accumulate the sums of four
// blocks x four slots in ONE N = 16 accumulator. Four warps issue (matrix x
// half), four MMAs and one commit each per step; the A, B and quant stages of
// a step are released by the epilogue, which sees the step's completion. What
// bounds the launch then is the f32 epilogue (about 300 dependent instructions
// per weight row and step, one warp per SM sub-partition) and, per item, its
// SwiGLU and block quantiser.
//
// Work items (as the f16 fused launch, experts_tc.cu): gate/up = (problem, 128
// rows of the intermediate dim, chunk of up to 4 slots), matrix 0 = gate,
// 1 = up, K = H; down = (problem, 256 output rows, chunk), matrix 0/1 = the
// two 128-row halves, K = I (or S). The gate/up epilogue applies SwiGLU and
// the int8 block quantiser and stores the down operand rows (aq / ad / as);
// the down items of a chunk start once all of its gate/up tiles have counted
// themselves done (bounded wait; all gate/up items precede all down items and
// each CTA takes its items in order).
//
// Operands: A = Q8_0 quants straight from the TMA quant tiles (two 128-row x
// 128-byte tiles per matrix and step, 128-byte swizzle), or Q4_K nibbles
// unpacked to u8 by the unpack warps into TMEM (one weight row per lane, four
// values per column in K order). B = the block-diagonal tiles (two per step,
// 16 rows x 128 bytes, 128-byte swizzle, zero outside the diagonal), filled
// by the act warp with 16-byte cp.async copies that arrive on the stage's
// barrier. Block scales of the slots: copied per item into shared memory by
// the act warp. Weight scales: read by the epilogue from the quant stage's
// 16-byte scale rows.
// Warp roles (448 threads, one CTA per SM; four warps per SM sub-partition
// cap a thread at 128 registers):
//   0       TMA producer of the quant ring
//   1       act: B operand copies, the item's activation block scales, the
//           down items' dependency waits
//   2..5    MMA issue, lane 0 of warp 2 + i: matrix i & 1, blocks
//           4 (i >> 1) .. 4 (i >> 1) + 3 of every step; warp 2 owns the TMEM
//   6..9    unpack (Q4_K) of the warp's TMEM lane quarter, thread = weight
//           row, both matrices
//   10..13  epilogue, thread = weight row = TMEM lane
// Rings: quant stages (TMA -> unpack / MMA / epilogue), A stages in TMEM
// (unpack -> MMA), B stages (act -> MMA), block sums in TMEM (MMA ->
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
constexpr int kYKS = 256;                         // K values per step (eight 32-value blocks)
constexpr int kYCap = 4;                          // slots per item
constexpr int kYN = 16;                           // MMA N: 4 blocks x 4 slots
constexpr int kYTma = 0, kYAct = 1, kYMma0 = 2, kYMmas = 4, kYUnp0 = 6, kYUnps = 4, kYEpi0 = 10, kYEpis = 4;
constexpr int kYThreads = (kYEpi0 + kYEpis) * 32;
constexpr int kYTile = kYM * 128;                 // one 128-row x 128-byte quant tile (16 KB)
constexpr int kYMetaBytes = kYM * 16;             // 16-byte scale row per weight row and step
constexpr int kYBHalf = kYN * 128;                // B tile of a half step (16 rows x 128 bytes)
constexpr int kYBStage = 2 * kYBHalf;
constexpr int kYBst = 6;                          // B ring depth
constexpr int kYMaxQst = 4;
constexpr int kYAccS = 4;                         // block-sum stages in TMEM
constexpr int kYAccCols = 4 * kYN;                // a stage: [matrix][half][16] int32
constexpr int kYA0 = kYAccS * kYAccCols;          // then the A stages (Q4_K)
constexpr int kYAs = 2;                           // A stages: [matrix][64 columns of u8 x 4]
constexpr int kYACols = 128;
constexpr long long kYDepWaitCycles = 4000000000LL;
static_assert(kYA0 + kYAs * kYACols <= 512, "TMEM");

struct YCfg {
    int mode;                // 0 routed problems, 1 shared only, 2 both
    int qst;                 // quant ring depth
    int mstride;             // bytes of one matrix in a quant stage (tiles, then scale rows)
    int max_q;               // capacity of the problem table
    int kb_max;              // largest K / 32 of the launch's matrices (item scale rows)
    int smem_q, smem_b, smem_sc, smem_tab, smem_bar;
};

struct YMaps {
    CUtensorMap gq[2], gm[2];   // routed gate/up: quants (128 x 128 B, swizzle 128B), scales (128 x 16 B)
    CUtensorMap dq, dm;         // routed down
    CUtensorMap sq[2], sm[2];   // shared gate/up
    CUtensorMap sdq, sdm;       // shared down
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

// Offset in a quant stage of matrix m's scale rows: after its tiles (one for
// Q4_K, two for Q8_0).
__device__ __forceinline__ uint32_t y_meta_off(int mstride, int m, bool q4)
{
    return (uint32_t)(m * mstride + (q4 ? 1 : 2) * kYTile);
}

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

struct YEpi {
    uint64_t *q_full, *q_empty, *acc_full, *acc_empty, *b_empty, *a_empty;
    uint32_t sq;
    uint32_t sc;             // shared address of the item's scale buffer
    int kb;                  // K / 32 of the item (scale row length)
    int qst, mstride;
    volatile int *abort_flag;
};

// The K steps of one item for the epilogue: the f32 sums of matrix 0 and 1 for
// row r and the item's slots (a0 / a1; slots >= n hold nothing of use). The
// weight scales come from the quant stage (waited for, then released), the
// slot scales from the item's scale buffer sc: [slot][kb] dx, then [slot][kb] sx.
template <bool DBG>
__device__ __forceinline__ bool epi_steps(const FwdParams &p, const YEpi &e, bool q4, int K, uint32_t tb0, int r,
                                          RingPos &qr, RingPos &cr, RingPos &br, RingPos &ar, float (&a0)[kYCap],
                                          float (&a1)[kYCap], int32_t *dbg, int n)
{
    const int nk = (K + kYKS - 1) / kYKS;
#pragma unroll
    for (int j = 0; j < kYCap; j++) { a0[j] = 0.0f; a1[j] = 0.0f; }
    const uint32_t m0 = y_meta_off(e.mstride, 0, q4), m1 = y_meta_off(e.mstride, 1, q4);
    for (int kk = 0; kk < nk; kk++) {
        if (!ywait_warp(&e.q_full[qr.slot], qr.phase, e.abort_flag, p.err)) return false;
        const uint32_t st = e.sq + (uint32_t)(qr.slot * 2 * e.mstride) + (uint32_t)(r * 16);
        const uint4 meta0 = lds128(st + m0), meta1 = lds128(st + m1);
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
        const int kh = min(2, (K - kk * kYKS) / 128);   // halves in this step (a Q8_0 K may end on one)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (h >= kh) break;
            // the slots' dx (and sx) of blocks 8 kk + 4 h .. + 3: 16 contiguous bytes per slot
            const uint32_t scs = e.sc + 4u * (uint32_t)(8 * kk + 4 * h);
            uint4 dx[kYCap], sx[kYCap];
#pragma unroll
            for (int j = 0; j < kYCap; j++) {
                dx[j] = lds128(scs + 4u * (uint32_t)(j * e.kb));
                sx[j] = q4 ? lds128(scs + 4u * (uint32_t)((kYCap + j) * e.kb)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int m = 0; m < 2; m++) {
                uint32_t S[kYN];   // column 4 b + j: block 4 h + b, slot j
                tmem_ld16(tb + (uint32_t)((2 * m + h) * kYN), S);
                float w[4], mn[4];
                const uint4 &meta = m ? meta1 : meta0;
                if (q4) {
                    q4_scales4(meta, h, w, mn);
                } else {
                    q8_scales4(meta, h, w);
#pragma unroll
                    for (int b = 0; b < 4; b++) mn[b] = 0.0f;
                }
                tmem_ld_wait();
                if (DBG) {   // parity probe: the raw int32 block sums, [slot][matrix][row][block]
#pragma unroll
                    for (int j = 0; j < kYCap; j++)
#pragma unroll
                        for (int b = 0; b < 4; b++)
                            if (j < n)
                                dbg[((size_t)j * 2 + m) * p.I * (size_t)(K >> 5) + 8 * kk + 4 * h + b] =
                                    (int32_t)S[4 * b + j];
                }
#pragma unroll
                for (int j = 0; j < kYCap; j++) {
                    const float dxv[4] = {__uint_as_float(dx[j].x), __uint_as_float(dx[j].y),
                                          __uint_as_float(dx[j].z), __uint_as_float(dx[j].w)};
                    const float sxv[4] = {__uint_as_float(sx[j].x), __uint_as_float(sx[j].y),
                                          __uint_as_float(sx[j].z), __uint_as_float(sx[j].w)};
                    float acc = m ? a1[j] : a0[j];
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        acc = __fmaf_rn(w[b], __fmul_rn(dxv[b], i2f_small((int)S[4 * b + j])), acc);
                        if (q4) acc = __fmaf_rn(-mn[b], sxv[b], acc);
                    }
                    if (m) a1[j] = acc;
                    else a0[j] = acc;
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) {
            mbar_arrive(&e.acc_empty[cr.slot]);
            mbar_arrive(&e.q_empty[qr.slot]);
        }
        cr.advance(kYAccS);
        qr.advance(e.qst);
    }
    return true;
}

// SwiGLU of the item's slots and the int8 block quantiser of the down operand
// (quant_block32's arithmetic), the slots' warp reductions interleaved: the
// warp's 32 lanes are one 32-row block (rows r0 ..) of the intermediate dim.
__device__ __forceinline__ void swiglu_quant_slots(const FwdParams &p, const XItem &x, int r0,
                                                   const float (&g)[kYCap], const float (&u)[kYCap], int lane)
{
    float v[kYCap], am[kYCap];
#pragma unroll
    for (int j = 0; j < kYCap; j++) {
        v[j] = swiglu(g[j], u[j]);
        am[j] = fabsf(v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < kYCap; j++) am[j] = fmaxf(am[j], __shfl_xor_sync(0xffffffffu, am[j], o));
    int q[kYCap], qs[kYCap];
#pragma unroll
    for (int j = 0; j < kYCap; j++) {
        am[j] = fmaxf(am[j], 0.0f);   // all-NaN block -> 0, as the oracle's running max from 0
        const float id = am[j] > 0.0f ? __fdiv_rn(127.0f, am[j]) : 0.0f;
        const float rr = fminf(fmaxf(roundf(__fmul_rn(v[j], id)), -127.0f), 127.0f);
        q[j] = (int)rr;
        qs[j] = q[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < kYCap; j++) qs[j] += __shfl_xor_sync(0xffffffffu, qs[j], o);
    const size_t W = (size_t)p.W;
#pragma unroll
    for (int j = 0; j < kYCap; j++) {
        if (j < x.n) {
            const size_t sl = (size_t)x.slot + j;
            p.aq[sl * W + r0 + lane] = (int8_t)q[j];
            if (lane == 0) {
                const float d = __fdiv_rn(am[j], 127.0f);
                p.ad[sl * (W >> 5) + (r0 >> 5)] = d;
                p.as[sl * (W >> 5) + (r0 >> 5)] = d * (float)qs[j];
            }
        }
    }
}

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

    // the B tiles are zero outside their block diagonals: cleared once here,
    // the act warp only ever writes the diagonals
    for (int i = threadIdx.x; i < kYBst * kYBStage / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(sb)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();

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
            // epilogue warp once the block sums of the step are complete. A B
            // stage fills with one cp.async arrival per act lane.
            for (int i = 0; i < c.qst; i++) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], kYUnps + kYEpis); }
            for (int i = 0; i < kYAs; i++) { mbar_init(&a_full[i], kYUnps); mbar_init(&a_empty[i], 1); }
            for (int i = 0; i < kYBst; i++) { mbar_init(&b_full[i], 32); mbar_init(&b_empty[i], 1); }
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
                const int nks = (M.cols + kYKS - 1) / kYKS;
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
                const int nt = q4 ? 1 : 2;   // 128-byte quant tiles per row and full step
                for (int ks = 0; ks < nks; ks++) {
                    if (!ywait(&q_empty[qr.slot], qr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    // tiles of this step: a Q8_0 K may end on a 128-value half step
                    const int ntk = q4 ? 1 : min(2, (M.cols - ks * kYKS) / 128);
                    uint64_t *bar = &q_full[qr.slot];
                    mbar_arrive_expect_tx(bar, (uint32_t)(2 * (ntk * kYTile + kYMetaBytes)));
                    uint8_t *dst = sq + (size_t)qr.slot * 2 * c.mstride;
                    for (int t = 0; t < ntk; t++) {
                        tma_load_2d(dst + t * kYTile, mq0, 16 * (nt * ks + t), y0, bar);
                        tma_load_2d(dst + c.mstride + t * kYTile, mq1, 16 * (nt * ks + t), y1, bar);
                    }
                    tma_load_2d(dst + nt * kYTile, mm0, 2 * ks, y0, bar);
                    tma_load_2d(dst + c.mstride + nt * kYTile, mm1, 2 * ks, y1, bar);
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
        // this lane's 16 bytes of a half step's B tile: row R = 4 b + j
        // (block b of the half, slot j), unit t of the block's 32 bytes, at
        // its 128-byte-swizzled place
        const int R = lane >> 1, t = lane & 1, bq = R >> 2, jq = R & 3;
        const uint32_t dst_off = (uint32_t)(R * 128 + (((2 * bq + t) ^ (R & 7)) * 16));
        const uint32_t sb0 = smem_addr(sb);
        RingPos br, sr;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const int K = x_mat(L, x).cols, nks = (K + kYKS - 1) / kYKS, kb = K >> 5;
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
            }
            // the item's activation block scales: [slot][kb] dx, then [4 + slot][kb] sx
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
            // B operand: slot jq's int8 row (token row of xq, or slot row of aq)
            const int8_t *row = nullptr;
            if (jq < x.n)
                row = x.phase == 0 ? p.xq + (size_t)p.perm_token[x.slot + jq] * (size_t)p.H
                                   : p.aq + ((size_t)x.slot + jq) * (size_t)p.W;
            for (int ks = 0; ks < nks; ks++) {
                if (!ywait_warp(&b_empty[br.slot], br.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                const uint32_t stage = sb0 + (uint32_t)(br.slot * kYBStage);
                const int kh = min(2, (K - ks * kYKS) / 128);
#pragma unroll
                for (int h = 0; h < 2; h++)
                    if (row && h < kh)
                        cp_async16_s(stage + (uint32_t)(h * kYBHalf) + dst_off,
                                     row + (size_t)ks * kYKS + h * 128 + 32 * bq + 16 * t);
                cp_async_mbar_arrive_noinc(&b_full[br.slot]);
                br.advance(kYBst);
            }
        }
        cp_async_wait<0>();   // no copy outlives the CTA
    } else if (warp < kYUnp0) {
        // MMA issue: lane 0 of warp kYMma0 + i issues matrix i & 1, blocks
        // 4 (i >> 1) .. 4 (i >> 1) + 3 of every step into its own N = 16
        // accumulator, and one commit per step.
        if (lane == 0) {
            const int iss = warp - kYMma0, m_i = iss & 1, h = iss >> 1;
            const uint64_t q_desc0 = umma_desc_sw128(smem_addr(sq)), b_desc0 = umma_desc_sw128(smem_addr(sb));
            RingPos qr, br, ar, cr;
            bool ok = true, issued = false;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
                const DevMatrix &M = x_mat(L, x);
                const bool q4 = M.type == FMT_Q4_K;
                const int nks = (M.cols + kYKS - 1) / kYKS;
                // s32 accumulate; A u8 (Q4_K nibbles) or s8 (Q8_0), B s8; K-major; N = 16, M = 128
                const uint32_t idesc = (2u << 4) | ((q4 ? 0u : 1u) << 7) | (1u << 10) | ((uint32_t)(kYN >> 3) << 17) |
                                       ((uint32_t)(kYM >> 4) << 24);
                for (int ks = 0; ks < nks; ks++) {
                    if ((!q4 && !ywait(&q_full[qr.slot], qr.phase, abort_flag, p.err)) ||
                        !ywait(&acc_empty[cr.slot], cr.phase ^ 1u, abort_flag, p.err) ||
                        !ywait(&b_full[br.slot], br.phase, abort_flag, p.err) ||
                        !ywait(&a_full[ar.slot], ar.phase, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    fence_async_smem();   // the cp.async B rows -> the tensor core's reads
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(cr.slot * kYAccCols + (2 * m_i + h) * kYN);
                    const uint64_t bd = b_desc0 + (uint64_t)((br.slot * kYBStage + h * kYBHalf) >> 4);
                    if (h * 128 >= M.cols - ks * kYKS) {
                        // the step ends before this half (Q8_0): nothing to issue, the commit still counts
                    } else if (q4) {
                        const uint32_t a = tmem + (uint32_t)(kYA0 + ar.slot * kYACols + 64 * m_i + 32 * h);
#pragma unroll
                        for (int b = 0; b < 4; b++) tc_mma_i8_ts(d, a + 8u * b, bd + 2 * b, idesc, b > 0);
                    } else {
                        const uint64_t ad =
                            q_desc0 + (uint64_t)((qr.slot * 2 * c.mstride + m_i * c.mstride + h * kYTile) >> 4);
#pragma unroll
                        for (int b = 0; b < 4; b++) tc_mma_i8(d, ad + 2 * b, bd + 2 * b, idesc, b > 0);
                    }
                    issued = true;
                    tc_commit(&acc_full[cr.slot]);
                    qr.advance(c.qst);
                    br.advance(kYBst);
                    ar.advance(kYAs);
                    cr.advance(kYAccS);
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
        RingPos qr, ar;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const DevMatrix &M = x_mat(L, x);
            const bool q4 = M.type == FMT_Q4_K;
            const int nks = (M.cols + kYKS - 1) / kYKS;
            for (int ks = 0; ks < nks; ks++) {
                if (!ywait_warp(&q_full[qr.slot], qr.phase, abort_flag, p.err)) { ok = false; break; }
                // the A stage is free once the MMAs that read it last are
                // complete. Waited for on every step, Q8_0 ones too, so that
                // the A stage phases never run a lap ahead of the MMA issuers.
                if (!ywait_warp(&a_empty[ar.slot], ar.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                if (q4) {
#pragma unroll
                    for (int m = 0; m < 2; m++) {
#pragma unroll
                        for (int hh = 0; hh < 2; hh++) {
                            uint4 qv[4];
#pragma unroll
                            for (int i = 0; i < 4; i++)   // sub-block 4 hh + i of the 256-value quant row
                                qv[i] = lds128(q_row + (uint32_t)(qr.slot * 2 * c.mstride + m * c.mstride) +
                                               16u * ((uint32_t)(4 * hh + i) ^ swz));
                            uint32_t v[32];
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                const uint4 q = qv[i];
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
                            tmem_st32(arow + (uint32_t)(ar.slot * kYACols + 64 * m + 32 * hh), v);
                        }
                    }
                    tmem_st_wait();
                    tc_fence_before();
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[ar.slot]);
                    mbar_arrive(&q_empty[qr.slot]);   // Q8_0: the epilogue's release follows the MMAs
                }
                ar.advance(kYAs);
                qr.advance(c.qst);
            }
        }
    } else {
        const int wq = warp & 3;
        const YEpi e{q_full, q_empty, acc_full, acc_empty, b_empty, a_empty, smem_addr(sq), 0u, 0, c.qst,
                     c.mstride, abort_flag};
        const uint32_t tb0 = tmem + ((uint32_t)(32 * wq) << 16);
        const int r = 32 * wq + lane;
        RingPos qr, cr, sr, br, ar;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it, kYCap);
            const DevMatrix &M = x_mat(L, x);
            const bool q4 = M.type == FMT_Q4_K;
            if (!ywait_warp(&sc_full[sr.slot], sr.phase, abort_flag, p.err)) break;
            YEpi ei = e;
            ei.sc = smem_addr(ssc + (size_t)sr.slot * sc_stride);
            ei.kb = M.cols >> 5;
            float a0[kYCap], a1[kYCap];
            int32_t *dbg = p.dbg_isum && x.phase == 0 && !x.shared
                               ? p.dbg_isum + ((size_t)x.slot * 2 * p.I + (size_t)x.tile * kYM + r) * (size_t)(M.cols >> 5)
                               : nullptr;
            // the parity probe's stores in their own instance, off the production loop
            const bool ok = dbg ? epi_steps<true>(p, ei, q4, M.cols, tb0, r, qr, cr, br, ar, a0, a1, dbg, x.n)
                                : epi_steps<false>(p, ei, q4, M.cols, tb0, r, qr, cr, br, ar, a0, a1, nullptr, x.n);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sc_empty[sr.slot]);
            sr.advance(2);
            if (!ok) break;
            if (x.phase == 0) {
                // SwiGLU and the int8 block quantiser of the down operand: the
                // warp's 32 lanes are one 32-row block of the intermediate dim
                swiglu_quant_slots(p, x, x.tile * kYM + 32 * wq, a0, a1, lane);
                __syncwarp();
                if (lane == 0) red_release_add(p.dep + x.chunk, 1);
            } else {
                const int f0 = x.tile * 2 * kYM + r;
#pragma unroll
                for (int j = 0; j < kYCap; j++) {
                    if (j < x.n) {
                        float *yr = p.y + y_row(p, (size_t)x.slot + j) * p.H;
                        yr[f0] = a0[j];
                        yr[f0 + kYM] = a1[j];
                    }
                }
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

// Q4_K: whole super-blocks; Q8_0: whole 128-value halves (the last step of
// a K that ends on one has a single half)
bool y_matrix_ok(const DevMatrix &m, int row_tile)
{
    if (m.rows % row_tile != 0 || m.cols < 128) return false;
    return (m.type == FMT_Q4_K && m.cols % kYKS == 0) || (m.type == FMT_Q8_0 && m.cols % 128 == 0);
}

bool y_aligned(const void *ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

bool y_any_q8(const LayerDev &L, bool shared)
{
    bool q8 = L.gate.type == FMT_Q8_0 || L.up.type == FMT_Q8_0 || L.down.type == FMT_Q8_0;
    if (shared) q8 = q8 || L.sh_gate.type == FMT_Q8_0 || L.sh_up.type == FMT_Q8_0 || L.sh_down.type == FMT_Q8_0;
    return q8;
}

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
    // B rows: 16-byte copies out of xq token rows and aq slot rows; block scales as float4 rows
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
    YCfg c{};
    c.mode = mode;
    c.max_q = p.max_problems;
    c.kb_max = (p.H > p.W ? p.H : p.W) / 32;
    // a quant stage holds both matrices: Q8_0 two tiles per row and step, Q4_K one
    c.mstride = (y_any_q8(L, p.S > 0) ? 2 : 1) * kYTile + kYMetaBytes;
    const int tab = (((c.max_q + 4) & ~3) * 3 * 4 + c.max_q * 16 + 15) / 16 * 16;
    const int bar_bytes = (2 * kYMaxQst + 2 * kYAs + 2 * kYBst + 2 * kYAccS + 4 + kYMmas) * 8 + 16;
    const int sc_bytes = 2 * 2 * kYCap * c.kb_max * 4;
    const int fixed = kYBst * kYBStage + sc_bytes + tab + bar_bytes + 1024;   // + alignment slack
    c.qst = kYMaxQst;
    while (c.qst > 2 && (size_t)c.qst * 2 * c.mstride + fixed > 232448) c.qst--;
    c.smem_q = 0;
    c.smem_b = c.smem_q + c.qst * 2 * c.mstride;
    c.smem_sc = c.smem_b + kYBst * kYBStage;
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
