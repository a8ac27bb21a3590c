// prefill.cu -- grouped expert GEMMs on the 5th-generation tensor cores for
// large token counts (tcgen05.mma kind::f16, fp32 accumulators in TMEM).
//
// One work item is (problem, 128 weight rows, chunk of up to 128 / 256 slots).
// The MMA runs with the weights as the M = 128 operand and the expert's token
// slots as N (a multiple of 16 up to the chunk cap), so the tensor work follows
// the expert's real token count instead of padding it to a 128-slot tile:
//   A = weight rows, TMA-loaded as GGUF blocks (Q4_K / Q8_0) in the 128-byte
//       swizzle and expanded to f16 by eight dequant warps;
//   B = the problem's activation slots in f16, TMA-loaded (boxes of 32 rows).
// Both are K-major in the 128-byte swizzle layout. Each aligned group of four
// K positions holds the values (0, 2, 1, 3): that is the order in which the
// dequant warps unpack a 32-bit word of quants, and the activation operands
// are written in the same order, so the dot products are unchanged.
// gate/up items carry two accumulators (gate, up); their epilogue applies
// SwiGLU and the int8 block quantiser of the decode path (so both paths feed
// the down projection the same values) and stores the down operand in f16.
// down items store y in f32. Items are spread over a persistent grid, slot
// chunks innermost so neighbouring CTAs share a weight tile in L2. Every wait
// is bounded.
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

constexpr int kM = 128;                         // weight rows per item (MMA M, TMEM lanes)
constexpr int kKS = 64;                         // K per stage: one 128-byte swizzled row of f16
constexpr int kCapGU = 128, kCapDN = 256;       // slots per item (MMA N) of the gate/up and down launches
constexpr int kXBoxRows = 32, kXBoxBytes = kXBoxRows * 128;
// two MMA-issuing warps: one thread completes about one tcgen05 instruction per
// 130-250 cycles, so gate/up (eight MMAs per K step) issues matrix m from warp
// kWarpMma + m; down items of at most 128 slots split each K step's four MMAs
// over the two (own accumulators, added by the epilogue), larger ones use the first
constexpr int kWarpTma = 0, kWarpMma = 1, kMmaWarps = 2, kDeqWarp0 = 3, kDeqWarps = 8, kEpiWarp0 = 11, kEpiWarps = 4;
constexpr int kTcThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kMaxStages = 6;
constexpr int kTmemCols = 512, kAccCols = 256;  // two accumulator buffers of 256 columns
constexpr int kWTileBytes = kM * 128;           // dequantised weights: one matrix, one K step (16 KB)
constexpr int kQuantBox = kM * 128;             // quants of one matrix per quantised stage (16 KB)
constexpr int kQBytes = kQuantBox + kM * 16;    // + 16 bytes of scales per row (18 KB)

struct TcCfg {
    int mode;                // 0 routed problems, 1 shared only, 2 both
    int cap;                 // slots per item
    int kst, qst;            // ring depths: K steps (activation + dequantised tiles), quantised stages
    int x_bytes;             // bytes of one activation stage (cap rows)
    int max_q;               // capacity of the item table
    int smem_x, smem_w, smem_q, smem_tab, smem_bar;   // region offsets
};

struct TcMaps {
    CUtensorMap a;                        // activations f16 [slots][K], box 64 x 32, swizzle 128B
    CUtensorMap wq[2], wm[2];             // routed weights: quants (swizzle 128B), scales (box 128 rows)
    CUtensorMap sq[2], sm[2];             // shared expert weights
};


// Output position of K index f within its group of four: (0, 2, 1, 3).
__device__ __forceinline__ int k_perm(int f) { return (f & ~3) | ((f & 1) << 1) | ((f >> 1) & 1); }

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }

// 16 values of a Q4_K sub-block word pair are unpacked per 32-bit quant word w
// (bytes b0..b3): halves (b0, b2) and (b1, b3) of the low nibbles, then of the
// high nibbles. 0x6400 | q is the f16 1024 + q; 0x6400 | (q << 4) is 1024 + 16q,
// which (x / 16 - 64) turns into q exactly. Weight = q * dsc - dmn.
__device__ __forceinline__ void q4_word_f16(uint32_t w, __half2 dsc, __half2 ndmn, uint32_t &lo0, uint32_t &lo1,
                                            uint32_t &hi0, uint32_t &hi1)
{
    const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
    const __half2 k16th = __half2half2(__ushort_as_half(0x2C00));   // 1/16
    const __half2 km64 = __half2half2(__ushort_as_half(0xD400));    // -64
    const uint32_t w8 = w >> 8;
    const __half2 l0 = __hsub2(bits_h2((w & 0x000F000Fu) | 0x64006400u), k1024);
    const __half2 l1 = __hsub2(bits_h2((w8 & 0x000F000Fu) | 0x64006400u), k1024);
    const __half2 h0 = __hfma2(bits_h2((w & 0x00F000F0u) | 0x64006400u), k16th, km64);
    const __half2 h1 = __hfma2(bits_h2((w8 & 0x00F000F0u) | 0x64006400u), k16th, km64);
    lo0 = h2_bits(__hfma2(l0, dsc, ndmn));
    lo1 = h2_bits(__hfma2(l1, dsc, ndmn));
    hi0 = h2_bits(__hfma2(h0, dsc, ndmn));
    hi1 = h2_bits(__hfma2(h1, dsc, ndmn));
}

// Four Q8_0 values of word w (signed bytes b0..b3) as halves (b0, b2), (b1, b3):
// (byte ^ 0x80) | 0x6400 is the f16 1024 + 128 + b.
__device__ __forceinline__ void q8_word_f16(uint32_t w, __half2 d, uint32_t &o0, uint32_t &o1)
{
    const __half2 k1152 = __half2half2(__ushort_as_half(0x6480));
    const __half2 e = __hsub2(bits_h2((w & 0x00FF00FFu) ^ 0x64806480u), k1152);
    const __half2 o = __hsub2(bits_h2(((w >> 8) & 0x00FF00FFu) ^ 0x64806480u), k1152);
    o0 = h2_bits(__hmul2(e, d));
    o1 = h2_bits(__hmul2(o, d));
}


template <int FMT, int NMAT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_expert_kernel(FwdParams p, LayerDev L, TcCfg c, const __grid_constant__ TcMaps maps)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment of the operand tiles (swizzle atoms)
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sx = base + c.smem_x, *sw = base + c.smem_w, *sq = base + c.smem_q;
    int *s_off = reinterpret_cast<int *>(base + c.smem_tab);
    int4 *s_prob = reinterpret_cast<int4 *>(s_off + ((c.max_q + 4) & ~3));
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + c.smem_bar);
    // a K-step stage holds one activation tile (TMA, x_full) and the dequantised
    // weight tiles (dequant warps, w_full); one tensor-core commit frees both
    uint64_t *x_full = bars, *w_full = x_full + kMaxStages, *k_empty = w_full + kMaxStages;
    uint64_t *q_full = k_empty + kMaxStages, *q_empty = q_full + kMaxStages;
    uint64_t *acc_full = q_empty + kMaxStages, *acc_empty = acc_full + 2, *drain_bar = acc_empty + 2;   // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int QK = FMT == FMT_Q4_K ? 4 : 2;   // K steps per quantised stage (256 / 128 values)

    // the launch's problems: routed ones, then the shared expert
    const int n_routed = c.mode == 1 ? 0 : *p.n_active;
    const bool with_shared = c.mode != 0 && p.S > 0;
    const int nq = min(n_routed + (with_shared ? 1 : 0), c.max_q);
    const int32_t *tile_off = p.tile_off + (NMAT == 2 ? 0 : 2 * kTileOffStride) + (c.mode == 1 ? kTileOffStride : 0);
    for (int i = threadIdx.x; i <= nq; i += blockDim.x) s_off[i] = tile_off[i];
    for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        const bool sh = i >= n_routed;
        const Problem pr = sh ? p.problems[p.max_problems - 1] : p.problems[i];
        s_prob[i] = make_int4(pr.expert, pr.slot0, pr.count, sh ? 1 : 0);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < c.kst; i++) {
            mbar_init(&x_full[i], 1);
            mbar_init(&w_full[i], kDeqWarps);
            mbar_init(&k_empty[i], kMmaWarps);   // one commit per issuing warp
        }
        for (int i = 0; i < c.qst; i++) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], kDeqWarps); }
        for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], kMmaWarps); mbar_init(&acc_empty[i], kEpiWarps); }
        mbar_init(&drain_bar[0], 1);
        mbar_init(&drain_bar[1], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = nq > 0 ? s_off[nq] : 0;

    if (warp == kWarpTma) {
        if (lane == 0) {
            RingPos kr, qr;
            uint32_t gx = 0, gq = 0;   // uses issued, for the drain after an abort
            bool ok = true;
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(s_off, s_prob, nq, c.cap, it);
                const DevMatrix &M0 = NMAT == 2 ? (x.shared ? L.sh_gate : L.gate) : (x.shared ? L.sh_down : L.down);
                const int nk = M0.cols / kKS;
                const int wy = x.expert * M0.rows + x.nt * kM;
                const int nbox = (x.n + kXBoxRows - 1) / kXBoxRows;
                const CUtensorMap *mq0 = x.shared ? &maps.sq[0] : &maps.wq[0], *mm0 = x.shared ? &maps.sm[0] : &maps.wm[0];
                const CUtensorMap *mq1 = x.shared ? &maps.sq[1] : &maps.wq[1], *mm1 = x.shared ? &maps.sm[1] : &maps.wm[1];
                for (int kk = 0; kk < nk; kk++) {
                    if ((kk & (QK - 1)) == 0) {
                        if (!tc_wait(&q_empty[qr.slot], qr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                        uint64_t *bar = &q_full[qr.slot];
                        mbar_arrive_expect_tx(bar, (uint32_t)(NMAT * kQBytes));
                        uint8_t *dst = sq + (size_t)qr.slot * NMAT * kQBytes;
                        tma_load_2d(dst, mq0, (kk / QK) * 16, wy, bar);
                        tma_load_2d(dst + kQuantBox, mm0, (kk >> 2) * 2, wy, bar);
                        if (NMAT == 2) {
                            tma_load_2d(dst + kQBytes, mq1, (kk / QK) * 16, wy, bar);
                            tma_load_2d(dst + kQBytes + kQuantBox, mm1, (kk >> 2) * 2, wy, bar);
                        }
                        qr.advance(c.qst);
                        gq++;
                    }
                    if (!tc_wait(&k_empty[kr.slot], kr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint64_t *bar = &x_full[kr.slot];
                    mbar_arrive_expect_tx(bar, (uint32_t)(nbox * kXBoxBytes));
                    uint8_t *dst = sx + (size_t)kr.slot * c.x_bytes;
                    for (int b = 0; b < nbox; b++)
                        tma_load_2d(dst + b * kXBoxBytes, &maps.a, kk * kKS, x.slot + b * kXBoxRows, bar);
                    kr.advance(c.kst);
                    gx++;
                }
            }
            if (!ok) {   // wait (bounded) for the copies still in flight
                for (uint32_t g = gx > (uint32_t)c.kst ? gx - c.kst : 0; g < gx; g++)
                    drain_wait(&x_full[g % c.kst], (g / c.kst) & 1);
                for (uint32_t g = gq > (uint32_t)c.qst ? gq - c.qst : 0; g < gq; g++)
                    drain_wait(&q_full[g % c.qst], (g / c.qst) & 1);
            }
        }
    } else if (warp < kWarpMma + kMmaWarps) {
        // issuer mi: gate/up, matrix mi of every K step; down, the 16-value sub-steps
        // 2 mi and 2 mi + 1 of every step into the accumulator at column 128 mi when
        // the item has at most 128 slots, else (mi = 0) all of them. Both issuers
        // wait for every stage and commit every stage and item, so the barrier
        // counts never depend on the item.
        const int mi = warp - kWarpMma;
        if (lane == 0) {
            RingPos kr, ar;
            bool ok = true, issued = false;
            // smem descriptors of stage 0; a stage, matrix or 16-value K step moves the
            // start address field (address / 16) by a constant
            const uint64_t a_desc0 = umma_desc_sw128(smem_addr(sw)), b_desc0 = umma_desc_sw128(smem_addr(sx));
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const TcItem x = tc_item(s_off, s_prob, nq, c.cap, it);
                const int K = NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                        : (x.shared ? L.sh_down.cols : L.down.cols);
                const int nk = K / kKS;
                const uint32_t npad = (uint32_t)((x.n + 15) & ~15);
                // instruction descriptor: f32 accumulate, f16 A and B, both K-major, N = npad, M = 128
                const uint32_t idesc = (1u << 4) | ((npad >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
                if (!tc_wait(&acc_empty[ar.slot], ar.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dbase = tmem + (uint32_t)(ar.slot * kAccCols);
                for (int kk = 0; kk < nk; kk++) {
                    const int st = kr.slot;
                    if (!tc_wait(&x_full[st], kr.phase, abort_flag, p.err) ||
                        !tc_wait(&w_full[st], kr.phase, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bd = b_desc0 + (uint64_t)((st * c.x_bytes) >> 4);
                    if (NMAT == 2) {
                        const uint64_t ad = a_desc0 + (uint64_t)(((st * NMAT + mi) * kWTileBytes) >> 4);
                        const uint32_t d = dbase + (uint32_t)(mi * kCapGU);
#pragma unroll
                        for (int k16 = 0; k16 < kKS / 16; k16++)
                            tc_mma_f16(d, ad + 2 * k16, bd + 2 * k16, idesc, (kk | k16) != 0);
                        issued = true;
                    } else if (npad <= 128) {
                        const uint64_t ad = a_desc0 + (uint64_t)((st * kWTileBytes) >> 4);
                        const uint32_t d = dbase + (uint32_t)(mi * 128);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int k16 = 2 * mi + h;
                            tc_mma_f16(d, ad + 2 * k16, bd + 2 * k16, idesc, (kk | h) != 0);
                        }
                        issued = true;
                    } else if (mi == 0) {
                        const uint64_t ad = a_desc0 + (uint64_t)((st * kWTileBytes) >> 4);
#pragma unroll
                        for (int k16 = 0; k16 < kKS / 16; k16++)
                            tc_mma_f16(dbase, ad + 2 * k16, bd + 2 * k16, idesc, (kk | k16) != 0);
                        issued = true;
                    }
                    tc_commit(&k_empty[st]);
                    kr.advance(c.kst);
                }
                if (!ok) break;
                tc_commit(&acc_full[ar.slot]);
                ar.advance(2);
            }
            if (issued) {   // every MMA of this issuer has completed before the CTA may release TMEM
                tc_commit(&drain_bar[mi]);
                drain_wait(&drain_bar[mi], 0);
            }
        }
    } else if (warp < kEpiWarp0) {
        // dequant warps: thread d owns weight row d % 128 and one 32-value half of each 64-value K step
        const int d = threadIdx.x - kDeqWarp0 * 32, r = d & (kM - 1), hf = d >> 7;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t q_row = smem_addr(sq) + (uint32_t)r * 128, m_row = smem_addr(sq) + kQuantBox + (uint32_t)r * 16;
        const uint32_t w_row = smem_addr(sw) + (uint32_t)r * 128;
        RingPos qr, kr;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const TcItem x = tc_item(s_off, s_prob, nq, c.cap, it);
            const int K = NMAT == 2 ? (x.shared ? L.sh_gate.cols : L.gate.cols)
                                    : (x.shared ? L.sh_down.cols : L.down.cols);
            const int nk = K / kKS;
            for (int kk = 0; kk < nk; kk++) {
                const int qi = kk & (QK - 1), s_q = qr.slot, s_w = kr.slot;
                if (qi == 0 && !tc_wait(&q_full[s_q], qr.phase, abort_flag, p.err)) { ok = false; break; }
                if (!tc_wait(&k_empty[s_w], kr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const uint32_t qb = q_row + (uint32_t)(s_q * NMAT + m) * kQBytes;
                    const uint32_t mb = m_row + (uint32_t)(s_q * NMAT + m) * kQBytes;
                    const uint32_t wb = w_row + (uint32_t)(s_w * NMAT + m) * kWTileBytes;
                    uint4 out[4];
                    if (FMT == FMT_Q4_K) {
                        const int j = 2 * qi + hf;   // sub-block of the super-step = 16-byte chunk of the row
                        const uint4 q = lds128(qb + 16u * ((uint32_t)j ^ swz));
                        const float2 sc = q4_scales(lds128(mb), j);   // (d*sc/16, dmin*m)
                        const __half2 dsc = __float2half2_rn(sc.x * 16.0f), ndmn = __float2half2_rn(-sc.y);
                        q4_word_f16(q.x, dsc, ndmn, out[0].x, out[0].y, out[2].x, out[2].y);
                        q4_word_f16(q.y, dsc, ndmn, out[0].z, out[0].w, out[2].z, out[2].w);
                        q4_word_f16(q.z, dsc, ndmn, out[1].x, out[1].y, out[3].x, out[3].y);
                        q4_word_f16(q.w, dsc, ndmn, out[1].z, out[1].w, out[3].z, out[3].w);
                    } else {
                        const int jb = 2 * qi + hf;   // 32-value block of the 128-value stage
                        const uint4 q0 = lds128(qb + 16u * ((uint32_t)(2 * jb) ^ swz));
                        const uint4 q1 = lds128(qb + 16u * ((uint32_t)(2 * jb + 1) ^ swz));
                        const int blk = 4 * ((kk >> 1) & 1) + jb;   // block of the 256-value scale row
                        const __half2 dd = __half2half2(__ushort_as_half((unsigned short)lds16(mb + 2u * blk)));
                        q8_word_f16(q0.x, dd, out[0].x, out[0].y);
                        q8_word_f16(q0.y, dd, out[0].z, out[0].w);
                        q8_word_f16(q0.z, dd, out[1].x, out[1].y);
                        q8_word_f16(q0.w, dd, out[1].z, out[1].w);
                        q8_word_f16(q1.x, dd, out[2].x, out[2].y);
                        q8_word_f16(q1.y, dd, out[2].z, out[2].w);
                        q8_word_f16(q1.z, dd, out[3].x, out[3].y);
                        q8_word_f16(q1.w, dd, out[3].z, out[3].w);
                    }
#pragma unroll
                    for (int cc = 0; cc < 4; cc++) sts128(wb + 16u * ((uint32_t)(4 * hf + cc) ^ swz), out[cc]);
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&w_full[s_w]);
                kr.advance(c.kst);
                if (qi == QK - 1 || kk == nk - 1) {
                    if (lane == 0) mbar_arrive(&q_empty[s_q]);
                    qr.advance(c.qst);
                }
            }
        }
    } else {
        // epilogue warps: TMEM lane = weight row = output feature, column = slot
        const int wq = warp & 3;
        RingPos ar;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const TcItem x = tc_item(s_off, s_prob, nq, c.cap, it);
            const int buf = ar.slot;
            if (!tc_wait(&acc_full[buf], ar.phase, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            const int f = x.nt * kM + 32 * wq + lane;
            const uint32_t tb = tmem + ((uint32_t)(32 * wq) << 16) + (uint32_t)(buf * kAccCols);
            const int ncc = (x.n + 31) >> 5;
#pragma unroll 1
            for (int cc = 0; cc < ncc; cc++) {
                const int n_here = min(32, x.n - 32 * cc);
                uint32_t g[32];
                tmem_ld32(tb + 32 * cc, g);
                if (NMAT == 2) {
                    uint32_t u[32];
                    tmem_ld32(tb + kCapGU + 32 * cc, u);
                    tmem_ld_wait();
                    // one slot per column; the warp's 32 lanes are one 32-feature quantisation
                    // block, so a column's amax is a warp max; lane i keeps column i's and
                    // computes its scales once, the others read them with a shuffle
                    float a[32];
                    uint32_t own = 0;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        a[i] = swiglu(__uint_as_float(g[i]), __uint_as_float(u[i]));
                        const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(fabsf(a[i]), 0.0f)));
                        own = lane == i ? m : own;
                    }
                    const float amax = __uint_as_float(own);
                    const float id_own = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                    const float dq_own = __fdiv_rn(amax, 127.0f);
                    __half *dst = static_cast<__half *>(p.a16dn) + (size_t)(x.slot + 32 * cc) * p.a16dn_stride + k_perm(f);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float id = __shfl_sync(0xffffffffu, id_own, i);
                        const float dq = __shfl_sync(0xffffffffu, dq_own, i);
                        const float q = fminf(fmaxf(roundf(__fmul_rn(a[i], id)), -127.0f), 127.0f);
                        if (i < n_here) dst[(size_t)i * p.a16dn_stride] = __float2half_rn(q * dq);
                    }
                } else {
                    if (x.n <= 128) {   // two issuers' accumulators: columns c and 128 + c
                        uint32_t g2[32];
                        tmem_ld32(tb + 128 + 32 * cc, g2);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            g[i] = __float_as_uint(__fadd_rn(__uint_as_float(g[i]), __uint_as_float(g2[i])));
                    } else {
                        tmem_ld_wait();
                    }
                    const size_t s0 = (size_t)x.slot + 32 * cc;
                    if (p.y_rows) {   // expert parallel: the output row of each slot is its received row
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (i < n_here) p.y[(size_t)p.y_rows[s0 + i] * p.H + f] = __uint_as_float(g[i]);
                    } else {
                        float *dst = p.y + s0 * p.H + f;
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (i < n_here) dst[(size_t)i * p.H] = __uint_as_float(g[i]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
            ar.advance(2);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// B operand of the gate/up GEMM: slot s holds f16(xq * d) of its token (the
// activation blocks the decode path uses), each group of four values in the
// order (0, 2, 1, 3). One warp per slot row, 16 values per lane: bytes go to
// f32 exactly with a byte permute and one add (2^23 + 128 + q - (2^23 + 128)),
// then f32(q) * d and one f16 rounding per value, as (float)q * d would.
__device__ __forceinline__ float q8_to_f32(uint32_t flipped, int byte_idx)
{
    const uint32_t b = __byte_perm(flipped, 0x4B000000u, 0x7540u | (uint32_t)byte_idx);
    return __int_as_float((int)b) - 8388736.0f;   // 2^23 + 128
}

// perm: slot -> token row, or null for slot s = row s.
__global__ void __launch_bounds__(256) gather_act_f16_kernel(const int32_t *perm, const int8_t *xq, const float *xd,
                                                             int H, __half *a16, int stride, int n_slots)
{
    const int chunks = H >> 4;
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int n_warps = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    for (int s = warp; s < n_slots; s += n_warps) {
        const size_t tok = perm ? (size_t)perm[s] : (size_t)s;
        const int8_t *xr = xq + tok * H;
        const float *dr = xd + tok * (H >> 5);
        __half *dst = a16 + (size_t)s * stride;
        for (int c = lane; c < chunks; c += 32) {
            const uint4 q = *reinterpret_cast<const uint4 *>(xr + 16 * c);
            const float d = dr[c >> 1];
            const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
            uint32_t h[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                h[2 * i] = h2_bits(__floats2half2_rn(q8_to_f32(w[i], 0) * d, q8_to_f32(w[i], 2) * d));
                h[2 * i + 1] = h2_bits(__floats2half2_rn(q8_to_f32(w[i], 1) * d, q8_to_f32(w[i], 3) * d));
            }
            uint4 *o = reinterpret_cast<uint4 *>(dst + 16 * c);
            o[0] = make_uint4(h[0], h[1], h[2], h[3]);
            o[1] = make_uint4(h[4], h[5], h[6], h[7]);
        }
    }
}

// Item offsets of the tensor-core launches (one thread): for each launch
// layout (gate/up routed+shared, gate/up shared only, down routed+shared, down
// shared only) the prefix over problems of slot chunks * 128-row weight tiles.
__global__ void tile_plan_kernel(FwdParams p, int rows_gu, int rows_gu_sh, int rows_dn)
{
    if (threadIdx.x != 0) return;
    const int nr = *p.n_active;
    const int sh_gu = p.S > 0 ? chunk_count(p.T, kCapGU) * (rows_gu_sh / kM) : 0;
    const int sh_dn = p.S > 0 ? chunk_count(p.T, kCapDN) * (rows_dn / kM) : 0;
    int32_t *gu = p.tile_off, *gu_sh = p.tile_off + kTileOffStride;
    int32_t *dn = p.tile_off + 2 * kTileOffStride, *dn_sh = p.tile_off + 3 * kTileOffStride;
    int a = 0, b = 0;
    for (int q = 0; q < nr; q++) {
        gu[q] = a;
        dn[q] = b;
        const int cnt = p.problems[q].count;
        a += chunk_count(cnt, kCapGU) * (rows_gu / kM);
        b += chunk_count(cnt, kCapDN) * (rows_dn / kM);
    }
    gu[nr] = a;
    dn[nr] = b;
    gu[nr + 1] = a + sh_gu;
    dn[nr + 1] = b + sh_dn;
    gu_sh[0] = 0;
    dn_sh[0] = 0;
    gu_sh[1] = sh_gu;
    dn_sh[1] = sh_dn;
}

// One problem of T slots over the rows of a single matrix (the down layout):
// its entry, the active count and its item offsets for slot chunks of cap.
__global__ void dense_plan_kernel(Problem *prob, int32_t *n_active, int32_t *tile_off, int T, int rows, int cap)
{
    prob[0] = Problem{0, 0, T, 0};
    *n_active = 1;
    int32_t *dn = tile_off + 2 * kTileOffStride;
    dn[0] = 0;
    dn[1] = chunk_count(T, cap) * (rows / kM);
    dn[2] = dn[1];
}

// f16 activation operand [rows][cols] with row stride stride_elems: box 64 x 32, 128-byte swizzle.
cudaError_t encode_f16_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint64_t stride_elems)
{
    return encode_tiled(m, 0, base, rows, cols, stride_elems * 2, kKS, kXBoxRows, 1) == 0 ? cudaSuccess
                                                                                          : cudaErrorInvalidValue;
}

// cap > 0 (down only): slot chunks of cap (a multiple of 32) instead of
// kCapDN, and as many K-step stages as the smaller activation tiles leave room for.
template <int FMT, int NMAT>
cudaError_t launch_tc(const FwdParams &p, const LayerDev &L, const LayerMaps &lm, int mode, int num_sms,
                      cudaStream_t st, int cap = 0)
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
    c.mode = mode;
    c.cap = NMAT == 2 ? kCapGU : kCapDN;
    c.x_bytes = c.cap * 128;
    // ring depths by shared-memory room: a K step is 48 KB (gate/up: x 16 + w 32;
    // down: x 32 + w 16), a quantised stage 36 KB (gate/up) or 18 KB (down)
    c.kst = 3;
    c.qst = NMAT == 2 ? 2 : 3;
    if (NMAT == 1 && cap > 0) {
        if (cap % kXBoxRows != 0 || cap > kCapDN) return cudaErrorInvalidValue;
        c.cap = cap;
        c.x_bytes = cap * 128;
        const int room = 200 * 1024 - c.qst * kQBytes;
        c.kst = room / (c.x_bytes + kWTileBytes);
        c.kst = c.kst < 3 ? 3 : (c.kst > kMaxStages ? kMaxStages : c.kst);
    }
    c.max_q = p.max_problems;
    c.smem_x = 0;
    c.smem_w = c.smem_x + c.kst * c.x_bytes;
    c.smem_q = c.smem_w + c.kst * NMAT * kWTileBytes;
    c.smem_tab = c.smem_q + c.qst * NMAT * kQBytes;
    c.smem_bar = c.smem_tab + (((c.max_q + 4) & ~3) * 4 + c.max_q * 16 + 15) / 16 * 16;
    const size_t smem = (size_t)c.smem_bar + (5 * kMaxStages + 6) * 8 + 16 + 1024;   // barriers + alignment slack
    if (smem > 232448) return cudaErrorInvalidValue;
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
    gather_act_f16_kernel<<<num_sms * 8, 256, 0, st>>>(p.perm_token, p.xq, p.xd, p.H, static_cast<__half *>(p.a16),
                                                       p.a16_stride, n_slots);
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

bool dense_f16_ok(const FwdParams &p, const LayerDev &L)
{
    const DevMatrix &m = L.down;
    return (m.type == FMT_Q4_K || m.type == FMT_Q8_0) && m.rows % kM == 0 && m.cols % kKS == 0 && p.H == m.rows &&
           p.W == m.cols && p.a16dn && p.tile_off && p.a16dn_stride % 8 == 0 && p.slots_cap >= p.T;
}

cudaError_t launch_dense_f16(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                             cudaStream_t st)
{
    if (!dense_f16_ok(p, L)) return cudaErrorInvalidValue;
    gather_act_f16_kernel<<<num_sms * 4, 256, 0, st>>>(nullptr, p.xq, p.xd, p.W, static_cast<__half *>(p.a16dn),
                                                       p.a16dn_stride, p.T);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // a few rows (decode batches): chunks of 64 slots, six K-step stages
    const int cap = p.T <= 64 ? 64 : kCapDN;
    dense_plan_kernel<<<1, 1, 0, st>>>(p.problems, p.n_active, p.tile_off, p.T, L.down.rows, cap);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return L.down.type == FMT_Q4_K ? launch_tc<FMT_Q4_K, 1>(p, L, maps, 0, num_sms, st, cap)
                                   : launch_tc<FMT_Q8_0, 1>(p, L, maps, 0, num_sms, st, cap);
}

}  // namespace jmoe
