// experts_tc.cu -- the expert FFN of a small batch (decode) as ONE persistent
// launch on the 5th-generation tensor cores: the gate/up projections with
// SwiGLU and the down projection, with f16 operands and f32 accumulators that
// sum over the whole K in TMEM.
//
// At decode sizes every weight value is used by a handful of tokens, so the
// launch is bound by streaming the expert weights from HBM. Each weight value
// is expanded from its GGUF block (Q4_K or Q8_0, scales folded in) to f16 once,
// straight into TMEM as the A operand (tcgen05.st), and one MMA per 16 K values
// multiplies it with all of the item's tokens. Per weight value that is about
// two instructions of the expansion, against four per value and token pair of
// the int8 dot-product kernels, and no per-block hand-off between the tensor
// cores and the CUDA cores (the block scales are folded into A, so the
// accumulators run over the whole K).
//
// Work items, in one list per launch:
//   gate/up: (problem, 128 rows of the intermediate dim, slot chunk): matrix 0
//            = gate rows, matrix 1 = up rows, K = H; the epilogue applies
//            SwiGLU and the int8 block quantiser of the other paths and stores
//            the quantised values as the f16 down operand rows (a16dn), then
//            counts itself done in the chunk's dependency counter;
//   down:    (problem, 256 output rows, slot chunk): matrix 0/1 = the two 128-row
//            halves, K = I (or S); the act warp starts a down item's operand
//            rows once every gate/up tile of that chunk has counted itself done.
// All gate/up items come before all down items, and each CTA takes its items in
// increasing order, so every item a down item waits for is taken by a CTA that
// never waits first: the wait always ends (and is bounded anyway).
//
// A = weight tile in TMEM: the dequant warps read the TMA-loaded quant tile
//     (128 rows x 128 bytes, 128-byte swizzle) and the 16-byte scale row of
//     each row, and write f16 weights d*sc*q - dmin*m (Q4_K) or d*q (Q8_0),
//     one weight row per TMEM lane. Within each aligned group of four K
//     positions the values sit in the order (0, 2, 1, 3), the order in which a
//     32-bit word of quants unpacks into two f16 pairs.
// B = the item's slot rows in f16 in shared memory (128-byte swizzle, same K
//     order), loaded by the act warp with one TMA box per row and K step from
//     rows that are already f16 in that order: the token rows f16(q * d) of the
//     activation blocks, which the routing kernel writes (x16), and the slot
//     rows of the quantised SwiGLU output (a16dn). These are the operand values
//     of the f16 tensor-core prefill path.
// Warp roles (576 threads, one CTA per SM):
//   0       TMA producer of the quant ring
//   1..4    MMA issue, one thread each: issuer (h, m) = matrix m of the K steps
//           of parity h, into its own accumulator (warp 1 owns the TMEM)
//   5       act: B operand loads and the down items' dependency waits
//   6..13   dequant: warps 6..9 matrix 0, 10..13 matrix 1, thread = weight row
//   14..17  epilogue, thread = TMEM lane = weight row; adds the two parities
// Every wait is bounded; a timeout sets the status word and the CTA drains.
//
// Semantics followed: the per-token expert FFN of dispatch_qwen3_moe_ffn
// (src/qwen_deepseek.rs:847-951, run_single_swiglu_expert :748-771) over GGUF
// Q4_K / Q8_0 weights, with the activation blocks of the other paths.
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

constexpr int kXM = 128;                          // rows of a matrix tile (MMA M, TMEM lanes)
constexpr int kXKS = 64;                          // K values per step (one 128-byte f16 row of B)
constexpr int kXCap = 32;                         // slots per item (MMA N: 16 or 32)
constexpr int kXTma = 0, kXMma0 = 1, kXMmas = 4, kXAct = 5, kXDeq0 = 6, kXDeqs = 8, kXEpi0 = 14, kXEpis = 4;
constexpr int kXThreads = (kXEpi0 + kXEpis) * 32;
constexpr int kXQuantBox = kXM * 128;             // quants of one matrix tile per quant stage (16 KB)
constexpr int kXQBytes = kXQuantBox + kXM * 16;   // + one 16-byte scale row per weight row (18 KB)
constexpr int kXStage = 2 * kXQBytes;             // a quant stage holds both matrices (36 KB)
constexpr int kXBTile = kXCap * 128;              // B operand of one K step
constexpr int kXBst = 16;                         // B ring depth (a power of two)
constexpr int kXMaxQst = 5;
constexpr int kXAccCols = 128;                    // accumulator buffer: issuer (h, m) at column 32 (2 h + m)
constexpr int kXA0 = 2 * kXAccCols;               // two accumulator buffers, then the A stages
constexpr int kXAs = (512 - kXA0) / 64;           // A stages (64 columns: two matrices x 32)
static_assert((kXAs & (kXAs - 1)) == 0 && (kXBst & (kXBst - 1)) == 0, "ring sizes are powers of two");
constexpr long long kXDepWaitCycles = 4000000000LL;
static_assert(kXA0 + kXAs * 64 <= 512, "TMEM");

struct XCfg {
    int mode;                // 0 routed problems, 1 shared only, 2 both
    int qst;                 // quant ring depth
    int max_q;               // capacity of the problem table
    int smem_q, smem_b, smem_tab, smem_bar;
};

struct XMaps {
    CUtensorMap gq[2], gm[2];   // routed gate/up: quants (128 x 128 B, swizzle 128B), scales (128 x 16 B)
    CUtensorMap dq, dm;         // routed down
    CUtensorMap sq[2], sm[2];   // shared gate/up
    CUtensorMap sdq, sdm;       // shared down
    CUtensorMap bx, bd;         // B rows: x16 token rows, a16dn slot rows (box 64 f16 x 1 row, swizzle 128B)
};

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }

// One 32-bit word of a Q4_K sub-block (bytes b0..b3: values b (low nibble)
// and 16 + b (high nibble)) as f16 weights q * dsc + ndmn: lo0 = values
// (b0, b2), lo1 = (b1, b3) of the low nibbles, hi0 / hi1 the same of the high
// nibbles. 0x6400 | q is the f16 1024 + q, exact; 0x6400 | (q << 4) is
// 1024 + 16 q, which x / 16 - 64 turns into q exactly.
__device__ __forceinline__ void q4w(uint32_t w, __half2 dsc, __half2 ndmn, uint32_t &lo0, uint32_t &lo1,
                                    uint32_t &hi0, uint32_t &hi1)
{
    const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
    const __half2 k16th = __half2half2(__ushort_as_half(0x2C00));
    const __half2 km64 = __half2half2(__ushort_as_half(0xD400));
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

// Four Q8_0 values (signed bytes b0..b3) times d as f16 pairs (b0, b2), (b1, b3):
// (byte ^ 0x80) | 0x6400 is the f16 1024 + 128 + b.
__device__ __forceinline__ void q8w(uint32_t w, __half2 d, uint32_t &o0, uint32_t &o1)
{
    const __half2 k1152 = __half2half2(__ushort_as_half(0x6480));
    const __half2 e = __hsub2(bits_h2((w & 0x00FF00FFu) ^ 0x64806480u), k1152);
    const __half2 o = __hsub2(bits_h2(((w >> 8) & 0x00FF00FFu) ^ 0x64806480u), k1152);
    o0 = h2_bits(__hmul2(e, d));
    o1 = h2_bits(__hmul2(o, d));
}

// Every role waits suspended in try_wait (the warp issues nothing until the
// phase completes): spinning waiters measurably took issue slots from the
// dequant warps, which are issue-bound.
template <bool SPIN>
__device__ __forceinline__ bool xwait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
{
    return tc_wait(bar, parity, abort_flag, err);
}

__global__ void __launch_bounds__(kXThreads, 1)
    fused_expert_kernel(FwdParams p, LayerDev L, XCfg c, const __grid_constant__ XMaps maps)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sq = base + c.smem_q, *sb = base + c.smem_b;
    const int tab_n = (c.max_q + 4) & ~3;
    int *s_o0 = reinterpret_cast<int *>(base + c.smem_tab);
    int *s_o1 = s_o0 + tab_n, *s_cb = s_o1 + tab_n;
    int4 *s_prob = reinterpret_cast<int4 *>(s_cb + tab_n);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + c.smem_bar);
    uint64_t *q_full = bars, *q_empty = q_full + kXMaxQst;
    uint64_t *a_full = q_empty + kXMaxQst, *a_empty = a_full + kXAs;
    uint64_t *b_full = a_empty + kXAs, *b_empty = b_full + kXBst;
    uint64_t *acc_full = b_empty + kXBst, *acc_empty = acc_full + 2, *drain_bar = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + kXMmas);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *s_last = reinterpret_cast<int *>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    pdl_wait();   // launched as a dependent: the routing output is complete
    pdl_trigger();

    // the launch's problems (routed ones, then the shared expert), their first
    // items of each phase and their first slot chunks
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
                vc = chunk_count(pr.z, kXCap);
                v0 = vc * ((pr.w ? L.sh_gate.rows : L.gate.rows) / kXM);
                v1 = vc * (p.H / (2 * kXM));
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
            for (int i = 0; i < c.qst; i++) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], kXDeqs); }
            // a step's A and B stages are read by the two issuers of its parity
            for (int i = 0; i < kXAs; i++) { mbar_init(&a_full[i], kXDeqs); mbar_init(&a_empty[i], 2); }
            for (int i = 0; i < kXBst; i++) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 2); }
            for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], kXMmas); mbar_init(&acc_empty[i], kXEpis); }
            for (int i = 0; i < kXMmas; i++) mbar_init(&drain_bar[i], 1);
            *abort_flag = 0;
            fence_barrier_init();
        }
    }
    if (warp == kXMma0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = nq > 0 ? s_o0[nq] + s_o1[nq] : 0;
    // chunk counters beyond the capacity would alias: such a launch does no work
    const bool fits = nq == 0 || s_cb[nq] <= p.dep_cap;
    const int n_items = fits ? total : 0;
    if (!fits && threadIdx.x == 0) atomicExch(p.err, kErrTimeout + 1);

    if (warp == kXTma) {
        if (lane == 0) {
            RingPos qr;
            uint32_t gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it);
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
                    y0 = y1 = x.expert * M.rows + x.tile * kXM;
                } else {
                    mq0 = mq1 = x.shared ? &maps.sdq : &maps.dq;
                    mm0 = mm1 = x.shared ? &maps.sdm : &maps.dm;
                    y0 = x.expert * M.rows + x.tile * 2 * kXM;
                    y1 = y0 + kXM;
                }
                for (int qs = 0; qs < nqs; qs++) {
                    if (!xwait<false>(&q_empty[qr.slot], qr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint64_t *bar = &q_full[qr.slot];
                    mbar_arrive_expect_tx(bar, (uint32_t)kXStage);
                    uint8_t *dst = sq + (size_t)qr.slot * kXStage;
                    const int mx = q4 ? 2 * qs : 2 * (qs >> 1);   // 16-byte scale row of the 256-value group
                    tma_load_2d(dst, mq0, 16 * qs, y0, bar);
                    tma_load_2d(dst + kXQuantBox, mm0, mx, y0, bar);
                    tma_load_2d(dst + kXQBytes, mq1, 16 * qs, y1, bar);
                    tma_load_2d(dst + kXQBytes + kXQuantBox, mm1, mx, y1, bar);
                    qr.advance(c.qst);
                    gq++;
                }
            }
            if (!ok)   // wait (bounded) for the copies still in flight
                for (uint32_t g = gq > (uint32_t)c.qst ? gq - c.qst : 0; g < gq; g++)
                    drain_wait(&q_full[g % c.qst], (g / c.qst) & 1);
        }
    } else if (warp < kXMma0 + kXMmas) {
        // four issuing threads: one tcgen05.mma stream from a single thread
        // completes one instruction per ~130 cycles whatever N is, so issuer
        // (h, m) takes matrix m of the K steps of parity h into its own
        // accumulator, and the epilogue adds the two parities
        if (lane == 0) {
            const int iss = warp - kXMma0, m = iss & 1, h = iss >> 1;
            RingPos cr;
            uint32_t g = 0;   // K steps of the CTA's earlier items (the rings' sequence)
            bool ok = true, issued = false;
            const uint64_t b_desc0 = umma_desc_sw128(smem_addr(sb));
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it);
                const int nk = x_mat(L, x).cols / kXKS;
                const uint32_t npad = x.n <= 16 ? 16u : 32u;
                // f32 accumulate, f16 A and B, both K-major, N = npad, M = 128
                const uint32_t idesc = (1u << 4) | ((npad >> 3) << 17) | ((uint32_t)(kXM >> 4) << 24);
                if (!xwait<false>(&acc_empty[cr.slot], cr.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(cr.slot * kXAccCols + 32 * (2 * h + m));
                for (int kk = h; kk < nk; kk += 2) {
                    const uint32_t st = g + (uint32_t)kk;
                    const int as = (int)(st & (kXAs - 1)), bs = (int)(st & (kXBst - 1));
                    const uint32_t aph = (st / kXAs) & 1u, bph = (st / kXBst) & 1u;
                    if (!xwait<true>(&a_full[as], aph, abort_flag, p.err) ||
                        !xwait<true>(&b_full[bs], bph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bd = b_desc0 + (uint64_t)((bs * kXBTile) >> 4);
                    const uint32_t a0 = tmem + (uint32_t)(kXA0 + as * 64 + 32 * m);
#pragma unroll
                    for (int k16 = 0; k16 < kXKS / 16; k16++)
                        tc_mma_f16_ts(d, a0 + 8u * k16, bd + 2 * k16, idesc, (kk != h || k16 != 0) ? 1u : 0u);
                    issued = true;
                    tc_commit(&a_empty[as]);
                    tc_commit(&b_empty[bs]);
                }
                if (!ok) break;
                tc_commit(&acc_full[cr.slot]);
                g += (uint32_t)nk;
                cr.advance(2);
            }
            if (issued) {   // every MMA has completed before the CTA may release TMEM
                tc_commit(&drain_bar[iss]);
                drain_wait(&drain_bar[iss], 0);
            }
        }
    } else if (warp == kXAct) {
        // B operand: one TMA box per slot row and K step (64 f16 = one 128-byte
        // row, written with the 128-byte swizzle of its row in the stage),
        // completing on the stage's b_full; issued as far ahead as the B ring
        // allows. Lane l loads row l of the item. A down item's loads start
        // once its chunk's gate/up tiles are all done (the wait is bounded).
        const int tiles_gu_r = L.gate.rows / kXM, tiles_gu_s = p.S > 0 ? L.sh_gate.rows / kXM : 0;
        RingPos br;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it);
            const int nk = x_mat(L, x).cols / kXKS;
            if (x.phase == 1) {
                const int need = kXEpis * (x.shared ? tiles_gu_s : tiles_gu_r);
                const long long t0 = clock64();
                while (ld_acquire_gpu(p.dep + x.chunk) < need) {
                    if (*abort_flag) { ok = false; break; }
                    if (clock64() - t0 > kXDepWaitCycles) {
                        *abort_flag = 1;
                        atomicExch(p.err, kErrTimeout);
                        ok = false;
                        break;
                    }
                    __nanosleep(256);
                }
                if (!ok) break;
                fence_proxy_async_global();   // the generic stores seen above -> the TMA reads below
            }
            const CUtensorMap *map = x.phase == 0 ? &maps.bx : &maps.bd;
            const int row = lane < x.n ? (x.phase == 0 ? p.perm_token[x.slot + lane] : x.slot + lane) : 0;
            for (int kk = 0; kk < nk; kk++) {
                // the slot's previous contents have been read by their MMAs
                if (!xwait<true>(&b_empty[br.slot], br.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                if (lane == 0) mbar_arrive_expect_tx(&b_full[br.slot], (uint32_t)(x.n * 128));
                __syncwarp();
                if (lane < x.n)
                    tma_load_2d(sb + (size_t)br.slot * kXBTile + lane * 128, map, kk * kXKS, row, &b_full[br.slot]);
                br.advance(kXBst);
            }
        }
        if (!ok && lane == 0) {   // wait (bounded) for the loads still in flight
            for (int i = 0; i < kXBst; i++) {
                drain_wait(&b_full[br.slot], br.phase ^ 1u);
                br.advance(kXBst);
            }
        }
    } else if (warp < kXEpi0) {
        // dequant: thread = (matrix m, weight row r = its TMEM lane)
        const int m = (warp - kXDeq0) >> 2;
        const int r = 32 * (warp & 3) + lane;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t q_row = smem_addr(sq) + (uint32_t)(m * kXQBytes + r * 128);
        const uint32_t m_row = smem_addr(sq) + (uint32_t)(m * kXQBytes + kXQuantBox + r * 16);
        const uint32_t arow = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(kXA0 + 32 * m);
        RingPos qr, ar;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it);
            const DevMatrix &M = x_mat(L, x);
            const bool q4 = M.type == FMT_Q4_K;
            const int nqs = M.cols / (q4 ? 256 : 128);
            for (int qs = 0; qs < nqs && ok; qs++) {
                if (!xwait<true>(&q_full[qr.slot], qr.phase, abort_flag, p.err)) { ok = false; break; }
                const uint32_t qb = q_row + (uint32_t)(qr.slot * kXStage);
                const uint4 meta = lds128(m_row + (uint32_t)(qr.slot * kXStage));
                if (q4) {
                    float s8[8], m8[8];
                    q4_scales_all(meta, s8, m8);
#pragma unroll
                    for (int kq = 0; kq < 4; kq++) {
                        // expand first, then wait for the A stage: the expansion
                        // overlaps the MMAs that still read the stage
                        uint32_t v[32];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int j = 2 * kq + h;   // sub-block = 16-byte chunk of the quant row
                            const uint4 q = lds128(qb + 16u * ((uint32_t)j ^ swz));
                            const __half2 dsc = __float2half2_rn(s8[j]), ndmn = __float2half2_rn(-m8[j]);
                            uint32_t *o = v + 16 * h;
                            q4w(q.x, dsc, ndmn, o[0], o[1], o[8], o[9]);
                            q4w(q.y, dsc, ndmn, o[2], o[3], o[10], o[11]);
                            q4w(q.z, dsc, ndmn, o[4], o[5], o[12], o[13]);
                            q4w(q.w, dsc, ndmn, o[6], o[7], o[14], o[15]);
                        }
                        if (!xwait<true>(&a_empty[ar.slot], ar.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();   // the MMAs that read this A stage have completed
                        tmem_st32(arow + (uint32_t)(ar.slot * 64), v);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[ar.slot]);
                        ar.advance(kXAs);
                    }
                } else {
                    // the 16-byte scale row covers 256 values: this stage is half (qs & 1) of it
                    const uint32_t dw[2] = {(qs & 1) ? meta.z : meta.x, (qs & 1) ? meta.w : meta.y};
#pragma unroll
                    for (int kq = 0; kq < 2; kq++) {
                        uint32_t v[32];
                        const uint32_t dpair = dw[kq];   // f16 d of blocks 2 kq, 2 kq + 1 of the stage
                        const __half2 d0 = __low2half2(bits_h2(dpair)), d1 = __high2half2(bits_h2(dpair));
#pragma unroll
                        for (int cc = 0; cc < 4; cc++) {   // 16-byte chunk 4 kq + cc: values 16 cc .. of the step
                            const uint4 q = lds128(qb + 16u * ((uint32_t)(4 * kq + cc) ^ swz));
                            const __half2 d = cc < 2 ? d0 : d1;
                            q8w(q.x, d, v[8 * cc + 0], v[8 * cc + 1]);
                            q8w(q.y, d, v[8 * cc + 2], v[8 * cc + 3]);
                            q8w(q.z, d, v[8 * cc + 4], v[8 * cc + 5]);
                            q8w(q.w, d, v[8 * cc + 6], v[8 * cc + 7]);
                        }
                        if (!xwait<true>(&a_empty[ar.slot], ar.phase ^ 1u, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                        tmem_st32(arow + (uint32_t)(ar.slot * 64), v);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[ar.slot]);
                        ar.advance(kXAs);
                    }
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&q_empty[qr.slot]);
                qr.advance(c.qst);
            }
        }
    } else {
        // epilogue: thread = TMEM lane = weight row of the tile
        const int wq = warp & 3;
        RingPos cr;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const XItem x = x_item(s_o0, s_o1, s_cb, s_prob, nq, it);
            if (!xwait<false>(&acc_full[cr.slot], cr.phase, abort_flag, p.err)) break;
            tc_fence_after();
            const uint32_t tb = tmem + ((uint32_t)(32 * wq) << 16) + (uint32_t)(cr.slot * kXAccCols);
            // matrix m = columns [32 m, 32 m + 32) (parity 0) + [64 + 32 m, ...)
            // (parity 1); slots in halves of 16 columns, each finished before the
            // next is loaded; the buffer is released after the last half
            const int pos = x.tile * kXM + 32 * wq + ((lane & ~3) | ((lane & 1) << 1) | ((lane >> 1) & 1));
            const int f0 = x.tile * 2 * kXM + 32 * wq + lane;
            for (int hf = 0; hf < 2 && 16 * hf < x.n; hf++) {
                uint32_t a0[16], a1[16], b0[16], b1[16];
                tmem_ld16(tb + 16 * hf, a0);
                tmem_ld16(tb + 64 + 16 * hf, a1);
                tmem_ld16(tb + 32 + 16 * hf, b0);
                tmem_ld16(tb + 96 + 16 * hf, b1);
                tmem_ld_wait();
                const int n_here = min(16, x.n - 16 * hf);
                const size_t s0 = (size_t)x.slot + 16 * hf;
                if (x.phase == 0) {
                    // SwiGLU, then the int8 block quantiser (the values of
                    // quant_block32; the warp's 32 lanes are one 32-row block of
                    // the intermediate dim), stored as the f16 down operand
                    // f16(q * d) in the order (0, 2, 1, 3)
                    __half *dst = static_cast<__half *>(p.a16dn) + s0 * p.a16dn_stride + pos;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (j < n_here) {
                            const float gv = __fadd_rn(__uint_as_float(a0[j]), __uint_as_float(a1[j]));
                            const float uv = __fadd_rn(__uint_as_float(b0[j]), __uint_as_float(b1[j]));
                            const float a = swiglu(gv, uv);
                            const float amax = fmaxf(warp_max(fabsf(a)), 0.0f);
                            const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                            const float q = fminf(fmaxf(roundf(__fmul_rn(a, id)), -127.0f), 127.0f);
                            dst[(size_t)j * p.a16dn_stride] = __float2half_rn(q * __fdiv_rn(amax, 127.0f));
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (j < n_here) {
                            float *yr = y_dst(p, s0 + j);
                            yr[f0] = __fadd_rn(__uint_as_float(a0[j]), __uint_as_float(a1[j]));
                            yr[f0 + kXM] = __fadd_rn(__uint_as_float(b0[j]), __uint_as_float(b1[j]));
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[cr.slot]);
            cr.advance(2);
            if (x.phase == 0) {
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(p.dep + x.chunk, 1);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kXMma0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    // the last CTA returns the chunk counters and the ticket to zero (and,
    // returning rows over peer memory, raises the output flags once every
    // CTA's stores are fenced at system scope)
    if (threadIdx.x == 0) {
        if (p.y_peer) __threadfence_system();
        else __threadfence();
        *s_last = atomicAdd(p.dep_done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (*s_last) {
        __threadfence();
        const int n = min(nq > 0 ? s_cb[nq] : 0, p.dep_cap);
        for (int i = threadIdx.x; i < n; i += blockDim.x) p.dep[i] = 0;
        if (threadIdx.x == 0) *p.dep_done = 0;
        if (p.y_peer && threadIdx.x < p.y_world && *p.y_ok) {
            __threadfence_system();
            uint32_t *flag = reinterpret_cast<uint32_t *>(p.y_peer[threadIdx.x] + p.y_flag_off);
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(p.y_epoch) : "memory");
        }
    }
}

bool x_matrix_ok(const DevMatrix &m, int row_tile)
{
    return (m.type == FMT_Q4_K || m.type == FMT_Q8_0) && m.rows % row_tile == 0 &&
           m.cols % (m.type == FMT_Q4_K ? 256 : 128) == 0 && m.cols >= 128;
}

bool x_aligned(const void *ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace

bool fused_experts_ok(const FwdParams &p, const LayerDev &L)
{
    if (!x_matrix_ok(L.gate, kXM) || !x_matrix_ok(L.up, kXM) || !x_matrix_ok(L.down, 2 * kXM)) return false;
    if (L.gate.type != L.up.type || L.gate.rows != L.up.rows) return false;
    if (p.S > 0 && (!x_matrix_ok(L.sh_gate, kXM) || !x_matrix_ok(L.sh_up, kXM) || !x_matrix_ok(L.sh_down, 2 * kXM) ||
                    L.sh_gate.type != L.sh_up.type))
        return false;
    if (!p.dep || !p.dep_done || p.dep_cap <= 0) return false;
    // B rows: token rows of x16 and slot rows of a16dn, copied in 16-byte chunks
    if (!p.x16 || !p.a16dn || p.x_qstride != 0 || p.y_rows) return false;
    if (p.H % 64 != 0 || p.a16dn_stride % 8 != 0 || p.a16dn_stride < p.W) return false;
    if (!x_aligned(p.x16, 16) || !x_aligned(p.a16dn, 16)) return false;
    return true;
}

cudaError_t launch_fused_experts(const FwdParams &p, const LayerDev &L, const LayerMaps &lm, int mode, int num_sms,
                                 cudaStream_t st)
{
    XMaps maps;
    maps.gq[0] = lm.gate_tc.qs; maps.gm[0] = lm.gate_tc.meta;
    maps.gq[1] = lm.up_tc.qs; maps.gm[1] = lm.up_tc.meta;
    maps.dq = lm.down_tc.qs; maps.dm = lm.down_tc.meta;
    maps.sq[0] = lm.sh_gate_tc.qs; maps.sm[0] = lm.sh_gate_tc.meta;
    maps.sq[1] = lm.sh_up_tc.qs; maps.sm[1] = lm.sh_up_tc.meta;
    maps.sdq = lm.sh_down_tc.qs; maps.sdm = lm.sh_down_tc.meta;
    const int tx = p.T, sx = p.T * p.k + (p.S > 0 ? p.T : 0);
    if (encode_tiled(&maps.bx, 0, p.x16, (uint64_t)tx, (uint64_t)p.H, (uint64_t)p.H * 2, kXKS, 1, 1) != 0 ||
        encode_tiled(&maps.bd, 0, p.a16dn, (uint64_t)sx, (uint64_t)p.W, (uint64_t)p.a16dn_stride * 2, kXKS, 1, 1) != 0)
        return cudaErrorInvalidValue;
    XCfg c{};
    c.mode = mode;
    c.max_q = p.max_problems;
    const int tab = (((c.max_q + 4) & ~3) * 3 * 4 + c.max_q * 16 + 15) / 16 * 16;
    const int bar_bytes = (2 * kXMaxQst + 2 * kXAs + 2 * kXBst + 4 + kXMmas) * 8 + 16;
    const int fixed = kXBst * kXBTile + tab + bar_bytes + 1024;   // + alignment slack
    c.qst = kXMaxQst;
    while (c.qst > 2 && (size_t)c.qst * kXStage + fixed > 232448) c.qst--;
    c.smem_q = 0;
    c.smem_b = c.smem_q + c.qst * kXStage;
    c.smem_tab = c.smem_b + kXBst * kXBTile;
    c.smem_bar = c.smem_tab + tab;
    const size_t smem = (size_t)c.smem_bar + bar_bytes + 1024;
    if (smem > 232448) return cudaErrorInvalidValue;
    static int opted[64];
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || opted[dev] < (int)smem) {
        e = cudaFuncSetAttribute(fused_expert_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) opted[dev] = (int)smem;
    }
    return launch_dependent(fused_expert_kernel, dim3(num_sms), dim3(kXThreads), smem, st, p, L, c, maps);
}

}  // namespace jmoe
