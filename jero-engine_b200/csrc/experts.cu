// experts.cu -- grouped SwiGLU experts over quantised weights and the combine.
//
// Quantised experts run as weight-streaming kernels: the HBM traffic of a
// decode-sized MoE layer is the weight rows of the routed experts, read once.
// Each CTA owns a contiguous range of work items (problem, 32- or 64-row tile);
// a producer warp streams the tiles' weight chunks into a shared-memory ring
// with bulk async copies (cp.async.bulk, completion on mbarriers) while eight
// consumer warps dot them against the problem's int8 activation blocks, which
// sit in shared memory. The copy stream does not stop between work items.
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
constexpr int kGuChunkRows = 8, kGuItemRows = 32;    // gate/up: one warp per row, 32 lanes
constexpr int kDnChunkRows = 16, kDnItemRows = 64;   // down: two rows per warp, 16 lanes each
constexpr long long kWaitCycles = 4000000000LL;      // ~2 s: a wait that long means a fault
constexpr int kRingBudget = 80 * 1024;
constexpr int kErrTimeout = 1;

// Bounded mbarrier wait: gives up (and flags the CTA and the forward) after
// kWaitCycles or when another thread of the CTA gave up.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err)
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

struct Item {
    Problem pr;
    bool shared;
    int rt;
};

__device__ __forceinline__ Item item_at(const FwdParams &p, const StreamCfg &c, int nr, int it)
{
    Item x;
    if (it < nr * c.rt_routed) {
        x.pr = p.problems[it / c.rt_routed];
        x.rt = it % c.rt_routed;
        x.shared = false;
    } else {
        x.pr = p.problems[p.max_problems - 1];
        x.rt = it - nr * c.rt_routed;
        x.shared = true;
    }
    return x;
}

struct Smem {
    uint8_t *ring;
    int8_t *xq;
    float *xd, *xs, *g, *u;
    uint64_t *full, *empty;
    volatile int *abort_flag;
};

__host__ __device__ inline size_t smem_bytes(const StreamCfg &c)
{
    return (size_t)c.stages * c.stage_bytes + (size_t)kTT * c.act_k + 2 * (size_t)kTT * (c.act_k / 32) * 4 +
           2 * (size_t)kTT * 32 * 4 + 16 * (size_t)c.stages + 16;
}

__device__ __forceinline__ Smem carve(uint8_t *base, const StreamCfg &c)
{
    Smem s;
    s.ring = base;
    s.xq = reinterpret_cast<int8_t *>(base + (size_t)c.stages * c.stage_bytes);
    s.xd = reinterpret_cast<float *>(s.xq + (size_t)kTT * c.act_k);
    s.xs = s.xd + kTT * (c.act_k / 32);
    s.g = s.xs + kTT * (c.act_k / 32);
    s.u = s.g + kTT * 32;
    s.full = reinterpret_cast<uint64_t *>(s.u + kTT * 32);
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
        while (!mbar_try_wait(&s.full[k % stages], (k / stages) & 1))
            if (clock64() - t0 > kWaitCycles) break;
    }
}

// Activation blocks of nt rows into shared memory: q [kTT][K] int8 and the
// per-block scale d and d*sum(q). Rows come from perm (token ids) or are
// consecutive slots starting at row0.
__device__ __forceinline__ void stage_act(const Smem &s, const int8_t *gq, const float *gd, const float *gs,
                                          size_t q_stride, size_t d_stride, const int32_t *perm, int row0, int nt,
                                          int K)
{
    const int nv = K >> 4, nb = K >> 5;
    for (int v = threadIdx.x; v < nt * nv; v += kConsumers) {
        const int i = v / nv, c = v % nv;
        const size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        reinterpret_cast<uint4 *>(s.xq + (size_t)i * K)[c] = __ldg(reinterpret_cast<const uint4 *>(gq + row * q_stride) + c);
    }
    for (int v = threadIdx.x; v < nt * nb; v += kConsumers) {
        const int i = v / nb, c = v % nb;
        const size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        s.xd[i * nb + c] = __ldg(gd + row * d_stride + c);
        s.xs[i * nb + c] = __ldg(gs + row * d_stride + c);
    }
}

// ---------------------------------------------------------------- gate/up

template <int FMT>
__global__ void __launch_bounds__(kStreamThreads, 2) gate_up_stream_kernel(FwdParams p, LayerDev L, StreamCfg c)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, c);
    const int S = c.stages;
    init_ring(s, S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nr = c.mode == 1 ? 0 : *p.n_active;
    const int total = nr * c.rt_routed + ((c.mode != 0 && p.S > 0) ? c.rt_shared : 0);
    const int it0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int it1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    constexpr int CR = kGuChunkRows, IR = kGuItemRows;

    if (warp == kConsumerWarps) {   // producer
        if (lane != 0) return;
        uint32_t g = 0;
        for (int it = it0; it < it1; it++) {
            const Item x = item_at(p, c, nr, it);
            const DevMatrix &G = x.shared ? L.sh_gate : L.gate;
            const DevMatrix &U = x.shared ? L.sh_up : L.up;
            const size_t qsr = G.qs_rstride, mr = G.meta_rstride;
            const uint8_t *gq = G.qs + (size_t)x.pr.expert * G.qs_estride;
            const uint8_t *gm = G.meta + (size_t)x.pr.expert * G.meta_estride;
            const uint8_t *uq = U.qs + (size_t)x.pr.expert * U.qs_estride;
            const uint8_t *um = U.meta + (size_t)x.pr.expert * U.meta_estride;
            const int r0 = x.rt * IR, nrow = min(IR, G.rows - r0), nch = (nrow + CR - 1) / CR;
            const int tiles = (x.pr.count + kTT - 1) / kTT;
            for (int tt = 0; tt < tiles; tt++) {
                for (int ch = 0; ch < nch; ch++) {
                    const int st = g % S;
                    const uint32_t use = g / S;
                    if (use > 0 && !wait_bar(&s.empty[st], (use - 1) & 1, s.abort_flag, p.err)) {
                        drain(s, S, g);
                        return;
                    }
                    const size_t rr = (size_t)r0 + ch * CR;
                    const uint32_t qb = (uint32_t)(CR * qsr), mb = (uint32_t)(CR * mr);
                    uint8_t *dst = s.ring + (size_t)st * c.stage_bytes;
                    mbar_arrive_expect_tx(&s.full[st], 2 * (qb + mb));
                    bulk_g2s(dst, gq + rr * qsr, qb, &s.full[st]);
                    bulk_g2s(dst + qb, gm + rr * mr, mb, &s.full[st]);
                    bulk_g2s(dst + qb + mb, uq + rr * qsr, qb, &s.full[st]);
                    bulk_g2s(dst + 2 * qb + mb, um + rr * mr, mb, &s.full[st]);
                    g++;
                }
            }
        }
        return;
    }

    // consumers
    uint32_t g = 0;
    int staged_slot = -1, staged_tile = -1;
    const int H = p.H;
    for (int it = it0; it < it1; it++) {
        const Item x = item_at(p, c, nr, it);
        const DevMatrix &G = x.shared ? L.sh_gate : L.gate;
        const int K = G.cols, NU = K >> 5;
        const size_t qsr = G.qs_rstride, mr = G.meta_rstride;
        const int r0 = x.rt * IR, nrow = min(IR, G.rows - r0), nch = (nrow + CR - 1) / CR;
        const int tiles = (x.pr.count + kTT - 1) / kTT;
        const int down_f32 = c.down_f32;
        for (int tt = 0; tt < tiles; tt++) {
            const int t0 = tt * kTT, nt = min(kTT, x.pr.count - t0);
            if (staged_slot != x.pr.slot0 || staged_tile != tt) {
                named_bar(1, kConsumers);
                stage_act(s, p.xq, p.xd, p.xs, (size_t)H, (size_t)(H >> 5), p.perm_token, x.pr.slot0 + t0, nt, K);
                named_bar(1, kConsumers);
                staged_slot = x.pr.slot0;
                staged_tile = tt;
            }
            for (int ch = 0; ch < nch; ch++) {
                const int st = g % S;
                if (!wait_bar(&s.full[st], (g / S) & 1, s.abort_flag, p.err)) return;
                const uint8_t *base = s.ring + (size_t)st * c.stage_bytes;
                const int rl = ch * CR + warp;
                float ag[kTT], au[kTT];
#pragma unroll
                for (int t = 0; t < kTT; t++) { ag[t] = 0.0f; au[t] = 0.0f; }
                if (rl < nrow) {
                    const size_t qb = CR * qsr, mb = CR * mr;
                    const uint8_t *gqr = base + warp * qsr, *gmr = base + qb + warp * mr;
                    const uint8_t *uqr = base + qb + mb + warp * qsr, *umr = base + 2 * qb + mb + warp * mr;
                    for (int u = lane; u < NU; u += 32) {
                        WUnit<FMT> wg, wu;
                        wg.load(gqr, gmr, u);
                        wu.load(uqr, umr, u);
#pragma unroll
                        for (int t = 0; t < kTT; t++) {
                            if (t < nt) {
                                const int8_t *xq = s.xq + (size_t)t * K + 32 * u;
                                const float xd = s.xd[t * NU + u], xs = s.xs[t * NU + u];
                                ag[t] += wg.dot(xq, xd, xs);
                                au[t] += wu.dot(xq, xd, xs);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.empty[st]);
                g++;
#pragma unroll
                for (int t = 0; t < kTT; t++) {
                    float a = ag[t], b = au[t];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        a += __shfl_xor_sync(0xffffffffu, a, o);
                        b += __shfl_xor_sync(0xffffffffu, b, o);
                    }
                    if (lane == 0 && t < nt && rl < nrow) {
                        s.g[t * 32 + rl] = a;
                        s.u[t * 32 + rl] = b;
                    }
                }
            }
            named_bar(1, kConsumers);
            if (warp < nt) {
                const size_t slot = (size_t)x.pr.slot0 + t0 + warp;
                const float a = lane < nrow ? swiglu(s.g[warp * 32 + lane], s.u[warp * 32 + lane]) : 0.0f;
                if (down_f32) {
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

// ------------------------------------------------------------------- down

template <int FMT>
__global__ void __launch_bounds__(kStreamThreads, 2) down_stream_kernel(FwdParams p, LayerDev L, StreamCfg c)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, c);
    const int S = c.stages;
    init_ring(s, S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nr = c.mode == 1 ? 0 : *p.n_active;
    const int total = nr * c.rt_routed + ((c.mode != 0 && p.S > 0) ? c.rt_shared : 0);
    const int it0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int it1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    constexpr int CR = kDnChunkRows, IR = kDnItemRows;

    if (warp == kConsumerWarps) {
        if (lane != 0) return;
        uint32_t g = 0;
        for (int it = it0; it < it1; it++) {
            const Item x = item_at(p, c, nr, it);
            const DevMatrix &D = x.shared ? L.sh_down : L.down;
            const size_t qsr = D.qs_rstride, mr = D.meta_rstride;
            const uint8_t *dq = D.qs + (size_t)x.pr.expert * D.qs_estride;
            const uint8_t *dm = D.meta + (size_t)x.pr.expert * D.meta_estride;
            const int r0 = x.rt * IR, nrow = min(IR, D.rows - r0), nch = (nrow + CR - 1) / CR;
            const int tiles = (x.pr.count + kTT - 1) / kTT;
            for (int tt = 0; tt < tiles; tt++) {
                for (int ch = 0; ch < nch; ch++) {
                    const int st = g % S;
                    const uint32_t use = g / S;
                    if (use > 0 && !wait_bar(&s.empty[st], (use - 1) & 1, s.abort_flag, p.err)) {
                        drain(s, S, g);
                        return;
                    }
                    const size_t rr = (size_t)r0 + ch * CR;
                    const uint32_t qb = (uint32_t)(CR * qsr), mb = (uint32_t)(CR * mr);
                    uint8_t *dst = s.ring + (size_t)st * c.stage_bytes;
                    mbar_arrive_expect_tx(&s.full[st], qb + mb);
                    bulk_g2s(dst, dq + rr * qsr, qb, &s.full[st]);
                    bulk_g2s(dst + qb, dm + rr * mr, mb, &s.full[st]);
                    g++;
                }
            }
        }
        return;
    }

    uint32_t g = 0;
    int staged_slot = -1, staged_tile = -1;
    const int half = lane >> 4, hl = lane & 15;
    for (int it = it0; it < it1; it++) {
        const Item x = item_at(p, c, nr, it);
        const DevMatrix &D = x.shared ? L.sh_down : L.down;
        const int K = D.cols, NU = K >> 5;
        const size_t qsr = D.qs_rstride, mr = D.meta_rstride;
        const int r0 = x.rt * IR, nrow = min(IR, D.rows - r0), nch = (nrow + CR - 1) / CR;
        const int tiles = (x.pr.count + kTT - 1) / kTT;
        for (int tt = 0; tt < tiles; tt++) {
            const int t0 = tt * kTT, nt = min(kTT, x.pr.count - t0);
            if (staged_slot != x.pr.slot0 || staged_tile != tt) {
                named_bar(1, kConsumers);
                stage_act(s, p.aq, p.ad, p.as, (size_t)p.W, (size_t)(p.W >> 5), nullptr, x.pr.slot0 + t0, nt, K);
                named_bar(1, kConsumers);
                staged_slot = x.pr.slot0;
                staged_tile = tt;
            }
            for (int ch = 0; ch < nch; ch++) {
                const int st = g % S;
                if (!wait_bar(&s.full[st], (g / S) & 1, s.abort_flag, p.err)) return;
                const uint8_t *base = s.ring + (size_t)st * c.stage_bytes;
                const int rw = 2 * warp + half;        // row within the chunk
                const int rl = ch * CR + rw;           // row within the item
                float acc[kTT];
#pragma unroll
                for (int t = 0; t < kTT; t++) acc[t] = 0.0f;
                if (rl < nrow) {
                    const uint8_t *qr = base + rw * qsr, *mrow = base + CR * qsr + rw * mr;
                    for (int u = hl; u < NU; u += 16) {
                        WUnit<FMT> w;
                        w.load(qr, mrow, u);
#pragma unroll
                        for (int t = 0; t < kTT; t++)
                            if (t < nt) acc[t] += w.dot(s.xq + (size_t)t * K + 32 * u, s.xd[t * NU + u], s.xs[t * NU + u]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.empty[st]);
                g++;
#pragma unroll
                for (int t = 0; t < kTT; t++) {
                    float v = acc[t];
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (hl == 0 && t < nt && rl < nrow)
                        p.y[((size_t)x.pr.slot0 + t0 + t) * p.H + r0 + rl] = v;
                }
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
        if (l8 == 0 && row < rows) p.y[slot * p.H + row] = v;
    }
}

// ---------------------------------------------------------------- combine

// out[t] = 0 + shared(x_t), then += w_r * y_r in rank order, each step a
// separately rounded multiply and add (src/qwen_deepseek.rs:858-938).
__global__ void __launch_bounds__(256) combine_kernel(FwdParams p)
{
    __shared__ long long s_pos[kMaxK];
    __shared__ float s_w[kMaxK];
    const int t = blockIdx.y, k = p.k, mw = p.mask_words;
    if (threadIdx.x < k) {
        const int r = threadIdx.x;
        const int e = p.sel_idx[(size_t)t * k + r];
        long long pos = -1;
        if (e >= 0) {
            const uint32_t m = p.mask[(size_t)e * mw + (t >> 5)];
            pos = p.offsets[e] + p.wprefix[(size_t)e * mw + (t >> 5)] + __popc(m & ((1u << (t & 31)) - 1u));
        }
        s_pos[r] = pos;
        s_w[r] = p.sel_w[(size_t)t * k + r];
    }
    __syncthreads();
    const int H = p.H;
    const size_t shared_row = (size_t)p.T * k + t;
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x) {
        float v = 0.0f;
        if (p.S > 0) v = __fadd_rn(v, p.y[shared_row * H + h]);
        for (int r = 0; r < k; r++)
            if (s_pos[r] >= 0) v = __fadd_rn(v, __fmul_rn(s_w[r], p.y[(size_t)s_pos[r] * H + h]));
        p.out[(size_t)t * H + h] = v;
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
cudaError_t launch_stream(Kern kern, const FwdParams &p, const LayerDev &L, StreamCfg c, int upper, int num_sms,
                          cudaStream_t st)
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
    kern<<<grid, kStreamThreads, sm, st>>>(p, L, c);
    return cudaGetLastError();
}

int ring_stages(int stage_bytes)
{
    int s = kRingBudget / stage_bytes;
    return s < 2 ? 2 : (s > 16 ? 16 : s);
}

}  // namespace

cudaError_t launch_gate_up(const FwdParams &p, const LayerDev &L, int mode, int num_sms, cudaStream_t st)
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
    c.item_rows = kGuItemRows;
    c.rt_routed = mode == 1 ? 0 : (L.gate.rows + kGuItemRows - 1) / kGuItemRows;
    c.rt_shared = (mode != 0 && p.S > 0) ? (L.sh_gate.rows + kGuItemRows - 1) / kGuItemRows : 0;
    c.down_f32 = (mode == 1 ? L.sh_down.type : L.down.type) == FMT_F32;
    c.act_k = p.H;
    size_t per_row = G0.qs_rstride + G0.meta_rstride;
    c.stage_bytes = (int)(((2 * kGuChunkRows * per_row) + 127) / 128 * 128);
    c.stages = ring_stages(c.stage_bytes);
    const int upper = (mode == 1 ? 0 : (p.max_problems - (p.S > 0 ? 1 : 0)) * c.rt_routed) + c.rt_shared;
    if (G0.type == FMT_Q4_K) return launch_stream(gate_up_stream_kernel<FMT_Q4_K>, p, L, c, upper, num_sms, st);
    return launch_stream(gate_up_stream_kernel<FMT_Q8_0>, p, L, c, upper, num_sms, st);
}

cudaError_t launch_down(const FwdParams &p, const LayerDev &L, int mode, int num_sms, cudaStream_t st)
{
    const DevMatrix &D0 = mode == 1 ? L.sh_down : L.down;
    if (D0.type == FMT_F32) {
        const int ny = mode == 1 ? 1 : (mode == 2 ? p.max_problems : p.max_problems - (p.S > 0 ? 1 : 0));
        down_f32_kernel<<<dim3((p.H + 31) / 32, ny), 256, 0, st>>>(p, L, mode);
        return cudaGetLastError();
    }
    StreamCfg c{};
    c.mode = mode;
    c.item_rows = kDnItemRows;
    c.rt_routed = mode == 1 ? 0 : (p.H + kDnItemRows - 1) / kDnItemRows;
    c.rt_shared = (mode != 0 && p.S > 0) ? (p.H + kDnItemRows - 1) / kDnItemRows : 0;
    size_t per_row = D0.qs_rstride + D0.meta_rstride;
    int act = D0.cols;
    if (mode == 2) {
        const size_t sh_row = L.sh_down.qs_rstride + L.sh_down.meta_rstride;
        per_row = per_row > sh_row ? per_row : sh_row;
        act = act > L.sh_down.cols ? act : L.sh_down.cols;
    }
    c.act_k = act;
    c.stage_bytes = (int)((kDnChunkRows * per_row + 127) / 128 * 128);
    c.stages = ring_stages(c.stage_bytes);
    const int upper = (mode == 1 ? 0 : (p.max_problems - (p.S > 0 ? 1 : 0)) * c.rt_routed) + c.rt_shared;
    if (D0.type == FMT_Q4_K) return launch_stream(down_stream_kernel<FMT_Q4_K>, p, L, c, upper, num_sms, st);
    return launch_stream(down_stream_kernel<FMT_Q8_0>, p, L, c, upper, num_sms, st);
}

cudaError_t launch_combine(const FwdParams &p, cudaStream_t st)
{
    dim3 grid((p.H + 255) / 256 < 8 ? (p.H + 255) / 256 : 8, p.T);
    combine_kernel<<<grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace jmoe
