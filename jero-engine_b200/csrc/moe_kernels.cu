// moe_kernels.cu -- router, dispatch permutation, grouped SwiGLU experts and
// combine for the batched MoE block (CUDA cores; sm_100a).
//
// One forward = memset(mask) -> router -> topk -> scan -> gate_up -> down -> combine.
// Every kernel reads its work from device-side counters written by the one
// before it, so the sequence needs no host round trip and can be captured in
// a CUDA graph. No kernel waits on another CTA.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "moe_device.h"

namespace jmoe {

namespace {

constexpr int kTT = 8;          // tokens per expert-kernel tile
constexpr int kRouterTT = 8;    // tokens per router CTA
constexpr int kMaxLaneE = 8;    // experts per lane in topk (E <= 256)
constexpr int kMaxK = 16;

__device__ __forceinline__ int32_t total_key(float f)
{
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

__device__ __forceinline__ bool rank_before(int32_t ka, int ia, int32_t kb, int ib)
{
    return ka > kb || (ka == kb && ia < ib);
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_isum(int v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Activation block quantiser: 32 lanes hold the 32 values of one block.
// q = clamp(round(v * 127/amax), -127, 127), NaN -> -127; d = amax/127.
__device__ __forceinline__ void quant_block32(float v, int8_t *q_out, float *d_out, float *s_out, int lane)
{
    float amax = warp_max(fabsf(v));
    float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    float r = roundf(__fmul_rn(v, id));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    int q = (int)r;
    q_out[lane] = (int8_t)q;
    int qs = warp_isum(q);
    if (lane == 0) {
        float d = __fdiv_rn(amax, 127.0f);
        *d_out = d;
        *s_out = d * (float)qs;
    }
}

__device__ __forceinline__ int byte_of(uint32_t a, uint32_t b, uint32_t c, int i)
{
    uint32_t w = i < 4 ? a : (i < 8 ? b : c);
    return (int)((w >> (8 * (i & 3))) & 0xFFu);
}

// ----------------------------------------------------------------- router

// logits[t][e] = router row e . x_t in the canonical order (element h to
// partial (h/4) mod 32, fmaf chain per partial, xor butterfly 16..1), then
// + logit_bias[e]. CTAs also quantise x into int8 blocks when p.quant_x.
template <int EPW>
__global__ void __launch_bounds__(128) router_kernel(FwdParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = (blockIdx.x * 4 + warp) * EPW;
    const int t0 = blockIdx.y * kRouterTT;
    const int H = p.H, E = p.E, T = p.T;

    if (p.quant_x) {
        const int nb = H >> 5;
        const int ntok = min(kRouterTT, T - t0);
        const int ntask = ntok * nb;
        for (int i = blockIdx.x + gridDim.x * warp; i < ntask; i += gridDim.x * 4) {
            int t = t0 + i / nb, b = i % nb;
            float v = p.x[(size_t)t * H + 32 * b + lane];
            quant_block32(v, p.xq + (size_t)t * H + 32 * b, p.xd + (size_t)t * nb + b,
                          p.xs + (size_t)t * nb + b, lane);
        }
    }
    if (e0 >= E) return;

    float acc[kRouterTT][EPW];
#pragma unroll
    for (int t = 0; t < kRouterTT; t++)
#pragma unroll
        for (int j = 0; j < EPW; j++) acc[t][j] = 0.0f;

    if ((H & 3) == 0) {
        for (int h4 = lane; h4 < (H >> 2); h4 += 32) {
            float4 w[EPW];
#pragma unroll
            for (int j = 0; j < EPW; j++)
                w[j] = (e0 + j < E) ? __ldg(reinterpret_cast<const float4 *>(p.router + (size_t)(e0 + j) * H) + h4)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int t = 0; t < kRouterTT; t++) {
                if (t0 + t < T) {
                    float4 xv = __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)(t0 + t) * H) + h4);
#pragma unroll
                    for (int j = 0; j < EPW; j++) {
                        acc[t][j] = __fmaf_rn(w[j].x, xv.x, acc[t][j]);
                        acc[t][j] = __fmaf_rn(w[j].y, xv.y, acc[t][j]);
                        acc[t][j] = __fmaf_rn(w[j].z, xv.z, acc[t][j]);
                        acc[t][j] = __fmaf_rn(w[j].w, xv.w, acc[t][j]);
                    }
                }
            }
        }
    } else {
        for (int hb = 4 * lane; hb < H; hb += 128) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                int h = hb + c;
                if (h < H) {
#pragma unroll
                    for (int t = 0; t < kRouterTT; t++) {
                        if (t0 + t < T) {
                            float xv = p.x[(size_t)(t0 + t) * H + h];
#pragma unroll
                            for (int j = 0; j < EPW; j++)
                                if (e0 + j < E)
                                    acc[t][j] = __fmaf_rn(p.router[(size_t)(e0 + j) * H + h], xv, acc[t][j]);
                        }
                    }
                }
            }
        }
    }

#pragma unroll
    for (int t = 0; t < kRouterTT; t++) {
#pragma unroll
        for (int j = 0; j < EPW; j++) {
            float v = acc[t][j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0 && t0 + t < T && e0 + j < E) {
                if (p.logit_bias) v = __fadd_rn(v, p.logit_bias[e0 + j]);
                p.logits[(size_t)(t0 + t) * E + e0 + j] = v;
            }
        }
    }
}

// ------------------------------------------------------------------- topk

// One warp per token: softmax, (group-limited) top-k, weights, and the token
// bit in the expert mask. Semantics of select_top_k_experts /
// select_experts_with_optional_bias (src/gemma.rs:362-442,
// src/qwen_deepseek.rs:773-831); ranking by total_cmp key, ties to the lower index.
__global__ void __launch_bounds__(128) topk_kernel(FwdParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + warp;
    if (t >= p.T) return;
    const int E = p.E;
    float lg[kMaxLaneE];
    int32_t key[kMaxLaneE];
    bool cand[kMaxLaneE];
#pragma unroll
    for (int i = 0; i < kMaxLaneE; i++) {
        int e = lane + 32 * i;
        bool valid = e < E;
        lg[i] = valid ? p.logits[(size_t)t * E + e] : 0.0f;
        float s = (valid && p.sel_bias) ? __fadd_rn(lg[i], p.sel_bias[e]) : lg[i];
        key[i] = valid ? total_key(isfinite(s) ? s : -INFINITY) : INT32_MIN;
        cand[i] = valid;
    }
    int k = min(p.k, E);
    if (p.route_mode == 1 && p.n_groups > 0 && p.topk_groups > 0 && p.topk_groups < p.n_groups) {
        const int G = p.n_groups, gs = E / G;
        int32_t mykey = INT32_MIN;
        for (int g = 0; g < G; g++) {
            int32_t local = INT32_MIN;
#pragma unroll
            for (int i = 0; i < kMaxLaneE; i++) {
                int e = lane + 32 * i;
                if (e < E && e / gs == g) local = max(local, key[i]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) local = max(local, __shfl_xor_sync(0xffffffffu, local, o));
            if (lane == g) mykey = local;
        }
        uint32_t gmask = 0;
        for (int r = 0; r < p.topk_groups; r++) {
            int32_t bk = (lane < G && !((gmask >> lane) & 1u)) ? mykey : INT32_MIN;
            int bi = (lane < G && !((gmask >> lane) & 1u)) ? lane : 0x7fffffff;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                int32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
                int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (rank_before(ok, oi, bk, bi)) { bk = ok; bi = oi; }
            }
            gmask |= 1u << bi;
        }
#pragma unroll
        for (int i = 0; i < kMaxLaneE; i++) {
            int e = lane + 32 * i;
            cand[i] = cand[i] && ((gmask >> (e / gs)) & 1u);
        }
        k = min(k, p.topk_groups * gs);
    }

    int sel[kMaxK];
    int nsel = 0;
    for (int r = 0; r < k; r++) {
        int32_t bk = INT32_MIN;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxLaneE; i++) {
            int e = lane + 32 * i;
            if (cand[i] && (bi == 0x7fffffff || rank_before(key[i], e, bk, bi))) { bk = key[i]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            int32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || rank_before(ok, oi, bk, bi))) { bk = ok; bi = oi; }
        }
        if (bi == 0x7fffffff) break;
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < kMaxLaneE; i++)
                if (i == (bi >> 5)) cand[i] = false;
        }
        sel[r] = bi;
        nsel = r + 1;
    }

    // softmax of the (logit-biased) router logits over all E
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxLaneE; i++)
        if (lane + 32 * i < E && isfinite(lg[i])) mx = fmaxf(mx, lg[i]);
    mx = warp_max(mx);
    float pv[kMaxLaneE];
    float psum = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxLaneE; i++) {
        bool ok = lane + 32 * i < E && isfinite(lg[i]) && isfinite(mx);
        pv[i] = ok ? expf(lg[i] - mx) : 0.0f;
        psum = __fadd_rn(psum, pv[i]);
    }
    psum = warp_sum(psum);
    const bool sum_ok = psum > 0.0f && isfinite(psum);

    float w[kMaxK];
    for (int r = 0; r < nsel; r++) {
        int e = sel[r];
        float mine = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxLaneE; i++)
            if (i == (e >> 5)) mine = pv[i];
        float pe = __shfl_sync(0xffffffffu, mine, e & 31);
        if (p.sel_bias) {
            w[r] = sum_ok ? __fdiv_rn(pe, psum) : 0.0f;
        } else {
            w[r] = sum_ok ? __fdiv_rn(pe, psum) : __fdiv_rn(1.0f, (float)E);
        }
    }
    if (p.sel_bias || p.normalize) {
        float ss = 0.0f;
        for (int r = 0; r < nsel; r++) ss = __fadd_rn(ss, w[r]);
        const bool ok = ss > 0.0f && isfinite(ss);
        for (int r = 0; r < nsel; r++) w[r] = ok ? __fdiv_rn(w[r], ss) : __fdiv_rn(1.0f, (float)nsel);
    } else if (p.routed_scale != 1.0f) {
        for (int r = 0; r < nsel; r++) w[r] = __fmul_rn(w[r], p.routed_scale);
    }

    const int mw = p.mask_words;
    for (int r = 0; r < p.k; r++) {
        if (lane == (r & 31)) {
            int e = r < nsel ? sel[r] : -1;
            p.sel_idx[(size_t)t * p.k + r] = e;
            p.sel_w[(size_t)t * p.k + r] = r < nsel ? w[r] : 0.0f;
            if (e >= 0) atomicOr(p.mask + (size_t)e * mw + (t >> 5), 1u << (t & 31));
        }
    }
}

// ------------------------------------------------------------------- scan

// Single CTA: per-expert token counts from the bit masks, slot offsets
// (experts ascending), the list of experts that received tokens, and the
// slot -> token permutation (tokens ascending inside an expert).
__global__ void __launch_bounds__(1024) scan_kernel(FwdParams p)
{
    extern __shared__ int s_scan[];
    int *s_count = s_scan;           // [E]
    int *s_off = s_scan + p.E;       // [E+1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int E = p.E, mw = p.mask_words;

    for (int e = warp; e < E; e += nwarps) {
        int run = 0;
        for (int c = 0; c < mw; c += 32) {
            int word = c + lane;
            uint32_t m = word < mw ? p.mask[(size_t)e * mw + word] : 0u;
            int pc = __popc(m), incl = pc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (word < mw) p.wprefix[(size_t)e * mw + word] = run + incl - pc;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) s_count[e] = run;
    }
    __syncthreads();
    if (warp == 0) {
        const int chunk = (E + 31) / 32;
        int b = lane * chunk, local = 0;
        for (int i = 0; i < chunk; i++)
            if (b + i < E) local += s_count[b + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < chunk; i++) {
            if (b + i < E) {
                s_off[b + i] = run;
                p.offsets[b + i] = run;
                run += s_count[b + i];
            }
        }
        if (lane == 31) { s_off[E] = incl; p.offsets[E] = incl; }
    }
    __syncthreads();
    if (warp == 0) {
        int nact = 0;
        for (int c = 0; c < E; c += 32) {
            int e = c + lane;
            bool act = e < E && s_count[e] > 0;
            uint32_t bal = __ballot_sync(0xffffffffu, act);
            int pos = nact + __popc(bal & ((1u << lane) - 1u));
            if (act) {
                Problem pr;
                pr.expert = e; pr.slot0 = s_off[e]; pr.count = s_count[e]; pr.is_shared = 0;
                p.problems[pos] = pr;
            }
            nact += __popc(bal);
        }
        if (lane == 0) {
            *p.n_active = nact;
            if (p.S > 0) {
                Problem pr;
                pr.expert = 0; pr.slot0 = p.T * p.k; pr.count = p.T; pr.is_shared = 1;
                p.problems[p.max_problems - 1] = pr;
            }
        }
    }
    for (int e = warp; e < E; e += nwarps) {
        if (s_count[e] == 0) continue;
        for (int c = 0; c < mw; c += 32) {
            int word = c + lane;
            if (word < mw) {
                uint32_t m = p.mask[(size_t)e * mw + word];
                int pos = s_off[e] + p.wprefix[(size_t)e * mw + word];
                while (m) {
                    int bit = __ffs(m) - 1;
                    p.perm_token[pos++] = word * 32 + bit;
                    m &= m - 1u;
                }
            }
        }
    }
    if (p.S > 0)
        for (int i = threadIdx.x; i < p.T; i += blockDim.x) p.perm_token[(size_t)p.T * p.k + i] = i;
}

// ----------------------------------------------------- expert weight units

// One 32-value block of a quantised row (a Q8_0 block or a Q4_K sub-block),
// held in registers and dotted against many tokens.
template <int FMT>
struct WUnit;

template <>
struct WUnit<FMT_Q4_K> {
    uint4 q;
    float dsc, dmn;
    __device__ __forceinline__ void load(const DevMatrix &M, const uint8_t *qs_row, const uint8_t *meta_row, int u)
    {
        q = __ldg(reinterpret_cast<const uint4 *>(qs_row + 16 * (size_t)u));
        uint4 m = __ldg(reinterpret_cast<const uint4 *>(meta_row + 16 * (size_t)(u >> 3)));
        float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xFFFFu)));
        float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
        int j = u & 7, sc, mn;
        if (j < 4) {
            sc = byte_of(m.y, m.z, m.w, j) & 63;
            mn = byte_of(m.y, m.z, m.w, j + 4) & 63;
        } else {
            sc = (byte_of(m.y, m.z, m.w, j + 4) & 0x0F) | ((byte_of(m.y, m.z, m.w, j - 4) >> 6) << 4);
            mn = (byte_of(m.y, m.z, m.w, j + 4) >> 4) | ((byte_of(m.y, m.z, m.w, j) >> 6) << 4);
        }
        dsc = d * (float)sc;
        dmn = dmin * (float)mn;
    }
    __device__ __forceinline__ int isum(const int8_t *xq) const
    {
        const int4 a = *reinterpret_cast<const int4 *>(xq);
        const int4 b = *reinterpret_cast<const int4 *>(xq + 16);
        const uint32_t m4 = 0x0F0F0F0Fu;
        int s = __dp4a((int)(q.x & m4), a.x, 0);
        s = __dp4a((int)(q.y & m4), a.y, s);
        s = __dp4a((int)(q.z & m4), a.z, s);
        s = __dp4a((int)(q.w & m4), a.w, s);
        s = __dp4a((int)((q.x >> 4) & m4), b.x, s);
        s = __dp4a((int)((q.y >> 4) & m4), b.y, s);
        s = __dp4a((int)((q.z >> 4) & m4), b.z, s);
        s = __dp4a((int)((q.w >> 4) & m4), b.w, s);
        return s;
    }
    __device__ __forceinline__ float dot(const int8_t *xq, float xd, float xs) const
    {
        return xd * (dsc * (float)isum(xq)) - xs * dmn;
    }
};

template <>
struct WUnit<FMT_Q8_0> {
    uint4 q0, q1;
    float d;
    __device__ __forceinline__ void load(const DevMatrix &M, const uint8_t *qs_row, const uint8_t *meta_row, int u)
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(qs_row + 32 * (size_t)u);
        q0 = __ldg(src);
        q1 = __ldg(src + 1);
        d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(meta_row) + u)));
    }
    __device__ __forceinline__ int isum(const int8_t *xq) const
    {
        const int4 a = *reinterpret_cast<const int4 *>(xq);
        const int4 b = *reinterpret_cast<const int4 *>(xq + 16);
        int s = __dp4a((int)q0.x, a.x, 0);
        s = __dp4a((int)q0.y, a.y, s);
        s = __dp4a((int)q0.z, a.z, s);
        s = __dp4a((int)q0.w, a.w, s);
        s = __dp4a((int)q1.x, b.x, s);
        s = __dp4a((int)q1.y, b.y, s);
        s = __dp4a((int)q1.z, b.z, s);
        s = __dp4a((int)q1.w, b.w, s);
        return s;
    }
    __device__ __forceinline__ float dot(const int8_t *xq, float xd, float xs) const
    {
        return (d * xd) * (float)isum(xq);
    }
};

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
    int y = blockIdx.y;
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

// Stages the activation blocks of tokens [t0, t0+nt) of a problem into shared
// memory: xq [kTT][K], xd [kTT][K/32], xs [kTT][K/32]. gather: token ids come
// from perm_token (gate/up: rows of x); otherwise rows are consecutive slots.
__device__ __forceinline__ void stage_act(int8_t *s_xq, float *s_xd, float *s_xs, const int8_t *gq,
                                          const float *gd, const float *gs, size_t q_stride, size_t d_stride,
                                          const int32_t *perm, int row0, int nt, int K)
{
    const int nv = K >> 4, nb = K >> 5;
    for (int v = threadIdx.x; v < nt * nv; v += blockDim.x) {
        int i = v / nv, c = v % nv;
        size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        reinterpret_cast<uint4 *>(s_xq + (size_t)i * K)[c] = __ldg(reinterpret_cast<const uint4 *>(gq + row * q_stride) + c);
    }
    for (int v = threadIdx.x; v < nt * nb; v += blockDim.x) {
        int i = v / nb, c = v % nb;
        size_t row = perm ? (size_t)perm[row0 + i] : (size_t)(row0 + i);
        s_xd[i * nb + c] = __ldg(gd + row * d_stride + c);
        s_xs[i * nb + c] = __ldg(gs + row * d_stride + c);
    }
}

// Gate and up projections of one 32-row tile for every token of one problem,
// a = silu(g) * u, quantised into one int8 block per token (or stored as f32
// when the down matrix is F32). 8 warps x 4 rows, 8 lanes per row.
template <int FMT>
__global__ void __launch_bounds__(256) gate_up_q_kernel(FwdParams p, LayerDev L, int shared_mode, int down_f32)
{
    ProblemSel ps = pick_problem(p, shared_mode);
    if (!ps.ok) return;
    const DevMatrix &G = ps.shared ? L.sh_gate : L.gate;
    const DevMatrix &U = ps.shared ? L.sh_up : L.up;
    const int rows = G.rows, K = G.cols, NU = K >> 5;
    const int r0 = blockIdx.x * 32;
    if (r0 >= rows) return;

    extern __shared__ __align__(16) uint8_t smem[];
    int8_t *s_xq = reinterpret_cast<int8_t *>(smem);
    float *s_xd = reinterpret_cast<float *>(smem + (size_t)kTT * K);
    float *s_xs = s_xd + kTT * NU;
    float *s_g = s_xs + kTT * NU;   // [kTT][32]
    float *s_u = s_g + kTT * 32;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane >> 3, l8 = lane & 7;
    const int rl = warp * 4 + sub, row = r0 + rl;
    const bool row_ok = row < rows;
    const int e = ps.pr.expert;
    const uint8_t *gq = G.qs + (size_t)e * G.qs_estride + (size_t)row * G.qs_rstride;
    const uint8_t *gm = G.meta + (size_t)e * G.meta_estride + (size_t)row * G.meta_rstride;
    const uint8_t *uq = U.qs + (size_t)e * U.qs_estride + (size_t)row * U.qs_rstride;
    const uint8_t *um = U.meta + (size_t)e * U.meta_estride + (size_t)row * U.meta_rstride;

    for (int t0 = 0; t0 < ps.pr.count; t0 += kTT) {
        const int nt = min(kTT, ps.pr.count - t0);
        __syncthreads();
        stage_act(s_xq, s_xd, s_xs, p.xq, p.xd, p.xs, (size_t)p.H, (size_t)(p.H >> 5), p.perm_token,
                  ps.pr.slot0 + t0, nt, K);
        __syncthreads();

        float ag[kTT], au[kTT];
#pragma unroll
        for (int t = 0; t < kTT; t++) { ag[t] = 0.0f; au[t] = 0.0f; }
        if (row_ok) {
            for (int u = l8; u < NU; u += 8) {
                WUnit<FMT> wg, wu;
                wg.load(G, gq, gm, u);
                wu.load(U, uq, um, u);
#pragma unroll
                for (int t = 0; t < kTT; t++) {
                    if (t < nt) {
                        const int8_t *xq = s_xq + (size_t)t * K + 32 * u;
                        float xd = s_xd[t * NU + u], xs = s_xs[t * NU + u];
                        ag[t] += wg.dot(xq, xd, xs);
                        au[t] += wu.dot(xq, xd, xs);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kTT; t++) {
            float g = ag[t], u = au[t];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) {
                g += __shfl_xor_sync(0xffffffffu, g, o);
                u += __shfl_xor_sync(0xffffffffu, u, o);
            }
            if (l8 == 0 && t < nt) {
                s_g[t * 32 + rl] = g;
                s_u[t * 32 + rl] = u;
            }
        }
        __syncthreads();
        if (warp < nt) {
            const int t = warp;
            const size_t slot = (size_t)ps.pr.slot0 + t0 + t;
            float a = 0.0f;
            if (r0 + lane < rows) {
                float g = s_g[t * 32 + lane], u = s_u[t * 32 + lane];
                a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
            }
            if (down_f32) {
                if (r0 + lane < rows) p.af[slot * p.W + r0 + lane] = a;
            } else {
                quant_block32(a, p.aq + slot * p.W + r0, p.ad + slot * (p.W >> 5) + (r0 >> 5),
                              p.as + slot * (p.W >> 5) + (r0 >> 5), lane);
            }
        }
    }
}

// Down projection of one 32-row tile (rows of H) for every slot of one problem.
template <int FMT>
__global__ void __launch_bounds__(256) down_q_kernel(FwdParams p, LayerDev L, int shared_mode)
{
    ProblemSel ps = pick_problem(p, shared_mode);
    if (!ps.ok) return;
    const DevMatrix &D = ps.shared ? L.sh_down : L.down;
    const int rows = D.rows, K = D.cols, NU = K >> 5;
    const int r0 = blockIdx.x * 32;
    if (r0 >= rows) return;

    extern __shared__ __align__(16) uint8_t smem[];
    int8_t *s_xq = reinterpret_cast<int8_t *>(smem);
    float *s_xd = reinterpret_cast<float *>(smem + (size_t)kTT * K);
    float *s_xs = s_xd + kTT * NU;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane >> 3, l8 = lane & 7;
    const int row = r0 + warp * 4 + sub;
    const bool row_ok = row < rows;
    const int e = ps.pr.expert;
    const uint8_t *dq = D.qs + (size_t)e * D.qs_estride + (size_t)row * D.qs_rstride;
    const uint8_t *dm = D.meta + (size_t)e * D.meta_estride + (size_t)row * D.meta_rstride;

    for (int t0 = 0; t0 < ps.pr.count; t0 += kTT) {
        const int nt = min(kTT, ps.pr.count - t0);
        __syncthreads();
        stage_act(s_xq, s_xd, s_xs, p.aq, p.ad, p.as, (size_t)p.W, (size_t)(p.W >> 5), nullptr,
                  ps.pr.slot0 + t0, nt, K);
        __syncthreads();
        float acc[kTT];
#pragma unroll
        for (int t = 0; t < kTT; t++) acc[t] = 0.0f;
        if (row_ok) {
            for (int u = l8; u < NU; u += 8) {
                WUnit<FMT> w;
                w.load(D, dq, dm, u);
#pragma unroll
                for (int t = 0; t < kTT; t++)
                    if (t < nt) acc[t] += w.dot(s_xq + (size_t)t * K + 32 * u, s_xd[t * NU + u], s_xs[t * NU + u]);
            }
        }
#pragma unroll
        for (int t = 0; t < kTT; t++) {
            float v = acc[t];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (l8 == 0 && row_ok && t < nt) p.y[((size_t)ps.pr.slot0 + t0 + t) * p.H + row] = v;
        }
    }
}

// F32 expert matrices (the reference's own unit tests use F32 stacks): one
// token at a time, activations read from global memory, any shape.
__global__ void __launch_bounds__(256) gate_up_f32_kernel(FwdParams p, LayerDev L, int shared_mode)
{
    ProblemSel ps = pick_problem(p, shared_mode);
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
        if (l8 == 0 && row < rows) p.af[slot * p.W + row] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

__global__ void __launch_bounds__(256) down_f32_kernel(FwdParams p, LayerDev L, int shared_mode)
{
    ProblemSel ps = pick_problem(p, shared_mode);
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
    __shared__ size_t s_pos[kMaxK];
    __shared__ float s_w[kMaxK];
    const int t = blockIdx.y, k = p.k, mw = p.mask_words;
    if (threadIdx.x < k) {
        int r = threadIdx.x;
        int e = p.sel_idx[(size_t)t * k + r];
        size_t pos = (size_t)-1;
        if (e >= 0) {
            uint32_t m = p.mask[(size_t)e * mw + (t >> 5)];
            pos = (size_t)(p.offsets[e] + p.wprefix[(size_t)e * mw + (t >> 5)] + __popc(m & ((1u << (t & 31)) - 1u)));
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
            if (s_pos[r] != (size_t)-1) v = __fadd_rn(v, __fmul_rn(s_w[r], p.y[s_pos[r] * H + h]));
        p.out[(size_t)t * H + h] = v;
    }
}

// ------------------------------------------------------------ parity probe

__global__ void quantize_rows_kernel(const float *x, int n, int cols, int8_t *xq, float *xd, float *xs)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = cols >> 5;
    if (warp >= n * nb) return;
    int r = warp / nb, b = warp % nb;
    quant_block32(x[(size_t)r * cols + 32 * b + lane], xq + (size_t)r * cols + 32 * b, xd + (size_t)r * nb + b,
                  xs + (size_t)r * nb + b, lane);
}

template <int FMT>
__global__ void block_dots_kernel(DevMatrix m, const int8_t *xq, int n, int32_t *isum)
{
    const int nb = m.cols >> 5;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nb) return;
    int r = i / nb, u = i % nb;
    WUnit<FMT> w;
    w.load(m, m.qs + (size_t)r * m.qs_rstride, m.meta + (size_t)r * m.meta_rstride, u);
    isum[i] = w.isum(xq + (size_t)r * m.cols + 32 * u);
}

inline size_t act_smem(int K) { return (size_t)kTT * K + 2 * (size_t)kTT * (K / 32) * 4 + 2 * kTT * 32 * 4; }

template <typename Kern>
cudaError_t set_smem(Kern k, size_t bytes)
{
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

cudaError_t launch_gate_up(const FwdParams &p, const LayerDev &L, const DevMatrix &G, int ny, int mode,
                           int down_f32, cudaStream_t st)
{
    dim3 grid((G.rows + 31) / 32, ny);
    if (G.type == FMT_F32) {
        gate_up_f32_kernel<<<grid, 256, 0, st>>>(p, L, mode);
        return cudaGetLastError();
    }
    size_t sm = act_smem(G.cols);
    cudaError_t err;
    if (G.type == FMT_Q4_K) {
        if ((err = set_smem(gate_up_q_kernel<FMT_Q4_K>, sm)) != cudaSuccess) return err;
        gate_up_q_kernel<FMT_Q4_K><<<grid, 256, sm, st>>>(p, L, mode, down_f32);
    } else {
        if ((err = set_smem(gate_up_q_kernel<FMT_Q8_0>, sm)) != cudaSuccess) return err;
        gate_up_q_kernel<FMT_Q8_0><<<grid, 256, sm, st>>>(p, L, mode, down_f32);
    }
    return cudaGetLastError();
}

cudaError_t launch_down(const FwdParams &p, const LayerDev &L, const DevMatrix &D, int ny, int mode, cudaStream_t st)
{
    dim3 grid((D.rows + 31) / 32, ny);
    if (D.type == FMT_F32) {
        down_f32_kernel<<<grid, 256, 0, st>>>(p, L, mode);
        return cudaGetLastError();
    }
    size_t sm = act_smem(D.cols);
    cudaError_t err;
    if (D.type == FMT_Q4_K) {
        if ((err = set_smem(down_q_kernel<FMT_Q4_K>, sm)) != cudaSuccess) return err;
        down_q_kernel<FMT_Q4_K><<<grid, 256, sm, st>>>(p, L, mode);
    } else {
        if ((err = set_smem(down_q_kernel<FMT_Q8_0>, sm)) != cudaSuccess) return err;
        down_q_kernel<FMT_Q8_0><<<grid, 256, sm, st>>>(p, L, mode);
    }
    return cudaGetLastError();
}

}  // namespace

int launch_forward(const FwdParams &p, const LayerDev &L, void *stream, const Marker &mk)
{
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t err;
    if (p.T == 0) return cudaSuccess;
    mk.mark(nullptr);
    if ((err = cudaMemsetAsync(p.mask, 0, sizeof(uint32_t) * (size_t)p.E * p.mask_words, st)) != cudaSuccess)
        return err;
    if (p.T <= 8) {
        dim3 grid((p.E + 3) / 4, (p.T + kRouterTT - 1) / kRouterTT);
        router_kernel<1><<<grid, 128, 0, st>>>(p);
    } else {
        dim3 grid((p.E + 15) / 16, (p.T + kRouterTT - 1) / kRouterTT);
        router_kernel<4><<<grid, 128, 0, st>>>(p);
    }
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    mk.mark("router");
    topk_kernel<<<(p.T + 3) / 4, 128, 0, st>>>(p);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    mk.mark("topk");
    scan_kernel<<<1, 1024, sizeof(int) * (2 * (size_t)p.E + 1), st>>>(p);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    mk.mark("scan");

    const int n_routed = p.max_problems - (p.S > 0 ? 1 : 0);
    const bool has_sh = p.S > 0;
    const bool same_gu = has_sh && L.sh_gate.type == L.gate.type;
    const bool same_d = has_sh && L.sh_down.type == L.down.type;
    // gate/up: one launch when the shared expert has the routed format
    // (grid.x covers the larger of I and S; CTAs past a problem's rows exit).
    if (same_gu) {
        DevMatrix G = L.gate;
        G.rows = L.gate.rows > L.sh_gate.rows ? L.gate.rows : L.sh_gate.rows;
        G.cols = L.gate.cols;
        if ((err = launch_gate_up(p, L, G, p.max_problems, 2, L.down.type == FMT_F32, st)) != cudaSuccess) return err;
        mk.mark("gate_up");
    } else {
        if ((err = launch_gate_up(p, L, L.gate, n_routed, 0, L.down.type == FMT_F32, st)) != cudaSuccess) return err;
        mk.mark("gate_up");
        if (has_sh) {
            if ((err = launch_gate_up(p, L, L.sh_gate, 1, 1, L.sh_down.type == FMT_F32, st)) != cudaSuccess)
                return err;
            mk.mark("gate_up_shared");
        }
    }
    if (same_d) {
        DevMatrix D = L.down;
        D.cols = L.down.cols > L.sh_down.cols ? L.down.cols : L.sh_down.cols;
        if ((err = launch_down(p, L, D, p.max_problems, 2, st)) != cudaSuccess) return err;
        mk.mark("down");
    } else {
        if ((err = launch_down(p, L, L.down, n_routed, 0, st)) != cudaSuccess) return err;
        mk.mark("down");
        if (has_sh) {
            if ((err = launch_down(p, L, L.sh_down, 1, 1, st)) != cudaSuccess) return err;
            mk.mark("down_shared");
        }
    }
    dim3 cgrid((p.H + 255) / 256 < 8 ? (p.H + 255) / 256 : 8, p.T);
    combine_kernel<<<cgrid, 256, 0, st>>>(p);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    mk.mark("combine");
    return cudaSuccess;
}

int launch_quantize_rows(const float *x, int n, int cols, int8_t *xq, float *xd, float *xs, void *stream)
{
    int warps = n * (cols / 32);
    quantize_rows_kernel<<<(warps + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, cols, xq, xd, xs);
    return cudaGetLastError();
}

int launch_block_dots(const DevMatrix &m, const int8_t *xq, int n, int32_t *isum, void *stream)
{
    int tot = n * (m.cols / 32);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (m.type == FMT_Q4_K)
        block_dots_kernel<FMT_Q4_K><<<(tot + 255) / 256, 256, 0, st>>>(m, xq, n, isum);
    else
        block_dots_kernel<FMT_Q8_0><<<(tot + 255) / 256, 256, 0, st>>>(m, xq, n, isum);
    return cudaGetLastError();
}

}  // namespace jmoe
