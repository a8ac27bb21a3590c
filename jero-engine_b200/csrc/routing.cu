// routing.cu -- router logits, top-k selection and the dispatch permutation.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace jmoe {
namespace {

// Batches up to this many tokens build the dispatch permutation inside the
// selection kernel (shared-memory masks); larger ones use scan_kernel.
constexpr int kFusedScanMaxT = kFusedRoutingMaxT;
constexpr int kFusedMaskWords = kFusedScanMaxT / 32;

// Quantises the activation blocks of tokens [t0, t0 + ntok): eight lanes per
// 32-value block, four blocks per warp pass; tasks are spread over the warps
// of all CTAs that share this token tile. Same arithmetic as quant_block32.
__device__ __forceinline__ void quantize_tile(const FwdParams &p, int t0, int ntok, int worker, int n_workers,
                                              int lane)
{
    const int H = p.H, nb = H >> 5, ntask = ntok * nb;
    const int sub = lane >> 3, l8 = lane & 7;
    for (int base = worker * 4; base < ntask; base += n_workers * 4) {
        const int i = base + sub;
        const bool ok = i < ntask;
        const int t = t0 + (ok ? i / nb : 0), b = ok ? i % nb : 0;
        float4 v = ok ? *reinterpret_cast<const float4 *>(p.x + (size_t)t * H + 32 * b + 4 * l8)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        amax = fmaxf(amax, 0.0f);
        const float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        auto q8 = [&](float a) {
            float r = roundf(__fmul_rn(a, id));
            return (int)fminf(fmaxf(r, -127.0f), 127.0f);
        };
        const int q0 = q8(v.x), q1 = q8(v.y), q2 = q8(v.z), q3 = q8(v.w);
        int qs = q0 + q1 + q2 + q3;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
        if (ok) {
            const uint32_t packed = (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) |
                                    ((uint32_t)(q2 & 0xFF) << 16) | ((uint32_t)(q3 & 0xFF) << 24);
            *reinterpret_cast<uint32_t *>(p.xq + (size_t)t * H + 32 * b + 4 * l8) = packed;
            const float d = __fdiv_rn(amax, 127.0f);
            if (l8 == 0) {
                p.xd[(size_t)t * nb + b] = d;
                p.xs[(size_t)t * nb + b] = d * (float)qs;
            }
            if (p.x16) {   // f16(q * d) in the tensor-core operand order (0, 2, 1, 3)
                const __half2 a = __floats2half2_rn((float)q0 * d, (float)q2 * d);
                const __half2 c = __floats2half2_rn((float)q1 * d, (float)q3 * d);
                *reinterpret_cast<uint2 *>(static_cast<__half *>(p.x16) + (size_t)t * H + 32 * b + 4 * l8) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&c));
            }
        }
    }
}

// logits[t][e] = router row e . x_t in the canonical order shared with the
// oracle: element h feeds partial (h/4) mod 32 (one lane each), every partial is
// an fmaf chain in increasing h, and the partials are combined by the xor
// butterfly 16, 8, 4, 2, 1; then + logit_bias[e]. Each warp owns EPW experts
// and TT tokens of the CTA's tile; CTAs also quantise x (p.quant_x).
template <int TT, int EPW>
__global__ void __launch_bounds__(128) router_kernel(FwdParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = (blockIdx.x * 4 + warp) * EPW;
    const int t0 = blockIdx.y * TT;
    const int H = p.H, E = p.E, T = p.T;
    const int ntok = min(TT, T - t0);

    if (p.quant_x) quantize_tile(p, t0, ntok, blockIdx.x * 4 + warp, gridDim.x * 4, lane);
    if (e0 >= E) return;

    float acc[TT][EPW];
#pragma unroll
    for (int t = 0; t < TT; t++)
#pragma unroll
        for (int j = 0; j < EPW; j++) acc[t][j] = 0.0f;

    if ((H & 3) == 0) {
        const int n4 = H >> 2;
#pragma unroll 2
        for (int h4 = lane; h4 < n4; h4 += 32) {
            float4 w[EPW];
#pragma unroll
            for (int j = 0; j < EPW; j++)
                w[j] = (e0 + j < E) ? __ldg(reinterpret_cast<const float4 *>(p.router + (size_t)(e0 + j) * H) + h4)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 xv[TT];
#pragma unroll
            for (int t = 0; t < TT; t++)
                xv[t] = (t < ntok) ? __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)(t0 + t) * H) + h4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int t = 0; t < TT; t++) {
#pragma unroll
                for (int j = 0; j < EPW; j++) {
                    acc[t][j] = __fmaf_rn(w[j].x, xv[t].x, acc[t][j]);
                    acc[t][j] = __fmaf_rn(w[j].y, xv[t].y, acc[t][j]);
                    acc[t][j] = __fmaf_rn(w[j].z, xv[t].z, acc[t][j]);
                    acc[t][j] = __fmaf_rn(w[j].w, xv[t].w, acc[t][j]);
                }
            }
        }
    } else {
        for (int hb = 4 * lane; hb < H; hb += 128) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int h = hb + c;
                if (h < H) {
#pragma unroll
                    for (int t = 0; t < TT; t++) {
                        if (t < ntok) {
                            const float xv = p.x[(size_t)(t0 + t) * H + h];
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
    for (int t = 0; t < TT; t++) {
#pragma unroll
        for (int j = 0; j < EPW; j++) {
            float v = acc[t][j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0 && t < ntok && e0 + j < E) {
                if (p.logit_bias) v = __fadd_rn(v, p.logit_bias[e0 + j]);
                p.logits[(size_t)(t0 + t) * E + e0 + j] = v;
            }
        }
    }
}

// Selection of token t by one warp: softmax over all E logits, (group-limited)
// top-k on the total_cmp key with ties to the lower index, the weights, and
// the token's bit in each chosen expert's mask. Semantics of
// select_top_k_experts and select_experts_with_optional_bias
// (src/gemma.rs:362-442, src/qwen_deepseek.rs:773-831). The r-th choice is
// the winner of the r-th round of a warp-wide 64-bit argmax over the
// candidates not chosen yet.
template <int NL>   // experts per lane: E <= 32 * NL
__device__ __forceinline__ void select_token(const FwdParams &p, int t, int lane)
{
    const int E = p.E;
    float lg[NL];
    int32_t key[NL];
    bool cand[NL];
#pragma unroll
    for (int i = 0; i < NL; i++) {
        const int e = lane + 32 * i;
        const bool valid = e < E;
        lg[i] = valid ? p.logits[(size_t)t * E + e] : 0.0f;
        const float s = (valid && p.sel_bias) ? __fadd_rn(lg[i], p.sel_bias[e]) : lg[i];
        key[i] = valid ? total_key(isfinite(s) ? s : -INFINITY) : INT32_MIN;
        cand[i] = valid;
    }

    // softmax of the logits (logit_bias already added) over all E
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NL; i++)
        if (lane + 32 * i < E && isfinite(lg[i])) mx = fmaxf(mx, lg[i]);
    mx = warp_max(mx);
    float pv[NL];
    float psum = 0.0f;
#pragma unroll
    for (int i = 0; i < NL; i++) {
        const bool ok = lane + 32 * i < E && isfinite(lg[i]) && isfinite(mx);
        pv[i] = ok ? expf(__fsub_rn(lg[i], mx)) : 0.0f;
        psum = __fadd_rn(psum, pv[i]);
    }
    psum = warp_sum(psum);
    const bool sum_ok = psum > 0.0f && isfinite(psum);

    int k = min(p.k, E);
    if (p.route_mode == 1 && p.n_groups > 0 && p.topk_groups > 0 && p.topk_groups < p.n_groups) {
        const int G = p.n_groups, gs = E / G;
        int32_t mykey = INT32_MIN;
        for (int g = 0; g < G; g++) {
            int32_t local = INT32_MIN;
#pragma unroll
            for (int i = 0; i < NL; i++) {
                const int e = lane + 32 * i;
                if (e < E && e / gs == g) local = max(local, key[i]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) local = max(local, __shfl_xor_sync(0xffffffffu, local, o));
            if (lane == g) mykey = local;
        }
        // group g (lane g) is kept when fewer than topk_groups groups rank before it
        int grank = 0;
        for (int src = 0; src < G; src++) {
            const int32_t ok = __shfl_sync(0xffffffffu, mykey, src);
            if (lane < G && rank_before(ok, src, mykey, lane)) grank++;
        }
        const uint32_t gmask = __ballot_sync(0xffffffffu, lane < G && grank < p.topk_groups);
#pragma unroll
        for (int i = 0; i < NL; i++) {
            const int e = lane + 32 * i;
            cand[i] = cand[i] && ((gmask >> (e / gs)) & 1u);
        }
        k = min(k, p.topk_groups * gs);
    }

    // k rounds of a warp argmax over the candidates. Each candidate is packed
    // as (key in unsigned order) << 32 | (0xFFFFFFFF - expert), so the 64-bit
    // maximum is the largest key with ties to the lower index; non-candidates
    // are 0. Round r's winner is the r-th choice; its owner lane clears it.
    uint64_t pk[NL];
#pragma unroll
    for (int i = 0; i < NL; i++)
        pk[i] = cand[i] ? ((uint64_t)((uint32_t)key[i] ^ 0x80000000u) << 32) |
                              (uint64_t)(0xFFFFFFFFu - (uint32_t)(lane + 32 * i))
                        : 0ull;
    int my_e = -1;
    float my_w = 0.0f, my_p = 0.0f;
    int nsel = 0;
    for (int r = 0; r < k; r++) {
        uint64_t loc = pk[0];
#pragma unroll
        for (int i = 1; i < NL; i++) loc = pk[i] > loc ? pk[i] : loc;
        const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(loc >> 32));
        const uint32_t lo = __reduce_max_sync(0xffffffffu, (uint32_t)(loc >> 32) == hi ? (uint32_t)loc : 0u);
        if (hi == 0u && lo == 0u) break;   // fewer candidates than k
        const int e = (int)(0xFFFFFFFFu - lo);
        float hp = 0.0f;
#pragma unroll
        for (int i = 0; i < NL; i++)
            if (lane + 32 * i == e) {
                pk[i] = 0ull;
                hp = pv[i];
            }
        const float bp = __shfl_sync(0xffffffffu, hp, e & 31);
        if (lane == r) {
            my_e = e;
            my_p = bp;
        }
        nsel = r + 1;
    }
    // the chosen probabilities, all ranks at once (lane r holds rank r)
    if (lane < nsel) {
        if (p.sel_bias) my_w = sum_ok ? __fdiv_rn(my_p, psum) : 0.0f;
        else my_w = sum_ok ? __fdiv_rn(my_p, psum) : __fdiv_rn(1.0f, (float)E);
    }
    if (p.sel_bias || p.normalize) {
        // sum of the chosen weights in rank order, as the reference adds them
        float ss = 0.0f;
        for (int r = 0; r < nsel; r++) ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, my_w, r));
        const bool ok = ss > 0.0f && isfinite(ss);
        if (lane < nsel) my_w = ok ? __fdiv_rn(my_w, ss) : __fdiv_rn(1.0f, (float)nsel);
    } else if (p.routed_scale != 1.0f) {
        my_w = __fmul_rn(my_w, p.routed_scale);
    }
    if (lane < p.k) {
        p.sel_idx[(size_t)t * p.k + lane] = my_e;
        p.sel_w[(size_t)t * p.k + lane] = my_e >= 0 ? my_w : 0.0f;
        if (my_e >= 0 && p.T > kFusedScanMaxT)   // small batches rebuild the masks in shared memory
            atomicOr(p.mask + (size_t)my_e * p.mask_words + (t >> 5), 1u << (t & 31));
    }
}

// The dispatch permutation from the expert masks, by nthreads threads of one
// CTA: per-expert token counts, slot offsets (experts ascending), the list of
// experts that received tokens, and slot -> token (tokens ascending inside an
// expert). s_count [E], s_off [E+1] in shared memory.
__device__ void build_permutation(const FwdParams &p, int *s_count, int *s_off)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int E = p.E, mw = p.mask_words;

    for (int e = warp; e < E; e += nwarps) {
        int run = 0;
        for (int c = 0; c < mw; c += 32) {
            const int word = c + lane;
            const uint32_t m = word < mw ? p.mask[(size_t)e * mw + word] : 0u;
            const int pc = __popc(m);
            int incl = pc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
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
        const int b = lane * chunk;
        int local = 0;
        for (int i = 0; i < chunk; i++)
            if (b + i < E) local += s_count[b + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
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
        if (lane == 31) {
            s_off[E] = incl;
            p.offsets[E] = incl;
        }
    }
    __syncthreads();
    if (warp == 0) {
        int nact = 0;
        for (int c = 0; c < E; c += 32) {
            const int e = c + lane;
            const bool act = e < E && s_count[e] > 0;
            const uint32_t bal = __ballot_sync(0xffffffffu, act);
            const int pos = nact + __popc(bal & ((1u << lane) - 1u));
            if (act) {
                Problem pr;
                pr.expert = e;
                pr.slot0 = s_off[e];
                pr.count = s_count[e];
                pr.is_shared = 0;
                p.problems[pos] = pr;
            }
            nact += __popc(bal);
        }
        if (lane == 0) {
            *p.n_active = nact;
            if (p.S > 0) {
                Problem pr;
                pr.expert = 0;
                pr.slot0 = p.T * p.k;
                pr.count = p.T;
                pr.is_shared = 1;
                p.problems[p.max_problems - 1] = pr;
            }
        }
    }
    for (int e = warp; e < E; e += nwarps) {
        if (s_count[e] == 0) continue;
        for (int c = 0; c < mw; c += 32) {
            const int word = c + lane;
            if (word < mw) {
                uint32_t m = p.mask[(size_t)e * mw + word];
                int pos = s_off[e] + p.wprefix[(size_t)e * mw + word];
                while (m) {
                    const int bit = __ffs(m) - 1;
                    p.perm_token[pos++] = word * 32 + bit;
                    m &= m - 1u;
                }
            }
        }
    }
    if (p.S > 0)
        for (int i = threadIdx.x; i < p.T; i += blockDim.x) p.perm_token[(size_t)p.T * p.k + i] = i;
}

// The same permutation for T <= 256 by the last CTA of the selection, in
// shared memory: per-expert token bit masks (shared-memory atomics on the
// selections), counts, slot offsets, problem list, slot -> token and the slot
// of each choice. No global masks are read or written.
__device__ void build_permutation_small(const FwdParams &p)
{
    __shared__ uint32_t s_mask[kMaxRouteExperts * kFusedMaskWords];
    __shared__ int s_wpre[kMaxRouteExperts * kFusedMaskWords];
    __shared__ int s_cnt[kMaxRouteExperts], s_off[kMaxRouteExperts + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = p.E, T = p.T, k = p.k, mw = p.mask_words, n = T * k;
    for (int i = threadIdx.x; i < E * mw; i += blockDim.x) s_mask[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = p.sel_idx[i], t = i / k;
        if (e >= 0) atomicOr(&s_mask[e * mw + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < mw; w++) {
            s_wpre[e * mw + w] = run;
            run += __popc(s_mask[e * mw + w]);
        }
        s_cnt[e] = run;
    }
    __syncthreads();
    if (warp == 0) {
        const int chunk = (E + 31) / 32, b = lane * chunk;
        int local = 0;
        for (int i = 0; i < chunk; i++)
            if (b + i < E) local += s_cnt[b + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < chunk; i++) {
            if (b + i < E) {
                s_off[b + i] = run;
                p.offsets[b + i] = run;
                run += s_cnt[b + i];
            }
        }
        if (lane == 31) {
            s_off[E] = incl;
            p.offsets[E] = incl;
        }
    }
    __syncthreads();
    if (warp == 1 || (blockDim.x == 32 && warp == 0)) {
        int nact = 0;
        for (int c = 0; c < E; c += 32) {
            const int e = c + lane;
            const bool act = e < E && s_cnt[e] > 0;
            const uint32_t bal = __ballot_sync(0xffffffffu, act);
            const int pos = nact + __popc(bal & ((1u << lane) - 1u));
            if (act) p.problems[pos] = Problem{e, s_off[e], s_cnt[e], 0};
            nact += __popc(bal);
        }
        if (lane == 0) {
            *p.n_active = nact;
            if (p.S > 0) p.problems[p.max_problems - 1] = Problem{0, T * k, T, 1};
        }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = p.sel_idx[i], t = i / k;
        int slot = -1;
        if (e >= 0) {
            const int w = e * mw + (t >> 5);
            slot = s_off[e] + s_wpre[w] + __popc(s_mask[w] & ((1u << (t & 31)) - 1u));
            p.perm_token[slot] = t;
        }
        p.slot_of[i] = slot;
    }
    if (p.S > 0)
        for (int i = threadIdx.x; i < T; i += blockDim.x) p.perm_token[(size_t)T * k + i] = i;
    if (threadIdx.x == 0) *p.sync = 0;   // ticket ready for the next selection
}

// Large batches: the router as a tiled f32 GEMM in the same canonical order.
// A CTA (16 warps) covers 32 tokens x 32 experts; warp (tg, eg) owns 8 tokens
// x 8 experts, lane l holding the partials of h4 = l (mod 32) for all 64, so
// every logit is still lane fmaf chains in increasing h plus the xor
// butterfly. Token and router rows are staged in shared memory 256 values at a
// time (cp.async, double-buffered), which cuts the L2 re-reads of the router
// rows by 4x and of the token rows by 2x against per-warp global loads.
constexpr int kRtTok = 32, kRtExp = 32, kRtChunk4 = 64;   // chunk: 64 float4 = 256 values


__global__ void __launch_bounds__(512, 1) router_tiled_kernel(FwdParams p)
{
    extern __shared__ float4 rt_smem[];   // [2][kRtTok + kRtExp][kRtChunk4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tg = warp & 3, eg = warp >> 2;
    const int t_base = blockIdx.y * kRtTok, e_base = blockIdx.x * kRtExp;
    const int H = p.H, E = p.E, T = p.T, n4 = H >> 2;
    const int nchunks = (n4 + kRtChunk4 - 1) / kRtChunk4;
    constexpr int kRows = kRtTok + kRtExp;

    auto stage = [&](int c, int buf) {
        float4 *dst = rt_smem + (size_t)buf * kRows * kRtChunk4;
        for (int i = threadIdx.x; i < kRows * kRtChunk4; i += blockDim.x) {
            const int r = i / kRtChunk4, c4 = i - r * kRtChunk4;
            const int h4 = c * kRtChunk4 + c4;
            const bool tok_row = r < kRtTok;
            const int g = tok_row ? t_base + r : e_base + (r - kRtTok);
            const bool valid = h4 < n4 && (tok_row ? g < T : g < E);
            const float *src = tok_row ? p.x + (size_t)(valid ? g : 0) * H : p.router + (size_t)(valid ? g : 0) * H;
            cp_async16(dst + i, reinterpret_cast<const float4 *>(src) + (valid ? h4 : 0), valid);
        }
        cp_async_commit();
    };

    float acc[8][8];
#pragma unroll
    for (int t = 0; t < 8; t++)
#pragma unroll
        for (int e = 0; e < 8; e++) acc[t][e] = 0.0f;

    stage(0, 0);
    for (int c = 0; c < nchunks; c++) {
        if (c + 1 < nchunks) {
            stage(c + 1, (c + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float4 *xs = rt_smem + (size_t)(c & 1) * kRows * kRtChunk4;
        const float4 *ws = xs + kRtTok * kRtChunk4;
#pragma unroll
        for (int j = 0; j < kRtChunk4 / 32; j++) {
            const int c4 = lane + 32 * j;
            if (c * kRtChunk4 + c4 < n4) {
                float4 w[8];
#pragma unroll
                for (int e = 0; e < 8; e++) w[e] = ws[(eg * 8 + e) * kRtChunk4 + c4];
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const float4 xv = xs[(tg * 8 + t) * kRtChunk4 + c4];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        acc[t][e] = __fmaf_rn(w[e].x, xv.x, acc[t][e]);
                        acc[t][e] = __fmaf_rn(w[e].y, xv.y, acc[t][e]);
                        acc[t][e] = __fmaf_rn(w[e].z, xv.z, acc[t][e]);
                        acc[t][e] = __fmaf_rn(w[e].w, xv.w, acc[t][e]);
                    }
                }
            }
        }
        __syncthreads();   // the buffer is refilled by the next iteration's stage
    }
#pragma unroll
    for (int t = 0; t < 8; t++) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float v = acc[t][e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            const int tok = t_base + tg * 8 + t, ex = e_base + eg * 8 + e;
            if (lane == ((t * 8 + e) & 31) && tok < T && ex < E) {
                if (p.logit_bias) v = __fadd_rn(v, p.logit_bias[ex]);
                p.logits[(size_t)tok * E + ex] = v;
            }
        }
    }
    // activation blocks of this CTA's tokens, shared over the expert tiles
    if (p.quant_x) {
        const int ntok = min(kRtTok, T - t_base);
        if (ntok > 0) quantize_tile(p, t_base, ntok, blockIdx.x * 16 + warp, gridDim.x * 16, lane);
    }
}

// Routing of a small batch (T <= 256) in one kernel. Logits in the canonical
// order of router_kernel, with the token tile staged in shared memory and each
// warp's router row held in registers 2048 values at a time (one DRAM round
// trip per 2048 values). The last CTA of a token tile to finish (ticket
// sync[1 + tile]) selects its TT tokens, one warp each; the last token tile
// (ticket sync[0]) builds the dispatch permutation. Tickets return to zero.
template <int TT, int NL>
__global__ void __launch_bounds__(128) router_small_kernel(FwdParams p)
{
    static_assert(TT == 4, "one selecting warp per token of the tile");
    pdl_wait();      // launched as a dependent: the previous forward's last kernel is done
    pdl_trigger();
    extern __shared__ float4 xs4[];   // [TT][H/4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 4 + warp;
    const int t0 = blockIdx.y * TT;
    const int H = p.H, E = p.E, n4 = H >> 2;
    const int ntok = min(TT, p.T - t0);
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *wr = reinterpret_cast<const float4 *>(p.router + (size_t)min(e, E - 1) * H);

    // issue the first row chunk before staging the tile, so both loads overlap
    float4 w[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int h4 = lane + 32 * i;
        w[i] = h4 < n4 ? __ldg(wr + h4) : zero4;
    }
    // the tile by asynchronous copies, all in flight at once (rows past the
    // batch are zero-filled)
    for (int i = threadIdx.x; i < TT * n4; i += blockDim.x) {
        const int t = i / n4, c = i - t * n4;
        const bool ok = t < ntok;
        cp_async16(xs4 + i, reinterpret_cast<const float4 *>(p.x + (size_t)(t0 + (ok ? t : 0)) * H) + c, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; t++) acc[t] = 0.0f;
    for (int base = 0; base < n4; base += 512) {
        if (base > 0) {
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int h4 = base + lane + 32 * i;
                w[i] = h4 < n4 ? __ldg(wr + h4) : zero4;
            }
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int h4 = base + lane + 32 * i;
            if (h4 < n4) {
#pragma unroll
                for (int t = 0; t < TT; t++) {
                    const float4 xv = xs4[t * n4 + h4];
                    acc[t] = __fmaf_rn(w[i].x, xv.x, acc[t]);
                    acc[t] = __fmaf_rn(w[i].y, xv.y, acc[t]);
                    acc[t] = __fmaf_rn(w[i].z, xv.z, acc[t]);
                    acc[t] = __fmaf_rn(w[i].w, xv.w, acc[t]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TT; t++) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0 && t < ntok && e < E) {
            if (p.logit_bias) v = __fadd_rn(v, p.logit_bias[e]);
            p.logits[(size_t)(t0 + t) * E + e] = v;
        }
    }
    if (p.quant_x) quantize_tile(p, t0, ntok, blockIdx.x * 4 + warp, gridDim.x * 4, lane);

    __shared__ int s_flag;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_flag = atomicAdd(&p.sync[1 + blockIdx.y], 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();   // the tile's logits from every CTA are visible
    if (t0 + warp < p.T) select_token<NL>(p, t0 + warp, lane);
    __syncthreads();
    if (gridDim.y == 1) {   // one token tile: this CTA saw every selection, no second ticket
        if (threadIdx.x == 0) p.sync[1] = 0;
        __threadfence();
        build_permutation_small(p);
        return;
    }
    if (threadIdx.x == 0) {
        p.sync[1 + blockIdx.y] = 0;
        __threadfence();
        s_flag = atomicAdd(&p.sync[0], 1) == (int)gridDim.y - 1;
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    build_permutation_small(p);
}

// One warp per token. With FUSE_SCAN (1024-thread CTAs, T <= 256) the last
// CTA to finish (a fence and a ticket on p.sync) also builds the dispatch
// permutation, so small batches need no separate scan launch; that CTA sets
// the ticket back to zero. Without it the selections go to the global masks
// for scan_kernel.
template <bool FUSE_SCAN, int NL>
__global__ void __launch_bounds__(FUSE_SCAN ? 1024 : 128, 1) select_kernel(FwdParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t < p.T) select_token<NL>(p, t, lane);
    if (!FUSE_SCAN) return;
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(p.sync, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    build_permutation_small(p);
}

__global__ void __launch_bounds__(1024) scan_kernel(FwdParams p)
{
    extern __shared__ int s_scan[];
    build_permutation(p, s_scan, s_scan + p.E);
}

// ------------------------------------------------------------ parity probes

__global__ void quantize_rows_kernel(const float *x, int n, int cols, int8_t *xq, float *xd, float *xs)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = cols >> 5;
    if (warp >= n * nb) return;
    const int r = warp / nb, b = warp % nb;
    quant_block32(x[(size_t)r * cols + 32 * b + lane], xq + (size_t)r * cols + 32 * b, xd + (size_t)r * nb + b,
                  xs + (size_t)r * nb + b, lane);
}

// Integer block sums with the dot routines of the expert kernels.
template <int FMT>
__global__ void block_dots_kernel(DevMatrix m, const int8_t *xq, int n, int32_t *isum)
{
    const int nb = m.cols >> 5;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nb) return;
    const int r = i / nb, u = i % nb;
    const uint8_t *qrow = m.qs + (size_t)r * m.qs_rstride;
    const int4 *x = reinterpret_cast<const int4 *>(xq + (size_t)r * m.cols + 32 * u);
    if (FMT == FMT_Q4_K) {
        const Q4Nib nb4 = q4_nibbles(*reinterpret_cast<const uint4 *>(qrow + 16 * (size_t)u));
        isum[i] = q4_isum16(nb4, x[0], x[1]) >> 4;   // exact: the sum is a multiple of 16
    } else {
        const uint4 *q = reinterpret_cast<const uint4 *>(qrow + 32 * (size_t)u);
        isum[i] = q8_isum(q[0], q[1], x[0], x[1]);
    }
}

cudaError_t launch_router(const FwdParams &p, cudaStream_t st)
{
    if (p.T <= 256) {
        dim3 grid((p.E + 3) / 4, (p.T + 3) / 4);
        router_kernel<4, 1><<<grid, 128, 0, st>>>(p);
    } else if ((p.H & 3) == 0) {
        const size_t smem = 2 * (size_t)(kRtTok + kRtExp) * kRtChunk4 * sizeof(float4);
        static size_t opted[64] = {};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64 || opted[dev] < smem) {
            e = cudaFuncSetAttribute(router_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) opted[dev] = smem;
        }
        dim3 grid((p.E + kRtExp - 1) / kRtExp, (p.T + kRtTok - 1) / kRtTok);
        router_tiled_kernel<<<grid, 512, smem, st>>>(p);
    } else {
        dim3 grid((p.E + 15) / 16, (p.T + 7) / 8);
        router_kernel<8, 4><<<grid, 128, 0, st>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t clear_routing_state(const FwdParams &p, cudaStream_t st)
{
    // small batches keep their masks in shared memory and reset their own
    // tickets; larger ones need zeroed global masks (tickets included)
    if (p.T <= kFusedScanMaxT) return cudaSuccess;
    return cudaMemsetAsync(p.sync, 0, kRoutingTicketBytes + sizeof(uint32_t) * (size_t)p.E * p.mask_words, st);
}

cudaError_t launch_select(const FwdParams &p, cudaStream_t st)
{
    if (p.E > kMaxRouteExperts) return cudaErrorInvalidValue;
    const bool small_e = p.E <= 128;
    if (p.T <= kFusedScanMaxT) {
        if (small_e) select_kernel<true, 4><<<(p.T + 31) / 32, 1024, 0, st>>>(p);
        else select_kernel<true, 8><<<(p.T + 31) / 32, 1024, 0, st>>>(p);
        return cudaGetLastError();
    }
    if (small_e) select_kernel<false, 4><<<(p.T + 3) / 4, 128, 0, st>>>(p);
    else select_kernel<false, 8><<<(p.T + 3) / 4, 128, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    scan_kernel<<<1, 1024, sizeof(int) * (2 * (size_t)p.E + 1), st>>>(p);
    return cudaGetLastError();
}

template <int NL>
cudaError_t launch_routing_small(const FwdParams &p, cudaStream_t st)
{
    constexpr int TT = 4;
    const size_t smem = (size_t)TT * p.H * 4;
    // the kernel also has static shared memory (the permutation), so the dynamic
    // part needs the opt-in attribute; set once per device and size
    static size_t opted[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || opted[dev] < smem) {
        e = cudaFuncSetAttribute(router_small_kernel<TT, NL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) opted[dev] = smem;
    }
    dim3 grid((p.E + 3) / 4, (p.T + TT - 1) / TT);
    return launch_dependent(router_small_kernel<TT, NL>, grid, dim3(128), smem, st, p);
}

}  // namespace

cudaError_t launch_routing(const FwdParams &p, cudaStream_t st, const Marker &mk)
{
    cudaError_t e;
    if (p.E > kMaxRouteExperts) return cudaErrorInvalidValue;
    // one kernel when the token tile fits in shared memory and the tile tickets in their region
    if (p.T <= kFusedScanMaxT && (p.H & 3) == 0 && p.H <= 12288 && 4 * (1 + (p.T + 3) / 4) <= kRoutingTicketBytes) {
        e = p.E <= 128 ? launch_routing_small<4>(p, st) : launch_routing_small<8>(p, st);
        if (e != cudaSuccess) return e;
        mk.mark("routing");
        return cudaSuccess;
    }
    if ((e = clear_routing_state(p, st)) != cudaSuccess) return e;
    if ((e = launch_router(p, st)) != cudaSuccess) return e;
    mk.mark("router");
    if ((e = launch_select(p, st)) != cudaSuccess) return e;
    mk.mark("select");
    return cudaSuccess;
}

int launch_quantize_rows(const float *x, int n, int cols, int8_t *xq, float *xd, float *xs, void *stream)
{
    const int warps = n * (cols / 32);
    quantize_rows_kernel<<<(warps + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, cols, xq, xd, xs);
    return cudaGetLastError();
}

int launch_block_dots(const DevMatrix &m, const int8_t *xq, int n, int32_t *isum, void *stream)
{
    const int tot = n * (m.cols / 32);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (m.type == FMT_Q4_K)
        block_dots_kernel<FMT_Q4_K><<<(tot + 255) / 256, 256, 0, st>>>(m, xq, n, isum);
    else
        block_dots_kernel<FMT_Q8_0><<<(tot + 255) / 256, 256, 0, st>>>(m, xq, n, isum);
    return cudaGetLastError();
}

}  // namespace jmoe

// ------------------------------------------------------------ FFN pre-norm

namespace jmoe {
namespace {

// RMSNorm of one token per warp in the fixed order shared with the oracle
// (orc_rmsnorm): element h feeds lane partial (h/4) mod 32 as x*x fmaf chains
// in increasing h, the xor butterfly 16..1 adds the partials, then
// mean = sum / H, inv = 1 / sqrt(mean + eps), y = (x * inv) * w, each step
// rounded once. Semantics of rmsnorm_standard (src/qwen_deepseek.rs:521-528),
// whose kernel (jero-kernels-rvv) fixes no order.
__global__ void __launch_bounds__(128) rmsnorm_kernel(FwdParams p)
{
    pdl_wait();   // the previous sublayer may still be writing the residual stream
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + warp;
    if (t >= p.T) return;
    const int H = p.H;
    const float *x = p.norm_in + (size_t)t * H;
    float *y = p.norm_out + (size_t)t * H;
    float acc = 0.0f;
    for (int hb = 4 * lane; hb < H; hb += 128)
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (hb + c < H) acc = __fmaf_rn(x[hb + c], x[hb + c], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    const float mean = __fdiv_rn(acc, (float)H);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.norm_eps)));
    for (int h = lane; h < H; h += 32) y[h] = __fmul_rn(__fmul_rn(x[h], inv), p.norm_w[h]);
}

}  // namespace

cudaError_t launch_rmsnorm(const FwdParams &p, cudaStream_t st)
{
    return launch_dependent(rmsnorm_kernel, dim3((p.T + 3) / 4), dim3(128), 0, st, p);
}

}  // namespace jmoe
