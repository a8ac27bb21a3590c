// common.cuh -- device helpers shared by the MoE kernels: ranking keys, warp
// reductions, the activation block quantiser and the quantised block dots.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "moe_device.h"

namespace jmoe {

constexpr int kTT = 8;         // tokens per expert-kernel tile
constexpr int kMaxK = 16;      // largest top_k
constexpr int kMaxLaneE = 8;   // experts per lane in topk (E <= 256)
constexpr int kMaxRouteExperts = 32 * kMaxLaneE;

// Rust f32::total_cmp order as a signed integer (src/gemma.rs:417).
__device__ __forceinline__ int32_t total_key(float f)
{
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// (ka, ia) ranks before (kb, ib): larger key first, ties to the lower index.
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

// Activation block quantiser (the oracle's orc_quantize_act): the 32 lanes of
// a warp hold the 32 values of one block. q = clamp(round(v * 127/amax), -127,
// 127) with NaN -> -127 (fmaxf keeps the non-NaN operand), d = amax/127;
// s = d * sum(q) feeds the min term of Q4_K dots.
__device__ __forceinline__ void quant_block32(float v, int8_t *q_out, float *d_out, float *s_out, int lane)
{
    float amax = fmaxf(warp_max(fabsf(v)), 0.0f);   // all-NaN block -> 0, as the oracle's running max from 0
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

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Exact int -> float for |v| < 2^22 with an integer add and a float add
// (keeps the conversion off the slow pipe).
__device__ __forceinline__ float i2f_small(int v)
{
    return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

// ---- Q4_K sub-block (32 values, 16 bytes of nibbles in the device layout:
// byte b = value b (low nibble) | value 16 + b (high nibble)) ----

// Nibbles of one sub-block prepared once for many tokens: lo holds values
// 0..15 as bytes, hi16 values 16..31 times 16 (the high nibble left in place).
struct Q4Nib {
    uint32_t lo[4], hi16[4];
};

__device__ __forceinline__ Q4Nib q4_nibbles(uint4 q)
{
    Q4Nib n;
    n.lo[0] = q.x & 0x0F0F0F0Fu; n.hi16[0] = q.x & 0xF0F0F0F0u;
    n.lo[1] = q.y & 0x0F0F0F0Fu; n.hi16[1] = q.y & 0xF0F0F0F0u;
    n.lo[2] = q.z & 0x0F0F0F0Fu; n.hi16[2] = q.z & 0xF0F0F0F0u;
    n.lo[3] = q.w & 0x0F0F0F0Fu; n.hi16[3] = q.w & 0xF0F0F0F0u;
    return n;
}

// 16 * sum(q * x) over the sub-block; a holds x[0..15], b holds x[16..31].
__device__ __forceinline__ int q4_isum16(const Q4Nib &n, int4 a, int4 b)
{
    int lo = dp4a_us(n.lo[0], a.x, 0);
    int hi = dp4a_us(n.hi16[0], b.x, 0);
    lo = dp4a_us(n.lo[1], a.y, lo);
    hi = dp4a_us(n.hi16[1], b.y, hi);
    lo = dp4a_us(n.lo[2], a.z, lo);
    hi = dp4a_us(n.hi16[2], b.z, hi);
    lo = dp4a_us(n.lo[3], a.w, lo);
    hi = dp4a_us(n.hi16[3], b.w, hi);
    return lo * 16 + hi;
}

// Q4_K scale and min of sub-block j from the device meta (16 bytes per
// super-block: f16 d, f16 dmin, then eight 12-bit fields sc_j | m_j << 6 at
// bit 12j of the remaining 96 bits). Returns (d*sc_j/16, dmin*m_j).
__device__ __forceinline__ float2 q4_scales(uint4 m, int j)
{
    const int bit = 12 * j, wi = bit >> 5, sh = bit & 31;
    const uint32_t lo = wi == 0 ? m.y : (wi == 1 ? m.z : m.w);
    const uint32_t hi = wi == 0 ? m.z : (wi == 1 ? m.w : 0u);
    const uint32_t f = __funnelshift_r(lo, hi, sh) & 0xFFFu;
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&m.x));
    return make_float2(dd.x * (float)(f & 63u) * 0.0625f, dd.y * (float)(f >> 6));
}

// ---- Q8_0 block (32 signed bytes, f16 scale) ----
__device__ __forceinline__ int q8_isum(uint4 q0, uint4 q1, int4 a, int4 b)
{
    int s0 = __dp4a((int)q0.x, a.x, 0);
    int s1 = __dp4a((int)q1.x, b.x, 0);
    s0 = __dp4a((int)q0.y, a.y, s0);
    s1 = __dp4a((int)q1.y, b.y, s1);
    s0 = __dp4a((int)q0.z, a.z, s0);
    s1 = __dp4a((int)q1.z, b.z, s1);
    s0 = __dp4a((int)q0.w, a.w, s0);
    s1 = __dp4a((int)q1.w, b.w, s1);
    return s0 + s1;
}

// SiLU(g) * u with silu(g) = g / (1 + exp(-g)), each operation rounded (the oracle's form).
// Row of y that holds the expert output of slot s.
__device__ __forceinline__ size_t y_row(const FwdParams &p, size_t s);

// Output row of slot s: this rank's y, or (expert parallel, fused launch) the
// source rank's output inbox over peer memory.
__device__ __forceinline__ float *y_dst(const FwdParams &p, size_t s)
{
    if (p.y_peer) {
        const int2 rr = p.y_ret[s];
        return reinterpret_cast<float *>(p.y_peer[rr.x] + p.y_peer_off) + (size_t)rr.y * p.H;
    }
    return p.y + y_row(p, s) * p.H;
}

__device__ __forceinline__ size_t y_row(const FwdParams &p, size_t s)
{
    return p.y_rows ? (size_t)p.y_rows[s] : s;
}

__device__ __forceinline__ float swiglu(float g, float u)
{
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

}  // namespace jmoe
