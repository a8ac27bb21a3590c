// common.cuh -- device helpers shared by the MoE kernels: ranking keys, warp
// reductions, the activation block quantiser and the quantised weight units.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "moe_device.h"

namespace jmoe {

constexpr int kTT = 8;         // tokens per expert-kernel tile
constexpr int kMaxK = 16;      // largest top_k
constexpr int kMaxLaneE = 8;   // experts per lane in topk (E <= 256)

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

__device__ __forceinline__ int byte_of(uint32_t a, uint32_t b, uint32_t c, int i)
{
    uint32_t w = i < 4 ? a : (i < 8 ? b : c);
    return (int)((w >> (8 * (i & 3))) & 0xFFu);
}

// One 32-value block of a quantised row (a Q8_0 block or a Q4_K sub-block)
// in the device layout, held in registers and dotted against many tokens.
// load() reads from global or shared memory through a generic pointer.
template <int FMT>
struct WUnit;

template <>
struct WUnit<FMT_Q4_K> {
    uint4 q;
    float dsc, dmn;
    __device__ __forceinline__ void load(const uint8_t *qs_row, const uint8_t *meta_row, int u)
    {
        q = *reinterpret_cast<const uint4 *>(qs_row + 16 * (size_t)u);
        const uint4 m = *reinterpret_cast<const uint4 *>(meta_row + 16 * (size_t)(u >> 3));
        const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
        const int j = u & 7;
        int sc, mn;
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
    __device__ __forceinline__ void load(const uint8_t *qs_row, const uint8_t *meta_row, int u)
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(qs_row + 32 * (size_t)u);
        q0 = src[0];
        q1 = src[1];
        d = __half2float(__ushort_as_half(reinterpret_cast<const unsigned short *>(meta_row)[u]));
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

// SiLU(g) * u with silu(g) = g / (1 + exp(-g)), each operation rounded (the oracle's form).
__device__ __forceinline__ float swiglu(float g, float u)
{
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

}  // namespace jmoe
