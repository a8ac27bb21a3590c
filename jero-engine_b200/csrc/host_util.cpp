// host_util.cpp -- the repository's GGUF quantiser and seeded input generator
// (host code; used to build synthetic layers for tests and the bench).
#include <math.h>

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/jeromoe.h"
#include "layout.h"

namespace {

// IEEE binary32 -> binary16, round to nearest even (overflow -> inf).
uint16_t f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);   // rounds past 65504
    if (ax < 0x38800000u) {                                      // below the f16 normal range
        if (ax < 0x33000000u) return (uint16_t)sign;             // below half the smallest subnormal
        const uint32_t man = (ax & 0x7FFFFFu) | 0x800000u;
        const int shift = 126 - (int)(ax >> 23);                 // 14 + (113 - exp)
        uint32_t r = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax >> 23) - 112) << 10 | ((ax >> 13) & 0x3FFu);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (!man) bits = sign;
        else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }

// Q8_0: d = amax/127 stored as f16, q = round(x / d_f16) clamped to +-127.
void quant_q8_0_row(const float *x, int cols, uint8_t *dst)
{
    for (int b = 0; b < cols / 32; b++) {
        const float *v = x + 32 * b;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = std::max(amax, fabsf(v[i]));
        const uint16_t dh = f32_to_f16(amax / 127.0f);
        const float d = f16_to_f32(dh);
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        uint8_t *o = dst + 34 * b;
        put16(o, dh);
        for (int i = 0; i < 32; i++) {
            float r = roundf(v[i] * id);
            r = std::min(127.0f, std::max(-127.0f, r));
            o[2 + i] = (uint8_t)(int8_t)r;
        }
    }
}

// Q4_K (asymmetric 4-bit with 6-bit sub-block scale and min): per 32-value
// sub-block j, scale_j = (max - min)/15 and min_j = -min (min clamped to <= 0);
// super-block d = max scale_j / 63, dmin = max min_j / 63 (f16); sc_j, m_j are
// the 6-bit ratios to the stored d / dmin; q = round((x + dmin*m_j) / (d*sc_j)).
void quant_q4_k_row(const float *x, int cols, uint8_t *dst)
{
    for (int s = 0; s < cols / 256; s++) {
        const float *v = x + 256 * s;
        float scale[8], mn[8];
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = -INFINITY;
            for (int i = 0; i < 32; i++) {
                lo = std::min(lo, v[32 * j + i]);
                hi = std::max(hi, v[32 * j + i]);
            }
            scale[j] = (hi - lo) / 15.0f;
            mn[j] = -lo;
        }
        float ms = 0.0f, mm = 0.0f;
        for (int j = 0; j < 8; j++) { ms = std::max(ms, scale[j]); mm = std::max(mm, mn[j]); }
        const uint16_t dh = f32_to_f16(ms / 63.0f), mh = f32_to_f16(mm / 63.0f);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        int sc[8], m[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.0f ? (int)std::min(63.0f, std::max(0.0f, roundf(scale[j] / d))) : 0;
            m[j] = dmin > 0.0f ? (int)std::min(63.0f, std::max(0.0f, roundf(mn[j] / dmin))) : 0;
        }
        uint8_t *o = dst + 144 * s;
        put16(o, dh);
        put16(o + 2, mh);
        uint8_t *sc12 = o + 4;
        for (int j = 0; j < 4; j++) {
            sc12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            sc12[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            sc12[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
        }
        uint8_t q[256];
        for (int j = 0; j < 8; j++) {
            const float ds = d * (float)sc[j], dm = dmin * (float)m[j];
            for (int i = 0; i < 32; i++) {
                float r = ds > 0.0f ? roundf((v[32 * j + i] + dm) / ds) : 0.0f;
                q[32 * j + i] = (uint8_t)std::min(15.0f, std::max(0.0f, r));
            }
        }
        uint8_t *qs = o + 16;
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
    }
}

inline uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename F>
void parallel_for(int64_t n, int threads, F f)
{
    threads = std::max(1, std::min<int>(threads, (int)std::min<int64_t>(n, 256)));
    if (threads == 1) { f(0, n); return; }
    std::vector<std::thread> pool;
    const int64_t chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; t++) {
        int64_t a = t * chunk, b = std::min(n, a + chunk);
        if (a >= b) break;
        pool.emplace_back([=] { f(a, b); });
    }
    for (auto &th : pool) th.join();
}

}  // namespace

extern "C" {

int moe_quantize_rows(int32_t quant, const float *src, int64_t rows, int32_t cols, void *dst, int32_t n_threads)
{
    if (!src || !dst || rows < 0) return MOE_ERR_INVALID_ARGS;
    const size_t rb = jmoe::gguf_row_bytes(quant, cols);
    if (!rb || (quant != MOE_QUANT_Q8_0 && quant != MOE_QUANT_Q4_K && quant != MOE_QUANT_F32))
        return MOE_ERR_CAPABILITY_MISMATCH;
    uint8_t *out = static_cast<uint8_t *>(dst);
    parallel_for(rows, n_threads, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; r++) {
            const float *x = src + r * cols;
            uint8_t *o = out + r * rb;
            if (quant == MOE_QUANT_F32) memcpy(o, x, rb);
            else if (quant == MOE_QUANT_Q8_0) quant_q8_0_row(x, cols, o);
            else quant_q4_k_row(x, cols, o);
        }
    });
    return MOE_OK;
}

// Normal pair m of stream (seed, s): u1 = (mix(k + (2m+1)G) >> 11 + 1) / 2^53,
// u2 = (mix(k + (2m+2)G) >> 11) / 2^53 with k = mix(seed ^ mix(s + G)) and G the
// splitmix64 increment; z = sqrt(-2 ln u1) * (cos, sin)(2 pi u2), times sigma.
int moe_gen_normal(uint64_t seed, uint64_t stream, uint64_t n, float sigma, float *dst, int32_t n_threads)
{
    if (!dst) return MOE_ERR_INVALID_ARGS;
    const uint64_t G = 0x9E3779B97F4A7C15ull;
    const uint64_t key = mix64(seed ^ mix64(stream + G));
    const int64_t pairs = (int64_t)((n + 1) / 2);
    parallel_for(pairs, n_threads, [&](int64_t a, int64_t b) {
        for (int64_t m = a; m < b; m++) {
            const uint64_t r1 = mix64(key + (uint64_t)(2 * m + 1) * G);
            const uint64_t r2 = mix64(key + (uint64_t)(2 * m + 2) * G);
            const double u1 = (double)((r1 >> 11) + 1) * 0x1.0p-53;
            const double u2 = (double)(r2 >> 11) * 0x1.0p-53;
            const double rad = sqrt(-2.0 * log(u1));
            const double th = 6.283185307179586 * u2;
            dst[2 * m] = (float)(rad * cos(th) * (double)sigma);
            if ((uint64_t)(2 * m + 1) < n) dst[2 * m + 1] = (float)(rad * sin(th) * (double)sigma);
        }
    });
    return MOE_OK;
}

}  // extern "C"
