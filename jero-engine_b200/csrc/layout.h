// layout.h -- GGUF block formats and the device layout sizes (host side).
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "moe_device.h"

namespace jmoe {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// GGUF bytes of one row (0 if cols is not a whole number of blocks).
inline size_t gguf_row_bytes(int type, int64_t cols)
{
    if (cols <= 0) return 0;
    switch (type) {
    case FMT_F32: return (size_t)cols * 4;
    case FMT_Q8_0: return (cols % 32) ? 0 : (size_t)(cols / 32) * 34;
    case FMT_Q4_K: return (cols % 256) ? 0 : (size_t)(cols / 256) * 144;
    default: return 0;
    }
}

// Device-layout row strides (see moe_device.h). Meta rows are padded to 16
// bytes so that every row (and every 256-value slice of it) starts on a bulk-copy boundary.
inline void dev_row_strides(int type, int cols, size_t *qs_r, size_t *meta_r)
{
    switch (type) {
    case FMT_F32: *qs_r = (size_t)cols * 4; *meta_r = 0; break;
    case FMT_Q8_0: *qs_r = (size_t)cols; *meta_r = align_up((size_t)(cols / 32) * 2, 16); break;
    default: *qs_r = (size_t)cols / 2; *meta_r = (size_t)(cols / 256) * 16; break;
    }
}

// Q4_K super-block header in the device layout: f16 d, f16 dmin as in GGUF,
// then the eight 6-bit scales and mins regrouped as 12-bit fields
// (sc_j | m_j << 6) at bit 12j, so a lane decodes its sub-block with one
// funnel shift. GGUF packs them as: j < 4: low 6 bits of byte j (scale) and
// byte j+4 (min); j >= 4: a nibble of byte j+4 plus the top two bits of byte
// j-4 (scale) / byte j (min).
inline void q4k_meta(const uint8_t *gguf_blk, uint8_t *out16)
{
    const uint8_t *s = gguf_blk + 4;
    memcpy(out16, gguf_blk, 4);
    uint32_t w[3] = {0, 0, 0};
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        if (j < 4) {
            sc = s[j] & 63;
            mn = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
            mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const uint64_t f = (uint64_t)(sc | (mn << 6)) << (12 * j % 32);
        const int wi = 12 * j / 32;
        w[wi] |= (uint32_t)f;
        if (wi < 2) w[wi + 1] |= (uint32_t)(f >> 32);
    }
    memcpy(out16 + 4, w, 12);
}

struct MatrixPlan {
    int type, rows, cols, n_experts;
    size_t qs_rstride, meta_rstride, qs_estride, meta_estride;
    size_t qs_bytes, meta_bytes;   // whole stack
};

inline MatrixPlan plan_matrix(int type, int rows, int cols, int n_experts)
{
    MatrixPlan m;
    m.type = type; m.rows = rows; m.cols = cols; m.n_experts = n_experts;
    dev_row_strides(type, cols, &m.qs_rstride, &m.meta_rstride);
    m.qs_estride = align_up(m.qs_rstride * rows, 128);
    m.meta_estride = align_up(m.meta_rstride * rows, 128);
    m.qs_bytes = m.qs_estride * n_experts;
    m.meta_bytes = m.meta_estride * n_experts;
    return m;
}

// Reorders the GGUF rows of a stack into the device layout. src holds
// n_experts * rows GGUF rows back to back; qs/meta receive the device bytes.
//   Q8_0: quants and f16 scales split into two arrays.
//   Q4_K: the 16-byte header (d, dmin, scales) of each super-block goes to meta
//         with its scales regrouped (q4k_meta); the 128 nibble bytes are regrouped per 32-value sub-block j
//         so that byte b of sub-block j holds value 32j+b (low) and 32j+16+b (high).
//         In GGUF, value 64g+l (l<32) is the low nibble of byte 32g+l and value
//         64g+32+l its high nibble.
inline void repack_rows(const MatrixPlan &m, const uint8_t *src, uint8_t *qs, uint8_t *meta)
{
    const size_t rb = gguf_row_bytes(m.type, m.cols);
    for (int e = 0; e < m.n_experts; e++) {
        for (int r = 0; r < m.rows; r++) {
            const uint8_t *row = src + ((size_t)e * m.rows + r) * rb;
            uint8_t *dq = qs + (size_t)e * m.qs_estride + (size_t)r * m.qs_rstride;
            uint8_t *dm = meta ? meta + (size_t)e * m.meta_estride + (size_t)r * m.meta_rstride : nullptr;
            if (m.type == FMT_F32) {
                memcpy(dq, row, rb);
            } else if (m.type == FMT_Q8_0) {
                for (int b = 0; b < m.cols / 32; b++) {
                    memcpy(dm + 2 * b, row + 34 * b, 2);
                    memcpy(dq + 32 * b, row + 34 * b + 2, 32);
                }
            } else {
                for (int s = 0; s < m.cols / 256; s++) {
                    const uint8_t *blk = row + 144 * s;
                    q4k_meta(blk, dm + 16 * s);
                    const uint8_t *g = blk + 16;
                    uint8_t nib[256];
                    for (int gi = 0; gi < 4; gi++)
                        for (int l = 0; l < 32; l++) {
                            nib[64 * gi + l] = g[32 * gi + l] & 0x0F;
                            nib[64 * gi + 32 + l] = g[32 * gi + l] >> 4;
                        }
                    uint8_t *o = dq + 128 * s;
                    for (int j = 0; j < 8; j++)
                        for (int b = 0; b < 16; b++)
                            o[16 * j + b] = (uint8_t)(nib[32 * j + b] | (nib[32 * j + 16 + b] << 4));
                }
            }
        }
    }
}

}  // namespace jmoe
