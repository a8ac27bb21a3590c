/*
 * moe_oracle.h -- CPU restatement of jero-engine's mixture-of-experts FFN path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path in
 * libjeromoe.so: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it. The product path never calls it.
 *
 * What it restates (paths are relative to the jero-engine source tree):
 *   - dispatch_qwen3_moe_ffn            src/qwen_deepseek.rs:847-951
 *   - select_experts_with_optional_bias src/qwen_deepseek.rs:773-831
 *   - run_single_swiglu_expert          src/qwen_deepseek.rs:748-771
 *   - select_top_k_experts              src/gemma.rs:362-442
 *   - matvec_any / matvec_f32 row split src/gemma.rs:100-189
 *   - per-token prefill loop            src/qwen_deepseek.rs:2298-2312
 *
 * Parity status. The arithmetic kernels behind the path live in the
 * un-vendored crate jero-kernels-rvv @ 93a778ef690ac2171aab915f7b58daf5d8bbfe79
 * (Cargo.lock:456-458): vec_dot_q8_0, BaselineKernel::vec_dot_q4_k_m,
 * swiglu_f32, dot_product_f32_scalar. No reference test pins their numeric
 * output, so this oracle DEFINES them (int8 activation blocks of 32 with an
 * f32 scale, int32 block sums, f32 scaling; a fixed f32 summation tree for
 * the router). Routing, tie-breaking, renormalisation, the shared-expert and
 * combine order, the GGUF block layouts and the dequantisation rules are
 * pinned by the reference's own tests (restated in tests/golden/).
 */
#ifndef JERO_MOE_ORACLE_H
#define JERO_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF ggml_type ids (the reference's QuantType variants of the same name). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12 };

enum {
    ORC_OK = 0,
    ORC_ERR_ARG = 1,       /* bad shape / unsupported type */
    ORC_ERR_NOMEM = 2
};

/* One weight matrix or a stack of per-expert matrices in GGUF byte layout:
 * row r of expert e starts at data + e*expert_stride + r*row_bytes(type, cols). */
typedef struct orc_matrix {
    int32_t type;
    int32_t rows;             /* output features */
    int32_t cols;             /* input features (contiguous) */
    int32_t _pad;
    const uint8_t *data;      /* NULL: tensor absent */
    uint64_t expert_stride;   /* bytes between consecutive experts (stacks) */
} orc_matrix;

/* Routing options. Fields marked [build] have no counterpart in the
 * reference (which only renormalises and only supports exp_probs_b). */
typedef struct orc_layer {
    int32_t hidden;           /* H */
    int32_t n_experts;        /* E */
    int32_t top_k;            /* k */
    int32_t normalize;        /* 1: renormalise selected weights (reference) */
    float   scale;            /* [build] routed scaling factor, applied when normalize==0 */
    int32_t n_groups;         /* [build] group-limited top-k: groups (0 = off) */
    int32_t topk_groups;      /* [build] groups kept */
    int32_t _pad;
    const float *router;      /* [E][H] f32, blk.L.ffn_gate_inp.weight */
    const float *sel_bias;    /* [E] or NULL: blk.L.exp_probs_b.bias (selection only) */
    const float *logit_bias;  /* [E] or NULL: [build] added to logits before routing */
    orc_matrix gate, up, down;            /* stacks: gate/up [I x H], down [H x I] per expert */
    orc_matrix sh_gate, sh_up, sh_down;   /* shared expert (data NULL if absent) */
} orc_layer;

/* ---- formats ---- */
float    orc_f16_to_f32(uint16_t h);
size_t   orc_row_bytes(int type, int cols);      /* 0 if cols not allowed */
int      orc_dequantize_row(int type, const uint8_t *row, int cols, float *dst);

/* ---- activation blocks (int8 per 32 values + f32 scale) ---- */
int  orc_quantize_act(const float *x, int cols, int8_t *xq, float *dx);
/* int32 sums of each 32-wide block: isum[b] = sum w_q * x_q; for Q4_K also
 * xsum[b] = sum x_q (the term that multiplies the block min). */
int  orc_block_dots(int type, const uint8_t *wrow, const int8_t *xq, int cols,
                    int32_t *isum, int32_t *xsum);
/* one output feature of a quantised matvec (activation already quantised) */
float orc_row_dot_q(int type, const uint8_t *wrow, const int8_t *xq, const float *dx, int cols);

/* ---- router ---- */
void orc_router_logits(const float *w, const float *x, int E, int H, float *logits);
void orc_rmsnorm(const float *x, const float *w, int H, float eps, float *out);
int  orc_select(const orc_layer *L, const float *logits, int32_t *idx, float *w);

/* ---- the layer ---- */
int orc_moe_forward(const orc_layer *L, int T, const float *x, float *out,
                    int32_t *sel_idx, float *sel_w, int n_threads);

/* project_lm_head for T rows (see moe_oracle.c). */
int orc_lm_head(int type, const uint8_t *head, int shaped, int64_t head_rows, int hidden, int T,
                const float *normed, int n_logits, float *logits);

/* Canonical dispatch permutation: slots sorted by (expert asc, token asc).
 * offsets[E+1]; perm_token[T*k] = token of each slot. */
int orc_permutation(const int32_t *sel_idx, int T, int k, int E,
                    int32_t *offsets, int32_t *perm_token);

/* orc_moe_forward with act_f32 = 1: quantised weight rows dequantised to f32
 * and dotted with f32 activations (no activation blocks), the other reading
 * of the reference's vec_dot_q8_0 / vec_dot_q4_k_m. act_f32 = 0 is
 * orc_moe_forward. */
int orc_moe_forward_ex(const orc_layer *L, int T, const float *x, float *out,
                       int32_t *sel_idx, float *sel_w, int n_threads, int act_f32);

/* ---- synthetic inputs (same bytes as the library's moe_gen_normal and
 * moe_quantize_rows; used to build the benchmark's layers without it) ---- */
int orc_gen_normal(uint64_t seed, uint64_t stream, uint64_t n, float sigma, float *dst, int n_threads);
int orc_quantize_rows(int type, const float *src, int64_t rows, int cols, uint8_t *dst, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
