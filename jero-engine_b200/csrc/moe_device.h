// moe_device.h -- device-side data layout and launch interface of the MoE path.
//
// Weights live in HBM in an expert-major structure-of-arrays layout derived
// from the GGUF blocks at upload time (a byte permutation of the same values,
// no requantisation):
//   Q8_0  qs   [E][rows][cols]        int8 quants
//         meta [E][rows][cols/32]     f16 block scale d
//   Q4_K  qs   [E][rows][cols/2]      16 bytes per 32-value sub-block j: byte b holds
//                                     value 32j+b (low nibble) and 32j+16+b (high nibble)
//         meta [E][rows][cols/256][16] f16 d, f16 dmin, 12 bytes of packed 6-bit scales/mins
//   F32   qs   [E][rows][cols]        f32
// Every expert slab starts on a 128-byte boundary.
#pragma once

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>
#include <vector_types.h>

namespace jmoe {

enum Fmt : int { FMT_F32 = 0, FMT_Q8_0 = 8, FMT_Q4_K = 12 };

struct DevMatrix {
    int type;                // Fmt
    int rows;                // output features
    int cols;                // input features
    int n_experts;
    const uint8_t *qs;
    const uint8_t *meta;
    size_t qs_estride;       // bytes per expert slab (multiple of 128)
    size_t meta_estride;
    size_t qs_rstride;       // bytes per row
    size_t meta_rstride;
    int ks;                  // values per K-slice streamed by the expert kernels
    int qs_box;              // bytes of one row's slice of quants (TMA box width)
    int meta_box;            // bytes of one row's slice of scales (TMA box width)
    int _pad;
};

// 2-D TMA descriptors of one quantised stack viewed as [E*rows][row bytes]
// (u64 elements); the box is 32 rows by one K-slice.
struct MatMaps {
    CUtensorMap qs, meta;
};

struct LayerMaps {
    MatMaps gate, up, down, sh_gate, sh_up, sh_down;            // streaming kernels: 32-row boxes per K-slice
    MatMaps gate_tc, up_tc, down_tc, sh_gate_tc, sh_up_tc, sh_down_tc;  // tensor-core path: 128-row boxes per 256 values
};

// Batches up to this many tokens route in one kernel and get the slot of each
// choice in FwdParams::slot_of; larger ones leave the global expert masks.
constexpr int kFusedRoutingMaxT = 256;

// Bytes of the routing tickets in front of the expert masks: [0] the last
// token tile, [1 + j] the CTAs of token tile j (fused routing, T <= 256).
constexpr int kRoutingTicketBytes = 1024;

// Entries per launch layout in FwdParams::tile_off (problems + 2).
constexpr int kTileOffStride = 260;

// One group of slots that share a weight set: a routed expert, or the shared
// expert (is_shared = 1, all T tokens in order).
struct Problem {
    int expert;
    int slot0;
    int count;
    int is_shared;
};

struct FwdParams {
    int T, H, E, k, I, S;        // S = 0: no shared expert
    int route_mode, normalize, n_groups, topk_groups;
    float routed_scale;
    int mask_words;              // ceil(T/32)
    int quant_x;                 // x needs int8 blocks (some gate/up matrix is quantised)
    int max_problems;            // grid.y of the expert kernels
    int use_tc;                  // experts on the f16 tensor-core path (prefill.cu)
    int use_dtc;                 // experts on the int8 tensor-core path (decode_tc.cu)
    int use_xtc;                 // experts in one fused f16 tensor-core launch (experts_tc.cu)
    int use_xi8;                 // experts in one fused int8 tensor-core launch (experts_i8.cu)

    const float *x;              // [T][H]
    const float *router;         // [E][H]
    const float *logit_bias;     // [E] or null
    const float *sel_bias;       // [E] or null

    int8_t *xq;                  // [T][H] (row stride x_qstride bytes when set)
    int x_qstride, x_dstride;    // 0: H and H/32. Expert-parallel inbox rows are packed
                                 // [H int8 | H/32 d | H/32 s], read in place with these strides
    float *xd;                   // [T][H/32] block scale
    void *x16;                   // null, or [T][H] f16(q * d) of the activation blocks, each aligned group
                                 // of four values in the order (0, 2, 1, 3) (fused tensor-core launch)
    float *xs;                   // [T][H/32] block scale * block sum of quants
    float *logits;               // [T][E]
    int32_t *sel_idx;            // [T][k]
    float *sel_w;                // [T][k]
    int *sync;                   // routing tickets [kRoutingTicketBytes / 4]; the masks follow (one memset clears both)
    uint32_t *mask;              // [E][mask_words]: bit t of expert e = token t chose e
    int32_t *wprefix;            // [E][mask_words]: set bits of expert e before word w
    int32_t *offsets;            // [E+1]
    int32_t *perm_token;         // [T*k + T]
    int32_t *slot_of;            // [T][k] slot of each choice (-1: none), for the combine
    Problem *problems;           // [max_problems]
    int32_t *n_active;           // [1]

    int8_t *aq;                  // [slots][W] quantised SwiGLU output, W = max(I, S)
    float *ad;                   // [slots][W/32]
    float *as;                   // [slots][W/32]
    float *af;                   // [slots][W] f32 SwiGLU output (F32 down matrices)
    int W;
    float *y;                    // [slots][H] expert outputs
    const int32_t *y_rows;       // null: y row = slot; else y row of slot s = y_rows[s] (expert-parallel
                                 // receive order, so rows go back to their source rank in its order)
    float *out;                  // [T][H]
    int *err;                    // device status word: 0 ok, 1 a bounded wait ran out

    // FFN sublayer (moe_forward_block): norm_out = rmsnorm(norm_in, norm_w,
    // norm_eps) before the routing (x = norm_out), and out = residual + block
    // in the combine. null norm_in / residual: plain moe_forward.
    const float *norm_in;
    float *norm_out;
    const float *norm_w;
    float norm_eps;
    const float *residual;

    // tensor-core (prefill) path
    void *a16;                   // [slots_cap][a16_stride] f16: gate/up operand (activation blocks dequantised)
    void *a16dn;                 // [slots_cap][a16dn_stride] f16: down operand (quantised SwiGLU output)
    int a16_stride, a16dn_stride, slots_cap;
    int32_t *tile_off;           // [4][kTileOffStride] work-item offsets of the tensor-core launches

    // fused expert launch (experts_tc.cu): per slot chunk, the number of
    // gate/up epilogue warps that have stored their SwiGLU rows (the down
    // items of that chunk wait for all of them), and a ticket of finished
    // CTAs; the last CTA returns both to zero. dep_cap entries.
    int32_t *dep;
    int32_t *dep_done;
    int dep_cap;

    // expert-parallel return through peer memory (the fused f16 expert
    // launch): when y_peer is set, the down epilogue stores the output row of
    // local slot s straight into its source rank's output inbox, at
    // y_peer[y_ret[s].x] + y_peer_off, row y_ret[s].y; the launch's last CTA
    // then raises this rank's output flag (value y_epoch, at y_flag_off in
    // every rank's arena) once every CTA's stores are fenced at system scope,
    // unless *y_ok is 0 (the forward's exchange has failed).
    uint8_t *const *y_peer;
    const int2 *y_ret;
    size_t y_peer_off, y_flag_off;
    uint32_t y_epoch;
    int y_world;
    const int *y_ok;

    // parity probe (null in production): the int8 tensor-core gate/up launch
    // stores each routed slot's raw int32 block sums here,
    // [slot][matrix 0 gate / 1 up][row of I][block of H/32]
    int32_t *dbg_isum;
};

// Entries of FwdParams::dep a forward over T tokens may use: one per slot
// chunk (of at least 4 slots, the smallest item cap) of every problem.
inline int dep_entries(int T, int k, int E) { return (T * k + T) / 4 + (E < T * k ? E : T * k) + 2; }

struct LayerDev {
    DevMatrix gate, up, down;
    DevMatrix sh_gate, sh_up, sh_down;   // rows == 0: absent
};

// Called after each kernel of the forward sequence is enqueued (profiling).
struct Marker {
    void (*fn)(void *user, const char *kernel);
    void *user;
    void mark(const char *k) const { if (fn) fn(user, k); }
};

// Launch sequence of one forward on stream; returns cudaError_t as int.
// num_sms sizes the grids of the streaming expert kernels.
int launch_forward(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, void *stream, const Marker &mk,
                   int num_sms);

// K-slice and TMA box widths of a quantised matrix (host side, at upload).
void plan_slices(DevMatrix &m);

// Builds the two TMA descriptors of a quantised stack; returns a CUresult.
// box_rows 32: one K-slice per box (streaming kernels); box_rows 128: 256 values
// per box (tensor-core path).
int make_matrix_maps(const DevMatrix &m, MatMaps *out, int box_rows);

// 2-D tiled TMA descriptor. dtype 0: f16 elements, 1: u64 elements. cols in
// elements, row_bytes the global row stride, box_cols x box_rows the box,
// swizzle128: 128-byte swizzle (else none). Returns a CUresult.
int encode_tiled(CUtensorMap *map, int dtype, const void *base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                 uint32_t box_cols, uint32_t box_rows, int swizzle128);

// Stores the message that moe_last_error_message(NULL) returns on this thread.
void record_error(const char *msg);

// Integer block sums for the parity probe (same device code as the forward path).
int launch_block_dots(const DevMatrix &m, const int8_t *xq, int n, int32_t *isum, void *stream);
int launch_quantize_rows(const float *x, int n, int cols, int8_t *xq, float *xd, float *xs,
                         void *stream);

}  // namespace jmoe
