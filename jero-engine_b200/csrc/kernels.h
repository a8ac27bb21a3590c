// kernels.h -- host-side launchers of the MoE kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>

#include "moe_device.h"

namespace jmoe {

// Work split of the streaming expert kernels, chosen on the host.
struct StreamCfg {
    int stages;        // ring depth
    int stage_bytes;   // bytes of one ring stage (multiple of 128)
    int act_k;         // largest activation row (values) staged in shared memory
    int mode;          // 0: routed problems, 1: the shared expert only, 2: both
    int down_f32;      // gate_up: store a in f32 (F32 down matrices)
    int rt_routed;     // row tiles per routed problem
    int rt_shared;     // row tiles of the shared problem
    int ks;            // values per K-slice (one ring stage holds 32 rows of one slice)
    int qs_row;        // shared-memory bytes of one row's slice of quants
    int meta_row;      // shared-memory bytes of one row's slice of scales (multiple of 16)
    int max_q;         // capacity of the shared-memory problem table (routed + shared)
};

// Router logits, top-k selection and the dispatch permutation. Small batches
// (T <= 256) run it as one kernel; larger ones clear the expert masks, then
// router, selection and scan kernels. Marks "routing" or "router"/"select".
cudaError_t launch_routing(const FwdParams &p, cudaStream_t st, const Marker &mk);

// Launch with programmatic stream serialization: the kernel may be scheduled
// while its predecessor finishes, so it must call pdl_wait() before touching
// memory (the decode-path kernels do so on entry).
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}
// Routed and shared matrices can share one streaming launch when their slice plans match.
bool stream_plans_match(const DevMatrix &a, const DevMatrix &b);
cudaError_t launch_gate_up(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                           cudaStream_t st);
cudaError_t launch_down(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                        cudaStream_t st);
cudaError_t launch_combine(const FwdParams &p, cudaStream_t st);

// RMSNorm of the T rows of p.norm_in into p.norm_out (moe_forward_block).
cudaError_t launch_rmsnorm(const FwdParams &p, cudaStream_t st);

// Tensor-core expert path (gather of the f16 operand, item plan, gate/up and
// down GEMMs); replaces launch_gate_up / launch_down for large token counts.
cudaError_t launch_prefill(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                           const Marker &mk, cudaStream_t st);
// One dense problem on the f16 tensor-core down launch: slots 0 .. p.T-1 (the
// int8 blocks p.xq / p.xd of rows of p.W values, expanded to f16 into p.a16dn)
// times the p.H rows of L.down, into p.y [T][p.H]; item offsets in p.tile_off.
// The LM head's product for larger batches.
bool dense_f16_ok(const FwdParams &p, const LayerDev &L);
cudaError_t launch_dense_f16(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                             cudaStream_t st);

// Tensor-core expert path with integer operands for small batches: the gate/up
// and down launches (routed problems, plus the shared expert when p.S > 0), or
// the shared expert alone. decode_tc_ok: the layer's formats, shapes and
// buffers suit it.
bool decode_tc_ok(const FwdParams &p, const LayerDev &L);
cudaError_t launch_decode_tc(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                             const Marker &mk, cudaStream_t st, bool shared_only = false);
// The down launch alone over the routed problems (one matrix of rows of p.H,
// K = p.W): the LM head's product. decode_tc_down_ok: formats, shapes, buffers.
bool decode_tc_down_ok(const FwdParams &p, const LayerDev &L);
cudaError_t launch_decode_tc_down(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int num_sms,
                                  cudaStream_t st);

// The expert FFN of small batches as one persistent launch on the tensor
// cores with f16 operands (experts_tc.cu): gate/up + SwiGLU and down, the
// down items of a slot chunk waiting for its gate/up tiles. mode: 0 routed
// problems, 1 the shared expert only, 2 both. fused_experts_ok: the layer's
// formats, shapes and buffers suit it.
bool fused_experts_ok(const FwdParams &p, const LayerDev &L);
cudaError_t launch_fused_experts(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                                 cudaStream_t st);

// The same fused launch with integer operands (experts_i8.cu): exact int32
// block sums from tcgen05 kind::i8 scaled per block by the epilogue; items of
// up to 16 slots. fused_i8_ok: the layer's formats, shapes and buffers suit it.
bool fused_i8_ok(const FwdParams &p, const LayerDev &L);
cudaError_t launch_fused_i8(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, int mode, int num_sms,
                            cudaStream_t st);

// LM head (lm_head.cu): the problem entry of its product on the down-projection
// kernels, the rows past the head's rows, the synthetic logits without a head.
cudaError_t launch_lm_head_prep(Problem *prob, int32_t *n_active, int T, cudaStream_t st);
cudaError_t launch_lm_head_scatter(const float *y, int ystride, int target, const float *normed, int hidden,
                                   float *logits, int n, int T, int num_sms, cudaStream_t st);
cudaError_t launch_lm_head_synth(const float *normed, int hidden, float *logits, int n, int T, cudaStream_t st);

// Expert-parallel exchange (ep.cu): bytes of one packed token row, and the
// pack / unpack / receive-plan kernels.
size_t ep_row_bytes(int H);
cudaError_t launch_ep_pack(const int8_t *xq, const float *xd, const float *xs, const int32_t *perm, int n_rows, int H,
                           void *out, int num_sms, cudaStream_t st);
cudaError_t launch_ep_unpack(const void *in, int n_rows, int H, int8_t *xq, float *xd, float *xs, int num_sms,
                             cudaStream_t st);
cudaError_t launch_ep_segments(const void *segs, int n_segs, int32_t *perm, int num_sms, cudaStream_t st);

}  // namespace jmoe
