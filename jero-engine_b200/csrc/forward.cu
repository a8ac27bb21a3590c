// forward.cu -- the launch sequence of one batched MoE forward:
// routing (router, top-k, permutation) -> gate_up -> down -> combine.
// Each kernel reads its work from device-side counters written by the one
// before it, so the sequence needs no host round trip.
#include <cuda_runtime.h>

#include "kernels.h"
#include "moe_device.h"

namespace jmoe {

int launch_forward(const FwdParams &p, const LayerDev &L, const LayerMaps &maps, void *stream, const Marker &mk,
                   int num_sms)
{
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t err;
    if (p.T == 0) return cudaSuccess;
    mk.mark(nullptr);
    if (p.norm_in) {
        if ((err = launch_rmsnorm(p, st)) != cudaSuccess) return err;
        mk.mark("ffn_norm");
    }
    if ((err = launch_routing(p, st, mk)) != cudaSuccess) return err;

    if (p.use_tc) {
        if ((err = launch_prefill(p, L, maps, num_sms, mk, st)) != cudaSuccess) return err;
        if ((err = launch_combine(p, st)) != cudaSuccess) return err;
        mk.mark("combine");
        return cudaSuccess;
    }
    if (p.use_xi8) {
        if ((err = launch_fused_i8(p, L, maps, p.S > 0 ? 2 : 0, num_sms, st)) != cudaSuccess) return err;
        mk.mark("experts_i8");
        if ((err = launch_combine(p, st)) != cudaSuccess) return err;
        mk.mark("combine");
        return cudaSuccess;
    }
    if (p.use_xtc) {
        if ((err = launch_fused_experts(p, L, maps, p.S > 0 ? 2 : 0, num_sms, st)) != cudaSuccess) return err;
        mk.mark("experts_tc");
        if ((err = launch_combine(p, st)) != cudaSuccess) return err;
        mk.mark("combine");
        return cudaSuccess;
    }
    if (p.use_dtc) {
        if ((err = launch_decode_tc(p, L, maps, num_sms, mk, st)) != cudaSuccess) return err;
        if ((err = launch_combine(p, st)) != cudaSuccess) return err;
        mk.mark("combine");
        return cudaSuccess;
    }
    const bool has_sh = p.S > 0;
    // one launch covers routed and shared problems when they share a format and slice plan
    const bool same_gu = has_sh && stream_plans_match(L.sh_gate, L.gate);
    const bool same_d = has_sh && stream_plans_match(L.sh_down, L.down);
    if ((err = launch_gate_up(p, L, maps, same_gu ? 2 : 0, num_sms, st)) != cudaSuccess) return err;
    mk.mark("gate_up");
    if (has_sh && !same_gu) {
        if ((err = launch_gate_up(p, L, maps, 1, num_sms, st)) != cudaSuccess) return err;
        mk.mark("gate_up_shared");
    }
    if ((err = launch_down(p, L, maps, same_d ? 2 : 0, num_sms, st)) != cudaSuccess) return err;
    mk.mark("down");
    if (has_sh && !same_d) {
        if ((err = launch_down(p, L, maps, 1, num_sms, st)) != cudaSuccess) return err;
        mk.mark("down_shared");
    }
    if ((err = launch_combine(p, st)) != cudaSuccess) return err;
    mk.mark("combine");
    return cudaSuccess;
}

}  // namespace jmoe
