// noalloc.cu -- routing and dispatch permutation without any allocation.
//
// For callers that cannot allocate device memory themselves or let a library
// do it: a runtime that owns all device memory through its own pool, or a
// decode loop that must not allocate once it is running (jero-engine holds its
// decode step to zero heap allocations). The caller passes device inputs and
// outputs; the working memory of the routing kernels (logits, expert masks,
// prefix counts, problem list) lives in one fixed static device array below.
//
// Properties a caller must know:
//   - The array is kNoAllocScratchBytes per device and stays resident on every
//     GPU that loads the library until the process exits.
//   - All calls share the array: calls that overlap on the GPU (different
//     streams, or several host threads) race on it. Serialise them.
//   - The first call on a device resolves the array's device address
//     (cudaGetSymbolAddress); make that first call before capturing a stream
//     into a CUDA graph.
//   - The calling thread's current device is the same after the call.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/jeromoe.h"
#include "kernels.h"
#include "moe_device.h"

namespace jmoe {
namespace {

constexpr int kNoAllocMaxTokens = 1024;
constexpr int kNoAllocMaxExperts = 256;
constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;   // 2 MiB per device
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices];

// Failures are reported through moe_last_error_message(NULL).
int fail(int code, const char *msg)
{
    record_error(msg);
    return code;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace
}  // namespace jmoe

using namespace jmoe;

extern "C" int moe_route_noalloc(int32_t device, const float *x, const float *router, const float *logit_bias,
                                 const float *sel_bias, int32_t T, int32_t H, int32_t E, int32_t top_k,
                                 int32_t normalize, float routed_scale, int32_t n_groups, int32_t topk_groups,
                                 int32_t *sel_idx, float *sel_w, int32_t *offsets, int32_t *perm_token, void *stream)
{
    if (!x || !router || !sel_idx || !sel_w || !offsets || !perm_token)
        return fail(MOE_ERR_INVALID_ARGS, "null input or output pointer");
    if (device < 0 || device >= kMaxDevices) return fail(MOE_ERR_INVALID_ARGS, "device ordinal out of range");
    if (T < 0 || H <= 0 || E <= 0 || top_k <= 0 || top_k > 16 || top_k > E)
        return fail(MOE_ERR_INVALID_ARGS, "bad shape (need H > 0, 0 < top_k <= min(16, E))");
    if (T > kNoAllocMaxTokens || E > kNoAllocMaxExperts)
        return fail(MOE_ERR_CONTEXT_LENGTH,
                    "moe_route_noalloc takes at most 1024 tokens and 256 experts per call (fixed 2 MiB scratch)");
    const bool grouped = n_groups > 0;
    if (grouped && (n_groups > 32 || E % n_groups || topk_groups <= 0 || topk_groups >= n_groups ||
                    top_k > topk_groups * (E / n_groups)))
        return fail(MOE_ERR_CAPABILITY_MISMATCH, "bad group-limited routing parameters");
    if (((uintptr_t)x | (uintptr_t)router) & 15) return fail(MOE_ERR_INVALID_ARGS, "x and router must be 16-byte aligned");
    if (T == 0) return MOE_OK;

    // carve the static array for this call's shape
    const int mw = (T + 31) / 32;
    const int max_problems = (E < T * top_k ? E : T * top_k);
    size_t off = 0;
    // the selection ticket sits at a fixed place (offset 0): small batches leave
    // it at zero when they finish, and the array starts zeroed
    const size_t o_mask = off;     off += align256(kRoutingTicketBytes + (size_t)E * mw * 4);   // tickets + masks
    const size_t o_logits = off;   off += align256((size_t)T * E * 4);
    const size_t o_wprefix = off;  off += align256((size_t)E * mw * 4);
    const size_t o_problems = off; off += align256((size_t)(max_problems + 1) * sizeof(Problem));
    const size_t o_nactive = off;  off += 256;
    const size_t o_slot_of = off;  off += align256((size_t)T * top_k * 4);
    if (off > kNoAllocScratchBytes) return fail(MOE_ERR_CONTEXT_LENGTH, "routing scratch for this shape exceeds 2 MiB");

    // the caller's current device is restored before returning
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return fail(MOE_ERR_CUDA, cudaGetErrorString(e));
    if ((e = cudaSetDevice(device)) != cudaSuccess) return fail(MOE_ERR_CUDA, cudaGetErrorString(e));
    struct Restore {
        int dev;
        ~Restore() { cudaSetDevice(dev); }
    } restore{prev};
    unsigned char *base;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_ptr[device]) {
            void *ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_route_scratch);
            if (e != cudaSuccess) return fail(MOE_ERR_CUDA, cudaGetErrorString(e));
            g_scratch_ptr[device] = ptr;
        }
        base = static_cast<unsigned char *>(g_scratch_ptr[device]);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    FwdParams p{};
    p.T = T; p.H = H; p.E = E; p.k = top_k; p.I = 0; p.S = 0;
    p.route_mode = grouped ? MOE_ROUTE_GROUP_LIMITED : MOE_ROUTE_SOFTMAX_TOPK;
    p.normalize = normalize;
    p.n_groups = grouped ? n_groups : 0;
    p.topk_groups = grouped ? topk_groups : 0;
    p.routed_scale = routed_scale;
    p.mask_words = mw;
    p.quant_x = 0;
    p.max_problems = max_problems;
    p.x = x; p.router = router; p.logit_bias = logit_bias; p.sel_bias = sel_bias;
    p.logits = reinterpret_cast<float *>(base + o_logits);
    p.sync = reinterpret_cast<int *>(base + o_mask);
    p.mask = reinterpret_cast<uint32_t *>(base + o_mask + kRoutingTicketBytes);
    p.wprefix = reinterpret_cast<int32_t *>(base + o_wprefix);
    p.problems = reinterpret_cast<Problem *>(base + o_problems);
    p.n_active = reinterpret_cast<int32_t *>(base + o_nactive);
    p.slot_of = reinterpret_cast<int32_t *>(base + o_slot_of);
    p.sel_idx = sel_idx; p.sel_w = sel_w; p.offsets = offsets; p.perm_token = perm_token;

    if ((e = launch_routing(p, st, Marker{nullptr, nullptr})) != cudaSuccess)
        return fail(MOE_ERR_CUDA, cudaGetErrorString(e));
    return MOE_OK;
}
