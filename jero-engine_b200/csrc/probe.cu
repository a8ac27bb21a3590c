// probe.cu -- tensor-core throughput probe: back-to-back tcgen05.mma of one
// shape on every SM, from operands already in shared memory (or A in TMEM),
// timed with CUDA events. It gives the int8 (kind::i8) and f16 (kind::f16)
// dense peaks of this GPU that the expert GEMMs are measured against, and the
// cost of one MMA instruction at the small N that decode batches produce.
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/jeromoe.h"
#include "kernels.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace jmoe {
namespace {

constexpr int kProbeSmem = 64 * 1024 + 1024;   // A (up to 16 KB) + B (up to 32 KB) + barriers
constexpr int kProbeSmemHalf = 50 * 1024;      // two CTAs per SM: B up to 128 rows

// ctas_per_sm CTAs per SM; in each, n_acc warps issue n_mma MMAs apiece
// (K = 16 f16 or 32 int8 values each) into their own accumulator, commit and
// wait (bounded) for them; the clock cycles of warp 0 from its first issue to
// completion go to cycles[blockIdx.x].
__global__ void __launch_bounds__(128)
    tc_probe_kernel(int kind, int M, int N, int a_tmem, int n_acc, int n_mma, int cols, long long *cycles, int *err)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sa = base, *sb = base + 16384;
    const int bytes = cols == 512 ? 65536 : 49152;
    uint64_t *bar = reinterpret_cast<uint64_t *>(base + bytes - 128);   // one per issuer (<= 8)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 8);
    const int warp = threadIdx.x >> 5;
    // zero operands: every product is 0, no special values
    for (int i = threadIdx.x; i < (bytes - 128) / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(base)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < 8; i++) mbar_init(&bar[i], 1);
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, (uint32_t)cols);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t a_col = (uint32_t)cols / 2;
    if (a_tmem && warp < 4) {   // A operand columns [cols / 2, cols) hold zeros
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; i++) z[i] = 0u;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
        for (uint32_t c = a_col; c < (uint32_t)cols; c += 32) tmem_st32(lane_base + c, z);
        tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // issuers = n_acc: lane 0 of warp w issues every MMA into accumulator w
    // (columns [w N, (w + 1) N)), one independent K loop per issuing warp
    // n_acc > 0: issuer w = lane 0 of warp w; n_acc < 0: issuers = lanes 0..-n_acc-1 of warp 0
    const bool lanes = n_acc < 0;
    const int n_iss = lanes ? -n_acc : n_acc;
    const int iss = lanes ? (threadIdx.x & 31) : warp;
    if (lanes ? (warp == 0 && (threadIdx.x & 31) < n_iss) : ((threadIdx.x & 31) == 0 && warp < n_iss)) {
        const uint64_t ad = umma_desc_sw128(smem_addr(sa)), bd = umma_desc_sw128(smem_addr(sb));
        // D f32 (f16 kind) or s32 (i8 kind, s8 x s8), both K-major
        const uint32_t idesc = kind == 0 ? ((1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24))
                                         : ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                                            ((uint32_t)(M >> 4) << 24));
        const uint32_t d = tmem + (uint32_t)(iss * N);
        const long long t0 = clock64();
        for (int i = 0; i < n_mma; i++) {
            const uint32_t acc = i > 0 ? 1u : 0u;
            const uint32_t at = tmem + a_col + (uint32_t)(8 * (i & 3));
            if (kind == 0) {
                if (a_tmem) tc_mma_f16_ts(d, at, bd, idesc, acc);
                else tc_mma_f16(d, ad, bd, idesc, acc);
            } else {
                if (a_tmem) tc_mma_i8_ts(d, at, bd, idesc, acc);
                else tc_mma_i8(d, ad, bd, idesc, acc);
            }
        }
        tc_commit(&bar[iss]);
        volatile int never = 0;
        tc_wait(&bar[iss], 0, &never, err);
        if (iss == 0) cycles[blockIdx.x] = clock64() - t0;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)cols);
    }
}

}  // namespace
}  // namespace jmoe

extern "C" int moe_probe_tensor(int32_t device, int32_t kind, int32_t m, int32_t n, int32_t a_tmem, int32_t n_acc,
                                int32_t ctas_per_sm, int32_t n_mma, double *tops, double *cycles_per_mma)
{
    using namespace jmoe;
    if ((kind != 0 && kind != 1) || (m != 64 && m != 128) || n < 16 || n > 256 || n % 16 || n_mma < 4 ||
        n_acc == 0 || n_acc > 4 || n_acc < -8 || (ctas_per_sm != 1 && ctas_per_sm != 2) ||
        (n_acc < 0 ? -n_acc : n_acc) * n > 256 / ctas_per_sm ||
        (ctas_per_sm == 2 && n > 128) || !tops || !cycles_per_mma)
        return MOE_ERR_INVALID_ARGS;
    if (m == 64 && a_tmem) return MOE_ERR_INVALID_ARGS;   // A from TMEM: M = 128 only here
    cudaError_t e;
    if ((e = cudaSetDevice(device)) != cudaSuccess) { record_error(cudaGetErrorString(e)); return MOE_ERR_CUDA; }
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) {
        record_error(cudaGetErrorString(e));
        return MOE_ERR_CUDA;
    }
    const int grid = sms * ctas_per_sm, cols = ctas_per_sm == 1 ? 512 : 256;
    const int smem = ctas_per_sm == 1 ? kProbeSmem : kProbeSmemHalf;
    long long *cyc = nullptr;
    int *err = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    int rc = MOE_OK;
    auto cleanup = [&]() {
        if (cyc) cudaFree(cyc);
        if (err) cudaFree(err);
        if (a) cudaEventDestroy(a);
        if (b) cudaEventDestroy(b);
    };
    if ((e = cudaMalloc(&cyc, sizeof(long long) * grid)) != cudaSuccess ||
        (e = cudaMalloc(&err, sizeof(int))) != cudaSuccess || (e = cudaMemset(err, 0, sizeof(int))) != cudaSuccess ||
        (e = cudaEventCreate(&a)) != cudaSuccess || (e = cudaEventCreate(&b)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(tc_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem)) !=
            cudaSuccess) {
        record_error(cudaGetErrorString(e));
        cleanup();
        return MOE_ERR_CUDA;
    }
    float ms = 0.0f;
    for (int rep = 0; rep < 2 && rc == MOE_OK; rep++) {   // the first launch warms up
        cudaEventRecord(a);
        tc_probe_kernel<<<grid, 128, smem>>>(kind, m, n, a_tmem, n_acc, n_mma, cols, cyc, err);
        cudaEventRecord(b);
        if ((e = cudaEventSynchronize(b)) != cudaSuccess || (e = cudaGetLastError()) != cudaSuccess) {
            record_error(cudaGetErrorString(e));
            rc = MOE_ERR_CUDA;
        }
    }
    int herr = 0;
    std::vector<long long> hc(grid);
    if (rc == MOE_OK && ((e = cudaEventElapsedTime(&ms, a, b)) != cudaSuccess ||
                         (e = cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess ||
                         (e = cudaMemcpy(hc.data(), cyc, sizeof(long long) * grid, cudaMemcpyDeviceToHost)) !=
                             cudaSuccess)) {
        record_error(cudaGetErrorString(e));
        rc = MOE_ERR_CUDA;
    }
    if (rc == MOE_OK && herr) {
        record_error("tensor-core probe: a bounded wait ran out");
        rc = MOE_ERR_TIMEOUT;
    }
    if (rc == MOE_OK) {
        const double k = kind == 0 ? 16.0 : 32.0;
        *tops = 2.0 * m * n * k * (double)n_mma * (n_acc < 0 ? -n_acc : n_acc) * grid / (ms * 1e-3) / 1e12;
        long long mx = 0;
        for (long long c : hc) mx = c > mx ? c : mx;
        *cycles_per_mma = (double)mx / n_mma;
    }
    cleanup();
    return rc;
}
