// ep.cu -- device side of the expert-parallel exchange: packing the routed
// token rows (int8 activation blocks with their scales) into the send buffer,
// unpacking received rows, and expanding the receive plan into the slot ->
// received-row map of the local expert problems.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ep_plan.h"
#include "kernels.h"

namespace jmoe {
namespace {

// One packed row: [H int8 quants][H/32 f32 d][H/32 f32 d * sum q], as 32-bit words.
__device__ __forceinline__ void row_words(int H, int &wq, int &ws, int &wr)
{
    wq = H >> 2;
    ws = H >> 5;
    wr = wq + 2 * ws;
}

// Send buffer: row r = the activation blocks of token perm[r] (slots in the
// sender's canonical order).
__global__ void ep_pack_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xd,
                               const float *__restrict__ xs, const int32_t *__restrict__ perm, int n_rows, int H,
                               uint32_t *__restrict__ out)
{
    int wq, ws, wr;
    row_words(H, wq, ws, wr);
    const long long total = (long long)n_rows * wr;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / wr), w = (int)(i % wr);
        const size_t tok = (size_t)perm[r];
        uint32_t v;
        if (w < wq) v = reinterpret_cast<const uint32_t *>(xq + tok * H)[w];
        else if (w < wq + ws) v = __float_as_uint(xd[tok * ws + (w - wq)]);
        else v = __float_as_uint(xs[tok * ws + (w - wq - ws)]);
        out[i] = v;
    }
}

// Received rows back into the dense activation arrays the expert kernels read.
__global__ void ep_unpack_kernel(const uint32_t *__restrict__ in, int n_rows, int H, int8_t *__restrict__ xq,
                                 float *__restrict__ xd, float *__restrict__ xs)
{
    int wq, ws, wr;
    row_words(H, wq, ws, wr);
    const long long total = (long long)n_rows * wr;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const size_t r = (size_t)(i / wr);
        const int w = (int)(i % wr);
        const uint32_t v = in[i];
        if (w < wq) reinterpret_cast<uint32_t *>(xq + r * H)[w] = v;
        else if (w < wq + ws) xd[r * ws + (w - wq)] = __uint_as_float(v);
        else xs[r * ws + (w - wq - ws)] = __uint_as_float(v);
    }
}

__global__ void ep_segments_kernel(const EpSegment *__restrict__ segs, int n_segs, int32_t *__restrict__ perm)
{
    for (int g = blockIdx.x; g < n_segs; g += gridDim.x) {
        const EpSegment sg = segs[g];
        for (int i = threadIdx.x; i < sg.count; i += blockDim.x) perm[sg.slot_base + i] = sg.row_base + i;
    }
}

int grid_for(long long work, int num_sms)
{
    const long long blocks = (work + 255) / 256;
    const long long cap = 8LL * num_sms;
    return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

size_t ep_row_bytes(int H) { return (size_t)H + 8 * (size_t)(H / 32); }

cudaError_t launch_ep_pack(const int8_t *xq, const float *xd, const float *xs, const int32_t *perm, int n_rows, int H,
                           void *out, int num_sms, cudaStream_t st)
{
    if (n_rows <= 0) return cudaSuccess;
    const long long work = (long long)n_rows * (long long)(ep_row_bytes(H) / 4);
    ep_pack_kernel<<<grid_for(work, num_sms), 256, 0, st>>>(xq, xd, xs, perm, n_rows, H, static_cast<uint32_t *>(out));
    return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const void *in, int n_rows, int H, int8_t *xq, float *xd, float *xs, int num_sms,
                             cudaStream_t st)
{
    if (n_rows <= 0) return cudaSuccess;
    const long long work = (long long)n_rows * (long long)(ep_row_bytes(H) / 4);
    ep_unpack_kernel<<<grid_for(work, num_sms), 256, 0, st>>>(static_cast<const uint32_t *>(in), n_rows, H, xq, xd,
                                                              xs);
    return cudaGetLastError();
}

cudaError_t launch_ep_segments(const void *segs, int n_segs, int32_t *perm, int num_sms, cudaStream_t st)
{
    if (n_segs <= 0) return cudaSuccess;
    const int grid = n_segs < 2 * num_sms ? n_segs : 2 * num_sms;
    ep_segments_kernel<<<grid, 256, 0, st>>>(static_cast<const EpSegment *>(segs), n_segs, perm);
    return cudaGetLastError();
}

}  // namespace jmoe
