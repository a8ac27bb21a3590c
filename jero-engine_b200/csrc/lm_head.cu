// lm_head.cu -- the pieces of the LM head (project_lm_head,
// src/qwen_deepseek.rs:584-632) around its matrix-vector product, which runs
// on the expert down-projection kernels (one problem of T tokens over the head
// matrix): the problem entry, the rows past the head's rows, and the synthetic
// logits of a model without a head.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "kernels.h"
#include "moe_device.h"

namespace jmoe {
namespace {

// One problem: "expert" 0 (the head), slots 0 .. T-1 (the tokens).
__global__ void lm_head_prep_kernel(Problem *prob, int32_t *n_active, int T)
{
    prob[0] = Problem{0, 0, T, 0};
    *n_active = 1;
}

// logits[t][i] for i < target from the product rows y [T][ystride], and for
// target <= i < n the reference's filler normed[t][i mod hidden] * 0.05.
__global__ void lm_head_scatter_kernel(const float *y, int ystride, int target, const float *normed, int hidden,
                                       float *logits, int n, int T)
{
    const long long total = (long long)T * n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / n), c = (int)(i - (long long)t * n);
        logits[i] = c < target ? y[(size_t)t * ystride + c] : __fmul_rn(normed[(size_t)t * hidden + c % hidden], 0.05f);
    }
}

// No head: base = tanh(sum(normed) / 16) with the sum taken in element order,
// then logits[idx] = base + normed[idx mod hidden] * 0.1 + (idx mod 13) * 0.01.
// One CTA per token; thread 0 takes the sequential sum.
__global__ void lm_head_synth_kernel(const float *normed, int hidden, float *logits, int n)
{
    __shared__ float s_base;
    const float *x = normed + (size_t)blockIdx.x * hidden;
    if (threadIdx.x == 0) {
        float sum = 0.0f;
        for (int i = 0; i < hidden; i++) sum = __fadd_rn(sum, x[i]);
        s_base = tanhf(__fdiv_rn(sum, 16.0f));
    }
    __syncthreads();
    float *out = logits + (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = __fadd_rn(__fadd_rn(s_base, __fmul_rn(x[i % hidden], 0.1f)), __fmul_rn((float)(i % 13), 0.01f));
}

}  // namespace

cudaError_t launch_lm_head_prep(Problem *prob, int32_t *n_active, int T, cudaStream_t st)
{
    lm_head_prep_kernel<<<1, 1, 0, st>>>(prob, n_active, T);
    return cudaGetLastError();
}

cudaError_t launch_lm_head_scatter(const float *y, int ystride, int target, const float *normed, int hidden,
                                   float *logits, int n, int T, int num_sms, cudaStream_t st)
{
    const long long total = (long long)T * n;
    long long blocks = (total + 255) / 256;
    if (blocks > 4LL * num_sms) blocks = 4LL * num_sms;
    if (blocks < 1) blocks = 1;
    lm_head_scatter_kernel<<<(int)blocks, 256, 0, st>>>(y, ystride, target, normed, hidden, logits, n, T);
    return cudaGetLastError();
}

cudaError_t launch_lm_head_synth(const float *normed, int hidden, float *logits, int n, int T, cudaStream_t st)
{
    lm_head_synth_kernel<<<T, 256, 0, st>>>(normed, hidden, logits, n);
    return cudaGetLastError();
}

}  // namespace jmoe
