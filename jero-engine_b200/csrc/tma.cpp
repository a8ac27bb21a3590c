// tma.cpp -- K-slice planning and TMA tensor-map descriptors for the
// quantised expert stacks and the tensor-core operands (host side).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>

#include "moe_device.h"

namespace jmoe {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

}  // namespace

int encode_tiled(CUtensorMap *map, int dtype, const void *base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                 uint32_t box_cols, uint32_t box_rows, int swizzle128)
{
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT64, 2,
              const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// A K-slice is at most 1024 values (Q4_K) or 512 (Q8_0), a whole number of
// super-blocks, so one ring stage (2 matrices x 32 rows) stays near 36 KB and
// every slice starts on a 16-byte boundary of its row (TMA box x-alignment).
void plan_slices(DevMatrix &m)
{
    if (m.type == FMT_Q4_K) {
        m.ks = m.cols < 1024 ? m.cols : 1024;
        m.qs_box = m.ks / 2;
        m.meta_box = (m.ks / 256) * 16;
    } else if (m.type == FMT_Q8_0) {
        m.ks = m.cols < 512 ? m.cols : 512;
        m.qs_box = m.ks;
        m.meta_box = ((m.ks / 32) * 2 + 15) & ~15;
    } else {
        m.ks = m.qs_box = m.meta_box = 0;
    }
}

// Each quantised stack is the dense array [E*rows][row bytes] of u64 elements.
// box_rows 32: the streaming kernels' K-slice boxes; box_rows 128: the
// tensor-core path's boxes of 128 bytes of quants per row (Q4_K 256 values,
// Q8_0 128 values) and 16 bytes of scales per row (one 256-value super-step).
int make_matrix_maps(const DevMatrix &m, MatMaps *out, int box_rows)
{
    memset(out, 0, sizeof *out);
    if (m.type != FMT_Q4_K && m.type != FMT_Q8_0) return CUDA_SUCCESS;
    const uint64_t rows_total = (uint64_t)m.n_experts * m.rows;
    // the tensor-core path lands quants in 128-byte rows with the 128-byte
    // swizzle (Q8_0: two boxes per 256 values), so its dequant warps read them
    // without bank conflicts
    const bool tc = box_rows != 32;
    const uint32_t qbox = tc ? 128u : (uint32_t)m.qs_box;
    const uint32_t mbox = tc ? 16u : (uint32_t)m.meta_box;
    int r = encode_tiled(&out->qs, 1, m.qs, rows_total, m.qs_rstride / 8, m.qs_rstride, qbox / 8, box_rows, tc);
    if (r != CUDA_SUCCESS) return r;
    return encode_tiled(&out->meta, 1, m.meta, rows_total, m.meta_rstride / 8, m.meta_rstride, mbox / 8, box_rows, 0);
}

}  // namespace jmoe
