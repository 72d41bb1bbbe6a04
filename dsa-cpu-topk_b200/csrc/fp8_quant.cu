// Per-row FP8 (e4m3) quantisation for the FP8 Lightning Indexer.
//
// Each row of D values is stored as e4m3(x / s) with s = max|x| / 448 (448
// is e4m3's largest finite value; an all-zero row gets s = 1), so every row
// uses the whole e4m3 range.  The indexer then takes the per-key scales of k
// as k_scale (multiplying each score column) and the per-(query, head)
// scales of q folded into the head weights w (ReLU(c x) = c ReLU(x) for c >
// 0).  The DeepSeek-V3.2 indexer runs its q/k in FP8 with scales in the same
// way; the reference's Triton indexer is fp32 only (lightning_indexer.py:54-97).
#include "common.cuh"

namespace dsa {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ x, int64_t rows, int D,
                                                            int64_t row_stride, __nv_fp8_e4m3* __restrict__ out,
                                                            float* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;   // warp-uniform
    const T* xr = x + row * row_stride;
    float m = 0.f;
    for (int i = lane; i < D; i += 32) m = fmaxf(m, fabsf(Elem<T>::to_f(xr[i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? m / 448.f : 1.f;
    const float inv = 1.f / s;
    __nv_fp8_e4m3* orow = out + row * D;
    for (int i = lane; i < D; i += 32) orow[i] = __nv_fp8_e4m3(Elem<T>::to_f(xr[i]) * inv);
    if (lane == 0) scale[row] = s;
}

template <typename T>
int launch_q(const void* x, int64_t rows, int64_t D, int64_t stride, void* out, float* scale, cudaStream_t st) {
    const int64_t grid = (rows + 7) / 8;
    if (grid > INT32_MAX) return fail(DSA_ERR_INVALID, "quantize_fp8_rows: too many rows");
    quantize_rows_kernel<T><<<(unsigned)grid, 256, 0, st>>>(static_cast<const T*>(x), rows, (int)D, stride,
                                                            static_cast<__nv_fp8_e4m3*>(out), scale);
    return check_launch("quantize_rows_kernel");
}

}  // namespace
DSA_DEBUG_FLAGS_READER(fp8_quant)

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_quantize_fp8_rows(const void* x, int dtype, int64_t rows, int64_t D, int64_t row_stride,
                                     void* out_e4m3, float* scale_out, void* stream) {
    clear_error();
    if (rows < 0 || D < 1 || D > INT32_MAX || row_stride < D)
        return fail(DSA_ERR_INVALID, "quantize_fp8_rows: bad sizes");
    if (rows == 0) return DSA_OK;
    if (!x || !out_e4m3 || !scale_out) return fail(DSA_ERR_INVALID, "quantize_fp8_rows: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    switch (dtype) {
        case DSA_F32: return launch_q<float>(x, rows, D, row_stride, out_e4m3, scale_out, st);
        case DSA_BF16: return launch_q<__nv_bfloat16>(x, rows, D, row_stride, out_e4m3, scale_out, st);
        case DSA_F16: return launch_q<__half>(x, rows, D, row_stride, out_e4m3, scale_out, st);
        default: return fail(DSA_ERR_INVALID, "quantize_fp8_rows: dtype must be fp32, bf16 or fp16");
    }
}
