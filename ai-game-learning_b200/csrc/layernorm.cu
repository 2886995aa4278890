// Row LayerNorm with learned gain and bias (pbg/core/tensor_ops.py LayerNorm,
// F.layer_norm over the last dimension, eps as given): one warp per row, fp32
// statistics (mean, then the centred second moment), input fp32 or bf16,
// output bf16 (the next tensor-core map's operand) or fp32, written with its
// own row stride (so it can fill a slice of a wider operand buffer).
#include <cuda_bf16.h>

#include "pbg_common.cuh"

namespace pbg {

// Row i of the launch is row i % group_rows of group i / group_rows: x rows at
// x + group * x_group_stride + r * ldx, y rows likewise (elements), so a launch
// can normalise a row block of every sequence of a batch (e.g. the leading
// private rows of each decision's token sequence) without gathering it first.
template <typename In, typename Out>
__global__ void layernorm_kernel(int64_t rows, int d, int64_t group_rows, const In* __restrict__ x,
                                 int64_t x_group_stride, int64_t ldx, const float* __restrict__ gain,
                                 const float* __restrict__ bias, float eps, Out* __restrict__ y,
                                 int64_t y_group_stride, int64_t ldy) {
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const int64_t group = row / group_rows, r = row - group * group_rows;
    const In* xr = x + group * x_group_stride + r * ldx;
    float v[32];  // d <= 1024
    int count = 0;
    float sum = 0.0f;
    for (int c = lane; c < d; c += 32) {
        const float t = (float)xr[c];
        v[count++] = t;
        sum += t;
    }
    sum = warp_sum(sum);
    const float mean = sum / (float)d;
    float sq = 0.0f;
    for (int i = 0; i < count; ++i) sq += (v[i] - mean) * (v[i] - mean);
    sq = warp_sum(sq);
    const float inv = rsqrtf(sq / (float)d + eps);
    Out* yr = y + group * y_group_stride + r * ldy;
    count = 0;
    for (int c = lane; c < d; c += 32) {
        float t = (v[count++] - mean) * inv;
        if (gain) t *= gain[c];
        if (bias) t += bias[c];
        yr[c] = (Out)t;
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_layernorm_rows(int64_t rows, int32_t d, int64_t group_rows, const void* x, int32_t x_bf16,
                                  int64_t x_group_stride, int64_t ldx, const float* gain, const float* bias, float eps,
                                  void* y, int32_t y_bf16, int64_t y_group_stride, int64_t ldy, void* stream) {
    PBG_REQUIRE(rows >= 0 && d >= 1 && d <= 1024, "layernorm: width must be in [1, 1024]");
    PBG_REQUIRE(ldy >= d && ldx >= d, "layernorm: row strides must be at least the width");
    PBG_REQUIRE(group_rows >= 1, "layernorm: rows per group must be positive");
    PBG_REQUIRE(rows == 0 || (x && y), "layernorm: null pointer");
    if (rows == 0) return 0;
    const unsigned blocks = (unsigned)((rows * 32 + 255) / 256);
    cudaStream_t s = as_stream(stream);
    if (x_bf16 && y_bf16)
        layernorm_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, 256, 0, s>>>(
            rows, d, group_rows, (const __nv_bfloat16*)x, x_group_stride, ldx, gain, bias, eps, (__nv_bfloat16*)y,
            y_group_stride, ldy);
    else if (x_bf16)
        layernorm_kernel<__nv_bfloat16, float><<<blocks, 256, 0, s>>>(rows, d, group_rows, (const __nv_bfloat16*)x,
                                                                      x_group_stride, ldx, gain, bias, eps, (float*)y,
                                                                      y_group_stride, ldy);
    else if (y_bf16)
        layernorm_kernel<float, __nv_bfloat16><<<blocks, 256, 0, s>>>(rows, d, group_rows, (const float*)x,
                                                                      x_group_stride, ldx, gain, bias, eps,
                                                                      (__nv_bfloat16*)y, y_group_stride, ldy);
    else
        layernorm_kernel<float, float><<<blocks, 256, 0, s>>>(rows, d, group_rows, (const float*)x, x_group_stride,
                                                              ldx, gain, bias, eps, (float*)y, y_group_stride, ldy);
    return launch_status("layernorm");
}

extern "C" int pbg_layernorm(int64_t rows, int32_t d, const void* x, int32_t x_bf16, const float* gain,
                             const float* bias, float eps, void* y, int32_t y_bf16, int64_t ldy, void* stream) {
    return pbg_layernorm_rows(rows, d, rows > 0 ? rows : 1, x, x_bf16, 0, d, gain, bias, eps, y, y_bf16, 0, ldy,
                              stream);
}
