// Row LayerNorm with learned gain and bias (pbg/core/tensor_ops.py LayerNorm,
// F.layer_norm over the last dimension, eps as given): one warp per row, fp32
// statistics (mean, then the centred second moment), input fp32 or bf16,
// output bf16 (the next tensor-core map's operand) or fp32, written with its
// own row stride (so it can fill a slice of a wider operand buffer).  The
// model's case (fp32 residual stream in, bf16 out, width a multiple of 128)
// moves 16-byte vectors.
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

// fp32 input of width d = 128 * V: each lane holds V float4 (columns 4 lane + 128 i), bf16 output with
// 8-byte stores of the same columns; one warp per row
template <int V>
__global__ void layernorm_f32_vec_kernel(int64_t rows, int d, int64_t group_rows, const float* __restrict__ x,
                                         int64_t x_group_stride, int64_t ldx, const float* __restrict__ gain,
                                         const float* __restrict__ bias, float eps, __nv_bfloat16* __restrict__ y,
                                         int64_t y_group_stride, int64_t ldy) {
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const int64_t group = row / group_rows, r = row - group * group_rows;
    const float4* xr = reinterpret_cast<const float4*>(x + group * x_group_stride + r * ldx);
    float4 v[V];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        v[i] = __ldg(xr + lane + 32 * i);
        sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    sum = warp_sum(sum);
    const float mean = sum / (float)d;
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
        sq += (a * a + b * b) + (c * c + e * e);
    }
    sq = warp_sum(sq);
    const float inv = rsqrtf(sq / (float)d + eps);
    __nv_bfloat16* yr = y + group * y_group_stride + r * ldy;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = 4 * lane + 128 * i;
        float o[4] = {(v[i].x - mean) * inv, (v[i].y - mean) * inv, (v[i].z - mean) * inv, (v[i].w - mean) * inv};
        if (gain) {
            const float4 g = __ldg(reinterpret_cast<const float4*>(gain + c));
            o[0] *= g.x;
            o[1] *= g.y;
            o[2] *= g.z;
            o[3] *= g.w;
        }
        if (bias) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + c));
            o[0] += bb.x;
            o[1] += bb.y;
            o[2] += bb.z;
            o[3] += bb.w;
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t*>(&lo);
        w.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(yr + c) = w;
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
    const bool vec = !x_bf16 && y_bf16 && d % 128 == 0 && d <= 512 && ldx % 4 == 0 && x_group_stride % 4 == 0 &&
                     ldy % 4 == 0 && y_group_stride % 4 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 8) == 0 &&
                     (!gain || ((uintptr_t)gain % 16) == 0) && (!bias || ((uintptr_t)bias % 16) == 0);
    if (vec) {
        const int V = d / 128;
        auto run = [&](auto kernel) {
            kernel<<<blocks, 256, 0, s>>>(rows, d, group_rows, (const float*)x, x_group_stride, ldx, gain, bias, eps,
                                         (__nv_bfloat16*)y, y_group_stride, ldy);
        };
        if (V == 1) run(layernorm_f32_vec_kernel<1>);
        else if (V == 2) run(layernorm_f32_vec_kernel<2>);
        else if (V == 3) run(layernorm_f32_vec_kernel<3>);
        else run(layernorm_f32_vec_kernel<4>);
        return launch_status("layernorm");
    }
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
