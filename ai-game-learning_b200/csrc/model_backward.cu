// The element-wise and row-wise parts of the policy/value network's backward
// (pbg/games/poker/model/primitives.py FFN and MHA, pbg/core/tensor_ops.py
// LayerNorm, as differentiated by torch autograd in the reference's learner
// step, pbg/core/training.py:381-403).  The dense products of the backward
// (dX = dY W, dW = dY^T X, and the four attention products) are library
// GEMMs; these kernels sit between them.
//
//   gelu_backward      dpre = dy * (Phi(pre) + pre * phi(pre)) for the exact
//                      (erf) GELU, bf16 out: the operand of the map's dX / dW
//                      products
//   layernorm_backward warp per row: the statistics recomputed from the row,
//                      dx = inv * (g dy - mean(g dy) - xhat mean(g dy xhat)),
//                      and per-block column sums of dy * xhat (gain) and dy
//                      (bias) in a fixed order (the host adds the blocks' rows)
//   attention_softmax_backward
//                      one CTA per score row (sequence, head, query): from the
//                      raw content scores q.k and dP = dO V^T it recomputes the
//                      row's softmax of s * scale_h + key_bias (absent keys
//                      excluded; a row without keys is all zeros), writes P
//                      (bf16, for dV = P^T dO), the logit gradient
//                      dZ = P (dP - sum(P dP)) times scale_h (bf16, for
//                      dQ = dZ K and dK = dZ^T Q), and the row's sum of
//                      dZ * s (the gradient of the head's score scale)
#include <cuda_bf16.h>

#include <cmath>

#include "pbg_common.cuh"

namespace pbg {
namespace {

constexpr int GB_THREADS = 256;
constexpr int LNB_WARPS = 8;
constexpr int LNB_MAX_PER_LANE = 16;  // d <= 512
constexpr int ASB_THREADS = 256;

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void store_f(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename DY>
__global__ void gelu_backward_kernel(int64_t M, int N, const float* __restrict__ pre, int64_t ldp,
                                     const DY* __restrict__ dy, int64_t ldd, __nv_bfloat16* __restrict__ out,
                                     int64_t ldo) {
    const int64_t n = M * N;
    const float inv_sqrt2 = 0.70710678118654752f;
    const float inv_sqrt2pi = 0.39894228040143268f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / N;
        const int c = (int)(i - m * N);
        const float x = pre[m * ldp + c];
        const float cdf = 0.5f * (1.0f + erff(x * inv_sqrt2));
        const float pdf = inv_sqrt2pi * expf(-0.5f * x * x);
        out[m * ldo + c] = __float2bfloat16_rn(load_f(dy + m * ldd + c) * (cdf + x * pdf));
    }
}

template <typename In, typename DY, typename Out>
__global__ void __launch_bounds__(LNB_WARPS * 32)
layernorm_backward_kernel(int64_t rows, int d, const In* __restrict__ x, int64_t ldx, const float* __restrict__ gain,
                          float eps, const DY* __restrict__ dy, int64_t ldy, Out* __restrict__ dx, int64_t lddx,
                          float* __restrict__ partial) {
    __shared__ float red[LNB_WARPS][2 * 32 * LNB_MAX_PER_LANE];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = d >> 5;
    float acc_g[LNB_MAX_PER_LANE], acc_b[LNB_MAX_PER_LANE];
    #pragma unroll
    for (int i = 0; i < LNB_MAX_PER_LANE; ++i) acc_g[i] = acc_b[i] = 0.0f;
    const int64_t warps = (int64_t)gridDim.x * LNB_WARPS;
    for (int64_t r = (int64_t)blockIdx.x * LNB_WARPS + warp; r < rows; r += warps) {
        const In* xr = x + r * ldx;
        const DY* dr = dy + r * ldy;
        float v[LNB_MAX_PER_LANE], g[LNB_MAX_PER_LANE];
        float sum = 0.0f;
        #pragma unroll
        for (int i = 0; i < LNB_MAX_PER_LANE; ++i) {
            if (i < per) {
                v[i] = load_f(xr + lane + 32 * i);
                sum += v[i];
            }
        }
        const float mean = warp_sum(sum) / (float)d;
        float sq = 0.0f;
        #pragma unroll
        for (int i = 0; i < LNB_MAX_PER_LANE; ++i)
            if (i < per) sq += (v[i] - mean) * (v[i] - mean);
        const float inv = rsqrtf(warp_sum(sq) / (float)d + eps);
        float s1 = 0.0f, s2 = 0.0f;
        #pragma unroll
        for (int i = 0; i < LNB_MAX_PER_LANE; ++i) {
            if (i < per) {
                const int c = lane + 32 * i;
                const float t = load_f(dr + c);
                const float xh = (v[i] - mean) * inv;
                v[i] = xh;
                acc_g[i] += t * xh;
                acc_b[i] += t;
                g[i] = gain ? t * gain[c] : t;
                s1 += g[i];
                s2 += g[i] * xh;
            }
        }
        s1 = warp_sum(s1) / (float)d;
        s2 = warp_sum(s2) / (float)d;
        Out* out = dx + r * lddx;
        #pragma unroll
        for (int i = 0; i < LNB_MAX_PER_LANE; ++i)
            if (i < per) store_f(out + lane + 32 * i, inv * (g[i] - s1 - v[i] * s2));
    }
    #pragma unroll
    for (int i = 0; i < LNB_MAX_PER_LANE; ++i) {
        if (i < per) {
            red[warp][lane + 32 * i] = acc_g[i];
            red[warp][d + lane + 32 * i] = acc_b[i];
        }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < 2 * d; c += blockDim.x) {
        float t = 0.0f;
        for (int w = 0; w < LNB_WARPS; ++w) t += red[w][c];
        partial[(int64_t)blockIdx.x * 2 * d + c] = t;
    }
}

template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? fmaxf(v, u) : v + u;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();  // the previous reduction's readers are done with scratch
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = scratch[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = MAX ? fmaxf(t, scratch[w]) : t + scratch[w];
    return t;
}

__global__ void __launch_bounds__(ASB_THREADS)
attention_softmax_backward_kernel(int64_t rows, int L, int heads, const float* __restrict__ score,
                                  const float* __restrict__ dprob, const float* __restrict__ key_bias,
                                  const uint8_t* __restrict__ key_mask, const float* __restrict__ q_scale,
                                  __nv_bfloat16* __restrict__ prob, __nv_bfloat16* __restrict__ dlogit,
                                  float* __restrict__ scale_partial) {
    __shared__ float scratch[ASB_THREADS / 32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t bh = r / L;
        const int64_t b = bh / heads;
        const int h = (int)(bh - b * heads);
        const float scale = q_scale[h];
        const float* s = score + r * (int64_t)L;
        const float* dp = dprob + r * (int64_t)L;
        const float* bias = key_bias ? key_bias + b * (int64_t)L : nullptr;
        const uint8_t* mask = key_mask ? key_mask + b * (int64_t)L : nullptr;
        __nv_bfloat16* pr = prob + r * (int64_t)L;
        __nv_bfloat16* dz = dlogit + r * (int64_t)L;
        float top = -INFINITY;
        for (int j = threadIdx.x; j < L; j += blockDim.x) {
            if (mask && !mask[j]) continue;
            const float z = s[j] * scale + (bias ? bias[j] : 0.0f);
            top = fmaxf(top, z);
        }
        top = block_reduce<true>(top, scratch);
        if (top == -INFINITY) {  // no key: the forward's row is zero, so is every gradient
            for (int j = threadIdx.x; j < L; j += blockDim.x) {
                pr[j] = __float2bfloat16_rn(0.0f);
                dz[j] = __float2bfloat16_rn(0.0f);
            }
            if (threadIdx.x == 0) scale_partial[r] = 0.0f;
            continue;
        }
        float total = 0.0f;
        for (int j = threadIdx.x; j < L; j += blockDim.x) {
            if (mask && !mask[j]) continue;
            total += expf(s[j] * scale + (bias ? bias[j] : 0.0f) - top);
        }
        const float inv_total = 1.0f / block_reduce<false>(total, scratch);
        float dot = 0.0f;
        for (int j = threadIdx.x; j < L; j += blockDim.x) {
            float p = 0.0f;
            if (!mask || mask[j]) p = expf(s[j] * scale + (bias ? bias[j] : 0.0f) - top) * inv_total;
            pr[j] = __float2bfloat16_rn(p);
            dot += p * dp[j];
        }
        dot = block_reduce<false>(dot, scratch);
        float ds = 0.0f;
        for (int j = threadIdx.x; j < L; j += blockDim.x) {
            float g = 0.0f;
            const float raw = s[j];
            if (!mask || mask[j]) g = expf(raw * scale + (bias ? bias[j] : 0.0f) - top) * inv_total * (dp[j] - dot);
            dz[j] = __float2bfloat16_rn(g * scale);
            ds += g * raw;
        }
        ds = block_reduce<false>(ds, scratch);
        if (threadIdx.x == 0) scale_partial[r] = ds;
    }
}

int layernorm_backward_grid(int64_t rows) {
    const int64_t need = (rows + LNB_WARPS - 1) / LNB_WARPS;
    const int64_t cap = 4 * (int64_t)sm_count();
    return (int)(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace
}  // namespace pbg

using namespace pbg;

extern "C" {

int pbg_gelu_backward(int64_t M, int32_t N, const float* pre, int64_t ldp, const void* dy, int32_t dy_bf16,
                      int64_t ldd, void* out, int64_t ldo, void* stream) {
    PBG_REQUIRE(M >= 0 && N >= 1 && pre && dy && out && ldp >= N && ldd >= N && ldo >= N,
                "gelu_backward: bad arguments");
    if (M == 0) return PBG_OK;
    const int grid = stride_grid(M * (int64_t)N, GB_THREADS);
    auto* o = static_cast<__nv_bfloat16*>(out);
    if (dy_bf16)
        gelu_backward_kernel<<<grid, GB_THREADS, 0, as_stream(stream)>>>(
            M, N, pre, ldp, static_cast<const __nv_bfloat16*>(dy), ldd, o, ldo);
    else
        gelu_backward_kernel<<<grid, GB_THREADS, 0, as_stream(stream)>>>(M, N, pre, ldp,
                                                                         static_cast<const float*>(dy), ldd, o, ldo);
    return launch_status("gelu_backward");
}

int64_t pbg_layernorm_backward_partials(int64_t rows, int32_t d) {
    if (rows < 0 || d < 32 || d % 32 || d > 32 * LNB_MAX_PER_LANE) return -1;
    return (int64_t)layernorm_backward_grid(rows) * 2 * d;
}

int pbg_layernorm_backward(int64_t rows, int32_t d, const void* x, int32_t x_bf16, int64_t ldx, const float* gain,
                           float eps, const void* dy, int32_t dy_bf16, int64_t ldy, void* dx, int32_t dx_bf16,
                           int64_t lddx, float* partial, int64_t partial_len, void* stream) {
    PBG_REQUIRE(rows >= 0 && d >= 32 && d % 32 == 0 && d <= 32 * LNB_MAX_PER_LANE,
                "layernorm_backward: width %d must be a multiple of 32 up to %d", (int)d, 32 * LNB_MAX_PER_LANE);
    PBG_REQUIRE(x && dy && dx && partial && ldx >= d && ldy >= d && lddx >= d, "layernorm_backward: bad arguments");
    const int grid = layernorm_backward_grid(rows);
    PBG_REQUIRE(partial_len >= (int64_t)grid * 2 * d, "layernorm_backward: partials hold %lld floats, need %lld",
                (long long)partial_len, (long long)grid * 2 * d);
    cudaStream_t s = as_stream(stream);
    const dim3 block(LNB_WARPS * 32);
#define PBG_LNB(IN, DYT, OUT)                                                                                     \
    layernorm_backward_kernel<IN, DYT, OUT><<<grid, block, 0, s>>>(rows, d, static_cast<const IN*>(x), ldx, gain, \
                                                                   eps, static_cast<const DYT*>(dy), ldy,         \
                                                                   static_cast<OUT*>(dx), lddx, partial)
    if (x_bf16) {
        if (dy_bf16) {
            if (dx_bf16) PBG_LNB(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16); else PBG_LNB(__nv_bfloat16, __nv_bfloat16, float);
        } else {
            if (dx_bf16) PBG_LNB(__nv_bfloat16, float, __nv_bfloat16); else PBG_LNB(__nv_bfloat16, float, float);
        }
    } else {
        if (dy_bf16) {
            if (dx_bf16) PBG_LNB(float, __nv_bfloat16, __nv_bfloat16); else PBG_LNB(float, __nv_bfloat16, float);
        } else {
            if (dx_bf16) PBG_LNB(float, float, __nv_bfloat16); else PBG_LNB(float, float, float);
        }
    }
#undef PBG_LNB
    return launch_status("layernorm_backward");
}

int pbg_attention_softmax_backward(int64_t rows, int32_t len, int32_t heads, const float* score, const float* dprob,
                                   const float* key_bias, const uint8_t* key_mask, const float* q_scale, void* prob,
                                   void* dlogit, float* scale_partial, void* stream) {
    PBG_REQUIRE(rows >= 0 && len >= 1 && heads >= 1 && rows % ((int64_t)len * heads) == 0,
                "attention_softmax_backward: rows must be sequences x heads x length");
    PBG_REQUIRE(score && dprob && q_scale && prob && dlogit && scale_partial,
                "attention_softmax_backward: null argument");
    if (rows == 0) return PBG_OK;
    const int64_t cap = 16 * (int64_t)sm_count();
    const int grid = (int)(rows < cap ? rows : cap);
    attention_softmax_backward_kernel<<<grid, ASB_THREADS, 0, as_stream(stream)>>>(
        rows, len, heads, score, dprob, key_bias, key_mask, q_scale,
        static_cast<__nv_bfloat16*>(prob), static_cast<__nv_bfloat16*>(dlogit), scale_partial);
    return launch_status("attention_softmax_backward");
}

}  // extern "C"
