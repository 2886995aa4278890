// Fused categorical PPO loss backward: one HBM pass over the decisions.
//
// Per row: masked log-softmax of the logits (the categorical policy of
// tests/categorical_policy_fixture.py:33-57), the clipped and
// negative-advantage-capped importance ratio of pbg/core/learner.py:2021-2077,
// the entropy bonus, the row's decision-mass weight, and d total / d logits.
// torch.minimum's half split at ties and torch.clamp's inclusive gradient
// bounds are restated exactly, so the gradient is the reference's autograd
// gradient, not an approximation of it.
//
// Layout: logits/dlogits [N,A] (bf16 or fp32), mask [N,A] u8, action [N]
// i32, old_logp/adv/weight [N] f32.  For A == 8 with 16-byte aligned rows
// one thread moves a whole row with 16/8/16-byte vector accesses (56 B per
// row with bf16 logits); other shapes take a scalar path.  Per-block loss
// statistics go to a caller scratch array and are summed in a fixed order by
// a one-block finalise kernel, so results are deterministic.
#include <cuda_bf16.h>

#include "pbg_common.cuh"

namespace pbg {

constexpr int LOSS_BLOCK = 256;
constexpr int LOSS_STATS = 8;
constexpr int LOSS_MAX_A = 32;

struct LossControls {
    float clip, cap, cent, coef_scale;  // coef_scale = scale * inv_count
};

__device__ __forceinline__ LossControls load_controls(const float* c) {
    LossControls k;
    k.clip = c[0];
    k.cap = c[1];
    k.cent = c[2];
    k.coef_scale = c[3] * c[4];
    return k;
}

struct RowStats {
    float v[LOSS_STATS];
    __device__ void zero() {
        #pragma unroll
        for (int i = 0; i < LOSS_STATS; ++i) v[i] = 0.0f;
    }
};

// d(policy_row)/d(log_ratio) and the row's policy loss (learner.py:2021-2047).
__device__ __forceinline__ float ratio_terms(float lr, float adv, const LossControls& k, float& prow,
                                             float& ratio_out) {
    float ratio = expf(lr);
    float lo = 1.0f - k.clip, hi = 1.0f + k.clip;
    float clipped = fminf(fmaxf(ratio, lo), hi);
    bool negative = adv < 0.0f;
    float neg_ratio = expf(fminf(lr, k.cap));
    float pr = negative ? neg_ratio : ratio;
    float f1 = pr * adv, f2 = clipped * adv;
    prow = -fminf(f1, f2);
    float g1 = f1 < f2 ? 1.0f : (f1 == f2 ? 0.5f : 0.0f);
    float g2 = f2 < f1 ? 1.0f : (f1 == f2 ? 0.5f : 0.0f);
    float dpr = negative ? neg_ratio * (lr < k.cap ? 1.0f : (lr == k.cap ? 0.5f : 0.0f)) : ratio;
    float dcl = (ratio >= lo && ratio <= hi) ? ratio : 0.0f;
    ratio_out = ratio;
    return -(g1 * adv * dpr + g2 * adv * dcl);
}

__device__ __forceinline__ void accumulate(RowStats& s, float coef, float w, float prow, float ent, float ratio,
                                           float lr, const LossControls& k, float adv) {
    s.v[0] += coef * (prow - k.cent * ent);
    s.v[1] += w * prow;
    s.v[2] += w * ent;
    s.v[3] += w * ((ratio - 1.0f) - lr);
    s.v[4] += fabsf(ratio - 1.0f) > k.clip ? 1.0f : 0.0f;
    s.v[5] += (adv < 0.0f && lr > k.cap) ? 1.0f : 0.0f;
    s.v[6] += w;
    s.v[7] += 1.0f;
}

// One row held in registers: x[j] logits, legal bitmask.
template <int A>
__device__ __forceinline__ void row_backward(float (&x)[A], unsigned legal, int act, float old, float adv, float w,
                                             const LossControls& k, RowStats& s) {
    float mx = -INFINITY;
    #pragma unroll
    for (int j = 0; j < A; ++j) if ((legal >> j) & 1u) mx = fmaxf(mx, x[j]);
    float e[A];
    float se = 0.0f;
    #pragma unroll
    for (int j = 0; j < A; ++j) {
        e[j] = ((legal >> j) & 1u) ? expf(x[j] - mx) : 0.0f;
        se += e[j];
    }
    float lse = mx + logf(se);
    float inv = __frcp_rn(se);
    float ent = 0.0f, lpa = 0.0f;
    #pragma unroll
    for (int j = 0; j < A; ++j) {
        float lp = x[j] - lse;
        if ((legal >> j) & 1u) ent -= e[j] * inv * lp;
        if (j == act) lpa = lp;
        x[j] = lp;  // reuse as log-probability
    }
    float lr = lpa - old;
    float prow, ratio;
    float dprow = ratio_terms(lr, adv, k, prow, ratio);
    float coef = k.coef_scale * w;
    #pragma unroll
    for (int j = 0; j < A; ++j) {
        float p = e[j] * inv;
        float g = dprow * ((j == act ? 1.0f : 0.0f) - p) + k.cent * p * (x[j] + ent);
        x[j] = ((legal >> j) & 1u) ? coef * g : 0.0f;  // reuse as dlogit
    }
    accumulate(s, coef, w, prow, ent, ratio, lr, k, adv);
}

// Block reduction of the 8 statistics into partials[block*8 + i].
__device__ __forceinline__ void block_stats(RowStats& s, double* partials) {
    __shared__ float red[LOSS_BLOCK / 32][LOSS_STATS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    #pragma unroll
    for (int i = 0; i < LOSS_STATS; ++i) {
        float v = warp_sum(s.v[i]);
        if (lane == 0) red[warp][i] = v;
    }
    __syncthreads();
    if (threadIdx.x < LOSS_STATS) {
        double acc = 0.0;
        for (int w = 0; w < LOSS_BLOCK / 32; ++w) acc += (double)red[w][threadIdx.x];
        partials[(int64_t)blockIdx.x * LOSS_STATS + threadIdx.x] = acc;
    }
}

__device__ __forceinline__ void bf16x8_to_float(const uint4& v, float (&x)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ uint4 float8_to_bf16(const float (&x)[8]) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
    #pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    return v;
}

__device__ __forceinline__ unsigned mask8(const uint2& m) {
    unsigned bits = 0;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        bits |= (((m.x >> (8 * j)) & 0xffu) != 0 ? 1u : 0u) << j;
        bits |= (((m.y >> (8 * j)) & 0xffu) != 0 ? 1u : 0u) << (j + 4);
    }
    return bits;
}

// A == 8, bf16: a row is one uint4 of logits, one uint2 of mask.
__global__ void __launch_bounds__(LOSS_BLOCK) ppo_bf16x8_kernel(int64_t N, const uint4* __restrict__ logits,
                                                                 const uint2* __restrict__ mask,
                                                                 const int32_t* __restrict__ action,
                                                                 const float* __restrict__ old_logp,
                                                                 const float* __restrict__ adv,
                                                                 const float* __restrict__ weight,
                                                                 const float* __restrict__ controls,
                                                                 uint4* __restrict__ dlogits, double* partials) {
    LossControls k = load_controls(controls);
    RowStats s;
    s.zero();
    const int64_t stride = (int64_t)gridDim.x * LOSS_BLOCK;
    int64_t r = (int64_t)blockIdx.x * LOSS_BLOCK + threadIdx.x;
    // two rows in flight per thread
    for (; r + stride < N; r += 2 * stride) {
        uint4 v0 = __ldcs(logits + r), v1 = __ldcs(logits + r + stride);
        uint2 m0 = __ldcs(mask + r), m1 = __ldcs(mask + r + stride);
        int a0 = __ldcs(action + r), a1 = __ldcs(action + r + stride);
        float o0 = __ldcs(old_logp + r), o1 = __ldcs(old_logp + r + stride);
        float d0 = __ldcs(adv + r), d1 = __ldcs(adv + r + stride);
        float w0 = __ldcs(weight + r), w1 = __ldcs(weight + r + stride);
        float x0[8], x1[8];
        bf16x8_to_float(v0, x0);
        bf16x8_to_float(v1, x1);
        row_backward<8>(x0, mask8(m0), a0, o0, d0, w0, k, s);
        row_backward<8>(x1, mask8(m1), a1, o1, d1, w1, k, s);
        __stcs(dlogits + r, float8_to_bf16(x0));
        __stcs(dlogits + r + stride, float8_to_bf16(x1));
    }
    if (r < N) {
        uint4 v0 = __ldcs(logits + r);
        uint2 m0 = __ldcs(mask + r);
        float x0[8];
        bf16x8_to_float(v0, x0);
        row_backward<8>(x0, mask8(m0), __ldcs(action + r), __ldcs(old_logp + r), __ldcs(adv + r),
                        __ldcs(weight + r), k, s);
        __stcs(dlogits + r, float8_to_bf16(x0));
    }
    block_stats(s, partials);
}

// Generic rows (A <= 32, fp32 or bf16, any alignment).
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(LOSS_BLOCK) ppo_generic_kernel(int64_t N, int A, const T* __restrict__ logits,
                                                                  const uint8_t* __restrict__ mask,
                                                                  const int32_t* __restrict__ action,
                                                                  const float* __restrict__ old_logp,
                                                                  const float* __restrict__ adv,
                                                                  const float* __restrict__ weight,
                                                                  const float* __restrict__ controls,
                                                                  T* __restrict__ dlogits, double* partials) {
    LossControls k = load_controls(controls);
    RowStats s;
    s.zero();
    for (int64_t r = (int64_t)blockIdx.x * LOSS_BLOCK + threadIdx.x; r < N; r += (int64_t)gridDim.x * LOSS_BLOCK) {
        float x[LOSS_MAX_A];
        unsigned legal = 0;
        #pragma unroll
        for (int j = 0; j < LOSS_MAX_A; ++j) {
            x[j] = 0.0f;
            if (j < A) {
                x[j] = to_f<T>(logits[r * A + j]);
                legal |= (mask[r * A + j] != 0 ? 1u : 0u) << j;
            }
        }
        row_backward<LOSS_MAX_A>(x, legal, action[r], old_logp[r], adv[r], weight[r], k, s);
        #pragma unroll
        for (int j = 0; j < LOSS_MAX_A; ++j)
            if (j < A) dlogits[r * A + j] = from_f<T>(x[j]);
    }
    block_stats(s, partials);
}

// Fixed-order sum of per-block statistics.
__global__ void ppo_finalize_kernel(int blocks, const double* partials, double* stats) {
    __shared__ double red[LOSS_BLOCK];
    for (int i = 0; i < LOSS_STATS; ++i) {
        double acc = 0.0;
        for (int b = threadIdx.x; b < blocks; b += blockDim.x) acc += partials[(int64_t)b * LOSS_STATS + i];
        red[threadIdx.x] = acc;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
            __syncthreads();
        }
        if (threadIdx.x == 0) stats[i] = red[0];
        __syncthreads();
    }
}

int ppo_grid(int64_t N) {
    // enough rows in flight to cover HBM latency: 8 resident blocks per SM
    return stride_grid(N, LOSS_BLOCK, 8);
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_ppo_partials_size(int64_t N, int32_t A) {
    (void)A;
    return (int64_t)ppo_grid(N > 0 ? N : 1) * LOSS_STATS;
}

int pbg_ppo_categorical_backward(int64_t N, int32_t A, int32_t dtype, const void* logits, const uint8_t* mask,
                                 const int32_t* action, const float* old_logp, const float* adv,
                                 const float* weight, const float* controls, void* dlogits, double* partials,
                                 double* stats, void* stream) {
    PBG_REQUIRE(N >= 0 && A >= 1 && A <= LOSS_MAX_A, "ppo: need N >= 0 and A in [1,32]");
    PBG_REQUIRE(dtype == 0 || dtype == 1, "ppo: dtype must be 0 (fp32) or 1 (bf16)");
    PBG_REQUIRE(logits && mask && action && old_logp && adv && weight && controls && dlogits && partials && stats,
                "ppo: null argument");
    cudaStream_t s = as_stream(stream);
    int grid = ppo_grid(N > 0 ? N : 1);
    bool vec = dtype == 1 && A == 8 && ((uintptr_t)logits % 16 == 0) && ((uintptr_t)dlogits % 16 == 0) &&
               ((uintptr_t)mask % 8 == 0);
    if (vec) {
        ppo_bf16x8_kernel<<<grid, LOSS_BLOCK, 0, s>>>(N, (const uint4*)logits, (const uint2*)mask, action, old_logp,
                                                      adv, weight, controls, (uint4*)dlogits, partials);
    } else if (dtype == 1) {
        ppo_generic_kernel<__nv_bfloat16><<<grid, LOSS_BLOCK, 0, s>>>(
            N, A, (const __nv_bfloat16*)logits, mask, action, old_logp, adv, weight, controls,
            (__nv_bfloat16*)dlogits, partials);
    } else {
        ppo_generic_kernel<float><<<grid, LOSS_BLOCK, 0, s>>>(N, A, (const float*)logits, mask, action, old_logp, adv,
                                                              weight, controls, (float*)dlogits, partials);
    }
    int rc = launch_status("ppo_categorical_backward");
    if (rc) return rc;
    ppo_finalize_kernel<<<1, LOSS_BLOCK, 0, s>>>(grid, partials, stats);
    return launch_status("ppo_finalize");
}

}  // extern "C"
