// Fused flat-buffer Adam/AdamW step for one optimizer lane.
//
// Restates pbg/core/optimization.py:182-233 (adam_transition) for K = 1:
// unscale by the loss scale, global 2-norm and finiteness, norm clipping,
// coupled or decoupled weight decay, bias-corrected moments, and the
// all-or-nothing rule (a non-finite gradient leaves masters and moments
// untouched and zeroes the gradient rows).  Two stream-ordered launches:
// per-block sum of squares, whose last block to finish computes the step's
// scalars (norm, clip scale, bias corrections) -> apply (four parameters per
// thread when the streams are 16-byte aligned).
// Algorithmic traffic: 4 B per parameter for the norm pass, 32 B for the apply.
// The dynamic fp16 loss-scale update (growth/backoff trackers) is not part
// of this step: the scale is read from controls[6] as given.
#include "pbg_common.cuh"

namespace pbg {

constexpr int ADAM_BLOCK = 256;

// report: [applied, finite, norm, clip_scale, step_after, c1, c2, unused]
// Run by one block of ADAM_BLOCK threads.
__device__ __forceinline__ void adam_finalize(int blocks, const double* partials, const float* controls,
                                              int64_t* step, double* report) {
    __shared__ double red[2][ADAM_BLOCK];
    double ss = 0.0, bad = 0.0;
    for (int b = threadIdx.x; b < blocks; b += blockDim.x) {
        ss += __ldcg(partials + 2 * (int64_t)b);
        bad += __ldcg(partials + 2 * (int64_t)b + 1);
    }
    red[0][threadIdx.x] = ss;
    red[1][threadIdx.x] = bad;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            red[0][threadIdx.x] += red[0][threadIdx.x + o];
            red[1][threadIdx.x] += red[1][threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        double norm = sqrt(red[0][0]);
        bool finite = red[1][0] == 0.0 && isfinite(norm);
        double clip = controls[5];
        double scale = fmin(clip / fmax(norm, 1.0e-12), 1.0);
        if (!finite) scale = 0.0;
        int64_t t = step[0] + (finite ? 1 : 0);
        double b1 = controls[1], b2 = controls[2];
        report[0] = finite ? 1.0 : 0.0;
        report[1] = finite ? 1.0 : 0.0;
        report[2] = finite ? norm : INFINITY;
        report[3] = scale;
        report[4] = (double)t;
        report[5] = fmax(1.0 - pow(b1, (double)t), 1.0e-30);
        report[6] = fmax(1.0 - pow(b2, (double)t), 1.0e-30);
        report[7] = 0.0;
        step[0] = t;
    }
}

__global__ void __launch_bounds__(ADAM_BLOCK) adam_norm_kernel(int64_t n, const float4* __restrict__ grad4,
                                                                const float* __restrict__ grad,
                                                                const float* controls, double* partials,
                                                                int64_t* step, double* report) {
    float inv_scale = 1.0f / controls[6];
    float ss = 0.0f;
    float bad = 0.0f;
    int64_t n4 = n / 4;
    for (int64_t i = (int64_t)blockIdx.x * ADAM_BLOCK + threadIdx.x; i < n4; i += (int64_t)gridDim.x * ADAM_BLOCK) {
        float4 g = __ldcs(grad4 + i);
        float a = g.x * inv_scale, b = g.y * inv_scale, c = g.z * inv_scale, d = g.w * inv_scale;
        ss += a * a + b * b + c * c + d * d;
        bad += (isfinite(a) && isfinite(b) && isfinite(c) && isfinite(d)) ? 0.0f : 1.0f;
    }
    for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * ADAM_BLOCK + threadIdx.x; i < n; i += (int64_t)gridDim.x * ADAM_BLOCK) {
        float a = grad[i] * inv_scale;
        ss += a * a;
        bad += isfinite(a) ? 0.0f : 1.0f;
    }
    __shared__ float red[2][ADAM_BLOCK / 32];
    float s1 = warp_sum(ss), s2 = warp_sum(bad);
    if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = s1; red[1][threadIdx.x >> 5] = s2; }
    __syncthreads();
    if (threadIdx.x < 2) {
        double acc = 0.0;
        for (int w = 0; w < ADAM_BLOCK / 32; ++w) acc += (double)red[threadIdx.x][w];
        partials[2 * (int64_t)blockIdx.x + threadIdx.x] = acc;
    }
    // the last block to arrive turns the per-block sums into the step's scalars (in block order, as a
    // separate one-block launch would) and clears the arrival counter for the next step
    __shared__ bool last;
    unsigned int* counter = reinterpret_cast<unsigned int*>(partials + 2 * (int64_t)gridDim.x);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    adam_finalize(gridDim.x, partials, controls, step, report);
    if (threadIdx.x == 0) *counter = 0u;
}


__global__ void __launch_bounds__(ADAM_BLOCK) adam_apply_kernel(int64_t n, float* __restrict__ master,
                                                                 float* __restrict__ grad, float* __restrict__ first,
                                                                 float* __restrict__ second, const float* controls,
                                                                 int decoupled, const double* report) {
    bool applied = report[0] != 0.0;
    float lr = controls[0], b1 = controls[1], b2 = controls[2], eps = controls[3], decay = controls[4];
    float inv_scale = 1.0f / controls[6];
    float clipping = (float)report[3];
    float coupled = decoupled ? 0.0f : decay;
    float inv_c1 = (float)(1.0 / report[5]);
    float inv_sqrt_c2 = (float)(1.0 / sqrt(report[6]));
    float shrink = 1.0f - lr * (decoupled ? decay : 0.0f);
    for (int64_t i = (int64_t)blockIdx.x * ADAM_BLOCK + threadIdx.x; i < n; i += (int64_t)gridDim.x * ADAM_BLOCK) {
        if (!applied) { grad[i] = 0.0f; continue; }
        float w = master[i];
        float g = grad[i] * inv_scale * clipping + coupled * w;
        float m = b1 * first[i] + (1.0f - b1) * g;
        float v = b2 * second[i] + (1.0f - b2) * g * g;
        float den = sqrtf(v) * inv_sqrt_c2 + eps;
        float dir = m * inv_c1 / den;
        master[i] = w * shrink - lr * dir;
        first[i] = m;
        second[i] = v;
        grad[i] = g;
    }
}

// The same update four parameters per thread (16-byte accesses), when every stream is 16-byte
// aligned; per element the arithmetic is the scalar kernel's, so the results are identical.
struct AdamScalars {
    bool applied;
    float lr, b1, b2, eps, inv_scale, clipping, coupled, inv_c1, inv_sqrt_c2, shrink;
};

__device__ __forceinline__ AdamScalars adam_scalars(const float* controls, int decoupled, const double* report) {
    AdamScalars k;
    k.applied = report[0] != 0.0;
    k.lr = controls[0];
    k.b1 = controls[1];
    k.b2 = controls[2];
    k.eps = controls[3];
    const float decay = controls[4];
    k.inv_scale = 1.0f / controls[6];
    k.clipping = (float)report[3];
    k.coupled = decoupled ? 0.0f : decay;
    k.inv_c1 = (float)(1.0 / report[5]);
    k.inv_sqrt_c2 = (float)(1.0 / sqrt(report[6]));
    k.shrink = 1.0f - k.lr * (decoupled ? decay : 0.0f);
    return k;
}

__device__ __forceinline__ void adam_one(const AdamScalars& k, float& w, float& g, float& m, float& v) {
    g = g * k.inv_scale * k.clipping + k.coupled * w;
    m = k.b1 * m + (1.0f - k.b1) * g;
    v = k.b2 * v + (1.0f - k.b2) * g * g;
    const float den = sqrtf(v) * k.inv_sqrt_c2 + k.eps;
    const float dir = m * k.inv_c1 / den;
    w = w * k.shrink - k.lr * dir;
}

__global__ void __launch_bounds__(ADAM_BLOCK) adam_apply4_kernel(int64_t n, float4* __restrict__ master,
                                                                  float4* __restrict__ grad, float4* __restrict__ first,
                                                                  float4* __restrict__ second, float* __restrict__ master1,
                                                                  float* __restrict__ grad1, float* __restrict__ first1,
                                                                  float* __restrict__ second1, const float* controls,
                                                                  int decoupled, const double* report) {
    const AdamScalars k = adam_scalars(controls, decoupled, report);
    const int64_t n4 = n / 4;
    const int64_t stride = (int64_t)gridDim.x * ADAM_BLOCK;
    for (int64_t i = (int64_t)blockIdx.x * ADAM_BLOCK + threadIdx.x; i < n4; i += stride) {
        if (!k.applied) {
            __stcs(grad + i, make_float4(0.0f, 0.0f, 0.0f, 0.0f));
            continue;
        }
        float4 w = __ldcs(master + i), g = __ldcs(grad + i), m = __ldcs(first + i), v = __ldcs(second + i);
        adam_one(k, w.x, g.x, m.x, v.x);
        adam_one(k, w.y, g.y, m.y, v.y);
        adam_one(k, w.z, g.z, m.z, v.z);
        adam_one(k, w.w, g.w, m.w, v.w);
        __stcs(master + i, w);
        __stcs(first + i, m);
        __stcs(second + i, v);
        __stcs(grad + i, g);
    }
    for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * ADAM_BLOCK + threadIdx.x; i < n; i += stride) {
        if (!k.applied) {
            grad1[i] = 0.0f;
            continue;
        }
        float w = master1[i], g = grad1[i], m = first1[i], v = second1[i];
        adam_one(k, w, g, m, v);
        master1[i] = w;
        first1[i] = m;
        second1[i] = v;
        grad1[i] = g;
    }
}

int adam_grid(int64_t n) { return stride_grid((n + 3) / 4, ADAM_BLOCK, 4); }

}  // namespace pbg

using namespace pbg;

extern "C" {

// per-block sums of squares and non-finite counts, then the arrival counter of the last-block finalise
int64_t pbg_adam_partials_size(int64_t n) { return 2 * (int64_t)adam_grid(n > 0 ? n : 1) + 1; }

int pbg_adam_step(int64_t n, float* master, float* grad, float* first, float* second, const float* controls,
                  int64_t* step, int32_t decoupled, double* partials, double* report, void* stream) {
    PBG_REQUIRE(n >= 0 && master && grad && first && second && controls && step && partials && report,
                "adam_step: null argument");
    PBG_REQUIRE(((uintptr_t)grad % 16) == 0, "adam_step: grad must be 16-byte aligned");
    cudaStream_t s = as_stream(stream);
    int grid = adam_grid(n > 0 ? n : 1);
    adam_norm_kernel<<<grid, ADAM_BLOCK, 0, s>>>(n, (const float4*)grad, grad, controls, partials, step, report);
    int rc = launch_status("adam_norm");
    if (rc) return rc;
    const bool vec = (uintptr_t)master % 16 == 0 && (uintptr_t)first % 16 == 0 && (uintptr_t)second % 16 == 0;
    if (n > 0 && vec)
        adam_apply4_kernel<<<adam_grid(n), ADAM_BLOCK, 0, s>>>(n, (float4*)master, (float4*)grad, (float4*)first,
                                                               (float4*)second, master, grad, first, second, controls,
                                                               decoupled, report);
    else if (n > 0)
        adam_apply_kernel<<<stride_grid(n, ADAM_BLOCK, 4), ADAM_BLOCK, 0, s>>>(n, master, grad, first, second,
                                                                             controls, decoupled, report);
    return launch_status("adam_apply");
}

}  // extern "C"
