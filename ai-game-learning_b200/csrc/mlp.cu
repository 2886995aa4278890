// The fp32 preflop-class MLP of cfg1 (two hidden layers of 256, ReLU) behind
// the reference's ModelOperation protocol (pbg/core/learner.py:324-350): the
// element-wise parts of its forward and backward around the dense maps.
//
//   bias_relu          y = max(y + b, 0) in place after the GEMM of a hidden layer
//   heads              the policy and value heads of the sampled class row,
//                      with the reference head's activations
//                      (pbg/games/poker/model/heads.py:28-62): type logits as
//                      they are, omega = softmax, mu = sigmoid, s = softplus +
//                      s_min, iota = sigmoid; value the row's value column
//   heads_backward     their vector-Jacobian product into the output row
//   relu_backward_bias dy *= (y > 0) and the bias gradient as column sums in a
//                      fixed order (blocks of 32 rows in row order, the blocks'
//                      sums strided over a warp's lanes, then a butterfly)
//
// The output row of the last dense map holds, for each of the K class rows,
// [type 3 | omega logits M | mu logits M | s pre-activations M | iota logit]
// and then the K values.
#include <cfloat>

#include "pbg_common.cuh"

namespace pbg {
namespace {

constexpr int MLP_THREADS = 256;
constexpr int MLP_MAXM = 8;
constexpr int MLP_ROW_BLOCK = 32;  // rows per partial column sum (loaded all at once)

__global__ void bias_relu_kernel(int64_t M, int N, float* __restrict__ y, const float* __restrict__ bias) {
    const int64_t n = M * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = __fadd_rn(y[i], bias[i % N]);
        y[i] = v > 0.0f ? v : 0.0f;
    }
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// torch.nn.functional.softplus with beta 1 and threshold 20
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__global__ void heads_kernel(int64_t S, int K, int M, float s_min, const float* __restrict__ z, int64_t ldz,
                             const float* __restrict__ bias, const int32_t* __restrict__ cls,
                             float* __restrict__ type_logits, float* __restrict__ omega, float* __restrict__ mu,
                             float* __restrict__ scale, float* __restrict__ iota, float* __restrict__ value,
                             uint32_t* __restrict__ status) {
    const int R = 4 + 3 * M;  // outputs per class row
    for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < S; s += (int64_t)gridDim.x * blockDim.x) {
        int c = cls[s];
        if (c < 0 || c >= K) {
            atomicOr(status, 1u);
            c = 0;
        }
        const float* row = z + s * ldz;
        const int base = c * R;
        #pragma unroll
        for (int j = 0; j < 3; ++j) type_logits[s * 3 + j] = __fadd_rn(row[base + j], bias[base + j]);
        float w[MLP_MAXM];
        float top = -FLT_MAX;
        for (int j = 0; j < M; ++j) {
            w[j] = __fadd_rn(row[base + 3 + j], bias[base + 3 + j]);
            top = fmaxf(top, w[j]);
        }
        float total = 0.0f;
        for (int j = 0; j < M; ++j) {
            w[j] = expf(w[j] - top);
            total += w[j];
        }
        for (int j = 0; j < M; ++j) {
            omega[s * M + j] = w[j] / total;
            mu[s * M + j] = sigmoid_f(__fadd_rn(row[base + 3 + M + j], bias[base + 3 + M + j]));
            scale[s * M + j] = __fadd_rn(softplus_f(__fadd_rn(row[base + 3 + 2 * M + j], bias[base + 3 + 2 * M + j])),
                                         s_min);
        }
        iota[s] = sigmoid_f(__fadd_rn(row[base + 3 + 3 * M], bias[base + 3 + 3 * M]));
        value[s] = __fadd_rn(row[K * R + c], bias[K * R + c]);
    }
}

__global__ void heads_backward_kernel(int64_t S, int K, int M, const float* __restrict__ z, int64_t ldz,
                                      const float* __restrict__ bias, const int32_t* __restrict__ cls,
                                      const float* __restrict__ omega, const float* __restrict__ mu,
                                      const float* __restrict__ iota, const float* __restrict__ d_type,
                                      const float* __restrict__ d_omega, const float* __restrict__ d_mu,
                                      const float* __restrict__ d_scale, const float* __restrict__ d_iota,
                                      const float* __restrict__ d_value, float* __restrict__ dz, int64_t lddz) {
    const int R = 4 + 3 * M;
    for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < S; s += (int64_t)gridDim.x * blockDim.x) {
        int c = cls[s];
        if (c < 0 || c >= K) c = 0;  // flagged by the forward
        float* out = dz + s * lddz;
        const int base = c * R;
        #pragma unroll
        for (int j = 0; j < 3; ++j) out[base + j] = d_type[s * 3 + j];
        float dot = 0.0f;
        for (int j = 0; j < M; ++j) dot += omega[s * M + j] * d_omega[s * M + j];
        for (int j = 0; j < M; ++j) {
            const float o = omega[s * M + j];
            out[base + 3 + j] = o * (d_omega[s * M + j] - dot);
            const float m = mu[s * M + j];
            out[base + 3 + M + j] = d_mu[s * M + j] * (m * (1.0f - m));
            const float pre = __fadd_rn(z[s * ldz + base + 3 + 2 * M + j], bias[base + 3 + 2 * M + j]);
            out[base + 3 + 2 * M + j] = pre > 20.0f ? d_scale[s * M + j] : d_scale[s * M + j] * sigmoid_f(pre);
        }
        const float io = iota[s];
        out[base + 3 + 3 * M] = d_iota[s] * (io * (1.0f - io));
        out[K * R + c] = d_value[s];
    }
}

// Per block: the column sums of rows [r0, r0 + MLP_ROW_BLOCK) after the ReLU mask; each thread
// loads its column's 32 rows at once and adds them in row order.
__global__ void relu_backward_partial_kernel(int64_t M, int N, float* __restrict__ dy, const float* __restrict__ y,
                                             float* __restrict__ partial) {
    const int64_t blocks = (M + MLP_ROW_BLOCK - 1) / MLP_ROW_BLOCK;
    for (int64_t blk = blockIdx.x; blk < blocks; blk += gridDim.x) {
        const int64_t r0 = blk * MLP_ROW_BLOCK;
        const int rows = (int)min((int64_t)MLP_ROW_BLOCK, M - r0);
        for (int n = threadIdx.x; n < N; n += blockDim.x) {
            float g[MLP_ROW_BLOCK];
            bool keep[MLP_ROW_BLOCK];
            #pragma unroll
            for (int r = 0; r < MLP_ROW_BLOCK; ++r) {
                g[r] = r < rows ? dy[(r0 + r) * N + n] : 0.0f;
                keep[r] = r < rows && (!y || y[(r0 + r) * N + n] > 0.0f);
            }
            float acc = 0.0f;
            #pragma unroll
            for (int r = 0; r < MLP_ROW_BLOCK; ++r) {
                if (r < rows && !keep[r]) dy[(r0 + r) * N + n] = 0.0f;
                acc += keep[r] ? g[r] : 0.0f;
            }
            partial[blk * N + n] = acc;
        }
    }
}

// One warp per column: lane l adds the partials of blocks l, l + 32, ... in order, then a fixed
// butterfly adds the lanes.
__global__ void column_total_kernel(int64_t blocks, int N, const float* __restrict__ partial, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t n = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
        float acc = 0.0f;
        for (int64_t b = lane; b < blocks; b += 32) acc += partial[b * N + n];
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) out[n] = acc;
    }
}

}  // namespace
}  // namespace pbg

using namespace pbg;

extern "C" {

int pbg_mlp_bias_relu(int64_t M, int32_t N, float* y, const float* bias, void* stream) {
    PBG_REQUIRE(M >= 0 && N >= 1 && y && bias, "mlp_bias_relu: bad arguments");
    if (M == 0) return PBG_OK;
    bias_relu_kernel<<<stride_grid(M * N, MLP_THREADS), MLP_THREADS, 0, as_stream(stream)>>>(M, N, y, bias);
    return launch_status("mlp_bias_relu");
}

int pbg_mlp_heads(int64_t S, int32_t K, int32_t M, float s_min, const float* z, int64_t ldz, const float* bias,
                  const int32_t* cls, float* type_logits, float* omega, float* mu, float* scale, float* iota,
                  float* value, uint32_t* status, void* stream) {
    PBG_REQUIRE(S >= 0 && K >= 1 && M >= 1 && M <= MLP_MAXM && ldz >= (int64_t)K * (5 + 3 * M),
                "mlp_heads: bad shape");
    PBG_REQUIRE(z && bias && cls && type_logits && omega && mu && scale && iota && value && status,
                "mlp_heads: null argument");
    if (S == 0) return PBG_OK;
    heads_kernel<<<stride_grid(S, MLP_THREADS), MLP_THREADS, 0, as_stream(stream)>>>(
        S, K, M, s_min, z, ldz, bias, cls, type_logits, omega, mu, scale, iota, value, status);
    return launch_status("mlp_heads");
}

int pbg_mlp_heads_backward(int64_t S, int32_t K, int32_t M, const float* z, int64_t ldz, const float* bias,
                           const int32_t* cls, const float* omega, const float* mu, const float* iota,
                           const float* d_type, const float* d_omega, const float* d_mu, const float* d_scale,
                           const float* d_iota, const float* d_value, float* dz, int64_t lddz, void* stream) {
    PBG_REQUIRE(S >= 0 && K >= 1 && M >= 1 && M <= MLP_MAXM && ldz >= (int64_t)K * (5 + 3 * M) &&
                    lddz >= (int64_t)K * (5 + 3 * M),
                "mlp_heads_backward: bad shape");
    PBG_REQUIRE(z && bias && cls && omega && mu && iota && d_type && d_omega && d_mu && d_scale && d_iota && d_value &&
                    dz,
                "mlp_heads_backward: null argument");
    if (S == 0) return PBG_OK;
    int err = cuda_status(cudaMemsetAsync(dz, 0, (size_t)S * lddz * sizeof(float), as_stream(stream)),
                          "mlp_heads_backward: clear");
    if (err) return err;
    heads_backward_kernel<<<stride_grid(S, MLP_THREADS), MLP_THREADS, 0, as_stream(stream)>>>(
        S, K, M, z, ldz, bias, cls, omega, mu, iota, d_type, d_omega, d_mu, d_scale, d_iota, d_value, dz, lddz);
    return launch_status("mlp_heads_backward");
}

int64_t pbg_mlp_bias_partials(int64_t M, int32_t N) {
    if (M < 0 || N < 1) return -1;
    return ((M + MLP_ROW_BLOCK - 1) / MLP_ROW_BLOCK) * (int64_t)N;
}

int pbg_mlp_relu_backward_bias(int64_t M, int32_t N, float* dy, const float* y, float* dbias, float* partial,
                               int64_t partial_len, void* stream) {
    PBG_REQUIRE(M >= 0 && N >= 1 && dy && dbias && partial, "mlp_relu_backward_bias: bad arguments");
    const int64_t blocks = (M + MLP_ROW_BLOCK - 1) / MLP_ROW_BLOCK;
    PBG_REQUIRE(partial_len >= blocks * N, "mlp_relu_backward_bias: partials hold %lld floats, need %lld",
                (long long)partial_len, (long long)(blocks * N));
    if (M == 0) {
        return cuda_status(cudaMemsetAsync(dbias, 0, (size_t)N * sizeof(float), as_stream(stream)),
                           "mlp_relu_backward_bias: clear");
    }
    const int grid = (int)(blocks < 16 * (int64_t)sm_count() ? blocks : 16 * (int64_t)sm_count());
    relu_backward_partial_kernel<<<grid, MLP_THREADS, 0, as_stream(stream)>>>(M, N, dy, y, partial);
    int err = launch_status("mlp_relu_backward_bias: partials");
    if (err) return err;
    column_total_kernel<<<(N + 7) / 8, MLP_THREADS, 0, as_stream(stream)>>>(blocks, N, partial, dbias);
    return launch_status("mlp_relu_backward_bias: totals");
}

}  // extern "C"
