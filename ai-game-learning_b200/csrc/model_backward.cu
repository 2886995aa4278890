// The element-wise and row-wise parts of the policy/value network's backward
// (pbg/games/poker/model/primitives.py FFN and MHA, pbg/core/tensor_ops.py
// LayerNorm, as differentiated by torch autograd in the reference's learner
// step, pbg/core/training.py:381-403).  The dense maps' products (dX = dY W,
// dW = dY^T X) are library GEMMs; these kernels sit between them, and the
// attention backward is one fused pass of its own.
//
//   gelu_backward      dpre = dy * (Phi(pre) + pre * phi(pre)) for the exact
//                      (erf) GELU, bf16 out: the operand of the map's dX / dW
//                      products (for maps with an fp32 output; a bf16-output
//                      map gets dpre from its GEMM's epilogue,
//                      pbg_linear_gelu_backward)
//   layernorm_backward warp per row: the statistics recomputed from the row,
//                      dx = inv * (g dy - mean(g dy) - xhat mean(g dy xhat)),
//                      and per-block column sums of dy * xhat (gain) and dy
//                      (bias) in a fixed order (the host adds the blocks' rows)
//   attention backward (fused, below): dQ, dK, dV and the score-scale
//                      gradient from the forward's log-sum-exp, the scores
//                      recomputed tile by tile on the tensor cores
#include <cuda_bf16.h>

#include <cmath>

#include "pbg_common.cuh"

namespace pbg {
namespace {

constexpr int GB_THREADS = 256;
constexpr int LNB_WARPS = 8;
constexpr int LNB_MAX_WIDTH = 512;

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

// PER: the columns a lane holds (d <= 32 PER)
template <int PER, typename In, typename DY, typename Out>
__global__ void __launch_bounds__(LNB_WARPS * 32)
layernorm_backward_kernel(int64_t rows, int d, const In* __restrict__ x, int64_t ldx, const float* __restrict__ gain,
                          float eps, const DY* __restrict__ dy, int64_t ldy, Out* __restrict__ dx, int64_t lddx,
                          float* __restrict__ partial) {
    __shared__ float red[LNB_WARPS][2 * 32 * PER];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = d >> 5;
    float acc_g[PER], acc_b[PER];
    #pragma unroll
    for (int i = 0; i < PER; ++i) acc_g[i] = acc_b[i] = 0.0f;
    const int64_t warps = (int64_t)gridDim.x * LNB_WARPS;
    for (int64_t r = (int64_t)blockIdx.x * LNB_WARPS + warp; r < rows; r += warps) {
        const In* xr = x + r * ldx;
        const DY* dr = dy + r * ldy;
        float v[PER], g[PER];
        float sum = 0.0f;
        #pragma unroll
        for (int i = 0; i < PER; ++i) {
            if (i < per) {
                v[i] = load_f(xr + lane + 32 * i);
                sum += v[i];
            }
        }
        const float mean = warp_sum(sum) / (float)d;
        float sq = 0.0f;
        #pragma unroll
        for (int i = 0; i < PER; ++i)
            if (i < per) sq += (v[i] - mean) * (v[i] - mean);
        const float inv = rsqrtf(warp_sum(sq) / (float)d + eps);
        float s1 = 0.0f, s2 = 0.0f;
        #pragma unroll
        for (int i = 0; i < PER; ++i) {
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
        for (int i = 0; i < PER; ++i)
            if (i < per) store_f(out + lane + 32 * i, inv * (g[i] - s1 - v[i] * s2));
    }
    #pragma unroll
    for (int i = 0; i < PER; ++i) {
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

// ---------------------------------------------------------------- fused attention backward
// FlashAttention-style: the scores never leave the chip.  With the forward's base-2 log-sum-exp
// lse2 of every (sequence, head, query) row and delta = sum_d dO O of the row, for a query/key tile
// pair: z2 = s * scale_h * log2(e) + bias * log2(e) (absent key: -inf), P = 2^(z2 - lse2),
// dP = dO V^T, dZ = P (dP - delta) (the logit gradient), and with dS = dZ * scale_h:
// dQ = dS K, dK = dS^T Q, dV = P^T dO; the head's scale gradient sums dZ * s.  Two kernels, no
// atomics: one CTA per 64-query block computes dQ (looping over key blocks), one per 64-key block
// dK and dV (looping over query blocks).  Each of the 4 warps owns 16 rows; the products run on
// mma.sync m16n8k16 (bf16 operands, fp32 accumulation) with operand tiles staged in shared memory
// row-major at a stride of 40 elements, which makes every ldmatrix read bank-conflict free; the
// products that contract over a tile's rows read it with ldmatrix.trans.
constexpr int AB_TILE = 64;
constexpr int AB_LD = 40;
constexpr float AB_LOG2E = 1.4426950408889634f;
constexpr int AB_DKV_BLOCKS = 2;  // 16-key row blocks per warp in the dK/dV kernel
constexpr int AB_DQ_BLOCKS = 2;   // 16-query row blocks per warp in the dQ kernel

__device__ __forceinline__ void ab_mma(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ab_pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float ab_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t ab_ld32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// four 8x8 bf16 matrices from shared memory; lane l gives the address of row l % 8 of matrix l / 8
// and receives, of each matrix i, the pair (row l / 4, columns 2 (l % 4) + {0, 1}) in r[i]: with the
// rows of a tile as the MMA's n index and 8 consecutive k per matrix, r[0..1] and r[2..3] are the
// B fragments of two consecutive k steps of 16
// the same four matrices transposed: lane l receives (rows 2 (l % 4) + {0, 1}, column l / 4), the B
// fragment of an MMA whose k index runs along the stored rows (a row-major [k][n] tile)
__device__ __forceinline__ void ab_ldm4t(uint32_t r[4], const __nv_bfloat16* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p))
                 : "memory");
}

__device__ __forceinline__ void ab_ldm4(uint32_t r[4], const __nv_bfloat16* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p))
                 : "memory");
}

// A fragments (two k-steps of 16 columns) of a warp's 16 rows x 32 columns of a row-major bf16
// matrix in global memory (rows at or past `rows` read as zero)
__device__ __forceinline__ void ab_rows_a(const __nv_bfloat16* base, int64_t ld, int row0, int rows, int g, int t,
                                          uint32_t a[2][4]) {
    const bool v0 = row0 + g < rows, v1 = row0 + g + 8 < rows;
    const __nv_bfloat16* r0 = base + (int64_t)(row0 + g) * ld;
    const __nv_bfloat16* r1 = base + (int64_t)(row0 + g + 8) * ld;
#pragma unroll
    for (int kt = 0; kt < 2; ++kt) {
        a[kt][0] = v0 ? ab_ld32(r0 + 16 * kt + 2 * t) : 0u;
        a[kt][1] = v1 ? ab_ld32(r1 + 16 * kt + 2 * t) : 0u;
        a[kt][2] = v0 ? ab_ld32(r0 + 16 * kt + 2 * t + 8) : 0u;
        a[kt][3] = v1 ? ab_ld32(r1 + 16 * kt + 2 * t + 8) : 0u;
    }
}

// A tile of 64 rows x 32 columns (row r at base + (row0 + r) * ld; absent rows zero) moves through
// registers: ab_fetch loads this thread's 16 columns of one row, ab_put stores them into `tile`
// (row-major, stride AB_LD).  The kernels fetch the next tile before computing on the current one,
// so its load latency overlaps the tensor-core work.
__device__ __forceinline__ void ab_fetch(const __nv_bfloat16* base, int64_t ld, int row0, int rows, uint4 v[2]) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    v[0] = v[1] = make_uint4(0u, 0u, 0u, 0u);
    if (row0 + r < rows) {
        const uint4* src = reinterpret_cast<const uint4*>(base + (int64_t)(row0 + r) * ld + 16 * half);
        v[0] = src[0];
        v[1] = src[1];
    }
}

__device__ __forceinline__ void ab_put(const uint4 v[2], __nv_bfloat16* tile) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    uint4* dst = reinterpret_cast<uint4*>(tile + r * AB_LD + 16 * half);
    dst[0] = v[0];
    dst[1] = v[1];
}

__device__ __forceinline__ float ab_key_term(const float* bias, const uint8_t* mask, int64_t at, bool present) {
    if (!present || (mask && !mask[at])) return -INFINITY;
    return bias ? bias[at] * AB_LOG2E : 0.0f;
}

struct AttnBackArgs {
    int batch, len, heads;
    const __nv_bfloat16* qkv;   // [batch, len, 3 * heads * 32]
    const __nv_bfloat16* dout;  // [batch, len, heads * 32]
    const float* lse;           // [batch, heads, len] base 2
    const float* delta;         // [batch, heads, len]
    const float* key_bias;      // [batch, len] or null
    const uint8_t* key_mask;    // [batch, len] or null
    const float* q_scale;       // [heads]
    __nv_bfloat16* dqkv;        // [batch, len, 3 * heads * 32]
    float* scale_partial;       // [batch, heads, len]
};

__global__ void __launch_bounds__(128) attention_delta_kernel(int64_t rows, int heads, const __nv_bfloat16* out,
                                                              const __nv_bfloat16* dout, int len, float* delta) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x) {
        // i = (b * len + q) * heads + h
        const int h = (int)(i % heads);
        const int64_t bq = i / heads;
        const uint4* o = reinterpret_cast<const uint4*>(out + i * 32);
        const uint4* g = reinterpret_cast<const uint4*>(dout + i * 32);
        float acc = 0.0f;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const uint4 a = o[v], c = g[v];
            const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
            const __nv_bfloat162* pc = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 fa = __bfloat1622float2(pa[e]), fc = __bfloat1622float2(pc[e]);
                acc += fa.x * fc.x + fa.y * fc.y;
            }
        }
        const int64_t b = bq / len, q = bq - b * len;
        delta[(b * heads + h) * len + q] = acc;
    }
}

// RB row blocks of 16 queries per warp (4 * 16 * RB queries per CTA), as in the dK/dV kernel: every
// K / V fragment read from shared memory feeds RB products; keys taken in two halves of 32
template <int RB>
__global__ void __launch_bounds__(128, RB == 1 ? 4 : 2) attention_dq_kernel(AttnBackArgs A) {
    __shared__ __align__(16) __nv_bfloat16 ks[AB_TILE * AB_LD], vs[AB_TILE * AB_LD];
    __shared__ __align__(8) float kterm[AB_TILE];
    constexpr int QUERIES = 64 * RB;  // queries per CTA
    const int qblocks = (A.len + QUERIES - 1) / QUERIES;
    const int qb = blockIdx.x % qblocks;
    const int h = (blockIdx.x / qblocks) % A.heads;
    const int b = blockIdx.x / (qblocks * A.heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int lrow = lane & 7, lmat = lane >> 3;
    const int d = A.heads * 32, width = 3 * d;
    const int q0 = qb * QUERIES + 16 * RB * warp;  // row block r: queries q0 + 16 r + {g, g + 8}
    const float scale = A.q_scale[h], scale2 = scale * AB_LOG2E;
    const __nv_bfloat16* seq = A.qkv + (int64_t)b * A.len * width + h * 32;
    const int64_t row_base = ((int64_t)b * A.heads + h) * A.len;
    uint32_t qa[RB][2][4], da[RB][2][4];
    float lse0[RB], lse1[RB], dl0[RB], dl1[RB], th0[RB], th1[RB];
    float dq[RB][4][4];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        const int qr = q0 + 16 * r;
        ab_rows_a(seq, width, qr, A.len, g, t, qa[r]);
        ab_rows_a(A.dout + (int64_t)b * A.len * d + h * 32, d, qr, A.len, g, t, da[r]);
        const bool v0 = qr + g < A.len, v1 = qr + g + 8 < A.len;
        lse0[r] = v0 ? A.lse[row_base + qr + g] : INFINITY;
        lse1[r] = v1 ? A.lse[row_base + qr + g + 8] : INFINITY;
        dl0[r] = v0 ? A.delta[row_base + qr + g] : 0.0f;
        dl1[r] = v1 ? A.delta[row_base + qr + g + 8] : 0.0f;
        th0[r] = th1[r] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) dq[r][i][0] = dq[r][i][1] = dq[r][i][2] = dq[r][i][3] = 0.0f;
    }
    const int kblocks = (A.len + AB_TILE - 1) / AB_TILE;
    uint4 kv[2], vv[2];
    float term = 0.0f;
    ab_fetch(seq + d, width, 0, A.len, kv);
    ab_fetch(seq + 2 * d, width, 0, A.len, vv);
    if (threadIdx.x < AB_TILE)
        term = ab_key_term(A.key_bias, A.key_mask, (int64_t)b * A.len + threadIdx.x, (int)threadIdx.x < A.len);
    for (int kb = 0; kb < kblocks; ++kb) {
        __syncthreads();  // the previous block's tiles are consumed
        ab_put(kv, ks);
        ab_put(vv, vs);
        if (threadIdx.x < AB_TILE) kterm[threadIdx.x] = term;
        __syncthreads();
        if (kb + 1 < kblocks) {  // the next block's rows, in flight during this block's products
            const int k1 = (kb + 1) * AB_TILE;
            ab_fetch(seq + d, width, k1, A.len, kv);
            ab_fetch(seq + 2 * d, width, k1, A.len, vv);
            if (threadIdx.x < AB_TILE)
                term = ab_key_term(A.key_bias, A.key_mask, (int64_t)b * A.len + k1 + threadIdx.x,
                                   k1 + (int)threadIdx.x < A.len);
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // keys 32 half .. 32 half + 31 of the block
            float s[RB][4][4], dp[RB][4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int nt = 4 * half + j;
                uint32_t kb4[4], vb4[4];
                ab_ldm4(kb4, ks + (8 * nt + lrow) * AB_LD + 8 * lmat);
                ab_ldm4(vb4, vs + (8 * nt + lrow) * AB_LD + 8 * lmat);
#pragma unroll
                for (int r = 0; r < RB; ++r) {
                    s[r][j][0] = s[r][j][1] = s[r][j][2] = s[r][j][3] = 0.0f;
                    dp[r][j][0] = dp[r][j][1] = dp[r][j][2] = dp[r][j][3] = 0.0f;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        ab_mma(s[r][j], qa[r][k], kb4[2 * k], kb4[2 * k + 1]);
                        ab_mma(dp[r][j], da[r][k], vb4[2 * k], vb4[2 * k + 1]);
                    }
                }
            }
            uint32_t dsa[RB][2][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 tp = *reinterpret_cast<const float2*>(kterm + 8 * (4 * half + j) + 2 * t);
                const float t0 = tp.x, t1 = tp.y;
#pragma unroll
                for (int r = 0; r < RB; ++r) {
                    const float p0 = ab_exp2(fmaf(s[r][j][0], scale2, t0) - lse0[r]);
                    const float p1 = ab_exp2(fmaf(s[r][j][1], scale2, t1) - lse0[r]);
                    const float p2 = ab_exp2(fmaf(s[r][j][2], scale2, t0) - lse1[r]);
                    const float p3 = ab_exp2(fmaf(s[r][j][3], scale2, t1) - lse1[r]);
                    const float z0 = p0 * (dp[r][j][0] - dl0[r]), z1 = p1 * (dp[r][j][1] - dl0[r]);
                    const float z2 = p2 * (dp[r][j][2] - dl1[r]), z3 = p3 * (dp[r][j][3] - dl1[r]);
                    th0[r] += z0 * s[r][j][0] + z1 * s[r][j][1];
                    th1[r] += z2 * s[r][j][2] + z3 * s[r][j][3];
                    // C fragment of n-tile j -> half of the A fragment of key step j / 2
                    dsa[r][j >> 1][(j & 1) * 2] = ab_pack(z0 * scale, z1 * scale);
                    dsa[r][j >> 1][(j & 1) * 2 + 1] = ab_pack(z2 * scale, z3 * scale);
                }
            }
            // dQ += dS K: the k index (keys) runs along the rows of the K tile
#pragma unroll
            for (int kl = 0; kl < 2; ++kl) {
                const int kk = 2 * half + kl;
#pragma unroll
                for (int nt = 0; nt < 4; nt += 2) {
                    uint32_t b4[4];
                    ab_ldm4t(b4, ks + (16 * kk + 8 * (lmat & 1) + lrow) * AB_LD + 8 * (nt + (lmat >> 1)));
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        ab_mma(dq[r][nt], dsa[r][kl], b4[0], b4[1]);
                        ab_mma(dq[r][nt + 1], dsa[r][kl], b4[2], b4[3]);
                    }
                }
            }
        }
    }
    __nv_bfloat16* out = A.dqkv + (int64_t)b * A.len * width + h * 32;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        float a = th0[r], c = th1[r];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        const int qr = q0 + 16 * r;
        const bool v0 = qr + g < A.len, v1 = qr + g + 8 < A.len;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            if (v0)
                *reinterpret_cast<uint32_t*>(out + (int64_t)(qr + g) * width + 8 * nt + 2 * t) =
                    ab_pack(dq[r][nt][0], dq[r][nt][1]);
            if (v1)
                *reinterpret_cast<uint32_t*>(out + (int64_t)(qr + g + 8) * width + 8 * nt + 2 * t) =
                    ab_pack(dq[r][nt][2], dq[r][nt][3]);
        }
        if (t == 0) {
            if (v0) A.scale_partial[row_base + qr + g] = a;
            if (v1) A.scale_partial[row_base + qr + g + 8] = c;
        }
    }
}

// RB row blocks of 16 keys per warp (4 * 16 * RB keys per CTA): every B fragment read from shared
// memory feeds RB products, which divides the kernel's shared-memory traffic per pair by RB (it is
// bound by that traffic); the queries of a tile are taken in two halves of 32 to bound registers
template <int RB>
__global__ void __launch_bounds__(128, RB == 1 ? 4 : 2) attention_dkv_kernel(AttnBackArgs A) {
    __shared__ __align__(16) __nv_bfloat16 qs[AB_TILE * AB_LD], gs[AB_TILE * AB_LD];
    __shared__ __align__(8) float lse_s[AB_TILE], delta_s[AB_TILE];
    constexpr int KEYS = 64 * RB;  // keys per CTA
    const int kblocks = (A.len + KEYS - 1) / KEYS;
    const int kb = blockIdx.x % kblocks;
    const int h = (blockIdx.x / kblocks) % A.heads;
    const int b = blockIdx.x / (kblocks * A.heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int lrow = lane & 7, lmat = lane >> 3;
    const int d = A.heads * 32, width = 3 * d;
    const int k0 = kb * KEYS + 16 * RB * warp;  // row block r: keys k0 + 16 r + {g, g + 8}
    const float scale = A.q_scale[h], scale2 = scale * AB_LOG2E;
    const __nv_bfloat16* seq = A.qkv + (int64_t)b * A.len * width + h * 32;
    const __nv_bfloat16* grad = A.dout + (int64_t)b * A.len * d + h * 32;
    uint32_t ka[RB][2][4], va[RB][2][4];
    float kt0[RB], kt1[RB];
    float dk[RB][4][4], dv[RB][4][4];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        const int kr = k0 + 16 * r;
        ab_rows_a(seq + d, width, kr, A.len, g, t, ka[r]);
        ab_rows_a(seq + 2 * d, width, kr, A.len, g, t, va[r]);
        kt0[r] = ab_key_term(A.key_bias, A.key_mask, (int64_t)b * A.len + kr + g, kr + g < A.len);
        kt1[r] = ab_key_term(A.key_bias, A.key_mask, (int64_t)b * A.len + kr + g + 8, kr + g + 8 < A.len);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dk[r][i][0] = dk[r][i][1] = dk[r][i][2] = dk[r][i][3] = 0.0f;
            dv[r][i][0] = dv[r][i][1] = dv[r][i][2] = dv[r][i][3] = 0.0f;
        }
    }
    const int64_t row_base = ((int64_t)b * A.heads + h) * A.len;
    const int qblocks = (A.len + AB_TILE - 1) / AB_TILE;
    uint4 qv[2], gv[2];
    float lv = INFINITY, dv_ = 0.0f;
    ab_fetch(seq, width, 0, A.len, qv);
    ab_fetch(grad, d, 0, A.len, gv);
    if (threadIdx.x < AB_TILE && (int)threadIdx.x < A.len) {
        lv = A.lse[row_base + threadIdx.x];
        dv_ = A.delta[row_base + threadIdx.x];
    }
    for (int qb = 0; qb < qblocks; ++qb) {
        __syncthreads();
        ab_put(qv, qs);
        ab_put(gv, gs);
        if (threadIdx.x < AB_TILE) {
            lse_s[threadIdx.x] = lv;
            delta_s[threadIdx.x] = dv_;
        }
        __syncthreads();
        if (qb + 1 < qblocks) {  // the next block's rows, in flight during this block's products
            const int q1 = (qb + 1) * AB_TILE;
            ab_fetch(seq, width, q1, A.len, qv);
            ab_fetch(grad, d, q1, A.len, gv);
            const bool v = threadIdx.x < AB_TILE && q1 + (int)threadIdx.x < A.len;
            lv = v ? A.lse[row_base + q1 + threadIdx.x] : INFINITY;
            dv_ = v ? A.delta[row_base + q1 + threadIdx.x] : 0.0f;
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // queries 32 half .. 32 half + 31
            float s[RB][4][4], dp[RB][4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int nt = 4 * half + j;
                uint32_t qb4[4], gb4[4];
                ab_ldm4(qb4, qs + (8 * nt + lrow) * AB_LD + 8 * lmat);
                ab_ldm4(gb4, gs + (8 * nt + lrow) * AB_LD + 8 * lmat);
#pragma unroll
                for (int r = 0; r < RB; ++r) {
                    s[r][j][0] = s[r][j][1] = s[r][j][2] = s[r][j][3] = 0.0f;
                    dp[r][j][0] = dp[r][j][1] = dp[r][j][2] = dp[r][j][3] = 0.0f;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        ab_mma(s[r][j], ka[r][k], qb4[2 * k], qb4[2 * k + 1]);
                        ab_mma(dp[r][j], va[r][k], gb4[2 * k], gb4[2 * k + 1]);
                    }
                }
            }
            uint32_t pa[RB][2][4], dsa[RB][2][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = 8 * (4 * half + j) + 2 * t;
                const float2 lp = *reinterpret_cast<const float2*>(lse_s + c);
                const float2 ep = *reinterpret_cast<const float2*>(delta_s + c);
                const float l0 = lp.x, l1 = lp.y, e0 = ep.x, e1 = ep.y;
#pragma unroll
                for (int r = 0; r < RB; ++r) {
                    // rows: keys g (regs 0, 1) and g + 8 (regs 2, 3) of block r; columns: queries c, c + 1
                    const float p0 = ab_exp2(fmaf(s[r][j][0], scale2, kt0[r]) - l0);
                    const float p1 = ab_exp2(fmaf(s[r][j][1], scale2, kt0[r]) - l1);
                    const float p2 = ab_exp2(fmaf(s[r][j][2], scale2, kt1[r]) - l0);
                    const float p3 = ab_exp2(fmaf(s[r][j][3], scale2, kt1[r]) - l1);
                    const float z0 = p0 * (dp[r][j][0] - e0), z1 = p1 * (dp[r][j][1] - e1);
                    const float z2 = p2 * (dp[r][j][2] - e0), z3 = p3 * (dp[r][j][3] - e1);
                    pa[r][j >> 1][(j & 1) * 2] = ab_pack(p0, p1);
                    pa[r][j >> 1][(j & 1) * 2 + 1] = ab_pack(p2, p3);
                    dsa[r][j >> 1][(j & 1) * 2] = ab_pack(z0 * scale, z1 * scale);
                    dsa[r][j >> 1][(j & 1) * 2 + 1] = ab_pack(z2 * scale, z3 * scale);
                }
            }
            // dV += P^T dO and dK += dS^T Q: the k index (queries) runs along the rows of the dO and Q tiles
#pragma unroll
            for (int kl = 0; kl < 2; ++kl) {
                const int kk = 2 * half + kl;
#pragma unroll
                for (int nt = 0; nt < 4; nt += 2) {
                    const int at = (16 * kk + 8 * (lmat & 1) + lrow) * AB_LD + 8 * (nt + (lmat >> 1));
                    uint32_t gb4[4], qb4[4];
                    ab_ldm4t(gb4, gs + at);
                    ab_ldm4t(qb4, qs + at);
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        ab_mma(dv[r][nt], pa[r][kl], gb4[0], gb4[1]);
                        ab_mma(dv[r][nt + 1], pa[r][kl], gb4[2], gb4[3]);
                        ab_mma(dk[r][nt], dsa[r][kl], qb4[0], qb4[1]);
                        ab_mma(dk[r][nt + 1], dsa[r][kl], qb4[2], qb4[3]);
                    }
                }
            }
        }
    }
    __nv_bfloat16* out = A.dqkv + (int64_t)b * A.len * width + h * 32;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        const int kr = k0 + 16 * r;
        const bool v0 = kr + g < A.len, v1 = kr + g + 8 < A.len;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int col = 8 * nt + 2 * t;
            if (v0) {
                *reinterpret_cast<uint32_t*>(out + (int64_t)(kr + g) * width + d + col) = ab_pack(dk[r][nt][0], dk[r][nt][1]);
                *reinterpret_cast<uint32_t*>(out + (int64_t)(kr + g) * width + 2 * d + col) =
                    ab_pack(dv[r][nt][0], dv[r][nt][1]);
            }
            if (v1) {
                *reinterpret_cast<uint32_t*>(out + (int64_t)(kr + g + 8) * width + d + col) =
                    ab_pack(dk[r][nt][2], dk[r][nt][3]);
                *reinterpret_cast<uint32_t*>(out + (int64_t)(kr + g + 8) * width + 2 * d + col) =
                    ab_pack(dv[r][nt][2], dv[r][nt][3]);
            }
        }
    }
}

int layernorm_backward_grid(int64_t rows) {
    const int64_t need = (rows + LNB_WARPS - 1) / LNB_WARPS;
    const int64_t cap = 8 * (int64_t)sm_count();
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
    if (rows < 0 || d < 32 || d % 32 || d > LNB_MAX_WIDTH) return -1;
    return (int64_t)layernorm_backward_grid(rows) * 2 * d;
}

int pbg_layernorm_backward(int64_t rows, int32_t d, const void* x, int32_t x_bf16, int64_t ldx, const float* gain,
                           float eps, const void* dy, int32_t dy_bf16, int64_t ldy, void* dx, int32_t dx_bf16,
                           int64_t lddx, float* partial, int64_t partial_len, void* stream) {
    PBG_REQUIRE(rows >= 0 && d >= 32 && d % 32 == 0 && d <= LNB_MAX_WIDTH,
                "layernorm_backward: width %d must be a multiple of 32 up to %d", (int)d, LNB_MAX_WIDTH);
    PBG_REQUIRE(x && dy && dx && partial && ldx >= d && ldy >= d && lddx >= d, "layernorm_backward: bad arguments");
    const int grid = layernorm_backward_grid(rows);
    PBG_REQUIRE(partial_len >= (int64_t)grid * 2 * d, "layernorm_backward: partials hold %lld floats, need %lld",
                (long long)partial_len, (long long)grid * 2 * d);
    cudaStream_t s = as_stream(stream);
    const dim3 block(LNB_WARPS * 32);
#define PBG_LNB_PER(PER, IN, DYT, OUT)                                                                    \
    layernorm_backward_kernel<PER, IN, DYT, OUT><<<grid, block, 0, s>>>(                                   \
        rows, d, static_cast<const IN*>(x), ldx, gain, eps, static_cast<const DYT*>(dy), ldy, static_cast<OUT*>(dx), \
        lddx, partial)
#define PBG_LNB(IN, DYT, OUT)                  \
    do {                                       \
        if (d <= 128)                          \
            PBG_LNB_PER(4, IN, DYT, OUT);      \
        else if (d <= 256)                     \
            PBG_LNB_PER(8, IN, DYT, OUT);      \
        else                                   \
            PBG_LNB_PER(16, IN, DYT, OUT);     \
    } while (0)
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
#undef PBG_LNB_PER
    return launch_status("layernorm_backward");
}

int pbg_attention_backward(int32_t batch, int32_t len, int32_t heads, const void* qkv, const void* out,
                           const void* dout, const float* lse, const float* key_bias, const uint8_t* key_mask,
                           const float* q_scale, void* dqkv, float* delta, float* scale_partial, void* stream) {
    PBG_REQUIRE(batch >= 0 && len >= 0 && heads >= 1, "attention_backward: bad shape");
    PBG_REQUIRE(qkv && out && dout && lse && q_scale && dqkv && delta && scale_partial,
                "attention_backward: null argument");
    PBG_REQUIRE(((uintptr_t)qkv | (uintptr_t)out | (uintptr_t)dout | (uintptr_t)dqkv) % 16 == 0,
                "attention_backward: qkv, out, dout and dqkv must be 16-byte aligned");
    if (batch == 0 || len == 0) return PBG_OK;
    cudaStream_t s = as_stream(stream);
    const int64_t rows = (int64_t)batch * len * heads;
    attention_delta_kernel<<<stride_grid(rows, 128), 128, 0, s>>>(rows, heads, static_cast<const __nv_bfloat16*>(out),
                                                                  static_cast<const __nv_bfloat16*>(dout), len, delta);
    int err = launch_status("attention_backward: delta");
    if (err) return err;
    AttnBackArgs A;
    A.batch = batch;
    A.len = len;
    A.heads = heads;
    A.qkv = static_cast<const __nv_bfloat16*>(qkv);
    A.dout = static_cast<const __nv_bfloat16*>(dout);
    A.lse = lse;
    A.delta = delta;
    A.key_bias = key_bias;
    A.key_mask = key_mask;
    A.q_scale = q_scale;
    A.dqkv = static_cast<__nv_bfloat16*>(dqkv);
    A.scale_partial = scale_partial;
    const int64_t grid = (int64_t)batch * heads * ((len + AB_TILE - 1) / AB_TILE);
    PBG_REQUIRE(grid <= INT32_MAX, "attention_backward: too many blocks");
    const int64_t grid_q = (int64_t)batch * heads * ((len + 64 * AB_DQ_BLOCKS - 1) / (64 * AB_DQ_BLOCKS));
    attention_dq_kernel<AB_DQ_BLOCKS><<<(unsigned)grid_q, 128, 0, s>>>(A);
    err = launch_status("attention_backward: dq");
    if (err) return err;
    const int64_t grid_kv = (int64_t)batch * heads * ((len + 64 * AB_DKV_BLOCKS - 1) / (64 * AB_DKV_BLOCKS));
    attention_dkv_kernel<AB_DKV_BLOCKS><<<(unsigned)grid_kv, 128, 0, s>>>(A);
    return launch_status("attention_backward: dk dv");
}

}  // extern "C"
