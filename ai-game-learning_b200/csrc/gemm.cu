// Dense bf16 linear layer on the 5th-generation tensor cores:
//     y[M, N] = act(x[M, K] . w[N, K]^T * row_scale[M] + bias[N] + residual[M, N])
// bf16 operands, fp32 accumulate, bf16 or fp32 output; the Linear / FFN /
// attention-projection maps of the poker model (pbg/games/poker/model/
// primitives.py:35-60 FFN, :97-117 MHA projections, pbg/core/tensor_ops.py
// Linear: weight [out, in], bias [out]) with the elementwise steps that follow
// them in the model fused into the epilogue: the per-row mass scale of the
// incidence source map, the fp32 residual add of the attention output and FFN
// maps, the pre-activation residual of the incidence query map
// (pbg/games/poker/model/incidence.py:57-84), and the per-decision context
// projection that a factored FFN adds to every row of its decision
// (pbg/games/poker/model/primitives.py:62-71, a residual row per group of rows).  x, residual and y take their own
// row strides, so a map can read or fill a column slice of a wider buffer.
//
// One persistent CTA per SM walks 128 x BN output tiles (BN <= 256, a
// divisor of N).  Warp roles:
//   warp 0  TMA producer: 128x64 x-tiles and BNx64 w-tiles (both K-major,
//           128-byte swizzle) into a 4-stage shared-memory ring, completion
//           counted on the stage's "full" mbarrier;
//   warp 1  owns the tensor memory (2*BN fp32 columns: two accumulators) and
//           one elected thread issues tcgen05.mma (M=128, N=BN, K=16, both
//           operands from shared memory) four times per 64-wide k-block, then
//           tcgen05.commit frees the stage ("empty") and, after the last
//           k-block, publishes the accumulator ("acc_full");
//   warps 2-17 epilogue, four warps per TMEM lane quadrant, each on a quarter
//           of the tile's columns: a thread owns one accumulator row, loads 32
//           columns at a time with tcgen05.ld, applies the row scale, bias,
//           residual (128 contiguous bytes of its row) and GELU (erf form,
//           torch's default), packs bf16 (or keeps fp32) into a 64-byte-swizzled
//           shared-memory block (conflict-free) and one lane TMA-stores the
//           32x32 bf16 block (two 32x16 fp32 blocks; rows past M are clipped by
//           the tensor map); then the warp releases the accumulator
//           ("acc_empty") so the next tile's MMAs overlap this epilogue.
// Every wait is bounded; a wait that runs out records an error code, stops
// the CTA's loops, waits (bounded) for its own copies and MMAs in flight,
// frees its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <mutex>

#include "pbg_common.cuh"

namespace pbg {

constexpr int GM_BM = 128;
constexpr int GM_BK = 64;  // one 128-byte swizzle row of bf16
constexpr int GM_STAGES = 4;
constexpr int GM_EPI_WARPS = 16;  // four per TMEM lane quadrant, each on a quarter of the tile's columns
constexpr int GM_THREADS = 64 + 32 * GM_EPI_WARPS;
constexpr int GM_STAGE_OUT = 32 * 64;  // one warp's 32 x 32 bf16 output block (64-byte swizzled rows)
constexpr uint32_t GM_WAIT_TRIES = 1u << 26;

struct GemmArgs {
    int64_t M;
    int N, K, BN, tiles_n;
    int64_t tiles;
    const float* bias;
    const float* row_scale;  // [M] or null
    const float* residual;   // fp32, row m at residual + (m / res_div) * ldr, or null
    int64_t ldr, res_div;
    const __nv_bfloat16* grad;  // act 2: bf16 [M, N] row stride ldg, the gradient of the GELU's output
    int64_t ldg;
    int act;                 // 0 none, 1 gelu, 2 GELU backward: grad * GELU'(pre-activation)
    int out_f32;             // 0 bf16, 1 fp32
    uint32_t* error;
};

__device__ __forceinline__ uint32_t gm_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void gm_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void gm_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void gm_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool gm_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; also gives up when another role has aborted the CTA.
__device__ __forceinline__ bool gm_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < GM_WAIT_TRIES; ++i) {
        if (gm_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && *abort_flag) return false;
    }
    return false;
}

__device__ __forceinline__ void gm_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// K-major operand tile, 128-byte swizzle: rows of 128 B, 8-row (1024 B) atoms.
__device__ __forceinline__ uint64_t gm_desc(uint32_t smem_addr) {
    const uint64_t start = (smem_addr >> 4) & 0x3FFFu;
    const uint64_t lbo = 1;                 // unused by swizzled K-major layouts
    const uint64_t sbo = 1024 >> 4;         // next 8-row atom
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46) /* sm100 descriptor version */ |
           (2ull << 61) /* SWIZZLE_128B */;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> fp32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t gm_idesc(int bn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(GM_BM >> 4) << 24);
}

__device__ __forceinline__ void gm_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void gm_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void gm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void gm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void gm_tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// erf by the rational approximation of Abramowitz & Stegun, Handbook of
// Mathematical Functions, formula 7.1.26 (|error| <= 1.5e-7 for all x):
//   erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2),  t = 1 / (1 + p x),  x >= 0,
// odd in x.  Far below the bf16 rounding of the layer's output; one reciprocal and one exponential
// on the SFU instead of a branchy library erf.
__device__ __forceinline__ float gm_erf(float x) {
    const float ax = fabsf(x);
    const float t = __fdividef(1.0f, fmaf(0.3275911f, ax, 1.0f));
    float poly = fmaf(1.061405429f, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    const float y = fmaf(-poly * t, __expf(-ax * ax), 1.0f);
    return copysignf(y, x);
}

// GELU, erf form (torch's default): x * Phi(x) = 0.5 x (1 + erf(x / sqrt 2)).  The erf error above
// is absolute: relative to the output it stays below 1e-4 for x >= -3; further out the output is
// below 1e-5 in magnitude and the deviation below 1e-6.
__device__ __forceinline__ float gm_gelu(float x) { return 0.5f * x * (1.0f + gm_erf(x * 0.70710678118654752f)); }

// GELU's derivative, erf form: Phi(x) + x phi(x)
__device__ __forceinline__ float gm_gelu_grad(float x) {
    return 0.5f * (1.0f + gm_erf(x * 0.70710678118654752f)) + x * 0.39894228040143268f * __expf(-0.5f * x * x);
}

// activation and bf16 packing of one thread's 32 finished columns (two at a time: few live registers)
template <int ACT>
__device__ __forceinline__ void gm_pack_bf16(const float* v, uint32_t* packed) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const float x0 = ACT == 1 ? gm_gelu(v[j]) : v[j];
        const float x1 = ACT == 1 ? gm_gelu(v[j + 1]) : v[j + 1];
        __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        packed[j / 2] = *reinterpret_cast<uint32_t*>(&h);
    }
}

// one 32 x 64-byte block row (`lane`) of the swizzled staging block: chunk q at position q ^ ((row >> 1) & 3)
__device__ __forceinline__ void gm_stage_row(uint32_t blk, int lane, const uint32_t* words) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t addr = blk + (uint32_t)lane * 64u + (uint32_t)((q ^ ((lane >> 1) & 3)) * 16);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(words[4 * q]), "r"(words[4 * q + 1]),
                     "r"(words[4 * q + 2]), "r"(words[4 * q + 3])
                     : "memory");
    }
}

__device__ __forceinline__ void gm_store_block(const CUtensorMap* map, uint32_t blk, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(blk)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(GM_THREADS, 1)
    linear_tcgen05_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                          const __grid_constant__ CUtensorMap map_y, GemmArgs G) {
    extern __shared__ __align__(16) unsigned char gm_raw[];
    __shared__ __align__(8) uint64_t full[GM_STAGES], empty[GM_STAGES], acc_full[2], acc_empty[2], done_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;
    // 1024-byte aligned ring (the 128-byte swizzle atom)
    const uint32_t raw = gm_smem(gm_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    const uint32_t a_bytes = GM_BM * GM_BK * 2;
    const uint32_t b_bytes = (uint32_t)G.BN * GM_BK * 2;
    const uint32_t stage_bytes = a_bytes + b_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = G.K / GM_BK;
    const uint32_t tmem_cols = G.BN * 2 <= 32 ? 32 : (G.BN * 2 <= 64 ? 64 : (G.BN * 2 <= 128 ? 128 : (G.BN * 2 <= 256 ? 256 : 512)));

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < GM_STAGES; ++s) {
            gm_mbar_init(gm_smem(&full[s]), 1);
            gm_mbar_init(gm_smem(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            gm_mbar_init(gm_smem(&acc_full[b]), 1);
            gm_mbar_init(gm_smem(&acc_empty[b]), 32 * GM_EPI_WARPS);
        }
        gm_mbar_init(gm_smem(&done_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(gm_smem(&tmem_base_s)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    gm_fence_before();
    __syncthreads();
    gm_fence_after();
    const uint32_t tmem_base = tmem_base_s;

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; ok && t < G.tiles; t += gridDim.x) {
                const int m_blk = (int)(t / G.tiles_n), n_blk = (int)(t % G.tiles_n);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % GM_STAGES;
                    const uint32_t phase = (it / GM_STAGES) & 1u;
                    if (!gm_wait(gm_smem(&empty[s]), phase ^ 1u, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = ring + s * stage_bytes;
                    gm_expect_tx(gm_smem(&full[s]), stage_bytes);
                    gm_tma_2d(sa, &map_x, kb * GM_BK, m_blk * GM_BM, gm_smem(&full[s]));
                    gm_tma_2d(sa + a_bytes, &map_w, kb * GM_BK, n_blk * G.BN, gm_smem(&full[s]));
                }
            }
            if (!ok) {
                atomicCAS(G.error, 0u, 1u);
                abort_flag = 1;
            }
            // every stage's last copy has landed before the CTA can exit
            const uint32_t issued = it;
            for (uint32_t k = issued > GM_STAGES ? issued - GM_STAGES : 0; k < issued; ++k) {
                const uint32_t s = k % GM_STAGES, phase = (k / GM_STAGES) & 1u;
                for (uint32_t i = 0; i < GM_WAIT_TRIES && !gm_try_wait(gm_smem(&full[s]), phase); ++i) {
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issue
        if (lane == 0) {
            const uint32_t idesc = gm_idesc(G.BN);
            uint32_t it = 0, acc_it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; ok && t < G.tiles; t += gridDim.x, ++acc_it) {
                const uint32_t b = acc_it & 1u, aphase = (acc_it >> 1) & 1u;
                if (!gm_wait(gm_smem(&acc_empty[b]), aphase ^ 1u, &abort_flag)) {
                    ok = false;
                    break;
                }
                gm_fence_after();
                const uint32_t d_tmem = tmem_base + b * (uint32_t)G.BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % GM_STAGES;
                    const uint32_t phase = (it / GM_STAGES) & 1u;
                    if (!gm_wait(gm_smem(&full[s]), phase, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    gm_fence_after();
                    const uint32_t sa = ring + s * stage_bytes;
#pragma unroll
                    for (int k = 0; k < GM_BK / 16; ++k)
                        gm_mma(d_tmem, gm_desc(sa + k * 32), gm_desc(sa + a_bytes + k * 32), idesc,
                               (kb > 0 || k > 0) ? 1u : 0u);
                    gm_commit(gm_smem(&empty[s]));
                }
                if (ok) gm_commit(gm_smem(&acc_full[b]));
            }
            if (!ok) {
                atomicCAS(G.error, 0u, 2u);
                abort_flag = 1;
            }
            // all MMAs this thread issued have completed before the memory is freed
            gm_commit(gm_smem(&done_bar));
            for (uint32_t i = 0; i < GM_WAIT_TRIES && !gm_try_wait(gm_smem(&done_bar), 0u); ++i) {
            }
        }
    } else {
        // ---------------------------------------------------------- epilogue
        const int e = warp - 2;
        const int quad = warp & 3;  // TMEM lanes this warp may read
        const int part = e >> 2;    // which quarter of the tile's columns
        const int cols = G.BN / 4;  // a multiple of 32
        // one 2 KB output block per warp, after the operand ring
        const uint32_t blk = ring + GM_STAGES * stage_bytes + (uint32_t)e * GM_STAGE_OUT;
        uint32_t acc_it = 0;
        for (int64_t t = blockIdx.x; t < G.tiles; t += gridDim.x, ++acc_it) {
            const int m_blk = (int)(t / G.tiles_n), n_blk = (int)(t % G.tiles_n);
            const uint32_t b = acc_it & 1u, aphase = (acc_it >> 1) & 1u;
            if (!gm_wait(gm_smem(&acc_full[b]), aphase, &abort_flag)) {
                if (lane == 0) atomicCAS(G.error, 0u, 3u);
                abort_flag = 1;
                break;
            }
            gm_fence_after();
            const int col_base = n_blk * G.BN + part * cols;
            for (int c = 0; c < cols; c += 32) {
                float v[32];
                gm_tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + b * (uint32_t)G.BN + (uint32_t)(part * cols + c),
                             v);
                const int64_t row = (int64_t)m_blk * GM_BM + quad * 32 + lane;
                const bool live = row < G.M;
                if (G.row_scale) {
                    const float scale = live ? G.row_scale[row] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] *= scale;
                }
                if (G.bias) {
                    const float* bias = G.bias + col_base + c;
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += bias[j];
                }
                if (G.residual && live) {
                    const float4* r4 =
                        reinterpret_cast<const float4*>(G.residual + (row / G.res_div) * G.ldr + col_base + c);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        float4 r[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) r[q] = __ldg(r4 + 4 * half + q);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            v[16 * half + 4 * q] += r[q].x;
                            v[16 * half + 4 * q + 1] += r[q].y;
                            v[16 * half + 4 * q + 2] += r[q].z;
                            v[16 * half + 4 * q + 3] += r[q].w;
                        }
                    }
                }
                if (G.act == 2) {  // the gradient through the GELU: grad * GELU'(pre-activation); 0 past M
                    const uint4* g4 = reinterpret_cast<const uint4*>(G.grad + row * G.ldg + col_base + c);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint4 raw = live ? __ldg(g4 + q) : make_uint4(0u, 0u, 0u, 0u);
                        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 g = __bfloat1622float2(h[e]);
                            v[8 * q + 2 * e] = g.x * gm_gelu_grad(v[8 * q + 2 * e]);
                            v[8 * q + 2 * e + 1] = g.y * gm_gelu_grad(v[8 * q + 2 * e + 1]);
                        }
                    }
                }
                const int y0 = m_blk * GM_BM + quad * 32;
                const bool gelu = G.act == 1;
                if (!G.out_f32) {
                    uint32_t packed[16];
                    if (gelu) gm_pack_bf16<1>(v, packed);
                    else gm_pack_bf16<0>(v, packed);
                    // the previous TMA store has finished reading the block
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    __syncwarp();
                    gm_stage_row(blk, lane, packed);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) gm_store_block(&map_y, blk, col_base + c, y0);
                } else {
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        if (gelu) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) v[16 * half + j] = gm_gelu(v[16 * half + j]);
                        }
                        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                        __syncwarp();
                        gm_stage_row(blk, lane, reinterpret_cast<const uint32_t*>(v + 16 * half));
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) gm_store_block(&map_y, blk, col_base + c + 16 * half, y0);
                    }
                }
            }
            gm_fence_before();
            gm_arrive(gm_smem(&acc_empty[b]));
        }
        // the output blocks must be read out before the CTA's shared memory is released
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    __syncthreads();
    if (warp == 1) {
        gm_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols) : "memory");
    }
}

// ------------------------------------------------------------------ host

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D row-major map (bf16 or fp32): rows x cols (cols contiguous, `ld` elements between rows), box
// box_rows x box_cols.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int cols, int64_t ld, int box_rows,
                    int box_cols, CUtensorMapSwizzle swizzle, bool f32 = false) {
    auto fn = encode_fn();
    PBG_REQUIRE(fn != nullptr, "linear: cuTensorMapEncodeTiled is unavailable");
    const int esize = f32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * esize};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    PBG_REQUIRE(r == CUDA_SUCCESS, "linear: tensor map encoding failed (%d)", (int)r);
    return 0;
}

}  // namespace pbg

using namespace pbg;

extern "C" {

static int linear_launch(int64_t M, int32_t N, int32_t K, const void* x, int64_t ldx, const void* w,
                         const float* bias, const float* row_scale, const float* residual, int64_t ldr,
                         int64_t residual_row_div, const void* grad, int64_t ldg, void* y, int64_t ldy, int32_t y_f32,
                         int32_t activation, uint32_t* error, void* stream);

int pbg_linear_ex(int64_t M, int32_t N, int32_t K, const void* x, int64_t ldx, const void* w, const float* bias,
                  const float* row_scale, const float* residual, int64_t ldr, int64_t residual_row_div, void* y,
                  int64_t ldy, int32_t y_f32, int32_t activation, uint32_t* error, void* stream) {
    PBG_REQUIRE(activation == 0 || activation == 1, "linear: activation must be 0 (none) or 1 (gelu)");
    return linear_launch(M, N, K, x, ldx, w, bias, row_scale, residual, ldr, residual_row_div, nullptr, 0, y, ldy,
                         y_f32, activation, error, stream);
}

int pbg_linear_gelu_backward(int64_t M, int32_t N, int32_t K, const void* x, int64_t ldx, const void* w,
                             const float* bias, const float* row_scale, const float* residual, int64_t ldr,
                             int64_t residual_row_div, const void* dy, int64_t ldd, void* out, int64_t ldo,
                             uint32_t* error, void* stream) {
    PBG_REQUIRE(dy && ldd >= N && ldd % 8 == 0 && ((uintptr_t)dy % 16) == 0,
                "linear_gelu_backward: dy must be 16-byte aligned with a row stride >= N and a multiple of 8");
    return linear_launch(M, N, K, x, ldx, w, bias, row_scale, residual, ldr, residual_row_div, dy, ldd, out, ldo, 0, 2,
                         error, stream);
}

static int linear_launch(int64_t M, int32_t N, int32_t K, const void* x, int64_t ldx, const void* w,
                         const float* bias, const float* row_scale, const float* residual, int64_t ldr,
                         int64_t residual_row_div, const void* grad, int64_t ldg, void* y, int64_t ldy, int32_t y_f32,
                         int32_t activation, uint32_t* error, void* stream) {
    PBG_REQUIRE(M >= 0 && N > 0 && K > 0, "linear: bad shape");
    PBG_REQUIRE(K % GM_BK == 0, "linear: K must be a multiple of %d", GM_BK);
    PBG_REQUIRE(N % 128 == 0, "linear: N must be a multiple of 128");
    PBG_REQUIRE(activation != 2 || (grad && y_f32 == 0), "linear: the GELU backward takes a gradient, bf16 out");
    PBG_REQUIRE(y_f32 == 0 || y_f32 == 1, "linear: y_f32 must be 0 (bf16) or 1 (fp32)");
    PBG_REQUIRE(x && w && y && error, "linear: null pointer");
    PBG_REQUIRE(ldx >= K && (ldx * 2) % 16 == 0, "linear: x row stride must be >= K and a multiple of 8");
    PBG_REQUIRE(ldy >= N && (ldy * (y_f32 ? 4 : 2)) % 16 == 0, "linear: y row stride must be >= N, 16-byte rows");
    PBG_REQUIRE(!residual || (ldr >= N && ldr % 4 == 0 && ((uintptr_t)residual % 16) == 0 && residual_row_div >= 1),
                "linear: residual must be 16-byte aligned with a row stride >= N and a multiple of 4");
    PBG_REQUIRE(((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && ((uintptr_t)y % 16) == 0,
                "linear: x, w and y must be 16-byte aligned");
    if (M == 0) return 0;
    // the widest tile (<= 256 columns, a multiple of 128: four epilogue quarters of 32-column blocks) dividing N
    int BN = 0;
    for (int c = 256; c >= 128; c -= 128)
        if (N % c == 0) {
            BN = c;
            break;
        }
    PBG_REQUIRE(BN > 0, "linear: N must be a multiple of 128");
    CUtensorMap mx, mw, my;
    int rc = make_map(&mx, x, M, K, ldx, GM_BM, GM_BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_map(&mw, w, N, K, K, BN, GM_BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // output blocks of 32 rows x 64 bytes: 32 bf16 or 16 fp32 columns
    rc = make_map(&my, y, M, N, ldy, 32, y_f32 ? 16 : 32, CU_TENSOR_MAP_SWIZZLE_64B, y_f32 != 0);
    if (rc) return rc;
    GemmArgs G;
    G.M = M;
    G.N = N;
    G.K = K;
    G.BN = BN;
    G.tiles_n = N / BN;
    G.tiles = ((M + GM_BM - 1) / GM_BM) * (int64_t)G.tiles_n;
    G.bias = bias;
    G.row_scale = row_scale;
    G.residual = residual;
    G.ldr = ldr;
    G.res_div = residual_row_div >= 1 ? residual_row_div : 1;
    G.grad = static_cast<const __nv_bfloat16*>(grad);
    G.ldg = ldg;
    G.act = activation;
    G.out_f32 = y_f32;
    G.error = error;
    const size_t smem = 1024 + (size_t)GM_STAGES * (GM_BM * GM_BK * 2 + (size_t)BN * GM_BK * 2) +
                        (size_t)GM_EPI_WARPS * GM_STAGE_OUT;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        rc = cuda_status(cudaFuncSetAttribute(linear_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              1024 + GM_STAGES * (GM_BM * GM_BK * 2 + 256 * GM_BK * 2) +
                                                  GM_EPI_WARPS * GM_STAGE_OUT),
                         "linear: shared memory size");
        if (rc) return rc;
        configured[dev] = 1;
    }
    const int64_t grid = G.tiles < sm_count() ? G.tiles : sm_count();
    linear_tcgen05_kernel<<<(unsigned)grid, GM_THREADS, smem, as_stream(stream)>>>(mx, mw, my, G);
    return launch_status("linear_bf16");
}

int pbg_linear_bf16(int64_t M, int32_t N, int32_t K, const void* x, const void* w, const float* bias, void* y,
                    int32_t activation, uint32_t* error, void* stream) {
    return pbg_linear_ex(M, N, K, x, K, w, bias, nullptr, nullptr, 0, 1, y, N, 0, activation, error, stream);
}

}  // extern "C"
