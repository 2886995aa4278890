// Reach-biased multi-head self-attention core on the tensor cores
// (pbg/games/poker/model/primitives.py:63-283, MHA: scores
// (q / temperature_h) . k / sqrt(d_head) + key_bias, masked keys -inf,
// softmax over keys, times v; heads of width 32).
//
// One CTA per (sequence, head, group of T = 2, 3 or 4 query tiles of 128 rows),
// warp-specialised so that staging, tensor-core work and the softmax of
// different tiles and key blocks overlap:
//   warps 4t..4t+3  softmax warpgroup of tile t; thread r owns query row r.
//                   Per block of 64 keys it reads its row of S from tensor
//                   memory in one load, forms the base-2 logits, updates the
//                   running maximum (the shift moves only when the maximum
//                   grows by more than 2^8, so most blocks leave the output
//                   untouched; when it moves, the thread rescales its output
//                   row in tensor memory), writes its row of P (bf16 pairs)
//                   into the tile's P columns and adds the row sum;
//   warps 4T, 4T+1  loader: thread k stages key k of the block into a
//                   four-stage ring (K rows and V^T columns in the 128-byte
//                   swizzled K-major layout, and the key's base-2 bias, -inf
//                   for an absent key);
//   warp 4T+2       owns the tensor memory; one thread issues, per key block
//                   and tile, O += P . V of the previous block (P from tensor
//                   memory, V^T from shared memory) and S = Q . K^T of this
//                   block, and commits them to the tiles' barriers.
// Tensor memory: S of tile t at 64 t, P at 64 T + 32 t, O at 96 T + 32 t.
// Every wait is bounded; a wait that runs out records an error code and stops
// the CTA's loops; the MMA thread waits (bounded) for its MMAs before the
// memory is freed.
#include <cuda_bf16.h>

#include <cmath>

#include "pbg_common.cuh"

namespace pbg {

constexpr int AT_DH = 32;
constexpr int AT_BLOCK = 128;  // queries per CTA and keys per step
constexpr uint32_t AT_WAIT_TRIES = 1u << 22;

__device__ __forceinline__ uint32_t at_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool at_try_wait(uint32_t bar, uint32_t parity) {
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

// max(a, b, c) in one instruction
__device__ __forceinline__ float at_max3(float a, float b, float c) {
    float m;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
    return m;
}

// 2^x on the special-function unit (ex2.approx: relative error about 2^-22; 0 for -inf)
__device__ __forceinline__ float at_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint64_t at_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ constexpr uint32_t at_idesc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void at_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// D = A . B with A read from tensor memory (M = 128 lanes, K packed two bf16 per column)
__device__ __forceinline__ void at_mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// this thread's lane, 16 consecutive 32-bit columns
__device__ __forceinline__ void at_st16(uint32_t taddr, const uint32_t* w) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]),
          "r"(w[8]), "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
        : "memory");
}

__device__ __forceinline__ void at_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void at_ld32(uint32_t taddr, float* v) {
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

// 64 consecutive columns of this thread's lane: two loads in flight, one wait
__device__ __forceinline__ void at_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t* o = r + 32 * half;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
            "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
            "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]), "=r"(o[4]), "=r"(o[5]), "=r"(o[6]), "=r"(o[7]),
              "=r"(o[8]), "=r"(o[9]), "=r"(o[10]), "=r"(o[11]), "=r"(o[12]), "=r"(o[13]), "=r"(o[14]), "=r"(o[15]),
              "=r"(o[16]), "=r"(o[17]), "=r"(o[18]), "=r"(o[19]), "=r"(o[20]), "=r"(o[21]), "=r"(o[22]), "=r"(o[23]),
              "=r"(o[24]), "=r"(o[25]), "=r"(o[26]), "=r"(o[27]), "=r"(o[28]), "=r"(o[29]), "=r"(o[30]), "=r"(o[31])
            : "r"(taddr + 32u * half));
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j]);
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled block
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) * 16);
}

struct AttnArgs {
    int batch, len, heads, qblocks, qgroups;
    const __nv_bfloat16* qkv;  // [batch, len, 3 * heads * 32]: q | k | v, head-major inside each
    const float* key_bias;     // [batch, len] or null
    const uint8_t* key_mask;   // [batch, len] (nonzero = key present) or null
    const float* q_scale;      // [heads]: 1 / (temperature_h * sqrt(32))
    __nv_bfloat16* out;        // [batch, len, heads * 32]
    float* lse;                // [batch, heads, len] base-2 log-sum-exp of each row's logits (+inf: no key), or null
    uint32_t* error;
};

constexpr int AT_KB = 64;                // keys per block
constexpr int AT_STAGES = 4;
constexpr int AT_STAGE = 8192 + 4096;    // K [64 x 128 B] + V^T [32 x 128 B]
constexpr float AT_RESCALE = 8.0f;       // base-2 growth of the maximum that moves the shift

template <int T>
struct AttnPlan {
    static constexpr int threads = 32 * (4 * T + 3);
    static constexpr int kv = T * 16384;                       // after the Q tiles
    static constexpr int smem = kv + AT_STAGES * AT_STAGE;     // + 1024 alignment
    static constexpr uint32_t s_col = 0, p_col = 64 * T, o_col = 96 * T;
    static constexpr uint32_t tmem_cols = 96 * T + 32 * T <= 256 ? 256 : 512;
};

// bounded wait that also gives up when another role has aborted the CTA
__device__ __forceinline__ bool at_wait_abort(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < AT_WAIT_TRIES; ++i) {
        if (at_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && *abort_flag) return false;
    }
    return false;
}

__device__ __forceinline__ void at_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <int T>
__global__ void __launch_bounds__(AttnPlan<T>::threads, 1) attention_kernel(AttnArgs A) {
    using Plan = AttnPlan<T>;
    extern __shared__ __align__(16) unsigned char at_raw[];
    __shared__ __align__(8) uint64_t kv_full[AT_STAGES], kv_empty[AT_STAGES], s_full[T], p_full[T], done_bar;
    __shared__ uint32_t tmem_s;
    __shared__ volatile int abort_flag;
    __shared__ __align__(16) float kterm_s[AT_STAGES][AT_KB];  // base-2 bias per key, or -inf when absent
    const uint32_t base = (at_smem(at_raw) + 1023u) & ~1023u;
    unsigned char* sm = at_raw + (base - at_smem(at_raw));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qg = blockIdx.x % A.qgroups;
    const int h = (blockIdx.x / A.qgroups) % A.heads;
    const int b = blockIdx.x / (A.qgroups * A.heads);
    const int width = 3 * A.heads * AT_DH;  // qkv row stride (elements)
    const int64_t row0 = (int64_t)b * A.len;
    const int kblocks = (A.len + AT_KB - 1) / AT_KB;
    constexpr int mma_warp = 4 * T + 2;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < AT_STAGES; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(at_smem(&kv_full[s])), "r"(AT_KB) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&kv_empty[s])) : "memory");
        }
        for (int t = 0; t < T; ++t) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&s_full[t])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(at_smem(&p_full[t])), "r"(AT_BLOCK) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&done_bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == mma_warp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(at_smem(&tmem_s)),
                     "r"(Plan::tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    const int tile = warp >> 2;  // softmax warpgroup when tile < T
    const int r = 32 * (warp & 3) + lane;
    if (tile < T) {
        // stage this warpgroup's Q tile: row r = query (qg * T + tile) * 128 + r, zero past the sequence
        const int q = (qg * T + tile) * AT_BLOCK + r;
        uint4 c[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (q < A.len) {
            const uint4* src = reinterpret_cast<const uint4*>(A.qkv + (row0 + q) * width + h * AT_DH);
#pragma unroll
            for (int j = 0; j < 4; ++j) c[j] = src[j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(sm + tile * 16384 + sw128(r, j)) = c[j];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_s;

    if (tile < T) {
        // ------------------------------------------------------------ softmax
        const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t s_cols = tmem + lanes + Plan::s_col + (uint32_t)(tile * 64);
        const uint32_t p_cols = tmem + lanes + Plan::p_col + (uint32_t)(tile * 32);
        const uint32_t o_cols = tmem + lanes + Plan::o_col + (uint32_t)(tile * 32);
        const float scale2 = A.q_scale[h] * 1.4426950408889634f;  // base-2 logits
        const float2 scale2x2 = make_float2(scale2, scale2);
        float shift = -INFINITY, l = 0.0f;  // the shift of every P written so far, and their sum
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
            const int stage = kb % AT_STAGES;
            // the warp decides together: the tensor-memory accesses below are warp-collective
            const bool ready = at_wait_abort(at_smem(&s_full[tile]), (uint32_t)(kb & 1), &abort_flag) &&
                               at_wait_abort(at_smem(&kv_full[stage]), (uint32_t)((kb / AT_STAGES) & 1), &abort_flag);
            if (!__all_sync(0xffffffffu, ready)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float sv[AT_KB];
            at_ld64(s_cols, sv);
            const float4* kterm4 = reinterpret_cast<const float4*>(kterm_s[stage]);
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
            for (int j = 0; j < AT_KB; j += 4) {
                const float4 kt = kterm4[j >> 2];
                const float2 t0 = __ffma2_rn(make_float2(sv[j], sv[j + 1]), scale2x2, make_float2(kt.x, kt.y));
                const float2 t1 = __ffma2_rn(make_float2(sv[j + 2], sv[j + 3]), scale2x2, make_float2(kt.z, kt.w));
                sv[j] = t0.x;
                sv[j + 1] = t0.y;
                sv[j + 2] = t1.x;
                sv[j + 3] = t1.y;
                const int a = (j >> 2) & 3;
                mx[2 * a] = at_max3(mx[2 * a], t0.x, t0.y);
                mx[2 * a + 1] = at_max3(mx[2 * a + 1], t1.x, t1.y);
            }
            const float bmax = at_max3(at_max3(mx[0], mx[1], mx[2]), at_max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
            // move the shift to the new maximum when it grows past the threshold: earlier P values
            // (in the output and the sum) are rescaled by 2^(shift - new shift); the first present key
            // always sets it (the output is still empty then: the first product overwrites it)
            const bool rescale = __any_sync(0xffffffffu, bmax > shift + AT_RESCALE);
            float corr = 1.0f;
            if (rescale) {
                const float next = bmax > shift + AT_RESCALE ? bmax : shift;
                corr = shift == -INFINITY ? 0.0f : at_exp2(shift - next);
                l *= corr;
                shift = next;
            }
            const float2 neg_shift = shift == -INFINITY ? make_float2(0.0f, 0.0f) : make_float2(-shift, -shift);
            float2 acc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
            uint32_t packed[AT_KB / 2];
#pragma unroll
            for (int j = 0; j < AT_KB; j += 4) {
                const float2 t0 = __fadd2_rn(make_float2(sv[j], sv[j + 1]), neg_shift);
                const float2 t1 = __fadd2_rn(make_float2(sv[j + 2], sv[j + 3]), neg_shift);
                const float2 p0 = make_float2(at_exp2(t0.x), at_exp2(t0.y));
                const float2 p1 = make_float2(at_exp2(t1.x), at_exp2(t1.y));
                acc[(j >> 2) & 3] = __fadd2_rn(acc[(j >> 2) & 3], __fadd2_rn(p0, p1));
                __nv_bfloat162 h0 = __floats2bfloat162_rn(p0.x, p0.y), h1 = __floats2bfloat162_rn(p1.x, p1.y);
                packed[j / 2] = *reinterpret_cast<uint32_t*>(&h0);
                packed[j / 2 + 1] = *reinterpret_cast<uint32_t*>(&h1);
            }
            at_st16(p_cols, packed);
            at_st16(p_cols + 16u, packed + 16);
            const float2 acc2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
            l += acc2.x + acc2.y;
            if (rescale && kb > 0) {
                // the accumulated output moves to the new shift before this block's product is added
                // (the previous product has completed: it was issued before this block's S)
                float o[AT_DH];
                at_ld32(o_cols, o);
#pragma unroll
                for (int j = 0; j < AT_DH; ++j) o[j] *= corr;
                at_st16(o_cols, reinterpret_cast<const uint32_t*>(o));
                at_st16(o_cols + 16u, reinterpret_cast<const uint32_t*>(o + 16));
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            at_arrive(at_smem(&p_full[tile]));
        }
        if (ok) ok = __all_sync(0xffffffffu, at_wait_abort(at_smem(&done_bar), 0u, &abort_flag));
        if (!ok) {
            if (r == 0) atomicOr(A.error, 1u);
            abort_flag = 1;
        } else {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float o[AT_DH];
            at_ld32(o_cols, o);
            const int q = (qg * T + tile) * AT_BLOCK + r;
            if (q < A.len) {
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
                if (A.lse) A.lse[((int64_t)b * A.heads + h) * A.len + q] = l > 0.0f ? shift + log2f(l) : INFINITY;
                uint32_t packed[16];
#pragma unroll
                for (int j = 0; j < AT_DH; j += 2) {
                    __nv_bfloat162 hv = __floats2bfloat162_rn(o[j] * inv, o[j + 1] * inv);
                    packed[j / 2] = *reinterpret_cast<uint32_t*>(&hv);
                }
                uint4* dst = reinterpret_cast<uint4*>(A.out + (row0 + q) * (A.heads * AT_DH) + h * AT_DH);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            }
        }
    } else if (warp < mma_warp) {
        // ------------------------------------------------------------- loader
        // key k of each block; the next block's rows are fetched into registers as soon as this
        // block is staged, so their latency overlaps the wait for a free stage
        const int k = threadIdx.x - 128 * T;
        uint4 kc[4], vc[4];
        float term;
        auto fetch = [&](int kb) {
            const int key = kb * AT_KB + k;
#pragma unroll
            for (int j = 0; j < 4; ++j) kc[j] = vc[j] = make_uint4(0, 0, 0, 0);
            term = -INFINITY;
            if (key < A.len) {
                const __nv_bfloat16* rowp = A.qkv + (row0 + key) * width;
                const uint4* ks = reinterpret_cast<const uint4*>(rowp + (A.heads + h) * AT_DH);
                const uint4* vs = reinterpret_cast<const uint4*>(rowp + (2 * A.heads + h) * AT_DH);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    kc[j] = ks[j];
                    vc[j] = vs[j];
                }
                if (!A.key_mask || A.key_mask[row0 + key])
                    term = A.key_bias ? A.key_bias[row0 + key] * 1.4426950408889634f : 0.0f;
            }
        };
        fetch(0);
        for (int kb = 0; kb < kblocks; ++kb) {
            const int stage = kb % AT_STAGES;
            if (kb >= AT_STAGES &&
                !at_wait_abort(at_smem(&kv_empty[stage]), (uint32_t)((kb / AT_STAGES - 1) & 1), &abort_flag)) {
                if (k == 0) atomicOr(A.error, 4u);
                abort_flag = 1;
                break;
            }
            unsigned char* st = sm + Plan::kv + stage * AT_STAGE;
#pragma unroll
            for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(st + sw128(k, j)) = kc[j];
            kterm_s[stage][k] = term;
            {
                // V^T: element (d, key) at byte key * 2 of row d (one 64-key column block)
                const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(vc);
#pragma unroll
                for (int d = 0; d < AT_DH; ++d)
                    *reinterpret_cast<__nv_bfloat16*>(st + 8192 + sw128(d, k >> 3) + (uint32_t)((k & 7) * 2)) = v[d];
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            at_arrive(at_smem(&kv_full[stage]));
            if (kb + 1 < kblocks) fetch(kb + 1);
        }
    } else {
        // ---------------------------------------------------------------- MMA
        if (lane == 0) {
            bool ok = true;
            for (int kb = 0; ok && kb <= kblocks; ++kb) {
                const int stage = kb % AT_STAGES, prev = (kb + AT_STAGES - 1) % AT_STAGES;
                if (kb < kblocks &&
                    !at_wait_abort(at_smem(&kv_full[stage]), (uint32_t)((kb / AT_STAGES) & 1), &abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int t = 0; t < T; ++t) {
                    if (kb > 0) {
                        // O += P . V of the previous block once this tile's P is written
                        if (!at_wait_abort(at_smem(&p_full[t]), (uint32_t)((kb - 1) & 1), &abort_flag)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t vt = base + Plan::kv + prev * AT_STAGE + 8192;
#pragma unroll
                        for (int u = 0; u < AT_KB / 16; ++u)
                            at_mma_ts(tmem + Plan::o_col + t * 32, tmem + Plan::p_col + t * 32 + (uint32_t)(u * 8),
                                      at_desc(vt + u * 32), at_idesc(AT_DH), (kb > 1 || u > 0) ? 1u : 0u);
                    }
                    if (kb < kblocks) {
                        const uint32_t q = base + t * 16384;
                        const uint32_t kt = base + Plan::kv + stage * AT_STAGE;
#pragma unroll
                        for (int u = 0; u < AT_DH / 16; ++u)
                            at_mma(tmem + Plan::s_col + t * 64, at_desc(q + u * 32), at_desc(kt + u * 32),
                                   at_idesc(AT_KB), u > 0);
                        at_commit(at_smem(&s_full[t]));
                    }
                }
                if (!ok) break;
                if (kb > 0) at_commit(at_smem(&kv_empty[prev]));  // every MMA reading the previous stage is issued
            }
            if (!ok) {
                atomicOr(A.error, 2u);
                abort_flag = 1;
            }
            // all MMAs this thread issued have completed before the results are read or the memory freed
            at_commit(at_smem(&done_bar));
            for (uint32_t i = 0; i < AT_WAIT_TRIES && !at_try_wait(at_smem(&done_bar), 0u); ++i) {
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == mma_warp) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Plan::tmem_cols)
                     : "memory");
    }
}

template <int T>
static int launch_attention(const AttnArgs& A, int64_t grid, cudaStream_t stream) {
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int rc = cuda_status(cudaFuncSetAttribute(attention_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  AttnPlan<T>::smem + 1024),
                             "attention: shared memory size");
        if (rc) return rc;
        configured[dev] = 1;
    }
    attention_kernel<T><<<(unsigned)grid, AttnPlan<T>::threads, AttnPlan<T>::smem + 1024, stream>>>(A);
    return launch_status("attention_bf16");
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_attention_bf16_lse(int32_t batch, int32_t len, int32_t heads, const void* qkv,
                                      const float* key_bias, const uint8_t* key_mask, const float* q_scale, void* out,
                                      float* lse, uint32_t* error, void* stream);

extern "C" int pbg_attention_bf16(int32_t batch, int32_t len, int32_t heads, const void* qkv, const float* key_bias,
                                  const uint8_t* key_mask, const float* q_scale, void* out, uint32_t* error,
                                  void* stream) {
    return pbg_attention_bf16_lse(batch, len, heads, qkv, key_bias, key_mask, q_scale, out, nullptr, error, stream);
}

extern "C" int pbg_attention_bf16_lse(int32_t batch, int32_t len, int32_t heads, const void* qkv,
                                      const float* key_bias, const uint8_t* key_mask, const float* q_scale, void* out,
                                      float* lse, uint32_t* error, void* stream) {
    PBG_REQUIRE(batch >= 0 && len >= 0 && heads >= 1, "attention: bad shape");
    PBG_REQUIRE(qkv && q_scale && out && error, "attention: null pointer");
    PBG_REQUIRE(((uintptr_t)qkv % 16) == 0 && ((uintptr_t)out % 16) == 0, "attention: qkv and out must be 16-byte aligned");
    if (batch == 0 || len == 0) return 0;
    AttnArgs A;
    A.batch = batch;
    A.len = len;
    A.heads = heads;
    A.qblocks = (len + AT_BLOCK - 1) / AT_BLOCK;
    // as many query tiles per CTA as fit (more softmax warps cover the tensor-core round trips)
    // unless that computes more than one extra tile past the sequence
    auto waste = [&](int t) { return t * ((A.qblocks + t - 1) / t) - A.qblocks; };
    const int tiles = (A.qblocks >= 4 && waste(4) <= waste(2) + 1)   ? 4
                      : (A.qblocks >= 3 && waste(3) <= waste(2) + 1) ? 3
                                                                     : 2;
    A.qgroups = (A.qblocks + tiles - 1) / tiles;
    A.qkv = static_cast<const __nv_bfloat16*>(qkv);
    A.key_bias = key_bias;
    A.key_mask = key_mask;
    A.q_scale = q_scale;
    A.out = static_cast<__nv_bfloat16*>(out);
    A.lse = lse;
    A.error = error;
    const int64_t grid = (int64_t)batch * heads * A.qgroups;
    PBG_REQUIRE(grid <= INT32_MAX, "attention: too many blocks");
    if (tiles == 4) return launch_attention<4>(A, grid, as_stream(stream));
    return tiles == 3 ? launch_attention<3>(A, grid, as_stream(stream)) : launch_attention<2>(A, grid, as_stream(stream));
}
