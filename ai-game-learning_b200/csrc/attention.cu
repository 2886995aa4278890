// Reach-biased multi-head self-attention core on the tensor cores
// (pbg/games/poker/model/primitives.py:63-283, MHA: scores
// (q / temperature_h) . k / sqrt(d_head) + key_bias, masked keys -inf,
// softmax over keys, times v; heads of width 32).
//
// One CTA of 128 threads per (sequence, head, block of 128 queries); thread r
// owns query row r.  Per block of 128 keys:
//   1. the CTA stages K (128 keys x 32) and V^T (32 x 128 keys) in shared
//      memory in the 128-byte-swizzled K-major layout of the tensor core;
//   2. one thread issues S = Q . K^T (tcgen05.mma, M=128, N=128, K=32) into
//      tensor memory;
//   3. each thread reads its row of S from tensor memory (tcgen05.ld, 32
//      columns at a time, twice: block maximum, then probabilities), keeps
//      the running maximum and sum (online softmax, base 2) and writes its
//      row of P (bf16) to shared memory;
//   4. one thread issues P . V (M=128, N=32, K=128) into the same tensor
//      memory columns; each thread rescales its 32 output accumulators in
//      registers and adds its row.
// Q is staged once.  Every operand row is 128 bytes (64 bf16, the 32-wide
// head zero-padded), the layout the 128-byte swizzle and the MMA descriptors
// expect.  Waits on MMA completion are bounded; a wait that runs out sets
// *error, and the CTA waits (bounded) for its MMAs, frees its tensor memory
// and returns.
#include <cuda_bf16.h>

#include <cmath>

#include "pbg_common.cuh"

namespace pbg {

constexpr int AT_THREADS = 128;
constexpr int AT_DH = 32;
constexpr int AT_BLOCK = 128;  // queries per CTA and keys per step
constexpr uint32_t AT_WAIT_TRIES = 1u << 26;
// shared layout (bytes, each region 1024-aligned): Q [128 x 128 B], K [128 x 128 B],
// V^T two column blocks [32 x 128 B], P two column blocks [128 x 128 B]
constexpr int AT_Q = 0, AT_K = 16384, AT_VT = 32768, AT_P = 40960, AT_SMEM = 73728;

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

__device__ __forceinline__ bool at_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < AT_WAIT_TRIES; ++i)
        if (at_try_wait(bar, parity)) return true;
    return false;
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

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled block
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) * 16);
}

struct AttnArgs {
    int batch, len, heads, qblocks;
    const __nv_bfloat16* qkv;  // [batch, len, 3 * heads * 32]: q | k | v, head-major inside each
    const float* key_bias;     // [batch, len] or null
    const uint8_t* key_mask;   // [batch, len] (nonzero = key present) or null
    const float* q_scale;      // [heads]: 1 / (temperature_h * sqrt(32))
    __nv_bfloat16* out;        // [batch, len, heads * 32]
    uint32_t* error;
};

__global__ void __launch_bounds__(AT_THREADS) attention_kernel(AttnArgs A) {
    extern __shared__ __align__(16) unsigned char at_raw[];
    __shared__ __align__(8) uint64_t bar_s, bar_pv, bar_done;
    __shared__ uint32_t tmem_s;
    __shared__ float kterm[AT_BLOCK];  // per key of the block: base-2 bias, or -inf when absent
    const uint32_t base = (at_smem(at_raw) + 1023u) & ~1023u;
    unsigned char* sm = at_raw + (base - at_smem(at_raw));
    const int r = threadIdx.x, warp = r >> 5;
    const int qb = blockIdx.x % A.qblocks;
    const int h = (blockIdx.x / A.qblocks) % A.heads;
    const int b = blockIdx.x / (A.qblocks * A.heads);
    const int width = 3 * A.heads * AT_DH;  // qkv row stride (elements)
    const int64_t row0 = (int64_t)b * A.len;

    if (r == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&bar_s)) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&bar_pv)) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(at_smem(&bar_done)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(at_smem(&tmem_s))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // stage Q: row r = query qb*128 + r, 64 bytes in chunks 0..3 (zero past the sequence)
    {
        const int q = qb * AT_BLOCK + r;
        uint4 c[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (q < A.len) {
            const uint4* src = reinterpret_cast<const uint4*>(A.qkv + (row0 + q) * width + h * AT_DH);
#pragma unroll
            for (int j = 0; j < 4; ++j) c[j] = src[j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(sm + AT_Q + sw128(r, j)) = c[j];
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_s;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const float scale2 = A.q_scale[h] * 1.4426950408889634f;  // base-2 logits
    float m = -INFINITY, l = 0.0f;
    float o[AT_DH];
#pragma unroll
    for (int j = 0; j < AT_DH; ++j) o[j] = 0.0f;
    bool ok = true;
    const int kblocks = (A.len + AT_BLOCK - 1) / AT_BLOCK;
    for (int kb = 0; kb < kblocks && ok; ++kb) {
        const uint32_t parity = (uint32_t)(kb & 1);
        // 1. stage K (row = key) and V^T (row = head dim, column = key)
        const int key = kb * AT_BLOCK + r;
        uint4 kc[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        uint4 vc[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (key < A.len) {
            const __nv_bfloat16* rowp = A.qkv + (row0 + key) * width;
            const uint4* ks = reinterpret_cast<const uint4*>(rowp + (A.heads + h) * AT_DH);
            const uint4* vs = reinterpret_cast<const uint4*>(rowp + (2 * A.heads + h) * AT_DH);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                kc[j] = ks[j];
                vc[j] = vs[j];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(sm + AT_K + sw128(r, j)) = kc[j];
        {
            const bool present = key < A.len && (!A.key_mask || A.key_mask[row0 + key]);
            kterm[r] = present ? (A.key_bias ? A.key_bias[row0 + key] * 1.4426950408889634f : 0.0f) : -INFINITY;
        }
        {
            // V^T: element (d, key) in column block key / 64, byte (key % 64) * 2 of row d
            const int blk = r >> 6, col = r & 63;
            const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(vc);
#pragma unroll
            for (int d = 0; d < AT_DH; ++d) {
                const uint32_t off = AT_VT + blk * 4096 + sw128(d, col >> 3) + (uint32_t)((col & 7) * 2);
                *reinterpret_cast<__nv_bfloat16*>(sm + off) = v[d];
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        // 2. S = Q . K^T into tensor-memory columns [0, 128)
        if (r == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int t = 0; t < AT_DH / 16; ++t)
                at_mma(tmem, at_desc(base + AT_Q + t * 32), at_desc(base + AT_K + t * 32), at_idesc(128), t > 0);
            at_commit(at_smem(&bar_s));
        }
        // every thread takes the same decision, so no thread leaves a barrier the others reach
        if (!__syncthreads_and(at_wait(at_smem(&bar_s), parity))) {
            ok = false;
            if (r == 0) atomicOr(A.error, 1u);
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // 3. online softmax over this block's keys (base 2); absent keys carry -inf
        float bmax = -INFINITY;
        for (int c = 0; c < AT_BLOCK; c += 32) {
            float s[32];
            at_ld32(lane_base + (uint32_t)c, s);
#pragma unroll
            for (int j = 0; j < 32; ++j) bmax = fmaxf(bmax, fmaf(s[j], scale2, kterm[c + j]));
        }
        const float m_new = fmaxf(m, bmax);
        const bool any = m_new != -INFINITY;  // some key so far is present
        const float corr = any ? exp2f(m - m_new) : 1.0f;
        const float shift = any ? m_new : 0.0f;
        float sum = 0.0f;
        for (int c = 0; c < AT_BLOCK; c += 32) {
            float s[32];
            at_ld32(lane_base + (uint32_t)c, s);
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float p0 = exp2f(fmaf(s[j], scale2, kterm[c + j]) - shift);
                const float p1 = exp2f(fmaf(s[j + 1], scale2, kterm[c + j + 1]) - shift);
                sum += p0 + p1;
                __nv_bfloat162 hv = __floats2bfloat162_rn(p0, p1);
                packed[j / 2] = *reinterpret_cast<uint32_t*>(&hv);
            }
            // row r of P: keys c..c+31 are chunks c/8 .. c/8+3 of column block c / 64
            const int blk = c >> 6, chunk0 = (c & 63) >> 3;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                *reinterpret_cast<uint4*>(sm + AT_P + blk * 16384 + sw128(r, chunk0 + q)) =
                    make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
        l = l * corr + sum;
        m = m_new;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        // 4. PV = P . V into tensor-memory columns [0, 32) (S has been read)
        if (r == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int t = 0; t < AT_BLOCK / 16; ++t)
                at_mma(tmem, at_desc(base + AT_P + (t >> 2) * 16384 + (t & 3) * 32),
                       at_desc(base + AT_VT + (t >> 2) * 4096 + (t & 3) * 32), at_idesc(AT_DH), t > 0);
            at_commit(at_smem(&bar_pv));
        }
        if (!__syncthreads_and(at_wait(at_smem(&bar_pv), parity))) {
            ok = false;
            if (r == 0) atomicOr(A.error, 2u);
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float pv[AT_DH];
        at_ld32(lane_base, pv);
#pragma unroll
        for (int j = 0; j < AT_DH; ++j) o[j] = fmaf(o[j], corr, pv[j]);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    // every MMA this CTA issued has completed before the tensor memory is freed
    if (r == 0) {
        at_commit(at_smem(&bar_done));
        for (uint32_t i = 0; i < AT_WAIT_TRIES && !at_try_wait(at_smem(&bar_done), 0u); ++i) {
        }
    }
    __syncthreads();
    if (ok) {
        const int q = qb * AT_BLOCK + r;
        if (q < A.len) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
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
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_attention_bf16(int32_t batch, int32_t len, int32_t heads, const void* qkv, const float* key_bias,
                                  const uint8_t* key_mask, const float* q_scale, void* out, uint32_t* error,
                                  void* stream) {
    PBG_REQUIRE(batch >= 0 && len >= 0 && heads >= 1, "attention: bad shape");
    PBG_REQUIRE(qkv && q_scale && out && error, "attention: null pointer");
    PBG_REQUIRE(((uintptr_t)qkv % 16) == 0 && ((uintptr_t)out % 16) == 0, "attention: qkv and out must be 16-byte aligned");
    if (batch == 0 || len == 0) return 0;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int rc = cuda_status(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  AT_SMEM + 1024),
                             "attention: shared memory size");
        if (rc) return rc;
        configured[dev] = 1;
    }
    AttnArgs A;
    A.batch = batch;
    A.len = len;
    A.heads = heads;
    A.qblocks = (len + AT_BLOCK - 1) / AT_BLOCK;
    A.qkv = static_cast<const __nv_bfloat16*>(qkv);
    A.key_bias = key_bias;
    A.key_mask = key_mask;
    A.q_scale = q_scale;
    A.out = static_cast<__nv_bfloat16*>(out);
    A.error = error;
    const int64_t grid = (int64_t)batch * heads * A.qblocks;
    PBG_REQUIRE(grid <= INT32_MAX, "attention: too many blocks");
    attention_kernel<<<(unsigned)grid, AT_THREADS, AT_SMEM + 1024, as_stream(stream)>>>(A);
    return launch_status("attention_bf16");
}
