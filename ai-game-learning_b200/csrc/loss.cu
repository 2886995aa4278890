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
// Algebra used to keep the row cheap (x logits, legal set L, e_j =
// exp(x_j - max) on L and 0 off L, s = sum e, lse = max + log s,
// p_j = e_j / s):
//   entropy       H      = lse - sum_j p_j x_j
//   d lp_a / d x_j       = [j == a] - p_j
//   d H / d x_j          = -p_j (x_j - lse + H)
//   d total / d x_j      = coef * ( g [j == a] + p_j (c x_j + c (H - lse) - g) )
// with g = d policy_row / d log_ratio and c the entropy coefficient; illegal
// entries vanish through e_j = 0.  Exponentials and logarithms run base 2 on
// the special-function unit (exp2f, __log2f: documented CUDA functions with a
// few-ulp error), about 1e-6 relative on the gradient.
//
// Layout: logits/dlogits [N,A] (bf16 or fp32), mask [N,A] u8 (0/1), action
// [N] i32, old_logp/adv/weight [N] f32.  For A == 8 with aligned rows one
// thread moves a whole row with 16/8/16-byte accesses (56 B per row with bf16
// logits), prefetches the next row before computing the current one, and
// does the elementwise work on bf16/f32 pairs.  Compiled with -ftz=true:
// denormal probabilities flush to zero.
// When every stream is 16-byte aligned and at least one 992-row tile exists,
// the rows are staged through shared memory by bulk-async copies (see
// ppo_bf16x8_bulk_kernel).  Per-block statistics go to caller scratch; the
// last block to finish sums them in block order (deterministic) and clears
// the arrival counter.
#include <cuda_bf16.h>

#include <algorithm>

#include "pbg_common.cuh"

namespace pbg {

constexpr int LOSS_BLOCK = 256;
constexpr int LOSS_STATS = 8;
constexpr int LOSS_MAX_A = 32;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct LossControls {
    float clip, cap, exp_cap, cent, coef_scale;  // coef_scale = scale * inv_count
    float lo, hi;                                // 1 - clip, 1 + clip
};

__device__ __forceinline__ LossControls load_controls(const float* c) {
    LossControls k;
    k.clip = c[0];
    k.cap = c[1];
    k.exp_cap = expf(c[1]);
    k.cent = c[2];
    k.coef_scale = c[3] * c[4];
    k.lo = 1.0f - c[0];
    k.hi = 1.0f + c[0];
    return k;
}

struct RowStats {
    float v[LOSS_STATS];  // v[7] (rows) is added once per thread by the kernel, not per row
    __device__ void zero() {
        #pragma unroll
        for (int i = 0; i < LOSS_STATS; ++i) v[i] = 0.0f;
    }
};

// Row objective pieces from the log ratio (learner.py:2021-2047): returns
// g = d policy_row / d log_ratio and writes policy_row and the ratio.
// policy_row = -min(f1, f2) with f1 = (capped) ratio * A, f2 = clip(ratio) * A;
// torch.minimum sends the gradient to the smaller operand and half to each
// at a tie; torch.clamp passes it inside [lo, hi] inclusive.
__device__ __forceinline__ float ratio_terms(float lr, float adv, const LossControls& k, float& prow,
                                             float& ratio_out) {
    float ratio = exp2f(lr * LOG2E);
    float clipped = fminf(fmaxf(ratio, k.lo), k.hi);
    bool negative = adv < 0.0f;
    // exp(min(lr, cap)) without a second exponential
    float neg_ratio = lr <= k.cap ? ratio : k.exp_cap;
    float pr = negative ? neg_ratio : ratio;
    float f1 = pr * adv, f2 = clipped * adv;
    prow = -fminf(f1, f2);
    float dpr = negative ? (lr < k.cap ? neg_ratio : (lr == k.cap ? 0.5f * neg_ratio : 0.0f)) : ratio;
    float dcl = (ratio >= k.lo && ratio <= k.hi) ? ratio : 0.0f;
    float d = f1 < f2 ? dpr : (f2 < f1 ? dcl : 0.5f * (dpr + dcl));
    ratio_out = ratio;
    return -adv * d;
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
}

// One row in registers: x[j] logits (overwritten with dlogits), legal(j) flags.
template <int A, class Legal>
__device__ __forceinline__ void row_backward(float (&x)[A], const Legal& legal, int act, float old, float adv,
                                             float w, const LossControls& k, RowStats& s) {
    float my = -INFINITY;
    #pragma unroll
    for (int j = 0; j < A; ++j) if (legal(j)) my = fmaxf(my, x[j] * LOG2E);
    float e[A];
    float se = 0.0f, sx = 0.0f, xa = 0.0f;
    #pragma unroll
    for (int j = 0; j < A; ++j) {
        bool on = legal(j);
        e[j] = on ? exp2f(fmaf(x[j], LOG2E, -my)) : 0.0f;
        se += e[j];
        sx = on ? fmaf(e[j], x[j], sx) : sx;  // masked logits may be -inf
        xa = j == act ? x[j] : xa;
    }
    float inv = __frcp_rn(se);
    float lse = (my + __log2f(se)) * LN2;
    float ent = lse - sx * inv;
    float lr = (xa - lse) - old;
    float prow, ratio;
    float g = ratio_terms(lr, adv, k, prow, ratio);
    float coef = k.coef_scale * w;
    float pscale = inv * coef;
    float K = k.cent * (ent - lse) - g;
    float ga = coef * g;
    #pragma unroll
    for (int j = 0; j < A; ++j) {
        float d = legal(j) ? (e[j] * pscale) * fmaf(k.cent, x[j], K) : 0.0f;
        x[j] = j == act ? d + ga : d;
    }
    accumulate(s, coef, w, prow, ent, ratio, lr, k, adv);
}

struct LegalBits {
    unsigned bits;
    __device__ bool operator()(int j) const { return (bits >> j) & 1u; }
};

// Scratch layout: slot 0 holds the arrival counter (low 32 bits) and an
// error word (high 32 bits); block b's sums are slots 1 + 8b .. 8 + 8b.  The
// fixed counter slot lets launches with different grids share one buffer.
// The last block to arrive sums all blocks in block order (deterministic),
// publishes stats (rows = -1 if any block reported an error) and clears slot 0.
// Returns true in the last block (every block's earlier global writes are then
// visible to it).
template <int BLOCK>
__device__ __forceinline__ bool block_stats(RowStats& s, double* partials, double* stats, bool failed = false) {
    __shared__ float red[BLOCK / 32][LOSS_STATS];
    __shared__ bool last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    #pragma unroll
    for (int i = 0; i < LOSS_STATS; ++i) {
        float v = warp_sum(s.v[i]);
        if (lane == 0) red[warp][i] = v;
    }
    __syncthreads();
    unsigned int* word = reinterpret_cast<unsigned int*>(partials);  // [0] counter, [1] error
    if (threadIdx.x < LOSS_STATS) {
        double acc = 0.0;
        for (int w = 0; w < BLOCK / 32; ++w) acc += (double)red[w][threadIdx.x];
        partials[1 + (int64_t)blockIdx.x * LOSS_STATS + threadIdx.x] = acc;
    }
    if (threadIdx.x == 0 && failed) atomicOr(word + 1, 1u);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(word, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return false;
    __threadfence();
    if (threadIdx.x < LOSS_STATS) {
        double acc = 0.0;
        for (unsigned b = 0; b < gridDim.x; ++b) acc += __ldcg(partials + 1 + (int64_t)b * LOSS_STATS + threadIdx.x);
        bool bad = __ldcg(reinterpret_cast<const unsigned long long*>(partials)) >> 32;
        stats[threadIdx.x] = (bad && threadIdx.x == LOSS_STATS - 1) ? -1.0 : acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<unsigned long long*>(partials) = 0ull;  // ready for the next launch
    return true;
}

// Rows a grid-stride loop starting at r0 with step `stride` visits below N.
__device__ __forceinline__ float strided_rows(int64_t r0, int64_t stride, int64_t N) {
    return r0 < N ? (float)((N - 1 - r0) / stride + 1) : 0.0f;
}

struct Row8 {
    uint4 logits;
    uint2 mask;
    int act;
    float old, adv, w;
};

__device__ __forceinline__ Row8 load_row8(int64_t r, const uint4* logits, const uint2* mask, const int32_t* action,
                                          const float* old_logp, const float* adv, const float* weight) {
    Row8 v;
    v.logits = __ldcs(logits + r);
    v.mask = __ldcs(mask + r);
    v.act = __ldcs(action + r);
    v.old = __ldcs(old_logp + r);
    v.adv = __ldcs(adv + r);
    v.w = __ldcs(weight + r);
    return v;
}

// A == 8, bf16 rows as four bf16x2 pairs ----------------------------------
//
// Mask bytes are 0/1 (torch.bool).  A pair's two bytes become a 32-bit lane
// mask w (0xFFFF per legal element) with one byte permute and one multiply;
// (x & w) | (-2^100 & ~w) is the logit pair with illegal entries at -2^100
// (one LOP3).
// Elementwise arithmetic runs on float2 with the packed FP32 instructions.
__device__ __forceinline__ float2 bf2_to_f2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

__device__ __forceinline__ void row8_backward(const Row8& row, const LossControls& k, RowStats& s, uint4& out) {
    const uint32_t v[4] = {row.logits.x, row.logits.y, row.logits.z, row.logits.w};
    const uint32_t mw[4] = {__byte_perm(row.mask.x, 0u, 0x1100) * 0xffu, __byte_perm(row.mask.x, 0u, 0x3322) * 0xffu,
                            __byte_perm(row.mask.y, 0u, 0x1100) * 0xffu, __byte_perm(row.mask.y, 0u, 0x3322) * 0xffu};
    // illegal entries become -2^100: exp underflows to exactly 0 and every product with
    // that 0 stays finite, so they drop out of the sums and get a zero gradient
    uint32_t xm[4];
    #pragma unroll
    for (int p = 0; p < 4; ++p) xm[p] = (v[p] & mw[p]) | (0xf180f180u & ~mw[p]);
    // masked max in bf16 (exact)
    __nv_bfloat162 m01 = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&xm[0]),
                                 *reinterpret_cast<const __nv_bfloat162*>(&xm[1]));
    __nv_bfloat162 m23 = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&xm[2]),
                                 *reinterpret_cast<const __nv_bfloat162*>(&xm[3]));
    __nv_bfloat162 mm = __hmax2(m01, m23);
    float my = fmaxf(__low2float(mm), __high2float(mm)) * LOG2E;
    const float2 L2 = make_float2(LOG2E, LOG2E), NMY = make_float2(-my, -my);
    float2 X[4], E[4];
    #pragma unroll
    for (int p = 0; p < 4; ++p) {
        X[p] = bf2_to_f2(xm[p]);
        float2 t = __ffma2_rn(X[p], L2, NMY);
        E[p] = make_float2(exp2f(t.x), exp2f(t.y));
    }
    float2 S = __fadd2_rn(__fadd2_rn(E[0], E[1]), __fadd2_rn(E[2], E[3]));
    float2 SX = __ffma2_rn(E[3], X[3], __ffma2_rn(E[2], X[2], __ffma2_rn(E[1], X[1], __fmul2_rn(E[0], X[0]))));
    float se = S.x + S.y, sx = SX.x + SX.y;
    const int act = row.act, ka = act >> 1;
    float2 Xa = ka == 0 ? X[0] : ka == 1 ? X[1] : ka == 2 ? X[2] : X[3];
    float xa = (act & 1) ? Xa.y : Xa.x;
    float inv = __fdividef(1.0f, se);
    float lse = (my + __log2f(se)) * LN2;
    float ent = lse - sx * inv;
    float lr = (xa - lse) - row.old;
    float prow, ratio;
    float g = ratio_terms(lr, row.adv, k, prow, ratio);
    float coef = k.coef_scale * row.w;
    float pscale = inv * coef;
    float K = k.cent * (ent - lse) - g;
    float ga = coef * g;
    const float2 PS = make_float2(pscale, pscale), C2 = make_float2(k.cent, k.cent), K2 = make_float2(K, K);
    const float2 GA = (act & 1) ? make_float2(0.0f, ga) : make_float2(ga, 0.0f);
    uint32_t o[4];
    #pragma unroll
    for (int p = 0; p < 4; ++p) {
        float2 d = __fmul2_rn(__fmul2_rn(E[p], PS), __ffma2_rn(C2, X[p], K2));
        if (p == ka) d = __fadd2_rn(d, GA);
        __nv_bfloat162 h = __floats2bfloat162_rn(d.x, d.y);
        o[p] = *reinterpret_cast<uint32_t*>(&h);
    }
    out = make_uint4(o[0], o[1], o[2], o[3]);
    accumulate(s, coef, row.w, prow, ent, ratio, lr, k, row.adv);
}

// A == 8, bf16: software-pipelined, one row per thread per step.
__global__ void __launch_bounds__(LOSS_BLOCK, 4) ppo_bf16x8_kernel(int64_t N, const uint4* __restrict__ logits,
                                                                    const uint2* __restrict__ mask,
                                                                    const int32_t* __restrict__ action,
                                                                    const float* __restrict__ old_logp,
                                                                    const float* __restrict__ adv,
                                                                    const float* __restrict__ weight,
                                                                    const float* __restrict__ controls,
                                                                    uint4* __restrict__ dlogits, double* partials,
                                                                    double* stats) {
    LossControls k = load_controls(controls);
    RowStats s;
    s.zero();
    const int64_t stride = (int64_t)gridDim.x * LOSS_BLOCK;
    int64_t r = (int64_t)blockIdx.x * LOSS_BLOCK + threadIdx.x;
    Row8 cur;
    if (r < N) cur = load_row8(r, logits, mask, action, old_logp, adv, weight);
    while (r < N) {
        int64_t nr = r + stride;
        Row8 nxt;
        if (nr < N) nxt = load_row8(nr, logits, mask, action, old_logp, adv, weight);
        uint4 out;
        row8_backward(cur, k, s, out);
        __stcs(dlogits + r, out);
        cur = nxt;
        r = nr;
    }
    s.v[7] = strided_rows((int64_t)blockIdx.x * LOSS_BLOCK + threadIdx.x, stride, N);
    block_stats<LOSS_BLOCK>(s, partials, stats);
}

// A == 8, bf16, bulk-async staged, warp-specialised -----------------------
//
// One persistent CTA per SM (1024 threads): warp 31 is the producer, warps
// 0..30 consume.  Tiles of BULK_T = 992 rows (one row per consumer thread)
// stream through a ring of BULK_STAGES shared-memory stages.  The producer's
// lane 0 fills a stage with six plain 1D bulk copies (cp.async.bulk global ->
// shared, no tensor map, no multicast) completing on the stage's "full"
// mbarrier; each consumer warp waits on it, computes its 32 rows, stores
// dlogits straight to global memory and arrives on the stage's "empty"
// mbarrier; the producer refills a stage once all 31 warps have released it.
// No warp waits on another warp's compute.  Every wait is bounded: a wait
// that runs out marks the launch failed (stats rows = -1), the producer
// waits (bounded again) for its copies still in flight, and the launch ends.
constexpr int BULK_CONSUMER_WARPS = 31;
constexpr int BULK_THREADS = 32 * (BULK_CONSUMER_WARPS + 1);
constexpr int BULK_T = 32 * BULK_CONSUMER_WARPS;  // 992 rows
constexpr int BULK_STAGES = 4;
constexpr uint32_t BULK_OFF_MASK = BULK_T * 16;
constexpr uint32_t BULK_OFF_ACT = BULK_OFF_MASK + BULK_T * 8;
constexpr uint32_t BULK_OFF_OLD = BULK_OFF_ACT + BULK_T * 4;
constexpr uint32_t BULK_OFF_ADV = BULK_OFF_OLD + BULK_T * 4;
constexpr uint32_t BULK_OFF_W = BULK_OFF_ADV + BULK_T * 4;
constexpr uint32_t BULK_TILE_BYTES = BULK_OFF_W + BULK_T * 4;  // 39,680 B, every offset a multiple of 16
constexpr size_t BULK_SMEM = (size_t)BULK_STAGES * BULK_TILE_BYTES;
constexpr uint32_t BULK_WAIT_TRIES = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < BULK_WAIT_TRIES; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

struct BulkArgs {
    int64_t N;
    const uint4* logits;
    const uint2* mask;
    const int32_t* action;
    const float* old_logp;
    const float* adv;
    const float* weight;
    const float* controls;
    uint4* dlogits;
    double* partials;
    double* stats;
};

__device__ __forceinline__ void bulk_issue(const BulkArgs& a, unsigned char* ring, uint32_t full_bar, int st,
                                           int64_t tile) {
    uint32_t dst = smem_u32(ring + (size_t)st * BULK_TILE_BYTES);
    int64_t r0 = tile * BULK_T;
    mbar_expect_tx(full_bar, BULK_TILE_BYTES);
    bulk_g2s(dst, a.logits + r0, BULK_T * 16, full_bar);
    bulk_g2s(dst + BULK_OFF_MASK, a.mask + r0, BULK_T * 8, full_bar);
    bulk_g2s(dst + BULK_OFF_ACT, a.action + r0, BULK_T * 4, full_bar);
    bulk_g2s(dst + BULK_OFF_OLD, a.old_logp + r0, BULK_T * 4, full_bar);
    bulk_g2s(dst + BULK_OFF_ADV, a.adv + r0, BULK_T * 4, full_bar);
    bulk_g2s(dst + BULK_OFF_W, a.weight + r0, BULK_T * 4, full_bar);
}

__global__ void __launch_bounds__(BULK_THREADS, 1) ppo_bf16x8_bulk_kernel(BulkArgs a) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t full[BULK_STAGES], empty[BULK_STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    LossControls k = load_controls(a.controls);
    RowStats s;
    s.zero();
    const int64_t ntiles = a.N / BULK_T;
    if (threadIdx.x == 0) {
        for (int st = 0; st < BULK_STAGES; ++st) {
            mbar_init(smem_u32(&full[st]), 1);
            mbar_init(smem_u32(&empty[st]), BULK_CONSUMER_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    bool failed = false;
    if (warp == BULK_CONSUMER_WARPS) {
        // producer
        if (lane == 0) {
            int64_t issued = 0;
            for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++issued) {
                const int st = (int)(issued % BULK_STAGES);
                if (issued >= BULK_STAGES &&
                    !mbar_wait_bounded(smem_u32(&empty[st]), (uint32_t)((issued / BULK_STAGES - 1) & 1))) {
                    failed = true;
                    break;
                }
                bulk_issue(a, ring, smem_u32(&full[st]), st, tile);
            }
            if (failed) {
                // copies of the last BULK_STAGES issued tiles may still be in flight
                int64_t first = issued > BULK_STAGES ? issued - BULK_STAGES : 0;
                for (int64_t m = first; m < issued; ++m)
                    mbar_wait_bounded(smem_u32(&full[m % BULK_STAGES]), (uint32_t)((m / BULK_STAGES) & 1));
            }
        }
    } else {
        // consumers: one row per thread per tile
        int64_t used = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++used) {
            const int st = (int)(used % BULK_STAGES);
            bool ok = mbar_wait_bounded(smem_u32(&full[st]), (uint32_t)((used / BULK_STAGES) & 1));
            if (!__all_sync(0xffffffffu, ok)) {
                failed = true;
                break;
            }
            const unsigned char* base = ring + (size_t)st * BULK_TILE_BYTES;
            const int rr = threadIdx.x;  // warp * 32 + lane < BULK_T
            Row8 row;
            row.logits = reinterpret_cast<const uint4*>(base)[rr];
            row.mask = reinterpret_cast<const uint2*>(base + BULK_OFF_MASK)[rr];
            row.act = reinterpret_cast<const int32_t*>(base + BULK_OFF_ACT)[rr];
            row.old = reinterpret_cast<const float*>(base + BULK_OFF_OLD)[rr];
            row.adv = reinterpret_cast<const float*>(base + BULK_OFF_ADV)[rr];
            row.w = reinterpret_cast<const float*>(base + BULK_OFF_W)[rr];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty[st]));  // this warp's rows are in registers
            uint4 out;
            row8_backward(row, k, s, out);
            __stcs(a.dlogits + tile * BULK_T + rr, out);
        }
        // rows after the last full tile: direct loads
        if (!failed) {
            const int64_t t0 = ntiles * BULK_T + (int64_t)blockIdx.x * BULK_T + threadIdx.x;
            s.v[7] = (float)used + strided_rows(t0, (int64_t)gridDim.x * BULK_T, a.N);
            for (int64_t r = t0; r < a.N; r += (int64_t)gridDim.x * BULK_T) {
                Row8 row = load_row8(r, a.logits, a.mask, a.action, a.old_logp, a.adv, a.weight);
                uint4 out;
                row8_backward(row, k, s, out);
                __stcs(a.dlogits + r, out);
            }
        }
    }
    block_stats<BULK_THREADS>(s, a.partials, a.stats, __syncthreads_or(failed));
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
                                                                  T* __restrict__ dlogits, double* partials,
                                                                  double* stats) {
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
        row_backward<LOSS_MAX_A>(x, LegalBits{legal}, action[r], old_logp[r], adv[r], weight[r], k, s);
        #pragma unroll
        for (int j = 0; j < LOSS_MAX_A; ++j)
            if (j < A) dlogits[r * A + j] = from_f<T>(x[j]);
    }
    s.v[7] = strided_rows((int64_t)blockIdx.x * LOSS_BLOCK + threadIdx.x, (int64_t)gridDim.x * LOSS_BLOCK, N);
    block_stats<LOSS_BLOCK>(s, partials, stats);
}

// Loss backward fused with the readout's weight gradient ------------------
//
// The learner's readout maps a hidden row h_r (bf16, width d) to the A = 8
// logits, x_r = W h_r + b.  Its gradients are rank-8 sums over the decisions,
// dW[a][k] = sum_r dx_r[a] h_r[k] and db[a] = sum_r dx_r[a], taken of the bf16
// dlogits this pass writes (the operand a separate weight-gradient GEMM would
// read back).  With 8 outputs that is 16 FLOPs per hidden element, about 8
// FLOP/B: below the FP32 ridge, so the sum runs on the FMA pipe inside the
// loss pass and the pass stays HBM bound at 56 + 2d bytes per row, with no
// second launch re-reading dlogits.
//
// Warps take 32-row chunks: lane l computes row l's dlogits (row8_backward),
// then the warp walks the chunk's 32 hidden rows in groups of 4 or 8: lane l
// holds columns [l*DC, l*DC + DC) of each row (one coalesced 2d-byte row per
// warp load) and adds the row's dlogits (staged once as fp32 in shared memory,
// read back as broadcasts) times its columns into packed fp32 accumulators.  A CTA's warps add their partial sums
// in warp order in shared memory; CTA partials go to caller scratch after the
// loss statistics, and the last CTA adds them in CTA order (in double), so
// the result does not depend on scheduling.
constexpr int RO_WARPS = 8;
constexpr int RO_THREADS = 32 * RO_WARPS;

// hidden rows loaded per batch, and the occupancy the register budget is set for
template <int DC>
__host__ __device__ constexpr int ro_group() {
    return DC == 8 ? 4 : 8;
}

template <int DC>
struct HiddenVec;
template <>
struct HiddenVec<2> {
    using T = uint32_t;
};
template <>
struct HiddenVec<4> {
    using T = uint2;
};
template <>
struct HiddenVec<8> {
    using T = uint4;
};

template <int DC>
__host__ __device__ constexpr int ro_min_blocks() {
    return DC == 2 ? 3 : (DC == 4 ? 2 : 1);
}

template <int DC>
constexpr size_t ro_smem() {
    return (size_t)RO_WARPS * (8 * 32 * DC + 8) * sizeof(float);
}

template <int DC>
__global__ void __launch_bounds__(RO_THREADS, ro_min_blocks<DC>())
ppo_readout_kernel(int64_t N, const uint4* __restrict__ logits, const uint2* __restrict__ mask,
                   const int32_t* __restrict__ action, const float* __restrict__ old_logp,
                   const float* __restrict__ adv, const float* __restrict__ weight,
                   const float* __restrict__ controls, const typename HiddenVec<DC>::T* __restrict__ hidden,
                   uint4* __restrict__ dlogits, float* __restrict__ dweight, float* __restrict__ dbias,
                   double* partials, double* stats) {
    using HV = typename HiddenVec<DC>::T;
    constexpr int D = 32 * DC;
    constexpr int OUT = 8 * D + 8;  // dW [8][D], then db [8]
    extern __shared__ float ro_red[];  // [RO_WARPS][OUT]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    LossControls k = load_controls(controls);
    RowStats s;
    s.zero();
    float2 acc[8][DC / 2];
    float db[8];
    #pragma unroll
    for (int a = 0; a < 8; ++a) {
        db[a] = 0.0f;
        #pragma unroll
        for (int j = 0; j < DC / 2; ++j) acc[a][j] = make_float2(0.0f, 0.0f);
    }
    float rows_done = 0.0f;
    const int64_t chunks = (N + 31) / 32;
    const int64_t wstride = (int64_t)gridDim.x * RO_WARPS;
    constexpr int G = ro_group<DC>();
    // Software pipeline: while a group of hidden rows is summed, the next group (or the next chunk's
    // first group) and the next chunk's loss row are already loading.
    auto load_group = [&](int64_t first, HV (&hv)[G]) {
        #pragma unroll
        for (int i = 0; i < G; ++i) {
            const int64_t rr = first + i;
            hv[i] = rr < N ? __ldcs(hidden + rr * 32 + lane) : HV{};
        }
    };
    float* staged = ro_red + warp * 32 * 8;  // [32][8] fp32 dlogits of the warp's chunk
    int64_t c = (int64_t)blockIdx.x * RO_WARPS + warp;
    Row8 row;
    HV cur[G];
    if (c < chunks) {
        if (c * 32 + lane < N) row = load_row8(c * 32 + lane, logits, mask, action, old_logp, adv, weight);
        load_group(c * 32, cur);
    }
    for (; c < chunks; c += wstride) {
        const int64_t r = c * 32 + lane;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (r < N) {
            row8_backward(row, k, s, out);
            __stcs(dlogits + r, out);
            rows_done += 1.0f;
        }
        const int64_t nc = c + wstride;
        if (nc < chunks && nc * 32 + lane < N) row = load_row8(nc * 32 + lane, logits, mask, action, old_logp, adv, weight);
        {
            // the row's dlogits as fp32, once, into the warp's staging rows (read back as broadcasts)
            const float2 d01 = bf2_to_f2(out.x), d23 = bf2_to_f2(out.y), d45 = bf2_to_f2(out.z),
                         d67 = bf2_to_f2(out.w);
            db[0] += d01.x; db[1] += d01.y; db[2] += d23.x; db[3] += d23.y;
            db[4] += d45.x; db[5] += d45.y; db[6] += d67.x; db[7] += d67.y;
            float4* mine = reinterpret_cast<float4*>(staged + lane * 8);
            mine[0] = make_float4(d01.x, d01.y, d23.x, d23.y);
            mine[1] = make_float4(d45.x, d45.y, d67.x, d67.y);
        }
        __syncwarp();
        #pragma unroll 1
        for (int g = 0; g < 32; g += G) {
            HV nxt[G];
            if (g + G < 32) load_group(c * 32 + g + G, nxt);
            else if (nc < chunks) load_group(nc * 32, nxt);
            #pragma unroll
            for (int i = 0; i < G; ++i) {
                const float4 lo = reinterpret_cast<const float4*>(staged + (g + i) * 8)[0];
                const float4 hi = reinterpret_cast<const float4*>(staged + (g + i) * 8)[1];
                const float dl[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                const uint32_t* hw = reinterpret_cast<const uint32_t*>(&cur[i]);
                float2 h[DC / 2];
                #pragma unroll
                for (int j = 0; j < DC / 2; ++j) h[j] = bf2_to_f2(hw[j]);
                #pragma unroll
                for (int a = 0; a < 8; ++a) {
                    const float2 da = make_float2(dl[a], dl[a]);
                    #pragma unroll
                    for (int j = 0; j < DC / 2; ++j) acc[a][j] = __ffma2_rn(h[j], da, acc[a][j]);
                }
            }
            #pragma unroll
            for (int i = 0; i < G; ++i) cur[i] = nxt[i];
        }
        __syncwarp();  // every lane has read the staging rows before the next chunk rewrites them
    }
    // this warp's partial sums (over the staging rows: every warp is past its loop), then the CTA's
    // in warp order
    __syncthreads();
    float* mine = ro_red + warp * OUT;
    #pragma unroll
    for (int a = 0; a < 8; ++a) {
        #pragma unroll
        for (int j = 0; j < DC / 2; ++j)
            *reinterpret_cast<float2*>(mine + a * D + lane * DC + 2 * j) = acc[a][j];
        const float t = warp_sum(db[a]);
        if (lane == 0) mine[8 * D + a] = t;
    }
    __syncthreads();
    float* cta = reinterpret_cast<float*>(partials + 1 + (int64_t)gridDim.x * LOSS_STATS) + (int64_t)blockIdx.x * OUT;
    for (int o = threadIdx.x; o < OUT; o += RO_THREADS) {
        float v = 0.0f;
        #pragma unroll
        for (int w = 0; w < RO_WARPS; ++w) v += ro_red[w * OUT + o];
        cta[o] = v;
    }
    s.v[7] = rows_done;
    if (block_stats<RO_THREADS>(s, partials, stats)) {
        const float* all = reinterpret_cast<const float*>(partials + 1 + (int64_t)gridDim.x * LOSS_STATS);
        for (int o = threadIdx.x; o < OUT; o += RO_THREADS) {
            double v = 0.0;
            for (unsigned b = 0; b < gridDim.x; ++b) v += (double)__ldcg(all + (int64_t)b * OUT + o);
            if (o < 8 * D) dweight[o] = (float)v;
            else dbias[o - 8 * D] = (float)v;
        }
    }
}

// Staged variant (every stream 16-byte aligned): each warp (12 per CTA; 16 at
// d = 64, 6 at d = 256) keeps its own ring of two chunk stages in shared memory, filled by
// plain 1D bulk copies (cp.async.bulk global -> shared, no tensor map, no
// multicast) that its lane 0 issues STAGES chunks ahead, completing on the
// stage's mbarrier.  A
// chunk's 32 hidden rows are contiguous in [N, d], so one copy brings all of
// them, and six more bring the loss inputs; the loads no longer hold registers,
// so a CTA of 12 warps keeps up to 24 chunks (227 KB at d = 128) in flight.  After a lane has
// its loss row in registers, the stage's first 1,024 bytes (logits, mask,
// action, old log pi) are reused as the fp32 dlogits staging rows.  Every wait
// is bounded: one that runs out marks the launch failed (stats rows = -1),
// lane 0 waits (bounded again) for its copies still in flight, and the warp
// stops.  The rows after the last whole chunk go through direct loads.
template <int DC>
struct RoBulk {
    static constexpr int D = 32 * DC;
    static constexpr uint32_t HID = 32u * 2u * D;  // the chunk's hidden rows
    static constexpr uint32_t LOGITS = HID, MASK = HID + 512, ACT = MASK + 256, OLD = ACT + 128, ADV = OLD + 128,
                              WGT = ADV + 128, BYTES = WGT + 128;  // every offset a multiple of 16
    static constexpr int STAGES = 2;
    static constexpr int WARPS = DC == 8 ? 6 : (DC == 2 ? 16 : 12);
    static constexpr int THREADS = 32 * WARPS;
    static constexpr size_t SMEM = (size_t)WARPS * STAGES * BYTES;
};

struct RoArgs {
    int64_t N;
    const uint4* logits;
    const uint2* mask;
    const int32_t* action;
    const float* old_logp;
    const float* adv;
    const float* weight;
    const float* controls;
    const unsigned char* hidden;
    uint4* dlogits;
    float* dweight;
    float* dbias;
    double* partials;
    double* stats;
};

// dW += dl[row] (x) h[row] for the chunk's 32 rows: h rows from `hid` ([32][32] HV), fp32 dlogits
// from `staged` ([32][8]).  acc[p][c] holds (dW[2p][col], dW[2p+1][col]) for the lane's column c: the
// logit pairs come straight from the staged row, only the hidden value is duplicated per pair.
template <int DC>
__device__ __forceinline__ void ro_accumulate(const typename HiddenVec<DC>::T* hid, const float* staged, int lane,
                                              float2 (&acc)[4][DC]) {
    using HV = typename HiddenVec<DC>::T;
    #pragma unroll 4
    for (int r = 0; r < 32; ++r) {
        const HV hv = hid[r * 32 + lane];
        const float4 lo = reinterpret_cast<const float4*>(staged + r * 8)[0];
        const float4 hi = reinterpret_cast<const float4*>(staged + r * 8)[1];
        const float2 dp[4] = {make_float2(lo.x, lo.y), make_float2(lo.z, lo.w), make_float2(hi.x, hi.y),
                              make_float2(hi.z, hi.w)};
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv);
        #pragma unroll
        for (int j = 0; j < DC / 2; ++j) {
            const float h0 = __uint_as_float(hw[j] << 16), h1 = __uint_as_float(hw[j] & 0xffff0000u);
            const float2 hh0 = make_float2(h0, h0), hh1 = make_float2(h1, h1);
            #pragma unroll
            for (int q = 0; q < 4; ++q) {
                acc[q][2 * j] = __ffma2_rn(dp[q], hh0, acc[q][2 * j]);
                acc[q][2 * j + 1] = __ffma2_rn(dp[q], hh1, acc[q][2 * j + 1]);
            }
        }
    }
}

__device__ __forceinline__ void ro_stage_dl(const uint4& out, float* staged, int lane, float (&db)[8]) {
    const float2 d01 = bf2_to_f2(out.x), d23 = bf2_to_f2(out.y), d45 = bf2_to_f2(out.z), d67 = bf2_to_f2(out.w);
    db[0] += d01.x; db[1] += d01.y; db[2] += d23.x; db[3] += d23.y;
    db[4] += d45.x; db[5] += d45.y; db[6] += d67.x; db[7] += d67.y;
    float4* mine = reinterpret_cast<float4*>(staged + lane * 8);
    mine[0] = make_float4(d01.x, d01.y, d23.x, d23.y);
    mine[1] = make_float4(d45.x, d45.y, d67.x, d67.y);
}

template <int DC>
__global__ void __launch_bounds__(RoBulk<DC>::THREADS, 1) ppo_readout_bulk_kernel(RoArgs a) {
    using B = RoBulk<DC>;
    using HV = typename HiddenVec<DC>::T;
    constexpr int D = B::D, OUT = 8 * D + 8, S = B::STAGES, W = B::WARPS;
    extern __shared__ __align__(128) unsigned char ro_ring[];
    __shared__ __align__(8) uint64_t full[W][S];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* ring = ro_ring + (size_t)warp * S * B::BYTES;
    LossControls k = load_controls(a.controls);
    RowStats s;
    s.zero();
    float2 acc[4][DC];
    float db[8];
    #pragma unroll
    for (int q = 0; q < 8; ++q) db[q] = 0.0f;
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
        #pragma unroll
        for (int j = 0; j < DC; ++j) acc[q][j] = make_float2(0.0f, 0.0f);
    }
    float rows_done = 0.0f;
    const int64_t whole = a.N / 32;
    const int64_t gw = (int64_t)blockIdx.x * W + warp;
    const int64_t wstride = (int64_t)gridDim.x * W;
    if (lane == 0) {
        for (int st = 0; st < S; ++st) mbar_init(smem_u32(&full[warp][st]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int64_t chunk, int st) {
        const uint32_t dst = smem_u32(ring + (size_t)st * B::BYTES), bar = smem_u32(&full[warp][st]);
        const int64_t r0 = chunk * 32;
        // order this warp's earlier generic accesses to the stage before the copies overwrite it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bar, B::BYTES);
        bulk_g2s(dst, a.hidden + r0 * 2 * D, B::HID, bar);
        bulk_g2s(dst + B::LOGITS, a.logits + r0, 512, bar);
        bulk_g2s(dst + B::MASK, a.mask + r0, 256, bar);
        bulk_g2s(dst + B::ACT, a.action + r0, 128, bar);
        bulk_g2s(dst + B::OLD, a.old_logp + r0, 128, bar);
        bulk_g2s(dst + B::ADV, a.adv + r0, 128, bar);
        bulk_g2s(dst + B::WGT, a.weight + r0, 128, bar);
    };
    int64_t issued = 0;  // chunks this warp has requested (lane 0's count; the same on every lane)
    for (int st = 0; st < S; ++st) {
        const int64_t chunk = gw + st * wstride;
        if (chunk >= whole) break;
        if (lane == 0) issue(chunk, st);
        ++issued;
    }
    bool failed = false;
    int64_t used = 0;
    for (int64_t c = gw; c < whole; c += wstride, ++used) {
        const int st = (int)(used % S);
        const bool ok = mbar_wait_bounded(smem_u32(&full[warp][st]), (uint32_t)((used / S) & 1));
        if (!__all_sync(0xffffffffu, ok)) {
            failed = true;
            break;
        }
        unsigned char* base = ring + (size_t)st * B::BYTES;
        Row8 row;
        row.logits = reinterpret_cast<const uint4*>(base + B::LOGITS)[lane];
        row.mask = reinterpret_cast<const uint2*>(base + B::MASK)[lane];
        row.act = reinterpret_cast<const int32_t*>(base + B::ACT)[lane];
        row.old = reinterpret_cast<const float*>(base + B::OLD)[lane];
        row.adv = reinterpret_cast<const float*>(base + B::ADV)[lane];
        row.w = reinterpret_cast<const float*>(base + B::WGT)[lane];
        __syncwarp();  // every lane holds its row: the logits .. old log pi bytes become the staging rows
        uint4 out;
        row8_backward(row, k, s, out);
        __stcs(a.dlogits + c * 32 + lane, out);
        rows_done += 1.0f;
        float* staged = reinterpret_cast<float*>(base + B::LOGITS);
        ro_stage_dl(out, staged, lane, db);
        __syncwarp();
        ro_accumulate<DC>(reinterpret_cast<const HV*>(base), staged, lane, acc);
        __syncwarp();  // the stage is consumed
        const int64_t next = c + S * wstride;
        if (next < whole) {
            if (lane == 0) issue(next, st);
            ++issued;
        }
    }
    if (failed) {
        // copies of the chunks requested but not consumed may still be in flight
        if (lane == 0)
            for (int64_t m = used; m < issued; ++m)
                mbar_wait_bounded(smem_u32(&full[warp][m % S]), (uint32_t)((m / S) & 1));
        __syncwarp();
    } else if (a.N % 32 && gw == whole % wstride) {
        // the rows after the last whole chunk: direct loads, staged through this warp's first stage
        const int64_t r = whole * 32 + lane;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (r < a.N) {
            Row8 row = load_row8(r, a.logits, a.mask, a.action, a.old_logp, a.adv, a.weight);
            row8_backward(row, k, s, out);
            __stcs(a.dlogits + r, out);
            rows_done += 1.0f;
        }
        HV* hid = reinterpret_cast<HV*>(ring);
        const HV* src = reinterpret_cast<const HV*>(a.hidden);
        for (int rr = 0; rr < 32; ++rr)
            hid[rr * 32 + lane] = whole * 32 + rr < a.N ? __ldcs(src + (whole * 32 + rr) * 32 + lane) : HV{};
        float* staged = reinterpret_cast<float*>(ring + B::LOGITS);
        ro_stage_dl(out, staged, lane, db);
        __syncwarp();
        ro_accumulate<DC>(hid, staged, lane, acc);
    }
    // every warp is past the ring: it now holds the warps' partial sums, then the CTA's in warp order
    __syncthreads();
    float* red = reinterpret_cast<float*>(ro_ring);
    float* mine = red + warp * OUT;
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
        #pragma unroll
        for (int j = 0; j < DC; ++j) {
            mine[(2 * q) * D + lane * DC + j] = acc[q][j].x;
            mine[(2 * q + 1) * D + lane * DC + j] = acc[q][j].y;
        }
    }
    #pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float t = warp_sum(db[q]);
        if (lane == 0) mine[8 * D + q] = t;
    }
    __syncthreads();
    float* cta = reinterpret_cast<float*>(a.partials + 1 + (int64_t)gridDim.x * LOSS_STATS) + (int64_t)blockIdx.x * OUT;
    for (int o = threadIdx.x; o < OUT; o += B::THREADS) {
        float v = 0.0f;
        #pragma unroll
        for (int w = 0; w < W; ++w) v += red[w * OUT + o];
        cta[o] = v;
    }
    s.v[7] = rows_done;
    if (block_stats<B::THREADS>(s, a.partials, a.stats, __syncthreads_or(failed))) {
        const float* all = reinterpret_cast<const float*>(a.partials + 1 + (int64_t)gridDim.x * LOSS_STATS);
        for (int o = threadIdx.x; o < OUT; o += B::THREADS) {
            double v = 0.0;
            for (unsigned b = 0; b < gridDim.x; ++b) v += (double)__ldcg(all + (int64_t)b * OUT + o);
            if (o < 8 * D) a.dweight[o] = (float)v;
            else a.dbias[o - 8 * D] = (float)v;
        }
    }
}

// CTAs of the staged launch: one per SM at most, each with work for every warp where there is enough.
template <int DC>
int readout_bulk_grid(int64_t N) {
    const int64_t whole = N / 32;
    const int64_t need = (whole + RoBulk<DC>::WARPS - 1) / RoBulk<DC>::WARPS;
    return (int)std::max<int64_t>(1, std::min<int64_t>(need, sm_count()));
}

template <int DC>
int readout_bulk_launch(const RoArgs& a, cudaStream_t s) {
    static bool ready[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!ready[dev]) {
        int rc = cuda_status(cudaFuncSetAttribute(ppo_readout_bulk_kernel<DC>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RoBulk<DC>::SMEM),
                             "ppo_readout: shared-memory opt-in");
        if (rc) return rc;
        ready[dev] = true;
    }
    ppo_readout_bulk_kernel<DC><<<readout_bulk_grid<DC>(a.N), RoBulk<DC>::THREADS, RoBulk<DC>::SMEM, s>>>(a);
    return PBG_OK;
}

template <int DC>
int readout_grid_dc(int64_t N) {
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = dev >= 0 && dev < 64 ? dev : 0;
    if (per_sm[slot] == 0) {
        int n = 0;
        if (cudaFuncSetAttribute(ppo_readout_kernel<DC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)ro_smem<DC>()) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ppo_readout_kernel<DC>, RO_THREADS, ro_smem<DC>()) !=
                cudaSuccess ||
            n <= 0)
            n = 1;
        per_sm[slot] = n;
    }
    return stride_grid((N + 31) / 32, RO_WARPS, per_sm[slot]);
}

int readout_grid(int64_t N, int d) {
    return d == 64 ? readout_grid_dc<2>(N) : d == 128 ? readout_grid_dc<4>(N) : readout_grid_dc<8>(N);
}

// One wave of resident blocks (occupancy of the vector kernel), grid-stride beyond.
int ppo_grid(int64_t N) {
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int slot = dev >= 0 && dev < 64 ? dev : 0;
    if (per_sm[slot] == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ppo_bf16x8_kernel, LOSS_BLOCK, 0) != cudaSuccess || n <= 0)
            n = 4;
        per_sm[slot] = n;
    }
    return stride_grid(N, LOSS_BLOCK, per_sm[slot]);
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_ppo_partials_size(int64_t N, int32_t A) {
    (void)A;
    // one counter/error slot plus per-block statistics of the widest launch
    return 1 + (int64_t)ppo_grid(N > 0 ? N : 1) * LOSS_STATS;
}

int pbg_ppo_categorical_backward_grid(int64_t N, int32_t A, int32_t dtype, const void* logits, const uint8_t* mask,
                                      const int32_t* action, const float* old_logp, const float* adv,
                                      const float* weight, const float* controls, void* dlogits, double* partials,
                                      double* stats, int32_t max_ctas, void* stream) {
    PBG_REQUIRE(max_ctas >= 0, "ppo: max_ctas must be >= 0 (0 = no cap)");
    PBG_REQUIRE(N >= 0 && A >= 1 && A <= LOSS_MAX_A, "ppo: need N >= 0 and A in [1,32]");
    PBG_REQUIRE(dtype == 0 || dtype == 1, "ppo: dtype must be 0 (fp32) or 1 (bf16)");
    PBG_REQUIRE(controls && partials && stats, "ppo: null controls or scratch");
    PBG_REQUIRE(N == 0 || (logits && mask && action && old_logp && adv && weight && dlogits), "ppo: null argument");
    cudaStream_t s = as_stream(stream);
    int grid = ppo_grid(N > 0 ? N : 1);
    bool vec = dtype == 1 && A == 8 && ((uintptr_t)logits % 16 == 0) && ((uintptr_t)dlogits % 16 == 0) &&
               ((uintptr_t)mask % 8 == 0);
    bool bulk = vec && N >= BULK_T && ((uintptr_t)mask % 16 == 0) && ((uintptr_t)action % 16 == 0) &&
                ((uintptr_t)old_logp % 16 == 0) && ((uintptr_t)adv % 16 == 0) && ((uintptr_t)weight % 16 == 0);
    if (bulk) {
        static bool smem_ready[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) dev = 0;
        if (!smem_ready[dev]) {
            int rc = cuda_status(cudaFuncSetAttribute(ppo_bf16x8_bulk_kernel,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BULK_SMEM),
                                 "ppo: shared-memory opt-in");
            if (rc) return rc;
            smem_ready[dev] = true;
        }
        int64_t tiles = N / BULK_T;
        int bgrid = (int)(tiles < sm_count() ? tiles : sm_count());
        if (max_ctas > 0 && bgrid > max_ctas) bgrid = max_ctas;  // leave SMs to concurrent work
        BulkArgs a{N, (const uint4*)logits, (const uint2*)mask, action, old_logp, adv, weight, controls,
                   (uint4*)dlogits, partials, stats};
        ppo_bf16x8_bulk_kernel<<<bgrid, BULK_THREADS, BULK_SMEM, s>>>(a);
    } else if (vec) {
        ppo_bf16x8_kernel<<<grid, LOSS_BLOCK, 0, s>>>(N, (const uint4*)logits, (const uint2*)mask, action, old_logp,
                                                      adv, weight, controls, (uint4*)dlogits, partials, stats);
    } else if (dtype == 1) {
        ppo_generic_kernel<__nv_bfloat16><<<grid, LOSS_BLOCK, 0, s>>>(
            N, A, (const __nv_bfloat16*)logits, mask, action, old_logp, adv, weight, controls,
            (__nv_bfloat16*)dlogits, partials, stats);
    } else {
        ppo_generic_kernel<float><<<grid, LOSS_BLOCK, 0, s>>>(N, A, (const float*)logits, mask, action, old_logp, adv,
                                                              weight, controls, (float*)dlogits, partials, stats);
    }
    return launch_status("ppo_categorical_backward");
}

int pbg_ppo_categorical_backward(int64_t N, int32_t A, int32_t dtype, const void* logits, const uint8_t* mask,
                                 const int32_t* action, const float* old_logp, const float* adv,
                                 const float* weight, const float* controls, void* dlogits, double* partials,
                                 double* stats, void* stream) {
    return pbg_ppo_categorical_backward_grid(N, A, dtype, logits, mask, action, old_logp, adv, weight, controls,
                                             dlogits, partials, stats, 0, stream);
}

int64_t pbg_ppo_readout_partials_size(int64_t N, int32_t A, int32_t d) {
    if (A != 8 || !(d == 64 || d == 128 || d == 256)) return -1;
    // the wider of the two launches (direct-load and staged) sizes the per-block partials
    const int64_t n = N > 0 ? N : 1;
    const int64_t staged = d == 64 ? readout_bulk_grid<2>(n) : d == 128 ? readout_bulk_grid<4>(n) : readout_bulk_grid<8>(n);
    const int64_t grid = std::max<int64_t>(readout_grid(n, d), staged);
    const int64_t floats = grid * (8LL * d + 8);
    // counter/error slot, per-block statistics, then per-block dW/db partials (two floats per slot)
    return 1 + grid * LOSS_STATS + (floats + 1) / 2;
}

int pbg_ppo_readout_backward(int64_t N, int32_t A, const void* logits, const uint8_t* mask, const int32_t* action,
                             const float* old_logp, const float* adv, const float* weight, const float* controls,
                             const void* hidden, int32_t d, void* dlogits, float* dweight, float* dbias,
                             double* partials, double* stats, void* stream) {
    PBG_REQUIRE(N >= 0 && A == 8, "ppo_readout: need N >= 0 and A == 8");
    PBG_REQUIRE(d == 64 || d == 128 || d == 256, "ppo_readout: hidden width must be 64, 128 or 256");
    PBG_REQUIRE(controls && partials && stats && dweight && dbias, "ppo_readout: null controls, scratch or output");
    PBG_REQUIRE(N == 0 || (logits && mask && action && old_logp && adv && weight && hidden && dlogits),
                "ppo_readout: null argument");
    PBG_REQUIRE(N == 0 || ((uintptr_t)logits % 16 == 0 && (uintptr_t)dlogits % 16 == 0 && (uintptr_t)mask % 8 == 0 &&
                           (uintptr_t)hidden % 16 == 0),
                "ppo_readout: logits, dlogits and hidden must be 16-byte aligned, mask 8-byte aligned");
    cudaStream_t s = as_stream(stream);
    const bool staged = N >= 32 && (uintptr_t)mask % 16 == 0 && (uintptr_t)action % 16 == 0 &&
                        (uintptr_t)old_logp % 16 == 0 && (uintptr_t)adv % 16 == 0 && (uintptr_t)weight % 16 == 0;
    if (staged) {
        RoArgs a{N, (const uint4*)logits, (const uint2*)mask, action, old_logp, adv, weight, controls,
                 (const unsigned char*)hidden, (uint4*)dlogits, dweight, dbias, partials, stats};
        const int rc = d == 64    ? readout_bulk_launch<2>(a, s)
                       : d == 128 ? readout_bulk_launch<4>(a, s)
                                  : readout_bulk_launch<8>(a, s);
        if (rc) return rc;
        return launch_status("ppo_readout_backward");
    }
    const int grid = readout_grid(N > 0 ? N : 1, d);
    if (d == 64) {
        ppo_readout_kernel<2><<<grid, RO_THREADS, ro_smem<2>(), s>>>(
            N, (const uint4*)logits, (const uint2*)mask, action, old_logp, adv, weight, controls,
            (const uint32_t*)hidden, (uint4*)dlogits, dweight, dbias, partials, stats);
    } else if (d == 128) {
        ppo_readout_kernel<4><<<grid, RO_THREADS, ro_smem<4>(), s>>>(
            N, (const uint4*)logits, (const uint2*)mask, action, old_logp, adv, weight, controls,
            (const uint2*)hidden, (uint4*)dlogits, dweight, dbias, partials, stats);
    } else {
        ppo_readout_kernel<8><<<grid, RO_THREADS, ro_smem<8>(), s>>>(
            N, (const uint4*)logits, (const uint2*)mask, action, old_logp, adv, weight, controls,
            (const uint4*)hidden, (uint4*)dlogits, dweight, dbias, partials, stats);
    }
    return launch_status("ppo_readout_backward");
}

}  // extern "C"

// ===================================================== allocation-free variant
//
// Some callers cannot call cudaMalloc: host applications that hand all
// device memory to their own pool and forbid allocations once training
// starts, plugins whose binding has no way to pass a scratch buffer, and code
// that must not stall on the allocator in the middle of a step.  For them
// the per-block loss statistics live in a fixed array compiled into this
// library instead of in caller scratch.  Every GPU that loads the library
// holds the array (about 128 KiB) until the process exits.
#include <mutex>

namespace pbg {

constexpr int NOALLOC_MAX_BLOCKS = 2048;  // statistics of at most 2048 thread blocks
static __device__ __align__(256) double g_ppo_noalloc_scratch[NOALLOC_MAX_BLOCKS * LOSS_STATS + 1];

static std::mutex g_noalloc_mutex;
static double* g_noalloc_ptr[64] = {nullptr};

// Device address of the array on the current device.  The array's name is
// only a host-side stand-in, so the address is looked up once per device,
// with that device current, and cached.
static int noalloc_scratch(double** out) {
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev), "ppo_noalloc: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) {
        set_error("ppo_noalloc: device ordinal %d is beyond the 64 supported", dev);
        return PBG_ERANGE;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        rc = cuda_status(cudaGetSymbolAddress(&p, g_ppo_noalloc_scratch), "ppo_noalloc: cudaGetSymbolAddress");
        if (rc) return rc;
        g_noalloc_ptr[dev] = static_cast<double*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return PBG_OK;
}

}  // namespace pbg

extern "C" int pbg_ppo_categorical_backward_noalloc(int64_t N, int32_t A, int32_t dtype, const void* logits,
                                                    const uint8_t* mask, const int32_t* action,
                                                    const float* old_logp, const float* adv, const float* weight,
                                                    const float* controls, void* dlogits, double* stats,
                                                    void* stream) {
    // Reject bad arguments before anything touches the shared array: a refused call must not
    // queue a write that could race with another caller's launch.
    PBG_REQUIRE(N >= 0 && A >= 1 && A <= LOSS_MAX_A, "ppo_noalloc: need N >= 0 and A in [1,32]");
    PBG_REQUIRE(dtype == 0 || dtype == 1, "ppo_noalloc: dtype must be 0 (fp32) or 1 (bf16)");
    PBG_REQUIRE(controls && stats, "ppo_noalloc: null controls or statistics");
    PBG_REQUIRE(N == 0 || (logits && mask && action && old_logp && adv && weight && dlogits),
                "ppo_noalloc: null argument");
    int grid = ppo_grid(N > 0 ? N : 1);
    if (grid > NOALLOC_MAX_BLOCKS) {
        set_error("ppo_noalloc: this launch needs statistics for %d blocks; the built-in scratch holds %d "
                  "(use pbg_ppo_categorical_backward with caller scratch)", grid, NOALLOC_MAX_BLOCKS);
        return PBG_ERANGE;
    }
    double* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // The arrival counter and error word (slot 0) must start at zero; clear them in stream order.
    rc = cuda_status(cudaMemsetAsync(scratch, 0, sizeof(double), as_stream(stream)),
                     "ppo_noalloc: clearing the arrival counter");
    if (rc) return rc;
    return pbg_ppo_categorical_backward(N, A, dtype, logits, mask, action, old_logp, adv, weight, controls, dlogits,
                                        scratch, stats, stream);
}
