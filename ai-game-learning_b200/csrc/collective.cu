// Flat fp32 gradient SUM over NVLink SHARP (NVLS) multicast memory.
//
// Replaces the NCCL all_reduce(SUM) of pbg/core/replica.py:352-362 for a
// gradient buffer allocated in symmetric memory and bound to a multicast
// object.  Every rank owns 1/world of the buffer: it reads that slice with
// multimem.ld_reduce (the NVSwitch returns the sum over all ranks' copies)
// and writes the sum back with multimem.st (the switch stores it into every
// rank's copy).  Two cross-rank barriers bracket the reduction: the first
// makes every rank's gradient complete before anyone reads it, the second
// makes every rank's multicast stores complete before anyone uses the sum.
//
// Barrier protocol: CTA c of rank r signals peer p by a release store of 1
// into p's signal pad at slot ((phase * grid + c) * world + r), then waits
// (acquire) for its own slots ((phase * grid + c) * world + p) of every peer
// and clears them.  The host caps the grid to what the pad holds.  Barrier 1 and barrier 2
// use disjoint slot ranges, which is enough for back-to-back calls: a peer can
// only signal a slot again after this rank has cleared it (the intervening
// barrier orders it).  Every wait is bounded; a wait that runs out sets
// *error and the kernel returns without touching the buffer further.  The
// error word is sticky: a launch that finds it set returns at entry, before
// signalling anyone, so slots left stale by a timed-out barrier are never
// read by a later call (clear the pads and the word together to reuse them).
#include "pbg_common.cuh"

namespace pbg {

constexpr int NVLS_THREADS = 512;
constexpr int NVLS_MAX_BLOCKS = 160;
constexpr int NVLS_MAX_WORLD = 8;
constexpr int NVLS_UNROLL = 4;
constexpr uint32_t NVLS_WAIT_TRIES = 1u << 22;

__device__ __forceinline__ void signal_release(uint32_t* addr) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(1u) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// Cross-rank barrier of CTA blockIdx.x; returns false when a wait ran out.
__device__ bool rank_barrier(uint32_t* const* pads, int rank, int world, int phase, uint32_t* error) {
    __shared__ int ok_shared;
    if (threadIdx.x == 0) ok_shared = 1;
    __syncthreads();
    const int slot_base = (phase * (int)gridDim.x + (int)blockIdx.x) * world;
    if (threadIdx.x < world) {
        const int peer = threadIdx.x;
        __threadfence_system();
        signal_release(pads[peer] + slot_base + rank);
        uint32_t* mine = pads[rank] + slot_base + peer;
        bool done = false;
        for (uint32_t i = 0; i < NVLS_WAIT_TRIES; ++i) {
            if (load_acquire(mine) != 0u) {
                done = true;
                break;
            }
        }
        if (done) {
            *mine = 0u;
        } else {
            ok_shared = 0;
            atomicOr(error, 1u);
        }
    }
    __syncthreads();
    return ok_shared != 0;
}

__device__ __forceinline__ float4 multimem_ld_reduce_add(const float* addr) {
    float4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void multimem_st(float* addr, const float4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

// Each thread walks its vectors of the rank's slice in rounds of NVLS_UNROLL, software-pipelined:
// the multimem loads of round k+1 are issued before the multicast stores of round k, so this GPU's
// outbound NVLink traffic (the switch gathering every copy for the reductions) overlaps its inbound
// traffic (the switch delivering other ranks' reduced slices) instead of running as two phases.
__global__ void __launch_bounds__(NVLS_THREADS) nvls_sum_kernel(int64_t n, float* mc, uint32_t* const* pads, int rank,
                                                                int world, uint32_t* error) {
    if (*reinterpret_cast<volatile uint32_t*>(error) != 0u) return;  // an earlier call failed: stay off
    if (!rank_barrier(pads, rank, world, 0, error)) return;
    const int64_t slice = n / world;  // multiple of 4 floats by contract
    const int64_t v0 = (int64_t)rank * slice / 4, vn = slice / 4;
    const int64_t stride = (int64_t)gridDim.x * NVLS_THREADS;
    constexpr int U = NVLS_UNROLL;  // independent multimem loads in flight per thread
    int64_t i = (int64_t)blockIdx.x * NVLS_THREADS + threadIdx.x;
    float4 cur[U];
    bool have[U];
    #pragma unroll
    for (int u = 0; u < U; ++u) {
        have[u] = i + u * stride < vn;
        if (have[u]) cur[u] = multimem_ld_reduce_add(mc + 4 * (v0 + i + u * stride));
    }
    for (; i < vn; i += U * stride) {
        const int64_t nx = i + U * stride;
        float4 nxt[U];
        bool nhave[U];
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            nhave[u] = nx + u * stride < vn;
            if (nhave[u]) nxt[u] = multimem_ld_reduce_add(mc + 4 * (v0 + nx + u * stride));
        }
        #pragma unroll
        for (int u = 0; u < U; ++u)
            if (have[u]) multimem_st(mc + 4 * (v0 + i + u * stride), cur[u]);
        #pragma unroll
        for (int u = 0; u < U; ++u) {
            cur[u] = nxt[u];
            have[u] = nhave[u];
        }
    }
    __syncthreads();
    rank_barrier(pads, rank, world, 1, error);
}

}  // namespace pbg

using namespace pbg;

extern "C" {

// Signal-pad bytes one CTA needs per rank of the group (two barrier phases).
int64_t pbg_nvls_signal_bytes(void) { return (int64_t)2 * NVLS_MAX_WORLD * sizeof(uint32_t); }

int pbg_nvls_allreduce_sum_f32_grid(int64_t n, void* multicast, const void* signal_pads, int64_t pad_bytes,
                                    int32_t rank, int32_t world, uint32_t* error, int32_t max_ctas, void* stream) {
    PBG_REQUIRE(max_ctas >= 0, "nvls_sum: max_ctas must be >= 0 (0 = no cap)");
    PBG_REQUIRE(world >= 2 && world <= NVLS_MAX_WORLD && rank >= 0 && rank < world, "nvls_sum: bad rank/world");
    PBG_REQUIRE(n > 0 && n % (4 * world) == 0, "nvls_sum: n must be a positive multiple of 4*world");
    PBG_REQUIRE(multicast && signal_pads && error, "nvls_sum: null argument");
    PBG_REQUIRE(((uintptr_t)multicast % 16) == 0, "nvls_sum: multicast address must be 16-byte aligned");
    // as many SMs issuing multimem requests as the slice allows (one round of NVLS_UNROLL
    // float4 per thread at least), capped at one CTA per SM and by the barrier slots the pad holds
    int64_t vn = n / world / 4;
    int64_t want = (vn + (int64_t)NVLS_THREADS * NVLS_UNROLL - 1) / ((int64_t)NVLS_THREADS * NVLS_UNROLL);
    int cap = sm_count() < NVLS_MAX_BLOCKS ? sm_count() : NVLS_MAX_BLOCKS;
    int64_t fit = pad_bytes / (2 * (int64_t)world * (int64_t)sizeof(uint32_t));  // barrier slots the pad holds
    PBG_REQUIRE(fit >= 1, "nvls_sum: signal pad of %lld bytes is too small", (long long)pad_bytes);
    if (fit < cap) cap = (int)fit;
    if (max_ctas > 0 && max_ctas < cap) cap = max_ctas;  // leave SMs to concurrent work
    int blocks = (int)(want < cap ? want : cap);
    if (blocks < 1) blocks = 1;
    nvls_sum_kernel<<<blocks, NVLS_THREADS, 0, as_stream(stream)>>>(n, (float*)multicast, (uint32_t* const*)signal_pads,
                                                                    rank, world, error);
    return launch_status("nvls_allreduce_sum_f32");
}

int pbg_nvls_allreduce_sum_f32(int64_t n, void* multicast, const void* signal_pads, int64_t pad_bytes, int32_t rank,
                               int32_t world, uint32_t* error, void* stream) {
    return pbg_nvls_allreduce_sum_f32_grid(n, multicast, signal_pads, pad_bytes, rank, world, error, 0, stream);
}

}  // extern "C"
