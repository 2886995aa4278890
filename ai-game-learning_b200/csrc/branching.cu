// Branched learner sampling metadata (pbg/core/csrc/alias_table.cu and
// pbg/core/csrc/branching_metadata.cu run these as single-thread launches).
//
// Walker alias table (Vose's two-stack construction, float64):
//   The reference pushes every index onto a "small" (scaled < 1) or "large"
//   stack in index order, then pops one of each until a stack empties: the
//   small index gets probability = its scaled value and alias = the large
//   index, the large index loses 1 - that value and goes back onto the small
//   or the large stack.  Because both stacks are LIFO, the only element that
//   ever moves between them is the large just popped, and it is popped again
//   at once: it is the "current large" (still >= 1, back on the large stack)
//   or the "pending small" (dropped below 1).  Every other element is read
//   once, in stack order, with its original value.  So:
//     1. alias_classify / alias_scatter (parallel): probability = 1,
//        alias = index, and an order-preserving partition of the indices into
//        the two stacks, each entry stored with its original scaled value;
//     2. alias_pair_kernel (one warp running one scalar loop): the pairing
//        loop with the moving element held in registers, reading the two
//        stacks from their tops through shared-memory windows, writing
//        probability / alias of each small.
//   The arithmetic (scaled[high] -= 1 - p_low, compared with 1.0) and the
//   pop order are the reference's, so the table is identical.
//
// Decision log mass: log_mass[node] = log_mass[parent] - logf(degree[parent])
// along parent links that always point to a smaller index.  A thread per node
// walks its ancestors and sums root-down in the same fp32 order as the
// reference's sequential loop, so every value is identical; the first failing
// node in index order (parent >= node: code 1; a parent of degree <= 0:
// code 2) sets *failure, as the reference's loop does before it stops.
#include <climits>

#include "pbg_common.cuh"

namespace pbg {

constexpr int BR_THREADS = 256;

// ------------------------------------------------------------ alias table

__global__ void alias_classify_kernel(int64_t n, const double* __restrict__ scaled, double* __restrict__ probability,
                                      int32_t* __restrict__ alias, int32_t* __restrict__ block_small) {
    __shared__ int count;
    if (threadIdx.x == 0) count = 0;
    __syncthreads();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    bool small = false;
    if (i < n) {
        probability[i] = 1.0;
        alias[i] = (int32_t)i;
        small = scaled[i] < 1.0;
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, small);
    if ((threadIdx.x & 31) == 0) atomicAdd(&count, __popc(ballot));
    __syncthreads();
    if (threadIdx.x == 0) block_small[blockIdx.x] = count;
}

// exclusive prefix of per-block small counts (one block; blocks <= 1024 * chunk)
__global__ void alias_block_scan_kernel(int blocks, int32_t* __restrict__ block_small, int64_t* __restrict__ totals) {
    __shared__ int64_t carry;
    __shared__ int64_t warp_sums[32];
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < blocks; base += blockDim.x) {
        const int i = base + threadIdx.x;
        int64_t v = i < blocks ? block_small[i] : 0;
        int64_t x = v;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int64_t w = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            warp_sums[lane] = w;
        }
        __syncthreads();
        const int64_t inclusive = x + (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
        if (i < blocks) block_small[i] = (int32_t)(inclusive - v);
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = inclusive;
        __syncthreads();
    }
    if (threadIdx.x == 0) totals[0] = carry;
}

// Stack entries: values in `vals` (small stack at [0, ns), large stack at
// [ns, n)), indices in `idx` (same positions), both in index order.
__global__ void alias_scatter_kernel(int64_t n, const double* __restrict__ scaled,
                                     const int32_t* __restrict__ block_small, const int64_t* __restrict__ totals,
                                     double* __restrict__ vals, int32_t* __restrict__ idx) {
    __shared__ int warp_counts[BR_THREADS / 32];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool small = i < n && scaled[i] < 1.0;
    const unsigned ballot = __ballot_sync(0xffffffffu, small);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_counts[warp] = __popc(ballot);
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += warp_counts[w];
    const int64_t small_before = (int64_t)block_small[blockIdx.x] + before + __popc(ballot & ((1u << lane) - 1u));
    if (i < n) {
        const int64_t ns = totals[0];
        const int64_t pos = small ? small_before : ns + (i - small_before);
        vals[pos] = scaled[i];
        idx[pos] = (int32_t)i;
    }
}

// One warp.  Every lane runs the same scalar pairing loop on the same data (so
// control flow is uniform); the next stack entries come from shared-memory
// windows that the whole warp refills with coalesced loads when a stack's
// top leaves its window; lane 0 writes the results.
constexpr int ALIAS_WINDOW = 1024;

__global__ void __launch_bounds__(32) alias_pair_kernel(int64_t n, const int64_t* __restrict__ totals,
                                                        const double* __restrict__ vals,
                                                        const int32_t* __restrict__ idx, double* __restrict__ scaled,
                                                        double* __restrict__ probability, int32_t* __restrict__ alias) {
    // whole static stacks staged through shared memory in windows; the loop below is the
    // reference's pop order written as: a large H absorbs smalls (static ones, top first)
    // until it drops below 1 or the smalls run out; a large that drops below 1 is itself the
    // next small, absorbed by the next static large.
    __shared__ double small_val[ALIAS_WINDOW], large_val[ALIAS_WINDOW];
    __shared__ int32_t small_idx[ALIAS_WINDOW], large_idx[ALIAS_WINDOW];
    const int lane = threadIdx.x;
    const int64_t ns = totals[0];
    int64_t ss = ns, sl = n - ns;  // static entries not yet consumed (tops at ss-1, sl-1)
    int64_t s_lo = ss, l_lo = sl;  // window starts
    auto small_at = [&](int64_t k, int32_t& id, double& v) {  // k < ss, reads through the window
        if (k < s_lo) {
            s_lo = k + 1 > ALIAS_WINDOW ? k + 1 - ALIAS_WINDOW : 0;
            __syncwarp();
            for (int64_t q = s_lo + lane; q <= k; q += 32) {
                small_val[q - s_lo] = vals[q];
                small_idx[q - s_lo] = idx[q];
            }
            __syncwarp();
        }
        id = small_idx[k - s_lo];
        v = small_val[k - s_lo];
    };
    auto large_at = [&](int64_t k, int32_t& id, double& v) {
        if (k < l_lo) {
            l_lo = k + 1 > ALIAS_WINDOW ? k + 1 - ALIAS_WINDOW : 0;
            __syncwarp();
            for (int64_t q = l_lo + lane; q <= k; q += 32) {
                large_val[q - l_lo] = vals[ns + q];
                large_idx[q - l_lo] = idx[ns + q];
            }
            __syncwarp();
        }
        id = large_idx[k - l_lo];
        v = large_val[k - l_lo];
    };
    // step k's result is held by lane k % 32 and written by the whole warp every 32 steps
    uint32_t step = 0;
    int32_t held_low = -1, held_alias = 0;
    double held_prob = 0.0;
    bool held_scaled = false;
    auto emit = [&](int32_t low, double p, int32_t high, bool converted) {
        if ((int)(step & 31u) == lane) {
            held_low = low;
            held_prob = p;
            held_alias = high;
            held_scaled = converted;  // a converted large keeps its final value in scaled[]
        }
        if ((++step & 31u) == 0) {
            if (held_low >= 0) {
                probability[held_low] = held_prob;
                alias[held_low] = held_alias;
                if (held_scaled) scaled[held_low] = held_prob;
            }
            held_low = -1;
        }
    };
    bool pending = false;  // a converted large waiting to be popped as the next small
    int32_t p_idx = 0;
    double p_val = 0.0;
    int32_t h_idx = 0;
    double h_val = 0.0;
    bool have_h = false;
    while (true) {
        if (!have_h) {  // pop the next large
            if (sl == 0) break;
            --sl;
            large_at(sl, h_idx, h_val);
            have_h = true;
        }
        if (pending) {  // the converted large is the small popped first
            if (sl == 0 && !have_h) break;
            emit(p_idx, p_val, h_idx, true);
            h_val -= 1.0 - p_val;
            pending = false;
            if (h_val < 1.0) {
                pending = true;
                p_idx = h_idx;
                p_val = h_val;
                have_h = false;
                continue;
            }
        }
        // absorb static smalls into H until it drops below 1 or they run out
        if (ss == 0) break;
        int32_t s_id;
        double s_v;
        small_at(ss - 1, s_id, s_v);
        bool dropped = false;
        while (true) {
            --ss;
            int32_t next_id = 0;
            double next_v = 0.0;
            if (ss > 0) small_at(ss - 1, next_id, next_v);  // fetched before it is needed
            emit(s_id, s_v, h_idx, false);
            h_val -= 1.0 - s_v;
            if (h_val < 1.0) {
                dropped = true;
                break;
            }
            if (ss == 0) break;
            s_id = next_id;
            s_v = next_v;
        }
        if (dropped) {
            pending = true;
            p_idx = h_idx;
            p_val = h_val;
            have_h = false;
        } else {
            break;  // smalls exhausted with H still >= 1
        }
    }
    // flush the held results of the last partial group
    if (held_low >= 0) {
        probability[held_low] = held_prob;
        alias[held_low] = held_alias;
        if (held_scaled) scaled[held_low] = held_prob;
    }
    // the element left over keeps its final value in scaled[]
    if (lane == 0) {
        if (pending) scaled[p_idx] = p_val;
        else if (have_h) scaled[h_idx] = h_val;
    }
}

// ------------------------------------------------------ decision log mass

__global__ void decision_log_mass_kernel(int64_t n, const int32_t* __restrict__ parent,
                                         const int32_t* __restrict__ degree, float* __restrict__ log_mass,
                                         unsigned long long* __restrict__ first_failure) {
    const int64_t node = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (node >= n) return;
    const int32_t ancestor = parent[node];
    if (ancestor >= node) {
        atomicMin(first_failure, ((unsigned long long)node << 2) | 1ull);
        return;
    }
    if (ancestor < 0) {
        log_mass[node] = 0.0f;
        return;
    }
    if (degree[ancestor] <= 0) {
        atomicMin(first_failure, ((unsigned long long)node << 2) | 2ull);
        return;
    }
    // ancestors nearest first; sum root-down as the sequential loop does
    constexpr int DEPTH = 64;
    float terms[DEPTH];
    int depth = 0;
    int64_t at = node;
    bool deep = false;
    while (true) {
        const int32_t p = parent[at];
        if (p < 0 || p >= at) break;  // root reached (or an invalid link, reported at its own node)
        if (depth == DEPTH) {
            deep = true;
            break;
        }
        terms[depth++] = logf((float)degree[p]);
        at = p;
    }
    float value = 0.0f;
    if (!deep) {
        for (int k = depth - 1; k >= 0; --k) value = value - terms[k];
    } else {
        // deeper than the local buffer: count the path, then subtract from the root down
        int64_t length = 0;
        for (int64_t a = node; parent[a] >= 0 && parent[a] < a; a = parent[a]) ++length;
        for (int64_t k = length - 1; k >= 0; --k) {
            int64_t a = node;
            for (int64_t s = 0; s < k; ++s) a = parent[a];
            value = value - logf((float)degree[parent[a]]);
        }
    }
    log_mass[node] = value;
}

__global__ void failure_finish_kernel(const unsigned long long* __restrict__ first_failure, int32_t* failure) {
    const unsigned long long v = *first_failure;
    if (v != ~0ull) *failure = (int32_t)(v & 3ull);
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_alias_workspace_bytes(int64_t n) {
    if (n <= 0) return -1;
    const int64_t blocks = (n + BR_THREADS - 1) / BR_THREADS;
    return 8 * n + 4 * n + 4 * blocks + 16 + 64;
}

int pbg_alias_table(int64_t n, double* scaled, double* probability, int32_t* alias, void* workspace, void* stream) {
    PBG_REQUIRE(n > 0 && n <= INT32_MAX, "alias_table: size must be in [1, 2^31)");
    PBG_REQUIRE(scaled && probability && alias && workspace, "alias_table: null pointer");
    PBG_REQUIRE(((uintptr_t)workspace % 16) == 0, "alias_table: workspace must be 16-byte aligned");
    cudaStream_t s = as_stream(stream);
    const int64_t blocks = (n + BR_THREADS - 1) / BR_THREADS;
    PBG_REQUIRE(blocks <= INT32_MAX, "alias_table: too many blocks");
    unsigned char* w = static_cast<unsigned char*>(workspace);
    double* vals = reinterpret_cast<double*>(w);
    int32_t* idx = reinterpret_cast<int32_t*>(w + 8 * n);
    int32_t* block_small = reinterpret_cast<int32_t*>(w + 12 * n);
    int64_t* totals = reinterpret_cast<int64_t*>(w + ((12 * n + 4 * blocks + 15) & ~(int64_t)15));
    alias_classify_kernel<<<(unsigned)blocks, BR_THREADS, 0, s>>>(n, scaled, probability, alias, block_small);
    alias_block_scan_kernel<<<1, 1024, 0, s>>>((int)blocks, block_small, totals);
    alias_scatter_kernel<<<(unsigned)blocks, BR_THREADS, 0, s>>>(n, scaled, block_small, totals, vals, idx);
    alias_pair_kernel<<<1, 32, 0, s>>>(n, totals, vals, idx, scaled, probability, alias);
    return launch_status("alias_table");
}

int pbg_decision_log_mass(int64_t n, const int32_t* parent, const int32_t* degree, float* log_mass, int32_t* failure,
                          void* workspace, void* stream) {
    PBG_REQUIRE(n >= 0, "decision_log_mass: bad size");
    PBG_REQUIRE(failure && workspace && (n == 0 || (parent && degree && log_mass)), "decision_log_mass: null pointer");
    cudaStream_t s = as_stream(stream);
    unsigned long long* first = static_cast<unsigned long long*>(workspace);
    int rc = cuda_status(cudaMemsetAsync(first, 0xff, sizeof(unsigned long long), s), "decision_log_mass: init");
    if (rc) return rc;
    if (n > 0)
        decision_log_mass_kernel<<<(unsigned)((n + BR_THREADS - 1) / BR_THREADS), BR_THREADS, 0, s>>>(
            n, parent, degree, log_mass, first);
    failure_finish_kernel<<<1, 1, 0, s>>>(first, failure);
    return launch_status("decision_log_mass");
}

}  // extern "C"
