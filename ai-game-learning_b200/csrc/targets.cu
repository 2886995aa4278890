// Layered lambda-return targets over a topology forest, all layers in one
// cooperative launch (pbg/core/csrc/layered_targets.cu:117-411 computes the
// same quantities with one launch per layer and one 256-thread block per
// node).
//
// Per node (reverse layer order, children already final):
//   * mass / moment of each (player p, component d): the mean over the
//     node's target children of their work values, converted from the
//     child's output partition to the node's (conversion table sums the
//     source components that map to d);
//   * at the owner's seat: the sigma value target, one advantage per target
//     child (child value minus a baseline that mixes the siblings'
//     continuation with the old value head by lambda), and the lambda-mixed
//     value written back to the work arena;
//   * branched trees: trace / cost / delta scalars of the trace head.
// Validity checks (finite values, non-negative masses) record the first
// failing node of each lane with atomicMin, and later nodes of a failed lane
// are skipped, as in the reference.
//
// B200 mapping: one warp per node, lanes over (p, d); a grid-strided warp
// loop over the layer's nodes; a bounded grid barrier between layers (the
// launch is cooperative, so every CTA is resident and the barrier completes).
// A barrier that does not complete within its bound writes -2 into every
// lane's failure word and the kernel returns.
#include <climits>

#include "pbg_common.cuh"

namespace pbg {

constexpr int TGT_THREADS = 256;
constexpr uint32_t TGT_WAIT_TRIES = 1u << 24;  // with a 64 ns back-off: seconds, far above any layer

struct TargetArgs {
    const int32_t* layer_ptr;
    int layers;
    pbg_target_nodes nd;
    pbg_target_children ch;
    pbg_target_tables t;
    int n_replica, input_count, output_count, action_partitions, p_train, max_width;
    float lambda;
    bool sampled, branched;
    int32_t* failure_min;
    uint32_t* sync;
};

__device__ __forceinline__ float* table_ptr(const int64_t* table, int index) {
    return reinterpret_cast<float*>(table[index]);
}

__device__ __forceinline__ int arena_of(int encoded) { return encoded < 0 ? 1 : 0; }
__device__ __forceinline__ int row_of(int encoded) { return encoded < 0 ? -encoded - 1 : encoded; }

// work[(((lane*cap + row)*2 + arena)*p_train + p)*width + d]
__device__ __forceinline__ float work_at(const TargetArgs& A, const int64_t* table, int part, int lane, int encoded,
                                         int p, int d) {
    if (!table) return 0.0f;
    const int64_t idx = ((((int64_t)lane * A.t.work_cap[part] + row_of(encoded)) * 2 + arena_of(encoded)) * A.p_train + p) *
                            A.t.width[part] + d;
    return __ldcg(table_ptr(table, part) + idx);
}

// value of component d of the node's partition `dst` from a child in partition `src`
__device__ __forceinline__ float child_value(const TargetArgs& A, const int64_t* table, int src, int dst, int lane,
                                             int encoded, int p, int d) {
    if (src == dst) return work_at(A, table, src, lane, encoded, p, d);
    const int32_t* map = A.t.conversion + ((int64_t)src * A.output_count + dst) * A.max_width;
    float total = 0.0f;
    for (int h = 0; h < A.t.width[src]; ++h)
        if (map[h] == d) total += work_at(A, table, src, lane, encoded, p, h);
    return total;
}

__device__ __forceinline__ float scalar_at(const TargetArgs& A, const int64_t* table, int part, int lane, int encoded) {
    if (!table) return 0.0f;
    return __ldcg(table_ptr(table, part) + ((int64_t)lane * A.t.work_cap[part] + row_of(encoded)) * 2 + arena_of(encoded));
}

__device__ __forceinline__ float trace_at(const TargetArgs& A, int part, int lane, int encoded, int p) {
    return __ldcg(table_ptr(A.t.trace, part) +
                  (((int64_t)lane * A.t.work_cap[part] + row_of(encoded)) * 2 + arena_of(encoded)) * A.p_train + p);
}

__device__ __forceinline__ bool bad_rb(float mass, float moment) {
    return !isfinite(moment) || mass < 0.0f || (mass == 0.0f && fabsf(moment) > 1.0e-7f);
}

// One node on one warp.
__device__ void target_node(const TargetArgs& A, int node, int arena) {
    const int lane_id = threadIdx.x & 31;
    const int lane = A.nd.replica[node];
    if (__ldcg(A.failure_min + lane) != INT_MAX) return;
    const int begin = A.nd.child_begin[node];
    const int ntgt = A.nd.target_degree[node];
    const int output = A.nd.output_type[node];
    const int input = A.nd.input_type[node];
    const int owner = A.nd.owner_slot[node];
    const int width = A.t.width[output];
    const int dest = A.nd.destination_row[node];
    const int cap = A.t.work_cap[output];
    const bool sampled = A.sampled;
    bool bad = false;
    for (int linear = lane_id; linear < A.p_train * width; linear += 32) {
        const int p = linear / width, d = linear % width;
        float mass_sum = 0.0f, moment_sum = 0.0f;
        for (int a = 0; a < ntgt; ++a) {
            const int e = begin + a;
            const float c0 = child_value(A, A.t.work0, A.ch.source_type[e], output, lane, A.ch.source_row[e], p, d);
            mass_sum += c0;
            if (!sampled) {
                const float c1 = child_value(A, A.t.work1, A.ch.source_type[e], output, lane, A.ch.source_row[e], p, d);
                moment_sum += c1;
                if (bad_rb(c0, c1)) bad = true;
            }
            if (!isfinite(c0)) bad = true;
        }
        float parent0 = mass_sum / (float)ntgt;
        float parent1 = sampled ? 0.0f : moment_sum / (float)ntgt;
        if (p == owner && input >= 0) {
            const float old_v = table_ptr(A.t.head_v, input)[((int64_t)lane * A.t.head_cap[input] + A.nd.sigma_head_row[node]) * width + d];
            const float sigma = sampled ? parent0 : (parent0 > 0.0f ? parent1 / parent0 : 0.0f);
            table_ptr(A.t.sigma_v, lane * A.input_count + input)[(int64_t)A.nd.sigma_target_row[node] * width + d] = sigma;
            const int part = A.branched ? output : input;
            float* adv = table_ptr(A.t.action_a, lane * A.action_partitions + part);
            float* post = sampled ? nullptr : table_ptr(A.t.action_p, lane * A.action_partitions + part);
            for (int a = 0; a < ntgt; ++a) {
                const int e = begin + a;
                const float c0 = ntgt == 1 ? mass_sum
                                           : child_value(A, A.t.work0, A.ch.source_type[e], output, lane, A.ch.source_row[e], p, d);
                const float c1 = sampled ? 0.0f
                                         : (ntgt == 1 ? moment_sum
                                                      : child_value(A, A.t.work1, A.ch.source_type[e], output, lane,
                                                                    A.ch.source_row[e], p, d));
                float baseline = old_v;
                if (ntgt > 1) {
                    float s0 = 0.0f, s1 = 0.0f;
                    for (int sib = 0; sib < ntgt; ++sib) {
                        if (sib == a) continue;
                        const int se = begin + sib;
                        s0 += child_value(A, A.t.work0, A.ch.source_type[se], output, lane, A.ch.source_row[se], p, d);
                        if (!sampled)
                            s1 += child_value(A, A.t.work1, A.ch.source_type[se], output, lane, A.ch.source_row[se], p, d);
                    }
                    const float cont = sampled ? s0 / (float)(ntgt - 1) : (s0 > 0.0f ? s1 / s0 : 0.0f);
                    baseline = A.lambda * cont + (1.0f - A.lambda) * old_v;
                }
                const float q = sampled ? c0 : (c0 > 0.0f ? c1 / c0 : 0.0f);
                const int64_t row = A.nd.action_begin[node] + a;
                adv[row * width + d] = q - baseline;
                if (post) post[row * width + d] = c0;
                if (!isfinite(q) || !isfinite(baseline) ||
                    (!sampled && (c0 < 0.0f || (c0 == 0.0f && fabsf(c1) > 1.0e-7f))))
                    bad = true;
            }
            if (sampled) parent0 = A.lambda * parent0 + (1.0f - A.lambda) * old_v;
            else parent1 = A.lambda * parent1 + (1.0f - A.lambda) * parent0 * old_v;
        }
        if (!isfinite(parent0) || (!sampled && bad_rb(parent0, parent1))) bad = true;
        const int64_t widx = ((((int64_t)lane * cap + dest) * 2 + arena) * A.p_train + p) * width + d;
        if (A.t.work0) table_ptr(A.t.work0, output)[widx] = parent0;
        if (!sampled && A.t.work1) table_ptr(A.t.work1, output)[widx] = parent1;
    }
    if (A.branched && lane_id == 0) {
        float delta_bar = 0.0f, cost_raw = 0.0f;
        for (int a = 0; a < ntgt; ++a) {
            const int e = begin + a;
            delta_bar += scalar_at(A, A.t.delta, A.ch.source_type[e], lane, A.ch.source_row[e]);
            cost_raw += (float)A.ch.path[e] + A.ch.multiplier[e] * scalar_at(A, A.t.cost, A.ch.source_type[e], lane, A.ch.source_row[e]);
        }
        delta_bar /= (float)ntgt;
        cost_raw /= (float)ntgt;
        float trace_exec = 0.0f;
        for (int p = 0; p < A.p_train; ++p) {
            float mean = 0.0f;
            for (int a = 0; a < ntgt; ++a) {
                const int e = begin + a;
                const int src = A.ch.source_type[e], enc = A.ch.source_row[e];
                mean += trace_at(A, src, lane, enc, p);
            }
            mean /= (float)ntgt;
            table_ptr(A.t.trace, output)[(((int64_t)lane * cap + dest) * 2 + arena) * A.p_train + p] = mean;
            if (ntgt > 1) {
                for (int a = 0; a < ntgt; ++a) {
                    const int e = begin + a;
                    const int src = A.ch.source_type[e], enc = A.ch.source_row[e];
                    const float v = trace_at(A, src, lane, enc, p);
                    trace_exec += (v - mean) * (v - mean);
                }
            }
        }
        if (ntgt > 1) trace_exec /= (float)(ntgt - 1);
        float prop_delta = delta_bar / (float)ntgt;
        float prop_cost = cost_raw;
        if (input >= 0) {
            const int64_t hidx = (int64_t)lane * A.t.head_cap[input] + A.nd.sigma_head_row[node];
            const float old_t = table_ptr(A.t.head_t, input)[hidx];
            const float old_c = table_ptr(A.t.head_c, input)[hidx];
            const float trace_hat = ntgt > 1 ? fmaxf(0.0f, trace_exec - delta_bar) : 0.0f;
            const float t_star = ntgt > 1 ? trace_hat : old_t;
            prop_delta = (t_star + delta_bar) / (float)ntgt - t_star / (float)A.nd.nominal_degree[node];
            prop_cost = A.lambda * cost_raw + (1.0f - A.lambda) * old_c;
            table_ptr(A.t.sigma_t, lane * A.input_count + input)[A.nd.sigma_target_row[node]] = trace_hat;
            table_ptr(A.t.sigma_c, lane * A.input_count + input)[A.nd.sigma_target_row[node]] = cost_raw;
        }
        const int64_t sidx = ((int64_t)lane * cap + dest) * 2 + arena;
        if (A.t.cost) table_ptr(A.t.cost, output)[sidx] = prop_cost;
        if (A.t.delta) table_ptr(A.t.delta, output)[sidx] = prop_delta;
        if (!isfinite(trace_exec) || !isfinite(prop_cost) || !isfinite(prop_delta)) bad = true;
    }
    if (__any_sync(0xffffffffu, bad) && lane_id == 0) atomicMin(A.failure_min + lane, node);
}

__device__ __forceinline__ uint32_t load_acquire_gpu(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// Generation-counting grid barrier; false when the bounded wait ran out.
__device__ bool grid_barrier(uint32_t* count, uint32_t* gen, uint32_t& my_gen) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ok = 1;
        const uint32_t g = my_gen;
        __threadfence();
        if (atomicAdd(count, 1u) == gridDim.x - 1) {
            atomicExch(count, 0u);
            __threadfence();
            atomicAdd(gen, 1u);
        } else {
            uint32_t i = 0;
            while (load_acquire_gpu(gen) == g) {
                if (++i >= TGT_WAIT_TRIES) {
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        my_gen = g + 1;
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

__global__ void __launch_bounds__(TGT_THREADS) layered_targets_kernel(TargetArgs A) {
    uint32_t* count = A.sync;
    uint32_t* gen = A.sync + 1;
    __shared__ uint32_t my_gen_s;
    if (threadIdx.x == 0) my_gen_s = atomicAdd(gen, 0u);
    // the lane failure words start clean; visible to all CTAs after the first barrier
    if (blockIdx.x == 0)
        for (int l = threadIdx.x; l < A.n_replica; l += blockDim.x) A.failure_min[l] = INT_MAX;
    __syncthreads();
    uint32_t my_gen = my_gen_s;
    if (!grid_barrier(count, gen, my_gen)) goto timeout;
    {
        const int warps_total = gridDim.x * (TGT_THREADS / 32);
        const int warp_global = blockIdx.x * (TGT_THREADS / 32) + (threadIdx.x >> 5);
        for (int layer = 0; layer < A.layers; ++layer) {
            const int first = A.layer_ptr[layer], last = A.layer_ptr[layer + 1];
            for (int node = first + warp_global; node < last; node += warps_total) target_node(A, node, (layer + 1) & 1);
            if (!grid_barrier(count, gen, my_gen)) goto timeout;
        }
    }
    return;
timeout:
    if (threadIdx.x == 0)
        for (int l = 0; l < A.n_replica; ++l) atomicExch(A.failure_min + l, -2);
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_layered_targets(const int32_t* layer_ptr, int32_t layers, pbg_target_nodes nodes,
                                   pbg_target_children children, pbg_target_tables tables, int32_t n_replica,
                                   int32_t input_count, int32_t output_count, int32_t action_partition_count,
                                   int32_t p_train, int32_t max_width, float lambda, int32_t sampled, int32_t branched,
                                   int32_t* failure_min, uint32_t* sync, void* stream) {
    PBG_REQUIRE(layers >= 0 && layer_ptr && failure_min && sync && n_replica >= 1, "layered_targets: bad arguments");
    PBG_REQUIRE(p_train >= 1 && output_count >= 1 && input_count >= 0 && max_width >= 1,
                "layered_targets: bad partition counts");
    PBG_REQUIRE(tables.work_cap && tables.width && tables.conversion, "layered_targets: missing table");
    PBG_REQUIRE(lambda >= 0.0f && lambda <= 1.0f, "layered_targets: lambda must be in [0,1]");
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int slot = dev >= 0 && dev < 64 ? dev : 0;
    if (per_sm[slot] == 0) {
        int n = 0;
        int rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, layered_targets_kernel, TGT_THREADS, 0),
                             "layered_targets: occupancy");
        if (rc) return rc;
        per_sm[slot] = n > 0 ? n : 1;
    }
    // co-resident grid (a cooperative launch refuses more)
    int grid = sm_count() * (per_sm[slot] < 4 ? per_sm[slot] : 4);
    TargetArgs A;
    A.layer_ptr = layer_ptr; A.layers = layers; A.nd = nodes; A.ch = children; A.t = tables;
    A.n_replica = n_replica; A.input_count = input_count; A.output_count = output_count;
    A.action_partitions = action_partition_count; A.p_train = p_train; A.max_width = max_width;
    A.lambda = lambda; A.sampled = sampled != 0; A.branched = branched != 0;
    A.failure_min = failure_min; A.sync = sync;
    void* args[] = {&A};
    return cuda_status(cudaLaunchCooperativeKernel((const void*)layered_targets_kernel, dim3(grid), dim3(TGT_THREADS),
                                                   args, 0, as_stream(stream)),
                       "layered_targets: cooperative launch");
}
