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
// are skipped, as in the reference.  Every sum runs in the reference's order
// (children in edge order, siblings summed directly, never total minus
// child), so results are bit-identical with -fmad=false.
//
// B200 mapping.  The pass is a chain of dependent loads per node (node
// record -> edges -> children's rows), so the design minimises round trips
// and instructions per node rather than bytes.  A node has p_train*width
// independent (p, d) items, often fewer than 32, so a node gets a GROUP of G
// lanes (G = the power of two covering p_train*max_width, capped at 32; 32/G
// nodes per warp).  Each CTA keeps every output partition's arena pointers,
// capacity and width in shared memory.  Loads go out in three waves: the node
// record; then the lane failure word, the head rows and the target edges
// (staged in shared memory as the child row's arena offset, one edge per
// lane); then every child's work values of each lane's items and, for
// branched trees, every child's trace, cost term and delta, all independent.
// Mass, moment, per-action values and sibling sums then read shared memory.
// Nodes with more than TGT_MAX_CHILDREN target children read global memory
// directly.
// Layers are separated by a bounded grid barrier (the launch is cooperative,
// so every CTA is resident and the barrier completes); there is none before
// the first layer or after the last.  The failure codes live in a persistent
// workspace that every call leaves clean; the CTA that finishes last turns
// them into failure_min.  A barrier wait that runs out makes failure_min -2
// in every lane.
#include <climits>

#include "pbg_common.cuh"

namespace pbg {

constexpr int TGT_THREADS = 256;
constexpr int TGT_WARPS = TGT_THREADS / 32;
constexpr int TGT_MAX_CHILDREN = 8;  // target children staged in shared memory per node
constexpr int TGT_MAX_PARTS = 16;    // output partitions cached in shared memory
constexpr uint32_t TGT_WAIT_TRIES = 1u << 24;  // with a 64 ns back-off: seconds, far above any layer

// One output partition's arenas and strides.
struct TargetPart {
    float *w0, *w1, *trace, *cost, *delta;
    int cap, width;
};

struct TargetArgs {
    const int32_t* layer_ptr;
    int layers;
    pbg_target_nodes nd;
    pbg_target_children ch;
    pbg_target_tables t;
    int n_replica, input_count, output_count, action_partitions, p_train, max_width;
    int group;                    // lanes per node (power of two, <= 32)
    int warp_bytes;               // shared staging bytes per warp
    int off_part, off_value, off_tail;  // byte offsets inside a warp's staging area
    float lambda;
    bool sampled, branched;
    int32_t* failure_min;  // output
    uint32_t* ws;          // persistent workspace (layout below)
};

// Workspace words (zero before the first call; every completed call leaves
// the counters at zero again):  [0] grid-barrier arrivals, [32] barrier
// generation, [64] CTAs finished, [65] barrier timeout flag, [96 + lane]
// the lane's failure code (0 = none, else INT_MAX - first failing node, kept
// with atomicMax so the smallest node wins).
constexpr int WS_ARRIVE = 0, WS_GEN = 32, WS_DONE = 64, WS_TIMEOUT = 65, WS_FAIL = 96;

__device__ __forceinline__ float* table_ptr(const int64_t* table, int index) {
    return reinterpret_cast<float*>(table[index]);
}

__device__ __forceinline__ int arena_of(int encoded) { return encoded < 0 ? 1 : 0; }
__device__ __forceinline__ int row_of(int encoded) { return encoded < 0 ? -encoded - 1 : encoded; }

// arena offset of an encoded row of a lane: (lane*cap + row)*2 + arena
__device__ __forceinline__ int64_t row_offset(const TargetPart& P, int lane, int encoded) {
    return ((int64_t)lane * P.cap + row_of(encoded)) * 2 + arena_of(encoded);
}

// component d of the node's partition `dst` from a child (offset `off`) in partition `src`;
// work[((off*p_train + p)*width + d]
__device__ __forceinline__ float child_value(const TargetPart* parts, const int32_t* conversion, int output_count,
                                             int max_width, int p_train, bool second, int src, int dst, int64_t off,
                                             int p, int d) {
    const TargetPart& S = parts[src];
    const float* base = second ? S.w1 : S.w0;
    if (!base) return 0.0f;
    const float* row = base + (off * p_train + p) * S.width;
    if (src == dst) return row[d];
    const int32_t* map = conversion + ((int64_t)src * output_count + dst) * max_width;
    float total = 0.0f;
    for (int h = 0; h < S.width; ++h)
        if (map[h] == d) total += row[h];
    return total;
}

__device__ __forceinline__ bool bad_rb(float mass, float moment) {
    return !isfinite(moment) || mass < 0.0f || (mass == 0.0f && fabsf(moment) > 1.0e-7f);
}

__device__ __forceinline__ uint32_t load_acquire_gpu(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

// One node on one lane group.  `gl` is the lane's index in the group, `leader`
// the warp lane of the group's first lane, `gmask` the group's lanes; `wsm`
// the warp's staging area.
__device__ void target_node(const TargetArgs& A, const TargetPart* parts, unsigned char* wsm, int node, int arena,
                            int gl, int leader, unsigned gmask) {
    const int G = A.group;
    const int me = leader + gl;
    const int gi = leader / G;  // group index inside the warp
    const int P = A.p_train;
    // wave 1: the node record
    const int lane = A.nd.replica[node];
    const int begin = A.nd.child_begin[node];
    const int ntgt = A.nd.target_degree[node];
    const int output = A.nd.output_type[node];
    const int input = A.nd.input_type[node];
    const int owner = A.nd.owner_slot[node];
    const int dest = A.nd.destination_row[node];
    const int head_row = A.nd.sigma_head_row[node];
    const TargetPart& O = parts[output];
    const int width = O.width;
    const bool sampled = A.sampled;
    const bool staged = ntgt <= TGT_MAX_CHILDREN;
    int64_t* eoff = reinterpret_cast<int64_t*>(wsm) + gi * TGT_MAX_CHILDREN;
    int32_t* epart = reinterpret_cast<int32_t*>(wsm + A.off_part) + gi * TGT_MAX_CHILDREN;
    // wave 2: lane failure word, edges, head rows
    int failed = 0;
    if (gl == 0) failed = __ldcg(reinterpret_cast<const int32_t*>(A.ws + WS_FAIL) + lane) != 0;
    if (staged) {
        for (int a = gl; a < ntgt; a += G) {
            const int src = A.ch.source_type[begin + a];
            eoff[a] = row_offset(parts[src], lane, A.ch.source_row[begin + a]);
            epart[a] = src;
        }
    }
    // the first owner item (p = owner) this lane handles, and its head value, fetched now
    int d_pref = -1;
    if (input >= 0 && owner >= 0 && owner < P) {
        const int base = owner * width;
        const int first = base + (((gl - base) % G) + G) % G;
        if (first < base + width) d_pref = first - base;
    }
    const float* head_v = input >= 0 ? table_ptr(A.t.head_v, input) + ((int64_t)lane * A.t.head_cap[input] + head_row) * width
                                     : nullptr;
    float old_v_pref = 0.0f;
    if (d_pref >= 0) old_v_pref = head_v[d_pref];
    float old_t = 0.0f, old_c = 0.0f;
    if (A.branched && input >= 0 && gl == 0) {
        const int64_t hidx = (int64_t)lane * A.t.head_cap[input] + head_row;
        old_t = table_ptr(A.t.head_t, input)[hidx];
        old_c = table_ptr(A.t.head_c, input)[hidx];
    }
    if (__shfl_sync(gmask, failed, leader)) return;
    __syncwarp(gmask);
    auto off_of_edge = [&](int a) -> int64_t {
        return staged ? eoff[a] : row_offset(parts[A.ch.source_type[begin + a]], lane, A.ch.source_row[begin + a]);
    };
    auto part_of_edge = [&](int a) { return staged ? epart[a] : A.ch.source_type[begin + a]; };
    // wave 3a (branched): the group fetches every child's trace, cost term and delta
    float* tv = reinterpret_cast<float*>(wsm + A.off_tail) + gi * (P + 2) * TGT_MAX_CHILDREN;
    float* cterm = tv + P * ntgt;
    float* dterm = cterm + ntgt;
    const bool fits = A.branched && staged;
    if (fits) {
        for (int k = gl; k < P * ntgt; k += G) {
            const int p = k / ntgt, a = k - p * ntgt;
            tv[k] = parts[epart[a]].trace[eoff[a] * P + p];
        }
        for (int a = gl; a < ntgt; a += G) {
            const TargetPart& S = parts[epart[a]];
            cterm[a] = (float)A.ch.path[begin + a] + A.ch.multiplier[begin + a] * (S.cost ? S.cost[eoff[a]] : 0.0f);
            dterm[a] = S.delta ? S.delta[eoff[a]] : 0.0f;
        }
    }
    // wave 3b: each lane's children values of its items, then the item's targets
    float* v0 = reinterpret_cast<float*>(wsm + A.off_value) + me * 2 * TGT_MAX_CHILDREN;
    float* v1 = v0 + TGT_MAX_CHILDREN;
    const int32_t* conv = A.t.conversion;
    const int oc = A.output_count, mw = A.max_width;
    bool bad = false;
    for (int linear = gl; linear < P * width; linear += G) {
        const int p = linear / width, d = linear - p * width;
        if (staged) {
            // independent loads: every child's value of this item in flight at once
            for (int a = 0; a < ntgt; ++a) {
                v0[a] = child_value(parts, conv, oc, mw, P, false, epart[a], output, eoff[a], p, d);
                if (!sampled) v1[a] = child_value(parts, conv, oc, mw, P, true, epart[a], output, eoff[a], p, d);
            }
        }
        auto c0_of = [&](int a) {
            return staged ? v0[a] : child_value(parts, conv, oc, mw, P, false, part_of_edge(a), output, off_of_edge(a), p, d);
        };
        auto c1_of = [&](int a) {
            return staged ? v1[a] : child_value(parts, conv, oc, mw, P, true, part_of_edge(a), output, off_of_edge(a), p, d);
        };
        float mass_sum = 0.0f, moment_sum = 0.0f;
        for (int a = 0; a < ntgt; ++a) {
            const float c0 = c0_of(a);
            mass_sum += c0;
            if (!sampled) {
                const float c1 = c1_of(a);
                moment_sum += c1;
                if (bad_rb(c0, c1)) bad = true;
            }
            if (!isfinite(c0)) bad = true;
        }
        float parent0 = mass_sum / (float)ntgt;
        float parent1 = sampled ? 0.0f : moment_sum / (float)ntgt;
        if (p == owner && input >= 0) {
            const float old_v = d == d_pref ? old_v_pref : head_v[d];
            const float sigma = sampled ? parent0 : (parent0 > 0.0f ? parent1 / parent0 : 0.0f);
            table_ptr(A.t.sigma_v, lane * A.input_count + input)[(int64_t)A.nd.sigma_target_row[node] * width + d] = sigma;
            const int part = A.branched ? output : input;
            float* adv = table_ptr(A.t.action_a, lane * A.action_partitions + part);
            float* post = sampled ? nullptr : table_ptr(A.t.action_p, lane * A.action_partitions + part);
            const int64_t action_begin = A.nd.action_begin[node];
            for (int a = 0; a < ntgt; ++a) {
                const float c0 = ntgt == 1 ? mass_sum : c0_of(a);
                const float c1 = sampled ? 0.0f : (ntgt == 1 ? moment_sum : c1_of(a));
                float baseline = old_v;
                if (ntgt > 1) {
                    float s0 = 0.0f, s1 = 0.0f;
                    for (int sib = 0; sib < ntgt; ++sib) {
                        if (sib == a) continue;
                        s0 += c0_of(sib);
                        if (!sampled) s1 += c1_of(sib);
                    }
                    const float cont = sampled ? s0 / (float)(ntgt - 1) : (s0 > 0.0f ? s1 / s0 : 0.0f);
                    baseline = A.lambda * cont + (1.0f - A.lambda) * old_v;
                }
                const float q = sampled ? c0 : (c0 > 0.0f ? c1 / c0 : 0.0f);
                const int64_t row = action_begin + a;
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
        const int64_t widx = ((((int64_t)lane * O.cap + dest) * 2 + arena) * P + p) * width + d;
        if (O.w0) O.w0[widx] = parent0;
        if (!sampled && O.w1) O.w1[widx] = parent1;
    }
    if (A.branched) {
        __syncwarp(gmask);  // the tail rows are complete
        if (gl == 0) {
            float delta_bar = 0.0f, cost_raw = 0.0f;
            for (int a = 0; a < ntgt; ++a) {
                if (fits) {
                    delta_bar += dterm[a];
                    cost_raw += cterm[a];
                } else {
                    const TargetPart& S = parts[part_of_edge(a)];
                    const int64_t off = off_of_edge(a);
                    delta_bar += S.delta ? S.delta[off] : 0.0f;
                    cost_raw += (float)A.ch.path[begin + a] + A.ch.multiplier[begin + a] * (S.cost ? S.cost[off] : 0.0f);
                }
            }
            delta_bar /= (float)ntgt;
            cost_raw /= (float)ntgt;
            auto trace_of = [&](int p, int a) {
                return fits ? tv[p * ntgt + a] : parts[part_of_edge(a)].trace[off_of_edge(a) * P + p];
            };
            float trace_exec = 0.0f;
            const int64_t dst_off = ((int64_t)lane * O.cap + dest) * 2 + arena;
            for (int p = 0; p < P; ++p) {
                float mean = 0.0f;
                for (int a = 0; a < ntgt; ++a) mean += trace_of(p, a);
                mean /= (float)ntgt;
                O.trace[dst_off * P + p] = mean;
                if (ntgt > 1) {
                    for (int a = 0; a < ntgt; ++a) {
                        const float v = trace_of(p, a);
                        trace_exec += (v - mean) * (v - mean);
                    }
                }
            }
            if (ntgt > 1) trace_exec /= (float)(ntgt - 1);
            float prop_delta = delta_bar / (float)ntgt;
            float prop_cost = cost_raw;
            if (input >= 0) {
                const float trace_hat = ntgt > 1 ? fmaxf(0.0f, trace_exec - delta_bar) : 0.0f;
                const float t_star = ntgt > 1 ? trace_hat : old_t;
                prop_delta = (t_star + delta_bar) / (float)ntgt - t_star / (float)A.nd.nominal_degree[node];
                prop_cost = A.lambda * cost_raw + (1.0f - A.lambda) * old_c;
                table_ptr(A.t.sigma_t, lane * A.input_count + input)[A.nd.sigma_target_row[node]] = trace_hat;
                table_ptr(A.t.sigma_c, lane * A.input_count + input)[A.nd.sigma_target_row[node]] = cost_raw;
            }
            if (O.cost) O.cost[dst_off] = prop_cost;
            if (O.delta) O.delta[dst_off] = prop_delta;
            if (!isfinite(trace_exec) || !isfinite(prop_cost) || !isfinite(prop_delta)) bad = true;
        }
    }
    if (__any_sync(gmask, bad) && gl == 0) atomicMax(reinterpret_cast<int32_t*>(A.ws + WS_FAIL) + lane, INT_MAX - node);
    __syncwarp(gmask);  // the staging rows are reused by the group's next node
}

// Generation-counting grid barrier; false when the bounded wait ran out.
// Release: every thread's writes are ordered before thread 0's fence and
// arrival (CTA barrier, then a gpu-scope fence); acquire: thread 0 sees the
// new generation, fences, and the CTA barrier passes that on, so the plain
// loads of the next layer observe every write of the previous one.
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

// No barrier before the first layer (the failure codes are clean on entry)
// and none after the last: the CTA that finishes last publishes failure_min
// and clears the failure codes for the next call.
__global__ void __launch_bounds__(TGT_THREADS, 3) layered_targets_kernel(TargetArgs A) {
    extern __shared__ __align__(16) unsigned char tgt_smem_raw[];
    __shared__ TargetPart parts[TGT_MAX_PARTS];
    uint32_t* count = A.ws + WS_ARRIVE;
    uint32_t* gen = A.ws + WS_GEN;
    __shared__ uint32_t my_gen_s;
    if (threadIdx.x == 0) my_gen_s = load_acquire_gpu(gen);
    for (int i = threadIdx.x; i < A.output_count; i += blockDim.x) {
        TargetPart q;
        q.w0 = A.t.work0 ? table_ptr(A.t.work0, i) : nullptr;
        q.w1 = A.t.work1 ? table_ptr(A.t.work1, i) : nullptr;
        q.trace = A.t.trace ? table_ptr(A.t.trace, i) : nullptr;
        q.cost = A.t.cost ? table_ptr(A.t.cost, i) : nullptr;
        q.delta = A.t.delta ? table_ptr(A.t.delta, i) : nullptr;
        q.cap = A.t.work_cap[i];
        q.width = A.t.width[i];
        parts[i] = q;
    }
    __syncthreads();
    {
        uint32_t my_gen = my_gen_s;
        const int G = A.group;
        const int warp_lane = threadIdx.x & 31;
        const int gl = warp_lane & (G - 1);
        const int leader = warp_lane - gl;
        const unsigned gmask = (G == 32 ? 0xffffffffu : ((1u << G) - 1u)) << leader;
        const int groups_per_warp = 32 / G;
        const int groups_total = gridDim.x * TGT_WARPS * groups_per_warp;
        const int group_global = (blockIdx.x * TGT_WARPS + (threadIdx.x >> 5)) * groups_per_warp + leader / G;
        unsigned char* wsm = tgt_smem_raw + (size_t)(threadIdx.x >> 5) * A.warp_bytes;
        for (int layer = 0; layer < A.layers; ++layer) {
            const int first = A.layer_ptr[layer], last = A.layer_ptr[layer + 1];
            for (int node = first + group_global; node < last; node += groups_total)
                target_node(A, parts, wsm, node, (layer + 1) & 1, gl, leader, gmask);
            if (layer + 1 < A.layers && !grid_barrier(count, gen, my_gen)) {
                if (threadIdx.x == 0) atomicExch(A.ws + WS_TIMEOUT, 1u);
                break;
            }
        }
    }
    // epilogue: the last CTA to finish publishes the result and clears the codes
    __shared__ int last_cta;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last_cta = atomicAdd(A.ws + WS_DONE, 1u) == gridDim.x - 1;
        if (last_cta) __threadfence();
    }
    __syncthreads();
    if (last_cta) {
        // every other CTA has finished: plain accesses, spread over the CTA
        const bool timed_out = __ldcg(A.ws + WS_TIMEOUT) != 0u;
        int32_t* codes = reinterpret_cast<int32_t*>(A.ws + WS_FAIL);
        for (int l = threadIdx.x; l < A.n_replica; l += blockDim.x) {
            const int32_t code = __ldcg(codes + l);
            A.failure_min[l] = timed_out ? -2 : (code ? INT_MAX - code : INT_MAX);
            codes[l] = 0;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            A.ws[WS_TIMEOUT] = 0u;
            A.ws[WS_DONE] = 0u;
        }
    }
}

}  // namespace pbg

using namespace pbg;

static int align16(int x) { return (x + 15) & ~15; }
static constexpr int TGT_SMEM_CEILING = 200 * 1024;

extern "C" int64_t pbg_layered_targets_workspace_words(int32_t n_replica) {
    return n_replica < 0 ? -1 : (int64_t)WS_FAIL + n_replica;
}

extern "C" int pbg_layered_targets(const int32_t* layer_ptr, int32_t layers, pbg_target_nodes nodes,
                                   pbg_target_children children, pbg_target_tables tables, int32_t n_replica,
                                   int32_t input_count, int32_t output_count, int32_t action_partition_count,
                                   int32_t p_train, int32_t max_width, float lambda, int32_t sampled, int32_t branched,
                                   int32_t* failure_min, uint32_t* workspace, void* stream) {
    PBG_REQUIRE(layers >= 0 && layer_ptr && failure_min && workspace && n_replica >= 1,
                "layered_targets: bad arguments");
    PBG_REQUIRE(p_train >= 1 && output_count >= 1 && input_count >= 0 && max_width >= 1,
                "layered_targets: bad partition counts");
    PBG_REQUIRE(output_count <= TGT_MAX_PARTS, "layered_targets: at most %d output partitions", TGT_MAX_PARTS);
    PBG_REQUIRE(tables.work_cap && tables.width && tables.conversion, "layered_targets: missing table");
    PBG_REQUIRE(lambda >= 0.0f && lambda <= 1.0f, "layered_targets: lambda must be in [0,1]");
    int items = p_train * max_width;
    int group = 1;
    while (group < items && group < 32) group *= 2;
    const int gpw = 32 / group;
    // a warp's staging area: edge offsets, edge partitions, value rows, branched tails
    const int off_part = align16(gpw * TGT_MAX_CHILDREN * (int)sizeof(int64_t));
    const int off_value = off_part + align16(gpw * TGT_MAX_CHILDREN * (int)sizeof(int32_t));
    const int off_tail = off_value + align16(32 * 2 * TGT_MAX_CHILDREN * (int)sizeof(float));
    const int warp_bytes = off_tail + align16(gpw * (p_train + 2) * TGT_MAX_CHILDREN * (int)sizeof(float));
    const int smem = TGT_WARPS * warp_bytes;
    PBG_REQUIRE(smem <= TGT_SMEM_CEILING, "layered_targets: p_train %d needs too much staging memory", p_train);
    // occupancy per (device, staging size); the attribute calls run once per size
    static int cached_dev[8] = {-1, -1, -1, -1, -1, -1, -1, -1}, cached_smem[8], cached_blocks[8];
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = 0;
    for (int i = 0; i < 8; ++i)
        if (cached_dev[i] == dev && cached_smem[i] == smem) per_sm = cached_blocks[i];
    if (per_sm == 0) {
        int rc = cuda_status(cudaFuncSetAttribute(layered_targets_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                  100),
                             "layered_targets: carveout");
        if (!rc)  // the ceiling every staging size below stays under
            rc = cuda_status(cudaFuncSetAttribute(layered_targets_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  TGT_SMEM_CEILING),
                             "layered_targets: shared memory size");
        int n = 0;
        if (!rc)
            rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, layered_targets_kernel, TGT_THREADS, smem),
                             "layered_targets: occupancy");
        if (rc) return rc;
        per_sm = n > 0 ? n : 1;
        for (int i = 0; i < 8; ++i)
            if (cached_dev[i] < 0 || i == 7) {
                cached_dev[i] = dev; cached_smem[i] = smem; cached_blocks[i] = per_sm;
                break;
            }
    }
    // co-resident grid (a cooperative launch refuses more)
    int grid = sm_count() * per_sm;
    TargetArgs A;
    A.layer_ptr = layer_ptr; A.layers = layers; A.nd = nodes; A.ch = children; A.t = tables;
    A.n_replica = n_replica; A.input_count = input_count; A.output_count = output_count;
    A.action_partitions = action_partition_count; A.p_train = p_train; A.max_width = max_width;
    A.group = group; A.warp_bytes = warp_bytes; A.off_part = off_part; A.off_value = off_value; A.off_tail = off_tail;
    A.lambda = lambda; A.sampled = sampled != 0; A.branched = branched != 0;
    A.failure_min = failure_min; A.ws = workspace;
    void* args[] = {&A};
    return cuda_status(cudaLaunchCooperativeKernel((const void*)layered_targets_kernel, dim3(grid), dim3(TGT_THREADS),
                                                   args, (size_t)smem, as_stream(stream)),
                       "layered_targets: cooperative launch");
}
