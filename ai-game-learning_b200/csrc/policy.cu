// Composite poker policy entry points (warp per policy row).
// policy.py:113-204 (probabilities), :206-233 (selected_log_pi),
// :235-244 (policy_reductions entropy), :246-282 (sample_actor).
#include "pbg_common.cuh"
#include "policy.cuh"

namespace pbg {

enum PolicyMode { PROBS = 0, SELECTED = 1, ENTROPY = 2, SAMPLE = 3 };

template <int MODE>
__global__ void __launch_bounds__(256) policy_kernel(int64_t B, int E, pbg_policy pol, const uint8_t* mask,
                                                     const int32_t* action, const int32_t* hand,
                                                     const int64_t* keys, float* out, int32_t* out_action) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int C = (E + 31) / 32;
    const int T = E - 2;
    const int64_t rows = MODE == SAMPLE ? B : B * pol.rows;
    for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        int64_t b = MODE == SAMPLE ? r : r / pol.rows;
        int64_t prow = MODE == SAMPLE ? (b * pol.rows + (pol.rows > 1 ? hand[b] : 0)) : r;
        MaskRow legal{mask + b * E};
        RawRow raw = raw_row(pol, prow);
        float p[CHUNK_MAX];
        float mass = warp_policy_row(raw, legal, T, E, C, p);
        if (MODE == PROBS) {
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j) {
                int e = lane * C + j;
                if (j < C && e < E) out[r * E + e] = p[j];
            }
        } else if (MODE == SELECTED) {
            float v = warp_fetch(p, action[b], C);
            if (lane == 0) out[r] = logf(fmaxf(v, POLICY_EPS));
        } else if (MODE == ENTROPY) {
            float part = 0.0f;
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j) {
                int e = lane * C + j;
                if (j < C && e < E) part = __fadd_rn(part, __fmul_rn(p[j], logf(fmaxf(p[j], POLICY_EPS))));
            }
            float s = warp_sum(part);
            if (lane == 0) out[r] = -s;
        } else {
            int act = warp_sample(p, E, C, mass, keys[b]);
            float v = warp_fetch(p, act, C);
            if (lane == 0) {
                out_action[b] = act;
                out[b] = logf(fmaxf(v, POLICY_EPS));
            }
        }
    }
}

static int check_policy(int64_t B, int32_t E, const pbg_policy& pol, const uint8_t* mask) {
    PBG_REQUIRE(B >= 0 && E > RAISE_OFFSET && E <= 32 * CHUNK_MAX && mask, "policy: bad shape or mask");
    PBG_REQUIRE(pol.type_logits && pol.omega && pol.mu && pol.scale && pol.iota, "policy: null field");
    PBG_REQUIRE(pol.rows >= 1 && pol.mixtures >= 1 && pol.mixtures <= 8, "policy: rows >= 1, mixtures in [1,8]");
    return PBG_OK;
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int pbg_policy_probabilities(int64_t B, int32_t E, pbg_policy pol, const uint8_t* mask, float* out, void* stream) {
    int rc = check_policy(B, E, pol, mask);
    if (rc) return rc;
    PBG_REQUIRE(out, "policy_probabilities: null output");
    if (B == 0) return PBG_OK;
    policy_kernel<PROBS><<<stride_grid(B * pol.rows * 32, 256), 256, 0, as_stream(stream)>>>(
        B, E, pol, mask, nullptr, nullptr, nullptr, out, nullptr);
    return launch_status("policy_probabilities");
}

int pbg_policy_selected_log_pi(int64_t B, int32_t E, pbg_policy pol, const uint8_t* mask, const int32_t* action,
                               float* out, void* stream) {
    int rc = check_policy(B, E, pol, mask);
    if (rc) return rc;
    PBG_REQUIRE(out && action, "policy_selected_log_pi: null argument");
    if (B == 0) return PBG_OK;
    policy_kernel<SELECTED><<<stride_grid(B * pol.rows * 32, 256), 256, 0, as_stream(stream)>>>(
        B, E, pol, mask, action, nullptr, nullptr, out, nullptr);
    return launch_status("policy_selected_log_pi");
}

int pbg_policy_entropy(int64_t B, int32_t E, pbg_policy pol, const uint8_t* mask, float* out, void* stream) {
    int rc = check_policy(B, E, pol, mask);
    if (rc) return rc;
    PBG_REQUIRE(out, "policy_entropy: null output");
    if (B == 0) return PBG_OK;
    policy_kernel<ENTROPY><<<stride_grid(B * pol.rows * 32, 256), 256, 0, as_stream(stream)>>>(
        B, E, pol, mask, nullptr, nullptr, nullptr, out, nullptr);
    return launch_status("policy_entropy");
}

int pbg_policy_sample_actor(int64_t B, int32_t E, pbg_policy pol, const uint8_t* mask, const int32_t* hand,
                            const int64_t* keys, int32_t* action, float* selected_log, void* stream) {
    int rc = check_policy(B, E, pol, mask);
    if (rc) return rc;
    PBG_REQUIRE(keys && action && selected_log && (hand || pol.rows == 1), "policy_sample_actor: null argument");
    if (B == 0) return PBG_OK;
    policy_kernel<SAMPLE><<<stride_grid(B * 32, 256), 256, 0, as_stream(stream)>>>(
        B, E, pol, mask, nullptr, hand, keys, selected_log, action);
    return launch_status("policy_sample_actor");
}

}  // extern "C"
