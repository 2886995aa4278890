// Warp-cooperative composite poker policy (one policy row per warp).
//
// Restates pbg/games/poker/queued/policy.py:113-204 (probabilities with
// _discretized_logistic): a discretised-logistic raise mixture over the tick
// grid, an all-in atom on the highest legal tick, and a masked softmax over
// [fold, check/call, raise ticks].  Events are split across lanes in
// contiguous chunks of C = ceil(E/32) so that the CDF needed by sampling is
// a lane-local prefix plus one warp scan.  fp32 throughout; the library's
// own transcendental functions (expf, expm1f, logf) are used as-is.
#pragma once

#include "pbg_common.cuh"

namespace pbg {

constexpr int CHUNK_MAX = 9;  // E <= 288
constexpr float POLICY_EPS = 1.0e-12f;
constexpr float FLT_TINY = 1.17549435e-38f;

// torch.linspace(0, 1, T+1)[i] in fp32 (two-sided formula).
__device__ __forceinline__ float edge_of(int i, int T) {
    float step = __fdiv_rn(1.0f, (float)T);
    int half = (T + 1) / 2;
    return i < half ? __fmul_rn((float)i, step) : __fsub_rn(1.0f, __fmul_rn(step, (float)(T - i)));
}

__device__ __forceinline__ float sigmoid_f(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}

// One mixture component of the discretised logistic over T ticks: edges
// x_i = linspace(0, 1, T+1)[i], z_i = (x_i - mu) / s.  Tick k has mass
// sigma(z_{k+1}) * sigma(-z_k) * (-expm1(z_k - z_{k+1})); the edges are equally
// spaced, so the last factor is one constant per component, and each edge's
// sigmoid pair costs one exponential and one reciprocal:
//   sigma(z) = 1 / (1 + e^{-z}),  sigma(-z) = e^{-z} sigma(z)  (1 when e^{-z} overflows).
// The normaliser sigma(z_T) sigma(-z_0) (-expm1(z_0 - z_T)) keeps the
// reference's form.
struct MixtureEdges {
    float loc, inv_scale, width, inv_norm;
};

__device__ __forceinline__ MixtureEdges mixture_edges(float loc, float sc, int T) {
    MixtureEdges m;
    m.loc = loc;
    m.inv_scale = __fdiv_rn(1.0f, sc);
    float z0 = __fdiv_rn(__fsub_rn(0.0f, loc), sc);
    float zT = __fdiv_rn(__fsub_rn(edge_of(T, T), loc), sc);
    float norm = __fmul_rn(__fmul_rn(sigmoid_f(zT), sigmoid_f(-z0)), -expm1f(__fsub_rn(z0, zT)));
    m.inv_norm = __fdiv_rn(1.0f, fmaxf(norm, FLT_TINY));
    m.width = -expm1f(-__fmul_rn(__fdiv_rn(1.0f, (float)T), m.inv_scale));
    return m;
}

__device__ __forceinline__ void edge_sigmoids(const MixtureEdges& m, int i, int T, float& sig, float& sm) {
    float z = __fmul_rn(__fsub_rn(edge_of(i, T), m.loc), m.inv_scale);
    float ex = expf(-z);
    sig = __fdividef(1.0f, __fadd_rn(1.0f, ex));
    sm = isinf(ex) ? 1.0f : __fmul_rn(ex, sig);
}

// Legal-event sources ------------------------------------------------------
struct MaskRow {           // a materialised [E] uint8 row
    const uint8_t* m;
    __device__ bool operator()(int e) const { return m[e] != 0; }
};

struct LegalSummary {      // compact legality: call bit + contiguous raise ticks
    bool alive, call_legal;
    int lo, hi;            // legal raise ticks [lo, hi]; lo > hi when none
    __device__ bool operator()(int e) const {
        if (!alive) return false;
        if (e == 0) return call_legal;
        if (e == 1) return true;
        int k = e - 2;
        return k >= lo && k <= hi;
    }
};

struct RawRow {
    const float* logits;  // [3]
    const float* omega;   // [M]
    const float* mu;
    const float* scale;
    float iota;
    int M;
};

__device__ __forceinline__ RawRow raw_row(const pbg_policy& pol, int64_t row) {
    RawRow r;
    r.M = pol.mixtures;
    r.logits = pol.type_logits + row * 3;
    r.omega = pol.omega + row * pol.mixtures;
    r.mu = pol.mu + row * pol.mixtures;
    r.scale = pol.scale + row * pol.mixtures;
    r.iota = pol.iota[row];
    return r;
}

// Probabilities of one row: lane holds events [lane*C, lane*C + C).
// Returns the sum of probabilities (the categorical "mass").
template <class Legal>
__device__ float warp_policy_row(const RawRow& raw, const Legal& legal, int T, int E, int C,
                                 float (&p)[CHUNK_MAX]) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * C;
    float mix[CHUNK_MAX];
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) mix[j] = 0.0f;
    for (int m = 0; m < raw.M; ++m) {
        MixtureEdges mx_m = mixture_edges(raw.mu[m], raw.scale[m], T);
        float tick[CHUNK_MAX];
        float part = 0.0f;
        // ticks of this lane's chunk: tick k needs sigma(-z_k) and sigma(z_{k+1})
        const int k0 = e0 - 2;
        float sig_unused, sm_prev;
        edge_sigmoids(mx_m, k0 > 0 ? k0 : 0, T, sig_unused, sm_prev);
        #pragma unroll
        for (int j = 0; j < CHUNK_MAX; ++j) {
            tick[j] = 0.0f;
            int e = e0 + j;
            int k = e - 2;
            if (j < C && k >= 0 && e < E) {
                float sig_next, sm_next;
                edge_sigmoids(mx_m, k + 1, T, sig_next, sm_next);
                float v = fmaxf(__fmul_rn(__fmul_rn(sig_next, sm_prev), mx_m.width), 0.0f);
                tick[j] = __fmul_rn(v, mx_m.inv_norm);
                part = __fadd_rn(part, tick[j]);
                sm_prev = sm_next;
            }
        }
        float total = fmaxf(warp_sum(part), FLT_TINY);
        float om = raw.omega[m];
        #pragma unroll
        for (int j = 0; j < CHUNK_MAX; ++j)
            mix[j] = __fadd_rn(mix[j], __fmul_rn(om, __fdiv_rn(tick[j], total)));
    }
    // mask the mixture, legal raise count, mass and all-in tick
    float part_mass = 0.0f;
    int part_count = 0, part_top = -1;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        bool ok = j < C && e >= 2 && e < E && legal(e);
        if (!ok) mix[j] = 0.0f;
        else {
            part_mass = __fadd_rn(part_mass, mix[j]);
            ++part_count;
            part_top = e - 2;
        }
    }
    float mass = warp_sum(part_mass);
    int count = __reduce_add_sync(0xffffffffu, part_count);
    int all_in = warp_max_int(part_top);
    float io = raw.iota;
    bool facing = legal(0);
    float l0 = raw.logits[0], l1 = raw.logits[1], l2 = raw.logits[2];
    float full[CHUNK_MAX];
    float mx = -INFINITY;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        full[j] = -INFINITY;
        if (j < C && e < E && legal(e)) {
            if (e == 0) full[j] = l0;
            else if (e == 1) full[j] = facing ? l1 : l0;
            else {
                float cond = mass > 0.0f ? __fdiv_rn(mix[j], fmaxf(mass, POLICY_EPS))
                                         : __fdiv_rn(1.0f, (float)max(count, 1));
                float atom = (e - 2) == all_in ? 1.0f : 0.0f;
                float rp = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, io), cond), __fmul_rn(io, atom));
                full[j] = rp > 0.0f ? __fadd_rn(l2, logf(fmaxf(rp, POLICY_EPS))) : -INFINITY;
            }
            mx = fmaxf(mx, full[j]);
        }
    }
    mx = warp_max(mx);
    float part_sum = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        p[j] = (j < C && e < E && legal(e)) ? expf(__fsub_rn(full[j], mx)) : 0.0f;
        part_sum = __fadd_rn(part_sum, p[j]);
    }
    float denom = warp_sum(part_sum);
    float part_p = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        if (j < C && e < E && legal(e)) p[j] = __fdiv_rn(p[j], denom);
        else p[j] = 0.0f;
        part_p = __fadd_rn(part_p, p[j]);
    }
    return warp_sum(part_p);
}

// Inverse-CDF sampling over the chunked row: first event whose inclusive
// prefix reaches min(u*mass, nextafter(mass, 0)); clamped to E-1.
__device__ __forceinline__ int warp_sample(const float (&p)[CHUNK_MAX], int E, int C, float mass,
                                           int64_t key) {
    const int lane = threadIdx.x & 31;
    float thr = __fmul_rn(key_uniform(key), mass);
    float cap = nextafterf(mass, 0.0f);
    thr = thr < cap ? thr : cap;
    float chunk = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) chunk = __fadd_rn(chunk, p[j]);
    // exclusive warp scan of chunk sums in lane order
    float incl = chunk;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __fadd_rn(v, incl);
    }
    float prev = __shfl_up_sync(0xffffffffu, incl, 1);
    float cdf = lane > 0 ? prev : 0.0f;
    int found = 0x7fffffff;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = lane * C + j;
        if (j < C && e < E) {
            cdf = __fadd_rn(cdf, p[j]);
            if (cdf >= thr && e < found) found = e;
        }
    }
    found = warp_min_int(found);
    return found >= E ? E - 1 : found;
}

// Value of p at event e (held by lane e / C), broadcast to the warp.
__device__ __forceinline__ float warp_fetch(const float (&p)[CHUNK_MAX], int e, int C) {
    const int lane = threadIdx.x & 31;
    float mine = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j)
        if (lane * C + j == e) mine = p[j];
    return __shfl_sync(0xffffffffu, mine, e / C);
}

}  // namespace pbg
