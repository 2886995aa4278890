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

namespace pbg {

// ---------------------------------------------------------------------------
// Closed-form composite policy of one row, one thread.
//
// For one logistic component with edges z_i = (x_i - mu) / s, the tick mass
// sigma(z_{k+1}) sigma(-z_k) (1 - e^{z_k - z_{k+1}}) equals
// sigma(z_{k+1}) - sigma(z_k), so the mass of any tick range [a, b) is the
// same product form with (a, b) in place of (k, k+1):
//     R(a, b) = sigma(z_b) sigma(-z_a) (-expm1(-(x_b - x_a) / s)),
// accurate in both tails because no difference of nearly equal sigmoids is
// taken and the edge gap is computed from the edges, not from rounded z's.
// Consequences used here (policy.py:113-204 is the per-tick definition):
//   * the legal raise mass needs one R per component, not one per tick;
//   * the conditional raise probabilities rp_k over the legal ticks sum to 1
//     ((1 - iota) mix/mass + iota at the all-in tick), so the softmax
//     denominator is e^{l0} [fold legal] + e^{l1'} + e^{l2} [raise legal];
//   * the CDF at any tick is O(M), so sampling is a binary search over ticks.
// Results equal the per-tick composition up to rounding.
struct ClosedPolicy {
    static constexpr int MMAX = 8;
    float loc[MMAX], inv_s[MMAX], wnorm[MMAX];  // wnorm = omega / normaliser
    int M, T;
    LegalSummary L;
    float mass, iota, pf, pc, pr;  // fold, check/call and total raise probability
    bool raise;

    __device__ float range(int m, int a, int b) const {
        if (b <= a) return 0.0f;
        float xa = edge_of(a, T), xb = edge_of(b, T);
        float za = __fmul_rn(__fsub_rn(xa, loc[m]), inv_s[m]);
        float zb = __fmul_rn(__fsub_rn(xb, loc[m]), inv_s[m]);
        float w = -expm1f(-__fmul_rn(__fsub_rn(xb, xa), inv_s[m]));
        return fmaxf(__fmul_rn(__fmul_rn(sigmoid_f(zb), sigmoid_f(-za)), w), 0.0f);
    }

    // normalised mixture mass of ticks [a, b)
    __device__ float mix(int a, int b) const {
        float acc = 0.0f;
        for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, __fmul_rn(wnorm[m], range(m, a, b)));
        return acc;
    }

    __device__ void init(const RawRow& raw, const LegalSummary& legal, int ticks) {
        M = raw.M;
        T = ticks;
        L = legal;
        iota = raw.iota;
        raise = L.alive && L.lo <= L.hi;
        for (int m = 0; m < M; ++m) {
            loc[m] = raw.mu[m];
            inv_s[m] = __fdiv_rn(1.0f, raw.scale[m]);
            wnorm[m] = 1.0f;
            float norm = range(m, 0, T);
            wnorm[m] = __fdiv_rn(raw.omega[m], fmaxf(norm, FLT_TINY));
        }
        mass = raise ? mix(L.lo, L.hi + 1) : 0.0f;
        float l0 = raw.logits[0], l1 = L.call_legal ? raw.logits[1] : raw.logits[0], l2 = raw.logits[2];
        float mx = l1;
        if (L.call_legal) mx = fmaxf(mx, l0);
        if (raise) mx = fmaxf(mx, l2);
        float ef = L.call_legal ? expf(__fsub_rn(l0, mx)) : 0.0f;
        float ec = expf(__fsub_rn(l1, mx));
        float er = raise ? expf(__fsub_rn(l2, mx)) : 0.0f;
        float d = __fadd_rn(__fadd_rn(ef, ec), er);
        pf = __fdiv_rn(ef, d);
        pc = __fdiv_rn(ec, d);
        pr = __fdiv_rn(er, d);
    }

    // conditional raise probability of tick k (legal, lo <= k <= hi)
    __device__ float rp(int k) const {
        int count = L.hi - L.lo + 1;
        float cond = mass > 0.0f ? __fdiv_rn(mix(k, k + 1), fmaxf(mass, POLICY_EPS)) : __fdiv_rn(1.0f, (float)count);
        return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, iota), cond), k == L.hi ? iota : 0.0f);
    }

    // conditional raise probability of ticks lo..k
    __device__ float rp_cum(int k) const {
        int count = L.hi - L.lo + 1;
        float cond = mass > 0.0f ? fminf(__fdiv_rn(mix(L.lo, k + 1), fmaxf(mass, POLICY_EPS)), 1.0f)
                                 : __fdiv_rn((float)(k - L.lo + 1), (float)count);
        return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, iota), cond), k == L.hi ? iota : 0.0f);
    }

    // probability of event e (legal by contract)
    __device__ float prob(int e) const {
        if (e == 0) return L.call_legal ? pf : 0.0f;
        if (e == 1) return pc;
        int k = e - 2;
        if (!raise || k < L.lo || k > L.hi) return 0.0f;
        float r = rp(k);
        return r > 0.0f ? __fmul_rn(pr, fmaxf(r, POLICY_EPS)) : 0.0f;
    }

    // inverse-CDF draw at uniform u over the event order fold, call, ticks
    // (rollout.py:237-267): first event whose cumulative probability reaches
    // min(u * total, nextafter(total, 0)); a threshold beyond the last
    // legal event (rounding) takes the last legal event.
    __device__ int sample(float u) const {
        float total = __fadd_rn(__fadd_rn(L.call_legal ? pf : 0.0f, pc), pr);
        float thr = __fmul_rn(u, total);
        float cap = nextafterf(total, 0.0f);
        thr = thr < cap ? thr : cap;
        float c0 = L.call_legal ? pf : 0.0f;
        if (L.call_legal && c0 >= thr) return 0;
        float c1 = __fadd_rn(c0, pc);
        if (c1 >= thr || !raise) return 1;
        int lo = L.lo, hi = L.hi;
        if (__fadd_rn(c1, __fmul_rn(pr, rp_cum(hi))) < thr) return hi + 2;
        while (lo < hi) {  // smallest k with c1 + pr * rp_cum(k) >= thr
            int mid = (lo + hi) >> 1;
            if (__fadd_rn(c1, __fmul_rn(pr, rp_cum(mid))) >= thr) hi = mid;
            else lo = mid + 1;
        }
        return lo + 2;
    }
};

}  // namespace pbg
