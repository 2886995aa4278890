// Fused poker learner objective: the composite policy forward, the loss of
// one physical learner batch and its gradient with respect to the raw policy
// fields, the value and the public heads, in one pass over the policy rows.
//
// Reference: pbg/core/learner.py:1824-2159 (LearnerOperation.forward_loss)
// with the poker policy operation pbg/games/poker/queued/policy.py:113-298
// (probabilities, selected_log_pi, policy_reductions, learner), followed by
// the backward of (total * objective_weight * loss_scale).sum()
// (pbg/core/training.py:403).  Autograd's conventions at the non-smooth points
// are kept: clamp / clamp_min pass the gradient on the closed interval,
// torch.minimum / maximum split a tie evenly, torch.where routes it to the
// selected branch, masked_fill blocks it.
//
// Layout.  Sigma rows s = 0..S-1 carry the model's raw fields over W columns
// (W = 1: the sampled private row; W = H: every private hand, Rao-Blackwell):
// policy row r = s*W + c.  Action rows i = action_ptr[s] .. action_ptr[s+1]-1
// belong to sigma row s (unit spans for sequential batches), each with an
// event id and [W] old log pi, advantage and posterior.
//
// Work split.  One warp per policy row: lanes hold contiguous chunks of the E
// events (as in policy.cuh).  The warp evaluates the row's probabilities once
// (and the reference row's, for KL), walks the row's action span to form the
// PPO terms and the gradient of each selected log-probability, adds the
// entropy and KL gradients, and runs the composite backward: masked softmax,
// the all-in atom and the conditional raise law, the mixture weights, and per
// component the discretised logistic back to (mu, s).  The tick mass is
// sigma(z_{k+1}) sigma(-z_k) (1 - e^{z_k - z_{k+1}}) = sigma(z_{k+1}) - sigma(z_k),
// so its exact derivative with respect to an interior edge is
// (dc_{k-1} - dc_k) sigma'(z_k): one product per edge, free of the
// cancellation between the two product-rule terms that autograd forms.
//
// Statistics are accumulated per (warp, lane of the batch) in double in
// shared memory, reduced per block in warp order and across blocks by the last
// block to arrive: each statistic strided over several of its threads (block
// b to thread b mod groups, in block order), then those threads in order
// (deterministic for a given grid).
#include <type_traits>

#include "pbg_common.cuh"
#include "policy.cuh"

namespace pbg {

constexpr int PL_THREADS = 256;
constexpr int PL_WARPS = PL_THREADS / 32;
constexpr int PL_MAX_LANES = 16;
// per-lane statistics: sums, then maxima
enum { ST_POLICY, ST_VALUE, ST_ENTROPY, ST_REFERENCE, ST_APPROX, ST_CLIP, ST_CAP, ST_TRACE, ST_COST, PL_SUMS };
constexpr int PL_STATS = PL_SUMS + 2;  // + negative log-ratio max, negative influence max
constexpr int PL_RESULT = 10;          // LossResult fields (learner.py:1739-1749)
constexpr int PL_MAX_BLOCKS = 2048;    // grid cap: sizes the statistics workspace independently of the device
static_assert(PL_MAX_LANES * PL_STATS <= PL_THREADS, "the last block reduces every statistic at once");

struct LearnerArgs {
    int64_t S, A, rows;  // sigma rows, action rows, policy rows S*W
    int E, W, lanes;
    pbg_policy raw, ref;  // ref.type_logits == nullptr: no reference KL
    const uint8_t* mask;  // [S,E]
    const int64_t* action_ptr;  // [S+1] or nullptr (unit spans)
    const int32_t* action;      // [A]
    const float *old_log, *advantage, *posterior;  // [A,W]; posterior nullptr = ones
    const float *value, *old_value, *target;       // [S,W]
    const float *trace_pred, *cost_pred, *trace_target, *cost_target;  // [S] or nullptr
    const float* controls;     // [lanes,10]
    const float* lane_weight;  // [lanes]
    pbg_policy_grad grad;
    float *d_value, *d_trace, *d_cost;
    const float *inv_post, *inv_vpost;  // [A], [S] (posterior normalisers; nullptr when W == 1)
    double* partials;
    float* result;  // [lanes,10]
};

// ------------------------------------------------------------------ row math
//
// The learner's own forward of the composite policy (policy.py:113-204): the
// same operations as warp_policy_row (policy.cuh), with every per-event
// division replaced by a multiplication with a correctly rounded reciprocal
// (__frcp_rn) and the edge spacing hoisted.  Results agree with the
// rounding-for-rounding forward to a few ulp, far inside the learner's
// tolerance; the rollout keeps the exact forward for its sampled actions.
// Lanes hold CH consecutive events (CH a compile-time chunk >= ceil(E / 32)).

struct Ticks {
    int T, E, half;
    float step;  // linspace(0, 1, T + 1) spacing
};

__device__ __forceinline__ Ticks make_ticks(int E) {
    Ticks g;
    g.E = E;
    g.T = E - 2;
    g.half = (g.T + 1) / 2;
    g.step = __fdiv_rn(1.0f, (float)g.T);
    return g;
}

// torch.linspace(0, 1, T+1)[i] in fp32 (two-sided formula)
__device__ __forceinline__ float edge_at(const Ticks& g, int i) {
    return i < g.half ? __fmul_rn((float)i, g.step) : __fsub_rn(1.0f, __fmul_rn(g.step, (float)(g.T - i)));
}

// sigma(z) and sigma(-z) from one exponential: sigma(-z) = e^{-z} sigma(z) (1 when e^{-z} overflows)
__device__ __forceinline__ void sig_pair(float z, float& sig, float& sm) {
    const float ex = expf(-z);
    sig = __frcp_rn(1.0f + ex);
    sm = isinf(ex) ? 1.0f : ex * sig;
}

// Per-component constants: 1/s, the tick width factor -expm1(-(1/T)/s) and the normaliser
// sigma(z_T) sigma(-z_0) (-expm1(z_0 - z_T)).
struct Comp {
    float loc, inv_s, width, norm, inv_norm;
};

__device__ __forceinline__ Comp comp_setup(float mu, float s, const Ticks& g) {
    Comp c;
    c.loc = mu;
    c.inv_s = __frcp_rn(s);
    const float z0 = -mu * c.inv_s;
    const float zT = (edge_at(g, g.T) - mu) * c.inv_s;
    float sT, smT, s0, sm0;
    sig_pair(zT, sT, smT);
    sig_pair(z0, s0, sm0);
    c.norm = sT * sm0 * -expm1f(z0 - zT);
    c.inv_norm = __frcp_rn(fmaxf(c.norm, FLT_TINY));
    c.width = -expm1f(-g.step * c.inv_s);
    return c;
}

template <int CH>
struct RowForward {
    float p[CH];     // probabilities, 0 where illegal
    float mix[CH];   // masked mixture on raise ticks
    float cond[CH];  // conditional raise probability
    float rp[CH];    // raise probability (1 - iota) cond + iota [all-in]
    bool ok[CH];     // event legal
    float mass;
    int all_in;      // highest legal raise tick, -1 when none
    bool facing;
};

template <int CH>
__device__ __forceinline__ float chunk_fetch(const float (&x)[CH], int e) {
    const int lane = threadIdx.x & 31;
    float mine = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j)
        if (lane * CH + j == e) mine = x[j];
    return __shfl_sync(0xffffffffu, mine, (e / CH) & 31);
}

template <int CH>
__device__ void policy_forward_fast(const RawRow& raw, const MaskRow& legal, const Ticks& g, RowForward<CH>& f) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * CH;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        f.ok[j] = e < g.E && legal(e);
        f.mix[j] = 0.0f;
    }
    const int kk = e0 - 2 > 0 ? e0 - 2 : 0;
    for (int m = 0; m < raw.M; ++m) {
        const Comp c = comp_setup(raw.mu[m], raw.scale[m], g);
        float sig, sm_prev;
        sig_pair((edge_at(g, kk) - c.loc) * c.inv_s, sig, sm_prev);
        float a[CH];
        float part = 0.0f;
        #pragma unroll
        for (int j = 0; j < CH; ++j) {
            const int e = e0 + j, k = e - 2;
            a[j] = 0.0f;
            if (k >= 0 && e < g.E) {
                float sig_next, sm_next;
                sig_pair((edge_at(g, k + 1) - c.loc) * c.inv_s, sig_next, sm_next);
                a[j] = fmaxf(sig_next * sm_prev * c.width, 0.0f) * c.inv_norm;
                part += a[j];
                sm_prev = sm_next;
            }
        }
        const float coef = raw.omega[m] * __frcp_rn(fmaxf(warp_sum(part), FLT_TINY));
        #pragma unroll
        for (int j = 0; j < CH; ++j) f.mix[j] += coef * a[j];
    }
    float part_mass = 0.0f;
    int part_count = 0, part_top = -1;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        if (e >= 2 && f.ok[j]) {
            part_mass += f.mix[j];
            ++part_count;
            part_top = e - 2;
        } else {
            f.mix[j] = 0.0f;
        }
    }
    f.mass = warp_sum(part_mass);
    const int count = __reduce_add_sync(0xffffffffu, part_count);
    f.all_in = warp_max_int(part_top);
    const float inv_mass = __frcp_rn(fmaxf(f.mass, POLICY_EPS));
    const float uniform = __frcp_rn((float)max(count, 1));
    const float io = raw.iota;
    f.facing = legal(0);
    const float l0 = raw.logits[0], l1 = raw.logits[1], l2 = raw.logits[2];
    float full[CH];
    float mx = -INFINITY;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        full[j] = -INFINITY;
        f.cond[j] = 0.0f;
        f.rp[j] = 0.0f;
        if (f.ok[j]) {
            if (e == 0) full[j] = l0;
            else if (e == 1) full[j] = f.facing ? l1 : l0;
            else {
                const float cond = f.mass > 0.0f ? f.mix[j] * inv_mass : uniform;
                const float rp = (1.0f - io) * cond + (e - 2 == f.all_in ? io : 0.0f);
                f.cond[j] = cond;
                f.rp[j] = rp;
                full[j] = rp > 0.0f ? l2 + __logf(fmaxf(rp, POLICY_EPS)) : -INFINITY;
            }
            mx = fmaxf(mx, full[j]);
        }
    }
    mx = warp_max(mx);
    float part_sum = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        f.p[j] = f.ok[j] ? expf(full[j] - mx) : 0.0f;
        part_sum += f.p[j];
    }
    const float inv_denom = __frcp_rn(warp_sum(part_sum));
    #pragma unroll
    for (int j = 0; j < CH; ++j) f.p[j] *= inv_denom;
}

// Backward of one mixture component: given d(total)/d(mixture_k) on the raise
// ticks held by this lane (0 elsewhere), add d omega_m, d mu_m, d s_m.
// Recomputes the forward's tick masses a_k = v_k / max(N, tiny) and their sum.
template <int CH>
__device__ void component_backward(const RawRow& raw, int m, const Ticks& g, const float (&dmix)[CH], float& d_om,
                                   float& d_mu, float& d_s) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * CH;
    const Comp c = comp_setup(raw.mu[m], raw.scale[m], g);
    float v[CH], a[CH], dlow[CH], zlow[CH];
    float dtop = 0.0f, ztop = 0.0f;  // sigma'(z_T) and z_T on the lane holding tick T-1
    float part = 0.0f;
    const int kk = e0 - 2 > 0 ? e0 - 2 : 0;
    float z_prev = (edge_at(g, kk) - c.loc) * c.inv_s;
    float sig_prev, sm_prev;
    sig_pair(z_prev, sig_prev, sm_prev);
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        v[j] = a[j] = dlow[j] = zlow[j] = 0.0f;
        const int e = e0 + j, k = e - 2;
        if (k >= 0 && e < g.E) {
            const float z_next = (edge_at(g, k + 1) - c.loc) * c.inv_s;
            float sig_next, sm_next;
            sig_pair(z_next, sig_next, sm_next);
            v[j] = fmaxf(sig_next * sm_prev * c.width, 0.0f);
            a[j] = v[j] * c.inv_norm;
            part += a[j];
            dlow[j] = sig_prev * sm_prev;  // sigma'(z_k)
            zlow[j] = z_prev;
            if (k + 1 == g.T) {
                dtop = sig_next * sm_next;
                ztop = z_next;
            }
            z_prev = z_next;
            sig_prev = sig_next;
            sm_prev = sm_next;
        }
    }
    const float total = warp_sum(part);
    const float inv_Sc = __frcp_rn(fmaxf(total, FLT_TINY));
    const float om = raw.omega[m];
    float pom = 0.0f, pq = 0.0f;
    float ddl[CH];
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        pom += dmix[j] * a[j];
        ddl[j] = dmix[j] * om;
        pq += ddl[j] * a[j];
    }
    d_om += warp_sum(pom) * inv_Sc;
    const float Q = warp_sum(pq);
    const float qterm = total >= FLT_TINY ? Q * inv_Sc * inv_Sc : 0.0f;
    float dc[CH];
    float pn = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j, k = e - 2;
        dc[j] = 0.0f;
        if (k >= 0 && e < g.E) {
            const float da = ddl[j] * inv_Sc - qterm;
            pn += da * v[j];
            dc[j] = da * c.inv_norm;
        }
    }
    const float sn = warp_sum(pn);
    const float dN = c.norm >= FLT_TINY ? -sn * c.inv_norm * c.inv_norm : 0.0f;
    float carry = __shfl_up_sync(0xffffffffu, dc[CH - 1], 1);  // dc of the tick just before this lane's chunk
    if (lane == 0) carry = 0.0f;
    float sdz = 0.0f, szdz = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j, k = e - 2;
        if (k >= 0 && e < g.E) {
            // edge k: lower edge of tick k, upper edge of tick k-1 (no tick before tick 0)
            const float before = k == 0 ? 0.0f : carry;
            float dz = (before - dc[j]) * dlow[j];
            if (k == 0) dz -= dN * dlow[j];
            sdz += dz;
            szdz += zlow[j] * dz;
            if (k + 1 == g.T) {
                const float dzT = (dc[j] + dN) * dtop;
                sdz += dzT;
                szdz += ztop * dzT;
            }
            carry = dc[j];
        }
    }
    d_mu += -warp_sum(sdz) * c.inv_s;
    d_s += -warp_sum(szdz) * c.inv_s;
}

__device__ __forceinline__ float tie_share(float a, float b) { return a < b ? 1.0f : (a == b ? 0.5f : 0.0f); }

// dL/dp of the entropy and KL reductions (policy.py:235-244) with upstream
// gradients g_ent (d/d entropy) and g_kl (d/d KL): entropy -sum p log max(p, eps)
// gives -(log max(p, eps) + [p >= eps]); KL sum p (log max(p, eps) - log max(q, eps))
// gives log max(p, eps) - log max(q, eps) + [p >= eps].  Illegal events get 0
// (the masked fill after the softmax).
template <int CH>
__device__ __forceinline__ void add_reduction_grads(const RowForward<CH>& f, const float (&logp)[CH],
                                                    const float (*logq)[CH], float g_ent, float g_kl,
                                                    float (&gp)[CH]) {
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        if (f.ok[j]) {
            const float ind = f.p[j] >= POLICY_EPS ? 1.0f : 0.0f;
            gp[j] += -g_ent * (logp[j] + ind);
            if (logq) gp[j] += g_kl * (logp[j] - (*logq)[j] + ind);
        } else {
            gp[j] = 0.0f;
        }
    }
}

// Composite backward of one policy row: given dL/dp on the legal events (gp),
// write d type_logits, d omega, d mu, d s, d iota of row r.
template <int CH>
__device__ void policy_row_backward(const RawRow& raw, const RowForward<CH>& f, const float (&gp)[CH],
                                    const Ticks& g, const pbg_policy_grad& grad, int64_t r) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * CH;
    // masked softmax (selected logits -inf where illegal)
    float psg = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) psg += gp[j] * f.p[j];
    const float sg = warp_sum(psg);
    float dx[CH];
    float pt0 = 0.0f, pt1 = 0.0f, pt2 = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        dx[j] = f.ok[j] ? f.p[j] * (gp[j] - sg) : 0.0f;
        if (e == 0) pt0 += dx[j];
        else if (e == 1) {
            if (f.facing) pt1 += dx[j];
            else pt0 += dx[j];
        } else pt2 += dx[j];
    }
    const float dt0 = warp_sum(pt0), dt1 = warp_sum(pt1), dt2 = warp_sum(pt2);
    // raise logits l2 + log max(rp, eps) where rp > 0; rp = (1 - iota) cond + iota [all-in tick]
    const float io = raw.iota;
    float dcond[CH];
    float pio = 0.0f, pdm = 0.0f;
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        dcond[j] = 0.0f;
        if (e >= 2 && f.ok[j]) {
            const float rp = f.rp[j];
            const float drp = (rp > 0.0f && rp >= POLICY_EPS) ? dx[j] * __frcp_rn(rp) : 0.0f;
            const float atom = (e - 2) == f.all_in ? 1.0f : 0.0f;
            pio += drp * (atom - f.cond[j]);
            dcond[j] = drp * (1.0f - io);
            pdm += dcond[j] * f.mix[j];
        }
    }
    const float dio = warp_sum(pio);
    // cond = mixture / max(mass, eps) when mass > 0, else the uniform law (no gradient)
    const float mass = f.mass;
    const float inv_mc = __frcp_rn(fmaxf(mass, POLICY_EPS));
    const float sdm = warp_sum(pdm);
    const float dmass = mass >= POLICY_EPS ? -sdm * inv_mc * inv_mc : 0.0f;
    float dmix[CH];
    #pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int e = e0 + j;
        dmix[j] = (mass > 0.0f && e >= 2 && f.ok[j]) ? dcond[j] * inv_mc + dmass : 0.0f;
    }
    float* gom = grad.omega + r * raw.M;
    float* gmu = grad.mu + r * raw.M;
    float* gsc = grad.scale + r * raw.M;
    for (int m = 0; m < raw.M; ++m) {
        float dom = 0.0f, dmu = 0.0f, dsc = 0.0f;
        component_backward<CH>(raw, m, g, dmix, dom, dmu, dsc);
        if (lane == 0) {
            gom[m] = dom;
            gmu[m] = dmu;
            gsc[m] = dsc;
        }
    }
    if (lane == 0) {
        grad.type_logits[r * 3 + 0] = dt0;
        grad.type_logits[r * 3 + 1] = dt1;
        grad.type_logits[r * 3 + 2] = dt2;
        grad.iota[r] = dio;
    }
}

// probabilities only (the reference row of the KL term)
template <int CH>
__device__ __forceinline__ void policy_probs_fast(const RawRow& raw, const MaskRow& legal, const Ticks& g,
                                                  float (&q)[CH]) {
    RowForward<CH> f;
    policy_forward_fast<CH>(raw, legal, g, f);
    #pragma unroll
    for (int j = 0; j < CH; ++j) q[j] = f.p[j];
}

template <int CH>
__global__ void __launch_bounds__(PL_THREADS, 2) learner_objective_kernel(LearnerArgs g) {
    __shared__ double wst[PL_WARPS][PL_MAX_LANES][PL_STATS];
    __shared__ bool last_block;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < PL_WARPS * PL_MAX_LANES * PL_STATS; i += PL_THREADS) {
        const int st = i % PL_STATS;
        (&wst[0][0][0])[i] = st >= PL_SUMS ? -INFINITY : 0.0;
    }
    __syncthreads();
    const Ticks tk = make_ticks(g.E);
    const int W = g.W;
    const int64_t rpl = g.S / g.lanes, apl = g.A / g.lanes;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = (int64_t)blockIdx.x * PL_WARPS + warp; r < g.rows; r += warps) {
        const int64_t s = r / W;
        const int c = (int)(r - s * W);
        const int ln = (int)(s / rpl);
        const float* ctl = g.controls + ln * 10;
        const float lw = g.lane_weight[ln] / (float)rpl;  // d (weighted total) / d (a sigma row's term)
        MaskRow legal{g.mask + s * g.E};
        RawRow raw = raw_row(g.raw, r);
        RowForward<CH> f;
        policy_forward_fast<CH>(raw, legal, tk, f);
        float logp[CH], gp[CH];
        float pent = 0.0f;
        #pragma unroll
        for (int j = 0; j < CH; ++j) {
            logp[j] = __logf(fmaxf(f.p[j], POLICY_EPS));
            pent += f.p[j] * logp[j];
            gp[j] = 0.0f;
        }
        const float entropy = -warp_sum(pent);
        float kl = 0.0f;
        float logq[CH];
        const bool with_ref = g.ref.type_logits != nullptr;
        if (with_ref) {
            float q[CH];
            policy_probs_fast<CH>(raw_row(g.ref, r), legal, tk, q);
            float pk = 0.0f;
            #pragma unroll
            for (int j = 0; j < CH; ++j) {
                logq[j] = __logf(fmaxf(q[j], POLICY_EPS));
                pk += f.p[j] * (logp[j] - logq[j]);
            }
            kl = warp_sum(pk);
        }
        // ---- action span: PPO rows, statistics, gradient of each selected log pi
        const int64_t a0 = g.action_ptr ? g.action_ptr[s] : s;
        const int64_t a1 = g.action_ptr ? g.action_ptr[s + 1] : s + 1;
        const float count = (float)(a1 - a0);
        double st[PL_SUMS];
        #pragma unroll
        for (int k = 0; k < PL_SUMS; ++k) st[k] = 0.0;
        float nlr_max = -INFINITY, ninf_max = -INFINITY;
        float wsum = 0.0f;  // sum over the span of normalised posterior / count
        for (int64_t i = a0; i < a1; ++i) {
            const float* actl = g.controls + (i / apl) * 10;
            const int act = g.action[i];
            const float pa = chunk_fetch<CH>(f.p, act);
            const float cur = __logf(fmaxf(pa, POLICY_EPS));
            const int64_t ic = i * W + c;
            const float post_raw = g.posterior ? g.posterior[ic] : 1.0f;
            const float post = g.inv_post ? post_raw * g.inv_post[i] : post_raw / fmaxf(post_raw, FLT_TINY);
            const float adv = g.advantage[ic];
            const float lr = cur - g.old_log[ic];
            const float ratio = expf(lr);
            const float clip = actl[0], cap = actl[1];
            const float clipped = fminf(fmaxf(ratio, 1.0f - clip), 1.0f + clip);
            const bool neg = adv < 0.0f;
            const float nratio = expf(fminf(lr, cap));
            const float pratio = neg ? nratio : ratio;
            const float X = pratio * adv, Y = clipped * adv;
            const float term = -fminf(X, Y);
            const float w = post / count;
            st[ST_POLICY] += (double)(w * term);
            st[ST_ENTROPY] += (double)(w * entropy);
            st[ST_REFERENCE] += (double)(w * kl);
            st[ST_APPROX] += (double)(w * ((ratio - 1.0f) - lr));
            st[ST_CLIP] += fabsf(ratio - 1.0f) > clip ? (double)w : 0.0;
            st[ST_CAP] += (neg && lr > cap) ? (double)w : 0.0;
            nlr_max = fmaxf(nlr_max, (neg && post > 0.0f) ? lr : 0.0f);
            ninf_max = fmaxf(ninf_max, post * fmaxf(-adv, 0.0f) * (neg ? pratio : 0.0f));
            wsum += w;
            // d(-min(X, Y)) / d cur, through the capped ratio and the clipped ratio
            const float dpr = neg ? nratio * tie_share(lr, cap) : ratio;
            const float dclip = (ratio >= 1.0f - clip && ratio <= 1.0f + clip) ? ratio : 0.0f;
            const float dcur = -lw * w * (tie_share(X, Y) * adv * dpr + tie_share(Y, X) * adv * dclip);
            const float dpa = pa >= POLICY_EPS ? dcur * __frcp_rn(pa) : 0.0f;
            #pragma unroll
            for (int j = 0; j < CH; ++j)
                if (lane * CH + j == act) gp[j] += dpa;
        }
        // ---- entropy (-c4) and KL (+c5) gradients, then the composite backward
        add_reduction_grads<CH>(f, logp, with_ref ? &logq : nullptr, -ctl[4] * lw * wsum, ctl[5] * lw * wsum, gp);
        policy_row_backward<CH>(raw, f, gp, tk, g.grad, r);
        // ---- value of this column under the sigma posterior: wsum (sum over the span of post / count)
        // normalised over the columns of the sigma row
        {
            const float vp = g.inv_vpost ? wsum * g.inv_vpost[s] : wsum / fmaxf(wsum, FLT_TINY);
            const int64_t sc_i = s * W + c;
            const float v = g.value[sc_i], ov = g.old_value[sc_i], tg = g.target[sc_i];
            const float veps = ctl[3];
            const float verr = (v - tg) * (v - tg);
            const float diff = v - ov;
            const float cv = ov + fminf(fmaxf(diff, -veps), veps);
            const float cerr = (cv - tg) * (cv - tg);
            const bool use_clip = ctl[9] != 0.0f;
            const float err = use_clip ? fmaxf(verr, cerr) : verr;
            st[ST_VALUE] += (double)(vp * err);
            const float dverr = 2.0f * (v - tg);
            const float dcerr = (diff >= -veps && diff <= veps) ? 2.0f * (cv - tg) : 0.0f;
            const float dv = use_clip ? tie_share(cerr, verr) * dverr + tie_share(verr, cerr) * dcerr : dverr;
            if (lane == 0) g.d_value[sc_i] = ctl[2] * lw * vp * dv;
        }
        // ---- public heads of branched batches (sigma-level, column 0)
        if (c == 0 && g.trace_pred) {
            const float eps8 = ctl[8];
            const float tp = g.trace_pred[s], cp = g.cost_pred[s], tt = g.trace_target[s], ct = g.cost_target[s];
            const float tden = fmaxf(tp, FLT_TINY) + eps8;
            const float tr = (tt + eps8) / tden;
            const bool deg2 = count >= 2.0f;
            st[ST_TRACE] += deg2 ? (double)(tr - logf(tr) - 1.0f) : 0.0;
            const float cpc = fmaxf(cp, FLT_TINY);
            const float cr = ct / cpc;
            st[ST_COST] += (double)(cr - logf(cr) - 1.0f);
            if (lane == 0) {
                g.d_trace[s] = (deg2 && tp >= FLT_TINY)
                                   ? ctl[6] * lw * (1.0f - 1.0f / tr) * (-(tt + eps8) / (tden * tden))
                                   : 0.0f;
                g.d_cost[s] = cp >= FLT_TINY ? ctl[7] * lw * (1.0f - 1.0f / cr) * (-ct / (cpc * cpc)) : 0.0f;
            }
        }
        if (lane == 0) {
            #pragma unroll
            for (int k = 0; k < PL_SUMS; ++k) wst[warp][ln][k] += st[k];
            // action-lane maxima (spans do not cross lane boundaries)
            const int al = (int)(a0 / apl);
            wst[warp][al][PL_SUMS] = fmax(wst[warp][al][PL_SUMS], (double)nlr_max);
            wst[warp][al][PL_SUMS + 1] = fmax(wst[warp][al][PL_SUMS + 1], (double)ninf_max);
        }
    }
    __syncthreads();
    // ---- block partials (warp order), then the last block reduces (block order)
    const int n = g.lanes * PL_STATS;
    unsigned int* word = reinterpret_cast<unsigned int*>(g.partials);
    for (int i = threadIdx.x; i < n; i += PL_THREADS) {
        const int l = i / PL_STATS, k = i % PL_STATS;
        double acc = k >= PL_SUMS ? -INFINITY : 0.0;
        for (int w = 0; w < PL_WARPS; ++w) acc = k >= PL_SUMS ? fmax(acc, wst[w][l][k]) : acc + wst[w][l][k];
        g.partials[1 + (int64_t)blockIdx.x * n + i] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_block = atomicAdd(word, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last_block) return;
    __threadfence();
    // the last block: each of the n statistics is reduced by `groups` threads, thread (i, grp) over
    // the blocks grp, grp + groups, ... in order, then the groups in order
    __shared__ double red[PL_THREADS];
    const int groups = PL_THREADS / n;  // n <= PL_MAX_LANES * PL_STATS < PL_THREADS
    if ((int)threadIdx.x < groups * n) {
        const int i = threadIdx.x % n, grp = threadIdx.x / n, k = i % PL_STATS;
        double acc = k >= PL_SUMS ? -INFINITY : 0.0;
        for (unsigned b = grp; b < gridDim.x; b += groups) {
            const double v = __ldcg(g.partials + 1 + (int64_t)b * n + i);
            acc = k >= PL_SUMS ? fmax(acc, v) : acc + v;
        }
        red[threadIdx.x] = acc;
    }
    __syncthreads();
    for (int l = threadIdx.x; l < g.lanes; l += PL_THREADS) {
        double acc[PL_STATS];
        for (int k = 0; k < PL_STATS; ++k) acc[k] = k >= PL_SUMS ? -INFINITY : 0.0;
        for (int grp = 0; grp < groups; ++grp)
            for (int k = 0; k < PL_STATS; ++k) {
                const double v = red[grp * n + l * PL_STATS + k];
                acc[k] = k >= PL_SUMS ? fmax(acc[k], v) : acc[k] + v;
            }
        const float* ctl = g.controls + l * 10;
        const double inv = 1.0 / (double)rpl;
        const double policy = acc[ST_POLICY] * inv, value = acc[ST_VALUE] * inv, ent = acc[ST_ENTROPY] * inv,
                     refk = acc[ST_REFERENCE] * inv, trace = acc[ST_TRACE] * inv, cost = acc[ST_COST] * inv;
        float* out = g.result + l * PL_RESULT;
        out[0] = (float)(policy + ctl[2] * value - ctl[4] * ent + ctl[5] * refk + ctl[6] * trace + ctl[7] * cost);
        out[1] = (float)policy;
        out[2] = (float)value;
        out[3] = (float)ent;
        out[4] = (float)refk;
        out[5] = (float)(acc[ST_APPROX] * inv);
        out[6] = (float)(acc[ST_CLIP] * inv);
        out[7] = (float)(acc[ST_CAP] * inv);
        out[8] = (float)acc[PL_SUMS];
        out[9] = (float)acc[PL_SUMS + 1];
    }
    __syncthreads();
    if (threadIdx.x == 0) *word = 0u;  // ready for the next launch
}

// PokerPolicyOperator.learner forward (policy.py:284-298) in one pass per
// policy row: selected log pi (clamped at eps), entropy and, with reference
// fields, KL(p || q).
template <int CH>
__global__ void __launch_bounds__(PL_THREADS, 2) policy_learner_fwd_kernel(int64_t B, int E, pbg_policy raw,
                                                                        pbg_policy ref, const uint8_t* mask,
                                                                        const int32_t* action, float* selected,
                                                                        float* entropy, float* kl) {
    const int lane = threadIdx.x & 31;
    const Ticks tk = make_ticks(E);
    const int64_t rows = B * raw.rows;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = ((int64_t)blockIdx.x * PL_THREADS + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t b = r / raw.rows;
        MaskRow legal{mask + b * E};
        float p[CH];
        policy_probs_fast<CH>(raw_row(raw, r), legal, tk, p);
        float logp[CH];
        float pe = 0.0f;
        #pragma unroll
        for (int j = 0; j < CH; ++j) {
            logp[j] = __logf(fmaxf(p[j], POLICY_EPS));
            pe += p[j] * logp[j];
        }
        const float ent = -warp_sum(pe);
        float k = 0.0f;
        if (ref.type_logits != nullptr) {
            float q[CH];
            policy_probs_fast<CH>(raw_row(ref, r), legal, tk, q);
            float pk = 0.0f;
            #pragma unroll
            for (int j = 0; j < CH; ++j) pk += p[j] * (logp[j] - __logf(fmaxf(q[j], POLICY_EPS)));
            k = warp_sum(pk);
        }
        const float pa = chunk_fetch<CH>(p, action[b]);
        if (lane == 0) {
            selected[r] = __logf(fmaxf(pa, POLICY_EPS));
            entropy[r] = ent;
            kl[r] = k;
        }
    }
}

// Vector-Jacobian product of PokerPolicyOperator.learner (policy.py:284-298):
// upstream gradients of the selected log-probability, the entropy and the
// reference KL of every policy row (B rows x `rows` columns, the action and
// legality shared by a row's columns) -> gradients of the raw fields.
template <int CH>
__global__ void __launch_bounds__(PL_THREADS, 2) policy_learner_vjp_kernel(int64_t B, int E, pbg_policy raw,
                                                                        pbg_policy ref, const uint8_t* mask,
                                                                        const int32_t* action, const float* g_sel,
                                                                        const float* g_ent, const float* g_kl,
                                                                        pbg_policy_grad grad) {
    const int lane = threadIdx.x & 31;
    const Ticks tk = make_ticks(E);
    const int64_t rows = B * raw.rows;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = ((int64_t)blockIdx.x * PL_THREADS + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t b = r / raw.rows;
        MaskRow legal{mask + b * E};
        RawRow rr = raw_row(raw, r);
        RowForward<CH> f;
        policy_forward_fast<CH>(rr, legal, tk, f);
        float logp[CH], gp[CH], logq[CH];
        #pragma unroll
        for (int j = 0; j < CH; ++j) {
            logp[j] = __logf(fmaxf(f.p[j], POLICY_EPS));
            gp[j] = 0.0f;
        }
        const bool with_ref = ref.type_logits != nullptr && g_kl != nullptr;
        if (with_ref) {
            float q[CH];
            policy_probs_fast<CH>(raw_row(ref, r), legal, tk, q);
            #pragma unroll
            for (int j = 0; j < CH; ++j) logq[j] = __logf(fmaxf(q[j], POLICY_EPS));
        }
        if (g_sel) {
            const int act = action[b];
            const float pa = chunk_fetch<CH>(f.p, act);
            const float dpa = pa >= POLICY_EPS ? g_sel[r] * __frcp_rn(pa) : 0.0f;
            #pragma unroll
            for (int j = 0; j < CH; ++j)
                if (lane * CH + j == act) gp[j] += dpa;
        }
        add_reduction_grads<CH>(f, logp, with_ref ? &logq : nullptr, g_ent ? g_ent[r] : 0.0f,
                                with_ref ? g_kl[r] : 0.0f, gp);
        policy_row_backward<CH>(rr, f, gp, tk, grad, r);
    }
}

// Posterior normalisers of Rao-Blackwell batches (learner.py:2019-2021 and
// 2063-2071): inv_post[i] = 1 / max(sum_c posterior[i,c], tiny) per action
// row, inv_vpost[s] = 1 / max(sum_c sum_{i in s} post[i,c] / count_s, tiny).
__global__ void __launch_bounds__(256) posterior_norm_kernel(int64_t S, int W, const int64_t* action_ptr,
                                                             const float* posterior, float* inv_post,
                                                             float* inv_vpost) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * 8;
    for (int64_t s = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5; s < S; s += warps) {
        const int64_t a0 = action_ptr ? action_ptr[s] : s, a1 = action_ptr ? action_ptr[s + 1] : s + 1;
        float vsum = 0.0f;
        for (int64_t i = a0; i < a1; ++i) {
            float part = 0.0f;
            for (int c = lane; c < W; c += 32) part += posterior[i * W + c];
            const float inv = 1.0f / fmaxf(warp_sum(part), FLT_TINY);
            if (lane == 0) inv_post[i] = inv;
            vsum += part * inv;  // this lane's share of the normalised row
        }
        vsum = warp_sum(vsum) / (float)(a1 - a0);
        if (lane == 0) inv_vpost[s] = 1.0f / fmaxf(vsum, FLT_TINY);
    }
}

// Chunk of events per lane: the smallest instantiated CH with 32 * CH >= E.
template <class F>
static void with_chunk(int E, F&& f) {
    if (E <= 32) f(std::integral_constant<int, 1>{});
    else if (E <= 64) f(std::integral_constant<int, 2>{});
    else if (E <= 128) f(std::integral_constant<int, 4>{});
    else if (E <= 224) f(std::integral_constant<int, 7>{});
    else f(std::integral_constant<int, 9>{});
}

static int64_t stat_bytes(int32_t lanes) {
    return ((1 + (int64_t)PL_MAX_BLOCKS * lanes * PL_STATS) * (int64_t)sizeof(double) + 255) / 256 * 256;
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_learner_workspace_bytes(int64_t S, int64_t A, int32_t lanes) {
    if (S < 0 || A < 0 || lanes < 1 || lanes > PL_MAX_LANES) return -1;
    return stat_bytes(lanes) + ((A + S) * (int64_t)sizeof(float) + 255) / 256 * 256;
}

int pbg_poker_learner_objective(int64_t S, int64_t A, int32_t E, int32_t W, int32_t lanes, pbg_policy raw,
                                const pbg_policy* reference, const uint8_t* mask, const int64_t* action_ptr,
                                const int32_t* action, const float* old_log, const float* advantage,
                                const float* posterior, const float* value, const float* old_value,
                                const float* value_target, const float* trace_pred, const float* cost_pred,
                                const float* trace_target, const float* cost_target, const float* controls,
                                const float* lane_weight, pbg_policy_grad grad, float* d_value, float* d_trace,
                                float* d_cost, float* result, void* workspace, int64_t workspace_bytes,
                                void* stream) {
    PBG_REQUIRE(S >= 0 && A >= S && E > RAISE_OFFSET && E <= 32 * CHUNK_MAX, "learner: bad S/A/E");
    PBG_REQUIRE(W >= 1 && raw.rows == W && raw.mixtures >= 1 && raw.mixtures <= ClosedPolicy::MMAX,
                "learner: raw rows must equal W and mixtures lie in [1,8]");
    PBG_REQUIRE(lanes >= 1 && lanes <= PL_MAX_LANES && S % lanes == 0 && A % lanes == 0,
                "learner: lanes in [1,16] must divide the sigma and action rows");
    PBG_REQUIRE(action_ptr || A == S, "learner: ragged batches need action_ptr");
    PBG_REQUIRE(!reference || (reference->rows == W && reference->mixtures == raw.mixtures),
                "learner: reference fields must share the raw layout");
    PBG_REQUIRE(controls && lane_weight && result && workspace, "learner: null controls, weights or outputs");
    PBG_REQUIRE(S == 0 || (raw.type_logits && raw.omega && raw.mu && raw.scale && raw.iota && mask && action &&
                           old_log && advantage && value && old_value && value_target && grad.type_logits &&
                           grad.omega && grad.mu && grad.scale && grad.iota && d_value),
                "learner: null argument");
    PBG_REQUIRE(W == 1 || posterior, "learner: Rao-Blackwell rows (W > 1) need the posterior");
    const bool heads = trace_pred != nullptr;
    PBG_REQUIRE(!heads || (cost_pred && trace_target && cost_target && d_trace && d_cost && action_ptr),
                "learner: public heads need predictions, targets, gradients and action spans");
    const int64_t need = pbg_learner_workspace_bytes(S, A, lanes);
    PBG_REQUIRE(workspace_bytes >= need, "learner: workspace of %lld bytes, %lld needed", (long long)workspace_bytes,
                (long long)need);
    if (S == 0) return PBG_OK;
    cudaStream_t st = as_stream(stream);
    LearnerArgs g{};
    g.S = S;
    g.A = A;
    g.rows = S * (int64_t)W;
    g.E = E;
    g.W = W;
    g.lanes = lanes;
    g.raw = raw;
    if (reference) g.ref = *reference;
    g.mask = mask;
    g.action_ptr = action_ptr;
    g.action = action;
    g.old_log = old_log;
    g.advantage = advantage;
    g.posterior = posterior;
    g.value = value;
    g.old_value = old_value;
    g.target = value_target;
    g.trace_pred = trace_pred;
    g.cost_pred = cost_pred;
    g.trace_target = trace_target;
    g.cost_target = cost_target;
    g.controls = controls;
    g.lane_weight = lane_weight;
    g.grad = grad;
    g.d_value = d_value;
    g.d_trace = d_trace;
    g.d_cost = d_cost;
    g.result = result;
    g.partials = static_cast<double*>(workspace);
    int grid = stride_grid(g.rows * 32, PL_THREADS);
    if (grid > PL_MAX_BLOCKS) grid = PL_MAX_BLOCKS;
    if (W > 1) {
        float* norms = reinterpret_cast<float*>(static_cast<char*>(workspace) + stat_bytes(lanes));
        g.inv_post = norms;
        g.inv_vpost = norms + A;
        posterior_norm_kernel<<<stride_grid(S * 32, 256), 256, 0, st>>>(S, W, action_ptr, posterior, norms, norms + A);
    }
    with_chunk(E, [&](auto ch) { learner_objective_kernel<decltype(ch)::value><<<grid, PL_THREADS, 0, st>>>(g); });
    return launch_status("poker_learner_objective");
}

int pbg_policy_learner_forward(int64_t B, int32_t E, pbg_policy raw, const pbg_policy* reference,
                               const uint8_t* mask, const int32_t* action, float* selected, float* entropy,
                               float* kl, void* stream) {
    PBG_REQUIRE(B >= 0 && E > RAISE_OFFSET && E <= 32 * CHUNK_MAX, "policy_learner_forward: bad B or E");
    PBG_REQUIRE(raw.rows >= 1 && raw.mixtures >= 1 && raw.mixtures <= ClosedPolicy::MMAX,
                "policy_learner_forward: rows >= 1, mixtures in [1,8]");
    PBG_REQUIRE(!reference || (reference->rows == raw.rows && reference->mixtures == raw.mixtures),
                "policy_learner_forward: reference fields must share the raw layout");
    PBG_REQUIRE(B == 0 || (raw.type_logits && raw.omega && raw.mu && raw.scale && raw.iota && mask && action &&
                           selected && entropy && kl),
                "policy_learner_forward: null argument");
    if (B == 0) return PBG_OK;
    pbg_policy ref{};
    if (reference) ref = *reference;
    const int grid = stride_grid(B * raw.rows * 32, PL_THREADS);
    with_chunk(E, [&](auto ch) {
        policy_learner_fwd_kernel<decltype(ch)::value><<<grid, PL_THREADS, 0, as_stream(stream)>>>(
            B, E, raw, ref, mask, action, selected, entropy, kl);
    });
    return launch_status("policy_learner_forward");
}

int pbg_policy_learner_backward(int64_t B, int32_t E, pbg_policy raw, const pbg_policy* reference,
                                const uint8_t* mask, const int32_t* action, const float* g_selected,
                                const float* g_entropy, const float* g_kl, pbg_policy_grad grad, void* stream) {
    PBG_REQUIRE(B >= 0 && E > RAISE_OFFSET && E <= 32 * CHUNK_MAX, "policy_learner_backward: bad B or E");
    PBG_REQUIRE(raw.rows >= 1 && raw.mixtures >= 1 && raw.mixtures <= ClosedPolicy::MMAX,
                "policy_learner_backward: rows >= 1, mixtures in [1,8]");
    PBG_REQUIRE(!g_kl || (reference && reference->rows == raw.rows && reference->mixtures == raw.mixtures),
                "policy_learner_backward: a KL gradient needs reference fields of the raw layout");
    PBG_REQUIRE(!g_selected || action, "policy_learner_backward: a selected-log-pi gradient needs the actions");
    PBG_REQUIRE(B == 0 || (raw.type_logits && raw.omega && raw.mu && raw.scale && raw.iota && mask &&
                           grad.type_logits && grad.omega && grad.mu && grad.scale && grad.iota),
                "policy_learner_backward: null argument");
    if (B == 0) return PBG_OK;
    pbg_policy ref{};
    if (reference) ref = *reference;
    const int grid = stride_grid(B * raw.rows * 32, PL_THREADS);
    with_chunk(E, [&](auto ch) {
        policy_learner_vjp_kernel<decltype(ch)::value><<<grid, PL_THREADS, 0, as_stream(stream)>>>(
            B, E, raw, ref, mask, action, g_selected, g_entropy, g_kl, grad);
    });
    return launch_status("policy_learner_backward");
}

}  // extern "C"
