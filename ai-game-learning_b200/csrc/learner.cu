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
// shared memory, reduced per block in warp order and across blocks in block
// order by the last block to arrive (deterministic for a given grid).
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

// Forward of one row, keeping what the backward needs (lane chunk of C events).
struct RowForward {
    float p[CHUNK_MAX];     // probabilities, 0 where illegal
    float mix[CHUNK_MAX];   // masked mixture on raise ticks
    float cond[CHUNK_MAX];  // conditional raise probability
    float rp[CHUNK_MAX];    // raise probability (1 - iota) cond + iota [all-in]
    float mass;
    int all_in;             // highest legal raise tick, -1 when none
    bool facing;
};

// Same arithmetic as warp_policy_row (policy.cuh), rounding for rounding.
template <class Legal>
__device__ void policy_forward_ex(const RawRow& raw, const Legal& legal, int T, int E, int C, RowForward& f) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * C;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) f.mix[j] = 0.0f;
    for (int m = 0; m < raw.M; ++m) {
        MixtureEdges mx_m = mixture_edges(raw.mu[m], raw.scale[m], T);
        float tick[CHUNK_MAX];
        float part = 0.0f;
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
        for (int j = 0; j < CHUNK_MAX; ++j) f.mix[j] = __fadd_rn(f.mix[j], __fmul_rn(om, __fdiv_rn(tick[j], total)));
    }
    float part_mass = 0.0f;
    int part_count = 0, part_top = -1;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        bool ok = j < C && e >= 2 && e < E && legal(e);
        if (!ok) f.mix[j] = 0.0f;
        else {
            part_mass = __fadd_rn(part_mass, f.mix[j]);
            ++part_count;
            part_top = e - 2;
        }
    }
    f.mass = warp_sum(part_mass);
    int count = __reduce_add_sync(0xffffffffu, part_count);
    f.all_in = warp_max_int(part_top);
    const float io = raw.iota;
    f.facing = legal(0);
    const float l0 = raw.logits[0], l1 = raw.logits[1], l2 = raw.logits[2];
    float full[CHUNK_MAX];
    float mx = -INFINITY;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        full[j] = -INFINITY;
        f.cond[j] = 0.0f;
        f.rp[j] = 0.0f;
        if (j < C && e < E && legal(e)) {
            if (e == 0) full[j] = l0;
            else if (e == 1) full[j] = f.facing ? l1 : l0;
            else {
                float cond = f.mass > 0.0f ? __fdiv_rn(f.mix[j], fmaxf(f.mass, POLICY_EPS))
                                           : __fdiv_rn(1.0f, (float)max(count, 1));
                float atom = (e - 2) == f.all_in ? 1.0f : 0.0f;
                float rp = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, io), cond), __fmul_rn(io, atom));
                f.cond[j] = cond;
                f.rp[j] = rp;
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
        f.p[j] = (j < C && e < E && legal(e)) ? expf(__fsub_rn(full[j], mx)) : 0.0f;
        part_sum = __fadd_rn(part_sum, f.p[j]);
    }
    float denom = warp_sum(part_sum);
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        int e = e0 + j;
        f.p[j] = (j < C && e < E && legal(e)) ? __fdiv_rn(f.p[j], denom) : 0.0f;
    }
}

// Backward of one mixture component: given d(total)/d(mixture_k) on the raise
// ticks held by this lane (0 elsewhere), accumulate d omega_m, d mu_m, d s_m.
// Recomputes the forward's tick masses a_k = v_k / max(N, tiny) and their sum.
__device__ void component_backward(const RawRow& raw, int m, int T, int E, int C, const float (&dmix)[CHUNK_MAX],
                                   float& d_om, float& d_mu, float& d_s) {
    const int lane = threadIdx.x & 31;
    const int e0 = lane * C;
    const float loc = raw.mu[m], sc = raw.scale[m];
    const MixtureEdges mx = mixture_edges(loc, sc, T);
    const float z0 = __fdiv_rn(__fsub_rn(0.0f, loc), sc);
    const float zT = __fdiv_rn(__fsub_rn(edge_of(T, T), loc), sc);
    const float norm = __fmul_rn(__fmul_rn(sigmoid_f(zT), sigmoid_f(-z0)), -expm1f(__fsub_rn(z0, zT)));
    float v[CHUNK_MAX], a[CHUNK_MAX], dlow[CHUNK_MAX], zlow[CHUNK_MAX];
    float dtop = 0.0f, ztop = 0.0f;  // sigma'(z_T) and z_T on the lane holding tick T-1
    float part = 0.0f;
    const int k0 = e0 - 2;
    float sig_prev, sm_prev;
    edge_sigmoids(mx, k0 > 0 ? k0 : 0, T, sig_prev, sm_prev);
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        v[j] = a[j] = dlow[j] = zlow[j] = 0.0f;
        const int e = e0 + j, k = e - 2;
        if (j < C && k >= 0 && e < E) {
            float sig_next, sm_next;
            edge_sigmoids(mx, k + 1, T, sig_next, sm_next);
            v[j] = fmaxf(__fmul_rn(__fmul_rn(sig_next, sm_prev), mx.width), 0.0f);
            a[j] = __fmul_rn(v[j], mx.inv_norm);
            part = __fadd_rn(part, a[j]);
            dlow[j] = sig_prev * sm_prev;  // sigma'(z_k)
            zlow[j] = (edge_of(k, T) - loc) * mx.inv_scale;
            if (k + 1 == T) {
                dtop = sig_next * sm_next;
                ztop = (edge_of(T, T) - loc) * mx.inv_scale;
            }
            sig_prev = sig_next;
            sm_prev = sm_next;
        }
    }
    const float total = warp_sum(part);
    const float Sc = fmaxf(total, FLT_TINY);
    const float om = raw.omega[m];
    float pom = 0.0f, pq = 0.0f;
    float ddl[CHUNK_MAX];
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const float dl = __fdiv_rn(a[j], Sc);
        pom += dmix[j] * dl;
        ddl[j] = dmix[j] * om;
        pq += ddl[j] * a[j];
    }
    d_om += warp_sum(pom);
    const float Q = warp_sum(pq);
    const float qterm = total >= FLT_TINY ? Q / (Sc * Sc) : 0.0f;
    float dc[CHUNK_MAX];
    float pn = 0.0f, last = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = e0 + j, k = e - 2;
        dc[j] = 0.0f;
        if (j < C && k >= 0 && e < E) {
            const float da = ddl[j] / Sc - qterm;
            pn += da * v[j];
            dc[j] = da * mx.inv_norm;
        }
        if (j == C - 1) last = dc[j];
    }
    const float sn = warp_sum(pn);
    const float dN = norm >= FLT_TINY ? -sn * mx.inv_norm * mx.inv_norm : 0.0f;
    float carry = __shfl_up_sync(0xffffffffu, last, 1);  // dc of the tick just before this lane's chunk
    if (lane == 0) carry = 0.0f;
    float sdz = 0.0f, szdz = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = e0 + j, k = e - 2;
        const bool tick = j < C && k >= 0 && e < E;
        if (tick) {
            // edge k: lower edge of tick k, upper edge of tick k-1 (no tick before tick 0)
            const float before = k == 0 ? 0.0f : carry;
            float dz = (before - dc[j]) * dlow[j];
            if (k == 0) dz -= dN * dlow[j];
            sdz += dz;
            szdz += zlow[j] * dz;
            if (k + 1 == T) {
                const float dzT = (dc[j] + dN) * dtop;
                sdz += dzT;
                szdz += ztop * dzT;
            }
            carry = dc[j];
        }
    }
    d_mu += -warp_sum(sdz) * mx.inv_scale;
    d_s += -warp_sum(szdz) * mx.inv_scale;
}

__device__ __forceinline__ float tie_share(float a, float b) { return a < b ? 1.0f : (a == b ? 0.5f : 0.0f); }

// dL/dp of the entropy and KL reductions (policy.py:235-244) with upstream
// gradients g_ent (d/d entropy) and g_kl (d/d KL): entropy -sum p log max(p, eps)
// gives -(log max(p, eps) + [p >= eps]); KL sum p (log max(p, eps) - log max(q, eps))
// gives log max(p, eps) - log max(q, eps) + [p >= eps].  Illegal events get 0
// (the masked fill after the softmax).
__device__ __forceinline__ void add_reduction_grads(const RowForward& f, const float (&logp)[CHUNK_MAX],
                                                    const float (*logq)[CHUNK_MAX], const MaskRow& legal, int E,
                                                    int C, float g_ent, float g_kl, float (&gp)[CHUNK_MAX]) {
    const int lane = threadIdx.x & 31;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = lane * C + j;
        if (j < C && e < E && legal(e)) {
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
__device__ void policy_row_backward(const RawRow& raw, const RowForward& f, const float (&gp)[CHUNK_MAX],
                                    const MaskRow& legal, int T, int E, int C, const pbg_policy_grad& grad,
                                    int64_t r) {
    const int lane = threadIdx.x & 31;
    // masked softmax (selected logits -inf where illegal)
    float psg = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) psg += gp[j] * f.p[j];
    const float sg = warp_sum(psg);
    float dx[CHUNK_MAX];
    float pt0 = 0.0f, pt1 = 0.0f, pt2 = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = lane * C + j;
        dx[j] = (j < C && e < E && legal(e)) ? f.p[j] * (gp[j] - sg) : 0.0f;
        if (e == 0) pt0 += dx[j];
        else if (e == 1) {
            if (f.facing) pt1 += dx[j];
            else pt0 += dx[j];
        } else pt2 += dx[j];
    }
    const float dt0 = warp_sum(pt0), dt1 = warp_sum(pt1), dt2 = warp_sum(pt2);
    // raise logits l2 + log max(rp, eps) where rp > 0; rp = (1 - iota) cond + iota [all-in tick]
    const float io = raw.iota;
    float dcond[CHUNK_MAX];
    float pio = 0.0f, pdm = 0.0f;
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = lane * C + j;
        dcond[j] = 0.0f;
        if (j < C && e >= 2 && e < E && legal(e)) {
            const float rp = f.rp[j];
            const float drp = (rp > 0.0f && rp >= POLICY_EPS) ? dx[j] / rp : 0.0f;
            const float atom = (e - 2) == f.all_in ? 1.0f : 0.0f;
            pio += drp * (atom - f.cond[j]);
            dcond[j] = drp * (1.0f - io);
            pdm += dcond[j] * f.mix[j];
        }
    }
    const float dio = warp_sum(pio);
    // cond = mixture / max(mass, eps) when mass > 0, else the uniform law (no gradient)
    const float mass = f.mass;
    const float mc = fmaxf(mass, POLICY_EPS);
    const float sdm = warp_sum(pdm);
    const float dmass = mass >= POLICY_EPS ? -sdm / (mc * mc) : 0.0f;
    float dmix[CHUNK_MAX];
    #pragma unroll
    for (int j = 0; j < CHUNK_MAX; ++j) {
        const int e = lane * C + j;
        dmix[j] = (mass > 0.0f && j < C && e >= 2 && e < E && legal(e)) ? dcond[j] / mc + dmass : 0.0f;
    }
    float* gom = grad.omega + r * raw.M;
    float* gmu = grad.mu + r * raw.M;
    float* gsc = grad.scale + r * raw.M;
    for (int m = 0; m < raw.M; ++m) {
        float dom = 0.0f, dmu = 0.0f, dsc = 0.0f;
        component_backward(raw, m, T, E, C, dmix, dom, dmu, dsc);
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

__global__ void __launch_bounds__(PL_THREADS) learner_objective_kernel(LearnerArgs g) {
    __shared__ double wst[PL_WARPS][PL_MAX_LANES][PL_STATS];
    __shared__ bool last_block;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < PL_WARPS * PL_MAX_LANES * PL_STATS; i += PL_THREADS) {
        const int st = i % PL_STATS;
        (&wst[0][0][0])[i] = st >= PL_SUMS ? -INFINITY : 0.0;
    }
    __syncthreads();
    const int E = g.E, C = (E + 31) / 32, T = E - 2, W = g.W;
    const int64_t rpl = g.S / g.lanes, apl = g.A / g.lanes;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = (int64_t)blockIdx.x * PL_WARPS + warp; r < g.rows; r += warps) {
        const int64_t s = r / W;
        const int c = (int)(r - s * W);
        const int ln = (int)(s / rpl);
        const float* ctl = g.controls + ln * 10;
        const float lw = g.lane_weight[ln] / (float)rpl;  // d (weighted total) / d (a sigma row's term)
        MaskRow legal{g.mask + s * E};
        RawRow raw = raw_row(g.raw, r);
        RowForward f;
        policy_forward_ex(raw, legal, T, E, C, f);
        float logp[CHUNK_MAX], gp[CHUNK_MAX];
        float pent = 0.0f;
        #pragma unroll
        for (int j = 0; j < CHUNK_MAX; ++j) {
            logp[j] = logf(fmaxf(f.p[j], POLICY_EPS));
            pent += f.p[j] * logp[j];
            gp[j] = 0.0f;
        }
        const float entropy = -warp_sum(pent);
        float kl = 0.0f;
        float logq[CHUNK_MAX];
        const bool with_ref = g.ref.type_logits != nullptr;
        if (with_ref) {
            float q[CHUNK_MAX];
            warp_policy_row(raw_row(g.ref, r), legal, T, E, C, q);
            float pk = 0.0f;
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j) {
                logq[j] = logf(fmaxf(q[j], POLICY_EPS));
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
            const float pa = warp_fetch(f.p, act, C);
            const float cur = logf(fmaxf(pa, POLICY_EPS));
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
            const float dpa = pa >= POLICY_EPS ? dcur / pa : 0.0f;
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j)
                if (lane * C + j == act) gp[j] += dpa;
        }
        // ---- entropy (-c4) and KL (+c5) gradients, then the composite backward
        add_reduction_grads(f, logp, with_ref ? &logq : nullptr, legal, E, C, -ctl[4] * lw * wsum,
                            ctl[5] * lw * wsum, gp);
        policy_row_backward(raw, f, gp, legal, T, E, C, g.grad, r);
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
    for (int l = threadIdx.x; l < g.lanes; l += PL_THREADS) {
        double acc[PL_STATS];
        for (int k = 0; k < PL_STATS; ++k) acc[k] = k >= PL_SUMS ? -INFINITY : 0.0;
        for (unsigned b = 0; b < gridDim.x; ++b)
            for (int k = 0; k < PL_STATS; ++k) {
                const double v = __ldcg(g.partials + 1 + (int64_t)b * n + l * PL_STATS + k);
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
__global__ void __launch_bounds__(PL_THREADS) policy_learner_fwd_kernel(int64_t B, int E, pbg_policy raw,
                                                                        pbg_policy ref, const uint8_t* mask,
                                                                        const int32_t* action, float* selected,
                                                                        float* entropy, float* kl) {
    const int lane = threadIdx.x & 31;
    const int C = (E + 31) / 32, T = E - 2;
    const int64_t rows = B * raw.rows;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = ((int64_t)blockIdx.x * PL_THREADS + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t b = r / raw.rows;
        MaskRow legal{mask + b * E};
        float p[CHUNK_MAX];
        warp_policy_row(raw_row(raw, r), legal, T, E, C, p);
        float logp[CHUNK_MAX];
        float pe = 0.0f;
        #pragma unroll
        for (int j = 0; j < CHUNK_MAX; ++j) {
            logp[j] = logf(fmaxf(p[j], POLICY_EPS));
            pe += p[j] * logp[j];
        }
        const float ent = -warp_sum(pe);
        float k = 0.0f;
        if (ref.type_logits != nullptr) {
            float q[CHUNK_MAX];
            warp_policy_row(raw_row(ref, r), legal, T, E, C, q);
            float pk = 0.0f;
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j) pk += p[j] * (logp[j] - logf(fmaxf(q[j], POLICY_EPS)));
            k = warp_sum(pk);
        }
        const float pa = warp_fetch(p, action[b], C);
        if (lane == 0) {
            selected[r] = logf(fmaxf(pa, POLICY_EPS));
            entropy[r] = ent;
            kl[r] = k;
        }
    }
}

// Vector-Jacobian product of PokerPolicyOperator.learner (policy.py:284-298):
// upstream gradients of the selected log-probability, the entropy and the
// reference KL of every policy row (B rows x `rows` columns, the action and
// legality shared by a row's columns) -> gradients of the raw fields.
__global__ void __launch_bounds__(PL_THREADS) policy_learner_vjp_kernel(int64_t B, int E, pbg_policy raw,
                                                                        pbg_policy ref, const uint8_t* mask,
                                                                        const int32_t* action, const float* g_sel,
                                                                        const float* g_ent, const float* g_kl,
                                                                        pbg_policy_grad grad) {
    const int lane = threadIdx.x & 31;
    const int C = (E + 31) / 32, T = E - 2;
    const int64_t rows = B * raw.rows;
    const int64_t warps = (int64_t)gridDim.x * PL_WARPS;
    for (int64_t r = ((int64_t)blockIdx.x * PL_THREADS + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t b = r / raw.rows;
        MaskRow legal{mask + b * E};
        RawRow rr = raw_row(raw, r);
        RowForward f;
        policy_forward_ex(rr, legal, T, E, C, f);
        float logp[CHUNK_MAX], gp[CHUNK_MAX], logq[CHUNK_MAX];
        #pragma unroll
        for (int j = 0; j < CHUNK_MAX; ++j) {
            logp[j] = logf(fmaxf(f.p[j], POLICY_EPS));
            gp[j] = 0.0f;
        }
        const bool with_ref = ref.type_logits != nullptr && g_kl != nullptr;
        if (with_ref) {
            float q[CHUNK_MAX];
            warp_policy_row(raw_row(ref, r), legal, T, E, C, q);
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j) logq[j] = logf(fmaxf(q[j], POLICY_EPS));
        }
        if (g_sel) {
            const int act = action[b];
            const float pa = warp_fetch(f.p, act, C);
            const float dpa = pa >= POLICY_EPS ? g_sel[r] / pa : 0.0f;
            #pragma unroll
            for (int j = 0; j < CHUNK_MAX; ++j)
                if (lane * C + j == act) gp[j] += dpa;
        }
        add_reduction_grads(f, logp, with_ref ? &logq : nullptr, legal, E, C, g_ent ? g_ent[r] : 0.0f,
                            with_ref ? g_kl[r] : 0.0f, gp);
        policy_row_backward(rr, f, gp, legal, T, E, C, grad, r);
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
    learner_objective_kernel<<<grid, PL_THREADS, 0, st>>>(g);
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
    policy_learner_fwd_kernel<<<stride_grid(B * raw.rows * 32, PL_THREADS), PL_THREADS, 0, as_stream(stream)>>>(
        B, E, raw, ref, mask, action, selected, entropy, kl);
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
    policy_learner_vjp_kernel<<<stride_grid(B * raw.rows * 32, PL_THREADS), PL_THREADS, 0, as_stream(stream)>>>(
        B, E, raw, ref, mask, action, g_selected, g_entropy, g_kl, grad);
    return launch_status("policy_learner_backward");
}

}  // extern "C"
