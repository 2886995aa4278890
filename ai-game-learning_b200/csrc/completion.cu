// Rao-Blackwell leaf completion behind the contract-v2 `complete` and
// `complete_selected` signatures of the external poker_gpu_evaluator, called by
// RBCompletionBinding.leaf_to_layer_work (pbg/games/poker/queued/hooks.py:
// 2472-2477, 2512) on the rows that PokerStateMachine.rb_leaf captures
// (hooks.py:1218-1258).  The law is PreTerminalMC (docs/theory/core_math.tex:
// 664-684, 1360-1380): draw the private profile X from
//     P(x | tau) ∝ mu(x) * prod_q r_q(tau | x_q),
// mu uniform over card-disjoint deals (the chance reach of the dealt board is
// the same for every profile and cancels), complete the hand given X, and
// publish per seat p and private hand h the occurrence p_hat[p,h] ~ P(X_p = h)
// and the conditional mean return v_hat[p,h] ~ E(R_p | X_p = h), with the
// sampler's effective sample size n_eff.  The evaluator's own implementation is
// not part of the reference tree; this kernel is this build's own estimator of
// that law.
//
// Sampler (sequential importance sampling over the seats, as the reference's
// theory notes recommend).  For sample i of a row, seats q = 0..P-1 in order:
// the proposal for seat q is its board-legal range restricted to the hands
// disjoint from the cards of seats < q; the sample's weight is
//     w_i = prod_q Z_q(dead_q) / Z_q,
// Z_q the seat's board-legal mass and Z_q(dead) the mass of its hands disjoint
// from `dead` (inclusion-exclusion over the dead cards with per-card masses).
// A seat's draw is up to RB_ATTEMPTS proposals from its fp32 CDF, keeping the
// first one disjoint from `dead` (exactly the restricted law), then one exact
// scan of the restricted range.  The missing board cards are dealt uniformly
// from the unused deck, and the returns follow the contract-v2 stratum
// settlement (showdown.cuh).  Every draw is addressed by (row seed, sample,
// seat or board slot, attempt) through the counter hash, so results do not
// depend on the launch shape.
//
// Estimates are reduced in 64-bit fixed point (integer sums are associative,
// so the shared-memory atomics are deterministic): q_i = rint(w_i 2^(Q-e_w)),
// m_i,p = rint(w_i R_i,p 2^(Q-e_w-e_R)) with 2^e_w > max w and 2^e_R > max|R|;
// p_hat = sum q / sum q, v_hat = 2^e_R * sum m / sum q over the samples that
// drew hand h, n_eff = (sum q)^2 / sum q^2 (at most n_samples).
//
// One persistent CTA per leaf row, all tables in shared memory: the hand ->
// card table (once per CTA), the board-masked range [P,H] f32, its CDF [P,H]
// f32 (reused as the [2,H] int64 accumulators after sampling), per-card masses
// [P,D] f64, and the sample records (weight f64, hands u16 [P], returns f32
// [P]).  Rows with an invalid board card or selected seat set *status bit 1
// and publish zeros; rows whose every sample has weight 0 (a seat without
// board-legal mass) set bit 2 and publish n_eff = 0.
#include <cfloat>

#include "showdown.cuh"

namespace pbg {
namespace {

constexpr int RB_THREADS = 256;
constexpr int RB_WARPS = RB_THREADS / 32;
constexpr int RB_ATTEMPTS = 16;
constexpr uint32_t RB_BAD_INPUT = 1u, RB_NO_MASS = 2u;
constexpr int64_t RB_SMEM_MAX = 227 * 1024;

struct RBLayout {
    int64_t hc, wb, cdf, mass, zd, rw, rh, rr, red, total;
};

__host__ __device__ __forceinline__ int64_t align16(int64_t x) { return (x + 15) & ~(int64_t)15; }

__host__ __device__ __forceinline__ RBLayout rb_layout(int P, int H, int D, int N) {
    RBLayout L;
    int64_t o = 0;
    L.hc = o;
    o = align16(o + 2 * (int64_t)H);
    L.wb = o;
    o = align16(o + 4 * (int64_t)P * H);
    L.cdf = o;
    const int64_t cdf_bytes = 4 * (int64_t)P * H, acc_bytes = 16 * (int64_t)H;
    o = align16(o + (cdf_bytes > acc_bytes ? cdf_bytes : acc_bytes));
    L.mass = o;
    o = align16(o + 8 * (int64_t)P * D);
    L.zd = o;
    o = align16(o + 8 * (int64_t)P);
    L.rw = o;
    o = align16(o + 8 * (int64_t)N);
    L.rh = o;
    o = align16(o + 2 * (int64_t)N * P);
    L.rr = o;
    o = align16(o + 4 * (int64_t)N * P);
    L.red = o;
    o = align16(o + 8 * 4 * RB_WARPS);
    L.total = o;
    return L;
}

// Lexicographic id of the local card pair a < b in a deck of D cards.
__device__ __forceinline__ int pair_id(int D, int a, int b) { return a * (2 * D - a - 1) / 2 + b - a - 1; }

__device__ __forceinline__ int ceil_log2(int n) {
    int k = 0;
    while ((1 << k) < n) ++k;
    return k;
}

__device__ __forceinline__ double warp_max_double(double v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Butterfly sum: every lane ends with the same value (each step adds a commutative pair).
__device__ __forceinline__ double warp_butterfly_double(double v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ long long warp_sum_ll(long long v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(RB_THREADS)
rb_complete_kernel(Strength S, int R, int D, int first, int64_t F, int P, int strata, int N,
                   const uint8_t* __restrict__ board, const float* __restrict__ weights,
                   const int32_t* __restrict__ level, const float* __restrict__ baseline,
                   const float* __restrict__ amount, const int64_t* __restrict__ seed,
                   const int32_t* __restrict__ selected, float* __restrict__ p_hat, float* __restrict__ v_hat,
                   float* __restrict__ n_eff, uint32_t* __restrict__ status) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int H = D * (D - 1) / 2;
    const RBLayout L = rb_layout(P, H, D, N);
    uint8_t* hc = smem + L.hc;
    float* wb = reinterpret_cast<float*>(smem + L.wb);
    float* cdf = reinterpret_cast<float*>(smem + L.cdf);
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(smem + L.cdf);  // after sampling
    double* mass = reinterpret_cast<double*>(smem + L.mass);
    double* zd = reinterpret_cast<double*>(smem + L.zd);
    double* rw = reinterpret_cast<double*>(smem + L.rw);
    uint16_t* rh = reinterpret_cast<uint16_t*>(smem + L.rh);
    float* rr = reinterpret_cast<float*>(smem + L.rr);
    double* red = reinterpret_cast<double*>(smem + L.red);
    long long* red_ll = reinterpret_cast<long long*>(smem + L.red);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t deck = (1ull << D) - 1ull;  // D <= 52
    const int outputs = selected ? 1 : P;

    for (int h = tid; h < H; h += RB_THREADS) {
        int c0, c1;
        combo_cards(D, 0, h, c0, c1);
        hc[2 * h] = (uint8_t)c0;
        hc[2 * h + 1] = (uint8_t)c1;
    }
    __syncthreads();

    for (int64_t f = blockIdx.x; f < F; f += gridDim.x) {
        // ---- the row's public board and selected seat (every thread, broadcast loads)
        uint64_t bmask = 0;
        int bc[5];
        bool bad = false;
        #pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int c = board[f * 5 + j];
            bc[j] = c;
            if (c == PAD_CARD) continue;
            if (c < first || c >= 52 || ((bmask >> (c - first)) & 1ull)) {
                bad = true;
            } else {
                bmask |= 1ull << (c - first);
            }
        }
        const int sel = selected ? selected[f] : 0;
        if (selected && (sel < 0 || sel >= P)) bad = true;
        if (bad) {
            for (int64_t k = tid; k < (int64_t)outputs * H; k += RB_THREADS) {
                p_hat[f * outputs * H + k] = 0.0f;
                v_hat[f * outputs * H + k] = 0.0f;
            }
            if (tid == 0) {
                n_eff[f] = 0.0f;
                atomicOr(status, RB_BAD_INPUT);
            }
            continue;
        }

        // ---- board-masked range weights (non-positive and non-finite weigh 0)
        const float* wrow = weights + f * (int64_t)P * H;
        for (int idx = tid; idx < P * H; idx += RB_THREADS) {
            const int h = idx - (idx / H) * H;
            const float x = __ldg(wrow + idx);
            const bool conflict = ((bmask >> hc[2 * h]) | (bmask >> hc[2 * h + 1])) & 1ull;
            wb[idx] = (x > 0.0f && x <= FLT_MAX && !conflict) ? x : 0.0f;
        }
        __syncthreads();

        // ---- per seat: fp32 CDF from a double running sum (warp q: each lane a contiguous
        //      segment, segment bases from an inclusive warp scan of the segment totals)
        if (warp < P) {
            const float* w = wb + warp * H;
            float* c = cdf + warp * H;
            const int seg = (H + 31) / 32;
            const int lo = min(lane * seg, H), hi = min(lo + seg, H);
            double local = 0.0;
            for (int h = lo; h < hi; ++h) local = __dadd_rn(local, (double)w[h]);
            double v = local;
            #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v = __dadd_rn(n, v);
            }
            double run = __shfl_up_sync(0xffffffffu, v, 1);
            if (lane == 0) run = 0.0;
            for (int h = lo; h < hi; ++h) {
                run = __dadd_rn(run, (double)w[h]);
                c[h] = __double2float_rn(run);
            }
            if (lane == 31) zd[warp] = run;
        }
        // ---- per seat and card: the mass of the hands holding the card, in hand-id order
        for (int idx = tid; idx < P * D; idx += RB_THREADS) {
            const int q = idx / D, c = idx - q * D;
            const float* w = wb + q * H;
            double m = 0.0;
            for (int a = 0; a < c; ++a) m = __dadd_rn(m, (double)w[pair_id(D, a, c)]);
            for (int b = c + 1; b < D; ++b) m = __dadd_rn(m, (double)w[pair_id(D, c, b)]);
            mass[idx] = m;
        }
        __syncthreads();

        // ---- samples
        const uint64_t ns = rng_namespace(seed[f], 0, COMPLETION);
        const int32_t* lev_row = level + f * P;
        const float* base_row = baseline + f * P;
        const float* amt_row = amount + f * strata;
        for (int i = tid; i < N; i += RB_THREADS) {
            double weight = 1.0;
            uint64_t dead = 0;
            int hand[MAXP];
            #pragma unroll
            for (int q = 0; q < MAXP; ++q) hand[q] = 0;
            for (int q = 0; q < P; ++q) {
                const float* w = wb + q * H;
                const float* c = cdf + q * H;
                const double* m = mass + q * D;
                const double z = zd[q];
                double s1 = 0.0, s2 = 0.0;
                for (uint64_t rest = dead; rest; rest &= rest - 1) {
                    const int a = __ffsll((long long)rest) - 1;
                    s1 = __dadd_rn(s1, m[a]);
                    for (uint64_t r2 = rest & (rest - 1); r2; r2 &= r2 - 1)
                        s2 = __dadd_rn(s2, (double)w[pair_id(D, a, __ffsll((long long)r2) - 1)]);
                }
                const double zs = __dadd_rn(__dsub_rn(z, s1), s2);
                if (!(z > 0.0) || !(zs > 0.0)) {
                    weight = 0.0;
                    break;
                }
                weight = __dmul_rn(weight, __ddiv_rn(zs, z));
                int pick = -1;
                const float top = c[H - 1];
                if (top > 0.0f) {
                    const float below = __int_as_float(__float_as_int(top) - 1);  // nextafter(top, 0)
                    for (int a = 0; a < RB_ATTEMPTS; ++a) {
                        const float u = key_uniform(rng_key(ns, i, 0, a, q, 0));
                        const float t = fminf(__fmul_rn(u, top), below);
                        int lo = 0, hi = H;
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (c[mid] > t) hi = mid;
                            else lo = mid + 1;
                        }
                        if (lo >= H) lo = H - 1;
                        const bool clash = ((dead >> hc[2 * lo]) | (dead >> hc[2 * lo + 1])) & 1ull;
                        if (!clash && w[lo] > 0.0f) {
                            pick = lo;
                            break;
                        }
                    }
                }
                if (pick < 0) {  // exact scan of the restricted range
                    const double t = __dmul_rn((double)key_uniform(rng_key(ns, i, 0, RB_ATTEMPTS, q, 0)), zs);
                    double run = 0.0;
                    for (int h = 0; h < H; ++h) {
                        const float x = w[h];
                        if (!(x > 0.0f)) continue;
                        if (((dead >> hc[2 * h]) | (dead >> hc[2 * h + 1])) & 1ull) continue;
                        run = __dadd_rn(run, (double)x);
                        pick = h;
                        if (run > t) break;
                    }
                }
                if (pick < 0) {
                    weight = 0.0;
                    break;
                }
                hand[q] = pick;
                dead |= (1ull << hc[2 * pick]) | (1ull << hc[2 * pick + 1]);
            }
            float ret[MAXP];
            #pragma unroll
            for (int p = 0; p < MAXP; ++p) ret[p] = 0.0f;
            if (weight > 0.0) {
                uint64_t used = bmask | dead;
                HandCounts on_board;
                #pragma unroll
                for (int j = 0; j < 5; ++j) {
                    int card = bc[j];
                    if (card == PAD_CARD) {
                        const uint64_t avail = deck & ~used;
                        const int n = __popcll(avail);
                        const float u = key_uniform(rng_key(ns, i, 1, j, 0, 0));
                        int k = (int)__fmul_rn(u, (float)n);
                        if (k >= n) k = n - 1;
                        uint64_t r = avail;
                        for (; k > 0; --k) r &= r - 1;
                        const int local = __ffsll((long long)r) - 1;
                        used |= 1ull << local;
                        card = local + first;
                    }
                    on_board.add(card);
                }
                int64_t value[MAXP];
                int lev[MAXP];
                #pragma unroll
                for (int p = 0; p < MAXP; ++p) {
                    if (p >= P) break;
                    lev[p] = lev_row[p];
                    value[p] = -1;
                    if (lev[p] >= 0) {
                        HandCounts hv = on_board;
                        hv.add(hc[2 * hand[p]] + first);
                        hv.add(hc[2 * hand[p] + 1] + first);
                        value[p] = hand_value(hv, S, R);
                    }
                    ret[p] = base_row[p];
                }
                settle_strata(P, strata, value, lev, amt_row, ret);
            }
            rw[i] = weight;
            #pragma unroll
            for (int p = 0; p < MAXP; ++p) {
                if (p >= P) break;
                rh[i * P + p] = (uint16_t)hand[p];
                rr[i * P + p] = ret[p];
            }
        }
        __syncthreads();

        // ---- scales: 2^ew > max weight, 2^er > max |return| (maxima are order-free)
        double mw = 0.0, mr = 0.0;
        for (int i = tid; i < N; i += RB_THREADS) {
            const double x = rw[i];
            if (!(x > 0.0)) continue;
            mw = fmax(mw, x);
            for (int p = 0; p < P; ++p) mr = fmax(mr, fabs((double)rr[i * P + p]));
        }
        mw = warp_max_double(mw);
        mr = warp_max_double(mr);
        if (lane == 0) {
            red[warp] = mw;
            red[RB_WARPS + warp] = mr;
        }
        __syncthreads();
        mw = 0.0;
        mr = 0.0;
        for (int k = 0; k < RB_WARPS; ++k) {
            mw = fmax(mw, red[k]);
            mr = fmax(mr, red[RB_WARPS + k]);
        }
        int ew = 0, er = 0;
        frexp(mw, &ew);
        frexp(mr, &er);
        const int Q = 61 - ceil_log2(N);
        // ---- sum q and sum q^2 (thread-strided partial sums, warp butterfly, warps in order)
        long long wsum = 0;
        double sq = 0.0;
        for (int i = tid; i < N; i += RB_THREADS) {
            const long long qi = __double2ll_rn(ldexp(rw[i], Q - ew));
            wsum += qi;
            const double qd = (double)qi;
            sq = __dadd_rn(sq, __dmul_rn(qd, qd));
        }
        wsum = warp_sum_ll(wsum);
        sq = warp_butterfly_double(sq);
        if (lane == 0) {
            red_ll[2 * RB_WARPS + warp] = wsum;
            red[3 * RB_WARPS + warp] = sq;
        }
        __syncthreads();
        long long W = 0;
        double S2 = 0.0;
        for (int k = 0; k < RB_WARPS; ++k) {
            W += red_ll[2 * RB_WARPS + k];
            S2 = __dadd_rn(S2, red[3 * RB_WARPS + k]);
        }
        const double Wd = (double)W;

        // ---- per published seat: fixed-point occurrence and return sums, then the estimates
        for (int o = 0; o < outputs; ++o) {
            const int p = selected ? sel : o;
            for (int h = tid; h < 2 * H; h += RB_THREADS) acc[h] = 0ull;
            __syncthreads();
            for (int i = tid; i < N; i += RB_THREADS) {
                const double x = rw[i];
                if (!(x > 0.0)) continue;
                const long long qi = __double2ll_rn(ldexp(x, Q - ew));
                const long long mi = __double2ll_rn(ldexp(__dmul_rn(x, (double)rr[i * P + p]), Q - ew - er));
                const int h = rh[i * P + p];
                atomicAdd(&acc[h], (unsigned long long)qi);
                atomicAdd(&acc[H + h], (unsigned long long)mi);
            }
            __syncthreads();
            float* po = p_hat + (f * outputs + o) * (int64_t)H;
            float* vo = v_hat + (f * outputs + o) * (int64_t)H;
            for (int h = tid; h < H; h += RB_THREADS) {
                const long long a = (long long)acc[h], b = (long long)acc[H + h];
                __stcs(po + h, W > 0 ? __double2float_rn(__ddiv_rn((double)a, Wd)) : 0.0f);
                __stcs(vo + h, a != 0 ? __double2float_rn(ldexp(__ddiv_rn((double)b, (double)a), er)) : 0.0f);
            }
            __syncthreads();
        }
        if (tid == 0) {
            n_eff[f] = W > 0 ? __double2float_rn(fmin(__ddiv_rn(__dmul_rn(Wd, Wd), S2), (double)N)) : 0.0f;
            if (W <= 0) atomicOr(status, RB_NO_MASS);
        }
    }
}

int64_t rb_smem(int P, int D, int N) { return rb_layout(P, D * (D - 1) / 2, D, N).total; }

}  // namespace
}  // namespace pbg

using namespace pbg;

extern "C" {

int32_t pbg_rb_complete_max_samples(int32_t rank_count, int32_t P) {
    if (rank_count < 4 || rank_count > 13 || P < 2 || P > MAXP) return 0;
    const int D = 4 * rank_count;
    int32_t lo = 0, hi = 1 << 16;
    while (lo < hi) {  // largest N whose tables fit one CTA's shared memory
        const int32_t mid = (lo + hi + 1) / 2;
        if (rb_smem(P, D, mid) <= RB_SMEM_MAX) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

int pbg_rb_complete(int32_t rank_count, int64_t F, int32_t P, int32_t strata, int32_t n_samples,
                    const uint8_t* board, const float* range_weights, const int32_t* level, const float* baseline,
                    const float* amount, const int64_t* seed, const int32_t* selected, float* p_hat, float* v_hat,
                    float* n_eff, uint32_t* status, void* stream) {
    PBG_REQUIRE(rank_count >= 4 && rank_count <= 13, "rb_complete: rank_count must be in [4,13]");
    PBG_REQUIRE(P >= 2 && P <= MAXP && strata >= 1 && F >= 0, "rb_complete: bad shape");
    const int D = 4 * rank_count;
    PBG_REQUIRE(2 * P + 5 <= D, "rb_complete: %d seats and a five-card board do not fit a %d-card deck", P, D);
    PBG_REQUIRE(n_samples >= 1, "rb_complete: n_samples must be positive");
    const int32_t cap = pbg_rb_complete_max_samples(rank_count, P);
    PBG_REQUIRE(n_samples <= cap, "rb_complete: n_samples %d exceeds %d, the most one leaf's sample records hold",
                n_samples, cap);
    PBG_REQUIRE(board && range_weights && level && baseline && amount && seed && p_hat && v_hat && n_eff && status,
                "rb_complete: null argument");
    if (F == 0) return PBG_OK;
    const int64_t smem = rb_smem(P, D, n_samples);
    int err = cuda_status(cudaFuncSetAttribute(rb_complete_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem), "rb_complete: shared memory");
    if (err) return err;
    int per_sm = 0;
    err = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rb_complete_kernel, RB_THREADS,
                                                                    (size_t)smem), "rb_complete: occupancy");
    if (err) return err;
    if (per_sm < 1) per_sm = 1;
    const int64_t cap_grid = (int64_t)sm_count() * per_sm;
    const int grid = (int)(F < cap_grid ? F : cap_grid);
    rb_complete_kernel<<<grid, RB_THREADS, smem, as_stream(stream)>>>(
        category_strength(rank_count), rank_count, D, 52 - D, F, P, strata, n_samples, board, range_weights, level,
        baseline, amount, seed, selected, p_hat, v_hat, n_eff, status);
    return launch_status("rb_complete");
}

}  // extern "C"
