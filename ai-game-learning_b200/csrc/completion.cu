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
// A seat's draw is up to RB_ATTEMPTS proposals from its fp32 CDF (searched
// through a guide table, two proposals at a time), keeping the first one
// disjoint from `dead` (exactly the restricted law), then one exact scan of
// the restricted range.  The normalisers' sums are built incrementally: each
// drawn hand adds its terms to the accumulators of every later seat, in the
// order the definition fixes.  The missing board cards are dealt uniformly from the
// unused deck, and the returns follow the contract-v2 stratum settlement
// (showdown.cuh).  Every draw is addressed by (row seed, sample, draw code)
// through the counter hash, so results do not depend on the launch shape.
//
// Estimates are reduced in 64-bit fixed point (integer sums are associative,
// so the shared-memory atomics are deterministic): q_i = rint(w_i 2^(Q-e_w)),
// m_i,p = rint(w_i R_i,p 2^(Q-e_w-e_R)) with 2^e_w > max w and 2^e_R > max|R|;
// p_hat = float(sum q) * float(1 / W), W = sum q, and v_hat = float(sum m) *
// rcp(float(sum q)) * 2^e_R over the samples that drew hand h (single precision
// from the integer sums on); n_eff = W^2 / sum q^2 (at most n_samples).
//
// One persistent CTA per leaf row (256 threads, or 512 when the sample records
// leave room for one CTA per SM only), all tables in shared memory: the hand ->
// card table (once per CTA), the board-masked range [P,Hp] f32 (Hp = H rounded
// up to 4), its CDF [P,Hp] f32 (the two reused, after sampling, as the 64-bit
// accumulators of a few seats at a time, kept as 32-bit halves), the guide tables [P,RB_GUIDE+1] u16,
// per-card masses [P,D] f64, the sample records (weight f64, hands u16 [P],
// returns f32 [P]) and each thread's current cards.  Rows with an invalid board card or selected seat set *status bit 1
// and publish zeros; rows whose every sample has weight 0 (a seat without
// board-legal mass) set bit 2 and publish n_eff = 0.
#include <cfloat>

#include "showdown.cuh"

namespace pbg {
namespace {

constexpr int RB_ATTEMPTS = 16;  // proposals per seat before the exact scan (even: drawn in pairs)
constexpr int RB_GUIDE = 128;    // guide buckets per seat (a power of two)
constexpr int RB_SEG4 = 11;      // float4 chunks of one lane's CDF segment (H <= 1326)
constexpr int RB_PARTIALS = 256; // n_eff's sum of squares: partial sums over samples i = p mod 256
constexpr uint32_t RB_BAD_INPUT = 1u, RB_NO_MASS = 2u;
constexpr int64_t RB_SMEM_MAX = 227 * 1024;
constexpr int64_t RB_SMEM_TWO = 112 * 1024;  // two CTAs of this size share one SM

struct RBLayout {
    int64_t hc, wb, cdf, guide, mass, zd, rw, rh, rr, sc, red, total;
};

__host__ __device__ __forceinline__ int64_t align16(int64_t x) { return (x + 15) & ~(int64_t)15; }
__host__ __device__ __forceinline__ int padded_hands(int H) { return (H + 3) & ~3; }

__host__ __device__ __forceinline__ RBLayout rb_layout(int P, int H, int D, int N, int threads) {
    RBLayout L;
    const int64_t Hp = padded_hands(H);
    int64_t o = 0;
    L.hc = o;
    o = align16(o + 2 * (int64_t)H);
    L.wb = o;
    o = align16(o + 4 * (int64_t)P * Hp);
    L.cdf = o;
    const int64_t cdf_bytes = 4 * (int64_t)P * Hp, acc_bytes = 16 * (int64_t)H;
    o = align16(o + (cdf_bytes > acc_bytes ? cdf_bytes : acc_bytes));
    L.guide = o;
    o = align16(o + 2 * (int64_t)P * (RB_GUIDE + 1));
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
    L.sc = o;
    o = align16(o + 2 * MAXP * (int64_t)threads);
    L.red = o;
    o = align16(o + 8 * 4 * (threads / 32));
    L.total = o;
    return L;
}

// Lexicographic id of the local card pair {a, b} (a != b) in a deck of D cards.
__device__ __forceinline__ int pair_id(int D, int a, int b) {
    const int lo = min(a, b), hi = max(a, b);
    return lo * (2 * D - lo - 1) / 2 + hi - lo - 1;
}

__device__ __forceinline__ int ceil_log2(int n) {
    int k = 0;
    while ((1 << k) < n) ++k;
    return k;
}

// 2^e as a double, exact for e in [-1022, 1023].
__device__ __forceinline__ double pow2(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

// rint(x * 2^e) as an integer (ldexp is exact; the product by a representable 2^e is the same number).
__device__ __forceinline__ long long scaled_rint(double x, int e) {
    return __double2ll_rn(e <= 1023 && e >= -1022 ? __dmul_rn(x, pow2(e)) : ldexp(x, e));
}

// The uniform of draw `code` of a sample whose base key is `base`.
__device__ __forceinline__ float draw_uniform(int64_t base, int code) {
    return key_uniform(mix63((int64_t)(((uint64_t)base + (uint64_t)(code + 1) * 0x9E3779B97F4A7C15ULL) & M63)));
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

// 64-bit integer addition on a (low, high) pair of 32-bit shared words: native 32-bit atomics
// with the carry of the low word (integer sums: the result does not depend on the order).
__device__ __forceinline__ void atomic_add_split(unsigned* lo, unsigned* hi, unsigned long long v) {
    const unsigned vlo = (unsigned)v, vhi = (unsigned)(v >> 32);
    const unsigned old = atomicAdd(lo, vlo);
    const unsigned carry = (old + vlo < old) ? 1u : 0u;
    if (vhi + carry) atomicAdd(hi, vhi + carry);
}

template <int T>
__global__ void __launch_bounds__(T, 512 / T)
rb_complete_kernel(CategoryOrder O, int R, int D, int first, int64_t F, int P, int strata, int N,
                   const uint8_t* __restrict__ board, const float* __restrict__ weights,
                   const int32_t* __restrict__ level, const float* __restrict__ baseline,
                   const float* __restrict__ amount, const int64_t* __restrict__ seed,
                   const int32_t* __restrict__ selected, float* __restrict__ p_hat, float* __restrict__ v_hat,
                   float* __restrict__ n_eff, uint32_t* __restrict__ status) {
    constexpr int WARPS = T / 32;
    extern __shared__ __align__(16) unsigned char smem[];
    const int H = D * (D - 1) / 2, Hp = padded_hands(H);
    const RBLayout L = rb_layout(P, H, D, N, T);
    uint16_t* hc = reinterpret_cast<uint16_t*>(smem + L.hc);  // local cards c0 | c1 << 8
    float* wb = reinterpret_cast<float*>(smem + L.wb);
    float* cdf = reinterpret_cast<float*>(smem + L.cdf);
    uint16_t* guide = reinterpret_cast<uint16_t*>(smem + L.guide);
    double* mass = reinterpret_cast<double*>(smem + L.mass);
    double* zd = reinterpret_cast<double*>(smem + L.zd);
    double* rw = reinterpret_cast<double*>(smem + L.rw);
    uint16_t* rh = reinterpret_cast<uint16_t*>(smem + L.rh);
    float* rr = reinterpret_cast<float*>(smem + L.rr);
    uint8_t* sc = smem + L.sc + threadIdx.x;  // this thread's sample cards, [2 * MAXP] at stride T
    double* red = reinterpret_cast<double*>(smem + L.red);
    long long* red_ll = reinterpret_cast<long long*>(smem + L.red);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t deck = (1ull << D) - 1ull;  // D <= 52
    const int outputs = selected ? 1 : P;

    for (int h = tid; h < H; h += T) {
        int c0, c1;
        combo_cards(D, 0, h, c0, c1);
        hc[h] = (uint16_t)(c0 | (c1 << 8));
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
            for (int64_t k = tid; k < (int64_t)outputs * H; k += T) {
                p_hat[f * outputs * H + k] = 0.0f;
                v_hat[f * outputs * H + k] = 0.0f;
            }
            if (tid == 0) {
                n_eff[f] = 0.0f;
                atomicOr(status, RB_BAD_INPUT);
            }
            continue;
        }

        // ---- board-masked range weights (non-positive and non-finite weigh 0); H is even, so the
        //      row is read as float2 pairs of one seat, eight loads in flight per thread
        {
            const float2* src = reinterpret_cast<const float2*>(weights + f * (int64_t)P * H);
            const int pairs = P * H / 2;
            for (int k0 = tid; k0 < pairs; k0 += 8 * T) {
                float2 v[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int k = k0 + u * T;
                    v[u] = k < pairs ? __ldg(src + k) : make_float2(0.0f, 0.0f);
                }
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int k = k0 + u * T;
                    if (k >= pairs) break;
                    const int q = (2 * k) / H, h = 2 * k - q * H;
                    const unsigned c01 = hc[h], c23 = hc[h + 1];
                    const bool x0 = ((bmask >> (c01 & 0xFF)) | (bmask >> (c01 >> 8))) & 1ull;
                    const bool x1 = ((bmask >> (c23 & 0xFF)) | (bmask >> (c23 >> 8))) & 1ull;
                    wb[q * Hp + h] = (v[u].x > 0.0f && v[u].x <= FLT_MAX && !x0) ? v[u].x : 0.0f;
                    wb[q * Hp + h + 1] = (v[u].y > 0.0f && v[u].y <= FLT_MAX && !x1) ? v[u].y : 0.0f;
                }
            }
            for (int k = tid; k < P * (Hp - H); k += T) wb[(k / (Hp - H)) * Hp + H + k % (Hp - H)] = 0.0f;
        }
        __syncthreads();

        // ---- per seat: fp32 CDF from a double running sum (warp q: each lane a contiguous segment
        //      of `seg` hands, seg = ceil(H / 32) rounded up to 4; segment bases from an inclusive
        //      warp scan of the segment totals)
        if (warp < P) {
            const float* w = wb + warp * Hp;
            float* c = cdf + warp * Hp;
            const int seg = (((H + 31) / 32) + 3) & ~3;
            const int lo = min(lane * seg, H), hi = min(lo + seg, H);
            double local = 0.0;
            #pragma unroll
            for (int u = 0; u < RB_SEG4; ++u) {
                if (lo + 4 * u >= hi) break;
                const float4 x = *reinterpret_cast<const float4*>(w + lo + 4 * u);
                local = __dadd_rn(local, (double)x.x);
                local = __dadd_rn(local, (double)x.y);
                local = __dadd_rn(local, (double)x.z);
                local = __dadd_rn(local, (double)x.w);
            }
            double v = local;
            #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v = __dadd_rn(n, v);
            }
            double run = __shfl_up_sync(0xffffffffu, v, 1);
            if (lane == 0) run = 0.0;
            #pragma unroll
            for (int u = 0; u < RB_SEG4; ++u) {
                if (lo + 4 * u >= hi) break;
                const float4 x = *reinterpret_cast<const float4*>(w + lo + 4 * u);
                float4 y;
                run = __dadd_rn(run, (double)x.x);
                y.x = __double2float_rn(run);
                run = __dadd_rn(run, (double)x.y);
                y.y = __double2float_rn(run);
                run = __dadd_rn(run, (double)x.z);
                y.z = __double2float_rn(run);
                run = __dadd_rn(run, (double)x.w);
                y.w = __double2float_rn(run);
                *reinterpret_cast<float4*>(c + lo + 4 * u) = y;  // entries past H land in the padding
            }
            if (lane == 31) zd[warp] = run;
        }
        // ---- per seat and card: the mass of the hands holding the card, in hand-id order
        for (int idx = tid; idx < P * D; idx += T) {
            const int q = idx / D, c = idx - q * D;
            const float* w = wb + q * Hp;
            // the hands holding c in increasing id, t = 0..D-2: {t, c} for t < c, then {c, t + 1}; four
            // running sums (terms t = 0, 1, 2, 3 mod 4, each in order), then (s0 + s1) + (s2 + s3)
            const int row = c * (2 * D - c - 1) / 2 - c - 1;
            double part[4] = {0.0, 0.0, 0.0, 0.0};
            for (int t0 = 0; t0 < D - 1; t0 += 8) {
                float x[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = t0 + u;
                    const int id = t < c ? t * (2 * D - t - 1) / 2 + c - t - 1 : row + t + 1;
                    x[u] = t < D - 1 ? w[id] : 0.0f;
                }
                #pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (t0 + u < D - 1) part[u & 3] = __dadd_rn(part[u & 3], (double)x[u]);
            }
            mass[idx] = __dadd_rn(__dadd_rn(part[0], part[1]), __dadd_rn(part[2], part[3]));
        }
        __syncthreads();
        // ---- per seat: guide[k] = the first hand whose CDF exceeds (k / RB_GUIDE) * top, guide[RB_GUIDE] = H - 1
        for (int idx = tid; idx < P * (RB_GUIDE + 1); idx += T) {
            const int q = idx / (RB_GUIDE + 1), k = idx - q * (RB_GUIDE + 1);
            const float* c = cdf + q * Hp;
            const float top = c[H - 1];
            int lo = H - 1;
            if (k < RB_GUIDE && top > 0.0f) {
                const float thr = __fmul_rn((float)k * (1.0f / RB_GUIDE), top);
                int hi = H - 1;
                lo = 0;
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (c[mid] > thr) hi = mid;
                    else lo = mid + 1;
                }
            }
            guide[idx] = (uint16_t)lo;
        }
        __syncthreads();

        // ---- samples
        const uint64_t ns = rng_namespace(seed[f], 0, COMPLETION);
        const int32_t* lev_row = level + f * P;
        const float* base_row = baseline + f * P;
        const float* amt_row = amount + f * strata;
        for (int i = tid; i < N; i += T) {
            const int64_t key = rng_key(ns, i, 0, 0, 0, 0);
            double weight = 1.0;
            uint64_t dead = 0;
            // each later seat's normaliser sums: s1 = the dead cards' masses, s2 = the dead pairs' weights
            double s1[MAXP], s2[MAXP];
            #pragma unroll
            for (int q = 0; q < MAXP; ++q) {
                s1[q] = 0.0;
                s2[q] = 0.0;
            }
            int seated = 0;
            #pragma unroll 1
            for (int q = 0; q < P; ++q) {
                const float* w = wb + q * Hp;
                const float* c = cdf + q * Hp;
                const double z = zd[q];
                double s1q = 0.0, s2q = 0.0;
                #pragma unroll
                for (int r = 0; r < MAXP; ++r)
                    if (r == q) {
                        s1q = s1[r];
                        s2q = s2[r];
                    }
                // Z(dead) = (Z - sum of the dead cards' masses) + the weights of the dead-card pairs
                const double zs = __dadd_rn(__dsub_rn(z, s1q), s2q);
                if (!(z > 0.0) || !(zs > 0.0)) {
                    weight = 0.0;
                    break;
                }
                weight = __dmul_rn(weight, __ddiv_rn(zs, z));
                int pick = -1;
                const float top = c[H - 1];
                if (top > 0.0f) {
                    const float below = __int_as_float(__float_as_int(top) - 1);  // nextafter(top, 0)
                    const uint16_t* g = guide + q * (RB_GUIDE + 1);
                    for (int a = 0; a < RB_ATTEMPTS && pick < 0; a += 2) {
                        // two proposals searched together: the first entries above t0 and t1
                        const float u0 = draw_uniform(key, q * 32 + a), u1 = draw_uniform(key, q * 32 + a + 1);
                        const float t0 = fminf(__fmul_rn(u0, top), below), t1 = fminf(__fmul_rn(u1, top), below);
                        const int k0 = (int)__fmul_rn(u0, (float)RB_GUIDE), k1 = (int)__fmul_rn(u1, (float)RB_GUIDE);
                        int lo0 = g[k0], hi0 = g[k0 + 1], lo1 = g[k1], hi1 = g[k1 + 1];
                        while (lo0 < hi0 || lo1 < hi1) {
                            const int m0 = (lo0 + hi0) >> 1, m1 = (lo1 + hi1) >> 1;
                            const float c0 = c[m0], c1 = c[m1];
                            if (lo0 < hi0) {
                                if (c0 > t0) hi0 = m0;
                                else lo0 = m0 + 1;
                            }
                            if (lo1 < hi1) {
                                if (c1 > t1) hi1 = m1;
                                else lo1 = m1 + 1;
                            }
                        }
                        const unsigned cc0 = hc[lo0], cc1 = hc[lo1];
                        const bool ok0 = !(((dead >> (cc0 & 0xFF)) | (dead >> (cc0 >> 8))) & 1ull) && w[lo0] > 0.0f;
                        const bool ok1 = !(((dead >> (cc1 & 0xFF)) | (dead >> (cc1 >> 8))) & 1ull) && w[lo1] > 0.0f;
                        pick = ok0 ? lo0 : (ok1 ? lo1 : -1);
                    }
                }
                if (pick < 0) {  // exact scan of the restricted range
                    const double t = __dmul_rn((double)draw_uniform(key, q * 32 + RB_ATTEMPTS), zs);
                    double run = 0.0;
                    for (int h = 0; h < H; ++h) {
                        const float x = w[h];
                        if (!(x > 0.0f)) continue;
                        const unsigned cc = hc[h];
                        if (((dead >> (cc & 0xFF)) | (dead >> (cc >> 8))) & 1ull) continue;
                        run = __dadd_rn(run, (double)x);
                        pick = h;
                        if (run > t) break;
                    }
                }
                if (pick < 0) {
                    weight = 0.0;
                    break;
                }
                const unsigned cc = hc[pick];
                const int aj = cc & 0xFF, bj = cc >> 8;
                rh[i * P + q] = (uint16_t)pick;
                sc[(2 * q) * T] = (uint8_t)aj;
                sc[(2 * q + 1) * T] = (uint8_t)bj;
                dead |= (1ull << aj) | (1ull << bj);
                seated = q + 1;
                // the drawn hand's terms, added to every later seat's sums in the defined order:
                // its two cards' masses; its own pair, then its cross pairs with the earlier hands
                #pragma unroll
                for (int r = 1; r < MAXP; ++r) {
                    if (r <= q || r >= P) continue;
                    const float* wr = wb + r * Hp;
                    const double* mr = mass + r * D;
                    s1[r] = __dadd_rn(__dadd_rn(s1[r], mr[aj]), mr[bj]);
                    double x = __dadd_rn(s2[r], (double)wr[pick]);
                    for (int k = 0; k < q; ++k) {
                        const int ak = sc[(2 * k) * T], bk = sc[(2 * k + 1) * T];
                        x = __dadd_rn(x, (double)wr[pair_id(D, ak, aj)]);
                        x = __dadd_rn(x, (double)wr[pair_id(D, ak, bj)]);
                        x = __dadd_rn(x, (double)wr[pair_id(D, bk, aj)]);
                        x = __dadd_rn(x, (double)wr[pair_id(D, bk, bj)]);
                    }
                    s2[r] = x;
                }
            }
            for (int q = seated; q < P; ++q) rh[i * P + q] = 0;
            float ret[MAXP];
            #pragma unroll
            for (int p = 0; p < MAXP; ++p) ret[p] = 0.0f;
            if (weight > 0.0) {
                uint64_t used = bmask | dead;
                HandCounts on_board;
                #pragma unroll
                for (int j = 0; j < 5; ++j) {
                    int card = bc[j];
                    if (card == PAD_CARD) {  // the k-th unused card, k uniform
                        const uint64_t avail = deck & ~used;
                        const unsigned lo32 = (unsigned)avail, hi32 = (unsigned)(avail >> 32);
                        const int n_lo = __popc(lo32), n = n_lo + __popc(hi32);
                        int k = (int)__fmul_rn(draw_uniform(key, 1024 + j), (float)n);
                        if (k >= n) k = n - 1;
                        const int local = k < n_lo ? (int)__fns(lo32, 0, k + 1) : 32 + (int)__fns(hi32, 0, k - n_lo + 1);
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
                        hv.add(sc[(2 * p) * T] + first);
                        hv.add(sc[(2 * p + 1) * T] + first);
                        value[p] = hand_order(hv, O, R);
                    }
                    ret[p] = base_row[p];
                }
                settle_strata(P, strata, value, lev, amt_row, ret);
            }
            rw[i] = weight;
            #pragma unroll
            for (int p = 0; p < MAXP; ++p) {
                if (p >= P) break;
                rr[i * P + p] = ret[p];
            }
        }
        __syncthreads();

        // ---- scales: 2^ew > max weight, 2^er > max |return| (maxima are order-free); the publish
        //      accumulators (`group` seats of [4][H] words over the range and CDF tables) start at 0
        const int group = min(outputs, max(1, (int)((L.guide - L.wb) / (16 * (int64_t)H))));
        unsigned* accum = reinterpret_cast<unsigned*>(smem + L.wb);
        for (int k = tid; k < group * 4 * H; k += T) accum[k] = 0u;
        double mw = 0.0, mr = 0.0;
        for (int i = tid; i < N; i += T) {
            const double x = rw[i];
            if (!(x > 0.0)) continue;
            mw = fmax(mw, x);
            for (int p = 0; p < P; ++p) mr = fmax(mr, fabs((double)rr[i * P + p]));
        }
        mw = warp_max_double(mw);
        mr = warp_max_double(mr);
        if (lane == 0) {
            red[warp] = mw;
            red[WARPS + warp] = mr;
        }
        __syncthreads();
        mw = 0.0;
        mr = 0.0;
        for (int k = 0; k < WARPS; ++k) {
            mw = fmax(mw, red[k]);
            mr = fmax(mr, red[WARPS + k]);
        }
        int ew = 0, er = 0;
        frexp(mw, &ew);
        frexp(mr, &er);
        const int Q = 61 - ceil_log2(N);
        // ---- sum q and sum q^2: RB_PARTIALS partial sums over i = p mod RB_PARTIALS, a butterfly
        //      within each warp of them, then those warps in order
        long long wsum = 0;
        double sq = 0.0;
        if (tid < RB_PARTIALS) {
            for (int i = tid; i < N; i += RB_PARTIALS) {
                const double x = rw[i];
                const long long qi = x > 0.0 ? scaled_rint(x, Q - ew) : 0;
                wsum += qi;
                const double qd = (double)qi;
                sq = __dadd_rn(sq, __dmul_rn(qd, qd));
            }
        }
        wsum = warp_sum_ll(wsum);
        sq = warp_butterfly_double(sq);
        if (lane == 0) {
            red_ll[2 * WARPS + warp] = wsum;
            red[3 * WARPS + warp] = sq;
        }
        __syncthreads();
        long long W = 0;
        double S2 = 0.0;
        for (int k = 0; k < RB_PARTIALS / 32; ++k) {
            W += red_ll[2 * WARPS + k];
            S2 = __dadd_rn(S2, red[3 * WARPS + k]);
        }
        const double Wd = (double)W;
        const float inv_w = W > 0 ? __double2float_rn(__ddiv_rn(1.0, Wd)) : 0.0f;
        const float scale_r = ldexpf(1.0f, min(er, 127));  // exact: |returns| < 2^er

        // ---- per published seat, `group` seats per pass: fixed-point occurrence and return sums
        //      ([4][H] words per seat: occurrence low/high, return low/high), then the estimates;
        //      the output loop resets the words it read
        for (int o0 = 0; o0 < outputs; o0 += group) {
            const int g_end = min(group, outputs - o0);
            for (int i = tid; i < N; i += T) {
                const double x = rw[i];
                if (!(x > 0.0)) continue;
                const long long qi = scaled_rint(x, Q - ew);
                for (int g = 0; g < g_end; ++g) {
                    const int p = selected ? sel : o0 + g;
                    unsigned* a = accum + g * 4 * H;
                    const long long mi = scaled_rint(__dmul_rn(x, (double)rr[i * P + p]), Q - ew - er);
                    const int h = rh[i * P + p];
                    atomic_add_split(a + h, a + H + h, (unsigned long long)qi);
                    atomic_add_split(a + 2 * H + h, a + 3 * H + h, (unsigned long long)mi);
                }
            }
            __syncthreads();
            for (int g = 0; g < g_end; ++g) {
                unsigned* a = accum + g * 4 * H;
                float* po = p_hat + (f * outputs + o0 + g) * (int64_t)H;
                float* vo = v_hat + (f * outputs + o0 + g) * (int64_t)H;
                #pragma unroll 4
                for (int h = tid; h < H; h += T) {
                    const long long n = (long long)(((unsigned long long)a[H + h] << 32) | a[h]);
                    float pv = 0.0f, vv = 0.0f;
                    if (n != 0) {  // single precision from here: n and m rounded to float once each
                        const long long m = (long long)(((unsigned long long)a[3 * H + h] << 32) | a[2 * H + h]);
                        const float nf = __ll2float_rn(n), mf = __ll2float_rn(m);
                        pv = __fmul_rn(nf, inv_w);
                        vv = __fmul_rn(__fmul_rn(mf, __frcp_rn(nf)), scale_r);
                        a[h] = a[H + h] = a[2 * H + h] = a[3 * H + h] = 0u;
                    }
                    __stcs(po + h, pv);
                    __stcs(vo + h, vv);
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            n_eff[f] = W > 0 ? __double2float_rn(fmin(__ddiv_rn(__dmul_rn(Wd, Wd), S2), (double)N)) : 0.0f;
            if (W <= 0) atomicOr(status, RB_NO_MASS);
        }
    }
}

int64_t rb_smem(int P, int D, int N, int threads) { return rb_layout(P, D * (D - 1) / 2, D, N, threads).total; }

// 256 threads while two CTAs fit one SM, else 512 (one CTA per SM, twice the warps).
int rb_threads(int P, int D, int N) { return rb_smem(P, D, N, 256) <= RB_SMEM_TWO ? 256 : 512; }

template <int T>
int launch_rb(int64_t smem, int rank_count, int D, int64_t F, int P, int strata, int N, const uint8_t* board,
              const float* range_weights, const int32_t* level, const float* baseline, const float* amount,
              const int64_t* seed, const int32_t* selected, float* p_hat, float* v_hat, float* n_eff,
              uint32_t* status, cudaStream_t stream) {
    int err = cuda_status(cudaFuncSetAttribute(rb_complete_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem), "rb_complete: shared memory");
    if (err) return err;
    int per_sm = 0;
    err = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rb_complete_kernel<T>, T, (size_t)smem),
                      "rb_complete: occupancy");
    if (err) return err;
    if (per_sm < 1) per_sm = 1;
    const int64_t cap_grid = (int64_t)sm_count() * per_sm;
    const int grid = (int)(F < cap_grid ? F : cap_grid);
    rb_complete_kernel<T><<<grid, T, smem, stream>>>(category_order(rank_count), rank_count, D, 52 - D, F, P, strata,
                                                     N, board, range_weights, level, baseline, amount, seed, selected,
                                                     p_hat, v_hat, n_eff, status);
    return launch_status("rb_complete");
}

}  // namespace
}  // namespace pbg

using namespace pbg;

extern "C" {

int32_t pbg_rb_complete_max_samples(int32_t rank_count, int32_t P) {
    if (rank_count < 4 || rank_count > 13 || P < 2 || P > MAXP) return 0;
    const int D = 4 * rank_count;
    int32_t lo = 0, hi = 1 << 16;
    while (lo < hi) {  // largest N whose tables fit one 512-thread CTA's shared memory
        const int32_t mid = (lo + hi + 1) / 2;
        if (rb_smem(P, D, mid, 512) <= RB_SMEM_MAX) lo = mid;
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
    PBG_REQUIRE(((uintptr_t)range_weights & 7) == 0, "rb_complete: range_weights must be 8-byte aligned");
    if (F == 0) return PBG_OK;
    const int threads = rb_threads(P, D, n_samples);
    const int64_t smem = rb_smem(P, D, n_samples, threads);
    if (threads == 256)
        return launch_rb<256>(smem, rank_count, D, F, P, strata, n_samples, board, range_weights, level, baseline,
                              amount, seed, selected, p_hat, v_hat, n_eff, status, as_stream(stream));
    return launch_rb<512>(smem, rank_count, D, F, P, strata, n_samples, board, range_weights, level, baseline, amount,
                          seed, selected, p_hat, v_hat, n_eff, status, as_stream(stream));
}

}  // extern "C"
