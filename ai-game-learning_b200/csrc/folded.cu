// Multiway folded-range statistics: the finite-difference removal queries
// (pbg/games/poker/queued/folded.py:111-232, _phi_queries, evaluated by the
// reference in chunks of 64 queries over dense [B, Q, F, F, H] intermediates).
//
// For one decision row the estimator is evaluated on every removal query:
// query 0 removes no card, queries 1..C remove one card, queries C+1.. remove
// the card pair of private hand q-1-C (the triu order of folded.py:81-92 is the
// lexicographic hand order).  With at most two cards removed, every dense
// contraction of the reference collapses to lookups into the folder's hand
// probabilities (range matrix entry M[c][d] = p[hand(c, d)], diagonal zero):
//   linear_f       = m_f[a] + m_f[b]                 (m_f = row sums of M_f)
//   quadratic_f    = p_f[hand(a, b)]
//   surviving_f    = max(1 - linear_f + quadratic_f, tiny)
//   cond_f[c]      = (m_f[c] - M_f[c][a] - M_f[c][b]) * allowed[c] / surviving_f
//   delta_f[c]     = cond_f[c] - 2 / max(available, 1) * allowed[c]
// then phi = sum_f log surviving_f over folders, the packed-uniform terms, the
// pairwise disjointness terms (a C-wide dot product of conditional marginals
// and an H-wide sum over surviving hands per folder pair) and the triple
// cluster terms (an H-wide edge sum per tight pair and hub, plus C-wide
// diagonal / outer products).  Layout: one CTA per (decision, block of queries);
// the decision's probabilities [P][H], card marginals [P][C] and the hand ->
// card-pair table live in shared memory; each warp evaluates one query at a
// time with lanes over cards (two per lane) and over hands (strided), its
// conditional marginals and deltas in a per-warp shared scratch.  Output per
// query: phi + triple and triple, as _phi_queries returns them.
#include <cfloat>

#include "pbg_common.cuh"

namespace pbg {

constexpr int FD_MAXP = 6;     // NLHEGeometry seats (hooks.py:81-83)
constexpr int FD_MAXC = 52;
constexpr int FD_CPAD = 64;
constexpr int FD_WARPS = 8;
constexpr int FD_THREADS = 32 * FD_WARPS;
constexpr int FD_DENSE = 4;  // folders handled by the one-pass path
// pair s of four dense folder slots, (i < j) in lexicographic order, and the other two slots of the
// pair (its hubs, increasing): the seat order the reference accumulates pairs and hubs in.  Unrolled
// loops over s make these compile-time constants (register arrays stay in registers).
__device__ __forceinline__ constexpr int fd_pair_i(int s) { return s < 3 ? 0 : (s < 5 ? 1 : 2); }
__device__ __forceinline__ constexpr int fd_pair_j(int s) { return s < 3 ? s + 1 : (s < 5 ? s - 1 : 3); }
__device__ __forceinline__ constexpr int fd_hub(int s, int u) {
    // the u-th slot of {0, 1, 2, 3} outside {i, j}
    return u == 0 ? (fd_pair_i(s) == 0 ? (fd_pair_j(s) == 1 ? 2 : 1) : 0)
                  : (fd_pair_j(s) == 3 ? (fd_pair_i(s) == 2 ? 1 : 2) : 3);
}

__device__ __forceinline__ float fd_clamp_tiny(float x) {
    // torch's clamp_min: NaN passes through
    return x != x ? x : fmaxf(x, FLT_MIN);
}

__device__ __forceinline__ int fd_hand(int lo, int hi, int cards) {
    return lo * (2 * cards - lo - 1) / 2 + hi - lo - 1;
}

__device__ __forceinline__ float fd_pair(const float* __restrict__ p, int c, int d, int cards) {
    // range matrix entry M[c][d] (zero on the diagonal)
    if (c == d) return 0.0f;
    return c < d ? p[fd_hand(c, d, cards)] : p[fd_hand(d, c, cards)];
}

__device__ __forceinline__ float fd_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(FD_THREADS, 3)
folded_phi_kernel(int players, int cards, int hands, int queries, int queries_per_warp,
                  const float* __restrict__ probability, const uint8_t* __restrict__ folder_mask,
                  const uint8_t* __restrict__ tight_mask, const float* __restrict__ base_cards,
                  float* __restrict__ phi_out, float* __restrict__ triple_out) {
    extern __shared__ float4 fd_smem4[];
    __shared__ float fd_zero[FD_CPAD];  // the delta row of a slot that is not tight
    float* prob = reinterpret_cast<float*>(fd_smem4);                   // [P][H]
    float* marg = prob + players * hands;                                // [P][CPAD]
    uint16_t* comb = reinterpret_cast<uint16_t*>(marg + players * FD_CPAD);  // [H]: lo | hi << 8
    float* scratch = reinterpret_cast<float*>(comb + ((hands + 3) & ~3));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* cond = scratch + warp * 2 * FD_MAXP * FD_CPAD;                // [P][CPAD]
    float* delta = cond + FD_MAXP * FD_CPAD;                             // [P][CPAD]
    const int64_t row = blockIdx.y;

    unsigned fmask = 0, tmask = 0;
    for (int f = 0; f < players; ++f) {
        fmask |= (folder_mask[row * players + f] ? 1u : 0u) << f;
        tmask |= (tight_mask[row * players + f] ? 1u : 0u) << f;
    }
    const int folders = __popc(fmask);
    // the folders in seat order as dense slots, and which slots are tight
    int fseat[FD_DENSE] = {0, 0, 0, 0};
    unsigned dtight = 0;
    {
        int k = 0;
        for (int f = 0; f < players && k < FD_DENSE; ++f)
            if (fmask >> f & 1u) {
                fseat[k] = f;
                dtight |= (tmask >> f & 1u) << k;
                ++k;
            }
    }
    const float* src = probability + row * (int64_t)players * hands;
    for (int i = threadIdx.x; i < players * hands; i += FD_THREADS) prob[i] = src[i];
    if (threadIdx.x < FD_CPAD) fd_zero[threadIdx.x] = 0.0f;
    for (int h = threadIdx.x; h < hands; h += FD_THREADS) {
        int lo = 0;
        while (fd_hand(lo + 1, lo + 2, cards) <= h && lo + 2 < cards) ++lo;
        const int hi = h - fd_hand(lo, lo + 1, cards) + lo + 1;
        comb[h] = (uint16_t)(lo | (hi << 8));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < players * cards; i += FD_THREADS) {
        const int f = i / cards, c = i - f * cards;
        const float* pf = prob + f * hands;
        float s = 0.0f;
        for (int d = 0; d < cards; ++d) s += fd_pair(pf, c, d, cards);
        marg[f * FD_CPAD + c] = s;
    }
    __syncthreads();

    const float base = base_cards[row];
    const int first_query = (blockIdx.x * FD_WARPS + warp) * queries_per_warp;
    for (int k = 0; k < queries_per_warp; ++k) {
        const int q = first_query + k;
        if (q >= queries) break;
        int removed = 0, ra = -1, rb = -1;
        if (q >= 1 && q <= cards) {
            removed = 1;
            ra = q - 1;
        } else if (q > cards) {
            removed = 2;
            const uint16_t pr = comb[q - 1 - cards];
            ra = pr & 0xff;
            rb = pr >> 8;
        }
        const float available = base - (float)removed;
        const float flat = 2.0f / fmaxf(available, 1.0f);
        float surviving[FD_MAXP];
#pragma unroll
        for (int f = 0; f < FD_MAXP; ++f) {
            surviving[f] = 1.0f;
            if (f < players) {
                float linear = 0.0f, quadratic = 0.0f;
                if (removed >= 1) linear = marg[f * FD_CPAD + ra];
                if (removed == 2) {
                    linear = linear + marg[f * FD_CPAD + rb];
                    quadratic = prob[f * hands + fd_hand(ra, rb, cards)];
                }
                surviving[f] = fd_clamp_tiny((1.0f - linear) + quadratic);
            }
        }
        // conditional marginals and deltas of every seat, lanes over cards
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int c = lane + 32 * half;
            if (c < cards) {
                const float allowed = (c == ra || c == rb) ? 0.0f : 1.0f;
#pragma unroll
                for (int f = 0; f < FD_MAXP; ++f) {
                    if (f < players) {
                        const float* pf = prob + f * hands;
                        float column = 0.0f;
                        if (removed >= 1) column = fd_pair(pf, c, ra, cards);
                        if (removed == 2) column = column + fd_pair(pf, c, rb, cards);
                        const float cm = (marg[f * FD_CPAD + c] - column) * allowed / surviving[f];
                        cond[f * FD_CPAD + c] = cm;
                        delta[f * FD_CPAD + c] = cm - flat * allowed;
                    }
                }
            }
        }
        __syncwarp();

        float phi = 0.0f;
#pragma unroll
        for (int f = 0; f < FD_MAXP; ++f)
            if (f < players) phi = phi + logf(surviving[f]) * ((fmask >> f & 1u) ? 1.0f : 0.0f);
        const float denominator = available * (available - 1.0f) * 0.5f;
        for (int packed = 1; packed < players; ++packed) {
            const float numerator_cards = available - 2.0f * (float)packed;
            const float numerator = numerator_cards * (numerator_cards - 1.0f) * 0.5f;
            if (folders > packed) phi = phi + logf(fd_clamp_tiny(numerator / denominator));
        }

        float triple = 0.0f;
        if (folders <= FD_DENSE) {
            // the dense slots' surviving masses (selected with compile-time indices)
            float sd[FD_DENSE];
#pragma unroll
            for (int k = 0; k < FD_DENSE; ++k) {
                sd[k] = 1.0f;
#pragma unroll
                for (int f = 0; f < FD_MAXP; ++f) sd[k] = fseat[k] == f ? surviving[f] : sd[k];
            }
            // at most four folders (every decision with two live seats or more at six seats): one pass
            // over the surviving hands accumulates every folder pair's identical-hand sum and every tight
            // pair's edge sum against each of its (at most two) hubs
            float ident[6], tri[6][2];
#pragma unroll
            for (int i = 0; i < 6; ++i) ident[i] = tri[i][0] = tri[i][1] = 0.0f;
            // per slot: its seat's probability row, and its delta row or the zero row when the slot is not
            // tight (the loop then needs no selects).  Slots past the folder count read seat 0's row: the
            // sums they feed are never used.
            const float* prow[FD_DENSE];
            const float* drow[FD_DENSE];
#pragma unroll
            for (int i = 0; i < FD_DENSE; ++i) {
                prow[i] = prob + fseat[i] * hands;
                drow[i] = (dtight >> i & 1u) ? delta + fseat[i] * FD_CPAD : fd_zero;
            }
            for (int h = lane; h < hands; h += 32) {
                const uint16_t pr = comb[h];
                const int c1 = pr & 0xff, c2 = pr >> 8;
                if (c1 == ra || c1 == rb || c2 == ra || c2 == rb) continue;
                float ph[FD_DENSE], d1[FD_DENSE], d2[FD_DENSE];
#pragma unroll
                for (int i = 0; i < FD_DENSE; ++i) {
                    ph[i] = prow[i][h];
                    d1[i] = drow[i][c1];
                    d2[i] = drow[i][c2];
                }
#pragma unroll
                for (int s = 0; s < 6; ++s) {
                    const int i = fd_pair_i(s), j = fd_pair_j(s);
                    ident[s] += ph[i] * ph[j];
                    const float edge = d1[i] * d2[j] + d2[i] * d1[j];
                    tri[s][0] += edge * ph[fd_hub(s, 0)];
                    tri[s][1] += edge * ph[fd_hub(s, 1)];
                }
            }
            if (folders >= 2) {
                const float uniform_pair = fd_clamp_tiny((1.0f - 4.0f / available) + 1.0f / denominator);
#pragma unroll
                for (int s = 0; s < 6; ++s) {
                    const int i = fd_pair_i(s), j = fd_pair_j(s);
                    if (j >= folders) continue;
                    const int f = fseat[i], g = fseat[j];
                    float dot = 0.0f;
                    for (int c = lane; c < cards; c += 32) dot += cond[f * FD_CPAD + c] * cond[g * FD_CPAD + c];
                    dot = fd_warp_sum(dot);
                    const float same = 2.0f * fd_warp_sum(ident[s]) / (sd[i] * sd[j]);
                    const float disjoint = fd_clamp_tiny((1.0f - dot) + 0.5f * same);
                    phi = phi + logf(disjoint / uniform_pair);
                }
            }
#pragma unroll
            for (int s = 0; s < 6; ++s) {
                const int i = fd_pair_i(s), j = fd_pair_j(s);
                if (!((dtight >> i & 1u) && (dtight >> j & 1u))) continue;
                const float* left = delta + fseat[i] * FD_CPAD;
                const float* right = delta + fseat[j] * FD_CPAD;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int k = fd_hub(s, u);
                    if (k >= folders) continue;
                    const int hub = fseat[k];
                    const float matrix_term = fd_warp_sum(tri[s][u]) / sd[k];
                    const float* hm = cond + hub * FD_CPAD;
                    float diagonal = 0.0f, hl = 0.0f, hr = 0.0f;
                    for (int c = lane; c < cards; c += 32) {
                        diagonal += hm[c] * left[c] * right[c];
                        hl += hm[c] * left[c];
                        hr += hm[c] * right[c];
                    }
                    diagonal = fd_warp_sum(diagonal);
                    const float outer = fd_warp_sum(hl) * fd_warp_sum(hr);
                    triple = triple + ((matrix_term + diagonal) - outer);
                }
            }
        } else {
        // pairwise disjointness: H-wide sums of p_f p_g over surviving hands for every folder pair
        if (folders >= 2) {
            float ident[FD_MAXP * (FD_MAXP - 1) / 2];
#pragma unroll
            for (int i = 0; i < FD_MAXP * (FD_MAXP - 1) / 2; ++i) ident[i] = 0.0f;
            for (int h = lane; h < hands; h += 32) {
                const uint16_t pr = comb[h];
                const int c1 = pr & 0xff, c2 = pr >> 8;
                if (c1 == ra || c1 == rb || c2 == ra || c2 == rb) continue;
                float ph[FD_MAXP];
#pragma unroll
                for (int f = 0; f < FD_MAXP; ++f) ph[f] = f < players ? prob[f * hands + h] : 0.0f;
                int slot = 0;
#pragma unroll
                for (int f = 0; f < FD_MAXP; ++f)
#pragma unroll
                    for (int g = f + 1; g < FD_MAXP; ++g) ident[slot++] += ph[f] * ph[g];
            }
            const float uniform_pair = fd_clamp_tiny((1.0f - 4.0f / available) + 1.0f / denominator);
            int slot = 0;
#pragma unroll
            for (int f = 0; f < FD_MAXP; ++f) {
#pragma unroll
                for (int g = f + 1; g < FD_MAXP; ++g, ++slot) {
                    if (!((fmask >> f & 1u) && (fmask >> g & 1u))) continue;
                    float dot = 0.0f;
                    for (int c = lane; c < cards; c += 32) dot += cond[f * FD_CPAD + c] * cond[g * FD_CPAD + c];
                    dot = fd_warp_sum(dot);
                    const float same = 2.0f * fd_warp_sum(ident[slot]) / (surviving[f] * surviving[g]);
                    const float disjoint = fd_clamp_tiny((1.0f - dot) + 0.5f * same);
                    phi = phi + logf(disjoint / uniform_pair);
                }
            }
        }

        // triple clusters: for each tight pair, the edge sum over surviving hands weighted by every hub
        for (int f = 0; f < players; ++f) {
            for (int g = f + 1; g < players; ++g) {
                if (!((tmask >> f & 1u) && (tmask >> g & 1u))) continue;
                unsigned hubs = fmask & ~(1u << f) & ~(1u << g);
                if (!hubs) continue;
                const float* left = delta + f * FD_CPAD;
                const float* right = delta + g * FD_CPAD;
                float edge_sum[FD_MAXP];
#pragma unroll
                for (int hub = 0; hub < FD_MAXP; ++hub) edge_sum[hub] = 0.0f;
                for (int h = lane; h < hands; h += 32) {
                    const uint16_t pr = comb[h];
                    const int c1 = pr & 0xff, c2 = pr >> 8;
                    if (c1 == ra || c1 == rb || c2 == ra || c2 == rb) continue;
                    const float edge = left[c1] * right[c2] + left[c2] * right[c1];
#pragma unroll
                    for (int hub = 0; hub < FD_MAXP; ++hub)
                        if (hubs >> hub & 1u) edge_sum[hub] += edge * prob[hub * hands + h];
                }
#pragma unroll
                for (int hub = 0; hub < FD_MAXP; ++hub) {
                    if (!(hubs >> hub & 1u)) continue;
                    const float matrix_term = fd_warp_sum(edge_sum[hub]) / surviving[hub];
                    const float* hm = cond + hub * FD_CPAD;
                    float diagonal = 0.0f, hl = 0.0f, hr = 0.0f;
                    for (int c = lane; c < cards; c += 32) {
                        diagonal += hm[c] * left[c] * right[c];
                        hl += hm[c] * left[c];
                        hr += hm[c] * right[c];
                    }
                    diagonal = fd_warp_sum(diagonal);
                    const float outer = fd_warp_sum(hl) * fd_warp_sum(hr);
                    triple = triple + ((matrix_term + diagonal) - outer);
                }
            }
        }
        }
        if (lane == 0) {
            phi_out[row * queries + q] = phi + triple;
            triple_out[row * queries + q] = triple;
        }
        __syncwarp();
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_folded_query_count(int32_t cards) {
    if (cards < 2 || cards > FD_MAXC) return -1;
    return 1 + (int64_t)cards + (int64_t)cards * (cards - 1) / 2;
}

int pbg_folded_phi_queries(int64_t batch, int32_t players, int32_t cards, const float* probability,
                           const uint8_t* folder_mask, const uint8_t* tight_mask, const float* base_cards, float* phi,
                           float* triple, void* stream) {
    PBG_REQUIRE(batch >= 0 && batch <= 65535, "folded_phi_queries: batch must be in [0, 65535]");
    PBG_REQUIRE(players >= 1 && players <= FD_MAXP, "folded_phi_queries: players must be in [1, 6]");
    PBG_REQUIRE(cards >= 4 && cards <= FD_MAXC && cards % 4 == 0, "folded_phi_queries: cards must be 4R, R in [1, 13]");
    if (batch == 0) return PBG_OK;
    PBG_REQUIRE(probability && folder_mask && tight_mask && base_cards && phi && triple,
                "folded_phi_queries: null pointer");
    const int hands = cards * (cards - 1) / 2;
    const int queries = (int)pbg_folded_query_count(cards);
    // enough CTAs for about two waves of three per SM, at least one query per warp
    const int64_t target_ctas = 2 * 3 * 148;
    int64_t per_warp = (queries * batch + target_ctas * FD_WARPS - 1) / (target_ctas * FD_WARPS);
    if (per_warp < 1) per_warp = 1;
    if (per_warp > 64) per_warp = 64;
    const int per_block = FD_WARPS * (int)per_warp;
    const dim3 grid((unsigned)((queries + per_block - 1) / per_block), (unsigned)batch);
    const size_t smem = (size_t)players * hands * 4 + (size_t)players * FD_CPAD * 4 + (size_t)((hands + 3) & ~3) * 2 +
                        (size_t)FD_WARPS * 2 * FD_MAXP * FD_CPAD * 4;
    static bool configured = false;
    if (!configured) {
        int rc = cuda_status(cudaFuncSetAttribute(folded_phi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  96 * 1024),
                             "folded_phi_queries: shared memory");
        if (rc) return rc;
        configured = true;
    }
    PBG_REQUIRE(smem <= 96 * 1024, "folded_phi_queries: shared memory plan too large");
    folded_phi_kernel<<<grid, FD_THREADS, smem, as_stream(stream)>>>(players, cards, hands, queries, (int)per_warp,
                                                                    probability, folder_mask, tight_mask, base_cards,
                                                                    phi, triple);
    return launch_status("folded_phi_queries");
}

}  // extern "C"
