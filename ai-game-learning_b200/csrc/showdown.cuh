// Seven-card hand ranking and stratum settlement shared by the sampled
// showdown (showdown.cu) and the Rao-Blackwell completion (completion.cu).
//
// The category order of each deck is the rarity-consistent order of
// pbg/games/poker/cards.py:37-74 (category_profile): categories sorted by
// their exact five-card counts, equal counts in conventional order.  Within
// a category the usual kicker order applies; tied winners share equally.
#pragma once

#include "pbg_common.cuh"

namespace pbg {

enum Cat { HIGH_CARD, PAIR, TWO_PAIR, TRIPS, STRAIGHT, FLUSH, FULL_HOUSE, QUADS, STRAIGHT_FLUSH, N_CAT };

struct Strength {
    int s[N_CAT];
};

inline double comb_d(int n, int k) {
    if (k < 0 || k > n) return 0.0;
    double r = 1.0;
    for (int i = 1; i <= k; ++i) r = r * (n - k + i) / i;
    return r;
}

// Strength index of every category for a deck of R ranks (0 = weakest).
inline Strength category_strength(int R) {
    double total = comb_d(4 * R, 5);
    int seq = (R - 4 > 0 ? R - 4 : 0) + (R == 13 ? 1 : 0);
    double cr5 = R >= 5 ? comb_d(R, 5) : 0.0;
    double cnt[N_CAT];
    cnt[HIGH_CARD] = total;
    cnt[PAIR] = total - 1024.0 * cr5;
    cnt[TWO_PAIR] = 144.0 * (R - 2) * comb_d(R, 2) + 24.0 * R * (R - 1);
    cnt[TRIPS] = 64.0 * R * comb_d(R - 1, 2) + 28.0 * R * (R - 1);
    cnt[STRAIGHT] = 1024.0 * seq;
    cnt[FLUSH] = 4.0 * cr5;
    cnt[FULL_HOUSE] = 24.0 * R * (R - 1);
    cnt[QUADS] = 4.0 * R * (R - 1);
    cnt[STRAIGHT_FLUSH] = 4.0 * seq;
    Strength st;
    for (int c = 0; c < N_CAT; ++c) {
        int weaker = 0;
        for (int o = 0; o < N_CAT; ++o) {
            if (o == c || cnt[o] <= 0) continue;
            if (cnt[o] > cnt[c] || (cnt[o] == cnt[c] && o < c)) ++weaker;
        }
        st.s[c] = cnt[c] > 0 ? weaker : -1;
    }
    return st;
}

__device__ __forceinline__ int top_straight(unsigned mask, int R) {
    for (int top = 12; top >= 4; --top)
        if (((mask >> (top - 4)) & 0x1Fu) == 0x1Fu) return top;
    if (R == 13 && (mask & 0x100Fu) == 0x100Fu) return 3;  // A-2-3-4-5
    return -1;
}

__device__ __forceinline__ int64_t pack(int strength, int t0, int t1, int t2, int t3, int t4) {
    return ((((((int64_t)strength * 16 + t0) * 16 + t1) * 16 + t2) * 16 + t3) * 16) + t4;
}

// Highest set rank of mask below `below` (exclusive), or 0 when none.
__device__ __forceinline__ int next_rank(unsigned mask, int& cursor) {
    while (cursor >= 0 && !((mask >> cursor) & 1u)) --cursor;
    int r = cursor >= 0 ? cursor : 0;
    --cursor;
    return r;
}

// Rank multiplicities as bit planes (ranks held at least once / twice / three / four times) and
// the four suits' rank masks packed 16 bits apart: a card is added with a few register ops, so the
// board's planes are built once per hand and each seat only adds its two hole cards.
struct HandCounts {
    unsigned ge1 = 0, ge2 = 0, ge3 = 0, ge4 = 0;
    uint64_t suits = 0;

    __device__ __forceinline__ void add(int card) {
        const unsigned m = 1u << (card >> 2);
        ge4 |= ge3 & m;
        ge3 |= ge2 & m;
        ge2 |= ge1 & m;
        ge1 |= m;
        suits |= (uint64_t)m << (16 * (card & 3));
    }
};

__device__ __forceinline__ int64_t hand_value(const HandCounts& h, const Strength& S, int R) {
    const unsigned ranks = h.ge1, ge2 = h.ge2, ge3 = h.ge3, ge4 = h.ge4;
    int64_t best = -1;
    int flush_suit = -1;
    unsigned flush_mask = 0;
    #pragma unroll
    for (int s = 0; s < 4; ++s) {
        const unsigned m = (unsigned)(h.suits >> (16 * s)) & 0x1FFFu;
        if (__popc(m) >= 5) {
            flush_suit = s;
            flush_mask = m;
        }
    }
    if (flush_suit >= 0 && S.s[STRAIGHT_FLUSH] >= 0) {
        int top = top_straight(flush_mask, R);
        if (top >= 0) best = max(best, pack(S.s[STRAIGHT_FLUSH], top, 0, 0, 0, 0));
    }
    if (ge4) {
        int q = 31 - __clz(ge4);
        unsigned rest = ranks & ~(1u << q);
        int k = rest ? 31 - __clz(rest) : 0;
        best = max(best, pack(S.s[QUADS], q, k, 0, 0, 0));
    }
    if (ge3) {
        int t = 31 - __clz(ge3);
        unsigned pairs = ge2 & ~(1u << t);
        if (pairs) best = max(best, pack(S.s[FULL_HOUSE], t, 31 - __clz(pairs), 0, 0, 0));
    }
    if (flush_suit >= 0 && S.s[FLUSH] >= 0) {
        int cur = 12;
        unsigned m = flush_mask;
        int a = next_rank(m, cur), b = next_rank(m, cur), c = next_rank(m, cur), d = next_rank(m, cur), e = next_rank(m, cur);
        best = max(best, pack(S.s[FLUSH], a, b, c, d, e));
    }
    if (S.s[STRAIGHT] >= 0) {
        int top = top_straight(ranks, R);
        if (top >= 0) best = max(best, pack(S.s[STRAIGHT], top, 0, 0, 0, 0));
    }
    if (ge3) {
        int t = 31 - __clz(ge3);
        unsigned rest = ranks & ~(1u << t);
        int cur = 12;
        int a = next_rank(rest, cur), b = next_rank(rest, cur);
        best = max(best, pack(S.s[TRIPS], t, a, b, 0, 0));
    }
    if (__popc(ge2) >= 2) {
        int p1 = 31 - __clz(ge2);
        unsigned others = ge2 & ~(1u << p1);
        int p2 = 31 - __clz(others);
        unsigned rest = ranks & ~(1u << p1) & ~(1u << p2);
        int k = rest ? 31 - __clz(rest) : 0;
        best = max(best, pack(S.s[TWO_PAIR], p1, p2, k, 0, 0));
    }
    if (ge2) {
        int p = 31 - __clz(ge2);
        unsigned rest = ranks & ~(1u << p);
        int cur = 12;
        int a = next_rank(rest, cur), b = next_rank(rest, cur), c = next_rank(rest, cur);
        best = max(best, pack(S.s[PAIR], p, a, b, c, 0));
    }
    {
        int cur = 12;
        int a = next_rank(ranks, cur), b = next_rank(ranks, cur), c = next_rank(ranks, cur), d = next_rank(ranks, cur),
            e = next_rank(ranks, cur);
        best = max(best, pack(S.s[HIGH_CARD], a, b, c, d, e));
    }
    return best;
}


// ---------------------------------------------------- order-equivalent values
// Settlement needs only the order (and ties) of the seats' hands, so the
// showdown and completion kernels rank with hand_order: for any two hands of
// one deck its values compare exactly as hand_value's packed values do.  The
// strongest category present decides (hand_value's maximum over all categories
// is that one): every category's presence is set at its strength's bit and the
// highest bit wins, without a data-dependent loop; its kickers are rank masks
// (the k highest ranks of a set: equal-size masks compare as the descending
// rank lists do).
struct CategoryOrder {
    unsigned bit[N_CAT];  // 1 << strength of each category present in the deck, 0 if absent
};

inline CategoryOrder category_order(int R) {
    const Strength S = category_strength(R);
    CategoryOrder o;
    for (int c = 0; c < N_CAT; ++c) o.bit[c] = S.s[c] >= 0 ? 1u << S.s[c] : 0u;
    return o;
}

// The k highest set bits of m (m holds at most seven ranks).
__device__ __forceinline__ unsigned keep_top(unsigned m, int k) {
    #pragma unroll
    for (int r = 0; r < 6; ++r)
        if (__popc(m) > k) m &= m - 1;
    return m;
}

// Highest rank of a five-rank run in m (the wheel A-2-3-4-5 counts on the full deck), -1 if none.
__device__ __forceinline__ int straight_top(unsigned m, int R) {
    const unsigned run = m & (m >> 1) & (m >> 2) & (m >> 3) & (m >> 4);
    if (run) return 35 - __clz(run);
    return (R == 13 && (m & 0x100Fu) == 0x100Fu) ? 3 : -1;
}

__device__ __forceinline__ int64_t hand_order(const HandCounts& h, const CategoryOrder& O, int R) {
    const unsigned ranks = h.ge1, ge2 = h.ge2, ge3 = h.ge3, ge4 = h.ge4;
    unsigned flush = 0;
    #pragma unroll
    for (int s = 0; s < 4; ++s) {
        const unsigned m = (unsigned)(h.suits >> (16 * s)) & 0x1FFFu;
        if (__popc(m) >= 5) flush = m;
    }
    const int sf = flush ? straight_top(flush, R) : -1;
    const int st = straight_top(ranks, R);
    const int t = ge3 ? 31 - __clz(ge3) : 0;
    const unsigned fh = ge3 ? (ge2 & ~(1u << t)) : 0u;
    unsigned present = O.bit[HIGH_CARD];
    if (ge2) present |= O.bit[PAIR];
    if (__popc(ge2) >= 2) present |= O.bit[TWO_PAIR];
    if (ge3) present |= O.bit[TRIPS];
    if (st >= 0) present |= O.bit[STRAIGHT];
    if (flush) present |= O.bit[FLUSH];
    if (fh) present |= O.bit[FULL_HOUSE];
    if (ge4) present |= O.bit[QUADS];
    if (sf >= 0) present |= O.bit[STRAIGHT_FLUSH];
    const int strength = 31 - __clz(present);
    const unsigned top = 1u << strength;
    unsigned a = 0, b = 0;
    if (top == O.bit[STRAIGHT_FLUSH]) {
        a = (unsigned)sf;
    } else if (top == O.bit[QUADS]) {
        const int q = 31 - __clz(ge4);
        a = q;
        b = keep_top(ranks & ~(1u << q), 1);
    } else if (top == O.bit[FULL_HOUSE]) {
        a = t;
        b = 31 - __clz(fh);
    } else if (top == O.bit[FLUSH]) {
        b = keep_top(flush, 5);
    } else if (top == O.bit[STRAIGHT]) {
        a = (unsigned)st;
    } else if (top == O.bit[TRIPS]) {
        a = t;
        b = keep_top(ranks & ~(1u << t), 2);
    } else if (top == O.bit[TWO_PAIR]) {
        a = keep_top(ge2, 2);
        b = keep_top(ranks & ~a, 1);
    } else if (top == O.bit[PAIR]) {
        const int p = 31 - __clz(ge2);
        a = p;
        b = keep_top(ranks & ~(1u << p), 3);
    } else {
        b = keep_top(ranks, 5);
    }
    return ((int64_t)strength << 26) | ((int64_t)a << 13) | b;
}

// Chip settlement of one hand (the contract-v2 payoff: hooks.py:2252-2295): each
// seat starts from its baseline; stratum k's amount goes in equal shares to the
// strongest seats among those with level >= k and a valid hand (value >= 0).
__device__ __forceinline__ void settle_strata(int P, int strata, const int64_t* value, const int* lev,
                                              const float* amount, float* acc) {
    for (int k = 0; k < strata; ++k) {
        const float amt = amount[k];
        if (!(amt > 0.0f)) continue;
        int64_t best = -1;
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            if (value[p] >= 0 && lev[p] >= k && value[p] > best) best = value[p];
        }
        if (best < 0) continue;
        int winners = 0;
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            winners += value[p] == best && lev[p] >= k;
        }
        const float share = __fdiv_rn(amt, (float)winners);
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            if (value[p] == best && lev[p] >= k) acc[p] = __fadd_rn(acc[p], share);
        }
    }
}

}  // namespace pbg
