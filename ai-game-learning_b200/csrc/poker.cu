// NLHE public state machine, chance, settlement inputs and the fused
// sampled rollout step (sm_100a).
//
// The per-hand transition restates pbg/games/poker/queued/hooks.py:
//   initial_roots      :357-454      legality          :464-510
//   step_player        :883-979      needs_chance      :981-987
//   deal_next_street   :989-1126     history appends   :708-810
//   sampled_leaf       :1145-1216    combo_cards/class :1128-1143, :655-674
// Chip amounts are half big blinds, exact in fp32, so every state column is
// bit-exact against the reference.  A hand's state lives in registers
// (seat loops unrolled for the compile-time player count P) and is written
// back once per call.
#include "pbg_common.cuh"
#include "policy.cuh"

namespace pbg {

template <int P>
struct Hand {
    uint8_t board[5];
    int combo[P];
    int button, street, to_act;
    float stacks[P], committed[P], cs[P];
    int status[P];
    float bet, lfr;
    bool pending[P], can[P];
    bool terminal;

    __device__ void load(const pbg_state& s, int64_t b) {
        #pragma unroll
        for (int i = 0; i < 5; ++i) board[i] = s.board[b * 5 + i];
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            combo[p] = s.combo[b * P + p];
            stacks[p] = s.stacks[b * P + p];
            committed[p] = s.committed[b * P + p];
            cs[p] = s.committed_street[b * P + p];
            status[p] = s.status[b * P + p];
            pending[p] = s.pending[b * P + p] != 0;
            can[p] = s.can_raise[b * P + p] != 0;
        }
        button = s.button[b];
        street = s.street[b];
        to_act = s.to_act[b];
        bet = s.current_bet[b];
        lfr = s.last_full_raise[b];
        terminal = s.terminal[b] != 0;
    }

    __device__ void store(const pbg_state& s, int64_t b) const {
        #pragma unroll
        for (int i = 0; i < 5; ++i) s.board[b * 5 + i] = board[i];
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            s.combo[b * P + p] = combo[p];
            s.stacks[b * P + p] = stacks[p];
            s.committed[b * P + p] = committed[p];
            s.committed_street[b * P + p] = cs[p];
            s.status[b * P + p] = (int8_t)status[p];
            s.pending[b * P + p] = pending[p];
            s.can_raise[b * P + p] = can[p];
        }
        s.button[b] = button;
        s.street[b] = street;
        s.to_act[b] = to_act;
        s.current_bet[b] = bet;
        s.last_full_raise[b] = lfr;
        s.terminal[b] = terminal;
    }

    // seat-indexed reads without local memory
    __device__ float get(const float (&v)[P], int a) const {
        float r = 0.0f;
        #pragma unroll
        for (int p = 0; p < P; ++p) if (p == a) r = v[p];
        return r;
    }
    __device__ int get(const int (&v)[P], int a) const {
        int r = 0;
        #pragma unroll
        for (int p = 0; p < P; ++p) if (p == a) r = v[p];
        return r;
    }
    __device__ bool get(const bool (&v)[P], int a) const {
        bool r = false;
        #pragma unroll
        for (int p = 0; p < P; ++p) if (p == a) r = v[p];
        return r;
    }

    __device__ int live_count() const {
        int n = 0;
        #pragma unroll
        for (int p = 0; p < P; ++p) n += status[p] == LIVE;
        return n;
    }

    __device__ float pot() const {
        float s = 0.0f;
        #pragma unroll
        for (int p = 0; p < P; ++p) s = __fadd_rn(s, committed[p]);
        return s;
    }

    // hooks.py:342-348 (_next_seat) over LIVE seats.
    __device__ int next_live(int after) const {
        int found = -1;
        #pragma unroll
        for (int o = P; o >= 1; --o) {
            int c = (after + o) % P;
            if (get(status, c) == LIVE) found = c;
        }
        return found >= 0 ? found : (after + 1) % P;
    }

    // hooks.py:464-510 as a summary: call bit and contiguous raise ticks.
    __device__ LegalSummary legality(int T) const {
        LegalSummary L;
        int a = to_act;
        float stack = get(stacks, a), street_c = get(cs, a);
        float call = fmaxf(__fsub_rn(bet, street_c), 0.0f);
        float maximum = __fadd_rn(street_c, stack);
        float minimum = __fadd_rn(bet, lfr);
        bool raising = live_count() > 1 && get(can, a);
        L.alive = !terminal;
        L.call_legal = call > 0.0f;
        L.lo = 1;
        L.hi = 0;
        if (raising) {
            // tick k has target (k+1)/2; twice a half-integer is an integer
            int max2 = (int)__fmul_rn(maximum, 2.0f);
            int min2 = (int)ceilf(__fmul_rn(minimum, 2.0f));
            int hi = min(max2 - 1, T - 1);
            if (min2 <= max2) {
                L.lo = max(min2 - 1, 0);
                L.hi = hi;
            } else if (maximum > bet && max2 - 1 >= 0 && max2 - 1 <= T - 1) {
                L.lo = max2 - 1;
                L.hi = max2 - 1;
            }
        }
        return L;
    }

    // hooks.py:883-979 (step_player); the action is legal by contract.
    __device__ void step(int action) {
        int a = to_act;
        bool fold = action == FOLD, call_action = action == CHECK_CALL, raise_action = action >= RAISE_OFFSET;
        float ac = get(cs, a), astack = get(stacks, a);
        float call = fmaxf(__fsub_rn(bet, ac), 0.0f);
        float paid_call = fminf(call, astack);
        float paid = call_action ? paid_call : 0.0f;
        float raise_to = __fmul_rn(__fadd_rn(__fsub_rn((float)action, 2.0f), 1.0f), 0.5f);
        float paid_raise = fmaxf(__fsub_rn(raise_to, ac), 0.0f);
        if (raise_action) paid = paid_raise;
        if (fold) paid = 0.0f;
        float next_stack = __fsub_rn(astack, paid);
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            if (p != a) continue;
            if (fold) status[p] = FOLDED;
            pending[p] = false;
            stacks[p] = next_stack;
            committed[p] = __fadd_rn(committed[p], paid);
            cs[p] = __fadd_rn(cs[p], paid);
            if (next_stack == 0.0f && !fold) status[p] = ALL_IN;
        }
        float old_bet = bet;
        if (raise_action) bet = raise_to;
        float raise_size = __fsub_rn(raise_to, old_bet);
        bool full = raise_action && raise_size >= lfr;
        if (full) lfr = raise_size;
        bool any_outstanding = false;
        int contenders = 0;
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            bool active = status[p] == LIVE;
            if (full && active) { can[p] = true; pending[p] = true; }
            if (p == a) can[p] = false;
            if (active && cs[p] < bet) pending[p] = true;
            if (p == a) pending[p] = false;
            contenders += status[p] != FOLDED;
            any_outstanding |= pending[p] && active;
        }
        terminal = contenders <= 1 || (!any_outstanding && street == 3);
        to_act = next_live(a);
    }

    __device__ bool needs_chance() const {
        bool outstanding = false;
        #pragma unroll
        for (int p = 0; p < P; ++p) outstanding |= pending[p] && status[p] == LIVE;
        return !terminal && !outstanding && street < 3;
    }

    // 64-bit set of compact deck cards held privately or on the board.
    __device__ uint64_t used_cards(int D, int first) const {
        uint64_t used = 0;
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            int c0, c1;
            combo_cards(D, first, combo[p], c0, c1);
            used |= 1ULL << (c0 - first);
            used |= 1ULL << (c1 - first);
        }
        #pragma unroll
        for (int i = 0; i < 5; ++i)
            if (board[i] != PAD_CARD) used |= 1ULL << (board[i] - first);
        return used;
    }

    // hooks.py:989-1074 given the three smallest (key, card) unused cards.
    __device__ void apply_deal(bool needs, const int (&dealt)[3], int first) {
        if (needs) {
            if (street == 0) { board[0] = (uint8_t)(first + dealt[0]); board[1] = (uint8_t)(first + dealt[1]); board[2] = (uint8_t)(first + dealt[2]); }
            else if (street == 1) board[3] = (uint8_t)(first + dealt[0]);
            else if (street == 2) board[4] = (uint8_t)(first + dealt[0]);
        }
        street += needs ? 1 : 0;
        int live = live_count();
        if (needs) {
            #pragma unroll
            for (int p = 0; p < P; ++p) {
                bool np = status[p] == LIVE && live > 1;
                pending[p] = np;
                can[p] = np;
                cs[p] = 0.0f;
            }
            to_act = next_live(button);
            bet = 0.0f;
            lfr = 1.0f;
        }
        bool outstanding = false;
        #pragma unroll
        for (int p = 0; p < P; ++p) outstanding |= pending[p] && status[p] == LIVE;
        if (street == 3 && !outstanding) terminal = true;
    }
};

// Three smallest (key, index) among unused cards, one thread.
__device__ __forceinline__ void smallest3(const int64_t* key, uint64_t used, int D, int (&out)[3]) {
    int64_t bk[3] = {INT64_MAX, INT64_MAX, INT64_MAX};
    int bi[3] = {D, D, D};
    for (int c = 0; c < D; ++c) {
        int64_t k = ((used >> c) & 1ULL) ? INT64_MAX : key[c];
        // insert (k, c) keeping ascending (key, index) order
        if (k < bk[2] || (k == bk[2] && c < bi[2])) {
            bk[2] = k; bi[2] = c;
            if (bk[2] < bk[1] || (bk[2] == bk[1] && bi[2] < bi[1])) {
                int64_t tk = bk[1]; int ti = bi[1]; bk[1] = bk[2]; bi[1] = bi[2]; bk[2] = tk; bi[2] = ti;
                if (bk[1] < bk[0] || (bk[1] == bk[0] && bi[1] < bi[0])) {
                    tk = bk[0]; ti = bi[0]; bk[0] = bk[1]; bi[0] = bi[1]; bk[1] = tk; bi[1] = ti;
                }
            }
        }
    }
    out[0] = bi[0]; out[1] = bi[1]; out[2] = bi[2];
}

// History slot writes ------------------------------------------------------
struct HistoryToken {
    int64_t actor, street, action;
    float amount, pot, call, bet, lo, hi;
};

__device__ __forceinline__ void write_token(const pbg_history& h, int64_t b, int pos, const HistoryToken& t) {
    int64_t i = b * h.tokens + pos;
    h.actor[i] = t.actor; h.street[i] = t.street; h.action[i] = t.action;
    h.amount[i] = t.amount; h.pot_before[i] = t.pot; h.call_amount[i] = t.call;
    h.current_bet[i] = t.bet; h.min_raise_to[i] = t.lo; h.max_raise_to[i] = t.hi;
    h.mask[i] = 1;
}

__device__ __forceinline__ int history_length(const pbg_history& h, int64_t b) {
    int n = 0;
    for (int t = 0; t < h.tokens; ++t) n += h.mask[b * h.tokens + t] != 0;
    return n;
}

template <int P>
__device__ HistoryToken player_token(const Hand<P>& s, int action, int T) {
    LegalSummary L = s.legality(T);
    HistoryToken t;
    bool has = L.alive && L.lo <= L.hi;
    t.lo = has ? __fmul_rn((float)(L.lo + 1), 0.5f) : 0.0f;
    t.hi = has ? __fmul_rn((float)(L.hi + 1), 0.5f) : 0.0f;
    int a = s.to_act;
    float stack = s.get(s.stacks, a), ac = s.get(s.cs, a);
    float call = fmaxf(__fsub_rn(s.bet, ac), 0.0f);
    float paid_call = fminf(call, stack);
    float raise_to = __fmul_rn(__fadd_rn(__fsub_rn((float)action, 2.0f), 1.0f), 0.5f);
    bool raised = action >= RAISE_OFFSET, called = action == CHECK_CALL;
    t.amount = raised ? raise_to : (called ? paid_call : 0.0f);
    t.action = raised ? 2 : (called ? 1 : 0);
    t.actor = a;
    t.street = s.street;
    t.pot = s.pot();
    t.call = call;
    t.bet = s.bet;
    return t;
}

template <int P>
__device__ HistoryToken chance_token(const Hand<P>& s) {
    HistoryToken t;
    t.actor = -1; t.street = s.street + 1; t.action = 3;
    t.amount = 0.0f; t.pot = s.pot(); t.call = 0.0f; t.bet = s.bet; t.lo = 0.0f; t.hi = 0.0f;
    return t;
}

// hooks.py:1145-1216 for one hand (one thread).
template <int P>
__device__ void write_leaf(const Hand<P>& s, int D, int first, const pbg_leaf& leaf, int64_t b) {
    int contenders = 0;
    #pragma unroll
    for (int p = 0; p < P; ++p) contenders += s.status[p] != FOLDED;
    bool early = contenders == 1;
    float pot = s.pot();
    #pragma unroll
    for (int p = 0; p < P; ++p) {
        bool contender = s.status[p] != FOLDED;
        float base = -s.committed[p];
        if (early) base = __fadd_rn(base, __fmul_rn(contender ? 1.0f : 0.0f, pot));
        leaf.baseline[b * P + p] = base;
        leaf.amount[b * P + p] = (!early && p == 0) ? pot : 0.0f;
        leaf.level[b * P + p] = (!early && contender) ? 0 : -1;
        leaf.combo[b * P + p] = (!early && contender) ? s.combo[p] : -1;
    }
    uint64_t free_cards = ~s.used_cards(D, first) & (D == 64 ? ~0ULL : ((1ULL << D) - 1));
    #pragma unroll
    for (int i = 0; i < 5; ++i) {
        uint8_t c = s.board[i];
        if (early && c == PAD_CARD) {
            int low = __ffsll((long long)free_cards) - 1;
            free_cards &= free_cards - 1;
            c = (uint8_t)(first + low);
        }
        leaf.board[b * 5 + i] = c;
    }
}

// ----------------------------------------------------------------- kernels

template <int P>
__global__ void roots_kernel(Geo d, int64_t rows, uint64_t ns, int64_t epoch, int64_t base, int64_t lane_id,
                             const int32_t* buttons, float stack_bb, pbg_state st) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < rows; b += (int64_t)gridDim.x * blockDim.x) {
        int64_t root = base + b;
        int64_t key[MAXD];
        for (int c = 0; c < d.D; ++c) key[c] = rng_key(ns, root, 0, c, lane_id, epoch);
        // 2P smallest keys in stable order: repeated selection
        uint64_t taken = 0;
        int order[2 * MAXP];
        for (int r = 0; r < 2 * P; ++r) {
            int best = -1;
            for (int c = 0; c < d.D; ++c) {
                if ((taken >> c) & 1ULL) continue;
                if (best < 0 || key[c] < key[best]) best = c;
            }
            taken |= 1ULL << best;
            order[r] = best;
        }
        Hand<P> h;
        #pragma unroll
        for (int i = 0; i < 5; ++i) h.board[i] = PAD_CARD;
        int button = buttons ? buttons[b] : (int)(root % P);
        int sb, bb, first_actor;
        if (P == 2) { sb = button; bb = (button + 1) % 2; first_actor = button; }
        else { sb = (button + 1) % P; bb = (button + 2) % P; first_actor = (button + 3) % P; }
        #pragma unroll
        for (int p = 0; p < P; ++p) {
            h.combo[p] = combo_id(d.D, d.first, d.first + order[2 * p], d.first + order[2 * p + 1]);
            float c = p == bb ? 1.0f : (p == sb ? 0.5f : 0.0f);
            h.committed[p] = c;
            h.cs[p] = c;
            h.stacks[p] = __fsub_rn(stack_bb, c);
            h.status[p] = LIVE;
            h.pending[p] = true;
            h.can[p] = true;
        }
        h.button = button;
        h.street = 0;
        h.to_act = first_actor;
        h.bet = 1.0f;
        h.lfr = 1.0f;
        h.terminal = false;
        h.store(st, b);
    }
}

template <int P>
__global__ void legality_kernel(Geo d, int64_t B, pbg_state st, uint8_t* mask) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        LegalSummary L = h.legality(d.T);
        for (int e = 0; e < d.E; ++e) mask[b * d.E + e] = L(e) ? 1 : 0;
    }
}

template <int P>
__global__ void input_type_kernel(int64_t B, pbg_state st, int32_t* out) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        int contenders = 0;
        for (int p = 0; p < P; ++p) contenders += st.status[b * P + p] != FOLDED;
        out[b] = st.street[b] == 0 ? 0 : contenders - 1;
    }
}

template <int P>
__global__ void step_kernel(int64_t B, pbg_state st, const int32_t* action) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        h.step(action[b]);
        h.store(st, b);
    }
}

template <int P>
__global__ void needs_chance_kernel(int64_t B, pbg_state st, uint8_t* out) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        out[b] = h.needs_chance();
    }
}

// keys: explicit [B,D] (keyed == false) or CHANCE keys derived in-kernel.
template <int P>
__global__ void deal_kernel(Geo d, int64_t B, pbg_state st, const int64_t* keys, const uint8_t* active,
                            bool keyed, uint64_t ns, const int64_t* root, const int64_t* path, int64_t draw,
                            const int64_t* retry, const int64_t* lane) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        bool needs = h.needs_chance() && (active ? active[b] != 0 : true);
        int dealt[3] = {0, 1, 2};
        uint64_t used = h.used_cards(d.D, d.first);
        int64_t k[MAXD];
        for (int c = 0; c < d.D; ++c) {
            if (keyed) k[c] = needs ? rng_key(ns, root[b], path[b], draw * d.D + c, lane[b], retry[b]) : 0;
            else k[c] = keys[b * d.D + c];
        }
        smallest3(k, used, d.D, dealt);
        h.apply_deal(needs, dealt, d.first);
        h.store(st, b);
    }
}

template <int P>
__global__ void history_kernel(Geo d, int64_t B, pbg_state st, const int32_t* action, const uint8_t* active,
                               pbg_history hist) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        bool on;
        HistoryToken t;
        if (action) { on = !h.terminal; t = player_token(h, action[b], d.T); }
        else { on = active[b] != 0; t = chance_token(h); }
        if (!on) continue;
        int len = hist.length ? hist.length[b] : history_length(hist, b);
        if (len < hist.tokens) write_token(hist, b, len, t);
        if (hist.length) hist.length[b] = len + 1 < hist.tokens ? len + 1 : hist.tokens;
    }
}

template <int P>
__global__ void leaf_kernel(Geo d, int64_t B, pbg_state st, pbg_leaf leaf) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        Hand<P> h;
        h.load(st, b);
        write_leaf(h, d.D, d.first, leaf, b);
    }
}

__global__ void combo_cards_kernel(Geo d, int64_t n, const int32_t* ids, int64_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int a, b;
        combo_cards(d.D, d.first, ids[i], a, b);
        out[2 * i] = a;
        out[2 * i + 1] = b;
    }
}

__global__ void combo_class_kernel(Geo d, int32_t* out) {
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < d.H; h += gridDim.x * blockDim.x) {
        int a, b;
        combo_cards(d.D, d.first, h, a, b);
        out[h] = combo_class(d.R, a, b);
    }
}

// Fused sampled rollout step: one thread per hand ---------------------------
struct StepArgs {
    Geo d;
    int64_t B;
    const int32_t* list;   // work list mode: *list = live hands, list[1..] their indices (else NULL)
    pbg_state st;
    pbg_history hist;
    int64_t* root_path;
    const int64_t* lane;
    const int64_t* retry;
    uint64_t ns_action, ns_chance;
    pbg_policy pol;
    int32_t* action;
    float* selected;
    int32_t* decision;
    uint8_t* new_leaf;
    pbg_leaf leaf;
};

// The address terms of a hand's CHANCE keys other than the draw: rng_key(ns, root, path, draw,
// lane, epoch) = mix63((base + draw * C_draw) mod 2^63) with this base.
__device__ __forceinline__ uint64_t chance_base(uint64_t ns, int64_t root, int64_t path, int64_t lane_id,
                                                int64_t epoch) {
    return (uint64_t)root * 0x1C69B3F74AC4AE35ULL + (uint64_t)path * 0x3C79AC492BA7B653ULL +
           (uint64_t)lane_id * 0x4A7484AA6EA6E483ULL + (uint64_t)epoch * 0x2E1B21385C26C926ULL + ns;
}
constexpr uint64_t CHANCE_DRAW_MUL = 0x1F83D9ABFB41BD6BULL;

// Three smallest (key, card) CHANCE keys among one hand's unused cards,
// computed by a whole warp: lane l keys cards l and l+32, then three
// shuffle-argmin rounds over (key, card) pairs (stable by card index).
__device__ __forceinline__ void warp_smallest3(uint64_t base, int64_t draw_base, uint64_t used, int D,
                                               int (&out)[3]) {
    const int lane = threadIdx.x & 31;
    int64_t k0 = INT64_MAX, k1 = INT64_MAX;
    int c0 = lane, c1 = lane + 32;
    if (c0 < D && !((used >> c0) & 1ULL))
        k0 = mix63((int64_t)((base + (uint64_t)(draw_base + c0) * CHANCE_DRAW_MUL) & M63));
    if (c1 < D && !((used >> c1) & 1ULL))
        k1 = mix63((int64_t)((base + (uint64_t)(draw_base + c1) * CHANCE_DRAW_MUL) & M63));
    if (c0 >= D) c0 = 64;
    if (c1 >= D) c1 = 64;
    #pragma unroll
    for (int r = 0; r < 3; ++r) {
        bool first_is_min = (k0 < k1) || (k0 == k1 && c0 < c1);
        int64_t bk = first_is_min ? k0 : k1;
        int bc = first_is_min ? c0 : c1;
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            int64_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
            int oc = __shfl_xor_sync(0xffffffffu, bc, o);
            if (ok < bk || (ok == bk && oc < bc)) { bk = ok; bc = oc; }
        }
        out[r] = bc;
        if (bc == c0) { k0 = INT64_MAX; c0 = 64; }
        if (bc == c1) { k1 = INT64_MAX; c1 = 64; }
    }
}

// The same three cards computed by one thread for its own hand: used when many
// hands of a warp deal at once, where the warp-wide version would run once per hand.
__device__ __forceinline__ void thread_smallest3(uint64_t base, int64_t draw_base, uint64_t used, int D,
                                                 int (&out)[3]) {
    int64_t bk[3] = {INT64_MAX, INT64_MAX, INT64_MAX};
    int bi[3] = {64, 64, 64};
    uint64_t acc = base + (uint64_t)draw_base * CHANCE_DRAW_MUL;
    for (int c = 0; c < D; ++c, acc += CHANCE_DRAW_MUL) {
        if ((used >> c) & 1ULL) continue;
        const int64_t k = mix63((int64_t)(acc & M63));
        if (k < bk[2]) {  // cards arrive in increasing order: equal keys keep the earlier card
            if (k < bk[1]) {
                bk[2] = bk[1]; bi[2] = bi[1];
                if (k < bk[0]) {
                    bk[1] = bk[0]; bi[1] = bi[0];
                    bk[0] = k; bi[0] = c;
                } else {
                    bk[1] = k; bi[1] = c;
                }
            } else {
                bk[2] = k; bi[2] = c;
            }
        }
    }
    out[0] = bi[0]; out[1] = bi[1]; out[2] = bi[2];
}

// Fused sampled rollout step: one thread per hand.  Consecutive threads own
// consecutive hands, so every state column is read and written coalesced.
// The loop is warp-uniform: when a few hands of a warp must deal a street they
// are dealt by the whole warp (warp_smallest3), one hand at a time; from
// DEAL_PER_THREAD pending hands on, each deals its own (thread_smallest3).
constexpr int DEAL_PER_THREAD = 6;
constexpr int ROLLOUT_BLOCK = 128;  // 64 measured the same
//
// Work list mode (A.list): a compaction pass has already written the outputs of
// the terminal hands and listed the live ones, so every lane of a warp owns a
// live hand and late steps, where few hands are left, run dense warps.
template <int P>
__global__ void __launch_bounds__(ROLLOUT_BLOCK) rollout_step_kernel(StepArgs A) {
    const Geo& d = A.d;
    const int lane = threadIdx.x & 31;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t n = A.list ? (int64_t)A.list[0] : A.B;
    for (int64_t base = blockIdx.x * (int64_t)blockDim.x + (threadIdx.x & ~31); base < n; base += stride) {
        const bool valid = base + lane < n;
        const int64_t b = A.list ? (valid ? (int64_t)A.list[1 + base + lane] : 0) : base + lane;
        const bool live = valid && (A.list || !A.st.terminal[b]);
        if (valid && !live) {
            A.action[b] = -1;
            A.selected[b] = 0.0f;
            if (A.new_leaf) A.new_leaf[b] = 0;
            if (A.decision) {
                A.decision[4 * b] = -1; A.decision[4 * b + 1] = -1; A.decision[4 * b + 2] = 1; A.decision[4 * b + 3] = 0;
            }
        }
        if (__ballot_sync(0xffffffffu, live) == 0u) continue;
        Hand<P> h;
        int64_t root = 0, path = 0, rl = 0, re = 0;
        int act = 1, a = 0, street_before = 0, len = 0;
        float logp = 0.0f;
        LegalSummary L;
        L.alive = false; L.call_legal = false; L.lo = 1; L.hi = 0;
        const bool with_history = A.hist.tokens > 0;
        if (live) {
            h.load(A.st, b);
            root = A.root_path[2 * b];
            path = A.root_path[2 * b + 1];
            rl = A.lane ? A.lane[b] : 0;
            re = A.retry ? A.retry[b] : 0;
            // sample at the owner's private row (rollout.py:1604-1621, hooks.py:1489-1541)
            L = h.legality(d.T);
            a = h.to_act;
            int64_t row = 0;
            if (A.pol.rows > 1) {
                int combo = h.get(h.combo, a);
                if (h.street == 0) {
                    int c0, c1;
                    combo_cards(d.D, d.first, combo, c0, c1);
                    row = combo_class(d.R, c0, c1);
                } else {
                    row = combo;
                }
            }
            ClosedPolicy pol;
            pol.init(raw_row(A.pol, b * A.pol.rows + row), L, d.T);
            const int64_t key = rng_key(A.ns_action, root, path, 0, rl, re);
            act = pol.sample(key_uniform(key));
            logp = logf(fmaxf(pol.prob(act), POLICY_EPS));
            // transition (hooks.py:1656-1700)
            if (with_history) len = A.hist.length ? A.hist.length[b] : history_length(A.hist, b);
            if (with_history && len < A.hist.tokens) write_token(A.hist, b, len, player_token(h, act, d.T));
            ++len;
            street_before = h.street;
            h.step(act);
        }
        for (int gen = 0; gen < 3; ++gen) {
            const bool needs = live && h.needs_chance();
            unsigned pending = __ballot_sync(0xffffffffu, needs);
            if (pending == 0u) continue;
            uint64_t used = 0;
            if (needs) {
                if (with_history && len < A.hist.tokens) write_token(A.hist, b, len, chance_token(h));
                ++len;
                used = h.used_cards(d.D, d.first);
            }
            int dealt[3] = {0, 1, 2};
            const uint64_t base = chance_base(A.ns_chance, root, path, rl, re);
            if (__popc(pending) >= DEAL_PER_THREAD) {
                if (needs) thread_smallest3(base, (int64_t)gen * d.D, used, d.D, dealt);
            } else {
                while (pending) {
                    const int src = __ffs(pending) - 1;
                    pending &= pending - 1;
                    int out3[3];
                    warp_smallest3(__shfl_sync(0xffffffffu, base, src), (int64_t)gen * d.D,
                                   __shfl_sync(0xffffffffu, used, src), d.D, out3);
                    if (lane == src) { dealt[0] = out3[0]; dealt[1] = out3[1]; dealt[2] = out3[2]; }
                }
            }
            if (live) h.apply_deal(needs, dealt, d.first);
        }
        if (!live) continue;
        if (with_history && A.hist.length) A.hist.length[b] = len < A.hist.tokens ? len : A.hist.tokens;
        h.store(A.st, b);
        A.action[b] = act;
        A.selected[b] = logp;
        A.root_path[2 * b + 1] = child_path(path, 1);
        if (A.decision) {
            A.decision[4 * b] = a;
            A.decision[4 * b + 1] = street_before;
            A.decision[4 * b + 2] = L.lo;
            A.decision[4 * b + 3] = (L.hi & 0xffff) | ((L.call_legal ? 1 : 0) << 16);
        }
        if (A.new_leaf) A.new_leaf[b] = h.terminal;
        if (h.terminal) write_leaf(h, d.D, d.first, A.leaf, b);
    }
}

// Work list of a rollout step: the terminal hands get the step's "no decision"
// outputs (action -1, no leaf), the live ones are appended to list[1..] with one
// atomic per warp (list order does not matter: every draw is addressed by the
// hand's own root and path).  list[0] must be 0 on entry.
__global__ void __launch_bounds__(256) rollout_list_kernel(int64_t B, const uint8_t* terminal, int32_t* action,
                                                           float* selected, int32_t* decision, uint8_t* new_leaf,
                                                           int32_t* list) {
    const int lane = threadIdx.x & 31;
    for (int64_t base = blockIdx.x * (int64_t)blockDim.x + (threadIdx.x & ~31); base < B;
         base += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = base + lane;
        const bool valid = b < B;
        const bool live = valid && !terminal[b];
        if (valid && !live) {
            action[b] = -1;
            selected[b] = 0.0f;
            if (new_leaf) new_leaf[b] = 0;
            if (decision) {
                decision[4 * b] = -1; decision[4 * b + 1] = -1; decision[4 * b + 2] = 1; decision[4 * b + 3] = 0;
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, live);
        if (m == 0u) continue;
        int start = 0;
        if (lane == 0) start = atomicAdd(list, __popc(m));
        start = __shfl_sync(0xffffffffu, start, 0);
        if (live) list[1 + start + __popc(m & ((1u << lane) - 1u))] = (int32_t)b;
    }
}

// log pi(act) of one composite-policy row, one thread (hooks.py:1641-1645 via
// policy.py:113-233), through the closed-form composition.
__device__ __forceinline__ float selected_log_row(const RawRow& raw, const LegalSummary& L, int T, int act) {
    ClosedPolicy pol;
    pol.init(raw, L, T);
    return logf(fmaxf(pol.prob(act), POLICY_EPS));
}

// Reach update: block per hand, thread per private row --------------------
// The hand -> (cards, class) table is decoded once per block into shared
// memory, and each thread's log-reach values are loaded before the policy rows
// are evaluated (they do not depend on them), so their latency overlaps.
constexpr int RC_THREADS = 256;
constexpr int RC_MAXH = 1326;                                    // 52 cards
constexpr int RC_CHUNKS = (RC_MAXH + RC_THREADS - 1) / RC_THREADS;  // private rows per thread

template <int P>
__global__ void __launch_bounds__(RC_THREADS) reach_kernel(Geo d, int64_t B, pbg_state st, pbg_policy pol,
                                                           const int32_t* action, const int32_t* decision,
                                                           float* log_reach) {
    extern __shared__ float sel[];  // [H]
    __shared__ uint16_t pair_s[RC_MAXH];  // (c0 - first) | (c1 - first) << 8
    __shared__ uint8_t class_s[RC_MAXH];
    for (int h = threadIdx.x; h < d.H; h += RC_THREADS) {
        int c0, c1;
        combo_cards(d.D, d.first, h, c0, c1);
        pair_s[h] = (uint16_t)((c0 - d.first) | ((c1 - d.first) << 8));
        class_s[h] = (uint8_t)combo_class(d.R, c0, c1);
    }
    __syncthreads();
    for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
        int a = decision[4 * b];
        if (a < 0) continue;  // hand was already terminal
        int street_before = decision[4 * b + 1];
        LegalSummary L;
        L.alive = true;
        L.lo = decision[4 * b + 2];
        L.hi = (int16_t)(decision[4 * b + 3] & 0xffff);
        L.call_legal = (decision[4 * b + 3] >> 16) & 1;
        int act = action[b];
        int rows = street_before == 0 ? d.K : d.H;
        float* reach = log_reach + (int64_t)b * P * d.H;
        float held[RC_CHUNKS][P];
        #pragma unroll
        for (int k = 0; k < RC_CHUNKS; ++k) {
            const int hnd = threadIdx.x + k * RC_THREADS;
            #pragma unroll
            for (int p = 0; p < P; ++p) held[k][p] = hnd < d.H ? reach[p * d.H + hnd] : 0.0f;
        }
        for (int r = threadIdx.x; r < rows; r += RC_THREADS) {
            sel[r] = selected_log_row(raw_row(pol, b * pol.rows + r), L, d.T, act);
        }
        __syncthreads();
        // board after the chance closure
        uint64_t board_cards = 0;
        for (int i = 0; i < 5; ++i) {
            int c = st.board[b * 5 + i];
            if (c != PAD_CARD) board_cards |= 1ULL << (c - d.first);
        }
        #pragma unroll
        for (int k = 0; k < RC_CHUNKS; ++k) {
            const int hnd = threadIdx.x + k * RC_THREADS;
            if (hnd >= d.H) break;
            const unsigned pc = pair_s[hnd];
            const int r = street_before == 0 ? (int)class_s[hnd] : hnd;
            const bool conflict = ((board_cards >> (pc & 0xffu)) | (board_cards >> (pc >> 8))) & 1ULL;
            #pragma unroll
            for (int p = 0; p < P; ++p) {
                float v = held[k][p];
                if (p == a) v = __fadd_rn(v, sel[r]);
                if (conflict) v = -INFINITY;
                reach[p * d.H + hnd] = v;
            }
        }
        __syncthreads();
    }
}


// Model-input rows (hooks.py:531-612 direct_model_input, hooks.py:630-648
// _compact_preflop_reach): one block per hand.  Layout: public 8+10P |
// log-reach P*K (preflop, class-compact) or P*H | 10 history columns of
// `tokens` | zeros for the folded summary of post rows when P > 2.
__device__ __forceinline__ float public_column(const pbg_state& st, int64_t b, int t, int P, const Geo& d,
                                               float scale) {
    if (t == 0) return __fdiv_rn((float)st.street[b], 3.0f);
    t -= 1;
    if (t < 5) {
        int c = st.board[b * 5 + t];
        return c == PAD_CARD ? -1.0f : __fdiv_rn(__fsub_rn((float)c, (float)d.first), (float)max(1, d.D - 1));
    }
    t -= 5;
    if (t < P) return st.to_act[b] == t ? 1.0f : 0.0f;
    t -= P;
    if (t < P) return st.button[b] == t ? 1.0f : 0.0f;
    t -= P;
    if (t < P) return __fdiv_rn(st.stacks[b * P + t], scale);
    t -= P;
    if (t < P) return __fdiv_rn(st.committed[b * P + t], scale);
    t -= P;
    if (t < P) return __fdiv_rn(st.committed_street[b * P + t], scale);
    t -= P;
    if (t < 3 * P) return st.status[b * P + t / 3] == t % 3 ? 1.0f : 0.0f;
    t -= 3 * P;
    if (t < P) return st.pending[b * P + t] ? 1.0f : 0.0f;
    t -= P;
    if (t == 0) return __fdiv_rn(st.current_bet[b], scale);
    if (t == 1) return __fdiv_rn(st.last_full_raise[b], scale);
    t -= 2;
    return st.can_raise[b * P + t] ? 1.0f : 0.0f;
}

// Compact combo ids of preflop class k (class matrix of hooks.py:655-674):
// pair (6 combos), suited (4) or offsuit (12).
__device__ __forceinline__ int class_members(const Geo& d, int k, int (&ids)[12]) {
    const int R = d.R, i = k / R, j = k % R, shift = 13 - R;
    int n = 0;
    if (i == j) {
        int r = R - 1 - i + shift;
        for (int s1 = 0; s1 < 4; ++s1)
            for (int s2 = s1 + 1; s2 < 4; ++s2) ids[n++] = combo_id(d.D, d.first, 4 * r + s1, 4 * r + s2);
    } else if (i < j) {
        int hi = R - 1 - i + shift, lo = R - 1 - j + shift;
        for (int s = 0; s < 4; ++s) ids[n++] = combo_id(d.D, d.first, 4 * hi + s, 4 * lo + s);
    } else {
        int hi = R - 1 - j + shift, lo = R - 1 - i + shift;
        for (int s1 = 0; s1 < 4; ++s1)
            for (int s2 = 0; s2 < 4; ++s2)
                if (s1 != s2) ids[n++] = combo_id(d.D, d.first, 4 * hi + s1, 4 * lo + s2);
    }
    return n;
}

template <int P>
__global__ void model_input_kernel(Geo d, int64_t B, pbg_state st, int pre, const float* reach, pbg_history hist,
                                   int tokens, float* out, int64_t width, float scale) {
    __shared__ float gauge[MAXP];
    __shared__ float red[32];
    const int nt = blockDim.x;
    for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
        float* row = out + b * width;
        const int npub = 8 + 10 * P;
        for (int t = threadIdx.x; t < npub; t += nt) row[t] = public_column(st, b, t, P, d, scale);
        int64_t off = npub;
        if (pre) {
            if (reach) {
                // per-seat gauge: max of the finite exact reaches
                for (int p = 0; p < P; ++p) {
                    float m = -INFINITY;
                    for (int h = threadIdx.x; h < d.H; h += nt) {
                        float v = reach[(b * P + p) * d.H + h];
                        if (isfinite(v)) m = fmaxf(m, v);
                    }
                    m = warp_max(m);
                    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        float g = -INFINITY;
                        for (int w = 0; w < (nt + 31) / 32; ++w) g = fmaxf(g, red[w]);
                        gauge[p] = isfinite(g) ? g : 0.0f;
                    }
                    __syncthreads();
                }
            }
            for (int i = threadIdx.x; i < P * d.K; i += nt) {
                int p = i / d.K, k = i % d.K;
                int ids[12];
                int n = class_members(d, k, ids);
                float v;
                if (!reach) {
                    v = logf((float)n);
                } else {
                    float sum = 0.0f, g = gauge[p];
                    for (int m = 0; m < n; ++m) {
                        float x = reach[(b * P + p) * d.H + ids[m]];
                        if (isfinite(x)) sum = __fadd_rn(sum, expf(__fsub_rn(x, g)));
                    }
                    v = sum > 0.0f ? __fadd_rn(logf(fmaxf(sum, FLT_TINY)), g) : -INFINITY;
                }
                row[off + i] = v;
            }
            off += (int64_t)P * d.K;
        } else {
            for (int i = threadIdx.x; i < P * d.H; i += nt) row[off + i] = reach ? reach[b * P * d.H + i] : 0.0f;
            off += (int64_t)P * d.H;
        }
        for (int i = threadIdx.x; i < 10 * tokens; i += nt) {
            int c = i / tokens, t = i % tokens;
            int64_t at = b * tokens + t;
            float v;
            if (!hist.mask) v = c < 3 ? -1.0f : 0.0f;
            else if (c == 0) v = (float)hist.actor[at];
            else if (c == 1) v = (float)hist.street[at];
            else if (c == 2) v = (float)hist.action[at];
            else if (c == 3) v = hist.amount[at];
            else if (c == 4) v = hist.pot_before[at];
            else if (c == 5) v = hist.call_amount[at];
            else if (c == 6) v = hist.current_bet[at];
            else if (c == 7) v = hist.min_raise_to[at];
            else if (c == 8) v = hist.max_raise_to[at];
            else v = hist.mask[at] ? 1.0f : 0.0f;
            row[off + i] = v;
        }
        off += 10 * (int64_t)tokens;
        for (int64_t i = off + threadIdx.x; i < width; i += nt) row[i] = 0.0f;  // folded summary
        __syncthreads();
    }
}

}  // namespace pbg

// ====================================================================== ABI
using namespace pbg;

#define PBG_DISPATCH_P(P, ...)                                           \
    switch (P) {                                                         \
        case 2: { constexpr int PP = 2; __VA_ARGS__; break; }            \
        case 3: { constexpr int PP = 3; __VA_ARGS__; break; }            \
        case 4: { constexpr int PP = 4; __VA_ARGS__; break; }            \
        case 5: { constexpr int PP = 5; __VA_ARGS__; break; }            \
        case 6: { constexpr int PP = 6; __VA_ARGS__; break; }            \
        default: set_error("players must be in [2,6]"); return PBG_EINVAL; \
    }

static bool state_ok(const pbg_state& s) {
    return s.board && s.combo && s.button && s.street && s.to_act && s.stacks && s.committed &&
           s.committed_street && s.status && s.current_bet && s.last_full_raise && s.pending &&
           s.can_raise && s.terminal;
}

extern "C" {

int pbg_initial_roots(pbg_geometry g, int64_t rows, int64_t seed, int64_t iteration, int64_t retry_epoch,
                      int64_t logical_base, int64_t lane, const int32_t* buttons, pbg_state st, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(rows >= 0 && state_ok(st), "initial_roots: bad rows or state");
    if (rows == 0) return PBG_OK;
    Geo d = derive(g);
    uint64_t ns = rng_namespace(seed, iteration, PRIVATE);
    float stack_bb = 0.5f * (float)g.stack_ticks;
    PBG_DISPATCH_P(g.players, roots_kernel<PP><<<stride_grid(rows, 128), 128, 0, as_stream(stream)>>>(
        d, rows, ns, retry_epoch, logical_base, lane, buttons, stack_bb, st));
    return launch_status("initial_roots");
}

int pbg_legality(pbg_geometry g, int64_t B, pbg_state st, uint8_t* mask, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && mask, "legality: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    PBG_DISPATCH_P(g.players, legality_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(d, B, st, mask));
    return launch_status("legality");
}

int pbg_input_type(pbg_geometry g, int64_t B, pbg_state st, int32_t* out, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && out, "input_type: bad arguments");
    if (B == 0) return PBG_OK;
    PBG_DISPATCH_P(g.players, input_type_kernel<PP><<<stride_grid(B, 256), 256, 0, as_stream(stream)>>>(B, st, out));
    return launch_status("input_type");
}

int pbg_step_player(pbg_geometry g, int64_t B, pbg_state st, const int32_t* action, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && action, "step_player: bad arguments");
    if (B == 0) return PBG_OK;
    PBG_DISPATCH_P(g.players, step_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(B, st, action));
    return launch_status("step_player");
}

int pbg_needs_chance(pbg_geometry g, int64_t B, pbg_state st, uint8_t* out, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && out, "needs_chance: bad arguments");
    if (B == 0) return PBG_OK;
    PBG_DISPATCH_P(g.players, needs_chance_kernel<PP><<<stride_grid(B, 256), 256, 0, as_stream(stream)>>>(B, st, out));
    return launch_status("needs_chance");
}

int pbg_deal_next_street(pbg_geometry g, int64_t B, pbg_state st, const int64_t* keys, const uint8_t* active,
                         void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && keys, "deal_next_street: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    PBG_DISPATCH_P(g.players, deal_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(
        d, B, st, keys, active, false, 0, nullptr, nullptr, 0, nullptr, nullptr));
    return launch_status("deal_next_street");
}

int pbg_deal_next_street_keyed(pbg_geometry g, int64_t B, pbg_state st, int64_t seed, int64_t iteration,
                               const int64_t* root, const int64_t* path, int64_t draw, const int64_t* retry,
                               const int64_t* lane, const uint8_t* active, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && root && path && retry && lane, "deal_next_street_keyed: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    uint64_t ns = rng_namespace(seed, iteration, CHANCE);
    PBG_DISPATCH_P(g.players, deal_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(
        d, B, st, nullptr, active, true, ns, root, path, draw, retry, lane));
    return launch_status("deal_next_street_keyed");
}

int pbg_append_player_history(pbg_geometry g, int64_t B, pbg_state st, const int32_t* action, pbg_history h,
                              void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && action && h.mask && h.tokens > 0, "append_player_history: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    PBG_DISPATCH_P(g.players, history_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(
        d, B, st, action, nullptr, h));
    return launch_status("append_player_history");
}

int pbg_append_chance_history(pbg_geometry g, int64_t B, pbg_state st, const uint8_t* active, pbg_history h,
                              void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && active && h.mask && h.tokens > 0, "append_chance_history: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    PBG_DISPATCH_P(g.players, history_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(
        d, B, st, nullptr, active, h));
    return launch_status("append_chance_history");
}

int pbg_sampled_leaf(pbg_geometry g, int64_t B, pbg_state st, pbg_leaf leaf, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(B >= 0 && state_ok(st) && leaf.board && leaf.combo && leaf.level && leaf.baseline && leaf.amount,
                "sampled_leaf: bad arguments");
    if (B == 0) return PBG_OK;
    Geo d = derive(g);
    PBG_DISPATCH_P(g.players, leaf_kernel<PP><<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(d, B, st, leaf));
    return launch_status("sampled_leaf");
}

int pbg_combo_cards(pbg_geometry g, int64_t n, const int32_t* ids, int64_t* out, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(n >= 0 && ids && out, "combo_cards: bad arguments");
    if (n == 0) return PBG_OK;
    combo_cards_kernel<<<stride_grid(n, 256), 256, 0, as_stream(stream)>>>(derive(g), n, ids, out);
    return launch_status("combo_cards");
}

int pbg_combo_class(pbg_geometry g, int32_t* out, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    PBG_REQUIRE(out, "combo_class: null output");
    Geo d = derive(g);
    combo_class_kernel<<<stride_grid(d.H, 256), 256, 0, as_stream(stream)>>>(d, out);
    return launch_status("combo_class");
}

static int rollout_step_impl(pbg_geometry g, int64_t B, pbg_state st, pbg_history hist, int64_t* root_path,
                             const int64_t* lane, const int64_t* retry_epoch, int64_t seed, int64_t iteration,
                             pbg_policy pol, int32_t* action, float* selected_log, int32_t* decision,
                             uint8_t* new_leaf, pbg_leaf leaf, int32_t* worklist, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    Geo d = derive(g);
    PBG_REQUIRE(B >= 0 && state_ok(st) && root_path && action && selected_log, "rollout_step: bad arguments");
    PBG_REQUIRE(pol.type_logits && pol.omega && pol.mu && pol.scale && pol.iota, "rollout_step: null policy field");
    PBG_REQUIRE(pol.mixtures >= 1 && pol.mixtures <= 8, "rollout_step: mixtures must be in [1,8]");
    PBG_REQUIRE(pol.rows == 1 || pol.rows >= d.H, "rollout_step: policy rows must be 1 or >= H (%d)", d.H);
    PBG_REQUIRE(leaf.board && leaf.combo && leaf.level && leaf.baseline && leaf.amount, "rollout_step: null leaf column");
    PBG_REQUIRE(hist.tokens == 0 || hist.mask, "rollout_step: history without mask");
    PBG_REQUIRE(B <= INT32_MAX, "rollout_step: at most 2^31 - 1 hands");
    if (B == 0) return PBG_OK;
    if (worklist) {
        int err = cuda_status(cudaMemsetAsync(worklist, 0, sizeof(int32_t), as_stream(stream)), "rollout_step: list");
        if (err) return err;
        rollout_list_kernel<<<stride_grid(B, 256, 8), 256, 0, as_stream(stream)>>>(B, st.terminal, action,
                                                                                   selected_log, decision, new_leaf,
                                                                                   worklist);
        err = launch_status("rollout_step: list");
        if (err) return err;
    }
    StepArgs A;
    A.d = d; A.B = B; A.list = worklist; A.st = st; A.hist = hist; A.root_path = root_path; A.lane = lane;
    A.retry = retry_epoch;
    A.ns_action = rng_namespace(seed, iteration, ACTION);
    A.ns_chance = rng_namespace(seed, iteration, CHANCE);
    A.pol = pol; A.action = action; A.selected = selected_log; A.decision = decision; A.new_leaf = new_leaf;
    A.leaf = leaf;
    const int block = ROLLOUT_BLOCK;
    PBG_DISPATCH_P(g.players, rollout_step_kernel<PP><<<stride_grid(B, block, 16), block, 0, as_stream(stream)>>>(A));
    return launch_status("rollout_step");
}

int pbg_rollout_step(pbg_geometry g, int64_t B, pbg_state st, pbg_history hist, int64_t* root_path,
                     const int64_t* lane, const int64_t* retry_epoch, int64_t seed, int64_t iteration,
                     pbg_policy pol, int32_t* action, float* selected_log, int32_t* decision, uint8_t* new_leaf,
                     pbg_leaf leaf, void* stream) {
    return rollout_step_impl(g, B, st, hist, root_path, lane, retry_epoch, seed, iteration, pol, action,
                             selected_log, decision, new_leaf, leaf, nullptr, stream);
}

int pbg_rollout_step_listed(pbg_geometry g, int64_t B, pbg_state st, pbg_history hist, int64_t* root_path,
                            const int64_t* lane, const int64_t* retry_epoch, int64_t seed, int64_t iteration,
                            pbg_policy pol, int32_t* action, float* selected_log, int32_t* decision,
                            uint8_t* new_leaf, pbg_leaf leaf, int32_t* worklist, void* stream) {
    PBG_REQUIRE(worklist, "rollout_step_listed: null work list");
    return rollout_step_impl(g, B, st, hist, root_path, lane, retry_epoch, seed, iteration, pol, action,
                             selected_log, decision, new_leaf, leaf, worklist, stream);
}

int pbg_reach_update(pbg_geometry g, int64_t B, pbg_state st, pbg_policy pol, const int32_t* action,
                     const int32_t* decision, float* log_reach, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    Geo d = derive(g);
    PBG_REQUIRE(B >= 0 && state_ok(st) && action && decision && log_reach, "reach_update: bad arguments");
    PBG_REQUIRE(pol.rows >= d.H && pol.mixtures >= 1 && pol.mixtures <= 8, "reach_update: policy rows must be >= H");
    if (B == 0) return PBG_OK;
    int blocks = stride_grid(B * RC_THREADS, RC_THREADS, 8);
    PBG_REQUIRE(d.H <= RC_MAXH, "reach_update: at most 52 cards");
    PBG_DISPATCH_P(g.players, reach_kernel<PP><<<blocks, RC_THREADS, d.H * sizeof(float), as_stream(stream)>>>(
        d, B, st, pol, action, decision, log_reach));
    return launch_status("reach_update");
}

int pbg_direct_model_input(pbg_geometry g, int64_t B, pbg_state st, int32_t input_type, const float* log_reach,
                           pbg_history hist, float* out, int64_t width, void* stream) {
    int rc = check_geometry(g);
    if (rc) return rc;
    Geo d = derive(g);
    PBG_REQUIRE(B >= 0 && state_ok(st) && out && (input_type == 0 || input_type == 1), "direct_model_input: bad arguments");
    PBG_REQUIRE(hist.tokens > 0, "direct_model_input: history token capacity required");
    const int P = g.players;
    int64_t folded = (input_type == 1 && P > 2) ? (int64_t)d.H + d.D + d.D * d.D + P + P * d.D + 2 : 0;
    int64_t expect = 8 + 10 * P + (int64_t)P * (input_type == 0 ? d.K : d.H) + 10 * (int64_t)hist.tokens + folded;
    PBG_REQUIRE(width == expect, "direct_model_input: width %lld, the layout needs %lld", (long long)width,
                (long long)expect);
    if (B == 0) return PBG_OK;
    float scale = 0.5f * (float)g.stack_ticks;
    PBG_DISPATCH_P(g.players, model_input_kernel<PP><<<stride_grid(B * 256, 256, 8), 256, 0, as_stream(stream)>>>(
        d, B, st, input_type == 0, log_reach, hist, hist.tokens, out, width, scale));
    return launch_status("direct_model_input");
}


}  // extern "C"
