/*
 * pbg_oracle.c -- CPU restatement of the pbg data-parallel hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under ai-game-learning_b200/csrc.  Only tests/, the smoke() check
 * in __graft_entry__.py and bench.py's cpu_baseline / reference leg may load
 * it.  The product path never calls it and has no CPU fallback.
 *
 * Every function restates one reference function; the citation is given as
 * `path:line` inside the pbg project (pbustillo05/ai-game-learning).  The
 * restatement is pinned against golden vectors produced by running the
 * reference itself (tests/golden/make_golden.py).
 *
 * Float semantics: integer, card and half-big-blind chip arithmetic is
 * exact.  Policy composition follows the reference's fp32 operation order;
 * the PPO loss and Adam are evaluated in double precision as the truth that
 * fp32 kernels are compared against within a stated tolerance.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -shared).  Callers
 * that want several host threads split rows across threads themselves.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#define M63 0x7FFFFFFFFFFFFFFFULL
#define PAD_CARD 255
#define LIVE 0
#define FOLDED 1
#define ALL_IN 2
#define FOLD 0
#define CHECK_CALL 1
#define RAISE_OFFSET 2
#define MAXP 6
#define MAXD 52

/* ------------------------------------------------------------------ RNG */

/* pbg/core/rollout.py:96-106 (_mix63).  Signed shifts are arithmetic, as in
 * torch.bitwise_right_shift on int64; products wrap modulo 2^64 and are then
 * masked to 63 bits. */
static int64_t mix63(int64_t v) {
    int64_t f = v ^ (v >> 30);
    f = (int64_t)(((uint64_t)f * 0x3C79AC492BA7B653ULL) & M63);
    int64_t s = f ^ (f >> 27);
    s = (int64_t)(((uint64_t)s * 0x1C69B3F74AC4AE35ULL) & M63);
    return (int64_t)((uint64_t)(s ^ (s >> 31)) & M63);
}

/* pbg/core/rollout.py:109-119 (_scalar_counter_hash) on Python ints. */
static uint64_t scalar_hash(uint64_t v) {
    v &= M63;
    v = ((v ^ (v >> 30)) * 0x3C79AC492BA7B653ULL) & M63;
    v = ((v ^ (v >> 27)) * 0x1C69B3F74AC4AE35ULL) & M63;
    return (v ^ (v >> 31)) & M63;
}

/* pbg/core/rollout.py:158-163: the (seed, iteration, purpose) namespace. */
static uint64_t rng_namespace(int64_t seed, int64_t iteration, int64_t purpose) {
    uint64_t ns = scalar_hash(((uint64_t)seed & M63) ^
                              (((uint64_t)iteration + 0x6A09E667F3BCC909ULL) & M63));
    return scalar_hash(ns ^ (((uint64_t)purpose + 0x5BE0CD19137E2179ULL) & M63));
}

static int64_t rng_key(uint64_t ns, int64_t root, int64_t path, int64_t draw,
                       int64_t lane, int64_t epoch) {
    /* pbg/core/rollout.py:164-172 */
    uint64_t c = (uint64_t)root * 0x1C69B3F74AC4AE35ULL + (uint64_t)path * 0x3C79AC492BA7B653ULL +
                 (uint64_t)draw * 0x1F83D9ABFB41BD6BULL + (uint64_t)lane * 0x4A7484AA6EA6E483ULL +
                 (uint64_t)epoch * 0x2E1B21385C26C926ULL + ns;
    return mix63((int64_t)(c & M63));
}

/* pbg/core/rollout.py:122-181 (logical_rng_keys), elementwise after the
 * caller broadcast every address column to length n. */
void orc_rng_keys(int64_t seed, int64_t iteration, int64_t purpose, int64_t n,
                  const int64_t *root, const int64_t *path, const int64_t *draw,
                  const int64_t *lane, const int64_t *epoch, const uint8_t *active,
                  int64_t *out) {
    uint64_t ns = rng_namespace(seed, iteration, purpose);
    for (int64_t i = 0; i < n; ++i) {
        int64_t k = rng_key(ns, root[i], path[i], draw[i], lane[i], epoch[i]);
        out[i] = (active && !active[i]) ? 0 : k;
    }
}

/* pbg/core/rollout.py:184-202 (child_path_keys). */
void orc_child_path(int64_t n, const int64_t *path, const int64_t *ordinal, int64_t *out) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = mix63(path[i] ^ (int64_t)(((uint64_t)ordinal[i] + 0x243F6A8885A308D3ULL) & M63));
}

/* pbg/core/rollout.py:205-234 (logical_uniform), fp32 arithmetic. */
static float uniform_of(int64_t key) {
    float mant = (float)((key >> 39) & ((1LL << 24) - 1));
    float u = (mant + 0.5f) * (1.0f / 16777216.0f);
    float top = nextafterf(1.0f, 0.0f);
    return u < top ? u : top;
}

void orc_uniform(int64_t n, const int64_t *keys, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = uniform_of(keys[i]);
}

/* pbg/core/rollout.py:237-267 (logical_categorical).  The CDF is a
 * sequential fp32 prefix sum.  `margin` (optional) receives the distance
 * from the threshold to the nearest CDF edge that bounds the chosen bin,
 * divided by the row mass: a small margin flags a near-tie where another
 * summation order may legitimately pick the neighbouring bin. */
void orc_categorical(int64_t B, int64_t E, const float *p, const int64_t *keys,
                     const float *mass_in, int64_t *out, double *margin) {
    for (int64_t b = 0; b < B; ++b) {
        const float *row = p + b * E;
        float mass = 0.0f;
        if (mass_in) mass = mass_in[b];
        else for (int64_t e = 0; e < E; ++e) mass += row[e];
        float thr = uniform_of(keys[b]) * mass;
        float cap = nextafterf(mass, 0.0f);
        if (cap < thr) thr = cap;
        float cdf = 0.0f, prev = 0.0f;
        int64_t sel = E;
        for (int64_t e = 0; e < E; ++e) {
            prev = cdf;
            cdf += row[e];
            if (cdf >= thr) { sel = e; break; }
        }
        if (sel >= E) { sel = E - 1; prev = cdf; }
        out[b] = sel;
        if (margin) {
            double lo = fabs((double)thr - (double)prev);
            double hi = fabs((double)cdf - (double)thr);
            double m = lo < hi ? lo : hi;
            margin[b] = mass > 0 ? m / (double)mass : 0.0;
        }
    }
}

/* ------------------------------------------------------------- geometry */

typedef struct {
    int32_t players;
    float stack_bb;
    int32_t rank_count;
} orc_geom;

typedef struct {
    int D, first, H, K, T, E, P, tokens;
} geom_d;

static geom_d derive(orc_geom g) {
    /* pbg/games/poker/queued/hooks.py:72-192 (NLHEGeometry) and
     * pbg/games/poker/model/capacity.py:12-25 (history token bound). */
    geom_d d;
    d.P = g.players;
    d.D = 4 * g.rank_count;
    d.first = 52 - d.D;
    d.H = d.D * (d.D - 1) / 2;
    d.K = g.rank_count * g.rank_count;
    d.T = (int)lround(g.stack_bb * 2.0);
    d.E = d.T + 2;
    double nodes = ceil((double)g.stack_bb * g.players + 3.0 * g.players - g.stack_bb + 1.0);
    d.tokens = (int)nodes + 3;
    return d;
}

int32_t orc_history_tokens(orc_geom g) { return derive(g).tokens; }

/* hooks.py:187-192 (combo_id): lexicographic compact pair index. */
static int32_t combo_id(const geom_d *d, int a, int b) {
    int lo = (a < b ? a : b) - d->first, hi = (a < b ? b : a) - d->first;
    return (int32_t)(lo * (2 * d->D - lo - 1) / 2 + hi - lo - 1);
}

/* hooks.py:1128-1143 (combo_cards). */
static void combo_cards(const geom_d *d, int32_t id, int *c0, int *c1) {
    int lo = 0;
    for (int f = 0; f < d->D - 1; ++f) {
        int start = f * (2 * d->D - f - 1) / 2;
        if (id >= start) lo = f;
    }
    int start = lo * (2 * d->D - lo - 1) / 2;
    int hi = lo + (id - start) + 1;
    *c0 = lo + d->first;
    *c1 = hi + d->first;
}

void orc_combo_cards(orc_geom g, int64_t n, const int32_t *ids, int64_t *out) {
    geom_d d = derive(g);
    for (int64_t i = 0; i < n; ++i) {
        int a, b;
        combo_cards(&d, ids[i], &a, &b);
        out[2 * i] = a;
        out[2 * i + 1] = b;
    }
}

void orc_combo_id(orc_geom g, int64_t n, const int64_t *first, const int64_t *second, int32_t *out) {
    geom_d d = derive(g);
    for (int64_t i = 0; i < n; ++i) out[i] = combo_id(&d, (int)first[i], (int)second[i]);
}

/* hooks.py:655-674 (_combo_class): preflop class of every compact combo. */
void orc_combo_class(orc_geom g, int32_t *out) {
    geom_d d = derive(g);
    int R = g.rank_count;
    for (int h = 0; h < d.H; ++h) {
        int a, b;
        combo_cards(&d, h, &a, &b);
        int ra = a / 4 - (13 - R), rb = b / 4 - (13 - R);
        int high = ra > rb ? ra : rb, low = ra > rb ? rb : ra;
        int hp = R - 1 - high, lp = R - 1 - low;
        int suited_or_pair = (ra == rb) || (a % 4 == b % 4);
        out[h] = suited_or_pair ? hp * R + lp : lp * R + hp;
    }
}

/* ---------------------------------------------------------------- state */

typedef struct {
    uint8_t *board;          /* [B,5] */
    int32_t *combo;          /* [B,P] */
    int32_t *button, *street, *to_act;   /* [B] */
    float *stacks, *committed, *committed_street; /* [B,P] */
    int8_t *status;          /* [B,P] */
    float *current_bet, *last_full_raise; /* [B] */
    uint8_t *pending, *can_raise; /* [B,P] */
    uint8_t *terminal;       /* [B] */
} orc_state;

typedef struct {
    int64_t *actor, *street, *action;   /* [B,T] */
    float *amount, *pot_before, *call_amount, *current_bet, *min_raise_to, *max_raise_to;
    uint8_t *mask;
} orc_history;

/* Stable ascending argsort of n int64 keys (insertion sort; n <= 52). */
static void stable_argsort(const int64_t *key, int n, int *perm) {
    for (int i = 0; i < n; ++i) perm[i] = i;
    for (int i = 1; i < n; ++i) {
        int v = perm[i], j = i - 1;
        while (j >= 0 && key[perm[j]] > key[v]) { perm[j + 1] = perm[j]; --j; }
        perm[j + 1] = v;
    }
}

/* hooks.py:342-348 (_next_seat): first seat after `after` in table order
 * whose mask is set; seat after+1 when none is. */
static int next_seat(const uint8_t *mask, int P, int after) {
    for (int o = 1; o <= P; ++o) {
        int c = (after + o) % P;
        if (mask[c]) return c;
    }
    return (after + 1) % P;
}

/* hooks.py:357-454 (PokerStateMachine.initial_roots). */
void orc_initial_roots(orc_geom g, int64_t rows, int64_t seed, int64_t iteration,
                       int64_t retry_epoch, int64_t logical_base, int64_t lane,
                       const int32_t *buttons, orc_state *s) {
    geom_d d = derive(g);
    int P = d.P;
    uint64_t ns = rng_namespace(seed, iteration, 1 /* PRIVATE */);
    int64_t keys[MAXD];
    int perm[MAXD];
    for (int64_t b = 0; b < rows; ++b) {
        int64_t root = logical_base + b;
        for (int c = 0; c < d.D; ++c) keys[c] = rng_key(ns, root, 0, c, lane, retry_epoch);
        stable_argsort(keys, d.D, perm);
        for (int p = 0; p < P; ++p)
            s->combo[b * P + p] = combo_id(&d, d.first + perm[2 * p], d.first + perm[2 * p + 1]);
        int button = buttons ? buttons[b] : (int)(root % P);
        int sb, bb, first;
        if (P == 2) { sb = button; bb = (button + 1) % 2; first = button; }
        else { sb = (button + 1) % P; bb = (button + 2) % P; first = (button + 3) % P; }
        for (int c = 0; c < 5; ++c) s->board[b * 5 + c] = PAD_CARD;
        s->button[b] = button;
        s->street[b] = 0;
        s->to_act[b] = first;
        for (int p = 0; p < P; ++p) {
            float c = p == bb ? 1.0f : (p == sb ? 0.5f : 0.0f);
            s->committed[b * P + p] = c;
            s->committed_street[b * P + p] = c;
            s->stacks[b * P + p] = g.stack_bb - c;
            s->status[b * P + p] = LIVE;
            s->pending[b * P + p] = 1;
            s->can_raise[b * P + p] = 1;
        }
        s->current_bet[b] = 1.0f;
        s->last_full_raise[b] = 1.0f;
        s->terminal[b] = 0;
    }
}

/* hooks.py:456-462 (input_type). */
void orc_input_type(orc_geom g, int64_t B, const orc_state *s, int32_t *out) {
    int P = g.players;
    for (int64_t b = 0; b < B; ++b) {
        int contenders = 0;
        for (int p = 0; p < P; ++p) contenders += s->status[b * P + p] != FOLDED;
        out[b] = s->street[b] == 0 ? 0 : contenders - 1;
    }
}

/* hooks.py:464-510 (legality) for one row; mask has E entries. */
static void legality_row(const geom_d *d, const orc_state *s, int64_t b, uint8_t *mask) {
    int P = d->P, a = s->to_act[b];
    float stack = s->stacks[b * P + a];
    float street_c = s->committed_street[b * P + a];
    float call = s->current_bet[b] - street_c;
    if (call < 0.0f) call = 0.0f;
    float maximum = street_c + stack;
    float minimum = s->current_bet[b] + s->last_full_raise[b];
    int live = 0;
    for (int p = 0; p < P; ++p) live += s->status[b * P + p] == LIVE;
    int raising = live > 1 && s->can_raise[b * P + a];
    int alive = !s->terminal[b];
    mask[0] = alive && call > 0.0f;
    mask[1] = alive;
    for (int k = 0; k < d->T; ++k) {
        float target = (float)(k + 1) * 0.5f;
        int full = target >= minimum && target <= maximum;
        int shortall = target == maximum && maximum > s->current_bet[b];
        mask[2 + k] = alive && raising && (full || shortall);
    }
}

void orc_legality(orc_geom g, int64_t B, const orc_state *s, uint8_t *mask) {
    geom_d d = derive(g);
    for (int64_t b = 0; b < B; ++b) legality_row(&d, s, b, mask + b * d.E);
}

/* hooks.py:883-979 (step_player) for one row. */
static void step_row(const geom_d *d, orc_state *s, int64_t b, int action) {
    int P = d->P, a = s->to_act[b];
    float *stacks = s->stacks + b * P, *com = s->committed + b * P, *cs = s->committed_street + b * P;
    int8_t *status = s->status + b * P;
    uint8_t *pending = s->pending + b * P, *can = s->can_raise + b * P;
    int fold = action == FOLD, call_action = action == CHECK_CALL, raise_action = action >= RAISE_OFFSET;
    if (fold) status[a] = FOLDED;
    pending[a] = 0;
    float ac = cs[a], astack = stacks[a];
    float call = s->current_bet[b] - ac;
    if (call < 0.0f) call = 0.0f;
    float paid_call = call < astack ? call : astack;
    float paid = call_action ? paid_call : 0.0f;
    float raise_to = ((float)action - 2.0f + 1.0f) * 0.5f;
    float paid_raise = raise_to - ac;
    if (paid_raise < 0.0f) paid_raise = 0.0f;
    if (raise_action) paid = paid_raise;
    if (fold) paid = 0.0f;
    float next_stack = astack - paid;
    stacks[a] = next_stack;
    com[a] += paid;
    cs[a] += paid;
    if (next_stack == 0.0f && !fold) status[a] = ALL_IN;
    float old_bet = s->current_bet[b];
    if (raise_action) s->current_bet[b] = raise_to;
    float raise_size = raise_to - old_bet;
    int full = raise_action && raise_size >= s->last_full_raise[b];
    if (full) s->last_full_raise[b] = raise_size;
    uint8_t active[MAXP];
    for (int p = 0; p < P; ++p) active[p] = status[p] == LIVE;
    for (int p = 0; p < P; ++p) {
        if (full && active[p]) { can[p] = 1; pending[p] = 1; }
    }
    can[a] = 0;
    for (int p = 0; p < P; ++p)
        if (active[p] && cs[p] < s->current_bet[b]) pending[p] = 1;
    pending[a] = 0;
    int contenders = 0, outstanding = 0;
    for (int p = 0; p < P; ++p) {
        contenders += status[p] != FOLDED;
        outstanding |= pending[p] && active[p];
    }
    int terminal = contenders <= 1;
    if (!outstanding && s->street[b] == 3) terminal = 1;
    s->terminal[b] = (uint8_t)terminal;
    s->to_act[b] = next_seat(active, P, a);
}

void orc_step_player(orc_geom g, int64_t B, orc_state *s, const int32_t *action) {
    geom_d d = derive(g);
    for (int64_t b = 0; b < B; ++b) step_row(&d, s, b, action[b]);
}

/* hooks.py:981-987 (needs_chance). */
static int needs_chance_row(int P, const orc_state *s, int64_t b) {
    int outstanding = 0;
    for (int p = 0; p < P; ++p)
        outstanding |= s->pending[b * P + p] && s->status[b * P + p] == LIVE;
    return !s->terminal[b] && !outstanding && s->street[b] < 3;
}

void orc_needs_chance(orc_geom g, int64_t B, const orc_state *s, uint8_t *out) {
    for (int64_t b = 0; b < B; ++b) out[b] = (uint8_t)needs_chance_row(g.players, s, b);
}

/* hooks.py:989-1074 (deal_next_street) for one row with its D chance keys. */
static void deal_row(const geom_d *d, orc_state *s, int64_t b, const int64_t *key, int active_in) {
    int P = d->P;
    int needs = needs_chance_row(P, s, b) && active_in;
    uint8_t used[MAXD] = {0};
    for (int p = 0; p < P; ++p) {
        int c0, c1;
        combo_cards(d, s->combo[b * P + p], &c0, &c1);
        used[c0 - d->first] = 1;
        used[c1 - d->first] = 1;
    }
    for (int i = 0; i < 5; ++i) {
        int c = s->board[b * 5 + i];
        if (c != PAD_CARD && c >= d->first && c < 52) used[c - d->first] = 1;
    }
    int64_t ordering[MAXD];
    int perm[MAXD];
    for (int c = 0; c < d->D; ++c) ordering[c] = used[c] ? INT64_MAX : key[c];
    stable_argsort(ordering, d->D, perm);
    int street = s->street[b];
    if (needs) {
        if (street == 0)
            for (int i = 0; i < 3; ++i) s->board[b * 5 + i] = (uint8_t)(d->first + perm[i]);
        else if (street == 1) s->board[b * 5 + 3] = (uint8_t)(d->first + perm[0]);
        else if (street == 2) s->board[b * 5 + 4] = (uint8_t)(d->first + perm[0]);
    }
    int new_street = street + needs;
    s->street[b] = new_street;
    uint8_t active[MAXP];
    int live = 0;
    for (int p = 0; p < P; ++p) { active[p] = s->status[b * P + p] == LIVE; live += active[p]; }
    if (needs) {
        for (int p = 0; p < P; ++p) {
            uint8_t np = active[p] && live > 1;
            s->pending[b * P + p] = np;
            s->can_raise[b * P + p] = np;
            s->committed_street[b * P + p] = 0.0f;
        }
        s->to_act[b] = next_seat(active, P, s->button[b]);
        s->current_bet[b] = 0.0f;
        s->last_full_raise[b] = 1.0f;
    }
    int outstanding = 0;
    for (int p = 0; p < P; ++p) outstanding |= s->pending[b * P + p] && active[p];
    if (new_street == 3 && !outstanding) s->terminal[b] = 1;
}

void orc_deal_next_street(orc_geom g, int64_t B, orc_state *s, const int64_t *keys, const uint8_t *active) {
    geom_d d = derive(g);
    for (int64_t b = 0; b < B; ++b) deal_row(&d, s, b, keys + b * d.D, active ? active[b] : 1);
}

/* hooks.py:1076-1126 (deal_next_street_keyed): CHANCE keys at the row's
 * (root, path) with draw = generation*D + card ordinal; inactive rows get
 * the zero key and do not deal. */
void orc_deal_next_street_keyed(orc_geom g, int64_t B, orc_state *s, int64_t seed, int64_t iteration,
                                const int64_t *root, const int64_t *path, int64_t draw,
                                const int64_t *retry, const int64_t *lane, const uint8_t *active) {
    geom_d d = derive(g);
    uint64_t ns = rng_namespace(seed, iteration, 5 /* CHANCE */);
    int64_t keys[MAXD];
    for (int64_t b = 0; b < B; ++b) {
        int on = needs_chance_row(d.P, s, b) && (active ? active[b] : 1);
        for (int c = 0; c < d.D; ++c)
            keys[c] = on ? rng_key(ns, root[b], path[b], draw * d.D + c, lane[b], retry[b]) : 0;
        deal_row(&d, s, b, keys, on);
    }
}

/* hooks.py:708-731 (_append_history) for one row. */
static void append_row(orc_history *h, int tokens, int64_t b, int active, int64_t actor, int64_t street,
                       int64_t action, float amount, float pot, float call, float bet, float lo, float hi) {
    if (!active) return;
    int64_t len = 0;
    for (int t = 0; t < tokens; ++t) len += h->mask[b * tokens + t] != 0;
    if (len >= tokens) return; /* reference asserts; callers never exceed the bound */
    int64_t i = b * tokens + len;
    h->actor[i] = actor; h->street[i] = street; h->action[i] = action;
    h->amount[i] = amount; h->pot_before[i] = pot; h->call_amount[i] = call;
    h->current_bet[i] = bet; h->min_raise_to[i] = lo; h->max_raise_to[i] = hi;
    h->mask[i] = 1;
}

/* hooks.py:733-785 (append_player_history), from the pre-action state. */
void orc_append_player_history(orc_geom g, int64_t B, const orc_state *s, const int32_t *action, orc_history *h) {
    geom_d d = derive(g);
    uint8_t mask[2 + 2 * 128 + 2];
    int P = d.P;
    for (int64_t b = 0; b < B; ++b) {
        legality_row(&d, s, b, mask);
        float lo = INFINITY, hi = -INFINITY;
        int has = 0;
        for (int k = 0; k < d.T; ++k) {
            if (!mask[2 + k]) continue;
            float t = (float)(k + 1) * 0.5f;
            has = 1;
            if (t < lo) lo = t;
            if (t > hi) hi = t;
        }
        if (!has) { lo = 0.0f; hi = 0.0f; }
        int a = s->to_act[b];
        float stack = s->stacks[b * P + a], ac = s->committed_street[b * P + a];
        float call = s->current_bet[b] - ac;
        if (call < 0.0f) call = 0.0f;
        float paid_call = call < stack ? call : stack;
        int act = action[b];
        float raise_to = ((float)act - 2.0f + 1.0f) * 0.5f;
        int raised = act >= RAISE_OFFSET, called = act == CHECK_CALL;
        float amount = raised ? raise_to : (called ? paid_call : 0.0f);
        int64_t type = raised ? 2 : (called ? 1 : 0);
        float pot = 0.0f;
        for (int p = 0; p < P; ++p) pot += s->committed[b * P + p];
        append_row(h, d.tokens, b, !s->terminal[b], a, s->street[b], type, amount, pot, call,
                   s->current_bet[b], lo, hi);
    }
}

/* hooks.py:787-810 (append_chance_history). */
void orc_append_chance_history(orc_geom g, int64_t B, const orc_state *s, const uint8_t *active, orc_history *h) {
    geom_d d = derive(g);
    int P = d.P;
    for (int64_t b = 0; b < B; ++b) {
        float pot = 0.0f;
        for (int p = 0; p < P; ++p) pot += s->committed[b * P + p];
        append_row(h, d.tokens, b, active[b], -1, s->street[b] + 1, 3, 0.0f, pot, 0.0f,
                   s->current_bet[b], 0.0f, 0.0f);
    }
}

/* hooks.py:1145-1216 (sampled_leaf) for states treated as terminal. */
void orc_sampled_leaf(orc_geom g, int64_t B, const orc_state *s, uint8_t *board, int32_t *combo,
                      int32_t *level, float *baseline, float *amount) {
    geom_d d = derive(g);
    int P = d.P;
    for (int64_t b = 0; b < B; ++b) {
        int contenders = 0;
        float pot = 0.0f;
        for (int p = 0; p < P; ++p) {
            contenders += s->status[b * P + p] != FOLDED;
            pot += s->committed[b * P + p];
        }
        int early = contenders == 1;
        for (int p = 0; p < P; ++p) {
            int contender = s->status[b * P + p] != FOLDED;
            float base = -s->committed[b * P + p];
            if (early) base = base + (contender ? 1.0f : 0.0f) * pot;
            baseline[b * P + p] = base;
            amount[b * P + p] = (!early && p == 0) ? pot : 0.0f;
            level[b * P + p] = (!early && contender) ? 0 : -1;
            combo[b * P + p] = (!early && contender) ? s->combo[b * P + p] : -1;
        }
        uint8_t used[MAXD] = {0};
        for (int p = 0; p < P; ++p) {
            int c0, c1;
            combo_cards(&d, s->combo[b * P + p], &c0, &c1);
            used[c0 - d.first] = 1;
            used[c1 - d.first] = 1;
        }
        for (int i = 0; i < 5; ++i) {
            int c = s->board[b * 5 + i];
            if (c != PAD_CARD) used[c - d.first] = 1;
        }
        int unused[MAXD], n_unused = 0;
        for (int c = 0; c < d.D; ++c) if (!used[c]) unused[n_unused++] = d.first + c;
        int missing = 0;
        for (int i = 0; i < 5; ++i) {
            uint8_t c = s->board[b * 5 + i];
            if (early && c == PAD_CARD) {
                c = (uint8_t)unused[missing];
                ++missing;
            } else if (c == PAD_CARD) {
                ++missing;
            }
            board[b * 5 + i] = c;
        }
    }
}

/* ------------------------------------------------------------- showdown */
/*
 * The reference calls the external poker_gpu_evaluator (contract v2) for
 * showdowns (hooks.py:2277-2295); it is not part of the reference tree.
 * This restates standard 7-card NLHE ranking with the short-deck category
 * order from pbg/games/poker/cards.py:37-74 (rarity-consistent strength:
 * categories sorted by their exact five-card counts, ties in conventional
 * order) and equal shares among tied winners.  Parity is unpinned against
 * the external evaluator.
 */

enum { HIGH_CARD, PAIR, TWO_PAIR, TRIPS, STRAIGHT, FLUSH, FULL_HOUSE, QUADS, STRAIGHT_FLUSH, N_CAT };

static double comb(int n, int k) {
    if (k < 0 || k > n) return 0.0;
    double r = 1.0;
    for (int i = 1; i <= k; ++i) r = r * (n - k + i) / i;
    return r;
}

/* strength[cat] = 0 for the weakest category present, larger is stronger. */
static void category_strength(int R, int *strength) {
    double total = comb(4 * R, 5);
    int seq = (R - 4 > 0 ? R - 4 : 0) + (R == 13);
    double cr5 = R >= 5 ? comb(R, 5) : 0.0;
    double cnt[N_CAT];
    cnt[HIGH_CARD] = total;
    cnt[PAIR] = total - 1024.0 * cr5;
    cnt[TWO_PAIR] = 144.0 * (R - 2) * comb(R, 2) + 24.0 * R * (R - 1);
    cnt[TRIPS] = 64.0 * R * comb(R - 1, 2) + 28.0 * R * (R - 1);
    cnt[STRAIGHT] = 1024.0 * seq;
    cnt[FLUSH] = 4.0 * cr5;
    cnt[FULL_HOUSE] = 24.0 * R * (R - 1);
    cnt[QUADS] = 4.0 * R * (R - 1);
    cnt[STRAIGHT_FLUSH] = 4.0 * seq;
    /* Conventional index: straight_flush=0 ... high_card=8 (strongest first). */
    for (int c = 0; c < N_CAT; ++c) {
        /* Count categories that are strictly weaker: more common, or equally
         * common and conventionally weaker.  Absent categories never rank. */
        int weaker = 0;
        for (int o = 0; o < N_CAT; ++o) {
            if (o == c || cnt[o] <= 0) continue;
            if (cnt[o] > cnt[c] || (cnt[o] == cnt[c] && o < c)) ++weaker;
        }
        strength[c] = cnt[c] > 0 ? weaker : -1;
    }
}

/* Value of a five-card hand: strength index then tie-break ranks (0..12,
 * global rank = card/4), 4 bits each. */
static int64_t five_value(const int *cards, const int *strength, int R) {
    int rc[13] = {0};
    int flush = 1;
    for (int i = 0; i < 5; ++i) {
        rc[cards[i] / 4]++;
        if (cards[i] % 4 != cards[0] % 4) flush = 0;
    }
    int distinct = 0, top = -1;
    for (int r = 0; r < 13; ++r) distinct += rc[r] > 0;
    int straight = 0;
    if (distinct == 5) {
        int hi = -1, lo = 13;
        for (int r = 0; r < 13; ++r) if (rc[r]) { if (r > hi) hi = r; if (r < lo) lo = r; }
        if (hi - lo == 4) { straight = 1; top = hi; }
        else if (R == 13 && rc[12] && rc[0] && rc[1] && rc[2] && rc[3]) { straight = 1; top = 3; }
    }
    /* group ranks by (count desc, rank desc) */
    int order[5], n = 0;
    for (int c = 4; c >= 1; --c)
        for (int r = 12; r >= 0; --r)
            if (rc[r] == c) order[n++] = r;
    int cat;
    if (straight && flush) cat = STRAIGHT_FLUSH;
    else if (rc[order[0]] == 4) cat = QUADS;
    else if (rc[order[0]] == 3 && n >= 2 && rc[order[1]] == 2) cat = FULL_HOUSE;
    else if (flush) cat = FLUSH;
    else if (straight) cat = STRAIGHT;
    else if (rc[order[0]] == 3) cat = TRIPS;
    else if (rc[order[0]] == 2 && rc[order[1]] == 2) cat = TWO_PAIR;
    else if (rc[order[0]] == 2) cat = PAIR;
    else cat = HIGH_CARD;
    int64_t v = strength[cat];
    int tb[5] = {0, 0, 0, 0, 0};
    if (cat == STRAIGHT || cat == STRAIGHT_FLUSH) tb[0] = top;
    else for (int i = 0; i < n; ++i) tb[i] = order[i];
    for (int i = 0; i < 5; ++i) v = v * 16 + tb[i];
    return v;
}

int64_t orc_hand_value7(int32_t rank_count, const int32_t *cards7) {
    int strength[N_CAT];
    category_strength(rank_count, strength);
    int64_t best = -1;
    int sub[5];
    for (int a = 0; a < 7; ++a)
        for (int b2 = a + 1; b2 < 7; ++b2) {
            int n = 0;
            for (int i = 0; i < 7; ++i) if (i != a && i != b2) sub[n++] = cards7[i];
            int64_t v = five_value(sub, strength, rank_count);
            if (v > best) best = v;
        }
    return best;
}

/* Contract-v2 evaluate_showdowns: payoff = baseline + sum over strata k of
 * an equal share of amount[k] among the best hands whose level >= k. */
void orc_evaluate_showdowns(int32_t rank_count, int64_t B, int32_t P, int32_t strata,
                            const uint8_t *board, const int32_t *combo, const int32_t *level,
                            const float *baseline, const float *amount, float *out) {
    orc_geom g = {P, 8.0f, rank_count};
    geom_d d = derive(g);
    for (int64_t b = 0; b < B; ++b) {
        int64_t value[MAXP];
        for (int p = 0; p < P; ++p) {
            value[p] = -1;
            int32_t id = combo[b * P + p];
            if (id < 0 || level[b * P + p] < 0) continue;
            int c7[7], c0, c1;
            combo_cards(&d, id, &c0, &c1);
            for (int i = 0; i < 5; ++i) c7[i] = board[b * 5 + i];
            c7[5] = c0;
            c7[6] = c1;
            value[p] = orc_hand_value7(rank_count, c7);
        }
        for (int p = 0; p < P; ++p) out[b * P + p] = baseline[b * P + p];
        for (int k = 0; k < strata; ++k) {
            float amt = amount[b * strata + k];
            if (!(amt > 0.0f)) continue;
            int64_t best = -1;
            for (int p = 0; p < P; ++p)
                if (value[p] >= 0 && level[b * P + p] >= k && value[p] > best) best = value[p];
            if (best < 0) continue;
            int winners = 0;
            for (int p = 0; p < P; ++p)
                winners += value[p] == best && level[b * P + p] >= k;
            float share = amt / (float)winners;
            for (int p = 0; p < P; ++p)
                if (value[p] == best && level[b * P + p] >= k) out[b * P + p] += share;
        }
    }
}

/* --------------------------------------------------------------- policy */

/* torch.linspace(0, 1, T+1) in fp32 (the two-sided formula torch uses). */
static float linspace_edge(int i, int T) {
    float step = 1.0f / (float)T;
    int half = (T + 1) / 2;
    return i < half ? (float)i * step : 1.0f - step * (float)(T - i);
}

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* pbg/games/poker/queued/policy.py:113-204 (PokerPolicyOperator.probabilities
 * with _discretized_logistic), one policy row at a time.  `mask` rows are
 * shared by `rows_per_mask` consecutive policy rows (the [B,H,E] broadcast of
 * a [B,E] legality). */
void orc_policy_probabilities(int64_t rows, int32_t T, int32_t M, int64_t rows_per_mask,
                              const float *type_logits, const float *omega, const float *mu,
                              const float *scale, const float *iota, const uint8_t *mask,
                              float *out) {
    const float eps = 1.0e-12f, tiny = FLT_MIN;
    int E = T + 2;
    float *z = malloc(sizeof(float) * (T + 1));
    float *tick = malloc(sizeof(float) * T);
    float *mix = malloc(sizeof(float) * T);
    float *full = malloc(sizeof(float) * E);
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t *mk = mask + (r / rows_per_mask) * E;
        for (int k = 0; k < T; ++k) mix[k] = 0.0f;
        for (int m = 0; m < M; ++m) {
            float loc = mu[r * M + m], sc = scale[r * M + m];
            for (int i = 0; i <= T; ++i) z[i] = (linspace_edge(i, T) - loc) / sc;
            float norm = sigm(z[T]) * sigm(-z[0]) * (-expm1f(z[0] - z[T]));
            if (norm < tiny) norm = tiny;
            float sum = 0.0f;
            for (int k = 0; k < T; ++k) {
                float p = sigm(z[k + 1]) * sigm(-z[k]) * (-expm1f(z[k] - z[k + 1]));
                if (p < 0.0f) p = 0.0f;
                tick[k] = p / norm;
                sum += tick[k];
            }
            if (sum < tiny) sum = tiny;
            for (int k = 0; k < T; ++k) mix[k] += omega[r * M + m] * (tick[k] / sum);
        }
        float mass = 0.0f;
        int count = 0, all_in = -1;
        for (int k = 0; k < T; ++k) {
            if (!mk[2 + k]) { mix[k] = 0.0f; continue; }
            mass += mix[k];
            ++count;
            all_in = k;
        }
        float io = iota[r];
        const float *lg = type_logits + r * 3;
        full[0] = lg[0];
        full[1] = mk[0] ? lg[1] : lg[0];
        for (int k = 0; k < T; ++k) {
            float rp = 0.0f;
            if (mk[2 + k]) {
                float cond = mass > 0.0f ? mix[k] / (mass > eps ? mass : eps)
                                         : 1.0f / (float)(count > 1 ? count : 1);
                rp = (1.0f - io) * cond + io * (k == all_in ? 1.0f : 0.0f);
            }
            full[2 + k] = lg[2] + (rp > 0.0f ? logf(rp > eps ? rp : eps) : -INFINITY);
        }
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) if (mk[e] && full[e] > mx) mx = full[e];
        float sum = 0.0f;
        for (int e = 0; e < E; ++e) {
            float v = mk[e] ? expf(full[e] - mx) : 0.0f;
            out[r * E + e] = v;
            sum += v;
        }
        for (int e = 0; e < E; ++e) out[r * E + e] = mk[e] ? out[r * E + e] / sum : 0.0f;
    }
    free(z); free(tick); free(mix); free(full);
}

/* ----------------------------------------------------------------- loss */
/*
 * PPO / entropy objective for the game-neutral categorical policy
 * (tests/categorical_policy_fixture.py:33-57 for log pi and entropy;
 * pbg/core/learner.py:2021-2077 for the ratio, clip and negative-advantage
 * log cap).  Per row r with decision-mass weight w_r:
 *   loss_r = w_r * (policy_row_r - c_ent * entropy_r)
 *   total  = scale * sum_r loss_r * inv_count
 * dlogits is d total / d logits (masked entries zero).  torch.minimum and
 * torch.clamp gradients are restated exactly, including the half split of
 * minimum at ties (the unclipped case) and clamp's inclusive bounds.
 *
 * controls: [clip, log_cap, ent_coef, scale, inv_count]
 * sums (double[8]): total, policy_sum, entropy_sum, approx_kl_sum,
 *                   clip_count, negcap_count, weight_sum, rows
 */
void orc_ppo_categorical(int64_t N, int32_t A, const float *logits, const uint8_t *mask,
                         const int32_t *action, const float *old_logp, const float *adv,
                         const float *weight, const float *controls, float *dlogits,
                         double *sums) {
    double clip = controls[0], cap = controls[1], cent = controls[2];
    double scale = controls[3], inv = controls[4];
    double acc[8] = {0};
    {
        double *loc = acc;
        double *lp = malloc(sizeof(double) * A);
        for (int64_t r = 0; r < N; ++r) {
            const float *x = logits + r * A;
            const uint8_t *mk = mask + r * A;
            double mx = -INFINITY;
            for (int j = 0; j < A; ++j) if (mk[j] && x[j] > mx) mx = x[j];
            double se = 0.0;
            for (int j = 0; j < A; ++j) if (mk[j]) se += exp((double)x[j] - mx);
            double lse = mx + log(se);
            double ent = 0.0;
            for (int j = 0; j < A; ++j) {
                lp[j] = mk[j] ? (double)x[j] - lse : 0.0;
                if (mk[j]) ent -= exp(lp[j]) * lp[j];
            }
            int a = action[r];
            double adv_r = adv[r], w = weight[r];
            double lr = lp[a] - (double)old_logp[r];
            double ratio = exp(lr);
            double lo = 1.0 - clip, hi = 1.0 + clip;
            double clipped = ratio < lo ? lo : (ratio > hi ? hi : ratio);
            int negative = adv_r < 0.0;
            double capped_lr = lr < cap ? lr : cap;
            double neg_ratio = exp(capped_lr);
            double pratio = negative ? neg_ratio : ratio;
            double f1 = pratio * adv_r, f2 = clipped * adv_r;
            double prow = -(f1 < f2 ? f1 : f2);
            /* d prow / d lr */
            double g1 = f1 < f2 ? 1.0 : (f1 == f2 ? 0.5 : 0.0);
            double g2 = f2 < f1 ? 1.0 : (f1 == f2 ? 0.5 : 0.0);
            double dpr = negative ? neg_ratio * (lr < cap ? 1.0 : (lr == cap ? 0.5 : 0.0)) : ratio;
            double dcl = (ratio >= lo && ratio <= hi) ? ratio : 0.0;
            double dprow_dlr = -(g1 * adv_r * dpr + g2 * adv_r * dcl);
            double coef = scale * w * inv;
            for (int j = 0; j < A; ++j) {
                double g = 0.0;
                if (mk[j]) {
                    double p = exp(lp[j]);
                    g = dprow_dlr * ((j == a ? 1.0 : 0.0) - p) + cent * p * (lp[j] + ent);
                    g *= coef;
                }
                if (dlogits) dlogits[r * A + j] = (float)g;
            }
            loc[0] += coef * (prow - cent * ent);
            loc[1] += w * prow;
            loc[2] += w * ent;
            loc[3] += w * ((ratio - 1.0) - lr);
            loc[4] += fabs(ratio - 1.0) > clip ? 1.0 : 0.0;
            loc[5] += (negative && lr > cap) ? 1.0 : 0.0;
            loc[6] += w;
            loc[7] += 1.0;
        }
        free(lp);
    }
    for (int i = 0; i < 8; ++i) sums[i] = acc[i];
}

/* ----------------------------------------------------------------- Adam */
/*
 * pbg/core/optimization.py:182-233 (adam_transition) for one lane (K=1).
 * controls: [lr, beta1, beta2, epsilon, decay, clip, scale, growth, backoff,
 * interval]; decoupled selects AdamW.  Returns 1 when the step applied.
 * Evaluated in double; `norm_out` receives the unscaled gradient 2-norm.
 */
int32_t orc_adam(int64_t n, float *master, float *grad, float *first, float *second,
                 const float *controls, int64_t *step, int32_t decoupled, double *norm_out) {
    double lr = controls[0], b1 = controls[1], b2 = controls[2], epsv = controls[3];
    double decay = controls[4], clip = controls[5], scale = controls[6];
    double ss = 0.0;
    int finite = 1;
    for (int64_t i = 0; i < n; ++i) {
        double g = (double)grad[i] / scale;
        if (!isfinite(g)) finite = 0;
        ss += g * g;
    }
    double norm = sqrt(ss);
    if (!isfinite(norm)) finite = 0;
    *norm_out = norm;
    if (!finite) {
        for (int64_t i = 0; i < n; ++i) grad[i] = 0.0f;
        return 0;
    }
    double nn = norm > 1.0e-12 ? norm : 1.0e-12;
    double clipping = clip / nn;
    if (clipping > 1.0) clipping = 1.0;
    double coupled = decoupled ? 0.0 : decay;
    int64_t t = *step + 1;
    double c1 = 1.0 - pow(b1, (double)t), c2 = 1.0 - pow(b2, (double)t);
    if (c1 < 1.0e-30) c1 = 1.0e-30;
    if (c2 < 1.0e-30) c2 = 1.0e-30;
    double shrink = 1.0 - lr * (decoupled ? decay : 0.0);
    for (int64_t i = 0; i < n; ++i) {
        double g = (double)grad[i] / scale * clipping + coupled * (double)master[i];
        double m = b1 * first[i] + (1.0 - b1) * g;
        double v = b2 * second[i] + (1.0 - b2) * g * g;
        double den = sqrt(v) / sqrt(c2) + epsv;
        double dir = m / c1 / den;
        master[i] = (float)(master[i] * shrink - lr * dir);
        first[i] = (float)m;
        second[i] = (float)v;
        grad[i] = (float)g;
    }
    *step = t;
    return 1;
}

/* ------------------------------------------------------- layered targets */

/*
 * pbg/core/csrc/layered_targets.cu:117-411 (layered_target_kernel, run_layers):
 * lambda-return targets over a topology forest, one node after another in
 * layer order.  Tables hold HOST addresses (int64, 0 = absent) in the layout
 * the CUDA entry point binds: t[0..4] = work0, work1, trace, cost, delta per
 * output; t[5..7] = head_v, head_t, head_c per input; t[8..10] = sigma_v,
 * sigma_t, sigma_c per (lane, input); t[11..12] = action_p, action_a per
 * (lane, action partition).  node columns n[0..11] and child columns follow
 * pbg/core/targets.py:272-282.  Float order follows the reference kernel.
 */
typedef struct {
    const int64_t *tab[13];
    const int32_t *work_cap, *head_cap, *width, *conversion;
    int32_t output_count, input_count, action_partitions, p_train, max_width;
} orc_tables;

static float *tab_f(const int64_t *table, int index) { return (float *)(intptr_t)table[index]; }

static float orc_work(const orc_tables *T, const int64_t *table, int part, int lane, int enc, int p, int d) {
    if (!table || !table[part]) return 0.0f;
    int arena = enc < 0 ? 1 : 0, row = enc < 0 ? -enc - 1 : enc;
    int64_t i = ((((int64_t)lane * T->work_cap[part] + row) * 2 + arena) * T->p_train + p) * T->width[part] + d;
    return tab_f(table, part)[i];
}

static float orc_convert(const orc_tables *T, const int64_t *table, int src, int dst, int lane, int enc, int p, int d) {
    if (src == dst) return orc_work(T, table, src, lane, enc, p, d);
    const int32_t *map = T->conversion + ((int64_t)src * T->output_count + dst) * T->max_width;
    float s = 0.0f;
    for (int h = 0; h < T->width[src]; ++h)
        if (map[h] == d) s += orc_work(T, table, src, lane, enc, p, h);
    return s;
}

static float orc_scalar(const orc_tables *T, const int64_t *table, int part, int lane, int enc) {
    if (!table || !table[part]) return 0.0f;
    int arena = enc < 0 ? 1 : 0, row = enc < 0 ? -enc - 1 : enc;
    return tab_f(table, part)[((int64_t)lane * T->work_cap[part] + row) * 2 + arena];
}

static float orc_trace(const orc_tables *T, int part, int lane, int enc, int p) {
    int arena = enc < 0 ? 1 : 0, row = enc < 0 ? -enc - 1 : enc;
    return tab_f(T->tab[2], part)[(((int64_t)lane * T->work_cap[part] + row) * 2 + arena) * T->p_train + p];
}

static int rb_invalid(float mass, float moment) {
    return !isfinite(moment) || mass < 0.0f || (mass == 0.0f && fabsf(moment) > 1.0e-7f);
}

void orc_layered_targets(const int32_t *layer_ptr, int32_t layers, const int32_t *const *n,
                         const int32_t *src_row, const int32_t *src_type, const int32_t *path,
                         const float *multiplier, const int64_t *const *tables, const int32_t *work_cap,
                         const int32_t *head_cap, const int32_t *width, const int32_t *conversion,
                         int32_t n_replica, int32_t input_count, int32_t output_count,
                         int32_t action_partitions, int32_t p_train, int32_t max_width, float lambda,
                         int32_t sampled, int32_t branched, int32_t *failure_min) {
    orc_tables T;
    for (int i = 0; i < 13; ++i) T.tab[i] = tables[i];
    T.work_cap = work_cap; T.head_cap = head_cap; T.width = width; T.conversion = conversion;
    T.output_count = output_count; T.input_count = input_count; T.action_partitions = action_partitions;
    T.p_train = p_train; T.max_width = max_width;
    const int64_t *W0 = T.tab[0], *W1 = T.tab[1];
    for (int l = 0; l < n_replica; ++l) failure_min[l] = INT32_MAX;
    for (int layer = 0; layer < layers; ++layer) {
        const int arena = (layer + 1) & 1;
        for (int node = layer_ptr[layer]; node < layer_ptr[layer + 1]; ++node) {
            const int lane = n[0][node], begin = n[1][node], dest = n[3][node];
            const int input = n[4][node], output = n[5][node], owner = n[6][node];
            const int nominal = n[7][node], ntgt = n[8][node], head_row = n[9][node], target_row = n[10][node];
            const int action_begin = n[11][node];
            if (failure_min[lane] != INT32_MAX) continue;
            const int w = width[output];
            int bad = 0;
            for (int p = 0; p < p_train; ++p) {
                for (int d = 0; d < w; ++d) {
                    float m0 = 0.0f, m1 = 0.0f;
                    for (int a = 0; a < ntgt; ++a) {
                        int e = begin + a;
                        float c0 = orc_convert(&T, W0, src_type[e], output, lane, src_row[e], p, d);
                        m0 += c0;
                        if (!sampled) {
                            float c1 = orc_convert(&T, W1, src_type[e], output, lane, src_row[e], p, d);
                            m1 += c1;
                            if (rb_invalid(c0, c1)) bad = 1;
                        }
                        if (!isfinite(c0)) bad = 1;
                    }
                    float v0 = m0 / (float)ntgt;
                    float v1 = sampled ? 0.0f : m1 / (float)ntgt;
                    if (p == owner && input >= 0) {
                        float old_v = tab_f(T.tab[5], input)[((int64_t)lane * head_cap[input] + head_row) * w + d];
                        float sigma = sampled ? v0 : (v0 > 0.0f ? v1 / v0 : 0.0f);
                        tab_f(T.tab[8], lane * input_count + input)[(int64_t)target_row * w + d] = sigma;
                        int part = branched ? output : input;
                        float *adv = tab_f(T.tab[12], lane * action_partitions + part);
                        float *post = sampled ? NULL : tab_f(T.tab[11], lane * action_partitions + part);
                        for (int a = 0; a < ntgt; ++a) {
                            int e = begin + a;
                            float c0 = ntgt == 1 ? m0 : orc_convert(&T, W0, src_type[e], output, lane, src_row[e], p, d);
                            float c1 = sampled ? 0.0f
                                               : (ntgt == 1 ? m1 : orc_convert(&T, W1, src_type[e], output, lane, src_row[e], p, d));
                            float base = old_v;
                            if (ntgt > 1) {
                                float s0 = 0.0f, s1 = 0.0f;
                                for (int b = 0; b < ntgt; ++b) {
                                    if (b == a) continue;
                                    int f = begin + b;
                                    s0 += orc_convert(&T, W0, src_type[f], output, lane, src_row[f], p, d);
                                    if (!sampled) s1 += orc_convert(&T, W1, src_type[f], output, lane, src_row[f], p, d);
                                }
                                float cont = sampled ? s0 / (float)(ntgt - 1) : (s0 > 0.0f ? s1 / s0 : 0.0f);
                                base = lambda * cont + (1.0f - lambda) * old_v;
                            }
                            float q = sampled ? c0 : (c0 > 0.0f ? c1 / c0 : 0.0f);
                            int64_t row = (int64_t)action_begin + a;
                            adv[row * w + d] = q - base;
                            if (post) post[row * w + d] = c0;
                            if (!isfinite(q) || !isfinite(base) ||
                                (!sampled && (c0 < 0.0f || (c0 == 0.0f && fabsf(c1) > 1.0e-7f))))
                                bad = 1;
                        }
                        if (sampled) v0 = lambda * v0 + (1.0f - lambda) * old_v;
                        else v1 = lambda * v1 + (1.0f - lambda) * v0 * old_v;
                    }
                    if (!isfinite(v0) || (!sampled && rb_invalid(v0, v1))) bad = 1;
                    int64_t wi = ((((int64_t)lane * work_cap[output] + dest) * 2 + arena) * p_train + p) * w + d;
                    if (W0 && W0[output]) tab_f(W0, output)[wi] = v0;
                    if (!sampled && W1 && W1[output]) tab_f(W1, output)[wi] = v1;
                }
            }
            if (branched) {
                float dbar = 0.0f, craw = 0.0f;
                for (int a = 0; a < ntgt; ++a) {
                    int e = begin + a;
                    dbar += orc_scalar(&T, T.tab[4], src_type[e], lane, src_row[e]);
                    craw += (float)path[e] + multiplier[e] * orc_scalar(&T, T.tab[3], src_type[e], lane, src_row[e]);
                }
                dbar /= (float)ntgt;
                craw /= (float)ntgt;
                float texec = 0.0f;
                for (int p = 0; p < p_train; ++p) {
                    float mean = 0.0f;
                    for (int a = 0; a < ntgt; ++a) mean += orc_trace(&T, src_type[begin + a], lane, src_row[begin + a], p);
                    mean /= (float)ntgt;
                    tab_f(T.tab[2], output)[(((int64_t)lane * work_cap[output] + dest) * 2 + arena) * p_train + p] = mean;
                    if (ntgt > 1)
                        for (int a = 0; a < ntgt; ++a) {
                            float dv = orc_trace(&T, src_type[begin + a], lane, src_row[begin + a], p) - mean;
                            texec += dv * dv;
                        }
                }
                if (ntgt > 1) texec /= (float)(ntgt - 1);
                float pdelta = dbar / (float)ntgt, pcost = craw;
                if (input >= 0) {
                    int64_t hi = (int64_t)lane * head_cap[input] + head_row;
                    float old_t = tab_f(T.tab[6], input)[hi], old_c = tab_f(T.tab[7], input)[hi];
                    float that = ntgt > 1 ? fmaxf(0.0f, texec - dbar) : 0.0f;
                    float tstar = ntgt > 1 ? that : old_t;
                    pdelta = (tstar + dbar) / (float)ntgt - tstar / (float)nominal;
                    pcost = lambda * craw + (1.0f - lambda) * old_c;
                    tab_f(T.tab[9], lane * input_count + input)[target_row] = that;
                    tab_f(T.tab[10], lane * input_count + input)[target_row] = craw;
                }
                int64_t si = ((int64_t)lane * work_cap[output] + dest) * 2 + arena;
                if (T.tab[3] && T.tab[3][output]) tab_f(T.tab[3], output)[si] = pcost;
                if (T.tab[4] && T.tab[4][output]) tab_f(T.tab[4], output)[si] = pdelta;
                if (!isfinite(texec) || !isfinite(pcost) || !isfinite(pdelta)) bad = 1;
            }
            if (bad && node < failure_min[lane]) failure_min[lane] = node;
        }
    }
}

/* --------------------------------------------- collision-conditioned sampler */

/*
 * pbg/games/poker/queued/rb_sampling.py:86-223
 * (CollisionConditionedProfileSampler.sample_children).  Per parent and seat:
 * board-conflicting private hands get weight 0; the seat's mass and CDF are
 * prefix sums accumulated in double and rounded to fp32 per entry (torch's
 * CPU cumsum).  Per fresh child row (active and ordinal > 0): for attempts
 * a = 0..max_attempts-1, every seat draws a POSTERIOR key at (root, path,
 * draw a, lane seat, retry epoch), target = min(u*mass, nextafter(mass, 0)),
 * and takes the first CDF entry strictly above the target (an 11-step fixed
 * bisection, rb_sampling.py:31-55); the first attempt whose seats' hands
 * share no card wins.  Other rows, and rows whose attempts all collide, keep
 * the parent's inherited profile.  `margin` (optional, per row) receives the
 * smallest distance from a target to a bounding CDF edge over the attempts
 * up to the accepted one, divided by the seat mass: where it is tiny another
 * summation order may pick a neighbouring hand.
 */
void orc_posterior_sample(orc_geom g, int64_t B, const float *weights, const uint8_t *board,
                          const int32_t *inherited, int64_t G, const int64_t *source, const int64_t *ordinal,
                          const uint8_t *active, const int64_t *root, const int64_t *path, int64_t seed,
                          int64_t iteration, const int64_t *epoch, int32_t max_attempts, int32_t *out,
                          int32_t *attempt_count, uint8_t *exhausted, int64_t *min_failing, double *margin) {
    const int P = g.players, D = 4 * g.rank_count, first = 52 - D, H = D * (D - 1) / 2;
    int *c0 = (int *)malloc(sizeof(int) * H), *c1 = (int *)malloc(sizeof(int) * H);
    for (int i = 0, id = 0; i < D; ++i)
        for (int j = i + 1; j < D; ++j, ++id) {
            c0[id] = i + first;
            c1[id] = j + first;
        }
    float *cdf = (float *)malloc(sizeof(float) * (size_t)B * P * H);
    float *mass = (float *)malloc(sizeof(float) * (size_t)B * P);
    for (int64_t b = 0; b < B; ++b) {
        for (int p = 0; p < P; ++p) {
            double run = 0.0;
            const float *w = weights + ((size_t)b * P + p) * H;
            float *c = cdf + ((size_t)b * P + p) * H;
            for (int h = 0; h < H; ++h) {
                int blocked = 0;
                for (int k = 0; k < 5; ++k) {
                    int card = board[b * 5 + k];
                    if (card != 255 && (card == c0[h] || card == c1[h])) blocked = 1;
                }
                run += blocked ? 0.0 : (double)w[h];
                c[h] = (float)run;
            }
            mass[(size_t)b * P + p] = (float)run;
        }
    }
    uint64_t ns = rng_namespace(seed, iteration, 3 /* POSTERIOR */);
    int64_t worst = INT64_MAX;
    int32_t *sel = (int32_t *)malloc(sizeof(int32_t) * P);
    for (int64_t r = 0; r < G; ++r) {
        const int64_t src = source[r];
        const int fresh = active[r] && ordinal[r] > 0;
        double row_margin = 1.0;
        attempt_count[r] = 0;
        exhausted[r] = 0;
        for (int p = 0; p < P; ++p) out[r * P + p] = inherited[src * P + p];
        if (fresh) {
            int accepted = -1;
            for (int a = 0; a < max_attempts && accepted < 0; ++a) {
                for (int p = 0; p < P; ++p) {
                    const float total = mass[(size_t)src * P + p];
                    const float *c = cdf + ((size_t)src * P + p) * H;
                    float target = uniform_of(rng_key(ns, root[r], path[r], a, p, epoch[r])) * total;
                    const float cap = nextafterf(total, 0.0f);
                    if (cap < target) target = cap;
                    int lo = 0, hi = H;
                    for (int step = 0; step < 11; ++step) {
                        int mid = (lo + hi) >> 1;
                        int safe = mid < H - 1 ? mid : H - 1;
                        int below = mid < H && c[safe] <= target;
                        if (below) lo = mid + 1;
                        else hi = mid;
                    }
                    sel[p] = lo < H - 1 ? lo : H - 1;
                    if (margin && total > 0.0f) {
                        double up = (double)c[sel[p]] - target;
                        double down = sel[p] > 0 ? (double)target - c[sel[p] - 1] : (double)target;
                        double m = (up < down ? up : down) / total;
                        if (m < 0) m = -m;
                        if (m < row_margin) row_margin = m;
                    }
                }
                int clash = 0;
                for (int p = 0; p < P && !clash; ++p)
                    for (int q = p + 1; q < P && !clash; ++q)
                        if (c0[sel[p]] == c0[sel[q]] || c0[sel[p]] == c1[sel[q]] || c1[sel[p]] == c0[sel[q]] ||
                            c1[sel[p]] == c1[sel[q]])
                            clash = 1;
                if (!clash) accepted = a;
            }
            if (accepted >= 0) {
                for (int p = 0; p < P; ++p) out[r * P + p] = sel[p];
                attempt_count[r] = accepted + 1;
            } else {
                exhausted[r] = 1;
                attempt_count[r] = max_attempts;
                if (path[r] < worst) worst = path[r];
            }
        }
        if (margin) margin[r] = row_margin;
    }
    *min_failing = worst;
    free(sel);
    free(mass);
    free(cdf);
    free(c0);
    free(c1);
}

/* ------------------------------------------------ branched learner sampling */

/* pbg/core/csrc/alias_table.cu:11-44: Vose's two-stack Walker construction
 * over scaled weights (float64), in the reference's push/pop order. */
void orc_alias_table(int64_t n, double *scaled, double *probability, int32_t *alias) {
    int64_t *small = (int64_t *)malloc(sizeof(int64_t) * n), *large = (int64_t *)malloc(sizeof(int64_t) * n);
    int64_t ns = 0, nl = 0;
    for (int64_t i = 0; i < n; ++i) {
        probability[i] = 1.0;
        alias[i] = (int32_t)i;
        if (scaled[i] < 1.0) small[ns++] = i;
        else large[nl++] = i;
    }
    while (ns != 0 && nl != 0) {
        int64_t low = small[--ns], high = large[--nl];
        double p = scaled[low];
        probability[low] = p;
        alias[low] = (int32_t)high;
        scaled[high] -= 1.0 - p;
        if (scaled[high] < 1.0) small[ns++] = high;
        else large[nl++] = high;
    }
    free(small);
    free(large);
}

/* pbg/core/csrc/branching_metadata.cu:9-31: decision log mass in node order;
 * returns the failure code (0, 1 or 2) of the first failing node. */
int32_t orc_decision_log_mass(int64_t n, const int32_t *parent, const int32_t *degree, float *log_mass) {
    for (int64_t v = 0; v < n; ++v) {
        int32_t a = parent[v];
        if (a >= v) return 1;
        if (a < 0) {
            log_mass[v] = 0.0f;
            continue;
        }
        if (degree[a] <= 0) return 2;
        log_mass[v] = log_mass[a] - logf((float)degree[a]);
    }
    return 0;
}

/* ------------------------------------------------ Rao-Blackwell completion */

/* Restatement of this build's estimator of the contract-v2 `complete` /
 * `complete_selected` law (PreTerminalMC, docs/theory/core_math.tex:664-684,
 * 1360-1380; called at pbg/games/poker/queued/hooks.py:2472-2477, 2512 on the
 * rows of PokerStateMachine.rb_leaf, hooks.py:1218-1258).  The external
 * evaluator's own implementation is not in the reference tree, so parity with
 * it is unpinned; this function fixes the estimator the device kernel must
 * reproduce bit for bit:
 *   - range weights: non-positive, non-finite and board-conflicting hands
 *     weigh 0;
 *   - per seat, an fp32 CDF rounded from a double running sum whose 32
 *     contiguous segments (ceil(H/32) rounded up to 4 hands) start from an
 *     inclusive Kogge-Stone scan of the segment totals; Z = the double total;
 *     per-card masses: the hands holding the card in hand-id order as four
 *     running sums of every fourth term, then (s0 + s1) + (s2 + s3);
 *   - sample i (base key rng_key(root i) in the COMPLETION namespace of the
 *     row's seed; draw `code` uses mix63(base + (code + 1) * 0x9E3779B97F4A7C15)),
 *     seats q in order: Z(dead) = (Z - the dead cards' masses, seat by seat) +
 *     (each earlier hand's own weight, then its four cross pairs with the hands
 *     before it); the weight multiplies by Z(dead)/Z; up to 16 CDF proposals
 *     (codes 32q + attempt), the first disjoint from `dead` with positive
 *     weight wins; else an exact scan of the restricted range (code 32q + 16);
 *   - missing board slots j dealt uniformly from the unused deck (code
 *     1024 + j); returns settled as evaluate_showdowns settles them;
 *   - 64-bit fixed-point sums of q_i = rint(w_i 2^(Q-ew)) and
 *     rint(w_i R 2^(Q-ew-er)), Q = 61 - ceil(log2 N); then in single precision
 *     p_hat = float(sum q) * float(1/W), v_hat = float(sum m) * (1 / float(sum q))
 *     * 2^er; n_eff = W^2 / sum q^2 with sum q^2 reduced
 *     as 256 thread-strided partial sums, 32-lane butterflies and warps in
 *     order.
 * Returns the status bits (1: invalid board card or selected seat, 2: a row
 * without sample mass). */

#define RB_THREADS 256
#define RB_ATTEMPTS 16

static int rb_pair_id(int D, int a, int b) {
    int lo = a < b ? a : b, hi = a < b ? b : a;
    return lo * (2 * D - lo - 1) / 2 + hi - lo - 1;
}

static float rb_uniform(int64_t base, int code) {
    return uniform_of(mix63((int64_t)(((uint64_t)base + (uint64_t)(code + 1) * 0x9E3779B97F4A7C15ULL) & M63)));
}

static int rb_ceil_log2(int n) {
    int k = 0;
    while ((1 << k) < n) ++k;
    return k;
}

static int64_t rb_hand_value(int R, const int *strength, const int *cards7) {
    int64_t best = -1;
    int sub[5];
    for (int a = 0; a < 7; ++a)
        for (int b2 = a + 1; b2 < 7; ++b2) {
            int n = 0;
            for (int i = 0; i < 7; ++i) if (i != a && i != b2) sub[n++] = cards7[i];
            int64_t v = five_value(sub, strength, R);
            if (v > best) best = v;
        }
    return best;
}

int32_t orc_rb_complete(int32_t R, int64_t F, int32_t P, int32_t strata, int32_t N, const uint8_t *board,
                        const float *weights, const int32_t *level, const float *baseline, const float *amount,
                        const int64_t *seed, const int32_t *selected, float *p_hat, float *v_hat, float *n_eff) {
    const int D = 4 * R, first = 52 - D, H = D * (D - 1) / 2;
    const uint64_t deck = (1ULL << D) - 1ULL;
    int strength[N_CAT];
    category_strength(R, strength);
    int *hc = malloc(sizeof(int) * 2 * H);
    float *wb = malloc(sizeof(float) * P * H), *cdf = malloc(sizeof(float) * P * H);
    double *mass = malloc(sizeof(double) * P * D), *zd = malloc(sizeof(double) * P);
    double *rw = malloc(sizeof(double) * N);
    int *rh = malloc(sizeof(int) * N * P);
    float *rr = malloc(sizeof(float) * N * P);
    long long *pacc = malloc(sizeof(long long) * H), *vacc = malloc(sizeof(long long) * H);
    int32_t status = 0;
    for (int a = 0, id = 0; a < D; ++a)
        for (int b = a + 1; b < D; ++b, ++id) {
            hc[2 * id] = a;
            hc[2 * id + 1] = b;
        }
    const int outputs = selected ? 1 : P;
    for (int64_t f = 0; f < F; ++f) {
        uint64_t bmask = 0;
        int bc[5], bad = 0;
        for (int j = 0; j < 5; ++j) {
            int c = board[f * 5 + j];
            bc[j] = c;
            if (c == 255) continue;
            if (c < first || c >= 52 || ((bmask >> (c - first)) & 1ULL)) bad = 1;
            else bmask |= 1ULL << (c - first);
        }
        int sel = selected ? selected[f] : 0;
        if (selected && (sel < 0 || sel >= P)) bad = 1;
        if (bad) {
            for (int64_t k = 0; k < (int64_t)outputs * H; ++k) {
                p_hat[f * outputs * H + k] = 0.0f;
                v_hat[f * outputs * H + k] = 0.0f;
            }
            n_eff[f] = 0.0f;
            status |= 1;
            continue;
        }
        for (int idx = 0; idx < P * H; ++idx) {
            int h = idx % H;
            float x = weights[f * P * H + idx];
            int conflict = (int)(((bmask >> hc[2 * h]) | (bmask >> hc[2 * h + 1])) & 1ULL);
            wb[idx] = (x > 0.0f && x <= FLT_MAX && !conflict) ? x : 0.0f;
        }
        for (int q = 0; q < P; ++q) {
            const float *w = wb + q * H;
            int seg = (((H + 31) / 32) + 3) & ~3;
            double v[32], nv[32];
            for (int l = 0; l < 32; ++l) {
                int lo = l * seg < H ? l * seg : H, hi = lo + seg < H ? lo + seg : H;
                double local = 0.0;
                for (int h = lo; h < hi; ++h) local = local + (double)w[h];
                v[l] = local;
            }
            for (int o = 1; o < 32; o <<= 1) {
                for (int l = 0; l < 32; ++l) nv[l] = l >= o ? v[l - o] + v[l] : v[l];
                memcpy(v, nv, sizeof v);
            }
            for (int l = 0; l < 32; ++l) {
                int lo = l * seg < H ? l * seg : H, hi = lo + seg < H ? lo + seg : H;
                double run = l ? v[l - 1] : 0.0;
                for (int h = lo; h < hi; ++h) {
                    run = run + (double)w[h];
                    cdf[q * H + h] = (float)run;
                }
                if (l == 31) zd[q] = run;
            }
            for (int c = 0; c < D; ++c) {
                double part[4] = {0.0, 0.0, 0.0, 0.0};
                for (int t = 0; t < D - 1; ++t) {
                    int id = t < c ? rb_pair_id(D, t, c) : rb_pair_id(D, c, t + 1);
                    part[t & 3] = part[t & 3] + (double)w[id];
                }
                mass[q * D + c] = (part[0] + part[1]) + (part[2] + part[3]);
            }
        }
        const uint64_t ns = rng_namespace(seed[f], 0, 6 /* COMPLETION */);
        for (int i = 0; i < N; ++i) {
            const int64_t key = rng_key(ns, i, 0, 0, 0, 0);
            double weight = 1.0;
            uint64_t dead = 0;
            int hand[6] = {0, 0, 0, 0, 0, 0}, ca[6] = {0, 0, 0, 0, 0, 0}, cb[6] = {0, 0, 0, 0, 0, 0};
            for (int q = 0; q < P; ++q) {
                const float *w = wb + q * H, *c = cdf + q * H;
                const double *m = mass + q * D;
                double z = zd[q], s1 = 0.0, s2 = 0.0;
                for (int j = 0; j < q; ++j) {
                    s1 = s1 + m[ca[j]];
                    s1 = s1 + m[cb[j]];
                }
                for (int j = 0; j < q; ++j) {
                    s2 = s2 + (double)w[hand[j]];
                    for (int k = 0; k < j; ++k) {
                        s2 = s2 + (double)w[rb_pair_id(D, ca[k], ca[j])];
                        s2 = s2 + (double)w[rb_pair_id(D, ca[k], cb[j])];
                        s2 = s2 + (double)w[rb_pair_id(D, cb[k], ca[j])];
                        s2 = s2 + (double)w[rb_pair_id(D, cb[k], cb[j])];
                    }
                }
                double zs = (z - s1) + s2;
                if (!(z > 0.0) || !(zs > 0.0)) {
                    weight = 0.0;
                    break;
                }
                weight = weight * (zs / z);
                int pick = -1;
                float top = c[H - 1];
                if (top > 0.0f) {
                    float below = nextafterf(top, 0.0f);
                    for (int a = 0; a < RB_ATTEMPTS; ++a) {
                        float u = rb_uniform(key, q * 32 + a);
                        float t = u * top;
                        if (t > below) t = below;
                        int lo = 0, hi = H;
                        while (lo < hi) {
                            int mid = (lo + hi) >> 1;
                            if (c[mid] > t) hi = mid;
                            else lo = mid + 1;
                        }
                        if (lo >= H) lo = H - 1;
                        int clash = (int)(((dead >> hc[2 * lo]) | (dead >> hc[2 * lo + 1])) & 1ULL);
                        if (!clash && w[lo] > 0.0f) {
                            pick = lo;
                            break;
                        }
                    }
                }
                if (pick < 0) {
                    double t = (double)rb_uniform(key, q * 32 + RB_ATTEMPTS) * zs;
                    double run = 0.0;
                    for (int h = 0; h < H; ++h) {
                        float x = w[h];
                        if (!(x > 0.0f)) continue;
                        if (((dead >> hc[2 * h]) | (dead >> hc[2 * h + 1])) & 1ULL) continue;
                        run = run + (double)x;
                        pick = h;
                        if (run > t) break;
                    }
                }
                if (pick < 0) {
                    weight = 0.0;
                    break;
                }
                hand[q] = pick;
                ca[q] = hc[2 * pick];
                cb[q] = hc[2 * pick + 1];
                dead |= (1ULL << ca[q]) | (1ULL << cb[q]);
            }
            float ret[6] = {0, 0, 0, 0, 0, 0};
            if (weight > 0.0) {
                uint64_t used = bmask | dead;
                int cards[7];
                for (int j = 0; j < 5; ++j) {
                    int card = bc[j];
                    if (card == 255) {
                        uint64_t avail = deck & ~used;
                        int n = __builtin_popcountll(avail);
                        float u = rb_uniform(key, 1024 + j);
                        int k = (int)(u * (float)n);
                        if (k >= n) k = n - 1;
                        uint64_t r = avail;
                        for (; k > 0; --k) r &= r - 1;
                        int local = __builtin_ctzll(r);
                        used |= 1ULL << local;
                        card = local + first;
                    }
                    cards[j] = card;
                }
                int64_t value[6];
                for (int p = 0; p < P; ++p) {
                    value[p] = -1;
                    if (level[f * P + p] >= 0) {
                        cards[5] = hc[2 * hand[p]] + first;
                        cards[6] = hc[2 * hand[p] + 1] + first;
                        value[p] = rb_hand_value(R, strength, cards);
                    }
                    ret[p] = baseline[f * P + p];
                }
                for (int k = 0; k < strata; ++k) {
                    float amt = amount[f * strata + k];
                    if (!(amt > 0.0f)) continue;
                    int64_t best = -1;
                    for (int p = 0; p < P; ++p)
                        if (value[p] >= 0 && level[f * P + p] >= k && value[p] > best) best = value[p];
                    if (best < 0) continue;
                    int winners = 0;
                    for (int p = 0; p < P; ++p) winners += value[p] == best && level[f * P + p] >= k;
                    float share = amt / (float)winners;
                    for (int p = 0; p < P; ++p)
                        if (value[p] == best && level[f * P + p] >= k) ret[p] += share;
                }
            }
            rw[i] = weight;
            for (int p = 0; p < P; ++p) {
                rh[i * P + p] = hand[p];
                rr[i * P + p] = ret[p];
            }
        }
        double mw = 0.0, mr = 0.0;
        for (int i = 0; i < N; ++i) {
            if (!(rw[i] > 0.0)) continue;
            mw = fmax(mw, rw[i]);
            for (int p = 0; p < P; ++p) mr = fmax(mr, fabs((double)rr[i * P + p]));
        }
        int ew = 0, er = 0;
        frexp(mw, &ew);
        frexp(mr, &er);
        const int Q = 61 - rb_ceil_log2(N);
        long long W = 0;
        double part[RB_THREADS];
        for (int t = 0; t < RB_THREADS; ++t) {
            double sq = 0.0;
            for (int i = t; i < N; i += RB_THREADS) {
                long long qi = llrint(ldexp(rw[i], Q - ew));
                W += qi;
                double qd = (double)qi;
                sq = sq + qd * qd;
            }
            part[t] = sq;
        }
        double S2 = 0.0;
        for (int wp = 0; wp < RB_THREADS / 32; ++wp) {
            double v[32], nv[32];
            memcpy(v, part + 32 * wp, sizeof v);
            for (int o = 16; o > 0; o >>= 1) {
                for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
                memcpy(v, nv, sizeof v);
            }
            S2 = S2 + v[0];
        }
        const double Wd = (double)W;
        const float inv_w = W > 0 ? (float)(1.0 / Wd) : 0.0f;
        const float scale_r = ldexpf(1.0f, er < 127 ? er : 127);
        for (int o = 0; o < outputs; ++o) {
            int p = selected ? sel : o;
            memset(pacc, 0, sizeof(long long) * H);
            memset(vacc, 0, sizeof(long long) * H);
            for (int i = 0; i < N; ++i) {
                double x = rw[i];
                if (!(x > 0.0)) continue;
                int h = rh[i * P + p];
                pacc[h] += llrint(ldexp(x, Q - ew));
                vacc[h] += llrint(ldexp(x * (double)rr[i * P + p], Q - ew - er));
            }
            float *po = p_hat + (f * outputs + o) * (int64_t)H, *vo = v_hat + (f * outputs + o) * (int64_t)H;
            for (int h = 0; h < H; ++h) {
                if (pacc[h] != 0) {
                    float nf = (float)pacc[h], mf = (float)vacc[h];
                    po[h] = nf * inv_w;
                    vo[h] = (mf * (1.0f / nf)) * scale_r;
                } else {
                    po[h] = 0.0f;
                    vo[h] = 0.0f;
                }
            }
        }
        n_eff[f] = W > 0 ? (float)fmin(Wd * Wd / S2, (double)N) : 0.0f;
        if (W <= 0) status |= 2;
    }
    free(hc); free(wb); free(cdf); free(mass); free(zd); free(rw); free(rh); free(rr); free(pacc); free(vacc);
    return status;
}
