/*
 * pbgb200.h -- C ABI of libpbgb200.so, the B200 (sm_100a) hot path of pbg.
 *
 * Conventions
 *   - Every pointer is a device pointer owned by the caller (torch tensors in
 *     the Python host layer).  No entry point allocates device memory unless
 *     its comment says so; scratch buffers are passed in by the caller.
 *   - `stream` is a cudaStream_t passed as void*; work is stream-ordered and
 *     asynchronous.  No entry point synchronises the host.
 *   - Every entry point returns 0 on success or a negative PBG_E* code; the
 *     message of the last failure on the calling thread is pbg_last_error().
 *     No exception crosses the ABI; no device code traps.
 *   - Dtypes mirror the reference's tensors: bool columns are uint8 (0/1),
 *     int8 status, int32 ids, fp32 chips, int64 logical keys.
 *
 * Reference interfaces are cited as path:line inside the pbg project
 * (pbustillo05/ai-game-learning).
 */
#ifndef PBGB200_H
#define PBGB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PBG_OK 0
#define PBG_EINVAL (-1)   /* bad argument (shape, geometry, null pointer) */
#define PBG_ECUDA (-2)    /* a CUDA runtime call failed */
#define PBG_ERANGE (-3)   /* a size exceeds a documented maximum */

/* NLHE geometry: hooks.py:72-192 (NLHEGeometry).  stack_ticks = 2*stack_bb. */
typedef struct {
    int32_t players;     /* P in [2,6] */
    int32_t stack_ticks; /* T in [16,256]; events E = T + 2 */
    int32_t rank_count;  /* R in [4,13]; deck D = 4R cards 52-D..51 */
} pbg_geometry;

/* Public state of B hands, hooks.py:250-326 (PokerState), SoA columns. */
typedef struct {
    uint8_t *board;            /* [B,5], PAD 255 */
    int32_t *combo;            /* [B,P] compact combo ids */
    int32_t *button;           /* [B] */
    int32_t *street;           /* [B] 0..3 */
    int32_t *to_act;           /* [B] */
    float *stacks;             /* [B,P] */
    float *committed;          /* [B,P] */
    float *committed_street;   /* [B,P] */
    int8_t *status;            /* [B,P] LIVE 0, FOLDED 1, ALL_IN 2 */
    float *current_bet;        /* [B] */
    float *last_full_raise;    /* [B] */
    uint8_t *pending;          /* [B,P] */
    uint8_t *can_raise;        /* [B,P] */
    uint8_t *terminal;         /* [B] */
} pbg_state;

/* Public action history, hooks.py:329-339 (PokerHistory), [B,tokens]. */
typedef struct {
    int64_t *actor;
    int64_t *street;
    int64_t *action;
    float *amount;
    float *pot_before;
    float *call_amount;
    float *current_bet;
    float *min_raise_to;
    float *max_raise_to;
    uint8_t *mask;
    int32_t tokens;  /* model/capacity.py:22-25 bound */
    int32_t *length; /* [B] tokens used, kept current by every append; NULL = count the mask */
} pbg_history;

/* Sampled settlement inputs, hooks.py:1145-1216 (sampled_leaf) output. */
typedef struct {
    uint8_t *board;       /* [B,5] leaf_public_state */
    int32_t *combo;       /* [B,P] leaf_private_profile */
    int32_t *level;       /* [B,P] stratum_level */
    float *baseline;      /* [B,P] payoff_baseline */
    float *amount;        /* [B,P] stratum_amount (K_strata = P) */
} pbg_leaf;

/* Raw composite-policy fields, policy.py:113-204, laid out [B, rows, ...]. */
typedef struct {
    const float *type_logits; /* [B,rows,3] */
    const float *omega;       /* [B,rows,M] */
    const float *mu;          /* [B,rows,M] */
    const float *scale;       /* [B,rows,M]  ("s") */
    const float *iota;        /* [B,rows] */
    int32_t rows;             /* 1 = already selected at the actor's row */
    int32_t mixtures;         /* M in [1,8] */
} pbg_policy;

/* Gradients of the raw composite-policy fields, same layout as pbg_policy. */
typedef struct {
    float *type_logits; /* [B,rows,3] */
    float *omega;       /* [B,rows,M] */
    float *mu;          /* [B,rows,M] */
    float *scale;       /* [B,rows,M] */
    float *iota;        /* [B,rows] */
} pbg_policy_grad;

const char *pbg_last_error(void);
int32_t pbg_abi_version(void);

/* ---------------------------------------------------------------- RNG */

/* rollout.py:122-181 (logical_rng_keys): out[i] = key of the address
 * (root[i], path[i], draw[i], lane[i], epoch[i]) in the (seed, iteration,
 * purpose) namespace; 0 where active[i]==0 (active may be NULL). */
int pbg_rng_keys(int64_t seed, int64_t iteration, int64_t purpose, int64_t n,
                 const int64_t *root, const int64_t *path, const int64_t *draw,
                 const int64_t *lane, const int64_t *epoch, const uint8_t *active,
                 int64_t *out, void *stream);

/* rollout.py:184-202 (child_path_keys). */
int pbg_child_path(int64_t n, const int64_t *path, const int64_t *ordinal, int64_t *out,
                   void *stream);

/* rollout.py:205-234 (logical_uniform). */
int pbg_logical_uniform(int64_t n, const int64_t *keys, float *out, void *stream);

/* rollout.py:237-267 (logical_categorical): p [B,E] fp32, mass [B] or NULL. */
int pbg_logical_categorical(int64_t B, int32_t E, const float *p, const int64_t *keys,
                            const float *mass, int64_t *out, void *stream);

/* ------------------------------------------------------- state machine */

/* hooks.py:357-454 (PokerStateMachine.initial_roots); buttons may be NULL. */
int pbg_initial_roots(pbg_geometry g, int64_t rows, int64_t seed, int64_t iteration,
                      int64_t retry_epoch, int64_t logical_base, int64_t lane,
                      const int32_t *buttons, pbg_state st, void *stream);

/* hooks.py:464-510 (legality): mask [B,E] uint8. */
int pbg_legality(pbg_geometry g, int64_t B, pbg_state st, uint8_t *mask, void *stream);

/* hooks.py:456-462 (input_type): pre=0, post_A=A-1. */
int pbg_input_type(pbg_geometry g, int64_t B, pbg_state st, int32_t *out, void *stream);

/* hooks.py:883-979 (step_player), in place. */
int pbg_step_player(pbg_geometry g, int64_t B, pbg_state st, const int32_t *action,
                    void *stream);

/* hooks.py:981-987 (needs_chance). */
int pbg_needs_chance(pbg_geometry g, int64_t B, pbg_state st, uint8_t *out, void *stream);

/* hooks.py:989-1074 (deal_next_street) with explicit keys [B,D]; active may
 * be NULL. In place. */
int pbg_deal_next_street(pbg_geometry g, int64_t B, pbg_state st, const int64_t *keys,
                         const uint8_t *active, void *stream);

/* hooks.py:1076-1126 (deal_next_street_keyed): CHANCE keys at (root, path)
 * with draw*D + card ordinal.  retry/lane are [B]. */
int pbg_deal_next_street_keyed(pbg_geometry g, int64_t B, pbg_state st, int64_t seed,
                               int64_t iteration, const int64_t *root, const int64_t *path,
                               int64_t draw, const int64_t *retry, const int64_t *lane,
                               const uint8_t *active, void *stream);

/* hooks.py:733-785 (append_player_history), from the pre-action state. */
int pbg_append_player_history(pbg_geometry g, int64_t B, pbg_state st, const int32_t *action,
                              pbg_history h, void *stream);

/* hooks.py:787-810 (append_chance_history). */
int pbg_append_chance_history(pbg_geometry g, int64_t B, pbg_state st, const uint8_t *active,
                              pbg_history h, void *stream);

/* hooks.py:1145-1216 (sampled_leaf) of every row treated as terminal. */
int pbg_sampled_leaf(pbg_geometry g, int64_t B, pbg_state st, pbg_leaf leaf, void *stream);

/* hooks.py:1128-1143 (combo_cards): out [n,2] int64. */
int pbg_combo_cards(pbg_geometry g, int64_t n, const int32_t *ids, int64_t *out, void *stream);

/* hooks.py:655-674 (_combo_class): out [H] int32. */
int pbg_combo_class(pbg_geometry g, int32_t *out, void *stream);

/* hooks.py:531-612 (direct_model_input) with hooks.py:630-648
 * (_compact_preflop_reach): out [B,width] fp32 rows.  input_type 0 = "pre"
 * (class-compact reach), 1 = "post_*" (exact reach, folded-summary zeros
 * when P > 2).  log_reach is the exact [B,P,H] reach or NULL (class counts
 * preflop, zeros after); hist.mask NULL means an empty history of
 * hist.tokens slots.  width must equal the reference's row width. */
int pbg_direct_model_input(pbg_geometry g, int64_t B, pbg_state st, int32_t input_type,
                           const float *log_reach, pbg_history hist, float *out, int64_t width,
                           void *stream);

/* ----------------------------------------------------------- showdown */

/* Contract-v2 evaluate_showdowns of the external poker_gpu_evaluator, as
 * called at hooks.py:2277-2295: payoff[b,p] = baseline[b,p] + equal shares
 * of amount[b,k] among the best 7-card hands of seats with level >= k.
 * Category order per deck follows cards.py:37-74 (category_profile). */
int pbg_evaluate_showdowns(int32_t rank_count, int64_t B, int32_t P, int32_t strata,
                           const uint8_t *board, const int32_t *combo, const int32_t *level,
                           const float *baseline, const float *amount, float *out,
                           void *stream);

/* Best 7-card hand values (strength-major) for n hands: cards [n,7] int32. */
int pbg_hand_values(int32_t rank_count, int64_t n, const int32_t *cards, int64_t *out,
                    void *stream);

/* Contract-v2 `complete` / `complete_selected` of the external
 * poker_gpu_evaluator, as called by RBCompletionBinding.leaf_to_layer_work
 * (hooks.py:2472-2477, 2512) on PokerStateMachine.rb_leaf rows
 * (hooks.py:1218-1258): the PreTerminalMC law of core_math.tex:664-684.
 * Per leaf row f: board u8 [F,5] (255 = not dealt), range_weights f32
 * [F,P,H], level i32 [F,P], baseline f32 [F,P], amount f32 [F,strata],
 * seed i64 [F]; n_samples importance-weighted profiles (sequential over the
 * seats), the missing board dealt uniformly, returns settled by strata.
 * selected NULL: p_hat, v_hat f32 [F,P,H]; else selected i32 [F] and p_hat,
 * v_hat f32 [F,H] (bit-identical to the dense slice).  n_eff f32 [F] (the
 * effective sample size, <= n_samples).  *status (device, caller-zeroed):
 * bit 1 an invalid board card or selected seat (the row publishes zeros),
 * bit 2 a row without sample mass (n_eff = 0).  Deterministic. */
int pbg_rb_complete(int32_t rank_count, int64_t F, int32_t P, int32_t strata, int32_t n_samples,
                    const uint8_t *board, const float *range_weights, const int32_t *level,
                    const float *baseline, const float *amount, const int64_t *seed,
                    const int32_t *selected, float *p_hat, float *v_hat, float *n_eff,
                    uint32_t *status, void *stream);

/* Largest n_samples pbg_rb_complete accepts for this deck and seat count
 * (one leaf's tables and sample records in one CTA's shared memory); 0 for
 * an invalid geometry. */
int32_t pbg_rb_complete_max_samples(int32_t rank_count, int32_t P);

/* ------------------------------------------------------------- policy */

/* policy.py:113-204 (PokerPolicyOperator.probabilities): out [B*rows,E];
 * mask [B,E] is shared by the `rows` policy rows of each hand. */
int pbg_policy_probabilities(int64_t B, int32_t E, pbg_policy pol, const uint8_t *mask,
                             float *out, void *stream);

/* policy.py:206-233 (selected_log_pi) for every policy row: out [B*rows]. */
int pbg_policy_selected_log_pi(int64_t B, int32_t E, pbg_policy pol, const uint8_t *mask,
                               const int32_t *action, float *out, void *stream);

/* policy.py:235-244 (policy_reductions) without reference: entropy [B*rows]. */
int pbg_policy_entropy(int64_t B, int32_t E, pbg_policy pol, const uint8_t *mask,
                       float *out, void *stream);

/* policy.py:246-282 (sample_actor): hand [B] selects the row of each hand. */
int pbg_policy_sample_actor(int64_t B, int32_t E, pbg_policy pol, const uint8_t *mask,
                            const int32_t *hand, const int64_t *keys, int32_t *action,
                            float *selected_log, void *stream);

/* PokerPolicyOperator.learner forward (pbg/games/poker/queued/policy.py:284-298):
 * per policy row [B*rows] the selected log pi of action[b] (clamped at
 * 1e-12), the entropy and KL(p || q) against reference fields of the same
 * layout (kl = 0 when reference is NULL). */
int pbg_policy_learner_forward(int64_t B, int32_t E, pbg_policy raw, const pbg_policy *reference,
                               const uint8_t *mask, const int32_t *action, float *selected,
                               float *entropy, float *kl, void *stream);

/* Vector-Jacobian product of PokerPolicyOperator.learner
 * (pbg/games/poker/queued/policy.py:284-298, the reference's autograd
 * backward through its composite policy): upstream gradients of the
 * selected log pi, entropy and reference KL [B*rows] (each may be NULL) ->
 * gradients of the raw fields [B, rows, ...].  The reference fields enter
 * the KL only (no gradient flows to them). */
int pbg_policy_learner_backward(int64_t B, int32_t E, pbg_policy raw, const pbg_policy *reference,
                                const uint8_t *mask, const int32_t *action,
                                const float *g_selected, const float *g_entropy,
                                const float *g_kl, pbg_policy_grad grad, void *stream);

/* ------------------------------------------------- poker learner objective */

/* Workspace bytes pbg_poker_learner_objective needs for S sigma rows, A
 * action rows and `lanes` replica lanes (-1 for invalid sizes).  Zero the
 * workspace once before its first use; every launch leaves it ready for the
 * next. */
int64_t pbg_learner_workspace_bytes(int64_t S, int64_t A, int32_t lanes);

/* The poker learner objective of one physical batch and its gradient, one
 * pass: LearnerOperation.forward_loss (pbg/core/learner.py:1824-2159) with the
 * poker policy operation (pbg/games/poker/queued/policy.py:113-298 through
 * hooks.py:2200-2246 PokerLearnerPolicy), then the backward of
 * (total * lane_weight).sum() (pbg/core/training.py:403, lane_weight =
 * objective weight x loss scale).  Replaces the autograd program the
 * reference's learner runs between the model forward and the weight-gradient
 * GEMMs.
 *   raw        current raw fields [S, W, ...] (W = 1 sampled row, W = H
 *              Rao-Blackwell hands); reference: same layout or NULL (no KL)
 *   mask       [S, E] legal events of each sigma row (canonical ids 0..E-1)
 *   action_ptr [S+1] ragged action spans (NULL: unit spans, A == S)
 *   action [A]; old_log, advantage, posterior [A, W] (posterior NULL = 1
 *              for W == 1); value, old_value, value_target [S, W]
 *   trace/cost pred+target [S] (branched public heads) or all NULL
 *   controls [lanes, 10] (learner.py:2162-2175 order); lane_weight [lanes]
 * Writes grad (same layout as raw), d_value [S, W], d_trace / d_cost [S]
 * and result [lanes, 10] in LossResult order (total, policy, value,
 * entropy, reference_kl, approximate_kl, clip_fraction,
 * negative_advantage_cap_fraction, negative_advantage_log_ratio_max,
 * negative_advantage_influence_max).  Action spans must not cross lane
 * boundaries (S/lanes sigma rows and A/lanes action rows per lane). */
int pbg_poker_learner_objective(int64_t S, int64_t A, int32_t E, int32_t W, int32_t lanes,
                                pbg_policy raw, const pbg_policy *reference,
                                const uint8_t *mask, const int64_t *action_ptr,
                                const int32_t *action, const float *old_log,
                                const float *advantage, const float *posterior,
                                const float *value, const float *old_value,
                                const float *value_target, const float *trace_pred,
                                const float *cost_pred, const float *trace_target,
                                const float *cost_target, const float *controls,
                                const float *lane_weight, pbg_policy_grad grad,
                                float *d_value, float *d_trace, float *d_cost, float *result,
                                void *workspace, int64_t workspace_bytes, void *stream);

/* ------------------------------------------------------ fused rollout */

/* One fused sampled rollout step for B independent hands (thread per hand),
 * composing rollout.py:1604-1621 (ACTION key at draw 0), hooks.py:1489-1541
 * (sample at the owner's private row), hooks.py:1656-1700 (history,
 * step_player, three keyed chance generations), hooks.py:1145-1216 (leaf
 * payload of rows that became terminal) and hooks.py:1870 (child path).
 *
 * root_path [B,2] holds (root, path); path is replaced by its child for
 * every row that acted.  Rows whose terminal flag is already set are left
 * untouched and emit action -1.  pol rows: 1 = raw already at the actor's
 * row; otherwise rows >= H and the row is the actor's preflop class
 * (street 0, row < K) or compact combo (later streets).
 *
 * decision [B,4] int32 (may be NULL) receives (actor, street_before,
 * raise_lo_tick, raise_hi_tick | call_legal<<16) for pbg_reach_update.
 * leaf columns are written only for rows that became terminal; new_leaf[B]
 * flags them. */
int pbg_rollout_step(pbg_geometry g, int64_t B, pbg_state st, pbg_history hist,
                     int64_t *root_path, const int64_t *lane, const int64_t *retry_epoch,
                     int64_t seed, int64_t iteration, pbg_policy pol, int32_t *action,
                     float *selected_log, int32_t *decision, uint8_t *new_leaf, pbg_leaf leaf,
                     void *stream);

/* pbg_rollout_step over a work list: a compaction pass writes the terminal
 * hands' outputs (action -1, no leaf) and lists the live hands in
 * worklist[1..] (worklist[0] = their count; B + 1 device int32, no other
 * contract), then the step runs one thread per listed hand, so warps stay
 * full when few hands are left.  Results are identical to pbg_rollout_step. */
int pbg_rollout_step_listed(pbg_geometry g, int64_t B, pbg_state st, pbg_history hist,
                            int64_t *root_path, const int64_t *lane, const int64_t *retry_epoch,
                            int64_t seed, int64_t iteration, pbg_policy pol, int32_t *action,
                            float *selected_log, int32_t *decision, uint8_t *new_leaf, pbg_leaf leaf,
                            int32_t *worklist, void *stream);

/* hooks.py:1641-1656 and 1688-1703: add the selected action's log policy of
 * every private hand to the actor's log-reach row, then mask hands whose
 * cards meet the (post-chance) board with -inf for every seat.
 * log_reach [B,P,H]; pol has rows >= H (class rows used preflop). */
int pbg_reach_update(pbg_geometry g, int64_t B, pbg_state st, pbg_policy pol,
                     const int32_t *action, const int32_t *decision, float *log_reach,
                     void *stream);

/* ---------------------------------------------------------------- loss */

/* Fused categorical PPO loss backward (masked log-softmax, clipped /
 * negative-advantage-capped ratio, entropy bonus, per-row decision-mass
 * weight, dlogits) in one HBM pass: pbg/core/learner.py:2021-2077 with the
 * categorical policy of tests/categorical_policy_fixture.py:33-57.
 *
 * logits [N,A] (dtype 0=fp32, 1=bf16), mask [N,A] uint8, action [N] int32,
 * old_logp/adv/weight [N] fp32.  dlogits [N,A] in the logits dtype.
 * controls (device fp32[5]): clip, log_cap, ent_coef, scale, inv_count.
 * partials: caller scratch of pbg_ppo_partials_size(N) doubles; stats
 * (device double[8]) receives total, sum w*policy, sum w*entropy,
 * sum w*approx_kl, clip count, neg-cap count, sum w, rows. A in [1,32]. */
int64_t pbg_ppo_partials_size(int64_t N, int32_t A);
int pbg_ppo_categorical_backward(int64_t N, int32_t A, int32_t dtype, const void *logits,
                                 const uint8_t *mask, const int32_t *action,
                                 const float *old_logp, const float *adv, const float *weight,
                                 const float *controls, void *dlogits, double *partials,
                                 double *stats, void *stream);

/* pbg_ppo_categorical_backward with the persistent kernel's grid capped at
 * max_ctas thread blocks (0 = one per SM), so that a collective launched on
 * another stream keeps SMs of its own while the loss runs.  The loss kernel
 * fills every register of an SM, so nothing else shares an SM it holds. */
int pbg_ppo_categorical_backward_grid(int64_t N, int32_t A, int32_t dtype, const void *logits,
                                      const uint8_t *mask, const int32_t *action,
                                      const float *old_logp, const float *adv, const float *weight,
                                      const float *controls, void *dlogits, double *partials,
                                      double *stats, int32_t max_ctas, void *stream);

/* The loss backward above fused with the gradient of the readout that
 * produced the logits, x = W h + b (pbg/core/tensor_ops.py:25-38, `linear`,
 * whose weight and bias gradients autograd forms after the loss's dlogits,
 * pbg/core/learner.py:2021-2077).  A == 8, bf16 logits and dlogits as in the
 * vectorised path; hidden [N,d] bf16 (d = 64, 128 or 256, 16-byte aligned).
 * Writes dlogits as pbg_ppo_categorical_backward does (same values) and
 * dweight [8,d] = sum_r dlogits[r,:]^T hidden[r,:], dbias [8] = sum_r
 * dlogits[r,:] in fp32, summed from the bf16 dlogits.  partials: caller
 * scratch of pbg_ppo_readout_partials_size(N, 8, d) doubles, zero before the
 * first call (the kernel leaves it cleared); stats as above. */
int64_t pbg_ppo_readout_partials_size(int64_t N, int32_t A, int32_t d);
int pbg_ppo_readout_backward(int64_t N, int32_t A, const void *logits, const uint8_t *mask,
                             const int32_t *action, const float *old_logp, const float *adv,
                             const float *weight, const float *controls, const void *hidden, int32_t d,
                             void *dlogits, float *dweight, float *dbias, double *partials,
                             double *stats, void *stream);

/* Allocation-free variant of pbg_ppo_categorical_backward (no counterpart
 * in the reference).  For callers that cannot allocate device memory --
 * hosts that own all device memory through their own pool, bindings with no
 * way to pass scratch -- the per-block statistics live in a fixed array
 * inside this library (statistics of at most 2048 thread blocks, about 128
 * KiB, held by every GPU that loads the library until exit).  Returns
 * PBG_ERANGE if a launch would need more blocks than that.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  All calls share the
 * array: calls that overlap on the GPU (concurrent streams, or several host
 * threads on one device) race and must be serialised by the caller.  No
 * allocation happens; arguments and results are as for the entry point
 * above, minus `partials`. */
int pbg_ppo_categorical_backward_noalloc(int64_t N, int32_t A, int32_t dtype, const void *logits,
                                         const uint8_t *mask, const int32_t *action,
                                         const float *old_logp, const float *adv,
                                         const float *weight, const float *controls, void *dlogits,
                                         double *stats, void *stream);

/* ---------------------------------------------------------------- Adam */

/* optimization.py:182-233 (adam_transition) for one lane of a flat fp32
 * master/grad/moment set of n parameters.  controls (device fp32[10]):
 * lr, beta1, beta2, eps, decay, clip, scale, growth, backoff, interval;
 * decoupled selects AdamW.  step (device int64[1]) advances when applied.
 * partials: caller scratch of pbg_adam_partials_size(n) doubles, zero before
 * the first call (the last slot is an arrival counter the step leaves cleared).
 * report (device double[4]): applied, finite, norm, clip scale. */
int64_t pbg_adam_partials_size(int64_t n);
int pbg_adam_step(int64_t n, float *master, float *grad, float *first, float *second,
                  const float *controls, int64_t *step, int32_t decoupled, double *partials,
                  double *report, void *stream);

/* ------------------------------------------- collision-conditioned sampler */

/* Workspace (device floats) for pbg_posterior_sample_children: the parents'
 * per-seat CDFs and masses, parents * players * (private_hands + 1). */
int64_t pbg_posterior_workspace_floats(pbg_geometry geometry, int64_t parents);

/* pbg/games/poker/queued/rb_sampling.py:86-223 (CollisionConditionedProfile
 * Sampler.sample_children): one generating profile per child row.
 * range_weights f32 [parents, P, H], board u8 [parents, 5], inherited i32
 * [parents, P]; per row: source, ordinal, root, path (int64), active (u8);
 * retry_epoch int64 [rows] or NULL (then retry_epoch_scalar).  Outputs:
 * profile i32 [rows, P], attempt_count i32 [rows], exhausted u8 [rows],
 * min_failing int64 [1] (smallest path of an exhausted row, INT64_MAX if
 * none).  *status (device, caller-zeroed) becomes 1 when a fresh row's seat
 * has no board-legal mass (the reference's device assert; here the row keeps
 * its inherited profile and the host raises). */
int pbg_posterior_sample_children(pbg_geometry geometry, int64_t parents, const float *range_weights,
                                  const uint8_t *board, const int32_t *inherited, int64_t rows,
                                  const int64_t *source, const int64_t *ordinal, const uint8_t *active,
                                  const int64_t *root, const int64_t *path, int64_t seed, int64_t iteration,
                                  const int64_t *retry_epoch, int64_t retry_epoch_scalar, int32_t max_attempts,
                                  float *workspace, int32_t *profile, int32_t *attempt_count, uint8_t *exhausted,
                                  int64_t *min_failing, uint32_t *status, void *stream);

/* ------------------------------------------------ branched learner sampling */

/* Workspace bytes (device, 16-byte aligned) for pbg_alias_table over n weights. */
int64_t pbg_alias_workspace_bytes(int64_t n);

/* pbg/core/csrc/alias_table.cu:11-44 (Walker alias table, Vose's two-stack
 * construction in float64; learner.py:1519-1543 builds scaled = n * softmax
 * of the log weights): probability f64 [n] and alias i32 [n]; scaled f64 [n]
 * is consumed as the reference consumes it.  Identical table to the
 * reference's single-thread kernel; replaces its small/large stacks with
 * `workspace`. */
int pbg_alias_table(int64_t n, double *scaled, double *probability, int32_t *alias, void *workspace, void *stream);

/* pbg/core/csrc/branching_metadata.cu:9-31 (decision_log_mass):
 * log_mass f32 [n] with log_mass[v] = log_mass[parent[v]] -
 * logf(degree[parent[v]]) (roots 0), parents at smaller indices.  *failure
 * (caller-zeroed) receives 1 (parent >= node) or 2 (parent degree <= 0) of
 * the first failing node in index order.  workspace: 8 device bytes. */
int pbg_decision_log_mass(int64_t n, const int32_t *parent, const int32_t *degree, float *log_mass,
                          int32_t *failure, void *workspace, void *stream);

/* ------------------------------------------- multiway folded statistics */

/* Removal queries of one decision row for a deck of `cards` cards: 1 + C + C(C-1)/2
 * (pbg/games/poker/queued/folded.py:81-92), or -1 outside [2, 52]. */
int64_t pbg_folded_query_count(int32_t cards);

/* pbg/games/poker/queued/folded.py:111-232 (_phi_queries over every removal
 * query, called in chunks at folded.py:313-327): probability f32 [B,P,H]
 * (each folded seat's normalised, board-masked range; zero for other seats),
 * folder_mask / tight_mask u8 [B,P], base_cards f32 [B] (deck cards minus
 * board cards) -> phi f32 [B,Q] (phi + triple, as _phi_queries returns it)
 * and triple f32 [B,Q].  P <= 6, cards = 4R <= 52, H = C(C-1)/2; fp32 within
 * rounding of the reference's own fp32 evaluation. */
int pbg_folded_phi_queries(int64_t batch, int32_t players, int32_t cards, const float *probability,
                           const uint8_t *folder_mask, const uint8_t *tight_mask, const float *base_cards,
                           float *phi, float *triple, void *stream);

/* Batched symmetric eigendecomposition, n <= 64 (the beta matrices of the
 * folded statistics, pbg/games/poker/queued/folded.py:352, there
 * torch.linalg.eigh): cyclic Jacobi with round-robin parallel ordering, one CTA
 * per matrix, fp32.  matrices f32 [batch, n, n] (the symmetric part is used),
 * values f32 [batch, n] and vectors f32 [batch, n, n] (eigenvector j in column
 * j), unsorted; at most max_sweeps sweeps. */
int pbg_symmetric_eigh(int64_t batch, int32_t n, const float *matrices, float *values, float *vectors,
                       int32_t max_sweeps, void *stream);

/* ------------------------------------------------------- layered targets */

/* Device tables of per-partition arena pointers (int64 device addresses, 0 =
 * absent), the layout pbg/core/csrc/layered_targets.cu:14-32 binds:
 * work0/work1/trace/cost/delta [output_count], head_v/head_t/head_c
 * [input_count], sigma_v/sigma_t/sigma_c [n_replica*input_count],
 * action_p/action_a [n_replica*action_partition_count]; work_cap/width
 * [output_count], head_cap [input_count] int32; conversion
 * [output_count, output_count, max_width] int32 (source component ->
 * destination component, -1 = none). */
typedef struct {
    const int64_t *work0, *work1, *trace, *cost, *delta;
    const int64_t *head_v, *head_t, *head_c;
    const int64_t *sigma_v, *sigma_t, *sigma_c;
    const int64_t *action_p, *action_a;
    const int32_t *work_cap, *head_cap, *width, *conversion;
} pbg_target_tables;

/* Topology nodes in reverse-layer order, int32 [node_count] columns
 * (targets.py:640 run_layers node tensors). */
typedef struct {
    const int32_t *replica, *child_begin, *child_count, *destination_row, *input_type, *output_type;
    const int32_t *owner_slot, *nominal_degree, *target_degree, *sigma_head_row, *sigma_target_row;
    const int32_t *action_begin;
} pbg_target_nodes;

/* Child edges: encoded source row (r >= 0 arena 0 row r; r < 0 arena 1 row
 * -r-1), source output partition, unit path cost, cost multiplier. */
typedef struct {
    const int32_t *source_row, *source_type, *path;
    const float *multiplier;
} pbg_target_children;

/* pbg/core/csrc/layered_targets.cu:117-411 (layered_target_kernel +
 * run_layers): lambda-returns, sigma targets and per-action advantages of
 * every topology node, layer by layer, in ONE cooperative launch.
 * layer_ptr [layers+1] (device) bounds each layer's nodes; layer l writes
 * work arena (l+1)&1.  failure_min [n_replica] (device, output) receives
 * INT_MAX or the first failing node of each lane, or -2 in every lane when a
 * grid-barrier wait ran out (bounded wait).  At most 16 output partitions.
 * workspace [pbg_layered_targets_workspace_words(n_replica)] (device
 * uint32): zero before the first call; each completed call leaves it ready
 * for the next one, a call that reported -2 does not (zero it again).
 * Calls sharing a workspace must be ordered on one stream.  The workspace has
 * no reference counterpart: the reference launches one kernel per layer from
 * a host loop instead. */
int64_t pbg_layered_targets_workspace_words(int32_t n_replica);
int pbg_layered_targets(const int32_t *layer_ptr, int32_t layers, pbg_target_nodes nodes,
                        pbg_target_children children, pbg_target_tables tables, int32_t n_replica,
                        int32_t input_count, int32_t output_count, int32_t action_partition_count,
                        int32_t p_train, int32_t max_width, float lambda, int32_t sampled,
                        int32_t branched, int32_t *failure_min, uint32_t *workspace, void *stream);

/* ------------------------------------------------------------ model GEMM */

/* pbg/games/poker/model/primitives.py:35-60 (FFN), :97-117 (MHA
 * projections) and pbg/core/tensor_ops.py Linear: y[M,N] = act(x[M,K] .
 * w[N,K]^T + bias[N]) with bf16 x, w, y (row-major, 16-byte aligned) and
 * fp32 bias (may be NULL), fp32 accumulation on the tensor cores (tcgen05,
 * TMA, tensor memory).  activation: 0 none, 1 GELU (erf form).  K must be a
 * multiple of 64 and N of 128.  error (device uint32) receives a nonzero code
 * if a bounded pipeline wait ran out (the output is then incomplete). */
int pbg_linear_bf16(int64_t M, int32_t N, int32_t K, const void *x, const void *w, const float *bias, void *y,
                    int32_t activation, uint32_t *error, void *stream);

/* The same map with the model's following elementwise steps fused into the
 * epilogue: y = act(acc * row_scale[m] + bias[n] + residual[m, n]), where acc
 * = x . w^T in fp32 and each term may be absent (NULL): the per-row mass scale
 * of the incidence source map (pbg/games/poker/model/incidence.py:57-58), the
 * fp32 residual adds after the attention output and FFN maps (preflop.py:
 * 634-641, postflop.py:678-685), and the pre-GELU residual of the incidence
 * query map (incidence.py:77-84), and the context projection of a factored
 * FFN (primitives.py:62-71), one residual row shared by residual_row_div
 * consecutive rows (row m reads residual row m / residual_row_div).  x rows
 * are ldx elements apart (ldx >= K, a multiple of 8), residual rows ldr
 * floats apart (>= N, a multiple of 4, 16-byte aligned), y rows ldy elements
 * apart; y is fp32 when y_f32 is 1, else bf16 (rows 16-byte aligned).  Other
 * rules as for pbg_linear_bf16. */
int pbg_linear_ex(int64_t M, int32_t N, int32_t K, const void *x, int64_t ldx, const void *w, const float *bias,
                  const float *row_scale, const float *residual, int64_t ldr, int64_t residual_row_div, void *y,
                  int64_t ldy, int32_t y_f32, int32_t activation, uint32_t *error, void *stream);
/* The gradient through a GELU map of pbg_linear_ex, recomputing its pre-activation on the tensor
 * cores: out = dy * GELU'(x . w^T * row_scale + bias + residual), bf16 [M, N] (row stride ldo), with dy
 * bf16 [M, N] (row stride ldd, a multiple of 8; 16-byte aligned).  The other arguments and rules are
 * pbg_linear_ex's. */
int pbg_linear_gelu_backward(int64_t M, int32_t N, int32_t K, const void *x, int64_t ldx, const void *w,
                             const float *bias, const float *row_scale, const float *residual, int64_t ldr,
                             int64_t residual_row_div, const void *dy, int64_t ldd, void *out, int64_t ldo,
                             uint32_t *error, void *stream);

/* pbg/games/poker/model/primitives.py:63-283 (MHA, self-attention, heads of
 * width 32): out[b, q, h] = softmax_k((q_h / temperature_h) . k_h / sqrt(32)
 * + key_bias[b, k], keys with key_mask 0 excluded) . v_h.  qkv bf16
 * [batch, len, 3 * heads * 32] (the fused in-projection: q | k | v, heads
 * contiguous inside each), key_bias f32 [batch, len] or NULL, key_mask u8
 * [batch, len] or NULL (all present), q_scale f32 [heads] = 1 /
 * (temperature_h * sqrt(32)), out bf16 [batch, len, heads * 32] (merged
 * heads).  Rows whose keys are all masked give 0.  error (device) as for
 * pbg_linear_bf16. */
int pbg_attention_bf16(int32_t batch, int32_t len, int32_t heads, const void *qkv, const float *key_bias,
                       const uint8_t *key_mask, const float *q_scale, void *out, uint32_t *error, void *stream);
/* pbg_attention_bf16 that also writes each row's base-2 log-sum-exp of its
 * logits, lse f32 [batch, heads, len] (+inf for a row without keys): the
 * input of pbg_attention_backward. */
int pbg_attention_bf16_lse(int32_t batch, int32_t len, int32_t heads, const void *qkv, const float *key_bias,
                           const uint8_t *key_mask, const float *q_scale, void *out, float *lse, uint32_t *error,
                           void *stream);

/* pbg/core/tensor_ops.py:70-81 (LayerNorm over the last dimension, d <= 1024):
 * y = (x - mean) / sqrt(var + eps) * gain + bias, fp32 statistics; x and y
 * are bf16 when x_bf16 / y_bf16 is nonzero, else fp32; gain and bias may be
 * NULL; row i of y starts at y + i * ldy elements (ldy >= d). */
int pbg_layernorm(int64_t rows, int32_t d, const void *x, int32_t x_bf16, const float *gain, const float *bias,
                  float eps, void *y, int32_t y_bf16, int64_t ldy, void *stream);

/* The same over a row block of every sequence of a batch: launch row i is
 * row r = i % group_rows of group g = i / group_rows, read at x + g *
 * x_group_stride + r * ldx and written at y + g * y_group_stride + r * ldy
 * (elements). */
int pbg_layernorm_rows(int64_t rows, int32_t d, int64_t group_rows, const void *x, int32_t x_bf16,
                       int64_t x_group_stride, int64_t ldx, const float *gain, const float *bias, float eps, void *y,
                       int32_t y_bf16, int64_t y_group_stride, int64_t ldy, void *stream);

/* pbg/games/poker/model/incidence.py:57-70 after the two card contractions:
 * source and overlap f32 [B, P, R, d] (contiguous), identical_scale f32
 * [B, R]; per (b, r, feature) over the seats p (sums in seat order):
 * same = source * scale, oe = sum(same) - same, oc = (sum(overlap) - overlap)
 * - 2 oe, own = overlap - 2 same.  Writes oe and own as bf16 into columns
 * col_equal / col_own of `inc` (row (b*P + p)*R + r, ld_inc elements apart),
 * oc as f32 into other_card [B, P, R, d], and, when ffn is not NULL, oc*oc and
 * oc*oe as bf16 into columns col_square / col_product of the FamilyFFN
 * operand row p*R + r of sequence b (ffn + b * ffn_batch_stride + row *
 * ld_ffn).  d, strides and column offsets are multiples of 4; P <= 9. */
/* Copy of a contiguous bf16 matrix [rows, d] into the row block of every
 * sequence of a wider buffer: row i goes to dst + (i / group_rows) *
 * group_stride + (i % group_rows) * ld (elements; d, ld, group_stride
 * multiples of 8, 16-byte aligned buffers).  Places the incidence residual j
 * into the FamilyFFN operand rows of the private tokens. */
int pbg_scatter_rows_bf16(int64_t rows, int32_t d, int64_t group_rows, const void *src, void *dst,
                          int64_t group_stride, int64_t ld, void *stream);

int pbg_incidence_combine(int64_t batch, int32_t players, int64_t rows, int32_t d, const float *source,
                          const float *overlap, const float *identical_scale, void *inc, int64_t ld_inc,
                          int32_t col_equal, int32_t col_own, float *other_card, void *ffn, int64_t ffn_batch_stride,
                          int64_t ld_ffn, int32_t col_square, int32_t col_product, void *stream);
/* Backward of pbg_incidence_combine for outputs laid out per row
 * (b * P + p) * R + r: g_pair bf16 [rows, 2d] (the gradients of oe | own),
 * g_other_card f32 [rows, d], g_ffn bf16 [rows, 2d] (of oc*oc | oc*oe); any
 * may be NULL (zero).  Writes d_source and d_overlap f32 [B, P, R, d]. */
int pbg_incidence_combine_backward(int64_t batch, int32_t players, int64_t rows, int32_t d, const float *source,
                                   const float *overlap, const float *identical_scale, const void *g_pair,
                                   const float *g_other_card, const void *g_ffn, float *d_source, float *d_overlap,
                                   void *stream);

/* ---------------------------------------------------------- collective */

/* replica.py:352-362 (all_reduce SUM of the flat fp32 gradient) over NVLink
 * SHARP: `multicast` is the multicast address of a symmetric-memory buffer
 * of n floats (n a multiple of 4*world), `signal_pads` a device array of the
 * world ranks' signal-pad pointers (pads of pad_bytes bytes, zero before
 * first use; the launch uses at most pad_bytes / pbg_nvls_signal_bytes() CTAs).  Each rank sums its 1/world slice in the
 * switch (multimem.ld_reduce) and stores it to every rank (multimem.st),
 * between two bounded cross-rank barriers; *error (device) becomes nonzero if
 * a barrier wait runs out.  Every rank must make the same call. */
int64_t pbg_nvls_signal_bytes(void); /* pad bytes one CTA uses per group of up to 8 ranks */
int pbg_nvls_allreduce_sum_f32(int64_t n, void *multicast, const void *signal_pads,
                               int64_t pad_bytes, int32_t rank, int32_t world, uint32_t *error,
                               void *stream);

/* pbg_nvls_allreduce_sum_f32 on at most max_ctas thread blocks (0 = as many
 * as the slice and the pad allow), for a SUM that overlaps compute on the
 * remaining SMs.  A bucket of a larger buffer is summed by passing the
 * multicast address of its first element and its length. */
int pbg_nvls_allreduce_sum_f32_grid(int64_t n, void *multicast, const void *signal_pads,
                                    int64_t pad_bytes, int32_t rank, int32_t world,
                                    uint32_t *error, int32_t max_ctas, void *stream);

/* ------------------------------------------------ cfg1 preflop-class MLP */

/* The element-wise parts of the fp32 preflop-class MLP (two hidden layers,
 * ReLU) that the reference's ModelOperation protocol admits
 * (learner.py:324-350); its heads apply the reference head activations
 * (model/heads.py:28-62).  Output row layout of the last dense map: per class
 * row [type 3 | omega logits M | mu logits M | s pre M | iota logit], then
 * the K values.  y [M,N] row-major. */
int pbg_mlp_bias_relu(int64_t M, int32_t N, float *y, const float *bias, void *stream);

/* Heads of the sampled class row cls[s] (z [S, ldz] before its bias):
 * type_logits [S,3], omega/mu/scale [S,M], iota [S], value [S].  *status
 * (device, caller-zeroed) gets bit 1 for a class id outside [0,K). */
int pbg_mlp_heads(int64_t S, int32_t K, int32_t M, float s_min, const float *z, int64_t ldz,
                  const float *bias, const int32_t *cls, float *type_logits, float *omega, float *mu,
                  float *scale, float *iota, float *value, uint32_t *status, void *stream);

/* Vector-Jacobian product of pbg_mlp_heads into dz [S, lddz] (zero outside
 * the sampled row's columns). */
int pbg_mlp_heads_backward(int64_t S, int32_t K, int32_t M, const float *z, int64_t ldz,
                           const float *bias, const int32_t *cls, const float *omega, const float *mu,
                           const float *iota, const float *d_type, const float *d_omega,
                           const float *d_mu, const float *d_scale, const float *d_iota,
                           const float *d_value, float *dz, int64_t lddz, void *stream);

/* Floats of scratch pbg_mlp_relu_backward_bias needs for M rows of N columns. */
int64_t pbg_mlp_bias_partials(int64_t M, int32_t N);

/* dy *= (y > 0) (y may be NULL: no mask) and dbias[n] = sum_m dy[m,n], summed
 * in blocks of 32 rows, the blocks' sums strided over 32 lanes and added by a
 * fixed butterfly (deterministic). */
int pbg_mlp_relu_backward_bias(int64_t M, int32_t N, float *dy, const float *y, float *dbias,
                               float *partial, int64_t partial_len, void *stream);

/* ---- policy/value network backward (pbg/core/training.py:381-403 autograd
 * through pbg/games/poker/model/primitives.py FFN / MHA and tensor_ops.py
 * LayerNorm): the element-wise and row-wise steps between the library GEMMs.
 */

/* out[m, c] = dy[m, c] * GELU'(pre[m, c]) (exact erf GELU), bf16 out; pre f32,
 * dy bf16 (dy_bf16 = 1) or f32; row strides in elements. */
int pbg_gelu_backward(int64_t M, int32_t N, const float *pre, int64_t ldp, const void *dy, int32_t dy_bf16,
                      int64_t ldd, void *out, int64_t ldo, void *stream);

/* Floats of scratch pbg_layernorm_backward needs for `rows` rows of width d
 * (-1 for a width it does not take: d a multiple of 32 up to 512). */
int64_t pbg_layernorm_backward_partials(int64_t rows, int32_t d);

/* Backward of y = (x - mean) / sqrt(var + eps) * gain + bias over rows of
 * width d: dx (f32 or bf16) from x (f32 or bf16), gain (NULL = 1) and dy, and
 * partial [blocks, 2d]: each block's column sums of dy * xhat (first d) and dy
 * (next d), rows in a fixed order; the gain / bias gradients are the sums of
 * the partial rows. */
int pbg_layernorm_backward(int64_t rows, int32_t d, const void *x, int32_t x_bf16, int64_t ldx, const float *gain,
                           float eps, const void *dy, int32_t dy_bf16, int64_t ldy, void *dx, int32_t dx_bf16,
                           int64_t lddx, float *partial, int64_t partial_len, void *stream);

/* Backward of pbg_attention_bf16 (fused: the scores are recomputed tile by
 * tile and never stored): from qkv, the forward's output `out` and its base-2
 * log-sum-exp `lse` [batch, heads, len] (pbg_attention_bf16_lse), the output
 * gradient dout bf16 [batch, len, heads * 32], the same key_bias / key_mask /
 * q_scale, writes dqkv bf16 [batch, len, 3 * heads * 32] (dQ | dK | dV) and
 * scale_partial f32 [batch, heads, len]: per query row the sum over keys of
 * dZ * (q.k), dZ the gradient of the row's logits (the head's q_scale
 * gradient is the sum over the head's rows).  delta f32 [batch, heads, len]
 * is scratch.  qkv, out, dout and dqkv 16-byte aligned. */
int pbg_attention_backward(int32_t batch, int32_t len, int32_t heads, const void *qkv, const void *out,
                           const void *dout, const float *lse, const float *key_bias, const uint8_t *key_mask,
                           const float *q_scale, void *dqkv, float *delta, float *scale_partial, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PBGB200_H */
