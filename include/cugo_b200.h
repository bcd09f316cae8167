/* cugo_b200 — C ABI of the B200 batch environment for Hangame Shin Matgo.
 *
 * Each entry point replaces one op of the reference's pybind extension
 * (python/csrc/torch50_ext.cpp:36-59, host wrappers python/csrc/torch50_ext.cu:478-686)
 * with the same arguments, output shapes and semantics, but as plain device
 * pointers and sizes:
 *
 *   states    uint8 [n_states, 248]  game rows, byte-compatible with the
 *                                    reference's TorchEnv50 (8-byte aligned)
 *   env_ids   int64 [m]              rows to read; an id outside [0, n_states)
 *                                    gives the documented "invalid id" outputs
 *   actions   int64 [m]              unified actions 0..178; other values are
 *                                    "not legal" (status 3), state unchanged
 *   features  float [m, 720]         16-byte aligned
 *   legal     bool  [m, 179]         4-byte aligned
 *
 * All pointers are device pointers of the current device.  Every call only
 * enqueues work on `stream` (no host synchronisation, no allocation), so calls
 * can be captured in CUDA graphs.  Return value: CUGO_B200_OK or a negative
 * CUGO_B200_ERR_* for a bad argument, a misaligned pointer or a launch
 * failure; per-row game errors are reported in the status outputs, never as
 * device faults.  Indexed ops that step (step_indexed, step_events_indexed)
 * must not list the same env id twice in one call.
 */
#ifndef CUGO_B200_H
#define CUGO_B200_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* cudaStream_t;

#if defined(__GNUC__)
#define CUGO_B200_API __attribute__((visibility("default")))
#else
#define CUGO_B200_API
#endif

#define CUGO_B200_ABI_VERSION 1
#define CUGO_B200_OK 0
#define CUGO_B200_ERR_ARG (-1)
#define CUGO_B200_ERR_ALIGN (-2)
#define CUGO_B200_ERR_LAUNCH (-3)
#define CUGO_B200_ERR_CAPACITY (-4) /* larger than a fixed internal buffer allows */

/* Version of this C ABI (1).  No counterpart in the reference. */
CUGO_B200_API int cugo_b200_abi_version(void);

/* Contract constants (python/csrc/torch50_ext.cpp:61-71). */
CUGO_B200_API int64_t cugo_b200_state_bytes(void);          /* STATE_BYTES = 248 */
CUGO_B200_API int64_t cugo_b200_feature_count(void);        /* FEATURE_COUNT = 720 */
CUGO_B200_API int64_t cugo_b200_action_count(void);         /* ACTION_COUNT = 179 */
CUGO_B200_API int64_t cugo_b200_primary_action_count(void); /* PRIMARY_ACTION_COUNT = 127 */
CUGO_B200_API int64_t cugo_b200_choice_action_begin(void);  /* CHOICE_ACTION_BEGIN = 127 */
CUGO_B200_API int64_t cugo_b200_event_words(void);          /* EVENT_WORDS = 9 */
CUGO_B200_API int64_t cugo_b200_start_words(void);          /* START_WORDS = 8 */
CUGO_B200_API int64_t cugo_b200_status_ok(void);            /* STATUS_OK = 0 */

/* create (torch50_ext.cu:478-499): fresh games from (seed, first_player & 1). */
CUGO_B200_API int cugo_b200_create(const int64_t* seeds, const int64_t* first_players, int64_t n,
                     uint8_t* states, cudaStream_t stream);

/* create from game indices (the drivers build the seed and first-player arrays from
 * an index with torch ops first, python/cugo_ppo_nets50.py:15-17): game i gets seed
 * seed_base + index[i] and first player index[i] & 1, the rows cugo_b200_create makes
 * from those two arrays.  No reference counterpart. */
CUGO_B200_API int cugo_b200_create_indexed(const int64_t* index, int64_t seed_base, int64_t n,
                                           uint8_t* states, cudaStream_t stream);

/* observe (torch50_ext.cu:501-518): features, legal mask, deciding player,
 * done flag and packet status of every row; read only. */
CUGO_B200_API int cugo_b200_observe(const uint8_t* states, int64_t n, float* features, bool* legal,
                      uint8_t* players, bool* done, int16_t* status, cudaStream_t stream);

/* observe_indexed (torch50_ext.cu:520-544): the same for rows env_ids; an invalid
 * id gives zero features, no legal action, player 0, done 1, status -1. */
CUGO_B200_API int cugo_b200_observe_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                              int64_t m, float* features, bool* legal, uint8_t* players,
                              bool* done, int16_t* status, cudaStream_t stream);

/* step (torch50_ext.cu:546-569): applies actions[i] to row i in place; outputs
 * player 0's reward (final once done), done, nagari, status and whether a
 * primary action was committed. */
CUGO_B200_API int cugo_b200_step(uint8_t* states, int64_t n, const int64_t* actions, float* reward, bool* done,
                   bool* nagari, int16_t* status, bool* committed, cudaStream_t stream);

/* step_indexed (torch50_ext.cu:571-600): rows env_ids in place; an invalid id
 * gives reward 0, done 1, nagari 0, status -1, committed 0. */
CUGO_B200_API int cugo_b200_step_indexed(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                           const int64_t* actions, int64_t m, float* reward, bool* done,
                           bool* nagari, int16_t* status, bool* committed, cudaStream_t stream);

/* step_indexed with the bookkeeping of a self-play round in the same kernel (no
 * reference counterpart; it replaces the per-round tensor updates of the collection
 * loop, python/cugo_ppo50.py:321-450): for row i of game id = env_ids[i] (distinct
 * ids), decision[id] += 1; a game that finishes gets reward0[id] (player 0's reward)
 * and nagari[id]; each status other than OK (0) and "finished" (9) adds 1 to *bad;
 * next_ids gets the ids of the games still running, in their env_ids order, and
 * *next_count their number.  scratch: int32 [2 * ceil(m / 32)] of the caller's
 * (per-warp masks and offsets); three launches, no allocation.  m_dev (optional, not
 * next_count): a device-resident int32 row count; only rows below min(m, *m_dev)
 * are stepped. */
CUGO_B200_API int cugo_b200_step_compact(uint8_t* states, int64_t n_states,
                                         const int64_t* env_ids, const int64_t* actions,
                                         int64_t m, int32_t* decision, float* reward0,
                                         bool* nagari, int64_t* bad, int64_t* next_ids,
                                         int32_t* next_count, int32_t* scratch,
                                         const int32_t* m_dev, cudaStream_t stream);

/* cugo_b200_step_compact with next_ids grouped by each running game's next
 * decision: the games about to make a primary play first, then those with a
 * pending floor choice, then those answering a prompt (Go/Stop, Gukjin,
 * Chongtong), each group in env_ids order.  A round that steps the groups in this
 * order runs one branch of the rule code per warp almost everywhere.  scratch:
 * int32 [6 * ceil(m / 32)].  No reference counterpart (as cugo_b200_step_compact). */
CUGO_B200_API int cugo_b200_step_compact_grouped(uint8_t* states, int64_t n_states,
                                                 const int64_t* env_ids, const int64_t* actions,
                                                 int64_t m, int32_t* decision, float* reward0,
                                                 bool* nagari, int64_t* bad, int64_t* next_ids,
                                                 int32_t* next_count, int32_t* scratch,
                                                 const int32_t* m_dev, cudaStream_t stream);

/* The running set of a freshly created batch for the self-play round loop (the
 * reference's drivers keep a live index list and compact it with torch ops,
 * python/cugo_ppo50.py:359,375): ids[0 .. *count) = the rows whose game the deal did
 * not end, in row order, ids[i] = i past them, and spare_ids[i] = i (optional: the
 * other list of a double-buffered loop), so every entry is a valid row; decision,
 * reward0 and nagari zeroed for all n rows; *bad = 0.  scratch: int32
 * [cugo_b200_running_init_scratch(n)] (= 2 * ceil(n / 32)); a shorter one returns
 * CUGO_B200_ERR_CAPACITY.  No reference counterpart. */
CUGO_B200_API int64_t cugo_b200_running_init_scratch(int64_t n);
CUGO_B200_API int cugo_b200_running_init(const uint8_t* states, int64_t n, int64_t* ids,
                                         int64_t* spare_ids, int32_t* count, int32_t* decision,
                                         float* reward0, bool* nagari, int64_t* bad,
                                         int32_t* scratch, int64_t scratch_len,
                                         cudaStream_t stream);

/* step_events_indexed (torch50_ext.cu:626-660): step_indexed plus the committed
 * action's event record, int64 [m, 9] (zero when nothing was committed). */
CUGO_B200_API int cugo_b200_step_events_indexed(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                  const int64_t* actions, int64_t m, float* reward, bool* done,
                                  bool* nagari, int16_t* status, bool* committed, int64_t* events,
                                  cudaStream_t stream);

/* branch_indexed (torch50_ext.cu:703-734): children[i] = row env_ids[i] stepped
 * with actions[i]; parents are not written; an invalid id gives a zero child
 * and the invalid-id step outputs. */
CUGO_B200_API int cugo_b200_branch_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                             const int64_t* actions, int64_t m, uint8_t* children, float* reward,
                             bool* done, bool* nagari, int16_t* status, bool* committed,
                             cudaStream_t stream);

/* clone_indexed (torch50_ext.cu:679-701): children[i] = row env_ids[i], zero row
 * for an invalid id. */
CUGO_B200_API int cugo_b200_clone_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, uint8_t* children, cudaStream_t stream);

/* hands_indexed (torch50_ext.cu:736-758): int64 [m, 2] hand masks, 0 when invalid. */
CUGO_B200_API int cugo_b200_hands_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, int64_t* hands, cudaStream_t stream);

/* stock_indexed (torch50_ext.cu:602-624): int64 [m], the next 8 stock draws one
 * card id per byte (0xFF past the end); -1 when invalid. */
CUGO_B200_API int cugo_b200_stock_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, int64_t* stock, cudaStream_t stream);

/* start (torch50_ext.cu:662-677): int64 [n, 8] opening records. */
CUGO_B200_API int cugo_b200_start(const uint8_t* states, int64_t n, int64_t* out, cudaStream_t stream);

/* ---- Benchmark drivers ------------------------------------------------------
 * These have no counterpart in the reference's extension: they run the seeded
 * random-legal rule of the benchmark configurations on the GPU.  Game i uses
 * seed seed_base + i and first player i & 1; decision d of game i takes the
 * floor(r0 * n / 2^32)-th of its n legal actions, with r0 the first word of
 * Philox4x32-10(counter {i lo, i hi, d, stream}, key {seed lo, seed hi}).
 */

/* Plays games game0 .. game0+n-1 to the end (at most max_decisions steps each; the
 * loop of python/torch50_smoke.py:13-59 run_games with random-legal actions, in one
 * launch):
 * final rows [n, 248], player 0's reward, decisions taken, events committed,
 * FNV-1a 64 hash of the start record and every event record, last step status
 * (-2 when a game had no legal action). */
CUGO_B200_API int cugo_b200_rollout_random(int64_t game0, int64_t n, int64_t seed_base,
                                           int32_t max_decisions, uint32_t stream_id,
                                           uint8_t* final_rows, int64_t* reward0,
                                           int32_t* decisions, int32_t* events, uint64_t* hashes,
                                           int16_t* last_status, cudaStream_t stream);

/* One decision of every slot (config 1: the run_games loop, python/torch50_smoke.py:
 * 13-59, as one launch per decision): a finished game is replaced by game index +
 * n_slots (counted in slot_completed), then the slot's observation is written to
 * features/legal exactly as observe() writes it, a random legal action is drawn
 * and stepped (counted in slot_steps).  actions: int64 [n_slots] scratch that
 * receives the drawn actions (-1 where a game ended at its deal). */
CUGO_B200_API int cugo_b200_selfplay_random_step(uint8_t* states, int64_t n_slots,
                                                 int64_t seed_base, int64_t* slot_game,
                                                 int32_t* slot_decision, int32_t* slot_completed,
                                                 int64_t* slot_steps, float* features, bool* legal,
                                                 int64_t* actions, cudaStream_t stream);

/* Branching roots for the branch benchmark (python/branch50_smoke.py:66-195, whose
 * parents are fresh games advanced by one step): game r advanced by k_r random-legal
 * decisions, k_r uniform in 0..20 (stream 2, decision 0xFFFF), stopping before a
 * decision that would end the game. */
CUGO_B200_API int cugo_b200_branch_roots(int64_t n_roots, int64_t seed_base, uint8_t* roots,
                                         cudaStream_t stream);

/* Branch i = r * per_root + b: env_ids[i] = r and a random legal action of root
 * r drawn from stream 1 with counter {r, b} (-1 when the root has none). */
CUGO_B200_API int cugo_b200_branch_actions(const uint8_t* roots, int64_t n_roots,
                                           int64_t per_root, int64_t seed_base, int64_t* env_ids,
                                           int64_t* actions, cudaStream_t stream);

/* ---- Policy sampling ----------------------------------------------------------
 * Replaces the sampling of the reference's collect loop (python/cugo_ppo50.py:74-82:
 * masked_fill(-1e30), softmax + multinomial, log_softmax gather) and the
 * Gumbel-max of its sequence self-play (python/cugo_seq_selfplay50.py:126-130).
 * logits: fp32 [m, ld] (ld >= 179, policy logits in columns 0..178); legal:
 * bool [m, 179]; game/decision: the row's game index and decision counter.
 * actions[i] = argmax over legal a of logits[i, a] + g(i, a) (g = 0 when
 * greedy), logp[i] = log_softmax(masked logits)[actions[i]]; -1 and 0 for a row
 * with no legal action.  Noise g(i, a) = -log(-log(u)), u from word (a & 3) of
 * Philox4x32-10({game lo, game hi, decision, 3 | (a >> 2) << 8}, {seed lo, seed hi})
 * with seed = seed_base + game. */
CUGO_B200_API int cugo_b200_sample_actions(const float* logits, int64_t ld, const bool* legal,
                                           int64_t m, const int64_t* game,
                                           const int32_t* decision, int64_t seed_base,
                                           int32_t greedy, int64_t* actions, float* logp,
                                           cudaStream_t stream);

/* ---- Policy network layers -------------------------------------------------------
 * One nn.Linear layer of the residual-MLP policy/value networks
 * (python/cugo_ppo_nets50.py:26-87; run under bf16 autocast, cugo_ppo50.py:366)
 * with its bias, activation and residual add fused, on tcgen05 tensor cores:
 *   out = act_after(act(A . W^T + bias) + residual)
 * A bf16 [m, k] (row stride lda), W bf16 [n, k] (ldw), bias bf16 [n] or NULL,
 * residual bf16 [m, n] (ldr) or NULL (may alias out; bf16 out only), out bf16
 * or fp32 [m, n] (ldo).  act/act_after: 0 none, 1 ReLU, 2 SiLU.  Pointers
 * 16-byte aligned, row strides multiples of 16 bytes.  `error` (device int, may
 * be NULL) is set to 1 if a pipeline wait timed out. */
CUGO_B200_API int cugo_b200_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw,
                                      const void* bias, const void* residual, int64_t ldr,
                                      void* out, int64_t ldo, int32_t out_fp32, int32_t act,
                                      int32_t act_after, int64_t m, int64_t n, int64_t k,
                                      int32_t* error, cudaStream_t stream);

/* The same layer for the sequence transformer's blocks (python/cugo_seq50.py:
 * 318-321, nn.Linear under autocast with an fp32 residual stream x):
 * bias is fp32 when bias_fp32 != 0; the residual has the output's type, so with
 * out_fp32 an fp32 residual stream is updated in place (residual == out);
 * act/act_after may also be 3 = GELU (erf form, nn.GELU()). */
CUGO_B200_API int cugo_b200_gemm_bf16_ex(const void* a, int64_t lda, const void* w, int64_t ldw,
                                         const void* bias, int32_t bias_fp32,
                                         const void* residual, int64_t ldr, void* out,
                                         int64_t ldo, int32_t out_fp32, int32_t act,
                                         int32_t act_after, int64_t m, int64_t n, int64_t k,
                                         int32_t* error, cudaStream_t stream);

/* out = act(a w^T + bias) (bf16) and pre = a w^T + bias (bf16, row stride ldp):
 * a layer of a training forward that keeps its pre-activation for act' in the
 * backward, in one launch (no residual, bf16 output only).  Arguments otherwise as
 * for cugo_b200_gemm_bf16_ex.  Replaces an nn.Linear followed by the activation
 * under bf16 autocast (python/cugo_ppo_nets50.py:26-64, ResidualMlp's fc1 and
 * activation, as autograd saves both). */
CUGO_B200_API int cugo_b200_gemm_bf16_pre(const void* a, int64_t lda, const void* w, int64_t ldw,
                                          const void* bias, int32_t bias_fp32, void* out,
                                          int64_t ldo, void* pre, int64_t ldp, int32_t act,
                                          int64_t m, int64_t n, int64_t k, int32_t* error,
                                          cudaStream_t stream);

/* cugo_b200_gemm_bf16_ex over a row window read from device memory when the
 * kernel starts: window = int32 {first row, rows} (clamped to [0, m]); only those
 * rows of a and out (and residual) are touched, the others keep their values
 * except that the last 128-row tile of the window may also write the up to 127
 * rows that follow it.  For CUDA graphs whose row counts change between replays
 * (m, the maps' extent, stays fixed).  No counterpart in the reference. */
CUGO_B200_API int cugo_b200_gemm_bf16_window(const void* a, int64_t lda, const void* w,
                                             int64_t ldw, const void* bias, int32_t bias_fp32,
                                             const void* residual, int64_t ldr, void* out,
                                             int64_t ldo, int32_t out_fp32, int32_t act,
                                             int32_t act_after, int64_t m, int64_t n, int64_t k,
                                             const int32_t* window, int32_t* error,
                                             cudaStream_t stream);

/* One-output layer (the scalar value head of OracleCritic, python/cugo_ppo_nets50.py:
 * 67-87: nn.Linear(hidden, 1) under autocast): out[r * ldo] = a[r, :k] . w + *bias,
 * a bf16 [m, k] (lda, 16-byte aligned rows), w fp32 [k] (the bf16-rounded weight
 * row), bias fp32 scalar or NULL; k a multiple of 8, at most 2,048.  A row
 * reduction at HBM speed instead of a 256-column GEMM tile. */
CUGO_B200_API int cugo_b200_rowdot_bf16(const void* a, int64_t lda, const float* w,
                                        const float* bias, int64_t m, int64_t k, float* out,
                                        int64_t ldo, cudaStream_t stream);

/* The whole residual MLP of hidden width 512 in one kernel (python/cugo_ppo_nets50.py:
 * 26-64, norm "none"): h = W[0] x + b[0]; per block h = h + W[2i+2] act(W[2i+1] h +
 * b[2i+1]) + b[2i+2]; out = W[last] act(h) + b[last].  The activations of each
 * 128-row tile stay in shared and tensor memory across all layers.  x bf16 [m, k_in]
 * (ldx; k_in a multiple of 8, at most 1,024); weights: HOST array of 2 + 2 * blocks
 * DEVICE pointers to contiguous bf16 [out, in] weights (hidden 512, blocks <= 4,
 * n_out <= 256); biases: HOST array of fp32 device pointers (or NULL / NULL
 * entries); act 0 none, 1 ReLU, 2 SiLU; out fp32 [m, n_out] (ldo a multiple of 4);
 * error as for cugo_b200_gemm_bf16.  All pointers 16-byte aligned. */
CUGO_B200_API int cugo_b200_mlp_fused(const void* x, int64_t ldx, int64_t m, int64_t k_in,
                                      int32_t blocks, const void* const* weights,
                                      const float* const* biases, int64_t n_out, int32_t act,
                                      float* out, int64_t ldo, int32_t* error,
                                      cudaStream_t stream);

/* cugo_b200_mlp_fused with the policy's sampling in the same kernel (the reference's
 * _act, python/cugo_ppo50.py:74-82, with Gumbel-max instead of torch.multinomial):
 * per row, the masked Gumbel-max action over the first 179 outputs and its log
 * probability, as cugo_b200_sample_actions computes them from the same logits (the
 * same Philox noise, lowest action on ties, -1 and log p 0 for a row without a legal
 * action).  legal_bits uint64 [m, 3] (bit a of word a / 64: what
 * cugo_b200_observe_indexed_bf16_bits writes, or cugo_b200_pack_legal makes from a
 * bool mask), game int64 [m], decision int32 [m], actions int64 [m], logp fp32 [m];
 * n_out >= 179; out (fp32 [m, ldo]) may be NULL when the logits are not needed.
 * rows (optional, int64 [m]): game and decision then hold n_games entries and row r
 * reads entry rows[r] (a batch's running games without a gather); a row whose entry
 * is outside [0, n_games) gets action -1 and log p 0.
 * m_dev (optional): a device-resident int32 row count, read when the kernel starts;
 * only rows below min(m, *m_dev) are computed (a loop can launch without reading the
 * count back).  No counterpart in the reference. */
CUGO_B200_API int cugo_b200_mlp_fused_sample(const void* x, int64_t ldx, int64_t m,
                                             int64_t k_in, int32_t blocks,
                                             const void* const* weights,
                                             const float* const* biases, int64_t n_out,
                                             int32_t act, const uint64_t* legal_bits,
                                             const int64_t* game, const int32_t* decision,
                                             const int64_t* rows, int64_t n_games,
                                             int64_t seed_base, int32_t greedy, int64_t* actions,
                                             float* logp, float* out, int64_t ldo,
                                             const int32_t* m_dev, int32_t* error,
                                             cudaStream_t stream);

/* Packs bool legal masks [m, 179] into uint64 [m, 3] (bit a of word a / 64), the
 * form the fused sampling head reads.  No counterpart in the reference. */
CUGO_B200_API int cugo_b200_pack_legal(const bool* legal, int64_t m, uint64_t* bits,
                                       cudaStream_t stream);

/* Self-test of the failure-detection path of every pipeline wait in the GEMM and
 * whole-network kernels (no counterpart in the reference): one block waits on an
 * mbarrier that nothing arrives on, with the same bounded wait those kernels use
 * (limited on the GPU's global timer; 0 < limit_ns <= 1 s here, ~2 s there); the
 * wait gives up, *error (int32, device) is set to 1, *waited_ns (int64, device,
 * optional) receives the time waited, and the kernel returns with the context
 * usable. */
CUGO_B200_API int cugo_b200_wait_timeout_probe(int64_t limit_ns, int32_t* error,
                                               int64_t* waited_ns, cudaStream_t stream);

/* ---- PPO update (PpoUpdater._step, python/cugo_ppo50.py:558-623) ----------------- */

/* The plain-target PPO losses of a minibatch of b rows and their gradients in one
 * pass (it replaces the masked log_softmax, gather, ratio, clipped surrogate,
 * entropy and smooth-L1 value loss of python/cugo_ppo50.py:572-603 and their
 * autograd backward): loss = mean(-min(r A, clamp(r, 1 - clip, 1 + clip) A))
 * - entropy_coef mean(entropy) + value_coef mean(smooth_l1(value, ret)), r =
 * exp(log p_new(action) - logp_old), log p from the logits masked to -1e30 where
 * legal is 0.  logits fp32 [b, ldl >= 179]; legal bool [b, 179]; actions int64;
 * logp_old, adv, ret fp32 [b]; value fp32 with row stride value_ld; entropy_coef a
 * device fp32 scalar.  Writes d loss / d logits as bf16 [b, ldd >= 179] (columns
 * 179 .. ldd - 1 zero), d loss / d value fp32 [b], and stats fp32 [5] = the
 * minibatch means of the policy loss, value loss, entropy, KL estimate
 * (r - 1) - log r and clip fraction (|r - 1| > clip). */
CUGO_B200_API int cugo_b200_ppo_loss(const float* logits, int64_t ldl, const bool* legal,
                                     const int64_t* actions, const float* logp_old,
                                     const float* adv, const float* value, int64_t value_ld,
                                     const float* ret, int64_t b, float clip,
                                     const float* entropy_coef, float value_coef, void* dlogits,
                                     int64_t ldd, float* dvalue, float* stats,
                                     cudaStream_t stream);

/* Column sums (fp32 [n], 8 <= n <= 2048, n a multiple of 8) of bf16 x [rows, n]
 * (row stride ldx); with z (bf16, ldz), of dz = x * act'(z) (act 0 none, 1 ReLU,
 * 2 SiLU), which is also written to dz (bf16, ldd).  The bias gradients of the
 * update's backward.  scratch: the caller's fp32 buffer of at least
 * cugo_b200_colsum_scratch_floats(rows, n) floats for the per-block partial sums,
 * which a second launch adds up in a fixed order (the same result on every run);
 * a smaller one returns CUGO_B200_ERR_CAPACITY.  No counterpart in the reference
 * (torch reductions there). */
CUGO_B200_API int cugo_b200_colsum_bf16(const void* x, int64_t ldx, const void* z, int64_t ldz,
                                        int32_t act, void* dz, int64_t ldd, int64_t rows,
                                        int32_t n, float* sums, float* scratch,
                                        int64_t scratch_floats, cudaStream_t stream);

/* Scratch floats cugo_b200_colsum_bf16 and cugo_b200_scalar_head_backward need for
 * `rows` rows of n columns. */
CUGO_B200_API int64_t cugo_b200_colsum_scratch_floats(int64_t rows, int32_t n);

/* Backward of a one-output head v = w . act(h) + b over h bf16 [rows, n] (the
 * critic's value head): dh = dv w act'(h) (bf16, ldd), dh_sums = its column sums,
 * dw = sum_i dv_i act(h_i) (fp32 [n]), db = sum_i dv_i (fp32 [1]); dv fp32 [rows],
 * w bf16 [n]; scratch as for cugo_b200_colsum_bf16.  No counterpart in the
 * reference. */
CUGO_B200_API int cugo_b200_scalar_head_backward(const float* dv, const void* w, const void* h,
                                                 int64_t ldh, int32_t act, void* dh, int64_t ldd,
                                                 int64_t rows, int32_t n, float* dh_sums,
                                                 float* dw, float* db, float* scratch,
                                                 int64_t scratch_floats, cudaStream_t stream);

/* Weight gradient of a linear layer: dw[o][i] = sum over the rows r of
 * dy[r][o] x[r][i] (fp32 out, row stride lddw), with dy bf16 [rows, n_out] (row
 * stride lddy) and x bf16 [rows, n_in] (ldx): both operands enter the tcgen05 MMA
 * transposed (MN-major), the rows split across the SMs, each split's partial tile
 * written to scratch and the splits added in a fixed order (the same result on
 * every run).  scratch: the caller's fp32 buffer (16-byte aligned) of at least
 * cugo_b200_wgrad_scratch_floats(rows, n_out, n_in) floats; a smaller one returns
 * CUGO_B200_ERR_CAPACITY.  dy, x 16-byte aligned, strides multiples of 8.  error
 * as for cugo_b200_gemm_bf16.  Replaces the weight gradients autograd computes
 * for the reference's nn.Linear layers under bf16 autocast (python/cugo_ppo50.py:
 * 558-623, PpoUpdater._step's backward). */
CUGO_B200_API int cugo_b200_wgrad_bf16(const void* dy, int64_t lddy, const void* x, int64_t ldx,
                                       int64_t rows, int64_t n_out, int64_t n_in, float* dw,
                                       int64_t lddw, float* scratch, int64_t scratch_floats,
                                       int32_t* error, cudaStream_t stream);

/* Scratch floats cugo_b200_wgrad_bf16 needs for `rows` rows of an n_out x n_in
 * weight. */
CUGO_B200_API int64_t cugo_b200_wgrad_scratch_floats(int64_t rows, int64_t n_out, int64_t n_in);

/* Policy forward that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory — for example a Go/Java/Rust
 * serving process that passes only its own fixed input and output buffers and keeps
 * cudaMalloc (which synchronises the device) off its request path, or a runtime
 * that reserved all device memory at start-up.  Runs the same layer chain as the
 * Python policy (ResidualMlpPolicy.forward) through cugo_b200_gemm_bf16:
 *   h = W[0] x + b[0]; per block h = h + W[2i+2] act(W[2i+1] h + b[2i+1]) + b[2i+2];
 *   out = W[last] act(h) + b[last]
 * x bf16 [m, inputs] (ldx); weights/biases: HOST arrays of 2 + 2*blocks DEVICE
 * pointers (bf16 [out, in] weights; biases may be NULL or hold NULL entries);
 * act 1 ReLU, 2 SiLU; out fp32 [m, outputs] (ldo, rows a multiple of 16 bytes);
 * error as for cugo_b200_gemm_bf16.  The hidden activations live in a buffer
 * compiled into the library (16 MiB held on every GPU that loads it until the
 * process exits): m * hidden must not exceed 4,194,304 (e.g. 8,192 rows at hidden
 * 512), larger calls return CUGO_B200_ERR_CAPACITY.  The first call on a device
 * looks up that buffer's device address, so make it before any stream capture;
 * the address is kept for the life of the process, so a device must not be reset
 * (cudaDeviceReset) after its first call.  All calls share the buffer: calls that
 * overlap on the GPU (other streams or threads) race and must be serialised by the
 * caller. */
CUGO_B200_API int cugo_b200_policy_forward_noalloc(const void* x, int64_t ldx, int64_t m,
                                                   int64_t inputs, int64_t hidden,
                                                   int32_t blocks, int64_t outputs,
                                                   const void* const* weights,
                                                   const void* const* biases, int32_t act,
                                                   float* out, int64_t ldo, int32_t* error,
                                                   cudaStream_t stream);

/* observe_indexed_bf16 (observe_indexed, torch50_ext.cu:520-544, with bf16 features)
 * with the legal mask written as bits, uint64 [m, 3] (bit a of word a / 64), for the
 * fused MLP's sampling head; no bool mask is written.  m_dev
 * (optional): a device-resident int32 row count; rows from min(m, *m_dev) on are left
 * alone. */
CUGO_B200_API int cugo_b200_observe_indexed_bf16_bits(const uint8_t* states, int64_t n_states,
                                                      const int64_t* env_ids, int64_t m,
                                                      void* features_bf16, uint64_t* legal_bits,
                                                      uint8_t* players, bool* done,
                                                      int16_t* status, const int32_t* m_dev,
                                                      cudaStream_t stream);

/* observe_indexed with the features written as bf16 [m, 720] (16-byte aligned):
 * the policy's input layer reads them directly.  Same values as observe_indexed
 * rounded to bf16 (the reference casts features to bf16 under autocast). */
CUGO_B200_API int cugo_b200_observe_indexed_bf16(const uint8_t* states, int64_t n_states,
                                                 const int64_t* env_ids, int64_t m,
                                                 void* features_bf16, bool* legal,
                                                 uint8_t* players, bool* done, int16_t* status,
                                                 cudaStream_t stream);

/* observe_indexed writing the sequence policy's hybrid query input in one pass
 * (python/cugo_seq50.py:196-208: cat(features, legal) cast to bf16): query bf16
 * [m, ldq] with features in columns 0..719, legal as 0/1 in 720..898 and zeros
 * in 899..ldq-1 (ldq >= 899, a multiple of 8, e.g. 904); legal/players/done/
 * status as observe_indexed. */
CUGO_B200_API int cugo_b200_observe_query_bf16(const uint8_t* states, int64_t n_states,
                                               const int64_t* env_ids, int64_t m, void* query,
                                               int64_t ldq, bool* legal, uint8_t* players,
                                               bool* done, int16_t* status, cudaStream_t stream);

/* observe_indexed writing the oracle critic's input in one pass (python/cugo_ppo50.py:
 * 478-482, _critic_input without stock planes, as action_values and _child_values
 * build it, :86-104, 214-225): critic_in bf16 [m, ldc] with the mover's features in
 * columns 0..719, the hand of the mover's opponent as 0/1 in 720..769 and zeros in
 * 770..ldc-1 (ldc >= 770, a multiple of 8, e.g. 776); players/done/status as
 * observe_indexed. */
CUGO_B200_API int cugo_b200_observe_critic_bf16(const uint8_t* states, int64_t n_states,
                                                const int64_t* env_ids, int64_t m, void* critic_in,
                                                int64_t ldc, uint8_t* players, bool* done,
                                                int16_t* status, cudaStream_t stream);

/* Redeal rows in place for an observer (python/cugo_ppo50.py:125-149, _redeal): the
 * opponent of seats[i] keeps the hand cards shown by a shake and gets the rest anew,
 * as many as before, uniformly from the cards seats[i] cannot see (those cards and
 * the stock); the stock is the remainder; the opponent's held set follows; the stock's
 * RNG word is reseeded in [-2^62, 2^62).  Randomness: Philox4x32-10 keyed by seed,
 * counter {row, attempt, stream}.  Rows must be distinct. */
CUGO_B200_API int cugo_b200_redeal(uint8_t* rows, int64_t n, const int64_t* seats, int64_t seed,
                                   int32_t attempt, cudaStream_t stream);

/* Redealt worlds in one launch (the loop of redeal_worlds, python/cugo_ppo50.py:
 * 152-177): out [worlds * r, 248] world-major, world row w = k * r + b a copy of
 * states[env_ids[b]] redealt for observer seats[b] so that the observer's
 * features and legal actions are unchanged.  Attempt a (0 .. tries - 1, tries <=
 * 127) is cugo_b200_redeal's draw with Philox counter w; the first attempt whose
 * observation and legal mask equal the real deal's is kept; a row that fails
 * every attempt keeps the real deal.  accepted (optional, int8 [worlds * r]) gets
 * the attempt kept or -1.  A bad env id gives a zero row. */
CUGO_B200_API int cugo_b200_redeal_worlds(const uint8_t* states, int64_t n_states,
                                          const int64_t* env_ids, int64_t r,
                                          const int64_t* seats, int64_t worlds, int64_t seed,
                                          int32_t tries, uint8_t* out, int8_t* accepted,
                                          cudaStream_t stream);

/* ---- Sequence policy decode ------------------------------------------------------
 * Single-query attention over a KV cache, replacing decode_attention and its
 * Triton _decode_kernel (python/cugo_seq_attention50.py:22-62), optionally fused
 * with cached_step's KV append (python/cugo_seq50.py:313-316).
 * q bf16: query i, head h at q + i*ldq + h*head_dim; keys/values bf16 [n_rows,
 * heads, slots, head_dim]; rows int64 [n] cache row of query i (NULL: row i);
 * pos int64: with pos_clamp < 0, pos[i] is query i's position (attend slots
 * 0..pos[i], as decode_attention's pos); with pos_clamp >= 0, pos is the cache's
 * per-row length array and the position is min(pos[rows[i]], pos_clamp) (the
 * clamp cached_step applies); out bf16 at out + i*ldo + h*head_dim;
 * scale = head_dim^-0.5 as the reference passes it.  With k_new/v_new (bf16,
 * row stride ldn, same head layout as q) the token's key/value are first
 * written to slot pos[i] of its row, which it then attends; the rows of one call
 * must then be distinct.  head_dim must be 32, slots <= 512; a query whose pos
 * or row is out of range gets zeros and sets *error (device int, may be NULL). */
CUGO_B200_API int cugo_b200_decode_attention(const void* q, int64_t ldq, const void* k_new,
                                             const void* v_new, int64_t ldn, void* keys,
                                             void* values, int64_t n_rows, int32_t heads,
                                             int32_t slots, int32_t head_dim,
                                             const int64_t* pos, int64_t pos_clamp,
                                             const int64_t* rows, int64_t n, float scale,
                                             void* out, int64_t ldo, int32_t* error,
                                             cudaStream_t stream);

/* cugo_b200_decode_attention restricted to the queries with active[i] set (bool [n],
 * device; NULL: all): an inactive query reads and writes no cache slot, appends
 * nothing, sets no error and gets zeros.  The sequence self-play wave passes its
 * unfinished games, whose rows alone feed a later decision (no counterpart in the
 * reference, whose wave runs every row). */
CUGO_B200_API int cugo_b200_decode_attention_active(
    const void* q, int64_t ldq, const void* k_new, const void* v_new, int64_t ldn, void* keys,
    void* values, int64_t n_rows, int32_t heads, int32_t slots, int32_t head_dim,
    const int64_t* pos, int64_t pos_clamp, const int64_t* rows, int64_t n, float scale, void* out,
    int64_t ldo, const bool* active, int32_t* error, cudaStream_t stream);

/* nn.LayerNorm(d) of fp32 rows (eps as given, biased variance) into bf16 rows,
 * the operand of the next GEMM (norm1/norm2/norm of the sequence transformer,
 * python/cugo_seq50.py:311,321; python/cugo_seq50.py:226).  d in {128, 256, 512,
 * 1024}; x, gamma, beta fp32, 16-byte aligned; out bf16 (8-byte aligned). */
CUGO_B200_API int cugo_b200_layernorm(const float* x, int64_t ldx, const float* gamma,
                                      const float* beta, int64_t d, float eps, void* out,
                                      int64_t ldo, int64_t n, cudaStream_t stream);

/* Event tokens (SeqNet.event_token, python/cugo_seq50.py:276-282 with
 * encode_events :91-109): out[i] = event_in(tokens(events[i % n_events],
 * seats[i])) + position[1 + min(index[i % n_events], 47)] + token_type_row.
 * weight_t is the transposed event_in weight, bf16 [414, d]; bias, position
 * ([49, d]) and token_type_row fp32; out fp32 [n, ldo]; d in {256, 512}.
 * index may be NULL (0). */
CUGO_B200_API int cugo_b200_event_embed(const int64_t* events, int64_t n_events,
                                        const int64_t* seats, const int64_t* index, int64_t n,
                                        const void* weight_t, const float* bias,
                                        const float* position, const float* token_type,
                                        int64_t d, float* out, int64_t ldo, cudaStream_t stream);

/* Opening tokens (SeqNet.start_token, python/cugo_seq50.py:271-274 with
 * encode_start :112-128): out[i] = start_in(tokens(start[i % n_start], seats[i]))
 * + position0 + token_type_row.  weight_t bf16 [274, d] (transposed start_in
 * weight); other arguments as cugo_b200_event_embed. */
CUGO_B200_API int cugo_b200_start_embed(const int64_t* start, int64_t n_start,
                                        const int64_t* seats, int64_t n, const void* weight_t,
                                        const float* bias, const float* position0,
                                        const float* token_type, int64_t d, float* out,
                                        int64_t ldo, cudaStream_t stream);

/* encode_events (python/cugo_seq50.py:91-109): observer-relative event tokens
 * [b_rows, length, 414] (fp32, or bf16 when tokens_bf16) of events int64
 * [b_rows, max_events, 9] for observer seats[b]; valid (optional) bool
 * [b_rows, length] = e < count[b].  Values are 0/1 and the opponent's drawn-card
 * count, exact in either type. */
CUGO_B200_API int cugo_b200_encode_events(const int64_t* events, int64_t max_events,
                                          const int64_t* count, const int64_t* seats,
                                          int64_t b_rows, int32_t length, void* tokens,
                                          int32_t tokens_bf16, bool* valid, cudaStream_t stream);

/* Attention of SeqNet.forward_games (python/cugo_seq50.py:240-265), 8 heads of 32
 * (d 256): qkv bf16 [rows, ldq >= 768] (q | k | v) holds the token rows in three
 * blocks: n_seq openings, then n_seq x length events (sequence-major), then
 * n_seq x queries decision queries; out bf16 [rows, ldo] gets each row's attention
 * output.  The opening sees itself, event e the opening and events 0..e, query q of
 * sequence s the opening, events 0 .. min(seen[s * queries + q], length) - 1 and
 * itself.  length <= 48; qkv and out 16-byte aligned, ldq and ldo multiples of 8. */
CUGO_B200_API int cugo_b200_games_attention(const void* qkv, int64_t ldq, int64_t n_seq,
                                            int32_t length, int32_t queries, const int64_t* seen,
                                            float scale, void* out, int64_t ldo,
                                            cudaStream_t stream);

/* One decision round of a training collection appended to a device-resident
 * transition store (no reference counterpart: it replaces the per-round
 * hands_indexed, stock_indexed, index_select and RolloutStorage.append of
 * python/cugo_ppo50.py:394-412).  Round row i < min(m, *m_dev) (m_dev optional)
 * plays game row active[i] of states; its bf16 features (row i of features, ldf
 * elements apart, 16-byte aligned), legal bit words (uint64 [m, 3], bit a of word
 * a / 64), player (players[i]), action, behaviour log p and learner flag (learner
 * NULL: every row is the learner's) go to store row sizes[parity] + i, with the
 * opponent's hand (hand word 1 - player of the game row) and the next 8 stock draws
 * (stock_indexed's packing) read from the game row; the legal bits are written as
 * a bool [capacity, 179] mask, features as bf16 [capacity, 720].
 * sizes[parity ^ 1] = sizes[parity] + rows: the store's size moves between the
 * two slots of sizes (int64 [2]) round by round.  Rows past capacity are not
 * written and set *overflow (optional) to 1. */
CUGO_B200_API int cugo_b200_record_transitions(
    const uint8_t* states, int64_t n_states, const int64_t* active, int64_t m,
    const int32_t* m_dev, const void* features, int64_t ldf, const uint64_t* legal_bits,
    const uint8_t* players, const int64_t* actions, const float* logp, const bool* learner,
    int64_t* sizes, int32_t parity, int64_t capacity, void* out_features, bool* out_legal,
    int64_t* out_actions, float* out_logp, int64_t* out_opp_hand, int64_t* out_stock,
    int64_t* out_env, int64_t* out_seat, bool* out_learner, int32_t* overflow,
    cudaStream_t stream);

/* The oracle critic's stock planes (python/cugo_ppo_nets50.py:104-110 stock_planes
 * of ext.stock_indexed, as python/cugo_ppo50.py:478-482 appends them): in bf16 row i
 * (ld elements apart) of rows, column first_column + 50 k + c is set to 1 where the
 * k-th of the next 8 stock draws of game row env_ids[i] is card c < 50 (env_ids
 * NULL: row i); other columns are not written (observe_critic_bf16 zero-fills the
 * row past the hand plane).  An invalid id leaves its row alone. */
CUGO_B200_API int cugo_b200_stock_planes_bf16(const uint8_t* states, int64_t n_states,
                                              const int64_t* env_ids, int64_t m, void* rows,
                                              int64_t ld, int32_t first_column,
                                              cudaStream_t stream);

/* The end of one decision step of the sequence self-play wave for its w games (no
 * reference counterpart: it replaces the tensor bookkeeping of WaveCollector._step,
 * python/cugo_seq_selfplay50.py:108-163).  Inputs per game g: the step's observe
 * outputs (done, status, player), the sampled action (-1: no legal action) and its
 * log p, and the outputs of step_events_indexed.  A game that was running:
 * counts a bad observe (status != 0 or no legal action) and a bad step (status != 0)
 * into *bad; when it finishes, final_reward0/final_nagari/finished are set and
 * *running drops by one; a committed event is written to slot min(count, max_events
 * - 1) of its event log (int64 [w, max_events, 9]), then count[g] and the KV-cache
 * lengths of both seats (cache_length[g], cache_length[w + g]) grow by one;
 * decision[g] grows by one.  Records (optional, [max_steps, w], rec_actions NULL:
 * none) at row *step_index: action, player, count before the step and log p of a
 * game that was running (a finished game's entries are not written), and
 * whether the game was running and the learner moved (learner, optional: per game,
 * whether the learner's network chose the action; NULL: always).  *step_index then
 * grows by one. */
CUGO_B200_API int cugo_b200_wave_tail(
    int64_t w, const bool* obs_done, const int16_t* obs_status, const uint8_t* players,
    const int64_t* actions, const float* logp, const float* reward0, const bool* new_done,
    const bool* nagari, const int16_t* status, const bool* committed, const int64_t* step_events,
    const bool* learner, float* final_reward0, bool* final_nagari, bool* finished, int64_t* bad, int32_t* running,
    int64_t* events, int32_t max_events, int64_t* count, int64_t* cache_length, int32_t* decision,
    int64_t* step_index, int64_t* rec_actions, int64_t* rec_seat, int64_t* rec_count,
    float* rec_logp, bool* rec_valid, int64_t max_steps, cudaStream_t stream);

/* Token widths of the sequence policy (python/cugo_seq50.py:37-38). */
CUGO_B200_API int64_t cugo_b200_event_inputs(void); /* EVENT_IN = 414 */
CUGO_B200_API int64_t cugo_b200_start_inputs(void); /* START_IN = 274 */

#ifdef __cplusplus
}
#endif

#endif
