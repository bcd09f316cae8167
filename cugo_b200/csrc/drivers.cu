// Seeded random-legal drivers of the benchmark configurations, on the GPU.
//
// The reference has no such driver (its rollouts use canonical actions or a
// host LCG, tests/torch50_test.cpp:196-200); these kernels play the rule
// defined once for every implementation:
//   game i: seed = seed_base + i, first player = i & 1
//   decision d of game i picks the floor(r0 * n / 2^32)-th of its n legal
//   actions, r0 = Philox4x32-10({i lo, i hi, d, stream}, {seed lo, seed hi})[0]
//   event hash: FNV-1a 64 over the start record and every committed event.
#include <cuda_runtime.h>
#include <stdint.h>

#include "engine/driver.cuh"
#include "tile.cuh"
#include "engine/env.cuh"
#include "../../include/cugo_b200.h"

using namespace cb;

// In-place step without per-row outputs (env_kernels.cu).
int cb_step_in_place(uint8_t* states, int64_t n, const int64_t* actions, cudaStream_t stream);

namespace {

using namespace cb::tile;
constexpr u64 kFnvOffset = 0xcbf29ce484222325ull;
constexpr u64 kFnvPrime = 0x100000001b3ull;

__device__ __forceinline__ u64 fnv_words(u64 h, const i64* words, int n) {
  for (int w = 0; w < n; ++w) {
    const u64 v = static_cast<u64>(words[w]);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      h ^= (v >> (8 * b)) & 0xffu;
      h *= kFnvPrime;
    }
  }
  return h;
}

// Whole games: thread k plays game game0 + k to the end (or max_decisions).
__global__ void __launch_bounds__(kBlock) rollout_kernel(
    i64 game0, i64 n, i64 seed_base, int max_decisions, u32 stream, u64* __restrict__ final_rows,
    i64* __restrict__ reward0_out, int32_t* __restrict__ decisions_out,
    int32_t* __restrict__ events_out, u64* __restrict__ hash_out, int16_t* __restrict__ status_out) {
  const i64 k = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const u64 game = static_cast<u64>(game0 + k);
  const u64 seed = static_cast<u64>(seed_base) + game;
  Game g;
  create_game(g, seed, static_cast<u32>(game & 1u));
  i64 words[kEventWords];
  start_words(g, words);
  u64 h = fnv_words(kFnvOffset, words, kStartWords);
  int d = 0, ev = 0;
  i32 st = 0;
  i64 rew = 0;
  while (!g.done() && d < max_decisions) {
    const LegalInfo li = torch_legal(g);
    const u32 r0 = game_draw(game, static_cast<u32>(d), stream, seed).v[0];
    const u32 a = pick_set_bit(li.legal.w0, li.legal.w1, li.legal.w2, r0);
    if (a == 0xffffu) {
      st = -2;
      break;
    }
    const EventBase before = event_base(g);
    const StepOut r = step_game(g, a);
    ++d;
    st = static_cast<i32>(r.status);
    rew = r.reward0;
    if (r.status != kOk) break;
    if (r.committed) {
      event_words(before, g, words);
      h = fnv_words(h, words, kEventWords);
      ++ev;
    }
  }
  zero_padding(g);
  u64* out = final_rows + k * kRowWords;
#pragma unroll
  for (int w = 0; w < kRowWords; ++w) out[w] = g.w[w];
  reward0_out[k] = rew;
  decisions_out[k] = d;
  events_out[k] = ev;
  hash_out[k] = h;
  status_out[k] = static_cast<int16_t>(st);
}

// Replaces every finished game by the slot's next game (index + n_slots, decision
// counter 0, completed + 1).  A block scans 4,096 slots (the done byte of each
// row), queues the finished ones in shared memory and deals them with consecutive
// threads, so a warp's deal work is not repeated for one finished lane among
// thirty-one live ones, as it would be inside the decision kernel.
constexpr int kResetSpan = 4096;

__global__ void __launch_bounds__(256) reset_finished_kernel(
    u64* __restrict__ states, i64 n_slots, i64 seed_base, i64* __restrict__ slot_game,
    int32_t* __restrict__ slot_decision, int32_t* __restrict__ slot_completed) {
  __shared__ int32_t queue[kResetSpan];
  __shared__ int count;
  if (threadIdx.x == 0) count = 0;
  __syncthreads();
  const i64 first = (i64)blockIdx.x * kResetSpan;
  const uint8_t* bytes = reinterpret_cast<const uint8_t*>(states);
  for (int k = threadIdx.x; k < kResetSpan; k += blockDim.x) {
    const i64 slot = first + k;
    if (slot < n_slots && bytes[slot * kRowBytes + kDoneByte] != 0)
      queue[atomicAdd(&count, 1)] = static_cast<int32_t>(k);
  }
  __syncthreads();
  for (int q = threadIdx.x; q < count; q += blockDim.x) {
    const i64 slot = first + queue[q];
    const i64 game = slot_game[slot] + n_slots;
    Game g;
    create_game(g, static_cast<u64>(seed_base + game), static_cast<u32>(game & 1));
    zero_padding(g);
    u64* row = states + slot * kRowWords;
#pragma unroll
    for (int w = 0; w < kRowWords; ++w) row[w] = g.w[w];
    slot_game[slot] = game;
    slot_decision[slot] = 0;
    slot_completed[slot] += 1;
  }
}

// The observation and random legal pick of every slot after the resets: features
// and masks written like observe() writes them, actions[slot] = the pick (-1 for a
// game finished at its deal), decision and step counters advanced.  The step itself
// is a second launch (the in-place step kernel): the rule code of observe and step
// in one kernel overflows the instruction cache (ncu: "no instruction" was the top
// stall of the fused kernel, 4.6 cycles per issued instruction).
__global__ void __launch_bounds__(kBlock, 5) selfplay_pick_kernel(
    const u64* __restrict__ states, i64 n_slots, i64 seed_base, const i64* __restrict__ slot_game,
    int32_t* __restrict__ slot_decision, int64_t* __restrict__ slot_steps,
    float* __restrict__ features, bool* __restrict__ legal_out, i64* __restrict__ actions) {
  WarpTile& t = my_tile();
  const i64 slot = (i64)blockIdx.x * kBlock + threadIdx.x;
  const i64 tile_base = (i64)blockIdx.x * kBlock + (threadIdx.x & ~31);
  gather_rows(t, states, slot < n_slots ? slot : -1);
  Game g;
  load_game(t, g);
  __syncwarp();  // rows are in registers: the tile now holds packets
  const PacketRef pk = lane_packet(t);
  ObsMeta meta;
  if (slot < n_slots) {
    observe_game(g, pk, meta);
    const i64 game = slot_game[slot];
    const u32 decision = static_cast<u32>(slot_decision[slot]);
    const u32 r0 = game_draw(static_cast<u64>(game), decision, 0u, static_cast<u64>(seed_base + game)).v[0];
    const u32 action = pick_set_bit(meta.legal.w0, meta.legal.w1, meta.legal.w2, r0);
    if (action != 0xffffu) {
      slot_decision[slot] = static_cast<int32_t>(decision + 1u);
      slot_steps[slot] += 1;
      actions[slot] = static_cast<i64>(action);
    } else {
      actions[slot] = -1;  // "not legal": the step leaves the row unchanged
    }
  } else {
    for (u32 k = 0; k < kBitWords; ++k) pk.bits[k] = 0;
    for (u32 k = 0; k < kScalarColumns; ++k) pk.scal[k] = 0.0f;
    meta.legal = Legal{};
  }
  store_legal(t, meta.legal);
  const i64 left = n_slots - tile_base;
  const int rows_here = left >= 32 ? 32 : (left > 0 ? (int)left : 0);
  emit_features(t, features, (i64)kFeatures, tile_base, rows_here);
  emit_legal(t, legal_out, tile_base, rows_here);
}

// Redeal of a row for the observer seat (the reference's _redeal,
// python/cugo_ppo50.py:125-149, on the device): the opponent's hand keeps its cards
// shown by a shake and gets the rest — as many cards as before — drawn uniformly
// from the cards the observer cannot see (those hand cards and the stock); the stock
// is what remains; `held` (every card ever in that hand) follows the new hand; the
// stock's draw stream gets a new seed in [-2^62, 2^62).  Draws: Philox4x32-10 with
// counter {ctr lo, ctr hi, attempt, 8 + k / 4} and key {seed lo, seed hi}, word
// k % 4: a uniform subset by successive picks of the floor(r * left / 2^32)-th
// remaining card; the seed from counter {ctr lo, ctr hi, attempt, 7}.
// W: a pointer to the row in memory or the row's words in registers (constant
// indices only, so a register row stays in registers).
template <typename W>
__device__ __forceinline__ void redeal_row(W& w, bool s0, i64 ctr, i64 seed, u32 attempt) {
  const u64 hand = s0 ? w[1] : w[0];
  const u64 held = s0 ? w[21] : w[20];
  const u64 fixed = hand & (s0 ? w[23] : w[22]);
  const u64 free = hand & ~fixed;
  const u64 unknown = free | w[3];
  u64 left = unknown, picked = 0;
  const u32 count = popc(free);
  u32 remaining = popc(left);
  const u32 c0 = static_cast<u32>(ctr), c1 = static_cast<u32>(static_cast<u64>(ctr) >> 32);
  const u32 k0 = static_cast<u32>(seed), k1 = static_cast<u32>(static_cast<u64>(seed) >> 32);
  Philox4 r{};
  for (u32 k = 0; k < count; ++k) {
    if ((k & 3u) == 0) r = philox4x32_10(c0, c1, attempt, 8u + (k >> 2), k0, k1);
    const u32 q = k & 3u;
    const u32 word = q == 0 ? r.v[0] : (q == 1 ? r.v[1] : (q == 2 ? r.v[2] : r.v[3]));
    const u64 bit = u64{1} << nth_card(left, static_cast<u32>((static_cast<u64>(word) * remaining) >> 32));
    picked |= bit;
    left &= ~bit;
    --remaining;
  }
  const u64 new_hand = fixed | picked;
  const u64 new_held = (held & ~hand) | new_hand;
  w[3] = unknown & ~picked;
  if (s0) {
    w[1] = new_hand;
    w[21] = new_held;
  } else {
    w[0] = new_hand;
    w[20] = new_held;
  }
  const Philox4 sd = philox4x32_10(c0, c1, attempt, 7u, k0, k1);
  const u64 bits63 = ((static_cast<u64>(sd.v[0]) << 32) | sd.v[1]) >> 1;  // [0, 2^63)
  w[6] = bits63 - (u64{1} << 62);  // as int64: [-2^62, 2^62)
}

// One attempt on rows in place; the Philox counter is the row index.
__global__ void __launch_bounds__(256) redeal_kernel(u64* __restrict__ rows, i64 n,
                                                     const i64* __restrict__ seats, i64 seed,
                                                     u32 attempt) {
  const i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  u64* w = rows + i * kRowWords;
  redeal_row(w, __ldg(seats + i) == 0, i, seed, attempt);
}

// The observer's view of a row for the acceptance test: the observation packet
// (features) and the legal mask, in a lane-private shared-memory row.
constexpr int kViewWords = kBitWords + kScalarColumns + 6;  // 67: odd, conflict-free rows

// Redealt worlds (the reference's redeal_worlds loop, python/cugo_ppo50.py:152-177,
// in one launch): world row w = k * r + b is a copy of states[env_ids[b]] in which
// the observer (seats[b]) keeps its view: attempts a = 0 .. tries - 1 redeal the
// real deal with counter w, and the first whose observation packet and legal mask
// equal the real deal's is kept; after `tries` failures the row is the real deal.
// accepted[w] (optional) gets the attempt kept, or -1.  The real deal's view sits
// in dynamic shared memory; the row stays in registers and only the five words a
// redeal touches are restored between attempts.
__global__ void __launch_bounds__(kBlock, 3) redeal_worlds_kernel(
    const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids, i64 r,
    const i64* __restrict__ seats, i64 total, i64 seed, int tries, u64* __restrict__ out,
    int8_t* __restrict__ accepted) {
  extern __shared__ u32 view_smem[];
  WarpTile& t = my_tile();
  u32* view = view_smem + threadIdx.x * kViewWords;
  const i64 row = (i64)blockIdx.x * kBlock + threadIdx.x;
  const i64 b = row < total ? row % r : -1;
  const i64 src = b >= 0 ? lane_source(ids, b, r, n_states) : -1;
  gather_rows(t, states, src);
  Game g;
  load_game(t, g);
  __syncwarp();
  const bool s0 = src >= 0 && __ldg(seats + b) == 0;
  const u64 h0 = g.w[0], h1 = g.w[1], st = g.w[3], rng = g.w[6], hd0 = g.w[20], hd1 = g.w[21];
  const PacketRef pk = lane_packet(t);
  int kept = -1;
  const int last = src >= 0 ? tries : -1;
  for (int a = -1; a < last; ++a) {
    if (a >= 0) {
      g.w[0] = h0; g.w[1] = h1; g.w[3] = st; g.w[6] = rng; g.w[20] = hd0; g.w[21] = hd1;
      redeal_row(g.w, s0, row, seed, static_cast<u32>(a));
    }
    ObsMeta meta;
    observe_game(g, pk, meta);
    const u32 lw[6] = {static_cast<u32>(meta.legal.w0), static_cast<u32>(meta.legal.w0 >> 32),
                       static_cast<u32>(meta.legal.w1), static_cast<u32>(meta.legal.w1 >> 32),
                       static_cast<u32>(meta.legal.w2), static_cast<u32>(meta.legal.w2 >> 32)};
    if (a < 0) {  // the real deal's view
      for (u32 k = 0; k < kBitWords; ++k) view[k] = pk.bits[k];
      for (u32 k = 0; k < kScalarColumns; ++k) view[kBitWords + k] = __float_as_uint(pk.scal[k]);
      for (int k = 0; k < 6; ++k) view[kBitWords + kScalarColumns + k] = lw[k];
      continue;
    }
    bool same = true;
    for (u32 k = 0; k < kBitWords; ++k) same &= view[k] == pk.bits[k];
    for (u32 k = 0; k < kScalarColumns; ++k) same &= __uint_as_float(view[kBitWords + k]) == pk.scal[k];
    for (int k = 0; k < 6; ++k) same &= view[kBitWords + kScalarColumns + k] == lw[k];
    if (same) {
      kept = a;
      break;
    }
  }
  if (kept < 0) {
    g.w[0] = h0; g.w[1] = h1; g.w[3] = st; g.w[6] = rng; g.w[20] = hd0; g.w[21] = hd1;
    if (src < 0)
      for (int k = 0; k < kRowWords; ++k) g.w[k] = 0;
  }
  __syncwarp();  // every lane is done with its packet before rows overwrite the tile
  store_game(t, g);
  store_tile(t, out, (i64)blockIdx.x * kBlock + (threadIdx.x & ~31), total, row < total ? row : -1);
  if (row < total && accepted) accepted[row] = static_cast<int8_t>(kept);
}

// Branching roots: game r advanced by k_r < 21 random-legal decisions, stopping
// before a decision that would finish the game.
__global__ void __launch_bounds__(kBlock) branch_roots_kernel(i64 n_roots, i64 seed_base,
                                                              u64* __restrict__ roots) {
  const i64 r = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_roots) return;
  const u64 seed = static_cast<u64>(seed_base + r);
  Game g;
  create_game(g, seed, static_cast<u32>(r & 1));
  const u32 k = static_cast<u32>((static_cast<u64>(game_draw(r, 0xffffu, 2u, seed).v[0]) * 21u) >> 32);
  for (u32 d = 0; d < k && !g.done(); ++d) {
    const LegalInfo li = torch_legal(g);
    const u32 a = pick_set_bit(li.legal.w0, li.legal.w1, li.legal.w2,
                               game_draw(r, d, 0u, seed).v[0]);
    if (a == 0xffffu) break;
    Game next = g;
    step_game(next, a);
    if (next.done()) break;
    g = next;
  }
  zero_padding(g);
  u64* out = roots + r * kRowWords;
#pragma unroll
  for (int w = 0; w < kRowWords; ++w) out[w] = g.w[w];
}

// Branch i of root r = i / per_root: (env id, a random legal action of the root
// drawn from stream 1 with counter {r, b}).
__global__ void __launch_bounds__(kBlock) branch_actions_kernel(const u64* __restrict__ roots,
                                                                i64 n_roots, i64 per_root,
                                                                i64 seed_base, i64* __restrict__ ids,
                                                                i64* __restrict__ actions) {
  const i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_roots * per_root) return;
  const i64 r = i / per_root, b = i - r * per_root;
  Game g;
  const u64* row = roots + r * kRowWords;
#pragma unroll
  for (int w = 0; w < kRowWords; ++w) g.w[w] = __ldg(row + w);
  const LegalInfo li = torch_legal(g);
  const u64 ctr = static_cast<u64>(r) | (static_cast<u64>(b) << 32);
  const u32 a = pick_set_bit(li.legal.w0, li.legal.w1, li.legal.w2,
                             game_draw(ctr, 0u, 1u, static_cast<u64>(seed_base + r)).v[0]);
  ids[i] = r;
  actions[i] = a == 0xffffu ? -1 : static_cast<i64>(a);
}

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

inline unsigned blocks_for(i64 n) { return static_cast<unsigned>((n + kBlock - 1) / kBlock); }

}  // namespace

extern "C" {

int cugo_b200_rollout_random(int64_t game0, int64_t n, int64_t seed_base, int32_t max_decisions,
                             uint32_t stream_id, uint8_t* final_rows, int64_t* reward0,
                             int32_t* decisions, int32_t* events, uint64_t* hashes,
                             int16_t* last_status, cudaStream_t stream) {
  if (n < 0 || max_decisions < 0) return CUGO_B200_ERR_ARG;
  if (n > 0 && (!final_rows || !reward0 || !decisions || !events || !hashes || !last_status))
    return CUGO_B200_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(final_rows) & 7u) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  rollout_kernel<<<blocks_for(n), kBlock, 0, stream>>>(
      game0, n, seed_base, max_decisions, stream_id, reinterpret_cast<u64*>(final_rows), reward0,
      decisions, events, hashes, last_status);
  return launch_status();
}

int cugo_b200_selfplay_random_step(uint8_t* states, int64_t n_slots, int64_t seed_base,
                                   int64_t* slot_game, int32_t* slot_decision,
                                   int32_t* slot_completed, int64_t* slot_steps, float* features,
                                   bool* legal, int64_t* actions, cudaStream_t stream) {
  if (n_slots < 0) return CUGO_B200_ERR_ARG;
  if (n_slots > 0 && (!states || !slot_game || !slot_decision || !slot_completed || !slot_steps ||
                      !features || !legal || !actions))
    return CUGO_B200_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(states) & 7u) || (reinterpret_cast<uintptr_t>(features) & 15u) ||
      (reinterpret_cast<uintptr_t>(legal) & 3u) || (reinterpret_cast<uintptr_t>(actions) & 7u))
    return CUGO_B200_ERR_ALIGN;
  if (n_slots == 0) return CUGO_B200_OK;
  reset_finished_kernel<<<static_cast<unsigned>((n_slots + kResetSpan - 1) / kResetSpan), 256, 0,
                          stream>>>(reinterpret_cast<u64*>(states), n_slots, seed_base, slot_game,
                                    slot_decision, slot_completed);
  selfplay_pick_kernel<<<blocks_for(n_slots), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_slots, seed_base, slot_game, slot_decision, slot_steps,
      features, legal, actions);
  if (launch_status() != CUGO_B200_OK) return CUGO_B200_ERR_LAUNCH;
  return cb_step_in_place(states, n_slots, actions, stream);
}

int cugo_b200_redeal(uint8_t* rows, int64_t n, const int64_t* seats, int64_t seed, int32_t attempt,
                     cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!rows || !seats)) || attempt < 0) return CUGO_B200_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(rows) & 7u) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  redeal_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<u64*>(rows), n, seats, seed, static_cast<u32>(attempt));
  return launch_status();
}

int cugo_b200_redeal_worlds(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t r, const int64_t* seats, int64_t worlds, int64_t seed,
                            int32_t tries, uint8_t* out, int8_t* accepted, cudaStream_t stream) {
  if (n_states < 0 || r < 0 || worlds < 0 || tries < 0 || tries > 127) return CUGO_B200_ERR_ARG;
  const int64_t total = r * worlds;
  if (total > 0 && (!env_ids || !seats || !out || (n_states > 0 && !states))) return CUGO_B200_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(states) & 7u) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return CUGO_B200_ERR_ALIGN;
  if (total == 0) return CUGO_B200_OK;
  constexpr int kViewBytes = kBlock * kViewWords * 4;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(redeal_worlds_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kViewBytes) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  redeal_worlds_kernel<<<blocks_for(total), kBlock, kViewBytes, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, r, seats, total, seed, tries,
      reinterpret_cast<u64*>(out), accepted);
  return launch_status();
}

int cugo_b200_branch_roots(int64_t n_roots, int64_t seed_base, uint8_t* roots, cudaStream_t stream) {
  if (n_roots < 0 || (n_roots > 0 && !roots)) return CUGO_B200_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(roots) & 7u) return CUGO_B200_ERR_ALIGN;
  if (n_roots == 0) return CUGO_B200_OK;
  branch_roots_kernel<<<blocks_for(n_roots), kBlock, 0, stream>>>(n_roots, seed_base,
                                                                 reinterpret_cast<u64*>(roots));
  return launch_status();
}

int cugo_b200_branch_actions(const uint8_t* roots, int64_t n_roots, int64_t per_root,
                             int64_t seed_base, int64_t* env_ids, int64_t* actions,
                             cudaStream_t stream) {
  if (n_roots < 0 || per_root < 0) return CUGO_B200_ERR_ARG;
  const i64 n = n_roots * per_root;
  if (n > 0 && (!roots || !env_ids || !actions)) return CUGO_B200_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(roots) & 7u) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  branch_actions_kernel<<<blocks_for(n), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(roots), n_roots, per_root, seed_base, env_ids, actions);
  return launch_status();
}

}  // extern "C"
