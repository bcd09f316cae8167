// Device-side bookkeeping of the training collectors, and their C ABI
// (include/cugo_b200.h).
//
//   record_kernel     appends one decision round of a self-play collection to the
//                     transition store: rows [0, *m_dev) of the round (position i
//                     plays game row active[i]) go to store rows base + i, where
//                     base is the store's device-resident size; the kernel also
//                     reads the opponent's hand and the next 8 stock draws straight
//                     from the game row, and expands the legal bit words to the
//                     bool mask the update reads.  Warp per round row: the 1,440-byte
//                     bf16 feature row moves as 90 16-byte vectors.
//   stock_planes_kernel  the one-hot planes of the next 8 stock draws in the oracle
//                     critic's input rows (OracleCritic with stock planes)
//   wave_tail_kernel  the end of one decision step of the sequence self-play wave:
//                     bad-status counts, final rewards, the event log, the
//                     per-decision records, and the cache-length / event-count /
//                     decision advances, one thread per game (it replaces ~15
//                     tensor launches per step).
//
// Sizes and counters live in device memory, so neither kernel needs a host read
// and both can sit in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "engine/env.cuh"
#include "../../include/cugo_b200.h"

using namespace cb;

namespace {

constexpr int kRecordWarps = 8;
constexpr int kFeatureVecs = kFeatures * 2 / 16;  // 16-byte vectors of a bf16 feature row
static_assert(kFeatures * 2 % 16 == 0, "bf16 feature rows are whole 16-byte vectors");

struct RecordOut {
  __nv_bfloat16* features;  // [capacity, 720]
  bool* legal;              // [capacity, 179]
  int64_t* actions;
  float* logp;
  int64_t* opp_hand;
  int64_t* stock;
  int64_t* env;
  int64_t* seat;
  bool* learner;
};

__global__ void __launch_bounds__(32 * kRecordWarps) record_kernel(
    const u64* __restrict__ states, i64 n_states, const i64* __restrict__ active, i64 m,
    const int32_t* __restrict__ m_dev, const __nv_bfloat16* __restrict__ features, i64 ldf,
    const u64* __restrict__ legal_bits, const uint8_t* __restrict__ players,
    const i64* __restrict__ actions, const float* __restrict__ logp,
    const bool* __restrict__ learner, i64* __restrict__ sizes, int parity, i64 capacity,
    int32_t* __restrict__ overflow, RecordOut out) {
  i64 rows = m;
  if (m_dev) {
    const i64 md = __ldg(m_dev);
    rows = md < 0 ? 0 : (md < m ? md : m);
  }
  // Every block reads the size before any block could write it: the new size goes
  // to the other slot of the ping-pong pair.
  const i64 base = sizes[parity];
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    sizes[parity ^ 1] = base + rows;
    if (base + rows > capacity && overflow) atomicExch(overflow, 1);
  }
  const int lane = threadIdx.x & 31;
  const i64 warp0 = (i64)blockIdx.x * kRecordWarps + (threadIdx.x >> 5);
  const i64 stride = (i64)gridDim.x * kRecordWarps;
  for (i64 r = warp0; r < rows; r += stride) {
    const i64 dst = base + r;
    if (dst >= capacity) break;
    const uint4* src = reinterpret_cast<const uint4*>(features + r * ldf);
    uint4* to = reinterpret_cast<uint4*>(out.features + dst * kFeatures);
    for (int j = lane; j < kFeatureVecs; j += 32) to[j] = __ldg(src + j);
    const u64 w0 = __ldg(legal_bits + 3 * r), w1 = __ldg(legal_bits + 3 * r + 1),
              w2 = __ldg(legal_bits + 3 * r + 2);
    bool* lrow = out.legal + dst * kActions;
    for (int a = lane; a < kActions; a += 32) {
      const u64 w = a < 64 ? w0 : (a < 128 ? w1 : w2);
      lrow[a] = (w >> (a & 63)) & 1u;
    }
    if (lane == 0) {
      const i64 pos = __ldg(active + r);
      const i64 seat = __ldg(players + r) & 1;
      u64 opp = 0, preview = ~0ull;
      if (pos >= 0 && pos < n_states) {
        const u64* row = states + pos * kRowWords;
        opp = __ldg(row + (1 - seat));  // hand words 0 and 1
        Game g;
        g.w[3] = __ldg(row + 3);
        g.w[6] = __ldg(row + 6);
        preview = stock_preview(g);
      }
      out.actions[dst] = __ldg(actions + r);
      out.logp[dst] = __ldg(logp + r);
      out.opp_hand[dst] = static_cast<i64>(opp);
      out.stock[dst] = static_cast<i64>(preview);
      out.env[dst] = pos;
      out.seat[dst] = seat;
      out.learner[dst] = learner ? learner[r] : true;
    }
  }
}

// ---- stock planes of the oracle critic's input -----------------------------------

// Sets column first + 50 k + card of each of the next 8 stock draws of game
// row ids[i] to 1 in bf16 row i (the other columns are left as they are: the
// observe pass that wrote the row zero-fills them).
__global__ void __launch_bounds__(256) stock_planes_kernel(
    const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids, i64 m,
    __nv_bfloat16* __restrict__ rows, i64 ld, int first) {
  const i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const i64 id = ids ? __ldg(ids + i) : i;
  if (id < 0 || id >= n_states) return;
  Game g;
  g.w[3] = __ldg(states + id * kRowWords + 3);
  g.w[6] = __ldg(states + id * kRowWords + 6);
  const u64 packed = stock_preview(g);
  __nv_bfloat16* row = rows + i * ld + first;
  const __nv_bfloat16 one = __float2bfloat16(1.0f);
  for (int k = 0; k < 8; ++k) {
    const u32 card = static_cast<u32>(packed >> (8 * k)) & 0xffu;
    if (card < 50u) row[50 * k + card] = one;
  }
}

// ---- sequence wave ---------------------------------------------------------------

struct WaveState {
  float* final_reward0;  // [w]
  bool* final_nagari;    // [w]
  bool* finished;        // [w]
  int64_t* bad;          // [1]
  int32_t* running;      // [1] games of the wave not finished yet
  int64_t* events;       // [w, max_events, 9]
  int64_t* count;        // [w] committed events so far
  int64_t* cache_length; // [2w] KV-cache lengths (row seat * w + game)
  int32_t* decision;     // [w]
  int64_t* step_index;   // [1]
  int max_events;
  // per-decision records [max_steps, w] (rec_actions == nullptr: not recorded)
  int64_t* rec_actions;
  int64_t* rec_seat;
  int64_t* rec_count;
  float* rec_logp;
  bool* rec_valid;
  int64_t max_steps;
};

__global__ void __launch_bounds__(256) wave_tail_kernel(
    int64_t w, const bool* __restrict__ obs_done, const int16_t* __restrict__ obs_status,
    const uint8_t* __restrict__ players, const int64_t* __restrict__ actions,
    const float* __restrict__ logp, const float* __restrict__ reward0,
    const bool* __restrict__ new_done, const bool* __restrict__ nagari,
    const int16_t* __restrict__ status, const bool* __restrict__ committed,
    const int64_t* __restrict__ step_events, const bool* __restrict__ learner, WaveState s) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // The step index advances in a one-thread launch after this kernel (stream
  // order), so every thread here reads the same value.
  const int64_t step = __ldg(s.step_index);
  if (g < w) {
    const bool active = !obs_done[g];
    const int64_t a = actions[g];
    int bad = 0;
    if (active && (obs_status[g] != 0 || a < 0)) ++bad;  // no legal action or bad observe
    if (active && status[g] != 0) ++bad;
    if (s.rec_actions && step < s.max_steps) {
      // A finished game's entries are left alone (only its valid flag is cleared),
      // so steps replayed after the wave ended change no record.
      const int64_t at = step * w + g;
      if (active) {
        s.rec_actions[at] = a;
        s.rec_seat[at] = players[g];
        s.rec_count[at] = s.count[g];
        s.rec_logp[at] = logp[g];
      }
      s.rec_valid[at] = active && (learner == nullptr || learner[g]);
    }
    if (active && new_done[g]) {
      s.final_reward0[g] = reward0[g];
      if (nagari[g]) s.final_nagari[g] = true;
      s.finished[g] = true;
      atomicSub(s.running, 1);
    }
    if (active && committed[g]) {
      const int64_t c = s.count[g];
      const int64_t slot = c < s.max_events - 1 ? c : s.max_events - 1;
      int64_t* dst = s.events + (g * s.max_events + slot) * kEventWords;
      const int64_t* src = step_events + g * kEventWords;
      for (int k = 0; k < kEventWords; ++k) dst[k] = src[k];
      s.count[g] = c + 1;
      s.cache_length[g] += 1;
      s.cache_length[w + g] += 1;
    }
    if (active) s.decision[g] += 1;
    if (bad) atomicAdd(reinterpret_cast<unsigned long long*>(s.bad), (unsigned long long)bad);
  }
}

__global__ void advance_step_kernel(int64_t* step_index) { *step_index += 1; }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int cugo_b200_record_transitions(const uint8_t* states, int64_t n_states, const int64_t* active,
                                 int64_t m, const int32_t* m_dev, const void* features,
                                 int64_t ldf, const uint64_t* legal_bits, const uint8_t* players,
                                 const int64_t* actions, const float* logp, const bool* learner,
                                 int64_t* sizes, int32_t parity, int64_t capacity,
                                 void* out_features, bool* out_legal, int64_t* out_actions,
                                 float* out_logp, int64_t* out_opp_hand, int64_t* out_stock,
                                 int64_t* out_env, int64_t* out_seat, bool* out_learner,
                                 int32_t* overflow, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || capacity < 0 || (parity != 0 && parity != 1) || !sizes)
    return CUGO_B200_ERR_ARG;
  if (m > 0 && (!states || !active || !features || !legal_bits || !players || !actions || !logp ||
                !out_features || !out_legal || !out_actions || !out_logp || !out_opp_hand ||
                !out_stock || !out_env || !out_seat || !out_learner))
    return CUGO_B200_ERR_ARG;
  if (ldf < kFeatures && m > 0) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(features, 16) || !aligned(out_features, 16) ||
      (ldf * 2) % 16 != 0 || !aligned(legal_bits, 8) || !aligned(sizes, 8))
    return CUGO_B200_ERR_ALIGN;
  // Even an empty round writes the next size slot.
  const int64_t launch_rows = m > 0 ? m : 1;
  int blocks = static_cast<int>((launch_rows + kRecordWarps - 1) / kRecordWarps);
  if (blocks > 148 * 16) blocks = 148 * 16;
  RecordOut out{static_cast<__nv_bfloat16*>(out_features), out_legal, out_actions, out_logp,
                out_opp_hand, out_stock, out_env, out_seat, out_learner};
  record_kernel<<<blocks, 32 * kRecordWarps, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, active, m, m_dev,
      static_cast<const __nv_bfloat16*>(features), ldf, legal_bits, players, actions, logp, learner,
      sizes, parity, capacity, overflow, out);
  return launch_status();
}

int cugo_b200_stock_planes_bf16(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                int64_t m, void* rows, int64_t ld, int32_t first_column,
                                cudaStream_t stream) {
  if (n_states < 0 || m < 0 || first_column < 0 || ld < first_column + 400) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!states || !rows)) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(rows, 2)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  stock_planes_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m,
      static_cast<__nv_bfloat16*>(rows), ld, first_column);
  return launch_status();
}

int cugo_b200_wave_tail(int64_t w, const bool* obs_done, const int16_t* obs_status,
                        const uint8_t* players, const int64_t* actions, const float* logp,
                        const float* reward0, const bool* new_done, const bool* nagari,
                        const int16_t* status, const bool* committed, const int64_t* step_events,
                        const bool* learner, float* final_reward0, bool* final_nagari, bool* finished, int64_t* bad,
                        int32_t* running, int64_t* events, int32_t max_events, int64_t* count,
                        int64_t* cache_length, int32_t* decision, int64_t* step_index,
                        int64_t* rec_actions, int64_t* rec_seat, int64_t* rec_count,
                        float* rec_logp, bool* rec_valid, int64_t max_steps,
                        cudaStream_t stream) {
  if (w < 0 || max_events <= 0 || max_steps < 0) return CUGO_B200_ERR_ARG;
  if (w > 0 && (!obs_done || !obs_status || !players || !actions || !logp || !reward0 ||
                !new_done || !nagari || !status || !committed || !step_events || !final_reward0 ||
                !final_nagari || !finished || !bad || !running || !events || !count ||
                !cache_length || !decision || !step_index))
    return CUGO_B200_ERR_ARG;
  if (rec_actions && (!rec_seat || !rec_count || !rec_logp || !rec_valid)) return CUGO_B200_ERR_ARG;
  if (!aligned(bad, 8)) return CUGO_B200_ERR_ALIGN;
  if (w == 0) return CUGO_B200_OK;
  WaveState s{final_reward0, final_nagari, finished, bad, running, events, count, cache_length,
              decision, step_index, max_events, rec_actions, rec_seat, rec_count, rec_logp,
              rec_valid, max_steps};
  wave_tail_kernel<<<static_cast<unsigned>((w + 255) / 256), 256, 0, stream>>>(
      w, obs_done, obs_status, players, actions, logp, reward0, new_done, nagari, status,
      committed, step_events, learner, s);
  advance_step_kernel<<<1, 1, 0, stream>>>(step_index);
  return launch_status();
}

}  // extern "C"
