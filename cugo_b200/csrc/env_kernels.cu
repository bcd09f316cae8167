// Batch-environment kernels for sm_100a and their C ABI (include/cugo_b200.h).
//
// Layout in HBM: game rows are the reference's 248-byte TorchEnv50 images,
// [N, 248] uint8 (31 little-endian u64 words each); features are fp32 [M, 720],
// legal masks bool [M, 179].
//
// Kernel shape: 128-thread blocks, one game per thread, one 32-game tile per
// warp.  A warp moves its 32 rows between HBM and shared memory cooperatively
// (each row is one 248-byte coalesced access of 31 lanes, gathered through the
// id list for indexed ops), each thread runs the rule code on its row held in
// registers, and the warp writes the 32 feature rows (2,880 B each) and the
// 5,728-byte block of legal masks with 16-byte and 4-byte vector stores.
// Nothing is allocated; every launch goes to the caller's stream, so all
// entry points can be captured in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "engine/env.cuh"
#include "engine/driver.cuh"
#include "tile.cuh"
#include "../../include/cugo_b200.h"

using namespace cb;

// Blocks per SM the rules kernels (observe, step) are compiled for: their
// register budget is 65,536 / (128 x this).
#ifndef CB_ENGINE_MIN_BLOCKS
#define CB_ENGINE_MIN_BLOCKS 5
#endif

namespace {

using namespace cb::tile;

// ---- kernels -------------------------------------------------------------------

// seeds == nullptr: game i is deal seed_base + index[i] with first player index[i] & 1
// (the drivers' seeding, without materialising the two arrays).
__global__ void __launch_bounds__(kBlock) create_kernel(const i64* __restrict__ seeds,
                                                        const i64* __restrict__ first, i64 n,
                                                        u64* __restrict__ rows,
                                                        const i64* __restrict__ index = nullptr,
                                                        i64 seed_base = 0) {
  WarpTile& t = my_tile();
  const i64 row = (i64)blockIdx.x * kBlock + threadIdx.x;
  Game g;
  if (row < n) {
    if (seeds) {
      create_game(g, static_cast<u64>(__ldg(seeds + row)), static_cast<u32>(__ldg(first + row) & 1));
    } else {
      const i64 gi = __ldg(index + row);
      create_game(g, static_cast<u64>(seed_base + gi), static_cast<u32>(gi & 1));
    }
  } else {
    for (int k = 0; k < kRowWords; ++k) g.w[k] = 0;
  }
  store_game(t, g);
  scatter_rows(t, rows, row < n ? row : -1);
}

// observe / observe_indexed: ids == nullptr reads row i for output i.
template <typename F>
__global__ void __launch_bounds__(kBlock, CB_ENGINE_MIN_BLOCKS) observe_kernel(
    const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids, i64 m,
    F* __restrict__ features, i64 ld, int legal_cols, bool* __restrict__ legal,
    uint8_t* __restrict__ players, bool* __restrict__ done, int16_t* __restrict__ status,
    int hand_plane = 0, u64* __restrict__ legal_bits = nullptr,
    const int32_t* __restrict__ m_dev = nullptr) {
  if (m_dev) {  // a device-resident row count (rows past it are left alone)
    const i64 md = __ldg(m_dev);
    m = md < 0 ? 0 : (md < m ? md : m);
  }
  // A grid sized for the batch's capacity: blocks past a device count have nothing
  // to write (no block-wide barrier below, so they may leave at once).
  if ((i64)blockIdx.x * kBlock >= m) return;
  WarpTile& t = my_tile();
  const i64 row = (i64)blockIdx.x * kBlock + threadIdx.x;
  const i64 src = lane_source(ids, row, m, n_states);
  gather_rows(t, states, src);
  Game g;
  load_game(t, g);
  __syncwarp();  // rows are in registers: the tile now holds packets
  const PacketRef pk = lane_packet(t);
  ObsMeta meta;
  if (src >= 0) {
    observe_game(g, pk, meta);
  } else {
    for (u32 k = 0; k < kBitWords; ++k) pk.bits[k] = 0;
    for (u32 k = 0; k < kScalarColumns; ++k) pk.scal[k] = 0.0f;
    meta.legal = Legal{};
    meta.player = 0;
    meta.done = 1;
    meta.status = -1;
  }
  // With hand_plane the extra columns carry the hand of the mover's opponent.
  store_legal(t, hand_plane ? Legal{src >= 0 ? g.hand(meta.player ^ 1u) : 0ull, 0ull, 0ull}
                            : meta.legal);
  const i64 tile_base = (i64)blockIdx.x * kBlock + (threadIdx.x & ~31);
  const i64 left = m - tile_base;
  const int rows_here = left >= 32 ? 32 : (left > 0 ? (int)left : 0);
  emit_features(t, features, ld, tile_base, rows_here);
  if constexpr (sizeof(F) == 2) {
    if (legal_cols > 0)
      emit_legal_columns(t, features, ld, tile_base, rows_here, legal_cols,
                         hand_plane ? 50u : kActions);
  }
  if (legal) emit_legal(t, legal, tile_base, rows_here);
  if (row < m) {
    players[row] = static_cast<uint8_t>(meta.player);
    done[row] = meta.done != 0;
    status[row] = static_cast<int16_t>(meta.status);
    if (legal_bits) {  // the mask as three words: bit a of word a / 64
      legal_bits[row * 3 + 0] = meta.legal.w0;
      legal_bits[row * 3 + 1] = meta.legal.w1;
      legal_bits[row * 3 + 2] = meta.legal.w2;
    }
  }
}

// step / step_indexed / step_events_indexed / branch_indexed.
//   ids == nullptr: row i steps state i in place.
//   children != nullptr: the stepped copy goes to children[i] (branch); the
//   parent row is not written; a bad id gives a zero child.
// The bookkeeping of a self-play round folded into the step (step_compact): per row
// of game id, decision[id] += 1; a finished game's reward0[id] and nagari[id]; a
// status other than OK and "finished" counted in *bad; per warp, the ballot of its
// rows still running (keep[warp]), from which compact_scan_kernel and
// compact_scatter_kernel build the next id list in the same order.
struct RoundTail {
  int32_t* decision;
  float* reward0;
  bool* nagari;
  i64* bad;
  uint32_t* keep;        // [groups][stride]: per group and warp, the ballot of its rows
  const int32_t* m_dev;  // optional device-resident row count (at most m)
  int groups;            // 1: the running rows in order; 3: grouped by their next decision
  i64 stride;            // ceil(m / 32)
};

// Group of a running game's next decision for grouped compaction: 0 a primary play,
// 1 a pending floor choice, 2 a prompt (Go/Stop, Gukjin, Chongtong).  A warp of one
// group runs one branch of the rule code in the next round.
__device__ __forceinline__ int next_decision_group(const Game& g) {
  if (g.pend_active()) return 1;
  return decision_kind(g) == kDecPrimary ? 0 : 2;
}

__device__ __forceinline__ i64 device_rows(const int32_t* m_dev, i64 m) {
  if (!m_dev) return m;
  const i64 md = __ldg(m_dev);
  return md < 0 ? 0 : (md < m ? md : m);
}

// Rule path a row's step takes, for the block's partition of its rows: 0 a card play,
// 1 a bonus play, 2 a shake, bomb, grenade or bomb credit, 3 a floor choice, 4 a
// prompt answer, a finished row or an action outside the primary range, 5 no row.
__device__ __forceinline__ int step_path(const u64* row, u32 action, bool live) {
  if (!live) return 5;
  Game g;  // only the two words read below
  g.w[27] = row[27];
  g.w[29] = row[29];
  if (g.done()) return 4;
  if (g.pend_active()) return 3;
  if (action < 48u) return 0;
  if (action < 50u) return 1;
  if (action <= 122u) return 2;
  return 4;
}
constexpr int kStepPaths = 6;

// kPartition: a block's 128 rows are stepped in the order of their rule path (a
// stable counting sort through shared memory), so a warp runs mostly one path of the
// rules instead of every path its rows take (rows in random order with random legal
// actions: a warp of 32 almost always mixes card plays with a choice or a special
// play); each warp then writes the rows it stepped straight to their destinations.
// Without it (the self-play round tail, whose running list is already grouped by next
// decision) every warp steps its own 32 rows and the round's bookkeeping follows.
template <bool kPartition>
__global__ void __launch_bounds__(kBlock, CB_ENGINE_MIN_BLOCKS) step_kernel(
    u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids,
    const i64* __restrict__ actions, i64 m, u64* __restrict__ children,
    float* __restrict__ reward, bool* __restrict__ done, bool* __restrict__ nagari,
    int16_t* __restrict__ status, bool* __restrict__ committed, i64* __restrict__ events,
    RoundTail tail = RoundTail{}) {
  m = device_rows(tail.m_dev, m);
  if ((i64)blockIdx.x * kBlock >= m) return;  // past a device count: nothing to write
  WarpTile& t = my_tile();
  const int lane = threadIdx.x & 31;
  const i64 row = (i64)blockIdx.x * kBlock + threadIdx.x;
  const i64 src = lane_source(ids, row, m, n_states);
  gather_rows(t, states, src);
  const u32 action = src >= 0 ? torch_action(__ldg(actions + row)) : kNoAction;
  // The row this thread steps: its own, or with kPartition its place in path order.
  int mine = threadIdx.x;
  i64 msrc = src;
  u32 maction = action;
  if constexpr (kPartition) {
    __shared__ i64 src_s[kBlock];
    __shared__ u32 action_s[kBlock];
    __shared__ int16_t perm[kBlock];
    __shared__ int path_count[kWarpsPerBlock][kStepPaths];
    const int warp = threadIdx.x >> 5;
    src_s[threadIdx.x] = src;
    action_s[threadIdx.x] = action;
    const int path = step_path(t.rows[lane], action, src >= 0);
    int rank = 0;
#pragma unroll
    for (int c = 0; c < kStepPaths; ++c) {
      const unsigned b = __ballot_sync(kFull, path == c);
      if (lane == 0) path_count[warp][c] = __popc(b);
      if (path == c) rank = __popc(b & ((1u << lane) - 1u));
    }
    __syncthreads();  // every tile gathered, every warp's counts written
    int at = rank;
    for (int c = 0; c < path; ++c)
#pragma unroll
      for (int w = 0; w < kWarpsPerBlock; ++w) at += path_count[w][c];
    for (int w = 0; w < warp; ++w) at += path_count[w][path];
    perm[at] = static_cast<int16_t>(threadIdx.x);
    __syncthreads();
    mine = perm[threadIdx.x];
    msrc = src_s[mine];
    maction = action_s[mine];
  }
  WarpTile& mt = tile_of_block_row(mine);
  const int mr = mine & 31;
  const i64 mrow = (i64)blockIdx.x * kBlock + mine;
  Game g;
  load_game_row(mt, mr, g);
  StepOut out{static_cast<u32>(-1), 0, 1, 0, 0};
  i64 ev[kEventWords];
#pragma unroll
  for (int k = 0; k < (int)kEventWords; ++k) ev[k] = 0;
  if (msrc >= 0) {
    const EventBase before = event_base(g);
    out = step_game(g, maction);
    if (events && out.committed) event_words(before, g, ev);
  } else if (children) {
    for (int k = 0; k < kRowWords; ++k) g.w[k] = 0;
  }
  store_game_row(mt, mr, g);
  if constexpr (kPartition) {
    // This warp's 32 stepped rows, one 248-byte row per pass, to their destinations.
    __syncwarp();
    const i64 dst = children ? (mrow < m ? mrow : -1) : msrc;
    u64* base = children ? children : states;
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
      const int br = __shfl_sync(kFull, mine, r);
      const i64 d = __shfl_sync(kFull, dst, r);
      if (d >= 0 && lane < kRowWords)
        base[d * kRowWords + lane] = tile_of_block_row(br).rows[br & 31][lane];
    }
  } else {
    const i64 tile_base = (i64)blockIdx.x * kBlock + (threadIdx.x & ~31);
    if (children) store_tile(t, children, tile_base, m, row < m ? row : -1);
    else if (!ids) store_tile(t, states, tile_base, m, src);  // in place, rows in order
    else scatter_rows(t, states, src);
  }
  if (!kPartition && tail.keep) {  // ids are distinct (one row per game)
    const bool fin = src >= 0 && out.done != 0;
    if (src >= 0) {
      tail.decision[src] += 1;
      if (fin) {
        tail.reward0[src] = static_cast<float>(out.reward0);
        tail.nagari[src] = out.nagari != 0;
      }
      const u32 st = static_cast<u32>(out.status);
      if (st != kOk && st != kFinished) atomicAdd(reinterpret_cast<unsigned long long*>(tail.bad), 1ull);
    }
    const bool running = src >= 0 && !fin;
    const i64 w = ((i64)blockIdx.x * kBlock + (threadIdx.x & ~31)) >> 5;
    if (tail.groups == 1) {
      const unsigned mask = __ballot_sync(kFull, running);
      if (lane == 0 && w * 32 < m) tail.keep[w] = mask;
    } else {
      const int grp = running ? next_decision_group(g) : -1;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const unsigned mask = __ballot_sync(kFull, grp == q);
        if (lane == 0 && w * 32 < m) tail.keep[q * tail.stride + w] = mask;
      }
    }
  }
  if (mrow < m && reward) {  // internal callers may skip the per-row outputs
    reward[mrow] = static_cast<float>(out.reward0);
    done[mrow] = out.done != 0;
    nagari[mrow] = out.nagari != 0;
    status[mrow] = static_cast<int16_t>(static_cast<i32>(out.status));
    committed[mrow] = out.committed != 0;
    if (events) {
#pragma unroll
      for (int k = 0; k < (int)kEventWords; ++k) events[mrow * kEventWords + k] = ev[k];
    }
  }
}

// branch_indexed with identical children made once.  A child depends only on
// (parent row, action), so each warp takes kBranchEntries consecutive entries on its
// own (no block-wide barrier: while one warp runs the rule code, the others on the
// SM write children), finds the distinct (parent, action) pairs among them in a
// shared-memory hash keyed by the pair (numbered in order of first occurrence),
// steps the distinct pairs 32 per pass, and writes the child row and outputs of
// every entry from the stepped tile.  Entries with an invalid parent id share one
// zero child (status -1, done 1, as step_indexed reports it).
constexpr int kBranchWarps = 2;      // independent warps per block
#ifndef CB_BRANCH_MIN_BLOCKS
#define CB_BRANCH_MIN_BLOCKS 6
#endif
constexpr int kBranchEntries = 256;  // entries per warp
constexpr int kBranchPerLane = kBranchEntries / 32;
constexpr int kBranchHash = 2 * kBranchEntries;  // open addressing, load factor <= 1/2
constexpr unsigned long long kBranchEmpty = ~0ull;
constexpr unsigned long long kBranchInvalid = ~0ull - 1;  // every entry with a bad parent id

struct BranchWarpShared {
  u64 rows[32][kRowWords];          // stepped children of the current pass
  unsigned long long keys[kBranchHash];
  int16_t slot_u[kBranchHash];      // key -> its pair's index among the distinct ones
  int16_t uniq_of[kBranchEntries];  // entry -> pair index (-1 past m)
  int16_t head[kBranchEntries];     // pair -> its first entry
  float reward[32];                 // outputs of the current pass's pairs
  int16_t status[32];
  uint8_t flags[32];                // done | nagari << 1 | committed << 2
};

__global__ void __launch_bounds__(32 * kBranchWarps, CB_BRANCH_MIN_BLOCKS) branch_warp_kernel(
    const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids,
    const i64* __restrict__ actions, i64 m, u64* __restrict__ children,
    float* __restrict__ reward, bool* __restrict__ done, bool* __restrict__ nagari,
    int16_t* __restrict__ status, bool* __restrict__ committed) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  BranchWarpShared& sh = reinterpret_cast<BranchWarpShared*>(smem_raw)[warp];
  const i64 base = ((i64)blockIdx.x * kBranchWarps + warp) * kBranchEntries;
  if (base >= m) return;
  for (int k = lane; k < kBranchHash; k += 32) sh.keys[k] = kBranchEmpty;
  __syncwarp();
  const unsigned below = (1u << lane) - 1u;
  // Keys of the warp's entries, all loads in flight at once.
  unsigned long long key[kBranchPerLane];
#pragma unroll
  for (int j = 0; j < kBranchPerLane; ++j) {
    const i64 e = base + 32 * j + lane;
    const i64 src = lane_source(ids, e, m, n_states);
    const u32 act = e < m ? torch_action(__ldg(actions + e)) : kNoAction;
    key[j] = e >= m ? kBranchEmpty
                    : (src >= 0 ? (static_cast<unsigned long long>(src) << 16) | act : kBranchInvalid);
  }
  // Number the distinct keys in order of first occurrence.  Within one round of 32
  // entries equal keys elect one leader (match), so a key is inserted by one lane
  // only; keys of earlier rounds are found by a plain read.
  int distinct = 0;
#pragma unroll
  for (int j = 0; j < kBranchPerLane; ++j) {
    const unsigned long long k = key[j];
    const unsigned grp = __match_any_sync(kFull, k);
    const int leader = __ffs(grp) - 1;
    const bool live = k != kBranchEmpty;
    bool fresh = false;
    int h = -1;
    if (live && lane == leader) {
      h = static_cast<int>((k * 0x9E3779B97F4A7C15ull) >> 40) & (kBranchHash - 1);
      for (;;) {
        unsigned long long cur = sh.keys[h];
        if (cur == kBranchEmpty) {
          cur = atomicCAS(&sh.keys[h], kBranchEmpty, k);
          if (cur == kBranchEmpty) { fresh = true; break; }
        }
        if (cur == k) break;
        h = (h + 1) & (kBranchHash - 1);
      }
    }
    const unsigned fresh_ballot = __ballot_sync(kFull, fresh);
    int u = -1;
    if (fresh) {
      u = distinct + __popc(fresh_ballot & below);
      sh.slot_u[h] = static_cast<int16_t>(u);
      sh.head[u] = static_cast<int16_t>(32 * j + lane);
    } else if (live && lane == leader) {
      u = sh.slot_u[h];  // inserted in an earlier round
    }
    distinct += __popc(fresh_ballot);
    u = __shfl_sync(kFull, u, leader);
    sh.uniq_of[32 * j + lane] = static_cast<int16_t>(live ? u : -1);
    __syncwarp();  // this round's numbers are visible to the next round's reads
  }
  __syncwarp();
  const i64 rows_here = m - base < kBranchEntries ? m - base : kBranchEntries;
  // Full 256-entry groups made in one pass leave as row pairs: 496 contiguous bytes,
  // 31 vectors of 16 bytes, vector l of a pair holding words 2l and 2l + 1 -- the
  // same two word positions (and row of the pair) for lane l in every pair.
  const bool pairs = distinct <= 32 && rows_here == kBranchEntries &&
                     (reinterpret_cast<uintptr_t>(children) & 15u) == 0;
  const int w_a = 2 * lane, w_b = 2 * lane + 1;
  const int r_a = w_a >= kRowWords, r_b = w_b >= kRowWords;
  const int o_a = w_a - r_a * kRowWords, o_b = w_b - r_b * kRowWords;
#pragma unroll 1
  for (int first = 0; first < distinct; first += 32) {
    const int u = first + lane;
    const int e = u < distinct ? sh.head[u] : -1;
    const i64 src = e >= 0 ? lane_source(ids, base + e, m, n_states) : -1;
    // Rows of the pass: every valid lane of a branch group usually names one parent,
    // fetched once and replicated.
    {
      i64 id0 = -1;
      const unsigned have = __ballot_sync(kFull, src >= 0);
      if (have) id0 = __shfl_sync(kFull, src, __ffs(have) - 1);
      const bool one_parent = __all_sync(kFull, src < 0 || src == id0);
      if (one_parent && id0 >= 0) {
        const u64 w = lane < kRowWords ? __ldg(states + id0 * kRowWords + lane) : 0ull;
#pragma unroll 8
        for (int r = 0; r < 32; ++r)
          if (lane < kRowWords) sh.rows[r][lane] = w;
      } else {
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
          const i64 id = __shfl_sync(kFull, src, r);
          if (lane < kRowWords) sh.rows[r][lane] = id >= 0 ? __ldg(states + id * kRowWords + lane) : 0ull;
        }
      }
      __syncwarp();
    }
    Game g;
#pragma unroll
    for (int w = 0; w < kRowWords; ++w) g.w[w] = sh.rows[lane][w];
    __syncwarp();
    StepOut out{static_cast<u32>(-1), 0, 1, 0, 0};
    if (src >= 0) {
      out = step_game(g, torch_action(__ldg(actions + base + e)));
    } else {
      for (int w = 0; w < kRowWords; ++w) g.w[w] = 0;
    }
    zero_padding(g);
#pragma unroll
    for (int w = 0; w < kRowWords; ++w) sh.rows[lane][w] = g.w[w];
    sh.reward[lane] = static_cast<float>(out.reward0);
    sh.status[lane] = static_cast<int16_t>(static_cast<i32>(out.status));
    sh.flags[lane] = static_cast<uint8_t>((out.done != 0) | ((out.nagari != 0) << 1) |
                                          ((out.committed != 0) << 2));
    __syncwarp();
    if (pairs) {
      ulonglong2* dst = reinterpret_cast<ulonglong2*>(children + base * kRowWords);
#pragma unroll 4
      for (int p = 0; p < kBranchEntries / 2; ++p) {
        const int q0 = sh.uniq_of[2 * p], q1 = sh.uniq_of[2 * p + 1];
        if (lane < kRowWords) {
          const u64 a = sh.rows[r_a ? q1 : q0][o_a];
          const u64 b = sh.rows[r_b ? q1 : q0][o_b];
          __stcs(dst + p * kRowWords + lane, make_ulonglong2(a, b));
        }
      }
    } else {
#pragma unroll 4
      for (int r = 0; r < rows_here; ++r) {
        const int q = sh.uniq_of[r] - first;
        if (q >= 0 && q < 32 && lane < kRowWords)
          __stcs(children + (base + r) * kRowWords + lane, sh.rows[q][lane]);
      }
    }
#pragma unroll
    for (int j = 0; j < kBranchPerLane; ++j) {
      const int en = 32 * j + lane;
      const int q = sh.uniq_of[en] - first;
      if (en < rows_here && q >= 0 && q < 32) {
        const uint8_t f = sh.flags[q];
        reward[base + en] = sh.reward[q];
        status[base + en] = sh.status[q];
        done[base + en] = f & 1u;
        nagari[base + en] = (f >> 1) & 1u;
        committed[base + en] = (f >> 2) & 1u;
      }
    }
    __syncwarp();
  }
}

// Exclusive prefix over the warps' running counts (one block): offsets[q][w] for
// each group q (group q's rows follow every row of groups < q), and the total in
// *count.  The groups (at most kMaxGroups) are scanned together: every thread loads
// its consecutive warps' words of all groups at once, and one round of block
// barriers serves them all.
constexpr int kMaxGroups = 3;

__global__ void __launch_bounds__(1024) compact_scan_kernel(const uint32_t* __restrict__ keep,
                                                            i64 m, const int32_t* __restrict__ m_dev,
                                                            int32_t* __restrict__ offsets,
                                                            int32_t* __restrict__ count, int groups,
                                                            i64 stride) {
  __shared__ int32_t sums[kMaxGroups][32];
  const i64 warps = (device_rows(m_dev, m) + 31) / 32;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  const i64 per = (warps + blockDim.x - 1) / blockDim.x;  // consecutive warps per thread
  const i64 w0 = t * per;
  const i64 w1 = w0 + per < warps ? w0 + per : warps;
  // A thread's words move as 16-byte vectors when its whole span [w0, w0 + per) lies
  // in the arrays and starts 16-byte aligned (words past the row count read as zero;
  // their offsets are written but never read): a warp's loads and stores then touch a
  // quarter of the sectors the word-by-word loop does.
  const bool vec = per % 4 == 0 && stride % 4 == 0 && w0 < warps && w0 + per <= stride &&
                   (reinterpret_cast<uintptr_t>(keep) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(offsets) & 15u) == 0;
  int32_t mine[kMaxGroups] = {0, 0, 0};
  if (vec) {
    for (i64 w = w0; w < w0 + per; w += 4) {
#pragma unroll
      for (int q = 0; q < kMaxGroups; ++q) {
        if (q < groups) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(keep + q * stride + w));
          mine[q] += (w < warps ? __popc(v.x) : 0) + (w + 1 < warps ? __popc(v.y) : 0) +
                     (w + 2 < warps ? __popc(v.z) : 0) + (w + 3 < warps ? __popc(v.w) : 0);
        }
      }
    }
  } else {
    for (i64 w = w0; w < w1; ++w) {
#pragma unroll
      for (int q = 0; q < kMaxGroups; ++q)
        if (q < groups) mine[q] += __popc(__ldg(keep + q * stride + w));
    }
  }
  int32_t incl[kMaxGroups];
#pragma unroll
  for (int q = 0; q < kMaxGroups; ++q) incl[q] = mine[q];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int q = 0; q < kMaxGroups; ++q) {
      const int32_t v = __shfl_up_sync(kFull, incl[q], o);
      if (lane >= o) incl[q] += v;
    }
  }
  if (lane == 31) {
#pragma unroll
    for (int q = 0; q < kMaxGroups; ++q) sums[q][wid] = incl[q];
  }
  __syncthreads();
  if (wid < groups) {  // warp q scans group q's warp totals
    int32_t v = lane < nwarps ? sums[wid][lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(kFull, v, o);
      if (lane >= o) v += u;
    }
    sums[wid][lane] = v;  // inclusive over warps 0..lane
  }
  __syncthreads();
  int32_t run[kMaxGroups];
  int32_t base = 0;
#pragma unroll
  for (int q = 0; q < kMaxGroups; ++q) {
    if (q < groups) {
      run[q] = base + incl[q] - mine[q] + (wid > 0 ? sums[q][wid - 1] : 0);
      base += sums[q][31];
    } else {
      run[q] = 0;
    }
  }
  if (vec) {
    for (i64 w = w0; w < w0 + per; w += 4) {
#pragma unroll
      for (int q = 0; q < kMaxGroups; ++q) {
        if (q < groups) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(keep + q * stride + w));
          int4 o;
          o.x = run[q];
          o.y = o.x + (w < warps ? __popc(v.x) : 0);
          o.z = o.y + (w + 1 < warps ? __popc(v.y) : 0);
          o.w = o.z + (w + 2 < warps ? __popc(v.z) : 0);
          run[q] = o.w + (w + 3 < warps ? __popc(v.w) : 0);
          *reinterpret_cast<int4*>(offsets + q * stride + w) = o;
        }
      }
    }
  } else {
    for (i64 w = w0; w < w1; ++w) {
#pragma unroll
      for (int q = 0; q < kMaxGroups; ++q) {
        if (q < groups) {
          offsets[q * stride + w] = run[q];
          run[q] += __popc(__ldg(keep + q * stride + w));
        }
      }
    }
  }
  if (t == 0) *count = base;
}

// next_ids[offsets[q][w] + rank of the row among its warp's rows of group q] = ids[row]
// (the row itself without ids).
__global__ void __launch_bounds__(256) compact_scatter_kernel(const uint32_t* __restrict__ keep,
                                                              const int32_t* __restrict__ offsets,
                                                              const i64* __restrict__ ids, i64 m,
                                                              const int32_t* __restrict__ m_dev,
                                                              i64* __restrict__ next_ids, int groups,
                                                              i64 stride) {
  const i64 row = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= device_rows(m_dev, m)) return;
  const int lane = static_cast<int>(row & 31);
  for (int q = 0; q < groups; ++q) {
    const uint32_t mask = __ldg(keep + q * stride + (row >> 5));
    if ((mask >> lane) & 1u) {
      next_ids[__ldg(offsets + q * stride + (row >> 5)) + __popc(mask & ((1u << lane) - 1u))] =
          ids ? __ldg(ids + row) : row;
      return;
    }
  }
}

// A batch's running set at the deal: per row, zero decision count, reward and nagari,
// and ids[row] = spare[row] = row (so every entry of both id lists is a valid row);
// per warp, the ballot of its rows whose game the deal did not end (done byte 0);
// *bad = 0.  compact_scan_kernel and compact_scatter_kernel then list those rows.
__global__ void __launch_bounds__(256) running_flags_kernel(const uint8_t* __restrict__ states, i64 n,
                                                            i64* __restrict__ ids,
                                                            i64* __restrict__ spare,
                                                            uint32_t* __restrict__ keep,
                                                            int32_t* __restrict__ decision,
                                                            float* __restrict__ reward0,
                                                            bool* __restrict__ nagari,
                                                            i64* __restrict__ bad) {
  const i64 row = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  const bool running = row < n && __ldg(states + row * (kRowWords * 8) + kDoneByte) == 0;
  const unsigned mask = __ballot_sync(kFull, running);
  if (row < n) {
    ids[row] = row;
    if (spare) spare[row] = row;
    decision[row] = 0;
    reward0[row] = 0.0f;
    nagari[row] = false;
    if ((threadIdx.x & 31) == 0) keep[row >> 5] = mask;
  }
  if (row == 0) *bad = 0;
}

__global__ void __launch_bounds__(kBlock) clone_kernel(const u64* __restrict__ states, i64 n_states,
                                                       const i64* __restrict__ ids, i64 m,
                                                       u64* __restrict__ children) {
  WarpTile& t = my_tile();
  const i64 row = (i64)blockIdx.x * kBlock + threadIdx.x;
  gather_rows(t, states, lane_source(ids, row, m, n_states));
  store_tile(t, children, (i64)blockIdx.x * kBlock + (threadIdx.x & ~31), m, row < m ? row : -1);
}

__global__ void hands_kernel(const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids,
                             i64 m, i64* __restrict__ hands) {
  const i64 row = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= m) return;
  const i64 id = lane_source(ids, row, m, n_states);
  const u64 h0 = id >= 0 ? __ldg(states + id * kRowWords + 0) : 0;
  const u64 h1 = id >= 0 ? __ldg(states + id * kRowWords + 1) : 0;
  reinterpret_cast<longlong2*>(hands)[row] = make_longlong2((long long)h0, (long long)h1);
}

__global__ void stock_kernel(const u64* __restrict__ states, i64 n_states, const i64* __restrict__ ids,
                             i64 m, i64* __restrict__ out) {
  const i64 row = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= m) return;
  const i64 id = lane_source(ids, row, m, n_states);
  u64 packed = ~0ull;
  if (id >= 0) {
    Game g;
    g.w[3] = __ldg(states + id * kRowWords + 3);
    g.w[6] = __ldg(states + id * kRowWords + 6);
    packed = stock_preview(g);
  }
  out[row] = static_cast<i64>(packed);
}

__global__ void start_kernel(const u64* __restrict__ states, i64 n, i64* __restrict__ out) {
  const i64 row = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  Game g;
  const u64* s = states + row * kRowWords;
  g.w[0] = __ldg(s + 0);
  g.w[1] = __ldg(s + 1);
  g.w[2] = __ldg(s + 2);
  g.w[4] = __ldg(s + 4);
  g.w[5] = __ldg(s + 5);
  g.w[9] = __ldg(s + 9);
  g.w[10] = __ldg(s + 10);
  g.w[11] = __ldg(s + 11);
  g.w[18] = __ldg(s + 18);
  g.w[19] = __ldg(s + 19);
  start_words(g, out + row * kStartWords);
}

// ---- launch helpers ------------------------------------------------------------

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

inline unsigned blocks_for(i64 n, int per_block) { return static_cast<unsigned>((n + per_block - 1) / per_block); }

}  // namespace

extern "C" {

int cugo_b200_abi_version(void) { return CUGO_B200_ABI_VERSION; }
int64_t cugo_b200_state_bytes(void) { return kRowBytes; }
int64_t cugo_b200_feature_count(void) { return kFeatures; }
int64_t cugo_b200_action_count(void) { return kActions; }
int64_t cugo_b200_primary_action_count(void) { return kPrimaryActions; }
int64_t cugo_b200_choice_action_begin(void) { return kChoiceBegin; }
int64_t cugo_b200_event_words(void) { return kEventWords; }
int64_t cugo_b200_start_words(void) { return kStartWords; }
int64_t cugo_b200_status_ok(void) { return kOk; }

int cugo_b200_create_indexed(const int64_t* index, int64_t seed_base, int64_t n, uint8_t* states,
                             cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!index || !states))) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8)) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  create_kernel<<<blocks_for(n, kBlock), kBlock, 0, stream>>>(
      nullptr, nullptr, n, reinterpret_cast<u64*>(states), index, seed_base);
  return launch_status();
}

int64_t cugo_b200_running_init_scratch(int64_t n) { return n < 0 ? -1 : 2 * ((n + 31) / 32); }

int cugo_b200_running_init(const uint8_t* states, int64_t n, int64_t* ids, int64_t* spare_ids,
                           int32_t* count,
                           int32_t* decision, float* reward0, bool* nagari, int64_t* bad,
                           int32_t* scratch, int64_t scratch_len, cudaStream_t stream) {
  if (n < 0 || n > INT32_MAX) return CUGO_B200_ERR_ARG;
  if (!count || !bad || !scratch) return CUGO_B200_ERR_ARG;
  if (n > 0 && (!states || !ids || !decision || !reward0 || !nagari)) return CUGO_B200_ERR_ARG;
  const i64 words = (n + 31) / 32;
  if (scratch_len < 2 * words) return CUGO_B200_ERR_CAPACITY;
  uint32_t* keep = reinterpret_cast<uint32_t*>(scratch);
  int32_t* offsets = scratch + words;
  running_flags_kernel<<<static_cast<unsigned>(n > 0 ? (n + 255) / 256 : 1), 256, 0, stream>>>(
      states, n, ids, spare_ids, keep, decision, reward0, nagari, bad);
  compact_scan_kernel<<<1, 1024, 0, stream>>>(keep, n, nullptr, offsets, count, 1, words);
  if (n > 0)
    compact_scatter_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        keep, offsets, nullptr, n, nullptr, ids, 1, words);
  return launch_status();
}

int cugo_b200_create(const int64_t* seeds, const int64_t* first_players, int64_t n,
                     uint8_t* states, cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!seeds || !first_players || !states))) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8)) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  create_kernel<<<blocks_for(n, kBlock), kBlock, 0, stream>>>(seeds, first_players, n,
                                                             reinterpret_cast<u64*>(states));
  return launch_status();
}

static int observe_common(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                          int64_t m, float* features, bool* legal, uint8_t* players, bool* done,
                          int16_t* status, cudaStream_t stream) {
  if (n_states < 0 || m < 0) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!features || !legal || !players || !done || !status)) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(features, 16) || !aligned(legal, 4)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  observe_kernel<float><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m, features, (i64)kFeatures, 0, legal,
      players, done, status);
  return launch_status();
}

int cugo_b200_observe_indexed_bf16(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                   int64_t m, void* features, bool* legal, uint8_t* players,
                                   bool* done, int16_t* status, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && !env_ids)) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!features || !legal || !players || !done || !status)) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(features, 16) || !aligned(legal, 4)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  observe_kernel<__nv_bfloat16><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m,
      static_cast<__nv_bfloat16*>(features), (i64)kFeatures, 0, legal, players, done, status);
  return launch_status();
}

int cugo_b200_observe_indexed_bf16_bits(const uint8_t* states, int64_t n_states,
                                        const int64_t* env_ids, int64_t m, void* features,
                                        uint64_t* legal_bits, uint8_t* players, bool* done,
                                        int16_t* status, const int32_t* m_dev,
                                        cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && !env_ids)) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!features || !legal_bits || !players || !done || !status)) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(features, 16) || !aligned(legal_bits, 8))
    return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  observe_kernel<__nv_bfloat16><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m,
      static_cast<__nv_bfloat16*>(features), (i64)kFeatures, 0, nullptr, players, done, status, 0,
      reinterpret_cast<u64*>(legal_bits), m_dev);
  return launch_status();
}

int cugo_b200_observe_query_bf16(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                 int64_t m, void* query, int64_t ldq, bool* legal,
                                 uint8_t* players, bool* done, int16_t* status,
                                 cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && !env_ids)) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!query || !legal || !players || !done || !status)) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (ldq < (int64_t)(kFeatures + kActions)) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(query, 16) || ldq % 8 || !aligned(legal, 4))
    return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  // Legal columns fill the row up to ldq (zeros past action 178), in groups of 8.
  observe_kernel<__nv_bfloat16><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m,
      static_cast<__nv_bfloat16*>(query), ldq, static_cast<int>(ldq - kFeatures), legal, players,
      done, status);
  return launch_status();
}

int cugo_b200_observe_critic_bf16(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                  int64_t m, void* critic_in, int64_t ldc, uint8_t* players,
                                  bool* done, int16_t* status, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && !env_ids)) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!critic_in || !players || !done || !status)) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (ldc < (int64_t)(kFeatures + 50)) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(critic_in, 16) || ldc % 8) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  observe_kernel<__nv_bfloat16><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m,
      static_cast<__nv_bfloat16*>(critic_in), ldc, static_cast<int>(ldc - kFeatures), nullptr,
      players, done, status, 1);
  return launch_status();
}

int cugo_b200_observe(const uint8_t* states, int64_t n, float* features, bool* legal,
                      uint8_t* players, bool* done, int16_t* status, cudaStream_t stream) {
  return observe_common(states, n, nullptr, n, features, legal, players, done, status, stream);
}

int cugo_b200_observe_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                              int64_t m, float* features, bool* legal, uint8_t* players,
                              bool* done, int16_t* status, cudaStream_t stream) {
  if (m > 0 && !env_ids) return CUGO_B200_ERR_ARG;
  return observe_common(states, n_states, env_ids, m, features, legal, players, done, status,
                        stream);
}

}  // extern "C"

// In-place step of rows 0..n-1 with actions[i] and no per-row outputs, for the
// drivers in other translation units (not part of the C ABI).
int cb_step_in_place(uint8_t* states, int64_t n, const int64_t* actions, cudaStream_t stream) {
  if (n <= 0) return CUGO_B200_OK;
  step_kernel<true><<<blocks_for(n, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<u64*>(states), n, nullptr, actions, n, nullptr, nullptr, nullptr, nullptr,
      nullptr, nullptr, nullptr);
  return launch_status();
}

extern "C" {

static int step_common(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                       const int64_t* actions, int64_t m, uint8_t* children, float* reward,
                       bool* done, bool* nagari, int16_t* status, bool* committed,
                       int64_t* events, cudaStream_t stream) {
  if (n_states < 0 || m < 0) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!actions || !reward || !done || !nagari || !status || !committed))
    return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(children, 8) || !aligned(events, 8)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  step_kernel<true><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<u64*>(states), n_states, env_ids, actions, m,
      reinterpret_cast<u64*>(children), reward, done, nagari, status, committed, events);
  return launch_status();
}

int cugo_b200_step(uint8_t* states, int64_t n, const int64_t* actions, float* reward, bool* done,
                   bool* nagari, int16_t* status, bool* committed, cudaStream_t stream) {
  return step_common(states, n, nullptr, actions, n, nullptr, reward, done, nagari, status,
                     committed, nullptr, stream);
}

int cugo_b200_step_indexed(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                           const int64_t* actions, int64_t m, float* reward, bool* done,
                           bool* nagari, int16_t* status, bool* committed, cudaStream_t stream) {
  if (m > 0 && !env_ids) return CUGO_B200_ERR_ARG;
  return step_common(states, n_states, env_ids, actions, m, nullptr, reward, done, nagari, status,
                     committed, nullptr, stream);
}

static int step_compact_common(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                               const int64_t* actions, int64_t m, int32_t* decision,
                               float* reward0, bool* nagari, int64_t* bad, int64_t* next_ids,
                               int32_t* next_count, int32_t* scratch, const int32_t* m_dev,
                               int groups, cudaStream_t stream) {
  if (n_states < 0 || m < 0) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!env_ids || !actions || !decision || !reward0 || !nagari || !bad || !next_ids ||
                !next_count || !scratch))
    return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(scratch, 4)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) {
    cudaMemsetAsync(next_count, 0, sizeof(int32_t), stream);
    return launch_status();
  }
  const i64 warps = (m + 31) / 32;  // capacity; the kernels use the device count
  uint32_t* keep = reinterpret_cast<uint32_t*>(scratch);
  int32_t* offsets = scratch + groups * warps;
  if (m_dev == next_count) return CUGO_B200_ERR_ARG;  // the count is rewritten mid-call
  RoundTail tail{decision, reward0, nagari, bad, keep, m_dev, groups, warps};
  step_kernel<false><<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<u64*>(states), n_states, env_ids, actions, m, nullptr, nullptr, nullptr,
      nullptr, nullptr, nullptr, nullptr, tail);
  compact_scan_kernel<<<1, 1024, 0, stream>>>(keep, m, m_dev, offsets, next_count, groups, warps);
  compact_scatter_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, stream>>>(
      keep, offsets, env_ids, m, m_dev, next_ids, groups, warps);
  return launch_status();
}

int cugo_b200_step_compact(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                           const int64_t* actions, int64_t m, int32_t* decision, float* reward0,
                           bool* nagari, int64_t* bad, int64_t* next_ids, int32_t* next_count,
                           int32_t* scratch, const int32_t* m_dev, cudaStream_t stream) {
  return step_compact_common(states, n_states, env_ids, actions, m, decision, reward0, nagari, bad,
                             next_ids, next_count, scratch, m_dev, 1, stream);
}

int cugo_b200_step_compact_grouped(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                   const int64_t* actions, int64_t m, int32_t* decision,
                                   float* reward0, bool* nagari, int64_t* bad, int64_t* next_ids,
                                   int32_t* next_count, int32_t* scratch, const int32_t* m_dev,
                                   cudaStream_t stream) {
  return step_compact_common(states, n_states, env_ids, actions, m, decision, reward0, nagari, bad,
                             next_ids, next_count, scratch, m_dev, 3, stream);
}

int cugo_b200_step_events_indexed(uint8_t* states, int64_t n_states, const int64_t* env_ids,
                                  const int64_t* actions, int64_t m, float* reward, bool* done,
                                  bool* nagari, int16_t* status, bool* committed, int64_t* events,
                                  cudaStream_t stream) {
  if (m > 0 && (!env_ids || !events)) return CUGO_B200_ERR_ARG;
  return step_common(states, n_states, env_ids, actions, m, nullptr, reward, done, nagari, status,
                     committed, events, stream);
}

int cugo_b200_branch_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                             const int64_t* actions, int64_t m, uint8_t* children, float* reward,
                             bool* done, bool* nagari, int16_t* status, bool* committed,
                             cudaStream_t stream) {
  if (n_states < 0 || m < 0) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!env_ids || !children || !actions || !reward || !done || !nagari || !status ||
                !committed))
    return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(children, 8)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  constexpr size_t smem = kBranchWarps * sizeof(BranchWarpShared);
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(branch_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    configured = true;
  }
  branch_warp_kernel<<<blocks_for(m, kBranchWarps * kBranchEntries), 32 * kBranchWarps, smem,
                       stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, actions, m,
      reinterpret_cast<u64*>(children), reward, done, nagari, status, committed);
  return launch_status();
}

int cugo_b200_clone_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, uint8_t* children, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && (!env_ids || !children))) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(children, 8)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  clone_kernel<<<blocks_for(m, kBlock), kBlock, 0, stream>>>(
      reinterpret_cast<const u64*>(states), n_states, env_ids, m, reinterpret_cast<u64*>(children));
  return launch_status();
}

int cugo_b200_hands_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, int64_t* hands, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && (!env_ids || !hands))) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8) || !aligned(hands, 16)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  hands_kernel<<<blocks_for(m, 256), 256, 0, stream>>>(reinterpret_cast<const u64*>(states), n_states,
                                                       env_ids, m, hands);
  return launch_status();
}

int cugo_b200_stock_indexed(const uint8_t* states, int64_t n_states, const int64_t* env_ids,
                            int64_t m, int64_t* stock, cudaStream_t stream) {
  if (n_states < 0 || m < 0 || (m > 0 && (!env_ids || !stock))) return CUGO_B200_ERR_ARG;
  if (m > 0 && n_states > 0 && !states) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8)) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  stock_kernel<<<blocks_for(m, 256), 256, 0, stream>>>(reinterpret_cast<const u64*>(states), n_states,
                                                       env_ids, m, stock);
  return launch_status();
}

int cugo_b200_start(const uint8_t* states, int64_t n, int64_t* out, cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!states || !out))) return CUGO_B200_ERR_ARG;
  if (!aligned(states, 8)) return CUGO_B200_ERR_ALIGN;
  if (n == 0) return CUGO_B200_OK;
  start_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(reinterpret_cast<const u64*>(states), n, out);
  return launch_status();
}

}  // extern "C"
