// Oracle harness (TEST INFRASTRUCTURE ONLY): a C ABI over the reference's own
// header-only engine, compiled from the sources where they lie
// (<reference>/include/cugo/**, see oracle/Makefile) into oracle/_ref/.
//
// Every entry point runs the reference functions unchanged:
//   create            -> make_torch_env50                (cugo/game/torch50.h:231-236)
//   observe           -> make_torch_packet50 + encode_torch_packet50
//                        (torch50.h:245-296, 334-470), the per-row body of
//                        observe_kernel (python/csrc/torch50_ext.cu:125-141)
//   step / events     -> torch_step50 / torch_step_event50 + pack_torch_event50
//                        (torch50.h:491-540, 668-707; torch50_ext.cu:161-178, 299-334)
//   start, hands, stock -> pack_torch_start50, the hands/stock kernels' bodies
//                        (torch50.h:684-698; torch50_ext.cu:388-435)
//   rollout_random    -> the seeded random-legal driver of oracle/driver.h
// Rows are written in canonical form: every field at its TorchEnv50 offset and
// all padding bytes zero, so rows compare byte for byte.
#include <cstdint>
#include <cstring>
#include <cstddef>
#include <thread>
#include <vector>
#include <algorithm>

#include "cugo/game/torch50.h"
#include "driver.h"

using namespace cugo::game;
namespace core = cugo::core;

namespace {

static_assert(sizeof(TorchEnv50) == 248, "TorchEnv50 layout");

template <typename T>
void put(uint8_t* out, size_t off, const T& v) { std::memcpy(out + off, &v, sizeof(T)); }

// Field-wise copy into a zeroed row (padding bytes stay zero).
void canonical_row(const TorchEnv50& e, uint8_t* out) {
  std::memset(out, 0, sizeof(TorchEnv50));
  const TurnState50& t = e.game.special.game.turn;
#define T(f) put(out, offsetof(TorchEnv50, game.special.game.turn.f), t.f)
  T(hand0); T(hand1); T(floor); T(stock); T(captured0); T(captured1); T(rng_state);
  T(pending_bonus_mask); T(ppuk_months); T(ppuk_owner1_months); T(bonus2_ppuk_months);
  T(bonus3_ppuk_months); T(turn_index); T(actor); T(phase); T(pending_played);
  T(pending_drawn); T(mission_cards); T(neutral_ppuk_months);
#undef T
  const GameState50& g = e.game.special.game;
#define G(f) put(out, offsetof(TorchEnv50, game.special.game.f), g.f)
  G(go_count0); G(go_count1); G(last_go_base_score0); G(last_go_base_score1);
  G(decision_actor); G(winner); G(gukjin_decision);
#undef G
  const SpecialGameState50& s = e.game.special;
#define S(f) put(out, offsetof(TorchEnv50, game.special.f), s.f)
  S(shaken0); S(shaken1); S(bombs0); S(bombs1); S(credits0); S(credits1); S(shaken4_0); S(shaken4_1);
#undef S
  const TerminalGameState50& m = e.game;
#define M(f) put(out, offsetof(TorchEnv50, game.f), m.f)
  M(ppuk_count0); M(ppuk_count1); M(ppuk_streak0); M(ppuk_streak1); M(pending_chongtong_actor);
  M(pending_chongtong_months); M(terminal_winner); M(terminal_reason); M(terminal_points);
  M(side_points0); M(round_multiplier); M(mission_type); M(mission_multiplier);
  M(mission_multi0); M(mission_multi1); M(held0); M(held1); M(revealed0); M(revealed1);
#undef M
  const PostChancePending50& p = e.pending;
#define P(f) put(out, offsetof(TorchEnv50, pending.f), p.f)
  P(action.kind); P(action.card); P(action.month); P(action.resolve_choices.played_match);
  P(action.resolve_choices.drawn_match); P(action.pi_selection.cards); P(selected_pi);
  P(primary_action); P(actor); P(active);
#undef P
#define E(f) put(out, offsetof(TorchEnv50, f), e.f)
  E(primary_actions); E(choice_actions); E(resolve_choices); E(pi_choices);
  E(bonus_actions); E(special_actions); E(go_actions); E(status); E(done); E(nagari);
#undef E
}

TorchEnv50 load_row(const uint8_t* row) {
  TorchEnv50 e;
  std::memcpy(&e, row, sizeof(e));
  return e;
}

template <typename F>
void parallel_rows(int64_t n, int threads, F&& fn) {
  if (n <= 0) return;
  if (threads <= 1 || n < 64) {
    fn(int64_t{0}, n);
    return;
  }
  const int64_t workers = std::min<int64_t>(threads, (n + 63) / 64);
  const int64_t chunk = (n + workers - 1) / workers;
  std::vector<std::thread> pool;
  for (int64_t w = 0; w < workers; ++w) {
    const int64_t lo = w * chunk, hi = std::min<int64_t>(n, lo + chunk);
    if (lo >= hi) break;
    pool.emplace_back([&fn, lo, hi] { fn(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

void observe_one(const TorchEnv50& env, float* features, uint8_t* legal,
                 uint8_t* player, uint8_t* done, int16_t* status) {
  const TorchPacket50 packet = make_torch_packet50(env);
  encode_torch_packet50(packet, features);
  for (uint16_t a = 0; a < kTorch50ActionCount; ++a)
    legal[a] = has_torch_action50(packet.legal_actions, a) ? 1 : 0;
  *player = packet.decision_player;
  *done = env.done != 0;
  *status = static_cast<int16_t>(packet.status);
}

uint16_t torch_action(int64_t raw) {
  return raw >= 0 && raw < kTorch50ActionCount ? static_cast<uint16_t>(raw)
                                               : kInvalidTorch50Action;
}

}  // namespace

extern "C" {

int cugo_ref_state_bytes() { return static_cast<int>(sizeof(TorchEnv50)); }

void cugo_ref_canonicalize(uint8_t* rows, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const TorchEnv50 e = load_row(rows + i * 248);
    canonical_row(e, rows + i * 248);
  }
}

void cugo_ref_create(const int64_t* seeds, const int64_t* first, int64_t n,
                     uint8_t* rows, int threads) {
  parallel_rows(n, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      const TorchEnv50 e = make_torch_env50(static_cast<uint64_t>(seeds[i]),
                                            static_cast<uint8_t>(first[i] & 1));
      canonical_row(e, rows + i * 248);
    }
  });
}

void cugo_ref_observe(const uint8_t* rows, int64_t n, float* features, uint8_t* legal,
                      uint8_t* player, uint8_t* done, int16_t* status, int threads) {
  parallel_rows(n, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      observe_one(load_row(rows + i * 248), features + i * kTorch50FeatureCount,
                  legal + i * kTorch50ActionCount, player + i, done + i, status + i);
    }
  });
}

// In-place step of every row; events (nullable) receives 9 words per row.
void cugo_ref_step(uint8_t* rows, const int64_t* actions, int64_t n, float* reward,
                   uint8_t* done, uint8_t* nagari, int16_t* status, uint8_t* committed,
                   int64_t* events, int threads) {
  parallel_rows(n, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      TorchEnv50 e = load_row(rows + i * 248);
      TorchEvent50 ev{};
      const TorchStepResult50 r = torch_step_event50(e, torch_action(actions[i]), ev);
      reward[i] = static_cast<float>(r.reward0);
      done[i] = r.done != 0;
      nagari[i] = r.nagari != 0;
      status[i] = static_cast<int16_t>(r.status);
      committed[i] = r.primary_committed != 0;
      if (events != nullptr) pack_torch_event50(ev, events + i * kTorch50EventWords);
      canonical_row(e, rows + i * 248);
    }
  });
}

void cugo_ref_start(const uint8_t* rows, int64_t n, int64_t* out) {
  for (int64_t i = 0; i < n; ++i)
    pack_torch_start50(load_row(rows + i * 248), out + i * kTorch50StartWords);
}

void cugo_ref_hands(const uint8_t* rows, int64_t n, int64_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const TorchEnv50 e = load_row(rows + i * 248);
    out[2 * i] = static_cast<int64_t>(e.game.special.game.turn.hand0);
    out[2 * i + 1] = static_cast<int64_t>(e.game.special.game.turn.hand1);
  }
}

void cugo_ref_stock(const uint8_t* rows, int64_t n, int64_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const TorchEnv50 e = load_row(rows + i * 248);
    core::CardMask remaining = e.game.special.game.turn.stock;
    uint64_t rng = e.game.special.game.turn.rng_state;
    uint64_t packed = ~0ull;
    for (int k = 0; k < 8; ++k) {
      const core::CardId card = draw_stock_card(remaining, rng);
      if (!core::is_standard_card(card)) break;
      packed &= ~(0xFFull << (8 * k));
      packed |= static_cast<uint64_t>(card) << (8 * k);
    }
    out[i] = static_cast<int64_t>(packed);
  }
}

// Settlement summary of a finished row: final_points, reward0 and the multipliers.
// out[0..9] = status, reason, winner, final_points, go_count, go_multiplier,
//             bomb_shake_multiplier, bak_multiplier, mission_multiplier, side_points0
void cugo_ref_settle(const uint8_t* row, int64_t* out) {
  const TorchEnv50 e = load_row(row);
  const Settlement50 s = settle_terminal50(e.game);
  out[0] = static_cast<int64_t>(s.status);
  out[1] = static_cast<int64_t>(s.reason);
  out[2] = s.winner;
  out[3] = static_cast<int64_t>(s.final_points);
  out[4] = s.winner_go_count;
  out[5] = static_cast<int64_t>(s.go_multiplier);
  out[6] = static_cast<int64_t>(s.bomb_shake_multiplier);
  out[7] = static_cast<int64_t>(s.bak_multiplier);
  out[8] = static_cast<int64_t>(s.mission_multiplier);
  out[9] = s.side_points0;
}

// Seeded random-legal rollouts of games game0 .. game0+n-1 (oracle/driver.h).
// Per game: final canonical row, reward0, decisions taken, committed events,
// FNV-1a event hash, and the last step status.
void cugo_ref_rollout_random(int64_t game0, int64_t n, int64_t seed_base, int max_decisions,
                             uint32_t stream, uint8_t* final_rows, int64_t* reward0,
                             int32_t* decisions, int32_t* events, uint64_t* hashes,
                             int16_t* last_status, int threads) {
  parallel_rows(n, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t k = lo; k < hi; ++k) {
      const uint64_t game = static_cast<uint64_t>(game0 + k);
      const uint64_t seed = static_cast<uint64_t>(seed_base) + game;
      TorchEnv50 env = make_torch_env50(seed, static_cast<uint8_t>(game & 1u));
      int64_t start[kTorch50StartWords];
      pack_torch_start50(env, start);
      uint64_t h = oracle_fnv_words(ORACLE_FNV_OFFSET, start, kTorch50StartWords);
      int32_t d = 0, ev_count = 0;
      int16_t st = 0;
      int64_t rew = 0;
      while (env.done == 0 && d < max_decisions) {
        const TorchPacket50 packet = make_torch_packet50(env);
        uint8_t legal[kTorch50ActionCount];
        for (uint16_t a = 0; a < kTorch50ActionCount; ++a)
          legal[a] = has_torch_action50(packet.legal_actions, a) ? 1 : 0;
        const uint32_t r0 = oracle_driver_word(game, static_cast<uint32_t>(d), stream, seed);
        const int pick = oracle_pick_legal(legal, kTorch50ActionCount, r0);
        if (pick < 0) { st = -2; break; }
        TorchEvent50 e{};
        const TorchStepResult50 r = torch_step_event50(env, static_cast<uint16_t>(pick), e);
        ++d;
        st = static_cast<int16_t>(r.status);
        rew = r.reward0;
        if (r.status != ActionStatus50::kOk) break;
        if (r.primary_committed) {
          int64_t words[kTorch50EventWords];
          pack_torch_event50(e, words);
          h = oracle_fnv_words(h, words, kTorch50EventWords);
          ++ev_count;
        }
      }
      canonical_row(env, final_rows + k * 248);
      reward0[k] = rew;
      decisions[k] = d;
      events[k] = ev_count;
      hashes[k] = h;
      last_status[k] = st;
    }
  });
}

// Branching roots (config 2): game r advanced by k_r random-legal decisions,
// k_r = floor(r0 * 21 / 2^32) with r0 from (game r, decision 0xFFFF, stream 2),
// stopping before a decision that would end the game.
void cugo_ref_branch_roots(int64_t n_roots, int64_t seed_base, uint8_t* rows, int threads) {
  parallel_rows(n_roots, threads, [&](int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; ++r) {
      const uint64_t seed = static_cast<uint64_t>(seed_base + r);
      TorchEnv50 env = make_torch_env50(seed, static_cast<uint8_t>(r & 1));
      const uint32_t k = static_cast<uint32_t>(
          (static_cast<uint64_t>(oracle_driver_word(static_cast<uint64_t>(r), 0xffffu, 2u, seed)) * 21u) >> 32);
      for (uint32_t d = 0; d < k && env.done == 0; ++d) {
        const TorchPacket50 packet = make_torch_packet50(env);
        uint8_t legal[kTorch50ActionCount];
        for (uint16_t a = 0; a < kTorch50ActionCount; ++a)
          legal[a] = has_torch_action50(packet.legal_actions, a) ? 1 : 0;
        const int pick = oracle_pick_legal(legal, kTorch50ActionCount,
                                           oracle_driver_word(static_cast<uint64_t>(r), d, 0u, seed));
        if (pick < 0) break;
        TorchEnv50 next = env;
        torch_step50(next, static_cast<uint16_t>(pick));
        if (next.done != 0) break;
        env = next;
      }
      canonical_row(env, rows + r * 248);
    }
  });
}

// Branch i = r * per_root + b of config 2: env id r and the legal action of root r
// drawn with counter {r, b, 0, 1} (-1 when the root has none).
void cugo_ref_branch_actions(const uint8_t* roots, int64_t n_roots, int64_t per_root,
                             int64_t seed_base, int64_t* ids, int64_t* actions) {
  for (int64_t r = 0; r < n_roots; ++r) {
    const TorchEnv50 env = load_row(roots + r * 248);
    const TorchPacket50 packet = make_torch_packet50(env);
    uint8_t legal[kTorch50ActionCount];
    for (uint16_t a = 0; a < kTorch50ActionCount; ++a)
      legal[a] = has_torch_action50(packet.legal_actions, a) ? 1 : 0;
    const uint64_t seed = static_cast<uint64_t>(seed_base + r);
    for (int64_t b = 0; b < per_root; ++b) {
      const uint64_t ctr = static_cast<uint64_t>(r) | (static_cast<uint64_t>(b) << 32);
      const int pick = oracle_pick_legal(legal, kTorch50ActionCount,
                                         oracle_driver_word(ctr, 0u, 1u, seed));
      ids[r * per_root + b] = r;
      actions[r * per_root + b] = pick;
    }
  }
}

uint32_t cugo_ref_philox_word(uint64_t game, uint32_t decision, uint32_t stream, uint64_t seed) {
  return oracle_driver_word(game, decision, stream, seed);
}

}  // extern "C"
