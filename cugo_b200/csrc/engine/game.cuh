// One game's state as 31 little-endian 64-bit words: the exact byte image of the
// reference's 248-byte TorchEnv50 row (cugo/game/torch50.h:108-121, offsets
// measured with offsetof; the Python callers read words 0,1,3,6,20..23 of a row,
// cugo_ppo50.py:109-146).  Keeping the row as packed words lets a thread hold a
// whole game in ~62 registers and mutate it in place; every accessor uses a
// constant word index so nothing spills to local memory by indexing.
//
// Padding bytes are always written as zero.
#pragma once

#include "cards.cuh"

namespace cb {

constexpr int kRowBytes = 248;
constexpr int kDoneByte = 239;  // TorchEnv50::done (word 29, bits 56..63)
constexpr int kRowWords = 31;

// Decision kinds as the policy sees them (cugo/game/policy50.h:36-42,
// postchance50.h:15-20).
enum Decision : u32 {
  kDecNone = 0,
  kDecPrimary = 1,
  kDecGoStop = 2,
  kDecChongtong = 3,
  kDecFloorPlayed = 4,
  kDecFloorDrawn = 5,
  kDecPiCard = 6,
  kDecGukjin = 7,
};

// Action kinds stored in the pending record (cugo/game/rollout50.h:18-31).
enum ActKind : u32 {
  kActPlay = 0,
  kActBonus = 1,
  kActShake = 2,
  kActBomb = 3,
  kActGrenade = 4,
  kActCredit = 5,
  kActGo = 6,
  kActStop = 7,
  kActChongWin = 8,
  kActChongGo = 9,
  kActGukjinPi = 10,
  kActGukjinAnimal = 11,
};

// Step status codes (cugo/game/rollout50.h:33-44).
enum Status : u32 {
  kOk = 0,
  kWrongPhase = 1,
  kInvalidAction = 2,
  kNotLegal = 3,
  kStockEmpty = 4,
  kChoiceRequired = 5,
  kInvalidChoice = 6,
  kPiRequired = 7,
  kInvalidPi = 8,
  kFinished = 9,
};

// Why a game ended (cugo/game/terminal50.h:44-51).
enum EndReason : u32 {
  kEndNone = 0,
  kEndStop = 1,
  kEndDealtChongtong = 2,
  kEndFloorChongtong = 3,
  kEndBonusChongtong = 4,
  kEndThreePpuk = 5,
};

// Turn phases (cugo/game/turn50.h:39-43).
enum Phase : u32 { kPhasePlay = 0, kPhaseDraw = 1, kPhaseResolve = 2 };

constexpr u32 kNobody = 0xffu;

// Extra flags kept in the high bits of the ppuk-owner word
// (cugo/game/gukjin_state.h:336-347): bit 12+p = player p scores Gukjin as a
// double pi, bit 14+p = player p's Gukjin role is locked.
constexpr u32 kGukjinPiFlag0 = 1u << 12;
constexpr u32 kGukjinLockFlag0 = 1u << 14;
CB_HD u32 gukjin_pi_flag(u32 p) { return kGukjinPiFlag0 << (p & 1u); }
CB_HD u32 gukjin_lock_flag(u32 p) { return kGukjinLockFlag0 << (p & 1u); }

struct Game {
  u64 w[kRowWords];

  // -- generic sub-word access (W: word, S: bit shift, B: width) ---------------
  template <int W, int S, int B>
  CB_HD u32 get() const {
    return static_cast<u32>(w[W] >> S) & static_cast<u32>((u64{1} << B) - 1);
  }
  template <int W, int S, int B>
  CB_HD void put(u32 v) {
    constexpr u64 m = ((u64{1} << B) - 1) << S;
    w[W] = (w[W] & ~m) | ((static_cast<u64>(v) << S) & m);
  }

  // -- table (TurnState50, bytes 0..95) ---------------------------------------
  CB_HD Mask hand(u32 p) const { return p ? w[1] : w[0]; }
  CB_HD void set_hand(u32 p, Mask v) { if (p) w[1] = v; else w[0] = v; }
  CB_HD Mask floor() const { return w[2]; }
  CB_HD void set_floor(Mask v) { w[2] = v; }
  CB_HD Mask stock() const { return w[3]; }
  CB_HD void set_stock(Mask v) { w[3] = v; }
  CB_HD Mask pile(u32 p) const { return p ? w[5] : w[4]; }
  CB_HD void set_pile(u32 p, Mask v) { if (p) w[5] = v; else w[4] = v; }
  CB_HD u64 rng() const { return w[6]; }
  CB_HD void set_rng(u64 v) { w[6] = v; }
  // Bonus cards flipped from the stock during the current turn.
  CB_HD Mask flip_bonus() const { return w[7]; }
  CB_HD void set_flip_bonus(Mask v) { w[7] = v; }
  CB_HD u32 ppuk_months() const { return get<8, 0, 16>(); }
  CB_HD void set_ppuk_months(u32 v) { put<8, 0, 16>(v); }
  // Low 12 bits: ppuk months owned by player 1; high bits: Gukjin flags.
  CB_HD u32 owner1() const { return get<8, 16, 16>(); }
  CB_HD void set_owner1(u32 v) { put<8, 16, 16>(v); }
  CB_HD u32 ppuk_bonus2() const { return get<8, 32, 16>(); }
  CB_HD void set_ppuk_bonus2(u32 v) { put<8, 32, 16>(v); }
  CB_HD u32 ppuk_bonus3() const { return get<8, 48, 16>(); }
  CB_HD void set_ppuk_bonus3(u32 v) { put<8, 48, 16>(v); }
  CB_HD u32 turn() const { return get<9, 0, 16>(); }
  CB_HD void set_turn(u32 v) { put<9, 0, 16>(v); }
  CB_HD u32 actor() const { return get<9, 16, 8>(); }
  CB_HD void set_actor(u32 v) { put<9, 16, 8>(v); }
  CB_HD u32 phase() const { return get<9, 24, 8>(); }
  CB_HD void set_phase(u32 v) { put<9, 24, 8>(v); }
  CB_HD u32 played() const { return get<9, 32, 8>(); }
  CB_HD void set_played(u32 v) { put<9, 32, 8>(v); }
  CB_HD u32 drawn() const { return get<9, 40, 8>(); }
  CB_HD void set_drawn(u32 v) { put<9, 40, 8>(v); }
  CB_HD Mask mission() const { return w[10]; }
  CB_HD void set_mission(Mask v) { w[10] = v; }
  CB_HD u32 neutral_ppuk() const { return get<11, 0, 16>(); }
  CB_HD void set_neutral_ppuk(u32 v) { put<11, 0, 16>(v); }

  // -- Go/Stop bookkeeping (GameState50, bytes 96..103) ------------------------
  CB_HD u32 go(u32 p) const { return p ? get<12, 8, 8>() : get<12, 0, 8>(); }
  CB_HD void set_go(u32 p, u32 v) { if (p) put<12, 8, 8>(v); else put<12, 0, 8>(v); }
  CB_HD u32 last_go(u32 p) const { return p ? get<12, 24, 8>() : get<12, 16, 8>(); }
  CB_HD void set_last_go(u32 p, u32 v) { if (p) put<12, 24, 8>(v); else put<12, 16, 8>(v); }
  CB_HD u32 gostop_actor() const { return get<12, 32, 8>(); }
  CB_HD void set_gostop_actor(u32 v) { put<12, 32, 8>(v); }
  CB_HD u32 winner() const { return get<12, 40, 8>(); }
  CB_HD void set_winner(u32 v) { put<12, 40, 8>(v); }
  // 0 = no Gukjin prompt, otherwise prompted player + 1.
  CB_HD u32 gukjin_prompt() const { return get<12, 48, 8>(); }
  CB_HD void set_gukjin_prompt(u32 v) { put<12, 48, 8>(v); }

  // -- special plays (SpecialGameState50, bytes 104..119) ----------------------
  CB_HD u32 shaken(u32 p) const { return p ? get<13, 16, 16>() : get<13, 0, 16>(); }
  CB_HD void set_shaken(u32 p, u32 v) { if (p) put<13, 16, 16>(v); else put<13, 0, 16>(v); }
  CB_HD u32 bombs(u32 p) const { return p ? get<13, 40, 8>() : get<13, 32, 8>(); }
  CB_HD void set_bombs(u32 p, u32 v) { if (p) put<13, 40, 8>(v); else put<13, 32, 8>(v); }
  CB_HD u32 credits(u32 p) const { return p ? get<13, 56, 8>() : get<13, 48, 8>(); }
  CB_HD void set_credits(u32 p, u32 v) { if (p) put<13, 56, 8>(v); else put<13, 48, 8>(v); }
  CB_HD u32 shaken4(u32 p) const { return p ? get<14, 16, 16>() : get<14, 0, 16>(); }
  CB_HD void set_shaken4(u32 p, u32 v) { if (p) put<14, 16, 16>(v); else put<14, 0, 16>(v); }

  // -- game end and Hangame extras (TerminalGameState50, bytes 120..191) -------
  CB_HD u32 ppuk_count(u32 p) const { return p ? get<15, 8, 8>() : get<15, 0, 8>(); }
  CB_HD void set_ppuk_count(u32 p, u32 v) { if (p) put<15, 8, 8>(v); else put<15, 0, 8>(v); }
  CB_HD u32 ppuk_streak(u32 p) const { return p ? get<15, 24, 8>() : get<15, 16, 8>(); }
  CB_HD void set_ppuk_streak(u32 p, u32 v) { if (p) put<15, 24, 8>(v); else put<15, 16, 8>(v); }
  CB_HD u32 chong_actor() const { return get<15, 32, 8>(); }
  CB_HD void set_chong_actor(u32 v) { put<15, 32, 8>(v); }
  CB_HD u32 chong_months() const { return get<15, 48, 16>(); }
  CB_HD void set_chong_months(u32 v) { put<15, 48, 16>(v); }
  CB_HD u32 end_winner() const { return get<16, 0, 8>(); }
  CB_HD void set_end_winner(u32 v) { put<16, 0, 8>(v); }
  CB_HD u32 end_reason() const { return get<16, 8, 8>(); }
  CB_HD void set_end_reason(u32 v) { put<16, 8, 8>(v); }
  CB_HD u64 end_points() const { return w[17]; }
  CB_HD void set_end_points(u64 v) { w[17] = v; }
  CB_HD i32 side0() const { return static_cast<i32>(get<18, 0, 32>()); }
  CB_HD void set_side0(i32 v) { put<18, 0, 32>(static_cast<u32>(v)); }
  CB_HD u32 round_raw() const { return get<18, 32, 8>(); }
  CB_HD void set_round_raw(u32 v) { put<18, 32, 8>(v); }
  CB_HD u32 round_mult() const { const u32 r = round_raw(); return r == 0 ? 1u : r; }
  CB_HD u32 mission_type() const { return get<18, 40, 8>(); }
  CB_HD void set_mission_type(u32 v) { put<18, 40, 8>(v); }
  CB_HD u32 mission_mult() const { return get<18, 48, 8>(); }
  CB_HD void set_mission_mult(u32 v) { put<18, 48, 8>(v); }
  CB_HD u32 mission_multi(u32 p) const { return p ? get<19, 0, 8>() : get<18, 56, 8>(); }
  CB_HD void set_mission_multi(u32 p, u32 v) { if (p) put<19, 0, 8>(v); else put<18, 56, 8>(v); }
  // Every card a hand has held; cards shown by a shake declaration.
  CB_HD Mask held(u32 p) const { return p ? w[21] : w[20]; }
  CB_HD void set_held(u32 p, Mask v) { if (p) w[21] = v; else w[20] = v; }
  CB_HD Mask shown(u32 p) const { return p ? w[23] : w[22]; }
  CB_HD void set_shown(u32 p, Mask v) { if (p) w[23] = v; else w[22] = v; }

  // -- pending decision record (PostChancePending50, bytes 192..223) -----------
  CB_HD u32 pa_kind() const { return get<24, 0, 8>(); }
  CB_HD void set_pa_kind(u32 v) { put<24, 0, 8>(v); }
  CB_HD u32 pa_card() const { return get<24, 8, 8>(); }
  CB_HD void set_pa_card(u32 v) { put<24, 8, 8>(v); }
  CB_HD u32 pa_month() const { return get<24, 16, 8>(); }
  CB_HD void set_pa_month(u32 v) { put<24, 16, 8>(v); }
  CB_HD u32 pa_played_pick() const { return get<24, 24, 8>(); }
  CB_HD void set_pa_played_pick(u32 v) { put<24, 24, 8>(v); }
  CB_HD u32 pa_drawn_pick() const { return get<24, 32, 8>(); }
  CB_HD void set_pa_drawn_pick(u32 v) { put<24, 32, 8>(v); }
  CB_HD Mask pa_pi_pick() const { return w[25]; }
  CB_HD void set_pa_pi_pick(Mask v) { w[25] = v; }
  CB_HD Mask pend_selected_pi() const { return w[26]; }
  CB_HD u32 pend_primary() const { return get<27, 0, 16>(); }
  CB_HD void set_pend_primary(u32 v) { put<27, 0, 16>(v); }
  CB_HD u32 pend_actor() const { return get<27, 16, 8>(); }
  CB_HD void set_pend_actor(u32 v) { put<27, 16, 8>(v); }
  CB_HD u32 pend_active() const { return get<27, 24, 8>(); }
  CB_HD void set_pend_active(u32 v) { put<27, 24, 8>(v); }

  // -- counters and step outcome (bytes 224..247) ------------------------------
  CB_HD u32 n_primary() const { return get<28, 0, 16>(); }
  CB_HD void set_n_primary(u32 v) { put<28, 0, 16>(v); }
  CB_HD u32 n_choice() const { return get<28, 16, 16>(); }
  CB_HD void set_n_choice(u32 v) { put<28, 16, 16>(v); }
  CB_HD u32 n_resolve() const { return get<28, 32, 16>(); }
  CB_HD void set_n_resolve(u32 v) { put<28, 32, 16>(v); }
  CB_HD u32 n_pi() const { return get<28, 48, 16>(); }
  CB_HD void set_n_pi(u32 v) { put<28, 48, 16>(v); }
  CB_HD u32 n_bonus() const { return get<29, 0, 16>(); }
  CB_HD void set_n_bonus(u32 v) { put<29, 0, 16>(v); }
  CB_HD u32 n_special() const { return get<29, 16, 16>(); }
  CB_HD void set_n_special(u32 v) { put<29, 16, 16>(v); }
  CB_HD u32 n_go() const { return get<29, 32, 16>(); }
  CB_HD void set_n_go(u32 v) { put<29, 32, 16>(v); }
  CB_HD u32 status() const { return get<29, 48, 8>(); }
  CB_HD void set_status(u32 v) { put<29, 48, 8>(v); }
  CB_HD u32 done() const { return get<29, 56, 8>(); }
  CB_HD void set_done(u32 v) { put<29, 56, 8>(v); }
  CB_HD u32 nagari() const { return get<30, 0, 8>(); }
  CB_HD void set_nagari(u32 v) { put<30, 0, 8>(v); }

  // -- derived predicates -------------------------------------------------------
  CB_HD bool ended() const { return end_reason() != kEndNone; }
  CB_HD bool chong_pending() const { return chong_actor() <= 1u; }
  CB_HD bool gostop_pending() const { return gostop_actor() <= 1u; }
  CB_HD bool gukjin_pending() const { return gukjin_prompt() != 0; }
  CB_HD bool prompt_pending() const { return gostop_pending() || gukjin_pending(); }
  CB_HD bool decided() const { return winner() <= 1u; }
  CB_HD bool last_turn() const { return turn() >= 18u; }
  CB_HD Mask floor_std() const { return floor() & kStandardDeck; }
};

// Clears every padding byte of a row image (bytes 78-79, 90-95, 103, 116-119,
// 125, 130-135, 153-159, 197-199, 220-223, 241-247).
CB_HD void zero_padding(Game& g) {
  g.w[9] &= 0x0000'ffff'ffff'ffffull;
  g.w[11] &= 0xffffull;
  g.w[12] &= 0x00ff'ffff'ffff'ffffull;
  g.w[14] &= 0xffff'ffffull;
  g.w[15] &= 0xffff'00ff'ffff'ffffull;
  g.w[16] &= 0xffffull;
  g.w[19] &= 0xffull;
  g.w[24] &= 0xff'ffff'ffffull;
  g.w[27] &= 0xffff'ffffull;
  g.w[30] &= 0xffull;
}

}  // namespace cb
