// The batch-environment contract on one Game: create, observe, step, start
// record, stock preview and the event diff.  Behaviour matches the reference
// extension's per-row bodies (python/csrc/torch50_ext.cu:125-435) over
// cugo/game/torch50.h; the implementation is this engine's own.
#pragma once

#include <math.h>

#include "rules.cuh"

namespace cb {

constexpr u32 kFeatures = 720;
constexpr u32 kActions = 179;
constexpr u32 kPrimaryActions = 127;
constexpr u32 kChoiceBegin = 127;
constexpr u32 kGukjinPiAction = 177;
constexpr u32 kGukjinAnimalAction = 178;
constexpr u32 kEventWords = 9;
constexpr u32 kStartWords = 8;
constexpr u32 kNoAction = 0xffffu;

// ---- settlement (cugo/game/settlement50.h:95-225) ----------------------------

struct Settlement {
  bool ok;
  u32 winner;
  u64 final_points;
};

CB_HD Settlement settle(const Game& g) {
  Settlement s{false, kNobody, 0};
  if (!g.ended() || g.end_winner() > 1u) return s;
  const u32 w = g.end_winner(), l = w ^ 1u;
  s.ok = true;
  s.winner = w;
  const u64 round = g.round_mult();
  const u32 reason = g.end_reason();
  if (reason == kEndDealtChongtong || reason == kEndFloorChongtong ||
      reason == kEndBonusChongtong || reason == kEndThreePpuk) {
    s.final_points = g.end_points() * round;
    return s;
  }
  const Score ws = player_score(g, w), ls = player_score(g, l);
  const u32 go = g.go(w);
  const u64 after_go = (static_cast<u64>(ws.points) + go) * go_multiplier(go);
  const u64 special = pow2_u8((g.bombs(w) + shake_count(g, w)) & 0xffu);
  u64 bak = 1;
  if (ws.meongtta) bak *= 2u;
  if (ws.pi >= 10u && ls.pi >= 1u && ls.pi <= 7u) bak *= 2u;
  if (ws.bright >= 3u && ls.bright == 0u) bak *= 2u;
  if (g.go(l) != 0u) bak *= 2u;
  u64 mission = g.mission_multi(w);
  if (mission == 0) mission = 1;
  s.final_points = g.pile(l) == 0 ? 0u : after_go * special * bak * mission * round;
  return s;
}

// Zero-sum reward of player 0 for a finished game: the settled points plus the
// immediate side payments; a nagari pays only the side payments
// (torch_reward0_50, cugo/game/torch50.h:472-478).
CB_HD i64 reward0(const Game& g) {
  if (!g.done()) return 0;
  if (g.nagari()) return g.side0();
  const Settlement s = settle(g);
  if (!s.ok) return 0;
  const i64 pts = static_cast<i64>(s.final_points);
  return (s.winner == 0 ? pts : -pts) + g.side0();
}

// ---- decisions and legal actions (cugo/game/policy50.h:151-236) --------------

CB_HD u32 decision_kind(const Game& g) {
  if (g.ended()) return kDecNone;
  if (g.chong_pending()) return kDecChongtong;
  if (g.gukjin_pending()) return kDecGukjin;
  if (g.gostop_pending()) return kDecGoStop;
  return g.phase() == kPhasePlay ? kDecPrimary : kDecNone;
}

CB_HD u32 decision_player(const Game& g) {
  if (g.ended()) return kNobody;
  if (g.chong_pending()) return g.chong_actor();
  if (g.gukjin_pending()) return g.gukjin_prompt() - 1u;
  if (g.gostop_pending()) return g.gostop_actor();
  return g.actor();
}

// The player an observation is written for.
CB_HD u32 observer_seat(const Game& g) {
  const u32 p = decision_player(g);
  return p > 1u ? (g.actor() & 1u) : p;
}

struct Legal {
  u64 w0 = 0, w1 = 0, w2 = 0;  // actions 0..63, 64..127, 128..178
  CB_HD void set(u32 a) {
    const u64 b = u64{1} << (a & 63u);
    if (a < 64u) w0 |= b;
    else if (a < 128u) w1 |= b;
    else if (a < kActions) w2 |= b;
  }
  CB_HD bool has(u32 a) const {
    if (a >= kActions) return false;
    const u64 b = u64{1} << (a & 63u);
    return ((a < 64u ? w0 : a < 128u ? w1 : w2) & b) != 0;
  }
  CB_HD u32 count() const { return popc(w0) + popc(w1) + popc(w2); }
};

// legal_primary_actions50: bombs and grenades are forced for their months.
CB_HD Legal primary_legal(const Game& g) {
  Legal m;
  const u32 kind = decision_kind(g);
  if (kind == kDecChongtong) {
    m.w1 = (u64{1} << (125 - 64)) | (u64{1} << (126 - 64));
    return m;
  }
  if (kind == kDecGoStop) {
    m.w1 = (u64{1} << (123 - 64)) | (u64{1} << (124 - 64));
    return m;
  }
  if (kind != kDecPrimary || g.stock() == 0) return m;
  const u32 a = g.actor();
  const Mask hand = g.hand(a);
  const u32 bombs = bomb_months(g), grenades = grenade_months(g);
  const u32 forced = bombs | grenades;
  const u32 shakes = shake_months(g);
  // Spread a month set to the four card bits of each month.
  auto month_spread = [](u32 months) {
    Mask out = 0;
CB_UNROLL
    for (u32 mo = 0; mo < 12; ++mo)
      if (months & (1u << mo)) out |= month_cards(mo);
    return out;
  };
  const Mask std = hand & kStandardDeck;
  const Mask playable = std & ~month_spread(forced);
  const Mask shakeable = std & month_spread(shakes);
  // Card plays 0..47, bonus plays 48..49 (bits 48/49 of the hand), shakes 50..97.
  m.w0 = playable | (hand & kBonusCards) | (shakeable << 50);
  m.w1 = shakeable >> 14;
  // Bombs 98..109, grenades 110..121, bomb credit 122.
  m.w1 |= static_cast<u64>(bombs) << (98 - 64);
  m.w1 |= static_cast<u64>(grenades) << (110 - 64);
  if (g.credits(a) != 0) m.w1 |= u64{1} << (122 - 64);
  return m;
}

// primary_legal(g).has(action) without building the mask: the step needs only the
// one action's bit, and the mask's month sets (bombs, grenades, shakes over all twelve
// months) cost more than the rest of a plain play's legality.  The same rules for the
// action's own month.
CB_HD bool primary_action_legal(const Game& g, u32 action) {
  const u32 kind = decision_kind(g);
  if (kind == kDecChongtong) return action == 125u || action == 126u;
  if (kind == kDecGoStop) return action == 123u || action == 124u;
  if (kind != kDecPrimary || g.stock() == 0) return false;
  const u32 a = g.actor();
  const Mask hand = g.hand(a);
  if (action >= 48u && action < 50u) return (hand & card_bit(action)) != 0;  // bonus play
  if (action == 122u) return g.credits(a) != 0;
  if (action >= 123u) return false;
  // A card play (0..47), shake (50..97), bomb (98..109) or grenade (110..121): the
  // counts of the month's cards in hand and on the floor decide.
  u32 month, card = kNoCard;
  if (action < 48u) card = action;
  else if (action < 98u) card = action - 50u;
  if (card != kNoCard) {
    if (!(hand & card_bit(card))) return false;
    month = card_month(card);
  } else {
    month = action < 110u ? action - 98u : action - 110u;
  }
  const Mask mc = month_cards(month);
  const u32 in_hand = popc(hand & mc), on_floor = popc(g.floor_std() & mc);
  const bool bomb = in_hand == 3u && on_floor == 1u;
  const bool grenade = in_hand == 2u && on_floor == 2u;
  const u32 mb = 1u << month;
  if (action < 48u) return !(bomb || grenade);  // forced months take no single play
  if (action < 98u)
    return on_floor == 0u && ((in_hand == 3u && !(g.shaken(a) & mb)) ||
                              (in_hand == 4u && !(g.shaken4(a) & mb)));
  return action < 110u ? bomb : grenade;
}

// ---- pending floor choices (cugo/game/postchance50.h:150-456) ----------------
//
// A primary action whose flipped card leaves a two-card floor choice stays
// pending; the chooser picks the floor card with a choice action (127 + card).
// peek_pending() answers, without mutating the game, whether the pending
// action needs another choice.

struct Peek {
  u32 status = kOk;
  u32 decision = kDecNone;  // kDecFloorPlayed, kDecFloorDrawn or kDecNone
  Mask choices = 0;         // floor cards the choice may take
  u32 revealed = kNoCard;   // the standard card the stock flip showed
  // The flip itself, for the commit that follows a complete probe: the bonus cards
  // flipped before `revealed`, and the stock and its random stream after it.
  Mask flip_bonus = 0;
  Mask stock_after = 0;
  u64 rng_after = 0;
};

// The floor after `card` lands on it, given the pick for a two-card match.
// Returns false and sets `need` when a pick is missing, or sets `bad` when the
// pick is not one of the matches.
CB_HD Mask floor_after(Mask floor_std, u32 card, u32 pick, bool& need, bool& bad) {
  const Mask matches = floor_std & month_cards(card_month(card));
  const u32 n = popc(matches);
  need = bad = false;
  if (n == 0) return floor_std | card_bit(card);
  if (n != 2) return floor_std & ~matches;
  if (auto_pick(matches) && !in_set(matches, pick)) pick = lowest_card(matches);
  if (pick == kNoCard) {
    need = true;
    return floor_std;
  }
  if (!is_standard(pick) || !in_set(matches, pick)) {
    bad = true;
    return floor_std;
  }
  return floor_std & ~card_bit(pick);
}

// A card play or shake (`card` lands on the floor, then the flipped card), or a bomb,
// grenade or bomb credit (card = kNoCard: the bomb's month leaves the floor, then only
// the flipped card lands).  Both kinds share one body so that a warp whose rows mix
// them runs it once: they differ only in the floor before the flip and in the
// played card's resolution.
CB_HD Peek peek_turn(const Game& g, u32 kind, u32 card, u32 month, u32 played_pick,
                     u32 drawn_pick) {
  Peek p;
  const bool regular = card != kNoCard;
  Mask floor = g.floor_std();
  if (!regular && kind != kActCredit) floor &= ~month_cards(month);
  Mask stock = g.stock();
  u64 rng = g.rng();
  const Flip f = flip_stock(stock, rng);
  if (f.card == kNoCard) {
    p.status = kStockEmpty;
    return p;
  }
  p.revealed = f.card;
  p.flip_bonus = f.bonuses;
  p.stock_after = stock;
  p.rng_after = rng;
  Mask after_played = floor;
  if (regular) {
    const Mask pm = floor & month_cards(card_month(card));
    const u32 pmc = popc(pm);
    const bool same = card_month(card) == card_month(f.card);
    if (same && ((pmc == 1 && !g.last_turn()) || pmc == 0 || pmc == 2)) return p;
    bool need, bad;
    after_played = floor_after(floor, card, played_pick, need, bad);
    if (need) {
      p.decision = kDecFloorPlayed;
      p.choices = pm;
      return p;
    }
    if (bad) {
      p.status = kInvalidChoice;
      return p;
    }
  }
  bool need, bad;
  const Mask dm = after_played & month_cards(card_month(f.card));
  floor_after(after_played, f.card, drawn_pick, need, bad);
  if (need) {
    p.decision = kDecFloorDrawn;
    p.choices = dm;
  } else if (bad) {
    p.status = kInvalidChoice;
  }
  return p;
}

CB_HD Peek peek_pending(const Game& g) {
  const u32 kind = g.pa_kind();
  if (kind == kActPlay || kind == kActShake)
    return peek_turn(g, kind, g.pa_card(), 0xffu, g.pa_played_pick(), g.pa_drawn_pick());
  if (kind == kActBomb || kind == kActGrenade || kind == kActCredit)
    return peek_turn(g, kind, kNoCard, g.pa_month(), kNoCard, g.pa_drawn_pick());
  return Peek{};  // bonus plays and prompts never open a floor choice
}

// Turns `v` into the table the chooser sees at the pending choice: the card
// played and the stock flipped (the flip of `p`, the row's probe); for a drawn-card
// choice also the played card already resolved (postchance50.h:188-198, 288-292,
// 391-399).
CB_HD void stage_pending_view(Game& v, const Peek& p) {
  const u32 a = v.actor();
  const u32 kind = v.pa_kind();
  if (kind == kActPlay || kind == kActShake) {
    const u32 card = v.pa_card();
    if (kind == kActShake) {
      const u32 mb = month_bit(card);
      if (popc(v.hand(a) & month_cards(card_month(card))) == 4) v.set_shaken4(a, v.shaken4(a) | mb);
      else v.set_shaken(a, v.shaken(a) | mb);
    }
    v.set_hand(a, v.hand(a) & ~card_bit(card));
    v.set_played(card);
    v.set_stock(p.stock_after);
    v.set_rng(p.rng_after);
    v.set_drawn(p.revealed);
    v.set_flip_bonus(p.flip_bonus);
    v.set_phase(kPhaseResolve);
    if (p.decision == kDecFloorDrawn) {
      Tally t;
      resolve_card(v, card, v.pa_played_pick(), t);
      v.set_played(kNoCard);
    }
    return;
  }
  // Bomb, grenade or credit.
  if (kind == kActCredit) {
    v.set_credits(a, v.credits(a) - 1u);
  } else {
    const u32 m = v.pa_month();
    const Mask hc = v.hand(a) & month_cards(m);
    const Mask fc = v.floor_std() & month_cards(m);
    v.set_hand(a, v.hand(a) & ~hc);
    v.set_floor(v.floor() & ~fc);
    v.set_pile(a, v.pile(a) | hc | fc);
    const bool grenade = kind == kActGrenade;
    v.set_credits(a, (v.credits(a) + (grenade ? 1u : 2u)) & 0xffu);
    if (!grenade) v.set_bombs(a, (v.bombs(a) + 1u) & 0xffu);
  }
  v.set_stock(p.stock_after);
  v.set_rng(p.rng_after);
  v.set_drawn(p.revealed);
  v.set_flip_bonus(p.flip_bonus);
}

// ---- observation packet ------------------------------------------------------
//
// The 720 features (contract v4, cugo/game/torch50.h:334-470) are 0/1 except 37
// columns.  A packet holds the 0/1 columns as a 720-bit map and the others as
// floats; kernels expand packets into feature rows cooperatively.

constexpr u32 kScalarColumns = 37;
constexpr u32 kBitWords = 24;

// Where a packet is written: a thread's own slice of a shared-memory tile in the
// kernels (no registers or local memory held for it), or an ObsPacket on the host.
struct PacketRef {
  u32* bits;    // [kBitWords]
  float* scal;  // [kScalarColumns]
};

struct ObsPacket {
  u32 bits[kBitWords];
  float scal[kScalarColumns];
  CB_HD PacketRef ref() { return PacketRef{bits, scal}; }
};

// Slot of a non-binary feature column in ObsPacket::scal, or -1.
CB_HD int scalar_slot(u32 c) {
  if (c == 452u) return 0;                         // opponent hand count
  if (c >= 453u && c <= 468u) return 1 + (int)(c - 453u);   // scalars s0..s15
  if (c >= 471u && c <= 478u) return 17 + (int)(c - 471u);  // scalars s18..s25
  if (c >= 491u && c <= 495u) return 25 + (int)(c - 491u);  // table counts
  if (c >= 549u && c <= 551u) return 30 + (int)(c - 549u);  // mission multipliers
  if (c == 556u) return 33;                        // side payments
  if (c == 557u) return 34;                        // round multiplier
  if (c == 710u) return 35;                        // own ribbons
  if (c == 711u) return 36;                        // opponent ribbons
  return -1;
}

CB_HD float feature_value(const ObsPacket& pk, u32 c) {
  const int s = scalar_slot(c);
  if (s >= 0) return pk.scal[s];
  return ((pk.bits[c >> 5] >> (c & 31u)) & 1u) ? 1.0f : 0.0f;
}

CB_HD float fdiv(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}

// torch_unit50: value / scale clamped to 1.
CB_HD float unit(u32 v, u32 scale) {
  const float r = fdiv(static_cast<float>(v), static_cast<float>(scale));
  return r > 1.0f ? 1.0f : r;
}

CB_HD void or_word(u32* bits, u32 off, u32 x) {
  const u32 wi = off >> 5, sh = off & 31u;
  bits[wi] |= x << sh;
  if (sh != 0) bits[wi + 1] |= x >> (32u - sh);
}

// ORs `n` (<= 64) low bits of `val` into the map at column `off`.
CB_HD void put_bits(u32* bits, u32 off, u64 val) {
  or_word(bits, off, static_cast<u32>(val));
  or_word(bits, off + 32u, static_cast<u32>(val >> 32));
}

CB_HD void put_flag(u32* bits, u32 col, bool on) {
  if (on) bits[col >> 5] |= 1u << (col & 31u);
}

// Settled points if the Go/Stop decider stopped now (stop_points50,
// cugo/game/policy50.h:354-365), saturated to 32 bits.
CB_HD u32 stop_points(const Game& g) {
  if (decision_kind(g) != kDecGoStop) return 0;
  Game s = g;
  const u32 a = s.gostop_actor();
  settle_loser_gukjin(s, a ^ 1u);
  s.set_winner(a);
  s.set_gostop_actor(kNobody);
  sync_stop(s);
  if (!s.ended()) return 0;
  const Settlement st = settle(s);
  if (!st.ok) return 0;
  return st.final_points > 0xffffffffull ? 0xffffffffu : static_cast<u32>(st.final_points);
}

struct PacketInputs {
  u32 decision;     // decision kind written to the one-hot (0 when done)
  u32 primary;      // pending primary action or kNoAction
  u32 revealed;     // flipped card shown at a pending choice or kNoCard
  Mask choices;     // floor cards selectable at a pending choice
  bool pending_view;
};

// pack_policy_observation50 + encode_torch_packet50 for the observer's seat.
CB_HD void pack_observation(const Game& g, const PacketInputs& in, PacketRef pk) {
  for (u32 i = 0; i < kBitWords; ++i) pk.bits[i] = 0;
  const u32 me = observer_seat(g), op = me ^ 1u;
  const Mask own_hand = g.hand(me), opp_hand = g.hand(op);
  const Mask own_pile = g.pile(me), opp_pile = g.pile(op);
  const Mask floor = g.floor();
  Mask pending_public = g.flip_bonus();
  if (is_standard(g.played())) pending_public |= card_bit(g.played());
  if (is_standard(g.drawn())) pending_public |= card_bit(g.drawn());
  const Mask known = own_hand | floor | own_pile | opp_pile | pending_public;
  const Mask opp_known_hand = g.shown(op) & kFullDeck & ~known;
  Mask unseen = kFullDeck & ~known & ~opp_known_hand;
  if (in.pending_view && is_card(in.revealed) && !(known & card_bit(in.revealed))) {
    pending_public |= card_bit(in.revealed);
    unseen &= ~card_bit(in.revealed);
  }
  const u32 owner1_m = g.owner1() & 0xfffu;
  const u32 owner0_m = g.ppuk_months() & ~owner1_m;
  const u32 shaken0 = g.shaken(0) | g.shaken4(0), shaken1 = g.shaken(1) | g.shaken4(1);
  const Score os = player_score(g, me), xs = player_score(g, op);

  u32* b = pk.bits;
  put_bits(b, 0, own_hand);
  put_bits(b, 50, floor);
  put_bits(b, 100, own_pile);
  put_bits(b, 150, opp_pile);
  put_bits(b, 200, pending_public);
  put_bits(b, 250, unseen);
  put_bits(b, 300, me ? shaken1 : shaken0);
  put_bits(b, 312, me ? shaken0 : shaken1);
  put_bits(b, 324, g.ppuk_months() & 0xfffu);
  put_bits(b, 336, me ? owner1_m : owner0_m);
  put_bits(b, 348, me ? owner0_m : owner1_m);
  put_bits(b, 360, g.ppuk_bonus2() & 0xfffu);
  put_bits(b, 372, g.ppuk_bonus3() & 0xfffu);
  put_bits(b, 384, g.chong_months() & 0xfffu);
  put_bits(b, 396, in.choices & kFullDeck);
  const bool first = ((g.actor() ^ g.turn()) & 1u) == me;
  put_flag(b, 446, first);
  for (u32 k = 1; k <= 5u; ++k) put_flag(b, 446 + k, in.decision == k);  // constant columns
  put_flag(b, 469, (g.owner1() & gukjin_pi_flag(me)) != 0);
  put_flag(b, 470, (g.owner1() & gukjin_pi_flag(op)) != 0);
  put_bits(b, 479, g.neutral_ppuk() & 0xfffu);
  put_bits(b, 496, g.mission() & kStandardDeck);
  const u32 mt = g.mission_type();
  put_flag(b, 544, mt == kMissionEasy);
  put_flag(b, 545, mt == kMissionNormal);
  put_flag(b, 546, mt == kMissionHard);
  put_flag(b, 547, mt == kMissionAll);
  put_flag(b, 548, mt == kMissionTriple);
  put_flag(b, 552, in.decision == kDecGukjin);
  put_flag(b, 553, (g.owner1() & gukjin_lock_flag(me)) != 0);
  put_flag(b, 554, (g.owner1() & gukjin_lock_flag(op)) != 0);
  put_flag(b, 555, g.last_turn());
  const u32 own_streak = g.ppuk_streak(me), opp_streak = g.ppuk_streak(op);
  put_flag(b, 558, own_streak == kPpukFirst || own_streak == kPpukSecond);
  put_flag(b, 559, opp_streak == kPpukFirst || opp_streak == kPpukSecond);
  put_bits(b, 560, g.held(me) & ~own_hand);
  put_bits(b, 610, g.held(op) & ~opp_hand);
  put_bits(b, 660, opp_known_hand);

  float* s = pk.scal;
  s[0] = unit(popc(opp_hand), 10);
  s[1] = unit(g.turn(), 32);
  s[2] = unit(popc(g.stock()), 30);
  s[3] = unit(g.go(me), 8);
  s[4] = unit(g.go(op), 8);
  s[5] = unit(g.last_go(me), 64);
  s[6] = unit(g.last_go(op), 64);
  s[7] = unit(os.points, 64);
  s[8] = unit(xs.points, 64);
  s[9] = unit(g.bombs(me), 4);
  s[10] = unit(g.bombs(op), 4);
  s[11] = unit(g.credits(me), 4);
  s[12] = unit(g.credits(op), 4);
  s[13] = unit(g.ppuk_count(me), 3);
  s[14] = unit(g.ppuk_count(op), 3);
  s[15] = unit(own_streak <= 3u ? own_streak : 0u, 3);
  s[16] = unit(opp_streak <= 3u ? opp_streak : 0u, 3);
  {
    const float bits = log2f(1.0f + static_cast<float>(stop_points(g))) / 12.0f;
    s[17] = bits > 1.0f ? 1.0f : bits;
  }
  s[18] = in.primary < kPrimaryActions
              ? fdiv(static_cast<float>(in.primary + 1u), static_cast<float>(kPrimaryActions))
              : 0.0f;
  s[19] = is_card(in.revealed) ? fdiv(static_cast<float>(in.revealed + 1u), 50.0f) : 0.0f;
  s[20] = unit(os.pi, 20);
  s[21] = unit(popc(in.choices & kFullDeck), 50);
  s[22] = unit(popc(own_hand), 50);
  s[23] = unit(popc(floor), 50);
  s[24] = unit(popc(unseen), 50);
  s[25] = unit(xs.pi, 20);
  s[26] = unit(os.bright, 5);
  s[27] = unit(xs.bright, 5);
  s[28] = unit(os.animal, 10);
  s[29] = unit(xs.animal, 10);
  s[30] = unit(g.mission_mult(), 4);
  s[31] = unit(g.mission_multi(me), 8);
  s[32] = unit(g.mission_multi(op), 8);
  {
    const i32 side = me == 0 ? g.side0() : -g.side0();
    const float x = static_cast<float>(side) / 64.0f;
    s[33] = x > 1.0f ? 1.0f : (x < -1.0f ? -1.0f : x);
  }
  s[34] = unit(g.round_mult(), 8);
  s[35] = unit(os.ribbon, 10);
  s[36] = unit(xs.ribbon, 10);
}

// The packet of an observation whose pending probe failed: an all-zero
// observation except the pending action and the revealed card.
CB_HD void pack_failed_probe(u32 primary, u32 revealed, PacketRef pk) {
  for (u32 i = 0; i < kBitWords; ++i) pk.bits[i] = 0;
  for (u32 i = 0; i < kScalarColumns; ++i) pk.scal[i] = 0.0f;
  pk.scal[18] = primary < kPrimaryActions
                    ? fdiv(static_cast<float>(primary + 1u), static_cast<float>(kPrimaryActions))
                    : 0.0f;
  pk.scal[19] = is_card(revealed) ? fdiv(static_cast<float>(revealed + 1u), 50.0f) : 0.0f;
}

struct ObsMeta {
  Legal legal;
  u32 player;
  u32 done;
  i32 status;
};

// Legal actions of the floor choice: 127 + card for each selectable card.
CB_HD Legal choice_legal(Mask choices) {
  Legal m;
  choices &= kFullDeck;
  m.w1 = (choices & 1u) ? (u64{1} << 63) : 0;  // card 0 is action 127
  m.w2 = choices >> 1;                         // cards 1..49 are actions 128..176
  return m;
}

// The legal mask and packet status of make_torch_packet50 without the features.
struct LegalInfo {
  Legal legal;
  u32 status = kOk;
  u32 kind = kDecNone;  // decision kind written to the observation (0 when done)
  Peek peek;            // the pending probe, when a floor choice is pending
};

CB_HD LegalInfo torch_legal(const Game& g) {
  LegalInfo r;
  if (g.pend_active()) {
    r.peek = peek_pending(g);
    r.status = r.peek.status;
    if (r.status == kOk) {
      r.legal = choice_legal(r.peek.choices);
      r.kind = r.peek.decision;
    }
    return r;
  }
  if (g.done()) return r;
  r.kind = decision_kind(g);
  if (r.kind == kDecGukjin) r.legal.w2 = (u64{1} << (177 - 128)) | (u64{1} << (178 - 128));
  else r.legal = primary_legal(g);
  return r;
}

// make_torch_packet50 + encode: the observation of one row.
CB_HD void observe_game(const Game& g, PacketRef pk, ObsMeta& meta) {
  meta.done = g.done() ? 1u : 0u;
  const LegalInfo li = torch_legal(g);
  meta.legal = li.legal;
  meta.status = static_cast<i32>(li.status);
  if (g.pend_active()) {
    meta.player = g.pend_actor();
    if (li.status != kOk) {
      pack_failed_probe(g.pend_primary(), li.peek.revealed, pk);
      return;
    }
    Game v = g;
    if (li.peek.decision != kDecNone) stage_pending_view(v, li.peek);
    v.set_actor(g.pend_actor());
    PacketInputs in{li.peek.decision, g.pend_primary(), li.peek.revealed, li.peek.choices, true};
    pack_observation(v, in, pk);
    return;
  }
  meta.player = observer_seat(g);
  PacketInputs in{li.kind, kNoAction, kNoCard, 0, false};
  pack_observation(g, in, pk);
}

// ---- committing actions (cugo/game/rollout50.h:231-399 and the layers below) --

// A card play or shake (play, flip, resolve both cards), or a bomb, grenade or bomb
// credit (the month's cards captured, then only the flipped card resolved), followed
// by the steal and the end-of-turn checks.  One body for both kinds, so a warp whose
// rows mix them runs the resolution and the end of the turn once; the order of every
// state change is the reference's for each kind.  `flip` is the complete probe of this
// action (peek_pending on the same row): its stock flip is the one the commit makes.
CB_HD void commit_turn(Game& g, u32 kind, u32 card, u32 month, const Peek& flip) {
  const u32 a = g.actor();
  const Mask before = g.pile(a);
  const bool regular = kind == kActPlay || kind == kActShake;
  u32 base_steal = 0;
  if (regular) {
    if (kind == kActShake) {
      const Mask mc = month_cards(card_month(card));
      g.set_shown(a, g.shown(a) | (g.hand(a) & mc));
      const u32 mb = month_bit(card);
      if (popc(g.hand(a) & mc) == 4) g.set_shaken4(a, g.shaken4(a) | mb);
      else g.set_shaken(a, g.shaken(a) | mb);
    }
    g.set_hand(a, g.hand(a) & ~card_bit(card));
  } else if (kind == kActCredit) {
    g.set_credits(a, g.credits(a) - 1u);
  } else {
    const Mask hc = g.hand(a) & month_cards(month);
    const Mask fc = g.floor_std() & month_cards(month);
    g.set_hand(a, g.hand(a) & ~hc);
    g.set_floor(g.floor() & ~fc);
    g.set_pile(a, g.pile(a) | hc | fc);
    const bool grenade = kind == kActGrenade;
    g.set_credits(a, (g.credits(a) + (grenade ? 1u : 2u)) & 0xffu);
    if (!grenade) g.set_bombs(a, (g.bombs(a) + 1u) & 0xffu);
    base_steal = g.last_turn() ? 0u : 1u;
  }
  g.set_played(regular ? card : kNoCard);
  g.set_stock(flip.stock_after);
  g.set_rng(flip.rng_after);
  g.set_drawn(flip.revealed);
  g.set_flip_bonus(flip.flip_bonus);
  g.set_phase(kPhaseResolve);
  Tally t;
  resolve_turn(g, g.pa_played_pick(), g.pa_drawn_pick(), t);
  steal_pi(g, a, (base_steal + steal_count(t)) & 0xffu);
  after_turn(g, a);
  if ((t.events & kEvTtadak) && g.turn() == 1u) side_payment(g, a, 7);
  missions_update(g, a, g.pile(a) & ~before);
  if (t.events & kEvPpuk) record_ppuk(g, a);
  sync_stop(g);
}

// A bonus card from hand: captured at once, replaced from the stock, one pi
// stolen; a replacement completing a month in hand offers a Chongtong.
CB_HD void commit_bonus(Game& g, u32 card) {
  const u32 a = g.actor();
  const u32 full_before = full_months(g.hand(a));
  Mask stock = g.stock();
  u64 rng = g.rng();
  const u32 repl = draw_card(stock, rng);
  g.set_stock(stock);
  g.set_rng(rng);
  g.set_hand(a, (g.hand(a) & ~card_bit(card)) | card_bit(repl));
  g.set_pile(a, g.pile(a) | card_bit(card));
  const Mask taken = steal_pi(g, a, g.last_turn() ? 0u : 1u);
  if (taken) missions_update(g, a, taken);
  const u32 newly = full_months(g.hand(a)) & ~full_before;
  if (!g.ended() && !g.chong_pending() && newly != 0) {
    g.set_chong_actor(a);
    g.set_chong_months(newly & 0xfffu);
  }
}

// Commits the pending action; `probe` is its complete probe (peek_pending).
CB_HD void commit_pending(Game& g, const Peek& probe) {
  g.set_held(0, g.held(0) | g.hand(0));
  g.set_held(1, g.held(1) | g.hand(1));
  const u32 kind = g.pa_kind();
  switch (kind) {
    case kActPlay:
    case kActShake:
    case kActBomb:
    case kActGrenade:
    case kActCredit:  // one call site: these rows of a warp share one inlined turn
      commit_turn(g, kind, g.pa_card(), g.pa_month(), probe);
      break;
    case kActBonus: commit_bonus(g, g.pa_card()); break;
    case kActGo:
    case kActStop: {
      const u32 d = g.gostop_actor();
      if (kind == kActStop) {
        settle_loser_gukjin(g, d ^ 1u);
        g.set_winner(d);
      } else {
        const u32 base = player_score(g, d).points;
        g.set_go(d, (g.go(d) + 1u) & 0xffu);
        g.set_last_go(d, base);
      }
      g.set_gostop_actor(kNobody);
      sync_stop(g);
      break;
    }
    case kActGukjinPi:
    case kActGukjinAnimal: {
      const u32 p = g.gukjin_prompt() - 1u;
      decide_gukjin(g, p, kind == kActGukjinPi);
      g.set_gukjin_prompt(0);
      open_gostop(g, p);
      sync_stop(g);
      break;
    }
    case kActChongWin:
      mark_end(g, g.chong_actor(), kEndBonusChongtong, 10u);
      break;
    default:  // kActChongGo
      g.set_chong_actor(kNobody);
      g.set_chong_months(0);
      break;
  }
  g.set_held(0, g.held(0) | g.hand(0));
  g.set_held(1, g.held(1) | g.hand(1));
}

// refresh_torch_done50.
CB_HD void refresh_done(Game& g) {
  if (g.ended()) {
    g.set_done(1);
    g.set_nagari(0);
    return;
  }
  const bool exhausted = g.phase() == kPhasePlay && g.hand(0) == 0 && g.hand(1) == 0 &&
                         g.credits(0) == 0 && g.credits(1) == 0;
  const bool nagari = !g.pend_active() && !g.chong_pending() && !g.prompt_pending() && exhausted;
  g.set_done(nagari ? 1u : 0u);
  g.set_nagari(nagari ? 1u : 0u);
}

// Pending record for a primary action or prompt answer
// (decode_primary_action50_raw + start_postchance_action50).
CB_HD void begin_pending(Game& g, u32 action) {
  u32 kind = kActPlay, card = kNoCard, month = 0xffu;
  if (action < 48u) {
    card = action;
  } else if (action < 50u) {
    kind = kActBonus;
    card = action;
  } else if (action < 98u) {
    kind = kActShake;
    card = action - 50u;
    month = card_month(card);
  } else if (action < 110u) {
    kind = kActBomb;
    month = action - 98u;
  } else if (action < 122u) {
    kind = kActGrenade;
    month = action - 110u;
  } else if (action == 122u) {
    kind = kActCredit;
  } else if (action == 123u) {
    kind = kActGo;
  } else if (action == 124u) {
    kind = kActStop;
  } else if (action == 125u) {
    kind = kActChongWin;
  } else if (action == 126u) {
    kind = kActChongGo;
  } else if (action == kGukjinPiAction) {
    kind = kActGukjinPi;
  } else {
    kind = kActGukjinAnimal;
  }
  const u32 seat = observer_seat(g);
  g.w[24] = static_cast<u64>(kind) | (static_cast<u64>(card) << 8) |
            (static_cast<u64>(month) << 16) | (u64{0xff} << 24) | (u64{0xff} << 32);
  g.w[25] = 0;
  g.w[26] = 0;
  g.w[27] = static_cast<u64>(action) | (static_cast<u64>(seat) << 16) | (u64{1} << 24);
}

struct StepOut {
  u32 status;
  i64 reward0;
  u32 done, nagari, committed;
};

// torch_step50: one unified action (0..178; anything else is kNoAction).  A row at a
// floor choice probes its pending action twice (to validate the choice, then with the
// choice made); every other row once, after its pending record is written.  Both go
// through one probe call site, so the probe's code is in the kernel once.
CB_HD StepOut step_game(Game& g, u32 action) {
  StepOut out{kOk, 0, 0, 0, 0};
  if (g.done()) {
    g.set_status(kFinished);
    return StepOut{kFinished, reward0(g), g.done(), g.nagari(), 0};
  }
  const bool choosing = g.pend_active() != 0;
  if (!choosing) {  // torch_legal without a pending probe, for this action only
    const bool ok = decision_kind(g) == kDecGukjin ? (action == 177u || action == 178u)
                                                     : primary_action_legal(g, action);
    if (!ok) {
      g.set_status(kNotLegal);
      return StepOut{kNotLegal, 0, g.done(), g.nagari(), 0};
    }
    begin_pending(g, action);
  }
  Peek next;
CB_NO_UNROLL
  for (u32 pass = choosing ? 0u : 1u; pass < 2u; ++pass) {
    next = peek_pending(g);
    if (pass == 1u || next.status != kOk) break;
    // A choosing row's first probe: the choice must be one of its floor cards.
    if (!choice_legal(next.choices).has(action)) {
      g.set_status(kNotLegal);
      return StepOut{kNotLegal, 0, g.done(), g.nagari(), 0};
    }
    if (next.decision == kDecPiCard) g.set_n_pi(g.n_pi() + 1u);
    else g.set_n_resolve(g.n_resolve() + 1u);
    g.set_n_choice(g.n_choice() + 1u);
    const u32 card = action - kChoiceBegin;
    if (next.decision == kDecFloorPlayed) g.set_pa_played_pick(card);
    else if (next.decision == kDecFloorDrawn) g.set_pa_drawn_pick(card);
  }
  if (next.status != kOk) {
    g.set_status(next.status);
    return StepOut{next.status, 0, g.done(), g.nagari(), 0};
  }
  if (next.decision == kDecNone) {
    commit_pending(g, next);
    if (g.pend_selected_pi() != 0) g.set_pa_pi_pick(g.pend_selected_pi());
    g.set_pend_active(0);
    const u32 k = g.pa_kind();
    g.set_n_primary(g.n_primary() + 1u);
    if (k == kActBonus) g.set_n_bonus(g.n_bonus() + 1u);
    if (k == kActShake || k == kActBomb || k == kActGrenade || k == kActCredit)
      g.set_n_special(g.n_special() + 1u);
    if (k == kActGo) g.set_n_go(g.n_go() + 1u);
    out.committed = 1;
  }
  g.set_status(kOk);
  refresh_done(g);
  out.reward0 = reward0(g);
  out.done = g.done();
  out.nagari = g.nagari();
  return out;
}

// ---- event diff, opening record, stock preview (torch50.h:644-698) -----------

struct EventBase {
  Mask hand0, hand1, stock, pile0, pile1, shown0, shown1;
};

CB_HD EventBase event_base(const Game& g) {
  return EventBase{g.hand(0), g.hand(1), g.stock(), g.pile(0), g.pile(1), g.shown(0), g.shown(1)};
}

// make_torch_event50 + pack_torch_event50 of a committed step.
CB_HD void event_words(const EventBase& b, const Game& g, i64* out) {
  const u32 a = g.pend_actor() & 1u;
  const Mask hb = a ? b.hand1 : b.hand0, ha = g.hand(a);
  const Mask played = hb & ~ha, drawn = ha & ~hb;
  out[0] = static_cast<i64>(played);
  out[1] = static_cast<i64>(drawn);
  out[2] = static_cast<i64>(b.stock & ~g.stock() & ~drawn);
  out[3] = static_cast<i64>(g.pile(0) & ~b.pile0);
  out[4] = static_cast<i64>(g.pile(1) & ~b.pile1);
  out[5] = static_cast<i64>(b.pile0 & ~g.pile(0));
  out[6] = static_cast<i64>(b.pile1 & ~g.pile(1));
  out[7] = static_cast<i64>(g.shown(a) & ~(a ? b.shown1 : b.shown0));
  out[8] = static_cast<i64>(a) | (static_cast<i64>(g.pa_kind()) << 8);
}

CB_HD void start_words(const Game& g, i64* out) {
  out[0] = static_cast<i64>(g.hand(0));
  out[1] = static_cast<i64>(g.hand(1));
  out[2] = static_cast<i64>(g.floor());
  out[3] = static_cast<i64>(g.pile(0));
  out[4] = static_cast<i64>(g.pile(1));
  out[5] = static_cast<i64>(g.mission());
  out[6] = static_cast<i64>(g.neutral_ppuk());
  out[7] = static_cast<i64>(g.mission_type()) | (static_cast<i64>(g.mission_mult()) << 8) |
           (static_cast<i64>(g.actor() & 1u) << 16) |
           (static_cast<i64>(g.mission_multi(0)) << 24) |
           (static_cast<i64>(g.mission_multi(1)) << 32);
}

// The next eight stock draws, one card id per byte, 0xFF past the first
// non-standard draw.
CB_HD u64 stock_preview(const Game& g) {
  Mask stock = g.stock();
  u64 rng = g.rng();
  u64 packed = ~0ull;
CB_NO_UNROLL
  for (u32 k = 0; k < 8; ++k) {
    const u32 c = draw_card(stock, rng);
    if (!is_standard(c)) break;
    packed &= ~(0xffull << (8 * k));
    packed |= static_cast<u64>(c) << (8 * k);
  }
  return packed;
}

// ---- a fresh game (make_torch_env50, cugo/game/torch50.h:218-236) ------------

// Mission card sets (cugo/game/terminal50.h:128-159, Hangame card n = id n - 1).
CB_HD Mask mission_set(u32 type, u32 index) {
  if (type == kMissionEasy) return index == 10u ? cards_of(8, 28) : cards_of(4 * index, 4 * index + 1);
  if (type == kMissionNormal) return month_cards(index);
  if (type != kMissionHard && type != kMissionTriple) return 0;
  // Hard sets 0..13; the triple list skips hard set 4 and orders 5.. differently.
  // (Switches rather than local arrays: a runtime-indexed local table would be
  // copied to every thread's stack.)
  if (type == kMissionTriple && index >= 4u) ++index;
  if (index < 5u) {
    switch (index) {
      case 0: return cards_of(21, 33, 37);
      case 1: return cards_of(1, 5, 9);
      case 2: return cards_of(13, 17, 25);
      case 3: return cards_of(4, 12, 29);
      default: return cards_of(32, 41, 47);
    }
  }
  if (index > 13u) return 0;
  // Hard 5..13 read tail sets 0..8; triple 5..13 read tail sets 8, 0..7.
  const u32 tail = type == kMissionTriple ? (index - 5u + 8u) % 9u : index - 5u;
  switch (tail) {
    case 0: return cards_of(20, 24, 36);
    case 1: return cards_of(0, 8, 28);
    case 2: return cards_of(0, 8, 40);
    case 3: return cards_of(0, 28, 40);
    case 4: return cards_of(8, 28, 40);
    case 5: return cards_of(4, 12, 45);
    case 6: return cards_of(4, 29, 45);
    case 7: return cards_of(12, 29, 45);
    default: return cards_of(4, 24, 45);
  }
}

CB_HD void create_game(Game& g, u64 seed, u32 first) {
  for (int i = 0; i < kRowWords; ++i) g.w[i] = 0;
  first &= 1u;
  u64 rng = seed;
  Mask rest = kFullDeck, h0 = 0, h1 = 0, fl = 0;
  for (int i = 0; i < 10; ++i) h0 |= card_bit(draw_card(rest, rng));
  for (int i = 0; i < 10; ++i) h1 |= card_bit(draw_card(rest, rng));
  for (int i = 0; i < 8; ++i) fl |= card_bit(draw_card(rest, rng));
  const u64 deal_rng = rng;
  // Floor bonus cards go to the first player; the floor is refilled.
  Mask first_pile = fl & kBonusCards;
  fl &= ~kBonusCards;
  u32 missing = popc(first_pile);
  while (missing > 0 && rest != 0) {
    const u32 c = draw_card(rest, rng);
    if (is_bonus(c)) {
      first_pile |= card_bit(c);
      continue;
    }
    fl |= card_bit(c);
    --missing;
  }
  g.set_hand(0, h0);
  g.set_hand(1, h1);
  g.set_floor(fl);
  g.set_stock(rest);
  g.set_pile(first, first_pile);
  g.set_rng(rng);
  g.set_actor(first);
  g.set_phase(kPhasePlay);
  g.set_played(kNoCard);
  g.set_drawn(kNoCard);
  g.set_neutral_ppuk(triple_months(fl));
  g.set_gostop_actor(kNobody);
  g.set_winner(kNobody);
  g.set_chong_actor(kNobody);
  g.set_end_winner(kNobody);
  g.set_round_raw(1);
  // Mission from a hash of the pre-refill deal stream (terminal50.h:164-183).
  u64 mrng = deal_rng ^ 0x6d697373696f6e35ull;
  const u32 kind = bounded_draw(mrng, 5u);
  const u32 mult = 2u + bounded_draw(mrng, 3u);
  // kind 0..4 -> Easy (11 sets), Normal (12), Hard (14), All (none), Triple (13).
  const u32 type = kind == 0 ? kMissionEasy
                 : kind == 1 ? kMissionNormal
                 : kind == 2 ? kMissionHard
                 : kind == 3 ? kMissionAll
                             : kMissionTriple;
  const u32 options = kind == 0 ? 11u : kind == 1 ? 12u : kind == 2 ? 14u : kind == 3 ? 0u : 13u;
  const u32 index = options == 0 ? 0u : bounded_draw(mrng, options);
  g.set_mission_type(type);
  g.set_mission_mult(type == kMissionTriple ? 0u : mult);
  g.set_mission(mission_set(type, index));
  if (type == kMissionAll) {
    g.set_mission_multi(0, mult);
    g.set_mission_multi(1, mult);
  }
  missions_update(g, 0, 0);
  missions_update(g, 1, 0);
  g.set_held(0, h0);
  g.set_held(1, h1);
  // Chongtong on the deal: a whole month on the floor, or in a hand.
  const u32 c0 = full_months(h0), c1 = full_months(h1), cf = full_months(fl);
  if (cf != 0) mark_end(g, first, kEndFloorChongtong, 10u);
  else if (c0 != 0 && c1 != 0) mark_end(g, first, kEndDealtChongtong, 10u);
  else if (c0 != 0) mark_end(g, 0, kEndDealtChongtong, 10u);
  else if (c1 != 0) mark_end(g, 1, kEndDealtChongtong, 10u);
  g.set_done(g.ended() ? 1u : 0u);
}

}  // namespace cb
