// Shin Matgo rules applied in place on a Game.
//
// The rules are the reference's (Hangame Shin Matgo as locked by the reference's
// rule tests); they must produce identical rows, so every function states the
// reference code it agrees with.  The structure is different: the reference
// stacks four state layers (turn/game/special/terminal) and makes each layer
// transactional by copying the whole state and committing on success
// (e.g. cugo/game/turn50.h:431, game50.h:290, terminal50.h:476, rollout50.h:238).
// Here a step first decides, without mutating anything (see peek_* in env.cuh),
// whether the action completes; only then is it applied, once, in place.  Every
// function below is therefore called only on a path that cannot fail, which is
// why none of them keeps a copy of the state.
#pragma once

#include "game.cuh"

namespace cb {

// ---- scoring (cugo/game/hwatu.h:132-199) ------------------------------------

struct Score {
  u32 bright, animal, ribbon, pi, points;
  bool meongtta;  // seven or more animals
};

// Pi units of a pile; the Gukjin adds two when it counts as a double pi.
CB_HD u32 pi_units(Mask pile, bool gukjin_pi) {
  u32 v = popc(pile & kPlainPi) + 2u * popc(pile & kDoublePi);
  v += (pile & card_bit(kBonusTwo)) ? 2u : 0u;
  v += (pile & card_bit(kBonusThree)) ? 3u : 0u;
  v += (gukjin_pi && (pile & card_bit(kGukjin))) ? 2u : 0u;
  return v;
}

CB_HD Score score_pile(Mask pile, bool gukjin_pi) {
  Score s;
  s.bright = popc(pile & kBrights);
  const Mask animals = pile & kAnimals & ~(gukjin_pi ? card_bit(kGukjin) : Mask{0});
  s.animal = popc(animals);
  s.ribbon = popc(pile & kRibbons);
  s.pi = pi_units(pile, gukjin_pi);
  u32 bright_pts = 0;
  if (s.bright == 3) bright_pts = (pile & card_bit(kRainBright)) ? 2u : 3u;
  else if (s.bright == 4) bright_pts = 4;
  else if (s.bright == 5) bright_pts = 15;
  u32 animal_pts = s.animal >= 5 ? s.animal - 4 : 0;
  if ((animals & kGodori) == kGodori) animal_pts += 5;
  u32 ribbon_pts = s.ribbon >= 5 ? s.ribbon - 4 : 0;
  if ((pile & kRedRibbons) == kRedRibbons) ribbon_pts += 3;
  if ((pile & kGrassRibbons) == kGrassRibbons) ribbon_pts += 3;
  if ((pile & kBlueRibbons) == kBlueRibbons) ribbon_pts += 3;
  const u32 pi_pts = s.pi >= 10 ? s.pi - 9 : 0;
  s.points = (bright_pts + animal_pts + ribbon_pts + pi_pts) & 0xffu;
  s.meongtta = s.animal >= 7;
  return s;
}

// ---- Gukjin role (cugo/game/gukjin_state.h:372-466) --------------------------

CB_HD bool gukjin_counts_pi(const Game& g, u32 p) {
  return (g.pile(p) & card_bit(kGukjin)) && (g.owner1() & gukjin_pi_flag(p));
}

CB_HD Score player_score(const Game& g, u32 p) {
  return score_pile(g.pile(p), gukjin_counts_pi(g, p));
}

CB_HD bool gukjin_undecided(const Game& g, u32 p) {
  return (g.pile(p) & card_bit(kGukjin)) &&
         !(g.owner1() & (gukjin_pi_flag(p) | gukjin_lock_flag(p)));
}

// One-time role decision; either answer locks it.
CB_HD void decide_gukjin(Game& g, u32 p, bool as_pi) {
  if (!gukjin_undecided(g, p)) return;
  g.set_owner1(g.owner1() | gukjin_lock_flag(p) | (as_pi ? gukjin_pi_flag(p) : 0u));
}

// Ask after the player's turn: >= 8 pi and the conversion reaches 7 points.
CB_HD bool gukjin_prompt_due(const Game& g, u32 p) {
  if (!gukjin_undecided(g, p)) return false;
  const Mask pile = g.pile(p);
  if (pi_units(pile, false) < 8u) return false;
  return score_pile(pile, true).points + g.go(p) >= 7u;
}

// The loser's undecided Gukjin is settled in the loser's favour.
CB_HD void settle_loser_gukjin(Game& g, u32 loser) {
  const u32 pi = pi_units(g.pile(loser), gukjin_counts_pi(g, loser));
  if (pi == 6u || pi == 7u) decide_gukjin(g, loser, true);
  else if (pi == 0u) decide_gukjin(g, loser, false);
}

// ---- Go/Stop prompts (cugo/game/game50.h:117-199) ----------------------------

CB_HD u64 go_multiplier(u32 go) {
  return go >= 3u ? (go - 2u >= 64u ? 0ull : (1ull << (go - 2u))) : 1ull;
}

// Score a player would stop with: (base + go) * go multiplier * 2^(bombs + shakes)
// (cugo/game/special50.h:107-119).
CB_HD u32 shake_count(const Game& g, u32 p) {
  return (popc16(g.shaken(p)) + popc16(g.shaken4(p))) & 0xffu;
}

CB_HD u64 pow2_u8(u32 n) { return n >= 64u ? 0ull : (1ull << n); }

CB_HD u64 stop_value(const Game& g, u32 p) {
  const u32 go = g.go(p);
  const u64 after_go = (static_cast<u64>(player_score(g, p).points) + go) * go_multiplier(go);
  return after_go * pow2_u8((g.bombs(p) + shake_count(g, p)) & 0xffu);
}

// maybe_open_go_stop_decision50: reaching the threshold opens Go/Stop, or stops
// automatically on the last two turns.
CB_HD bool open_gostop(Game& g, u32 a) {
  if (a > 1u || g.decided() || g.prompt_pending()) return false;
  const u32 base = player_score(g, a).points;
  const u32 go = g.go(a);
  const bool eligible = go == 0 ? base >= 7u : base > g.last_go(a);
  if (!eligible) return false;
  settle_loser_gukjin(g, a ^ 1u);
  if (g.turn() > 18u) {
    g.set_winner(a);
    return false;
  }
  g.set_gostop_actor(a);
  return true;
}

// finish_turn_game50: the Gukjin prompt first, then Go/Stop.
CB_HD void after_turn(Game& g, u32 a) {
  if (a > 1u || g.decided() || g.prompt_pending()) return;
  if (gukjin_prompt_due(g, a)) {
    g.set_gukjin_prompt(a + 1u);
    return;
  }
  open_gostop(g, a);
}

// ---- game end bookkeeping (cugo/game/terminal50.h:104-362) -------------------

constexpr u32 kMissionEasy = 1, kMissionNormal = 2, kMissionHard = 3, kMissionAll = 4,
              kMissionTriple = 6;

CB_HD void mark_end(Game& g, u32 winner, u32 reason, u64 points) {
  g.set_end_winner(winner & 1u);
  g.set_end_reason(reason);
  g.set_end_points(points);
  g.set_chong_actor(kNobody);
  g.set_chong_months(0);
  g.set_gostop_actor(kNobody);
  g.set_gukjin_prompt(0);
}

// sync_game_stop50: a decided Go/Stop becomes the game's end.
CB_HD void sync_stop(Game& g) {
  if (g.ended() || !g.decided()) return;
  const u32 w = g.winner();
  g.set_end_winner(w);
  g.set_end_reason(kEndStop);
  g.set_end_points(stop_value(g, w));
}

CB_HD void side_payment(Game& g, u32 receiver, i32 base) {
  const i32 amount = base * static_cast<i32>(g.round_mult());
  g.set_side0(g.side0() + ((receiver & 1u) == 0 ? amount : -amount));
}

// update_missions50 after the player acquired cards.
CB_HD void missions_update(Game& g, u32 p, Mask acquired) {
  const Mask mission = g.mission();
  const Mask mine = g.pile(p);
  if (g.mission_type() == kMissionTriple) {
    g.set_mission_multi(p, (1u << popc(mission & mine)) & 0xffu);
    return;
  }
  if (mission == 0 || (acquired & mission) == 0) return;
  if ((mission & ~mine) == 0) g.set_mission_multi(p, g.mission_mult());
}

// Ppuk streak states (cugo/game/terminal50.h:24-32).
constexpr u32 kPpukNone = 0, kPpukFirst = 1, kPpukSecond = 2, kPpukThird = 3, kPpukOne = 4,
              kPpukTwo = 5, kPpukThree = 6;

// record_completed_turn_ppuk50: 7/14/21 payments for the first player's opening
// ppuk chain; any third ppuk ends the game.  `turn` is already advanced.
CB_HD void record_ppuk(Game& g, u32 a) {
  if (g.ended()) return;
  a &= 1u;
  const u32 count = g.ppuk_count(a);
  if (count != 0xffu) g.set_ppuk_count(a, count + 1u);
  const u32 t = g.turn();
  u32 s = g.ppuk_streak(a);
  switch (s) {
    case kPpukNone: s = t <= 1u ? kPpukFirst : kPpukOne; break;
    case kPpukFirst: s = t <= 3u ? kPpukSecond : kPpukTwo; break;
    case kPpukSecond: s = t <= 5u ? kPpukThird : kPpukThree; break;
    case kPpukOne: s = kPpukTwo; break;
    case kPpukTwo: s = kPpukThree; break;
    default: break;
  }
  g.set_ppuk_streak(a, s);
  if (s == kPpukFirst || s == kPpukSecond || s == kPpukThird)
    side_payment(g, a, 7 * static_cast<i32>(s));
  if (s == kPpukThird || s == kPpukThree) mark_end(g, a, kEndThreePpuk, 7u);
}

// ---- card resolution against the floor (cugo/game/turn50.h:198-508) ----------

constexpr u32 kEvPpuk = 1, kEvJjok = 2, kEvTtadak = 4, kEvSweep = 8;

struct Tally {
  u32 events = 0;
  u32 own_ppuk = 0;   // own ppuk stacks captured
  u32 opp_ppuk = 0;   // opponent or ownerless ppuk stacks captured
  Mask captured = 0;  // everything this turn put into the actor's pile
  bool last = false;  // the turn is one of the last two
};

// Two floor candidates that are both plain pi are interchangeable: the lower
// card is taken automatically.
CB_HD bool auto_pick(Mask matches) {
  return popc(matches) == 2 && (matches & ~kPlainPi) == 0;
}

CB_HD bool in_set(Mask set, u32 c) { return c < 64u && (set & card_bit(c)); }

CB_HD void capture(Game& g, Mask cards, Tally& t) {
  const u32 a = g.actor();
  g.set_pile(a, g.pile(a) | cards);
  t.captured |= cards;
}

// resolve_card_against_floor50.  Only called with a pick that is complete for
// this card (a two-card match has a valid `pick` or is an automatic pair).
CB_HD void resolve_card(Game& g, u32 card, u32 pick, Tally& t) {
  const Mask b = card_bit(card);
  const Mask matches = g.floor_std() & month_cards(card_month(card));
  const u32 n = popc(matches);
  if (n == 0) {
    g.set_floor(g.floor() | b);
    return;
  }
  Mask take;
  if (n == 1) {
    take = matches;
  } else if (n == 2) {
    if (auto_pick(matches) && !in_set(matches, pick)) pick = lowest_card(matches);
    take = card_bit(pick);
  } else {
    take = matches;
    const u32 mb = month_bit(card);
    if (g.ppuk_months() & mb) {
      // A ppuk stack carries the bonus cards that were flipped onto it.
      if (g.ppuk_bonus2() & mb) take |= card_bit(kBonusTwo);
      if (g.ppuk_bonus3() & mb) take |= card_bit(kBonusThree);
      g.set_ppuk_bonus2(g.ppuk_bonus2() & ~mb);
      g.set_ppuk_bonus3(g.ppuk_bonus3() & ~mb);
      const u32 owner = (g.owner1() & mb) ? 1u : 0u;
      if (owner == g.actor()) ++t.own_ppuk;
      else ++t.opp_ppuk;
      g.set_ppuk_months(g.ppuk_months() & ~mb);
      g.set_owner1(g.owner1() & ~mb);
    } else if (g.neutral_ppuk() & mb) {
      g.set_neutral_ppuk(g.neutral_ppuk() & ~mb);
      ++t.opp_ppuk;
    }
  }
  g.set_floor(g.floor() & ~take);
  capture(g, take | b, t);
}

// End of a turn: the other player moves next.
CB_HD void close_turn(Game& g) {
  g.set_played(kNoCard);
  g.set_drawn(kNoCard);
  g.set_flip_bonus(0);
  g.set_phase(kPhasePlay);
  g.set_actor(g.actor() ^ 1u);
  g.set_turn(g.turn() + 1u);
}

// resolve_turn50: the played and the drawn card against the floor, with ppuk,
// ttadak, jjok and sweep.  Phase must be kPhaseResolve.  Without a played card
// (a bomb, grenade or bomb credit) only the drawn card and its bonus cards resolve
// (the draw-only resolution of a special play, cugo/game/special50.h:140-158).
CB_HD void resolve_turn(Game& g, u32 played_pick, u32 drawn_pick, Tally& t) {
  const u32 played = g.played(), drawn = g.drawn();
  const bool has_played = played != kNoCard;
  const Mask pm = has_played ? g.floor_std() & month_cards(card_month(played)) : Mask{0};
  const u32 pmc = popc(pm);
  const bool same = has_played && card_month(played) == card_month(drawn);
  t.last = g.last_turn();
  const Mask pair = (has_played ? card_bit(played) : Mask{0}) | card_bit(drawn);
  const Mask bonus = g.flip_bonus();
  if (same && pmc == 1 && !t.last) {
    // Ppuk: the three cards of the month stay on the floor as a stack.
    g.set_floor(g.floor() | pair | bonus);
    const u32 mb = month_bit(played);
    g.set_ppuk_months(g.ppuk_months() | mb);
    g.set_owner1(g.actor() == 0 ? (g.owner1() & ~mb) : (g.owner1() | mb));
    if (bonus & card_bit(kBonusTwo)) g.set_ppuk_bonus2(g.ppuk_bonus2() | mb);
    if (bonus & card_bit(kBonusThree)) g.set_ppuk_bonus3(g.ppuk_bonus3() | mb);
    t.events |= kEvPpuk;
  } else if (same && pmc == 2) {
    g.set_floor(g.floor() & ~pm);
    capture(g, pm | pair | bonus, t);
    t.events |= kEvTtadak;
  } else if (same && pmc == 0) {
    capture(g, pair | bonus, t);
    if (!t.last) t.events |= kEvJjok;
  } else {
    if (has_played) resolve_card(g, played, played_pick, t);
    resolve_card(g, drawn, drawn_pick, t);
    if (bonus) capture(g, bonus, t);
  }
  if (g.floor() == 0 && t.captured != 0) t.events |= kEvSweep;
  close_turn(g);
}

// resolve_pi_steal_card_count: one per jjok, ttadak, sweep, opponent/neutral
// ppuk, two per own ppuk, one per captured bonus card; none on the last turns.
CB_HD u32 steal_count(const Tally& t) {
  if (t.last) return 0;
  u32 n = t.opp_ppuk + 2u * t.own_ppuk;
  n += (t.events & kEvJjok) ? 1u : 0u;
  n += (t.events & kEvTtadak) ? 1u : 0u;
  n += (t.events & kEvSweep) ? 1u : 0u;
  n += popc(t.captured & kBonusCards);
  return n & 0xffu;
}

// Takes the `count` lowest cards of `pool`.
CB_HD Mask take_lowest(Mask pool, u32& count) {
  Mask out = 0;
  while (pool != 0 && count != 0) {
    const Mask low = pool & (~pool + 1);
    out |= low;
    pool ^= low;
    --count;
  }
  return out;
}

// hangame_pi_steal_selection50: lowest pi value first, non-mission before
// mission on ties (all non-mission first when the victim owns the whole
// mission), ties broken by card id.
CB_HD Mask select_stolen_pi(Mask candidates, Mask mission, bool owns_mission, u32 count) {
  const Mask by_value[3] = {kPlainPi, kDoublePi | card_bit(kBonusTwo) | card_bit(kGukjin),
                            card_bit(kBonusThree)};
  Mask chosen = 0;
CB_UNROLL
  for (u32 key = 0; key < 6; ++key) {
    const bool in_mission = owns_mission ? key >= 3u : (key & 1u) != 0;
    const u32 value = owns_mission ? key % 3u : key / 2u;
    const Mask pool = candidates & by_value[value] & (in_mission ? mission : ~mission);
    chosen |= take_lowest(pool, count);
  }
  return chosen;
}

// apply_pi_steal50 with the automatic selection: returns the cards moved.
CB_HD Mask steal_pi(Game& g, u32 thief, u32 requested) {
  thief &= 1u;
  const u32 victim = thief ^ 1u;
  const Mask vpile = g.pile(victim);
  const Mask cand = (vpile & (kPlainPi | kDoublePi | kBonusCards)) |
                    (gukjin_counts_pi(g, victim) ? (vpile & card_bit(kGukjin)) : 0);
  const u32 avail = popc(cand);
  if (requested == 0) return 0;
  if (avail == 0) {
    decide_gukjin(g, victim, false);
    return 0;
  }
  Mask transfer = cand;
  if (avail > requested) {
    const Mask mission = g.mission();
    const bool owns = mission != 0 && (mission & ~vpile) == 0;
    transfer = select_stolen_pi(cand, mission, owns, requested);
  }
  g.set_pile(victim, vpile & ~transfer);
  g.set_pile(thief, g.pile(thief) | transfer);
  if (transfer & card_bit(kGukjin))
    g.set_owner1(g.owner1() & ~(gukjin_pi_flag(thief) | gukjin_pi_flag(victim)));
  if (avail < requested) decide_gukjin(g, victim, false);
  return transfer;
}

// ---- stock flips -------------------------------------------------------------

// draw_stock_with_bonus_chain: bonus cards flipped on the way are collected.
struct Flip {
  u32 card;      // the standard card flipped, kNoCard if the stock ran out
  Mask bonuses;  // bonus cards flipped before it
};

CB_HD Flip flip_stock(Mask& stock, u64& rng) {
  Flip f{kNoCard, 0};
  while (stock != 0) {
    const u32 c = draw_card(stock, rng);
    if (is_bonus(c)) {
      f.bonuses |= card_bit(c);
      continue;
    }
    f.card = c;
    break;
  }
  return f;
}

// ---- special plays (cugo/game/special50.h:63-106) ----------------------------

// Months where the actor holds `in_hand` cards and the floor `on_floor`.
CB_HD u32 special_months(const Game& g, u32 in_hand, u32 on_floor) {
  const u64 hc = month_counts(g.hand(g.actor()));
  const u64 fc = month_counts(g.floor_std());
  return months_with_count(hc, in_hand) & months_with_count(fc, on_floor);
}

// Shakes: three (or all four) cards of a month absent from the floor, not yet
// shaken at that size.
CB_HD u32 shake_months(const Game& g) {
  const u32 a = g.actor();
  return (special_months(g, 3, 0) & ~g.shaken(a)) | (special_months(g, 4, 0) & ~g.shaken4(a));
}
CB_HD u32 bomb_months(const Game& g) { return special_months(g, 3, 1); }
CB_HD u32 grenade_months(const Game& g) { return special_months(g, 2, 2); }

}  // namespace cb
