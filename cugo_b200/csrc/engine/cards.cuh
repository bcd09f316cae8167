// Card encoding, card classes, the stock random stream and bit utilities.
//
// Card ids follow the reference contract (cugo/core/card.h:14-30): a standard
// card is month * 4 + slot (0..47), 48 is the two-pi bonus and 49 the three-pi
// bonus; a set of cards is a 64-bit mask.  The card classes are the Hwatu deck's
// (cugo/game/hwatu.h:18-90) and the stock stream is SplitMix64 with Lemire's
// bounded draw (cugo/core/rng.h:13-54), because a state row must evolve exactly
// as the reference's does.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define CB_HD __host__ __device__ __forceinline__
#define CB_DEV __device__ __forceinline__
#else
#define CB_HD inline
#define CB_DEV inline
#endif

#if defined(__CUDACC__)
#define CB_HDC __host__ __device__ constexpr
#else
#define CB_HDC constexpr
#endif

#if defined(__CUDACC__)
#define CB_UNROLL _Pragma("unroll")
#define CB_NO_UNROLL _Pragma("unroll 1")
#else
#define CB_UNROLL
#define CB_NO_UNROLL
#endif

namespace cb {

using u8 = uint8_t;
using u16 = uint16_t;
using u32 = uint32_t;
using u64 = uint64_t;
using i32 = int32_t;
using i64 = int64_t;
using Mask = uint64_t;

constexpr u32 kNoCard = 0xffu;
constexpr u32 kBonusTwo = 48u;
constexpr u32 kBonusThree = 49u;
constexpr Mask kStandardDeck = (Mask{1} << 48) - 1;
constexpr Mask kBonusCards = Mask{3} << 48;
constexpr Mask kFullDeck = (Mask{1} << 50) - 1;

CB_HDC Mask cards_of(u32 a, u32 b, u32 c = 64, u32 d = 64, u32 e = 64) {
  return (Mask{1} << a) | (Mask{1} << b) | (c < 64 ? Mask{1} << c : 0) |
         (d < 64 ? Mask{1} << d : 0) | (e < 64 ? Mask{1} << e : 0);
}

// Card classes by id (month * 4 + slot).
constexpr Mask kBrights = cards_of(0, 8, 28, 40, 44);
constexpr u32 kRainBright = 44;
constexpr Mask kAnimals = cards_of(4, 12, 16, 20, 24) | cards_of(29, 32, 36, 45);
constexpr u32 kGukjin = 32;  // the September animal that may count as a double pi
constexpr Mask kRibbons = cards_of(1, 5, 9, 13, 17) | cards_of(21, 25, 33, 37, 46);
// Plain pi: slots 2 and 3 of months 0..10.
constexpr Mask kPlainPi = 0x0000'0ccc'cccc'ccccull;
constexpr Mask kDoublePi = cards_of(41, 47);
constexpr Mask kGodori = cards_of(4, 12, 29);
constexpr Mask kRedRibbons = cards_of(1, 5, 9);
constexpr Mask kGrassRibbons = cards_of(13, 17, 25);
constexpr Mask kBlueRibbons = cards_of(21, 33, 37);

static_assert((kBrights | kAnimals | kRibbons | kPlainPi | kDoublePi) == kStandardDeck,
              "card classes cover the standard deck");
static_assert((kBrights & kAnimals) == 0 && (kAnimals & kRibbons) == 0 &&
                  (kBrights & kRibbons) == 0 && (kPlainPi & kDoublePi) == 0,
              "card classes are disjoint");

CB_HD Mask card_bit(u32 c) { return Mask{1} << c; }
CB_HD u32 card_month(u32 c) { return c >> 2; }
CB_HD Mask month_cards(u32 m) { return Mask{0xf} << (4u * m); }
CB_HD u32 month_bit(u32 c) { return 1u << (c >> 2); }
CB_HD bool is_standard(u32 c) { return c < 48u; }
CB_HD bool is_bonus(u32 c) { return c == kBonusTwo || c == kBonusThree; }
CB_HD bool is_card(u32 c) { return c < 50u; }

CB_HD u32 popc(Mask m) {
#if defined(__CUDA_ARCH__)
  return static_cast<u32>(__popcll(m));
#else
  return static_cast<u32>(__builtin_popcountll(m));
#endif
}

CB_HD u32 popc16(u32 m) {
#if defined(__CUDA_ARCH__)
  return static_cast<u32>(__popc(m));
#else
  return static_cast<u32>(__builtin_popcount(m));
#endif
}

// Lowest card of a set, kNoCard when empty.
CB_HD u32 lowest_card(Mask m) {
#if defined(__CUDA_ARCH__)
  return m == 0 ? kNoCard : static_cast<u32>(__ffsll(static_cast<long long>(m)) - 1);
#else
  return m == 0 ? kNoCard : static_cast<u32>(__builtin_ctzll(m));
#endif
}

// The rank-th (0-based) card of a set in ascending id order, kNoCard if absent.
CB_HD u32 nth_card(Mask m, u32 rank) {
#if defined(__CUDA_ARCH__)
  const u32 lo = static_cast<u32>(m);
  const u32 nlo = static_cast<u32>(__popc(lo));
  if (rank < nlo) return __fns(lo, 0u, static_cast<int>(rank) + 1);
  const u32 hi = static_cast<u32>(m >> 32);
  const u32 r = rank - nlo;
  if (r >= static_cast<u32>(__popc(hi))) return kNoCard;
  return __fns(hi, 0u, static_cast<int>(r) + 1) + 32u;
#else
  if (rank >= popc(m)) return kNoCard;
  for (u32 k = 0; k < rank; ++k) m &= m - 1;
  return lowest_card(m);
#endif
}

// Per-month card counts of a standard-card set packed as 12 nibbles
// (month m's count in bits 4m..4m+3).
CB_HD u64 month_counts(Mask m) {
  m &= kStandardDeck;
  m = m - ((m >> 1) & 0x5555'5555'5555'5555ull);
  return (m & 0x3333'3333'3333'3333ull) + ((m >> 2) & 0x3333'3333'3333'3333ull);
}

// 12-bit month set of the nibbles of `counts` equal to `value` (0..4).
CB_HD u32 months_with_count(u64 counts, u32 value) {
  const u64 x = counts ^ (0x1111'1111'1111ull * value);  // zero nibble where equal
  // A nibble is zero iff (nibble | nibble>>1 | nibble>>2 | nibble>>3) & 1 == 0.
  const u64 any = (x | (x >> 1) | (x >> 2) | (x >> 3)) & 0x1111'1111'1111ull;
  const u64 eq = any ^ 0x1111'1111'1111ull;
  // Compress bit 4m into bit m.
  u32 out = 0;
CB_UNROLL
  for (u32 mo = 0; mo < 12; ++mo) out |= static_cast<u32>((eq >> (4 * mo)) & 1u) << mo;
  return out;
}

// Months whose four cards are all in the set.
CB_HD u32 full_months(Mask m) { return months_with_count(month_counts(m), 4); }

// Months with exactly three cards of the set.
CB_HD u32 triple_months(Mask m) { return months_with_count(month_counts(m), 3); }

// ---- stock stream: SplitMix64 + Lemire bounded draws -------------------------

CB_HD u64 splitmix_next(u64& state) {
  u64 z = (state += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Uniform integer in [0, bound) by multiply-shift with rejection of the biased
// low products (Lemire 2019); bound <= 1 draws nothing.
CB_HD u32 bounded_draw(u64& state, u32 bound) {
  if (bound <= 1u) return 0u;
  for (;;) {
    const u32 x = static_cast<u32>(splitmix_next(state) >> 32);
    const u64 prod = static_cast<u64>(x) * bound;
    const u32 low = static_cast<u32>(prod);
    if (low < bound && low < (0u - bound) % bound) continue;
    return static_cast<u32>(prod >> 32);
  }
}

// Removes and returns a uniformly drawn card of `pool` (kNoCard if empty).
CB_HD u32 draw_card(Mask& pool, u64& state) {
  const u32 n = popc(pool);
  if (n == 0) return kNoCard;
  const u32 c = nth_card(pool, bounded_draw(state, n));
  pool &= ~card_bit(c);
  return c;
}

}  // namespace cb
