// Seeded counter-based draws for the benchmark drivers (random-legal play,
// branch selection, Gumbel sampling).
//
// Philox4x32-10 as published by Salmon, Moraes, Dror and Shaw, "Parallel Random
// Numbers: As Easy as 1, 2, 3" (SC'11): ten rounds of two 32x32->64 multiplies
// with the published multipliers and Weyl key increments.  A draw is addressed
// by (game, decision, stream) under the game's seed, so any GPU thread, any
// rank, and the CPU oracle reproduce it without shared state:
//   counter = {game lo, game hi, decision, stream}, key = {seed lo, seed hi}.
#pragma once

#include "cards.cuh"

namespace cb {

struct Philox4 {
  u32 v[4];
};

CB_HD void mul_hi_lo(u32 a, u32 b, u32& hi, u32& lo) {
#if defined(__CUDA_ARCH__)
  hi = __umulhi(a, b);
  lo = a * b;
#else
  const u64 p = static_cast<u64>(a) * b;
  hi = static_cast<u32>(p >> 32);
  lo = static_cast<u32>(p);
#endif
}

CB_HD Philox4 philox4x32_10(u32 c0, u32 c1, u32 c2, u32 c3, u32 k0, u32 k1) {
  CB_UNROLL
  for (int round = 0; round < 10; ++round) {
    u32 hi0, lo0, hi1, lo1;
    mul_hi_lo(0xD2511F53u, c0, hi0, lo0);
    mul_hi_lo(0xCD9E8D57u, c2, hi1, lo1);
    const u32 n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return Philox4{{c0, c1, c2, c3}};
}

CB_HD Philox4 game_draw(u64 game, u32 decision, u32 stream, u64 seed) {
  return philox4x32_10(static_cast<u32>(game), static_cast<u32>(game >> 32), decision, stream,
                       static_cast<u32>(seed), static_cast<u32>(seed >> 32));
}

// Position of the floor(r * n / 2^32)-th set bit of a 179-bit mask held as
// three words (actions 0..63, 64..127, 128..178), or kNoCard-like 0xffff when empty.
CB_HD u32 pick_set_bit(u64 w0, u64 w1, u64 w2, u32 r) {
  const u32 c0 = popc(w0), c1 = popc(w1), c2 = popc(w2);
  const u32 n = c0 + c1 + c2;
  if (n == 0) return 0xffffu;
  const u32 rank = static_cast<u32>((static_cast<u64>(r) * n) >> 32);
  if (rank < c0) return nth_card(w0, rank);
  if (rank < c0 + c1) return 64u + nth_card(w1, rank - c0);
  return 128u + nth_card(w2, rank - c0 - c1);
}

}  // namespace cb
