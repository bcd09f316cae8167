/* Seeded random-legal driver for the oracle (TEST INFRASTRUCTURE ONLY).
 *
 * The reference has no such driver: its rollouts use canonical actions or a
 * host LCG (tests/torch50_test.cpp:196-200).  The benchmark configurations
 * need one seeded, counter-based rule that a CPU oracle and the GPU engine can
 * both evaluate, so it is defined here in plain C and restated independently
 * in the product (cugo_b200/csrc/engine/driver.cuh):
 *
 *   game i      : seed = seed_base + i (12345 + i), first player = i & 1
 *   decision d  : counts every step call of the game from 0
 *   random word : Philox4x32-10(counter = {i lo, i hi, d, stream},
 *                               key     = {seed lo, seed hi})   (Salmon et al.,
 *                 "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11)
 *   legal pick  : with n legal actions, take the floor(r0 * n / 2^32)-th set
 *                 bit of the 179-bit mask in ascending action order
 *   event hash  : FNV-1a 64 over the little-endian bytes of the 8 start words,
 *                 then the 9 words of every committed event, in order
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this.
 */
#ifndef CUGO_ORACLE_DRIVER_H
#define CUGO_ORACLE_DRIVER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Philox4x32 round multipliers and Weyl key increments, as published. */
#define ORACLE_PHILOX_M0 0xD2511F53u
#define ORACLE_PHILOX_M1 0xCD9E8D57u
#define ORACLE_PHILOX_W0 0x9E3779B9u
#define ORACLE_PHILOX_W1 0xBB67AE85u

static inline void oracle_philox4x32_10(const uint32_t ctr_in[4],
                                        const uint32_t key_in[2],
                                        uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = (uint64_t)ORACLE_PHILOX_M0 * c0;
    const uint64_t p1 = (uint64_t)ORACLE_PHILOX_M1 * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += ORACLE_PHILOX_W0;
    k1 += ORACLE_PHILOX_W1;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* First output word for (game, decision, stream) under the game's seed. */
static inline uint32_t oracle_driver_word(uint64_t game, uint32_t decision,
                                          uint32_t stream, uint64_t seed) {
  const uint32_t ctr[4] = {(uint32_t)game, (uint32_t)(game >> 32), decision, stream};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t out[4];
  oracle_philox4x32_10(ctr, key, out);
  return out[0];
}

/* Index of the chosen action in a legal mask given as 179 bytes (0/1), or -1. */
static inline int oracle_pick_legal(const uint8_t* legal, int count, uint32_t r0) {
  int n = 0;
  for (int a = 0; a < count; ++a) n += legal[a] != 0;
  if (n == 0) return -1;
  uint32_t rank = (uint32_t)(((uint64_t)r0 * (uint32_t)n) >> 32);
  for (int a = 0; a < count; ++a) {
    if (!legal[a]) continue;
    if (rank == 0) return a;
    --rank;
  }
  return -1;
}

#define ORACLE_FNV_OFFSET 0xcbf29ce484222325ull
#define ORACLE_FNV_PRIME 0x100000001b3ull

static inline uint64_t oracle_fnv_words(uint64_t h, const int64_t* words, int count) {
  for (int w = 0; w < count; ++w) {
    uint64_t v = (uint64_t)words[w];
    for (int b = 0; b < 8; ++b) {
      h ^= (v >> (8 * b)) & 0xffu;
      h *= ORACLE_FNV_PRIME;
    }
  }
  return h;
}

#ifdef __cplusplus
}
#endif

#endif
