// Warp tiles of game rows in shared memory, shared by the batch-environment and
// driver kernels.
//
// Kernel shape: 128-thread blocks, one game per thread, one 32-game tile per warp.
// A warp moves its 32 rows (248-byte TorchEnv50 images, 31 u64 words) between HBM
// and shared memory cooperatively — gathered with asynchronous 8-byte copies through
// the id list, written back row by row or, for a full tile of rows in order, with
// one 7,936-byte bulk copy — each thread runs the rule code on its row held in
// registers, writes its observation packet straight into the tile, and the warp
// writes the 32 feature rows and the legal-mask block with vector stores.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "engine/env.cuh"

namespace cb {
namespace tile {

constexpr int kWarpsPerBlock = 4;
constexpr int kBlock = 32 * kWarpsPerBlock;
constexpr unsigned kFull = 0xffffffffu;

// Per-warp shared staging: the 32 row images, reused for the 32 packets.
struct alignas(16) WarpTile {
  union {
    u64 rows[32][kRowWords];
    struct {
      u32 bits[32][kBitWords + 1];  // odd stride: conflict-free per-lane stores
      float scal[32][kScalarColumns];
    } pk;
  };
  u64 legal[32][3];
};
static_assert(sizeof(WarpTile) <= 9 * 1024, "tile fits the shared budget");

__device__ __forceinline__ WarpTile* block_tiles() {
  __shared__ WarpTile tiles[kWarpsPerBlock];
  return tiles;
}

__device__ __forceinline__ WarpTile& my_tile() { return block_tiles()[threadIdx.x >> 5]; }

// The tile holding row r (0..127) of the block.
__device__ __forceinline__ WarpTile& tile_of_block_row(int r) { return block_tiles()[r >> 5]; }

// Row id this lane's game reads: ids[row] for indexed ops, row itself otherwise;
// -1 past the end of the batch or for an id outside [0, n_states).
__device__ __forceinline__ i64 lane_source(const i64* ids, i64 row, i64 m, i64 n_states) {
  if (row >= m) return -1;
  const i64 id = ids ? __ldg(ids + row) : row;
  return (id >= 0 && id < n_states) ? id : -1;
}

// Gathers the warp's 32 source rows into the tile (zero rows for missing ids).
// Asynchronous 8-byte copies (cp.async) put all 32 rows in flight at once
// instead of a load -> shared store chain per word.
__device__ __forceinline__ void gather_rows(WarpTile& t, const u64* __restrict__ src, i64 my_src) {
  const int lane = threadIdx.x & 31;
  // Branching reads one parent for many children: when every lane names the same
  // row, fetch it once and replicate it in shared memory.
  const i64 id0 = __shfl_sync(kFull, my_src, 0);
  if (__all_sync(kFull, my_src == id0) && id0 >= 0) {
    const u64 w = lane < kRowWords ? __ldg(src + id0 * kRowWords + lane) : 0ull;
#pragma unroll 8
    for (int r = 0; r < 32; ++r)
      if (lane < kRowWords) t.rows[r][lane] = w;
    __syncwarp();
    return;
  }
#pragma unroll 8
  for (int r = 0; r < 32; ++r) {
    const i64 id = __shfl_sync(kFull, my_src, r);
    if (lane < kRowWords) {
      if (id >= 0) {
        const u32 dst = static_cast<u32>(__cvta_generic_to_shared(&t.rows[r][lane]));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst),
                     "l"(src + id * kRowWords + lane)
                     : "memory");
      } else {
        t.rows[r][lane] = 0ull;
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
}

// Writes tile rows back to dst[dst_row] for every lane whose dst_row >= 0.
__device__ __forceinline__ void scatter_rows(const WarpTile& t, u64* __restrict__ dst, i64 my_dst) {
  __syncwarp();
  const int lane = threadIdx.x & 31;
#pragma unroll 8
  for (int r = 0; r < 32; ++r) {
    const i64 id = __shfl_sync(kFull, my_dst, r);
    if (id >= 0 && lane < kRowWords) dst[id * kRowWords + lane] = t.rows[r][lane];
  }
}

// Writes the tile's 32 rows to the contiguous rows dst[0..31] (7,936 bytes) with one
// bulk copy from shared memory when dst is 16-byte aligned; false (nothing written)
// otherwise.  The tile's rows were written by every lane (store_game) before.
__device__ __forceinline__ bool store_tile_bulk(const WarpTile& t, u64* __restrict__ dst) {
  if (reinterpret_cast<uintptr_t>(dst) & 15u) return false;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the bulk copy
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                 "r"(static_cast<u32>(__cvta_generic_to_shared(&t.rows[0][0]))),
                 "r"(32u * kRowWords * 8u)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    // The tile may be reused (or the warp may exit) once the copy has read it;
    // its global writes complete with the grid.
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncwarp();
  return true;
}

// Rows of a full 32-row tile go to contiguous destination rows `base`..`base + 31`
// in one bulk copy; otherwise (partial tile, unaligned pointer) row by row.
__device__ __forceinline__ void store_tile(const WarpTile& t, u64* __restrict__ dst, i64 base,
                                          i64 m, i64 my_dst) {
  __syncwarp();
  if (base + 32 <= m && store_tile_bulk(t, dst + base * kRowWords)) return;
  scatter_rows(t, dst, my_dst);
}

__device__ __forceinline__ void load_game(const WarpTile& t, Game& g) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kRowWords; ++k) g.w[k] = t.rows[lane][k];
}

__device__ __forceinline__ void store_game(WarpTile& t, Game g) {
  zero_padding(g);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kRowWords; ++k) t.rows[lane][k] = g.w[k];
}

// Row r of a tile (another lane's, or another warp's tile).
__device__ __forceinline__ void load_game_row(const WarpTile& t, int r, Game& g) {
#pragma unroll
  for (int k = 0; k < kRowWords; ++k) g.w[k] = t.rows[r][k];
}

__device__ __forceinline__ void store_game_row(WarpTile& t, int r, Game g) {
  zero_padding(g);
#pragma unroll
  for (int k = 0; k < kRowWords; ++k) t.rows[r][k] = g.w[k];
}

// This lane's packet slice of the tile (valid once every lane has loaded its row).
__device__ __forceinline__ PacketRef lane_packet(WarpTile& t) {
  const int lane = threadIdx.x & 31;
  return PacketRef{t.pk.bits[lane], t.pk.scal[lane]};
}

__device__ __forceinline__ void store_legal(WarpTile& t, const Legal& legal) {
  const int lane = threadIdx.x & 31;
  t.legal[lane][0] = legal.w0;
  t.legal[lane][1] = legal.w1;
  t.legal[lane][2] = legal.w2;
}

__device__ __forceinline__ void store4(float* row, int q, const float* v) {
  __stcs(reinterpret_cast<float4*>(row) + q, make_float4(v[0], v[1], v[2], v[3]));
}

__device__ __forceinline__ void store4(__nv_bfloat16* row, int q, const float* v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(v[2], v[3]);
  uint2 raw;
  raw.x = *reinterpret_cast<const u32*>(&lo);
  raw.y = *reinterpret_cast<const u32*>(&hi);
  __stcs(reinterpret_cast<uint2*>(row) + q, raw);
}

// Cooperative write of the tile's feature rows: row `base + r` for r < rows.
// Lane l owns 4-column groups l, l+32, ... of every row (fp32 or bf16 rows).
template <typename F>
__device__ __forceinline__ void emit_features(const WarpTile& t, F* __restrict__ out, i64 ld,
                                              i64 base, int rows) {
  __syncwarp();
  const int lane = threadIdx.x & 31;
  // Per lane: for each of its 24 columns, the scalar slot or (word, bit).
  int slot[6][4];
  u32 word[6][4], bitpos[6][4];
#pragma unroll
  for (int k = 0; k < 6; ++k)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const u32 c = 4u * (lane + 32u * k) + j;
      slot[k][j] = c < kFeatures ? scalar_slot(c) : -1;
      word[k][j] = c >> 5;
      bitpos[k][j] = c & 31u;
    }
  for (int r = 0; r < rows; ++r) {
    F* row = out + (base + r) * ld;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      const int q = lane + 32 * k;
      if (q < (int)(kFeatures / 4)) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[j] = slot[k][j] >= 0 ? t.pk.scal[r][slot[k][j]]
                                 : ((t.pk.bits[r][word[k][j]] >> bitpos[k][j]) & 1u ? 1.0f : 0.0f);
        store4(row, q, v);
      }
    }
  }
}

// Cooperative write of bits 0 .. nbits-1 of the tile's per-row `legal` words as
// bf16 0/1 into columns 720 .. 720 + cols - 1 of each feature row (bits past nbits
// read 0): the legal mask for the sequence policy's query input [features, legal]
// (python/cugo_seq50.py:196-208), or the opponent's hand plane for the critic's
// input [features, hand] (python/cugo_ppo50.py:478-482).
__device__ __forceinline__ void emit_legal_columns(const WarpTile& t, __nv_bfloat16* __restrict__ out,
                                                   i64 ld, i64 base, int rows, int cols,
                                                   u32 nbits = kActions) {
  const int lane = threadIdx.x & 31;
  const int groups = cols >> 3;
  for (int k = lane; k < rows * groups; k += 32) {
    const int r = k / groups, g = k - r * groups;
    u32 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const u32 a0 = 8u * g + 2u * e, a1 = a0 + 1u;
      const u32 b0 = a0 < nbits ? static_cast<u32>((t.legal[r][a0 >> 6] >> (a0 & 63)) & 1ull) : 0u;
      const u32 b1 = a1 < nbits ? static_cast<u32>((t.legal[r][a1 >> 6] >> (a1 & 63)) & 1ull) : 0u;
      h[e] = (b0 ? 0x3F80u : 0u) | ((b1 ? 0x3F80u : 0u) << 16);  // bf16 1.0 = 0x3F80
    }
    __stcs(reinterpret_cast<uint4*>(out + (base + r) * ld + kFeatures) + g,
           make_uint4(h[0], h[1], h[2], h[3]));
  }
}

// Cooperative write of the tile's legal masks (bool [rows, 179], contiguous
// from row `base`); whole 4-byte words, then the tail bytes.
__device__ __forceinline__ void emit_legal(const WarpTile& t, bool* __restrict__ out, i64 base,
                                           int rows) {
  const int lane = threadIdx.x & 31;
  uint8_t* block = reinterpret_cast<uint8_t*>(out) + base * (i64)kActions;
  const int bytes = rows * (int)kActions;
  const int words = bytes >> 2;
  for (int wi = lane; wi < words; wi += 32) {
    u32 v = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = 4 * wi + j;
      const int r = b / (int)kActions, a = b - r * (int)kActions;
      const u64 w = t.legal[r][a >> 6];
      v |= static_cast<u32>((w >> (a & 63)) & 1ull) << (8 * j);
    }
    reinterpret_cast<u32*>(block)[wi] = v;
  }
  for (int b = 4 * words + lane; b < bytes; b += 32) {
    const int r = b / (int)kActions, a = b - r * (int)kActions;
    block[b] = static_cast<uint8_t>((t.legal[r][a >> 6] >> (a & 63)) & 1ull);
  }
}

__device__ __forceinline__ u32 torch_action(i64 raw) {
  return raw >= 0 && raw < (i64)kActions ? static_cast<u32>(raw) : kNoAction;
}

}  // namespace tile
}  // namespace cb
