// Policy-side kernels: masked Gumbel-max sampling of the unified action.
//
// The reference samples with softmax + torch.multinomial and takes the
// log-softmax of the chosen action (python/cugo_ppo50.py:74-82); its sequence
// self-play uses argmax(logits + Gumbel) (cugo_seq_selfplay50.py:126-130).
// Here one warp handles one row: masked logits (illegal -> -1e30, as the
// reference masks), Gumbel noise from Philox4x32-10 addressed by
// (game, decision, action block), argmax, and log p of the chosen action from a
// warp-wide log-sum-exp, in a single launch with no host synchronisation.
//
// Noise of action a at decision d of game i: word (a & 3) of
//   Philox4x32-10({i lo, i hi, d, 3 | (a >> 2) << 8}, {seed lo, seed hi}),
// u = (word >> 8 + 0.5) * 2^-24 in (0, 1), g = -log(-log(u)).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "engine/driver.cuh"
#include "../../include/cugo_b200.h"

using namespace cb;

namespace {

constexpr int kActionsPadded = 180;  // 45 blocks of 4 actions

__device__ __forceinline__ float gumbel_of(u32 word) {
  const float u = (static_cast<float>(word >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

// logits: [m, ld] fp32 (columns 0..178 are the policy logits); legal: [m, 179].
__global__ void __launch_bounds__(256) sample_kernel(const float* __restrict__ logits, int64_t ld,
                                                     const bool* __restrict__ legal, int64_t m,
                                                     const int64_t* __restrict__ game,
                                                     const int32_t* __restrict__ decision,
                                                     int64_t seed_base, int greedy,
                                                     int64_t* __restrict__ action_out,
                                                     float* __restrict__ logp_out) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= m) return;  // whole warps exit together
  const int lane = threadIdx.x & 31;
  const float* lrow = logits + row * ld;
  const uint8_t* grow = reinterpret_cast<const uint8_t*>(legal) + row * 179;
  const u64 g = static_cast<u64>(__ldg(game + row));
  const u32 d = static_cast<u32>(__ldg(decision + row));
  const u64 seed = static_cast<u64>(seed_base) + g;
  float best = -INFINITY;
  int best_a = -1;
  float mx = -INFINITY;
  float logit_of[8];
  int count = 0;
  // Lane l takes action blocks l and l + 32 (4 actions each).
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int blk = lane + 32 * pass;
    if (blk < kActionsPadded / 4) {
      Philox4 r{};
      if (!greedy) r = philox4x32_10(static_cast<u32>(g), static_cast<u32>(g >> 32), d,
                                     3u | (static_cast<u32>(blk) << 8), static_cast<u32>(seed),
                                     static_cast<u32>(seed >> 32));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int a = 4 * blk + j;
        float x = -1.0e30f;
        if (a < 179 && grow[a]) x = __ldg(lrow + a);
        logit_of[pass * 4 + j] = x;
        if (a < 179) {
          mx = fmaxf(mx, x);
          const float score = greedy ? x : x + gumbel_of(r.v[j]);
          if (grow[a] && score > best) {
            best = score;
            best_a = a;
          }
          count += grow[a] ? 1 : 0;
        }
      }
    }
  }
  // Warp argmax (lowest action on ties) and max.
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int oa = __shfl_xor_sync(0xffffffffu, best_a, off);
    if (ob > best || (ob == best && oa >= 0 && (best_a < 0 || oa < best_a))) {
      best = ob;
      best_a = oa;
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    count += __shfl_xor_sync(0xffffffffu, count, off);
  }
  // log-sum-exp over the masked logits (illegal ones contribute exp(-1e30 - mx) = 0).
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int a = 4 * (lane + 32 * (k >> 2)) + (k & 3);
    if (a < 179 && (lane + 32 * (k >> 2)) < kActionsPadded / 4) s += expf(logit_of[k] - mx);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    if (count == 0) {
      action_out[row] = -1;
      logp_out[row] = 0.0f;
    } else {
      action_out[row] = best_a;
      logp_out[row] = __ldg(lrow + best_a) - (mx + logf(s));
    }
  }
}

}  // namespace

extern "C" {

int cugo_b200_sample_actions(const float* logits, int64_t ld, const bool* legal, int64_t m,
                             const int64_t* game, const int32_t* decision, int64_t seed_base,
                             int32_t greedy, int64_t* actions, float* logp, cudaStream_t stream) {
  if (m < 0 || ld < 179) return CUGO_B200_ERR_ARG;
  if (m > 0 && (!logits || !legal || !game || !decision || !actions || !logp)) return CUGO_B200_ERR_ARG;
  if (m == 0) return CUGO_B200_OK;
  const unsigned blocks = static_cast<unsigned>((m + 7) / 8);
  sample_kernel<<<blocks, 256, 0, stream>>>(logits, ld, legal, m, game, decision, seed_base, greedy,
                                            actions, logp);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // extern "C"
