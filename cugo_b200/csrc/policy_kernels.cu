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
#include "gumbel.cuh"
#include "../../include/cugo_b200.h"

using namespace cb;

namespace {

// logits: [m, ld] fp32 (columns 0..178 are the policy logits); legal: [m, 179].
//
// The warp first compacts the row's legal actions (six ballots over the 179 mask
// bytes); lane j then takes the j-th legal action (j, j + 32, ... when a row has
// more than 32), so Philox and the two logarithms of the Gumbel noise run once per
// legal action instead of once per action.  Illegal actions cannot win and add
// exp(-1e30 - max) = 0 to the log-sum-exp, so leaving them out changes nothing.
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
  constexpr int kWords = (179 + 31) / 32;  // 6 ballots
  u32 bits[kWords];
  int n = 0;
#pragma unroll
  for (int k = 0; k < kWords; ++k) {
    const int a = lane + 32 * k;
    bits[k] = __ballot_sync(0xffffffffu, a < 179 && grow[a] != 0);
    n += __popc(bits[k]);
  }
  if (n == 0) {
    if (lane == 0) {
      action_out[row] = -1;
      logp_out[row] = 0.0f;
    }
    return;
  }
  const u64 g = static_cast<u64>(__ldg(game + row));
  const u32 d = static_cast<u32>(__ldg(decision + row));
  const u64 seed = static_cast<u64>(seed_base) + g;
  float best = -INFINITY, mx = -INFINITY;
  int best_a = -1;
  float xs[kWords];
#pragma unroll
  for (int c = 0; c < kWords; ++c) {
    xs[c] = -INFINITY;
    const int j = 32 * c + lane;  // this lane's rank among the legal actions
    if (32 * c < n && j < n) {
      int rank = j, a = -1;
#pragma unroll
      for (int k = 0; k < kWords; ++k) {
        const int cnt = __popc(bits[k]);
        if (a < 0 && rank < cnt) a = 32 * k + static_cast<int>(__fns(bits[k], 0u, rank + 1));
        else if (a < 0) rank -= cnt;
      }
      const float x = __ldg(lrow + a);
      float score = x;
      if (!greedy) {
        const Philox4 r = philox4x32_10(static_cast<u32>(g), static_cast<u32>(g >> 32), d,
                                        3u | (static_cast<u32>(a >> 2) << 8),
                                        static_cast<u32>(seed), static_cast<u32>(seed >> 32));
        const int q = a & 3;
        const u32 word = q == 0 ? r.v[0] : (q == 1 ? r.v[1] : (q == 2 ? r.v[2] : r.v[3]));
        score = x + gumbel_of(word);
      }
      xs[c] = x;
      mx = fmaxf(mx, x);
      if (score > best) {  // ascending actions per lane: the first maximum is the lowest
        best = score;
        best_a = a;
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
  }
  // log-sum-exp over the legal logits.
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < kWords; ++c)
    if (xs[c] != -INFINITY) s += expf(xs[c] - mx);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    action_out[row] = best_a;
    logp_out[row] = __ldg(lrow + best_a) - (mx + logf(s));
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
