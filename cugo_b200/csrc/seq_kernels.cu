// Decode kernels of the event-sequence policy (sm_100a).
//
// The sequence policy (python/cugo_seq50.py:131-339) runs one token per cache row
// per call: an opening token, one token per committed event for each seat, and a
// query token per decision.  Its per-layer work around the GEMMs is here:
//
//   decode_attention_kernel  single-query attention over a bf16 KV cache
//                            (python/cugo_seq_attention50.py:22-62), optionally
//                            appending the token's own key/value to its slot in
//                            the same pass (the KV append of cached_step,
//                            python/cugo_seq50.py:313-316);
//   layernorm_kernel         LayerNorm of the fp32 residual stream into the bf16
//                            operand of the next GEMM (nn.LayerNorm under
//                            autocast: fp32 math, bf16 consumer);
//   event_embed_kernel       event tokens (encode_events + event_in + position +
//   start_embed_kernel       token type, python/cugo_seq50.py:91-129,271-289) as
//                            sums of the weight columns of the token's set bits:
//                            a token is a multi-hot vector with a few dozen ones
//                            among 414 (274) inputs, so a gather-sum reads ~30
//                            weight rows instead of running a K=414 GEMM.
//
//   encode_events_kernel     the observer-relative event tokens themselves
//                            (encode_events, python/cugo_seq50.py:91-109) for
//                            callers that feed them to their own layers;
//   games_attention_kernel   the attention of the training forward over whole
//                            games (SeqNet.forward_games, python/cugo_seq50.py:
//                            240-265): per (game, seat) sequence the opening,
//                            causal event tokens and one query per decision that
//                            sees the events visible at that decision and itself.
//
// All of them are memory- or latency-bound; they use warp-per-row (or
// warp-per-(query, head)) mappings with 16-byte accesses.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <atomic>
#include <stdint.h>

#include "../../include/cugo_b200.h"

namespace {

using i64 = int64_t;
using u64 = uint64_t;
using u32 = uint32_t;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kDh = 32;         // head width of the decode kernel (d_model 256 / 8 heads)
constexpr int kMaxSlots = 512;  // cache capacity the decode kernel accepts
constexpr int kEventIn = 8 * 50 + 12 + 2;   // python/cugo_seq50.py:37
constexpr int kStartIn = 5 * 50 + 12 + 8 + 4;  // python/cugo_seq50.py:38
constexpr int kMaxEvents = 48;               // python/cugo_seq50.py:34

__device__ __forceinline__ void bf16x8(const uint4 raw, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

// d += A B for one m16n8k16 tile (bf16 operands, fp32 accumulators) in the register
// fragments of mma.sync: a0..a3 rows (g, g + 8) x K columns (2c, 2c + 1, 2c + 8, 2c + 9),
// b0, b1 K rows (2c, 2c + 1), (2c + 8, 2c + 9) of column g; d rows g, g + 8 x columns
// 2c, 2c + 1 (g = lane / 4, c = lane % 4; the lower K index in the lower 16 bits).
__device__ __forceinline__ void mma_m16n8k16_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// ---- decode attention -------------------------------------------------------------
//
// One warp per (query i, head h).  Lanes 2j and 2j+1 own slot j of each group of 16
// slots, each for one 16-dimension half of the head: a lane loads its 32-byte halves
// of the slot's key and value rows, the pair adds its partial dot products with one
// shuffle, and every lane keeps a running max, sum and weighted value sum for its
// half (online softmax).  Two groups (32 slots) are loaded before either is used.
// The 16 slot states are then merged: a warp max, a rescale, a warp sum of the
// denominators and a butterfly reduce-scatter of the 16-wide value sums within each
// half (15 shuffles), after which lane l holds dimension 16 (l & 1) + (l >> 1).
// With an append, the lanes of slot pos[i] use the new key/value from registers
// and write them to the cache; the cache rows of different queries must then be
// distinct (as in cached_step).
__global__ void __launch_bounds__(256, 3) decode_attention_kernel(
    const __nv_bfloat16* __restrict__ q, i64 ldq, const __nv_bfloat16* __restrict__ k_new,
    const __nv_bfloat16* __restrict__ v_new, i64 ldn, __nv_bfloat16* keys, __nv_bfloat16* values,
    i64 n_rows, int heads, int slots, const i64* __restrict__ pos, i64 pos_clamp,
    const i64* __restrict__ rows, i64 n, float scale, __nv_bfloat16* __restrict__ out, i64 ldo,
    int32_t* error, const bool* __restrict__ active) {
  const i64 gw = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= n * heads) return;
  const int lane = threadIdx.x & 31, half = lane & 1, sl = lane >> 1;
  const i64 i = gw / heads;
  const int h = static_cast<int>(gw - i * heads);
  if (active && !active[i]) {  // an inactive query: zero output, no cache access
    out[i * ldo + h * kDh + lane] = __float2bfloat16_rn(0.0f);
    return;
  }
  const i64 r = rows ? __ldg(rows + i) : i;
  i64 p = -1;
  if (pos_clamp < 0) {
    p = __ldg(pos + i);
  } else if (r >= 0 && r < n_rows) {  // pos holds per-row lengths
    p = __ldg(pos + r);
    p = p < pos_clamp ? p : pos_clamp;
  }
  __nv_bfloat16* o = out + i * ldo + h * kDh;
  if (p < 0 || p >= slots || r < 0 || r >= n_rows) {
    o[lane] = __float2bfloat16_rn(0.0f);
    if (lane == 0 && error) atomicExch(error, 1);
    return;
  }
  float qf[16];
  {
    const uint4* qp = reinterpret_cast<const uint4*>(q + i * ldq + h * kDh + half * 16);
    bf16x8(__ldg(qp), qf);
    bf16x8(__ldg(qp + 1), qf + 8);
  }
  const i64 base = (r * heads + h) * static_cast<i64>(slots) * kDh;
  uint4* kc = reinterpret_cast<uint4*>(keys + base) + 2 * half;    // 4 uint4 per slot
  uint4* vc = reinterpret_cast<uint4*>(values + base) + 2 * half;
  const int last = static_cast<int>(p);
  float m = -INFINITY, l = 0.0f, acc[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) acc[d] = 0.0f;
  for (int t0 = 0; t0 <= last; t0 += 32) {
    uint4 kr[2][2], vr[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int t = t0 + 16 * u + sl;
      if (t > last) continue;
      if (k_new && t == last) {
        const uint4* kn = reinterpret_cast<const uint4*>(k_new + i * ldn + h * kDh + half * 16);
        const uint4* vn = reinterpret_cast<const uint4*>(v_new + i * ldn + h * kDh + half * 16);
        kr[u][0] = __ldg(kn);
        kr[u][1] = __ldg(kn + 1);
        vr[u][0] = __ldg(vn);
        vr[u][1] = __ldg(vn + 1);
        kc[4 * t] = kr[u][0];
        kc[4 * t + 1] = kr[u][1];
        vc[4 * t] = vr[u][0];
        vc[4 * t + 1] = vr[u][1];
      } else {
        kr[u][0] = __ldg(kc + 4 * t);
        kr[u][1] = __ldg(kc + 4 * t + 1);
        vr[u][0] = __ldg(vc + 4 * t);
        vr[u][1] = __ldg(vc + 4 * t + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int t = t0 + 16 * u + sl;
      float s = 0.0f;
      if (t <= last) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float kf[8];
          bf16x8(kr[u][c], kf);
#pragma unroll
          for (int e = 0; e < 8; ++e) s = fmaf(kf[e], qf[8 * c + e], s);
        }
      }
      s += __shfl_xor_sync(kFull, s, 1);  // both halves of the slot
      if (t <= last) {
        s *= scale;
        if (s > m) {
          const float c = expf(m - s);
          l *= c;
#pragma unroll
          for (int d = 0; d < 16; ++d) acc[d] *= c;
          m = s;
        }
        const float w = expf(s - m);
        l += w;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float vf[8];
          bf16x8(vr[u][c], vf);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[8 * c + e] = fmaf(w, vf[e], acc[8 * c + e]);
        }
      }
    }
  }
  // Merge the slot states (both lanes of a slot hold the same m and l).
  const float mx = warp_max(m);
  const float f = expf(m - mx);  // 0 for a lane without slots (m = -inf)
  const float denom = warp_sum(half == 0 ? l * f : 0.0f);
#pragma unroll
  for (int d = 0; d < 16; ++d) acc[d] *= f;
  // Butterfly reduce-scatter over lane bits 4..1 (same half): after the level of
  // width w the lane's acc[0..w-1] hold its half's dimensions
  // ((lane >> 1) & ~(w-1)) .. +w-1 summed over the lanes that differ from it only
  // in bits >= 2w of the lane id.
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
    const bool upper = (lane & (2 * w)) != 0;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const float send = upper ? acc[j] : acc[j + w];
      const float keep = upper ? acc[j + w] : acc[j];
      acc[j] = keep + __shfl_xor_sync(kFull, send, 2 * w);
    }
  }
  o[half * 16 + sl] = __float2bfloat16_rn(acc[0] / denom);
}

// ---- LayerNorm ----------------------------------------------------------------------
//
// One warp per row; lane l owns 4-column groups l, l+32, ... of the row.  Mean,
// then the mean squared deviation from it (two passes over registers), then
// (x - mean) * rsqrt(var + eps) * gamma + beta rounded to bf16.
template <int V>
__global__ void __launch_bounds__(256) layernorm_kernel(const float* __restrict__ x, i64 ldx,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps,
                                                        __nv_bfloat16* __restrict__ out, i64 ldo,
                                                        i64 n) {
  const i64 row = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const int lane = threadIdx.x & 31;
  constexpr int d = 128 * V;
  const float4* xr = reinterpret_cast<const float4*>(x + row * ldx);
  float4 v[V];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    v[j] = __ldg(xr + lane + 32 * j);
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  const float mean = warp_sum(s) / d;
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, e = v[j].w - mean;
    ss += (a * a + b * b) + (c * c + e * e);
  }
  const float rstd = rsqrtf(warp_sum(ss) / d + eps);
  uint2* orow = reinterpret_cast<uint2*>(out + row * ldo);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c4 = lane + 32 * j;
    const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c4);
    const float4 b = __ldg(reinterpret_cast<const float4*>(beta) + c4);
    const __nv_bfloat162 lo = __floats2bfloat162_rn((v[j].x - mean) * rstd * g.x + b.x,
                                                    (v[j].y - mean) * rstd * g.y + b.y);
    const __nv_bfloat162 hi = __floats2bfloat162_rn((v[j].z - mean) * rstd * g.z + b.z,
                                                    (v[j].w - mean) * rstd * g.w + b.w);
    uint2 raw;
    raw.x = *reinterpret_cast<const u32*>(&lo);
    raw.y = *reinterpret_cast<const u32*>(&hi);
    orow[c4] = raw;
  }
}

// ---- token embeddings ----------------------------------------------------------------
//
// Embedding rows are d_model = 256 * G wide; lane l owns columns g*256 + 8l .. +7
// of every group g.  `wt` is the transposed input weight, bf16 [inputs, d_model]
// (one 512-byte row per input column), so an active input adds one row.

template <int G>
struct Acc {
  float v[G][8];
};

template <int G>
__device__ __forceinline__ void acc_init(Acc<G>& a) {
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) a.v[g][e] = 0.0f;
}

// Adds the weight rows of every set bit of masks[k] (input column bases[k] + bit).
// The columns are taken eight at a time and their rows loaded together, so a token
// costs a few L2 round trips instead of one per active input.  The masks are the
// same for the whole warp, so the index walk is warp-uniform.
template <int G, int NM>
__device__ __forceinline__ void acc_masks(Acc<G>& a, const __nv_bfloat16* __restrict__ wt,
                                          u64 (&masks)[NM], const int (&bases)[NM]) {
  const int lane = threadIdx.x & 31;
  int k = 0;
  for (;;) {
    int col[8];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      while (k < NM && masks[k] == 0) ++k;
      col[j] = -1;
      if (k < NM) {
        const int b = __ffsll(static_cast<long long>(masks[k])) - 1;
        masks[k] &= masks[k] - 1;
        col[j] = bases[k] + b;
        ++cnt;
      }
    }
    uint4 raw[8][G];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (col[j] >= 0) {
        const uint4* src = reinterpret_cast<const uint4*>(wt + static_cast<i64>(col[j]) * (256 * G));
#pragma unroll
        for (int g = 0; g < G; ++g) raw[j][g] = __ldg(src + 32 * g + lane);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (col[j] >= 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float f[8];
          bf16x8(raw[j][g], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) a.v[g][e] += f[e];
        }
      }
    }
    if (cnt < 8) break;
  }
}

// Adds scale[j] x row col[j] for the (up to 5) scalar inputs, loaded together.
template <int G, int N>
__device__ __forceinline__ void acc_scaled(Acc<G>& a, const __nv_bfloat16* __restrict__ wt,
                                           const int (&col)[N], const float (&scale)[N]) {
  const int lane = threadIdx.x & 31;
  uint4 raw[N][G];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if (scale[j] != 0.0f) {
      const uint4* src = reinterpret_cast<const uint4*>(wt + static_cast<i64>(col[j]) * (256 * G));
#pragma unroll
      for (int g = 0; g < G; ++g) raw[j][g] = __ldg(src + 32 * g + lane);
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if (scale[j] != 0.0f) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float f[8];
        bf16x8(raw[j][g], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) a.v[g][e] = fmaf(scale[j], f[e], a.v[g][e]);
      }
    }
  }
}

// out row = acc + bias + pos_row + type_row, fp32.
template <int G>
__device__ __forceinline__ void acc_store(const Acc<G>& a, const float* __restrict__ bias,
                                          const float* __restrict__ pos_row,
                                          const float* __restrict__ type_row, float* out) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int c = 256 * g + 8 * lane;
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; e += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c + e));
      const float4 p = __ldg(reinterpret_cast<const float4*>(pos_row + c + e));
      const float4 t = __ldg(reinterpret_cast<const float4*>(type_row + c + e));
      r[e] = a.v[g][e] + b.x + p.x + t.x;
      r[e + 1] = a.v[g][e + 1] + b.y + p.y + t.y;
      r[e + 2] = a.v[g][e + 2] + b.z + p.z + t.z;
      r[e + 3] = a.v[g][e + 3] + b.w + p.w + t.w;
    }
    reinterpret_cast<float4*>(out + c)[0] = make_float4(r[0], r[1], r[2], r[3]);
    reinterpret_cast<float4*>(out + c)[1] = make_float4(r[4], r[5], r[6], r[7]);
  }
}

// Event token of row i: event words events[i % n_events], observer seat seats[i],
// events before it index[i % n_events] (position 1 + min(index, 47)).  Inputs:
// 8 card planes (played, drawn — own draws only, flipped, my gain, opponent gain,
// my loss, opponent loss, shown), one-hot kind (clamped to 11), "mine" flag and
// the opponent's drawn-card count (python/cugo_seq50.py:91-109).
template <int G>
__global__ void __launch_bounds__(256) event_embed_kernel(
    const i64* __restrict__ events, i64 n_events, const i64* __restrict__ seats,
    const i64* __restrict__ index, i64 n, const __nv_bfloat16* __restrict__ wt,
    const float* __restrict__ bias, const float* __restrict__ position,
    const float* __restrict__ type_row, float* __restrict__ out, i64 ldo) {
  const i64 i = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (i >= n) return;
  const i64 e = i % n_events;
  const i64* ev = events + e * 9;
  const i64 seat = __ldg(seats + i);
  const i64 header = __ldg(ev + 8);
  const bool me = (header & 0xFF) == seat;
  const i64 kind = (header >> 8) & 0xFF;
  const bool first = seat == 0;
  const u64 w[8] = {static_cast<u64>(__ldg(ev + 0)), static_cast<u64>(__ldg(ev + 1)),
                    static_cast<u64>(__ldg(ev + 2)), static_cast<u64>(__ldg(ev + 3)),
                    static_cast<u64>(__ldg(ev + 4)), static_cast<u64>(__ldg(ev + 5)),
                    static_cast<u64>(__ldg(ev + 6)), static_cast<u64>(__ldg(ev + 7))};
  Acc<G> a;
  acc_init(a);
  constexpr u64 k50 = (1ull << 50) - 1;
  u64 masks[8] = {w[0] & k50, me ? (w[1] & k50) : 0ull, w[2] & k50, (first ? w[3] : w[4]) & k50,
                  (first ? w[4] : w[3]) & k50, (first ? w[5] : w[6]) & k50,
                  (first ? w[6] : w[5]) & k50, w[7] & k50};
  const int bases[8] = {0, 50, 100, 150, 200, 250, 300, 350};
  acc_masks(a, wt, masks, bases);
  const int opp_drawn = me ? 0 : __popcll(w[1] & k50);
  const int cols[3] = {400 + static_cast<int>(kind < 11 ? kind : 11), 412, 413};
  const float scales[3] = {1.0f, me ? 1.0f : 0.0f, static_cast<float>(opp_drawn)};
  acc_scaled(a, wt, cols, scales);
  i64 at = index ? __ldg(index + e) : 0;
  at = at < 0 ? 0 : (at > kMaxEvents - 1 ? kMaxEvents - 1 : at);
  acc_store(a, bias, position + (1 + at) * (256 * G), type_row, out + i * ldo);
}

// Opening token of row i: start words start[i % n_start], observer seat seats[i]
// (python/cugo_seq50.py:112-128): planes own hand, floor, my captures, opponent
// captures, mission cards; 12 neutral-month bits; one-hot mission type (clamped
// to 7); multiplier / 4, "first mover is me", my and the opponent's multi / 8.
template <int G>
__global__ void __launch_bounds__(256) start_embed_kernel(
    const i64* __restrict__ start, i64 n_start, const i64* __restrict__ seats, i64 n,
    const __nv_bfloat16* __restrict__ wt, const float* __restrict__ bias,
    const float* __restrict__ pos_row, const float* __restrict__ type_row,
    float* __restrict__ out, i64 ldo) {
  const i64 i = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (i >= n) return;
  const i64* st = start + (i % n_start) * 8;
  const i64 seat = __ldg(seats + i);
  const bool first = seat == 0;
  const i64 header = __ldg(st + 7);
  Acc<G> a;
  acc_init(a);
  constexpr u64 k50 = (1ull << 50) - 1;
  u64 masks[6] = {static_cast<u64>(__ldg(st + (first ? 0 : 1))) & k50,
                  static_cast<u64>(__ldg(st + 2)) & k50,
                  static_cast<u64>(__ldg(st + (first ? 3 : 4))) & k50,
                  static_cast<u64>(__ldg(st + (first ? 4 : 3))) & k50,
                  static_cast<u64>(__ldg(st + 5)) & k50,
                  static_cast<u64>(__ldg(st + 6)) & 0xFFFull};
  const int bases[6] = {0, 50, 100, 150, 200, 250};
  acc_masks(a, wt, masks, bases);
  const i64 mtype = header & 0xFF;
  const i64 m24 = (header >> 24) & 0xFF, m32 = (header >> 32) & 0xFF;
  const int cols[5] = {262 + static_cast<int>(mtype < 7 ? mtype : 7), 270, 271, 272, 273};
  const float scales[5] = {1.0f, static_cast<float>((header >> 8) & 0xFF) / 4.0f,
                           (((header >> 16) & 1) == seat) ? 1.0f : 0.0f,
                           static_cast<float>(first ? m24 : m32) / 8.0f,
                           static_cast<float>(first ? m32 : m24) / 8.0f};
  acc_scaled(a, wt, cols, scales);
  acc_store(a, bias, pos_row, type_row, out + i * ldo);
}

bool aligned(const void* p, uintptr_t q) { return (reinterpret_cast<uintptr_t>(p) % q) == 0; }

int launch_status() { return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH; }

unsigned blocks_for_warps(i64 warps) { return static_cast<unsigned>((warps + 7) / 8); }

// encode_events (python/cugo_seq50.py:91-109): token (b, e) for e < length of
// sequence b, 414 columns: 8 card planes of 50 (played, drawn — the observer's own
// draws only, flipped, my gain, opponent gain, my loss, opponent loss, shown), the
// event kind one-hot (clamped to 11), "mine" and the opponent's drawn-card count;
// valid[b, e] = e < count[b].  Positions past the count are encoded from their
// (zero) words as the reference does.  A warp per token, lanes over columns.
template <typename T>
__global__ void __launch_bounds__(256) encode_events_kernel(
    const i64* __restrict__ events, i64 max_events, const i64* __restrict__ count,
    const i64* __restrict__ seats, i64 b_rows, int length, T* __restrict__ out,
    bool* __restrict__ valid) {
  const i64 tok = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= b_rows * length) return;
  const i64 b = tok / length;
  const int e = static_cast<int>(tok - b * length);
  const i64* ev = events + (b * max_events + e) * 9;
  const i64 seat = __ldg(seats + b);
  const i64 header = __ldg(ev + 8);
  const bool me = (header & 0xFF) == seat;
  const int kind = static_cast<int>((header >> 8) & 0xFF);
  const bool first = seat == 0;
  constexpr u64 k50 = (1ull << 50) - 1;
  const u64 w1 = static_cast<u64>(__ldg(ev + 1));
  const u64 masks[8] = {static_cast<u64>(__ldg(ev + 0)) & k50, me ? (w1 & k50) : 0ull,
                        static_cast<u64>(__ldg(ev + 2)) & k50,
                        static_cast<u64>(__ldg(ev + (first ? 3 : 4))) & k50,
                        static_cast<u64>(__ldg(ev + (first ? 4 : 3))) & k50,
                        static_cast<u64>(__ldg(ev + (first ? 5 : 6))) & k50,
                        static_cast<u64>(__ldg(ev + (first ? 6 : 5))) & k50,
                        static_cast<u64>(__ldg(ev + 7)) & k50};
  const float opp_drawn = me ? 0.0f : static_cast<float>(__popcll(w1 & k50));
  const int hot = 400 + (kind < 11 ? kind : 11);
  T* row = out + tok * kEventIn;
  for (int c = lane; c < kEventIn; c += 32) {
    float v;
    if (c < 400) {
      const int slot = c / 50;
      u64 m = masks[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) m = slot == k ? masks[k] : m;
      v = static_cast<float>((m >> (c - 50 * slot)) & 1ull);
    } else if (c < 412) {
      v = c == hot ? 1.0f : 0.0f;
    } else {
      v = c == 412 ? (me ? 1.0f : 0.0f) : opp_drawn;
    }
    if constexpr (sizeof(T) == 2) row[c] = __float2bfloat16_rn(v);
    else row[c] = v;
  }
  if (lane == 0 && valid) valid[tok] = e < __ldg(count + b);
}

// Attention of SeqNet.forward_games (python/cugo_seq50.py:240-265, _encode :200-222)
// for 8 heads of 32.  Token rows of the [qkv] buffer come in three blocks: the S
// openings (row s), the S x L events (row S + s L + e) and the S x Q decision
// queries (row S + S L + s Q + q).  The opening sees itself; event e sees the
// opening and events 0..e; query q sees the opening, the first min(seen[s, q], L)
// events and itself.
//
// One block per sequence (grid-stride): the keys and values of its opening and
// events — the keys every token of the sequence shares — are staged once in shared
// memory.  A warp item is (head, 32 consecutive tokens of the sequence), one token
// per lane: the lane holds its q (and, for a query, its own k and v) in registers
// and walks the shared keys in order with an online softmax.  At each step every
// lane reads the same key and value rows (shared-memory broadcasts), so the item
// runs without shuffles; lanes whose token sees fewer keys idle through the tail.
constexpr int kKvPitch = 256 + 8;  // bf16 per staged row (528 bytes)
constexpr int kGamesBlock = 128;

__device__ __forceinline__ void load_head(const __nv_bfloat16* p, float* f) {
#pragma unroll
  for (int q = 0; q < 4; ++q) bf16x8(__ldg(reinterpret_cast<const uint4*>(p) + q), f + 8 * q);
}

__global__ void __launch_bounds__(kGamesBlock, 4) games_attention_kernel(
    const __nv_bfloat16* __restrict__ qkv, i64 ldq, int n_seq, int length, int queries,
    const i64* __restrict__ seen, float scale, __nv_bfloat16* __restrict__ out, i64 ldo) {
  extern __shared__ uint4 kv_raw[];
  const int pre = 1 + length;  // opening + events
  __nv_bfloat16* kp = reinterpret_cast<__nv_bfloat16*>(kv_raw);
  __nv_bfloat16* vp = kp + pre * kKvPitch;
  const int warp = threadIdx.x >> 5, warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int tokens = pre + queries;
  const int groups = (tokens + 31) >> 5;
  const i64 ev0 = n_seq, q0 = (i64)n_seq + (i64)n_seq * length;
  for (int s = blockIdx.x; s < n_seq; s += gridDim.x) {
    __syncthreads();  // the previous sequence's readers are done with the stage
    for (int idx = threadIdx.x; idx < pre * 64; idx += blockDim.x) {
      const int row = idx >> 6, piece = idx & 63, part = piece >> 5, p = piece & 31;
      const i64 g = row == 0 ? (i64)s : ev0 + (i64)s * length + (row - 1);
      const uint4 val = __ldg(reinterpret_cast<const uint4*>(qkv + g * ldq + 256 * (1 + part)) + p);
      reinterpret_cast<uint4*>((part ? vp : kp) + row * kKvPitch)[p] = val;
    }
    __syncthreads();
    for (int item = warp; item < groups * 8; item += warps) {
      const int h = item & 7;
      const int i = (item >> 3) * 32 + lane;  // this lane's token
      const bool live = i < tokens;
      i64 r = 0;
      int n_pre = 0;
      bool self = false;
      if (live) {
        if (i == 0) {
          r = s;
          n_pre = 1;
        } else if (i <= length) {
          r = ev0 + (i64)s * length + (i - 1);
          n_pre = i + 1;
        } else {
          const int q = i - pre;
          r = q0 + (i64)s * queries + q;
          i64 sn = __ldg(seen + (i64)s * queries + q);
          sn = sn < 0 ? 0 : (sn > length ? length : sn);
          n_pre = 1 + static_cast<int>(sn);
          self = true;
        }
      }
      const __nv_bfloat16* row = qkv + r * ldq + h * kDh;
      float qv[kDh], acc[kDh];
      if (live) load_head(row, qv);
#pragma unroll
      for (int d = 0; d < kDh; ++d) {
        qv[d] = live ? qv[d] * scale : 0.0f;
        acc[d] = 0.0f;
      }
      float m = -INFINITY, l = 0.0f;
      int n_max = n_pre;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) n_max = max(n_max, __shfl_xor_sync(kFull, n_max, o));
      for (int j = 0; j < n_max; ++j) {
        const __nv_bfloat16* krow = kp + j * kKvPitch + h * kDh;
        float part[4];  // four independent chains instead of one 32-long one
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float kf[8];
          bf16x8(reinterpret_cast<const uint4*>(krow)[p], kf);
          part[p] = 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) part[p] = fmaf(qv[8 * p + e], kf[e], part[p]);
        }
        const float dot = (part[0] + part[1]) + (part[2] + part[3]);
        if (j < n_pre) {
          if (dot > m) {  // a new maximum: rescale what has been summed (rare after a few keys)
            const float c = __expf(m - dot);  // 0 on the first key (m = -inf)
            l *= c;
#pragma unroll
            for (int d = 0; d < kDh; ++d) acc[d] *= c;
            m = dot;
          }
          const float pj = __expf(dot - m);
          l += pj;
          const __nv_bfloat16* vrow = vp + j * kKvPitch + h * kDh;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            float vf[8];
            bf16x8(reinterpret_cast<const uint4*>(vrow)[p], vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[8 * p + e] = fmaf(pj, vf[e], acc[8 * p + e]);
          }
        }
      }
      if (self) {  // a query's own key and value, from its row
        float kf[kDh], vf[kDh];
        load_head(row + 256, kf);
        load_head(row + 512, vf);
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int d = 0; d < kDh; ++d) part[d & 3] = fmaf(qv[d], kf[d], part[d & 3]);
        const float dot = (part[0] + part[1]) + (part[2] + part[3]);
        const float m_new = fmaxf(m, dot);
        const float c = __expf(m - m_new), pj = __expf(dot - m_new);
        l = fmaf(l, c, pj);
#pragma unroll
        for (int d = 0; d < kDh; ++d) acc[d] = fmaf(acc[d], c, pj * vf[d]);
      }
      if (live) {
        const float inv = 1.0f / l;
        __nv_bfloat16* o = out + r * ldo + h * kDh;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint4 raw;
          __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            hh[e] = __floats2bfloat162_rn(acc[8 * p + 2 * e] * inv, acc[8 * p + 2 * e + 1] * inv);
          reinterpret_cast<uint4*>(o)[p] = raw;
        }
      }
    }
  }
}

// Dynamic shared memory of games_attention_kernel for `length` events.
constexpr int games_smem_bytes(int length) { return 2 * (1 + length) * kKvPitch * 2; }

// ---- decode attention, staged through shared memory by bulk copies ----------------
//
// For caches of up to kStagedSlots slots and up to kStagedHeads heads (the sequence
// policy's 50 slots and 8 heads).  A persistent block takes its queries in order (all
// heads of one query at a time).  The block reads every query's cache row and
// position first, then warp 0 keeps a ring of shared memory filled: each query takes
// 2 x heads x (pos + 1) x 64 contiguous bytes of the ring (its attended key slots of
// every head, then its value slots) followed by its query row and, with an append,
// its new key and value rows (heads x 64 bytes each), loaded by one bulk copy
// (cp.async.bulk) per head and tensor and one per row, all completing on the query's
// mbarrier -- as many queries in flight as the ring holds (a query's bytes grow with
// its position, so the ring is filled by bytes, not by a fixed number of stages).
// Nothing a query needs is read from global memory after its wait: under a saturated
// memory system a load issued there would cost a full round trip per query.  Warp h then works on head h from shared
// memory: four lanes per slot take the 32-dimension dot product of 8 slots per pass,
// the warp forms the softmax over the slots (fp32), and lane d sums the weighted
// values of dimension d.  With an append, the slot pos row is not copied: the new key
// and value go to the ring from the token's own k_new / v_new and to the cache in
// global memory.  Every wait is bounded (about 2 s on the global timer); a wait that
// gives up sets *error and the block stops after its copies in flight have landed.
constexpr int kStagedSlots = 64;
constexpr int kStagedHeads = 8;
constexpr int kStagedThreads = 32 * kStagedHeads;
constexpr int kRingItems = 16;          // queries in flight at most (one mbarrier each)
constexpr int kMaxItemsPerBlock = 64;  // queries a block takes (their rows and positions are prefetched)
constexpr uint64_t kStagedWaitNs = 2'000'000'000ull;

struct StageInfo {
  i64 row;  // cache row, -1 for an invalid query
  int pos;
  int pad;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool stage_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok = 0;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255u) == 255u && global_ns() - t0 > kStagedWaitNs) return false;
  }
}

// Persistent: block b takes queries b, b + grid, ... (at most kMaxItemsPerBlock).
__global__ void __launch_bounds__(kStagedThreads, 4) decode_attention_staged_kernel(
    const __nv_bfloat16* __restrict__ q, i64 ldq, const __nv_bfloat16* __restrict__ k_new,
    const __nv_bfloat16* __restrict__ v_new, i64 ldn, __nv_bfloat16* keys, __nv_bfloat16* values,
    i64 n_rows, int heads, int slots, const i64* __restrict__ pos, i64 pos_clamp,
    const i64* __restrict__ rows, i64 n, float scale, __nv_bfloat16* __restrict__ out, i64 ldo,
    int32_t* error, int ring_bytes, const bool* __restrict__ active) {
  extern __shared__ __align__(128) unsigned char smem[];
  // Layout: the ring, the per-warp slot weights, the items' rows and positions, the
  // ring offsets of the items in flight, their mbarriers.
  unsigned char* ring = smem;
  float* weights = reinterpret_cast<float*>(smem + ring_bytes);
  StageInfo* info = reinterpret_cast<StageInfo*>(weights + kStagedHeads * kStagedSlots);
  int* ring_off = reinterpret_cast<int*>(info + kMaxItemsPerBlock);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring_off + kRingItems);
  const int t = threadIdx.x, lane = t & 31, h = t >> 5;
  const i64 grid = gridDim.x;
  const int items = n > blockIdx.x ? static_cast<int>((n - blockIdx.x + grid - 1) / grid) : 0;
  for (int k = t; k < items; k += kStagedThreads) {
    const i64 i = blockIdx.x + k * grid;
    const i64 r = rows ? __ldg(rows + i) : i;
    i64 p = -1;
    if (r >= 0 && r < n_rows) {
      if (pos_clamp < 0) {
        p = __ldg(pos + i);
      } else {
        p = __ldg(pos + r);
        p = p < pos_clamp ? p : pos_clamp;
      }
    }
    const bool ok = p >= 0 && p < slots && r >= 0 && r < n_rows;
    const bool skip = active && !active[i];  // inactive: no copies, zero output, no error
    info[k].row = skip ? -2 : (ok ? r : -1);
    info[k].pos = ok && !skip ? static_cast<int>(p) : -1;
  }
  if (t == 0) {
    for (int s = 0; s < kRingItems; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // Ring bookkeeping, warp 0 (every lane keeps the same copy): items [consumed,
  // issued) are in flight, taking live_bytes bytes; the next one goes at `head` (or
  // wraps to 0).
  int issued = 0, head = 0, live_bytes = 0;
  const int row_bytes = heads * kDh * 2;  // one token's query (or key, or value) row
  const int token_rows = k_new ? 3 : 1;
  const auto item_bytes = [&](int k) {
    return info[k].row >= 0 ? (2 * (info[k].pos + 1) + token_rows) * row_bytes : 0;
  };
  // Item k's copies (warp 0): lane 0 posts the expected bytes on the item's mbarrier,
  // then lane j < 2 x heads copies the key (j < heads) or value slots of head j % heads,
  // lane 2 x heads the query row, lanes 2 x heads + 1 and + 2 the new key and value.
  const auto issue = [&](int k, int at) {
    const i64 r = info[k].row;
    uint64_t* bar = &full[k % kRingItems];
    const int p1 = info[k].pos + 1;
    const int copied = r >= 0 ? (k_new ? p1 - 1 : p1) : 0;
    const uint32_t bytes = static_cast<uint32_t>(copied) * kDh * 2;
    const uint32_t total =
        r >= 0 ? bytes * 2u * static_cast<uint32_t>(heads) + static_cast<uint32_t>(token_rows * row_bytes)
               : 0u;
    if (lane == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                   "r"(total)
                   : "memory");
    __syncwarp();
    if (r < 0) return;
    const void* from;
    unsigned char* dst;
    uint32_t size;
    if (lane < 2 * heads) {
      if (bytes == 0) return;
      const int hh = lane < heads ? lane : lane - heads;
      from = (lane < heads ? keys : values) + (r * heads + hh) * static_cast<i64>(slots) * kDh;
      dst = ring + at + (lane < heads ? hh : heads + hh) * p1 * kDh * 2;
      size = bytes;
    } else if (lane < 2 * heads + token_rows) {
      const int j = lane - 2 * heads;  // 0 query, 1 new key, 2 new value
      const i64 i = blockIdx.x + static_cast<i64>(k) * grid;
      from = j == 0 ? q + i * ldq : (j == 1 ? k_new : v_new) + i * ldn;
      dst = ring + at + (2 * heads * p1 * kDh * 2) + j * row_bytes;
      size = static_cast<uint32_t>(row_bytes);
    } else {
      return;
    }
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(from), "r"(size), "r"(smem_u32(bar))
        : "memory");
  };
  // Issues items while the ring has room (warp 0, every lane the same decisions;
  // `consumed`: the oldest live item).
  const auto fill = [&](int consumed) {
    while (issued < items && issued - consumed < kRingItems) {
      const int need = item_bytes(issued);
      int at;
      if (live_bytes == 0) {
        at = 0;
      } else {
        // The live bytes start at the oldest item in flight that holds any (an item
        // without bytes -- an invalid or inactive query -- may sit at an offset that
        // bounds nothing: a later item can have gone to offset 0 when the ring was
        // empty).  live_bytes > 0, so one exists before `issued`.
        int oldest = consumed;
        while (item_bytes(oldest) == 0) ++oldest;
        const int tail = ring_off[oldest % kRingItems];
        if (head > tail) {  // live bytes in [tail, head)
          if (head + need <= ring_bytes) at = head;
          else if (need <= tail) at = 0;
          else break;
        } else if (head < tail) {  // wrapped: live in [tail, end) and [0, head)
          if (head + need <= tail) at = head;
          else break;
        } else {
          break;  // head == tail with live bytes: the ring is full
        }
      }
      if (lane == 0) ring_off[issued % kRingItems] = at;
      head = at + need;
      live_bytes += need;
      issue(issued, at);
      ++issued;
    }
  };

  if (h == 0) fill(0);
  float* wrow = weights + h * kStagedSlots;
  bool failed = false;
  for (int k = 0; k < items; ++k) {
    if (!stage_wait(&full[k % kRingItems], static_cast<uint32_t>((k / kRingItems) & 1))) {
      failed = true;
      if (t == 0 && error) atomicExch(error, 1);
      break;
    }
    const i64 i = blockIdx.x + k * grid;
    const i64 r = info[k].row;
    const int p = info[k].pos;
    if (h < heads) {
      __nv_bfloat16* o = out + i * ldo + h * kDh;
      if (r < 0) {
        o[lane] = __float2bfloat16_rn(0.0f);
        if (r == -1 && lane == 0 && error) atomicExch(error, 1);
      } else {
        const int at = ring_off[k % kRingItems];
        __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(ring + at) + h * (p + 1) * kDh;
        __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(ring + at) + (heads + h) * (p + 1) * kDh;
        // The token rows behind the slots: query, then (append) new key and new value.
        const __nv_bfloat16* tok =
            reinterpret_cast<const __nv_bfloat16*>(ring + at) + 2 * heads * (p + 1) * kDh + h * kDh;
        if (k_new) {  // the token's own key and value: slot p of the ring and the cache
          const __nv_bfloat16 kn = tok[heads * kDh + lane];
          const __nv_bfloat16 vn = tok[2 * heads * kDh + lane];
          ks[p * kDh + lane] = kn;
          vs[p * kDh + lane] = vn;
          const i64 dst = ((r * heads + h) * static_cast<i64>(slots) + p) * kDh + lane;
          keys[dst] = kn;
          values[dst] = vn;
          __syncwarp();
        }
        // Scores on the tensor cores: mma.sync m16n8k16 (bf16 in, fp32 out) with the
        // block's 16 slots as the A rows and the query in every B column.  The 32
        // dimensions go in as two K steps in a permuted order (the same for A and B,
        // so the dot products are unchanged): lane (g, c) = (lane / 4, lane % 4) loads
        // dimensions 8c .. 8c + 7 of slots g and g + 8 as one 16-byte read each (a
        // warp reads 512 contiguous bytes: no bank conflicts) and the same 8 query
        // dimensions; its bf16 pairs are K columns (2c, 2c + 1) and (2c + 8, 2c + 9)
        // of the two steps.  Lane (g, c) gets the scores of slots g and g + 8 of the
        // block.  Rows past p read slot p and are masked.
        const int g = lane >> 2, c = lane & 3;
        const uint4 qb = reinterpret_cast<const uint4*>(tok)[c];
        const int nblk = (p >> 4) + 1;  // p < kStagedSlots = 64: at most 4 blocks
        float sc[kStagedSlots / 16][2];
        float mx = -INFINITY;
#pragma unroll
        for (int b = 0; b < kStagedSlots / 16; ++b) {
          if (b < nblk) {
            const int s0 = 16 * b + g, s1 = s0 + 8;
            const uint4 k0 = *reinterpret_cast<const uint4*>(ks + (s0 <= p ? s0 : p) * kDh + 8 * c);
            const uint4 k1 = *reinterpret_cast<const uint4*>(ks + (s1 <= p ? s1 : p) * kDh + 8 * c);
            float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma_m16n8k16_bf16(d, k0.x, k1.x, k0.y, k1.y, qb.x, qb.y);
            mma_m16n8k16_bf16(d, k0.z, k1.z, k0.w, k1.w, qb.z, qb.w);
            sc[b][0] = s0 <= p ? d[0] * scale : -INFINITY;
            sc[b][1] = s1 <= p ? d[2] * scale : -INFINITY;
            mx = fmaxf(mx, fmaxf(sc[b][0], sc[b][1]));
          }
        }
        // The four lanes of a row group hold the same scores: reduce over g only.
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
        float sum = 0.0f;
#pragma unroll
        for (int b = 0; b < kStagedSlots / 16; ++b) {
          if (b < nblk) {
            const float w0 = expf(sc[b][0] - mx), w1 = expf(sc[b][1] - mx);  // 0 past p
            sum += w0 + w1;
            if (c == 0) {
              wrow[16 * b + g] = w0;
              wrow[16 * b + g + 8] = w1;
            }
          }
        }
        sum += __shfl_xor_sync(kFull, sum, 4);
        sum += __shfl_xor_sync(kFull, sum, 8);
        sum += __shfl_xor_sync(kFull, sum, 16);
        __syncwarp();
        // Output: lane l sums dimensions 2 (l % 16), 2 (l % 16) + 1 over slots l / 16,
        // l / 16 + 2, ... (two partial sums per dimension in flight), then the two slot
        // halves meet by one shuffle; all additions in a fixed order.
        const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(vs) + (lane & 15);
        float ax0 = 0.0f, ay0 = 0.0f, ax1 = 0.0f, ay1 = 0.0f;
        int j = lane >> 4;
        for (; j + 2 <= p; j += 4) {
          const float2 v0 = __bfloat1622float2(vp[j * (kDh / 2)]);
          const float2 v1 = __bfloat1622float2(vp[(j + 2) * (kDh / 2)]);
          const float w0 = wrow[j], w1 = wrow[j + 2];
          ax0 = fmaf(w0, v0.x, ax0);
          ay0 = fmaf(w0, v0.y, ay0);
          ax1 = fmaf(w1, v1.x, ax1);
          ay1 = fmaf(w1, v1.y, ay1);
        }
        if (j <= p) {
          const float2 v0 = __bfloat1622float2(vp[j * (kDh / 2)]);
          ax0 = fmaf(wrow[j], v0.x, ax0);
          ay0 = fmaf(wrow[j], v0.y, ay0);
        }
        float ax = ax0 + ax1, ay = ay0 + ay1;
        const float bx = __shfl_xor_sync(kFull, ax, 16), by = __shfl_xor_sync(kFull, ay, 16);
        if (lane < 16) {
          const float inv = 1.0f / sum;
          reinterpret_cast<__nv_bfloat162*>(o)[lane] =
              __floats2bfloat162_rn((ax + bx) * inv, (ay + by) * inv);
        }
      }
    }
    __syncthreads();  // item k's ring bytes and the weights are free again
    if (h == 0) {
      live_bytes -= item_bytes(k);
      fill(k + 1);
    }
  }
  // After a failed wait (decided over the whole block, so every thread takes the same
  // barriers) let copies already issued land before the shared memory goes away.
  if (__syncthreads_or(failed) && t == 0)
    for (int k = 0; k < issued; ++k)
      stage_wait(&full[k % kRingItems], static_cast<uint32_t>((k / kRingItems) & 1));
  __syncthreads();
}

// The ring holds the largest query of this cache (2 x heads x slots x 64 bytes of slots
// and three token rows of heads x 64 bytes, so a query always fits an empty ring),
// rounded up to 1 KB: at the sequence policy's 8 heads and 50 slots four blocks (32
// warps) fit an SM.
int ring_bytes_for(int heads, int slots) {
  return ((2 * slots + 3) * heads * kDh * 2 + 1023) / 1024 * 1024;
}

size_t staged_smem_bytes(int heads, int slots) {
  return static_cast<size_t>(ring_bytes_for(heads, slots)) + kStagedHeads * kStagedSlots * 4 +
         kMaxItemsPerBlock * sizeof(StageInfo) + kRingItems * sizeof(int) +
         kRingItems * sizeof(uint64_t);
}

}  // namespace

extern "C" {

int cugo_b200_decode_attention_active(const void* q, int64_t ldq, const void* k_new,
                                      const void* v_new, int64_t ldn, void* keys, void* values,
                                      int64_t n_rows, int32_t heads, int32_t slots,
                                      int32_t head_dim, const int64_t* pos, int64_t pos_clamp,
                                      const int64_t* rows, int64_t n, float scale, void* out,
                                      int64_t ldo, const bool* active, int32_t* error,
                                      cudaStream_t stream) {
  if (n < 0 || heads <= 0 || slots <= 0 || slots > kMaxSlots || head_dim != kDh || n_rows <= 0)
    return CUGO_B200_ERR_ARG;
  if (n == 0) return CUGO_B200_OK;
  if (!q || !keys || !values || !pos || !out || (!k_new) != (!v_new)) return CUGO_B200_ERR_ARG;
  if (ldq < heads * kDh || ldo < heads * kDh || (k_new && ldn < heads * kDh)) return CUGO_B200_ERR_ARG;
  if (!aligned(q, 16) || ldq % 8 || !aligned(keys, 16) || !aligned(values, 16) || !aligned(out, 2) ||
      (k_new && (!aligned(k_new, 16) || !aligned(v_new, 16) || ldn % 8)))
    return CUGO_B200_ERR_ALIGN;
  // The staged kernel stores the output as bf16 pairs (4-byte aligned rows).
  if (heads <= kStagedHeads && slots <= kStagedSlots && aligned(out, 4) && ldo % 2 == 0 &&
      staged_smem_bytes(heads, slots) <= static_cast<size_t>(227 * 1024)) {
    const size_t smem = staged_smem_bytes(heads, slots);
    // The shared-memory opt-in is a per-device function attribute.
    static std::atomic<size_t> configured[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
    if (smem > configured[dev].load(std::memory_order_acquire)) {
      if (cudaFuncSetAttribute(decode_attention_staged_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return CUGO_B200_ERR_LAUNCH;
      configured[dev].store(smem, std::memory_order_release);
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_attention_staged_kernel,
                                                      kStagedThreads, smem) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    i64 grid = n < per_sm * sms ? n : static_cast<i64>(per_sm) * sms;
    if ((n + grid - 1) / grid > kMaxItemsPerBlock) grid = (n + kMaxItemsPerBlock - 1) / kMaxItemsPerBlock;
    decode_attention_staged_kernel<<<static_cast<unsigned>(grid), kStagedThreads, smem, stream>>>(
        static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k_new),
        static_cast<const __nv_bfloat16*>(v_new), ldn, static_cast<__nv_bfloat16*>(keys),
        static_cast<__nv_bfloat16*>(values), n_rows, heads, slots, pos, pos_clamp, rows, n, scale,
        static_cast<__nv_bfloat16*>(out), ldo, error, ring_bytes_for(heads, slots), active);
    return launch_status();
  }
  decode_attention_kernel<<<blocks_for_warps(n * heads), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k_new),
      static_cast<const __nv_bfloat16*>(v_new), ldn, static_cast<__nv_bfloat16*>(keys),
      static_cast<__nv_bfloat16*>(values), n_rows, heads, slots, pos, pos_clamp, rows, n, scale,
      static_cast<__nv_bfloat16*>(out), ldo, error, active);
  return launch_status();
}

int cugo_b200_decode_attention(const void* q, int64_t ldq, const void* k_new, const void* v_new,
                               int64_t ldn, void* keys, void* values, int64_t n_rows,
                               int32_t heads, int32_t slots, int32_t head_dim,
                               const int64_t* pos, int64_t pos_clamp, const int64_t* rows,
                               int64_t n, float scale, void* out, int64_t ldo, int32_t* error,
                               cudaStream_t stream) {
  return cugo_b200_decode_attention_active(q, ldq, k_new, v_new, ldn, keys, values, n_rows, heads,
                                           slots, head_dim, pos, pos_clamp, rows, n, scale, out,
                                           ldo, nullptr, error, stream);
}

int cugo_b200_layernorm(const float* x, int64_t ldx, const float* gamma, const float* beta,
                        int64_t d, float eps, void* out, int64_t ldo, int64_t n,
                        cudaStream_t stream) {
  if (n < 0 || (d != 128 && d != 256 && d != 512 && d != 1024) || ldx < d || ldo < d)
    return CUGO_B200_ERR_ARG;
  if (n == 0) return CUGO_B200_OK;
  if (!x || !gamma || !beta || !out) return CUGO_B200_ERR_ARG;
  if (!aligned(x, 16) || ldx % 4 || !aligned(gamma, 16) || !aligned(beta, 16) || !aligned(out, 8) ||
      ldo % 4)
    return CUGO_B200_ERR_ALIGN;
  const unsigned grid = blocks_for_warps(n);
  auto* o = static_cast<__nv_bfloat16*>(out);
  switch (d) {
    case 128: layernorm_kernel<1><<<grid, 256, 0, stream>>>(x, ldx, gamma, beta, eps, o, ldo, n); break;
    case 256: layernorm_kernel<2><<<grid, 256, 0, stream>>>(x, ldx, gamma, beta, eps, o, ldo, n); break;
    case 512: layernorm_kernel<4><<<grid, 256, 0, stream>>>(x, ldx, gamma, beta, eps, o, ldo, n); break;
    default: layernorm_kernel<8><<<grid, 256, 0, stream>>>(x, ldx, gamma, beta, eps, o, ldo, n); break;
  }
  return launch_status();
}

int cugo_b200_event_embed(const int64_t* events, int64_t n_events, const int64_t* seats,
                          const int64_t* index, int64_t n, const void* weight_t,
                          const float* bias, const float* position, const float* token_type,
                          int64_t d, float* out, int64_t ldo, cudaStream_t stream) {
  if (n < 0 || (n > 0 && n_events <= 0) || (d != 256 && d != 512) || ldo < d) return CUGO_B200_ERR_ARG;
  if (n == 0) return CUGO_B200_OK;
  if (!events || !seats || !weight_t || !bias || !position || !token_type || !out)
    return CUGO_B200_ERR_ARG;
  if (!aligned(weight_t, 16) || !aligned(bias, 16) || !aligned(position, 16) ||
      !aligned(token_type, 16) || !aligned(out, 16) || ldo % 4)
    return CUGO_B200_ERR_ALIGN;
  const unsigned grid = blocks_for_warps(n);
  const auto* w = static_cast<const __nv_bfloat16*>(weight_t);
  if (d == 256)
    event_embed_kernel<1><<<grid, 256, 0, stream>>>(events, n_events, seats, index, n, w, bias,
                                                    position, token_type, out, ldo);
  else
    event_embed_kernel<2><<<grid, 256, 0, stream>>>(events, n_events, seats, index, n, w, bias,
                                                    position, token_type, out, ldo);
  return launch_status();
}

int cugo_b200_start_embed(const int64_t* start, int64_t n_start, const int64_t* seats, int64_t n,
                          const void* weight_t, const float* bias, const float* position0,
                          const float* token_type, int64_t d, float* out, int64_t ldo,
                          cudaStream_t stream) {
  if (n < 0 || (n > 0 && n_start <= 0) || (d != 256 && d != 512) || ldo < d) return CUGO_B200_ERR_ARG;
  if (n == 0) return CUGO_B200_OK;
  if (!start || !seats || !weight_t || !bias || !position0 || !token_type || !out)
    return CUGO_B200_ERR_ARG;
  if (!aligned(weight_t, 16) || !aligned(bias, 16) || !aligned(position0, 16) ||
      !aligned(token_type, 16) || !aligned(out, 16) || ldo % 4)
    return CUGO_B200_ERR_ALIGN;
  const unsigned grid = blocks_for_warps(n);
  const auto* w = static_cast<const __nv_bfloat16*>(weight_t);
  if (d == 256)
    start_embed_kernel<1><<<grid, 256, 0, stream>>>(start, n_start, seats, n, w, bias, position0,
                                                    token_type, out, ldo);
  else
    start_embed_kernel<2><<<grid, 256, 0, stream>>>(start, n_start, seats, n, w, bias, position0,
                                                    token_type, out, ldo);
  return launch_status();
}

int64_t cugo_b200_event_inputs(void) { return kEventIn; }
int64_t cugo_b200_start_inputs(void) { return kStartIn; }

int cugo_b200_encode_events(const int64_t* events, int64_t max_events, const int64_t* count,
                            const int64_t* seats, int64_t b_rows, int32_t length, void* tokens,
                            int32_t tokens_bf16, bool* valid, cudaStream_t stream) {
  if (b_rows < 0 || length < 0 || length > max_events || max_events <= 0) return CUGO_B200_ERR_ARG;
  const i64 n = b_rows * length;
  if (n == 0) return CUGO_B200_OK;
  if (!events || !count || !seats || !tokens) return CUGO_B200_ERR_ARG;
  const unsigned grid = static_cast<unsigned>((n * 32 + 255) / 256);
  if (tokens_bf16)
    encode_events_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        events, max_events, count, seats, b_rows, length, static_cast<__nv_bfloat16*>(tokens), valid);
  else
    encode_events_kernel<float><<<grid, 256, 0, stream>>>(events, max_events, count, seats, b_rows,
                                                          length, static_cast<float*>(tokens), valid);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

int cugo_b200_games_attention(const void* qkv, int64_t ldq, int64_t n_seq, int32_t length,
                              int32_t queries, const int64_t* seen, float scale, void* out,
                              int64_t ldo, cudaStream_t stream) {
  if (n_seq < 0 || n_seq > INT32_MAX || length < 0 || length > kMaxEvents || queries < 0 ||
      ldq < 768 || ldo < 256)
    return CUGO_B200_ERR_ARG;
  if (n_seq == 0) return CUGO_B200_OK;
  if (!qkv || !out || (queries > 0 && !seen)) return CUGO_B200_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15u) || ldq % 8 || (reinterpret_cast<uintptr_t>(out) & 15u) ||
      ldo % 8)
    return CUGO_B200_ERR_ALIGN;
  const int smem = games_smem_bytes(length);
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(games_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             games_smem_bytes(kMaxEvents)) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const i64 cap = static_cast<i64>(sms) * 4;
  const unsigned grid = static_cast<unsigned>(n_seq < cap ? n_seq : cap);
  games_attention_kernel<<<grid, kGamesBlock, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(qkv), ldq, static_cast<int>(n_seq), length, queries, seen,
      scale, static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // extern "C"
