// Kernels of the PPO update step (the reference's PpoUpdater._step,
// python/cugo_ppo50.py:558-623, plain policy target) around its GEMMs, and their
// C ABI (include/cugo_b200.h).
//
//   ppo_loss_kernel        the clipped-surrogate policy loss, entropy bonus and
//                          smooth-L1 value loss of a minibatch and their gradients
//                          in one pass: warp per row over the 179 masked logits
//                          (max, log-sum-exp, the action's log p, entropy), the
//                          row's d loss / d logits written as bf16 (the operand of
//                          the head's data-gradient GEMM) and d loss / d value as
//                          fp32; the minibatch means of the five statistics are
//                          accumulated per block and added with one atomic each
//   act_backward_colsum    dz = du * act'(z) (bf16) with the column sums of dz (the
//                          bias gradient) in the same pass
//   colsum                 column sums of a bf16 matrix (bias gradients of the
//                          residual stream)
//   scalar_head_backward   the backward of a one-output head g -> v = w . act(h) + b
//                          for the critic: dh = v' w * act'(h) with its column sums,
//                          the weight gradient sum_i v'_i act(h_i) and the bias
//                          gradient sum_i v'_i, in one pass over h
//
// Column sums: a block owns a range of rows and all columns, each thread 8
// consecutive columns (one 16-byte load per row), partial sums in registers, then
// one partial per column and block in the caller's scratch, summed in block order
// by a second launch (the same sums on every run, graph replay included).  Bias gradients
// are sums over the minibatch of bf16 values accumulated in fp32, as the
// reference's backward under bf16 autocast sums them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "../../include/cugo_b200.h"

namespace {

using i64 = int64_t;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kActions = 179;

enum Act : int { kActNone = 0, kActRelu = 1, kActSilu = 2 };

__device__ __forceinline__ void bf16x8(const uint4 raw, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
  return raw;
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

// act(z) and act'(z) of the networks' activations (SiLU: z sigmoid(z); its
// derivative s (1 + z (1 - s))).
__device__ __forceinline__ float act_value(float z, int act) {
  if (act == kActRelu) return z > 0.0f ? z : 0.0f;
  if (act == kActSilu) return __fdividef(z, 1.0f + __expf(-z));
  return z;
}

__device__ __forceinline__ float act_slope(float z, int act) {
  if (act == kActRelu) return z > 0.0f ? 1.0f : 0.0f;
  if (act == kActSilu) {
    // Fast exponential and divide (a few ulp, far below the bf16 rounding of the
    // stored gradient); IEEE division made this kernel compute-bound.
    const float s = __fdividef(1.0f, 1.0f + __expf(-z));
    return s * (1.0f + z * (1.0f - s));
  }
  return 1.0f;
}

// ---- the PPO losses and their gradients ---------------------------------------------

struct LossArgs {
  const float* logits;  // [b, ldl]
  i64 ldl;
  const bool* legal;    // [b, 179]
  const i64* actions;
  const float* logp_old;
  const float* adv;
  const float* value;   // [b] (row stride value_ld)
  i64 value_ld;
  const float* ret;
  i64 b;
  float clip, inv_b;
  const float* entropy_coef;  // device scalar (a graph keeps its address)
  float value_coef;
  __nv_bfloat16* dlogits;  // [b, ldd], columns 179 .. ldd - 1 written as 0
  i64 ldd;
  float* dvalue;           // [b]
  float* stats;            // [5]: policy loss, value loss, entropy, KL, clip fraction (means)
};

constexpr int kLossWarps = 8;

__global__ void __launch_bounds__(32 * kLossWarps) ppo_loss_kernel(LossArgs a) {
  __shared__ float part[kLossWarps][5];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const i64 row = (i64)blockIdx.x * kLossWarps + warp;
  float acc[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  if (row < a.b) {
    const float* lg = a.logits + row * a.ldl;
    const bool* lm = a.legal + row * kActions;
    // Lane l owns actions l, l + 32, ... (6 per lane; masked: -1e30, as the reference).
    float x[6];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      const int c = lane + 32 * k;
      x[k] = c < kActions ? (lm[c] ? lg[c] : -1.0e30f) : -INFINITY;
      mx = fmaxf(mx, x[k]);
    }
    mx = warp_max(mx);
    float se = 0.0f;
#pragma unroll
    for (int k = 0; k < 6; ++k) se += __expf(x[k] - mx);  // exp(-inf) = 0 past 179
    se = warp_sum(se);
    const float lse = mx + __logf(se);
    // p_j, log p_j and the entropy -sum p log p (masked actions: p = 0).
    float p[6], lp[6], h = 0.0f;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      lp[k] = x[k] - lse;
      p[k] = __expf(lp[k]);
      if (lane + 32 * k < kActions) h -= p[k] * lp[k];
    }
    h = warp_sum(h);
    const int act = static_cast<int>(a.actions[row]);
    const int owner = act & 31, slot = act >> 5;
    float lpa = 0.0f;
#pragma unroll
    for (int k = 0; k < 6; ++k)
      if (k == slot) lpa = lp[k];
    lpa = __shfl_sync(kFull, lpa, owner);
    const float log_ratio = lpa - a.logp_old[row];
    const float ratio = __expf(log_ratio);
    const float A = a.adv[row];
    const float clipped = fminf(fmaxf(ratio, 1.0f - a.clip), 1.0f + a.clip);
    const float unclipped_term = ratio * A, clipped_term = clipped * A;
    const float surrogate = fminf(unclipped_term, clipped_term);
    // d(-surrogate)/d log p_a: -ratio A where the unclipped term is the minimum (or
    // the clipped one still moves with the ratio), else 0.
    const bool moves = unclipped_term <= clipped_term || (ratio > 1.0f - a.clip && ratio < 1.0f + a.clip);
    const float g_logp = moves ? -ratio * A : 0.0f;
    const float ent_c = *a.entropy_coef;
    // loss = mean(-surrogate) - c_e mean(entropy) + c_v mean(smooth_l1(v, ret)).
    __nv_bfloat16* dl = a.dlogits + row * a.ldd;
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      const int c = lane + 32 * k;
      if (c < kActions) {
        const float g = g_logp * ((c == act ? 1.0f : 0.0f) - p[k]) + ent_c * p[k] * (lp[k] + h);
        dl[c] = __float2bfloat16_rn(g * a.inv_b);
      } else if (c < a.ldd) {
        dl[c] = __float2bfloat16_rn(0.0f);
      }
    }
    const float v = a.value[row * a.value_ld];
    const float d = v - a.ret[row];
    const float ad = fabsf(d);
    if (lane == 0) {
      a.dvalue[row] = a.value_coef * (ad < 1.0f ? d : (d > 0.0f ? 1.0f : -1.0f)) * a.inv_b;
      acc[0] = -surrogate;
      acc[1] = ad < 1.0f ? 0.5f * d * d : ad - 0.5f;
      acc[2] = h;
      acc[3] = (ratio - 1.0f) - log_ratio;
      acc[4] = fabsf(ratio - 1.0f) > a.clip ? 1.0f : 0.0f;
    }
  }
  if (lane == 0)
#pragma unroll
    for (int s = 0; s < 5; ++s) part[warp][s] = acc[s];
  __syncthreads();
  if (threadIdx.x < 5) {
    float t = 0.0f;
    for (int w = 0; w < kLossWarps; ++w) t += part[w][threadIdx.x];
    atomicAdd(a.stats + threadIdx.x, t * a.inv_b);
  }
}

// ---- column sums, with and without the activation backward ----------------------------

constexpr int kColThreads = 256;

// Rows [r0, r1) of x (bf16 [rows, n], ld elements apart), thread t of the block
// owning columns 8 (t % (n / 8)) .. + 7 of rows r0 + t / (n / 8), stepping by the
// block's row groups; with z, the sums are of dz = du act'(z) and dz is stored.
// Rows are taken kColBatch at a time with all their loads issued before use.
constexpr int kColBatch = 8;

__global__ void __launch_bounds__(kColThreads) colsum_kernel(
    const __nv_bfloat16* __restrict__ du, i64 ldu, const __nv_bfloat16* __restrict__ z, i64 ldz,
    int act, __nv_bfloat16* __restrict__ dz, i64 ldd, i64 rows, int n, i64 rows_per_block,
    float* __restrict__ partial) {
  extern __shared__ float shared_sums[];  // [groups][n]
  const int vecs = n / 8;
  const int groups = kColThreads / vecs;
  const int t = threadIdx.x;
  const int v = t % vecs, grp = t / vecs;
  const i64 r0 = (i64)blockIdx.x * rows_per_block;
  const i64 r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (grp < groups) {
    for (i64 rb = r0 + grp; rb < r1; rb += (i64)kColBatch * groups) {
      uint4 gx[kColBatch], gz[kColBatch];
#pragma unroll
      for (int k = 0; k < kColBatch; ++k) {
        const i64 r = rb + (i64)k * groups;
        if (r < r1) {
          gx[k] = __ldg(reinterpret_cast<const uint4*>(du + r * ldu) + v);
          if (z) gz[k] = __ldg(reinterpret_cast<const uint4*>(z + r * ldz) + v);
        }
      }
#pragma unroll
      for (int k = 0; k < kColBatch; ++k) {
        const i64 r = rb + (i64)k * groups;
        if (r >= r1) break;
        float g[8];
        bf16x8(gx[k], g);
        if (z) {
          float zz[8];
          bf16x8(gz[k], zz);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] *= act_slope(zz[e], act);
          const uint4 packed = pack8(g);
          reinterpret_cast<uint4*>(dz + r * ldd)[v] = packed;
          bf16x8(packed, g);  // the sums are of the stored (bf16) gradient
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] += g[e];
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) shared_sums[grp * n + 8 * v + e] = s[e];
  }
  __syncthreads();
  for (int c = t; c < n; c += kColThreads) {
    float tot = 0.0f;
    for (int q = 0; q < groups; ++q) tot += shared_sums[q * n + c];
    partial[(i64)blockIdx.x * n + c] = tot;
  }
}

// Column c of the block partials [blocks][width] summed in a fixed order: thread
// (c, y) of a 32 x 32 block adds the partials of blocks y, y + 32, ... in turn, then
// the 32 sums are added in order of y (deterministic, and every column's loads
// coalesced across the 32 columns of a block row).
constexpr int kSumRows = 32;

__device__ __forceinline__ bool sum_column(const float* __restrict__ partial, int blocks, int width,
                                           float& out) {
  __shared__ float ys[kSumRows][33];
  const int cx = threadIdx.x & 31, y = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cx;
  float tot = 0.0f;
  if (c < width) {
#pragma unroll 8
    for (int b = y; b < blocks; b += kSumRows) tot += __ldg(partial + (i64)b * width + c);
  }
  ys[y][cx] = tot;
  __syncthreads();
  if (y != 0 || c >= width) return false;
  out = 0.0f;
#pragma unroll
  for (int q = 0; q < kSumRows; ++q) out += ys[q][cx];
  return true;
}

// out[c] = sum over the blocks of partial[block][c].
__global__ void __launch_bounds__(32 * kSumRows) sum_partials_kernel(const float* __restrict__ partial,
                                                           int blocks, int n,
                                                           float* __restrict__ out) {
  float tot;
  if (sum_column(partial, blocks, n, tot)) out[blockIdx.x * 32 + (threadIdx.x & 31)] = tot;
}

// The critic's one-output head backward (v = w . act(h) + b, h [rows, n]):
// dh = dv w act'(h) (bf16), colsum(dh), dw = sum_i dv_i act(h_i), db = sum_i dv_i.
__global__ void __launch_bounds__(kColThreads) scalar_head_backward_kernel(
    const float* __restrict__ dv, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ h, i64 ldh, int act, __nv_bfloat16* __restrict__ dh,
    i64 ldd, i64 rows, int n, i64 rows_per_block, float* __restrict__ partial) {
  extern __shared__ float shared_sums[];  // [groups][2 n + 1]
  const int vecs = n / 8;
  const int groups = kColThreads / vecs;
  const int t = threadIdx.x;
  const int v = t % vecs, grp = t / vecs;
  const int stride = 2 * n + 1;
  const i64 r0 = (i64)blockIdx.x * rows_per_block;
  const i64 r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  float wf[8], s[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sb = 0.0f;
  bf16x8(__ldg(reinterpret_cast<const uint4*>(w) + v), wf);
  if (grp < groups) {
    for (i64 rb = r0 + grp; rb < r1; rb += (i64)kColBatch * groups) {
      uint4 hx[kColBatch];
      float dd[kColBatch];
#pragma unroll
      for (int k = 0; k < kColBatch; ++k) {
        const i64 r = rb + (i64)k * groups;
        if (r < r1) {
          hx[k] = __ldg(reinterpret_cast<const uint4*>(h + r * ldh) + v);
          dd[k] = __ldg(dv + r);
        }
      }
#pragma unroll
      for (int k = 0; k < kColBatch; ++k) {
        const i64 r = rb + (i64)k * groups;
        if (r >= r1) break;
        const float d = dd[k];
        float hh[8], g[8];
        bf16x8(hx[k], hh);
        // The head's input act(h) in bf16, as the forward's head GEMM read it, and
        // act'(h), from one sigmoid per element for SiLU.
        float gin[8], slope[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (act == kActSilu) {
            const float sg = __fdividef(1.0f, 1.0f + __expf(-hh[e]));
            gin[e] = hh[e] * sg;
            slope[e] = sg * (1.0f + hh[e] * (1.0f - sg));
          } else {
            gin[e] = act_value(hh[e], act);
            slope[e] = act_slope(hh[e], act);
          }
        }
        bf16x8(pack8(gin), gin);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          g[e] = d * wf[e] * slope[e];
          sw[e] += d * gin[e];
        }
        const uint4 packed = pack8(g);
        reinterpret_cast<uint4*>(dh + r * ldd)[v] = packed;
        bf16x8(packed, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] += g[e];
        if (v == 0) sb += d;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      shared_sums[grp * stride + 8 * v + e] = s[e];
      shared_sums[grp * stride + n + 8 * v + e] = sw[e];
    }
    if (v == 0) shared_sums[grp * stride + 2 * n] = sb;
  }
  __syncthreads();
  for (int c = t; c < 2 * n + 1; c += kColThreads) {
    float tot = 0.0f;
    for (int q = 0; q < groups; ++q) tot += shared_sums[q * stride + c];
    partial[(i64)blockIdx.x * (2 * n + 1) + c] = tot;
  }
}

// The scalar head's block partials [blocks][2n + 1] summed into dh_sums [n], dw [n]
// and db [1] (the order of sum_column).
__global__ void __launch_bounds__(32 * kSumRows) sum_head_partials_kernel(const float* __restrict__ partial,
                                                                int blocks, int n,
                                                                float* __restrict__ dh_sums,
                                                                float* __restrict__ dw,
                                                                float* __restrict__ db) {
  float tot;
  if (!sum_column(partial, blocks, 2 * n + 1, tot)) return;
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  if (c < n) dh_sums[c] = tot;
  else if (c < 2 * n) dw[c - n] = tot;
  else *db = tot;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

// Blocks and rows per block of a column-sum launch over `rows` rows.
inline void colsum_grid(i64 rows, unsigned& blocks, i64& per_block) {
  // Enough blocks that every SM holds several (the loads of a batch are all that a
  // thread keeps in flight), at least 32 rows each.
  const i64 target = 16 * 148;
  per_block = (rows + target - 1) / target;
  if (per_block < 32) per_block = 32;
  blocks = static_cast<unsigned>((rows + per_block - 1) / per_block);
}

bool colsum_shape_ok(int n) { return n >= 8 && n % 8 == 0 && n / 8 <= kColThreads; }

}  // namespace

extern "C" {

int cugo_b200_ppo_loss(const float* logits, int64_t ldl, const bool* legal, const int64_t* actions,
                       const float* logp_old, const float* adv, const float* value,
                       int64_t value_ld, const float* ret, int64_t b, float clip,
                       const float* entropy_coef, float value_coef, void* dlogits, int64_t ldd,
                       float* dvalue, float* stats, cudaStream_t stream) {
  if (b < 0 || ldl < kActions || ldd < kActions || value_ld < 1) return CUGO_B200_ERR_ARG;
  if (b > 0 && (!logits || !legal || !actions || !logp_old || !adv || !value || !ret ||
                !entropy_coef || !dlogits || !dvalue || !stats))
    return CUGO_B200_ERR_ARG;
  if (!aligned(stats, 4)) return CUGO_B200_ERR_ALIGN;
  if (cudaMemsetAsync(stats, 0, 5 * sizeof(float), stream) != cudaSuccess) return CUGO_B200_ERR_LAUNCH;
  if (b == 0) return CUGO_B200_OK;
  LossArgs a{logits, ldl, legal, actions, logp_old, adv, value, value_ld, ret, b, clip,
             1.0f / static_cast<float>(b), entropy_coef, value_coef,
             static_cast<__nv_bfloat16*>(dlogits), ldd, dvalue, stats};
  ppo_loss_kernel<<<static_cast<unsigned>((b + kLossWarps - 1) / kLossWarps), 32 * kLossWarps, 0,
                    stream>>>(a);
  return launch_status();
}

int cugo_b200_colsum_bf16(const void* x, int64_t ldx, const void* z, int64_t ldz, int32_t act,
                          void* dz, int64_t ldd, int64_t rows, int32_t n, float* sums,
                          float* scratch, int64_t scratch_floats, cudaStream_t stream) {
  if (rows < 0 || !colsum_shape_ok(n) || ldx < n || (z && (ldz < n || ldd < n)) ||
      (act != kActNone && act != kActRelu && act != kActSilu))
    return CUGO_B200_ERR_ARG;
  if (!sums || (rows > 0 && !x) || (z && !dz)) return CUGO_B200_ERR_ARG;
  if (!aligned(x, 16) || ldx % 8 || (z && (!aligned(z, 16) || !aligned(dz, 16) || ldz % 8 || ldd % 8)))
    return CUGO_B200_ERR_ALIGN;
  if (rows == 0) {
    return cudaMemsetAsync(sums, 0, n * sizeof(float), stream) == cudaSuccess ? CUGO_B200_OK
                                                                             : CUGO_B200_ERR_LAUNCH;
  }
  unsigned blocks;
  i64 per_block;
  colsum_grid(rows, blocks, per_block);
  if (!scratch || scratch_floats < static_cast<i64>(blocks) * n) return CUGO_B200_ERR_CAPACITY;
  const int groups = kColThreads / (n / 8);
  colsum_kernel<<<blocks, kColThreads, groups * n * sizeof(float), stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(z), ldz, act,
      static_cast<__nv_bfloat16*>(dz), ldd, rows, n, per_block, scratch);
  sum_partials_kernel<<<(n + 31) / 32, 32 * kSumRows, 0, stream>>>(scratch, static_cast<int>(blocks), n, sums);
  return launch_status();
}

int cugo_b200_scalar_head_backward(const float* dv, const void* w, const void* h, int64_t ldh,
                                   int32_t act, void* dh, int64_t ldd, int64_t rows, int32_t n,
                                   float* dh_sums, float* dw, float* db, float* scratch,
                                   int64_t scratch_floats, cudaStream_t stream) {
  if (rows < 0 || !colsum_shape_ok(n) || ldh < n || ldd < n ||
      (act != kActNone && act != kActRelu && act != kActSilu))
    return CUGO_B200_ERR_ARG;
  if (!w || !dh_sums || !dw || !db || (rows > 0 && (!dv || !h || !dh))) return CUGO_B200_ERR_ARG;
  if (!aligned(w, 16) || !aligned(h, 16) || !aligned(dh, 16) || ldh % 8 || ldd % 8)
    return CUGO_B200_ERR_ALIGN;
  if (rows == 0) {
    if (cudaMemsetAsync(dh_sums, 0, n * sizeof(float), stream) != cudaSuccess ||
        cudaMemsetAsync(dw, 0, n * sizeof(float), stream) != cudaSuccess ||
        cudaMemsetAsync(db, 0, sizeof(float), stream) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    return CUGO_B200_OK;
  }
  unsigned blocks;
  i64 per_block;
  colsum_grid(rows, blocks, per_block);
  if (!scratch || scratch_floats < static_cast<i64>(blocks) * (2 * n + 1)) return CUGO_B200_ERR_CAPACITY;
  const int groups = kColThreads / (n / 8);
  scalar_head_backward_kernel<<<blocks, kColThreads, groups * (2 * n + 1) * sizeof(float),
                                stream>>>(dv, static_cast<const __nv_bfloat16*>(w),
                                          static_cast<const __nv_bfloat16*>(h), ldh, act,
                                          static_cast<__nv_bfloat16*>(dh), ldd, rows, n, per_block,
                                          scratch);
  sum_head_partials_kernel<<<(2 * n + 1 + 31) / 32, 32 * kSumRows, 0, stream>>>(
      scratch, static_cast<int>(blocks), n, dh_sums, dw, db);
  return launch_status();
}

int64_t cugo_b200_colsum_scratch_floats(int64_t rows, int32_t n) {
  if (rows <= 0 || n <= 0) return 0;
  unsigned blocks;
  i64 per_block;
  colsum_grid(rows, blocks, per_block);
  return static_cast<int64_t>(blocks) * (2 * n + 1);
}

}  // extern "C"
