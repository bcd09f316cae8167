// bf16 GEMM with fused epilogue on the 5th-generation tensor cores (sm_100a).
//
//   out[M, N] = act_after(act(A[M, K] . W[N, K]^T + bias[N]) + residual[M, N])
//
// A and W are bf16, K-major (row-major A, nn.Linear weight layout); the product
// accumulates in fp32 in tensor memory; out is bf16 or fp32 and the residual has
// the output's type (an fp32 residual stream is updated in place); the bias is
// bf16 or fp32.  This is one layer of the policy/value MLP
// (python/cugo_ppo_nets50.py:26-64 run under bf16 autocast) or of the sequence
// transformer (python/cugo_seq50.py:318-321): nn.Linear + bias, then
// ReLU/SiLU/GELU and the residual add, fused.
//
// Kernel (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0     : TMA producer — one elected thread streams 128x64 A and 256x64 W
//                tiles (128-byte swizzle) into a 4-stage shared-memory ring;
//   warp 1     : owns the tensor memory (2 accumulators x 256 columns) and one
//                thread issues tcgen05.mma (M=128, N=256, K=16) per 16-wide K
//                slice, committing each stage back to the producer and each
//                finished tile to the epilogue;
//   warps 2..9 : epilogue — two warps per TMEM lane quadrant, each taking half of
//                the tile's 256 columns: tcgen05.ld of their 32 TMEM lanes, bias,
//                activation, residual; each 32-row x 64-byte chunk is transposed
//                through a swizzled shared buffer so that every warp store writes
//                whole 64-byte row segments.  A tile's epilogue overlaps the next
//                tile's MMAs through the second accumulator.
// Every mbarrier wait is bounded (about 2 s of %globaltimer); a wait that runs
// out sets *error and the kernel drains and returns instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "../../include/cugo_b200.h"
#include "engine/driver.cuh"
#include "gumbel.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int EPI_WARPS = 8;                    // two per TMEM lane quadrant
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int EPI_BUF = 2048;                   // one 32-row x 64-byte chunk
constexpr int EPI_STAGE_BYTES = EPI_WARPS * 2 * EPI_BUF;  // double-buffered per warp
constexpr uint32_t TMEM_COLS = 2 * BN;          // two accumulators
constexpr int BAR_BYTES = 512;  // mbarriers and the TMEM address
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + BAR_BYTES +
                           BN * 4 /*bias*/ + EPI_STAGE_BYTES;
constexpr uint64_t kWaitNs = 2'000'000'000ull;

// Shared memory and tensor memory of gemm_kernel at output tile width tbn (256, 128 or
// 64 columns; 256 everywhere else).
__host__ __device__ constexpr int g_stage_bytes(int tbn) { return A_BYTES + tbn * BK * 2; }
__host__ __device__ constexpr int g_smem_bytes(int tbn) {
  return STAGES * g_stage_bytes(tbn) + 1024 /*align*/ + BAR_BYTES + tbn * 4 /*bias*/ +
         EPI_STAGE_BYTES;
}
static_assert(g_smem_bytes(BN) == SMEM_BYTES, "the 256-wide tile is the default shape");

enum Act : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActGelu = 3 };

struct Epilogue {
  const void* bias;      // [N] bf16 (fp32 when bias_fp32) or null
  const void* residual;  // [M, ldr] of the output's type, or null
  int64_t ldr;
  void* out;
  int64_t ldo;
  int out_fp32;
  int bias_fp32;
  int act;        // applied to acc + bias, before the residual add
  int act_after;  // applied after the residual add
  int m, n, k;
  int* error;
  // Optional device-resident row window {first row, rows} of the M rows the maps
  // cover (read by the kernel, so a CUDA graph can change it between replays);
  // null: all M rows.
  const int32_t* window;
  // Nonzero: the residual's tensor map is instead a second bf16 output receiving
  // acc + bias before the activation (the pre-activation a training backward reads).
  int pre;
};

// The window's first row and row count, clamped to [0, M].
__device__ __forceinline__ void row_window(const Epilogue& ep, int& r0, int& rows) {
  r0 = 0;
  rows = ep.m;
  if (ep.window) {
    const int w0 = __ldg(ep.window), w1 = __ldg(ep.window + 1);
    r0 = w0 < 0 ? 0 : (w0 > ep.m ? ep.m : w0);
    rows = w1 < 0 ? 0 : (w1 > ep.m - r0 ? ep.m - r0 : w1);
  }
}

// ---- PTX wrappers ------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of parity `parity` to complete; false once limit_ns (~2 s by
// default) have passed on the global timer.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitNs) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 255u) == 0 && now_ns() - t0 > limit_ns) return false;
  }
}

// The timeout path of the bounded wait, run on purpose: thread 0 waits on an
// mbarrier that no thread arrives on, the wait gives up after limit_ns, *error is
// set and the time waited recorded; then the one expected arrival completes the
// phase so the barrier is left settled, and the kernel returns.
__global__ void wait_timeout_probe_kernel(uint64_t limit_ns, int* error,
                                          unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = now_ns();
    const bool completed = mbar_wait(&bar, 0, limit_ns);
    const uint64_t t1 = now_ns();
    if (!completed && error) atomicExch(error, 1);
    if (waited_ns) *waited_ns = t1 - t0;
    mbar_arrive(&bar);
    mbar_wait(&bar, 0, limit_ns);
  }
  __syncthreads();
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// Tile store from shared memory (the async proxy reads the staging buffer).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's tile stores still read shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1 KB apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;           // leading byte offset (unused here)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;           // descriptor version
  d |= static_cast<uint64_t>(2) << 61;           // 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: bf16 x bf16 -> fp32, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n) {
  return (1u << 4)                                  // D: fp32
         | (1u << 7) | (1u << 10)                   // A, B: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

#define CB_TMEM_LD32(taddr, r)                                                                  \
  asm volatile(                                                                                 \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"  \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"        \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),    \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),             \
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),          \
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),          \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),          \
        "=r"(r[31])                                                                             \
      : "r"(taddr))

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// SiLU as v * sigmoid(v) with the fast exponential and divide: a few instructions
// per element where IEEE division costs a dozen and an out-of-line slow path.  The
// error (a few fp32 ulp) is far below the bf16 rounding of the stored result.
__device__ __forceinline__ float silu_fast(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

__device__ __forceinline__ float activate(float v, int act) {
  if (act == kActRelu) return fmaxf(v, 0.0f);
  if (act == kActSilu) return silu_fast(v);
  if (act == kActGelu) return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));  // exact (erf) GELU
  return v;
}

// The activation over a chunk, the choice made once per chunk.
template <int CW>
__device__ __forceinline__ void activate_chunk(float* v, int act) {
  if (act == kActRelu) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = fmaxf(v[j], 0.0f);
  } else if (act == kActSilu) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = silu_fast(v[j]);
  } else if (act == kActGelu) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = activate(v[j], kActGelu);
  }
}

#define CB_TMEM_LD16(taddr, r)                                                                  \
  asm volatile(                                                                                 \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"  \
      "%14,%15}, [%16];"                                                                        \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),    \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),             \
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])                                                   \
      : "r"(taddr))

// ---- epilogue stores through shared memory ----------------------------------------
//
// A thread holds one output row of the chunk (TMEM lane = row): 64 bytes, i.e. 32
// bf16 or 16 fp32 columns.  Rows go to a per-warp 32 x 64-byte buffer whose 16-byte
// pieces are XOR-swizzled by row pair — the layout of a TMA tile with 64-byte
// swizzle, so the row-per-thread writes are bank-conflict free and one TMA store
// writes the chunk.  The residual comes in through the same layout (cp.async).

__device__ __forceinline__ uint32_t swz(int row, int piece) {
  return static_cast<uint32_t>(row * 64 + ((piece ^ ((row >> 1) & 3)) << 4));
}

// Writes this lane's row of the chunk into the staging buffer and has lane 0 store
// the 32 x 64-byte chunk with one TMA tile store (rows or columns outside the
// matrix are clipped by the tensor map).  The buffer's previous store has been
// waited for by the caller.
template <typename T>
__device__ __forceinline__ void store_chunk(uint8_t* stage, const float* v, const CUtensorMap* map_out,
                                            int row0, int col0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    uint4 raw;
    if constexpr (sizeof(T) == 2) {
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[p * 8 + 2 * e], v[p * 8 + 2 * e + 1]);
    } else {
      raw = make_uint4(__float_as_uint(v[p * 4]), __float_as_uint(v[p * 4 + 1]),
                       __float_as_uint(v[p * 4 + 2]), __float_as_uint(v[p * 4 + 3]));
    }
    *reinterpret_cast<uint4*>(stage + swz(lane, p)) = raw;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the TMA unit
  __syncwarp();
  if (lane == 0) tma_store_2d(map_out, stage, col0, row0);
}

// Residual chunks (32 rows x 64 bytes, the output's type) arrive by TMA tile loads
// into the same swizzled staging layout, one mbarrier per staging buffer; rows or
// columns outside the matrix read as zero.  Lane 0 issues, every lane waits.
__device__ __forceinline__ void residual_load(const CUtensorMap* map_res, uint64_t* bar,
                                              uint8_t* buf, int col0, int row0) {
  if ((threadIdx.x & 31) == 0) {
    mbar_expect_tx(bar, EPI_BUF);
    tma_load_2d(map_res, bar, buf, col0, row0);
  }
}

// Waits for a residual chunk in buffer b (bounded); false after a timeout.  Bit b of
// `phases` is the parity buffer b's barrier completes next.
__device__ __forceinline__ bool residual_wait(uint64_t* bar, uint32_t& phases, int b) {
  const bool ok = mbar_wait(bar, (phases >> b) & 1u);
  phases ^= 1u << b;
  return ok;
}

// Adds the staged residual row of this lane to v (the copies are complete).
template <typename T>
__device__ __forceinline__ void add_residual_row(const uint8_t* buf, float* v) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4 raw = *reinterpret_cast<const uint4*>(buf + swz(lane, p));
    if constexpr (sizeof(T) == 2) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        v[p * 8 + 2 * e] += f.x;
        v[p * 8 + 2 * e + 1] += f.y;
      }
    } else {
      const float* h = reinterpret_cast<const float*>(&raw);
#pragma unroll
      for (int e = 0; e < E; ++e) v[p * E + e] += h[e];
    }
  }
  __syncwarp();
}

// ---- epilogue of one tile (warps 2..9, 256 threads) ----------------------------------

// A warp's epilogue resources: tensor maps of the output and the residual, and the
// residual barriers of its two staging buffers with their phases.
struct EpiWarp {
  const CUtensorMap* map_out;
  const CUtensorMap* map_res;
  uint64_t* res_bar;     // [2]
  uint32_t res_phases;   // bit b: parity of buffer b's next completion
  bool ok;               // false once a residual wait timed out
};

// Epilogue warp w owns TMEM lanes 32 (w % 4) .. +31 (the hardware's lane quadrant
// for warp w) and columns 128 ((w - 2) / 4) .. +127 of the tile.
__device__ __forceinline__ int epi_quad(int warp) { return warp & 3; }
template <int TBN = BN>
__device__ __forceinline__ int epi_col0(int warp) { return ((warp - 2) >> 2) * (TBN / 2); }

// Starts the warp's first residual chunk and stages the tile's bias (fp32) in
// shared memory.
template <int TBN = BN>
__device__ __forceinline__ void epilogue_begin(const Epilogue& ep, EpiWarp& io, uint8_t* stage,
                                               float* bias_s, int epi_tid, int row0, int n0,
                                               int cbase) {
  // The previous tile's stores have read the staging buffers; then the first
  // residual chunk streams in while the accumulator is computed.
  if ((threadIdx.x & 31) == 0) tma_store_wait_read<0>();
  __syncwarp();
  if (ep.residual) residual_load(io.map_res, &io.res_bar[0], stage, n0 + cbase, row0);
  // The previous tile's readers of bias_s are past this barrier.
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
  for (int c = epi_tid; c < TBN; c += EPI_THREADS) {
    const int n = n0 + c;
    float b = 0.0f;
    if (ep.bias && n < ep.n)
      b = ep.bias_fp32 ? static_cast<const float*>(ep.bias)[n]
                       : __bfloat162float(static_cast<const __nv_bfloat16*>(ep.bias)[n]);
    bias_s[c] = b;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
}

// Waits for the accumulator; the epilogue threads agree on a timeout, so none is
// left on a named barrier.  False (after draining the residual copies) on timeout.
__device__ __forceinline__ bool epilogue_wait(uint64_t* acc_full, uint32_t parity) {
  const uint32_t timed_out = mbar_wait(acc_full, parity) ? 0u : 1u;
  uint32_t any_timed_out;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, 1, %2, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(any_timed_out)
      : "r"(timed_out), "n"(EPI_THREADS)
      : "memory");
  if (any_timed_out) return false;
  fence_after();
  return true;
}

// TMEM -> bias -> activation -> residual -> activation -> global for this warp's
// 32 rows x 128 columns (tile columns cbase .. cbase + 127; taddr: the warp's lane
// quadrant and accumulator buffer), in 64-byte-row chunks of CW columns.
template <typename T, int TBN = BN>
__device__ __forceinline__ void epilogue_cols(const Epilogue& ep, EpiWarp& io, uint32_t taddr,
                                              uint8_t* stage, const float* bias_s, int row0, int n0,
                                              int cbase) {
  constexpr int CW = 64 / static_cast<int>(sizeof(T));
  constexpr int CHUNKS = (TBN / 2) / CW;
  static_assert((TBN / 2) % CW == 0, "a warp's columns are whole chunks");
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int c = 0; c < CHUNKS; ++c) {
    const int c0 = cbase + c * CW;
    uint8_t* cur = stage + (c & 1) * EPI_BUF;
    uint32_t r[CW];
    if constexpr (CW == 32) {
      CB_TMEM_LD32(taddr + static_cast<uint32_t>(c0), r);
    } else {
      CB_TMEM_LD16(taddr + static_cast<uint32_t>(c0), r);
    }
    tmem_wait_ld();
    if (ep.residual) {
      // This chunk's residual (started one chunk earlier) has landed.
      if (!residual_wait(&io.res_bar[c & 1], io.res_phases, c & 1)) io.ok = false;
    }
    const bool live = n0 + c0 < ep.n;
    float v[CW];
    if (live) {
#pragma unroll
      for (int j = 0; j < CW; ++j) v[j] = __uint_as_float(r[j]) + bias_s[c0 + j];
      if constexpr (sizeof(T) == 2) {
        if (ep.pre) {  // the pre-activation through the other staging buffer
          if (lane == 0) tma_store_wait_read<0>();
          __syncwarp();
          store_chunk<T>(stage + ((c & 1) ^ 1) * EPI_BUF, v, io.map_res, row0, n0 + c0);
        }
      }
      activate_chunk<CW>(v, ep.act);
      if (ep.residual) add_residual_row<T>(cur, v);  // ends with __syncwarp
      activate_chunk<CW>(v, ep.act_after);
    }
    // The previous chunk's store must have read the other buffer before the next
    // residual lands there (and this buffer's store, two chunks back, long before).
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
    if (ep.residual && c + 1 < CHUNKS)
      residual_load(io.map_res, &io.res_bar[(c + 1) & 1], stage + ((c + 1) & 1) * EPI_BUF,
                    n0 + c0 + CW, row0);
    if (live) store_chunk<T>(cur, v, io.map_out, row0, n0 + c0);
  }
}

template <int TBN = BN>
__device__ __forceinline__ void epilogue_tile(const Epilogue& ep, EpiWarp& io, uint32_t taddr,
                                              uint8_t* stage, const float* bias_s, int row0, int n0,
                                              int cbase) {
  if (ep.out_fp32) epilogue_cols<float, TBN>(ep, io, taddr, stage, bias_s, row0, n0, cbase);
  else epilogue_cols<__nv_bfloat16, TBN>(ep, io, taddr, stage, bias_s, row0, n0, cbase);
}

// ---- the kernel ------------------------------------------------------------------

// TBN: output tile width (256, or 128 / 64 when wider tiles would leave SMs idle).
template <int TBN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_out,
                const __grid_constant__ CUtensorMap map_res, const Epilogue ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // Layout: operand stages | epilogue staging (1 KB aligned, as the 64-byte TMA
  // swizzle of the stores requires) | barriers | bias.
  constexpr int kStage = g_stage_bytes(TBN);
  constexpr uint32_t kTmemCols = 2 * TBN;  // two accumulators
  uint8_t* epi_stage = smem + STAGES * kStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drained = acc_empty + 2;
  uint64_t* res_bars = drained + 1;  // [EPI_WARPS][2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_bars + 2 * EPI_WARPS);
  float* bias_s = reinterpret_cast<float*>(epi_stage + EPI_STAGE_BYTES + BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int r0, m_rows;
  row_window(ep, r0, m_rows);
  const int tiles_m = (m_rows + BM - 1) / BM;
  const int tiles_n = (ep.n + TBN - 1) / TBN;
  const int tiles = tiles_m * tiles_n;
  const int k_tiles = (ep.k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);
    }
    mbar_init(drained, 1);
    for (int b = 0; b < 2 * EPI_WARPS; ++b) mbar_init(&res_bars[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool failed = false;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
        const int tm = t / tiles_n, tn = t - tm * tiles_n;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            failed = true;
            break;
          }
          uint8_t* sa = smem + stage * kStage;
          mbar_expect_tx(&full[stage], kStage);
          tma_load_2d(&map_a, &full[stage], sa, kt * BK, r0 + tm * BM);
          tma_load_2d(&map_w, &full[stage], sa + A_BYTES, kt * BK, tn * TBN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // After a failure, wait (bounded) for copies still in flight.
      if (failed) {
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full[s], 0);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BM, TBN);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++iter) {
        const int buf = iter & 1;
        const uint32_t use = static_cast<uint32_t>(iter >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u)) {
          failed = true;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * TBN);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase)) {
            failed = true;
            break;
          }
          fence_after();
          const uint32_t a_addr = smem_addr(smem + stage * kStage);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            mma_bf16(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                     (kt > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (failed) break;
        mma_commit(&acc_full[buf]);
      }
      // All issued MMAs complete before the accumulators are released.
      mma_commit(drained);
      mbar_wait(drained, 0);
    }
  } else {
    // ---- epilogue: warps 2..9 (two per TMEM lane quadrant) ----
    const int quad = epi_quad(warp);
    const int cbase = epi_col0<TBN>(warp);
    const int epi_tid = threadIdx.x - 64;  // 0..255
    uint8_t* stage = epi_stage + (warp - 2) * 2 * EPI_BUF;
    EpiWarp io{&map_out, &map_res, res_bars + 2 * (warp - 2), 0u, true};
    int iter = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++iter) {
      const int tm = t / tiles_n, tn = t - tm * tiles_n;
      const int n0 = tn * TBN;
      const int buf = iter & 1;
      const uint32_t use = static_cast<uint32_t>(iter >> 1);
      const int row0 = r0 + tm * BM + quad * 32;
      epilogue_begin<TBN>(ep, io, stage, bias_s, epi_tid, row0, n0, cbase);
      if (!epilogue_wait(&acc_full[buf], use & 1u)) {
        failed = true;
        break;
      }
      epilogue_tile<TBN>(ep, io,
                         tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(buf * TBN),
                    stage, bias_s, row0, n0, cbase);
      if (!io.ok) failed = true;
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) tma_store_wait_all();  // stores complete before the CTA leaves
  }
  if (failed) {
    if (ep.error) atomicExch(ep.error, 1);
    // Let copies still in flight land before the CTA leaves (bounded).
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 100'000ull) {
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols));
  }
}

// ---- the CTA-pair kernel (tcgen05 cta_group::2) ------------------------------------
//
// Two CTAs of a cluster share one 256 x 256 output tile: CTA r loads rows
// 128r..128r+127 of the A tile and rows 128r..128r+127 of the 256-row weight panel,
// and one thread of CTA 0 issues M=256 N=256 K=16 MMAs that read both CTAs' shared
// memory and accumulate each CTA's 128 rows in its own tensor memory.  Per SM
// this halves the weight bytes moved from L2 per FLOP (32 KB per 64-deep K step
// instead of 48 KB), which is what bounds the single-CTA kernel on the policy's
// narrow layers.  Both CTAs' copies count towards CTA 0's "full" barrier (only
// CTA 0 posts the expected byte count); CTA 0's MMA completion arrives on the
// "empty" and "accumulator full" barriers of both CTAs; each CTA's epilogue
// warps signal CTA 0's "accumulator empty" barrier once per tile.
constexpr int P_BN_HALF = BN / 2;                    // weight rows loaded per CTA
constexpr int P_STAGES = 6;
constexpr int P_B_BYTES = P_BN_HALF * BK * 2;        // 16 KB
constexpr int P_STAGE_BYTES = A_BYTES + P_B_BYTES;   // 32 KB
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 /*align*/ + BAR_BYTES +
                             BN * 4 /*bias*/ + EPI_STAGE_BYTES;
static_assert(P_SMEM_BYTES <= 232448, "fits the opt-in shared memory of one CTA");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}

// Tile copy whose completion is counted on the barrier at cluster address `bar`
// (CTA 0's), as the CTA pair's MMA requires.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar, void* dst,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrives on the barrier at this offset in both CTAs once the issued MMAs complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_addr(bar)), "h"(static_cast<uint16_t>(3))
      : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_out,
                     const __grid_constant__ CUtensorMap map_res, const Epilogue ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* epi_stage = smem + P_STAGES * P_STAGE_BYTES;  // 1 KB aligned (see gemm_kernel)
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* acc_full = empty + P_STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2], CTA 0's counts both CTAs' warps
  uint64_t* drained = acc_empty + 2;
  uint64_t* res_bars = drained + 1;  // [EPI_WARPS][2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_bars + 2 * EPI_WARPS);
  float* bias_s = reinterpret_cast<float*>(epi_stage + EPI_STAGE_BYTES + BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
  const int tiles_m = (ep.m + 2 * BM - 1) / (2 * BM);
  const int tiles_n = (ep.n + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int k_tiles = (ep.k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * EPI_WARPS);  // both CTAs' epilogue warps (used in CTA 0)
    }
    mbar_init(drained, 1);
    for (int b = 0; b < 2 * EPI_WARPS; ++b) mbar_init(&res_bars[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // both CTAs allocate together, same warp, same holder offset
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_holder)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool failed = false;
  __shared__ int any_failed;
  if (threadIdx.x == 0) any_failed = 0;
  __syncthreads();

  if (warp == 0) {
    // ---- TMA producer (both CTAs) ----
    if (lane == 0) {
      const uint32_t full0 = peer_addr(full, 0);  // CTA 0's full[0]
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < tiles && !failed; t += pairs) {
        const int tm = t / tiles_n, tn = t - tm * tiles_n;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            failed = true;
            break;
          }
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          const uint32_t bar = full0 + static_cast<uint32_t>(stage * 8);
          if (leader) mbar_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          tma_load_2d_pair(&map_a, bar, sa, kt * BK, tm * 2 * BM + static_cast<int>(rank) * BM);
          tma_load_2d_pair(&map_w, bar, sa + A_BYTES, kt * BK,
                           tn * BN + static_cast<int>(rank) * P_BN_HALF);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (CTA 0 only) ----
    if (leader && lane == 0) {
      constexpr uint32_t idesc = instr_desc(2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      for (int t = pair; t < tiles && !failed; t += pairs, ++iter) {
        const int buf = iter & 1;
        const uint32_t use = static_cast<uint32_t>(iter >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u)) {
          failed = true;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase)) {
            failed = true;
            break;
          }
          fence_after();
          const uint32_t a_addr = smem_addr(smem + stage * P_STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            mma_bf16_pair(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                          (kt > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty[stage]);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (failed) break;
        mma_commit_pair(&acc_full[buf]);
      }
      // All issued MMAs complete before the accumulators are released.
      mma_commit_pair_local(drained);
      mbar_wait(drained, 0);
    }
  } else {
    // ---- epilogue (both CTAs): warps 2..9 (two per TMEM lane quadrant) ----
    const int quad = epi_quad(warp);
    const int cbase = epi_col0(warp);
    const int epi_tid = threadIdx.x - 64;
    uint8_t* stage = epi_stage + (warp - 2) * 2 * EPI_BUF;
    EpiWarp io{&map_out, &map_res, res_bars + 2 * (warp - 2), 0u, true};
    int iter = 0;
    for (int t = pair; t < tiles; t += pairs, ++iter) {
      const int tm = t / tiles_n, tn = t - tm * tiles_n;
      const int n0 = tn * BN;
      const int buf = iter & 1;
      const uint32_t use = static_cast<uint32_t>(iter >> 1);
      const int row0 = tm * 2 * BM + static_cast<int>(rank) * BM + quad * 32;
      epilogue_begin(ep, io, stage, bias_s, epi_tid, row0, n0, cbase);
      if (!epilogue_wait(&acc_full[buf], use & 1u)) {
        failed = true;
        break;
      }
      epilogue_tile(ep, io,
                    tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                        static_cast<uint32_t>(buf * BN),
                    stage, bias_s, row0, n0, cbase);
      if (!io.ok) failed = true;
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_addr(&acc_empty[buf], 0));
    }
    if (lane == 0) tma_store_wait_all();  // stores complete before the CTA leaves
  }
  if (failed) {
    any_failed = 1;
    if (ep.error) atomicExch(ep.error, 1);
  }
  fence_before();
  __syncthreads();
  if (any_failed) {
    // Let copies and MMAs still in flight land before the pair leaves (bounded).
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 100'000ull) {
    }
  }
  cluster_sync_all();  // no cross-CTA signal is outstanding past this point
  fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

// ---- host side -------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over [rows, cols] (row stride ld elements), box box_rows x 64
// with 128-byte swizzle (the MMA operand layout).
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of the output [rows, cols] (bf16 or fp32, row stride ld elements) for
// the epilogue's stores: box 32 rows x 64 bytes with 64-byte swizzle.
bool make_out_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t ld, bool fp32) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int esz = fp32 ? 4 : 2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * esz)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(64 / esz), 32};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base,
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// CTA pairs of gemm_pair_kernel that fit on the device at once (clusters are placed
// within a GPC, so this can be below half the SM count).
int max_pairs(int dev) {
  static int cache[64] = {};
  if (!cache[dev]) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count() & ~1), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

// CUGO_B200_GEMM_SINGLE=1 selects the single-CTA kernel for every shape.
bool pair_kernel_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("CUGO_B200_GEMM_SINGLE");
    enabled = (v && v[0] == '1') ? 0 : 1;
  }
  return enabled == 1;
}

int gemm_launch(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                int32_t bias_fp32, const void* residual, int64_t ldr, void* out, int64_t ldo,
                int32_t out_fp32, int32_t act, int32_t act_after, int64_t m, int64_t n, int64_t k,
                const int32_t* window, int32_t* error, cudaStream_t stream,
                void* pre = nullptr, int64_t ldp = 0) {
  if (m < 0 || n <= 0 || k <= 0 || act < 0 || act > 3 || act_after < 0 || act_after > 3)
    return CUGO_B200_ERR_ARG;
  if (m == 0) return CUGO_B200_OK;
  if (!a || !w || !out || lda < k || ldw < k || ldo < n || (residual && ldr < n))
    return CUGO_B200_ERR_ARG;
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return CUGO_B200_ERR_ARG;
  if (pre && (residual || out_fp32 || ldp < n)) return CUGO_B200_ERR_ARG;
  if (pre && (reinterpret_cast<uintptr_t>(pre) % 16 || (ldp * 2) % 16)) return CUGO_B200_ERR_ALIGN;
  const int esz = out_fp32 ? 4 : 2;
  const auto al = [](const void* p, uintptr_t q) { return (reinterpret_cast<uintptr_t>(p) % q) == 0; };
  if (!al(a, 16) || !al(w, 16) || (lda * 2) % 16 || (ldw * 2) % 16 || !al(out, 16) ||
      (ldo * esz) % 16 || (residual && (!al(residual, 16) || (ldr * esz) % 16)) ||
      (bias && !al(bias, bias_fp32 ? 4 : 2)))
    return CUGO_B200_ERR_ALIGN;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {};
  if (dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             g_smem_bytes(256)) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             g_smem_bytes(128)) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             g_smem_bytes(64)) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             P_SMEM_BYTES) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  Epilogue ep{bias, residual, ldr, out, ldo, out_fp32 ? 1 : 0, bias_fp32 ? 1 : 0, act, act_after,
              static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), error, window,
              pre ? 1 : 0};
  CUtensorMap ma, mw, mo, mr;
  if (!make_out_map(&mo, out, m, n, ldo, out_fp32 != 0)) return CUGO_B200_ERR_LAUNCH;
  if (residual) {
    if (!make_out_map(&mr, const_cast<void*>(residual), m, n, ldr, out_fp32 != 0))
      return CUGO_B200_ERR_LAUNCH;
  } else if (pre) {
    if (!make_out_map(&mr, pre, m, n, ldp, false)) return CUGO_B200_ERR_LAUNCH;
  } else {
    mr = mo;  // unused
  }
  // Tile shape.  Wide tiles read each A tile fewer times per FLOP, so the single-CTA
  // kernel takes the widest output tile (256, then 128 columns, else 64) whose tiles
  // reach 60% of the SMs: narrower tiles pay only when wide ones would leave most SMs
  // idle (measured in CUDA graphs on B200: a 4,096 x 256 x 256 layer, 32 wide tiles,
  // 9.7 us at 256 columns and 5.7 us at 64; 4,096 x 768 x 256, 96 wide tiles, 7.1 us
  // at 256 and 7.6-8.0 us narrower; 32,768 x 512 x 512 21 us at 256, 25 us at 128).
  // The pair kernel halves the weight bytes each SM streams per FLOP, which pays when
  // the K loop is long and its 256 x 256 tiles fill every pair at least once
  // (262144x2048x2048 1,425 vs 1,317 TFLOP/s; but 4,096 x 256 x 1,024, 16 pair tiles,
  // 14.1 us against 9.2 us for 64-column single tiles).
  const int sms = sm_count();
  const int64_t tiles_m = (m + BM - 1) / BM;
  const int64_t enough = (3 * static_cast<int64_t>(sms)) / 5;
  int tbn = 64;
  for (int cand : {256, 128}) {
    if (tiles_m * ((n + cand - 1) / cand) >= enough) {
      tbn = cand;
      break;
    }
  }
  const int64_t pair_tiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + BN - 1) / BN);
  const bool pair = !window && m > BM && k >= 1024 && pair_kernel_enabled() &&
                    pair_tiles >= max_pairs(dev);
  if (!make_map(&ma, a, m, k, lda, BM) || !make_map(&mw, w, n, k, ldw, pair ? P_BN_HALF : tbn))
    return CUGO_B200_ERR_LAUNCH;
  if (pair) {
    // 256 x 256 tiles, one CTA pair per tile, persistent over the co-resident pairs.
    const int64_t pairs = pair_tiles < max_pairs(dev) ? pair_tiles : max_pairs(dev);
    gemm_pair_kernel<<<static_cast<unsigned>(2 * pairs), THREADS, P_SMEM_BYTES, stream>>>(
        ma, mw, mo, mr, ep);
  } else {
    const int64_t tiles = tiles_m * ((n + tbn - 1) / tbn);
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    if (tbn == 256)
      gemm_kernel<256><<<grid, THREADS, g_smem_bytes(256), stream>>>(ma, mw, mo, mr, ep);
    else if (tbn == 128)
      gemm_kernel<128><<<grid, THREADS, g_smem_bytes(128), stream>>>(ma, mw, mo, mr, ep);
    else
      gemm_kernel<64><<<grid, THREADS, g_smem_bytes(64), stream>>>(ma, mw, mo, mr, ep);
  }
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int cugo_b200_gemm_bf16_ex(const void* a, int64_t lda, const void* w, int64_t ldw,
                           const void* bias, int32_t bias_fp32, const void* residual,
                           int64_t ldr, void* out, int64_t ldo, int32_t out_fp32, int32_t act,
                           int32_t act_after, int64_t m, int64_t n, int64_t k, int32_t* error,
                           cudaStream_t stream) {
  return gemm_launch(a, lda, w, ldw, bias, bias_fp32, residual, ldr, out, ldo, out_fp32, act,
                     act_after, m, n, k, nullptr, error, stream);
}

int cugo_b200_gemm_bf16_pre(const void* a, int64_t lda, const void* w, int64_t ldw,
                            const void* bias, int32_t bias_fp32, void* out, int64_t ldo, void* pre,
                            int64_t ldp, int32_t act, int64_t m, int64_t n, int64_t k,
                            int32_t* error, cudaStream_t stream) {
  if (!pre) return CUGO_B200_ERR_ARG;
  return gemm_launch(a, lda, w, ldw, bias, bias_fp32, nullptr, 0, out, ldo, 0, act, 0, m, n, k,
                     nullptr, error, stream, pre, ldp);
}

int cugo_b200_gemm_bf16_window(const void* a, int64_t lda, const void* w, int64_t ldw,
                               const void* bias, int32_t bias_fp32, const void* residual,
                               int64_t ldr, void* out, int64_t ldo, int32_t out_fp32,
                               int32_t act, int32_t act_after, int64_t m, int64_t n, int64_t k,
                               const int32_t* window, int32_t* error, cudaStream_t stream) {
  if (!window || (reinterpret_cast<uintptr_t>(window) & 3u)) return CUGO_B200_ERR_ARG;
  return gemm_launch(a, lda, w, ldw, bias, bias_fp32, residual, ldr, out, ldo, out_fp32, act,
                     act_after, m, n, k, window, error, stream);
}

}  // extern "C"

namespace {

// ---- weight gradients: dW = dY^T X over the rows (split-K) --------------------------
//
// dW[o][i] = sum_r dY[r][o] X[r][i]: both operands are row-major over the reduction
// dimension (the minibatch rows), so they enter the MMA MN-major: TMA boxes of 64
// rows x 64 consecutive outputs (or inputs), 128-byte swizzled, stacked 8 KB apart
// along M (N); the shared-memory descriptors step 1 KB per 8-row group (stride
// byte offset) and 8 KB per 64-wide block (leading byte offset), and the
// instruction descriptor marks A and B transposed.  A 128 x 256 tile of dW has far
// too little work for the SM count over one K loop, so the rows are split: a work
// item is (tile, split), each writing its fp32 partial tile into a workspace
// [splits][Mpad][Npad]; wgrad_reduce_kernel adds the splits in order
// (deterministic).  Warp roles, barriers and bounded waits as in gemm_kernel.
struct WgradArgs {
  float* ws;
  int64_t mpad, npad;
  int tiles_m, tiles_n, splits, kt_per_split, k_tiles;
  int* error;
};

__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t addr) {
  uint64_t d = static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(8192 >> 4) << 16;   // leading byte offset: next 64-wide block
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1) << 46;           // descriptor version
  d |= static_cast<uint64_t>(2) << 61;           // 128-byte swizzle
  return d;
}

constexpr uint32_t kWgradIdesc = instr_desc(BM, BN) | (1u << 15) | (1u << 16);  // A, B MN-major

__global__ void __launch_bounds__(THREADS, 1)
    wgrad_kernel(const __grid_constant__ CUtensorMap map_dy, const __grid_constant__ CUtensorMap map_x,
                 const WgradArgs wa) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drained + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int items = wa.tiles_m * wa.tiles_n * wa.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);
    }
    mbar_init(drained, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_holder)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool failed = false;
  // Item -> (tile m, tile n, split) and its k-tile range [kt0, kt1).
  const auto decode = [&](int item, int& tm, int& tn, int& split, int& kt0, int& kt1) {
    const int tile = item / wa.splits;
    split = item - tile * wa.splits;
    tm = tile / wa.tiles_n;
    tn = tile - tm * wa.tiles_n;
    kt0 = split * wa.kt_per_split;
    kt1 = kt0 + wa.kt_per_split < wa.k_tiles ? kt0 + wa.kt_per_split : wa.k_tiles;
  };

  if (warp == 0) {
    // ---- TMA producer: per stage two 64-wide blocks of dY and four of X ----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int it = blockIdx.x; it < items && !failed; it += gridDim.x) {
        int tm, tn, split, kt0, kt1;
        decode(it, tm, tn, split, kt0, kt1);
        for (int kt = kt0; kt < kt1; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            failed = true;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          mbar_expect_tx(&full[stage], STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < BM / 64; ++h)
            tma_load_2d(&map_dy, &full[stage], sa + h * 8192, tm * BM + 64 * h, kt * BK);
#pragma unroll
          for (int q = 0; q < BN / 64; ++q)
            tma_load_2d(&map_x, &full[stage], sa + A_BYTES + q * 8192, tn * BN + 64 * q, kt * BK);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (failed) {
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full[s], 0);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      for (int it = blockIdx.x; it < items && !failed; it += gridDim.x, ++iter) {
        int tm, tn, split, kt0, kt1;
        decode(it, tm, tn, split, kt0, kt1);
        const int buf = iter & 1;
        const uint32_t use = static_cast<uint32_t>(iter >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u)) {
          failed = true;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kt = kt0; kt < kt1; ++kt) {
          if (!mbar_wait(&full[stage], phase)) {
            failed = true;
            break;
          }
          fence_after();
          const uint32_t a_addr = smem_addr(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {  // 16 rows = two 8-row groups
            mma_bf16(d_tmem, sw128_mn_desc(a_addr + kk * 2048), sw128_mn_desc(b_addr + kk * 2048),
                     kWgradIdesc, (kt > kt0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (failed) break;
        mma_commit(&acc_full[buf]);
      }
      mma_commit(drained);
      mbar_wait(drained, 0);
    }
  } else {
    // ---- epilogue: warps 2..9, two per TMEM lane quadrant, 128 columns each ----
    const int quad = epi_quad(warp);
    const int cbase = epi_col0(warp);
    int iter = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++iter) {
      int tm, tn, split, kt0, kt1;
      decode(it, tm, tn, split, kt0, kt1);
      const int buf = iter & 1;
      const uint32_t use = static_cast<uint32_t>(iter >> 1);
      if (!epilogue_wait(&acc_full[buf], use & 1u)) {
        failed = true;
        break;
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(buf * BN + cbase);
      float* row = wa.ws + ((int64_t)split * wa.mpad + (int64_t)tm * BM + quad * 32 + lane) * wa.npad +
                   (int64_t)tn * BN + cbase;
#pragma unroll 1
      for (int c = 0; c < BN / 2; c += 32) {
        uint32_t r[32];
        CB_TMEM_LD32(taddr + c, r);
        tmem_wait_ld();
        float4* dst = reinterpret_cast<float4*>(row + c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                               __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  if (failed) {
    if (wa.error) atomicExch(wa.error, 1);
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 100'000ull) {
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

// out[o][i] = sum over the splits, in order, of ws[split][o][i] (four columns per
// thread).
__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float* __restrict__ ws, int64_t mpad,
                                                           int64_t npad, int splits, int64_t m,
                                                           int64_t n, float* __restrict__ out,
                                                           int64_t ldo) {
  const int64_t quads = npad / 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= m * quads) return;
  const int64_t o = idx / quads, i0 = (idx - o * quads) * 4;
  if (i0 >= n) return;
  float4 acc = __ldg(reinterpret_cast<const float4*>(ws + o * npad + i0));
  for (int s = 1; s < splits; ++s) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(ws + ((int64_t)s * mpad + o) * npad + i0));
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  float* dst = out + o * ldo + i0;
  const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (i0 + e < n) dst[e] = a[e];
}

// Split count and k-tiles per split for a weight-gradient launch.
struct WgradPlan {
  int tiles_m, tiles_n, k_tiles, splits, kt_per_split;
  int64_t mpad, npad;
};

WgradPlan wgrad_plan(int64_t rows, int64_t n_out, int64_t n_in) {
  WgradPlan p{};
  p.tiles_m = static_cast<int>((n_out + BM - 1) / BM);
  p.tiles_n = static_cast<int>((n_in + BN - 1) / BN);
  p.k_tiles = static_cast<int>((rows + BK - 1) / BK);
  const int tiles = p.tiles_m * p.tiles_n;
  int want = sm_count() / tiles;  // at most one item per SM: no second wave
  if (want < 1) want = 1;
  p.kt_per_split = (p.k_tiles + want - 1) / want;
  if (p.kt_per_split < 4) p.kt_per_split = 4;  // at least 256 rows per item
  p.splits = (p.k_tiles + p.kt_per_split - 1) / p.kt_per_split;
  if (p.splits < 1) p.splits = 1;
  p.mpad = static_cast<int64_t>(p.tiles_m) * BM;
  p.npad = static_cast<int64_t>(p.tiles_n) * BN;
  return p;
}

}  // namespace

extern "C" {

int64_t cugo_b200_wgrad_scratch_floats(int64_t rows, int64_t n_out, int64_t n_in) {
  if (rows <= 0 || n_out <= 0 || n_in <= 0) return 0;
  const WgradPlan p = wgrad_plan(rows, n_out, n_in);
  return static_cast<int64_t>(p.splits) * p.mpad * p.npad;
}

int cugo_b200_wgrad_bf16(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t rows,
                         int64_t n_out, int64_t n_in, float* dw, int64_t lddw, float* scratch,
                         int64_t scratch_floats, int32_t* error, cudaStream_t stream) {
  if (rows < 0 || n_out <= 0 || n_in <= 0 || lddy < n_out || ldx < n_in || lddw < n_in || !dw)
    return CUGO_B200_ERR_ARG;
  if (rows > INT32_MAX || n_out > INT32_MAX || n_in > INT32_MAX) return CUGO_B200_ERR_ARG;
  if (rows == 0) {
    for (int64_t o = 0; o < n_out; ++o)
      if (cudaMemsetAsync(dw + o * lddw, 0, n_in * sizeof(float), stream) != cudaSuccess)
        return CUGO_B200_ERR_LAUNCH;
    return CUGO_B200_OK;
  }
  if (!dy || !x) return CUGO_B200_ERR_ARG;
  const auto al = [](const void* p, uintptr_t q) { return (reinterpret_cast<uintptr_t>(p) % q) == 0; };
  if (!al(dy, 16) || !al(x, 16) || (lddy * 2) % 16 || (ldx * 2) % 16 || !al(dw, 4))
    return CUGO_B200_ERR_ALIGN;
  const WgradPlan p = wgrad_plan(rows, n_out, n_in);
  const int64_t need = static_cast<int64_t>(p.splits) * p.mpad * p.npad;
  if (!scratch || scratch_floats < need) return CUGO_B200_ERR_CAPACITY;
  if (!al(scratch, 16)) return CUGO_B200_ERR_ALIGN;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {};
  if (dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
        cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  // Boxes of 64 rows (K) x 64 consecutive columns (M or N), 128-byte swizzle.
  CUtensorMap mdy, mx;
  if (!make_map(&mdy, dy, rows, n_out, lddy, BK) || !make_map(&mx, x, rows, n_in, ldx, BK))
    return CUGO_B200_ERR_LAUNCH;
  WgradArgs wa{scratch, p.mpad, p.npad, p.tiles_m, p.tiles_n, p.splits, p.kt_per_split, p.k_tiles, error};
  const int items = p.tiles_m * p.tiles_n * p.splits;
  const int grid = items < sm_count() ? items : sm_count();
  wgrad_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(mdy, mx, wa);
  const int64_t threads = n_out * (p.npad / 4);
  wgrad_reduce_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      scratch, p.mpad, p.npad, p.splits, n_out, n_in, dw, lddw);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // extern "C"

namespace {

// One-output layer (the scalar value head, python/cugo_ppo_nets50.py:82):
// out[r] = a[r, :k] . w[:k] + bias.  A GEMM tile would spend 255 of its 256
// columns on nothing, so this is a row reduction at HBM speed instead: a warp per
// row, each lane holding its 16-byte pieces of w in registers (k <= 2,048 and a
// multiple of 8), four rows in flight per warp, a fixed shuffle tree (the result
// does not depend on the launch shape).
constexpr int kDotMaxPieces = 8;  // 8 x 8 bf16 per lane: k <= 2,048

__global__ void __launch_bounds__(256) rowdot_kernel(const __nv_bfloat16* __restrict__ a,
                                                     int64_t lda, const float* __restrict__ w,
                                                     const float* __restrict__ bias, int64_t m,
                                                     int k, float* __restrict__ out, int64_t ldo) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int pieces = k >> 3;
  float wr[kDotMaxPieces][8];
#pragma unroll
  for (int j = 0; j < kDotMaxPieces; ++j) {
    const int p = lane + 32 * j;
#pragma unroll
    for (int e = 0; e < 8; ++e) wr[j][e] = p < pieces ? __ldg(w + 8 * p + e) : 0.0f;
  }
  const float b = bias ? __ldg(bias) : 0.0f;
  for (int64_t r0 = warp * 4; r0 < m; r0 += warps * 4) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < kDotMaxPieces; ++j) {
      const int p = lane + 32 * j;
      if (32 * j >= pieces) break;
      uint4 raw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        raw[q] = (p < pieces && r0 + q < m)
                     ? __ldcs(reinterpret_cast<const uint4*>(a + (r0 + q) * lda) + p)
                     : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[q] = fmaf(f.x, wr[j][2 * e], acc[q]);
          acc[q] = fmaf(f.y, wr[j][2 * e + 1], acc[q]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], off);
    }
    if (lane < 4 && r0 + lane < m) {
      const float v = lane == 0 ? acc[0] : (lane == 1 ? acc[1] : (lane == 2 ? acc[2] : acc[3]));
      out[(r0 + lane) * ldo] = v + b;
    }
  }
}

}  // namespace

extern "C" {

int cugo_b200_rowdot_bf16(const void* a, int64_t lda, const float* w, const float* bias,
                          int64_t m, int64_t k, float* out, int64_t ldo, cudaStream_t stream) {
  if (m < 0 || k <= 0 || k > 8 * 32 * kDotMaxPieces || k % 8 || lda < k || ldo < 1)
    return CUGO_B200_ERR_ARG;
  if (m == 0) return CUGO_B200_OK;
  if (!a || !w || !out) return CUGO_B200_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a) & 15u) || lda % 8 || (reinterpret_cast<uintptr_t>(w) & 3u))
    return CUGO_B200_ERR_ALIGN;
  const int64_t warps_needed = (m + 3) / 4;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8 * 8;  // 8 blocks of 8 warps per SM
  const int64_t warps = warps_needed < cap ? warps_needed : cap;
  rowdot_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(a), lda, w, bias, m, static_cast<int>(k), out, ldo);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

int cugo_b200_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                        const void* residual, int64_t ldr, void* out, int64_t ldo,
                        int32_t out_fp32, int32_t act, int32_t act_after, int64_t m, int64_t n,
                        int64_t k, int32_t* error, cudaStream_t stream) {
  if (act > 2 || act_after > 2) return CUGO_B200_ERR_ARG;
  if (residual && out_fp32) return CUGO_B200_ERR_ARG;  // this entry's residual stream is bf16
  return cugo_b200_gemm_bf16_ex(a, lda, w, ldw, bias, 0, residual, ldr, out, ldo, out_fp32, act,
                                act_after, m, n, k, error, stream);
}

}  // extern "C"

namespace {

// ---- the whole residual MLP in one kernel (hidden width 512) ------------------------
//
//   h = x W0^T + b0;  per block: h = h + act(h W1^T + b1) W2^T + b2;  out = act(h) Wo^T + bo
//
// (python/cugo_ppo_nets50.py:26-64, norm "none").  At hidden 512 every layer of the
// layer-per-launch path is bound by moving activations through HBM (a 512-wide bf16
// row is 1 KB in and 1 KB out per layer for 0.5 MFLOP); here the activations stay on
// chip for the whole network.  A CTA pair (cluster of 2, tcgen05 cta_group::2) owns a
// 256-row tile, 128 rows per CTA:
//   shared memory  ACT: the CTA's 128 x 512 bf16 activations (128 KB) in the
//                  128-byte-swizzled K-major layout the MMA reads (8 chunks of 64
//                  columns), rewritten in place layer after layer; during the input
//                  layer its chunks hold the x tiles streamed in by TMA, after the
//                  head it stages the fp32 output for TMA stores;
//                  a 5-stage ring of weight tiles: each stage is this CTA's half
//                  (128 rows x 64) of a 256-row tile (16 KB), so each SM streams
//                  half of every weight tile and the bytes in flight cover twice the
//                  MMA work a single CTA's would;
//                  the fp32 biases of the input and hidden layers (up to 8 vectors of
//                  512), copied in once per launch: the epilogue reads 16 columns'
//                  biases as four 16-byte broadcasts instead of a load and 16 shuffles;
//   tensor memory  the fp32 accumulator of a whole layer, 128 lanes x 512 columns;
//                  the head's (at most 256 columns) in the upper half, so the next
//                  tile's input-layer MMAs into the lower half overlap the head
//                  epilogue, and the sampling head's column groups meet there too.
// A block's residual never leaves the chip: the fc1 epilogue reads h from ACT, writes
// h + b2 into the accumulator columns it has just drained (tcgen05.st) and u = act(z)
// over h in ACT, so the fc2 MMAs accumulate u W2^T on top of h + b2.
// Warp roles: warp 0 of each CTA the TMA producer of its half (weights run ahead of
// the MMAs; x tiles wait for the previous tile's head MMAs, and for its output stores
// to leave ACT when there are any), warp 1
// of CTA 0 the MMA issuer (M = 256 MMAs reading both CTAs' shared memory), the other
// F_EPI_WARPS warps of each CTA the epilogue of its 128 rows (F_EPI_WARPS / 4 per
// TMEM lane quadrant, each a contiguous group of columns, 16 columns at a time).  Copies count on CTA 0's "full" barriers; MMA completions arrive on
// both CTAs' barriers; both CTAs' epilogue warps signal CTA 0's "ready" barrier.
// Every wait is bounded as in gemm_kernel.
constexpr int F_H = 512;
constexpr int F_CHUNKS = F_H / BK;            // 8
constexpr int F_CHUNK_BYTES = BM * BK * 2;    // 16 KB
constexpr int F_ACT_BYTES = F_CHUNKS * F_CHUNK_BYTES;
constexpr int F_WSTAGES = 5;
constexpr int F_BIAS_SLOTS = 8;                        // bias vectors kept in shared memory
constexpr int F_BIAS_BYTES = F_BIAS_SLOTS * F_H * 4;  // 16 KB
constexpr int F_W_ROWS = BN / 2;              // weight rows per CTA per stage
constexpr int F_W_BYTES = F_W_ROWS * BK * 2;  // 16 KB
constexpr int F_MAX_BLOCKS = 4;
constexpr int F_MAX_LAYERS = 2 + 2 * F_MAX_BLOCKS;
constexpr int F_MAX_KIN = 1024;
constexpr int F_SMEM_BYTES =
    F_ACT_BYTES + F_WSTAGES * F_W_BYTES + F_BIAS_BYTES + 1024 /*align*/ + 512 /*barriers*/;
// Epilogue warps per CTA: F_EPI_WARPS / 4 per TMEM lane quadrant, each draining
// 512 / (F_EPI_WARPS / 4) columns in 16-column chunks.
#ifndef CB_FUSED_EPI_WARPS
#define CB_FUSED_EPI_WARPS 16
#endif
constexpr int F_EPI_WARPS = CB_FUSED_EPI_WARPS;
constexpr int F_THREADS = 64 + 32 * F_EPI_WARPS;
constexpr int F_GROUPS = F_EPI_WARPS / 4;        // column groups per quadrant
constexpr int F_GROUP_COLS = F_H / F_GROUPS;
constexpr int F_CW = 16;                         // columns per epilogue chunk
static_assert(F_EPI_WARPS % 4 == 0 && F_GROUP_COLS % F_CW == 0, "epilogue split");
// The head's output staging sits in the upper half of ACT (chunks F_STAGE_CHUNK ..),
// so the next tile's first x chunks can load while the head stores.
constexpr int F_STAGE_CHUNK = F_CHUNKS / 2;
static_assert(F_EPI_WARPS * 2 * EPI_BUF <= F_ACT_BYTES - F_STAGE_CHUNK * F_CHUNK_BYTES,
              "output staging fits in the upper half of ACT");
static_assert(F_SMEM_BYTES <= 232448, "fits the opt-in shared memory of one CTA");

struct FusedMaps {
  CUtensorMap x;                    // bf16 [m, k_in], box 64 x 128
  CUtensorMap w[F_MAX_LAYERS];      // bf16 [n, k] per layer, box 64 x 128 (head: n_mma / 2)
  CUtensorMap out;                  // fp32 [m, n_out], box 16 x 32, 64-byte swizzle
};

struct FusedArgs {
  const float* bias[F_MAX_LAYERS];  // fp32 [n] or null
  int blocks, m, k_in, n_out, n_mma, act;
  int* error;
  int write_out;                    // store the outputs (maps.out) or not
  // Sampling head (actions != null): masked Gumbel-max over the first 179 outputs,
  // with the noise and tie rules of cugo_b200_sample_actions.
  const uint64_t* legal_bits;       // [m, 3]: bit a of word a / 64
  const int64_t* game;              // [m], or [n_games] read through rows
  const int32_t* decision;          // [m], or [n_games] read through rows
  const int64_t* rows;              // optional [m]: row r's entry of game and decision
  int64_t n_games;
  int64_t seed_base;
  int greedy;
  int64_t* actions;                 // [m]
  float* logp;                      // [m]
  const int32_t* m_dev;             // optional device-resident row count (at most m)
};

constexpr int F_ACTIONS = 179;

// A thread's running state of the sampling head over the columns it has seen.
struct SampleState {
  float best;   // best score (logit + noise), lowest action on ties
  int best_a;   // -1: no legal action seen
  float best_x; // the logit of best_a
  float mx;     // running maximum of the legal logits
  float sum;    // sum of exp(x - mx) over the legal logits
};

// Folds 16 outputs col0 .. col0 + 15 of the thread's row into the state (legal
// actions only); bits: the row's legal actions col0 .. col0 + 15.  The loop runs over
// the set bits in ascending order (the order, and so the result, of a scan over all
// 16 columns), so a warp pays for its lanes' legal actions, not for every column.
__device__ __forceinline__ void sample_chunk(const FusedArgs& args, uint64_t gid, uint32_t dec,
                                             int col0, uint32_t bits, const float* v,
                                             SampleState& st) {
  const uint64_t seed = static_cast<uint64_t>(args.seed_base) + gid;
  while (bits) {
    const int e = __ffs(bits) - 1;
    bits &= bits - 1;
    float x = v[0];
#pragma unroll
    for (int j = 1; j < 16; ++j) x = e == j ? v[j] : x;  // v[e] without local memory
    const int a = col0 + e;
    float score = x;
    if (!args.greedy) {
      const cb::Philox4 ph = cb::philox4x32_10(
          static_cast<uint32_t>(gid), static_cast<uint32_t>(gid >> 32), dec,
          3u | (static_cast<uint32_t>(a >> 2) << 8), static_cast<uint32_t>(seed),
          static_cast<uint32_t>(seed >> 32));
      const int w = a & 3;
      const uint32_t r = w == 0 ? ph.v[0] : (w == 1 ? ph.v[1] : (w == 2 ? ph.v[2] : ph.v[3]));
      score = x + cb::gumbel_of(r);
    }
    if (score > st.best) {  // ascending actions: the first maximum is kept
      st.best = score;
      st.best_a = a;
      st.best_x = x;
    }
    if (x > st.mx) {
      st.sum = st.sum * expf(st.mx - x) + 1.0f;  // exp(-inf) = 0 on the first legal logit
      st.mx = x;
    } else {
      st.sum += expf(x - st.mx);
    }
  }
}

// ACT address of 16-byte piece p (0..7) of row r in chunk kc: the TMA 128-byte swizzle.
__device__ __forceinline__ uint8_t* act_piece(uint8_t* act, int kc, int r, int p) {
  return act + kc * F_CHUNK_BYTES + r * 128 + ((p ^ (r & 7)) << 4);
}

// Row r's 16 columns col0 .. col0 + 15 (col0 a multiple of 16) as bf16 into ACT.
__device__ __forceinline__ void act_store16(uint8_t* act, int r, int col0, const float* v) {
  const int kc = col0 >> 6, p0 = (col0 & 63) >> 3;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
    *reinterpret_cast<uint4*>(act_piece(act, kc, r, p0 + j)) = raw;
  }
}

// act_store16 of max(v, 0): the ReLU folded into the bf16 conversion (the same bits as
// rounding max(v, 0)).
__device__ __forceinline__ void act_store16_relu(uint8_t* act, int r, int col0, const float* v) {
  const int kc = col0 >> 6, p0 = (col0 & 63) >> 3;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;"
          : "=r"(w[e])
          : "f"(v[8 * j + 2 * e + 1]), "f"(v[8 * j + 2 * e]));
    *reinterpret_cast<uint4*>(act_piece(act, kc, r, p0 + j)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__device__ __forceinline__ void act_load16(uint8_t* act, int r, int col0, float* v) {
  const int kc = col0 >> 6, p0 = (col0 & 63) >> 3;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint4 raw = *reinterpret_cast<const uint4*>(act_piece(act, kc, r, p0 + j));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[8 * j + 2 * e] = f.x;
      v[8 * j + 2 * e + 1] = f.y;
    }
  }
}

// The 16 biases col0 .. col0 + 15 (columns from `limit` on read 0): lanes 0..15 load
// one each and shuffles hand them to every lane.
__device__ __forceinline__ void fused_bias16(const float* b, int col0, int limit, float* out) {
  const int lane = threadIdx.x & 31;
  const float mine = (b && lane < 16 && col0 + lane < limit) ? __ldg(b + col0 + lane) : 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = __shfl_sync(0xffffffffu, mine, j);
}

// The 16 biases col0 .. col0 + 15 of layer `layer` (input or hidden, all columns below
// 512): from the shared-memory copy (every lane reads the same 16 bytes four times),
// or for a layer past the staged ones from global memory.
__device__ __forceinline__ void fused_layer_bias16(const float* bias_s, const float* b, int layer,
                                                   int col0, float* out) {
  if (layer >= F_BIAS_SLOTS) {
    fused_bias16(b, col0, F_H, out);
    return;
  }
  const float4* p = reinterpret_cast<const float4*>(bias_s + layer * F_H + col0);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 t = p[q];
    out[4 * q] = t.x;
    out[4 * q + 1] = t.y;
    out[4 * q + 2] = t.z;
    out[4 * q + 3] = t.w;
  }
}

#define CB_TMEM_ST16(taddr, r)                                                                  \
  asm volatile(                                                                                 \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"   \
      "%13,%14,%15,%16};" ::"r"(taddr),                                                         \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),   \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),        \
      "r"(r[15])                                                                                \
      : "memory")

// An epilogue phase is done: its TMEM reads/writes and ACT writes are visible to the
// pair's MMAs that follow (one arrive per epilogue warp on CTA 0's barrier).
__device__ __forceinline__ void fused_phase_done(uint32_t ready0) {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(ready0);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(F_THREADS, 1)
    fused_mlp_kernel(const __grid_constant__ FusedMaps maps, const __grid_constant__ FusedArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* act = smem;
  uint8_t* wring = smem + F_ACT_BYTES;
  float* bias_s = reinterpret_cast<float*>(wring + F_WSTAGES * F_W_BYTES);  // [F_BIAS_SLOTS][512]
  uint64_t* wfull = reinterpret_cast<uint64_t*>(wring + F_WSTAGES * F_W_BYTES + F_BIAS_BYTES);
  uint64_t* wempty = wfull + F_WSTAGES;
  uint64_t* xfull = wempty + F_WSTAGES;  // [8]
  uint64_t* xempty = xfull + F_CHUNKS;   // [8]
  uint64_t* acc_full = xempty + F_CHUNKS;
  uint64_t* act_ready = acc_full + 1;    // CTA 0's counts both CTAs' epilogue warps
  uint64_t* act_free = act_ready + 1;    // this CTA's ACT is free for the next x tiles
  uint64_t* drained = act_free + 1;
  uint64_t* sample_ready = drained + 1;  // [4]: a quadrant's other column groups posted
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sample_ready + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
  int m_rows = args.m;
  if (args.m_dev) {
    const int md = __ldg(args.m_dev);
    m_rows = md < 0 ? 0 : (md < m_rows ? md : m_rows);
  }
  const int tiles = (m_rows + 2 * BM - 1) / (2 * BM);
  const int kc0 = (args.k_in + BK - 1) / BK;
  const int kfirst = kc0 < F_CHUNKS ? kc0 : F_CHUNKS;  // input chunks in the first pass
  const int hidden_layers = 2 * args.blocks;
  const int head_rows = args.n_mma / 2;  // head weight rows per CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < F_WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < F_CHUNKS; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(act_ready, 2 * F_EPI_WARPS);
    mbar_init(act_free, F_EPI_WARPS);
    mbar_init(drained, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&sample_ready[q], F_GROUPS - 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // both CTAs allocate together, same warp, same holder offset
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_holder)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  // The biases of layers 0 .. min(hidden_layers, F_BIAS_SLOTS - 1) (zeros for none).
  const int staged = (hidden_layers + 1 < F_BIAS_SLOTS ? hidden_layers + 1 : F_BIAS_SLOTS) * F_H;
  for (int i = threadIdx.x; i < staged; i += blockDim.x) {
    const float* b = args.bias[i / F_H];
    bias_s[i] = b ? __ldg(b + i % F_H) : 0.0f;
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool failed = false;
  __shared__ int any_failed;
  if (threadIdx.x == 0) any_failed = 0;
  __syncthreads();

  if (warp == 0) {
    // ---- TMA producer (both CTAs): this CTA's halves of the weight tiles in MMA
    // order, its 128 rows of the x tiles into its ACT chunks ----
    if (lane == 0) {
      const uint32_t wfull0 = peer_addr(wfull, 0), xfull0 = peer_addr(xfull, 0);
      int ws = 0;
      uint32_t wph = 0, xuse = 0;
      auto load_w = [&](int layer, int kc, int row0, int tx_bytes) -> bool {
        if (!mbar_wait(&wempty[ws], wph ^ 1u)) return false;
        if (leader) mbar_expect_tx(&wfull[ws], static_cast<uint32_t>(tx_bytes));
        tma_load_2d_pair(&maps.w[layer], wfull0 + static_cast<uint32_t>(ws * 8),
                         wring + ws * F_W_BYTES, kc * BK, row0);
        if (++ws == F_WSTAGES) {
          ws = 0;
          wph ^= 1u;
        }
        return true;
      };
      const int rh = static_cast<int>(rank) * F_W_ROWS;  // this CTA's rows of a 256-row tile
      int iter = 0;
      for (int t = pair; t < tiles && !failed; t += pairs, ++iter) {
        const int row0 = t * 2 * BM + static_cast<int>(rank) * BM;
        // The input layer in the MMA's order: its first (up to) eight 64-column chunks
        // for accumulator half 0, the same chunks for half 1, then the rest of K
        // (chunk kc in ACT slot kc - 8) for half 0 and half 1.
        auto load_x = [&](int kc) -> bool {
          const int slot = kc & (F_CHUNKS - 1);
          if (iter > 0) {
            // ACT takes this tile's x once the previous tile's head MMAs have read it;
            // when the head stores outputs (through the upper chunks of ACT), chunks
            // from free_at on also wait for those stores to leave.  (A tile with
            // stores waits act_free exactly once, so no phase is skipped.)
            const int free_at = kfirst - 1 < F_STAGE_CHUNK ? kfirst - 1 : F_STAGE_CHUNK;
            if (kc == 0 && !(args.write_out && free_at == 0) &&
                !mbar_wait(acc_full, static_cast<uint32_t>(iter * (hidden_layers + 2) - 1) & 1u))
              return false;
            if (args.write_out && kc == free_at && !mbar_wait(act_free, (iter - 1) & 1)) return false;
          }
          // A slot's second x tile of this tile waits for the MMAs of its first.
          if (kc >= F_CHUNKS && !mbar_wait(&xempty[slot], ((xuse >> slot) & 1u) ^ 1u)) return false;
          if (leader) mbar_expect_tx(&xfull[slot], 2 * F_CHUNK_BYTES);
          tma_load_2d_pair(&maps.x, xfull0 + static_cast<uint32_t>(slot * 8),
                           act + slot * F_CHUNK_BYTES, kc * BK, row0);
          xuse ^= 1u << slot;
          return true;
        };
        // x chunk 8 + i goes into slot i as soon as half 1 has read chunk i, X_LAG
        // half-1 weight tiles later (the ring keeps the MMAs fed meanwhile).
        constexpr int X_LAG = 3;
        int next_x = F_CHUNKS;
        for (int kc = 0; kc < kfirst && !failed; ++kc)
          if (!load_w(0, kc, rh, 2 * F_W_BYTES) || !load_x(kc)) failed = true;
        for (int kc = 0; kc < kfirst && !failed; ++kc) {
          if (!load_w(0, kc, BN + rh, 2 * F_W_BYTES)) failed = true;
          if (!failed && kc >= X_LAG && next_x < kc0 && next_x - F_CHUNKS <= kc - X_LAG)
            if (!load_x(next_x++)) failed = true;
        }
        for (; next_x < kc0 && !failed; ++next_x)
          if (!load_x(next_x)) failed = true;
        for (int nh = 0; nh < 2 && !failed; ++nh)
          for (int kc = F_CHUNKS; kc < kc0 && !failed; ++kc)
            if (!load_w(0, kc, nh * BN + rh, 2 * F_W_BYTES)) failed = true;
        for (int l = 1; l <= hidden_layers && !failed; ++l)
          for (int kc = 0; kc < F_CHUNKS && !failed; ++kc)
            if (!load_w(l, kc, rh, 2 * F_W_BYTES) || !load_w(l, kc, BN + rh, 2 * F_W_BYTES))
              failed = true;
        for (int kc = 0; kc < F_CHUNKS && !failed; ++kc)
          if (!load_w(hidden_layers + 1, kc, static_cast<int>(rank) * head_rows,
                      args.n_mma * BK * 2))
            failed = true;
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (CTA 0 only) ----
    if (leader && lane == 0) {
      constexpr uint32_t idesc_h = instr_desc(2 * BM, BN);
      const uint32_t idesc_o = instr_desc(2 * BM, args.n_mma);
      int ws = 0;
      uint32_t wph = 0, xuse = 0, ready = 0;
      auto wait_ready = [&]() -> bool {
        const bool ok = mbar_wait(act_ready, ready & 1u);
        ++ready;
        fence_after();
        return ok;
      };
      // One 64-deep K step: a_addr the A chunk, into accumulator column block nh; only
      // the first `sub` 16-deep MMAs when the rest of the chunk is past K (zero fill).
      auto k_step = [&](uint32_t a_addr, int nh, uint32_t idesc, bool first,
                        int sub = BK / 16) -> bool {
        if (!mbar_wait(&wfull[ws], wph)) return false;
        fence_after();
        const uint32_t b_addr = smem_addr(wring + ws * F_W_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          if (kk < sub)
            mma_bf16_pair(tmem_base + static_cast<uint32_t>(nh * BN), sw128_desc(a_addr + kk * 32),
                          sw128_desc(b_addr + kk * 32), idesc, (first && kk == 0) ? 0u : 1u);
        mma_commit_pair(&wempty[ws]);
        if (++ws == F_WSTAGES) {
          ws = 0;
          wph ^= 1u;
        }
        return true;
      };
      int iter = 0;
      for (int t = pair; t < tiles && !failed; t += pairs, ++iter) {
        // Input layer, half 0 then half 1 over the resident x chunks, then the rest
        // of K.  Half 0 (columns 0..255) is free: the previous tile's last hidden
        // epilogue drained it before the head MMAs, whose accumulator is in half 1.
        // So these MMAs run while the previous tile's head epilogue samples; half 1
        // waits for it.
        for (int part = 0; part < 2 && !failed; ++part) {
          const int k0 = part ? F_CHUNKS : 0, k1 = part ? kc0 : kfirst;
          for (int nh = 0; nh < 2 && !failed; ++nh) {
            if (part == 0 && nh == 1 && iter > 0 && !wait_ready()) {
              failed = true;
              break;
            }
            for (int kc = k0; kc < k1 && !failed; ++kc) {
              const int slot = kc & (F_CHUNKS - 1);
              if (nh == 0) {
                if (!mbar_wait(&xfull[slot], (xuse >> slot) & 1u)) {
                  failed = true;
                  break;
                }
                xuse ^= 1u << slot;
                fence_after();
              }
              const int rest = (args.k_in - kc * BK + 15) / 16;  // 16-deep steps left in K
              if (!k_step(smem_addr(act + slot * F_CHUNK_BYTES), nh, idesc_h, kc == 0,
                          rest < BK / 16 ? rest : BK / 16)) {
                failed = true;
                break;
              }
              if (nh == 1) mma_commit_pair(&xempty[slot]);  // the chunk's last reader
            }
          }
        }
        if (failed) break;
        mma_commit_pair(acc_full);
        for (int l = 1; l <= hidden_layers && !failed; ++l) {
          if (!wait_ready()) {
            failed = true;
            break;
          }
          // fc2 (even l) accumulates onto h + b2, which its epilogue left in TMEM.
          const bool fresh = (l & 1) == 1;
          for (int kc = 0; kc < F_CHUNKS && !failed; ++kc) {
            const uint32_t a_addr = smem_addr(act + kc * F_CHUNK_BYTES);
            if (!k_step(a_addr, 0, idesc_h, fresh && kc == 0) ||
                !k_step(a_addr, 1, idesc_h, fresh && kc == 0))
              failed = true;
          }
          if (!failed) mma_commit_pair(acc_full);
        }
        if (failed || !wait_ready()) {
          failed = true;
          break;
        }
        // The head accumulates into half 1, so the next tile's half 0 need not wait
        // for the head epilogue.
        for (int kc = 0; kc < F_CHUNKS && !failed; ++kc)
          if (!k_step(smem_addr(act + kc * F_CHUNK_BYTES), 1, idesc_o, kc == 0)) failed = true;
        if (!failed) mma_commit_pair(acc_full);
      }
      // All issued MMAs complete before the accumulators are released.
      mma_commit_pair_local(drained);
      mbar_wait(drained, 0);
    }
  } else {
    // ---- epilogue (both CTAs): warps 2 .. 1 + F_EPI_WARPS ----
    const int quad = warp & 3;
    const int group = (warp - 2) >> 2;  // this warp's columns: group * F_GROUP_COLS ..
    const int r = quad * 32 + lane;     // this thread's row of the CTA's 128 rows
    const uint32_t tq = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t ready0 = peer_addr(act_ready, 0);
    uint8_t* stage = act + F_STAGE_CHUNK * F_CHUNK_BYTES + (warp - 2) * 2 * EPI_BUF;  // after the head MMAs
    uint32_t full_ph = 0;
    auto wait_full = [&]() -> bool {
      const bool ok = mbar_wait(acc_full, full_ph & 1u);
      ++full_ph;
      fence_after();
      return ok;
    };
    const int act_code = args.act;
    int iter = 0;
    for (int t = pair; t < tiles && !failed; t += pairs, ++iter) {
      const int row0 = t * 2 * BM + static_cast<int>(rank) * BM;
      // Input layer: h = x W0^T + b0 (+ act when there are no blocks).
      if (!wait_full()) {
        failed = true;
        break;
      }
      for (int c = 0; c < F_GROUP_COLS / F_CW; ++c) {
        const int col0 = group * F_GROUP_COLS + c * F_CW;
        uint32_t raw[F_CW];
        float v[F_CW];
        CB_TMEM_LD16(tq + static_cast<uint32_t>(col0), raw);
        fused_layer_bias16(bias_s, args.bias[0], 0, col0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < F_CW; ++j) v[j] += __uint_as_float(raw[j]);
        if (args.blocks == 0 && act_code == kActRelu) {
          act_store16_relu(act, r, col0, v);
        } else {
          if (args.blocks == 0) activate_chunk<F_CW>(v, act_code);
          act_store16(act, r, col0, v);
        }
      }
      fused_phase_done(ready0);
      for (int l = 1; l <= hidden_layers && !failed; ++l) {
        if (!wait_full()) {
          failed = true;
          break;
        }
        const bool fc1 = (l & 1) == 1;
        const bool last = l == hidden_layers;
        const bool relu_out = act_code == kActRelu && (fc1 || last);  // ReLU in the bf16 pack
        for (int c = 0; c < F_GROUP_COLS / F_CW; ++c) {
          const int col0 = group * F_GROUP_COLS + c * F_CW;
          uint32_t raw[F_CW];
          float v[F_CW];
          CB_TMEM_LD16(tq + static_cast<uint32_t>(col0), raw);
          if (fc1) {
            // u = act(h W1^T + b1) over h in ACT; h + b2 into the accumulator for fc2.
            float b2[F_CW], h[F_CW];
            fused_layer_bias16(bias_s, args.bias[l + 1], l + 1, col0, b2);
            act_load16(act, r, col0, h);
            fused_layer_bias16(bias_s, args.bias[l], l, col0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < F_CW; ++j) v[j] += __uint_as_float(raw[j]);
            if (!relu_out) activate_chunk<F_CW>(v, act_code);
#pragma unroll
            for (int j = 0; j < F_CW; ++j) raw[j] = __float_as_uint(h[j] + b2[j]);
            CB_TMEM_ST16(tq + static_cast<uint32_t>(col0), raw);
          } else {
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < F_CW; ++j) v[j] = __uint_as_float(raw[j]);
            if (last && !relu_out) activate_chunk<F_CW>(v, act_code);
          }
          if (relu_out) act_store16_relu(act, r, col0, v);
          else act_store16(act, r, col0, v);
        }
        fused_phase_done(ready0);
      }
      if (failed) break;
      // Head: out = act(h) Wo^T + bo, fp32, through the ACT staging and TMA stores.
      if (!wait_full()) {
        failed = true;
        break;
      }
      const int chunks = args.n_mma / 16;
      const float* bo = args.bias[hidden_layers + 1];
      const int64_t row_g = static_cast<int64_t>(row0) + r;
      const bool sampling = args.actions != nullptr;
      const bool live = sampling && row_g < m_rows;
      // The row's game: its own entry, or entry rows[row] (one outside the arrays is a
      // row without legal actions).
      int64_t gi = row_g;
      bool known = live;
      if (live && args.rows) {
        gi = __ldg(args.rows + row_g);
        known = gi >= 0 && gi < args.n_games;
      }
      const uint64_t gid = known ? static_cast<uint64_t>(__ldg(args.game + gi)) : 0;
      const uint32_t dec = known ? static_cast<uint32_t>(__ldg(args.decision + gi)) : 0;
      SampleState st{-INFINITY, -1, 0.0f, -INFINITY, 0.0f};
      uint64_t lw[3] = {0ull, 0ull, 0ull};
      if (known) {
        const uint64_t* p = args.legal_bits + row_g * 3;
        lw[0] = __ldg(p);
        lw[1] = __ldg(p + 1);
        lw[2] = __ldg(p + 2);
      }
      int used = 0;
      for (int c = group; c < chunks; c += F_GROUPS, ++used) {
        const int col0 = c * 16;
        uint32_t raw[16];
        float v[16];
        CB_TMEM_LD16(tq + static_cast<uint32_t>(BN + col0), raw);  // the head is in half 1
        fused_bias16(bo, col0, args.n_out, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += __uint_as_float(raw[j]);
        if (live && col0 < F_ACTIONS) {
          const int wi = col0 >> 6;  // the word holding actions col0 .. col0 + 15
          const uint64_t w = wi == 0 ? lw[0] : (wi == 1 ? lw[1] : lw[2]);
          sample_chunk(args, gid, dec, col0, static_cast<uint32_t>(w >> (col0 & 63)) & 0xffffu, v,
                       st);
        }
        if (args.write_out) {
          uint8_t* buf = stage + (used & 1) * EPI_BUF;
          // The store that last read this buffer (two chunks back) is done with it.
          if (lane == 0) tma_store_wait_read<1>();
          __syncwarp();
          if (col0 < args.n_out) store_chunk<float>(buf, v, &maps.out, row0 + quad * 32, col0);
        }
      }
      if (sampling) {
        // The quadrant's column groups meet in tensor memory: group g > 0 posts its
        // state over the first columns of its own first chunk (read already), group 0
        // combines and writes the row's action and log p.  Shared memory stays free
        // for the next tile's x.
        const uint32_t post = tq + static_cast<uint32_t>(BN);
        uint32_t raw[16];
        if (group > 0) {
          raw[0] = __float_as_uint(st.best);
          raw[1] = static_cast<uint32_t>(st.best_a);
          raw[2] = __float_as_uint(st.best_x);
          raw[3] = __float_as_uint(st.mx);
          raw[4] = __float_as_uint(st.sum);
#pragma unroll
          for (int j = 5; j < 16; ++j) raw[j] = 0u;
          CB_TMEM_ST16(post + static_cast<uint32_t>(group * 16), raw);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sample_ready[quad]);
        } else {
          // Decided by the whole warp: the TMEM loads below are warp-collective.
          const bool ok = __all_sync(0xffffffffu, mbar_wait(&sample_ready[quad], static_cast<uint32_t>(iter & 1)));
          if (!ok) failed = true;
          if (ok) {
            fence_after();
            for (int g2 = 1; g2 < F_GROUPS; ++g2) {
              CB_TMEM_LD16(post + static_cast<uint32_t>(g2 * 16), raw);
              tmem_wait_ld();
              const float best = __uint_as_float(raw[0]), mx = __uint_as_float(raw[3]);
              const int a = static_cast<int>(raw[1]);
              if (a >= 0 && (best > st.best || (best == st.best && (st.best_a < 0 || a < st.best_a)))) {
                st.best = best;
                st.best_a = a;
                st.best_x = __uint_as_float(raw[2]);
              }
              if (mx != -INFINITY) {
                const float m2 = fmaxf(st.mx, mx);
                st.sum = st.sum * expf(st.mx - m2) + __uint_as_float(raw[4]) * expf(mx - m2);
                st.mx = m2;
              }
            }
            if (live) {
              args.actions[row_g] = st.best_a;
              args.logp[row_g] = st.best_a < 0 ? 0.0f : st.best_x - (st.mx + logf(st.sum));
            }
          }
        }
      }
      if (lane == 0 && args.write_out) tma_store_wait_read<0>();  // ACT may take the next tile's x
      __syncwarp();
      fence_before();
      if (lane == 0) {
        mbar_arrive_cluster(ready0);
        mbar_arrive(act_free);
      }
    }
    if (lane == 0) tma_store_wait_all();
  }
  if (failed) {
    any_failed = 1;
    if (args.error) atomicExch(args.error, 1);
  }
  fence_before();
  __syncthreads();
  if (any_failed) {
    // Let copies and MMAs still in flight land before the pair leaves (bounded).
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 100'000ull) {
    }
  }
  cluster_sync_all();  // no cross-CTA signal is outstanding past this point
  fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512));
  }
}

// CTA pairs of fused_mlp_kernel that fit on the device at once.
int fused_max_pairs(int dev) {
  static int cache[64] = {};
  if (!cache[dev]) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count() & ~1), 1, 1);
    cfg.blockDim = dim3(F_THREADS, 1, 1);
    cfg.dynamicSmemBytes = F_SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fused_mlp_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    cache[dev] = n;
  }
  return cache[dev];
}



// Both entry points: out may be null when sampling (actions != null).
int fused_launch(const void* x, int64_t ldx, int64_t m, int64_t k_in, int32_t blocks,
                 const void* const* weights, const float* const* biases, int64_t n_out,
                 int32_t act, float* out, int64_t ldo, const uint64_t* legal, const int64_t* game,
                 const int32_t* decision, const int64_t* rows, int64_t n_games, int64_t seed_base,
                 int32_t greedy, int64_t* actions, float* logp, const int32_t* m_dev,
                 int32_t* error, cudaStream_t stream) {
  if (m < 0 || k_in <= 0 || k_in > F_MAX_KIN || blocks < 0 || blocks > F_MAX_BLOCKS ||
      n_out <= 0 || n_out > BN || !weights || act < 0 || act > 2)
    return CUGO_B200_ERR_ARG;
  if (m == 0) return CUGO_B200_OK;
  if (m > INT32_MAX || !x || (!out && !actions) || ldx < k_in || (out && ldo < n_out))
    return CUGO_B200_ERR_ARG;
  if (actions && (!logp || !legal || !game || !decision || n_out < F_ACTIONS)) return CUGO_B200_ERR_ARG;
  if (rows && (!actions || n_games < 0)) return CUGO_B200_ERR_ARG;
  const int layers = 2 + 2 * blocks;
  for (int l = 0; l < layers; ++l)
    if (!weights[l]) return CUGO_B200_ERR_ARG;
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(x) || ldx % 8 || (out && (!al(out) || ldo % 4)) || k_in % 8) return CUGO_B200_ERR_ALIGN;
  for (int l = 0; l < layers; ++l)
    if (!al(weights[l])) return CUGO_B200_ERR_ALIGN;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {};
  if (dev < 0 || dev >= 64) return CUGO_B200_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(fused_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             F_SMEM_BYTES) != cudaSuccess)
      return CUGO_B200_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  // The head's MMA width: n_out rounded up to 16, at least 32 (a multiple of 16 per
  // CTA of the pair, in whole 8-row swizzle atoms).
  const int n_mma = n_out <= 32 ? 32 : static_cast<int>((n_out + 15) / 16 * 16);
  FusedMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!make_map(&maps.x, x, m, k_in, ldx, BM)) return CUGO_B200_ERR_LAUNCH;
  if (!make_map(&maps.w[0], weights[0], F_H, k_in, k_in, F_W_ROWS)) return CUGO_B200_ERR_LAUNCH;
  for (int l = 1; l < layers - 1; ++l)
    if (!make_map(&maps.w[l], weights[l], F_H, F_H, F_H, F_W_ROWS)) return CUGO_B200_ERR_LAUNCH;
  if (!make_map(&maps.w[layers - 1], weights[layers - 1], n_out, F_H, F_H,
                static_cast<uint32_t>(n_mma / 2)))
    return CUGO_B200_ERR_LAUNCH;
  if (out && !make_out_map(&maps.out, out, m, n_out, ldo, true)) return CUGO_B200_ERR_LAUNCH;
  FusedArgs args{};
  args.write_out = out ? 1 : 0;
  args.legal_bits = legal;
  args.game = game;
  args.decision = decision;
  args.rows = rows;
  args.n_games = n_games;
  args.seed_base = seed_base;
  args.greedy = greedy;
  args.actions = actions;
  args.logp = logp;
  args.m_dev = m_dev;
  for (int l = 0; l < layers; ++l) args.bias[l] = biases ? biases[l] : nullptr;
  args.blocks = blocks;
  args.m = static_cast<int>(m);
  args.k_in = static_cast<int>(k_in);
  args.n_out = static_cast<int>(n_out);
  args.n_mma = n_mma;
  args.act = act;
  args.error = error;
  const int64_t tiles = (m + 2 * BM - 1) / (2 * BM);
  const int64_t cap = fused_max_pairs(dev);
  const int64_t pairs = tiles < cap ? tiles : cap;
  fused_mlp_kernel<<<static_cast<unsigned>(2 * pairs), F_THREADS, F_SMEM_BYTES, stream>>>(maps, args);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

// Packs bool masks [m, 179] into three words per row (bit a of word a / 64).
__global__ void __launch_bounds__(256) pack_legal_kernel(const bool* __restrict__ legal, int64_t m,
                                                         uint64_t* __restrict__ bits) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= m) return;  // whole warps
  const uint8_t* src = reinterpret_cast<const uint8_t*>(legal) + row * F_ACTIONS;
  uint32_t w[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const int a = 32 * k + lane;
    w[k] = __ballot_sync(0xffffffffu, a < F_ACTIONS && src[a] != 0);
  }
  if (lane < 3)
    bits[row * 3 + lane] = (static_cast<uint64_t>(lane == 0 ? w[1] : lane == 1 ? w[3] : w[5]) << 32) |
                           (lane == 0 ? w[0] : lane == 1 ? w[2] : w[4]);
}

}  // namespace

extern "C" {

int cugo_b200_pack_legal(const bool* legal, int64_t m, uint64_t* bits, cudaStream_t stream) {
  if (m < 0 || (m > 0 && (!legal || !bits))) return CUGO_B200_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(bits) & 7u) return CUGO_B200_ERR_ALIGN;
  if (m == 0) return CUGO_B200_OK;
  pack_legal_kernel<<<static_cast<unsigned>((m * 32 + 255) / 256), 256, 0, stream>>>(legal, m, bits);
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

int cugo_b200_mlp_fused(const void* x, int64_t ldx, int64_t m, int64_t k_in, int32_t blocks,
                        const void* const* weights, const float* const* biases, int64_t n_out,
                        int32_t act, float* out, int64_t ldo, int32_t* error, cudaStream_t stream) {
  if (m > 0 && !out) return CUGO_B200_ERR_ARG;
  return fused_launch(x, ldx, m, k_in, blocks, weights, biases, n_out, act, out, ldo, nullptr,
                      nullptr, nullptr, nullptr, 0, 0, 0, nullptr, nullptr, nullptr, error, stream);
}

int cugo_b200_mlp_fused_sample(const void* x, int64_t ldx, int64_t m, int64_t k_in, int32_t blocks,
                               const void* const* weights, const float* const* biases,
                               int64_t n_out, int32_t act, const uint64_t* legal_bits,
                               const int64_t* game, const int32_t* decision,
                               const int64_t* rows, int64_t n_games, int64_t seed_base,
                               int32_t greedy, int64_t* actions, float* logp, float* out,
                               int64_t ldo, const int32_t* m_dev, int32_t* error,
                               cudaStream_t stream) {
  if (m > 0 && (!actions || !logp)) return CUGO_B200_ERR_ARG;
  if (m > 0 && (reinterpret_cast<uintptr_t>(legal_bits) & 7u)) return CUGO_B200_ERR_ALIGN;
  return fused_launch(x, ldx, m, k_in, blocks, weights, biases, n_out, act, out, ldo, legal_bits,
                      game, decision, rows, n_games, seed_base, greedy, actions, logp, m_dev,
                      error, stream);
}

}  // extern "C"

extern "C" {

int cugo_b200_wait_timeout_probe(int64_t limit_ns, int32_t* error, int64_t* waited_ns,
                                 cudaStream_t stream) {
  if (limit_ns <= 0 || limit_ns > 1'000'000'000 || !error) return CUGO_B200_ERR_ARG;
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(
      static_cast<uint64_t>(limit_ns), error, reinterpret_cast<unsigned long long*>(waited_ns));
  return cudaGetLastError() == cudaSuccess ? CUGO_B200_OK : CUGO_B200_ERR_LAUNCH;
}

}  // extern "C"

// ---- policy forward without allocation --------------------------------------------
//
// For callers that may not allocate device memory: an FFI host (a Go, Java or Rust
// serving process) that hands this library only its own fixed input and output
// buffers and keeps cudaMalloc off its request path because it synchronises the
// device, or a runtime that has reserved all device memory up front.  The two bf16
// activation buffers the layer chain needs live in this file-scope array instead
// of being allocated per call; every GPU that loads the library holds it (16 MiB)
// until the process exits.

namespace {

// Per buffer: rows x hidden <= kNoAllocRowsTimesHidden bf16 elements.
constexpr int64_t kNoAllocRowsTimesHidden = int64_t{4} << 20;
static __device__ __align__(256) __nv_bfloat16 g_noalloc_activations[2 * kNoAllocRowsTimesHidden];

// Device address of g_noalloc_activations, looked up once per device with that
// device current (the name is only a host-side stand-in in host code).  The
// entries are atomic: two host threads making their first call on one device at
// the same time both look the address up and store the same value.  The cache
// outlives a cudaDeviceReset (after which the module is loaded again and the
// array may move), so resetting a device after its first call here is not
// supported.
void* noalloc_scratch(int* rc) {
  constexpr int kMaxDevices = 64;
  static std::atomic<void*> addr[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = CUGO_B200_ERR_LAUNCH;
    return nullptr;
  }
  void* p = addr[dev].load(std::memory_order_acquire);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_noalloc_activations) != cudaSuccess || !p) {
      *rc = CUGO_B200_ERR_LAUNCH;
      return nullptr;
    }
    addr[dev].store(p, std::memory_order_release);
  }
  *rc = CUGO_B200_OK;
  return p;
}

}  // namespace

extern "C" {

int cugo_b200_policy_forward_noalloc(const void* x, int64_t ldx, int64_t m, int64_t inputs,
                                     int64_t hidden, int32_t blocks, int64_t outputs,
                                     const void* const* weights, const void* const* biases,
                                     int32_t act, float* out, int64_t ldo, int32_t* error,
                                     cudaStream_t stream) {
  if (m < 0 || inputs <= 0 || hidden <= 0 || blocks < 0 || outputs <= 0 || !weights ||
      (act != kActRelu && act != kActSilu))
    return CUGO_B200_ERR_ARG;
  // rows x hidden against the buffer without forming the product (which can wrap
  // for caller-supplied sizes).
  if (hidden > kNoAllocRowsTimesHidden || m > kNoAllocRowsTimesHidden / hidden)
    return CUGO_B200_ERR_CAPACITY;
  if (m == 0) return CUGO_B200_OK;
  const int layers = 2 + 2 * blocks;
  for (int l = 0; l < layers; ++l)
    if (!weights[l]) return CUGO_B200_ERR_ARG;
  int rc = CUGO_B200_OK;
  void* scratch = noalloc_scratch(&rc);
  if (rc != CUGO_B200_OK) return rc;
  // h and u: each call writes every element it later reads (rows past m are
  // outside the tensor maps and read as zero), so no state carries over between
  // calls and nothing needs clearing.
  auto* h = static_cast<__nv_bfloat16*>(scratch);
  __nv_bfloat16* u = h + kNoAllocRowsTimesHidden;
  const auto bias = [&](int l) { return biases ? biases[l] : nullptr; };
  rc = cugo_b200_gemm_bf16(x, ldx, weights[0], inputs, bias(0), nullptr, 0, h, hidden, 0, 0,
                           blocks == 0 ? act : 0, m, hidden, inputs, error, stream);
  for (int i = 0; i < blocks && rc == CUGO_B200_OK; ++i) {
    rc = cugo_b200_gemm_bf16(h, hidden, weights[1 + 2 * i], hidden, bias(1 + 2 * i), nullptr, 0, u,
                             hidden, 0, act, 0, m, hidden, hidden, error, stream);
    if (rc == CUGO_B200_OK)
      rc = cugo_b200_gemm_bf16(u, hidden, weights[2 + 2 * i], hidden, bias(2 + 2 * i), h, hidden, h,
                               hidden, 0, 0, i == blocks - 1 ? act : 0, m, hidden, hidden, error,
                               stream);
  }
  if (rc == CUGO_B200_OK)
    rc = cugo_b200_gemm_bf16(h, hidden, weights[layers - 1], hidden, bias(layers - 1), nullptr, 0,
                             out, ldo, 1, 0, 0, m, outputs, hidden, error, stream);
  return rc;
}

}  // extern "C"
