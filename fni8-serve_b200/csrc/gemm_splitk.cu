// Decode W8A8 GEMM for 1..256 tokens: every SM streams weights.
//
//   acc^T[n, m] = sum_k W[n, k] * q[m, k]     (tcgen05.mma kind::i8, M=128 weight rows, N=NT tokens)
//   out[m, n]   = dtype((float(acc) * a_scale[m]) * w_scale[n] (+ bias[n]) (+ residual[m, n]))
//
// At decode sizes the GEMM reads W[N, K] once and is bound by how many SMs keep weight
// loads in flight, not by the tensor cores. The tile kernel gives one CTA per 128x256
// output tile (24-96 CTAs for a Qwen3-8B projection), the stream-K kernel reduces its
// partial tiles with global atomics whose count grows with the token count. Here:
//
//  * grid = n_tiles x S CTAs, clustered S (<= 8) at a time. A cluster owns 128 weight
//    rows; CTA rank r of the cluster the r-th slice of the K range, so n_tiles x S ~ the
//    SM count for any N and K (S lowered until all clusters are resident at once).
//  * warp 0 streams (weight, activation) k-blocks of its slice through a TMA ring. Weights
//    never depend on the previous kernel: the first ring of weight tiles is issued before
//    the grid-dependency wait; the int8 activations (written by the quantiser just
//    before) are loaded after it.
//  * warp 1 issues the MMAs into one TMEM accumulator of NT columns.
//  * warps 2-5 (one TMEM lane quarter each) reduce the S partial accumulators: every CTA
//    writes the token columns the other ranks own to its slab of the zero-maintained GEMM
//    workspace, the cluster synchronises (release/acquire), and each owner gathers its
//    peers' granules with cp.async, zeroes them again, adds its own columns from TMEM and
//    stores (staged in shared memory for 16-byte stores when the rows allow). Integer sums
//    are associative, so the result is bit-exact for every split.
//  * the next kernel is released (programmatic dependent launch) once the partial sums
//    are published; its weight loads then queue behind this kernel's.
// Shared memory stays under half an SM up to NT = 128, so two CTAs (or this kernel and
// the next) share an SM. Every mbarrier wait is bounded (fni8_common.cuh).
#include <mutex>

#include "fni8_common.cuh"
#include "gemm_internal.h"

#include <stdio.h>
#include <stdlib.h>

namespace fni8b {
namespace splitk {

constexpr int kThreads = 192;
constexpr int BNW = 128;  // weight rows per tile (MMA M)
constexpr int BK = 128;   // K elements per stage
constexpr int kMaxStages = 8;
// Weight k-blocks per CTA pulled into L2 (beyond the ring) before the dependency wait: none
// by default. Measured on B200 in chains of decode GEMMs, early prefetch of the next
// kernel's weights queues ahead of the running kernel's last loads and partial-sum stores
// and delays it more than the prefetch saves.
constexpr int kL2Ahead = 0;
constexpr int kBarBytes = 256;
constexpr int kAsBytes = 1024;  // per-token activation scales of up to 256 tokens

static __device__ int g_status;

// Timeline tracing for measurement builds only (-DFNI8_TRACE): per CTA, the globaltimer
// of the kernel's phases, in launch order.
#ifdef FNI8_TRACE
static __device__ unsigned long long g_trace[65536 * 8];
static __device__ unsigned int g_trace_seq;
#define FNI8_TRACE_SLOT                                                  \
  __shared__ unsigned int s_trace_slot;                                  \
  if (threadIdx.x == 0) s_trace_slot = atomicAdd(&g_trace_seq, 1u) % 65536u;
#define FNI8_TRACE_AT(i) (g_trace[s_trace_slot * 8u + (i)] = globaltimer_ns())
#define FNI8_TRACE_VAL(i, v) (g_trace[s_trace_slot * 8u + (i)] = (v))
#else
#define FNI8_TRACE_SLOT
#define FNI8_TRACE_AT(i) ((void)0)
#define FNI8_TRACE_VAL(i, v) ((void)0)
#endif

enum : int { kCodeProducer = 0x501, kCodeMma = 0x502, kCodeEpilogue = 0x503, kCodeDrain = 0x504 };
enum : int { kOutF16 = 0, kOutBF16 = 1, kOutI32 = 2 };

struct Epi {
  const float* a_scale;  // [M]
  const float* w_scale;  // [N]
  const void* bias;      // [N] or null
  const void* residual;  // [M, N] or null
  void* out;             // [M, N]
  int mode;
  int vec;      // fp16/bf16 out, no residual, rows 16-byte aligned: stage the tile, store 16 B per thread
  int l2ahead;  // weight k-blocks beyond the ring pulled into L2 before the dependency wait
  // when the next kernel is released: 0 at entry, 1 once this CTA's last load is issued,
  // 2 once its partial sums are published (its accumulator is complete when unsplit)
  int trigger;
};

template <int NT>
struct Cfg {
  static constexpr int W_BYTES = BNW * BK;
  static constexpr int X_BYTES = NT * BK;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte alignment of the 128B swizzle");
};

// out[m0 + j, n] for the CNT accumulator values of weight row n, tokens m0 + j < mlim,
// straight to global memory (int32 output, residual add, or unaligned rows). s_as holds
// the per-token scales in shared memory. Every load (scales, residual values, the epilogue
// parameters) is issued before the first store and every value is computed before it: a
// load issued after a store that might alias it waits for that store, which would cost a
// memory round trip per column.
template <typename T, int CNT>
__device__ __forceinline__ void emit_batch(const Epi& epi, const uint32_t (&acc)[CNT], int m0, int mlim, int n, int N,
                                           float wsn, float bn, const float* s_as) {
  const int mode = epi.mode;
  const bool has_bias = epi.bias != nullptr;
  const T* res = static_cast<const T*>(epi.residual);
  if (mode == kOutI32) {
    int32_t* o = static_cast<int32_t*>(epi.out);
#pragma unroll
    for (int j = 0; j < CNT; ++j)
      if (m0 + j < mlim) o[static_cast<int64_t>(m0 + j) * N + n] = static_cast<int32_t>(acc[j]);
    return;
  }
  T* o = static_cast<T*>(epi.out);
  float sa[CNT], rs[CNT];
#pragma unroll
  for (int j = 0; j < CNT; ++j) sa[j] = s_as[m0 + j < mlim ? m0 + j : m0];
#pragma unroll
  for (int j = 0; j < CNT; ++j)
    rs[j] = (res != nullptr && m0 + j < mlim) ? to_f32<T>(res[static_cast<int64_t>(m0 + j) * N + n]) : 0.0f;
  T h[CNT];
#pragma unroll
  for (int j = 0; j < CNT; ++j) {
    float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(acc[j])), sa[j]), wsn);
    if (has_bias) v = __fadd_rn(v, bn);
    if (res != nullptr) v = __fadd_rn(v, rs[j]);
    h[j] = from_f32<T>(v);
  }
#pragma unroll
  for (int j = 0; j < CNT; ++j)
    if (m0 + j < mlim) o[static_cast<int64_t>(m0 + j) * N + n] = h[j];
}

// Same values into the shared-memory output tile stage[m - m_base][128] (row n of the
// weight tile is column trow), for the coalesced copy-out; loads before stores likewise.
template <typename T, int CNT>
__device__ __forceinline__ void stage_batch(const uint32_t (&acc)[CNT], int m0, int mlim, int m_base, T* stage,
                                            int trow, float wsn, float bn, bool has_bias, const float* s_as) {
  float sa[CNT];
#pragma unroll
  for (int j = 0; j < CNT; ++j) sa[j] = s_as[m0 + j < mlim ? m0 + j : m0];
  T h[CNT];
#pragma unroll
  for (int j = 0; j < CNT; ++j) {
    float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(acc[j])), sa[j]), wsn);
    if (has_bias) v = __fadd_rn(v, bn);
    h[j] = from_f32<T>(v);
  }
#pragma unroll
  for (int j = 0; j < CNT; ++j)
    if (m0 + j < mlim) stage[(m0 + j - m_base) * BNW + trow] = h[j];
}

// Split-K ownership. The token columns that carry real tokens (the first mcols, M rounded
// up to 4) are dealt out in shares of `share` columns (a multiple of 16, so every 16-column
// batch of an owner lies inside the accumulator's NT columns) to the S CTAs of
// the cluster: CTA o sums and stores columns [o*share, (o+1)*share). The other CTAs'
// partial sums of those columns reach it through their workspace slabs: CTA b writes
// [NT/4 column groups][128 rows] of 16-byte granules at ws + b * (NT/4) * 128, the weight
// row innermost, so a warp's 32 stores or loads cover 512 contiguous bytes.
__host__ __device__ __forceinline__ int split_share(int mcols, int S) { return ((mcols + S - 1) / S + 15) & ~15; }

// Owned columns [own0, own0 + len) of row trow: this CTA's accumulator (TMEM) plus the
// peers' slab granules, all copied into `land` ([S-1][len/4][128] granules) by one batch
// of asynchronous copies and zeroed in the workspace again (it stays zero between calls);
// then staged for the copy-out or stored. 16 columns per batch.
template <typename T>
__device__ __forceinline__ void finish_owned(const Epi& epi, uint32_t taddr, uint4* ws, int nt4, int block0,
                                             uint32_t rank, uint32_t S, int own0, int len, int M, int N, int n,
                                             int trow, float wsn, float bn, const float* s_as, T* stage, uint4* land) {
  const int g_own = len >> 2;
  if (S > 1) {
    int pi = 0;
    for (uint32_t p = 0; p < S; ++p) {
      if (p == rank) continue;
      uint4* slab = ws + static_cast<int64_t>(block0 + static_cast<int>(p)) * nt4 * BNW + (own0 >> 2) * BNW + trow;
      for (int g = 0; g < g_own; ++g) cp_async_16(land + (pi * g_own + g) * BNW + trow, slab + g * BNW);
      ++pi;
    }
    cp_async_commit();
    cp_async_wait_group<0>();
    for (uint32_t p = 0; p < S; ++p) {
      if (p == rank) continue;
      uint4* slab = ws + static_cast<int64_t>(block0 + static_cast<int>(p)) * nt4 * BNW + (own0 >> 2) * BNW + trow;
      for (int g = 0; g < g_own; ++g) __stcg(slab + g * BNW, make_uint4(0, 0, 0, 0));
    }
  }
  // every lane of the warp runs the tcgen05.ld below (.sync.aligned): rows past N only
  // skip their stores
  const bool nvalid = n < N;
  const bool has_bias = epi.bias != nullptr;
  const int mlim = (own0 + len) < M ? own0 + len : M;
#pragma unroll 1
  for (int c0 = 0; c0 < len; c0 += 16) {
    uint32_t acc[16];
    tmem_ld16(taddr + static_cast<uint32_t>(own0 + c0), acc);  // own0 + c0 + 16 <= NT (shares of 16)
    tmem_ld_wait();
    for (int pi = 0; pi + 1 < static_cast<int>(S); ++pi) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        if (c0 + 4 * g < len) {
          const uint4 v = land[(pi * g_own + (c0 >> 2) + g) * BNW + trow];
          acc[4 * g] += v.x;
          acc[4 * g + 1] += v.y;
          acc[4 * g + 2] += v.z;
          acc[4 * g + 3] += v.w;
        }
      }
    }
    if (!nvalid || own0 + c0 >= M) continue;
    if (stage != nullptr) stage_batch<T, 16>(acc, own0 + c0, mlim, own0, stage, trow, wsn, bn, has_bias, s_as);
    else emit_batch<T, 16>(epi, acc, own0 + c0, mlim, n, N, wsn, bn, s_as);
  }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 2)
    w8a8_splitk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, Epi epi,
                       int M, int N, int K, int STG, uint4* ws) {
  using C = Cfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STG * C::STAGE);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_as = reinterpret_cast<float*>(smem + STG * C::STAGE + kBarBytes);  // [NT] activation scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t S = cluster_nctarank();
  const int tile = static_cast<int>(blockIdx.x / S);
  const int kb = (K + BK - 1) / BK;
  const int kbeg = static_cast<int>(static_cast<int64_t>(rank) * kb / S);
  const int nk = static_cast<int>(static_cast<int64_t>(rank + 1) * kb / S) - kbeg;

  FNI8_TRACE_SLOT
  if (threadIdx.x == 0) {
    FNI8_TRACE_AT(0);
    FNI8_TRACE_VAL(7, (static_cast<unsigned long long>(N) << 40) | (static_cast<unsigned long long>(K) << 16) |
                          blockIdx.x);
    for (int s = 0; s < STG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the next kernel may start its prologue (its weight loads compete with ours for HBM); it
  // waits for our completion before it reads what we write
  if (epi.trigger == 0) pdl_launch_dependents();

  auto stage_at = [&](int s) { return smem + s * C::STAGE; };
  int okt = 0;  // epilogue warps: the accumulator is complete
  const int n_row = tile * BNW + (warp & 3) * 32 + lane;  // epilogue warps: weight row of this thread
  float wsn = 0.0f, bn = 0.0f;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const int pre = nk < STG ? nk : STG;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE);
        tma_load_2d(&tmW, &full[i], stage_at(i), (kbeg + i) * BK, tile * BNW);
      }
      const int l2_end = (nk - pre) < epi.l2ahead ? nk : pre + epi.l2ahead;
      for (int i = pre; i < l2_end; ++i) tma_prefetch_l2_2d(&tmW, (kbeg + i) * BK, tile * BNW);
      pdl_wait();  // the activations come from the previous kernel
      FNI8_TRACE_AT(1);
      for (int i = 0; i < pre; ++i) tma_load_2d(&tmX, &full[i], stage_at(i) + C::W_BYTES, (kbeg + i) * BK, 0);
      int stage = pre % STG;
      uint32_t ph = (pre == STG) ? 1u : 0u;
      uint32_t armed = 0;
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&empty[stage], ph ^ 1u, &g_status, kCodeProducer)) break;
        mbar_arrive_expect_tx(&full[stage], C::STAGE);
        tma_load_2d(&tmW, &full[stage], stage_at(stage), (kbeg + i) * BK, tile * BNW);
        tma_load_2d(&tmX, &full[stage], stage_at(stage) + C::W_BYTES, (kbeg + i) * BK, 0);
        armed = (armed & ~(1u << stage)) | (ph << stage);
        ++issued;
        if (++stage == STG) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (epi.trigger == 1) pdl_launch_dependents();
      // every load still in flight lands before the ring is reused for the partial sums
      const int pending = issued < STG ? issued : STG;
      for (int i = 0; i < pending; ++i) {
        const int s = (stage - 1 - i + 2 * STG) % STG;
        mbar_wait(&full[s], (armed >> s) & 1u, &g_status, kCodeDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_i8(BNW, NT);
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        if (!mbar_wait(&full[stage], ph, &g_status, kCodeMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (i == 0) FNI8_TRACE_AT(2);
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(stage_at(stage)));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(stage_at(stage) + C::W_BYTES));
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk)
          umma_i8(tmem_base, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                  (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == STG) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (ok) umma_commit(tfull);
      FNI8_TRACE_AT(3);
      umma_commit(drain);
      mbar_wait(drain, 0, &g_status, kCodeDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    // While the mainloop runs: the per-token scales into shared memory, this thread's
    // weight-row scale and bias into registers (they may come from the previous kernel).
    pdl_wait();
    if (epi.mode != kOutI32) {
      for (int m = threadIdx.x - 64; m < M; m += 128) s_as[m] = __ldg(epi.a_scale + m);
      if (n_row < N) {
        wsn = __ldg(epi.w_scale + n_row);
        if (epi.bias != nullptr)
          bn = epi.mode == kOutBF16 ? to_f32<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(epi.bias)[n_row])
                                    : to_f32<__half>(static_cast<const __half*>(epi.bias)[n_row]);
      }
    }
    named_bar_sync(1, 128);
    if (lane == 0) okt = mbar_wait(tfull, 0, &g_status, kCodeEpilogue) ? 1 : 0;
    okt = __shfl_sync(0xffffffffu, okt, 0);
    tc_fence_after();
    if (threadIdx.x == 64) FNI8_TRACE_AT(4);
    if (epi.trigger == 2 && S == 1 && threadIdx.x == 64) pdl_launch_dependents();
  }
  __syncwarp();

  const int q = warp & 3;  // TMEM lane quarter this warp may read (warps 2-5 -> 2,3,0,1)
  const int trow = q * 32 + lane;
  const int n = n_row;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
  const int mcols = (M + 3) & ~3;
  const int share = S > 1 ? split_share(mcols, static_cast<int>(S)) : mcols;
  const int own0 = static_cast<int>(rank) * share;
  const int len = own0 < mcols ? (mcols - own0 < share ? mcols - own0 : share) : 0;
  // the producer drained the ring (every load landed) and the MMAs are complete: the ring
  // is free for the output tile
  __syncthreads();
  if (S > 1) {
    // publish the partial sums of the columns other CTAs own
    if (warp >= 2 && okt) {
      uint4* slab = ws + static_cast<int64_t>(blockIdx.x) * (NT / 4) * BNW;
      constexpr int CH = NT < 32 ? NT : 32;
#pragma unroll 1
      for (int c0 = 0; c0 < mcols; c0 += CH) {
        uint32_t r[CH];
        if constexpr (CH == 16) tmem_ld16(taddr + c0, reinterpret_cast<uint32_t(&)[16]>(r));
        else tmem_ld32(taddr + c0, reinterpret_cast<uint32_t(&)[32]>(r));
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < CH; j += 4) {
          const int col = c0 + j;
          if (col < mcols && (col < own0 || col >= own0 + share))
            __stcg(slab + (col >> 2) * BNW + trow, make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]));
        }
      }
    }
    cluster_sync_all();  // release/acquire at cluster scope: the slabs are visible to the owners
    if (epi.trigger == 2 && threadIdx.x == 64) pdl_launch_dependents();
    if (threadIdx.x == 64) FNI8_TRACE_AT(5);
  }
  if (warp >= 2 && okt && len > 0) {
    const int block0 = static_cast<int>(blockIdx.x) - static_cast<int>(rank);
    // drained ring: [output tile share x 128 x 2 B][landing area for the peers' granules]
    uint4* land = reinterpret_cast<uint4*>(smem + ((share * BNW * 2 + 15) & ~15));
    if (epi.mode == kOutBF16)
      finish_owned<__nv_bfloat16>(epi, taddr, ws, NT / 4, block0, rank, S, own0, len, M, N, n, trow, wsn, bn, s_as,
                                  epi.vec ? reinterpret_cast<__nv_bfloat16*>(smem) : nullptr, land);
    else
      finish_owned<__half>(epi, taddr, ws, NT / 4, block0, rank, S, own0, len, M, N, n, trow, wsn, bn, s_as,
                           epi.vec ? reinterpret_cast<__half*>(smem) : nullptr, land);
  }
  if (warp >= 2 && epi.vec) {
    // coalesced copy-out of the staged rows: 16 bytes per thread, 512 bytes per warp
    named_bar_sync(1, 128);
    const int rows = (okt && own0 < M) ? ((own0 + len < M ? own0 + len : M) - own0) : 0;
    const int n0 = tile * BNW;
    const int chunks_per_row = (N - n0) >= BNW ? BNW / 8 : (N - n0) / 8;
    const int ct = threadIdx.x - 64;
    const uint4* src = reinterpret_cast<const uint4*>(smem);
    uint16_t* dst = static_cast<uint16_t*>(epi.out);
    for (int i = ct; i < rows * (BNW / 8); i += 128) {
      const int r = i >> 4, ch = i & 15;
      if (ch < chunks_per_row)
        *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(own0 + r) * N + n0 + ch * 8) = src[i];
    }
  }

  if (threadIdx.x == 64) FNI8_TRACE_AT(6);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace splitk
}  // namespace fni8b

namespace fni8h {

using namespace fni8b;

#ifdef FNI8_TRACE
extern "C" __attribute__((visibility("default"))) int fni8_trace_read_splitk(unsigned long long* dst, int n_records) {
  const size_t bytes = static_cast<size_t>(n_records) * 8 * sizeof(unsigned long long);
  if (cudaMemcpyFromSymbol(dst, splitk::g_trace, bytes) != cudaSuccess) return FNI8_ERR_CUDA;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, splitk::g_trace) != cudaSuccess) return FNI8_ERR_CUDA;
  if (cudaMemset(p, 0, sizeof(splitk::g_trace)) != cudaSuccess) return FNI8_ERR_CUDA;
  unsigned int z = 0;
  if (cudaMemcpyToSymbol(splitk::g_trace_seq, &z, sizeof(z)) != cudaSuccess) return FNI8_ERR_CUDA;
  return FNI8_OK;
}
#endif

int splitk_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, splitk::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read split-K watchdog");
  e = cudaMemcpyToSymbol(splitk::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear split-K watchdog");
  *code = v;
  return FNI8_OK;
}

struct SplitPlan {
  int nt, S, grid, stages, smem;
  size_t ws_bytes;  // partial-sum slabs of the K split (zero-maintained GEMM workspace)
};

template <int NT>
static cudaError_t configure_splitk(int dev) {
  static std::atomic<bool> configured[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (configured[dev]) return cudaSuccess;
  auto kern = splitk::w8a8_splitk_kernel<NT>;
  // plans stay within 225 KB; the margin leaves room for static shared memory
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) configured[dev] = true;
  return e;
}

// Empty kernel: the occupancy calculator's stand-in for the tcgen05 kernels. (Asked about
// the split-K kernel itself, the CUDA 12.9 runtime answers one CTA per SM at any
// shared-memory size, while two of its CTAs measurably run on one SM together.)
static __global__ void __launch_bounds__(1024, 1) occupancy_standin() {}

// How many S-CTA clusters of `threads`-thread CTAs with `smem` bytes of shared memory can
// be resident at once (clusters live inside one GPC, so this is below SMs x CTAs-per-SM /
// S). Registers are not modelled (the callers' kernels fit two CTAs per SM by registers).
// -1 when the runtime cannot tell (no device).
int max_active_clusters(int threads, int smem, int S) {
  static std::atomic<bool> configured[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return -1;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(occupancy_standin, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return -1;
    }
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = -1;
  if (cudaOccupancyMaxActiveClusters(&n, occupancy_standin, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return n;
}

static int max_clusters(int nt, int smem, int S) {
  (void)nt;  // the ring size (smem) carries the token count's effect
  struct Entry { int dev, smem, S, n; };
  static Entry cache[64];
  static int used = 0;
  static std::mutex mu;  // GEMMs may be planned from several host threads
  std::lock_guard<std::mutex> lock(mu);
  const int dev = current_device();
  for (int i = 0; i < used; ++i)
    if (cache[i].dev == dev && cache[i].smem == smem && cache[i].S == S) return cache[i].n;
  const int n = max_active_clusters(splitk::kThreads, smem, S);
  if (n >= 0 && used < 64) cache[used++] = Entry{dev, smem, S, n};
  return n;
}

// NT: tokens rounded up to a power of two >= 16. S: the cluster size that brings the grid
// (n_tiles x S) closest to the SM count without exceeding it (at least 1, at most 8 and
// the number of K blocks), lowered until every cluster of the grid can be resident at
// once (a second wave of clusters would double the kernel's time). Ring: as many stages as
// fit in ~half an SM's shared memory (two CTAs per SM, so the next kernel can become
// resident), at least 3 when the K range is split (2 otherwise), else the whole SM; the
// drained ring must also hold the staged output tile of the CTA's columns.
// FNI8_TUNE_SPLITK_S, FNI8_TUNE_SPLITK_TARGET_PCT and FNI8_TUNE_SPLITK_SMEM_KB override
// the plan in a measurement build.
static bool plan_ring(int nt, int S, SplitPlan* p) {
  const int stage = splitk::BNW * splitk::BK + nt * splitk::BK;
  constexpr int forced_kb = FNI8_TUNE_SPLITK_SMEM_KB;
  const int sh = S > 1 ? splitk::split_share(nt, S) : nt;
  const int out_tile = ((sh * splitk::BNW * 2 + 15) & ~15) + (S - 1) * sh * splitk::BNW * 4;
  const int fixed = 1024 + splitk::kBarBytes + splitk::kAsBytes;
  int stages = 0;
  if (forced_kb > 0) {
    stages = (forced_kb * 1024 - fixed) / stage;
  } else {
    stages = (113 * 1024 - fixed) / stage;
    if (stages > splitk::kMaxStages) stages = splitk::kMaxStages;
    if (stages < (S > 1 ? 3 : 2) || stages * stage < out_tile) stages = (225 * 1024 - fixed) / stage;
  }
  if (stages > splitk::kMaxStages) stages = splitk::kMaxStages;
  if (stages < 2 || stages * stage < out_tile || fixed + stages * stage > 227 * 1024) return false;
  p->stages = stages;
  p->smem = fixed + stages * stage;
  return true;
}

static bool plan_splitk(int64_t M, int64_t N, int64_t K, SplitPlan* p) {
  if (M < 1 || M > kSplitkMaxM) return false;
  int nt = 16;
  while (nt < M) nt <<= 1;
  p->nt = nt;
  const int n_tiles = (int)((N + splitk::BNW - 1) / splitk::BNW);
  const int kb = (int)((K + splitk::BK - 1) / splitk::BK);
  const int sms = num_sms(current_device());
  constexpr int forced_s = FNI8_TUNE_SPLITK_S;
  constexpr int target_pct = FNI8_TUNE_SPLITK_TARGET_PCT;
  int S = forced_s;
  if (S < 1 || S > 8) {
    const int target = sms * target_pct / 100;
    S = n_tiles >= target ? 1 : target / n_tiles;
    if (S < 1) S = 1;
    if (S > 8) S = 8;
  }
  if (S > kb) S = kb;
  if (!plan_ring(nt, S, p)) return false;
  while (forced_s < 1 && S > 1) {
    const int mc = max_clusters(nt, p->smem, S);
    if (mc < 0 || n_tiles <= mc) break;
    --S;
    if (!plan_ring(nt, S, p)) return false;
  }
  p->S = S;
  p->grid = n_tiles * S;
  p->ws_bytes = S > 1 ? static_cast<size_t>(p->grid) * nt * splitk::BNW * 4 : 0;
  if (FNI8_TUNE_PLAN_LOG)
    fprintf(stderr, "fni8 split-K plan M=%lld N=%lld K=%lld: NT=%d S=%d grid=%d stages=%d smem=%d resident clusters=%d\n",
            (long long)M, (long long)N, (long long)K, nt, S, p->grid, p->stages, p->smem, max_clusters(nt, p->smem, S));
  return true;
}

template <int NT>
static int launch_splitk(const CUtensorMap& tw, const CUtensorMap& tx, const splitk::Epi& epi, int M, int N, int K,
                         const SplitPlan& p, uint4* ws, cudaStream_t st) {
  auto kern = splitk::w8a8_splitk_kernel<NT>;
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(FNI8_ERR_CUDA, "no current CUDA device");
  const cudaError_t ce = configure_splitk<NT>(dev);
  if (ce != cudaSuccess) return cuda_status(ce, "configure split-K gemm");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(splitk::kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, epi, M, N, K, p.stages, ws);
  if (e != cudaSuccess) return cuda_status(e, "launch split-K gemm");
  return FNI8_OK;
}

bool splitk_split_one_wave(int64_t M, int64_t N, int64_t K) {
  SplitPlan p;
  if (N >= (1LL << 31) || K >= (1LL << 31) || !plan_splitk(M, N, K, &p) || p.S < 2) return false;
  const int mc = max_clusters(p.nt, p.smem, p.S);
  return mc >= 0 && p.grid / p.S <= mc;
}

bool splitk_supported(int64_t M, int64_t N, int64_t K) {
  SplitPlan p;
  return N < (1LL << 31) && K < (1LL << 31) && plan_splitk(M, N, K, &p);
}

size_t splitk_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  SplitPlan p;
  return plan_splitk(M, N, K, &p) ? p.ws_bytes : 0;
}

int splitk_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws,
                size_t ws_bytes, cudaStream_t st) {
  if (M <= 0 || N <= 0) return FNI8_OK;
  SplitPlan p;
  if (!plan_splitk(M, N, K, &p))
    return fail(FNI8_ERR_UNSUPPORTED, "split-K decode GEMM takes 1 <= M <= %lld (got %lld)", (long long)kSplitkMaxM,
                (long long)M);
  if (p.ws_bytes > 0 && (ws == nullptr || ws_bytes < p.ws_bytes))
    return fail(FNI8_ERR_WORKSPACE, "split-K GEMM needs %zu workspace bytes (got %zu)", p.ws_bytes, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return fail(FNI8_ERR_ALIGN, "workspace must be 16-byte aligned");
  CUtensorMap tw, tx;
  if (int s = encode_tmap_2d_i8(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, 128)) return s;
  if (int s = encode_tmap_2d_i8(&tx, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, (uint32_t)p.nt)) return s;
  const int vec = out_mode != splitk::kOutI32 && residual == nullptr && N % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  // L2 prefetch depth (FNI8_TUNE_SPLITK_L2AHEAD, none) and when the next kernel is released
  // (FNI8_TUNE_SPLITK_TRIGGER: 0 entry, 1 after the last load, 2 after the partial sums are
  // published: the default, fastest in measured decode chains)
  constexpr int l2ahead = FNI8_TUNE_SPLITK_L2AHEAD > splitk::kL2Ahead ? FNI8_TUNE_SPLITK_L2AHEAD : splitk::kL2Ahead;
  constexpr int trigger = FNI8_TUNE_SPLITK_TRIGGER;
  splitk::Epi epi{a_scale, w_scale, bias, residual, out, out_mode, vec, l2ahead < 0 ? 0 : l2ahead, trigger};
  uint4* w4 = static_cast<uint4*>(ws);
  switch (p.nt) {
    case 16: return launch_splitk<16>(tw, tx, epi, (int)M, (int)N, (int)K, p, w4, st);
    case 32: return launch_splitk<32>(tw, tx, epi, (int)M, (int)N, (int)K, p, w4, st);
    case 64: return launch_splitk<64>(tw, tx, epi, (int)M, (int)N, (int)K, p, w4, st);
    case 128: return launch_splitk<128>(tw, tx, epi, (int)M, (int)N, (int)K, p, w4, st);
    default: return launch_splitk<256>(tw, tx, epi, (int)M, (int)N, (int)K, p, w4, st);
  }
}

}  // namespace fni8h
