// Dense and grouped W8A8 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   out[m, n] = dtype((float(sum_k a[m,k] * w[n,k]) * a_scale[m]) * w_scale[n] (+ bias[n]) (+ res[m,n]))
//
// Design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0      TMA producer: 128 x 128-byte tiles of A (activations) and BN x 128-byte
//               tiles of W (weights), 128-byte swizzled, into a STAGES-deep smem ring.
//   warp 1      allocates TMEM (2 x BN columns = a double-buffered int32 accumulator)
//               and, from one thread, issues tcgen05.mma.kind::i8 (M=128, N=BN, K=32;
//               4 per 128-byte stage); tcgen05.commit frees smem stages and publishes
//               finished accumulators.
//   warps 2-9   epilogue: tcgen05.ld of one accumulator row per thread, fp32 dequant
//               (+bias, +residual), rounding to fp16/bf16 (or raw int32), global stores;
//               two warps per TMEM lane quarter, each taking half of the BN columns, so
//               the epilogue keeps up with short K loops (e.g. the MoE down projection,
//               K=768). The other accumulator buffer is being filled meanwhile.
// Tiles are visited in bands of kGroupM m-tiles so a wave of 148 CTAs reuses the same
// A rows and W columns out of the 126 MB L2.
//
// PAIR: two CTAs of a cluster run each tile of 256 rows as one tcgen05.mma.cta_group::2
// (M=256): each loads its 128 A rows and half of the BN weight rows, so a weight tile is
// read once per 256 rows and each SM's shared memory holds and feeds half of it. The even
// CTA of the pair arms the stage barriers (the odd CTA's loads complete on them) and
// issues the MMAs; the commits reach both CTAs' barriers; each CTA stores its own rows.
//
// GROUPED: the A rows are split into segments (one per expert, or per (source rank,
// expert) pair under expert parallelism); segment s multiplies rows
// [off[s], off[s]+cnt[s]) by expert exp[s] of a [E, N, K] weight stack (3-D TMA map).
// A tile may load rows past its segment's end (they belong to the next segment); the
// epilogue simply does not store them.
//
// Every mbarrier wait is bounded (fni8_common.cuh); on a timeout the roles leave their
// loops, drain in-flight TMA loads and MMAs (bounded), free TMEM and exit, and the host
// sees FNI8_ERR_DEVICE_TIMEOUT from fni8_device_status().
#include "fni8_common.cuh"
#include "gemm_internal.h"

#include <stdlib.h>
#include <string.h>

namespace fni8b {
namespace tile {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes == int8 elements per stage along K
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kMaxSeg = fni8h::kTileMaxSeg;
constexpr int kGroupM = 16;
// Weight k-blocks per CTA prefetched into L2 (beyond the ring) before the PDL wait: none by
// default (measured on B200: the early prefetch competes with the upstream kernel's own
// loads and gains nothing in decode or prefill chains).
constexpr int kL2AheadUnits = 0;

static __device__ int g_status;  // watchdog word of this file

enum : int { kCodeProducer = 0x101, kCodeMma = 0x102, kCodeEpilogue = 0x103, kCodeDrain = 0x104, kCodeScatter = 0x105 };
constexpr int kMaxPeers = 8;
enum : int { kOutF16 = 0, kOutBF16 = 1, kOutI32 = 2 };

struct Epi {
  const float* a_scale;  // [rows]
  const float* w_scale;  // [N] or [E, N]
  const void* bias;      // [N] (out dtype) or null
  const void* residual;  // [rows, N] (out dtype) or null
  void* out;             // [rows, N]
  int mode;              // kOutF16 / kOutBF16 / kOutI32
  int l2ahead;           // weight k-blocks pulled into L2 (beyond the ring) before the PDL wait
  int trigger;           // next kernel released at entry (0) or after this CTA's last load (1)
  // Peer outputs (16-bit out, n_peers > 0; buffers of this GPU or of its NVLink peers
  // mapped into this process), instead of out:
  //  * column all-gather (dense, row_tag null): element (m, n) goes to element
  //    (m, peer_col + n) of every peer_out[p] ([rows, peer_ld] each);
  //  * row scatter (grouped, row_tag set): row r goes to row (row_tag[r] & 0xFFFFFF) of
  //    peer_out[row_tag[r] >> 24] ([peer_rows, N] each).
  void* peer_out[kMaxPeers];
  int n_peers;
  int peer_col;
  int64_t peer_ld;
  const int32_t* row_tag;
  int64_t peer_rows;
  int band;  // m-tiles per band of the dense tile order (0: kGroupM)
  // ACTMUL kernels (gate_up with act_and_mul in the epilogue): the weight holds the gate
  // rows [0, act_i) and the up rows [act_i, 2 act_i); tile n covers gate rows
  // [128 n, 128 n + 128) in accumulator columns 0-127 and the matching up rows in columns
  // 128-255; out is [rows, act_i]. act: FNI8_ACT_SILU or FNI8_ACT_GELU_TANH.
  int act;
  int act_i;
};
struct Groups {
  const int32_t* expert;
  const int32_t* off;
  const int32_t* cnt;
  int S;
};

template <int BN, bool PAIR>
struct Cfg {
  static constexpr int BMT = PAIR ? 2 * BM : BM;  // rows of a tile
  static constexpr int BNL = PAIR ? BN / 2 : BN;  // weight rows this CTA loads per stage
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BNL * BK;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? (BN == 256 ? 6 : 8) : ((BN == 256) ? 4 : 6);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SEG_BYTES = (kMaxSeg + 1 + 3 * kMaxSeg) * 4;
  // per epilogue warp, one 32 x 32 16-bit output staging buffer for the TMA store
  static constexpr int STG_BUF = 32 * 32 * 2;
  static constexpr int STG_BYTES = kEpiWarps * STG_BUF;
  static constexpr int STG_OFF = (STAGES * STAGE + BAR_BYTES + SEG_BYTES + 1023) / 1024 * 1024;  // swizzle-aligned
  static constexpr int SMEM = 1024 + STG_OFF + STG_BYTES + 2 * BN * 4;  // + per-tile column scales, bias
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
};

struct TileCoord {
  int row0;        // first A row of the tile (TMA y)
  int rows_valid;  // rows of this tile that belong to it (<= 128)
  int n_blk;
  int expert;
};

// Tile t -> rows [row0, row0 + rows_valid) (rows_valid <= BMT) and weight block n_blk.
// Dense tiles are visited in bands of `band` m-tiles, m-tile fastest within a band.
template <bool GROUPED, int BMT>
__device__ __forceinline__ TileCoord decode_tile(int t, int M, int m_tiles, int n_tiles, const int32_t* prefix,
                                                 const int32_t* soff, const int32_t* scnt, const int32_t* sexp,
                                                 int S, int band) {
  TileCoord tc;
  if constexpr (GROUPED) {
    const int mt = t / n_tiles;
    tc.n_blk = t - mt * n_tiles;
    int lo = 0, hi = S - 1;  // largest s with prefix[s] <= mt
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= mt) lo = mid;
      else hi = mid - 1;
    }
    const int ml = mt - prefix[lo];
    tc.row0 = soff[lo] + ml * BMT;
    tc.rows_valid = min(BMT, scnt[lo] - ml * BMT);
    tc.expert = sexp[lo];
  } else {
    const int band_tiles = band * n_tiles;
    const int b = t / band_tiles;
    const int first_m = b * band;
    const int gm = min(band, m_tiles - first_m);
    const int local = t - b * band_tiles;
    const int m_blk = first_m + local % gm;
    tc.n_blk = local / gm;
    tc.row0 = m_blk * BMT;
    tc.rows_valid = min(BMT, M - tc.row0);
    tc.expert = 0;
  }
  return tc;
}

// Per-thread stores of one 32-column chunk of one output row (the path for residual adds,
// rows cut by a segment end and unaligned outputs). ws/bs: the chunk's column scales and
// bias (fp32, from shared memory).
template <typename T>
__device__ __forceinline__ void store_chunk(const Epi& epi, const uint32_t (&r)[32], int64_t row, T* out, int n0,
                                            int N, float a_s, const float* ws, const float* bs, bool vec_ok) {
  const T* res = epi.residual ? static_cast<const T*>(epi.residual) + row * static_cast<int64_t>(N) : nullptr;
  const bool has_bias = epi.bias != nullptr;
  if (vec_ok && n0 + 32 <= N) {
#pragma unroll
    for (int j8 = 0; j8 < 32; j8 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j8 + j])), a_s), ws[j8 + j]);
        if (has_bias) v[j] = __fadd_rn(v[j], bs[j8 + j]);
      }
      if (res != nullptr) {
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(res + n0 + j8));
        const T* bb = reinterpret_cast<const T*>(&b);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], to_f32<T>(bb[j]));
      }
      uint4 o;
      T* oo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oo[j] = from_f32<T>(v[j]);
      *reinterpret_cast<uint4*>(out + n0 + j8) = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      if (n < N) {
        float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), a_s), ws[j]);
        if (has_bias) v = __fadd_rn(v, bs[j]);
        if (res != nullptr) v = __fadd_rn(v, to_f32<T>(res[n]));
        out[n] = from_f32<T>(v);
      }
    }
  }
}

__device__ __forceinline__ void store_chunk_i32(const Epi& epi, const uint32_t (&r)[32], int64_t row, int n0, int N,
                                                bool vec_ok) {
  int32_t* out = static_cast<int32_t*>(epi.out) + row * static_cast<int64_t>(N);
  if (vec_ok && n0 + 32 <= N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<int4*>(out + n0 + j) = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < N) out[n0 + j] = static_cast<int32_t>(r[j]);
  }
}

// act_and_mul of 32 output columns of one row from the gate accumulators rg and the up
// accumulators ru: each value is dequantised and rounded to T exactly as the plain
// epilogue stores it, then act(gate) * up is formed as the act_and_mul kernels form it
// (act_mul_one), so the fused result equals GEMM -> act_and_mul bit for bit. Packed as
// four 16-byte chunks of 8 outputs.
template <typename T, int ACT>
__device__ __forceinline__ void act_chunk(const uint32_t (&rg)[32], const uint32_t (&ru)[32], float a_s,
                                          const float* sg, const float* su, uint4 (&o)[4]) {
#pragma unroll
  for (int j8 = 0; j8 < 4; ++j8) {
    T* oo = reinterpret_cast<T*>(&o[j8]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j8 * 8 + j;
      const float g = round_trip<T>(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(rg[c])), a_s), sg[c]));
      const float u = round_trip<T>(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(ru[c])), a_s), su[c]));
      oo[j] = act_mul_one<T, ACT>(g, u);
    }
  }
}

// The plain epilogue's 32 outputs of one row: (float(acc) * a_s) * ws (+ bias) rounded once
// to fp16 (mode kOutF16) or bf16, packed as four 16-byte chunks.
__device__ __forceinline__ void dequant_chunk(int mode, const uint32_t (&r)[32], float a_s, const float* ws,
                                              const float* bs, bool has_bias, uint4 (&o)[4]) {
#pragma unroll
  for (int j8 = 0; j8 < 4; ++j8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j8 * 8 + j;
      v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[c])), a_s), ws[c]);
      if (has_bias) v[j] = __fadd_rn(v[j], bs[c]);
    }
    if (mode == kOutF16) {
      __half* oo = reinterpret_cast<__half*>(&o[j8]);
#pragma unroll
      for (int j = 0; j < 8; ++j) oo[j] = __float2half_rn(v[j]);
    } else {
      __nv_bfloat16* oo = reinterpret_cast<__nv_bfloat16*>(&o[j8]);
#pragma unroll
      for (int j = 0; j < 8; ++j) oo[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// One warp's 32 x 32 chunk of 16-bit outputs (lane = row of the slab, o = its four
// 16-byte pieces) to rows [row_base, row_base + 32), columns [n0, n0 + 32) of the output
// through one TMA store: staged in the warp's 2 KB buffer with the 64-byte swizzle of the
// store map (16-byte piece index ^= (row >> 1) & 3), reused only after the previous store
// from it has read it. (Measured on B200: copying the staged chunk out with coalesced
// 16-byte stores instead was slower.)
__device__ __forceinline__ void store_slab(uint8_t* buf, const uint4 (&o)[4], int lane, const CUtensorMap* tmOut,
                                           int n0, int row_base) {
  if (lane == 0) bulk_wait_group_read<0>();
  __syncwarp();
#pragma unroll
  for (int j8 = 0; j8 < 4; ++j8)
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((j8 ^ ((lane >> 1) & 3)) << 4)) = o[j8];
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmOut, buf, n0, row_base);
    bulk_commit_group();
  }
}

// Peer outputs leave 4 rows x 128 contiguous bytes per store instruction (measured on
// B200: twice the NVLink rate of 64-byte row pieces). Two consecutive 32-column chunks of
// the slab (o0, o1: this lane's row) pass through the warp's 2 KB buffer sixteen rows at a
// time (128 bytes per row, 16-byte pieces swizzled by row); put(r, g, v, tag) then stores
// piece g of slab row r (r < nrows) with lane r's tag.
template <typename Put>
__device__ __forceinline__ void stage_rows_128(uint8_t* buf, const uint4 (&o0)[4], const uint4 (&o1)[4], int lane,
                                               uint32_t tag, int nrows, Put&& put) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // slab rows [16h, 16h + 16)
    __syncwarp();  // every lane has read the previous rows out of the buffer
    if ((lane >> 4) == h) {
      const int rr = lane & 15;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        *reinterpret_cast<uint4*>(buf + rr * 128 + ((j ^ (rr & 7)) << 4)) = o0[j];
        *reinterpret_cast<uint4*>(buf + rr * 128 + (((j + 4) ^ (rr & 7)) << 4)) = o1[j];
      }
    }
    __syncwarp();
    const int g = lane & 7;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int rr = 4 * u + (lane >> 3);
      const int r = 16 * h + rr;
      const uint32_t tg = __shfl_sync(0xffffffffu, tag, r);
      if (r < nrows) put(r, g, *reinterpret_cast<const uint4*>(buf + rr * 128 + ((g ^ (rr & 7)) << 4)), tg);
    }
  }
}

// Column all-gather: columns [n0, n0 + 64) of rows [row_base, row_base + nrows) to columns
// [peer_col + n0, peer_col + n0 + 64) of every peer_out buffer (plain stores: the
// destinations may be other GPUs' memory).
__device__ __forceinline__ void store_cols_128(uint8_t* buf, const uint4 (&o0)[4], const uint4 (&o1)[4], int lane,
                                               const Epi& epi, int n0, int row_base, int nrows) {
  stage_rows_128(buf, o0, o1, lane, 0u, nrows, [&](int r, int g, const uint4& v, uint32_t) {
    const int64_t off = (static_cast<int64_t>(row_base + r) * epi.peer_ld + epi.peer_col + n0 + 8 * g) * 2;
    for (int p = 0; p < epi.n_peers; ++p) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(epi.peer_out[p]) + off) = v;
  });
}

// Row scatter: columns [n0, n0 + 64) of slab row r (tag: lane r's `tag`) to row
// (tag & 0xFFFFFF) of peer_out[tag >> 24]. A tag outside the buffers is skipped and
// recorded in the status word.
__device__ __forceinline__ void store_rows_128(uint8_t* buf, const uint4 (&o0)[4], const uint4 (&o1)[4], int lane,
                                               const Epi& epi, int n0, int N, uint32_t tag, int nrows, int* status) {
  stage_rows_128(buf, o0, o1, lane, tag, nrows, [&](int, int g, const uint4& v, uint32_t tg) {
    const int src = static_cast<int>(tg >> 24);
    const int64_t slot = static_cast<int64_t>(tg & 0xFFFFFFu);
    if (src < epi.n_peers && slot < epi.peer_rows)
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(epi.peer_out[src]) + (slot * N + n0 + 8 * g) * 2) = v;
    else if (g == 0)
      atomicExch(status, kCodeScatter);
  });
}

__device__ __forceinline__ void act_chunk_any(int mode, int act, const uint32_t (&rg)[32], const uint32_t (&ru)[32],
                                              float a_s, const float* sg, const float* su, uint4 (&o)[4]) {
  if (mode == kOutF16) {
    if (act == FNI8_ACT_SILU) act_chunk<__half, FNI8_ACT_SILU>(rg, ru, a_s, sg, su, o);
    else act_chunk<__half, FNI8_ACT_GELU_TANH>(rg, ru, a_s, sg, su, o);
  } else {
    if (act == FNI8_ACT_SILU) act_chunk<__nv_bfloat16, FNI8_ACT_SILU>(rg, ru, a_s, sg, su, o);
    else act_chunk<__nv_bfloat16, FNI8_ACT_GELU_TANH>(rg, ru, a_s, sg, su, o);
  }
}

template <int BN, bool GROUPED, bool PAIR, bool ACTMUL = false>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_tile_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut, Epi epi, Groups grp, int M, int N, int K, int vec_ok,
                     int tma_store) {
  static_assert(!ACTMUL || BN == 256, "act_and_mul tiles pair 128 gate with 128 up columns");
  using C = Cfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* full = bars;
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int32_t* prefix = reinterpret_cast<int32_t*>(smem + C::STAGES * C::STAGE + C::BAR_BYTES);
  int32_t* soff = prefix + kMaxSeg + 1;
  int32_t* scnt = soff + kMaxSeg;
  int32_t* sexp = scnt + kMaxSeg;
  uint8_t* stg = smem + C::STG_OFF;  // 1024-aligned: the 64B-swizzle pattern follows address bits

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pair role: half = 0 for the even CTA (arms the stage barriers, issues the MMAs)
  const uint32_t half = PAIR ? (cluster_ctarank() & 1u) : 0u;
  const uint32_t lead = PAIR ? (cluster_ctarank() & ~1u) : 0u;  // cluster rank of the even CTA
  const uint16_t pair_mask = static_cast<uint16_t>(3u << lead);
  const int t0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);  // one arrive per epilogue warp (of both CTAs)
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);  // both CTAs, same warp, same address
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
    tc_fence_before();
  }

  // Everything above touched only on-chip state; from here on we read upstream results.
  // In the dense case the TMA producer defers its wait: it first starts the weight loads
  // of its first ring of stages, which do not depend on the upstream kernel.
  // the next kernel may start its prologue; it waits for our completion
  if (epi.trigger == 0) pdl_launch_dependents();
  if (GROUPED || !(warp == 0 && lane == 0)) pdl_wait();

  const int n_tiles = (N + BN - 1) / BN;
  const int m_tiles = (M + C::BMT - 1) / C::BMT;
  const int band = epi.band > 0 ? epi.band : kGroupM;
  const int kb = (K + BK - 1) / BK;
  int S = 0;
  if constexpr (GROUPED) {
    S = grp.S;
    for (int i = threadIdx.x; i < S; i += kThreads) {
      soff[i] = grp.off[i];
      scnt[i] = max(grp.cnt[i], 0);
      sexp[i] = grp.expert[i];
    }
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      if (lane == 0) prefix[0] = 0;
      for (int base = 0; base < S; base += 32) {
        const int i = base + lane;
        int v = (i < S) ? (scnt[i] + C::BMT - 1) / C::BMT : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        if (i < S) prefix[i + 1] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
  }
  // a pair's CTAs signal each other's barriers from here on: both are initialised first
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = GROUPED ? prefix[S] * n_tiles : m_tiles * n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t armed = 0;  // parity each stage was last armed with (bit per stage)
      int issued = 0;
      bool ok = true;
      int t = t0, k = 0;
      TileCoord tc{};
      if (t < total) tc = decode_tile<GROUPED, C::BMT>(t, M, m_tiles, n_tiles, prefix, soff, scnt, sexp, S, band);
      // this CTA's A rows and weight rows of a tile; stage loads complete on the even CTA's
      // barrier under PAIR, which is armed with the bytes of both CTAs
      const int a_off = static_cast<int>(half) * BM;
      const int b_off = static_cast<int>(half) * C::BNL;
      constexpr uint32_t kStageTx = PAIR ? 2 * C::STAGE : C::STAGE;
      auto load_a = [&](int s, int kx, int row) {
        if constexpr (PAIR) tma_load_2d_pair(&tmA, mapa_shared(smem_u32(&full[s]), lead), smem + s * C::STAGE, kx, row + a_off);
        else tma_load_2d(&tmA, &full[s], smem + s * C::STAGE, kx, row);
      };
      auto load_b = [&](int s, int kx, int nb, int ex) {
        uint8_t* dst = smem + s * C::STAGE + C::A_BYTES;
        if constexpr (ACTMUL) {
          // gate rows [128 nb, +128) then up rows [act_i + 128 nb, +128): two 128-row boxes
          // that land where one 256-row box would (a pair's even CTA loads the gate half,
          // the odd CTA the up half)
          const int g_row = nb * 128, u_row = epi.act_i + nb * 128;
          if constexpr (PAIR) {
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), lead);
            const int r = half == 0 ? g_row : u_row;
            if constexpr (GROUPED) tma_load_3d_pair(&tmB, bar, dst, kx, r, ex);
            else tma_load_2d_pair(&tmB, bar, dst, kx, r);
          } else {
            if constexpr (GROUPED) {
              tma_load_3d(&tmB, &full[s], dst, kx, g_row, ex);
              tma_load_3d(&tmB, &full[s], dst + 128 * BK, kx, u_row, ex);
            } else {
              tma_load_2d(&tmB, &full[s], dst, kx, g_row);
              tma_load_2d(&tmB, &full[s], dst + 128 * BK, kx, u_row);
            }
          }
        } else if constexpr (PAIR) {
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), lead);
          if constexpr (GROUPED) tma_load_3d_pair(&tmB, bar, dst, kx, nb * BN + b_off, ex);
          else tma_load_2d_pair(&tmB, bar, dst, kx, nb * BN + b_off);
        } else {
          if constexpr (GROUPED) tma_load_3d(&tmB, &full[s], dst, kx, nb * BN, ex);
          else tma_load_2d(&tmB, &full[s], dst, kx, nb * BN);
        }
      };
      auto advance = [&]() {
        if (++k == kb) {
          k = 0;
          t += tstep;
          if (t < total) tc = decode_tile<GROUPED, C::BMT>(t, M, m_tiles, n_tiles, prefix, soff, scnt, sexp, S, band);
        }
      };
      if constexpr (!GROUPED) {
        int pre_row[C::STAGES], pre_k[C::STAGES];
        int pre = 0;
        for (; pre < C::STAGES && t < total; ++pre, advance()) {  // first use of each stage
          if (half == 0) mbar_arrive_expect_tx(&full[pre], kStageTx);
          load_b(pre, k * BK, tc.n_blk, 0);
          pre_row[pre] = tc.row0;
          pre_k[pre] = k;
        }
        {  // weight tiles of the next units into L2 (epi.l2ahead of them, none by default)
          int tt = t, kk = k, nb = tc.n_blk;
          for (int i = 0; i < epi.l2ahead && tt < total; ++i) {
            tma_prefetch_l2_2d(&tmB, kk * BK, nb * BN + b_off);
            if (++kk == kb) {
              kk = 0;
              tt += tstep;
              if (tt < total) nb = decode_tile<GROUPED, C::BMT>(tt, M, m_tiles, n_tiles, prefix, soff, scnt, sexp, S, band).n_blk;
            }
          }
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i) load_a(i, pre_k[i] * BK, pre_row[i]);
        issued = pre;
        stage = pre % C::STAGES;
        ph = (pre == C::STAGES) ? 1u : 0u;
      }
      for (; t < total && ok; advance()) {
        if (!mbar_wait(&empty[stage], ph ^ 1u, &g_status, kCodeProducer)) {
          ok = false;
          break;
        }
        if (half == 0) mbar_arrive_expect_tx(&full[stage], kStageTx);
        load_a(stage, k * BK, tc.row0);
        load_b(stage, k * BK, tc.n_blk, tc.expert);
        armed = (armed & ~(1u << stage)) | (ph << stage);
        ++issued;
        if (++stage == C::STAGES) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (epi.trigger == 1) pdl_launch_dependents();
      // Drain: the loads of the last min(issued, STAGES) stages must have landed before
      // the CTA may exit (normally they have: the MMA consumed them). The odd CTA of a pair
      // sees its loads land through the release of the stage (the MMA consumed them).
      uint64_t* done = half == 0 ? full : empty;
      const int pending = issued < C::STAGES ? issued : C::STAGES;
      for (int i = 0; i < pending; ++i) {
        const int s = (stage - 1 - i + 2 * C::STAGES) % C::STAGES;
        mbar_wait(&done[s], (armed >> s) & 1u, &g_status, kCodeDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && half == 0) {
      constexpr uint32_t kIdesc = idesc_i8(C::BMT, BN);
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int t = t0; t < total && ok; t += tstep) {
        if (!mbar_wait(&tempty[acc], aph ^ 1u, &g_status, kCodeMma)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int k = 0; k < kb; ++k) {
          if (!mbar_wait(&full[stage], ph, &g_status, kCodeMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + stage * C::STAGE;
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sa));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sa + C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            // advance the start address by kk * 32 bytes inside the 128-byte swizzle atom
            if constexpr (PAIR)
              umma_i8_pair(d, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                           (k | kk) != 0 ? 1u : 0u);
            else
              umma_i8(d, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                      (k | kk) != 0 ? 1u : 0u);
          }
          if constexpr (PAIR) umma_commit_pair_to(&empty[stage], pair_mask);
          else umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) umma_commit_pair_to(&tfull[acc], pair_mask);
        else umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      // All MMAs issued by this thread must retire before TMEM is freed.
      if constexpr (PAIR) umma_commit_pair(drain);
      else umma_commit(drain);
      mbar_wait(drain, 0, &g_status, kCodeDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // 8 warps; warp w reads TMEM lanes [32q, 32q+32), q = w % 4 (rows of the tile, one
    // per thread), and the columns [h*BN/2, (h+1)*BN/2) of its half h = (w - 2) / 4.
    // Per tile the column scales (and bias) are staged in shared memory; their loads are
    // issued before the accumulator wait so they overlap the MMA. 16-bit outputs leave
    // through a 64B-swizzled 32 x 32 staging buffer per warp and TMA stores.
    const int q = warp & 3;
    const int ew = warp - 2;                     // 0..7
    const int c_beg = (ew >> 2) * (BN / 2);      // this warp's columns of the tile
    const int row_local = q * 32 + lane;
    const int et = threadIdx.x - 64;  // 0..255 across the epilogue warps
    float* s_ws = reinterpret_cast<float*>(stg + C::STG_BYTES);
    float* s_bias = s_ws + BN;
    int acc = 0;
    uint32_t aph = 0;
    if (tma_store && lane == 0) tma_prefetch_desc(&tmOut);
    for (int t = t0; t < total; t += tstep) {
      const TileCoord tc = decode_tile<GROUPED, C::BMT>(t, M, m_tiles, n_tiles, prefix, soff, scnt, sexp, S, band);
      // this CTA's rows of the tile
      const int row0 = tc.row0 + static_cast<int>(half) * BM;
      const int rows_here = tc.rows_valid - static_cast<int>(half) * BM;
      const bool valid = row_local < rows_here;
      const int64_t row = static_cast<int64_t>(row0) + row_local;
      // this thread's output row (per-thread store path)
      uint8_t* orow = nullptr;
      if (valid && epi.mode != kOutI32 && epi.n_peers == 0)
        orow = static_cast<uint8_t*>(epi.out) + row * static_cast<int64_t>(ACTMUL ? epi.act_i : N) * 2;
      const int nb0 = tc.n_blk * BN;
      const float* wsc = epi.w_scale + static_cast<int64_t>(tc.expert) * N;
      static_assert(BN <= kEpiThreads, "one column scale per epilogue thread");
      float wreg = 0.0f, breg = 0.0f;
      float a_s = 0.0f;
      if (epi.mode != kOutI32) {
        // ACTMUL: staged scales 0-127 are the gate rows', 128-255 the matching up rows'
        const int col = !ACTMUL ? nb0 + et
                                : (et < 128 ? tc.n_blk * 128 + et : epi.act_i + tc.n_blk * 128 + (et - 128));
        if (et < BN && col < N) {
          wreg = __ldg(wsc + col);
          if (epi.bias != nullptr)
            breg = epi.mode == kOutF16 ? __half2float(static_cast<const __half*>(epi.bias)[col])
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(epi.bias)[col]);
        }
        if (valid) a_s = __ldg(epi.a_scale + row);
      }
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[acc], aph, &g_status, kCodeEpilogue) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // also: every reader of the previous tile's scales is done
      if (!named_bar_and(2, kEpiThreads, ok)) break;
      tc_fence_after();
      if (epi.mode != kOutI32) {
        if (et < BN) {
          s_ws[et] = wreg;
          s_bias[et] = breg;
        }
        named_bar_sync(2, kEpiThreads);
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      // TMA store of whole 32-row slabs; a slab cut by a segment end (grouped) or any
      // residual add takes the per-thread path. Column all-gather: every slab with rows.
      const bool slab_tma = tma_store && epi.residual == nullptr && (!GROUPED || rows_here - q * 32 >= 32) &&
                            q * 32 < rows_here;
      const bool slab_peer = !GROUPED && !ACTMUL && epi.n_peers > 0 && q * 32 < rows_here;
      const bool slab_rows = GROUPED && !ACTMUL && epi.row_tag != nullptr && q * 32 < rows_here;
      const uint32_t my_tag = (slab_rows && valid) ? static_cast<uint32_t>(__ldg(epi.row_tag + row)) : 0xFFFFFFFFu;
      if constexpr (ACTMUL) {
        // this warp's 64 of the tile's 128 product columns: gate accumulators at c, up at
        // 128 + c; outputs at column 128 n + c of the [rows, act_i] product
        // Software-pipelined: a chunk's outputs are formed in registers, then the next
        // chunk's TMEM loads are issued, so they overlap the staging-buffer wait and store.
        const int p_beg = (ew >> 2) * 64;
        uint32_t rg[32], ru[32];
        tmem_ld32(tbase + static_cast<uint32_t>(p_beg), rg);
        tmem_ld32(tbase + static_cast<uint32_t>(128 + p_beg), ru);
        tmem_ld_wait();
        tmem_regs_ready(rg);
        tmem_regs_ready(ru);
#pragma unroll 1
        for (int c = p_beg; c < p_beg + 64; c += 32) {
          const bool more = c + 32 < p_beg + 64;
          const int n0 = tc.n_blk * 128 + c;
          uint4 o[4];
          act_chunk_any(epi.mode, epi.act, rg, ru, a_s, s_ws + c, s_ws + 128 + c, o);
          if (more) {
            tmem_ld32(tbase + static_cast<uint32_t>(c + 32), rg);
            tmem_ld32(tbase + static_cast<uint32_t>(128 + c + 32), ru);
          }
          if (slab_tma) {
            store_slab(stg + ew * C::STG_BUF, o, lane, &tmOut, n0, row0 + q * 32);
          } else if (valid) {  // rows 16-byte aligned (checked on the host)
#pragma unroll
            for (int j8 = 0; j8 < 4; ++j8) *reinterpret_cast<uint4*>(orow + (n0 + 8 * j8) * 2) = o[j8];
          }
          if (more) {
            tmem_ld_wait();
            tmem_regs_ready(rg);
            tmem_regs_ready(ru);
          }
        }
      } else {
        const int c_end = c_beg + BN / 2;
        if (slab_rows || slab_peer) {
          // peer outputs: two chunks (64 columns) per round, each row leaving as 128 bytes
#pragma unroll 1
          for (int c = c_beg; c < c_end && nb0 + c < N; c += 64) {
            uint32_t r0[32], r1[32];
            tmem_ld32(tbase + static_cast<uint32_t>(c), r0);
            tmem_ld32(tbase + static_cast<uint32_t>(c + 32), r1);
            tmem_ld_wait();
            tmem_regs_ready(r0);
            tmem_regs_ready(r1);
            uint4 o0[4], o1[4];
            dequant_chunk(epi.mode, r0, a_s, s_ws + c, s_bias + c, epi.bias != nullptr, o0);
            dequant_chunk(epi.mode, r1, a_s, s_ws + c + 32, s_bias + c + 32, epi.bias != nullptr, o1);
            if (slab_rows)
              store_rows_128(stg + ew * C::STG_BUF, o0, o1, lane, epi, nb0 + c, N, my_tag,
                             min(32, rows_here - q * 32), &g_status);
            else
              store_cols_128(stg + ew * C::STG_BUF, o0, o1, lane, epi, nb0 + c, row0 + q * 32,
                             min(32, rows_here - q * 32));
          }
        } else {
          // Software-pipelined like the ACTMUL loop: dequantise a chunk into registers, issue
          // the next chunk's TMEM load, then wait for the staging buffer and store.
          uint32_t r[32];
          tmem_ld32(tbase + static_cast<uint32_t>(c_beg), r);
          tmem_ld_wait();
          tmem_regs_ready(r);
#pragma unroll 1
          for (int c = c_beg; c < c_end; c += 32) {
            const int n0 = nb0 + c;
            const bool more = c + 32 < c_end;
            if (slab_tma && n0 < N) {
              uint4 o[4];
              dequant_chunk(epi.mode, r, a_s, s_ws + c, s_bias + c, epi.bias != nullptr, o);
              if (more) tmem_ld32(tbase + static_cast<uint32_t>(c + 32), r);
              store_slab(stg + ew * C::STG_BUF, o, lane, &tmOut, n0, row0 + q * 32);
            } else {
              if (n0 < N && valid) {
                if (epi.mode == kOutI32) store_chunk_i32(epi, r, row, n0, N, vec_ok != 0);
                else if (epi.mode == kOutF16)
                  store_chunk<__half>(epi, r, row, reinterpret_cast<__half*>(orow), n0, N, a_s, s_ws + c, s_bias + c,
                                      vec_ok != 0);
                else
                  store_chunk<__nv_bfloat16>(epi, r, row, reinterpret_cast<__nv_bfloat16*>(orow), n0, N, a_s,
                                             s_ws + c, s_bias + c, vec_ok != 0);
              }
              if (more) tmem_ld32(tbase + static_cast<uint32_t>(c + 32), r);
            }
            if (more) {
              tmem_ld_wait();
              tmem_regs_ready(r);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (half == 0) mbar_arrive(&tempty[acc]);
        else mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), lead));  // the even CTA's MMA waits on it
      }
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
    }
    if (tma_store && lane == 0) bulk_wait_group<0>();  // stores complete before the CTA exits
    if (epi.n_peers > 0) __threadfence_system();  // peer stores performed before the kernel ends
    __syncwarp();
  }

  // under PAIR also: neither CTA exits while the other may still signal its barriers
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, bool GROUPED, bool PAIR, bool ACTMUL = false>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, bool tma_store, const Epi& epi,
           const Groups& grp, int M, int N, int K, int grid, bool vec_ok, cudaStream_t st) {
  using C = Cfg<BN, PAIR>;
  auto kern = w8a8_tile_kernel<BN, GROUPED, PAIR, ACTMUL>;
  static std::atomic<bool> configured[fni8h::kMaxDevices] = {};  // the attribute is set per device
  const int dev = fni8h::current_device();
  if (dev < 0 || dev >= fni8h::kMaxDevices) return fni8h::fail(FNI8_ERR_CUDA, "no current CUDA device");
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return fni8h::cuda_status(e, "cudaFuncSetAttribute(tile gemm)");
    // whole unified L1/shared array as shared memory: the next kernel on the stream can
    // then become resident next to this one (PDL) without an L1/shared reconfiguration
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return fni8h::cuda_status(e, "carveout(tile gemm)");
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fni8h::pdl_enabled();
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = PAIR ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, to, epi, grp, M, N, K, vec_ok ? 1 : 0, tma_store ? 1 : 0);
  if (e != cudaSuccess) return fni8h::cuda_status(e, "launch tile gemm");
  return FNI8_OK;
}

}  // namespace tile
}  // namespace fni8b

// ------------------------------------------------------------------------------------
// Internal host entry points (declared in gemm_internal.h, used by capi.cu / moe.cu)
// ------------------------------------------------------------------------------------

namespace fni8h {

using namespace fni8b;

int tile_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tile::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read tile watchdog");
  e = cudaMemcpyToSymbol(tile::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear tile watchdog");
  *code = v;
  return FNI8_OK;
}

// Measured on B200: CTA pairs raise the dense prefill GEMMs by 4-10 %, while the grouped
// expert GEMM, whose experts mostly hold fewer than 256 rows, loses ~10 % (a pair spends
// two SMs on a short segment). FNI8_TUNE_TILE_PAIR / FNI8_TUNE_GROUPED_PAIR.
bool tile_pair_enabled() { return FNI8_TUNE_TILE_PAIR != 0; }

bool grouped_pair_enabled() { return FNI8_TUNE_GROUPED_PAIR != 0; }

// L2 prefetch depth and the point where the next kernel is released (FNI8_TUNE_TILE_L2AHEAD
// and FNI8_TUNE_TILE_TRIGGER).
static int tile_l2ahead() { return FNI8_TUNE_TILE_L2AHEAD < 0 ? 0 : FNI8_TUNE_TILE_L2AHEAD; }

static int tile_trigger() { return FNI8_TUNE_TILE_TRIGGER; }

// Tensor map for the TMA-store epilogue: 16-bit outputs whose rows are 16-byte aligned.
// Returns false (per-thread stores) otherwise; no error is raised for that.
static bool out_tma_map(CUtensorMap* map, void* out, int out_mode, int64_t rows, int64_t N) {
  if (out_mode == tile::kOutI32 || (N * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) return false;
  if (encode_tmap_2d_16_sw(map, out, out_mode == tile::kOutBF16, (uint64_t)N, (uint64_t)rows, (uint64_t)N * 2, 32, 32,
                           true) != FNI8_OK)
    return false;
  return true;
}

int tile_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
              const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, int bn, bool pair,
              cudaStream_t st) {
  if (M <= 0 || N <= 0) return FNI8_OK;
  if (bn != 128 && bn != 256) return fail(FNI8_ERR_INVALID, "tile BN must be 128 or 256");
  CUtensorMap ta, tb;
  if (int s = encode_tmap_2d_i8(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, 128)) return s;
  if (int s = encode_tmap_2d_i8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, (uint32_t)(pair ? bn / 2 : bn)))
    return s;
  tile::Epi epi{a_scale, w_scale, bias, residual, out, out_mode, tile_l2ahead(), tile_trigger()};
  tile::Groups grp{nullptr, nullptr, nullptr, 0};
  const int bmt = pair ? 256 : 128;
  const int m_tiles = (int)((M + bmt - 1) / bmt);
  const int n_tiles = (int)((N + bn - 1) / bn);
  const int64_t tiles = (int64_t)m_tiles * n_tiles;
  const int sms = num_sms(current_device());
  // one CTA per tile (two per tile under PAIR), at most one per SM
  const int64_t ctas = pair ? 2 * tiles : tiles;
  const int cap = pair ? (sms & ~1) : sms;
  const int grid = (int)(ctas < cap ? ctas : cap);
  const size_t esz = out_mode == tile::kOutI32 ? 4 : 2;
  const bool vec_ok = ((N * (int64_t)esz) % 16 == 0) && (((uintptr_t)out & 15u) == 0) &&
                      (((uintptr_t)w_scale & 15u) == 0) && (bias == nullptr || ((uintptr_t)bias & 15u) == 0) &&
                      (residual == nullptr || ((uintptr_t)residual & 15u) == 0);
  CUtensorMap to;
  const bool tma_store = out_tma_map(&to, out, out_mode, M, N);
  if (pair) {
    if (bn == 256)
      return tile::launch<256, false, true>(ta, tb, to, tma_store, epi, grp, (int)M, (int)N, (int)K, grid, vec_ok, st);
    return tile::launch<128, false, true>(ta, tb, to, tma_store, epi, grp, (int)M, (int)N, (int)K, grid, vec_ok, st);
  }
  if (bn == 256)
    return tile::launch<256, false, false>(ta, tb, to, tma_store, epi, grp, (int)M, (int)N, (int)K, grid, vec_ok, st);
  return tile::launch<128, false, false>(ta, tb, to, tma_store, epi, grp, (int)M, (int)N, (int)K, grid, vec_ok, st);
}

int tile_gemm_peer_cols(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                        int out_mode, int64_t M, int64_t N, int64_t K, void* const* peer_out, int n_peers, int64_t ld,
                        int64_t col_off, int bn, bool pair, cudaStream_t st) {
  if (M <= 0 || N <= 0) return FNI8_OK;
  if (n_peers < 1 || n_peers > tile::kMaxPeers) return fail(FNI8_ERR_INVALID, "1 to %d destinations", tile::kMaxPeers);
  CUtensorMap ta, tb, to;
  if (int s = encode_tmap_2d_i8(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, 128)) return s;
  if (int s = encode_tmap_2d_i8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, (uint32_t)(pair ? bn / 2 : bn)))
    return s;
  memset(&to, 0, sizeof(to));
  tile::Epi epi{a_scale, w_scale, bias, nullptr, nullptr, out_mode, tile_l2ahead(), tile_trigger()};
  epi.n_peers = n_peers;
  epi.peer_col = (int)col_off;
  epi.peer_ld = ld;
  for (int i = 0; i < n_peers; ++i) epi.peer_out[i] = peer_out[i];
  // Tile bands (m-tiles per band): measured on B200s at M=4096, ld=28672 (K=8192), 2 and 4
  // ranks run fastest with the prefill's bands of 16 m-tiles, whose waves reuse the
  // weights from L2 (373 and 362 us per call; bands of 1 and 9 m-tiles: 425 and 513 us);
  // on 8 ranks those bands, with all 4096 rows in flight towards eight destinations, store
  // at ~60 GB/s (3.4 ms per call) and bands of 4 m-tiles (~1400 rows in flight) take 1.0 ms.
  epi.band = n_peers > 4 ? 4 : tile::kGroupM;
  tile::Groups grp{nullptr, nullptr, nullptr, 0};
  const int bmt = pair ? 256 : 128;
  const int64_t tiles = ((M + bmt - 1) / bmt) * ((N + bn - 1) / bn);
  const int64_t ctas = pair ? 2 * tiles : tiles;
  const int sms = num_sms(current_device());
  const int cap = pair ? (sms & ~1) : sms;
  const int grid = (int)(ctas < cap ? ctas : cap);
  const int Mi = (int)M, Ni = (int)N, Ki = (int)K;
  if (pair) {
    if (bn == 256) return tile::launch<256, false, true>(ta, tb, to, false, epi, grp, Mi, Ni, Ki, grid, true, st);
    return tile::launch<128, false, true>(ta, tb, to, false, epi, grp, Mi, Ni, Ki, grid, true, st);
  }
  if (bn == 256) return tile::launch<256, false, false>(ta, tb, to, false, epi, grp, Mi, Ni, Ki, grid, true, st);
  return tile::launch<128, false, false>(ta, tb, to, false, epi, grp, Mi, Ni, Ki, grid, true, st);
}

int tile_gemm_grouped(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w, const float* w_scale,
                      int64_t E, int64_t N, int64_t K, const int32_t* seg_expert, const int32_t* seg_off,
                      const int32_t* seg_cnt, int64_t S, void* out, int out_mode, int bn, bool pair,
                      cudaStream_t st, const int32_t* row_tag, void* const* peer_out, int n_peers,
                      int64_t peer_rows) {
  if (R <= 0 || N <= 0 || S <= 0) return FNI8_OK;
  if (S > tile::kMaxSeg) return fail(FNI8_ERR_UNSUPPORTED, "at most %d segments (got %lld)", tile::kMaxSeg, (long long)S);
  CUtensorMap ta, tb;
  if (int s = encode_tmap_2d_i8(&ta, a, (uint64_t)K, (uint64_t)R, (uint64_t)K, 128, 128)) return s;
  if (int s = encode_tmap_3d_i8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)E, (uint64_t)K, (uint64_t)(N * K), 128,
                                (uint32_t)(pair ? bn / 2 : bn)))
    return s;
  tile::Epi epi{a_scale, w_scale, nullptr, nullptr, out, out_mode, tile_l2ahead(), tile_trigger()};
  tile::Groups grp{seg_expert, seg_off, seg_cnt, (int)S};
  const int sms = num_sms(current_device());
  const int grid = pair ? (sms & ~1) : sms;
  const size_t esz = out_mode == tile::kOutI32 ? 4 : 2;
  const bool aligned = ((uintptr_t)out & 15u) == 0;
  const bool vec_ok = ((N * (int64_t)esz) % 16 == 0) && aligned && (((uintptr_t)w_scale & 15u) == 0) &&
                      ((N % 4) == 0);
  CUtensorMap to;
  bool tma_store = false;
  if (row_tag != nullptr) {  // rows scattered into peers' buffers (validated by the caller)
    memset(&to, 0, sizeof(to));
    epi.row_tag = row_tag;
    epi.n_peers = n_peers;
    epi.peer_rows = peer_rows;
    for (int i = 0; i < n_peers; ++i) epi.peer_out[i] = peer_out[i];
  } else {
    tma_store = out_tma_map(&to, out, out_mode, R, N);
  }
  if (pair) {
    if (bn == 256)
      return tile::launch<256, true, true>(ta, tb, to, tma_store, epi, grp, (int)R, (int)N, (int)K, grid, vec_ok, st);
    return tile::launch<128, true, true>(ta, tb, to, tma_store, epi, grp, (int)R, (int)N, (int)K, grid, vec_ok, st);
  }
  if (bn == 256)
    return tile::launch<256, true, false>(ta, tb, to, tma_store, epi, grp, (int)R, (int)N, (int)K, grid, vec_ok, st);
  return tile::launch<128, true, false>(ta, tb, to, tma_store, epi, grp, (int)R, (int)N, (int)K, grid, vec_ok, st);
}

int tile_gemm_act(const int8_t* a, const float* a_scale, int64_t M, const int8_t* w, const float* w_scale, int64_t E,
                  int64_t I, int64_t K, const int32_t* seg_expert, const int32_t* seg_off, const int32_t* seg_cnt,
                  int64_t S, int act, void* out, int out_mode, bool pair, cudaStream_t st) {
  if (M <= 0 || I <= 0) return FNI8_OK;
  if (I % 128 != 0) return fail(FNI8_ERR_UNSUPPORTED, "act_and_mul GEMM takes I a multiple of 128 (got %lld)", (long long)I);
  if (act != FNI8_ACT_SILU && act != FNI8_ACT_GELU_TANH) return fail(FNI8_ERR_INVALID, "unknown activation %d", act);
  if (out_mode != tile::kOutF16 && out_mode != tile::kOutBF16) return fail(FNI8_ERR_INVALID, "act GEMM out: F16 or BF16");
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) return fail(FNI8_ERR_ALIGN, "act GEMM output must be 16-byte aligned");
  const bool grouped = seg_expert != nullptr;
  if (grouped && S > tile::kMaxSeg)
    return fail(FNI8_ERR_UNSUPPORTED, "at most %d segments (got %lld)", tile::kMaxSeg, (long long)S);
  const int64_t N = 2 * I;  // weight rows: gate [0, I), up [I, 2I)
  CUtensorMap ta, tb;
  if (int s = encode_tmap_2d_i8(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, 128)) return s;
  if (grouped) {
    if (int s = encode_tmap_3d_i8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)E, (uint64_t)K, (uint64_t)(N * K), 128, 128))
      return s;
  } else if (int s = encode_tmap_2d_i8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, 128)) {
    return s;
  }
  tile::Epi epi{a_scale, w_scale, nullptr, nullptr, out, out_mode, 0, tile_trigger()};
  epi.act = act;
  epi.act_i = static_cast<int>(I);
  tile::Groups grp{seg_expert, seg_off, seg_cnt, grouped ? (int)S : 0};
  const int sms = num_sms(current_device());
  int grid = pair ? (sms & ~1) : sms;
  if (!grouped) {  // one CTA per tile (two under PAIR), at most one per SM
    const int64_t tiles = ((M + (pair ? 255 : 127)) / (pair ? 256 : 128)) * (I / 128);
    const int64_t ctas = pair ? 2 * tiles : tiles;
    grid = (int)(ctas < grid ? ctas : grid);
  }
  CUtensorMap to;
  const bool tma_store = out_tma_map(&to, out, out_mode, M, I);
  const int Mi = (int)M, Ni = (int)N, Ki = (int)K;
  if (grouped) {
    if (pair) return tile::launch<256, true, true, true>(ta, tb, to, tma_store, epi, grp, Mi, Ni, Ki, grid, true, st);
    return tile::launch<256, true, false, true>(ta, tb, to, tma_store, epi, grp, Mi, Ni, Ki, grid, true, st);
  }
  if (pair) return tile::launch<256, false, true, true>(ta, tb, to, tma_store, epi, grp, Mi, Ni, Ki, grid, true, st);
  return tile::launch<256, false, false, true>(ta, tb, to, tma_store, epi, grp, Mi, Ni, Ki, grid, true, st);
}

}  // namespace fni8h
