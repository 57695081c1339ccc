// W4A8 GEMM: int8 activations x 4-bit grouped weights (fni8.linear for per_group_i4 /
// int4 weights, fni8serve/layers/linear.py:8-10,58-69).
//
//   w[n, k]   = signed int4, packed two per byte along K (element 2j in the low nibble)
//   acc_g     = sum_{k in group g} q[m, k] * w[n, k]            (exact int32, group = 128 k)
//   out[m, n] = dtype((sum_g float(acc_g) * w_scale[n, g]) * a_scale[m] (+ bias[n]))
//
// Decode-shaped (up to 64 tokens per launch; the host walks larger M in 64-token chunks).
// The layout follows the int8 split-K kernel (gemm_splitk.cu): weights are the 128-row A
// operand (swap-AB), the tokens the MMA's N (NT = 16/32/64), and the K range of a weight
// tile is split over a cluster of S CTAs so every SM streams. Differences:
//  * the weight tiles arrive packed (64 B per row, half the HBM bytes of int8); warps 6-9
//    (one weight row per thread) unpack each k-block into the 128B-swizzled int8 tile the
//    MMA reads (a three-slot ring, so unpacking runs ahead of the tensor core),
//    sign-extending nibbles four at a time;
//  * a k-block is one scale group, so every k-block gets a fresh int32 accumulator (four
//    TMEM buffers in turn, so the tensor core runs ahead of the folding) that warps 2-5 (TMEM lane quarter = warp % 4) fold into fp32
//    running sums with the row's group scale while the tensor core works on the next one;
//  * the split-K partial sums are fp32; the cluster's CTA that owns a token column adds the
//    S partials in rank order (deterministic; the order differs from a one-pass sum over
//    the groups only in fp32 rounding).
// Every mbarrier wait is bounded (fni8_common.cuh).
#include "fni8_common.cuh"
#include "gemm_internal.h"

#include <stdlib.h>

namespace fni8b {
namespace w4 {

constexpr int kThreads = 320;  // producer, MMA, 4 folding warps, 4 unpacking warps
constexpr int BNW = 128;  // weight rows per tile (MMA M)
constexpr int BK = 128;   // K elements per stage = one scale group
constexpr int PW_BYTES = BNW * BK / 2;  // packed weight tile, 64 B per row (64B swizzle)
constexpr int A_BYTES = BNW * BK;       // unpacked int8 weight tile (128B swizzle)
constexpr int kASlots = 3;
constexpr int kAccBufs = 4;
constexpr int kMaxStages = 8;
constexpr int kL2Ahead = 0;  // no early L2 prefetch (it delays the upstream kernel in decode chains)
constexpr int kBarBytes = 512;

static __device__ int g_status;

enum : int { kCodeProducer = 0x701, kCodeMma = 0x702, kCodeConvert = 0x703, kCodeDrain = 0x704 };
enum : int { kOutF16 = 0, kOutBF16 = 1 };

struct Epi {
  const float* a_scale;  // [M]
  const float* w_scale;  // [N, G]
  const void* bias;      // [N] or null
  void* out;             // [M, N] (row stride ldo)
  int mode;
  int G;                 // scale groups along K
  int64_t ldo;
};

template <int NT>
struct Cfg {
  static constexpr int X_BYTES = NT * BK;
  static constexpr int STAGE = PW_BYTES + X_BYTES;
  static constexpr int TMEM_COLS = kAccBufs * NT < 32 ? 32 : kAccBufs * NT;
  static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte alignment of the 128B swizzle");
};

// Columns of the token share each cluster rank owns (a multiple of 4).
__host__ __device__ __forceinline__ int split_share(int mcols, int S) { return ((mcols + S - 1) / S + 3) & ~3; }

// Per-byte sign extension of 4-bit values (0..15 in each byte) to int8: bit 3 set means
// negative, i.e. the high nibble becomes 0xF. (v & 0x08) * 0x1E is 0xF0 or 0 in every byte,
// so the multiply never carries into the next byte: three integer ops per 4 values.
__device__ __forceinline__ uint32_t sext4_bytes(uint32_t v) { return v | ((v & 0x08080808u) * 0x1Eu); }

// 4 packed bytes (8 signed nibbles, element 2j low) -> 8 int8 values, in element order.
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t& lo4, uint32_t& hi4) {
  const uint32_t el = sext4_bytes(w & 0x0F0F0F0Fu);
  const uint32_t eh = sext4_bytes((w >> 4) & 0x0F0F0F0Fu);
  lo4 = __byte_perm(el, eh, 0x5140);  // elements 0..3 of the word
  hi4 = __byte_perm(el, eh, 0x7362);  // elements 4..7
}

template <typename T, int NT>
__device__ __forceinline__ void emit_col(const Epi& epi, int m, int n, float v, float bn) {
  float y = __fmul_rn(v, __ldg(epi.a_scale + m));
  if (epi.bias != nullptr) y = __fadd_rn(y, bn);
  static_cast<T*>(epi.out)[static_cast<int64_t>(m) * epi.ldo + n] = from_f32<T>(y);
}

// Up to 32 tokens two CTAs share an SM (the plan counts on it): registers capped for that.
template <int NT>
__global__ void __launch_bounds__(kThreads, NT <= 32 ? 2 : 1)
    w4a8_splitk_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmX, Epi epi,
                       int M, int N, int K, int STG, uint4* ws) {
  using C = Cfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aslot = smem;                           // [kASlots][A_BYTES] unpacked weights
  uint8_t* ring = smem + kASlots * A_BYTES;        // [STG][STAGE]: packed weights | activations
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STG * C::STAGE);
  uint64_t* empty = full + kMaxStages;
  uint64_t* a_full = empty + kMaxStages;
  uint64_t* a_empty = a_full + kASlots;
  uint64_t* acc_full = a_empty + kASlots;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint64_t* drain = acc_empty + kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t S = cluster_nctarank();
  const int tile = static_cast<int>(blockIdx.x / S);
  const int kb = (K + BK - 1) / BK;
  const int kbeg = static_cast<int>(static_cast<int64_t>(rank) * kb / S);
  const int nk = static_cast<int>(static_cast<int64_t>(rank + 1) * kb / S) - kbeg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kASlots; ++s) {
      mbar_init(&a_full[s], 4);  // one arrive per unpacking warp
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
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

  auto stage_at = [&](int s) { return ring + s * C::STAGE; };
  int okt = 1;  // folding warps: every wait succeeded
  float accf[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) accf[t] = 0.0f;
  const int trow = (warp & 3) * 32 + lane;  // warps 2-9: the weight row of this thread
  const int n = tile * BNW + trow;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmP);
      tma_prefetch_desc(&tmX);
      const int pre = nk < STG ? nk : STG;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE);
        tma_load_2d(&tmP, &full[i], stage_at(i), (kbeg + i) * (BK / 2), tile * BNW);
      }
      const int l2_end = (nk - pre) < kL2Ahead ? nk : pre + kL2Ahead;
      for (int i = pre; i < l2_end; ++i) tma_prefetch_l2_2d(&tmP, (kbeg + i) * (BK / 2), tile * BNW);
      pdl_wait();  // the activations come from the previous kernel
      for (int i = 0; i < pre; ++i) tma_load_2d(&tmX, &full[i], stage_at(i) + PW_BYTES, (kbeg + i) * BK, 0);
      int stage = pre % STG;
      uint32_t ph = (pre == STG) ? 1u : 0u;
      uint32_t armed = 0;
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&empty[stage], ph ^ 1u, &g_status, kCodeProducer)) break;
        mbar_arrive_expect_tx(&full[stage], C::STAGE);
        tma_load_2d(&tmP, &full[stage], stage_at(stage), (kbeg + i) * (BK / 2), tile * BNW);
        tma_load_2d(&tmX, &full[stage], stage_at(stage) + PW_BYTES, (kbeg + i) * BK, 0);
        armed = (armed & ~(1u << stage)) | (ph << stage);
        ++issued;
        if (++stage == STG) {
          stage = 0;
          ph ^= 1u;
        }
      }
      // the next kernel is released once this CTA's loads are all issued (its own loads
      // then queue behind ours); it waits for our completion before reading our output
      pdl_launch_dependents();
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
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % STG, a = i % kASlots, b = i % kAccBufs;
        const uint32_t ph_s = (i / STG) & 1, ph_a = (i / kASlots) & 1, ph_b = (i / kAccBufs) & 1;
        ok = mbar_wait(&a_full[a], ph_a, &g_status, kCodeMma) && mbar_wait(&full[s], ph_s, &g_status, kCodeMma) &&
             mbar_wait(&acc_empty[b], ph_b ^ 1u, &g_status, kCodeMma);
        if (!ok) break;
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(aslot + a * A_BYTES));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(stage_at(s) + PW_BYTES));
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * NT);
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk)
          umma_i8(d, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                  kk != 0 ? 1u : 0u);  // a fresh accumulator per scale group
        umma_commit(&empty[s]);
        umma_commit(&a_empty[a]);
        umma_commit(&acc_full[b]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, &g_status, kCodeDrain);
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------ unpacking
#pragma unroll 1
    for (int i = 0; i < nk; ++i) {
      const int st = i % STG, a = i % kASlots;
      int ok = 0;
      if (lane == 0)
        ok = (mbar_wait(&full[st], (i / STG) & 1, &g_status, kCodeConvert) &&
              mbar_wait(&a_empty[a], ((i / kASlots) & 1) ^ 1u, &g_status, kCodeConvert))
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const uint8_t* prow = stage_at(st) + trow * 64;
      uint8_t* arow = aslot + a * A_BYTES + trow * 128;
      // the four packed chunks are read before the first store (a shared-memory load issued
      // after a store it might alias waits for that store)
      uint4 pk[4];
#pragma unroll
      for (int c = 0; c < 4; ++c)  // 64B swizzle of the packed tile: chunk ^= (row >> 1) & 3
        pk[c] = *reinterpret_cast<const uint4*>(prow + ((c ^ ((trow >> 1) & 3)) << 4));
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 p = pk[c];
        uint4 o0, o1;
        unpack_word(p.x, o0.x, o0.y);
        unpack_word(p.y, o0.z, o0.w);
        unpack_word(p.z, o1.x, o1.y);
        unpack_word(p.w, o1.z, o1.w);
        // 128B swizzle of the MMA tile: chunk ^= row & 7
        *reinterpret_cast<uint4*>(arow + (((2 * c) ^ (trow & 7)) << 4)) = o0;
        *reinterpret_cast<uint4*>(arow + (((2 * c + 1) ^ (trow & 7)) << 4)) = o1;
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to tcgen05.mma
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[a]);
    }
  } else {
    // ------------------------------------------------------------ group scaling
    pdl_wait();  // scales may come from the previous kernel
    const uint32_t taddr_q = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float* wsr = epi.w_scale + static_cast<int64_t>(n < N ? n : 0) * epi.G + kbeg;
    float sw = n < N && nk > 0 ? __ldg(wsr) : 0.0f;
#pragma unroll 1
    for (int j = 0; j < nk; ++j) {
      // fold the accumulator of k-block j into the fp32 sums with the row's group scale
      // (all lanes: tcgen05.ld is .sync.aligned)
      const float sw_next = (j + 1 < nk && n < N) ? __ldg(wsr + j + 1) : 0.0f;
      const int b = j % kAccBufs;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&acc_full[b], (j / kAccBufs) & 1, &g_status, kCodeConvert) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      okt &= ok;
      if (!ok) break;
      tc_fence_after();
      uint32_t v[NT];
      if constexpr (NT == 16) {
        tmem_ld16(taddr_q + static_cast<uint32_t>(b * NT), reinterpret_cast<uint32_t(&)[16]>(v));
      } else {
#pragma unroll
        for (int h = 0; h < NT; h += 32)
          tmem_ld32(taddr_q + static_cast<uint32_t>(b * NT + h), *reinterpret_cast<uint32_t(*)[32]>(v + h));
      }
      tmem_ld_wait();
#pragma unroll
      for (int t = 0; t < NT; ++t)
        accf[t] = __fadd_rn(accf[t], __fmul_rn(__int2float_rn(static_cast<int>(v[t])), sw));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      sw = sw_next;
    }
  }
  __syncwarp();

  // ---------------------------------------------------------------- split-K reduction
  // Token columns [0, mcols) are dealt out in shares to the cluster's ranks; each CTA
  // publishes the fp32 sums of the columns other ranks own to its workspace slab
  // ([NT/4 granules][128 rows] of 16 bytes, the row innermost); after the cluster barrier
  // the owner gathers them, re-zeroes them and adds the S partials in rank order.
  const int mcols = (M + 3) & ~3;
  const int share = S > 1 ? split_share(mcols, static_cast<int>(S)) : mcols;
  const int own0 = static_cast<int>(rank) * share;
  const int len = own0 < mcols ? (mcols - own0 < share ? mcols - own0 : share) : 0;
  __syncthreads();  // every load landed and every MMA retired: the ring and A slots are free
  if (S > 1) {
    if (warp >= 2 && warp < 6 && okt) {
      uint4* slab = ws + static_cast<int64_t>(blockIdx.x) * (NT / 4) * BNW;
#pragma unroll
      for (int t = 0; t < NT; t += 4) {
        if (t < mcols && t / share != static_cast<int>(rank))
          __stcg(slab + (t >> 2) * BNW + trow, make_uint4(__float_as_uint(accf[t]), __float_as_uint(accf[t + 1]),
                                                          __float_as_uint(accf[t + 2]), __float_as_uint(accf[t + 3])));
      }
    }
    cluster_sync_all();  // release/acquire at cluster scope: the slabs are visible to the owners
  }
  if (warp >= 2 && warp < 6 && okt && len > 0) {
    const int g_own = len >> 2;
    const int block0 = static_cast<int>(blockIdx.x) - static_cast<int>(rank);
    uint4* land = reinterpret_cast<uint4*>(smem);  // [S-1][g_own][128] granules
    if (S > 1) {
      int pi = 0;
      for (uint32_t p = 0; p < S; ++p) {
        if (p == rank) continue;
        const uint4* slab = ws + static_cast<int64_t>(block0 + static_cast<int>(p)) * (NT / 4) * BNW +
                            (own0 >> 2) * BNW + trow;
        for (int g = 0; g < g_own; ++g) cp_async_16(land + (pi * g_own + g) * BNW + trow, slab + g * BNW);
        ++pi;
      }
      cp_async_commit();
      cp_async_wait_group<0>();
      for (uint32_t p = 0; p < S; ++p) {
        if (p == rank) continue;
        uint4* slab = ws + static_cast<int64_t>(block0 + static_cast<int>(p)) * (NT / 4) * BNW +
                      (own0 >> 2) * BNW + trow;
        for (int g = 0; g < g_own; ++g) __stcg(slab + g * BNW, make_uint4(0, 0, 0, 0));  // workspace stays zero
      }
    }
    if (n < N) {
      float bn = 0.0f;
      if (epi.bias != nullptr)
        bn = epi.mode == kOutBF16 ? to_f32<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(epi.bias)[n])
                                  : to_f32<__half>(static_cast<const __half*>(epi.bias)[n]);
      const float* landf = reinterpret_cast<const float*>(land);
      // all sums first, then all stores (a shared-memory load issued after a store it might
      // alias waits for that store)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= own0 && t < own0 + len && t < M) {
          const int lt = t - own0;
          float tot = 0.0f;
          int pi = 0;
          for (uint32_t p = 0; p < S; ++p) {  // rank order: deterministic for a given split
            float v;
            if (p == rank) {
              v = accf[t];
            } else {
              v = landf[((pi * g_own + (lt >> 2)) * BNW + trow) * 4 + (lt & 3)];
              ++pi;
            }
            tot = p == 0 ? v : __fadd_rn(tot, v);
          }
          accf[t] = tot;
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= own0 && t < own0 + len && t < M) {
          if (epi.mode == kOutBF16) emit_col<__nv_bfloat16, NT>(epi, t, n, accf[t], bn);
          else emit_col<__half, NT>(epi, t, n, accf[t], bn);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace w4
}  // namespace fni8b

namespace fni8h {

using namespace fni8b;

int w4a8_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, w4::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read W4A8 watchdog");
  e = cudaMemcpyToSymbol(w4::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear W4A8 watchdog");
  *code = v;
  return FNI8_OK;
}

struct W4Plan {
  int nt, S, grid, stages, smem;
  size_t ws_bytes;
};

// One launch covers up to 64 tokens. Up to 32 tokens a CTA fits in half an SM (registers
// and ~113 KB of shared memory), so S brings the grid to twice the SM count; 64 tokens take
// a whole SM. S is then lowered until every cluster can be resident at once. The ring fills the shared-memory budget next to the unpacked slots (at most
// 8 stages) and, drained, also holds the owner's landing area.
static bool plan_w4(int64_t M, int64_t N, int64_t K, W4Plan* p) {
  if (M < 1 || N < 1 || K < w4::BK) return false;
  const int64_t mc = M < kW4ChunkM ? M : kW4ChunkM;
  int nt = 16;
  while (nt < mc) nt <<= 1;
  p->nt = nt;
  const int stage = w4::PW_BYTES + nt * w4::BK;
  const int n_tiles = (int)((N + w4::BNW - 1) / w4::BNW);
  const int kb = (int)(K / w4::BK);
  const int sms = num_sms(current_device());
  const bool two = nt <= 32;
  const int target = two ? 2 * sms : sms;
  int S = n_tiles >= target ? 1 : target / n_tiles;
  if (S > 8) S = 8;
  if (S > kb) S = kb;
  const int fixed = 1024 + w4::kASlots * w4::A_BYTES + w4::kBarBytes;
  int stages = ((two ? 113 : 225) * 1024 - fixed) / stage;
  if (stages > w4::kMaxStages) stages = w4::kMaxStages;
  const int smem = fixed + stages * stage;
  // every cluster resident at once (a second wave of clusters doubles the time)
  while (S > 1) {
    const int mc = max_active_clusters(w4::kThreads, smem, S);
    if (mc < 0 || n_tiles <= mc) break;
    --S;
  }
  const int share = ((nt + S - 1) / S + 3) & ~3;
  const int land = (S - 1) * share * w4::BNW * 4;
  if (stages < 2 || land > w4::kASlots * w4::A_BYTES + stages * stage) return false;
  p->S = S;
  p->grid = n_tiles * S;
  p->stages = stages;
  p->smem = fixed + stages * stage;
  p->ws_bytes = S > 1 ? static_cast<size_t>(p->grid) * nt * w4::BNW * 4 : 0;
  return true;
}

size_t w4a8_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  W4Plan p;
  return plan_w4(M, N, K, &p) ? p.ws_bytes : 0;
}

template <int NT>
static int launch_w4(const CUtensorMap& tp, const CUtensorMap& tx, const w4::Epi& epi, int M, int N, int K,
                     const W4Plan& p, uint4* ws, cudaStream_t st) {
  auto kern = w4::w4a8_splitk_kernel<NT>;
  static std::atomic<bool> configured[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(FNI8_ERR_CUDA, "no current CUDA device");
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(w4a8 gemm)");
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "carveout(w4a8 gemm)");
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(w4::kThreads);
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tp, tx, epi, M, N, K, p.stages, ws);
  if (e != cudaSuccess) return cuda_status(e, "launch w4a8 gemm");
  return FNI8_OK;
}

int w4a8_gemm(const int8_t* a, const float* a_scale, const uint8_t* w4, const float* w_scale, const void* bias,
              void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (M <= 0) return FNI8_OK;
  W4Plan p;
  if (!plan_w4(M, N, K, &p)) return fail(FNI8_ERR_UNSUPPORTED, "W4A8 GEMM: shape does not fit");
  if (p.ws_bytes > 0 && (ws == nullptr || ws_bytes < p.ws_bytes))
    return fail(FNI8_ERR_WORKSPACE, "W4A8 GEMM needs %zu workspace bytes (got %zu)", p.ws_bytes, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return fail(FNI8_ERR_ALIGN, "workspace must be 16-byte aligned");
  CUtensorMap tp;
  if (int s = encode_tmap_2d_u8_sw64(&tp, w4, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), 64, 128)) return s;
  const size_t esz = 2;
  for (int64_t m0 = 0; m0 < M; m0 += kW4ChunkM) {  // 64 tokens per launch
    const int64_t mc = (M - m0) < kW4ChunkM ? (M - m0) : kW4ChunkM;
    W4Plan pc;
    plan_w4(mc, N, K, &pc);
    CUtensorMap tx;
    if (int s = encode_tmap_2d_i8(&tx, a + m0 * K, (uint64_t)K, (uint64_t)mc, (uint64_t)K, 128, (uint32_t)pc.nt))
      return s;
    w4::Epi epi{a_scale + m0, w_scale, bias, static_cast<uint8_t*>(out) + m0 * N * esz, out_mode, (int)(K / w4::BK), N};
    uint4* w = static_cast<uint4*>(ws);
    int s = FNI8_OK;
    switch (pc.nt) {
      case 16: s = launch_w4<16>(tp, tx, epi, (int)mc, (int)N, (int)K, pc, w, st); break;
      case 32: s = launch_w4<32>(tp, tx, epi, (int)mc, (int)N, (int)K, pc, w, st); break;
      default: s = launch_w4<64>(tp, tx, epi, (int)mc, (int)N, (int)K, pc, w, st); break;
    }
    if (s != FNI8_OK) return s;
  }
  return FNI8_OK;
}

}  // namespace fni8h
