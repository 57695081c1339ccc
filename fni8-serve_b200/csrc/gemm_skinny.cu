// Fused decode linear: fni8.linear(x, qt) for M <= 32 tokens in ONE launch.
//
//   out[m, n] = dtype((float(sum_k q[m,k] * w[n,k]) * s[m]) * w_scale[n] (+ bias[n]))
//   s[m] = absmax(x[m, :]) / 127,  q = round_half_even(x * (127 / absmax))   (per-token int8)
//
// At decode sizes a linear is a chain of short latencies (launch, first HBM round trip,
// cross-CTA reduction), so the activation quantisation and the split-K reduction live in
// the GEMM kernel itself instead of in extra kernels and global atomics:
//
//  * grid = n_tiles x S CTAs, clustered S at a time (S <= 8). A cluster owns one tile of
//    128 weight rows (the tcgen05 MMA's M), CTA rank r of the cluster the r-th slice of
//    the K range. Weights are the A operand (swap-AB), tokens the N operand (NT = 16/32).
//  * warp 0 streams the weight tiles of its K slice through a TMA ring. Weights never
//    depend on the previous kernel, so the first ring is issued before the
//    grid-dependency wait; the next kernel is released once every load is issued.
//  * warps 2-5 read the activations of the K slice, take each token's absmax over it,
//    exchange the S partial maxima through distributed shared memory (remote mbarrier
//    arrivals + ld.shared::cluster), then write the whole slice as int8 into shared memory
//    in the 128B-swizzled K-major layout the MMA reads.
//  * warp 1 issues tcgen05.mma kind::i8 (M=128, N=NT, K=32) into a TMEM accumulator.
//  * the S partial accumulators are summed by the cluster's rank-0 CTA over DSMEM and the
//    dequant epilogue stores out[m, n] (coalesced along n).
// No workspace, no atomics in global memory, and the results equal those of the separate
// quantiser + GEMM kernels bit for bit. Every wait is bounded (fni8_common.cuh).
#include "fni8_common.cuh"
#include "gemm_internal.h"

#include <stdlib.h>

namespace fni8b {
namespace skinny {

constexpr int kThreads = 192;
constexpr int BNW = 128;  // weight rows per tile (MMA M)
constexpr int BK = 128;   // K elements per stage
// Weight k-blocks per CTA pulled into L2 beyond the ring before the dependency wait: none
// (measured on B200 in decode chains: the next kernel's early prefetch delays this one).
constexpr int kL2Ahead = 0;
constexpr int kFullRowMaxM = 2;  // tokens for which each CTA reads the whole row instead of exchanging maxima

static __device__ int g_status;

// Timeline tracing for measurement builds only (-DFNI8_TRACE): per CTA, the globaltimer
// of the phases of the fused kernel, in launch order.
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

enum : int {
  kCodeProducer = 0x301,
  kCodeMma = 0x302,
  kCodeConvert = 0x303,
  kCodeEpilogue = 0x304,
  kCodeDrain = 0x305,
  kCodeExchange = 0x306
};

constexpr int kMaxStages = 8;
constexpr int W_BYTES = BNW * BK;  // one int8 weight tile, 128B swizzle

// Shared memory: [WST weight stages][nk_max int8 activation tiles of XR x 128 B][barriers].
// XR = NT rows, or 8 when M <= 8: the MMA then reads its second 8-row group from the first
// (group stride 0); those accumulator columns duplicate real ones and are never stored.
template <int NT>
struct Cfg {
  static constexpr int XI_BYTES = NT * BK;  // one int8 activation tile, 128B swizzle
  static constexpr int PART_LD = NT + 4;    // padded row of the int32 partial tile
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static constexpr int BAR_BYTES = 1024;
  static_assert(XI_BYTES % 1024 == 0, "activation tiles keep the 1024-byte swizzle alignment");
  static_assert(128 * PART_LD * 4 <= 2 * W_BYTES, "the partial tile reuses the weight ring");
};

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(h[i]);
}

__device__ __forceinline__ int8_t q8(float v, float inv) {  // inv = 127 / absmax (0 for a zero row)
  float q = rintf(__fmul_rn(v, inv));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(q));
}

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_linear_kernel(const __grid_constant__ CUtensorMap tmW, const T* __restrict__ x, const float* __restrict__ w_scale, const T* __restrict__ bias,
                         T* __restrict__ out, int M, int N, int K, int WST, int nk_max) {
  using C = Cfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xi_base = smem + WST * W_BYTES;
  const int xtile = (M <= 8 ? 8 : NT) * BK;  // bytes of one int8 activation tile
  const uint32_t xsbo = M <= 8 ? 0u : 1024u;
  uint64_t* full = reinterpret_cast<uint64_t*>(xi_base + nk_max * xtile);
  uint64_t* empty = full + kMaxStages;
  uint64_t* xready = empty + kMaxStages;
  uint64_t* tfull = xready + 1;
  uint64_t* pmax_bar = tfull + 1;
  uint64_t* red_bar = pmax_bar + 1;
  uint64_t* drain = red_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* s_pmax = reinterpret_cast<int*>(tmem_slot + 4);  // [32] absmax bits of this CTA's K slice
  float* s_scale = reinterpret_cast<float*>(s_pmax + 32);
  float* s_inv = s_scale + 32;
  int32_t* part = reinterpret_cast<int32_t*>(smem);  // [128][PART_LD] partial sums, after the mainloop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t S = cluster_nctarank();
  const int tile = static_cast<int>(blockIdx.x / S);
  const int kb = (K + BK - 1) / BK;
  const int kbeg = static_cast<int>(static_cast<int64_t>(rank) * kb / S);
  const int kend = static_cast<int>(static_cast<int64_t>(rank + 1) * kb / S);
  const int nk = kend - kbeg;

  FNI8_TRACE_SLOT
  if (threadIdx.x == 0) {
    FNI8_TRACE_AT(0);
    FNI8_TRACE_VAL(7, (static_cast<unsigned long long>(N) << 32) | (static_cast<unsigned long long>(M) << 24) |
                          blockIdx.x);
    for (int s = 0; s < WST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(xready, 4);
    mbar_init(tfull, 1);
    mbar_init(pmax_bar, S);
    mbar_init(red_bar, S);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) s_pmax[threadIdx.x] = 0;
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  // Peers arrive on our barriers remotely: all of the cluster is initialised first.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto w_at = [&](int s) { return smem + s * W_BYTES; };

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    // Weights only: they never depend on the previous kernel, so the whole stream starts
    // before the grid-dependency wait (the activations are read by warps 2-5).
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      const int pre = nk < WST ? nk : WST;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], W_BYTES);
        tma_load_2d(&tmW, &full[i], w_at(i), (kbeg + i) * BK, tile * BNW);
      }
      const int l2_end = (nk - pre) < kL2Ahead ? nk : pre + kL2Ahead;
      for (int i = pre; i < l2_end; ++i) tma_prefetch_l2_2d(&tmW, (kbeg + i) * BK, tile * BNW);
      int stage = pre % WST;
      uint32_t ph = (pre == WST) ? 1u : 0u;
      uint32_t armed = 0;
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&empty[stage], ph ^ 1u, &g_status, kCodeProducer)) break;
        mbar_arrive_expect_tx(&full[stage], W_BYTES);
        tma_load_2d(&tmW, &full[stage], w_at(stage), (kbeg + i) * BK, tile * BNW);
        armed = (armed & ~(1u << stage)) | (ph << stage);
        ++issued;
        if (++stage == WST) {
          stage = 0;
          ph ^= 1u;
        }
      }
      // the next kernel is released once every weight load of this CTA is issued (its own
      // loads then queue behind ours)
      pdl_launch_dependents();
      const int pending = issued < WST ? issued : WST;
      for (int i = 0; i < pending; ++i) {
        const int s = (stage - 1 - i + 2 * WST) % WST;
        mbar_wait(&full[s], (armed >> s) & 1u, &g_status, kCodeDrain);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_i8(BNW, NT);
      int stage = 0;
      uint32_t ph = 0;
      bool ok = mbar_wait(xready, 0, &g_status, kCodeMma);  // int8 activations of the whole slice
      for (int i = 0; i < nk && ok; ++i) {
        if (!mbar_wait(&full[stage], ph, &g_status, kCodeMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(w_at(stage)));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(xi_base + i * xtile), xsbo);
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk)
          umma_i8(tmem_base, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                  (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == WST) {
          stage = 0;
          ph ^= 1u;
        }
      }
      if (ok) umma_commit(tfull);
      umma_commit(drain);
      mbar_wait(drain, 0, &g_status, kCodeDrain);
    }
  } else {
    // -------------------------------------------------------------- quantise + epilogue
    const int ct = threadIdx.x - 64;  // 0..127
    pdl_wait();
    if (ct == 0) FNI8_TRACE_AT(1);
    // (1) absmax of each token, straight from global memory: over the CTA's own K slice
    //     (combined across the cluster below), or over the whole row when M is so small
    //     that reading it is cheaper than the cross-CTA exchange
    const bool full_row = M <= kFullRowMaxM;
    const int mrows = M < NT ? M : NT;
    int tpr = 128;  // threads per token row
    while (tpr > 1 && tpr * mrows > 128) tpr >>= 1;
    const int row = ct / tpr, sub = ct % tpr;
    float amax = 0.0f;
    if (row < mrows) {
      const int e0 = full_row ? 0 : kbeg * BK;
      const int e1 = full_row ? K : ((kend * BK < K) ? kend * BK : K);
      const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * K + e0);
      const int nch = (e1 - e0) >> 3;
      for (int c0 = sub; c0 < nch; c0 += 8 * tpr) {
        uint4 raw[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) raw[u] = (c0 + u * tpr < nch) ? __ldg(xr + c0 + u * tpr) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float f[8];
          unpack8<T>(raw[u], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
        }
      }
    }
    const int span = tpr < 32 ? tpr : 32;
    for (int o = 1; o < span; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (row < mrows && (sub & 31) == 0) atomicMax(&s_pmax[row], __float_as_int(amax));
    named_bar_sync(1, 128);
    if (ct == 0) FNI8_TRACE_AT(2);
    // (2) publish the slice maxima to every CTA of the cluster, then combine all slices
    bool ok = true;
    if (full_row) {
      if (ct < NT) {
        const float mx = __int_as_float(s_pmax[ct]);
        s_scale[ct] = __fdiv_rn(mx, 127.0f);
        s_inv[ct] = mx > 0.0f ? __fdiv_rn(127.0f, mx) : 0.0f;
      }
    } else {
      if (ct == 0)
        for (uint32_t p = 0; p < S; ++p) mbar_arrive_cluster(mapa_shared(smem_u32(pmax_bar), p));
      ok = __all_sync(0xffffffffu, mbar_wait_cluster(pmax_bar, 0, &g_status, kCodeExchange) ? 1 : 0) != 0;
      if (ct < NT) {
        int mx = 0;
        for (uint32_t p = 0; p < S; ++p)
          mx = max(mx, static_cast<int>(ld_dsmem_u32(mapa_shared(smem_u32(&s_pmax[ct]), p))));
        s_scale[ct] = __fdiv_rn(__int_as_float(mx), 127.0f);
        s_inv[ct] = __int_as_float(mx) > 0.0f ? __fdiv_rn(127.0f, __int_as_float(mx)) : 0.0f;
      }
    }
    named_bar_sync(1, 128);
    if (ct == 0) FNI8_TRACE_AT(3);
    // (3) the whole K slice of the activations -> int8, in the MMA's 128B-swizzled layout
    //     (rows >= M are never stored, so their bytes do not matter: the MMA columns they
    //     feed are discarded)
    if (ok) {
      const int per_kb = M * 8;  // 16-element chunks per k-block: (row, chunk-of-row)
      const int chunks = per_kb * nk;
      for (int c0 = ct; c0 < chunks; c0 += 4 * 128) {
        uint4 raw[4][2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // issue all loads of the batch first
          const int c = c0 + u * 128;
          raw[u][0] = raw[u][1] = make_uint4(0, 0, 0, 0);
          if (c < chunks) {
            const int kk = c / per_kb;
            const int rem = c - kk * per_kb;
            const int e = (kbeg + kk) * BK + (rem & 7) * 16;
            if (e < K) {  // K is a multiple of 16: a chunk is fully inside or past the end
              const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(rem >> 3) * K + e);
              raw[u][0] = __ldg(src);
              raw[u][1] = __ldg(src + 1);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * 128;
          if (c >= chunks) break;
          const int kk = c / per_kb;
          const int rem = c - kk * per_kb;
          const int r = rem >> 3, j = rem & 7;
          float f[16];
          unpack8<T>(raw[u][0], f);
          unpack8<T>(raw[u][1], f + 8);
          const float s = s_inv[r];
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            w4[q] = static_cast<uint32_t>(static_cast<uint8_t>(q8(f[4 * q], s))) |
                    (static_cast<uint32_t>(static_cast<uint8_t>(q8(f[4 * q + 1], s))) << 8) |
                    (static_cast<uint32_t>(static_cast<uint8_t>(q8(f[4 * q + 2], s))) << 16) |
                    (static_cast<uint32_t>(static_cast<uint8_t>(q8(f[4 * q + 3], s))) << 24);
          *reinterpret_cast<uint4*>(xi_base + kk * xtile + r * 128 + ((j ^ (r & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to tcgen05.mma
    }
    __syncwarp();
    if (lane == 0 && ok) mbar_arrive(xready);
    if (ct == 0) FNI8_TRACE_AT(4);
    // (4) accumulator -> partial sums -> rank 0 sums the cluster and stores
    const int q = warp & 3;
    const int trow = q * 32 + lane;
    int okt = 0;
    if (lane == 0 && ok) okt = mbar_wait(tfull, 0, &g_status, kCodeEpilogue) ? 1 : 0;
    okt = __shfl_sync(0xffffffffu, okt, 0);
    if (ct == 0) FNI8_TRACE_AT(5);
    uint32_t acc[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j] = 0;
    if (okt) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (NT == 16) tmem_ld16(taddr, reinterpret_cast<uint32_t(&)[16]>(acc));
      else tmem_ld32(taddr, reinterpret_cast<uint32_t(&)[32]>(acc));
      tmem_ld_wait();
    }
    tc_fence_before();
    bool store = (S == 1);
    if (S > 1) {
#pragma unroll
      for (int j = 0; j < NT; j += 4)
        *reinterpret_cast<uint4*>(part + trow * C::PART_LD + j) = make_uint4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      named_bar_sync(1, 128);
      if (ct == 0) mbar_arrive_cluster(mapa_shared(smem_u32(red_bar), 0));
      if (rank == 0) {
        const bool okr = mbar_wait_cluster(red_bar, 0, &g_status, kCodeEpilogue);
        if (okr) {
          for (uint32_t p = 1; p < S; ++p) {
            const uint32_t base = mapa_shared(smem_u32(part + trow * C::PART_LD), p);
#pragma unroll
            for (int j = 0; j < NT; j += 4) {
              const uint4 v = ld_dsmem_v4(base + j * 4);
              acc[j] += v.x;
              acc[j + 1] += v.y;
              acc[j + 2] += v.z;
              acc[j + 3] += v.w;
            }
          }
          store = okt != 0;
        }
      }
    }
    if (store && okt) {
      const int n = tile * BNW + trow;
      if (n < N) {
        const float wsn = __ldg(w_scale + n);
        const float bn = bias != nullptr ? to_f32<T>(bias[n]) : 0.0f;
        // every scale is read before the first store (a shared-memory load issued after a
        // store it might alias waits for that store)
        float sc[NT];
#pragma unroll
        for (int m = 0; m < NT; ++m) sc[m] = s_scale[m < M ? m : 0];
#pragma unroll
        for (int m = 0; m < NT; ++m) {
          if (m < M) {
            float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(acc[m])), sc[m]), wsn);
            if (bias != nullptr) v = __fadd_rn(v, bn);
            out[static_cast<int64_t>(m) * N + n] = from_f32<T>(v);
          }
        }
      }
    }
  }

  if (threadIdx.x == 64) FNI8_TRACE_AT(6);
  __syncwarp();
  cluster_sync_all();  // peers may still be reading this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace skinny
}  // namespace fni8b

namespace fni8h {

using namespace fni8b;

#ifdef FNI8_TRACE
extern "C" __attribute__((visibility("default"))) int fni8_trace_read_skinny(unsigned long long* dst, int n_records) {
  const size_t bytes = static_cast<size_t>(n_records) * 8 * sizeof(unsigned long long);
  if (cudaMemcpyFromSymbol(dst, skinny::g_trace, bytes) != cudaSuccess) return FNI8_ERR_CUDA;
  unsigned int z = 0;
  if (cudaMemcpyToSymbol(skinny::g_trace_seq, &z, sizeof(z)) != cudaSuccess) return FNI8_ERR_CUDA;
  return FNI8_OK;
}
#endif

int skinny_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, skinny::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read skinny watchdog");
  e = cudaMemcpyToSymbol(skinny::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear skinny watchdog");
  *code = v;
  return FNI8_OK;
}

struct SkinnyPlan {
  int nt, S, wst, nk_max, smem;
};

// Shared memory holds the int8 activations of the CTA's whole K slice plus a weight ring.
// Two CTAs share an SM when each needs <= 113 KB, which lets the grid go up to twice the SM
// count and the next kernel's CTAs start under PDL; the cluster size S (a power of two <= 8,
// S <= K blocks) is the largest that keeps the grid within that residency and the ring at
// >= 3 stages. Otherwise one CTA per SM with a deeper ring. FNI8_SKINNY_S forces S.
static bool plan_skinny(int64_t M, int64_t N, int64_t K, SkinnyPlan* p) {
  static const int forced = [] {
    const char* e = getenv("FNI8_SKINNY_S");
    return e ? atoi(e) : 0;
  }();
  p->nt = M <= 16 ? 16 : 32;
  const int xrows = M <= 8 ? 8 : p->nt;
  const int n_tiles = (int)((N + skinny::BNW - 1) / skinny::BNW);
  const int kb = (int)((K + skinny::BK - 1) / skinny::BK);
  const int sms = num_sms(current_device());
  auto fit = [&](int S, int budget_kb, int* wst) {
    const int nk = (kb + S - 1) / S;
    const int fixed = 2048 + nk * xrows * skinny::BK;
    int w = (budget_kb * 1024 - fixed) / skinny::W_BYTES;
    if (w > skinny::kMaxStages) w = skinny::kMaxStages;
    *wst = w;
    return nk;
  };
  for (int pass = 0; pass < 2; ++pass) {  // pass 0: two CTAs per SM; pass 1: one
    const int cap = pass == 0 ? 2 * sms : sms;
    const int budget = pass == 0 ? 113 : 225;
    int S = 1;
    if (forced == 1 || forced == 2 || forced == 4 || forced == 8) S = forced;
    else
      while (S < 8 && n_tiles * (S * 2) <= cap) S *= 2;
    while (S > 1 && S > kb) S >>= 1;
    int wst = 0;
    int nk = fit(S, budget, &wst);
    while (wst < 3 && S < 8 && S * 2 <= kb && forced == 0) {  // a deeper K split shrinks the activations
      S *= 2;
      nk = fit(S, budget, &wst);
    }
    if (wst >= 3 || (pass == 1 && wst >= 2)) {
      p->S = S;
      p->wst = wst;
      p->nk_max = nk;
      p->smem = 2048 + nk * xrows * skinny::BK + wst * skinny::W_BYTES;
      return true;
    }
  }
  return false;
}

template <typename T, int NT>
static int launch_skinny(const CUtensorMap& tw, const void* x, const float* w_scale, const void* bias, void* out,
                         int M, int N, int K, const SkinnyPlan& p, cudaStream_t st) {
  auto kern = skinny::skinny_linear_kernel<T, NT>;
  static std::atomic<bool> configured[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(FNI8_ERR_CUDA, "no current CUDA device");
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(skinny)");
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "carveout(skinny)");
    configured[dev] = true;
  }
  const int n_tiles = (N + skinny::BNW - 1) / skinny::BNW;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_tiles * p.S);
  cfg.blockDim = dim3(skinny::kThreads);
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, static_cast<const T*>(x), w_scale,
                                     static_cast<const T*>(bias), static_cast<T*>(out), M, N, K, p.wst, p.nk_max);
  if (e != cudaSuccess) return cuda_status(e, "launch skinny linear");
  return FNI8_OK;
}

bool skinny_supported(const void* x, int64_t M, int64_t N, int64_t K) {
  SkinnyPlan p;
  return M >= 1 && M <= kSkinnyMaxM && K % 16 == 0 && N < (1LL << 31) && K < (1LL << 31) &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && plan_skinny(M, N, K, &p);
}

// Largest M the AUTO choice of fni8_linear_w8a8 sends to the fused kernel: none by
// default — measured on B200, the quantiser + split-K GEMM pair is faster at every decode
// size, the fused kernel stays available as FNI8_PATH_FUSED (FNI8_SKINNY_AUTO_MAX_M
// overrides the AUTO choice for measurements).
int64_t skinny_auto_max_m() {
  static const int64_t m = [] {
    const char* e = getenv("FNI8_SKINNY_AUTO_MAX_M");
    const long v = e ? atol(e) : 0;
    return (int64_t)(v < 0 ? 0 : (v > kSkinnyMaxM ? kSkinnyMaxM : v));
  }();
  return m;
}

int skinny_linear(const void* x, bool bf16, const int8_t* w, const float* w_scale, const void* bias, void* out,
                  int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  SkinnyPlan p;
  if (!plan_skinny(M, N, K, &p)) return fail(FNI8_ERR_UNSUPPORTED, "fused decode linear: shape does not fit");
  CUtensorMap tw;
  if (int s = encode_tmap_2d_i8(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, 128)) return s;
  if (bf16)
    return p.nt == 16 ? launch_skinny<__nv_bfloat16, 16>(tw, x, w_scale, bias, out, (int)M, (int)N, (int)K, p, st)
                      : launch_skinny<__nv_bfloat16, 32>(tw, x, w_scale, bias, out, (int)M, (int)N, (int)K, p, st);
  return p.nt == 16 ? launch_skinny<__half, 16>(tw, x, w_scale, bias, out, (int)M, (int)N, (int)K, p, st)
                    : launch_skinny<__half, 32>(tw, x, w_scale, bias, out, (int)M, (int)N, (int)K, p, st);
}

}  // namespace fni8h
