// Skinny-M (decode) W8A8 GEMM: weight streaming at HBM speed on tcgen05.
//
// For M <= 256 tokens the GEMM is bound by reading W[N, K] once from HBM. The kernel
// swaps the operands so the weight rows fill the 128-row MMA dimension:
//     acc^T[n, m] = sum_k W[n, k] * x[m, k]      (tcgen05.mma kind::i8, M=128, N=NT, K=32)
// with NT = the token count rounded up to a power of two >= 16. Each accumulator lane is
// one weight row, each TMEM column one token, so the epilogue's stores of out[m, n] are
// coalesced along n.
//
// Work is split "stream-K" style: the (n-tile, k-block) units, n-tile major, are divided
// evenly over one persistent CTA per SM, so every SM streams the same number of bytes
// whatever N and K are. A CTA accumulates each maximal run of units that belong to one
// n-tile in TMEM (double-buffered), then
//   * a run covering the whole K range is finished directly (dequant epilogue), or
//   * a partial run is added with red.global.add.s32 into an int32 slot of the workspace
//     and counted; the CTA whose count completes the tile applies the epilogue from the
//     slot and zeroes it again. Integer addition is associative, so the result is
//     bit-exact and independent of the split. No CTA ever waits for another.
// The workspace (G slots of 128 x NT int32 + G counters, G = grid size) must be zero
// before the first call; every call leaves it zero.
#include "fni8_common.cuh"
#include "gemm_internal.h"

#include <stdlib.h>

namespace fni8b {
namespace strm {

constexpr int kThreads = 192;
constexpr int BNW = 128;  // weight rows per tile (MMA M)
constexpr int BK = 128;
// Weight units per CTA pulled into L2 beyond the ring before the dependency wait: none
// (measured on B200 in decode chains: early prefetch of the next kernel's weights delays
// the running kernel more than it saves).
constexpr int64_t kL2AheadUnits = 0;

static __device__ int g_status;

// Timeline tracing, compiled in only for measurement builds (-DFNI8_TRACE): per CTA, the
// globaltimer of a few pipeline events, in launch order.
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

enum : int { kCodeProducer = 0x201, kCodeMma = 0x202, kCodeEpilogue = 0x203, kCodeDrain = 0x204 };
enum : int { kOutF16 = 0, kOutBF16 = 1, kOutI32 = 2 };

struct Epi {
  const float* a_scale;  // [M]
  const float* w_scale;  // [N]
  const void* bias;      // [N] or null
  const void* residual;  // [M, N] or null
  void* out;             // [M, N]
  int mode;
};

// BUDGET_KB bounds the stage ring: at ~100 KB two CTAs fit on an SM, so the next kernel
// on the stream (launched early through PDL) can stream its first weight tiles while
// this one drains.
template <int NT, int BUDGET_KB>
struct Cfg {
  static constexpr int W_BYTES = BNW * BK;
  static constexpr int X_BYTES = NT * BK;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int STAGES_FIT = (BUDGET_KB * 1024) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 12 ? 12 : STAGES_FIT;
  static constexpr int TMEM_COLS = (2 * NT < 32) ? 32 : 2 * NT;
  static constexpr int SMEM = 1024 + STAGES * STAGE + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(STAGE % 1024 == 0, "stages must keep 1024-byte alignment for the 128B swizzle");
};

// Largest CTA index whose unit range starts at or before unit u.
__device__ __forceinline__ int owner_of(int64_t u, int64_t U, int G) {
  return static_cast<int>(((u + 1) * G + U - 1) / U) - 1;
}

template <typename T>
__device__ __forceinline__ void emit(const Epi& epi, int m, int n, int N, int32_t acc, float wsn, float bn) {
  const int64_t idx = static_cast<int64_t>(m) * N + n;
  if (epi.mode == kOutI32) {
    static_cast<int32_t*>(epi.out)[idx] = acc;
    return;
  }
  float v = __fmul_rn(__fmul_rn(__int2float_rn(acc), __ldg(epi.a_scale + m)), wsn);
  if (epi.bias != nullptr) v = __fadd_rn(v, bn);
  if (epi.residual != nullptr) v = __fadd_rn(v, to_f32<T>(static_cast<const T*>(epi.residual)[idx]));
  static_cast<T*>(epi.out)[idx] = from_f32<T>(v);
}

template <typename T, int NT>
__device__ __forceinline__ void epilogue_segment(const Epi& epi, uint32_t tbase, bool whole, int32_t* slot,
                                                 int32_t* counter, int seg_len, int kb, int tile, int M, int N,
                                                 int lane_row, int* s_flag) {
  const int n = tile * BNW + lane_row;
  const bool nvalid = n < N;
  float wsn = 0.0f, bn = 0.0f;
  if (nvalid && epi.mode != kOutI32) {
    wsn = __ldg(epi.w_scale + n);
    if (epi.bias != nullptr) bn = to_f32<T>(static_cast<const T*>(epi.bias)[n]);
  }
  constexpr int CH = NT < 32 ? NT : 32;
#pragma unroll 1
  for (int m0 = 0; m0 < NT; m0 += CH) {
    uint32_t r[CH];
    if constexpr (CH == 16) tmem_ld16(tbase + m0, reinterpret_cast<uint32_t(&)[16]>(r));
    else tmem_ld32(tbase + m0, reinterpret_cast<uint32_t(&)[32]>(r));
    tmem_ld_wait();
    if (m0 >= M) continue;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int m = m0 + j;
      if (m < M && nvalid) {
        if (whole) emit<T>(epi, m, n, N, static_cast<int32_t>(r[j]), wsn, bn);
        else red_add_s32(slot + m * BNW + lane_row, static_cast<int32_t>(r[j]));
      }
    }
  }
  if (whole) return;
  // publish this partial, then let the CTA that completes the tile finish it
  __threadfence();
  named_bar_sync(1, 128);
  if (threadIdx.x == 64) {
    const int old = atomicAdd(counter, seg_len);
    *s_flag = (old + seg_len == kb) ? 1 : 0;
  }
  named_bar_sync(1, 128);
  if (*s_flag == 0) return;
  __threadfence();
  if (nvalid) {
    for (int m = 0; m < M; ++m) {
      int32_t* p = slot + m * BNW + lane_row;
      emit<T>(epi, m, n, N, __ldcg(p), wsn, bn);
      __stcg(p, 0);
    }
  }
  if (threadIdx.x == 64) __stcg(counter, 0);
  named_bar_sync(1, 128);  // s_flag is reused by the next segment
}

template <int NT, int BUDGET_KB>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_stream_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, Epi epi,
                       int M, int N, int K, int32_t* ws) {
  using C = Cfg<NT, BUDGET_KB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* full = bars;
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* s_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  FNI8_TRACE_SLOT
  if (threadIdx.x == 0) {
    FNI8_TRACE_AT(0);
    FNI8_TRACE_VAL(7, (static_cast<unsigned long long>(N) << 32) | blockIdx.x);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = (N + BNW - 1) / BNW;
  const int kb = (K + BK - 1) / BK;
  const int64_t U = static_cast<int64_t>(n_tiles) * kb;
  const int G = gridDim.x;
  const int64_t u0 = static_cast<int64_t>(blockIdx.x) * U / G;
  const int64_t u1 = static_cast<int64_t>(blockIdx.x + 1) * U / G;

  // The weights never depend on the previous kernel, the activations do. The producer
  // therefore arms the first ring of stages and starts their weight loads before the
  // grid-dependency wait, so the first HBM round trip overlaps the upstream kernel's tail.
  if (!(warp == 0 && lane == 0)) pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0, armed = 0;
      int issued = 0;
      const int64_t pre_end = u0 + ((u1 - u0) < C::STAGES ? (u1 - u0) : C::STAGES);
      for (int64_t u = u0; u < pre_end; ++u, ++stage) {  // first use of each stage: no wait
        const int tile = static_cast<int>(u / kb);
        const int k = static_cast<int>(u - static_cast<int64_t>(tile) * kb);
        uint8_t* sw = smem + stage * C::STAGE;
        mbar_arrive_expect_tx(&full[stage], C::STAGE);
        tma_load_2d(&tmW, &full[stage], sw, k * BK, tile * BNW);
      }
      // Optionally pull the following weight tiles of this CTA into L2 as well
      // (kL2AheadUnits, none by default).
      {
        const int64_t l2_end = (u1 - pre_end) < kL2AheadUnits ? u1 : pre_end + kL2AheadUnits;
        for (int64_t u = pre_end; u < l2_end; ++u) {
          const int tile = static_cast<int>(u / kb);
          tma_prefetch_l2_2d(&tmW, static_cast<int>(u - static_cast<int64_t>(tile) * kb) * BK, tile * BNW);
        }
      }
      pdl_wait();
      FNI8_TRACE_AT(1);
      stage = 0;
      for (int64_t u = u0; u < pre_end; ++u, ++stage) {
        const int k = static_cast<int>(u % kb);
        tma_load_2d(&tmX, &full[stage], smem + stage * C::STAGE + C::W_BYTES, k * BK, 0);
        ++issued;
      }
      if (stage == C::STAGES) {
        stage = 0;
        ph = 1;
      }
      for (int64_t u = pre_end; u < u1; ++u) {
        const int tile = static_cast<int>(u / kb);
        const int k = static_cast<int>(u - static_cast<int64_t>(tile) * kb);
        if (!mbar_wait(&empty[stage], ph ^ 1u, &g_status, kCodeProducer)) break;
        uint8_t* sw = smem + stage * C::STAGE;
        mbar_arrive_expect_tx(&full[stage], C::STAGE);
        tma_load_2d(&tmW, &full[stage], sw, k * BK, tile * BNW);
        tma_load_2d(&tmX, &full[stage], sw + C::W_BYTES, k * BK, 0);
        armed = (armed & ~(1u << stage)) | (ph << stage);
        ++issued;
        if (++stage == C::STAGES) {
          stage = 0;
          ph ^= 1u;
        }
      }
      // the next kernel may start its prologue once this CTA's loads are all issued (its
      // loads then queue behind ours); it waits for our completion before reading
      pdl_launch_dependents();
      const int pending = issued < C::STAGES ? issued : C::STAGES;
      for (int i = 0; i < pending; ++i) {
        const int s = (stage - 1 - i + 2 * C::STAGES) % C::STAGES;
        mbar_wait(&full[s], (armed >> s) & 1u, &g_status, kCodeDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_i8(BNW, NT);
      int stage = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      int64_t u = u0;
      while (u < u1 && ok) {
        const int tile = static_cast<int>(u / kb);
        const int kbeg = static_cast<int>(u - static_cast<int64_t>(tile) * kb);
        const int kend = (kbeg + (u1 - u) < kb) ? static_cast<int>(kbeg + (u1 - u)) : kb;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, &g_status, kCodeMma)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * NT);
        for (int k = kbeg; k < kend; ++k) {
          if (!mbar_wait(&full[stage], ph, &g_status, kCodeMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (u == u0 && k == kbeg) FNI8_TRACE_AT(2);
          const uint8_t* sw = smem + stage * C::STAGE;
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sw));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sw + C::W_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            umma_i8(d, adesc + static_cast<uint64_t>(kk * 2), bdesc + static_cast<uint64_t>(kk * 2), kIdesc,
                    (k != kbeg || kk != 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
        u += kend - kbeg;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, &g_status, kCodeDrain);
      FNI8_TRACE_AT(3);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int lane_row = q * 32 + lane;
    int acc = 0;
    uint32_t aph = 0;
    int64_t u = u0;
    while (u < u1) {
      const int tile = static_cast<int>(u / kb);
      const int kbeg = static_cast<int>(u - static_cast<int64_t>(tile) * kb);
      const int kend = (kbeg + (u1 - u) < kb) ? static_cast<int>(kbeg + (u1 - u)) : kb;
      const bool whole = (kbeg == 0 && kend == kb);
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[acc], aph, &g_status, kCodeEpilogue) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // the finisher protocol below synchronises all four epilogue warps, so a timeout
      // in one warp must not leave the others waiting at a named barrier
      const int all_ok = named_bar_and(1, 128, ok);
      if (!all_ok) break;
      if (threadIdx.x == 64 && u == u0) FNI8_TRACE_AT(4);
      tc_fence_after();
      const int owner = owner_of(static_cast<int64_t>(tile) * kb, U, G);
      int32_t* slot = ws + static_cast<int64_t>(owner) * BNW * NT;
      int32_t* counter = ws + static_cast<int64_t>(G) * BNW * NT + owner;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * NT);
      if (epi.mode == kOutBF16)
        epilogue_segment<__nv_bfloat16, NT>(epi, tbase, whole, slot, counter, kend - kbeg, kb, tile, M, N, lane_row,
                                            s_flag);
      else
        epilogue_segment<__half, NT>(epi, tbase, whole, slot, counter, kend - kbeg, kb, tile, M, N, lane_row,
                                     s_flag);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
      u += kend - kbeg;
    }
    if (threadIdx.x == 64) FNI8_TRACE_AT(5);
  }

  __syncthreads();
  if (threadIdx.x == 0) FNI8_TRACE_AT(6);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace strm
}  // namespace fni8b

namespace fni8h {

using namespace fni8b;

#ifdef FNI8_TRACE
extern "C" __attribute__((visibility("default"))) int fni8_trace_read(unsigned long long* dst, int n_records) {
  const size_t bytes = static_cast<size_t>(n_records) * 8 * sizeof(unsigned long long);
  if (cudaMemcpyFromSymbol(dst, strm::g_trace, bytes) != cudaSuccess) return FNI8_ERR_CUDA;
  unsigned int z = 0;
  if (cudaMemcpyToSymbol(strm::g_trace_seq, &z, sizeof(z)) != cudaSuccess) return FNI8_ERR_CUDA;
  return FNI8_OK;
}
#endif

int stream_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, strm::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read stream watchdog");
  e = cudaMemcpyToSymbol(strm::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear stream watchdog");
  *code = v;
  return FNI8_OK;
}

static int stream_nt(int64_t M) {
  int nt = 16;
  while (nt < M) nt <<= 1;
  return nt;
}

static int64_t stream_grid(int64_t N, int64_t K, int sms) {
  const int64_t U = ((N + 127) / 128) * ((K + 127) / 128);
  return U < sms ? U : sms;
}

size_t stream_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || M > kStreamMaxM || N <= 0 || K <= 0) return 0;
  const int64_t G = stream_grid(N, K, num_sms(current_device()));
  return static_cast<size_t>(G) * (128 * static_cast<size_t>(stream_nt(M)) + 1) * sizeof(int32_t);
}

template <int NT, int BUDGET_KB>
static int launch_stream_cfg(const CUtensorMap& tw, const CUtensorMap& tx, const strm::Epi& epi, int M, int N, int K,
                             int grid, int32_t* ws, cudaStream_t st) {
  using C = strm::Cfg<NT, BUDGET_KB>;
  auto kern = strm::w8a8_stream_kernel<NT, BUDGET_KB>;
  static std::atomic<bool> configured[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(FNI8_ERR_CUDA, "no current CUDA device");
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(stream gemm)");
    // whole unified L1/shared array as shared memory: the next kernel on the stream can
    // then become resident next to this one (PDL) without an L1/shared reconfiguration
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "carveout(stream gemm)");
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(strm::kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fni8h::pdl_enabled();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, epi, M, N, K, ws);
  if (e != cudaSuccess) return cuda_status(e, "launch stream gemm");
  return FNI8_OK;
}

static int stream_budget_kb() { return FNI8_TUNE_STREAM_SMEM_KB == 200 ? 200 : 100; }

template <int NT>
static int launch_stream(const CUtensorMap& tw, const CUtensorMap& tx, const strm::Epi& epi, int M, int N, int K,
                         int grid, int32_t* ws, cudaStream_t st) {
  if (stream_budget_kb() == 200) return launch_stream_cfg<NT, 200>(tw, tx, epi, M, N, K, grid, ws, st);
  return launch_stream_cfg<NT, 100>(tw, tx, epi, M, N, K, grid, ws, st);
}

int stream_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws,
                size_t ws_bytes, cudaStream_t st) {
  if (M <= 0 || N <= 0) return FNI8_OK;
  if (M > kStreamMaxM) return fail(FNI8_ERR_UNSUPPORTED, "stream path takes M <= %lld (got %lld)",
                                   (long long)kStreamMaxM, (long long)M);
  const size_t need = stream_workspace_bytes(M, N, K);
  if (ws == nullptr || ws_bytes < need)
    return fail(FNI8_ERR_WORKSPACE, "stream GEMM needs %zu workspace bytes (got %zu)", need, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return fail(FNI8_ERR_ALIGN, "workspace must be 16-byte aligned");
  const int nt = stream_nt(M);
  CUtensorMap tw, tx;
  if (int s = encode_tmap_2d_i8(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, 128)) return s;
  if (int s = encode_tmap_2d_i8(&tx, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, (uint32_t)nt)) return s;
  strm::Epi epi{a_scale, w_scale, bias, residual, out, out_mode};
  const int grid = (int)stream_grid(N, K, num_sms(current_device()));
  int32_t* w32 = static_cast<int32_t*>(ws);
  switch (nt) {
    case 16: return launch_stream<16>(tw, tx, epi, (int)M, (int)N, (int)K, grid, w32, st);
    case 32: return launch_stream<32>(tw, tx, epi, (int)M, (int)N, (int)K, grid, w32, st);
    case 64: return launch_stream<64>(tw, tx, epi, (int)M, (int)N, (int)K, grid, w32, st);
    case 128: return launch_stream<128>(tw, tx, epi, (int)M, (int)N, (int)K, grid, w32, st);
    default: return launch_stream<256>(tw, tx, epi, (int)M, (int)N, (int)K, grid, w32, st);
  }
}

}  // namespace fni8h

// ------------------------------------------------------------------------------------
// Allocation-free variant of the skinny GEMM (fni8_gemm_w8a8_noalloc).
//
// The stream-K kernel needs a zero-maintained int32 scratch area for its partial tiles.
// Callers that cannot allocate device memory — an engine that has already reserved the
// whole HBM for its KV cache and weights, or a host program reaching this library through
// a thin FFI with no device allocator of its own — get that scratch from a fixed array
// compiled into the library instead. Every GPU that loads the library holds the array
// until the process exits. CUDA loads modules lazily by default, so the array is only
// materialised on a device when this file's module is first used there.
// ------------------------------------------------------------------------------------
#include <mutex>

namespace fni8b {
namespace strm {
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int64_t kNoAllocMaxM = 32;                        // rows of activations per call
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(int32_t)];

// Failure-detection self-test (fni8_watchdog_selftest): one warp, whose lane 0 waits on a
// flag that nothing in the library ever sets. The wait is bounded like every other wait in
// the library (globaltimer, at most kWaitBudgetNs), so the kernel always ends; when it
// gives up it records kCodeSelftest in this file's status word. With `dirty` set the warp
// first leaves non-zero partial sums and counts in the allocation-free scratch, the state a
// stream-K reduction abandoned by a timed-out wait would leave behind.
enum : int { kCodeSelftest = 0x2F0 };
static __device__ int g_selftest_flag;

__global__ void __launch_bounds__(32) watchdog_selftest_kernel(uint64_t budget_ns, int dirty) {
  if (dirty) {
    constexpr int n = static_cast<int>(kNoAllocScratchBytes / sizeof(int32_t));
    for (int i = threadIdx.x; i < n; i += 32) g_noalloc_scratch[i] = 0x5A5A0000 | (i & 0xFFFF);
    __threadfence();
  }
  if (threadIdx.x != 0) return;
  if (budget_ns > kWaitBudgetNs) budget_ns = kWaitBudgetNs;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (*reinterpret_cast<volatile int*>(&g_selftest_flag) != 0) return;
    if ((i & 63u) == 0u && globaltimer_ns() - t0 > budget_ns) {
      atomicCAS(&g_status, 0, kCodeSelftest);
      return;
    }
  }
}
}  // namespace strm
}  // namespace fni8b

namespace fni8h {

static std::mutex g_noalloc_mu;
static std::atomic<void*> g_noalloc_addr[kMaxDevices];

// Device address of the scratch array on the current device. The first call on a device
// looks the address up (in host code the array's name is only a stand-in for it) and
// zeroes the array on `st`; later calls read the cached address without taking the lock.
static int noalloc_scratch(int dev, cudaStream_t st, void** out) {
  void* p = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    p = g_noalloc_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      cudaError_t e = cudaGetSymbolAddress(&p, strm::g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
      e = cudaMemsetAsync(p, 0, strm::kNoAllocScratchBytes, st);
      if (e != cudaSuccess) return cuda_status(e, "clear no-alloc scratch");
      g_noalloc_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return FNI8_OK;
}

// Zero the allocation-free scratch of the current device again (synchronous). Called by
// fni8_device_status when a bounded wait has given up: a stream-K kernel that left its
// loop may have added partial sums or counts that no finishing CTA cleared.
int noalloc_scratch_reset() {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, strm::g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc scratch)");
  e = cudaMemset(p, 0, strm::kNoAllocScratchBytes);
  if (e != cudaSuccess) return cuda_status(e, "re-zero no-alloc scratch");
  return FNI8_OK;
}

}  // namespace fni8h

extern "C" int fni8_gemm_w8a8_noalloc(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                      const void* bias, const void* residual, void* out, int out_dtype, int64_t M,
                                      int64_t N, int64_t K, void* stream) {
  using namespace fni8h;
  if (M < 0 || N <= 0 || K <= 0) return fail(FNI8_ERR_INVALID, "bad GEMM shape M=%lld N=%lld K=%lld", (long long)M,
                                              (long long)N, (long long)K);
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "K=%lld must be a multiple of 16", (long long)K);
  if (N >= (1LL << 31) || K >= (1LL << 31)) return fail(FNI8_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  if (M > strm::kNoAllocMaxM)
    return fail(FNI8_ERR_UNSUPPORTED, "the allocation-free GEMM takes at most %lld rows (got %lld)",
                (long long)strm::kNoAllocMaxM, (long long)M);
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16)
    return fail(FNI8_ERR_INVALID, "out_dtype %d: expected F16 or BF16", out_dtype);
  if (M == 0) return FNI8_OK;
  if (a == nullptr || w == nullptr || out == nullptr || a_scale == nullptr || w_scale == nullptr)
    return fail(FNI8_ERR_INVALID, "null GEMM operand");
  const size_t need = stream_workspace_bytes(M, N, K);
  if (need > strm::kNoAllocScratchBytes)
    return fail(FNI8_ERR_UNSUPPORTED, "problem needs %zu scratch bytes, the built-in area holds %zu", need,
                strm::kNoAllocScratchBytes);
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(FNI8_ERR_CUDA, "no current CUDA device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if (int s = noalloc_scratch(dev, st, &scratch)) return s;
  return stream_gemm(a, a_scale, w, w_scale, bias, residual, out, out_dtype == FNI8_F16 ? 0 : 1, M, N, K, scratch,
                     strm::kNoAllocScratchBytes, st);
}

extern "C" int fni8_watchdog_selftest(int64_t wait_us, int dirty_scratch, void* stream) {
  using namespace fni8h;
  if (wait_us < 1 || wait_us > 1000000)
    return fail(FNI8_ERR_INVALID, "wait_us=%lld: expected 1 .. 1000000", (long long)wait_us);
  strm::watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(wait_us) * 1000ull, dirty_scratch != 0 ? 1 : 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "launch watchdog self-test");
  return FNI8_OK;
}
