// Expert-parallel row exchange over NVLink / NVSwitch peer memory (one process per GPU).
//
// The routed rows of an expert-parallel MoE layer move between GPUs as plain stores into
// peer memory mapped with CUDA IPC, so the split sizes never visit the host and the layer
// has no NCCL all_to_all:
//
//   dispatch  local rows sorted by expert (the plan) -> the owner rank d of the expert, at
//             dst_base[d][local expert] + the row's rank among this rank's rows of that
//             expert: int8 row, fp32 scale and a tag (source rank << 24 | the row's
//             index in the source's expert-sorted order)
//   return    every received row's expert output -> the back buffer of its source rank at
//             the tag's sorted-row index, where the source combines its tokens through
//             its own row map (row_of_slot). An owner's rows of one expert and one source
//             are consecutive sorted rows of that source, so the rows of a tile land in a
//             few contiguous runs of the sources' buffers rather than at random slots
//
// Ordering between ranks is the caller's: after each exchange kernel every rank runs a
// small NCCL all_reduce on the same stream, which a rank passes only once every rank's
// exchange kernel has completed. No kernel here waits on another GPU. Every store is
// checked against the receiving buffer's capacity; a row that would not fit is skipped and
// recorded in this file's status word (read through fni8_device_status).
#include "fni8_common.cuh"
#include "gemm_internal.h"

#include "fni8_b200.h"

#include <string.h>

namespace fni8b {
namespace ep {

constexpr int kMaxPeers = 8;
constexpr int kMaxE = 1024;
enum : int { kCodeDispatchOverflow = 0x701, kCodeReturnOverflow = 0x702, kCodeBarrier = 0x703 };

static __device__ int g_status;

struct Peers {
  void* p[kMaxPeers];
};

// Barrier of the ranks of one node over peer memory, optionally carrying n int32 words
// of this rank (the all-gather of an exchange's per-expert counts). Every rank holds a
// flag word per source rank in its buffer `flags` (this rank's flags: flags[me]) and an
// epoch counter in its own memory. The CTA (1) copies src[0 .. n) to words
// [me * n, me * n + n) of every rank's dst, (2) takes the next epoch, (3) stores it with
// release semantics into word `me` of every rank's flags, and (4) waits, with acquire
// loads, until every word of its own flags has reached the epoch. A rank can run at most
// one epoch ahead of another (it passes epoch e only after every rank has stored e), so
// `>= e` (wrap-safe) is the test. The wait is bounded by budget_ns: a rank that never
// arrives is recorded in the status word and the kernel returns, with no GPU waiting for
// good. Data stored into peers by kernels before this one on the stream are visible to a
// peer once it has passed the barrier (those kernels completed, then the release store).
__global__ void __launch_bounds__(256) barrier_kernel(Peers flags, int P, int me, uint32_t* epoch,
                                                      const int32_t* __restrict__ src, int n, Peers dst,
                                                      uint64_t budget_ns) {
  pdl_wait();  // every store of the previous kernel is done before the flags go out
  for (int i = threadIdx.x; i < P * n; i += blockDim.x) {
    const int p = i / n, j = i - p * n;
    static_cast<int32_t*>(dst.p[p])[me * n + j] = src[j];
  }
  __shared__ uint32_t s_e;
  if (threadIdx.x == 0) {
    s_e = *epoch + 1u;
    *epoch = s_e;
  }
  __threadfence_system();
  __syncthreads();
  const uint32_t e = s_e;
  if (threadIdx.x < P) {
    uint32_t* to = static_cast<uint32_t*>(flags.p[threadIdx.x]) + me;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(to), "r"(e) : "memory");
    const uint32_t* mine = static_cast<const uint32_t*>(flags.p[me]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (static_cast<int32_t>(v - e) >= 0) break;
      if ((i & 63u) == 0u && globaltimer_ns() - t0 > budget_ns) {
        atomicCAS(&g_status, 0, kCodeBarrier);
        break;
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();
}

// Placement of one exchange from cnt_all[s * E + e] (rows source rank s sends to global
// expert e; experts [d * El, (d + 1) * El) live on rank d). Rank d's receive buffer holds
// its local experts one after another, each expert's rows ordered by source rank. Lane d
// (< P) of the single warp walks owner d's local experts: dst_base[d * El + el] = where this
// rank's rows of (d, el) start in d's buffer; for d == rank also this rank's received
// segments (seg_off, seg_cnt) and their total (n_recv).
__global__ void placement_kernel(const int32_t* __restrict__ cnt_all, int P, int E, int me, int32_t* dst_base,
                                 int32_t* seg_off, int32_t* seg_cnt, int32_t* n_recv) {
  pdl_launch_dependents();
  pdl_wait();
  const int d = threadIdx.x, El = E / P;
  if (d >= P) return;
  int base = 0;
  for (int el = 0; el < El; ++el) {
    const int e = d * El + el;
    int tot = 0, before = 0;
    for (int s = 0; s < P; ++s) {
      const int c = cnt_all[s * E + e];
      tot += c;
      if (s < me) before += c;
    }
    dst_base[e] = base + before;
    if (d == me) {
      seg_off[el] = base;
      seg_cnt[el] = tot;
    }
    base += tot;
  }
  if (d == me) *n_recv = base;
}

// A warp copies `pieces` 16-byte pieces src -> dst. Each lane issues up to eight loads
// before it stores them: a store to a peer waits for its own load only, and more bytes
// stay in flight over NVLink (measured on 2 B200s: the expert-parallel layer with the
// dispatch and return kernels, 0.60 -> 0.57 ms per 4096-token step).
__device__ __forceinline__ void warp_copy(uint4* dst, const uint4* __restrict__ src, int pieces, int lane) {
  constexpr int kDepth = 8;
  for (int c0 = 0; c0 < pieces; c0 += kDepth * 32) {
    uint4 v[kDepth];
#pragma unroll
    for (int u = 0; u < kDepth; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < pieces) v[u] = __ldg(src + c);
    }
#pragma unroll
    for (int u = 0; u < kDepth; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < pieces) dst[c] = v[u];
    }
  }
}

// One warp per sorted row. offsets[E + 1]: first sorted row of each expert (offsets[E] =
// valid rows); dst_base[P * El]: where this rank's rows of (owner d, local expert el)
// start in d's receive buffers.
__global__ void dispatch_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                const int32_t* __restrict__ slot_of_row, const int32_t* __restrict__ offsets, int E,
                                int El, int k, int H, const int32_t* __restrict__ dst_base, int me, Peers pq, Peers ps,
                                Peers ptag, int64_t cap_rows) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_off[kMaxE + 1];
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = offsets[i];
  __syncthreads();
  const int n = s_off[E];
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); r < n;
       r += static_cast<int64_t>(gridDim.x) * warps) {
    int lo = 0, hi = E - 1;  // the expert whose rows contain r: largest e with s_off[e] <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int e = lo, d = e / El, el = e - d * El;
    const int64_t pos = static_cast<int64_t>(dst_base[d * El + el]) + (r - s_off[e]);
    if (pos < 0 || pos >= cap_rows) {  // uniform over the warp
      if (lane == 0) atomicExch(&g_status, kCodeDispatchOverflow);
      continue;
    }
    const int slot = slot_of_row[r];
    const int64_t t = slot / k;
    const uint4* src = reinterpret_cast<const uint4*>(q + t * H);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<int8_t*>(pq.p[d]) + pos * H);
    warp_copy(dst, src, H / 16, lane);
    if (lane == 0) {
      static_cast<float*>(ps.p[d])[pos] = __ldg(scale + t);
      static_cast<int32_t*>(ptag.p[d])[pos] = (me << 24) | static_cast<int32_t>(r);
    }
  }
  __threadfence_system();
}

// One warp per received row i < *n_recv: y[i] -> back buffer of the tag's source rank at
// the tag's sorted-row index.
template <typename T>
__global__ void return_kernel(const T* __restrict__ y, const int32_t* __restrict__ n_recv, int64_t cap_rows,
                              const int32_t* __restrict__ tag, int H, Peers pb, int P, int64_t back_rows) {
  pdl_launch_dependents();
  pdl_wait();
  int64_t n = *n_recv;
  n = n < cap_rows ? n : cap_rows;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int chunks = H * static_cast<int>(sizeof(T)) / 16;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); i < n;
       i += static_cast<int64_t>(gridDim.x) * warps) {
    const uint32_t tg = static_cast<uint32_t>(tag[i]);
    const int src = static_cast<int>(tg >> 24);
    const int64_t slot = static_cast<int64_t>(tg & 0xFFFFFFu);
    if (src >= P || slot >= back_rows) {  // uniform over the warp
      if (lane == 0) atomicExch(&g_status, kCodeReturnOverflow);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(y + i * H);
    uint4* d = reinterpret_cast<uint4*>(static_cast<T*>(pb.p[src]) + slot * H);
    warp_copy(d, s, chunks, lane);
  }
  __threadfence_system();
}

// Column all-gather step: 16-byte piece i of src [M, N] (16-bit, row stride N) to every
// destination's row at column col_off (row stride ld). Grid-stride over the M * N / 8 pieces.
__global__ void push_cols_kernel(const uint4* __restrict__ src, int64_t M, int64_t pieces_per_row, Peers dst, int P,
                                 int64_t ld, int64_t col_off) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = M * pieces_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  constexpr int kDepth = 4;  // loads in flight per thread before its stores
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < total; i0 += kDepth * stride) {
    uint4 v[kDepth];
#pragma unroll
    for (int u = 0; u < kDepth; ++u)
      if (i0 + u * stride < total) v[u] = __ldg(src + i0 + u * stride);
#pragma unroll
    for (int u = 0; u < kDepth; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < total) {
        const int64_t m = i / pieces_per_row, c = i - m * pieces_per_row;
        const int64_t off = (m * ld + col_off + 8 * c) * 2;
        for (int p = 0; p < P; ++p) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(dst.p[p]) + off) = v[u];
      }
    }
  }
  __threadfence_system();
}

}  // namespace ep
}  // namespace fni8b

using namespace fni8b;
using namespace fni8h;

namespace fni8h {
int ep_status_read_and_clear(int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, ep::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read expert-exchange status");
  e = cudaMemcpyToSymbol(ep::g_status, &z, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "clear expert-exchange status");
  *code = v;
  return FNI8_OK;
}

int push_cols(const void* src, int64_t M, int64_t N, void* const* peer_out, int n_peers, int64_t ld, int64_t col_off,
              cudaStream_t st) {
  if (M <= 0 || N <= 0) return FNI8_OK;
  if (n_peers < 1 || n_peers > ep::kMaxPeers) return fail(FNI8_ERR_INVALID, "push_cols: 1 to %d destinations", ep::kMaxPeers);
  ep::Peers d;
  for (int i = 0; i < n_peers; ++i) d.p[i] = peer_out[i];
  const int64_t pieces = M * (N / 8);
  const int64_t blocks = (pieces + 255) / 256;
  launch_pdl(ep::push_cols_kernel, dim3((int)(blocks < 148 * 8 ? blocks : 148 * 8)), dim3(256), 0, st,
             static_cast<const uint4*>(src), M, N / 8, d, n_peers, ld, col_off);
  FNI8_CHECK_LAUNCH("push_cols");
  return FNI8_OK;
}
}  // namespace fni8h

static_assert(sizeof(cudaIpcMemHandle_t) == FNI8_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int fni8_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return fail(FNI8_ERR_INVALID, "ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(ipc buffer)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "cudaIpcGetMemHandle");
  }
  *ptr = p;
  return FNI8_OK;
}

extern "C" int fni8_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(FNI8_ERR_INVALID, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
  return FNI8_OK;
}

extern "C" int fni8_ipc_close(void* ptr) {
  if (ptr == nullptr) return FNI8_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcCloseMemHandle");
  return FNI8_OK;
}

extern "C" int fni8_ipc_free(void* ptr) {
  if (ptr == nullptr) return FNI8_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_status(e, "cudaFree(ipc buffer)");
  return FNI8_OK;
}

static int load_peers(ep::Peers* out, void* const* ptrs, int P, const char* what) {
  for (int i = 0; i < ep::kMaxPeers; ++i) out->p[i] = nullptr;
  for (int i = 0; i < P; ++i) {
    if (ptrs[i] == nullptr) return fail(FNI8_ERR_INVALID, "%s: null peer buffer %d", what, i);
    out->p[i] = ptrs[i];
  }
  return FNI8_OK;
}

extern "C" int fni8_peer_barrier(void* const* peer_flags, int64_t world, int64_t rank, uint32_t* epoch,
                                 const int32_t* src, int64_t n, void* const* peer_dst, int64_t wait_us, void* stream) {
  if (world < 1 || world > ep::kMaxPeers || rank < 0 || rank >= world)
    return fail(FNI8_ERR_INVALID, "peer_barrier: 1 <= world <= %d, 0 <= rank < world", ep::kMaxPeers);
  if (n < 0 || n > 4096 || (n > 0 && (src == nullptr || peer_dst == nullptr)))
    return fail(FNI8_ERR_INVALID, "peer_barrier: 0 <= n <= 4096 words, src and peer_dst with n > 0");
  if (wait_us < 1 || wait_us > 1000000) return fail(FNI8_ERR_INVALID, "peer_barrier: wait_us in [1, 1000000]");
  if (peer_flags == nullptr || epoch == nullptr) return fail(FNI8_ERR_INVALID, "peer_barrier: null pointer");
  ep::Peers fl, dst{};
  if (int s = load_peers(&fl, peer_flags, (int)world, "peer_barrier")) return s;
  if (n > 0)
    if (int s = load_peers(&dst, peer_dst, (int)world, "peer_barrier")) return s;
  launch_pdl(ep::barrier_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), fl, (int)world, (int)rank,
             epoch, src, (int)n, dst, static_cast<uint64_t>(wait_us) * 1000ull);
  FNI8_CHECK_LAUNCH("peer_barrier");
  return FNI8_OK;
}

extern "C" int fni8_ep_placement(const int32_t* cnt_all, int64_t world, int64_t rank, int64_t E, int32_t* dst_base,
                                 int32_t* seg_off, int32_t* seg_cnt, int32_t* n_recv, void* stream) {
  if (world < 1 || world > ep::kMaxPeers || rank < 0 || rank >= world)
    return fail(FNI8_ERR_INVALID, "ep_placement: 1 <= world <= %d, 0 <= rank < world", ep::kMaxPeers);
  if (E <= 0 || E > ep::kMaxE || E % world != 0) return fail(FNI8_ERR_INVALID, "ep_placement: E must split over the ranks");
  if (!cnt_all || !dst_base || !seg_off || !seg_cnt || !n_recv) return fail(FNI8_ERR_INVALID, "ep_placement: null pointer");
  launch_pdl(ep::placement_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), cnt_all, (int)world, (int)E,
             (int)rank, dst_base, seg_off, seg_cnt, n_recv);
  FNI8_CHECK_LAUNCH("ep_placement");
  return FNI8_OK;
}

extern "C" int fni8_ep_dispatch_i8(const int8_t* q, const float* scale, const int32_t* slot_of_row,
                                   const int32_t* offsets, int64_t E, int64_t world, int64_t rank, int64_t top_k,
                                   int64_t H, const int32_t* dst_base, void* const* peer_q, void* const* peer_scale,
                                   void* const* peer_tag, int64_t cap_rows, int64_t max_rows, void* stream) {
  if (world < 1 || world > ep::kMaxPeers || rank < 0 || rank >= world)
    return fail(FNI8_ERR_INVALID, "ep_dispatch: 1 <= world <= %d, 0 <= rank < world", ep::kMaxPeers);
  if (E <= 0 || E > ep::kMaxE || E % world != 0) return fail(FNI8_ERR_INVALID, "ep_dispatch: E must split over the ranks");
  if (H <= 0 || H % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "ep_dispatch: H must be a multiple of 16");
  if (top_k <= 0 || cap_rows < 0 || max_rows < 0) return fail(FNI8_ERR_INVALID, "ep_dispatch: bad sizes");
  if (max_rows >= (1LL << 24)) return fail(FNI8_ERR_UNSUPPORTED, "ep_dispatch: at most 2^24 slots per rank");
  if (max_rows == 0) return FNI8_OK;
  if (!q || !scale || !slot_of_row || !offsets || !dst_base || !peer_q || !peer_scale || !peer_tag)
    return fail(FNI8_ERR_INVALID, "ep_dispatch: null pointer");
  if (reinterpret_cast<uintptr_t>(q) & 15u) return fail(FNI8_ERR_ALIGN, "ep_dispatch: rows must be 16-byte aligned");
  ep::Peers pq, ps, pt;
  if (int s = load_peers(&pq, peer_q, (int)world, "ep_dispatch")) return s;
  if (int s = load_peers(&ps, peer_scale, (int)world, "ep_dispatch")) return s;
  if (int s = load_peers(&pt, peer_tag, (int)world, "ep_dispatch")) return s;
  for (int i = 0; i < (int)world; ++i)
    if (reinterpret_cast<uintptr_t>(pq.p[i]) & 15u) return fail(FNI8_ERR_ALIGN, "ep_dispatch: peer rows must be 16-byte aligned");
  const int64_t blocks = (max_rows + 7) / 8;
  launch_pdl(ep::dispatch_kernel, dim3((int)(blocks < 148 * 16 ? blocks : 148 * 16)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), q, scale, slot_of_row, offsets, (int)E, (int)(E / world), (int)top_k,
             (int)H, dst_base, (int)rank, pq, ps, pt, cap_rows);
  FNI8_CHECK_LAUNCH("ep_dispatch");
  return FNI8_OK;
}

extern "C" int fni8_ep_return(const void* y, int dtype, const int32_t* n_recv, int64_t cap_rows, const int32_t* tag,
                              int64_t H, int64_t world, void* const* peer_back, int64_t back_rows, void* stream) {
  if (world < 1 || world > ep::kMaxPeers) return fail(FNI8_ERR_INVALID, "ep_return: 1 <= world <= %d", ep::kMaxPeers);
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "ep_return: dtype");
  if (H <= 0 || H % 8 != 0) return fail(FNI8_ERR_UNSUPPORTED, "ep_return: H must be a multiple of 8");
  if (cap_rows < 0 || back_rows < 0) return fail(FNI8_ERR_INVALID, "ep_return: bad sizes");
  if (cap_rows == 0) return FNI8_OK;
  if (!y || !n_recv || !tag || !peer_back) return fail(FNI8_ERR_INVALID, "ep_return: null pointer");
  if (reinterpret_cast<uintptr_t>(y) & 15u) return fail(FNI8_ERR_ALIGN, "ep_return: rows must be 16-byte aligned");
  ep::Peers pb;
  if (int s = load_peers(&pb, peer_back, (int)world, "ep_return")) return s;
  for (int i = 0; i < (int)world; ++i)
    if (reinterpret_cast<uintptr_t>(pb.p[i]) & 15u) return fail(FNI8_ERR_ALIGN, "ep_return: peer rows must be 16-byte aligned");
  const int64_t blocks = (cap_rows + 7) / 8;
  const dim3 grid((int)(blocks < 148 * 16 ? blocks : 148 * 16));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FNI8_F16)
    launch_pdl(ep::return_kernel<__half>, grid, dim3(256), 0, st, static_cast<const __half*>(y), n_recv, cap_rows, tag,
               (int)H, pb, (int)world, back_rows);
  else
    launch_pdl(ep::return_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, static_cast<const __nv_bfloat16*>(y), n_recv,
               cap_rows, tag, (int)H, pb, (int)world, back_rows);
  FNI8_CHECK_LAUNCH("ep_return");
  return FNI8_OK;
}
