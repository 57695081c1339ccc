// Routed-expert block of SparseMoE (fni8serve/models/moe.py:62-113) on the device:
//
//   route    one warp per token: softmax / sigmoid scores, optional group-limited
//            selection, top-k by warp arg-max rounds, renormalisation, scaling
//   plan     stable counting sort of the T*k (token, slot) pairs by expert in three
//            short kernels (per-chunk histograms, one-CTA column scan, per-chunk ranks
//            with __match_any_sync): row_of_slot / slot_of_row, deterministic order, and
//            the segment tables of the expert GEMMs
//   quant    each token quantised once, its int8 row written to the expert-grouped rows
//            of its slots (quant.cu, fni8_moe_quantize_scatter_i8)
//   GEMMs    the grouped tcgen05 tile GEMM (gemm_tile.cu): gate_up with SiLU*up in its
//            epilogue, the product quantised per row, then down; one segment per expert
//   combine  out[t] = sum_j w[t,j] * y[row_of_slot[t*k+j]] in fp32, one rounding
//
// Nothing here waits on another CTA, so there is no watchdog word in this file.
#include "fni8_common.cuh"
#include "gemm_internal.h"

namespace fni8b {
namespace moe {

constexpr int kMaxE = 1024;
constexpr int kMaxK = 32;
constexpr int kChunk = 1024;  // slots per plan CTA

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// warp-wide arg-max: larger value wins, ties go to the lower index
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// VPL = experts per lane (E <= 32 * VPL).
template <int VPL>
__global__ void route_kernel(const float* __restrict__ logits, int T, int E, int k, int scoring,
                             const float* __restrict__ sel_bias, int n_groups, int topk_group, int norm_topk,
                             float scaling, int wdtype, int32_t* __restrict__ topi, float* __restrict__ topw) {
  pdl_launch_dependents();
  pdl_wait();  // the logits come from the previous kernel
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* lr = logits + static_cast<int64_t>(t) * E;
  const float NEG = -INFINITY;
  float sc[VPL], sel[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    sc[i] = e < E ? lr[e] : NEG;
  }
  if (scoring == FNI8_SCORE_SOFTMAX) {
    float mx = NEG;
#pragma unroll
    for (int i = 0; i < VPL; ++i) mx = fmaxf(mx, sc[i]);
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      sc[i] = e < E ? expf(__fadd_rn(sc[i], -mx)) : 0.0f;
      sum = __fadd_rn(sum, sc[i]);
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      sc[i] = __fdiv_rn(sc[i], sum);
      sel[i] = (lane + 32 * i) < E ? sc[i] : NEG;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      sc[i] = e < E ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-sc[i]))) : 0.0f;
      sel[i] = e < E ? (sel_bias ? __fadd_rn(sc[i], sel_bias[e]) : sc[i]) : NEG;
    }
  }
  if (n_groups > 0 && topk_group > 0) {
    // keep only the topk_group groups with the largest max score
    const int epg = E / n_groups;
    unsigned keep = 0;  // bitmask over groups (n_groups <= 32)
    for (int r = 0; r < topk_group; ++r) {
      float best = NEG;
      int bg = 0x7fffffff;
      for (int g = 0; g < n_groups; ++g) {
        if (keep & (1u << g)) continue;
        float gm = NEG;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          const int e = lane + 32 * i;
          if (e < E && e / epg == g) gm = fmaxf(gm, sel[i]);
        }
        gm = warp_max(gm);
        if (gm > best) {
          best = gm;
          bg = g;
        }
      }
      if (bg != 0x7fffffff) keep |= 1u << bg;
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(keep & (1u << (e / epg)))) sel[i] = NEG;
    }
  }
  float my_w = 0.0f;
  int my_i = 0;
  float wsum = 0.0f;
  for (int j = 0; j < k; ++j) {
    float v = NEG;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (sel[i] > v || (sel[i] == v && e < idx))) {
        v = sel[i];
        idx = e;
      }
    }
    warp_argmax(v, idx);
    float w = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (lane + 32 * i == idx) {
        w = sc[i];
        sel[i] = NEG;  // taken
        // a -inf entry can only be re-picked if everything left is -inf; mark it below E
      }
    }
    w = __shfl_sync(0xffffffffu, w, idx & 31);
    if (lane == j) {  // slot j stays in lane j (k <= 32)
      my_w = w;
      my_i = idx;
    }
    wsum = __fadd_rn(wsum, w);  // in slot order, as the reference's sum over k
  }
  if (lane < k) {
    const float denom = fmaxf(wsum, 1e-9f);
    float w = norm_topk ? __fdiv_rn(my_w, denom) : my_w;
    w = __fmul_rn(w, scaling);
    if (wdtype == FNI8_F16) w = __half2float(__float2half_rn(w));
    else if (wdtype == FNI8_BF16) w = __bfloat162float(__float2bfloat16_rn(w));
    topi[static_cast<int64_t>(t) * k + lane] = my_i;
    topw[static_cast<int64_t>(t) * k + lane] = w;
  }
}

// ---------------------------------------------------------------- plan
// Every kernel of this file is launched with programmatic stream serialization: it lets
// the next kernel launch at once and waits for the previous one before touching global
// memory (so the launch latency, not the data, is what overlaps).
__global__ void plan_hist(const int32_t* __restrict__ topi, int64_t n, int E, int32_t* __restrict__ hist) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int h[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x;
  if (i < n) {
    const int e = topi[i];
    if (e >= 0 && e < E) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[static_cast<int64_t>(blockIdx.x) * E + e] = h[e];
}

// One CTA: counts, offsets and each chunk's starting row per expert (in place of hist).
// Each thread owns an expert column; its chunk counts are read 32 at a time before any of
// them is rewritten (a load issued after a store it might alias waits for that store).
constexpr int kScanThreads = 256;
// Optional `tables` [E]: the segment -> expert table (e) of a grouped launch over all experts.
__global__ void __launch_bounds__(kScanThreads) plan_scan(int32_t* __restrict__ hist, int n_chunks, int E,
                                                          int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                          int32_t* __restrict__ tables) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int tot[kMaxE];
  __shared__ int base[kMaxE];
  __shared__ int warp_tot[kScanThreads / 32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c0 = 0; c0 < n_chunks; c0 += 32) {
      const int nc = n_chunks - c0 < 32 ? n_chunks - c0 : 32;
      int v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = j < nc ? hist[static_cast<int64_t>(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < nc) {
          hist[static_cast<int64_t>(c0 + j) * E + e] = run;
          run += v[j];
        }
      }
    }
    tot[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  // exclusive scan of the expert totals, kScanThreads experts at a time (warp shuffles)
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += kScanThreads) {
      const int e = e0 + threadIdx.x;
      const int v = e < E ? tot[e] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) warp_tot[warp] = x;
      __syncthreads();
      int before = 0, all = 0;
#pragma unroll
      for (int w = 0; w < kScanThreads / 32; ++w) {
        before += w < warp ? warp_tot[w] : 0;
        all += warp_tot[w];
      }
      if (e < E) {
        const int off = carry + before + x - v;
        base[e] = off;
        offsets[e] = off;
        if (tables != nullptr) tables[e] = e;  // segment s -> expert s of a grouped launch
      }
      carry += all;
      __syncthreads();  // warp_tot is rewritten by the next round
    }
    if (threadIdx.x == 0) offsets[E] = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int b = base[e];
    for (int c0 = 0; c0 < n_chunks; c0 += 32) {
      const int nc = n_chunks - c0 < 32 ? n_chunks - c0 : 32;
      int v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = j < nc ? hist[static_cast<int64_t>(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nc) hist[static_cast<int64_t>(c0 + j) * E + e] = v[j] + b;
    }
  }
}

__global__ void plan_scatter(const int32_t* __restrict__ topi, int64_t n, int E, const int32_t* __restrict__ base,
                             int32_t* __restrict__ row_of_slot, int32_t* __restrict__ slot_of_row) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ int wc[];  // [32 warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x;
  int e = -1;
  if (i < n) e = topi[i];
  const bool ok = (i < n) && e >= 0 && e < E;
  const int key = ok ? e : -1 - lane;  // unique keys for lanes that take part in nothing
  const unsigned m = __match_any_sync(0xffffffffu, key);
  const int rank = __popc(m & ((1u << lane) - 1u));
  if (ok && rank == 0) wc[warp * E + e] = __popc(m);
  __syncthreads();
  if (ok) {
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wc[w * E + e];
    const int pos = base[static_cast<int64_t>(blockIdx.x) * E + e] + before + rank;
    row_of_slot[i] = pos;
    slot_of_row[pos] = static_cast<int32_t>(i);
  } else if (i < n) {
    row_of_slot[i] = -1;
  }
}

// ---------------------------------------------------------------- gather / combine
// n_rows_dev (optional): the number of valid rows lives on the device (offsets[E]).
__global__ void gather_rows(const int8_t* __restrict__ q, const float* __restrict__ scale,
                            const int32_t* __restrict__ slot_of_row, int64_t R, const int32_t* __restrict__ n_rows_dev,
                            int K, int k, int8_t* __restrict__ q_out, float* __restrict__ s_out) {
  pdl_launch_dependents();
  pdl_wait();
  if (n_rows_dev != nullptr) {
    const int64_t n = *n_rows_dev;
    R = n < R ? n : R;
  }
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5); r < R;
       r += static_cast<int64_t>(gridDim.x) * warps) {
    const int64_t t = slot_of_row[r] / k;
    const uint4* src = reinterpret_cast<const uint4*>(q + t * K);
    uint4* dst = reinterpret_cast<uint4*>(q_out + r * K);
    for (int c = lane; c < K / 16; c += 32) dst[c] = __ldg(src + c);
    if (lane == 0) s_out[r] = __ldg(scale + t);
  }
}

template <typename T>
__global__ void combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ row_of_slot,
                               const float* __restrict__ topw, int64_t Tn, int k, int H, T* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  // one CTA per token; each thread owns 8 consecutive columns
  for (int64_t t = blockIdx.x; t < Tn; t += gridDim.x) {
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < k; ++j) {
        const int r = row_of_slot[t * k + j];
        if (r < 0) continue;
        const float w = topw[t * k + j];
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(r) * H) + c);
        const T* v = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(w, to_f32<T>(v[e])));
      }
      uint4 o;
      T* oo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) oo[e] = from_f32<T>(acc[e]);
      reinterpret_cast<uint4*>(out + t * H)[c] = o;
    }
  }
}

// out[i] = map[ids[i]] for ids in [0, E), else ids[i] (the plan drops those).
__global__ void map_ids_kernel(const int32_t* __restrict__ ids, int64_t n, const int32_t* __restrict__ map, int E,
                               int32_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = ids[i];
    out[i] = (v >= 0 && v < E) ? __ldg(map + v) : v;
  }
}

}  // namespace moe
}  // namespace fni8b

using namespace fni8b;
using namespace fni8h;

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

extern "C" int fni8_moe_route(const float* logits, int64_t T, int64_t E, int64_t top_k, int scoring,
                              const float* sel_bias, int64_t n_groups, int64_t topk_group, int norm_topk,
                              float scaling, int weight_dtype, int32_t* topi, float* topw, void* stream) {
  if (T < 0 || E <= 0 || E > moe::kMaxE) return fail(FNI8_ERR_INVALID, "route: need 0 < E <= %d", moe::kMaxE);
  if (top_k <= 0 || top_k > moe::kMaxK || top_k > E) return fail(FNI8_ERR_INVALID, "route: bad top_k %lld", (long long)top_k);
  if (scoring != FNI8_SCORE_SOFTMAX && scoring != FNI8_SCORE_SIGMOID) return fail(FNI8_ERR_INVALID, "route: scoring");
  if (n_groups < 0 || n_groups > 32 || (n_groups > 0 && (E % n_groups != 0 || topk_group <= 0 || topk_group > n_groups)))
    return fail(FNI8_ERR_INVALID, "route: bad expert grouping");
  if (weight_dtype != FNI8_F16 && weight_dtype != FNI8_BF16 && weight_dtype != FNI8_F32)
    return fail(FNI8_ERR_INVALID, "route: weight_dtype");
  if (T == 0) return FNI8_OK;
  if (logits == nullptr || topi == nullptr || topw == nullptr) return fail(FNI8_ERR_INVALID, "route: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int threads = 256, per = threads / 32;
  const int grid = (int)((T + per - 1) / per);
  const int vpl = (int)((E + 31) / 32);
#define FNI8_ROUTE(V)                                                                                          \
  launch_pdl(moe::route_kernel<V>, dim3(grid), dim3(threads), 0, st, logits, (int)T, (int)E, (int)top_k, scoring, \
             sel_bias, (int)n_groups, (int)topk_group, norm_topk, scaling, weight_dtype, topi, topw)
  if (vpl <= 1) FNI8_ROUTE(1);
  else if (vpl <= 2) FNI8_ROUTE(2);
  else if (vpl <= 4) FNI8_ROUTE(4);
  else if (vpl <= 8) FNI8_ROUTE(8);
  else if (vpl <= 16) FNI8_ROUTE(16);
  else FNI8_ROUTE(32);
#undef FNI8_ROUTE
  FNI8_CHECK_LAUNCH("moe_route");
  return FNI8_OK;
}

extern "C" size_t fni8_moe_plan_workspace_bytes(int64_t n_slots, int64_t E) {
  const int64_t chunks = (n_slots + moe::kChunk - 1) / moe::kChunk;
  return align256(static_cast<size_t>(chunks > 0 ? chunks : 1) * E * 4);
}

// fni8_moe_plan, optionally also writing the segment tables of the expert GEMMs (4 x E
// ints, laid out as plan_scan documents) from its scan kernel.
static int moe_plan(const int32_t* topi, int64_t n_slots, int64_t E, int32_t* counts, int32_t* offsets,
                    int32_t* row_of_slot, int32_t* slot_of_row, void* workspace, size_t workspace_bytes,
                    int32_t* tables, void* stream) {
  if (n_slots < 0 || n_slots >= (1LL << 31) || E <= 0 || E > moe::kMaxE)
    return fail(FNI8_ERR_INVALID, "plan: bad sizes");
  if (counts == nullptr || offsets == nullptr) return fail(FNI8_ERR_INVALID, "plan: null counts/offsets");
  if (n_slots > 0 && (topi == nullptr || row_of_slot == nullptr || slot_of_row == nullptr))
    return fail(FNI8_ERR_INVALID, "plan: null pointer");
  const size_t need = fni8_moe_plan_workspace_bytes(n_slots, E);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(FNI8_ERR_WORKSPACE, "plan needs %zu workspace bytes", need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (int)((n_slots + moe::kChunk - 1) / moe::kChunk);
  int32_t* hist = static_cast<int32_t*>(workspace);
  if (chunks > 0) launch_pdl(moe::plan_hist, dim3(chunks), dim3(moe::kChunk), 0, st, topi, n_slots, (int)E, hist);
  launch_pdl(moe::plan_scan, dim3(1), dim3(moe::kScanThreads), 0, st, hist, chunks, (int)E, counts, offsets, tables);
  if (chunks > 0) {
    const size_t smem = 32 * E * sizeof(int);
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(moe::plan_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "plan_scatter smem");
    }
    launch_pdl(moe::plan_scatter, dim3(chunks), dim3(moe::kChunk), smem, st, topi, n_slots, (int)E,
               static_cast<const int32_t*>(hist), row_of_slot, slot_of_row);
  }
  FNI8_CHECK_LAUNCH("moe_plan");
  return FNI8_OK;
}

extern "C" int fni8_moe_plan(const int32_t* topi, int64_t n_slots, int64_t E, int32_t* counts, int32_t* offsets,
                             int32_t* row_of_slot, int32_t* slot_of_row, void* workspace, size_t workspace_bytes,
                             void* stream) {
  return moe_plan(topi, n_slots, E, counts, offsets, row_of_slot, slot_of_row, workspace, workspace_bytes, nullptr,
                  stream);
}

extern "C" int fni8_moe_map_ids(const int32_t* ids, int64_t n, const int32_t* map, int64_t E, int32_t* out,
                                void* stream) {
  if (n < 0 || E <= 0) return fail(FNI8_ERR_INVALID, "map_ids: bad sizes");
  if (n == 0) return FNI8_OK;
  if (!ids || !map || !out) return fail(FNI8_ERR_INVALID, "map_ids: null pointer");
  const int64_t blocks = (n + 255) / 256;
  launch_pdl(moe::map_ids_kernel, dim3((int)(blocks < 148 * 4 ? blocks : 148 * 4)), dim3(256), 0,
             static_cast<cudaStream_t>(stream), ids, n, map, (int)E, out);
  FNI8_CHECK_LAUNCH("moe_map_ids");
  return FNI8_OK;
}

extern "C" int fni8_moe_gather_rows_i8(const int8_t* q, const float* scale, const int32_t* slot_of_row, int64_t R,
                                       int64_t K, int64_t top_k, int8_t* q_out, float* scale_out, void* stream) {
  if (R < 0 || K <= 0 || top_k <= 0) return fail(FNI8_ERR_INVALID, "gather: bad sizes");
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "gather: K must be a multiple of 16");
  if (R == 0) return FNI8_OK;
  if (!q || !scale || !slot_of_row || !q_out || !scale_out) return fail(FNI8_ERR_INVALID, "gather: null pointer");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(q_out)) & 15u)
    return fail(FNI8_ERR_ALIGN, "gather: rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t blocks = (R + 7) / 8;
  launch_pdl(moe::gather_rows, dim3((int)(blocks < 148 * 16 ? blocks : 148 * 16)), dim3(256), 0, st, q, scale,
             slot_of_row, R, static_cast<const int32_t*>(nullptr), (int)K, (int)top_k, q_out, scale_out);
  FNI8_CHECK_LAUNCH("moe_gather_rows_i8");
  return FNI8_OK;
}

extern "C" int fni8_grouped_gemm_w8a8(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w,
                                      const float* w_scale, int64_t E, int64_t N, int64_t K, const int32_t* seg_expert,
                                      const int32_t* seg_off, const int32_t* seg_cnt, int64_t S, void* out,
                                      int out_dtype, void* stream) {
  if (R < 0 || E <= 0 || N <= 0 || K <= 0 || S < 0) return fail(FNI8_ERR_INVALID, "grouped: bad sizes");
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "grouped: K must be a multiple of 16");
  if (R >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) return fail(FNI8_ERR_UNSUPPORTED, "grouped: too large");
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16 && out_dtype != FNI8_I32)
    return fail(FNI8_ERR_INVALID, "grouped: out_dtype");
  if (R == 0 || S == 0) return FNI8_OK;
  if (!a || !w || !out || !seg_expert || !seg_off || !seg_cnt || (out_dtype != FNI8_I32 && (!a_scale || !w_scale)))
    return fail(FNI8_ERR_INVALID, "grouped: null pointer");
  const int mode = out_dtype == FNI8_F16 ? 0 : (out_dtype == FNI8_BF16 ? 1 : 2);
  const int bn = (N % 256 == 0 || N > 1024) ? 256 : 128;
  return tile_gemm_grouped(a, a_scale, R, w, w_scale, E, N, K, seg_expert, seg_off, seg_cnt, S, out, mode, bn,
                           grouped_pair_enabled(),
                           static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_grouped_gemm_w8a8_act(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w_gu,
                                          const float* s_gu, int64_t E, int64_t I, int64_t K, const int32_t* seg_expert,
                                          const int32_t* seg_off, const int32_t* seg_cnt, int64_t S, int act, void* out,
                                          int out_dtype, void* stream) {
  if (R < 0 || E <= 0 || I <= 0 || K <= 0 || S < 0) return fail(FNI8_ERR_INVALID, "grouped act: bad sizes");
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "grouped act: K must be a multiple of 16");
  if (R >= (1LL << 31) || 2 * I >= (1LL << 31) || K >= (1LL << 31))
    return fail(FNI8_ERR_UNSUPPORTED, "grouped act: too large");
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "grouped act: out_dtype");
  if (R == 0 || S == 0) return FNI8_OK;
  if (!a || !a_scale || !w_gu || !s_gu || !out || !seg_expert || !seg_off || !seg_cnt)
    return fail(FNI8_ERR_INVALID, "grouped act: null pointer");
  return tile_gemm_act(a, a_scale, R, w_gu, s_gu, E, I, K, seg_expert, seg_off, seg_cnt, S, act, out,
                       out_dtype == FNI8_F16 ? 0 : 1, grouped_pair_enabled(), static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_grouped_gemm_w8a8_scatter(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w,
                                              const float* w_scale, int64_t E, int64_t N, int64_t K,
                                              const int32_t* seg_expert, const int32_t* seg_off,
                                              const int32_t* seg_cnt, int64_t S, const int32_t* row_tag,
                                              void* const* peer_out, int64_t world, int64_t peer_rows, int out_dtype,
                                              void* stream) {
  if (R < 0 || E <= 0 || N <= 0 || K <= 0 || S < 0 || peer_rows < 0) return fail(FNI8_ERR_INVALID, "scatter: bad sizes");
  if (world < 1 || world > 8) return fail(FNI8_ERR_INVALID, "scatter: 1 <= world <= 8");
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "scatter: K must be a multiple of 16");
  if (N % 64 != 0) return fail(FNI8_ERR_UNSUPPORTED, "scatter: N must be a multiple of 64");
  if (R >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) return fail(FNI8_ERR_UNSUPPORTED, "scatter: too large");
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "scatter: out_dtype F16 or BF16");
  if (R == 0 || S == 0) return FNI8_OK;
  if (!a || !a_scale || !w || !w_scale || !seg_expert || !seg_off || !seg_cnt || !row_tag || !peer_out)
    return fail(FNI8_ERR_INVALID, "scatter: null pointer");
  for (int64_t i = 0; i < world; ++i) {
    if (peer_out[i] == nullptr) return fail(FNI8_ERR_INVALID, "scatter: null peer buffer %lld", (long long)i);
    if (reinterpret_cast<uintptr_t>(peer_out[i]) & 15u)
      return fail(FNI8_ERR_ALIGN, "scatter: peer buffer %lld must be 16-byte aligned", (long long)i);
  }
  const int bn = (N % 256 == 0 || N > 1024) ? 256 : 128;
  return tile_gemm_grouped(a, a_scale, R, w, w_scale, E, N, K, seg_expert, seg_off, seg_cnt, S, nullptr,
                           out_dtype == FNI8_F16 ? 0 : 1, bn, grouped_pair_enabled(), static_cast<cudaStream_t>(stream),
                           row_tag, peer_out, (int)world, peer_rows);
}

extern "C" int fni8_moe_combine(const void* y, int dtype, const int32_t* row_of_slot, const float* topw, int64_t T,
                                int64_t top_k, int64_t H, void* out, void* stream) {
  if (T < 0 || top_k <= 0 || H <= 0) return fail(FNI8_ERR_INVALID, "combine: bad sizes");
  if (H % 8 != 0) return fail(FNI8_ERR_UNSUPPORTED, "combine: H must be a multiple of 8");
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "combine: dtype");
  if (T == 0) return FNI8_OK;
  if (!y || !row_of_slot || !topw || !out) return fail(FNI8_ERR_INVALID, "combine: null pointer");
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(FNI8_ERR_ALIGN, "combine: 16-byte alignment");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = (int)(T < 148 * 8 ? T : 148 * 8);
  const int threads = (int)((H / 8) < 256 ? ((H / 8 + 31) / 32) * 32 : 256);
  if (dtype == FNI8_F16)
    launch_pdl(moe::combine_kernel<__half>, dim3(grid), dim3(threads), 0, st, static_cast<const __half*>(y),
               row_of_slot, topw, T, (int)top_k, (int)H, static_cast<__half*>(out));
  else
    launch_pdl(moe::combine_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, st,
               static_cast<const __nv_bfloat16*>(y), row_of_slot, topw, T, (int)top_k, (int)H,
               static_cast<__nv_bfloat16*>(out));
  FNI8_CHECK_LAUNCH("moe_combine");
  return FNI8_OK;
}

// Workspace layout of fni8_moe_experts_w8a8 (each piece 256-byte aligned).
struct MoeLayout {
  size_t plan, counts, offsets, tables, ros, sor, aq, as, h, hq, hs, y, total;
};
static MoeLayout moe_layout(int64_t T, int64_t H, int64_t k, int64_t E, int64_t I) {
  MoeLayout L;
  const size_t R = static_cast<size_t>(T) * k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.plan = take(fni8_moe_plan_workspace_bytes(static_cast<int64_t>(R), E));
  L.counts = take(static_cast<size_t>(E) * 4);
  L.offsets = take(static_cast<size_t>(E + 1) * 4);
  L.tables = take(static_cast<size_t>(E) * 4);
  L.ros = take(R * 4);
  L.sor = take(R * 4);
  L.aq = take(R * H);
  L.as = take(R * 4);
  L.h = take(R * 2 * I * 2);
  L.hq = take(R * I);
  L.hs = take(R * 4);
  L.y = take(R * H * 2);
  L.total = off;
  return L;
}

extern "C" size_t fni8_moe_experts_workspace_bytes(int64_t T, int64_t H, int64_t top_k, int64_t E, int64_t I) {
  if (T <= 0 || H <= 0 || top_k <= 0 || E <= 0 || I <= 0) return 0;
  return moe_layout(T, H, top_k, E, I).total;
}

extern "C" int fni8_moe_experts_w8a8(const void* x, int dtype, int64_t T, int64_t H, const int32_t* topi,
                                     const float* topw, int64_t top_k, const int8_t* w_gu, const float* s_gu,
                                     const int8_t* w_dn, const float* s_dn, int64_t E, int64_t I, int act, void* out,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "moe: dtype");
  if (T < 0 || H <= 0 || top_k <= 0 || E <= 0 || I <= 0) return fail(FNI8_ERR_INVALID, "moe: bad sizes");
  if (E > kTileMaxSeg) return fail(FNI8_ERR_UNSUPPORTED, "moe: at most %d experts", kTileMaxSeg);
  if (H % 16 != 0 || I % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "moe: H and I must be multiples of 16");
  if (T == 0) return FNI8_OK;
  if (!x || !topi || !topw || !w_gu || !s_gu || !w_dn || !s_dn || !out) return fail(FNI8_ERR_INVALID, "moe: null pointer");
  const MoeLayout L = moe_layout(T, H, top_k, E, I);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(FNI8_ERR_WORKSPACE, "moe needs %zu workspace bytes (got %zu)", L.total, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(FNI8_ERR_ALIGN, "moe: workspace must be 256-byte aligned");
  uint8_t* b = static_cast<uint8_t*>(workspace);
  int32_t* counts = reinterpret_cast<int32_t*>(b + L.counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(b + L.offsets);
  int32_t* tables = reinterpret_cast<int32_t*>(b + L.tables);
  int32_t* ros = reinterpret_cast<int32_t*>(b + L.ros);
  int32_t* sor = reinterpret_cast<int32_t*>(b + L.sor);
  int8_t* aq = reinterpret_cast<int8_t*>(b + L.aq);
  float* as = reinterpret_cast<float*>(b + L.as);
  void* h = b + L.h;
  int8_t* hq = reinterpret_cast<int8_t*>(b + L.hq);
  float* hs = reinterpret_cast<float*>(b + L.hs);
  void* y = b + L.y;
  const int64_t R = T * top_k;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // plan first (with the segment tables), then each token is quantised once and its int8
  // row written straight to the grouped rows of its slots (no [T, H] int8 copy, no gather)
  if (int s = moe_plan(topi, R, E, counts, offsets, ros, sor, b + L.plan, L.counts - L.plan, tables, stream))
    return s;
  if (int s = fni8_moe_quantize_scatter_i8(x, dtype, T, H, ros, top_k, aq, as, stream)) return s;
  // One segment per expert on single CTAs (measured on B200 at BASELINE config 3: CTA
  // pairs, for all rows or only for each expert's whole 256-row tiles, were slower).
  const int32_t* seg_e = tables;
  const int mode = dtype == FNI8_F16 ? 0 : 1;
  if (I % 128 == 0) {
    // gate_up with act_and_mul in its epilogue: the [R, I] product, then its int8 rows
    if (int s = tile_gemm_act(aq, as, R, w_gu, s_gu, E, I, H, seg_e, offsets, counts, E, act, h, mode,
                              grouped_pair_enabled(), st))
      return s;
    if (int s = fni8_quantize_rows_i8(h, dtype, R, I, hq, hs, stream)) return s;
  } else {
    if (int s = fni8_grouped_gemm_w8a8(aq, as, R, w_gu, s_gu, E, 2 * I, H, seg_e, offsets, counts, E, h, dtype, stream))
      return s;
    if (int s = fni8_act_and_mul_quant_i8(h, dtype, act, R, I, hq, hs, stream)) return s;
  }
  if (int s = fni8_grouped_gemm_w8a8(hq, hs, R, w_dn, s_dn, E, H, I, seg_e, offsets, counts, E, y, dtype, stream))
    return s;
  return fni8_moe_combine(y, dtype, ros, topw, T, top_k, H, out, stream);
}
