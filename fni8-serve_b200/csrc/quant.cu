// Row-wise producers of the W8A8 GEMM's A operand, all HBM-bound:
//   * per-token absmax int8 quantisation               (activation stage of fni8.linear)
//   * RMSNorm (+ residual add, + Gemma unit offset)    (fni8.rmsnorm)
//   * fused RMSNorm -> int8 quantisation               (one pass instead of two)
//   * act_and_mul (SiLU / tanh-GELU)                   (fni8.act_and_mul; act(gate) is
//     rounded to the storage dtype before the product, as the reference's own
//     F.silu(gate) * up does on fp16 tensors)
//   * fused act_and_mul -> int8 quantisation           (input of down_proj)
//
// One 128-thread CTA per row. Each thread keeps its 16-byte chunks of the row in
// registers (up to MAXC chunks of 8 elements), so a row is read from HBM once, reduced
// with warp shuffles + a 4-entry shared array, and written once. Rows whose K is not a
// multiple of 8 (or whose base is not 16-byte aligned) use a scalar two-pass kernel.
//
// Arithmetic is pinned so the int8 output is a pure function of the rounded input
// row: IEEE division and sqrt (__fdiv_rn, __fsqrt_rn), no contraction (__fmul_rn,
// __fadd_rn), round-half-even (rintf) — the same operations torch performs on CPU.
#include "fni8_common.cuh"

namespace fni8b {
namespace {

constexpr int kRowThreads = 128;

template <typename T>
struct Vec8;  // 8 elements in one 16-byte word
template <>
struct Vec8<__half> {
  __device__ static void unpack(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ static uint4 pack(const float (&f)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};
template <>
struct Vec8<__nv_bfloat16> {
  __device__ static void unpack(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ static uint4 pack(const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
};

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // protect `red` from the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kRowThreads / 32; ++w) r = fmaxf(r, red[w]);
  return r;
}
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kRowThreads / 32; ++w) r = __fadd_rn(r, red[w]);
  return r;
}

// scale = absmax / 127 is what the GEMM epilogue multiplies with; the codes are
// round_half_even(x * (127 / absmax)) — one reciprocal per row instead of a division per
// element (measured: the per-element IEEE division halved the quantiser's throughput).
__device__ __forceinline__ float quant_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
__device__ __forceinline__ float quant_inv(float amax) { return amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f; }
__device__ __forceinline__ int8_t quant_one(float v, float inv) {
  float q = rintf(__fmul_rn(v, inv));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(q));
}
__device__ __forceinline__ uint2 quant8(const float (&f)[8], float inv) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= (static_cast<uint32_t>(static_cast<uint8_t>(quant_one(f[i], inv)))) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= (static_cast<uint32_t>(static_cast<uint8_t>(quant_one(f[4 + i], inv)))) << (8 * i);
  return make_uint2(lo, hi);
}

// ---------------------------------------------------------------- vector kernels
// MODE 0: quantise rows of x.
template <typename T, int MAXC>
__global__ void __launch_bounds__(kRowThreads) quant_rows_vec(const T* __restrict__ x, int64_t M, int K,
                                                               int8_t* __restrict__ q, float* __restrict__ scale,
                                                               const int32_t* __restrict__ m_dev) {
  __shared__ float red[kRowThreads / 32];
  const int nch = K >> 3;
  pdl_launch_dependents();  // dependents may start now; they wait for our completion
  pdl_wait();
  if (m_dev != nullptr) {  // rows known only on the device: M is their upper bound
    const int64_t m = *m_dev;
    M = m < M ? m : M;
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    uint4 raw[MAXC];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        raw[i] = __ldg(xr + c);
        float f[8];
        Vec8<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
      }
    }
    amax = block_reduce_max(amax, red);
    const float s = quant_scale(amax), inv = quant_inv(amax);
    uint2* qr = reinterpret_cast<uint2*>(q + row * K);
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        float f[8];
        Vec8<T>::unpack(raw[i], f);
        qr[c] = quant8(f, inv);
      }
    }
    if (threadIdx.x == 0) scale[row] = s;
  }
}

// RMSNorm, optionally fused with quantisation. QUANT: emit q/scale. out may be null.
template <typename T, int MAXC, bool QUANT>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_vec(const T* __restrict__ x, const T* __restrict__ res,
                                                            const T* __restrict__ w, int64_t M, int K, float eps,
                                                            int unit_offset, T* __restrict__ out,
                                                            T* __restrict__ res_out, int8_t* __restrict__ q,
                                                            float* __restrict__ scale) {
  __shared__ float red[kRowThreads / 32];
  const int nch = K >> 3;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  pdl_launch_dependents();  // dependents may start now; they wait for our completion
  pdl_wait();
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    uint4 raw[MAXC];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        raw[i] = __ldg(xr + c);
        if (res != nullptr) {
          // x + residual in the storage dtype (one rounding), kept as the new residual
          const uint4 r = __ldg(reinterpret_cast<const uint4*>(res + row * K) + c);
          float a[8], b[8];
          Vec8<T>::unpack(raw[i], a);
          Vec8<T>::unpack(r, b);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] = __fadd_rn(a[j], b[j]);
          raw[i] = Vec8<T>::pack(a);
          reinterpret_cast<uint4*>(res_out + row * K)[c] = raw[i];
        }
        float f[8];
        Vec8<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(f[j], f[j]));
      }
    }
    ss = block_reduce_sum(ss, red);
    const float mean = __fdiv_rn(ss, static_cast<float>(K));
    const float rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        float f[8], g[8];
        Vec8<T>::unpack(raw[i], f);
        Vec8<T>::unpack(__ldg(wr + c), g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float gj = unit_offset ? __fadd_rn(1.0f, g[j]) : g[j];
          f[j] = round_trip<T>(__fmul_rn(__fmul_rn(f[j], rinv), gj));
          amax = fmaxf(amax, fabsf(f[j]));
        }
        raw[i] = Vec8<T>::pack(f);  // exact: f already holds T-representable values
        if (out != nullptr) reinterpret_cast<uint4*>(out + row * K)[c] = raw[i];
      }
    }
    if constexpr (QUANT) {
      amax = block_reduce_max(amax, red);
      const float s = quant_scale(amax), inv = quant_inv(amax);
      uint2* qr = reinterpret_cast<uint2*>(q + row * K);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        if (c < nch) {
          float f[8];
          Vec8<T>::unpack(raw[i], f);
          qr[c] = quant8(f, inv);
        }
      }
      if (threadIdx.x == 0) scale[row] = s;
    }
  }
}

// act(x[:, :I]) * x[:, I:], optionally quantised.
template <typename T, int MAXC, int ACT, bool QUANT>
__global__ void __launch_bounds__(kRowThreads) act_mul_vec(const T* __restrict__ x, int64_t M, int I,
                                                            T* __restrict__ out, int8_t* __restrict__ q,
                                                            float* __restrict__ scale, const int32_t* __restrict__ m_dev) {
  __shared__ float red[kRowThreads / 32];
  const int nch = I >> 3;
  pdl_launch_dependents();  // dependents may start now; they wait for our completion
  pdl_wait();
  if (m_dev != nullptr) {  // rows known only on the device: M is their upper bound
    const int64_t m = *m_dev;
    M = m < M ? m : M;
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* gr = reinterpret_cast<const uint4*>(x + row * 2 * static_cast<int64_t>(I));
    const uint4* ur = gr + nch;
    uint4 raw[MAXC];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        float g[8], u[8];
        Vec8<T>::unpack(__ldg(gr + c), g);
        Vec8<T>::unpack(__ldg(ur + c), u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          g[j] = round_trip<T>(__fmul_rn(round_trip<T>(act_fn<ACT>(g[j])), u[j]));
          amax = fmaxf(amax, fabsf(g[j]));
        }
        raw[i] = Vec8<T>::pack(g);
        if (!QUANT || out != nullptr) reinterpret_cast<uint4*>(out + row * I)[c] = raw[i];
      }
    }
    if constexpr (QUANT) {
      amax = block_reduce_max(amax, red);
      const float s = quant_scale(amax), inv = quant_inv(amax);
      uint2* qr = reinterpret_cast<uint2*>(q + row * I);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        if (c < nch) {
          float f[8];
          Vec8<T>::unpack(raw[i], f);
          qr[c] = quant8(f, inv);
        }
      }
      if (threadIdx.x == 0) scale[row] = s;
    }
  }
}

// ---------------------------------------------------------------- scalar kernels
// Any K, any alignment: two/three passes over the row from L2. Same arithmetic.
// OP 0: quant; 1: rmsnorm; 2: rmsnorm+quant; 3: act_mul; 4: act_mul+quant.
template <typename T, int OP, int ACT>
__global__ void __launch_bounds__(kRowThreads) row_scalar(const T* __restrict__ x, const T* __restrict__ res,
                                                           const T* __restrict__ w, int64_t M, int K, float eps,
                                                           int unit_offset, T* __restrict__ out,
                                                           T* __restrict__ res_out, int8_t* __restrict__ q,
                                                           float* __restrict__ scale) {
  __shared__ float red[kRowThreads / 32];
  constexpr bool NORM = (OP == 1 || OP == 2);
  constexpr bool ACTM = (OP == 3 || OP == 4);
  constexpr bool QUANT = (OP == 0 || OP == 2 || OP == 4);
  pdl_launch_dependents();  // dependents may start now; they wait for our completion
  pdl_wait();
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t in_ld = ACTM ? 2 * static_cast<int64_t>(K) : K;
    const T* xr = x + row * in_ld;
    auto value = [&](int k, float rinv) -> float {  // the rounded element that gets quantised
      if constexpr (NORM) {
        // with a residual, the first pass already stored x + residual in res_out (this
        // thread wrote index k itself), which also makes in-place residuals safe
        const float v = (res != nullptr) ? to_f32<T>(res_out[row * K + k]) : to_f32<T>(xr[k]);
        const float g = unit_offset ? __fadd_rn(1.0f, to_f32<T>(w[k])) : to_f32<T>(w[k]);
        return round_trip<T>(__fmul_rn(__fmul_rn(v, rinv), g));
      } else if constexpr (ACTM) {
        return round_trip<T>(__fmul_rn(round_trip<T>(act_fn<ACT>(to_f32<T>(xr[k]))), to_f32<T>(xr[K + k])));
      } else {
        return to_f32<T>(xr[k]);
      }
    };
    float rinv = 1.0f;
    if constexpr (NORM) {
      float ss = 0.0f;
      for (int k = threadIdx.x; k < K; k += kRowThreads) {
        float v = to_f32<T>(xr[k]);
        if (res != nullptr) {
          v = round_trip<T>(__fadd_rn(v, to_f32<T>(res[row * K + k])));
          res_out[row * K + k] = from_f32<T>(v);
        }
        ss = __fadd_rn(ss, __fmul_rn(v, v));
      }
      ss = block_reduce_sum(ss, red);
      rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
    }
    float amax = 0.0f;
    for (int k = threadIdx.x; k < K; k += kRowThreads) {
      const float v = value(k, rinv);
      amax = fmaxf(amax, fabsf(v));
      if (out != nullptr) out[row * K + k] = from_f32<T>(v);
    }
    if constexpr (QUANT) {
      amax = block_reduce_max(amax, red);
      const float s = quant_scale(amax), inv = quant_inv(amax);
      for (int k = threadIdx.x; k < K; k += kRowThreads) q[row * K + k] = quant_one(value(k, rinv), inv);
      if (threadIdx.x == 0) scale[row] = s;
    }
  }
}

// ---------------------------------------------------------------- warp-per-row kernels
// Rows of up to 32 * 8 * MW (<= 1024) elements: one warp per row, 8 rows per CTA, shuffle-only
// reductions (no block barriers), so many rows are in flight per SM. Same arithmetic as
// the CTA-per-row kernels above. OP: 0 quant, 1 rmsnorm, 2 rmsnorm+quant, 3 act_mul,
// 4 act_mul+quant.
constexpr int kWarpRows = 8;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename T, int OP, int ACT, int MW>
__global__ void __launch_bounds__(32 * kWarpRows) row_warp(const T* __restrict__ x, const T* __restrict__ res,
                                                            const T* __restrict__ w, int64_t M, int K, float eps,
                                                            int unit_offset, T* __restrict__ out,
                                                            T* __restrict__ res_out, int8_t* __restrict__ q,
                                                            float* __restrict__ scale, const int32_t* __restrict__ m_dev) {
  constexpr bool NORM = (OP == 1 || OP == 2);
  constexpr bool ACTM = (OP == 3 || OP == 4);
  constexpr bool QUANT = (OP == 0 || OP == 2 || OP == 4);
  pdl_launch_dependents();
  pdl_wait();
  if (m_dev != nullptr) {  // rows known only on the device: M is their upper bound
    const int64_t m = *m_dev;
    M = m < M ? m : M;
  }
  const int lane = threadIdx.x & 31;
  const int nch = K >> 3;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarpRows;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpRows + (threadIdx.x >> 5); row < M; row += stride) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * (ACTM ? 2 * static_cast<int64_t>(K) : K));
    uint4 raw[MW];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < MW; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        if constexpr (ACTM) {
          float g[8], u[8];
          Vec8<T>::unpack(__ldg(xr + c), g);
          Vec8<T>::unpack(__ldg(xr + nch + c), u);
#pragma unroll
          for (int j = 0; j < 8; ++j) g[j] = round_trip<T>(__fmul_rn(round_trip<T>(act_fn<ACT>(g[j])), u[j]));
          raw[i] = Vec8<T>::pack(g);
        } else if constexpr (NORM) {
          raw[i] = __ldg(xr + c);
          if (res != nullptr) {
            float a[8], b[8];
            Vec8<T>::unpack(raw[i], a);
            Vec8<T>::unpack(__ldg(reinterpret_cast<const uint4*>(res + row * K) + c), b);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = __fadd_rn(a[j], b[j]);
            raw[i] = Vec8<T>::pack(a);
            reinterpret_cast<uint4*>(res_out + row * K)[c] = raw[i];
          }
          float f[8];
          Vec8<T>::unpack(raw[i], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(f[j], f[j]));
        } else {
          raw[i] = __ldg(xr + c);
        }
      }
    }
    if constexpr (NORM) {
      ss = warp_sum_f(ss);
      const float rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
#pragma unroll
      for (int i = 0; i < MW; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          float f[8], g[8];
          Vec8<T>::unpack(raw[i], f);
          Vec8<T>::unpack(__ldg(reinterpret_cast<const uint4*>(w) + c), g);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float gj = unit_offset ? __fadd_rn(1.0f, g[j]) : g[j];
            f[j] = round_trip<T>(__fmul_rn(__fmul_rn(f[j], rinv), gj));
          }
          raw[i] = Vec8<T>::pack(f);
          if (out != nullptr) reinterpret_cast<uint4*>(out + row * K)[c] = raw[i];
        }
      }
    }
    if constexpr (ACTM) {  // the product itself (always without quantisation, optional with it)
      if (!QUANT || out != nullptr) {
#pragma unroll
        for (int i = 0; i < MW; ++i) {
          const int c = lane + 32 * i;
          if (c < nch) reinterpret_cast<uint4*>(out + row * K)[c] = raw[i];
        }
      }
    }
    if constexpr (QUANT) {
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < MW; ++i) {
        if (lane + 32 * i < nch) {
          float f[8];
          Vec8<T>::unpack(raw[i], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
        }
      }
      const float amax_w = warp_max_f(amax);
      const float s = quant_scale(amax_w), inv = quant_inv(amax_w);
      uint2* qr = reinterpret_cast<uint2*>(q + row * K);
#pragma unroll
      for (int i = 0; i < MW; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          float f[8];
          Vec8<T>::unpack(raw[i], f);
          qr[c] = quant8(f, inv);
        }
      }
      if (lane == 0) scale[row] = s;
    }
  }
}

// Launch the warp-per-row kernel for short rows (K <= 1024); returns false otherwise.
template <typename T, int OP, int ACT>
bool launch_row_warp(const T* x, const T* res, const T* w, int64_t M, int K, float eps, int uo, T* out, T* res_out,
                     int8_t* q, float* s, cudaStream_t st, const int32_t* m_dev = nullptr) {
  const int nch = K / 8;
  const int64_t ctas_needed = (M + kWarpRows - 1) / kWarpRows;
  const int grid = static_cast<int>(ctas_needed < 148LL * 8 ? ctas_needed : 148LL * 8);
  const dim3 blk(32 * kWarpRows);
  if (nch <= 32) fni8h::launch_pdl(row_warp<T, OP, ACT, 1>, dim3(grid), blk, 0, st, x, res, w, M, K, eps, uo, out, res_out, q, s, m_dev);
  else if (nch <= 64) fni8h::launch_pdl(row_warp<T, OP, ACT, 2>, dim3(grid), blk, 0, st, x, res, w, M, K, eps, uo, out, res_out, q, s, m_dev);
  else if (nch <= 128) fni8h::launch_pdl(row_warp<T, OP, ACT, 4>, dim3(grid), blk, 0, st, x, res, w, M, K, eps, uo, out, res_out, q, s, m_dev);
  else return false;  // longer rows: the CTA-per-row kernels spread a row over 4 warps (measured faster)
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int row_grid(int64_t M) {  // one row per CTA up to ~64 CTAs per SM (measured best)
  const int64_t cap = 148LL * 64LL;
  return static_cast<int>(M < cap ? M : cap);
}

template <typename T, int MAXC>
void launch_quant_vec(const void* x, int64_t M, int K, int8_t* q, float* s, cudaStream_t st, const int32_t* m_dev) {
  fni8h::launch_pdl(quant_rows_vec<T, MAXC>, dim3(row_grid(M)), dim3(kRowThreads), 0, st, static_cast<const T*>(x), M,
                    K, q, s, m_dev);
}

// m_dev (optional): the row count lives on the device, M is its upper bound (vector path
// only: the caller checks alignment first).
template <typename T>
int quant_dispatch(const void* x, int64_t M, int64_t K, int8_t* q, float* s, cudaStream_t st,
                   const int32_t* m_dev = nullptr) {
  const int64_t nch = K / 8;
  const bool vec = (K % 8 == 0) && aligned16(x) && aligned16(q) && nch <= 16 * kRowThreads;
  if (vec && launch_row_warp<T, 0, 0>(static_cast<const T*>(x), nullptr, nullptr, M, (int)K, 0.f, 0, nullptr, nullptr, q,
                                      s, st, m_dev)) {
    FNI8_CHECK_LAUNCH("quantize_rows_i8");
    return FNI8_OK;
  }
  if (vec) {
    if (nch <= 2 * kRowThreads) launch_quant_vec<T, 2>(x, M, (int)K, q, s, st, m_dev);
    else if (nch <= 4 * kRowThreads) launch_quant_vec<T, 4>(x, M, (int)K, q, s, st, m_dev);
    else if (nch <= 8 * kRowThreads) launch_quant_vec<T, 8>(x, M, (int)K, q, s, st, m_dev);
    else launch_quant_vec<T, 16>(x, M, (int)K, q, s, st, m_dev);
  } else {
    fni8h::launch_pdl(row_scalar<T, 0, 0>, dim3(row_grid(M)), dim3(kRowThreads), 0, st, static_cast<const T*>(x),
                      static_cast<const T*>(nullptr), static_cast<const T*>(nullptr), M, (int)K, 0.f, 0,
                      static_cast<T*>(nullptr), static_cast<T*>(nullptr), q, s);
  }
  FNI8_CHECK_LAUNCH("quantize_rows_i8");
  return FNI8_OK;
}

template <typename T, bool QUANT>
int norm_dispatch(const void* x, const void* res, const void* w, int64_t M, int64_t K, float eps, int uo, void* out,
                  void* res_out, int8_t* q, float* s, cudaStream_t st) {
  const int64_t nch = K / 8;
  const bool vec = (K % 8 == 0) && aligned16(x) && aligned16(w) && (out == nullptr || aligned16(out)) &&
                   (res == nullptr || (aligned16(res) && aligned16(res_out))) && (!QUANT || aligned16(q)) &&
                   nch <= 16 * kRowThreads;
  const T* xx = static_cast<const T*>(x);
  const T* rr = static_cast<const T*>(res);
  const T* ww = static_cast<const T*>(w);
  T* oo = static_cast<T*>(out);
  T* ro = static_cast<T*>(res_out);
  const int g = row_grid(M);
  if (vec && launch_row_warp<T, QUANT ? 2 : 1, 0>(xx, rr, ww, M, (int)K, eps, uo, oo, ro, q, s, st)) {
    FNI8_CHECK_LAUNCH(QUANT ? "rmsnorm_quant_i8" : "rmsnorm");
    return FNI8_OK;
  }
  if (vec) {
    if (nch <= 2 * kRowThreads)
      fni8h::launch_pdl(rmsnorm_vec<T, 2, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, rr, ww, M, (int)K, eps, uo, oo, ro, q, s);
    else if (nch <= 4 * kRowThreads)
      fni8h::launch_pdl(rmsnorm_vec<T, 4, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, rr, ww, M, (int)K, eps, uo, oo, ro, q, s);
    else if (nch <= 8 * kRowThreads)
      fni8h::launch_pdl(rmsnorm_vec<T, 8, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, rr, ww, M, (int)K, eps, uo, oo, ro, q, s);
    else
      fni8h::launch_pdl(rmsnorm_vec<T, 16, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, rr, ww, M, (int)K, eps, uo, oo, ro, q, s);
  } else {
    fni8h::launch_pdl(row_scalar<T, QUANT ? 2 : 1, 0>, dim3(g), dim3(kRowThreads), 0, st, xx, rr, ww, M, (int)K, eps, uo,
                      oo, ro, q, s);
  }
  FNI8_CHECK_LAUNCH(QUANT ? "rmsnorm_quant_i8" : "rmsnorm");
  return FNI8_OK;
}

template <typename T, int ACT, bool QUANT>
int act_dispatch(const void* x, int64_t M, int64_t I, void* out, int8_t* q, float* s, cudaStream_t st,
                 const int32_t* m_dev = nullptr) {
  const int64_t nch = I / 8;
  // QUANT with `out`: both the product and its int8 rows are written
  const bool vec = (I % 8 == 0) && aligned16(x) && (!QUANT || aligned16(q)) && (out == nullptr || aligned16(out)) &&
                   nch <= 16 * kRowThreads;
  const T* xx = static_cast<const T*>(x);
  T* oo = static_cast<T*>(out);
  const int g = row_grid(M);
  if (vec && launch_row_warp<T, QUANT ? 4 : 3, ACT>(xx, nullptr, nullptr, M, (int)I, 0.f, 0, oo, nullptr, q, s, st,
                                                    m_dev)) {
    FNI8_CHECK_LAUNCH(QUANT ? "act_and_mul_quant_i8" : "act_and_mul");
    return FNI8_OK;
  }
  if (vec) {
    if (nch <= 2 * kRowThreads) fni8h::launch_pdl(act_mul_vec<T, 2, ACT, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, M, (int)I, oo, q, s, m_dev);
    else if (nch <= 4 * kRowThreads)
      fni8h::launch_pdl(act_mul_vec<T, 4, ACT, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, M, (int)I, oo, q, s, m_dev);
    else if (nch <= 8 * kRowThreads)
      fni8h::launch_pdl(act_mul_vec<T, 8, ACT, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, M, (int)I, oo, q, s, m_dev);
    else
      fni8h::launch_pdl(act_mul_vec<T, 16, ACT, QUANT>, dim3(g), dim3(kRowThreads), 0, st, xx, M, (int)I, oo, q, s, m_dev);
  } else {
    fni8h::launch_pdl(row_scalar<T, QUANT ? 4 : 3, ACT>, dim3(g), dim3(kRowThreads), 0, st, xx,
                      static_cast<const T*>(nullptr), static_cast<const T*>(nullptr), M, (int)I, 0.f, 0, oo,
                      static_cast<T*>(nullptr), q, s);
  }
  FNI8_CHECK_LAUNCH(QUANT ? "act_and_mul_quant_i8" : "act_and_mul");
  return FNI8_OK;
}

int check_rows(const void* x, int dtype, int64_t M, int64_t K) {
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fni8h::fail(FNI8_ERR_INVALID, "dtype %d: expected F16 or BF16", dtype);
  if (M < 0 || K <= 0) return fni8h::fail(FNI8_ERR_INVALID, "bad shape M=%lld K=%lld", (long long)M, (long long)K);
  if (K > (1 << 30)) return fni8h::fail(FNI8_ERR_UNSUPPORTED, "K=%lld too large", (long long)K);
  if (M > 0 && x == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null input");
  if ((reinterpret_cast<uintptr_t>(x) & 1u) != 0) return fni8h::fail(FNI8_ERR_ALIGN, "input not 2-byte aligned");
  return FNI8_OK;
}

// Per-token quantisation whose int8 row goes straight to the expert-grouped rows of the
// token's routed slots: row row_of_slot[t * k + j] of q_out (and its scale) for every slot j
// that the plan placed (r >= 0). One CTA per token; the codes are those of quant_rows_vec.
template <typename T, int MAXC>
__global__ void __launch_bounds__(kRowThreads) quant_scatter_vec(const T* __restrict__ x, int64_t M, int K, int k,
                                                                  const int32_t* __restrict__ row_of_slot,
                                                                  int8_t* __restrict__ q_out,
                                                                  float* __restrict__ s_out) {
  __shared__ float red[kRowThreads / 32];
  const int nch = K >> 3;
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    uint4 raw[MAXC];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        raw[i] = __ldg(xr + c);
        float f[8];
        Vec8<T>::unpack(raw[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
      }
    }
    amax = block_reduce_max(amax, red);
    const float s = quant_scale(amax), inv = quant_inv(amax);
    uint2 qv[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nch) {
        float f[8];
        Vec8<T>::unpack(raw[i], f);
        qv[i] = quant8(f, inv);
      }
    }
    for (int j = 0; j < k; ++j) {
      const int32_t r = __ldg(row_of_slot + row * k + j);
      if (r < 0) continue;
      uint2* qr = reinterpret_cast<uint2*>(q_out + static_cast<int64_t>(r) * K);
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        if (c < nch) qr[c] = qv[i];
      }
      if (threadIdx.x == 0) s_out[r] = s;
    }
  }
}

template <typename T>
int quant_scatter_dispatch(const void* x, int64_t M, int64_t K, int64_t k, const int32_t* row_of_slot, int8_t* q,
                           float* s, cudaStream_t st) {
  const int64_t nch = K / 8;
  const dim3 g(row_grid(M)), b(kRowThreads);
  const T* xt = static_cast<const T*>(x);
#define FNI8_QS(C) fni8h::launch_pdl(quant_scatter_vec<T, C>, g, b, 0, st, xt, M, (int)K, (int)k, row_of_slot, q, s)
  if (nch <= kRowThreads) FNI8_QS(1);
  else if (nch <= 2 * kRowThreads) FNI8_QS(2);
  else if (nch <= 4 * kRowThreads) FNI8_QS(4);
  else if (nch <= 8 * kRowThreads) FNI8_QS(8);
  else FNI8_QS(16);
#undef FNI8_QS
  FNI8_CHECK_LAUNCH("quantize_scatter");
  return FNI8_OK;
}

}  // namespace
}  // namespace fni8b

using namespace fni8b;

extern "C" int fni8_moe_quantize_scatter_i8(const void* x, int dtype, int64_t T, int64_t K, const int32_t* row_of_slot,
                                            int64_t top_k, int8_t* q_out, float* scale_out, void* stream) {
  if (int st = check_rows(x, dtype, T, K)) return st;
  if (top_k <= 0 || top_k > 64) return fni8h::fail(FNI8_ERR_INVALID, "quantize_scatter: bad top_k %lld", (long long)top_k);
  if (T == 0) return FNI8_OK;
  if (row_of_slot == nullptr || q_out == nullptr || scale_out == nullptr)
    return fni8h::fail(FNI8_ERR_INVALID, "quantize_scatter: null pointer");
  if (K % 8 != 0 || K / 8 > 16 * kRowThreads || !aligned16(x) || !aligned16(q_out))
    return fni8h::fail(FNI8_ERR_UNSUPPORTED, "quantize_scatter: K a multiple of 8 (<= 16384), 16-byte aligned rows");
  if (K % 16 != 0) return fni8h::fail(FNI8_ERR_UNSUPPORTED, "quantize_scatter: K a multiple of 16");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == FNI8_F16 ? quant_scatter_dispatch<__half>(x, T, K, top_k, row_of_slot, q_out, scale_out, s)
                           : quant_scatter_dispatch<__nv_bfloat16>(x, T, K, top_k, row_of_slot, q_out, scale_out, s);
}

extern "C" int fni8_quantize_rows_i8(const void* x, int dtype, int64_t M, int64_t K, int8_t* q, float* scale,
                                     void* stream) {
  if (int st = check_rows(x, dtype, M, K)) return st;
  if (M > 0 && (q == nullptr || scale == nullptr)) return fni8h::fail(FNI8_ERR_INVALID, "null output");
  if (M == 0) return FNI8_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == FNI8_F16 ? quant_dispatch<__half>(x, M, K, q, scale, s)
                           : quant_dispatch<__nv_bfloat16>(x, M, K, q, scale, s);
}

static int norm_common(const void* x, const void* residual, const void* weight, int dtype, int64_t M, int64_t K,
                       float eps, int unit_offset, void* out, void* residual_out, int8_t* q, float* scale,
                       void* stream, bool quant) {
  if (int st = check_rows(x, dtype, M, K)) return st;
  if (weight == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null weight");
  if (residual != nullptr && residual_out == nullptr)
    return fni8h::fail(FNI8_ERR_INVALID, "residual given without residual_out");
  if (!quant && out == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null output");
  if (quant && M > 0 && (q == nullptr || scale == nullptr)) return fni8h::fail(FNI8_ERR_INVALID, "null q/scale");
  if (!(eps >= 0.0f)) return fni8h::fail(FNI8_ERR_INVALID, "eps must be >= 0");
  if (M == 0) return FNI8_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FNI8_F16)
    return quant ? norm_dispatch<__half, true>(x, residual, weight, M, K, eps, unit_offset, out, residual_out, q,
                                               scale, s)
                 : norm_dispatch<__half, false>(x, residual, weight, M, K, eps, unit_offset, out, residual_out,
                                                nullptr, nullptr, s);
  return quant ? norm_dispatch<__nv_bfloat16, true>(x, residual, weight, M, K, eps, unit_offset, out, residual_out,
                                                    q, scale, s)
               : norm_dispatch<__nv_bfloat16, false>(x, residual, weight, M, K, eps, unit_offset, out,
                                                     residual_out, nullptr, nullptr, s);
}

extern "C" int fni8_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int64_t M, int64_t K,
                            float eps, int unit_offset, void* out, void* residual_out, void* stream) {
  return norm_common(x, residual, weight, dtype, M, K, eps, unit_offset, out, residual_out, nullptr, nullptr, stream,
                     false);
}

extern "C" int fni8_rmsnorm_quant_i8(const void* x, const void* residual, const void* weight, int dtype, int64_t M,
                                     int64_t K, float eps, int unit_offset, void* out, void* residual_out, int8_t* q,
                                     float* scale, void* stream) {
  return norm_common(x, residual, weight, dtype, M, K, eps, unit_offset, out, residual_out, q, scale, stream, true);
}

static int act_common(const void* x, int dtype, int act, int64_t M, int64_t I, void* out, int8_t* q, float* scale,
                      void* stream, bool quant, const int32_t* m_dev = nullptr) {
  if (int st = check_rows(x, dtype, M, I)) return st;
  if (act != FNI8_ACT_SILU && act != FNI8_ACT_GELU_TANH) return fni8h::fail(FNI8_ERR_INVALID, "unknown act %d", act);
  if (!quant && M > 0 && out == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null output");
  if (quant && M > 0 && (q == nullptr || scale == nullptr)) return fni8h::fail(FNI8_ERR_INVALID, "null q/scale");
  if (M == 0) return FNI8_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FNI8_F16) {
    if (act == FNI8_ACT_SILU)
      return quant ? act_dispatch<__half, FNI8_ACT_SILU, true>(x, M, I, out, q, scale, s, m_dev)
                   : act_dispatch<__half, FNI8_ACT_SILU, false>(x, M, I, out, nullptr, nullptr, s, m_dev);
    return quant ? act_dispatch<__half, FNI8_ACT_GELU_TANH, true>(x, M, I, out, q, scale, s, m_dev)
                 : act_dispatch<__half, FNI8_ACT_GELU_TANH, false>(x, M, I, out, nullptr, nullptr, s, m_dev);
  }
  if (act == FNI8_ACT_SILU)
    return quant ? act_dispatch<__nv_bfloat16, FNI8_ACT_SILU, true>(x, M, I, out, q, scale, s, m_dev)
                 : act_dispatch<__nv_bfloat16, FNI8_ACT_SILU, false>(x, M, I, out, nullptr, nullptr, s, m_dev);
  return quant ? act_dispatch<__nv_bfloat16, FNI8_ACT_GELU_TANH, true>(x, M, I, out, q, scale, s, m_dev)
               : act_dispatch<__nv_bfloat16, FNI8_ACT_GELU_TANH, false>(x, M, I, out, nullptr, nullptr, s, m_dev);
}

extern "C" int fni8_act_and_mul(const void* x, int dtype, int act, int64_t M, int64_t I, void* out, void* stream) {
  return act_common(x, dtype, act, M, I, out, nullptr, nullptr, stream, false);
}

extern "C" int fni8_act_and_mul_quant_i8(const void* x, int dtype, int act, int64_t M, int64_t I, int8_t* q,
                                         float* scale, void* stream) {
  return act_common(x, dtype, act, M, I, nullptr, q, scale, stream, true);
}

extern "C" int fni8_quantize_rows_i8_rows(const void* x, int dtype, int64_t M, int64_t K, const int32_t* rows_dev,
                                          int8_t* q, float* scale, void* stream) {
  if (int st = check_rows(x, dtype, M, K)) return st;
  if (M == 0) return FNI8_OK;
  if (rows_dev == nullptr || q == nullptr || scale == nullptr)
    return fni8h::fail(FNI8_ERR_INVALID, "null device row count or output");
  if (K % 8 != 0 || K / 8 > 16 * kRowThreads || !aligned16(x) || !aligned16(q))
    return fni8h::fail(FNI8_ERR_UNSUPPORTED, "quantize_rows_i8_rows: K a multiple of 8 (<= 16384), 16-byte aligned rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == FNI8_F16 ? quant_dispatch<__half>(x, M, K, q, scale, s, rows_dev)
                           : quant_dispatch<__nv_bfloat16>(x, M, K, q, scale, s, rows_dev);
}

extern "C" int fni8_act_and_mul_quant_i8_rows(const void* x, int dtype, int act, int64_t M, int64_t I,
                                              const int32_t* rows_dev, int8_t* q, float* scale, void* stream) {
  if (M > 0 && rows_dev == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null device row count");
  return act_common(x, dtype, act, M, I, nullptr, q, scale, stream, true, rows_dev);
}

extern "C" int fni8_act_and_mul_dual(const void* x, int dtype, int act, int64_t M, int64_t I, void* out, int8_t* q,
                                     float* scale, void* stream) {
  if (M > 0 && out == nullptr) return fni8h::fail(FNI8_ERR_INVALID, "null output");
  return act_common(x, dtype, act, M, I, out, q, scale, stream, true);
}
