// Library plumbing behind include/fni8_b200.h: status strings, thread-local error
// messages, TMA descriptor encoding (through the runtime's driver entry point, so the
// library does not link libcuda and loads on machines without a GPU), and the dense
// GEMM / linear entry points that pick between the tile kernel (gemm_tile.cu), the
// split-K decode kernel (gemm_splitk.cu) and the stream-K kernel (gemm_stream.cu).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <stdlib.h>

#include <mutex>

#include "fni8_common.cuh"
#include "gemm_internal.h"

namespace fni8h {

static thread_local char g_msg[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  return fail(FNI8_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int num_sms(int device) {
  static std::atomic<int> cache[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static int encode(CUtensorMap* map, const void* base, cuuint32_t rank, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapDataType dt, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(FNI8_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(FNI8_ERR_ALIGN, "TMA base must be 16-byte aligned");
  for (cuuint32_t i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16 != 0) return fail(FNI8_ERR_ALIGN, "TMA stride %llu not a multiple of 16 bytes",
                                          (unsigned long long)strides[i]);
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FNI8_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FNI8_OK;
}

int encode_tmap_2d_i8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  return encode(map, base, 2, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_tmap_2d_u8_sw64(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  return encode(map, base, 2, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_64B);
}

int encode_tmap_3d_i8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                      uint64_t stride2, uint32_t box0, uint32_t box1) {
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1, stride2};
  const cuuint32_t box[3] = {box0, box1, 1};
  return encode(map, base, 3, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_tmap_2d_16_sw(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle64) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  return encode(map, base, 2, dims, strides, box,
                bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

int encode_tmap_2d_16(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  return encode(map, base, 2, dims, strides, box,
                bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Shape/pointer checks shared by the dense GEMM entry points.
static int check_gemm(const int8_t* a, const int8_t* w, const void* out, int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N <= 0 || K <= 0) return fail(FNI8_ERR_INVALID, "bad GEMM shape M=%lld N=%lld K=%lld", (long long)M,
                                              (long long)N, (long long)K);
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "K=%lld must be a multiple of 16", (long long)K);
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31))
    return fail(FNI8_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  if (M > 0 && (a == nullptr || w == nullptr || out == nullptr)) return fail(FNI8_ERR_INVALID, "null GEMM operand");
  return FNI8_OK;
}

// Largest M the AUTO choice sends to the stream-K kernel: none by default, the split-K
// kernel measured faster at every decode size on B200 (FNI8_TUNE_STREAM_AUTO_MAX_M).
static int64_t stream_auto_max_m() {
  constexpr int64_t m = FNI8_TUNE_STREAM_AUTO_MAX_M;
  return m < 0 ? 0 : (m > kStreamMaxM ? kStreamMaxM : m);
}

// Largest M the AUTO choice sends to the split-K kernel: measured on B200, it beats the
// tile kernel up to 256 tokens whenever its grid fits on the GPU in one wave
// (FNI8_TUNE_SPLITK_AUTO_MAX_M).
static int64_t splitk_auto_max_m() {
  constexpr int64_t m = FNI8_TUNE_SPLITK_AUTO_MAX_M;
  return m < 0 ? 0 : (m > kSplitkMaxM ? kSplitkMaxM : m);
}

// Above 64 tokens a weight matrix with at least this many 256-row tiles goes to the tile
// kernel, whose 256-column tiles let each MMA consume twice the weight bytes of a split-K
// MMA. Default: one tile per SM (an LM head, N = 151936, measured on B200);
// (FNI8_TUNE_WIDE_MIN_TILES).
static int64_t wide_min_tiles() {
  constexpr int64_t x = FNI8_TUNE_WIDE_MIN_TILES;
  return x > 0 ? x : num_sms(current_device());
}

static bool wide_weights(int64_t M, int64_t N) { return M > 64 && (N + 255) / 256 >= wide_min_tiles(); }

static int pick_path(int path, int64_t M, size_t ws_bytes, int64_t N, int64_t K) {
  if (path == FNI8_PATH_TILE || path == FNI8_PATH_STREAM || path == FNI8_PATH_SPLITK) return path;
  if (M <= stream_auto_max_m() && ws_bytes >= stream_workspace_bytes(M, N, K)) return FNI8_PATH_STREAM;
  const bool wide = wide_weights(M, N);
  // Above 128 tokens split-K wins only where it splits K over clusters that are all
  // resident at once (measured at M = 256: QKV, O and down projections; the unsplit
  // gate_up, 192 weight tiles, streams faster through the tile kernel).
  if (M <= splitk_auto_max_m() && !wide && splitk_supported(M, N, K) &&
      ws_bytes >= splitk_workspace_bytes(M, N, K) && (M <= 128 || splitk_split_one_wave(M, N, K)))
    return FNI8_PATH_SPLITK;
  return FNI8_PATH_TILE;
}

// Explicit GEMM kernel choices of the int8-activation entry points.
static int check_path(int path, int64_t M) {
  if (path != FNI8_PATH_AUTO && path != FNI8_PATH_TILE && path != FNI8_PATH_STREAM && path != FNI8_PATH_SPLITK)
    return fail(FNI8_ERR_INVALID, "unknown path %d", path);
  if (path == FNI8_PATH_STREAM && M > kStreamMaxM)
    return fail(FNI8_ERR_UNSUPPORTED, "stream path takes M <= %lld", (long long)kStreamMaxM);
  if (path == FNI8_PATH_SPLITK && M > kSplitkMaxM)
    return fail(FNI8_ERR_UNSUPPORTED, "split-K path takes M <= %lld", (long long)kSplitkMaxM);
  return FNI8_OK;
}

// Column width of a single-CTA tile: 256 where there are two 256-wide tiles per SM, else
// 128 (FNI8_TUNE_TILE_BN = 128 or 256 forces one).
static int pick_bn(int64_t M, int64_t N) {
  constexpr int forced = (FNI8_TUNE_TILE_BN == 128 || FNI8_TUNE_TILE_BN == 256) ? FNI8_TUNE_TILE_BN : 0;
  if (forced) return forced;
  const int64_t tiles256 = ((M + 127) / 128) * ((N + 255) / 256);
  return tiles256 >= 2 * num_sms(current_device()) ? 256 : 128;
}

static int gemm_any(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                    const void* residual, void* out, int mode, int64_t M, int64_t N, int64_t K, int path, void* ws,
                    size_t ws_bytes, cudaStream_t st) {
  const int p = pick_path(path, M, ws_bytes, N, K);
  if (p == FNI8_PATH_STREAM)
    return stream_gemm(a, a_scale, w, w_scale, bias, residual, out, mode, M, N, K, ws, ws_bytes, st);
  if (p == FNI8_PATH_SPLITK)
    return splitk_gemm(a, a_scale, w, w_scale, bias, residual, out, mode, M, N, K, ws, ws_bytes, st);
  // prefill sizes: 256-row tiles on CTA pairs, each SM holding half of a weight tile
  const bool pair = tile_pair_enabled() && M >= 256;
  return tile_gemm(a, a_scale, w, w_scale, bias, residual, out, mode, M, N, K, pair ? 256 : pick_bn(M, N), pair, st);
}

}  // namespace fni8h

using namespace fni8h;

extern "C" int fni8_abi_version(void) { return FNI8_ABI_VERSION; }

extern "C" const char* fni8_status_string(int status) {
  switch (status) {
    case FNI8_OK: return "ok";
    case FNI8_ERR_INVALID: return "invalid argument";
    case FNI8_ERR_UNSUPPORTED: return "unsupported";
    case FNI8_ERR_ALIGN: return "misaligned pointer or stride";
    case FNI8_ERR_CUDA: return "CUDA error";
    case FNI8_ERR_WORKSPACE: return "workspace missing or too small";
    case FNI8_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* fni8_last_error_message(void) { return g_msg; }

extern "C" int fni8_device_status(int* code_out) {
  if (code_out == nullptr) return fail(FNI8_ERR_INVALID, "null code_out");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceSynchronize");
  int codes[5] = {0, 0, 0, 0, 0};
  if (int s = tile_status_read_and_clear(&codes[0])) return s;
  if (int s = stream_status_read_and_clear(&codes[1])) return s;
  if (int s = splitk_status_read_and_clear(&codes[2])) return s;
  if (int s = w4a8_status_read_and_clear(&codes[3])) return s;
  if (int s = ep_status_read_and_clear(&codes[4])) return s;
  *code_out = 0;
  for (int v : codes)
    if (*code_out == 0) *code_out = v;
  if (*code_out == 0) return FNI8_OK;
  // a kernel that left its loop on a timed-out wait may have left partial sums in the
  // shared scratch of the allocation-free GEMM: zero it before the next call uses it
  if (int s = noalloc_scratch_reset()) return s;
  return fail(FNI8_ERR_DEVICE_TIMEOUT, "device watchdog code 0x%x", *code_out);
}

extern "C" size_t fni8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  const size_t a = stream_workspace_bytes(M, N, K), b = splitk_workspace_bytes(M, N, K);
  const size_t ab = a > b ? a : b, c = w4a8_workspace_bytes(M, N, K);
  return ab > c ? ab : c;
}

extern "C" int fni8_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (bytes == 0) return FNI8_OK;
  if (workspace == nullptr) return fail(FNI8_ERR_INVALID, "null workspace");
  cudaError_t e = cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(workspace)");
  return FNI8_OK;
}

extern "C" int fni8_gemm_w8a8_ex(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                 const void* bias, const void* residual, void* out, int out_dtype, int64_t M,
                                 int64_t N, int64_t K, int path, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  if (int s = check_gemm(a, w, out, M, N, K)) return s;
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16)
    return fail(FNI8_ERR_INVALID, "out_dtype %d: expected F16 or BF16", out_dtype);
  if (int s = check_path(path, M)) return s;
  if (M > 0 && (a_scale == nullptr || w_scale == nullptr)) return fail(FNI8_ERR_INVALID, "null scale");
  if (M == 0) return FNI8_OK;
  return gemm_any(a, a_scale, w, w_scale, bias, residual, out, out_dtype == FNI8_F16 ? 0 : 1, M, N, K, path,
                  workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_gemm_w8a8(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                              const void* bias, const void* residual, void* out, int out_dtype, int64_t M, int64_t N,
                              int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  return fni8_gemm_w8a8_ex(a, a_scale, w, w_scale, bias, residual, out, out_dtype, M, N, K, FNI8_PATH_AUTO,
                           workspace, workspace_bytes, stream);
}

extern "C" int fni8_gemm_w8a8_act(const int8_t* a, const float* a_scale, const int8_t* w_gu, const float* s_gu, int act,
                                  void* out, int out_dtype, int64_t M, int64_t I, int64_t K, void* stream) {
  if (int s = check_gemm(a, w_gu, out, M, 2 * I, K)) return s;
  if (I <= 0) return fail(FNI8_ERR_INVALID, "bad I=%lld", (long long)I);
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16)
    return fail(FNI8_ERR_INVALID, "out_dtype %d: expected F16 or BF16", out_dtype);
  if (M > 0 && (a_scale == nullptr || s_gu == nullptr)) return fail(FNI8_ERR_INVALID, "null scale");
  if (M == 0) return FNI8_OK;
  // 256-row tiles on CTA pairs from 256 tokens on (prefill), as the plain tile GEMM
  return tile_gemm_act(a, a_scale, M, w_gu, s_gu, 1, I, K, nullptr, nullptr, nullptr, 0, act, out,
                       out_dtype == FNI8_F16 ? 0 : 1, tile_pair_enabled() && M >= 256, static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_gemm_w8a8_peer_cols(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                        const void* bias, int out_dtype, int64_t M, int64_t N, int64_t K,
                                        void* const* peer_out, int n_peers, int64_t ld, int64_t col_off, void* tmp,
                                        size_t tmp_bytes, void* ws, size_t ws_bytes, void* stream) {
  if (int s = check_gemm(a, w, peer_out, M, N, K)) return s;
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16)
    return fail(FNI8_ERR_INVALID, "out_dtype %d: expected F16 or BF16", out_dtype);
  if (n_peers < 1 || n_peers > 8) return fail(FNI8_ERR_INVALID, "peer_cols: 1 to 8 destination buffers (got %d)", n_peers);
  if (N % 64 != 0) return fail(FNI8_ERR_UNSUPPORTED, "peer_cols: N=%lld must be a multiple of 64", (long long)N);
  if (col_off < 0 || ld < col_off + N) return fail(FNI8_ERR_INVALID, "peer_cols: columns [%lld, %lld) exceed ld=%lld",
                                                   (long long)col_off, (long long)(col_off + N), (long long)ld);
  if (ld % 8 != 0 || col_off % 8 != 0 || ld >= (1LL << 31))
    return fail(FNI8_ERR_ALIGN, "peer_cols: ld and col_off must be multiples of 8 (16 bytes)");
  if (M > 0 && (a_scale == nullptr || w_scale == nullptr)) return fail(FNI8_ERR_INVALID, "null scale");
  if (M == 0) return FNI8_OK;
  for (int i = 0; i < n_peers; ++i) {
    if (peer_out[i] == nullptr) return fail(FNI8_ERR_INVALID, "peer_cols: null destination %d", i);
    if (reinterpret_cast<uintptr_t>(peer_out[i]) & 15u)
      return fail(FNI8_ERR_ALIGN, "peer_cols: destination %d must be 16-byte aligned", i);
  }
  if ((reinterpret_cast<uintptr_t>(w_scale) & 15u) || (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 15u)))
    return fail(FNI8_ERR_ALIGN, "peer_cols: w_scale and bias must be 16-byte aligned");
  const int mode = out_dtype == FNI8_F16 ? 0 : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int p = pick_path(FNI8_PATH_AUTO, M, ws_bytes, N, K);
  if (p == FNI8_PATH_TILE) {
    const bool pair = tile_pair_enabled() && M >= 256;
    return tile_gemm_peer_cols(a, a_scale, w, w_scale, bias, mode, M, N, K, peer_out, n_peers, ld, col_off,
                               pair ? 256 : pick_bn(M, N), pair, st);
  }
  // decode sizes: the split-K (or stream-K) GEMM into tmp, then the copy to every buffer
  if (tmp == nullptr || tmp_bytes < (size_t)(M * N * 2))
    return fail(FNI8_ERR_WORKSPACE, "peer_cols: tmp needs %lld bytes", (long long)(M * N * 2));
  if (reinterpret_cast<uintptr_t>(tmp) & 15u) return fail(FNI8_ERR_ALIGN, "peer_cols: tmp must be 16-byte aligned");
  if (int s = gemm_any(a, a_scale, w, w_scale, bias, nullptr, tmp, mode, M, N, K, p, ws, ws_bytes, st)) return s;
  return push_cols(tmp, M, N, peer_out, n_peers, ld, col_off, st);
}

extern "C" int fni8_gemm_w8a8_i32(const int8_t* a, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                                  int path, void* workspace, size_t workspace_bytes, void* stream) {
  if (int s = check_gemm(a, w, acc, M, N, K)) return s;
  if (int s = check_path(path, M)) return s;
  if (M == 0) return FNI8_OK;
  return gemm_any(a, nullptr, w, nullptr, nullptr, nullptr, acc, 2, M, N, K, path, workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_linear_w8a8_ex(const void* x, int dtype, const int8_t* w, const float* w_scale, const void* bias,
                                   void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                                   int path, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "dtype %d: expected F16 or BF16", dtype);
  if (path < FNI8_PATH_AUTO || path > FNI8_PATH_SPLITK) return fail(FNI8_ERR_INVALID, "unknown path %d", path);
  if (path == FNI8_PATH_STREAM && M > kStreamMaxM)
    return fail(FNI8_ERR_UNSUPPORTED, "stream path takes M <= %lld", (long long)kStreamMaxM);
  if (path == FNI8_PATH_SPLITK && M > kSplitkMaxM)
    return fail(FNI8_ERR_UNSUPPORTED, "split-K path takes M <= %lld", (long long)kSplitkMaxM);
  if (M < 0 || N <= 0 || K <= 0) return fail(FNI8_ERR_INVALID, "bad linear shape M=%lld N=%lld K=%lld", (long long)M,
                                              (long long)N, (long long)K);
  if (K % 16 != 0) return fail(FNI8_ERR_UNSUPPORTED, "K=%lld must be a multiple of 16", (long long)K);
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31))
    return fail(FNI8_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  if (M == 0) return FNI8_OK;
  if (x == nullptr || w == nullptr || w_scale == nullptr || out == nullptr)
    return fail(FNI8_ERR_INVALID, "null linear operand");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (path == FNI8_PATH_FUSED)
    return fail(FNI8_ERR_UNSUPPORTED, "FNI8_PATH_FUSED is not built (measured slower than quantiser + split-K)");
  if (q_scratch == nullptr || s_scratch == nullptr) return fail(FNI8_ERR_INVALID, "null linear scratch");
  if (int s = fni8_quantize_rows_i8(x, dtype, M, K, q_scratch, s_scratch, stream)) return s;
  return gemm_any(q_scratch, s_scratch, w, w_scale, bias, nullptr, out, dtype == FNI8_F16 ? 0 : 1, M, N, K, path,
                  workspace, workspace_bytes, st);
}

extern "C" int fni8_linear_w8a8(const void* x, int dtype, const int8_t* w, const float* w_scale, const void* bias,
                                void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return fni8_linear_w8a8_ex(x, dtype, w, w_scale, bias, out, M, N, K, q_scratch, s_scratch, FNI8_PATH_AUTO,
                             workspace, workspace_bytes, stream);
}

// ------------------------------------------------------------------ W4A8 (per_group_i4, int4)
static int check_w4(const int8_t* a, const float* a_scale, const uint8_t* w4, const float* w_scale, const void* out,
                    int out_dtype, int64_t M, int64_t N, int64_t K, int64_t group_size) {
  if (M < 0 || N <= 0 || K <= 0) return fail(FNI8_ERR_INVALID, "bad W4A8 shape M=%lld N=%lld K=%lld", (long long)M,
                                              (long long)N, (long long)K);
  if (group_size != 128) return fail(FNI8_ERR_UNSUPPORTED, "W4A8 takes group_size 128 (got %lld)", (long long)group_size);
  if (K % 128 != 0) return fail(FNI8_ERR_UNSUPPORTED, "W4A8 takes K a multiple of 128 (got %lld)", (long long)K);
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31))
    return fail(FNI8_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  if (out_dtype != FNI8_F16 && out_dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "out_dtype %d", out_dtype);
  if (M > 0 && (a == nullptr || a_scale == nullptr || w4 == nullptr || w_scale == nullptr || out == nullptr))
    return fail(FNI8_ERR_INVALID, "null W4A8 operand");
  return FNI8_OK;
}

extern "C" int fni8_gemm_w4a8(const int8_t* a, const float* a_scale, const uint8_t* w4, const float* w_scale,
                              int64_t group_size, const void* bias, void* out, int out_dtype, int64_t M, int64_t N,
                              int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  if (int s = check_w4(a, a_scale, w4, w_scale, out, out_dtype, M, N, K, group_size)) return s;
  if (M == 0) return FNI8_OK;
  return w4a8_gemm(a, a_scale, w4, w_scale, bias, out, out_dtype == FNI8_F16 ? 0 : 1, M, N, K, workspace,
                   workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fni8_linear_w4a8(const void* x, int dtype, const uint8_t* w4, const float* w_scale, int64_t group_size,
                                const void* bias, void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch,
                                float* s_scratch, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != FNI8_F16 && dtype != FNI8_BF16) return fail(FNI8_ERR_INVALID, "dtype %d: expected F16 or BF16", dtype);
  if (M > 0 && (x == nullptr || q_scratch == nullptr || s_scratch == nullptr))
    return fail(FNI8_ERR_INVALID, "null linear input or scratch");
  if (int s = check_w4(M > 0 ? q_scratch : nullptr, s_scratch, w4, w_scale, out, dtype, M, N, K, group_size)) return s;
  if (M == 0) return FNI8_OK;
  if (int s = fni8_quantize_rows_i8(x, dtype, M, K, q_scratch, s_scratch, stream)) return s;
  return w4a8_gemm(q_scratch, s_scratch, w4, w_scale, bias, out, dtype == FNI8_F16 ? 0 : 1, M, N, K, workspace,
                   workspace_bytes, static_cast<cudaStream_t>(stream));
}
