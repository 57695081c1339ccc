// Host-side functions shared between the translation units of libfni8_b200.so. Not part
// of the public C ABI (include/fni8_b200.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "tuning.h"

namespace fni8h {

constexpr int kMaxDevices = 64;
constexpr int kTileMaxSeg = 512;  // segments of one grouped launch

// tcgen05 tile GEMM (gemm_tile.cu). out_mode: 0 fp16, 1 bf16, 2 int32 accumulators.
// pair: 256-row tiles on CTA pairs (tcgen05.mma.cta_group::2).
int tile_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
              const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, int bn, bool pair,
              cudaStream_t st);
int tile_gemm_grouped(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w, const float* w_scale,
                      int64_t E, int64_t N, int64_t K, const int32_t* seg_expert, const int32_t* seg_off,
                      const int32_t* seg_cnt, int64_t S, void* out, int out_mode, int bn, bool pair,
                      cudaStream_t st, const int32_t* row_tag = nullptr, void* const* peer_out = nullptr,
                      int n_peers = 0, int64_t peer_rows = 0);
// (row_tag set: output row r goes to row (row_tag[r] & 0xFFFFFF) of the [peer_rows, N]
// buffer peer_out[row_tag[r] >> 24] instead of out; 16-bit out_mode, N % 64 == 0, buffers
// 16-byte aligned, checked by the caller.)
// Dense tile GEMM whose epilogue writes output element (m, n) to element
// (m, col_off + n) of each of the n_peers (<= 8) buffers peer_out[p] (row stride ld
// elements; this GPU's memory or an NVLink peer's mapped into this process): a column
// shard's part of an all-gather. 16-bit out_mode, no residual; the caller validates
// alignment (buffers, ld and col_off 16-byte multiples, N % 64 == 0).
int tile_gemm_peer_cols(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                        int out_mode, int64_t M, int64_t N, int64_t K, void* const* peer_out, int n_peers, int64_t ld,
                        int64_t col_off, int bn, bool pair, cudaStream_t st);
// Tile GEMM over a merged gate_up weight (gate rows [0, I), up rows [I, 2I)) whose
// epilogue applies act_and_mul: out[M, I] in fp16/bf16 (out_mode 0/1), I % 128 == 0.
// Dense when seg_expert is null; grouped over S segments of a [E, 2I, K] stack otherwise.
int tile_gemm_act(const int8_t* a, const float* a_scale, int64_t M, const int8_t* w, const float* w_scale, int64_t E,
                  int64_t I, int64_t K, const int32_t* seg_expert, const int32_t* seg_off, const int32_t* seg_cnt,
                  int64_t S, int act, void* out, int out_mode, bool pair, cudaStream_t st);
// Whether dense (prefill-size) and grouped tile GEMMs run on CTA pairs.
bool tile_pair_enabled();
bool grouped_pair_enabled();
int tile_status_read_and_clear(int* code);

// Swap-AB stream-K GEMM for skinny M (gemm_stream.cu).
size_t stream_workspace_bytes(int64_t M, int64_t N, int64_t K);
int stream_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws,
                size_t ws_bytes, cudaStream_t st);
int stream_status_read_and_clear(int* code);
constexpr int64_t kStreamMaxM = 256;
// Re-zero the allocation-free GEMM's built-in scratch on the current device (synchronous).
int noalloc_scratch_reset();


// Cluster split-K swap-AB GEMM for decode (gemm_splitk.cu): int8 activations; partial sums
// of a split K range cross the zero-maintained GEMM workspace and are zeroed again.
constexpr int64_t kSplitkMaxM = 256;
bool splitk_supported(int64_t M, int64_t N, int64_t K);
// Clusters of S CTAs (`threads` threads, `smem` bytes of dynamic shared memory) that can
// be resident at once; -1 when the runtime cannot tell.
int max_active_clusters(int threads, int smem, int S);

// The split-K plan for this shape splits K (S > 1) and every one of its clusters can be
// resident at once.
bool splitk_split_one_wave(int64_t M, int64_t N, int64_t K);
size_t splitk_workspace_bytes(int64_t M, int64_t N, int64_t K);
int splitk_gemm(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, const void* bias,
                const void* residual, void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws,
                size_t ws_bytes, cudaStream_t st);
int splitk_status_read_and_clear(int* code);

// W4A8 decode-shaped GEMM (gemm_w4a8.cu): packed int4 weights [N, K/2] with fp32 scales
// per 128-channel group [N, K/128]; 64 tokens per launch.
constexpr int64_t kW4ChunkM = 64;
size_t w4a8_workspace_bytes(int64_t M, int64_t N, int64_t K);
int w4a8_gemm(const int8_t* a, const float* a_scale, const uint8_t* w4, const float* w_scale, const void* bias,
              void* out, int out_mode, int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes, cudaStream_t st);
int w4a8_status_read_and_clear(int* code);

// Expert-parallel exchange kernels (ep_p2p.cu): capacity-overflow status word.
int ep_status_read_and_clear(int* code);
// src [M, N] 16-bit rows (row stride N) to columns [col_off, col_off + N) of each of the
// n_peers buffers peer_out[p] (row stride ld elements): the all-gather step of a column
// shard whose GEMM wrote a local buffer. Same alignment rules as tile_gemm_peer_cols.
int push_cols(const void* src, int64_t M, int64_t N, void* const* peer_out, int n_peers, int64_t ld, int64_t col_off,
              cudaStream_t st);

}  // namespace fni8h
