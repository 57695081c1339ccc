// Tuning constants of the sm_100a kernels' launch choices, measured on B200. The shipped
// library reads no environment variables; a measurement build overrides one with
// -DFNI8_TUNE_<NAME>=<value> at compile time.
#pragma once

#ifndef FNI8_TUNE_PDL
#define FNI8_TUNE_PDL 1  // programmatic dependent launch between consecutive kernels
#endif
#ifndef FNI8_TUNE_TILE_PAIR
#define FNI8_TUNE_TILE_PAIR 1  // dense tile GEMMs from 256 rows on CTA pairs (4-10 % faster)
#endif
#ifndef FNI8_TUNE_GROUPED_PAIR
#define FNI8_TUNE_GROUPED_PAIR 0  // grouped (expert) GEMMs on CTA pairs (slower: short segments)
#endif
#ifndef FNI8_TUNE_TILE_L2AHEAD
#define FNI8_TUNE_TILE_L2AHEAD 0  // tile weight k-blocks pulled into L2 before the dependency wait
#endif
#ifndef FNI8_TUNE_TILE_TRIGGER
#define FNI8_TUNE_TILE_TRIGGER 1  // tile kernel releases the next kernel after its last load
#endif
#ifndef FNI8_TUNE_STREAM_AUTO_MAX_M
#define FNI8_TUNE_STREAM_AUTO_MAX_M 0  // AUTO never picks stream-K (split-K measured faster)
#endif
#ifndef FNI8_TUNE_SPLITK_AUTO_MAX_M
#define FNI8_TUNE_SPLITK_AUTO_MAX_M 256  // AUTO picks split-K up to 256 tokens (one wave)
#endif
#ifndef FNI8_TUNE_WIDE_MIN_TILES
#define FNI8_TUNE_WIDE_MIN_TILES 0  // 256-row weight tiles that send M > 64 to the tile kernel (0: SMs)
#endif
#ifndef FNI8_TUNE_TILE_BN
#define FNI8_TUNE_TILE_BN 0  // single-CTA tile width (0: 256 with two tiles per SM, else 128)
#endif
#ifndef FNI8_TUNE_STREAM_SMEM_KB
#define FNI8_TUNE_STREAM_SMEM_KB 100  // stream-K ring budget (100: two CTAs per SM)
#endif
#ifndef FNI8_TUNE_SPLITK_S
#define FNI8_TUNE_SPLITK_S 0  // split-K cluster size (0: planned per shape)
#endif
#ifndef FNI8_TUNE_SPLITK_TARGET_PCT
#define FNI8_TUNE_SPLITK_TARGET_PCT 100  // split-K grid target, % of the SM count
#endif
#ifndef FNI8_TUNE_SPLITK_SMEM_KB
#define FNI8_TUNE_SPLITK_SMEM_KB 0  // split-K ring budget (0: planned)
#endif
#ifndef FNI8_TUNE_SPLITK_L2AHEAD
#define FNI8_TUNE_SPLITK_L2AHEAD 0  // split-K weight k-blocks pulled into L2 before the wait
#endif
#ifndef FNI8_TUNE_SPLITK_TRIGGER
#define FNI8_TUNE_SPLITK_TRIGGER 2  // split-K releases the next kernel once its partial sums are out
#endif
#ifndef FNI8_TUNE_PLAN_LOG
#define FNI8_TUNE_PLAN_LOG 0  // print split-K plans to stderr
#endif
