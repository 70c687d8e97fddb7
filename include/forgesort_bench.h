/*
 * forgesort_bench.h -- seeded synthetic key generator for benchmarks and
 * large tests, exported by libforgesort.so.
 *
 * Replaces forge-bench's DataGenerator (kavanaghpatrick/gpu-forge,
 * metal-forge-compute/forge-bench/src/data_gen.rs:5-25: StdRng, uniform_u32)
 * with the generator the benchmark configs specify: Marsaglia xorshift64
 * (x ^= x<<13; x ^= x>>7; x ^= x<<17), element i = state after i+1 steps
 * from `seed`.  Any element range [start, start+n) is produced directly on
 * the GPU by jump-ahead (the step is linear over GF(2)), so shard r of a
 * multi-GPU input is exactly elements [r*m, (r+1)*m) of the one stream.
 */
#ifndef FORGESORT_BENCH_H
#define FORGESORT_BENCH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fs_gen_dist {
  FS_GEN_U32 = 0,      /* high 32 bits of each state                         */
  FS_GEN_U64 = 1,      /* the full state                                     */
  FS_GEN_SKEW_U32 = 2  /* w = state; (uint32)w % 10 < 7 ? 0x40000000 + (w>>44)
                          : (uint32)(w>>32)  -- 70 % of keys in one 2^20 range */
} fs_gen_dist;

/* Write elements [start, start+n) of distribution `dist` to device memory
 * `out` (4 or 8 bytes each), enqueued on `stream` (cudaStream_t, NULL =
 * legacy default stream) of the current device.  Returns an fs_status. */
int fs_generate(int dist, uint64_t seed, uint64_t start, uint64_t n, void* out,
                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FORGESORT_BENCH_H */
