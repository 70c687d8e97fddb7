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

typedef struct fs_sorter fs_sorter; /* declared in forgesort.h */

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

/* ---- failure-path hooks (tests) -------------------------------------------
 * The reference maps a failed command buffer to SortError::GpuExecution
 * (forge-sort src/lib.rs:396-406) and panics when a buffer allocation fails
 * (src/metal_helpers.rs:194-202).  These hooks make the corresponding paths
 * of this library run without faulting or hanging a GPU, so tests can check
 * that the call fails with the right status and that the sorter works again
 * afterwards. */

/* Keys-only sorts of 32-bit keys whose keys take at most `key_bytes` bytes
 * (more than the single-CTA limit, at most 14336 keys per SM) run as one
 * cooperative launch instead of the chain of 2 + 3P kernels; 0 always uses
 * the chain.  fs_create takes the limit from FORGESORT_COOP_MAX_BYTES
 * (default 8 MiB: 2^21 keys). */
int fs_set_single_launch_max(fs_sorter* s, uint64_t key_bytes);

/* Bound on every device-side wait of this sorter (the mbarrier waits of the
 * scatter's bulk copies), in milliseconds (> 0).  fs_create takes it from
 * FORGESORT_WAIT_TIMEOUT_MS (default 2000). */
int fs_set_wait_timeout_ms(fs_sorter* s, uint64_t ms);

typedef enum fs_test_inject_kind {
  /* The next radix-path sort (n above the single-CTA limit, 16-byte aligned
   * keys) leaves the first bulk copy of CTA 0's first scatter tile un-issued:
   * that CTA's bounded wait runs out, the kernels stop early and the call
   * returns FS_E_TIMEOUT.  Nothing is left in flight.  One-shot. */
  FS_TEST_WITHHOLD_COPY = 1,
  /* The arg-th next growth of the sorter's device scratch (arg >= 1) fails
   * as if cudaMalloc had run out of memory: the call returns FS_E_OOM and
   * the scratch slot is left empty (the next call grows it again). */
  FS_TEST_FAIL_ALLOC = 2,
  /* The next single-launch sort (fs_set_single_launch_max) runs with CTA 0
   * leaving before the first grid barrier: every other CTA's bounded wait
   * runs out (fs_set_wait_timeout_ms), the call returns FS_E_TIMEOUT and the
   * next sort clears the barrier state.  One-shot. */
  FS_TEST_SKIP_ARRIVAL = 3
} fs_test_inject_kind;

/* Arm one injected failure (kind above) on sorter `s`; arg as the kind says.
 * kind 0 disarms all. */
int fs_test_inject(fs_sorter* s, int kind, int arg);

#ifdef __cplusplus
}
#endif

#endif /* FORGESORT_BENCH_H */
