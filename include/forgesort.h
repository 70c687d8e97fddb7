/*
 * forgesort.h -- C ABI of the B200 (sm_100a) radix sort behind forge-sort's
 * GpuSorter API.
 *
 * Every entry point returns an fs_status (0 = success).  The text of the most
 * recent failure on a sorter is available from fs_last_error().  No torch or
 * CUDA C++ types cross this boundary: devices are ordinals, streams are
 * opaque `void*` (a cudaStream_t, or NULL for the sorter's own stream),
 * buffers are plain pointers and sizes.
 *
 * Reference interfaces replaced (paths inside kavanaghpatrick/gpu-forge,
 * crate metal-forge-compute/forge-sort):
 *   src/lib.rs:596-686      GpuSorter::new / with_context  -> fs_create
 *   src/lib.rs:160-281      SortBuffer<T>                  -> fs_buffer_*
 *   src/lib.rs:694-706      alloc_sort_buffer              -> fs_buffer_create
 *   src/lib.rs:708-738      sort_buffer (+ *_buffer forms) -> fs_sort_buffer
 *   src/lib.rs:749-785      encode_sort (caller encoder)   -> fs_sort_buffer(sync=0)
 *   src/lib.rs:791-2590     sort_{u32,i32,f32,u64,i64,f64} -> fs_host_sort_keys
 *   src/lib.rs:1675-2825    argsort_*                      -> fs_argsort / fs_host_argsort
 *   src/lib.rs:1923-3015    sort_pairs_*                   -> fs_sort_pairs / fs_host_sort_pairs
 *   src/lib.rs:94-104       SortError                      -> fs_status + fs_last_error
 *   src/metal_helpers.rs:194-217 alloc_buffer / init_device_and_queue
 *                                                          -> fs_alloc / fs_create
 */
#ifndef FORGESORT_H
#define FORGESORT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FS_ABI_VERSION 1

/* Key types.  Mirrors the sealed SortKey impls of src/lib.rs:16-88. */
typedef enum fs_dtype {
  FS_U32 = 0,
  FS_I32 = 1,
  FS_F32 = 2,
  FS_U64 = 3,
  FS_I64 = 4,
  FS_F64 = 5
} fs_dtype;

/* Status codes.  1..4 map one-to-one onto SortError's variants
 * (src/lib.rs:94-104); 5..8 are GPU-side failures that the Rust/C++/Python
 * layers report as SortError::GpuExecution(text). */
typedef enum fs_status {
  FS_OK = 0,
  FS_E_DEVICE_NOT_FOUND = 1,  /* SortError::DeviceNotFound            */
  FS_E_KERNEL_IMAGE = 2,      /* SortError::ShaderCompilation(text)   */
  FS_E_GPU_EXECUTION = 3,     /* SortError::GpuExecution(text)        */
  FS_E_LENGTH_MISMATCH = 4,   /* SortError::LengthMismatch{keys,values} */
  FS_E_TIMEOUT = 5,           /* a bounded device wait ran out        */
  FS_E_NCCL = 6,              /* collective failure (multi-GPU)       */
  FS_E_OOM = 7,               /* device allocation failed             */
  FS_E_INVALID = 8            /* bad argument (null pointer, size)    */
} fs_status;

typedef struct fs_sorter fs_sorter;

/* ---- lifetime ---------------------------------------------------------- */

/* Create a sorter bound to CUDA device `device`.  `stream` is a cudaStream_t
 * the sorter enqueues on (the analogue of with_context's command queue), or
 * NULL to create a private non-blocking stream (the analogue of new()).
 * Replaces src/lib.rs:596-686. */
int fs_create(int device, void* stream, fs_sorter** out);
/* Environment read by fs_create (all optional):
 *   FORGESORT_WAIT_TIMEOUT_MS  bound on every device-side wait (default 2000);
 *                              a wait that runs out fails the call with
 *                              FS_E_TIMEOUT instead of hanging
 *   FORGESORT_SMALL_SORT       largest n sorted by one CTA in shared memory
 *                              (default and maximum 8192 keys alone, 4096 with
 *                              a payload; 0: always the radix passes)
 *   FORGESORT_COOP_MAX_BYTES   keys-only sorts of 32-bit keys of up to this
 *                              many key bytes (default 8 MiB, and at most
 *                              14336 keys per SM) run as one cooperative
 *                              launch with grid barriers instead of the
 *                              chained kernels; 0: always chained
 *   FORGESORT_H16_MIN_KEYS     keys-only sorts of 32-bit keys of at least
 *                              this many keys (default 2^30) run only the
 *                              radix passes of the top two digits and then
 *                              sort each top-16-bit group by counting its
 *                              low 16 bits; 0: always the four passes
 * and once per process:
 *   FORGESORT_CHAIN_LAUNCH     0: launch a sort's kernels without programmatic
 *                              stream serialization (default: chained) */
int fs_destroy(fs_sorter* s);

/* Text of the last failure on `s` (never NULL; "" when none).  With s == NULL,
 * the text of the last failure on this thread of a call that has no sorter
 * (fs_create, fs_sort_keys_noalloc). */
const char* fs_last_error(const fs_sorter* s);

/* Replace the stream the sorter enqueues on (NULL = its private stream). */
int fs_set_stream(fs_sorter* s, void* stream);
/* Wait for all work enqueued by `s`, then report any device-side failure
 * (a bounded wait that ran out, an out-of-range scatter) that an
 * asynchronous call left behind. */
int fs_synchronize(fs_sorter* s);

/* ---- memory (SortBuffer backing) --------------------------------------- */

/* managed == 0: allocate `bytes` of device memory (cudaMalloc) for the
 * sorter's device.  managed != 0: a SortBuffer backing -- page-locked host
 * memory (cudaHostAlloc, portable + mapped) that the host reads and writes at
 * full speed through the same pointer, which is what
 * SortBuffer::as_slice/as_mut_slice rely on (src/lib.rs:694-706,
 * src/metal_helpers.rs:194-202).  The sorts below accept such a pointer:
 * they copy it into device staging memory at PCIe rate, sort in HBM and copy
 * it back, all on the sorter's stream.  (Managed memory from
 * cudaMallocManaged also works, prefetched to the device; but the host's
 * first read of pages that came back from the GPU maps them one fault at a
 * time: 436 ms for 1 GB measured, against ~20 ms for the copy back.) */
int fs_alloc(fs_sorter* s, size_t bytes, int managed, void** ptr);
int fs_free(fs_sorter* s, void* ptr);

/* ---- SortBuffer objects (zero-copy at device speed) ---------------------- */

/* A SortBuffer: `bytes` of device memory plus a page-locked host mirror of
 * the same size, kept coherent lazily.  The reference's SortBuffer is one
 * unified-memory Metal buffer that the CPU and GPU share
 * (src/lib.rs:160-281, alloc_sort_buffer :694-706); on a discrete GPU the
 * two copies stand in for it:
 *   - fs_sort_buffer / fs_sort_pairs_buffer sort the device copy in place and
 *     copy nothing back; before sorting they copy over only the leading bytes
 *     the host changed since the device last saw them.  Repeated sorts of a
 *     buffer the host does not touch run at device speed;
 *   - fs_buffer_host_read makes the host mirror current (waits for the sorts
 *     that touched the buffer, copies back what they changed): call it
 *     before reading fs_buffer_host(b) -- as_slice / copy_to_slice;
 *   - fs_buffer_host_write = host_read, then marks the device copy stale:
 *     call it before writing the host mirror -- as_mut_slice /
 *     copy_from_slice (write, then sort);
 *   - fs_buffer_device_use hands the device copy to other device code (a
 *     gather, a kernel of the caller's): makes its leading `bytes` current
 *     and counts them as possibly written, so the next host read waits for
 *     the device and copies them back.
 * A buffer lives on the creating sorter's device and may outlive that
 * sorter.  Buffer-only calls report errors through fs_last_error(NULL). */
typedef struct fs_buffer fs_buffer;
int fs_buffer_create(fs_sorter* s, uint64_t bytes, fs_buffer** out);
int fs_buffer_destroy(fs_buffer* b);
void* fs_buffer_host(const fs_buffer* b);
void* fs_buffer_device(const fs_buffer* b);
uint64_t fs_buffer_bytes(const fs_buffer* b);
int fs_buffer_host_read(fs_buffer* b);
int fs_buffer_host_write(fs_buffer* b);
int fs_buffer_device_use(fs_buffer* b, uint64_t bytes);
/* Sort the first n keys of `keys` in place on the device (sort_buffer,
 * sort_*_buffer, encode_sort: src/lib.rs:708-785, 1000-1117, 2301-2590);
 * sync == 0 only enqueues on the sorter's stream. */
int fs_sort_buffer(fs_sorter* s, int dtype, fs_buffer* keys, uint64_t n, int sync);
/* Stable pairs form over two buffers (additive: sort_pairs_buffer). */
int fs_sort_pairs_buffer(fs_sorter* s, int dtype, fs_buffer* keys, fs_buffer* vals,
                         uint64_t n, int sync);

/* ---- device-resident sorts (zero-copy path) ----------------------------- */

/* Sort n keys of type `dtype` in place at `keys`: device memory, managed
 * memory, or page-locked host memory (staged through the device).
 * Order: unsigned order for u32/u64, signed for i32/i64, IEEE totalOrder
 * (Rust f32::total_cmp) for f32/f64.  sync != 0 waits for completion and
 * reports device failures; sync == 0 only enqueues (encode_sort semantics:
 * the caller synchronises, e.g. with fs_synchronize).
 * Replaces sort_buffer / sort_*_buffer / encode_sort (src/lib.rs:708-785,
 * 1000-1117, 2301-2346, 2486-2590). */
int fs_sort_keys(fs_sorter* s, int dtype, void* keys, uint64_t n, int sync);

/* Sort (key, u32 value) pairs in place, stably by key (equal keys keep their
 * input order).  New zero-copy form of sort_pairs_* (src/lib.rs:1923-2236,
 * 2826-3015), used by SortBuffer-based pairs sorting. */
int fs_sort_pairs(fs_sorter* s, int dtype, void* keys, uint32_t* vals,
                  uint64_t n, int sync);

/* Write to idx_out the stable sorting permutation of keys (idx_out[i] = index
 * of the i-th smallest key; ties in index order).  `keys` is not modified.
 * n must be <= 2^32.  Replaces argsort_* (src/lib.rs:1675-1921, 2595-2825). */
int fs_argsort(fs_sorter* s, int dtype, const void* keys, uint32_t* idx_out,
               uint64_t n, int sync);

/* Out-of-place form: sorted copy of keys_in written to keys_out (device or
 * managed pointers, n keys each, non-overlapping); keys_in is not modified.
 * The reference's slice API does the same internally -- it copies the slice
 * into its own buffer before sorting (src/lib.rs:800-812) -- but fuses no
 * copy: the first pass reads keys_in and the last pass writes keys_out. */
int fs_sort_keys_copy(fs_sorter* s, int dtype, const void* keys_in,
                      void* keys_out, uint64_t n, int sync);

/* Out-of-place stable pairs sort: (keys_in, vals_in) sorted by key into
 * (keys_out, vals_out); equal keys keep their input order.  vals_in == NULL
 * takes the input positions as values (an argsort that also returns the
 * sorted keys).  Device or managed pointers, no two arrays overlapping; the
 * inputs are not modified.  The first pass reads the inputs and the last
 * pass writes the outputs (no extra copy). */
int fs_sort_pairs_copy(fs_sorter* s, int dtype, const void* keys_in,
                       const uint32_t* vals_in, void* keys_out,
                       uint32_t* vals_out, uint64_t n, int sync);

/* ---- host-slice sorts (sort_u32(&mut [u32]) etc.) ------------------------ */

/* Copy host keys to the device, sort, copy back; synchronous.  Pinned host
 * memory gives full copy bandwidth; pageable memory also works.
 * Replaces sort_u32/i32/f32/u64/i64/f64 (src/lib.rs:791-998, 2238-2485). */
int fs_host_sort_keys(fs_sorter* s, int dtype, void* host_keys, uint64_t n);
/* Length check first (LengthMismatch), then n <= 1 short-cut, as
 * src/lib.rs:1928-1937 orders them. */
int fs_host_sort_pairs(fs_sorter* s, int dtype, void* host_keys,
                       uint64_t n_keys, uint32_t* host_vals, uint64_t n_vals);
int fs_host_argsort(fs_sorter* s, int dtype, const void* host_keys,
                    uint32_t* host_idx_out, uint64_t n);
/* Host out-of-place form of sort_u32 etc.: host_in -> device -> sort ->
 * host_out (host_in untouched); synchronous.  Same copy-in / sort /
 * copy-out sequence as src/lib.rs:791-837. */
int fs_host_sort_keys_copy(fs_sorter* s, int dtype, const void* host_in,
                           void* host_out, uint64_t n);

/* Enqueue an out-of-place sort of n keys in host memory (host_in -> GPU ->
 * sort -> host_out) and return at once.  Consecutive calls overlap: the copy
 * of one call's keys to the GPU runs while the previous call sorts and copies
 * back (the sorter alternates between two device buffers and has copy
 * streams of its own).  host_in and host_out must stay untouched until
 * fs_synchronize returns; page-locked host memory (cudaHostAlloc) lets the
 * copies overlap.  Work enqueued on the sorter's stream before the first call
 * since the last fs_synchronize runs first; fs_synchronize waits for every
 * call and makes later work on the sorter's stream wait for it too.  No counterpart in the reference (its
 * sort_* calls are synchronous); this is the streaming form of
 * fs_host_sort_keys_copy. */
int fs_host_sort_keys_copy_async(fs_sorter* s, int dtype, const void* host_in,
                                 void* host_out, uint64_t n);

/* ---- permutation apply --------------------------------------------------- */

/* dst[i] = src[idx[i]] for i < n: elements of `width` bytes (4 or 8), u32
 * indices into a source of src_n elements; src, idx and dst are device,
 * managed or page-locked host memory (a SortBuffer) of the sorter's device,
 * and dst does not overlap src or idx.  Page-locked operands are staged
 * through device memory on the sorter's stream, except a page-locked source
 * more than 32x the gathered bytes, which the kernel reads in place.  An index >= src_n is skipped and reported as FS_E_GPU_EXECUTION at
 * the next synchronisation.  Replaces sort_gather_values
 * (shaders/sort.metal:792-800) and forge-runtime's GpuGather::gather_u32 /
 * gather_u64 (forge-runtime/src/gather.rs:82-134): applying an argsort
 * permutation to a payload. */
int fs_gather(fs_sorter* s, int width, const void* src, uint64_t src_n,
              const uint32_t* idx, void* dst, uint64_t n, int sync);

/* ---- streams --------------------------------------------------------------- */

/* A non-blocking CUDA stream on `device`, for callers that have no CUDA
 * runtime of their own: the command queue of forge-runtime's ForgeContext
 * (forge-runtime/src/context.rs:16-55), which sorters (fs_create) and
 * gathers then share so that their work runs in submission order.
 * fs_stream_synchronize is the analogue of commit + waitUntilCompleted
 * (forge-runtime/src/pipeline.rs:129-139).  Failures: FS_E_DEVICE_NOT_FOUND,
 * FS_E_GPU_EXECUTION; text via fs_last_error(NULL). */
int fs_stream_create(int device, void** stream);
int fs_stream_synchronize(void* stream);
int fs_stream_destroy(void* stream);

/* ---- per-kernel timing ---------------------------------------------------- */

/* on != 0: record a CUDA event pair around every kernel the sorter launches,
 * on its own stream (the forge-primitives GpuTimer analogue,
 * forge-primitives/src/timing.rs:9-47).  Off by default. */
int fs_set_kernel_timing(fs_sorter* s, int on);
/* After a synchronous sort with timing on: write up to `cap` durations in ms
 * and return how many were written (negative fs_status on failure).  Order:
 * first count (digit-0 counts + which digits vary), plan, then per digit pass
 * (count + slice scan, scatter), then finalize -- 3 + 2*P entries for
 * P = key bytes. */
int fs_last_kernel_times(fs_sorter* s, float* ms, int cap);

/* ---- multi-GPU sample sort building block -------------------------------- */

/* Stable partition of n keys (device pointers keys_in -> keys_out, which must
 * differ) into nsplit+1 contiguous buckets.  Bucket b holds the keys whose
 * (key, global position) pair is >= splitter b-1 and < splitter b, in the
 * same order as fs_sort_keys; a key's global position is gpos_base + its index.
 * splitter_keys (nsplit keys of `dtype`, raw bits) and splitter_gpos
 * (nsplit u64) are device pointers, ascending by (key, position).  Writes the
 * bucket sizes to bucket_counts (device, nsplit+1 u64).  0 <= nsplit <= 255.
 * No counterpart in the reference (it has no multi-GPU path); this is the
 * partition step of the 1-8 GPU sample sort. */
int fs_partition(fs_sorter* s, int dtype, const void* keys_in, uint64_t n,
                 uint64_t gpos_base, const void* splitter_keys,
                 const uint64_t* splitter_gpos, int nsplit, void* keys_out,
                 uint64_t* bucket_counts, int sync);

/* Sample-sort dispatch: partition and exchange in one pass over peer memory.
 * Step 1 counts: writes the nsplit+1 bucket sizes of the n keys to
 * bucket_counts_host (host memory) and keeps the per-slice counts in the
 * sorter's scratch; waits for the stream.  Same buckets as fs_partition. */
int fs_partition_count(fs_sorter* s, int dtype, const void* keys, uint64_t n,
                       uint64_t gpos_base, const void* splitter_keys,
                       const uint64_t* splitter_gpos, int nsplit,
                       uint64_t* bucket_counts_host);
/* Step 2 stores every key of bucket b at bucket_dst[b][0 .. count_b), in no
 * particular order within the bucket (keys only: the receiving rank's sort
 * orders them, and equal keys are identical bits; from 3 buckets up the pass
 * ranks with shared atomics) -- bucket_dst (host array of nsplit+1 device
 * pointers) may point
 * into other GPUs' memory (fs_ipc_open), which the kernel writes with plain
 * stores over NVLink; it makes those stores visible system-wide before it
 * ends.  Must directly follow fs_partition_count on the same sorter with the
 * same keys, n, dtype and splitters.  The caller orders the peers' reads of
 * their inboxes after this call (e.g. a stream-ordered collective). */
int fs_partition_dispatch(fs_sorter* s, int dtype, const void* keys, uint64_t n,
                          uint64_t gpos_base, const void* splitter_keys,
                          const uint64_t* splitter_gpos, int nsplit,
                          void* const* bucket_dst, int sync);

/* fs_partition_dispatch with a u32 payload, for a multi-GPU sort_pairs or
 * argsort: value i travels with key i to value_dst[b] at the key's position
 * in bucket_dst[b].  vals == NULL sends each key's global position
 * gpos_base + i instead (gpos_base + n <= 2^32).  Same pairing rule with
 * fs_partition_count; within a bucket the keys keep their input order, so a
 * stable local sort of the received pairs gives the globally stable order. */
int fs_partition_dispatch_pairs(fs_sorter* s, int dtype, const void* keys,
                                const uint32_t* vals, uint64_t n,
                                uint64_t gpos_base, const void* splitter_keys,
                                const uint64_t* splitter_gpos, int nsplit,
                                void* const* bucket_dst,
                                uint32_t* const* value_dst, int sync);

/* The same two steps without host round trips, for a sample-sort step that
 * waits on the host once (to size the receive buffers).
 * fs_partition_count_async: as fs_partition_count, but the bucket sizes go
 * to device memory bucket_counts_dev (nsplit+1 u64), stream-ordered, and the
 * call returns at once.
 * fs_partition_dispatch_matrix: as fs_partition_dispatch(_pairs) (with a
 * payload the keys keep their input order within a bucket, without one they
 * need not), with the
 * destinations computed on the device: send_matrix (device, G x G u64,
 * G = nsplit+1, row r = the bucket sizes rank r counted, e.g. the counts
 * all-gathered in rank order) and this rank's index `rank` give
 * bucket_dst[b] = inbox_keys[b] + (keys that ranks below `rank` send to
 * rank b), and likewise inbox_vals[b] for the values (payload != 0; vals
 * NULL sends global positions).  inbox_keys / inbox_vals: host arrays of G
 * device pointers (peers' inboxes, fs_ipc_open).  Must follow
 * fs_partition_count_async or fs_partition_count of the same keys. */
int fs_partition_count_async(fs_sorter* s, int dtype, const void* keys,
                             uint64_t n, uint64_t gpos_base,
                             const void* splitter_keys,
                             const uint64_t* splitter_gpos, int nsplit,
                             uint64_t* bucket_counts_dev);
int fs_partition_dispatch_matrix(fs_sorter* s, int dtype, const void* keys,
                                 const uint32_t* vals, int payload, uint64_t n,
                                 uint64_t gpos_base, const void* splitter_keys,
                                 const uint64_t* splitter_gpos, int nsplit,
                                 const uint64_t* send_matrix, int rank,
                                 void* const* inbox_keys,
                                 uint32_t* const* inbox_vals, int sync);

/* CUDA IPC for the dispatch inboxes (one process per GPU): export a handle to
 * device memory from cudaMalloc (fs_alloc with managed = 0), open a peer's
 * handle into this process (peer access enabled lazily), close it again
 * before the owner frees the memory. */
#define FS_IPC_HANDLE_BYTES 64
int fs_ipc_export(fs_sorter* s, void* dev_ptr, void* handle_out);
int fs_ipc_open(fs_sorter* s, const void* handle, void** peer_ptr);
int fs_ipc_close(fs_sorter* s, void* peer_ptr);

/* ---- several GPUs of one process (MultiGpuSorter) ----------------------- */

/* The sample sort driven from one process: one sorter (own stream) per
 * device, peer access enabled between every pair; fails with
 * FS_E_DEVICE_NOT_FOUND when a pair cannot reach each other.  1 <= g <= 16
 * distinct device ordinals.  No counterpart in the reference (single-device
 * only); the one-process-per-GPU form of the same algorithm is the Python
 * SampleSorter over torch.distributed. */
typedef struct fs_mg fs_mg;
int fs_mg_create(const int* devices, int g, fs_mg** out);
int fs_mg_destroy(fs_mg* mg);
const char* fs_mg_last_error(const fs_mg* mg);

/* Sort the concatenation shards[0] .. shards[g-1] (shard i: shard_n[i] keys
 * of `dtype` in device memory of devices[i], ready on that device's legacy
 * default stream; not modified).  On return out[i] (device memory of
 * devices[i], room for out_cap[i] keys) holds the i-th piece of the sorted
 * sequence and out_n[i] its length: concatenating the pieces in device order
 * gives the sorted keys, bit-exact with fs_sort_keys on the whole input.
 * Splitters come from regular samples with (key, global position) order, so
 * pieces stay within a few percent of the mean size even for skewed or
 * all-equal keys; if a piece would exceed its out_cap, nothing is sorted,
 * out_n holds the sizes needed and the call returns FS_E_INVALID. */
int fs_mg_sort_keys(fs_mg* mg, int dtype, void* const* shards,
                    const uint64_t* shard_n, void* const* out,
                    const uint64_t* out_cap, uint64_t* out_n);

/* fs_mg_sort_keys with a u32 payload: a stable multi-GPU sort_pairs, or an
 * argsort.  vals[i] (device memory of devices[i], shard_n[i] values) travels
 * with shard i's keys; vals == NULL sends each key's global position instead
 * (position = its index in the concatenated shards; at most 2^32 keys in
 * total).  out_vals[i] (device memory of devices[i], room for out_cap[i]
 * values) receives piece i's values.  Equal keys keep their global input
 * order.  Same sizing rule as fs_mg_sort_keys. */
int fs_mg_sort_pairs(fs_mg* mg, int dtype, void* const* shards,
                     const uint32_t* const* vals, const uint64_t* shard_n,
                     void* const* out, uint32_t* const* out_vals,
                     const uint64_t* out_cap, uint64_t* out_n);

/* ---- allocation-free form ------------------------------------------------ */

/* Sort n keys in place at `keys` (device memory of the current device),
 * enqueued on `stream` (a cudaStream_t; NULL = legacy default stream), then
 * wait for that stream and report device-side failures.  Same order as
 * fs_sort_keys.
 *
 * No counterpart in the reference.  This entry point allocates nothing -- no
 * cudaMalloc, cudaFree, pinned host memory or allocating library routine, and
 * no sorter object -- for callers that must not allocate: code running under
 * a fixed device-memory budget or a caching allocator that owns all device
 * memory, host threads that must not block in the driver's allocator, and
 * plugins embedded in runtimes that forbid device allocations at call time.
 * Its scratch is one fixed device array inside this library, sized for 4 MiB
 * of keys (2^20 u32/i32/f32 or 2^19 u64/i64/f64 keys); larger n returns
 * FS_E_INVALID with the limit in fs_last_error(NULL).  Every GPU that loads
 * the library holds that array (about 4.6 MB) until the process exits.
 *
 * The call is synchronous: it returns after the sort has finished on
 * `stream` (it waits for the stream to read back the device error word).
 * Device waits are bounded by FORGESORT_WAIT_TIMEOUT_MS (default 2 s), as
 * for sorters.  The first call on a device looks up the array's device
 * address (with that device current) and caches it for the process; make
 * that first call before any stream capture, and do not keep using the
 * library across a cudaDeviceReset of that device.  All calls share the one
 * array, which keeps the previous call's contents (each call clears what
 * must start at zero): calls that overlap on the GPU (other streams or host
 * threads, same device) race and corrupt each other's results, so serialise
 * them.  Errors: text in fs_last_error(NULL). */
int fs_sort_keys_noalloc(int dtype, void* keys, uint64_t n, void* stream);

/* ---- introspection ------------------------------------------------------- */

/* Bytes of device scratch the sorter holds right now (grow-only arena,
 * the analogue of ensure_buffers at src/lib.rs:1120-1289). */
uint64_t fs_scratch_bytes(const fs_sorter* s);
/* Number of kernels the last sort enqueued. */
int fs_last_launch_count(const fs_sorter* s);
/* ABI version (FS_ABI_VERSION). */
int fs_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FORGESORT_H */
