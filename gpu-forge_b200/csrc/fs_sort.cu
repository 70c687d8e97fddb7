// fs_sort.cu -- host orchestration and the C ABI (include/forgesort.h) of the
// single-GPU sort and the sample sort's partition kernels.  One fs_sorter =
// one device + one stream + a grow-only scratch arena; every sort is
// enqueued as
//   first count -> plan -> P x (count, slice scan, scatter) -> finalize
// on that stream (P = key bytes), with no host round trip in between.
#include "forgesort.h"
#include "forgesort_bench.h"
#include "fs_resident.cuh"
#include "fs_hoststage.h"
#include "fs_kernels.cuh"
#include "fs_histfill.cuh"

#include <cstdarg>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>

using namespace fs;

struct fs_sorter {
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t own_stream = nullptr;
  SortCtl* ctl = nullptr;
  int* host_err = nullptr;      // mapped pinned word written by k_finalize
  int* host_err_dev = nullptr;  // its device alias
  void* counts = nullptr;      // [slices][256] u32 per-pass slice counts
  size_t counts_bytes = 0;
  void* offsets = nullptr;     // [slices][256] u32 per-pass output offsets
  size_t offsets_bytes = 0;
  void* kother = nullptr;  // n keys of scratch (the OTHER slot)
  size_t kother_bytes = 0;
  void* kfinal2 = nullptr;  // argsort: keys are not an output, so FINAL is scratch too
  size_t kfinal2_bytes = 0;
  void* vother = nullptr;
  size_t vother_bytes = 0;
  void* dkeys = nullptr;  // staging for the host-slice API
  size_t dkeys_bytes = 0;
  void* dvals = nullptr;
  size_t dvals_bytes = 0;
  void* dst_tab = nullptr;  // sample-sort dispatch: 256 destination pointers
  // single-launch sort (k_resident_sort): two accumulator sets used by
  // alternate launches, per-CTA digit counts
  void* res_acc = nullptr;
  size_t res_acc_bytes = 0;
  void* res_counts = nullptr;
  size_t res_counts_bytes = 0;
  int res_parity = 0;
  void* hf = nullptr;  // histogram fill of keys-only 32-bit sorts (HfCtl)
  size_t hf_bytes = 0;
  uint64_t h16_min = 1ull << 30;  // keys-only 32-bit sorts of at least this many keys sort the top 16
                                  // bits by passes and the low 16 by the histogram fill
                                  // (FORGESORT_H16_MIN_KEYS; 0: never)
  // after a failure the device error word may be left set: the next sort
  // clears it first
  bool ctl_dirty = true;
  uint64_t coop_max_bytes = 8ull << 20;  // keys-only 32-bit sorts up to this many key bytes run as
                                         // one cooperative launch (FORGESORT_COOP_MAX_BYTES; 0: off)
  uint32_t small_max = SMALL_N_MAX;  // single-CTA sorts up to this n (FORGESORT_SMALL_SORT);
                                     // with a payload up to min(small_max, SMALL_N_PAYLOAD_MAX)
  // fs_host_sort_keys_copy_async: two device buffers used in turn, and copy
  // streams of their own so one call's copies overlap the next call's work
  struct PipeSlot {
    void* dkeys = nullptr;
    size_t bytes = 0;
    cudaEvent_t in_done = nullptr, sorted = nullptr, out_done = nullptr;
    bool used = false;
  } pipe[2];
  int pipe_next = 0;
  bool pipe_open = false;  // async calls since the last fs_synchronize
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t pipe_start = nullptr;
  // what the last fs_partition_count counted (fs_partition_dispatch must match)
  struct {
    bool ready = false;
    int dtype = -1, nsplit = -1;
    const void* keys = nullptr;
    uint64_t n = 0;
  } part;
  int sm_count = 0;
  uint64_t timeout_ns = 2000000000ull;
  int last_launches = 0;
  bool timing = false;  // fs_set_kernel_timing
  static constexpr int MAX_TIMED = 24;
  cudaEvent_t ev[2 * MAX_TIMED] = {};
  int ev_used = 0;
  HostStage stage;  // page-locked chunk ring for pageable host-slice copies
  int test_withhold = 0;    // fs_test_inject(FS_TEST_WITHHOLD_COPY): next radix sort
  int test_fail_alloc = 0;  // fs_test_inject(FS_TEST_FAIL_ALLOC): countdown to a failed growth
  int test_skip_arrival = 0;  // fs_test_inject(FS_TEST_SKIP_ARRIVAL): next single-launch sort
  std::unordered_map<void*, size_t> allocs;  // fs_alloc'd pointers -> bytes
  std::unordered_map<void*, int> managed;
  std::string err;
};

// A SortBuffer: device memory plus a page-locked host mirror, kept coherent
// lazily.  Sorts run on the device copy and copy nothing back; the host side
// is brought up to date only when the host reads it, and the device side
// only for the bytes a sort (or a device user) needs after the host wrote.
struct fs_buffer {
  int device = 0;
  void* dev = nullptr;
  void* host = nullptr;
  uint64_t bytes = 0;
  uint64_t dev_valid = 0;   // leading bytes the device copy holds as the host last wrote them
  uint64_t dev_newer = 0;   // leading bytes device work may have changed since the host last read
  cudaEvent_t done = nullptr;  // recorded after the last sort that touched the buffer
  bool pending = false;        // `done` marks work not yet waited for
  bool any_stream = false;     // handed out for device use on a stream not known here
};

namespace {

thread_local std::string g_create_err;

int fail(fs_sorter* s, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (s) {
    s->err = buf;
    s->ctl_dirty = true;  // a failed call may leave the device error word set
  } else {
    g_create_err = buf;
  }
  return code;
}

int cuda_fail(fs_sorter* s, cudaError_t e, const char* what) {
  cudaGetLastError();  // clear sticky-free errors
  if (e == cudaErrorMemoryAllocation) return fail(s, FS_E_OOM, "%s: %s", what, cudaGetErrorString(e));
  if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidKernelImage ||
      e == cudaErrorSharedObjectInitFailed)
    return fail(s, FS_E_KERNEL_IMAGE, "%s: %s", what, cudaGetErrorString(e));
  return fail(s, FS_E_GPU_EXECUTION, "%s: %s", what, cudaGetErrorString(e));
}

#define FS_CUDA(s, call)                                       \
  do {                                                         \
    cudaError_t e_ = (call);                                   \
    if (e_ != cudaSuccess) return cuda_fail((s), e_, #call);   \
  } while (0)

// Scatter tile shapes (threads x keys per thread, resident CTAs per SM,
// bulk-copy slots, 16-bit packed ranks).  The stable u32 pass runs with one
// copy slot and packed ranks at 4 CTAs/SM: measured on one B200, 2^30 u32
// keys, 4.23 -> 3.95 ms per stable pass (sort 18.4 -> 17.5 ms on that box);
// one slot made the unstable pass slower (2.9 -> 3.2-3.6 ms), so it keeps two.
// StableCfg ranks with the ballot multisplit (every pass of argsort / pairs,
// and the passes after the first of a keys-only sort); UnstableCfg ranks
// with one shared atomic per key (the first executed pass of a keys-only
// sort).  Measured on B200 with 2^30 u32 keys: stable 256x16 at 3 CTAs/SM
// 3.96 ms/pass (256x12 at 4: 4.67, 256x24 at 2: 4.29), unstable 256x32 at
// 2 CTAs/SM 2.58 ms/pass (256x24 at 2: 2.79).
#ifndef FS_U32_STABLE_IPT
#define FS_U32_STABLE_IPT 16
#endif
#ifndef FS_U32_STABLE_MINB
#define FS_U32_STABLE_MINB 4
#endif
#ifndef FS_U32_UNSTABLE_IPT
#define FS_U32_UNSTABLE_IPT 32
#endif
#ifndef FS_U32_UNSTABLE_MINB
#define FS_U32_UNSTABLE_MINB 2
#endif
template <typename K, bool VALS> struct StableCfg;
#ifndef FS_U32_STABLE_SLOTS
#define FS_U32_STABLE_SLOTS 1
#endif
#ifndef FS_U32_UNSTABLE_SLOTS
#define FS_U32_UNSTABLE_SLOTS 2
#endif
#ifndef FS_STABLE_PACK
#define FS_STABLE_PACK 1
#endif
#ifndef FS_UNSTABLE_PACK
#define FS_UNSTABLE_PACK 0
#endif
template <> struct StableCfg<uint32_t, false> {
  static constexpr int BLOCK = 256, IPT = FS_U32_STABLE_IPT, MINB = FS_U32_STABLE_MINB, SLOTS = FS_U32_STABLE_SLOTS;
  static constexpr bool PACK = FS_STABLE_PACK != 0;
};
template <> struct StableCfg<uint32_t, true> {
  static constexpr int BLOCK = 256, IPT = 16, MINB = 2, SLOTS = 2;
  static constexpr bool PACK = FS_STABLE_PACK != 0;
};
template <> struct StableCfg<uint64_t, false> {
  static constexpr int BLOCK = 256, IPT = 16, MINB = 2, SLOTS = 2;
  static constexpr bool PACK = FS_STABLE_PACK != 0;
};
template <> struct StableCfg<uint64_t, true> {
  static constexpr int BLOCK = 256, IPT = 8, MINB = 2, SLOTS = 2;
  static constexpr bool PACK = FS_STABLE_PACK != 0;
};
template <typename K> struct UnstableCfg;
template <> struct UnstableCfg<uint32_t> {
  static constexpr int BLOCK = 256, IPT = FS_U32_UNSTABLE_IPT, MINB = FS_U32_UNSTABLE_MINB,
                       SLOTS = FS_U32_UNSTABLE_SLOTS;
  static constexpr bool PACK = FS_UNSTABLE_PACK != 0;
};
template <> struct UnstableCfg<uint64_t> {
  static constexpr int BLOCK = 256, IPT = 16, MINB = 2, SLOTS = 2;
  static constexpr bool PACK = FS_UNSTABLE_PACK != 0;
};
// Sample-sort partition / dispatch pass: the stable tile with room for the
// splitter search (2 CTAs/SM; same tile as StableCfg<K, false>).
#ifndef FS_PART_MINB
#define FS_PART_MINB 4
#endif
#ifndef FS_PART_IPT
#define FS_PART_IPT 8
#endif
template <typename K> struct PartCfg {
  // 64-bit keys need the registers of 3 CTAs/SM (the splitters sit in registers)
  static constexpr int BLOCK = 256, IPT = FS_PART_IPT, MINB = sizeof(K) == 8 ? 3 : FS_PART_MINB, SLOTS = 2;
  static constexpr bool PACK = false;
  static_assert(StableCfg<K, false>::BLOCK * StableCfg<K, false>::IPT % (BLOCK * IPT) == 0,
                "partition tiles must divide the slice unit");
};
template <typename C> constexpr uint64_t tile_of() { return (uint64_t)C::BLOCK * C::IPT; }
constexpr uint64_t gcd64(uint64_t a, uint64_t b) { return b ? gcd64(b, a % b) : a; }
constexpr uint64_t lcm64(uint64_t a, uint64_t b) { return a / gcd64(a, b) * b; }

// Slices per SM: a multiple of 2, 3 and 4 so the scatter (2 or 3 CTAs/SM) and
// histogram/count (4 CTAs/SM) grids split the slices evenly.
constexpr int SLICES_PER_SM = 12;

constexpr int HIST_BLOCK = 512;  // histogram / count kernels: more loads in flight per SM

int key_bytes_of(int dtype) { return dtype >= FS_U64 ? 8 : 4; }

// Device ordinals the per-device caches below cover (fs_create refuses more).
constexpr int MAX_DEVICES = 64;

// Bound on every device-side wait: FORGESORT_WAIT_TIMEOUT_MS, default 2 s.
uint64_t wait_timeout_ns_env() {
  if (const char* t = getenv("FORGESORT_WAIT_TIMEOUT_MS")) {
    const long long ms = atoll(t);
    if (ms > 0) return (uint64_t)ms * 1000000ull;
  }
  return 2000000000ull;
}

int grow(fs_sorter* s, void** p, size_t* cap, size_t need, bool zero) {
  if (*cap >= need) return FS_OK;
  if (*p) {
    FS_CUDA(s, cudaStreamSynchronize(s->stream));
    FS_CUDA(s, cudaFree(*p));
    *p = nullptr;
    *cap = 0;
  }
  if (s && s->test_fail_alloc > 0 && --s->test_fail_alloc == 0)
    return fail(s, FS_E_OOM, "device allocation of %zu bytes failed: out of memory (injected by fs_test_inject)",
                need);
  cudaError_t e = cudaMalloc(p, need);
  if (e != cudaSuccess) {
    *p = nullptr;
    cudaGetLastError();
    return fail(s, FS_E_OOM, "device allocation of %zu bytes failed: %s", need, cudaGetErrorString(e));
  }
  *cap = need;
  if (zero) FS_CUDA(s, cudaMemsetAsync(*p, 0, need, s->stream));
  return FS_OK;
}

// Prefetch managed memory to the device before the kernels touch it (the
// SortBuffer path: host writes, then sorts in place).
int prepare_ptr(fs_sorter* s, const void* p, size_t bytes, const char* what) {
  cudaPointerAttributes at{};
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(s, FS_E_INVALID, "%s: not a CUDA pointer", what);
  }
  if (at.type == cudaMemoryTypeManaged) {
    FS_CUDA(s, cudaMemPrefetchAsync(p, bytes, s->device, s->stream));
    return FS_OK;
  }
  if (at.type != cudaMemoryTypeDevice)
    return fail(s, FS_E_INVALID, "%s: expected device or managed memory", what);
  if (at.device != s->device)
    return fail(s, FS_E_INVALID, "%s: pointer is on device %d, sorter on device %d", what, at.device,
                s->device);
  return FS_OK;
}

// Page-locked host memory (a SortBuffer, or any cudaHostAlloc buffer) is
// sorted through a device staging buffer: copied in, sorted in HBM, copied
// back, all on the sorter's stream.  is_pinned_host tells the kinds apart.
bool is_pinned_host(const void* p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

// The device pointer the kernels use for `p`: p itself (device or managed,
// checked and prefetched by prepare_ptr), or the staging buffer *buf, grown
// to `bytes` and filled from p when copy_in.
int device_view(fs_sorter* s, const void* p, size_t bytes, const char* what, void** buf, size_t* cap, bool copy_in,
                void** out) {
  if (is_pinned_host(p)) {
    int rc = grow(s, buf, cap, bytes, false);
    if (rc) return rc;
    if (copy_in) FS_CUDA(s, cudaMemcpyAsync(*buf, p, bytes, cudaMemcpyHostToDevice, s->stream));
    *out = *buf;
    return FS_OK;
  }
  *out = const_cast<void*>(p);
  return prepare_ptr(s, p, bytes, what);
}

// Host-slice copies.  Page-locked host memory is copied directly; pageable
// memory of at least STAGE_MIN bytes goes through the sorter's chunk ring
// (fs_hoststage.h), below that the driver's own path is as fast.
constexpr size_t STAGE_MIN = 1u << 20;

int host_to_device(fs_sorter* s, void* dev, const void* host, size_t bytes) {
  if (bytes < STAGE_MIN || is_pinned_host(host)) {
    FS_CUDA(s, cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, s->stream));
    return FS_OK;
  }
  FS_CUDA(s, s->stage.to_device(dev, host, bytes, s->stream));
  return FS_OK;
}

// Enqueued after the sort; for pageable memory this waits until the bytes
// have landed (the caller synchronises the stream next anyway).
int device_to_host(fs_sorter* s, void* host, const void* dev, size_t bytes) {
  if (bytes < STAGE_MIN || is_pinned_host(host)) {
    FS_CUDA(s, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, s->stream));
    return FS_OK;
  }
  FS_CUDA(s, s->stage.to_host(host, dev, bytes, s->stream));
  return FS_OK;
}

int copy_back(fs_sorter* s, void* host, const void* dev, size_t bytes) {
  if (host != dev) FS_CUDA(s, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, s->stream));
  return FS_OK;
}

// After a synchronous sort of managed memory (the SortBuffer path), move the
// result back to the host before returning: the caller reads it there next,
// and reading managed pages that still live on the GPU migrates them one
// fault at a time (measured 1.6 GB/s for a 1 GB buffer, against a full-rate
// prefetch).  Other memory is left alone.
int prefetch_to_host(fs_sorter* s, const void* p, size_t bytes) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return FS_OK;
  }
  if (at.type == cudaMemoryTypeManaged) FS_CUDA(s, cudaMemPrefetchAsync(p, bytes, cudaCpuDeviceId, s->stream));
  return FS_OK;
}

// Everything one enqueued sort needs: device and stream, the control block,
// scratch buffers that are already large enough, and where k_finalize
// reports device errors.  `s` (may be null) receives error text and owns the
// kernel-timing events.
struct Exec {
  int device;
  cudaStream_t stream;
  int sm_count;
  uint64_t timeout_ns;
  SortCtl* ctl;
  int* err_out;
  uint32_t* counts;      // >= slices * 256 words
  uint32_t* offsets;     // >= slices * 256 words
  HfCtl* hf;             // histogram fill scratch (h16 plans only)
  fs_sorter* s;
};

// Event pair around each launch when kernel timing is on.
void t_begin(const Exec& e) {
  fs_sorter* s = e.s;
  if (s && s->timing && s->ev_used < fs_sorter::MAX_TIMED) cudaEventRecord(s->ev[2 * s->ev_used], e.stream);
}
void t_end(const Exec& e) {
  fs_sorter* s = e.s;
  if (s && s->timing && s->ev_used < fs_sorter::MAX_TIMED) cudaEventRecord(s->ev[2 * s->ev_used++ + 1], e.stream);
}

// Resident CTAs per SM, or -(fs_status) on failure.
template <typename Kern>
int blocks_per_sm(fs_sorter* s, Kern k, int block, size_t smem) {
  int b = 0;
  const cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, block, smem);
  if (err != cudaSuccess) return -cuda_fail(s, err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  return b > 0 ? b : 1;
}

// Resident CTAs per SM of a scatter instantiation (cached per process; every
// device here is the same architecture).  Sets the kernel's shared-memory
// limit on the current device the first time; allocates nothing.
template <typename K, bool VALS, int XF, typename C, int MODE, typename D>
int scatter_occupancy(const Exec& e) {
  using Ly = ScatterLayout<K, VALS, C::BLOCK, C::IPT, D::STAGE, D::DIGITS, C::SLOTS>;
  auto kern = k_scatter<K, VALS, XF, C::BLOCK, C::IPT, C::MINB, MODE, D, C::SLOTS, C::PACK>;
  // sorters on several host threads may get here at once: the attribute
  // call is idempotent, the cache words are atomic
  static std::atomic<bool> configured[MAX_DEVICES];  // per device (the attribute is per context)
  static std::atomic<int> bps{0};
  if (e.device < 0 || e.device >= MAX_DEVICES)
    return -fail(e.s, FS_E_INVALID, "device %d outside [0, %d)", e.device, MAX_DEVICES);
  if (!configured[e.device].load()) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ly::BYTES);
    if (err != cudaSuccess) return -cuda_fail(e.s, err, "cudaFuncSetAttribute");
    const int b = blocks_per_sm(e.s, kern, C::BLOCK, Ly::BYTES);
    if (b < 0) return b;
    bps.store(b);
    configured[e.device].store(true);
  }
  return bps.load();
}

// Kernels of one sort follow each other on the sorter's stream.  Launched
// with programmatic stream serialization, each is scheduled while its
// predecessor drains instead of after it has finished; every such kernel
// opens with chain_wait(), which holds it until the predecessor's writes are
// visible, so results are unchanged.  FORGESORT_CHAIN_LAUNCH=0 launches
// them plainly.
bool chain_launch_on() {
  static const bool on = [] {
    const char* t = getenv("FORGESORT_CHAIN_LAUNCH");
    return !(t && atoi(t) == 0);
  }();
  return on;
}

template <typename... KArgs, typename... Args>
int chain_launch(const Exec& e, void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e.stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = chain_launch_on() ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, args...);
  if (err != cudaSuccess) return cuda_fail(e.s, err, "cudaLaunchKernelEx");
  return FS_OK;
}

template <typename K, bool VALS, int XF, typename C, int MODE, typename D>
int launch_scatter(const Exec& e, int pass, uint64_t n, const Slices& sl, const D& dfn, uint64_t gpos_base) {
  using Ly = ScatterLayout<K, VALS, C::BLOCK, C::IPT, D::STAGE, D::DIGITS, C::SLOTS>;
  const int bps = scatter_occupancy<K, VALS, XF, C, MODE, D>(e);
  if (bps < 0) return -bps;
  const uint64_t cap = (uint64_t)bps * e.sm_count;
  const unsigned grid = (unsigned)(sl.count < cap ? sl.count : cap);
  return chain_launch(e, k_scatter<K, VALS, XF, C::BLOCK, C::IPT, C::MINB, MODE, D, C::SLOTS, C::PACK>, grid, C::BLOCK,
                      Ly::BYTES,
                      e.ctl, pass, n, sl, static_cast<const uint32_t*>(e.offsets), e.timeout_ns, dfn, gpos_base);
}

// Cut n keys into contiguous slices of whole `unit`-key blocks (a multiple of
// every tile size used on them), about SLICES_PER_SM per SM.
Slices make_slices(const Exec& e, uint64_t n, uint64_t unit) {
  const uint64_t units = (n + unit - 1) / unit;
  const uint64_t target = (uint64_t)SLICES_PER_SM * e.sm_count;
  const uint64_t ups = (units + target - 1) / target;  // units per slice
  Slices sl{};
  sl.keys_per_slice = ups * unit;
  sl.count = (uint32_t)((units + ups - 1) / ups);
  return sl;
}

// Grid of the histogram / count kernels: 4 CTAs of HIST_BLOCK threads per SM.
unsigned stream_grid(const Exec& e, const Slices& sl) {
  const uint64_t cap = (uint64_t)4 * e.sm_count;
  return (unsigned)(sl.count < cap ? sl.count : cap);
}

template <typename K, int XF>
int enqueue_sort(const Exec& e, const PlanArgs& a, const Slices& sl, int* launches) {
  constexpr int P = (int)sizeof(K);
  const uint64_t n = a.n;
  const unsigned sg = stream_grid(e, sl);
  if (e.s) e.s->ev_used = 0;
  // 1. clear the accumulators; digit-0 slice counts + which digits vary
  t_begin(e);
  FS_CUDA(e.s, cudaMemsetAsync(e.ctl, 0, CTL_ACCUM_BYTES, e.stream));
  if ((reinterpret_cast<uintptr_t>(a.kin) & 15) == 0)
    k_first_count<K, XF, HIST_BLOCK, true>
        <<<sg, HIST_BLOCK, 0, e.stream>>>(static_cast<const K*>(a.kin), n, e.ctl, sl, e.counts, 0);
  else
    k_first_count<K, XF, HIST_BLOCK, false>
        <<<sg, HIST_BLOCK, 0, e.stream>>>(static_cast<const K*>(a.kin), n, e.ctl, sl, e.counts, 0);
  t_end(e);
  // 2. plan
  PlanArgs pa = a;
  pa.trivial_from_bits = 1;
  int rc;
  t_begin(e);
  if ((rc = chain_launch(e, k_plan, 1, RADIX, 0, e.ctl, pa))) return rc;
  t_end(e);
  // 3. passes: count (pass 0 was counted above), slice scan, scatter
  int nl = 2;
  for (int p = 0; p < P; ++p) {
    t_begin(e);
    if (p > 0) {
      if ((rc = chain_launch(e, k_count<K, XF, HIST_BLOCK>, sg, HIST_BLOCK, 0, e.ctl, p, n, sl, e.counts))) return rc;
      ++nl;
    }
    if ((rc = chain_launch(e, k_slice_scan, SCAN_GROUPS, SCAN_WARPS * 32, 0, e.ctl, p, sl,
                           static_cast<const uint32_t*>(e.counts), e.offsets, 0)))
      return rc;
    t_end(e);
    t_begin(e);
    const RadixDigit dg{p * RADIX_BITS};
    if (a.has_vals) {
      rc = launch_scatter<K, true, XF, StableCfg<K, true>, SCATTER_ANY>(e, p, n, sl, dg, 0ull);
    } else if (a.unstable_first && p == 0) {
      // pass 0, when it runs, is the first executed pass: it may rank
      // unstably.  (If it is trivial, the stable pass 1 kernel ranks pass 1.)
      rc = launch_scatter<K, false, XF, UnstableCfg<K>, SCATTER_UNSTABLE>(e, p, n, sl, dg, 0ull);
    } else if (a.unstable_first && sizeof(K) == 4 && p < P - 1) {
      // keys-only 32-bit passes 1 and 2: rounds whose keys agree on the lower
      // bits rank by atomics (PD_SORTED_BELOW), most rounds while the lower
      // bits are 8 or 16, so they take the first pass's wide tile; the top
      // pass (24 lower bits, rounds rarely agree) keeps the stable tile
      rc = launch_scatter<K, false, XF, UnstableCfg<K>, SCATTER_ANY>(e, p, n, sl, dg, 0ull);
    } else {
      rc = launch_scatter<K, false, XF, StableCfg<K, false>, SCATTER_ANY>(e, p, n, sl, dg, 0ull);
    }
    nl += 2;  // scan, scatter
    t_end(e);
    if (rc) return rc;
  }
  // 4. finalize
  uint64_t fb = (n + 255) / 256;
  const uint64_t fcap = (uint64_t)e.sm_count * 4;
  t_begin(e);
  if ((rc = chain_launch(e, k_finalize<K>, (unsigned)(fb < fcap ? fb : fcap), 256, 0, e.ctl, n, e.err_out)))
    return rc;
  t_end(e);
  if (launches) *launches = nl + 1;
  FS_CUDA(e.s, cudaGetLastError());
  return FS_OK;
}

// Keys-only 32-bit sort of many keys: the passes of digits 2 and 3 group the
// keys by their top 16 bits (digit 2 ranks unstably, being the first pass
// that can run; digit 3 stably), then the histogram fill sorts every group by
// its low 16 bits (fs_histfill.cuh).  Launches: first count (digit 2), plan,
// scan + scatter (digit 2), count + scan + scatter (digit 3), bounds, plan of
// the large groups, the per-group fill, the large groups' zero / count / scan
// / fill, finalize.
template <int XF>
int enqueue_h16(const Exec& e, const PlanArgs& a, const Slices& sl, int* launches) {
  using K = uint32_t;
  const uint64_t n = a.n;
  const unsigned sg = stream_grid(e, sl);
  if (e.s) e.s->ev_used = 0;
  t_begin(e);
  FS_CUDA(e.s, cudaMemsetAsync(e.ctl, 0, CTL_ACCUM_BYTES, e.stream));
  if ((reinterpret_cast<uintptr_t>(a.kin) & 15) == 0)
    k_first_count<K, XF, HIST_BLOCK, true>
        <<<sg, HIST_BLOCK, 0, e.stream>>>(static_cast<const K*>(a.kin), n, e.ctl, sl, e.counts, 2);
  else
    k_first_count<K, XF, HIST_BLOCK, false>
        <<<sg, HIST_BLOCK, 0, e.stream>>>(static_cast<const K*>(a.kin), n, e.ctl, sl, e.counts, 2);
  t_end(e);
  PlanArgs pa = a;
  pa.trivial_from_bits = 1;
  pa.h16 = 1;
  int rc;
  t_begin(e);
  if ((rc = chain_launch(e, k_plan, 1, RADIX, 0, e.ctl, pa))) return rc;
  t_end(e);
  for (int p = 2; p < 4; ++p) {
    t_begin(e);
    if (p == 3 && (rc = chain_launch(e, k_count<K, XF, HIST_BLOCK>, sg, HIST_BLOCK, 0, e.ctl, p, n, sl, e.counts)))
      return rc;
    if ((rc = chain_launch(e, k_slice_scan, SCAN_GROUPS, SCAN_WARPS * 32, 0, e.ctl, p, sl,
                           static_cast<const uint32_t*>(e.counts), e.offsets, 0)))
      return rc;
    t_end(e);
    t_begin(e);
    const RadixDigit dg{p * RADIX_BITS};
    // digit 3 on the first pass's wide tile too: its rounds rank by atomics
    // wherever their keys agree on digit 2 (PD_SORTED_BELOW), nearly always
    // (2^30 u32 keys: 3.18 ms against 3.88 on the stable pass's tile)
    rc = p == 2 ? launch_scatter<K, false, XF, UnstableCfg<K>, SCATTER_UNSTABLE>(e, p, n, sl, dg, 0ull)
                : launch_scatter<K, false, XF, UnstableCfg<K>, SCATTER_ANY>(e, p, n, sl, dg, 0ull);
    t_end(e);
    if (rc) return rc;
  }
  // histogram fill: one CTA per SM (136 KiB of counters each)
  static std::atomic<bool> configured[MAX_DEVICES];
  if (e.device < 0 || e.device >= MAX_DEVICES)
    return fail(e.s, FS_E_INVALID, "device %d outside [0, %d)", e.device, MAX_DEVICES);
  if (!configured[e.device].load()) {
    FS_CUDA(e.s, cudaFuncSetAttribute(k_hf_local<XF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)HF_LOCAL_SMEM_STAGED));
    FS_CUDA(e.s, cudaFuncSetAttribute(k_hf_big_count<XF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)HF_BIG_SMEM));
    configured[e.device].store(true);
  }
  t_begin(e);
  if ((rc = chain_launch(e, k_hf_bounds<XF>, (HF_GROUPS + 1 + 255) / 256, 256, 0, (const SortCtl*)e.ctl, e.hf, n)))
    return rc;
  if ((rc = chain_launch(e, k_hf_plan, 1, HF_BLOCK, 0, (const SortCtl*)e.ctl, e.hf))) return rc;
  t_end(e);
  t_begin(e);
  if ((rc = chain_launch(e, k_hf_local<XF>, (unsigned)e.sm_count, HF_BLOCK, HF_LOCAL_SMEM_STAGED, (const SortCtl*)e.ctl,
                         (const HfCtl*)e.hf)))
    return rc;
  t_end(e);
  t_begin(e);
  if ((rc = chain_launch(e, k_hf_big_zero, (unsigned)e.sm_count * 4, 256, 0, (const SortCtl*)e.ctl,
                         (const HfCtl*)e.hf)))
    return rc;
  if ((rc = chain_launch(e, k_hf_big_count<XF>, (unsigned)e.sm_count, HF_BLOCK, HF_BIG_SMEM, (const SortCtl*)e.ctl,
                         (const HfCtl*)e.hf)))
    return rc;
  if ((rc = chain_launch(e, k_hf_big_scan, (unsigned)e.sm_count, HF_BLOCK, 0, (const SortCtl*)e.ctl, e.hf)))
    return rc;
  if ((rc = chain_launch(e, k_hf_big_fill<XF>, (unsigned)e.sm_count, HF_BLOCK, 0, (const SortCtl*)e.ctl,
                         (const HfCtl*)e.hf)))
    return rc;
  t_end(e);
  uint64_t fb = (n + 255) / 256;
  const uint64_t fcap = (uint64_t)e.sm_count * 4;
  t_begin(e);
  if ((rc = chain_launch(e, k_finalize<K>, (unsigned)(fb < fcap ? fb : fcap), 256, 0, e.ctl, n, e.err_out)))
    return rc;
  t_end(e);
  if (launches) *launches = 15;
  FS_CUDA(e.s, cudaGetLastError());
  return FS_OK;
}

// Slice geometry for (dtype, n, payload, first-pass rank method).
Slices dispatch_slices(const Exec& e, int dtype, uint64_t n, bool vals, bool unstable_first) {
  const bool w = dtype >= FS_U64;
  uint64_t unit;
  if (vals)
    unit = w ? tile_of<StableCfg<uint64_t, true>>() : tile_of<StableCfg<uint32_t, true>>();
  else if (w)
    unit = unstable_first ? lcm64(tile_of<StableCfg<uint64_t, false>>(), tile_of<UnstableCfg<uint64_t>>())
                          : tile_of<StableCfg<uint64_t, false>>();
  else
    unit = unstable_first ? lcm64(tile_of<StableCfg<uint32_t, false>>(), tile_of<UnstableCfg<uint32_t>>())
                          : tile_of<StableCfg<uint32_t, false>>();
  return make_slices(e, n, unit);
}

int dispatch_enqueue(const Exec& e, int dtype, const PlanArgs& a, const Slices& sl, int* launches) {
  switch (dtype) {
    case FS_U32: return enqueue_sort<uint32_t, XF_NONE>(e, a, sl, launches);
    case FS_I32: return enqueue_sort<uint32_t, XF_SIGN>(e, a, sl, launches);
    case FS_F32: return enqueue_sort<uint32_t, XF_FLOAT>(e, a, sl, launches);
    case FS_U64: return enqueue_sort<uint64_t, XF_NONE>(e, a, sl, launches);
    case FS_I64: return enqueue_sort<uint64_t, XF_SIGN>(e, a, sl, launches);
    case FS_F64: return enqueue_sort<uint64_t, XF_FLOAT>(e, a, sl, launches);
    default: return fail(e.s, FS_E_INVALID, "unknown dtype %d", dtype);
  }
}

int ensure_slice_buffers(fs_sorter* s, const Slices& sl) {
  int rc = grow(s, &s->counts, &s->counts_bytes, (size_t)sl.count * RADIX * 4, false);
  if (!rc) rc = grow(s, &s->offsets, &s->offsets_bytes, (size_t)sl.count * RADIX * 4, false);
  return rc;
}

Exec exec_of(fs_sorter* s) {
  Exec e{};
  e.device = s->device;
  e.stream = s->stream;
  e.sm_count = s->sm_count;
  e.timeout_ns = s->timeout_ns;
  e.ctl = s->ctl;
  e.err_out = s->host_err_dev;
  e.s = s;
  return e;
}

// Small sorts: one CTA, everything in shared memory (k_small_sort).
template <typename K, int XF, bool VALS>
int launch_small(fs_sorter* s, const PlanArgs& a) {
  const uint32_t n = (uint32_t)a.n;
  uint32_t npad = 2;
  while (npad < n) npad <<= 1;
  const size_t smem = (size_t)npad * (sizeof(K) + (VALS ? 8 : 0));
  uint32_t block = npad / 4;
  if (block < 32) block = 32;
  if (block > (uint32_t)SMALL_BLOCK_MAX) block = SMALL_BLOCK_MAX;
  auto kern = k_small_sort<K, XF, VALS>;
  static std::atomic<bool> configured[MAX_DEVICES];  // opt-in shared memory, once per device
  if (s->device < 0 || s->device >= MAX_DEVICES)
    return fail(s, FS_E_INVALID, "device %d outside [0, %d)", s->device, MAX_DEVICES);
  if (!configured[s->device].load()) {
    FS_CUDA(s, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(SMALL_N_MAX * (sizeof(K) + (VALS ? 8 : 0)))));
    configured[s->device].store(true);
  }
  kern<<<1, block, smem, s->stream>>>(static_cast<const K*>(a.kin), static_cast<K*>(a.kfinal), a.vin, a.vfinal, n,
                                      npad, a.write_keys);
  s->last_launches = 1;
  FS_CUDA(s, cudaGetLastError());
  return FS_OK;
}

template <typename K, int XF>
int enqueue_small(fs_sorter* s, const PlanArgs& a) {
  return a.has_vals ? launch_small<K, XF, true>(s, a) : launch_small<K, XF, false>(s, a);
}

int dispatch_small(fs_sorter* s, int dtype, const PlanArgs& a) {
  switch (dtype) {
    case FS_U32: return enqueue_small<uint32_t, XF_NONE>(s, a);
    case FS_I32: return enqueue_small<uint32_t, XF_SIGN>(s, a);
    case FS_F32: return enqueue_small<uint32_t, XF_FLOAT>(s, a);
    case FS_U64: return enqueue_small<uint64_t, XF_NONE>(s, a);
    case FS_I64: return enqueue_small<uint64_t, XF_SIGN>(s, a);
    case FS_F64: return enqueue_small<uint64_t, XF_FLOAT>(s, a);
    default: return fail(s, FS_E_INVALID, "unknown dtype %d", dtype);
  }
}

// Clear the device error word after a failed call (stream-ordered, before
// the next sort's kernels): the single-launch sort leaves it set.
int rearm_ctl(fs_sorter* s) {
  if (!s->ctl_dirty) return FS_OK;
  FS_CUDA(s, cudaMemsetAsync(&s->ctl->err, 0, sizeof(int), s->stream));
  s->ctl_dirty = false;
  return FS_OK;
}

// Keys-only sorts of up to a few million keys: the whole sort in one
// cooperative launch (k_resident_sort), one CTA of RES_BLOCK threads per SM,
// every key in registers.  Keys per thread: the fewest of RES_IPTS that fit
// the keys on the SMs.
constexpr int RES_IPTS[] = {2, 4, 7, 14};
constexpr int RES_IPT_MAX = 14;

uint64_t resident_max_keys(int sm_count) {
  return (uint64_t)(sm_count < RES_MAX_CTAS ? sm_count : RES_MAX_CTAS) * RES_BLOCK * RES_IPT_MAX;
}

// Most-significant-digit first (a partition, then segments sorted in shared
// memory) where the segment keys fit the registers: up to 7 keys per thread.
#ifndef FS_RES_MSD
#define FS_RES_MSD 1
#endif

template <typename K, int XF, int IPT>
int launch_resident(fs_sorter* s, const PlanArgs& a) {
  constexpr bool MSD = FS_RES_MSD && IPT <= 7;
  using Ly = ResLayout<K, RES_BLOCK, IPT, MSD>;
  constexpr int P = (int)sizeof(K);
  auto kern = k_resident_sort<K, XF, RES_BLOCK, IPT, MSD>;
  static std::atomic<int> bps_dev[MAX_DEVICES];  // resident CTAs per SM, 0 = not configured yet
  int bps = bps_dev[s->device].load();
  if (bps == 0) {
    FS_CUDA(s, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ly::BYTES));
    bps = blocks_per_sm(s, kern, RES_BLOCK, Ly::BYTES);
    if (bps < 0) return -bps;
    bps_dev[s->device].store(bps);
  }
  const uint64_t grid = (a.n + Ly::TILE - 1) / Ly::TILE;
  if (grid > (uint64_t)bps * s->sm_count || grid > (uint64_t)RES_MAX_CTAS)
    return fail(s, FS_E_INVALID, "single-launch sort: %llu keys need %llu CTAs, %d fit", (unsigned long long)a.n,
                (unsigned long long)grid, bps * s->sm_count);
  // accumulators laid out for the most CTAs any launch of this sorter uses,
  // so alternate launches of different sizes clear what the next one reads
  // (every launch clears the set the next one uses before it waits anywhere,
  // so a launch that failed still leaves that set clean)
  const uint32_t max_grid = (uint32_t)RES_MAX_CTAS;
  const uint32_t groups = (max_grid + RES_GROUP - 1) / RES_GROUP;
  // a slot of RADIX words per digit pass, RES_MR / RADIX slots for the top-bits partition
  constexpr int SLOTS = MAX_PASSES + RES_MR / RADIX;
  const size_t set_words = res_acc_words(SLOTS, groups);
  int rc = grow(s, &s->res_acc, &s->res_acc_bytes, 2 * set_words * 4, true);
  if (!rc) rc = grow(s, &s->res_counts, &s->res_counts_bytes, (size_t)SLOTS * max_grid * RADIX * 4, false);
  if (rc) return rc;
  uint32_t* acc = static_cast<uint32_t*>(s->res_acc);
  ResArgs ra{};
  ra.kin = a.kin;
  ra.kout = a.kfinal;
  ra.n = a.n;
  ra.ctl = s->ctl;
  ra.counts = static_cast<uint32_t*>(s->res_counts);
  ra.acc = acc + (size_t)s->res_parity * set_words;
  ra.acc_next = acc + (size_t)(s->res_parity ^ 1) * set_words;
  ra.acc_words = (uint32_t)set_words;
  ra.groups = groups;
  ra.timeout_ns = s->timeout_ns;
  ra.host_err = s->host_err_dev;
  ra.test_skip_arrival = s->test_skip_arrival;
  s->test_skip_arrival = 0;  // one-shot
  void* params[] = {&ra};
  Exec e = exec_of(s);
  s->ev_used = 0;
  t_begin(e);
  FS_CUDA(s, cudaLaunchCooperativeKernel((const void*)kern, dim3((unsigned)grid), dim3(RES_BLOCK), params, Ly::BYTES,
                                         s->stream));
  t_end(e);
  s->res_parity ^= 1;
  s->last_launches = 1;
  static_assert(P <= MAX_PASSES, "accumulator sets sized for MAX_PASSES digit passes");
  return FS_OK;
}

template <typename K, int XF>
int enqueue_resident(fs_sorter* s, const PlanArgs& a) {
  if (s->device < 0 || s->device >= MAX_DEVICES)
    return fail(s, FS_E_INVALID, "device %d outside [0, %d)", s->device, MAX_DEVICES);
  const uint64_t per_cta = (a.n + s->sm_count - 1) / s->sm_count;
  if (per_cta <= (uint64_t)RES_BLOCK * RES_IPTS[0]) return launch_resident<K, XF, RES_IPTS[0]>(s, a);
  if (per_cta <= (uint64_t)RES_BLOCK * RES_IPTS[1]) return launch_resident<K, XF, RES_IPTS[1]>(s, a);
  if (per_cta <= (uint64_t)RES_BLOCK * RES_IPTS[2]) return launch_resident<K, XF, RES_IPTS[2]>(s, a);
  return launch_resident<K, XF, RES_IPTS[3]>(s, a);
}

int dispatch_resident(fs_sorter* s, int dtype, const PlanArgs& a) {
  switch (dtype) {
    case FS_U32: return enqueue_resident<uint32_t, XF_NONE>(s, a);
    case FS_I32: return enqueue_resident<uint32_t, XF_SIGN>(s, a);
    case FS_F32: return enqueue_resident<uint32_t, XF_FLOAT>(s, a);
    default: return fail(s, FS_E_INVALID, "single-launch sort: 32-bit keys only (dtype %d)", dtype);
  }
}

// The sorter's path: size the slices, grow its scratch, enqueue.
int dispatch(fs_sorter* s, int dtype, const PlanArgs& a) {
  s->part.ready = false;  // the slice counts of a pending dispatch are overwritten
  int rc = rearm_ctl(s);
  if (rc) return rc;
  const uint32_t small_cap = a.has_vals && s->small_max > SMALL_N_PAYLOAD_MAX ? SMALL_N_PAYLOAD_MAX : s->small_max;
  if (a.n <= small_cap) return dispatch_small(s, dtype, a);
  // measured on one B200 (device time per call): one launch 58-65 us against
  // 75 us chained for 2^14..2^19 u32 keys; slower from 2^20 (82 vs 78 us) and
  // for 64-bit keys at every size (8 passes: twice the grid barriers)
  if (!a.has_vals && a.unstable_first && !s->test_withhold && key_bytes_of(dtype) == 4 &&
      a.n * 4 <= s->coop_max_bytes && a.n <= resident_max_keys(s->sm_count))
    return dispatch_resident(s, dtype, a);
  Exec e = exec_of(s);
  const Slices sl = dispatch_slices(e, dtype, a.n, a.has_vals != 0, a.unstable_first != 0);
  rc = ensure_slice_buffers(s, sl);
  if (rc) return rc;
  e.counts = static_cast<uint32_t*>(s->counts);
  e.offsets = static_cast<uint32_t*>(s->offsets);
  PlanArgs pa = a;
  pa.test_withhold = s->test_withhold;
  s->test_withhold = 0;  // one-shot
  if (!a.has_vals && a.unstable_first && a.write_keys && key_bytes_of(dtype) == 4 && s->h16_min > 0 &&
      a.n >= s->h16_min && a.kother != nullptr && a.kother != a.kfinal) {
    if ((rc = grow(s, &s->hf, &s->hf_bytes, sizeof(HfCtl), false))) return rc;
    e.hf = static_cast<HfCtl*>(s->hf);
    switch (dtype) {
      case FS_U32: return enqueue_h16<XF_NONE>(e, pa, sl, &s->last_launches);
      case FS_I32: return enqueue_h16<XF_SIGN>(e, pa, sl, &s->last_launches);
      default: return enqueue_h16<XF_FLOAT>(e, pa, sl, &s->last_launches);
    }
  }
  return dispatch_enqueue(e, dtype, pa, sl, &s->last_launches);
}

// ---- sample-sort partition --------------------------------------------------
// The bucket count with the splitter search and counting mode fitted to the
// splitter count (register trees of 1-3 levels for 2-8 buckets, packed
// per-thread counters while a thread sees fewer than 2^16 keys of a slice).
template <typename K, int XF>
void launch_bucket_hist(const Exec& e, const Slices& sl, const void* keys, uint64_t n, const void* spl_keys,
                        const uint64_t* spl_gpos, int nsplit, uint64_t gpos_base) {
  const bool packed = sl.keys_per_slice / HIST_BLOCK < 60000;
  const unsigned grid = stream_grid(e, sl);
  auto go = [&](auto lv, auto pack) {
    using D = SplitterDigit<K, XF, decltype(lv)::value>;
    const D dfn{static_cast<const K*>(spl_keys), spl_gpos, nsplit};
    k_bucket_hist<K, XF, HIST_BLOCK, D, decltype(pack)::value><<<grid, HIST_BLOCK, 0, e.stream>>>(
        static_cast<const K*>(keys), n, e.ctl, sl, e.counts, dfn, gpos_base);
  };
  using std::integral_constant;
  if (nsplit <= 1 && packed)
    go(integral_constant<int, 1>{}, integral_constant<int, 2>{});
  else if (nsplit <= 3 && packed)
    go(integral_constant<int, 2>{}, integral_constant<int, 4>{});
  else if (nsplit <= 7 && packed)
    go(integral_constant<int, 3>{}, integral_constant<int, 8>{});
  else if (nsplit <= 7)
    go(integral_constant<int, 3>{}, integral_constant<int, 0>{});
  else
    go(integral_constant<int, 0>{}, integral_constant<int, 0>{});
}

// One stable pass that moves every key to the splitter bucket its (ordered
// key, global position) falls in: the same slice / count / scatter machinery
// as a radix pass, with the bucket index as the digit.
template <typename K, int XF>
int enqueue_partition(fs_sorter* s, const void* keys_in, void* keys_out, uint64_t n, uint64_t gpos_base,
                      const void* spl_keys, const uint64_t* spl_gpos, int nsplit, unsigned long long* counts_out) {
  s->part.ready = false;  // the slice counts of a pending dispatch are overwritten
  Exec e = exec_of(s);
  const Slices sl = make_slices(e, n, tile_of<StableCfg<K, false>>());
  int rc = ensure_slice_buffers(s, sl);
  if (rc) return rc;
  e.counts = static_cast<uint32_t*>(s->counts);
  e.offsets = static_cast<uint32_t*>(s->offsets);
  PlanArgs a{};
  a.n = n;
  a.kin = keys_in;
  a.kfinal = keys_out;
  a.kother = s->kother;
  a.passes = 1;
  a.has_vals = 0;
  a.write_keys = 1;
  a.key_bytes = (int)sizeof(K);
  a.counts_out = counts_out;
  a.ncounts = nsplit + 1;
  if (int rc0 = rearm_ctl(s)) return rc0;
  FS_CUDA(s, cudaMemsetAsync(e.ctl, 0, CTL_ACCUM_BYTES, e.stream));
  launch_bucket_hist<K, XF>(e, sl, keys_in, n, spl_keys, spl_gpos, nsplit, gpos_base);
  k_plan<<<1, RADIX, 0, e.stream>>>(e.ctl, a);
  k_slice_scan<<<SCAN_GROUPS, SCAN_WARPS * 32, 0, e.stream>>>(e.ctl, 0, sl, e.counts, e.offsets, 0);
  if (nsplit <= 7) {
    using D = SplitterDigit<K, XF, 3>;
    const D dfn{static_cast<const K*>(spl_keys), spl_gpos, nsplit};
    rc = launch_scatter<K, false, XF, PartCfg<K>, SCATTER_ANY>(e, 0, n, sl, dfn, gpos_base);
  } else {
    using D = SplitterDigit<K, XF, 0>;
    const D dfn{static_cast<const K*>(spl_keys), spl_gpos, nsplit};
    rc = launch_scatter<K, false, XF, PartCfg<K>, SCATTER_ANY>(e, 0, n, sl, dfn, gpos_base);
  }
  if (rc) return rc;
  uint64_t fb = (n + 255) / 256;
  const uint64_t fcap = (uint64_t)e.sm_count * 4;
  k_finalize<K><<<(unsigned)(fb < fcap ? fb : fcap), 256, 0, e.stream>>>(e.ctl, n, e.err_out);
  s->last_launches = 5;
  FS_CUDA(s, cudaGetLastError());
  return FS_OK;
}

// ---- sample-sort dispatch -----------------------------------------------------
// Count: per-slice bucket counts (kept in the sorter's scratch for the
// dispatch that follows) and the bucket totals, copied to the host.
// host_counts: copy the bucket sizes to host memory and wait; dev_counts
// (host_counts == nullptr): copy them to device memory, stream-ordered.
template <typename K, int XF>
int enqueue_partition_count(fs_sorter* s, const void* keys, uint64_t n, uint64_t gpos_base, const void* spl_keys,
                            const uint64_t* spl_gpos, int nsplit, unsigned long long* host_counts,
                            unsigned long long* dev_counts = nullptr) {
  Exec e = exec_of(s);
  const Slices sl = make_slices(e, n, tile_of<StableCfg<K, false>>());
  int rc = ensure_slice_buffers(s, sl);
  if (rc) return rc;
  e.counts = static_cast<uint32_t*>(s->counts);
  s->ev_used = 0;
  if (int rc0 = rearm_ctl(s)) return rc0;
  FS_CUDA(s, cudaMemsetAsync(e.ctl, 0, CTL_ACCUM_BYTES, e.stream));
  t_begin(e);
  launch_bucket_hist<K, XF>(e, sl, keys, n, spl_keys, spl_gpos, nsplit, gpos_base);
  t_end(e);
  FS_CUDA(s, cudaGetLastError());
  if (!host_counts) {
    FS_CUDA(s, cudaMemcpyAsync(dev_counts, &e.ctl->hist[0][0], (size_t)(nsplit + 1) * sizeof(unsigned long long),
                               cudaMemcpyDeviceToDevice, e.stream));
    s->last_launches = 1;
    return FS_OK;
  }
  FS_CUDA(s, cudaMemcpyAsync(host_counts, &e.ctl->hist[0][0], (size_t)(nsplit + 1) * sizeof(unsigned long long),
                             cudaMemcpyDeviceToHost, e.stream));
  FS_CUDA(s, cudaStreamSynchronize(e.stream));
  s->last_launches = 1;
  return FS_OK;
}

// Dispatch: one stable pass that stores every key at its rank within its
// bucket, straight into that bucket's destination (dst[b], this rank's region
// of rank b's inbox: plain stores over NVLink when it is another GPU's).
// Destinations of a dispatch computed on the device from the all-gathered
// send matrix M (G x G, row s = the bucket sizes rank s sends): this rank's
// keys of bucket b start after the keys that lower ranks send to rank b.
struct DispatchBases {
  uintptr_t key[RADIX];  // rank b's inbox (keys), this process's mapping
  uintptr_t val[RADIX];  // rank b's inbox (values), payload dispatches only
};

__global__ void __launch_bounds__(RADIX)
    k_dispatch_table(const unsigned long long* __restrict__ M, const int G, const int rank, const int kb,
                     const DispatchBases bases, const int payload, void** __restrict__ tab) {
  const int b = threadIdx.x;
  if (b >= G) return;
  unsigned long long before = 0;
  for (int r = 0; r < rank; ++r) before += M[(size_t)r * G + b];
  tab[b] = reinterpret_cast<void*>(bases.key[b] + before * (unsigned long long)kb);
  if (payload) tab[RADIX + b] = reinterpret_cast<void*>(bases.val[b] + before * 4ull);
}

// dst_host / vdst_host: destinations from the host (copied into the table);
// nullptr: the table was already written on the device (k_dispatch_table).
// Keys-only dispatch ranks with shared atomics from this many buckets up; with
// fewer, most lanes of a warp add to the same counter and the stable rank's
// ballots cost less.  Measured on one B200, 2^28 u32 keys, dispatch ms stable
// / atomics: 2 buckets 0.943 / 1.180, 3: 1.152 / 1.125, 4: 1.160 / 1.080,
// 6: 1.160 / 0.989, 8: 1.176 / 0.976.
#ifndef FS_DISPATCH_UNSTABLE_MIN
#define FS_DISPATCH_UNSTABLE_MIN 3
#endif

template <typename K, int XF, int NB, int LV, bool VALS>
int enqueue_partition_dispatch_nb(fs_sorter* s, const void* keys, const uint32_t* vals, uint64_t n,
                                  uint64_t gpos_base, const void* spl_keys, const uint64_t* spl_gpos, int nsplit,
                                  void* const* dst_host, uint32_t* const* vdst_host) {
  using D = SplitterDispatch<K, XF, NB, LV>;
  D dfn{};
  dfn.keys = static_cast<const K*>(spl_keys);
  dfn.gpos = spl_gpos;
  dfn.nsplit = nsplit;
  // [key destinations | value destinations], RADIX entries each
  if (!s->dst_tab) FS_CUDA(s, cudaMalloc(&s->dst_tab, 2 * RADIX * sizeof(void*)));
  void** tab = static_cast<void**>(s->dst_tab);
  // pageable sources: the copies are staged before cudaMemcpyAsync returns
  if (dst_host)
    FS_CUDA(s, cudaMemcpyAsync(tab, dst_host, (size_t)(nsplit + 1) * sizeof(void*), cudaMemcpyHostToDevice,
                               s->stream));
  if (VALS && vdst_host)
    FS_CUDA(s, cudaMemcpyAsync(tab + RADIX, vdst_host, (size_t)(nsplit + 1) * sizeof(void*), cudaMemcpyHostToDevice,
                               s->stream));
  dfn.dst = reinterpret_cast<K* const*>(tab);
  dfn.vdst = reinterpret_cast<uint32_t* const*>(tab + RADIX);
  Exec e = exec_of(s);
  const Slices sl = make_slices(e, n, tile_of<StableCfg<K, false>>());
  e.counts = static_cast<uint32_t*>(s->counts);
  e.offsets = static_cast<uint32_t*>(s->offsets);
  PlanArgs a{};
  a.n = n;
  a.kin = keys;
  a.kfinal = nullptr;  // not written: dispatch stores through dst[]
  a.kother = nullptr;
  a.passes = 1;
  a.write_keys = 1;
  a.key_bytes = (int)sizeof(K);
  a.force_exec = 1;
  // keys only: any order within a bucket (the receiving rank's sort orders
  // the keys, and equal keys are identical bits), so with enough buckets the
  // pass ranks with shared atomics; with a payload the input order is kept
  const bool unstable = !VALS && nsplit + 1 >= FS_DISPATCH_UNSTABLE_MIN;
  a.unstable_first = unstable ? 1 : 0;
  if (VALS) {
    a.has_vals = 1;
    a.vin = vals;  // nullptr: each key's global position, gpos_base + i
    a.vfinal = nullptr;  // not written either: dispatch stores through vdst[]
  }
  s->ev_used = 0;
  t_begin(e);
  k_plan<<<1, RADIX, 0, e.stream>>>(e.ctl, a);
  k_slice_scan<<<SCAN_GROUPS, SCAN_WARPS * 32, 0, e.stream>>>(e.ctl, 0, sl, e.counts, e.offsets, 1);
  t_end(e);
  int rc;
  t_begin(e);
  rc = unstable ? launch_scatter<K, VALS, XF, PartCfg<K>, SCATTER_UNSTABLE>(e, 0, n, sl, dfn, gpos_base)
                : launch_scatter<K, VALS, XF, PartCfg<K>, SCATTER_ANY>(e, 0, n, sl, dfn, gpos_base);
  t_end(e);
  if (rc) return rc;
  k_finalize<K><<<1, 256, 0, e.stream>>>(e.ctl, 0, e.err_out);  // error hand-off only
  s->last_launches = 4;
  FS_CUDA(s, cudaGetLastError());
  return FS_OK;
}


// Up to 8 buckets (the GPUs of one box) take the 8-digit instantiation, with
// the splitters in registers (one compare for 2 buckets, a 3-level tree for
// up to 8); more buckets search the shared-memory copy.
template <typename K, int XF>
int enqueue_partition_dispatch(fs_sorter* s, const void* keys, const uint32_t* vals, bool with_vals, uint64_t n,
                               uint64_t gpos_base, const void* spl_keys, const uint64_t* spl_gpos, int nsplit,
                               void* const* dst_host, uint32_t* const* vdst_host) {
#define FS_DISPATCH_NB(NB, LV)                                                                                     \
  (with_vals ? enqueue_partition_dispatch_nb<K, XF, NB, LV, true>(s, keys, vals, n, gpos_base, spl_keys, spl_gpos, \
                                                                   nsplit, dst_host, vdst_host)                   \
             : enqueue_partition_dispatch_nb<K, XF, NB, LV, false>(s, keys, nullptr, n, gpos_base, spl_keys,      \
                                                                    spl_gpos, nsplit, dst_host, nullptr))
  if (nsplit <= 1) return FS_DISPATCH_NB(8, 1);
  if (nsplit < 8) return FS_DISPATCH_NB(8, 3);
  return FS_DISPATCH_NB(RADIX, 0);
#undef FS_DISPATCH_NB
}

int finish(fs_sorter* s, int sync) {
  FS_CUDA(s, cudaGetLastError());
  if (!sync) return FS_OK;
  FS_CUDA(s, cudaStreamSynchronize(s->stream));
  const int he = *(volatile int*)s->host_err;
  if (he != 0) {
    *(volatile int*)s->host_err = 0;
    if (he == DEV_ERR_BOUNDS)
      return fail(s, FS_E_GPU_EXECUTION, "a device position fell out of range (scatter offset or gather index)");
    return fail(s, FS_E_TIMEOUT, "device wait timeout: a bulk copy or grid barrier did not complete within %llu ms",
                (unsigned long long)(s->timeout_ns / 1000000ull));
  }
  return FS_OK;
}

int check_common(fs_sorter* s, int dtype, uint64_t n) {
  if (!s) return FS_E_INVALID;
  if (dtype < FS_U32 || dtype > FS_F64) return fail(s, FS_E_INVALID, "unknown dtype %d", dtype);
  if (n > (1ull << 32)) return fail(s, FS_E_INVALID, "n = %llu exceeds 2^32 keys per GPU", (unsigned long long)n);
  return FS_OK;
}

int set_device(fs_sorter* s) {
  FS_CUDA(s, cudaSetDevice(s->device));
  return FS_OK;
}

// ---- allocation-free sorting ------------------------------------------------
// Scratch for fs_sort_keys_noalloc lives in one file-scope device array sized
// for NA_MAX_KEY_BYTES of keys.  Every device that loads this library holds it
// until the process exits.  Carved as:
//   [other-key buffer | slice counts | slice offsets | control block |
//    error word]
constexpr uint64_t NA_MAX_KEY_BYTES = 4ull << 20;  // 2^20 u32/i32/f32 or 2^19 u64/i64/f64 keys
constexpr uint32_t NA_MAX_SLICES = 256;            // >= tiles of the largest allowed sort
constexpr size_t NA_OFF_KEYS = 0;
constexpr size_t NA_OFF_COUNTS = NA_OFF_KEYS + NA_MAX_KEY_BYTES;
constexpr size_t NA_OFF_OFFSETS = NA_OFF_COUNTS + (size_t)NA_MAX_SLICES * RADIX * 4;
constexpr size_t NA_OFF_CTL = NA_OFF_OFFSETS + (size_t)NA_MAX_SLICES * RADIX * 4;
constexpr size_t NA_OFF_ERR = NA_OFF_CTL + ((sizeof(SortCtl) + 255) / 256) * 256;
constexpr size_t NA_BYTES = NA_OFF_ERR + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in: kernels must be given this address.
unsigned char* g_na_base[MAX_DEVICES] = {};
std::mutex g_na_mu;

int noalloc_base(int device, unsigned char** out) {
  if (device < 0 || device >= MAX_DEVICES) return fail(nullptr, FS_E_INVALID, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (!g_na_base[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // with `device` current
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_na_base[device] = static_cast<unsigned char*>(p);
  }
  *out = g_na_base[device];
  return FS_OK;
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

int fs_abi_version(void) { return FS_ABI_VERSION; }

const char* fs_last_error(const fs_sorter* s) { return s ? s->err.c_str() : g_create_err.c_str(); }

int fs_create(int device, void* stream, fs_sorter** out) {
  if (!out) return fail(nullptr, FS_E_INVALID, "out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(nullptr, FS_E_DEVICE_NOT_FOUND, "no CUDA device");
  }
  if (device < 0 || device >= count) return fail(nullptr, FS_E_DEVICE_NOT_FOUND, "no CUDA device %d", device);
  if (device >= MAX_DEVICES) return fail(nullptr, FS_E_INVALID, "device %d outside [0, %d)", device, MAX_DEVICES);
  fs_sorter* s = new fs_sorter();
  s->device = device;
  auto bail = [&](int rc) {
    g_create_err = s->err;
    fs_destroy(s);
    return rc;
  };
  int rc = set_device(s);
  if (rc) return bail(rc);
  if (cudaDeviceGetAttribute(&s->sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return bail(cuda_fail(s, cudaGetLastError(), "cudaDeviceGetAttribute"));
  if (stream) {
    s->stream = static_cast<cudaStream_t>(stream);
  } else {
    e = cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(cuda_fail(s, e, "cudaStreamCreate"));
    s->stream = s->own_stream;
  }
  e = cudaMalloc((void**)&s->ctl, sizeof(SortCtl));
  if (e != cudaSuccess) return bail(cuda_fail(s, e, "cudaMalloc(ctl)"));
  e = cudaMemset(s->ctl, 0, sizeof(SortCtl));
  if (e != cudaSuccess) return bail(cuda_fail(s, e, "cudaMemset(ctl)"));
  e = cudaHostAlloc((void**)&s->host_err, sizeof(int), cudaHostAllocMapped);
  if (e != cudaSuccess) return bail(cuda_fail(s, e, "cudaHostAlloc(err)"));
  *s->host_err = 0;
  e = cudaHostGetDevicePointer((void**)&s->host_err_dev, s->host_err, 0);
  if (e != cudaSuccess) return bail(cuda_fail(s, e, "cudaHostGetDevicePointer"));
  if (const char* t = getenv("FORGESORT_SMALL_SORT")) {  // 0: off; N: up to N keys (at most SMALL_N_MAX)
    const long long v = atoll(t);
    s->small_max = v <= 0 ? 0u : (uint32_t)(v < (long long)SMALL_N_MAX ? v : SMALL_N_MAX);
  }
  s->timeout_ns = wait_timeout_ns_env();
  if (const char* t = getenv("FORGESORT_COOP_MAX_BYTES")) {  // bytes of keys; 0: never one launch
    const long long v = atoll(t);
    s->coop_max_bytes = v <= 0 ? 0ull : (uint64_t)v;
  }
  if (const char* t = getenv("FORGESORT_H16_MIN_KEYS")) {  // keys; 0: never the histogram fill
    const long long v = atoll(t);
    s->h16_min = v <= 0 ? 0ull : (uint64_t)v;
  }
  *out = s;
  return FS_OK;
}

int fs_destroy(fs_sorter* s) {
  if (!s) return FS_OK;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  for (auto& kv : s->allocs) {
    if (s->managed.count(kv.first))
      cudaFreeHost(kv.first);
    else
      cudaFree(kv.first);
  }
  if (s->h2d) cudaStreamSynchronize(s->h2d);
  if (s->d2h) cudaStreamSynchronize(s->d2h);
  for (auto& sl : s->pipe) {
    if (sl.dkeys) cudaFree(sl.dkeys);
    for (cudaEvent_t e : {sl.in_done, sl.sorted, sl.out_done})
      if (e) cudaEventDestroy(e);
  }
  if (s->h2d) cudaStreamSynchronize(s->h2d), cudaStreamDestroy(s->h2d);
  if (s->d2h) cudaStreamSynchronize(s->d2h), cudaStreamDestroy(s->d2h);
  if (s->pipe_start) cudaEventDestroy(s->pipe_start);
  s->stage.release();
  void* bufs[] = {s->counts, s->offsets, s->kother, s->kfinal2, s->vother,    s->dkeys,
                  s->dvals,  s->dst_tab, s->ctl,    s->res_acc, s->res_counts, s->hf};
  for (void* b : bufs)
    if (b) cudaFree(b);
  if (s->host_err) cudaFreeHost(s->host_err);
  for (cudaEvent_t e : s->ev)
    if (e) cudaEventDestroy(e);
  if (s->own_stream) cudaStreamDestroy(s->own_stream);
  cudaGetLastError();
  delete s;
  return FS_OK;
}

int fs_set_stream(fs_sorter* s, void* stream) {
  if (!s) return FS_E_INVALID;
  int rc = set_device(s);
  if (rc) return rc;
  FS_CUDA(s, cudaStreamSynchronize(s->stream));
  if (stream) {
    s->stream = static_cast<cudaStream_t>(stream);
  } else {
    if (!s->own_stream) FS_CUDA(s, cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking));
    s->stream = s->own_stream;
  }
  return FS_OK;
}

int fs_synchronize(fs_sorter* s) {
  if (!s) return FS_E_INVALID;
  int rc = set_device(s);
  if (rc) return rc;
  // join the asynchronous host sorts: later work on the stream waits for
  // their copies back, then the host waits for the stream
  for (auto& sl : s->pipe)
    if (sl.used) FS_CUDA(s, cudaStreamWaitEvent(s->stream, sl.out_done, 0));
  s->pipe_open = false;
  return finish(s, 1);
}

int fs_host_sort_keys_copy_async(fs_sorter* s, int dtype, const void* host_in, void* host_out, uint64_t n) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n == 0) return FS_OK;
  if (!host_in || !host_out) return fail(s, FS_E_INVALID, "host_in or host_out is NULL");
  if ((rc = set_device(s))) return rc;
  const size_t bytes = (size_t)n * key_bytes_of(dtype);
  if (!s->h2d) {
    FS_CUDA(s, cudaStreamCreateWithFlags(&s->h2d, cudaStreamNonBlocking));
    FS_CUDA(s, cudaStreamCreateWithFlags(&s->d2h, cudaStreamNonBlocking));
    FS_CUDA(s, cudaEventCreateWithFlags(&s->pipe_start, cudaEventDisableTiming));
    for (auto& sl : s->pipe) {
      FS_CUDA(s, cudaEventCreateWithFlags(&sl.in_done, cudaEventDisableTiming));
      FS_CUDA(s, cudaEventCreateWithFlags(&sl.sorted, cudaEventDisableTiming));
      FS_CUDA(s, cudaEventCreateWithFlags(&sl.out_done, cudaEventDisableTiming));
    }
  }
  fs_sorter::PipeSlot& sl = s->pipe[s->pipe_next];
  s->pipe_next ^= 1;
  if (sl.bytes < bytes) {  // grow: the buffer's previous copy back must be done
    if (sl.used) FS_CUDA(s, cudaEventSynchronize(sl.out_done));
    if (sl.dkeys) FS_CUDA(s, cudaFree(sl.dkeys));
    sl.dkeys = nullptr;
    sl.bytes = 0;
    const cudaError_t e = cudaMalloc(&sl.dkeys, bytes);
    if (e != cudaSuccess) {
      sl.dkeys = nullptr;
      cudaGetLastError();
      return fail(s, FS_E_OOM, "device allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    }
    sl.bytes = bytes;
  }
  // The first call after a synchronize orders the copy streams after the
  // caller's work on the sorter's stream; later calls only wait for their
  // own buffer (waiting on the stream again would wait for the previous
  // call's sort and serialise the pipeline).
  if (!s->pipe_open) {
    FS_CUDA(s, cudaEventRecord(s->pipe_start, s->stream));
    FS_CUDA(s, cudaStreamWaitEvent(s->h2d, s->pipe_start, 0));
    FS_CUDA(s, cudaStreamWaitEvent(s->d2h, s->pipe_start, 0));
    s->pipe_open = true;
  }
  if (n == 1) {  // nothing to sort: a host copy in order with the copies out
    FS_CUDA(s, cudaMemcpyAsync(host_out, host_in, bytes, cudaMemcpyHostToHost, s->d2h));
    FS_CUDA(s, cudaEventRecord(sl.out_done, s->d2h));
    sl.used = true;
    return FS_OK;
  }
  // copy in once this buffer's last copy out is done
  if (sl.used) FS_CUDA(s, cudaStreamWaitEvent(s->h2d, sl.out_done, 0));
  FS_CUDA(s, cudaMemcpyAsync(sl.dkeys, host_in, bytes, cudaMemcpyHostToDevice, s->h2d));
  FS_CUDA(s, cudaEventRecord(sl.in_done, s->h2d));
  // sort on the sorter's stream (its scratch is used by one sort at a time)
  FS_CUDA(s, cudaStreamWaitEvent(s->stream, sl.in_done, 0));
  if ((rc = fs_sort_keys(s, dtype, sl.dkeys, n, 0))) return rc;
  FS_CUDA(s, cudaEventRecord(sl.sorted, s->stream));
  // copy out
  FS_CUDA(s, cudaStreamWaitEvent(s->d2h, sl.sorted, 0));
  FS_CUDA(s, cudaMemcpyAsync(host_out, sl.dkeys, bytes, cudaMemcpyDeviceToHost, s->d2h));
  FS_CUDA(s, cudaEventRecord(sl.out_done, s->d2h));
  sl.used = true;
  return FS_OK;
}

int fs_alloc(fs_sorter* s, size_t bytes, int managed, void** ptr) {
  if (!s || !ptr) return s ? fail(s, FS_E_INVALID, "ptr is NULL") : FS_E_INVALID;
  *ptr = nullptr;
  int rc = set_device(s);
  if (rc) return rc;
  const size_t b = bytes ? bytes : 16;
  cudaError_t e = managed ? cudaHostAlloc(ptr, b, cudaHostAllocPortable | cudaHostAllocMapped) : cudaMalloc(ptr, b);
  if (e != cudaSuccess) {
    *ptr = nullptr;
    cudaGetLastError();
    return fail(s, FS_E_OOM, "allocation of %zu bytes failed: %s", b, cudaGetErrorString(e));
  }
  s->allocs[*ptr] = b;
  if (managed) s->managed[*ptr] = 1;
  return FS_OK;
}

int fs_free(fs_sorter* s, void* ptr) {
  if (!s) return FS_E_INVALID;
  if (!ptr) return FS_OK;
  auto it = s->allocs.find(ptr);
  if (it == s->allocs.end()) return fail(s, FS_E_INVALID, "pointer was not allocated by fs_alloc");
  int rc = set_device(s);
  if (rc) return rc;
  FS_CUDA(s, cudaStreamSynchronize(s->stream));
  if (s->managed.count(ptr))
    FS_CUDA(s, cudaFreeHost(ptr));
  else
    FS_CUDA(s, cudaFree(ptr));
  s->allocs.erase(it);
  s->managed.erase(ptr);
  return FS_OK;
}

int fs_sort_keys(fs_sorter* s, int dtype, void* keys_arg, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n <= 1) return FS_OK;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  void* keys = nullptr;
  if ((rc = device_view(s, keys_arg, (size_t)n * kb, "keys", &s->dkeys, &s->dkeys_bytes, true, &keys))) return rc;
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  PlanArgs a{};
  a.n = n;
  a.kin = keys;
  a.kfinal = keys;
  a.kother = s->kother;
  a.passes = kb;
  a.has_vals = 0;
  a.write_keys = 1;
  a.key_bytes = kb;
  a.unstable_first = 1;  // keys only: equal keys are identical bits
  if ((rc = dispatch(s, dtype, a))) return rc;
  if ((rc = copy_back(s, keys_arg, keys, (size_t)n * kb))) return rc;
  if (sync && keys == keys_arg && (rc = prefetch_to_host(s, keys, (size_t)n * kb))) return rc;
  return finish(s, sync);
}

int fs_sort_pairs(fs_sorter* s, int dtype, void* keys_arg, uint32_t* vals_arg, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n <= 1) return FS_OK;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  void *keys = nullptr, *vv = nullptr;
  if ((rc = device_view(s, keys_arg, (size_t)n * kb, "keys", &s->dkeys, &s->dkeys_bytes, true, &keys))) return rc;
  if ((rc = device_view(s, vals_arg, (size_t)n * 4, "values", &s->dvals, &s->dvals_bytes, true, &vv))) return rc;
  uint32_t* vals = static_cast<uint32_t*>(vv);
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  if ((rc = grow(s, &s->vother, &s->vother_bytes, (size_t)n * 4, false))) return rc;
  PlanArgs a{};
  a.n = n;
  a.kin = keys;
  a.kfinal = keys;
  a.kother = s->kother;
  a.vin = vals;
  a.vfinal = vals;
  a.vother = static_cast<uint32_t*>(s->vother);
  a.passes = kb;
  a.has_vals = 1;
  a.write_keys = 1;
  a.key_bytes = kb;
  if ((rc = dispatch(s, dtype, a))) return rc;
  if ((rc = copy_back(s, keys_arg, keys, (size_t)n * kb))) return rc;
  if ((rc = copy_back(s, vals_arg, vals, (size_t)n * 4))) return rc;
  if (sync && keys == keys_arg && (rc = prefetch_to_host(s, keys, (size_t)n * kb))) return rc;
  if (sync && vals == vals_arg && (rc = prefetch_to_host(s, vals, (size_t)n * 4))) return rc;
  return finish(s, sync);
}

int fs_argsort(fs_sorter* s, int dtype, const void* keys_arg, uint32_t* idx_arg, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n == 0) return FS_OK;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  void* iv = nullptr;
  if ((rc = device_view(s, idx_arg, (size_t)n * 4, "idx_out", &s->dvals, &s->dvals_bytes, false, &iv))) return rc;
  uint32_t* idx_out = static_cast<uint32_t*>(iv);
  if (n == 1) {
    FS_CUDA(s, cudaMemsetAsync(idx_out, 0, 4, s->stream));
    if ((rc = copy_back(s, idx_arg, idx_out, 4))) return rc;
    s->last_launches = 0;
    return finish(s, sync);
  }
  void* kv = nullptr;
  if ((rc = device_view(s, keys_arg, (size_t)n * kb, "keys", &s->dkeys, &s->dkeys_bytes, true, &kv))) return rc;
  const void* keys = kv;
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  if ((rc = grow(s, &s->kfinal2, &s->kfinal2_bytes, (size_t)n * kb, false))) return rc;
  if ((rc = grow(s, &s->vother, &s->vother_bytes, (size_t)n * 4, false))) return rc;
  PlanArgs a{};
  a.n = n;
  a.kin = keys;
  a.kfinal = s->kfinal2;
  a.kother = s->kother;
  a.vin = nullptr;
  a.vfinal = idx_out;
  a.vother = static_cast<uint32_t*>(s->vother);
  a.passes = kb;
  a.has_vals = 1;
  a.write_keys = 0;
  a.key_bytes = kb;
  if ((rc = dispatch(s, dtype, a))) return rc;
  if ((rc = copy_back(s, idx_arg, idx_out, (size_t)n * 4))) return rc;
  if (sync && idx_out == idx_arg && (rc = prefetch_to_host(s, idx_out, (size_t)n * 4))) return rc;
  return finish(s, sync);
}

int fs_host_sort_keys(fs_sorter* s, int dtype, void* host_keys, uint64_t n) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n <= 1) return FS_OK;
  if (!host_keys) return fail(s, FS_E_INVALID, "keys is NULL");
  if ((rc = set_device(s))) return rc;
  const size_t bytes = (size_t)n * key_bytes_of(dtype);
  if ((rc = grow(s, &s->dkeys, &s->dkeys_bytes, bytes, false))) return rc;
  if ((rc = host_to_device(s, s->dkeys, host_keys, bytes))) return rc;
  if ((rc = fs_sort_keys(s, dtype, s->dkeys, n, 0))) return rc;
  if ((rc = device_to_host(s, host_keys, s->dkeys, bytes))) return rc;
  return finish(s, 1);
}

int fs_host_sort_pairs(fs_sorter* s, int dtype, void* host_keys, uint64_t n_keys, uint32_t* host_vals,
                       uint64_t n_vals) {
  if (!s) return FS_E_INVALID;
  if (n_keys != n_vals)
    return fail(s, FS_E_LENGTH_MISMATCH, "length mismatch: keys=%llu, values=%llu", (unsigned long long)n_keys,
                (unsigned long long)n_vals);
  int rc = check_common(s, dtype, n_keys);
  if (rc) return rc;
  const uint64_t n = n_keys;
  if (n <= 1) return FS_OK;
  if (!host_keys || !host_vals) return fail(s, FS_E_INVALID, "keys or values is NULL");
  if ((rc = set_device(s))) return rc;
  const size_t kbytes = (size_t)n * key_bytes_of(dtype), vbytes = (size_t)n * 4;
  if ((rc = grow(s, &s->dkeys, &s->dkeys_bytes, kbytes, false))) return rc;
  if ((rc = grow(s, &s->dvals, &s->dvals_bytes, vbytes, false))) return rc;
  if ((rc = host_to_device(s, s->dkeys, host_keys, kbytes))) return rc;
  if ((rc = host_to_device(s, s->dvals, host_vals, vbytes))) return rc;
  if ((rc = fs_sort_pairs(s, dtype, s->dkeys, static_cast<uint32_t*>(s->dvals), n, 0))) return rc;
  if ((rc = device_to_host(s, host_keys, s->dkeys, kbytes))) return rc;
  if ((rc = device_to_host(s, host_vals, s->dvals, vbytes))) return rc;
  return finish(s, 1);
}

int fs_host_argsort(fs_sorter* s, int dtype, const void* host_keys, uint32_t* host_idx_out, uint64_t n) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n == 0) return FS_OK;
  if (!host_keys || !host_idx_out) return fail(s, FS_E_INVALID, "keys or idx_out is NULL");
  if (n == 1) {
    host_idx_out[0] = 0;
    return FS_OK;
  }
  if ((rc = set_device(s))) return rc;
  const size_t kbytes = (size_t)n * key_bytes_of(dtype), vbytes = (size_t)n * 4;
  if ((rc = grow(s, &s->dkeys, &s->dkeys_bytes, kbytes, false))) return rc;
  if ((rc = grow(s, &s->dvals, &s->dvals_bytes, vbytes, false))) return rc;
  if ((rc = host_to_device(s, s->dkeys, host_keys, kbytes))) return rc;
  if ((rc = fs_argsort(s, dtype, s->dkeys, static_cast<uint32_t*>(s->dvals), n, 0))) return rc;
  if ((rc = device_to_host(s, host_idx_out, s->dvals, vbytes))) return rc;
  return finish(s, 1);
}

int fs_sort_keys_copy(fs_sorter* s, int dtype, const void* keys_in, void* keys_out, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  if (n == 0) return FS_OK;
  if (keys_in == keys_out) return fs_sort_keys(s, dtype, keys_out, n, sync);
  const char* a0 = static_cast<const char*>(keys_in);
  const char* b0 = static_cast<const char*>(keys_out);
  if (a0 < b0 + n * kb && b0 < a0 + n * kb) return fail(s, FS_E_INVALID, "keys_in and keys_out overlap");
  if ((rc = prepare_ptr(s, keys_in, (size_t)n * kb, "keys_in"))) return rc;
  if ((rc = prepare_ptr(s, keys_out, (size_t)n * kb, "keys_out"))) return rc;
  if (n == 1) {
    FS_CUDA(s, cudaMemcpyAsync(keys_out, keys_in, kb, cudaMemcpyDeviceToDevice, s->stream));
    s->last_launches = 0;
    return finish(s, sync);
  }
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  PlanArgs a{};
  a.n = n;
  a.kin = keys_in;
  a.kfinal = keys_out;
  a.kother = s->kother;
  a.passes = kb;
  a.has_vals = 0;
  a.write_keys = 1;
  a.key_bytes = kb;
  a.unstable_first = 1;  // keys only: equal keys are identical bits
  if ((rc = dispatch(s, dtype, a))) return rc;
  return finish(s, sync);
}

int fs_host_sort_keys_copy(fs_sorter* s, int dtype, const void* host_in, void* host_out, uint64_t n) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n == 0) return FS_OK;
  if (!host_in || !host_out) return fail(s, FS_E_INVALID, "host_in or host_out is NULL");
  const size_t bytes = (size_t)n * key_bytes_of(dtype);
  if (n == 1) {
    std::memmove(host_out, host_in, bytes);
    return FS_OK;
  }
  if ((rc = set_device(s))) return rc;
  if ((rc = grow(s, &s->dkeys, &s->dkeys_bytes, bytes, false))) return rc;
  if ((rc = host_to_device(s, s->dkeys, host_in, bytes))) return rc;
  if ((rc = fs_sort_keys(s, dtype, s->dkeys, n, 0))) return rc;
  if ((rc = device_to_host(s, host_out, s->dkeys, bytes))) return rc;
  return finish(s, 1);
}

int fs_set_kernel_timing(fs_sorter* s, int on) {
  if (!s) return FS_E_INVALID;
  int rc = set_device(s);
  if (rc) return rc;
  if (on && !s->ev[0]) {
    for (cudaEvent_t& e : s->ev) FS_CUDA(s, cudaEventCreate(&e));
  }
  s->timing = on != 0;
  s->ev_used = 0;
  return FS_OK;
}

int fs_last_kernel_times(fs_sorter* s, float* ms, int cap) {
  if (!s || (!ms && cap > 0)) return -FS_E_INVALID;
  if (!s->timing) return 0;
  if (set_device(s)) return -FS_E_GPU_EXECUTION;
  if (cudaStreamSynchronize(s->stream) != cudaSuccess) return -cuda_fail(s, cudaGetLastError(), "sync");
  int k = 0;
  for (; k < s->ev_used && k < cap; ++k) {
    if (cudaEventElapsedTime(&ms[k], s->ev[2 * k], s->ev[2 * k + 1]) != cudaSuccess)
      return -cuda_fail(s, cudaGetLastError(), "cudaEventElapsedTime");
  }
  return k;
}

int fs_sort_keys_noalloc(int dtype, void* keys, uint64_t n, void* stream) {
  if (dtype < FS_U32 || dtype > FS_F64) return fail(nullptr, FS_E_INVALID, "unknown dtype %d", dtype);
  const int kb = key_bytes_of(dtype);
  if (n > NA_MAX_KEY_BYTES / (uint64_t)kb)  // (n * kb could wrap for huge n)
    return fail(nullptr, FS_E_INVALID,
                "n = %llu keys exceeds the allocation-free limit of %llu bytes of keys (%llu keys of %d bytes)",
                (unsigned long long)n, (unsigned long long)NA_MAX_KEY_BYTES,
                (unsigned long long)(NA_MAX_KEY_BYTES / kb), kb);
  if (n <= 1) return FS_OK;
  if (!keys) return fail(nullptr, FS_E_INVALID, "keys is NULL");
  int device = 0;
  cudaError_t ce = cudaGetDevice(&device);
  if (ce != cudaSuccess) return cuda_fail(nullptr, ce, "cudaGetDevice");
  cudaPointerAttributes at{};
  ce = cudaPointerGetAttributes(&at, keys);
  if (ce != cudaSuccess || at.type != cudaMemoryTypeDevice || at.device != device) {
    cudaGetLastError();
    return fail(nullptr, FS_E_INVALID, "keys must be device memory of the current device %d", device);
  }
  unsigned char* base = nullptr;
  int rc = noalloc_base(device, &base);
  if (rc) return rc;
  Exec e{};
  e.device = device;
  e.stream = static_cast<cudaStream_t>(stream);
  ce = cudaDeviceGetAttribute(&e.sm_count, cudaDevAttrMultiProcessorCount, device);
  if (ce != cudaSuccess) return cuda_fail(nullptr, ce, "cudaDeviceGetAttribute");
  e.timeout_ns = wait_timeout_ns_env();
  e.ctl = reinterpret_cast<SortCtl*>(base + NA_OFF_CTL);
  e.err_out = reinterpret_cast<int*>(base + NA_OFF_ERR);
  e.counts = reinterpret_cast<uint32_t*>(base + NA_OFF_COUNTS);
  e.offsets = reinterpret_cast<uint32_t*>(base + NA_OFF_OFFSETS);
  e.s = nullptr;
  const Slices sl = dispatch_slices(e, dtype, n, false, true);
  if (sl.count > NA_MAX_SLICES) return fail(nullptr, FS_E_INVALID, "internal: %u slices exceed the fixed scratch", sl.count);
  // The arena keeps the previous call's contents: the histogram accumulates
  // from zero and the error words must start clear.
  ce = cudaMemsetAsync(e.ctl, 0, sizeof(SortCtl), e.stream);
  if (ce == cudaSuccess) ce = cudaMemsetAsync(e.err_out, 0, sizeof(int), e.stream);
  if (ce != cudaSuccess) return cuda_fail(nullptr, ce, "cudaMemsetAsync(noalloc scratch)");
  PlanArgs a{};
  a.n = n;
  a.kin = keys;
  a.kfinal = keys;
  a.kother = base + NA_OFF_KEYS;
  a.passes = kb;
  a.has_vals = 0;
  a.write_keys = 1;
  a.key_bytes = kb;
  a.unstable_first = 1;  // keys only: equal keys are identical bits
  if ((rc = dispatch_enqueue(e, dtype, a, sl, nullptr))) return rc;
  int dev_err = 0;
  ce = cudaMemcpyAsync(&dev_err, e.err_out, sizeof(int), cudaMemcpyDeviceToHost, e.stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(e.stream);
  if (ce != cudaSuccess) return cuda_fail(nullptr, ce, "fs_sort_keys_noalloc");
  if (dev_err == DEV_ERR_BOUNDS) return fail(nullptr, FS_E_GPU_EXECUTION, "scatter position out of range");
  if (dev_err != 0) return fail(nullptr, FS_E_TIMEOUT, "device wait timeout in fs_sort_keys_noalloc");
  return FS_OK;
}

int fs_partition(fs_sorter* s, int dtype, const void* keys_in, uint64_t n, uint64_t gpos_base,
                 const void* splitter_keys, const uint64_t* splitter_gpos, int nsplit, void* keys_out,
                 uint64_t* bucket_counts, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (nsplit < 0 || nsplit > RADIX - 1) return fail(s, FS_E_INVALID, "nsplit = %d outside [0, 255]", nsplit);
  if (!bucket_counts) return fail(s, FS_E_INVALID, "bucket_counts is NULL");
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  if ((rc = prepare_ptr(s, bucket_counts, (size_t)(nsplit + 1) * 8, "bucket_counts"))) return rc;
  if (n == 0) {
    FS_CUDA(s, cudaMemsetAsync(bucket_counts, 0, (size_t)(nsplit + 1) * 8, s->stream));
    return finish(s, sync);
  }
  if (keys_in == keys_out) return fail(s, FS_E_INVALID, "keys_in and keys_out must differ");
  if ((rc = prepare_ptr(s, keys_in, (size_t)n * kb, "keys_in"))) return rc;
  if ((rc = prepare_ptr(s, keys_out, (size_t)n * kb, "keys_out"))) return rc;
  if (nsplit > 0) {
    if ((rc = prepare_ptr(s, splitter_keys, (size_t)nsplit * kb, "splitter_keys"))) return rc;
    if ((rc = prepare_ptr(s, splitter_gpos, (size_t)nsplit * 8, "splitter_gpos"))) return rc;
  }
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  auto* counts = reinterpret_cast<unsigned long long*>(bucket_counts);
  switch (dtype) {
    case FS_U32: rc = enqueue_partition<uint32_t, XF_NONE>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
    case FS_I32: rc = enqueue_partition<uint32_t, XF_SIGN>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
    case FS_F32: rc = enqueue_partition<uint32_t, XF_FLOAT>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
    case FS_U64: rc = enqueue_partition<uint64_t, XF_NONE>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
    case FS_I64: rc = enqueue_partition<uint64_t, XF_SIGN>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
    default: rc = enqueue_partition<uint64_t, XF_FLOAT>(s, keys_in, keys_out, n, gpos_base, splitter_keys, splitter_gpos, nsplit, counts); break;
  }
  if (rc) return rc;
  return finish(s, sync);
}

#define FS_PARTITION_DTYPES(CALL)                \
  switch (dtype) {                               \
    case FS_U32: rc = CALL(uint32_t, XF_NONE); break;  \
    case FS_I32: rc = CALL(uint32_t, XF_SIGN); break;  \
    case FS_F32: rc = CALL(uint32_t, XF_FLOAT); break; \
    case FS_U64: rc = CALL(uint64_t, XF_NONE); break;  \
    case FS_I64: rc = CALL(uint64_t, XF_SIGN); break;  \
    default: rc = CALL(uint64_t, XF_FLOAT); break;     \
  }

int fs_partition_count(fs_sorter* s, int dtype, const void* keys, uint64_t n, uint64_t gpos_base,
                       const void* splitter_keys, const uint64_t* splitter_gpos, int nsplit,
                       uint64_t* bucket_counts_host) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (nsplit < 0 || nsplit > RADIX - 1) return fail(s, FS_E_INVALID, "nsplit = %d outside [0, 255]", nsplit);
  if (!bucket_counts_host) return fail(s, FS_E_INVALID, "bucket_counts_host is NULL");
  s->part.ready = false;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  if (n == 0) {  // nothing to send; the dispatch that follows is a no-op
    std::memset(bucket_counts_host, 0, (size_t)(nsplit + 1) * 8);
    s->part = {true, dtype, nsplit, keys, 0};
    return FS_OK;
  }
  if ((rc = prepare_ptr(s, keys, (size_t)n * kb, "keys"))) return rc;
  if (nsplit > 0) {
    if ((rc = prepare_ptr(s, splitter_keys, (size_t)nsplit * kb, "splitter_keys"))) return rc;
    if ((rc = prepare_ptr(s, splitter_gpos, (size_t)nsplit * 8, "splitter_gpos"))) return rc;
  }
  auto* hc = reinterpret_cast<unsigned long long*>(bucket_counts_host);
#define FS_PC(K, XF) enqueue_partition_count<K, XF>(s, keys, n, gpos_base, splitter_keys, splitter_gpos, nsplit, hc)
  FS_PARTITION_DTYPES(FS_PC)
#undef FS_PC
  if (rc) return rc;
  s->part = {true, dtype, nsplit, keys, n};
  return finish(s, 1);
}

int fs_partition_count_async(fs_sorter* s, int dtype, const void* keys, uint64_t n, uint64_t gpos_base,
                             const void* splitter_keys, const uint64_t* splitter_gpos, int nsplit,
                             uint64_t* bucket_counts_dev) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (nsplit < 0 || nsplit > RADIX - 1) return fail(s, FS_E_INVALID, "nsplit = %d outside [0, 255]", nsplit);
  if (!bucket_counts_dev) return fail(s, FS_E_INVALID, "bucket_counts_dev is NULL");
  s->part.ready = false;
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  if ((rc = prepare_ptr(s, bucket_counts_dev, (size_t)(nsplit + 1) * 8, "bucket_counts_dev"))) return rc;
  if (n == 0) {
    FS_CUDA(s, cudaMemsetAsync(bucket_counts_dev, 0, (size_t)(nsplit + 1) * 8, s->stream));
    s->part = {true, dtype, nsplit, keys, 0};
    return finish(s, 0);
  }
  if ((rc = prepare_ptr(s, keys, (size_t)n * kb, "keys"))) return rc;
  if (nsplit > 0) {
    if ((rc = prepare_ptr(s, splitter_keys, (size_t)nsplit * kb, "splitter_keys"))) return rc;
    if ((rc = prepare_ptr(s, splitter_gpos, (size_t)nsplit * 8, "splitter_gpos"))) return rc;
  }
  auto* dc = reinterpret_cast<unsigned long long*>(bucket_counts_dev);
#define FS_PC(K, XF) \
  enqueue_partition_count<K, XF>(s, keys, n, gpos_base, splitter_keys, splitter_gpos, nsplit, nullptr, dc)
  FS_PARTITION_DTYPES(FS_PC)
#undef FS_PC
  if (rc) return rc;
  s->part = {true, dtype, nsplit, keys, n};
  return finish(s, 0);
}

namespace {
int partition_dispatch(fs_sorter* s, int dtype, const void* keys, const uint32_t* vals, bool with_vals, uint64_t n,
                       uint64_t gpos_base, const void* splitter_keys, const uint64_t* splitter_gpos, int nsplit,
                       void* const* bucket_dst, uint32_t* const* value_dst, int sync,
                       const uint64_t* send_matrix = nullptr, int rank = 0) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (!s->part.ready || s->part.dtype != dtype || s->part.nsplit != nsplit || s->part.keys != keys ||
      s->part.n != n)
    return fail(s, FS_E_INVALID, "fs_partition_dispatch must follow fs_partition_count of the same keys and splitters");
  s->part.ready = false;
  if (n == 0) return FS_OK;
  if (!bucket_dst) return fail(s, FS_E_INVALID, "bucket_dst is NULL");
  if (with_vals && !value_dst) return fail(s, FS_E_INVALID, "value_dst is NULL");
  for (int b = 0; b <= nsplit; ++b) {
    if (!bucket_dst[b]) return fail(s, FS_E_INVALID, "bucket_dst[%d] is NULL", b);
    if (with_vals && !value_dst[b]) return fail(s, FS_E_INVALID, "value_dst[%d] is NULL", b);
  }
  if (with_vals && !vals && gpos_base + n > (1ull << 32))
    return fail(s, FS_E_INVALID, "global positions past 2^32 do not fit u32 indices");
  if (send_matrix && (rank < 0 || rank > nsplit))
    return fail(s, FS_E_INVALID, "rank %d outside [0, %d]", rank, nsplit);
  if ((rc = set_device(s))) return rc;
  if (with_vals && vals && (rc = prepare_ptr(s, vals, (size_t)n * 4, "values"))) return rc;
  void* const* kd = bucket_dst;
  uint32_t* const* vd = value_dst;
  if (send_matrix) {  // destinations = inbox bases + what lower ranks send, computed on the device
    const int G = nsplit + 1;
    if ((rc = prepare_ptr(s, send_matrix, (size_t)G * G * 8, "send_matrix"))) return rc;
    if (!s->dst_tab) FS_CUDA(s, cudaMalloc(&s->dst_tab, 2 * RADIX * sizeof(void*)));
    DispatchBases bases{};
    for (int b = 0; b < G; ++b) {
      bases.key[b] = reinterpret_cast<uintptr_t>(bucket_dst[b]);
      bases.val[b] = with_vals ? reinterpret_cast<uintptr_t>(value_dst[b]) : 0;
    }
    k_dispatch_table<<<1, RADIX, 0, s->stream>>>(reinterpret_cast<const unsigned long long*>(send_matrix), G, rank,
                                                 key_bytes_of(dtype), bases, with_vals ? 1 : 0,
                                                 static_cast<void**>(s->dst_tab));
    FS_CUDA(s, cudaGetLastError());
    kd = nullptr;  // the table is ready on the device
    vd = nullptr;
  }
#define FS_PD(K, XF)                                                                                         \
  enqueue_partition_dispatch<K, XF>(s, keys, vals, with_vals, n, gpos_base, splitter_keys, splitter_gpos, nsplit, \
                                    kd, vd)
  FS_PARTITION_DTYPES(FS_PD)
#undef FS_PD
  if (rc) return rc;
  return finish(s, sync);
}
}  // namespace

int fs_partition_dispatch_matrix(fs_sorter* s, int dtype, const void* keys, const uint32_t* vals, int payload,
                                 uint64_t n, uint64_t gpos_base, const void* splitter_keys,
                                 const uint64_t* splitter_gpos, int nsplit, const uint64_t* send_matrix, int rank,
                                 void* const* inbox_keys, uint32_t* const* inbox_vals, int sync) {
  if (!send_matrix) return s ? fail(s, FS_E_INVALID, "send_matrix is NULL") : FS_E_INVALID;
  return partition_dispatch(s, dtype, keys, vals, payload != 0, n, gpos_base, splitter_keys, splitter_gpos, nsplit,
                            inbox_keys, inbox_vals, sync, send_matrix, rank);
}

int fs_partition_dispatch(fs_sorter* s, int dtype, const void* keys, uint64_t n, uint64_t gpos_base,
                          const void* splitter_keys, const uint64_t* splitter_gpos, int nsplit,
                          void* const* bucket_dst, int sync) {
  return partition_dispatch(s, dtype, keys, nullptr, false, n, gpos_base, splitter_keys, splitter_gpos, nsplit,
                            bucket_dst, nullptr, sync);
}

int fs_partition_dispatch_pairs(fs_sorter* s, int dtype, const void* keys, const uint32_t* vals, uint64_t n,
                                uint64_t gpos_base, const void* splitter_keys, const uint64_t* splitter_gpos,
                                int nsplit, void* const* bucket_dst, uint32_t* const* value_dst, int sync) {
  return partition_dispatch(s, dtype, keys, vals, true, n, gpos_base, splitter_keys, splitter_gpos, nsplit,
                            bucket_dst, value_dst, sync);
}

int fs_sort_pairs_copy(fs_sorter* s, int dtype, const void* keys_in, const uint32_t* vals_in, void* keys_out,
                       uint32_t* vals_out, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  if (n == 0) return FS_OK;
  if (!keys_in || !keys_out || !vals_out) return fail(s, FS_E_INVALID, "keys_in, keys_out or vals_out is NULL");
  if ((rc = set_device(s))) return rc;
  const int kb = key_bytes_of(dtype);
  auto overlap = [n](const void* a, size_t ea, const void* b, size_t eb) {
    const char* x = static_cast<const char*>(a);
    const char* y = static_cast<const char*>(b);
    return x < y + n * eb && y < x + n * ea;
  };
  if (overlap(keys_in, kb, keys_out, kb) || overlap(keys_out, kb, vals_out, 4) ||
      (vals_in && (overlap(vals_in, 4, vals_out, 4) || overlap(vals_in, 4, keys_out, kb))))
    return fail(s, FS_E_INVALID, "inputs and outputs overlap");
  if ((rc = prepare_ptr(s, keys_in, (size_t)n * kb, "keys_in"))) return rc;
  if (vals_in && (rc = prepare_ptr(s, vals_in, (size_t)n * 4, "vals_in"))) return rc;
  if ((rc = prepare_ptr(s, keys_out, (size_t)n * kb, "keys_out"))) return rc;
  if ((rc = prepare_ptr(s, vals_out, (size_t)n * 4, "vals_out"))) return rc;
  if (n == 1) {
    FS_CUDA(s, cudaMemcpyAsync(keys_out, keys_in, kb, cudaMemcpyDeviceToDevice, s->stream));
    if (vals_in)
      FS_CUDA(s, cudaMemcpyAsync(vals_out, vals_in, 4, cudaMemcpyDeviceToDevice, s->stream));
    else
      FS_CUDA(s, cudaMemsetAsync(vals_out, 0, 4, s->stream));
    s->last_launches = 0;
    return finish(s, sync);
  }
  if ((rc = grow(s, &s->kother, &s->kother_bytes, (size_t)n * kb, false))) return rc;
  if ((rc = grow(s, &s->vother, &s->vother_bytes, (size_t)n * 4, false))) return rc;
  PlanArgs a{};
  a.n = n;
  a.kin = keys_in;
  a.kfinal = keys_out;
  a.kother = s->kother;
  a.vin = vals_in;  // nullptr: input positions (argsort with the sorted keys)
  a.vfinal = vals_out;
  a.vother = static_cast<uint32_t*>(s->vother);
  a.passes = kb;
  a.has_vals = 1;
  a.write_keys = 1;
  a.key_bytes = kb;
  if ((rc = dispatch(s, dtype, a))) return rc;
  return finish(s, sync);
}

int fs_gather(fs_sorter* s, int width, const void* src, uint64_t src_n, const uint32_t* idx, void* dst, uint64_t n,
              int sync) {
  if (!s) return FS_E_INVALID;
  if (width != 4 && width != 8) return fail(s, FS_E_INVALID, "width must be 4 or 8 bytes, got %d", width);
  if (n == 0) return FS_OK;
  if (!src || !idx || !dst) return fail(s, FS_E_INVALID, "src, idx or dst is NULL");
  int rc = set_device(s);
  if (rc) return rc;
  // Page-locked host operands (SortBuffers, ForgeContext buffers) go through
  // device staging as the sorts do.  A page-locked source much larger than
  // the gather is read in place over the bus instead: n random reads of one
  // 32-byte sector each cost less than copying all of it.
  void* srcv = const_cast<void*>(src);
  void* idxv = nullptr;
  void* dstv = nullptr;
  bool src_in_place = false;
  if (is_pinned_host(src) && n * 32 < src_n * (uint64_t)width) {
    cudaPointerAttributes at{};
    src_in_place = cudaPointerGetAttributes(&at, src) == cudaSuccess && at.devicePointer == src;
    cudaGetLastError();
  }
  if (!src_in_place &&
      (rc = device_view(s, src, (size_t)src_n * width, "src", &s->dkeys, &s->dkeys_bytes, true, &srcv)))
    return rc;
  if ((rc = device_view(s, idx, (size_t)n * 4, "idx", &s->dvals, &s->dvals_bytes, true, &idxv))) return rc;
  if ((rc = device_view(s, dst, (size_t)n * width, "dst", &s->kother, &s->kother_bytes, false, &dstv))) return rc;
  const uint64_t blocks = (n / 4 + 255) / 256 + 1;
  const uint64_t cap = (uint64_t)s->sm_count * 8;
  const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
  if (width == 4)
    k_gather<uint32_t><<<grid, 256, 0, s->stream>>>(static_cast<const uint32_t*>(srcv), src_n,
                                                  static_cast<const uint32_t*>(idxv), static_cast<uint32_t*>(dstv),
                                                  n, s->host_err_dev);
  else
    k_gather<uint64_t><<<grid, 256, 0, s->stream>>>(static_cast<const uint64_t*>(srcv), src_n,
                                                  static_cast<const uint32_t*>(idxv), static_cast<uint64_t*>(dstv),
                                                  n, s->host_err_dev);
  FS_CUDA(s, cudaGetLastError());
  if ((rc = copy_back(s, dst, dstv, (size_t)n * width))) return rc;
  s->last_launches = 1;
  return finish(s, sync);
}

// ---- streams for callers without a CUDA runtime of their own ----------------
int fs_stream_create(int device, void** stream) {
  if (!stream) return fail(nullptr, FS_E_INVALID, "stream is NULL");
  *stream = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(nullptr, FS_E_DEVICE_NOT_FOUND, "no CUDA device");
  }
  if (device < 0 || device >= count) return fail(nullptr, FS_E_DEVICE_NOT_FOUND, "no CUDA device %d", device);
  cudaStream_t st = nullptr;
  if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess) {
    cudaGetLastError();
    return fail(nullptr, FS_E_GPU_EXECUTION, "cudaStreamCreate: %s", cudaGetErrorString(e));
  }
  *stream = st;
  return FS_OK;
}

int fs_stream_synchronize(void* stream) {
  if (!stream) return fail(nullptr, FS_E_INVALID, "stream is NULL");
  const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(nullptr, FS_E_GPU_EXECUTION, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  }
  return FS_OK;
}

int fs_stream_destroy(void* stream) {
  if (!stream) return FS_OK;
  cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(nullptr, FS_E_GPU_EXECUTION, "cudaStreamDestroy: %s", cudaGetErrorString(e));
  }
  return FS_OK;
}

int fs_ipc_export(fs_sorter* s, void* ptr, void* handle_out) {
  if (!s || !ptr || !handle_out) return s ? fail(s, FS_E_INVALID, "fs_ipc_export: NULL argument") : FS_E_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == FS_IPC_HANDLE_BYTES, "IPC handle size");
  int rc = set_device(s);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  FS_CUDA(s, cudaIpcGetMemHandle(&h, ptr));
  std::memcpy(handle_out, &h, sizeof h);
  return FS_OK;
}

int fs_ipc_open(fs_sorter* s, const void* handle, void** ptr_out) {
  if (!s || !handle || !ptr_out) return s ? fail(s, FS_E_INVALID, "fs_ipc_open: NULL argument") : FS_E_INVALID;
  int rc = set_device(s);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  FS_CUDA(s, cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return FS_OK;
}

int fs_ipc_close(fs_sorter* s, void* ptr) {
  if (!s || !ptr) return s ? fail(s, FS_E_INVALID, "fs_ipc_close: NULL argument") : FS_E_INVALID;
  int rc = set_device(s);
  if (rc) return rc;
  FS_CUDA(s, cudaIpcCloseMemHandle(ptr));
  return FS_OK;
}

int fs_set_wait_timeout_ms(fs_sorter* s, uint64_t ms) {
  if (!s) return FS_E_INVALID;
  if (ms == 0 || ms > 3600000ull) return fail(s, FS_E_INVALID, "wait timeout %llu ms outside [1, 3600000]",
                                             (unsigned long long)ms);
  s->timeout_ns = ms * 1000000ull;
  return FS_OK;
}

int fs_set_single_launch_max(fs_sorter* s, uint64_t key_bytes) {
  if (!s) return FS_E_INVALID;
  s->coop_max_bytes = key_bytes;
  return FS_OK;
}

int fs_test_inject(fs_sorter* s, int kind, int arg) {
  if (!s) return FS_E_INVALID;
  switch (kind) {
    case 0:
      s->test_withhold = 0;
      s->test_fail_alloc = 0;
      s->test_skip_arrival = 0;
      return FS_OK;
    case FS_TEST_SKIP_ARRIVAL:
      s->test_skip_arrival = 1;
      return FS_OK;
    case FS_TEST_WITHHOLD_COPY:
      s->test_withhold = 1;
      return FS_OK;
    case FS_TEST_FAIL_ALLOC:
      if (arg < 1) return fail(s, FS_E_INVALID, "FS_TEST_FAIL_ALLOC needs arg >= 1, got %d", arg);
      s->test_fail_alloc = arg;
      return FS_OK;
    default:
      return fail(s, FS_E_INVALID, "unknown injection kind %d", kind);
  }
}

// ---- SortBuffer objects ------------------------------------------------------
// Buffer-only calls report errors through fs_last_error(NULL): a buffer may
// outlive the sorter that created it.
namespace {
// Wait for the device work that may have written the buffer.
int buffer_wait(fs_buffer* b) {
  if (b->any_stream) {
    FS_CUDA(nullptr, cudaDeviceSynchronize());
  } else if (b->pending) {
    FS_CUDA(nullptr, cudaEventSynchronize(b->done));
  }
  b->pending = false;
  return FS_OK;
}

// Bring the leading `need` bytes of the device copy up to date with the host
// mirror, enqueued on `st`.
int buffer_to_device(fs_sorter* s, fs_buffer* b, uint64_t need, cudaStream_t st) {
  if (b->dev_valid >= need) return FS_OK;
  FS_CUDA(s, cudaMemcpyAsync(static_cast<char*>(b->dev) + b->dev_valid, static_cast<char*>(b->host) + b->dev_valid,
                             need - b->dev_valid, cudaMemcpyHostToDevice, st));
  b->dev_valid = need;
  return FS_OK;
}

int check_buffer(fs_sorter* s, const fs_buffer* b, uint64_t need, const char* what) {
  if (!b) return fail(s, FS_E_INVALID, "%s is NULL", what);
  if (b->device != s->device)
    return fail(s, FS_E_INVALID, "%s lives on device %d, the sorter on device %d", what, b->device, s->device);
  if (need > b->bytes)
    return fail(s, FS_E_INVALID, "%s holds %llu bytes, %llu needed", what, (unsigned long long)b->bytes,
                (unsigned long long)need);
  return FS_OK;
}

// After a sort enqueued on s's stream wrote the leading `need` bytes.
int buffer_sorted(fs_sorter* s, fs_buffer* b, uint64_t need) {
  if (need > b->dev_newer) b->dev_newer = need;
  FS_CUDA(s, cudaEventRecord(b->done, s->stream));
  b->pending = true;
  b->any_stream = false;
  return FS_OK;
}
}  // namespace

int fs_buffer_create(fs_sorter* s, uint64_t bytes, fs_buffer** out) {
  if (!s || !out) return s ? fail(s, FS_E_INVALID, "out is NULL") : FS_E_INVALID;
  *out = nullptr;
  int rc = set_device(s);
  if (rc) return rc;
  const uint64_t b = bytes ? bytes : 16;
  fs_buffer* buf = new fs_buffer();
  buf->device = s->device;
  buf->bytes = b;
  cudaError_t e = cudaMalloc(&buf->dev, b);
  if (e == cudaSuccess) e = cudaHostAlloc(&buf->host, b, cudaHostAllocPortable);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&buf->done, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (buf->host) cudaFreeHost(buf->host);
    if (buf->dev) cudaFree(buf->dev);
    delete buf;
    return fail(s, e == cudaErrorMemoryAllocation ? FS_E_OOM : FS_E_GPU_EXECUTION, "SortBuffer of %llu bytes: %s",
                (unsigned long long)b, cudaGetErrorString(e));
  }
  *out = buf;
  return FS_OK;
}

int fs_buffer_destroy(fs_buffer* b) {
  if (!b) return FS_OK;
  cudaSetDevice(b->device);
  buffer_wait(b);
  cudaFree(b->dev);
  cudaFreeHost(b->host);
  cudaEventDestroy(b->done);
  cudaGetLastError();
  delete b;
  return FS_OK;
}

void* fs_buffer_host(const fs_buffer* b) { return b ? b->host : nullptr; }
void* fs_buffer_device(const fs_buffer* b) { return b ? b->dev : nullptr; }
uint64_t fs_buffer_bytes(const fs_buffer* b) { return b ? b->bytes : 0; }

int fs_buffer_host_read(fs_buffer* b) {
  if (!b) return fail(nullptr, FS_E_INVALID, "buffer is NULL");
  FS_CUDA(nullptr, cudaSetDevice(b->device));
  int rc = buffer_wait(b);
  if (rc) return rc;
  if (b->dev_newer) FS_CUDA(nullptr, cudaMemcpy(b->host, b->dev, b->dev_newer, cudaMemcpyDeviceToHost));
  b->dev_newer = 0;
  return FS_OK;
}

int fs_buffer_host_write(fs_buffer* b) {
  const int rc = fs_buffer_host_read(b);
  if (rc) return rc;
  b->dev_valid = 0;  // the host may change any byte: the device copy is stale
  return FS_OK;
}

int fs_buffer_device_use(fs_buffer* b, uint64_t bytes) {
  if (!b) return fail(nullptr, FS_E_INVALID, "buffer is NULL");
  if (bytes > b->bytes)
    return fail(nullptr, FS_E_INVALID, "SortBuffer holds %llu bytes, %llu requested", (unsigned long long)b->bytes,
                (unsigned long long)bytes);
  FS_CUDA(nullptr, cudaSetDevice(b->device));
  // no wait: a sort still in flight only touches bytes the device already
  // holds, and the copy below fills bytes past them
  if (b->dev_valid < bytes) {
    FS_CUDA(nullptr, cudaMemcpy(static_cast<char*>(b->dev) + b->dev_valid, static_cast<char*>(b->host) + b->dev_valid,
                                bytes - b->dev_valid, cudaMemcpyHostToDevice));
    b->dev_valid = bytes;
  }
  if (bytes > b->dev_newer) b->dev_newer = bytes;  // device code may write through the pointer
  b->any_stream = true;
  return FS_OK;
}

int fs_sort_buffer(fs_sorter* s, int dtype, fs_buffer* keys, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  const uint64_t need = n * (uint64_t)key_bytes_of(dtype);
  if ((rc = check_buffer(s, keys, need, "keys"))) return rc;
  if (n <= 1) return FS_OK;
  if ((rc = set_device(s))) return rc;
  if (keys->any_stream && (rc = buffer_wait(keys))) return fail(s, rc, "%s", fs_last_error(nullptr));
  if ((rc = buffer_to_device(s, keys, need, s->stream))) return rc;
  if ((rc = fs_sort_keys(s, dtype, keys->dev, n, sync))) return rc;
  return buffer_sorted(s, keys, need);
}

int fs_sort_pairs_buffer(fs_sorter* s, int dtype, fs_buffer* keys, fs_buffer* vals, uint64_t n, int sync) {
  int rc = check_common(s, dtype, n);
  if (rc) return rc;
  const uint64_t kneed = n * (uint64_t)key_bytes_of(dtype), vneed = n * 4;
  if ((rc = check_buffer(s, keys, kneed, "keys"))) return rc;
  if ((rc = check_buffer(s, vals, vneed, "values"))) return rc;
  if (keys == vals) return fail(s, FS_E_INVALID, "keys and values are the same SortBuffer");
  if (n <= 1) return FS_OK;
  if ((rc = set_device(s))) return rc;
  for (fs_buffer* b : {keys, vals})
    if (b->any_stream && (rc = buffer_wait(b))) return fail(s, rc, "%s", fs_last_error(nullptr));
  if ((rc = buffer_to_device(s, keys, kneed, s->stream))) return rc;
  if ((rc = buffer_to_device(s, vals, vneed, s->stream))) return rc;
  if ((rc = fs_sort_pairs(s, dtype, keys->dev, static_cast<uint32_t*>(vals->dev), n, sync))) return rc;
  if ((rc = buffer_sorted(s, keys, kneed))) return rc;
  return buffer_sorted(s, vals, vneed);
}

uint64_t fs_scratch_bytes(const fs_sorter* s) {
  if (!s) return 0;
  return s->counts_bytes + s->offsets_bytes + s->kother_bytes + s->kfinal2_bytes + s->vother_bytes + s->dkeys_bytes +
         s->dvals_bytes + sizeof(SortCtl);
}

int fs_last_launch_count(const fs_sorter* s) { return s ? s->last_launches : 0; }

}  // extern "C"
