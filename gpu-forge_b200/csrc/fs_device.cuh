// fs_device.cuh -- device-side building blocks of the LSD radix sort:
// key-order transforms, digit extraction, and the device-resident control
// block the host enqueues against.
#pragma once

#include <cstddef>

#include <cstdint>
#include <cuda_runtime.h>

namespace fs {

constexpr int RADIX_BITS = 8;
constexpr int RADIX = 1 << RADIX_BITS;
constexpr int MAX_PASSES = 8;

// Order-preserving bijections onto unsigned order.  Mode numbers follow the
// reference's SortKey constants (forge-sort src/lib.rs:16-88): i32/i64 flip the
// sign bit both ways; f32/f64 use FloatFlip forward and its inverse
// (shaders/sort.metal:812-868).  Here they run inside the first pass's load
// and the last pass's store instead of in separate passes.
enum Xform : int { XF_NONE = 0, XF_SIGN = 1, XF_FLOAT = 2 };

template <typename K> struct KeyBits;
template <> struct KeyBits<uint32_t> {
  using S = int32_t;
  static constexpr int BITS = 32;
  static constexpr uint32_t SIGN = 0x80000000u;
};
template <> struct KeyBits<uint64_t> {
  using S = int64_t;
  static constexpr int BITS = 64;
  static constexpr uint64_t SIGN = 0x8000000000000000ull;
};

// total_cmp order == unsigned order of: negative -> ~x, non-negative -> x^sign.
template <typename K, int XF>
__host__ __device__ __forceinline__ K to_ordered(K x) {
  using T = KeyBits<K>;
  if constexpr (XF == XF_SIGN) {
    return x ^ T::SIGN;
  } else if constexpr (XF == XF_FLOAT) {
    K neg = (K)((typename T::S)x >> (T::BITS - 1));  // all ones if negative
    return x ^ (neg | T::SIGN);
  } else {
    return x;
  }
}

template <typename K, int XF>
__host__ __device__ __forceinline__ K from_ordered(K y) {
  using T = KeyBits<K>;
  if constexpr (XF == XF_SIGN) {
    return y ^ T::SIGN;
  } else if constexpr (XF == XF_FLOAT) {
    K hi = (K)((typename T::S)y >> (T::BITS - 1));  // all ones if sign set
    return y ^ (~hi | T::SIGN);
  } else {
    return y;
  }
}

template <typename K>
__device__ __forceinline__ uint32_t digit_of(K x, int shift) {
  return (uint32_t)(x >> shift) & (RADIX - 1);
}

__device__ __forceinline__ int ld_relaxed_s32(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- device-resident control block ------------------------------------------
// Pass descriptors are written on the device by the plan kernel (which knows,
// from the histogram, which passes are trivial), so the host never waits for
// the histogram before enqueueing the passes.
enum PassFlags : uint32_t {
  PD_EXEC = 1u << 0,        // run this pass (not every key has the same digit)
  PD_XF_IN = 1u << 1,       // first executed pass: apply the forward transform
  PD_XF_OUT = 1u << 2,      // last executed pass: apply the inverse transform
  PD_SYNTH_IDX = 1u << 3,   // payload = input position (argsort), not loaded
  PD_WRITE_KEYS = 1u << 4,  // write keys (argsort's last pass does not)
  PD_FIRST = 1u << 5,       // first executed pass (reads the caller's keys)
  PD_UNSTABLE = 1u << 6,    // keys-only first pass: order among equal digits is free
  PD_TEST_WITHHOLD = 1u << 7,  // failure-path test: CTA 0 never issues its first bulk copy
  PD_SORTED_BELOW = 1u << 8,   // keys only: the input is sorted by the bits in `below`, and
                               // only their order has to survive among equal digits
};

struct PassDesc {
  const void* kin;
  void* kout;
  const uint32_t* vin;
  uint32_t* vout;
  uint32_t flags;
  uint32_t below;  // PD_SORTED_BELOW: bits of the (32-bit, ordered) key whose order the pass keeps
};

enum FinalOps : uint32_t {
  FIN_COPY_KEYS = 1u << 0,
  FIN_COPY_VALS = 1u << 1,
  FIN_IOTA_VALS = 1u << 2,
};

struct FinalDesc {
  const void* ksrc;
  void* kdst;
  const uint32_t* vsrc;
  uint32_t* vdst;
  uint32_t ops;
  uint32_t executed_passes;
};

// Device error codes (ctl->err).
constexpr int DEV_ERR_TIMEOUT = 1;  // a bounded wait (bulk-copy barrier) ran out
constexpr int DEV_ERR_BOUNDS = 2;  // a scatter position fell outside [0, n)

// Histogram-fill stage of a keys-only 32-bit sort (plan with `h16`): where
// the keys grouped by their top 16 bits are, and how to read them.
enum HfFlags : uint32_t {
  HF_ON = 1u << 0,     // the stage runs
  HF_XF_IN = 1u << 1,  // no pass ran: the source holds the caller's keys (apply the forward transform)
};

struct SortCtl {
  // Accumulators, cleared before every sort (the first CTL_ACCUM_BYTES):
  unsigned long long hist[MAX_PASSES][RADIX];  // global digit counts of each pass
  unsigned long long kor;    // OR of all ordered keys
  unsigned long long kandn;  // OR of all complemented ordered keys (= ~AND)
  PassDesc pass[MAX_PASSES];
  FinalDesc fin;
  const void* hf_src;  // keys grouped by their top 16 bits (ordered unless HF_XF_IN)
  void* hf_dst;        // where the histogram fill writes the sorted keys
  void* hf_pool;       // a buffer of n keys that is free during the fill: the
                       // histograms of the groups too large for one CTA
  uint32_t hf_flags;   // HfFlags
  int err;  // first device-side failure (DEV_ERR_*)
};

// Slice geometry shared by the histogram, count, scan and scatter kernels:
// slice c holds keys [c*keys_per_slice, min((c+1)*keys_per_slice, n)), a whole
// number of scatter tiles, and is owned by CTA c of each of those kernels.
struct Slices {
  uint64_t keys_per_slice;
  uint32_t count;
};

// Per-sort arguments of the plan kernel: where the keys and payload come from
// and where they must end up.
// Bytes of SortCtl that are zeroed before every sort: hist, kor and kandn.
constexpr size_t CTL_ACCUM_BYTES = sizeof(unsigned long long) * (MAX_PASSES * RADIX + 2);
static_assert(offsetof(SortCtl, pass) == CTL_ACCUM_BYTES, "accumulators lead SortCtl");

struct PlanArgs {
  uint64_t n;
  const void* kin;   // pass-1 key source (may be const user input)
  void* kfinal;      // where sorted keys must land
  void* kother;      // scratch of n keys (never equal to kfinal)
  const uint32_t* vin;  // payload source; nullptr = synthesise indices
  uint32_t* vfinal;
  uint32_t* vother;
  int passes;        // digit passes: 4 (32-bit keys) or 8 (64-bit keys)
  int has_vals;      // carry a payload
  int write_keys;    // keys are an output (false for argsort)
  int key_bytes;
  unsigned long long* counts_out;  // optional copy of pass-0 digit counts
  int ncounts;                     // entries of counts_out
  int unstable_first;              // keys-only LSD sort: first pass may reorder ties
  int force_exec;                  // single-pass plans: run the pass even if trivial
  int trivial_from_bits;           // 1: a pass is trivial when kor/kandn show its
                                   // digit never varies; 0: when hist[0] has one
                                   // digit holding all n keys (single-pass plans)
  int test_withhold;               // failure-path test (fs_test_inject): mark the
                                   // first executed pass PD_TEST_WITHHOLD
  int h16;                         // keys-only 32-bit sort: only the passes of the
                                   // top two digits run (the first may rank
                                   // unstably); the histogram fill sorts each
                                   // top-16-bit group by its low 16 bits
};

}  // namespace fs
