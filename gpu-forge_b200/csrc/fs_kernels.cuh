// fs_kernels.cuh -- the sm_100a kernels of one sort.
//
// Per sort (P = key bytes, one 8-bit digit per pass, LSD):
//   k_first_count    one read of the keys -> per-slice counts of digit 0 and
//                    their totals, OR / AND of all keys (which digits vary)
//   k_plan           trivial-pass detection, device-side buffer routing
// per executed pass:
//   k_count          per-slice counts of this pass's digit and their totals
//                    (pass 0: already counted by k_first_count)
//   k_slice_scan     per-(slice, digit) global output offsets
//   k_scatter        CTA c walks slice c tile by tile: warp multisplit rank,
//                    shared-memory staging by digit, coalesced scatter;
//                    payload carried alongside; next tile bulk-prefetched
// then:
//   k_finalize       copy-back / iota when the plan needs it; error hand-off
// (2 + 3P launches in a row on one stream, each after the first chained to
// its predecessor: chain_wait below.)  Up to a few thousand keys,
// k_small_sort does the whole sort in one CTA instead.
//
// The array is cut into contiguous slices (12 per SM, whole tiles each) that
// the scatter CTAs take in turn; no CTA ever waits on another: the offsets a
// slice needs come from the counts, not from a chained scan across
// concurrently running tiles.  That costs one extra read of the keys per pass
// after the first and removes the latency-bound inter-CTA dependency chain.
// The sample sort's partition reuses count, scan and scatter with the
// splitter bucket as the digit (k_bucket_hist, SplitterDigit, and
// SplitterDispatch, which stores each bucket into another GPU's inbox).
//
// Replaces the reference pipeline sort_msd_histogram -> sort_msd_prep ->
// sort_msd_atomic_scatter -> sort_inner_fused (+ sort_transform_*,
// sort_init_indices, sort_gather_values) of forge-sort shaders/sort.metal.
#pragma once

#include "fs_device.cuh"

#include <type_traits>

#ifndef FS_RANK_BALLOT
#define FS_RANK_BALLOT 3
#endif

namespace fs {

// ---- bulk-copy (TMA, non-tensor, no multicast) + mbarrier helpers ----------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Programmatic dependent launch: a kernel of the sort's chain may be
// scheduled while its predecessor on the stream is still draining, and
// waits here -- its first statement, on every path -- until the predecessor
// has completed and its memory operations are visible.  Launched without
// the attribute, the wait returns at once.
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// global -> shared bulk copy; both addresses 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
// Bounded wait on an mbarrier phase; false (and *err set) on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t timeout_ns, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && global_timer_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, DEV_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---- digit functors ------------------------------------------------------------
// A radix pass takes byte `shift/8` of the ordered key; the sample sort's
// partition pass takes the index of the splitter bucket that the element's
// (ordered key, global position) falls in.  The position breaks ties, so
// equal keys still spread over ranks in input order.
struct RadixDigit {
  int shift;
  static constexpr int DIGITS = RADIX;     // digit values 0 .. DIGITS-1
  static constexpr bool STAGE = false;     // recomputed from the staged key
  static constexpr bool DISPATCH = false;  // output is one contiguous array
  template <typename K>
  __device__ __forceinline__ uint32_t operator()(K k, uint64_t) const {
    // one byte-permute instruction instead of shift + mask
    if constexpr (sizeof(K) == 4) {
      return __byte_perm((uint32_t)k, 0u, 0x4440u | (uint32_t)(shift >> 3));
    } else {
      const uint32_t half = shift >= 32 ? (uint32_t)((uint64_t)k >> 32) : (uint32_t)k;
      return __byte_perm(half, 0u, 0x4440u | (uint32_t)((shift >> 3) & 3));
    }
  }
};

// LV: how the splitter search runs.  1, 2, 3: a fixed lower-bound tree of that
// many levels over 1, 3 or 7 splitters held in registers (2, 4 or 8 GPUs;
// unused entries hold the largest key); 0: a binary search over the
// shared-memory copy, for any count up to 255.
template <typename K, int XF, int LV = 3>
struct SplitterDigit {
  const K* keys;         // nsplit raw splitter keys, ascending by (key, gpos)
  const uint64_t* gpos;  // their global positions
  int nsplit;
  // shared-memory copy (ordered keys), set by stage_in before any lookup
  const K* s_keys = nullptr;
  const uint64_t* s_gpos = nullptr;
  uint32_t top = 0;  // largest power of two <= nsplit (0 if none)
  K r[7] = {};       // up to 7 splitters in registers, padded with the largest key
  static constexpr int DIGITS = RADIX;
  static constexpr bool STAGE = true;  // digits staged in shared memory
  static constexpr bool DISPATCH = false;
  static_assert(LV >= 0 && LV <= 3, "register tree of at most 3 levels");
  // Number of splitters <= (k, g) in (ordered key, position) order.  First
  // the splitters whose key is below k (lower bound); the search also yields
  // the first splitter key >= k, so a tie -- a key equal to a splitter key,
  // rare but possible with heavy duplicates -- is seen without another load,
  // and only then are positions compared.  gpos_of() returns the key's
  // global position and runs on that path only.
  template <typename G>
  __device__ __forceinline__ uint32_t operator()(K k, G&& gpos_of) const {
    uint32_t pos = 0;
    K cand = ~K(0);  // smallest splitter key >= k seen by the search
    if constexpr (LV == 1) {
      const bool right = r[0] < k;
      pos = right ? 1u : 0u;
      cand = right ? cand : r[0];
    } else if constexpr (LV == 2) {
      bool right = r[1] < k;
      pos = right ? 2u : 0u;
      cand = right ? cand : r[1];
      const K m = right ? r[2] : r[0];
      right = m < k;
      pos += right ? 1u : 0u;
      cand = right ? cand : m;
    } else if constexpr (LV == 3) {
      bool right = r[3] < k;
      pos = right ? 4u : 0u;
      cand = right ? cand : r[3];
      K m = right ? r[5] : r[1];
      right = m < k;
      pos += right ? 2u : 0u;
      cand = right ? cand : m;
      m = (pos & 4) ? ((pos & 2) ? r[6] : r[4]) : ((pos & 2) ? r[2] : r[0]);
      right = m < k;
      pos += right ? 1u : 0u;
      cand = right ? cand : m;
    } else {
      __builtin_assume(__isShared(s_keys));
      for (uint32_t step = top; step != 0; step >>= 1) {
        const uint32_t j = pos + step - 1;
        if (j < (uint32_t)nsplit && s_keys[j] < k) pos += step;
      }
      cand = pos < (uint32_t)nsplit ? s_keys[pos] : ~K(0);
    }
    if (cand == k && pos < (uint32_t)nsplit) {
      __builtin_assume(__isShared(s_keys) && __isShared(s_gpos));
      const uint64_t g = gpos_of();
      while (pos < (uint32_t)nsplit && s_keys[pos] == k && s_gpos[pos] <= g) ++pos;
    }
    return pos;
  }
  // Copy the splitters (ordered) into shared memory (at least 8 entries,
  // the unused ones set to the largest key) and point there; the caller
  // synchronises the CTA before the first lookup.
  __device__ __forceinline__ void stage_in(K* sk, uint64_t* sg) {
    const int len = nsplit > 8 ? nsplit : 8;
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
      sk[i] = i < nsplit ? to_ordered<K, XF>(keys[i]) : ~K(0);
      sg[i] = i < nsplit ? gpos[i] : 0ull;
    }
    s_keys = sk;
    s_gpos = sg;
    top = nsplit > 0 ? 1u << (31 - __clz(nsplit)) : 0u;
#pragma unroll
    for (int i = 0; i < 7; ++i) r[i] = i < nsplit ? to_ordered<K, XF>(keys[i]) : ~K(0);
  }
};

// Register-tree depth for nsplit splitters (0: shared-memory search).
__host__ __device__ constexpr int splitter_levels(int nsplit) {
  return nsplit <= 1 ? 1 : nsplit <= 3 ? 2 : nsplit <= 7 ? 3 : 0;
}

// Sample-sort dispatch: the splitter bucket is the digit, and bucket b's keys
// go to dst[b] -- this rank's region of rank b's inbox, which may be another
// GPU's memory reached with plain stores over NVLink -- at their stable rank
// within the bucket.
// NB = bucket capacity of the instantiation: 8 covers the GPUs of one box
// (tile counters and scans sized for 8 digits, ranking by three ballots);
// 256 covers any splitter count.
// With a payload, value i goes to vdst[b] at the same position as key i.
template <typename K, int XF, int NB = RADIX, int LV = 3>
struct SplitterDispatch : SplitterDigit<K, XF, LV> {
  static constexpr int DIGITS = NB;
  static constexpr bool DISPATCH = true;
  K* const* dst;          // device array of nsplit + 1 key destinations
  uint32_t* const* vdst;  // device array of nsplit + 1 value destinations (payload only)
};

// Visit the keys of [lo, hi) with the CTA's threads in coalesced order, 16-byte
// vector loads when `keys` is 16-byte aligned (VEC), four loads (64 bytes) in
// flight per thread to cover HBM latency; f(key, valid) is called by whole
// warps (valid = in range).
template <typename K, int BLOCK, bool VEC, typename F>
__device__ __forceinline__ void for_each_key(const K* __restrict__ keys, uint64_t lo, uint64_t hi, F&& f) {
  const uint32_t lane = threadIdx.x & 31, wbase = threadIdx.x & ~31u;
  uint64_t tail = lo;
  if constexpr (VEC) {
    constexpr int KV = 16 / (int)sizeof(K);
    constexpr int U = 4;
    // lo is a multiple of KV for every slice (slices are whole tiles)
    const uint64_t v0 = lo / KV, v1 = hi / KV;
    const uint4* kv = reinterpret_cast<const uint4*>(keys);
    uint64_t w = v0 + wbase;
    for (; w + (U - 1) * BLOCK + 32 <= v1; w += U * BLOCK) {
      uint4 a[U];
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = __ldcs(kv + w + u * BLOCK + lane);  // streamed: read once
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const K* ka = reinterpret_cast<const K*>(&a[u]);
#pragma unroll
        for (int q = 0; q < KV; ++q) f(ka[q], true);
      }
    }
    for (; w < v1; w += BLOCK) {
      const bool valid = w + lane < v1;
      const uint4 a = valid ? kv[w + lane] : make_uint4(0, 0, 0, 0);
      const K* ka = reinterpret_cast<const K*>(&a);
#pragma unroll
      for (int q = 0; q < KV; ++q) f(ka[q], valid);
    }
    tail = v1 * KV;
  }
  for (uint64_t w = tail + wbase; w < hi; w += BLOCK) {
    const bool valid = w + lane < hi;
    f(valid ? keys[w + lane] : K(0), valid);
  }
}

// --------------------------------------------------------------------------
// First count: one read of the keys gives
//   - the slice counts of the digit of pass `fpass` (0 for an LSD sort, 2
//     when only the top two digits are sorted by passes) of the ordered keys
//     (counts[c][d]) and their global totals (ctl->hist[fpass]),
//   - the OR of the ordered keys and the OR of their complements: a digit
//     whose bits never vary marks a pass that would be the identity, which the
//     plan skips before any scatter runs.
// Later passes count their own digit (k_count) when their input exists, so
// no pass needs a histogram taken up front; testing for trivial passes needs
// only the two bitwise reductions.
// Replaces sort_msd_histogram (shaders/sort.metal:64-142), which counted only
// the most significant byte, and the per-bucket histograms that
// sort_inner_fused recomputed (sort.metal:378-769).
// --------------------------------------------------------------------------
template <typename K, int XF, int BLOCK, bool VEC>
__global__ void __launch_bounds__(BLOCK)
    k_first_count(const K* __restrict__ keys, const uint64_t n, SortCtl* __restrict__ ctl, const Slices sl,
                  uint32_t* __restrict__ counts /* [count][RADIX] */, const int fpass) {
  chain_wait();
  constexpr int WARPS = BLOCK / 32;
  __shared__ uint32_t hw[WARPS][RADIX];
  __shared__ uint32_t tot[RADIX];
  uint32_t* h = hw[threadIdx.x >> 5];
  for (int i = threadIdx.x; i < WARPS * RADIX; i += BLOCK) (&hw[0][0])[i] = 0;
  for (int i = threadIdx.x; i < RADIX; i += BLOCK) tot[i] = 0;
  __syncthreads();
  K kor = 0, kandn = 0;
  const RadixDigit dg{fpass * RADIX_BITS};
  for (uint32_t c = blockIdx.x; c < sl.count; c += gridDim.x) {
    const uint64_t lo = (uint64_t)c * sl.keys_per_slice;
    const uint64_t hi = lo + sl.keys_per_slice < n ? lo + sl.keys_per_slice : n;
    for_each_key<K, BLOCK, VEC>(keys, lo, hi, [&](K x, bool valid) {
      if (valid) {
        const K o = to_ordered<K, XF>(x);
        kor |= o;
        kandn |= ~o;
        atomicAdd(&h[dg(o, 0)], 1u);
      }
    });
    __syncthreads();
    for (int b = threadIdx.x; b < RADIX; b += BLOCK) {
      uint32_t v = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        v += hw[w][b];
        hw[w][b] = 0;
      }
      counts[(size_t)c * RADIX + b] = v;
      tot[b] += v;
    }
    __syncthreads();
  }
  for (int b = threadIdx.x; b < RADIX; b += BLOCK)
    if (tot[b]) atomicAdd(&ctl->hist[fpass][b], (unsigned long long)tot[b]);
  // bitwise reductions: warp, then one atomic pair per warp
  uint32_t lo_or = __reduce_or_sync(0xffffffffu, (uint32_t)kor);
  uint32_t lo_an = __reduce_or_sync(0xffffffffu, (uint32_t)kandn);
  uint32_t hi_or = 0, hi_an = 0;
  if constexpr (sizeof(K) == 8) {
    hi_or = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kor >> 32));
    hi_an = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kandn >> 32));
  } else {
    hi_an = 0xffffffffu;  // bits above a 32-bit key never count as varying
  }
  if ((threadIdx.x & 31) == 0) {
    atomicOr(&ctl->kor, ((unsigned long long)hi_or << 32) | lo_or);
    atomicOr(&ctl->kandn, ((unsigned long long)hi_an << 32) | lo_an);
  }
}

// --------------------------------------------------------------------------
// Bucket histogram of the sample sort's partition pass (one pass, digit =
// splitter bucket): global counts into ctl->hist[0], slice counts into
// counts[c][*].  With few buckets (one per GPU) most lanes of a warp share a
// bucket, so the warp counts each bucket with one ballot instead of 32
// same-address atomics.
// --------------------------------------------------------------------------
// PACK: how a thread counts.  2 (one splitter): the number of keys in
// bucket 1 (bucket 0 is the rest of the slice); 4 / 8 (up to 3 / 7
// splitters): one add per key into 8-bit fields of a 32- / 64-bit register,
// folded every 250 or so keys into 16-bit fields (a thread sees fewer than
// 2^16 keys of a slice), summed by the warp once per slice; 0: one
// shared-memory atomic per key.
template <typename K, int XF, int BLOCK, typename D, int PACK>
__global__ void __launch_bounds__(BLOCK)
    k_bucket_hist(const K* __restrict__ keys, const uint64_t n, SortCtl* __restrict__ ctl, const Slices sl,
                  uint32_t* __restrict__ counts, const D dfn_in, const uint64_t gpos_base) {
  static_assert(PACK == 0 || PACK == 2 || PACK == 4 || PACK == 8, "counting mode");
  constexpr int KV = 16 / (int)sizeof(K);  // keys per 16-byte load
  __shared__ uint32_t h[RADIX];
  __shared__ uint32_t tot[RADIX];
  __shared__ K s_spk[RADIX];
  __shared__ uint64_t s_spg[RADIX];
  D dfn = dfn_in;
  dfn.stage_in(s_spk, s_spg);
  const uint32_t lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < RADIX; i += BLOCK) h[i] = tot[i] = 0;
  __syncthreads();
  using C8 = typename std::conditional<PACK == 8, uint64_t, uint32_t>::type;
  constexpr C8 EVEN = (C8)0x00ff00ff00ff00ffull;  // the 8-bit fields of even buckets, as 16-bit fields
  uint32_t c1 = 0;          // PACK 2: keys of bucket 1
  C8 c8 = 0;                // PACK 4 / 8: bucket b in bits [8b, 8b+8)
  C8 w_even = 0, w_odd = 0;  // 16-bit fields: buckets 0, 2, (4, 6) and 1, 3, (5, 7)
  auto add = [&](uint32_t b) {
    if constexpr (PACK == 2) {
      c1 += b;
    } else if constexpr (PACK == 4 || PACK == 8) {
      c8 += (C8)1 << (8 * b);
    } else {
      atomicAdd(&h[b], 1u);
    }
  };
  auto fold = [&]() {  // 8-bit fields -> 16-bit fields, before any can reach 256
    if constexpr (PACK == 4 || PACK == 8) {
      w_even += c8 & EVEN;
      w_odd += (c8 >> 8) & EVEN;
      c8 = 0;
    }
  };
  // keys a thread adds between folds: 2*KV per main-loop step, at most
  // KV + 1 more after the loop, never 256
  constexpr int FOLD_STEPS = (255 - KV - 1) / (2 * KV);
  const bool vec = (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
  for (uint32_t c = blockIdx.x; c < sl.count; c += gridDim.x) {
    const uint64_t lo = (uint64_t)c * sl.keys_per_slice;
    const uint64_t hi = lo + sl.keys_per_slice < n ? lo + sl.keys_per_slice : n;
    const uint32_t len = (uint32_t)(hi - lo);  // < 2^32: positions fit 32 bits
    const uint64_t g0 = gpos_base + lo;
    // slices start on whole tiles, so lo is a multiple of KV
    uint32_t done = 0;
    if (vec) {  // whole 16-byte vectors, two loads in flight per thread
      const uint4* kv = reinterpret_cast<const uint4*>(keys + lo);
      const uint32_t nv = len / KV;
      uint32_t v = threadIdx.x;
      int steps = 0;
      for (; v + BLOCK < nv; v += 2 * BLOCK) {
        if (++steps == FOLD_STEPS) {
          fold();
          steps = 0;
        }
        const uint4 a0 = __ldcs(kv + v), a1 = __ldcs(kv + v + BLOCK);
        const K* k0 = reinterpret_cast<const K*>(&a0);
        const K* k1 = reinterpret_cast<const K*>(&a1);
#pragma unroll
        for (int q = 0; q < KV; ++q) add(dfn(to_ordered<K, XF>(k0[q]), [&] { return g0 + (uint64_t)(v * KV + q); }));
#pragma unroll
        for (int q = 0; q < KV; ++q)
          add(dfn(to_ordered<K, XF>(k1[q]), [&] { return g0 + (uint64_t)((v + BLOCK) * KV + q); }));
      }
      for (; v < nv; v += BLOCK) {
        const uint4 a0 = __ldcs(kv + v);
        const K* k0 = reinterpret_cast<const K*>(&a0);
#pragma unroll
        for (int q = 0; q < KV; ++q) add(dfn(to_ordered<K, XF>(k0[q]), [&] { return g0 + (uint64_t)(v * KV + q); }));
      }
      done = nv * KV;
    }
    for (uint32_t i = done + threadIdx.x; i < len; i += BLOCK)
      add(dfn(to_ordered<K, XF>(keys[lo + i]), [&] { return g0 + i; }));
    if constexpr (PACK == 2) {
      const uint32_t v = __reduce_add_sync(0xffffffffu, c1);
      if (lane == 0 && v) atomicAdd(&h[1], v);
      c1 = 0;
    } else if constexpr (PACK != 0) {
      fold();
#pragma unroll
      for (int q = 0; q < PACK; ++q) {
        uint32_t v = (uint32_t)(((q & 1 ? w_odd : w_even) >> (16 * (q >> 1))) & 0xffffu);
        v = __reduce_add_sync(0xffffffffu, v);
        if (lane == 0 && v) atomicAdd(&h[q], v);
      }
      w_even = w_odd = 0;
    }
    __syncthreads();
    if constexpr (PACK == 2) {
      if (threadIdx.x == 0) h[0] = len - h[1];
      __syncthreads();
    }
    uint32_t* out = counts + (size_t)c * RADIX;
    for (int q = threadIdx.x; q < RADIX; q += BLOCK) {
      const uint32_t v = h[q];
      out[q] = v;
      tot[q] += v;
      h[q] = 0;
    }
    __syncthreads();
  }
  for (int q = threadIdx.x; q < RADIX; q += BLOCK)
    if (tot[q]) atomicAdd(&ctl->hist[0][q], (unsigned long long)tot[q]);
}

// --------------------------------------------------------------------------
// Plan: which passes run (a pass whose digit is the same for all n keys is the
// identity permutation and is skipped), then thread 0 routes the executed
// passes through the key and payload buffers so that the result lands where
// the caller wants it.  Replaces sort_msd_prep (shaders/sort.metal:153-181).
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(RADIX) k_plan(SortCtl* __restrict__ ctl, PlanArgs a) {
  chain_wait();
  const int d = threadIdx.x;
  __shared__ int s_exec[MAX_PASSES];
  const unsigned long long c0 = ctl->hist[0][d];
  if (a.counts_out != nullptr && d < a.ncounts) a.counts_out[d] = c0;
  if (a.trivial_from_bits) {
    const unsigned long long varying = ctl->kor & ctl->kandn;
    if (d < a.passes) s_exec[d] = ((varying >> (RADIX_BITS * d)) & (RADIX - 1)) != 0;
    if (a.h16 && d < 2) s_exec[d] = 0;  // the low 16 bits belong to the histogram fill
  } else {
    const int trivial = __syncthreads_or(c0 == a.n);
    if (d == 0) s_exec[0] = a.force_exec || !trivial;
  }
  __syncthreads();
  if (d != 0) return;

  int m = 0;
  for (int p = 0; p < a.passes; ++p) m += s_exec[p];
  const bool inplace_k = a.kin == a.kfinal;
  const bool inplace_v = a.has_vals && a.vin != nullptr && a.vin == a.vfinal;
  // Executed passes alternate between two slots, FINAL and OTHER.  Pass 1 may
  // not write the buffer it reads, so in-place sorts start in OTHER; with an
  // odd number of executed passes they then end in OTHER and copy back.
  const bool first_other = inplace_k || inplace_v;
  bool slot_final = first_other ? false : ((m & 1) != 0);  // slot of pass 1
  const void* kprev = a.kin;
  const uint32_t* vprev = a.vin;
  int i = 0;
  for (int p = 0; p < a.passes; ++p) {
    PassDesc pd{};
    if (s_exec[p]) {
      ++i;
      void* kdst = slot_final ? a.kfinal : a.kother;
      uint32_t* vdst = slot_final ? a.vfinal : a.vother;
      uint32_t f = PD_EXEC;
      if (i == 1) f |= PD_XF_IN | PD_FIRST;
      if (i == 1 && (p == 0 || a.h16) && !a.has_vals && a.unstable_first) f |= PD_UNSTABLE;
      if (i == 1 && a.has_vals && a.vin == nullptr) f |= PD_SYNTH_IDX;
      if (i == 1 && a.test_withhold) f |= PD_TEST_WITHHOLD;
      if (i == m && !a.h16) f |= PD_XF_OUT;  // h16: the histogram fill writes the caller's form
      if (a.write_keys || i < m || a.h16) f |= PD_WRITE_KEYS;
      // Keys only, not the first pass: the input is sorted by the digits
      // below (LSD: all lower bits; h16: digit 2 -- the fill orders the rest),
      // and equal keys are identical bits, so a warp round whose keys agree
      // on those bits may rank its equal digits in any order.
      // (64-bit keys: passes 1-3, whose lower bits fit the 32-bit mask).
      // Only where a value of those bits spans 64 keys or more on average;
      // with shorter runs few rounds agree and the check only costs
      // (2^26 u64 keys, pass 3: 0.395 ms with it, 0.375 without).
      const uint64_t run = a.n >> (a.h16 ? RADIX_BITS * 2 : RADIX_BITS * p);
      if (i > 1 && !a.has_vals && (a.key_bytes == 4 || p < 4) && run >= 64) {
        f |= PD_SORTED_BELOW;
        pd.below = a.h16 ? 0x00ff0000u : (uint32_t)((1ull << (RADIX_BITS * p)) - 1ull);
      }
      pd.kin = kprev;
      pd.kout = kdst;
      pd.vin = vprev;
      pd.vout = vdst;
      pd.flags = f;
      kprev = kdst;
      vprev = vdst;
      slot_final = !slot_final;
    }
    ctl->pass[p] = pd;
  }
  FinalDesc fin{};
  fin.executed_passes = (uint32_t)m;
  if (a.h16) {
    // The histogram fill reads the grouped keys wherever the passes left
    // them (in place is safe: each group is read whole before it is
    // written) and writes kfinal.  Keys that are all equal need neither.
    // The pool for the large groups' histograms takes the n-key buffer the
    // fill neither reads nor writes; a pass that sorted in place into OTHER
    // is filled there in place and copied back.
    const bool all_equal = (ctl->kor & ctl->kandn & 0xffffffffull) == 0;
    ctl->hf_src = kprev;
    ctl->hf_flags = all_equal ? 0u : (HF_ON | (m == 0 ? HF_XF_IN : 0u));
    if (kprev == a.kother) {  // in place, one pass
      ctl->hf_dst = a.kother;
      ctl->hf_pool = a.kfinal;
      if (!all_equal) {
        fin.ops |= FIN_COPY_KEYS;
        fin.ksrc = a.kother;
        fin.kdst = a.kfinal;
      }
    } else {
      ctl->hf_dst = a.kfinal;
      ctl->hf_pool = a.kother;
    }
    if (all_equal && a.kin != a.kfinal) {
      fin.ops |= FIN_COPY_KEYS;
      fin.ksrc = a.kin;
      fin.kdst = a.kfinal;
    }
    ctl->fin = fin;
    return;
  }
  if (m > 0) {
    if (kprev != a.kfinal) {  // ended in OTHER
      if (a.write_keys) {
        fin.ops |= FIN_COPY_KEYS;
        fin.ksrc = kprev;
        fin.kdst = a.kfinal;
      }
      if (a.has_vals) {
        fin.ops |= FIN_COPY_VALS;
        fin.vsrc = vprev;
        fin.vdst = a.vfinal;
      }
    }
  } else {
    if (a.write_keys && a.kin != a.kfinal) {
      fin.ops |= FIN_COPY_KEYS;
      fin.ksrc = a.kin;
      fin.kdst = a.kfinal;
    }
    if (a.has_vals) {
      if (a.vin == nullptr) {
        fin.ops |= FIN_IOTA_VALS;
        fin.vdst = a.vfinal;
      } else if (a.vin != a.vfinal) {
        fin.ops |= FIN_COPY_VALS;
        fin.vsrc = a.vin;
        fin.vdst = a.vfinal;
      }
    }
  }
  ctl->fin = fin;
}

// --------------------------------------------------------------------------
// Count: per-slice histogram of this pass's digit over the pass input, and its
// global totals (ctl->hist[pass]).  Pass 0 was counted by k_first_count.  The
// input holds ordered keys except for the first executed pass, which reads
// the caller's keys and transforms them as it counts.
// --------------------------------------------------------------------------
template <typename K, int XF, int BLOCK>
__global__ void __launch_bounds__(BLOCK)
    k_count(SortCtl* __restrict__ ctl, const int pass, const uint64_t n, const Slices sl,
            uint32_t* __restrict__ counts /* [count][RADIX] */) {
  chain_wait();
  const uint32_t flags = ctl->pass[pass].flags;
  if (!(flags & PD_EXEC) || pass == 0) return;
  const K* keys = static_cast<const K*>(ctl->pass[pass].kin);
  const bool xf = XF != XF_NONE && (flags & PD_XF_IN);
  // one histogram per warp: no atomic contention between warps
  constexpr int WARPS = BLOCK / 32;
  __shared__ uint32_t hw[WARPS][RADIX];
  __shared__ uint32_t tot[RADIX];
  uint32_t* h = hw[threadIdx.x >> 5];
  for (int i = threadIdx.x; i < WARPS * RADIX; i += BLOCK) (&hw[0][0])[i] = 0;
  for (int i = threadIdx.x; i < RADIX; i += BLOCK) tot[i] = 0;
  __syncthreads();
  const int shift = pass * RADIX_BITS;
  // one shared atomic per key (skewed digits only slow the warp that meets them)
  const RadixDigit dg{shift};
  auto f = [&](K x, bool valid) {
    if (valid) atomicAdd(&h[dg(xf ? to_ordered<K, XF>(x) : x, 0)], 1u);
  };
  const bool vec = (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
  for (uint32_t c = blockIdx.x; c < sl.count; c += gridDim.x) {
    const uint64_t lo = (uint64_t)c * sl.keys_per_slice;
    const uint64_t hi = lo + sl.keys_per_slice < n ? lo + sl.keys_per_slice : n;
    if (vec)
      for_each_key<K, BLOCK, true>(keys, lo, hi, f);
    else
      for_each_key<K, BLOCK, false>(keys, lo, hi, f);
    __syncthreads();
    for (int b = threadIdx.x; b < RADIX; b += BLOCK) {
      uint32_t v = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        v += hw[w][b];
        hw[w][b] = 0;
      }
      counts[(size_t)c * RADIX + b] = v;
      tot[b] += v;
    }
    __syncthreads();
  }
  for (int b = threadIdx.x; b < RADIX; b += BLOCK)
    if (tot[b]) atomicAdd(&ctl->hist[pass][b], (unsigned long long)tot[b]);
}

// --------------------------------------------------------------------------
// Slice scan: offsets[c][d] = (keys of digit < d in the whole pass) + (keys
// of digit d in slices c' < c), mod 2^32 (positions are < 2^32).  With
// `relative` the first term is dropped (positions within the digit's bucket,
// for the sample-sort dispatch).
// SCAN_GROUPS CTAs of 32 digits each; in a CTA, warp w owns a run of slices
// and lane l digit 32*blockIdx.x + l, so every load is one 128-byte row.
// --------------------------------------------------------------------------
constexpr int SCAN_GROUPS = RADIX / 32;
constexpr int SCAN_WARPS = 32;
__global__ void __launch_bounds__(SCAN_WARPS * 32)
    k_slice_scan(SortCtl* __restrict__ ctl, const int pass, const Slices sl,
                 const uint32_t* __restrict__ counts, uint32_t* __restrict__ offsets, const int relative) {
  chain_wait();
  const uint32_t flags = ctl->pass[pass].flags;
  if (!(flags & PD_EXEC)) return;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ uint32_t s_part[SCAN_WARPS][32];
  __shared__ uint32_t s_wtot[RADIX / 32];
  __shared__ uint32_t s_base[RADIX];
  // bucket starts: exclusive scan of the pass's global digit counts
  uint32_t t = 0, x = 0;
  if (tid < RADIX) {
    t = (uint32_t)ctl->hist[pass][tid];
    x = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if ((int)lane >= o) x += y;
    }
    if (lane == 31) s_wtot[warp] = x;
  }
  __syncthreads();
  if (tid < RADIX) {
    uint32_t pre = x - t;
    for (uint32_t w = 0; w < warp; ++w) pre += s_wtot[w];
    s_base[tid] = relative ? 0u : pre;  // relative: offsets within each digit's bucket
  }
  // Round-level atomic ranks (PD_SORTED_BELOW) only while no digit holds more
  // than an eighth of the keys: where many lanes of a round share a digit,
  // same-address atomics serialize (the skewed 2^32 input, 70% of keys on one
  // top digit: 60.0 ms a sort with them on digit 3, 54.9 without).  The
  // scatter of this pass reads the descriptor after this kernel.
  if (blockIdx.x == 0 && (flags & PD_SORTED_BELOW)) {
    __shared__ unsigned long long s_tot;
    if (tid == 0) s_tot = 0;
    __syncthreads();
    const unsigned long long c = tid < RADIX ? ctl->hist[pass][tid] : 0ull;
    if (c) atomicAdd(&s_tot, c);
    __syncthreads();
    if (__syncthreads_or(c > (s_tot >> 3)) && tid == 0) ctl->pass[pass].flags = flags & ~(uint32_t)PD_SORTED_BELOW;
  }
  // warp w sums its slices for the CTA's 32 digits
  const uint32_t d = blockIdx.x * 32 + lane;
  const uint32_t per = (sl.count + SCAN_WARPS - 1) / SCAN_WARPS;
  const uint32_t c0 = warp * per < sl.count ? warp * per : sl.count;
  const uint32_t c1 = c0 + per < sl.count ? c0 + per : sl.count;
  uint32_t sum = 0;
  for (uint32_t c = c0; c < c1; ++c) sum += counts[(size_t)c * RADIX + d];
  s_part[warp][lane] = sum;
  __syncthreads();
  uint32_t run = s_base[d];
  for (uint32_t w = 0; w < warp; ++w) run += s_part[w][lane];
  for (uint32_t c = c0; c < c1; ++c) {
    const uint32_t v = counts[(size_t)c * RADIX + d];
    offsets[(size_t)c * RADIX + d] = run;
    run += v;
  }
}

// --------------------------------------------------------------------------
// Scatter: CTA c sorts slice c's keys into their pass-output positions, one
// tile of BLOCK*IPT keys at a time, keeping a running output offset per digit.
//
// Tile layout: warp w owns the contiguous segment [w*32*IPT, (w+1)*32*IPT)
// and holds item k of lane l at k*32 + l, so ranking items in (k, lane) order
// IS input order -> the pass is stable, which argsort and pairs need (the
// reference's atomic MSD scatter was not: shaders/sort.metal:267-283).
//
//   A. keys -> registers from the bulk-copied shared-memory slot (plain loads
//      for the partial last tile and unaligned inputs); forward transform on
//      the first executed pass
//   B. warp multisplit rank: the lanes sharing a digit (eight ballots) read
//      the warp's running count for it, the group's highest lane advances
//      it; rank = count + lanes below in the group
//   C. per digit: warp bases, tile-local start, output offset = running
//      offset - start; running offset += tile count
//   D. stage: key (and payload) written to its slot in the digit-sorted tile
//   E. coalesced scatter: consecutive staged keys of one digit go to
//      consecutive output positions (+ inverse transform on the last pass)
// --------------------------------------------------------------------------

// Stable warp ranking.  Three ways to find the lanes that share this lane's
// digit were measured on B200 (2^30 u32 keys, 256x16 tiles, stable pass):
//   FS_RANK_BALLOT=3 (default): owner election through a per-warp byte per
//     digit, then five ballots over the owner's lane bits  3.96 ms/pass
//   FS_RANK_BALLOT=2: eight ballots over the digit's bits  4.75 ms/pass
//   FS_RANK_BALLOT=0: __match_any_sync                      ~2x slower again
// (The owner byte folded into the counter word, saving one shared load per
// key, measured 4.01 ms; the owner advancing the count with one shared atomic
// and the group reading it by shuffle, 4.03 ms: neither kept.)
// warp_peers serves 2 and 0; owner election is written out in scatter_tile.
// Invalid lanes of a partial tile match nobody but themselves.
template <bool FULL, int BITS = RADIX_BITS>
__device__ __forceinline__ uint32_t warp_peers(uint32_t d, bool valid) {
#if FS_RANK_BALLOT == 0
  if (BITS == RADIX_BITS) return __match_any_sync(0xffffffffu, valid ? d : 0xffffffffu);
#endif
  // lanes whose digit differs from mine in some bit, then complement
  uint32_t diff = FULL ? 0u : ~__ballot_sync(0xffffffffu, valid);
#pragma unroll
  for (int b = 0; b < BITS; ++b) {
    const uint32_t bit = (d >> b) & 1u;
    diff |= __ballot_sync(0xffffffffu, bit) ^ (0u - bit);
  }
  return valid ? ~diff : (1u << (threadIdx.x & 31));
}

__host__ __device__ constexpr int log2_of(int v) { return v <= 1 ? 0 : 1 + log2_of(v >> 1); }

// SLOTS: bulk-copy slots for the keys.  2: the next tile's copy lands in the
// other slot while this tile is processed.  1 (keys only): the next tile's
// copy is issued into the same slot as soon as this tile's keys are in
// registers -- half the shared memory, so more CTAs fit per SM.
template <typename K, bool VALS, int BLOCK, int IPT, bool STAGE_DIG, int R = RADIX, int SLOTS = 2>
struct ScatterLayout {
  static constexpr int WARPS = BLOCK / 32;
  static constexpr int TILE = BLOCK * IPT;
  static constexpr int SEG = 32 * IPT;
  static constexpr size_t KEYS = (size_t)TILE * sizeof(K);
  static constexpr size_t VALB = VALS ? (size_t)TILE * 4 : 0;
  static constexpr size_t SLOT = KEYS + VALB;  // one bulk-copy slot (keys | vals)
  // dynamic shared memory:
  //   [slot 0 | slot 1 | stage keys | stage vals | warp digit counters |
  //    warp digit owners | staged digits]
  static_assert(SLOTS == 2 || (SLOTS == 1 && !VALS), "one slot: keys-only passes");
  static constexpr size_t STAGE_OFF = SLOTS * SLOT;
  static constexpr size_t CNT_OFF = STAGE_OFF + KEYS + VALB;
  static constexpr size_t REP_OFF = CNT_OFF + (size_t)WARPS * R * 4;  // per-warp digit owners
  static constexpr size_t DIG_OFF = REP_OFF + (((size_t)WARPS * R + 15) & ~(size_t)15);
  static constexpr size_t BYTES = DIG_OFF + (STAGE_DIG ? (size_t)TILE : 0);
  static_assert(BLOCK >= R && BLOCK % 32 == 0, "one thread per digit needed");
  static_assert((R & (R - 1)) == 0 && R <= RADIX, "digit count: a power of two <= 256");
  static_assert(KEYS % 16 == 0, "bulk copies move multiples of 16 bytes");
};

// Per-key ranks of a tile: a register each, or (PACK) two 16-bit ranks per
// register (a rank is below 32 * IPT), which frees IPT/2 registers.
template <int IPT, bool PACK>
struct Ranks {
  uint32_t r[PACK ? (IPT + 1) / 2 : IPT];
  __device__ __forceinline__ void set(int k, uint32_t v) {
    if constexpr (PACK) {
      if (k & 1)
        r[k >> 1] |= v << 16;
      else
        r[k >> 1] = v;
    } else {
      r[k] = v;
    }
  }
  __device__ __forceinline__ uint32_t get(int k) const {
    if constexpr (PACK)
      return (k & 1) ? r[k >> 1] >> 16 : r[k >> 1] & 0xffffu;
    else
      return r[k];
  }
};

struct NoHook {
  __device__ __forceinline__ void operator()() const {}
};

// `on_loaded` runs on every thread once the tile's keys are in registers
// (single-slot scatter: it issues the next tile's copy into the slot).
template <typename K, bool VALS, int XF, int BLOCK, int IPT, bool FULL, bool FROM_SLOT, bool UNSTABLE,
          typename D, int SLOTS = 2, typename Hook = NoHook, bool PACK = false>
__device__ __forceinline__ void scatter_tile(const uint64_t tbase, const uint32_t tile_n, const uint64_t n,
                                             const uint32_t flags, const K* __restrict__ kin,
                                             K* __restrict__ kout, const uint32_t* __restrict__ vin,
                                             uint32_t* __restrict__ vout, const unsigned char* slot,
                                             unsigned char* dsm, uint32_t* s_run, uint32_t* s_off,
                                             uint32_t* s_wsum, SortCtl* __restrict__ ctl, const D& dfn,
                                             const uint64_t gpos_base, K* const* s_dst, const uint32_t* s_lim,
                                             uint32_t* const* s_vdst, const uint32_t below,
                                             const Hook& on_loaded = Hook{}) {
  constexpr int R = D::DIGITS;
  using Ly = ScatterLayout<K, VALS, BLOCK, IPT, D::STAGE, R, SLOTS>;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const uint64_t gbase = gpos_base + tbase;
  const uint32_t wofs = warp * Ly::SEG + lane;
  const K* slot_keys = reinterpret_cast<const K*>(slot);
  const uint32_t* slot_vals = reinterpret_cast<const uint32_t*>(slot + Ly::KEYS);
  K* skeys = reinterpret_cast<K*>(dsm + Ly::STAGE_OFF);
  uint32_t* svals = reinterpret_cast<uint32_t*>(dsm + Ly::STAGE_OFF + Ly::KEYS);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(dsm + Ly::CNT_OFF);
  uint8_t* sdig = dsm + Ly::DIG_OFF;
  uint32_t* wcnt = cnt + warp * R;
  uint8_t* wrep = dsm + Ly::REP_OFF + warp * R;

  // ---- A. keys -> registers ----------------------------------------------------
  K key[IPT];
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const uint32_t li = wofs + k * 32;
    if constexpr (FROM_SLOT)
      key[k] = slot_keys[li];
    else
      key[k] = (FULL || li < tile_n) ? kin[tbase + li] : K(0);
  }
  if constexpr (FROM_SLOT && SLOTS == 1) on_loaded();
  if constexpr (XF != XF_NONE) {
    if (flags & PD_XF_IN) {
#pragma unroll
      for (int k = 0; k < IPT; ++k) key[k] = to_ordered<K, XF>(key[k]);
    }
  }

  // Digits: a radix digit is one byte-permute and is recomputed where it is
  // needed; a splitter bucket (binary search) is computed once and kept
  // packed, four to a register.
  constexpr int DPK = D::STAGE ? (IPT + 3) / 4 : 1;
  uint32_t dpk[DPK];
  if constexpr (D::STAGE) {
#pragma unroll
    for (int q = 0; q < DPK; ++q) dpk[q] = 0;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const bool valid = FULL || (wofs + k * 32) < tile_n;
      const uint32_t d = valid ? dfn(key[k], [&] { return gbase + wofs + k * 32; }) : 0u;
      dpk[k >> 2] |= d << (8 * (k & 3));
    }
  }
  auto digit = [&](int k) -> uint32_t {
    if constexpr (D::STAGE)
      return (dpk[k >> 2] >> (8 * (k & 3))) & 0xffu;
    else
      return dfn(key[k], 0ull);  // the radix digit does not depend on the position
  };

  // ---- B. warp-local ranks -------------------------------------------------------
  // Per key: the lanes sharing its digit; all read the warp's running count
  // for that digit, the group's highest lane advances it.  After the loop
  // the counters hold the warp's per-digit totals.
  Ranks<IPT, PACK> rank;
  if constexpr (UNSTABLE) {
    // Keys-only first pass: no earlier order to keep, so any order among
    // equal digits is correct -- one shared atomic per key ranks it.
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const bool valid = FULL || (wofs + k * 32) < tile_n;
      const uint32_t d = digit(k);
      rank.set(k, valid ? atomicAdd(&wcnt[d], 1u) : 0u);
    }
  } else if constexpr (FS_RANK_BALLOT == 3 && R > 32) {
    // Owner election: every lane writes its lane number into its digit's
    // byte; after the warp syncs, all lanes of a digit read the same owner
    // (whichever write landed).  Lanes sharing a digit are then exactly the
    // lanes sharing an owner: five ballots over the owner's bits instead of
    // eight over the digit's.  The owner advances the running count.
    const bool sorted_below = !VALS && (flags & PD_SORTED_BELOW) != 0;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const bool valid = FULL || (wofs + k * 32) < tile_n;
      const uint32_t d = digit(k);
      if (sorted_below) {
        // the round's 32 consecutive keys agree on the bits below: any order
        // among equal digits is the stable one up to equal keys, so one
        // shared atomic per key ranks the round
        const uint32_t lb = (uint32_t)key[k] & below;
        const uint32_t mn = __reduce_min_sync(0xffffffffu, valid ? lb : 0xffffffffu);
        const uint32_t mx = __reduce_max_sync(0xffffffffu, valid ? lb : 0u);
        if (mn >= mx) {
          rank.set(k, valid ? atomicAdd(&wcnt[d], 1u) : 0u);
          __syncwarp();
          continue;
        }
      }
      if (valid) wrep[d] = (uint8_t)lane;
      __syncwarp();
      const uint32_t own = valid ? wrep[d] : lane;  // invalid lanes: groups of one
      uint32_t diff = 0;
#pragma unroll
      for (int b = 0; b < 5; ++b) {
        const uint32_t bit = (own >> b) & 1u;
        diff |= __ballot_sync(0xffffffffu, bit) ^ (0u - bit);
      }
      const uint32_t peers = ~diff;
      uint32_t old = 0;
      if (valid) old = wcnt[d];
      __syncwarp();
      if (valid && lane == own) wcnt[d] = old + __popc(peers);
      __syncwarp();
      rank.set(k, old + __popc(peers & lt_mask));
    }
  } else {
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const bool valid = FULL || (wofs + k * 32) < tile_n;
      const uint32_t d = digit(k);
      const uint32_t peers = warp_peers<FULL, (R > 32 ? RADIX_BITS : log2_of(R))>(d, valid);
      uint32_t old = 0;
      if (valid) old = wcnt[d];
      __syncwarp();
      if (valid && lane == 31u - __clz(peers)) wcnt[d] = old + __popc(peers);
      __syncwarp();
      rank.set(k, old + __popc(peers & lt_mask));
    }
  }
  __syncthreads();

  // ---- C. per-digit bases and output offsets ------------------------------------
  uint32_t tot = 0;
  if (tid < R) {
#pragma unroll
    for (int w = 0; w < Ly::WARPS; ++w) {
      const uint32_t c = cnt[w * R + tid];
      cnt[w * R + tid] = tot;
      tot += c;
    }
  }
  uint32_t x = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if ((int)lane >= o) x += y;
  }
  if (lane == 31 && tid < R) s_wsum[warp] = x;
  __syncthreads();
  if (tid < R) {
    uint32_t start = x - tot;
    for (uint32_t w = 0; w < warp; ++w) start += s_wsum[w];
#pragma unroll
    for (int w = 0; w < Ly::WARPS; ++w) cnt[w * R + tid] += start;
    s_off[tid] = s_run[tid] - start;
    s_run[tid] += tot;
  }
  __syncthreads();

  // ---- D. stage in digit order -----------------------------------------------------
  // cnt[w][d] now holds tile-local start of digit d + warp w's prefix
  const bool synth = VALS && (flags & PD_SYNTH_IDX);
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const uint32_t li = wofs + k * 32;
    if (FULL || li < tile_n) {
      const uint32_t d = digit(k);
      const uint32_t pos = wcnt[d] + rank.get(k);
      skeys[pos] = key[k];
      if constexpr (VALS) {
        uint32_t v;
        if (synth)  // the key's (global) position: gpos_base is 0 except in a sample-sort dispatch
          v = (uint32_t)(gbase + li);
        else if constexpr (FROM_SLOT)
          v = slot_vals[li];
        else
          v = vin[tbase + li];
        svals[pos] = v;
      }
      if constexpr (D::STAGE) sdig[pos] = (uint8_t)d;
    }
  }
  __syncthreads();

  // ---- E. coalesced scatter ---------------------------------------------------------
  // Positions are checked against n: a wrong offset records DEV_ERR_BOUNDS
  // and drops the write instead of touching foreign memory.
  const bool wkeys = (flags & PD_WRITE_KEYS) != 0;
  const bool xout = XF != XF_NONE && (flags & PD_XF_OUT);
  const uint32_t last = (uint32_t)(n - 1);  // n <= 2^32: positions fit 32 bits
  bool oob = false;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t i = j * BLOCK + tid;
    if (FULL || i < tile_n) {
      const K kk = skeys[i];
      uint32_t d;
      if constexpr (D::STAGE)
        d = sdig[i];
      else
        d = dfn(kk, 0);
      const uint32_t pos = s_off[d] + i;
      if constexpr (D::DISPATCH) {
        // position within bucket d; its region holds exactly s_lim[d] keys
        if (pos < s_lim[d]) {
          s_dst[d][pos] = xout ? from_ordered<K, XF>(kk) : kk;
          if constexpr (VALS) s_vdst[d][pos] = svals[i];
        } else {
          oob = true;
        }
      } else if (pos <= last) {
        if (wkeys) kout[pos] = xout ? from_ordered<K, XF>(kk) : kk;
        if constexpr (VALS) vout[pos] = svals[i];
      } else {
        oob = true;
      }
    }
  }
  if (oob) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
  for (int i = tid; i < Ly::WARPS * R; i += BLOCK) cnt[i] = 0;
  __syncthreads();  // staging reads done, counters zeroed: next tile may start
}

// Which passes a scatter instantiation takes.  The rank method is compiled
// in: SCATTER_UNSTABLE ranks with shared atomics and only runs a pass the
// plan marked PD_UNSTABLE (pass 0 of a keys-only sort when it executes);
// the others rank stably with ballots.
enum ScatterMode : int { SCATTER_ANY = 0, SCATTER_UNSTABLE = 1 };

// CTAs loop over slices (c = blockIdx.x, +gridDim.x, ...); tiles of a slice
// are processed in order with per-digit running offsets.  The next tile's
// keys (and payload) are bulk-copied (cp.async.bulk global->shared, no
// multicast) into the other of two slots while the current one is processed.
// Every mbarrier wait is bounded; no CTA exits with a copy still in flight.
template <typename K, bool VALS, int XF, int BLOCK, int IPT, int MINB, int MODE, typename D, int SLOTS = 2,
          bool PACK = false>
__global__ void __launch_bounds__(BLOCK, MINB)
    k_scatter(SortCtl* __restrict__ ctl, const int pass, const uint64_t n, const Slices sl,
              const uint32_t* __restrict__ offsets, const uint64_t timeout_ns, const D dfn_in,
              const uint64_t gpos_base) {
  constexpr int R = D::DIGITS;
  using Ly = ScatterLayout<K, VALS, BLOCK, IPT, D::STAGE, R, SLOTS>;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ uint32_t s_run[R];
  __shared__ uint32_t s_off[R];
  __shared__ uint32_t s_wsum[Ly::WARPS];
  __shared__ __align__(8) uint64_t s_bar[2];
  __shared__ int s_abort;
  __shared__ K* s_dst[D::DISPATCH ? R : 1];
  __shared__ uint32_t s_lim[D::DISPATCH ? R : 1];
  __shared__ uint32_t* s_vdst[D::DISPATCH && VALS ? R : 1];
  __shared__ K s_spk[D::STAGE ? (R < 8 ? 8 : R) : 1];  // the splitter search pads to 8
  __shared__ uint64_t s_spg[D::STAGE ? (R < 8 ? 8 : R) : 1];

  chain_wait();
  const PassDesc pd = ctl->pass[pass];
  if (!(pd.flags & PD_EXEC)) return;
  if (MODE == SCATTER_UNSTABLE && !(pd.flags & PD_UNSTABLE)) return;
  const K* kin = static_cast<const K*>(pd.kin);
  K* kout = static_cast<K*>(pd.kout);
  const bool copy_vals = VALS && !(pd.flags & PD_SYNTH_IDX);
  const bool bulk_ok = (reinterpret_cast<uintptr_t>(kin) & 15) == 0 &&
                       (!copy_vals || (reinterpret_cast<uintptr_t>(pd.vin) & 15) == 0);
  const uint32_t tid = threadIdx.x;

  // thread 0: start the copy of the tile at key `t0` of a slice ending at
  // `hi` into slot s (full tiles only)
  uint32_t armed = 0;  // thread 0: bit s = copy into slot s in flight
  // failure-path test: CTA 0 leaves its first copy un-issued (barrier never
  // armed, nothing in flight), so its bounded wait runs out
  bool withhold = (pd.flags & PD_TEST_WITHHOLD) != 0 && blockIdx.x == 0;
  auto issue = [&](uint64_t t0, uint64_t hi, int s) {
    if (bulk_ok && t0 + Ly::TILE <= hi) {
      if (withhold) {
        withhold = false;
        return;
      }
      unsigned char* dst = dsm + (size_t)s * Ly::SLOT;
      fence_proxy_async_smem();  // earlier generic reads of the slot precede the async write
      mbar_arrive_expect_tx(&s_bar[s], (uint32_t)(Ly::KEYS + (copy_vals ? Ly::VALB : 0)));
      bulk_g2s(dst, kin + t0, (uint32_t)Ly::KEYS, &s_bar[s]);
      if (copy_vals) bulk_g2s(dst + Ly::KEYS, pd.vin + t0, (uint32_t)Ly::VALB, &s_bar[s]);
      armed |= 1u << s;
    }
  };

  uint32_t* cnt = reinterpret_cast<uint32_t*>(dsm + Ly::CNT_OFF);
  for (int i = tid; i < Ly::WARPS * R; i += BLOCK) cnt[i] = 0;
  D dfn = dfn_in;
  if constexpr (D::STAGE) dfn.stage_in(s_spk, s_spg);  // visible after the slice loop's first barrier
  if constexpr (D::DISPATCH) {
    for (int b = tid; b < R; b += BLOCK) {
      const bool used = b <= dfn.nsplit;
      s_dst[b] = used ? dfn.dst[b] : nullptr;
      s_lim[b] = used ? (uint32_t)ctl->hist[0][b] : 0u;
      if constexpr (VALS) s_vdst[b] = used ? dfn.vdst[b] : nullptr;
    }
  }
  if (tid == 0) {
    mbar_init(&s_bar[0], 1);
    mbar_init(&s_bar[1], 1);
    fence_mbar_init();
    s_abort = 0;
  }

  uint32_t parity = 0;  // bit s: phase of slot s's barrier to wait for next
  int s = 0;
  bool aborted = false;
  for (uint32_t c = blockIdx.x; c < sl.count && !aborted; c += gridDim.x) {
    const uint64_t lo = (uint64_t)c * sl.keys_per_slice;
    const uint64_t hi = lo + sl.keys_per_slice < n ? lo + sl.keys_per_slice : n;
    __syncthreads();  // the previous slice's last tile is done with s_run
    if (tid < R) s_run[tid] = offsets[(size_t)c * RADIX + tid];  // row stride stays 256
    if (tid == 0) issue(lo, hi, s);
    __syncthreads();
    for (uint64_t t0 = lo; t0 < hi; t0 += Ly::TILE, s ^= (SLOTS == 2 ? 1 : 0)) {
      const uint32_t tile_n = hi - t0 < (uint64_t)Ly::TILE ? (uint32_t)(hi - t0) : (uint32_t)Ly::TILE;
      const bool full = tile_n == (uint32_t)Ly::TILE;
      const bool from_slot = full && bulk_ok;
      if (from_slot) {
        if (!mbar_wait_bounded(&s_bar[s], (parity >> s) & 1u, timeout_ns, &ctl->err)) s_abort = 1;
        parity ^= 1u << s;
        if (tid == 0) armed &= ~(1u << s);
      }
      if (tid == 0) {
        // two slots: the other one was consumed by the previous tile; one
        // slot: the copy is issued once this tile's keys are in registers
        if (SLOTS == 2) issue(t0 + Ly::TILE, hi, s ^ 1);
        if (ld_relaxed_s32(&ctl->err) != 0) s_abort = 1;
      }
      __syncthreads();  // one abort decision for the CTA
      if (s_abort) {
        aborted = true;
        break;
      }
      const unsigned char* slot = dsm + (size_t)s * Ly::SLOT;
      auto refill = [&]() {
        __syncthreads();  // every thread has read its keys from the slot
        if (tid == 0) issue(t0 + Ly::TILE, hi, 0);
      };
      if (from_slot)
        scatter_tile<K, VALS, XF, BLOCK, IPT, true, true, MODE == SCATTER_UNSTABLE, D, SLOTS, decltype(refill), PACK>(
            t0, tile_n, n, pd.flags, kin, kout, pd.vin, pd.vout, slot, dsm, s_run, s_off, s_wsum, ctl, dfn, gpos_base,
            s_dst, s_lim, s_vdst, pd.below, refill);
      else if (full)
        scatter_tile<K, VALS, XF, BLOCK, IPT, true, false, MODE == SCATTER_UNSTABLE, D, SLOTS, decltype(refill), PACK>(
            t0, tile_n, n, pd.flags, kin, kout, pd.vin, pd.vout, slot, dsm, s_run, s_off, s_wsum, ctl, dfn, gpos_base,
            s_dst, s_lim, s_vdst, pd.below, refill);
      else
        scatter_tile<K, VALS, XF, BLOCK, IPT, false, false, MODE == SCATTER_UNSTABLE, D, SLOTS, decltype(refill), PACK>(
            t0, tile_n, n, pd.flags, kin, kout, pd.vin, pd.vout, slot, dsm, s_run, s_off, s_wsum, ctl, dfn, gpos_base,
            s_dst, s_lim, s_vdst, pd.below, refill);
    }
  }
  // never leave a bulk copy into this CTA's shared memory in flight
  if (tid == 0) {
    for (int q = 0; q < 2; ++q)
      if (armed & (1u << q)) mbar_wait_bounded(&s_bar[q], (parity >> q) & 1u, timeout_ns, &ctl->err);
  }
  // dispatch: stores to peer GPUs are ordered before whatever this GPU does
  // next (the stream-ordered barrier that tells the peers their inbox is full)
  if constexpr (D::DISPATCH) __threadfence_system();
}

// --------------------------------------------------------------------------
// Small sorts (n <= SMALL_N_MAX): one CTA sorts everything in shared memory
// with a bitonic network, one launch instead of a radix pass chain, for the
// short arrays of e.g. gpu-search's argsort_u64
// (gpu-search/src/search/content.rs:849-884).  With a payload (argsort,
// pairs) the network orders (ordered key, input position), so equal keys keep
// their input order, as the radix passes do; keys alone need no position
// (equal keys are equal bits).  Inputs are staged first, so in-place calls
// are safe.
//
// The block has max(32, npad/4) threads (npad = n rounded up to a power of
// two, at most 1024 threads); every thread does PP = npad / (2 * threads)
// compare-exchanges per stage.  Warp w owns elements [w*E, (w+1)*E), E =
// 64 * PP: a stage with distance j <= E/2 only touches the warp's own
// elements, so it follows the previous warp-local stage after __syncwarp;
// only the stages with larger j (15 of the 78 at npad = 4096) and their
// neighbours need a block barrier.
// --------------------------------------------------------------------------
// Measured on B200 (one sort per launch, device time): the single CTA beats
// the radix chain up to 8192 keys without a payload (u32: 55 vs 63 us at
// 8192) and up to 4096 with one (argsort u32 at 4096: 42 vs 55 us; at 8192:
// 86 vs 56 us).
constexpr uint32_t SMALL_N_MAX = 8192;
constexpr uint32_t SMALL_N_PAYLOAD_MAX = 4096;
constexpr int SMALL_BLOCK_MAX = 1024;

template <typename K, bool VALS>
__device__ __forceinline__ void small_cx(K* sk, uint32_t* si, uint32_t i, uint32_t l, bool up) {
  const K a = sk[i], b = sk[l];
  bool swap;
  uint32_t ia = 0, ib = 0;
  if constexpr (VALS) {
    ia = si[i];
    ib = si[l];
    swap = (a > b || (a == b && ia > ib)) == up;
  } else {
    swap = (a > b) == up;
  }
  if (swap) {
    sk[i] = b;
    sk[l] = a;
    if constexpr (VALS) {
      si[i] = ib;
      si[l] = ia;
    }
  }
}

template <typename K, int XF, bool VALS>
__global__ void __launch_bounds__(SMALL_BLOCK_MAX)
    k_small_sort(const K* __restrict__ kin, K* __restrict__ kout, const uint32_t* __restrict__ vin,
                 uint32_t* __restrict__ vout, const uint32_t n, const uint32_t npad, const int write_keys) {
  extern __shared__ __align__(16) unsigned char sm[];
  K* sk = reinterpret_cast<K*>(sm);
  uint32_t* si = reinterpret_cast<uint32_t*>(sm + (size_t)npad * sizeof(K));  // input positions (VALS)
  uint32_t* sv = si + npad;                                                    // payload (VALS)
  const uint32_t B = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t pp = npad / (2 * B) > 0 ? npad / (2 * B) : 1;  // pairs per thread
  const uint32_t half = npad / 2;
  const uint32_t local_j = 32 * pp;  // j <= local_j: the stage stays inside each warp's elements
  for (uint32_t i = tid; i < npad; i += B) {
    if (i < n) {
      sk[i] = to_ordered<K, XF>(kin[i]);
      if constexpr (VALS) {
        si[i] = i;
        sv[i] = vin ? vin[i] : i;
      }
    } else {  // padding sorts after every real key: largest key (and position)
      sk[i] = ~K(0);
      if constexpr (VALS) si[i] = 0xffffffffu;
    }
  }
  uint32_t prev_j = npad;  // the loads above are block-strided: start with a barrier
  for (uint32_t k = 2; k <= npad; k <<= 1) {
    for (uint32_t j = k >> 1; j > 0; j >>= 1) {
      if (j > local_j || prev_j > local_j)
        __syncthreads();
      else
        __syncwarp();
      const uint32_t lj = 31 - __clz(j);
      for (uint32_t r = 0; r < pp; ++r) {
        const uint32_t q = warp * 32 * pp + r * 32 + lane;  // this warp's pairs
        if (q < half) {
          const uint32_t i = ((q >> lj) << (lj + 1)) | (q & (j - 1));  // q with a 0 bit inserted at lj
          small_cx<K, VALS>(sk, si, i, i | j, (i & k) == 0);
        }
      }
      prev_j = j;
    }
  }
  __syncthreads();
  for (uint32_t i = tid; i < n; i += B) {
    if (write_keys) kout[i] = from_ordered<K, XF>(sk[i]);
    if constexpr (VALS) vout[i] = sv[si[i]];
  }
}

// --------------------------------------------------------------------------
// Gather: dst[i] = src[idx[i]] -- applying a permutation (argsort result) to a
// payload.  Replaces sort_gather_values (shaders/sort.metal:792-800) and
// forge-runtime's GpuGather (forge-runtime/src/gather.rs:82-134).  Four
// indices per thread from one 16-byte load when aligned; an index outside the
// source is reported (DEV_ERR_BOUNDS to the mapped host word) and skipped.
// --------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256)
    k_gather(const T* __restrict__ src, const uint64_t src_n, const uint32_t* __restrict__ idx, T* __restrict__ dst,
             const uint64_t n, int* __restrict__ host_err) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  bool oob = false;
  if ((reinterpret_cast<uintptr_t>(idx) & 15) == 0) {
    const uint64_t n4 = n / 4;
    const uint4* iv = reinterpret_cast<const uint4*>(idx);
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4; q += stride) {
      const uint4 j = __ldcs(iv + q);
      const uint32_t jj[4] = {j.x, j.y, j.z, j.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (jj[r] < src_n)
          dst[4 * q + r] = src[jj[r]];
        else
          oob = true;
      }
    }
    for (uint64_t i = 4 * n4 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const uint32_t j = idx[i];
      if (j < src_n)
        dst[i] = src[j];
      else
        oob = true;
    }
  } else {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const uint32_t j = idx[i];
      if (j < src_n)
        dst[i] = src[j];
      else
        oob = true;
    }
  }
  if (oob) *(volatile int*)host_err = DEV_ERR_BOUNDS;
}

// --------------------------------------------------------------------------
// Finalize: copy-back for in-place sorts that ended in scratch, iota for an
// argsort whose keys were all equal; then hand any device error to the host
// (mapped pinned word; set-only, the host clears it) and re-arm ctl->err.
// --------------------------------------------------------------------------
template <typename K>
__global__ void __launch_bounds__(256)
    k_finalize(SortCtl* __restrict__ ctl, const uint64_t n, int* __restrict__ host_err) {
  chain_wait();
  const FinalDesc f = ctl->fin;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f.ops & FIN_COPY_KEYS) {
    const K* src = static_cast<const K*>(f.ksrc);
    K* dst = static_cast<K*>(f.kdst);
    for (uint64_t i = i0; i < n; i += stride) dst[i] = src[i];
  }
  if (f.ops & FIN_COPY_VALS)
    for (uint64_t i = i0; i < n; i += stride) f.vdst[i] = f.vsrc[i];
  if (f.ops & FIN_IOTA_VALS)
    for (uint64_t i = i0; i < n; i += stride) f.vdst[i] = (uint32_t)i;
  if (i0 == 0) {
    const int e = ld_relaxed_s32(&ctl->err);
    if (e != 0) {
      *(volatile int*)host_err = e;
      ctl->err = 0;
    }
  }
}

}  // namespace fs
