// fs_histfill.cuh -- the histogram fill that finishes a keys-only sort of
// 32-bit keys once the keys are grouped by their top 16 bits.
//
// In the ordered space (total order for floats, flipped sign for signed
// integers) keys that share their top 16 bits differ only in the low 16, and
// keys that share all 32 bits are the same bit pattern.  So a group is sorted
// by counting how many of its keys take each of the 65536 low values and then
// writing each value that many times, in value order: no ranking, no staging,
// one read and one sequential write per key.  The radix passes of the top two
// digits (the first may rank unstably, the second ranks stably) do the
// grouping, so a keys-only sort of 32-bit keys costs 2 scatter passes and
// this fill instead of 4 scatter passes.
//
//   k_hf_bounds   group g = [lower_bound(g << 16), lower_bound((g+1) << 16)),
//                 found by binary search over the grouped keys
//   k_hf_plan     one CTA: lists the groups larger than HF_LOCAL_MAX keys
//   k_hf_local    CTA c takes groups c, c + grid, ...: 65536 16-bit counters
//                 in shared memory (one extra bit per value records a count
//                 past 2^16), then the warps walk the counters in value order
//                 and write every key of the group once
//   k_hf_big_*    the large groups, spread over CTAs: each chunk's counts are
//                 added into a global histogram per group (held in a buffer of
//                 n keys that is idle during the fill), one exclusive scan per
//                 group, then each CTA writes one window of a group's output
//
// Replaces, for keys-only 32-bit sorts, the inner LSD passes over the low
// bytes (sort_inner_fused, shaders/sort.metal:378-769).
#pragma once

#include "fs_kernels.cuh"

namespace fs {

constexpr uint32_t HF_GROUPS = 1u << 16;       // groups: the top 16 bits
constexpr uint32_t HF_BINS = 1u << 16;         // bins: the low 16 bits
constexpr uint32_t HF_WORDS = HF_BINS / 2;     // two 16-bit counters per word
constexpr uint32_t HF_OVF_WORDS = HF_BINS / 32;  // one overflow bit per bin
constexpr int HF_BLOCK = 1024;
constexpr int HF_WARPS = HF_BLOCK / 32;
constexpr size_t HF_LOCAL_SMEM = (size_t)(HF_WORDS + HF_OVF_WORDS) * 4;  // 136 KiB
constexpr size_t HF_BIG_SMEM = (size_t)HF_WORDS * 4;                     // 128 KiB
// A group of up to HF_LOCAL_MAX keys is counted by one CTA.  A count past
// 0xffff wraps its 16-bit field; the thread that wraps it records the bit and
// takes back the carry into the neighbouring field.  With at most 126975 keys
// at most one of the two values sharing a word can reach 2^16, and the
// other stays below 61440, so the carry, present for a moment, never makes
// the neighbour look wrapped.
constexpr uint64_t HF_LOCAL_MAX = 126975;
// Large groups are counted and written in chunks of this many keys: a chunk's
// 16-bit counters never wrap.
constexpr uint64_t HF_CHUNK = 61440;
// A run of one value longer than this is written by the whole warp.
constexpr uint32_t HF_RUN = 8;
// Keys loaded per thread before they are counted.
#ifndef FS_HF_UNROLL
#define FS_HF_UNROLL 16
#endif
constexpr int HF_UNROLL = FS_HF_UNROLL;
// Groups of at least this many keys (dense: about one key per bin) are
// walked one counter word per lane, runs written straight to the output;
// sparser groups eight words per lane with a warp-synchronous cursor into the
// warp's staging buffer.  Measured per 2^32 / 2^30 u32 keys on one B200:
// dense walk 15.3 / 8.8 ms, cursor walk 17.2 / 7.3 ms (a loop over each
// lane's non-empty words with predicated stores: 15.3 / 9.0 ms).
constexpr uint64_t HF_DENSE = 32768;


// Device scratch of the fill (grow-only, per sorter).
struct HfCtl {
  uint64_t grp[HF_GROUPS + 1];      // group starts; grp[HF_GROUPS] = n
  uint64_t big_pre[HF_GROUPS + 1];  // chunks of the large groups listed before entry i
  uint32_t big_grp[HF_GROUPS];      // the large groups, in order
  uint32_t big_first[HF_GROUPS];    // first non-empty bin of each large group
  uint32_t nbig;
};

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t x) {
  const uint32_t lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if ((int)lane >= o) x += y;
  }
  return x;
}

// Exclusive scan over the block's threads (blockDim.x = 1024); *total gets
// the sum.  Ends with the block synchronised; s_tmp holds 33 words.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_tmp, uint32_t* total) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t x = warp_incl_scan(v);
  if (lane == 31) s_tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const uint32_t y = s_tmp[lane];
    const uint32_t ys = warp_incl_scan(y);
    s_tmp[lane] = ys - y;
    if (lane == 31) s_tmp[32] = ys;
  }
  __syncthreads();
  const uint32_t r = s_tmp[warp] + x - v;
  *total = s_tmp[32];
  __syncthreads();  // s_tmp may be reused
  return r;
}

// Write this lane's 16 runs: run b holds c[b] copies of bin `kbase + b`
// (ordered key) and the runs follow each other from out[p0].  Runs longer than
// HF_RUN are written by the whole warp, one run at a time (coalesced).
template <int XF>
__device__ __forceinline__ void hf_emit16(uint32_t* __restrict__ out, const uint32_t p0, const uint32_t (&c)[16],
                                          const uint32_t kbase) {
  bool large = false;
  uint32_t p = p0;
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    const uint32_t key = from_ordered<uint32_t, XF>(kbase + b);
    if (c[b] <= HF_RUN) {
      for (uint32_t q = 0; q < c[b]; ++q) out[p + q] = key;
    } else {
      large = true;
    }
    p += c[b];
  }
  if (__any_sync(0xffffffffu, large)) {
    const uint32_t lane = threadIdx.x & 31;
    p = p0;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      uint32_t mask = __ballot_sync(0xffffffffu, c[b] > HF_RUN);
      while (mask) {
        const int L = __ffs(mask) - 1;
        mask &= mask - 1;
        const uint32_t P = __shfl_sync(0xffffffffu, p, L);
        const uint32_t C = __shfl_sync(0xffffffffu, c[b], L);
        const uint32_t key = from_ordered<uint32_t, XF>(__shfl_sync(0xffffffffu, kbase, L) + b);
        for (uint32_t i = lane; i < C; i += 32) out[P + i] = key;
      }
      p += c[b];
    }
  }
}

// --------------------------------------------------------------------------
// Group bounds: binary search of each group's first key.  Before any pass
// ran (HF_XF_IN) every key has the same top 16 bits, and the search over the
// caller's keys, transformed as they are read, still finds them.
// --------------------------------------------------------------------------
template <int XF>
__global__ void __launch_bounds__(256)
    k_hf_bounds(const SortCtl* __restrict__ ctl, HfCtl* __restrict__ hf, const uint64_t n) {
  chain_wait();
  const uint32_t flags = ctl->hf_flags;
  if (!(flags & HF_ON)) return;
  const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g > HF_GROUPS) return;
  const uint32_t* src = static_cast<const uint32_t*>(ctl->hf_src);
  const bool xf = (flags & HF_XF_IN) != 0;
  uint64_t lo = 0, hi = n;
  if (g == HF_GROUPS) {
    lo = n;
  } else if (g > 0) {
    while (lo < hi) {
      const uint64_t mid = lo + ((hi - lo) >> 1);
      uint32_t x = src[mid];
      if (xf) x = to_ordered<uint32_t, XF>(x);
      if ((x >> 16) < g)
        lo = mid + 1;
      else
        hi = mid;
    }
  }
  hf->grp[g] = lo;
}

// --------------------------------------------------------------------------
// The large groups, listed in group order with the prefix of their chunk
// counts (one CTA; thread t looks at groups [64t, 64t + 64)).
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(HF_BLOCK) k_hf_plan(const SortCtl* __restrict__ ctl, HfCtl* __restrict__ hf) {
  chain_wait();
  if (!(ctl->hf_flags & HF_ON)) return;
  __shared__ uint32_t s_tmp[33];
  constexpr uint32_t PER = HF_GROUPS / HF_BLOCK;
  const uint32_t g0 = threadIdx.x * PER;
  uint32_t nb = 0, ch = 0;
  for (uint32_t k = 0; k < PER; ++k) {
    const uint64_t m = hf->grp[g0 + k + 1] - hf->grp[g0 + k];
    if (m > HF_LOCAL_MAX) {
      ++nb;
      ch += (uint32_t)((m + HF_CHUNK - 1) / HF_CHUNK);
    }
  }
  uint32_t nb_tot, ch_tot;
  uint32_t nb_at = block_excl_scan(nb, s_tmp, &nb_tot);
  uint32_t ch_at = block_excl_scan(ch, s_tmp, &ch_tot);
  for (uint32_t k = 0; k < PER && nb; ++k) {
    const uint64_t m = hf->grp[g0 + k + 1] - hf->grp[g0 + k];
    if (m > HF_LOCAL_MAX) {
      hf->big_grp[nb_at] = g0 + k;
      hf->big_pre[nb_at] = ch_at;
      ++nb_at;
      ch_at += (uint32_t)((m + HF_CHUNK - 1) / HF_CHUNK);
    }
  }
  if (threadIdx.x == 0) {
    hf->nbig = nb_tot;
    hf->big_pre[nb_tot] = ch_tot;
  }
}

// --------------------------------------------------------------------------
// One CTA per group of at most HF_LOCAL_MAX keys (groups c, c + grid, ...).
//   count: HF_UNROLL loads in flight per thread, then one shared reduction
//          (no return value) per key into packed 16-bit counters.  If the
//          counters then sum to less than the group's size, a low value
//          occurred 2^16 times or more and wrapped its field: the group is
//          counted again with atomics that return the old count, where the
//          thread that wraps a field records the bit (ovf) and takes back
//          the carry into the neighbouring field.
//   walk:  warp w owns words [1024w, 1024w + 1024) (bins [2048w, 2048w +
//          2048)).  The warps' totals give each warp its start, a warp scan
//          each lane's offset in a round.  Dense groups (>= HF_DENSE keys):
//          one word per lane per round, runs written straight out (lanes in
//          bin order, so a store instruction covers a short stretch).  Sparser
//          groups: 8 words per lane per round, a warp-synchronous cursor writes
//          every lane's next key into the warp's staging buffer, and the warp
//          copies the round out in order (coalesced); a round of more than
//          HF_STAGE keys is written directly.  Runs longer than HF_RUN are
//          written by the whole warp.  The counters are cleared as they are
//          read.
//   While a group is walked, the next group's keys are prefetched into L2
//   (cp.async.bulk.prefetch), so its count reads L2 while HBM streams.
// --------------------------------------------------------------------------
constexpr uint32_t HF_STAGE = 640;  // keys per warp
constexpr size_t HF_LOCAL_SMEM_STAGED = HF_LOCAL_SMEM + (size_t)HF_WARPS * HF_STAGE * 4;  // 216 KiB

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch the 16-byte-aligned interior of keys [lo, hi) into L2.
__device__ __forceinline__ void prefetch_keys_l2(const uint32_t* src, uint64_t lo, uint64_t hi) {
  uintptr_t a = reinterpret_cast<uintptr_t>(src + lo), z = reinterpret_cast<uintptr_t>(src + hi);
  a = (a + 15) & ~(uintptr_t)15;
  z &= ~(uintptr_t)15;
  constexpr uintptr_t PIECE = 64 << 10;
  for (; a + 16 <= z; a += PIECE) {
    const uintptr_t e = a + PIECE < z ? a + PIECE : z;
    prefetch_l2(reinterpret_cast<const void*>(a), (uint32_t)(e - a));
  }
}

// Sum of the two 16-bit fields of w.
__device__ __forceinline__ uint32_t fields(uint32_t w) { return __dp2a_lo(w, 0x0101u, 0u); }

template <int XF>
__global__ void __launch_bounds__(HF_BLOCK, 1)
    k_hf_local(const SortCtl* __restrict__ ctl, const HfCtl* __restrict__ hf) {
  chain_wait();
  const uint32_t flags = ctl->hf_flags;
  if (!(flags & HF_ON)) return;
  extern __shared__ __align__(16) uint32_t hsm[];
  uint32_t* cnt = hsm;
  uint32_t* ovf = hsm + HF_WORDS;
  __shared__ uint32_t s_wtot[HF_WARPS];
  const uint32_t* __restrict__ src = static_cast<const uint32_t*>(ctl->hf_src);
  uint32_t* __restrict__ dst = static_cast<uint32_t*>(ctl->hf_dst);
  const bool xf = (flags & HF_XF_IN) != 0;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* st = hsm + HF_WORDS + HF_OVF_WORDS + warp * HF_STAGE;
  for (uint32_t i = tid; i < (HF_WORDS + HF_OVF_WORDS) / 4; i += HF_BLOCK)
    reinterpret_cast<uint4*>(hsm)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  constexpr uint32_t WPW = HF_WORDS / HF_WARPS;  // 1024 words per warp
  constexpr uint32_t ROUNDS = WPW / (32 * 8);     // 4 rounds of 8 words per lane

  // one pass over the group's keys with f(ordered key)
  auto for_keys = [&](uint64_t lo, uint64_t hi, auto&& f) {
    uint64_t i = lo + tid;
    for (; i + (HF_UNROLL - 1) * HF_BLOCK < hi; i += HF_UNROLL * HF_BLOCK) {
      uint32_t x[HF_UNROLL];
#pragma unroll
      for (int k = 0; k < HF_UNROLL; ++k) x[k] = src[i + (uint64_t)k * HF_BLOCK];
#pragma unroll
      for (int k = 0; k < HF_UNROLL; ++k) f(xf ? to_ordered<uint32_t, XF>(x[k]) : x[k]);
    }
    for (; i + 3 * HF_BLOCK < hi; i += 4 * HF_BLOCK) {
      uint32_t x[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = src[i + (uint64_t)k * HF_BLOCK];
#pragma unroll
      for (int k = 0; k < 4; ++k) f(xf ? to_ordered<uint32_t, XF>(x[k]) : x[k]);
    }
    for (; i < hi; i += HF_BLOCK) f(xf ? to_ordered<uint32_t, XF>(src[i]) : src[i]);
  };

  for (uint32_t g = blockIdx.x; g < HF_GROUPS; g += gridDim.x) {
    const uint64_t lo = hf->grp[g], hi = hf->grp[g + 1];
    const uint64_t m = hi - lo;
    if (m == 0 || m > HF_LOCAL_MAX) continue;  // empty, or a large group (k_hf_big_*)
    if (m == 1) {
      if (tid == 0) {
        const uint32_t x = src[lo];
        dst[lo] = xf ? x : from_ordered<uint32_t, XF>(x);
      }
      continue;
    }
    // ---- count ----
    for_keys(lo, hi, [&](uint32_t x) {
      const uint32_t v = x & 0xffffu;
      atomicAdd(&cnt[v >> 1], 1u << ((v & 1u) << 4));  // result unused: a reduction
    });
    __syncthreads();
    // next group's keys into L2 while this one is walked
    if (tid == 0 && g + gridDim.x < HF_GROUPS) {
      const uint64_t lo2 = hf->grp[g + gridDim.x], hi2 = hf->grp[g + gridDim.x + 1];
      if (hi2 - lo2 > 1 && hi2 - lo2 <= HF_LOCAL_MAX) prefetch_keys_l2(src, lo2, hi2);
    }
    // ---- walk: warp totals ----
    uint32_t t = 0;
#pragma unroll
    for (uint32_t r = 0; r < ROUNDS; ++r) {
      const uint32_t j0 = warp * WPW + (r * 32 + lane) * 8;
      const uint4 w0 = *reinterpret_cast<const uint4*>(&cnt[j0]);
      const uint4 w1 = *reinterpret_cast<const uint4*>(&cnt[j0 + 4]);
      const uint32_t ob = (ovf[j0 >> 4] >> ((j0 & 15) << 1)) & 0xffffu;
      t += fields(w0.x) + fields(w0.y) + fields(w0.z) + fields(w0.w) + fields(w1.x) + fields(w1.y) +
           fields(w1.z) + fields(w1.w) + ((uint32_t)__popc(ob) << 16);
    }
    t = __reduce_add_sync(0xffffffffu, t);
    if (lane == 0) s_wtot[warp] = t;
    __syncthreads();
    if (__reduce_add_sync(0xffffffffu, s_wtot[lane]) != (uint32_t)m) {
      // a field wrapped: count again, exactly (rare: 2^16 equal keys in a group)
      __syncthreads();  // every warp has read s_wtot
      for (uint32_t i = tid; i < HF_WORDS / 4; i += HF_BLOCK)
        reinterpret_cast<uint4*>(cnt)[i] = make_uint4(0u, 0u, 0u, 0u);
      __syncthreads();
      for_keys(lo, hi, [&](uint32_t x) {
        const uint32_t v = x & 0xffffu, sh = (v & 1u) << 4;
        const uint32_t old = atomicAdd(&cnt[v >> 1], 1u << sh);
        if (((old >> sh) & 0xffffu) == 0xffffu) {  // this key wrapped the field
          if (sh == 0) atomicSub(&cnt[v >> 1], 1u << 16);
          atomicOr(&ovf[v >> 5], 1u << (v & 31));
        }
      });
      __syncthreads();
      t = 0;
#pragma unroll
      for (uint32_t r = 0; r < ROUNDS; ++r) {
        const uint32_t j0 = warp * WPW + (r * 32 + lane) * 8;
        const uint4 w0 = *reinterpret_cast<const uint4*>(&cnt[j0]);
        const uint4 w1 = *reinterpret_cast<const uint4*>(&cnt[j0 + 4]);
        const uint32_t ob = (ovf[j0 >> 4] >> ((j0 & 15) << 1)) & 0xffffu;
        t += fields(w0.x) + fields(w0.y) + fields(w0.z) + fields(w0.w) + fields(w1.x) + fields(w1.y) +
             fields(w1.z) + fields(w1.w) + ((uint32_t)__popc(ob) << 16);
      }
      t = __reduce_add_sync(0xffffffffu, t);
      if (lane == 0) s_wtot[warp] = t;
      __syncthreads();
    }
    uint32_t base = __reduce_add_sync(0xffffffffu, lane < warp ? s_wtot[lane] : 0u);
    uint32_t* out = dst + lo;
    if (m >= HF_DENSE) {
      // ---- walk: write, one word (two bins) per lane per round ----
      // Lanes hold consecutive words, so the lanes' runs follow each other in
      // lane order and each store instruction of the warp lands on a short
      // stretch of the output.  Runs up to HF_RUN by their lanes (the warp
      // loops to the longest), longer runs by the whole warp.
#pragma unroll 2
      for (uint32_t r = 0; r < WPW / 32; ++r) {
        const uint32_t j = warp * WPW + r * 32 + lane;
        const uint32_t wv = cnt[j];
        cnt[j] = 0u;
        const uint32_t e = (ovf[j >> 4] >> ((j & 15) << 1)) & 3u;
        const uint32_t c0 = (wv & 0xffffu) + ((e & 1u) << 16), c1 = (wv >> 16) + ((e >> 1) << 16);
        const uint32_t tl = c0 + c1;
        const uint32_t incl = warp_incl_scan(tl);
        const uint32_t p = base + incl - tl;
        base += __shfl_sync(0xffffffffu, incl, 31);
        const uint32_t kb = (g << 16) | (j << 1);
        const uint32_t k0 = from_ordered<uint32_t, XF>(kb), k1 = from_ordered<uint32_t, XF>(kb + 1);
        const bool small = c0 <= HF_RUN && c1 <= HF_RUN;
        const uint32_t s0 = small ? c0 : 0u, s1 = small ? c1 : 0u;
        const uint32_t qmax = __reduce_max_sync(0xffffffffu, s0 > s1 ? s0 : s1);
        for (uint32_t q = 0; q < qmax; ++q) {
          if (q < s0) out[p + q] = k0;
          if (q < s1) out[p + s0 + q] = k1;
        }
        uint32_t mask = __ballot_sync(0xffffffffu, !small);
        while (mask) {
          const int L = __ffs(mask) - 1;
          mask &= mask - 1;
          const uint32_t P = __shfl_sync(0xffffffffu, p, L);
          const uint32_t C0 = __shfl_sync(0xffffffffu, c0, L);
          const uint32_t C = C0 + __shfl_sync(0xffffffffu, c1, L);
          const uint32_t K0 = __shfl_sync(0xffffffffu, k0, L), K1 = __shfl_sync(0xffffffffu, k1, L);
          for (uint32_t i2 = lane; i2 < C; i2 += 32) out[P + i2] = i2 < C0 ? K0 : K1;
        }
      }
    } else {
      // ---- walk: write, eight words per lane per round (sparser groups) ----
#pragma unroll 1
      for (uint32_t r = 0; r < ROUNDS; ++r) {
        const uint32_t j0 = warp * WPW + (r * 32 + lane) * 8;
        uint4* wp = reinterpret_cast<uint4*>(&cnt[j0]);
        const uint4 w0 = wp[0], w1 = wp[1];
        const uint32_t ob = (ovf[j0 >> 4] >> ((j0 & 15) << 1)) & 0xffffu;
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint32_t tl = (uint32_t)__popc(ob) << 16;
#pragma unroll
        for (int k = 0; k < 8; ++k) tl += fields(w[k]);
        const uint32_t incl = warp_incl_scan(tl);
        const uint32_t p = incl - tl;                            // lane's offset in the round
        const uint32_t rt = __shfl_sync(0xffffffffu, incl, 31);  // keys of the round
        const uint32_t kbase = (g << 16) | (j0 << 1);
        const bool staged = rt <= HF_STAGE;
        uint32_t* o = staged ? st : out + base;  // generic: shared staging or global
        // Warp-synchronous cursor: step q writes every lane's q-th key, then
        // the lane moves to its next non-empty word when the current one is
        // spent.  Words holding a run longer than HF_RUN are skipped here (their
        // keys' positions left free) and written by the whole warp below.
        uint32_t wm = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) wm |= (uint32_t)((w[k] | ((ob >> (2 * k)) & 3u)) != 0u) << k;
        bool large = false;
        uint32_t pos = p, r0 = 0, r1 = 0, kk = 0;
        auto advance = [&]() {  // next non-empty word with short runs; skip the others
          while (wm) {
            kk = __ffs(wm) - 1;
            wm &= wm - 1;
            const uint32_t wv = cnt[j0 + kk];
            const uint32_t e = (ob >> (2 * kk)) & 3u;
            r0 = (wv & 0xffffu) + ((e & 1u) << 16);
            r1 = (wv >> 16) + ((e >> 1) << 16);
            if (r0 <= HF_RUN && r1 <= HF_RUN) return;
            large = true;
            pos += r0 + r1;
            r0 = r1 = 0;
          }
        };
        advance();
        while (__any_sync(0xffffffffu, (r0 | r1) != 0u)) {
          if (r0 | r1) {
            const uint32_t key = from_ordered<uint32_t, XF>(kbase + 2 * kk + (r0 ? 0u : 1u));
            o[pos++] = key;
            if (r0)
              --r0;
            else
              --r1;
            if ((r0 | r1) == 0u) advance();
          }
        }
        if (__any_sync(0xffffffffu, large)) {  // words with a long run: the whole warp writes them
          uint32_t pb = p;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t e = (ob >> (2 * k)) & 3u;
            const uint32_t c0 = (w[k] & 0xffffu) + ((e & 1u) << 16), c1 = (w[k] >> 16) + ((e >> 1) << 16);
            uint32_t mask = __ballot_sync(0xffffffffu, c0 > HF_RUN || c1 > HF_RUN);
            while (mask) {
              const int L = __ffs(mask) - 1;
              mask &= mask - 1;
              const uint32_t P = __shfl_sync(0xffffffffu, pb, L);
              const uint32_t C0 = __shfl_sync(0xffffffffu, c0, L);
              const uint32_t C = C0 + __shfl_sync(0xffffffffu, c1, L);
              const uint32_t kb = __shfl_sync(0xffffffffu, kbase, L) + 2 * k;
              const uint32_t k0 = from_ordered<uint32_t, XF>(kb), k1 = from_ordered<uint32_t, XF>(kb + 1);
              for (uint32_t i2 = lane; i2 < C; i2 += 32) o[P + i2] = i2 < C0 ? k0 : k1;
            }
            pb += c0 + c1;
          }
        }
        if (staged) {
          __syncwarp();
          for (uint32_t i2 = lane; i2 < rt; i2 += 32) out[base + i2] = st[i2];
          __syncwarp();  // staging read before the next round writes it
        }
        wp[0] = make_uint4(0u, 0u, 0u, 0u);
        wp[1] = make_uint4(0u, 0u, 0u, 0u);
        base += rt;
      }
    }
    __syncwarp();
    ovf[warp * (WPW / 16) + lane] = 0;  // only this warp read its bins' overflow bits
    ovf[warp * (WPW / 16) + 32 + lane] = 0;
    __syncthreads();  // counters clear before the next group's count
  }
}

// Large-group work item i -> (list entry b, chunk j), by binary search over
// the chunk prefix.
__device__ __forceinline__ void hf_big_item(const HfCtl* __restrict__ hf, uint32_t nbig, uint32_t i, uint32_t* b,
                                            uint32_t* j) {
  uint32_t lo = 0, hi = nbig;  // last entry with big_pre[entry] <= i
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (hf->big_pre[mid] <= i)
      lo = mid;
    else
      hi = mid;
  }
  *b = lo;
  *j = i - (uint32_t)hf->big_pre[lo];
}

// Zero the histograms of the large groups (pool entries 0 .. nbig-1).
__global__ void __launch_bounds__(256) k_hf_big_zero(const SortCtl* __restrict__ ctl, const HfCtl* __restrict__ hf) {
  chain_wait();
  if (!(ctl->hf_flags & HF_ON)) return;
  const uint64_t words = (uint64_t)hf->nbig * HF_BINS / 4;
  uint4* pool = static_cast<uint4*>(ctl->hf_pool);
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (uint64_t)gridDim.x * blockDim.x)
    pool[i] = make_uint4(0u, 0u, 0u, 0u);
}

// Count one chunk of a large group into shared 16-bit counters, then add the
// non-zero ones into the group's global histogram.
template <int XF>
__global__ void __launch_bounds__(HF_BLOCK, 1)
    k_hf_big_count(const SortCtl* __restrict__ ctl, const HfCtl* __restrict__ hf) {
  chain_wait();
  const uint32_t flags = ctl->hf_flags;
  if (!(flags & HF_ON)) return;
  const uint32_t nbig = hf->nbig;
  if (nbig == 0) return;
  extern __shared__ __align__(16) uint32_t hsm[];
  const uint32_t* __restrict__ src = static_cast<const uint32_t*>(ctl->hf_src);
  uint32_t* __restrict__ pool = static_cast<uint32_t*>(ctl->hf_pool);
  const bool xf = (flags & HF_XF_IN) != 0;
  const uint32_t tid = threadIdx.x;
  const uint32_t items = (uint32_t)hf->big_pre[nbig];
  for (uint32_t i = tid; i < HF_WORDS / 4; i += HF_BLOCK) reinterpret_cast<uint4*>(hsm)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
    uint32_t b, j;
    hf_big_item(hf, nbig, it, &b, &j);
    const uint32_t g = hf->big_grp[b];
    const uint64_t g0 = hf->grp[g], g1 = hf->grp[g + 1];
    const uint64_t lo = g0 + (uint64_t)j * HF_CHUNK;
    const uint64_t hi = lo + HF_CHUNK < g1 ? lo + HF_CHUNK : g1;
    auto count1 = [&](uint32_t x) {
      if (xf) x = to_ordered<uint32_t, XF>(x);
      const uint32_t v = x & 0xffffu;
      atomicAdd(&hsm[v >> 1], 1u << ((v & 1u) << 4));
    };
    uint64_t k0 = lo + tid;
    for (; k0 + (HF_UNROLL - 1) * HF_BLOCK < hi; k0 += HF_UNROLL * HF_BLOCK) {
      uint32_t x[HF_UNROLL];
#pragma unroll
      for (int k = 0; k < HF_UNROLL; ++k) x[k] = src[k0 + (uint64_t)k * HF_BLOCK];
#pragma unroll
      for (int k = 0; k < HF_UNROLL; ++k) count1(x[k]);
    }
    for (; k0 < hi; k0 += HF_BLOCK) count1(src[k0]);
    __syncthreads();
    uint32_t* h = pool + (size_t)b * HF_BINS;
    for (uint32_t w = tid; w < HF_WORDS; w += HF_BLOCK) {
      const uint32_t x = hsm[w];
      if (x) {
        hsm[w] = 0;
        if (x & 0xffffu) atomicAdd(&h[2 * w], x & 0xffffu);
        if (x >> 16) atomicAdd(&h[2 * w + 1], x >> 16);
      }
    }
    __syncthreads();
  }
}

// Exclusive scan of each large group's histogram, in place, and its first
// non-empty bin.  (A group of exactly 2^32 keys wraps the prefix after its
// last non-empty bin to 0; the fill tells those zeros from real ones by the
// first non-empty bin.)
__global__ void __launch_bounds__(HF_BLOCK)
    k_hf_big_scan(const SortCtl* __restrict__ ctl, HfCtl* __restrict__ hf) {
  chain_wait();
  if (!(ctl->hf_flags & HF_ON)) return;
  const uint32_t nbig = hf->nbig;
  __shared__ uint32_t s_tmp[33];
  __shared__ uint32_t s_first;
  uint32_t* pool = static_cast<uint32_t*>(ctl->hf_pool);
  constexpr uint32_t PER = HF_BINS / HF_BLOCK;  // 64 bins per thread
  for (uint32_t b = blockIdx.x; b < nbig; b += gridDim.x) {
    uint4* h = reinterpret_cast<uint4*>(pool + (size_t)b * HF_BINS + threadIdx.x * PER);
    if (threadIdx.x == 0) s_first = 0xffffffffu;
    uint32_t t = 0, first = 0xffffffffu;
#pragma unroll 4
    for (uint32_t q = 0; q < PER / 4; ++q) {
      const uint4 x = h[q];
      if (first == 0xffffffffu && (x.x | x.y | x.z | x.w))
        first = threadIdx.x * PER + 4 * q + (x.x ? 0 : x.y ? 1 : x.z ? 2 : 3);
      t += x.x + x.y + x.z + x.w;
    }
    __syncthreads();  // s_first initialised
    if (first != 0xffffffffu) atomicMin(&s_first, first);
    uint32_t tot;
    uint32_t run = block_excl_scan(t, s_tmp, &tot);
#pragma unroll 4
    for (uint32_t q = 0; q < PER / 4; ++q) {
      uint4 x = h[q];
      const uint32_t a = run, bb = a + x.x, cc = bb + x.y, dd = cc + x.z;
      run = dd + x.w;
      h[q] = make_uint4(a, bb, cc, dd);
    }
    if (threadIdx.x == 0) hf->big_first[b] = s_first;
    __syncthreads();
  }
}

// Write window j ([j*HF_CHUNK, min((j+1)*HF_CHUNK, m)) of the group's output)
// of a large group.  Bin v covers [P(v), P(v+1)) of the group, P the
// exclusive prefix (P(65536) = m); warp w takes the 512-bin blocks w, w + 32,
// ... from the first bin the window touches, lane l 16 bins of a block.
template <int XF>
__global__ void __launch_bounds__(HF_BLOCK)
    k_hf_big_fill(const SortCtl* __restrict__ ctl, const HfCtl* __restrict__ hf) {
  chain_wait();
  const uint32_t flags = ctl->hf_flags;
  if (!(flags & HF_ON)) return;
  const uint32_t nbig = hf->nbig;
  if (nbig == 0) return;
  __shared__ uint32_t s_v0;
  const uint32_t* __restrict__ pool = static_cast<const uint32_t*>(ctl->hf_pool);
  uint32_t* __restrict__ dst = static_cast<uint32_t*>(ctl->hf_dst);
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t items = (uint32_t)hf->big_pre[nbig];
  for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
    uint32_t b, j;
    hf_big_item(hf, nbig, it, &b, &j);
    const uint32_t g = hf->big_grp[b];
    const uint64_t g0 = hf->grp[g];
    const uint64_t m = hf->grp[g + 1] - g0;
    const uint64_t w0 = (uint64_t)j * HF_CHUNK;
    const uint64_t w1 = w0 + HF_CHUNK < m ? w0 + HF_CHUNK : m;
    const uint32_t* P = pool + (size_t)b * HF_BINS;
    const uint32_t first = hf->big_first[b];
    // P(v) as a 64-bit value: a stored 0 after the first non-empty bin is m
    auto pref = [&](uint32_t v) -> uint64_t {
      if (v >= HF_BINS) return m;
      const uint32_t x = P[v];
      return (x == 0 && v > first) ? m : (uint64_t)x;
    };
    if (tid == 0) {  // last bin with P(v) <= w0
      uint32_t lo = 0, hi = HF_BINS;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (pref(mid) <= w0)
          lo = mid;
        else
          hi = mid;
      }
      s_v0 = lo;
    }
    __syncthreads();
    const uint32_t v0 = s_v0;
    uint32_t* out = dst + g0 + w0;
    for (uint32_t blk = warp;; blk += HF_WARPS) {
      const uint32_t vb = v0 + blk * 512;  // first bin of this warp's block
      if (vb >= HF_BINS || pref(vb) >= w1) break;
      // the lane's bins are consecutive, so its clamped runs are too
      const uint32_t v = vb + lane * 16;
      uint32_t c[16];
      uint64_t s = pref(v);
      const uint32_t p0 = (uint32_t)((s > w0 ? (s < w1 ? s : w1) : w0) - w0);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const uint64_t e = pref(v + q + 1);
        const uint64_t a = s > w0 ? s : w0;
        const uint64_t z = e < w1 ? e : w1;
        c[q] = (v + q < HF_BINS && z > a) ? (uint32_t)(z - a) : 0u;
        s = e;
      }
      hf_emit16<XF>(out, p0, c, (g << 16) | (v & 0xffffu));
    }
    __syncthreads();  // s_v0 is rewritten for the next item
  }
}

}  // namespace fs
