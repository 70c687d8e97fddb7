// fs_resident.cuh -- a whole keys-only sort of up to a few million 32-bit
// keys in one cooperative launch, for the sizes where the chained launches of
// fs_kernels.cuh cost more than their kernels.  One CTA per SM, all resident;
// CTA c owns positions [c*TILE, (c+1)*TILE) (TILE = BLOCK*IPT) and holds them
// in registers from its first load.
//
// Main form (MSD, up to 7 keys a thread):
//   1. rank the tile by the top RES_MB bits with shared atomics (keys only:
//      any order among equal buckets), publish the CTA's bucket counts and add
//      them to 16-CTA group sums in L2;
//   2. grid barrier; each bucket's output base = the buckets before it (all
//      group sums) + the group sums before this CTA's group + the counts of
//      the CTAs before it in its group; stage the tile in bucket order and
//      write it;
//   3. grid barrier; load this CTA's segment -- the buckets that start in its
//      tile's range -- and sort it in shared memory: bitonic sorts of 256 keys
//      per warp in registers, then merge-path merges, no grid barrier.
// When a bucket holds more than a tile (skewed keys, or top bits that never
// vary) the same launch runs LSD passes instead, per executed 8-bit digit:
// rank (shared atomics for the first executed pass, owner election and five
// ballots after), publish, barrier, offsets, stage and write coalesced,
// barrier, reload.  The passes run in place in the output array: a pass's
// loads all happen before its first barrier and its stores after it.  The
// OR / AND words published with the first counts give every CTA the same
// plan (trivial digits skipped, the inverse transform on the last pass).
//
// Measured on one B200 (globaltimer stamps and clock64 laps per phase, 2^20
// u32 keys on 147 CTAs): a barrier built from a generation word cost 2.2-3.9
// us (four dependent L2 round trips), and one global OR per warp made the
// first barrier 6.6 us (4704 atomics on one word).  Here a barrier is one
// release reduction on a counter that only grows within a launch (the k-th
// barrier waits for k * gridDim.x arrivals) and the OR/AND words take one
// atomic per CTA.  Sorting segments with four local LSD passes cost ~6 us a
// pass (ranking at 70 instructions per 32 keys plus ~3 us of fixed scans
// and barriers); the merge sort replaced them.
//
// The accumulators (group sums, OR/AND words, barrier counter) come in two
// sets used by alternate launches: each launch clears the set the next one
// uses, so no memset precedes the launch.  Every barrier wait is bounded: on
// timeout the CTA records DEV_ERR_TIMEOUT (device word and the host's mapped
// error word) and returns.
#pragma once

#include "fs_kernels.cuh"

namespace fs {

constexpr int RES_GROUP = 16;   // CTAs per group sum
constexpr int RES_BLOCK = 1024;
constexpr int RES_MAX_CTAS = 2 * 148;  // 2048 threads per SM at most; the host checks the SM count

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier over all CTAs of a cooperative launch, the `k`-th of this
// launch (k = 1, 2, ...): thread 0 adds its arrival with a release (after the
// CTA's __syncthreads, so it covers every thread's stores) and waits with
// acquires until k * gridDim.x CTAs have arrived.  false: the wait ran out
// (DEV_ERR_TIMEOUT recorded in the device word and the host's mapped word).
__device__ __forceinline__ bool res_grid_sync(unsigned* bar, unsigned k, uint64_t timeout_ns, SortCtl* ctl,
                                              int* host_err, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = k * gridDim.x;
    red_add_release_u32(bar, 1u);
    if (ld_acquire_u32(bar) < target) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_u32(bar) >= target) break;
        if ((i & 63u) == 0 && global_timer_ns() - t0 > timeout_ns) {
          atomicCAS(&ctl->err, 0, DEV_ERR_TIMEOUT);
          *(volatile int*)host_err = DEV_ERR_TIMEOUT;
          ok = 0;
          break;
        }
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Accumulator set (32-bit words): [slots][groups][RADIX] group sums (one
// slot per digit pass, one more for the most-significant-digit partition),
// then the OR and ~AND words of the ordered keys (lo, hi each) and the
// barrier counter, padded to 16 bytes.
__host__ __device__ constexpr uint32_t res_acc_words(int slots, uint32_t groups) {
  return (uint32_t)slots * RADIX * groups + 8u;
}

struct ResArgs {
  const void* kin;
  void* kout;         // may equal kin (in place)
  uint64_t n;         // 2 .. gridDim.x * TILE
  SortCtl* ctl;       // err
  uint32_t* counts;   // [slots][gridDim.x][RADIX], plain stores
  uint32_t* acc;      // this launch's accumulator set (zero on entry)
  uint32_t* acc_next; // the next launch's set: cleared here
  uint32_t acc_words; // words of a set (the largest layout any launch uses)
  uint32_t groups;    // group sums per pass in a set (>= ceil(gridDim.x / RES_GROUP))
  uint64_t timeout_ns;
  int* host_err;      // mapped page-locked word the host reads after the sort
  int test_skip_arrival;  // failure-path test: CTA 0 leaves before the first barrier
};

template <typename K, int BLOCK, int IPT, bool MSD = false>
struct ResLayout {
  static constexpr int WARPS = BLOCK / 32;
  static constexpr int TILE = BLOCK * IPT;
  static constexpr int SEG = 32 * IPT;
  static constexpr int Q = BLOCK / RADIX;  // threads per digit in the per-digit phases
  static constexpr int MAXG = ((RES_MAX_CTAS + RES_GROUP - 1) / RES_GROUP + Q - 1) / Q;  // group loads a thread
  static constexpr int MAXW = (RES_GROUP - 1 + Q - 1) / Q;  // in-group count loads a thread
  // dynamic shared memory: [warp digit counters | warp digit owners | staged
  // keys: one tile, or (MSD) two buffers of a segment of up to two tiles,
  // rounded up to whole 256-key runs]
  static constexpr int STAGE_KEYS = MSD ? (2 * TILE + 255) / 256 * 256 : TILE;
  static constexpr size_t CNT_OFF = 0;
  static constexpr size_t REP_OFF = CNT_OFF + (size_t)WARPS * RADIX * 4;
  static constexpr size_t STAGE_OFF = REP_OFF + (size_t)WARPS * RADIX;
  static constexpr size_t BYTES =
      STAGE_OFF + (MSD ? 2 * (size_t)(STAGE_KEYS + STAGE_KEYS / 32) : (size_t)STAGE_KEYS) * sizeof(K);
  static_assert(!MSD || 2 * TILE <= 16 * BLOCK, "a merge level covers a segment in one round");
  static_assert(BLOCK % RADIX == 0 && WARPS % Q == 0, "whole warps per digit-thread group");
  static_assert(STAGE_OFF % 16 == 0, "staging alignment");
};

// Shared state of one CTA of k_resident_sort.
struct ResShared {
  uint32_t* cnt;    // [WARPS][RADIX] per-warp digit counters
  uint8_t* rep;     // [WARPS][RADIX] per-warp digit owners
  uint32_t (*q)[RADIX];   // [Q][RADIX] partial sums per digit-thread group
  uint32_t (*q2)[RADIX];  // [Q][RADIX] partial digit totals
  uint32_t* tpart;  // [RADIX] tile-local digit start within its warp of digits
  uint32_t* tstart; // [RADIX] tile-local start of each digit
  uint32_t* off;    // [RADIX] global position - staging index, per digit
  uint32_t* wsum;   // [RADIX / 32]
};

// Warp-local ranks of `rows` rows of 32 keys: lane l's k-th key is element
// wofs + 32k of the CTA's range (`lim` of them valid).  `unstable`: shared
// atomics (any order among equal digits); otherwise owner election through a
// byte per digit and five ballots over the owner's lane bits, which keeps the
// order.  After the loop wcnt holds the warp's count of each digit.
template <typename K, int NR, bool PACK>
__device__ __forceinline__ void res_rank(const K (&key)[NR], Ranks<NR, PACK>& rank, int rows, uint32_t wofs,
                                         uint32_t lim, int shift, bool unstable, uint32_t* wcnt, uint8_t* wrep) {
  const uint32_t lane = threadIdx.x & 31, lt_mask = (1u << lane) - 1u;
  if (unstable) {
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      if (k < rows) {
        const bool valid = wofs + k * 32 < lim;
        rank.set(k, valid ? atomicAdd(&wcnt[(uint32_t)(key[k] >> shift) & (RADIX - 1)], 1u) : 0u);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      if (k < rows) {
        const bool valid = wofs + k * 32 < lim;
        const uint32_t d = (uint32_t)(key[k] >> shift) & (RADIX - 1);
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
    }
  }
}

// After ranking (and a __syncthreads): turn the per-warp counters into each
// warp's start per digit (tile-local digit start + the counts of the earlier
// warps).  `on_total(tot)` runs on threads tid < RADIX with the CTA's count of
// digit tid, between the two internal barriers.  sh.tstart gets the
// tile-local digit starts.  Ends without a barrier.
template <int BLOCK, typename F>
__device__ __forceinline__ void res_warp_starts(const ResShared& sh, F&& on_total) {
  constexpr int Q = BLOCK / RADIX, WPQ = BLOCK / 32 / Q;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t d = tid % RADIX, q = tid / RADIX;
  {
    uint32_t sum = 0;
#pragma unroll
    for (int w = 0; w < WPQ; ++w) sum += sh.cnt[(q * WPQ + w) * RADIX + d];
    sh.q[q][d] = sum;
  }
  __syncthreads();
  {
    uint32_t run = 0, tot = 0;
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) {
      const uint32_t v = sh.q[qq][d];
      if (qq < (int)q) run += v;
      tot += v;
    }
#pragma unroll
    for (int w = 0; w < WPQ; ++w) {  // exclusive prefix over the warps, per digit
      uint32_t* cw = &sh.cnt[(q * WPQ + w) * RADIX + d];
      const uint32_t v = *cw;
      *cw = run;
      run += v;
    }
    if (tid < RADIX) {
      on_total(tot);
      uint32_t x = tot;  // tile-local digit starts: exclusive scan of tot over the digits
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if ((int)lane >= o) x += y;
      }
      if (lane == 31) sh.wsum[warp] = x;
      sh.tpart[tid] = x - tot;
    }
  }
  __syncthreads();
  uint32_t ts = sh.tpart[d];
  for (uint32_t w = 0; w < (d >> 5); ++w) ts += sh.wsum[w];
  if (q == 0) sh.tstart[d] = ts;
#pragma unroll
  for (int w = 0; w < WPQ; ++w) sh.cnt[(q * WPQ + w) * RADIX + d] += ts;
}

// After a grid barrier: the output base of each digit of accumulator slot
// `slot` for CTA c, minus the tile-local digit start (sh.off).  Loads first
// (at most MAXG + MAXW a thread), then two block barriers.
template <int BLOCK, int MAXG, int MAXW>
__device__ __forceinline__ void res_offsets(const ResShared& sh, const uint32_t* grp, const uint32_t* counts,
                                            uint32_t groups, int slot) {
  constexpr int Q = BLOCK / RADIX;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t d = tid % RADIX, q = tid / RADIX;
  const uint32_t c = blockIdx.x, G = gridDim.x;
  const uint32_t g_me = c / RES_GROUP, ngrp = (G + RES_GROUP - 1) / RES_GROUP;
  uint32_t gv[MAXG], wv[MAXW];
  {
    const uint32_t* gp = grp + (size_t)slot * groups * RADIX + d;
    const uint32_t* cp = counts + ((size_t)slot * G + g_me * RES_GROUP) * RADIX + d;
    const uint32_t nw = c - g_me * RES_GROUP;
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      const uint32_t g = q + i * Q;
      gv[i] = g < ngrp ? __ldcg(gp + (size_t)g * RADIX) : 0u;
    }
#pragma unroll
    for (int i = 0; i < MAXW; ++i) {
      const uint32_t j = q + i * Q;
      wv[i] = j < nw ? __ldcg(cp + (size_t)j * RADIX) : 0u;
    }
  }
  {
    uint32_t tot = 0, pre = 0;
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      tot += gv[i];
      if (q + i * Q < g_me) pre += gv[i];
    }
#pragma unroll
    for (int i = 0; i < MAXW; ++i) pre += wv[i];
    sh.q[q][d] = pre;
    sh.q2[q][d] = tot;
  }
  __syncthreads();
  if (tid < RADIX) {
    uint32_t tot = 0, pre = 0;
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) {
      tot += sh.q2[qq][tid];
      pre += sh.q[qq][tid];
    }
    uint32_t x = tot;  // digit starts: exclusive scan of the totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if ((int)lane >= o) x += y;
    }
    if (lane == 31) sh.wsum[warp] = x;
    sh.off[tid] = x - tot + pre - sh.tstart[tid];
  }
  __syncthreads();
  if (tid < RADIX) {
    uint32_t add = 0;
    for (uint32_t w = 0; w < (tid >> 5); ++w) add += sh.wsum[w];
    sh.off[tid] += add;
  }
}

// Stage the tile's keys in digit order (warp starts in sh.cnt plus ranks),
// then write them to kout at sh.off[digit] + staging index (`xout`: inverse
// order transform).  Out-of-range positions record DEV_ERR_BOUNDS and are
// dropped.  Ends without a barrier after the writes.
template <typename K, int XF, int BLOCK, int IPT, int STAGE_KEYS, bool PACK>
__device__ __forceinline__ void res_scatter(const ResShared& sh, K* stage, const K (&key)[IPT],
                                            const Ranks<IPT, PACK>& rank, uint32_t wofs, uint32_t tile_n, int shift,
                                            K* kout, uint64_t n, bool xout, SortCtl* ctl) {
  const uint32_t tid = threadIdx.x;
  const uint32_t* wcnt = sh.cnt + (tid >> 5) * RADIX;
  bool oob = false;
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    if (wofs + k * 32 < tile_n) {
      const uint32_t si = wcnt[(uint32_t)(key[k] >> shift) & (RADIX - 1)] + rank.get(k);
      if (si < (uint32_t)STAGE_KEYS)
        stage[si] = key[k];
      else
        oob = true;
    }
  }
  __syncthreads();
  const uint64_t lastpos = n - 1;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t i = j * BLOCK + tid;
    if (i < tile_n) {
      const K kk = stage[i];
      const uint64_t pos = (uint64_t)sh.off[(uint32_t)(kk >> shift) & (RADIX - 1)] + i;
      if (pos <= lastpos)
        kout[pos] = xout ? from_ordered<K, XF>(kk) : kk;
      else
        oob = true;
    }
  }
  if (oob) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
}

// ---- merge sort of a segment in shared memory (keys only) ----------------------
// Equal keys are identical bits, so no order among them has to be kept: a
// bitonic sort of 256 keys per warp in registers, then merge-path merges of
// sorted runs between two shared-memory buffers.
constexpr int RES_RUN = 256;  // keys a warp sorts in registers (8 a lane)

// Bitonic sort of 256 keys held blocked across the warp (lane l holds
// elements 8l .. 8l+7): the three low index bits are a lane's registers,
// the five high bits its lane number.
template <typename K>
__device__ __forceinline__ void warp_sort256(K (&x)[8]) {
  const uint32_t lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= RES_RUN; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 8) {  // partner: same register of lane ^ (j / 8)
        const uint32_t lm = (uint32_t)j >> 3;
        const bool lower = (lane & lm) == 0;
        const bool up = ((lane * 8) & (uint32_t)k) == 0;  // k >= 16: the block direction is the lane's
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const K y = __shfl_xor_sync(0xffffffffu, x[i], lm);
          x[i] = (lower == up) ? (x[i] < y ? x[i] : y) : (x[i] < y ? y : x[i]);
        }
      } else {  // partner: register i ^ j of the same lane
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int pi = i ^ j;
          if (pi > i) {
            const bool up = ((lane * 8 + (uint32_t)i) & (uint32_t)k) == 0;
            const K lo = x[i] < x[pi] ? x[i] : x[pi];
            const K hi = x[i] < x[pi] ? x[pi] : x[i];
            x[i] = up ? lo : hi;
            x[pi] = up ? hi : lo;
          }
        }
      }
    }
  }
}

// Segment buffers are indexed with one padding word per 32 keys, so that
// lanes 8 keys apart (a lane's run slice, a thread's merge outputs) fall in
// different banks.
__device__ __forceinline__ uint32_t res_pad(uint32_t i) { return i + (i >> 5); }
__host__ __device__ constexpr uint32_t res_padded(uint32_t n) { return n + n / 32; }

// One merge level: the sorted runs of length r in src[0, len) merged in
// pairs into dst (len a multiple of RES_RUN, r a power of two >= RES_RUN,
// len <= PER * BLOCK).  Thread t writes outputs [PER*t, PER*t + PER): a
// binary search on its merge-path diagonal, then PER merge steps.
template <typename K, int BLOCK, int PER>
__device__ __forceinline__ void res_merge_level(const K* src, K* dst, uint32_t len, uint32_t r) {
  const uint32_t o0 = threadIdx.x * PER;
  if (o0 >= len) return;
  const uint32_t base = o0 & ~(2 * r - 1);
  const uint32_t la = min(r, len - base);
  const uint32_t lb = min(r, len - base - la);
  const uint32_t a0 = base, b0 = base + la;
  const uint32_t diag = o0 - base;
  uint32_t lo = diag > lb ? diag - lb : 0u, hi = min(diag, la);
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (src[res_pad(a0 + mid)] <= src[res_pad(b0 + diag - 1 - mid)])
      lo = mid + 1;
    else
      hi = mid;
  }
  // merge steps without divergence: one load a step, of the run that advanced
  uint32_t ia = lo, ib = diag - lo;
  K ka = ia < la ? src[res_pad(a0 + ia)] : K(0), kb = ib < lb ? src[res_pad(b0 + ib)] : K(0);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const bool take_a = ib >= lb || (ia < la && ka <= kb);
    dst[res_pad(o0 + e)] = take_a ? ka : kb;
    ia += take_a;
    ib += !take_a;
    const uint32_t nx = take_a ? a0 + ia : b0 + ib;
    const bool in = take_a ? ia < la : ib < lb;
    const K v = in ? src[res_pad(nx)] : K(0);
    ka = take_a ? v : ka;
    kb = take_a ? kb : v;
  }
}

// Top-bits partition of the MSD form: 2^RES_MB buckets (about 512 keys each
// at 2^20 uniform keys, so every CTA's segment stays close to one tile).
constexpr int RES_MB = 11;
constexpr int RES_MR = 1 << RES_MB;

// Exclusive scan of one value a thread over the block (w32: 32 words of
// shared memory).  Two block barriers.
template <int BLOCK>
__device__ __forceinline__ uint32_t res_block_exclusive_scan(uint32_t v, uint32_t* w32) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if ((int)lane >= o) x += y;
  }
  if (lane == 31) w32[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t t = lane < (uint32_t)(BLOCK / 32) ? w32[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
      if ((int)lane >= o) t += y;
    }
    w32[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  return x - v + (warp ? w32[warp - 1] : 0u);
}

// MSD: first partition by the top digit across the grid (one pass, ranked
// with shared atomics), then each CTA sorts a segment of whole top-digit
// buckets -- those starting in its tile's range, at most two tiles when no
// bucket holds more than a tile -- in shared memory with the LSD passes of
// every varying digit and no grid barrier between them.  When a bucket is
// larger than a tile (skewed keys, or the top digit constant) the same launch
// runs the plain LSD passes instead.
template <typename K, int XF, int BLOCK, int IPT, bool MSD>
__global__ void __launch_bounds__(BLOCK, 1) k_resident_sort(const ResArgs a) {
  using Ly = ResLayout<K, BLOCK, IPT, MSD>;
  constexpr int P = (int)sizeof(K);
  constexpr int Q = Ly::Q;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ uint32_t s_q[Q][RADIX];
  __shared__ uint32_t s_q2[Q][RADIX];
  __shared__ uint32_t s_tpart[RADIX];
  __shared__ uint32_t s_tstart[RADIX];
  __shared__ uint32_t s_off[RADIX];
  __shared__ uint32_t s_wsum[RADIX / 32];
  __shared__ uint32_t s_or[4];
  __shared__ uint32_t s_seg[3];  // MSD: segment start, end, largest bucket
  __shared__ uint32_t s_w32[32];
  __shared__ int s_ok;

  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t c = blockIdx.x, G = gridDim.x;
  const uint64_t n = a.n;
  const uint64_t tbase = (uint64_t)c * Ly::TILE;
  const uint32_t tile_n = n - tbase < (uint64_t)Ly::TILE ? (uint32_t)(n - tbase) : (uint32_t)Ly::TILE;
  const uint32_t wofs = warp * Ly::SEG + lane;
  const ResShared sh{reinterpret_cast<uint32_t*>(dsm + Ly::CNT_OFF), dsm + Ly::REP_OFF, s_q, s_q2, s_tpart,
                     s_tstart, s_off, s_wsum};
  uint32_t* wcnt = sh.cnt + warp * RADIX;
  uint8_t* wrep = sh.rep + warp * RADIX;
  K* stage = reinterpret_cast<K*>(dsm + Ly::STAGE_OFF);
  SortCtl* ctl = a.ctl;
  // [P][groups][RADIX] per digit pass, then (MSD) [groups][RES_MR] for the partition
  constexpr int SLOTS = P + (MSD ? RES_MR / RADIX : 0);
  uint32_t* grp = a.acc;
  uint32_t* orand = a.acc + (size_t)SLOTS * a.groups * RADIX;  // or lo, or hi, ~and lo, ~and hi
  unsigned* bar = orand + 4;
  unsigned nbar = 0;
  const uint32_t g_me = c / RES_GROUP;
  K* kout = static_cast<K*>(a.kout);

  auto finish = [&]() {  // hand a device-side error to the host
    if (tid == 0) {
      const int e = ld_relaxed_s32(&ctl->err);
      if (e != 0) *(volatile int*)a.host_err = e;
    }
  };
  auto zero_cnt = [&]() {
    for (int i = tid; i < Ly::WARPS * RADIX; i += BLOCK) sh.cnt[i] = 0;
  };
  // publish the CTA's digit counts of accumulator slot `slot`
  auto publisher = [&](int slot, bool with_or) {
    return [&, slot, with_or](uint32_t tot) {
      __stcg(&a.counts[((size_t)slot * G + c) * RADIX + tid], tot);
      if (tot) atomicAdd(&grp[((size_t)slot * a.groups + g_me) * RADIX + tid], tot);
      if (with_or && tid < 4 && s_or[tid]) atomicOr(&orand[tid], s_or[tid]);
    };
  };
  auto or_reduce = [&](K kor, K kandn) {  // one shared OR per warp
    const uint32_t lo_or = __reduce_or_sync(0xffffffffu, (uint32_t)kor);
    const uint32_t lo_an = __reduce_or_sync(0xffffffffu, (uint32_t)kandn);
    uint32_t hi_or = 0, hi_an = 0;
    if constexpr (sizeof(K) == 8) {
      hi_or = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kor >> 32));
      hi_an = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kandn >> 32));
    }
    if (lane == 0) {
      atomicOr(&s_or[0], lo_or);
      atomicOr(&s_or[1], hi_or);
      atomicOr(&s_or[2], lo_an);
      atomicOr(&s_or[3], hi_an);
    }
  };
  auto plan_of = [&]() -> uint32_t {  // digits that vary across all keys
    const unsigned long long o = ((unsigned long long)__ldcg(&orand[1]) << 32) | __ldcg(&orand[0]);
    const unsigned long long an = ((unsigned long long)__ldcg(&orand[3]) << 32) | __ldcg(&orand[2]);
    const unsigned long long varying = o & an;
    uint32_t e = 0;
#pragma unroll
    for (int pp = 0; pp < P; ++pp)
      if ((varying >> (RADIX_BITS * pp)) & (RADIX - 1)) e |= 1u << pp;
    return e;
  };

  // clear the next launch's accumulators and this CTA's counters
  for (uint32_t i = c * BLOCK + tid; i < a.acc_words; i += G * BLOCK) a.acc_next[i] = 0;
  zero_cnt();
  if (tid < 4) s_or[tid] = 0;
  if (tid == 0) {
    s_seg[0] = (uint32_t)n;
    s_seg[1] = (uint32_t)n;
    s_seg[2] = 0;
  }

  // ---- keys -> registers (forward order transform) -----------------------------
  K key[IPT];
  K kor = 0, kandn = 0;
  {
    const K* kin = static_cast<const K*>(a.kin);
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const uint32_t li = wofs + k * 32;
      if (li < tile_n) {
        key[k] = to_ordered<K, XF>(kin[tbase + li]);
        kor |= key[k];
        kandn |= ~key[k];
      } else {
        key[k] = 0;
      }
    }
  }
  __syncthreads();

  Ranks<IPT, true> rank;
  uint32_t exec = 0;
  bool planned = false;

  if constexpr (MSD) {
    // ---- partition by the top MB bits --------------------------------------------------
    // CTA-wide counters (ranks by shared atomics: keys only, any order among
    // equal buckets), MR / BLOCK buckets a thread for the scans and offsets
    constexpr int DPT = RES_MR / BLOCK;
    constexpr int MSHIFT = 8 * P - RES_MB;
    static_assert(RES_MR % BLOCK == 0 && RES_MR <= Ly::WARPS * RADIX, "bucket counters fit the warp counters");
    static_assert(res_padded(Ly::STAGE_KEYS) * sizeof(K) >= 2 * RES_MR * sizeof(uint32_t),
                  "bucket offsets and starts fit the idle segment buffer");
    uint32_t* mcnt = sh.cnt;                                  // [MR]: counts, then tile-local starts
    uint32_t* moff = reinterpret_cast<uint32_t*>(stage + res_padded(Ly::STAGE_KEYS));  // [MR] in the idle buffer
    uint32_t* mstart = moff + RES_MR;                         // [MR] bucket starts
    uint32_t* grp_m = grp + (size_t)P * a.groups * RADIX;     // [groups][MR]
    uint32_t* cnt_m = a.counts + (size_t)P * G * RADIX;       // [G][MR]
    uint32_t mr[IPT];
#pragma unroll
    for (int k = 0; k < IPT; ++k)
      mr[k] = (wofs + k * 32 < tile_n) ? atomicAdd(&mcnt[(uint32_t)(key[k] >> MSHIFT)], 1u) : 0u;
    or_reduce(kor, kandn);
    __syncthreads();
    {
      uint32_t cv[DPT], sum = 0;
#pragma unroll
      for (int j = 0; j < DPT; ++j) {
        const uint32_t d = tid * DPT + j;
        cv[j] = mcnt[d];
        __stcg(&cnt_m[(size_t)c * RES_MR + d], cv[j]);
        if (cv[j]) atomicAdd(&grp_m[(size_t)g_me * RES_MR + d], cv[j]);
        sum += cv[j];
      }
      if (tid < 4 && s_or[tid]) atomicOr(&orand[tid], s_or[tid]);
      uint32_t run = res_block_exclusive_scan<BLOCK>(sum, s_w32);
#pragma unroll
      for (int j = 0; j < DPT; ++j) {
        mcnt[tid * DPT + j] = run;
        run += cv[j];
      }
    }
    if (a.test_skip_arrival && c == 0) return;
    if (!res_grid_sync(bar, ++nbar, a.timeout_ns, ctl, a.host_err, &s_ok)) return finish();
    exec = plan_of();  // (its loads are in flight with the offsets' loads)
    planned = true;
    {
      // bucket totals (all group sums) and this CTA's prefix (the group sums
      // before its group, the counts of the CTAs before it in its group)
      constexpr int NG = (RES_MAX_CTAS + RES_GROUP - 1) / RES_GROUP;
      const uint32_t ngrp = (G + RES_GROUP - 1) / RES_GROUP, nw = c - g_me * RES_GROUP;
      uint32_t tot[DPT], pre[DPT], sum = 0, mx = 0;
#pragma unroll
      for (int j = 0; j < DPT; ++j) {
        const uint32_t d = tid * DPT + j;
        uint32_t t = 0, q = 0;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const uint32_t v = (uint32_t)g < ngrp ? __ldcg(&grp_m[(size_t)g * RES_MR + d]) : 0u;
          t += v;
          if ((uint32_t)g < g_me) q += v;
        }
#pragma unroll
        for (int w = 0; w < RES_GROUP - 1; ++w)
          q += (uint32_t)w < nw ? __ldcg(&cnt_m[(size_t)(g_me * RES_GROUP + w) * RES_MR + d]) : 0u;
        tot[j] = t;
        pre[j] = q;
        sum += t;
        mx = max(mx, t);
      }
      uint32_t run = res_block_exclusive_scan<BLOCK>(sum, s_w32);
#pragma unroll
      for (int j = 0; j < DPT; ++j) {
        const uint32_t d = tid * DPT + j;
        mstart[d] = run;
        moff[d] = run + pre[j] - mcnt[d];
        run += tot[j];
      }
      mx = __reduce_max_sync(0xffffffffu, mx);
      if (lane == 0) atomicMax(&s_seg[2], mx);
    }
    __syncthreads();
    if (exec == 0) {  // every key equal: the output is the input
      if (a.kout != a.kin) {
#pragma unroll
        for (int k = 0; k < IPT; ++k) {
          const uint32_t li = wofs + k * 32;
          if (li < tile_n) kout[tbase + li] = from_ordered<K, XF>(key[k]);
        }
      }
      return finish();
    }
    if (s_seg[2] <= (uint32_t)Ly::TILE) {
      // this CTA's segment: the buckets starting in [c*TILE, (c+1)*TILE)
      {
        const uint32_t t0 = c * (uint32_t)Ly::TILE, t1 = t0 + (uint32_t)Ly::TILE;
#pragma unroll
        for (int j = 0; j < DPT; ++j) {
          const uint32_t d = tid * DPT + j;
          const uint32_t st = mstart[d], prev = d ? mstart[d - 1] : 0u;
          if (st >= t0 && (d == 0 || prev < t0)) s_seg[0] = st;
          if (st >= t1 && (d == 0 || prev < t1)) s_seg[1] = st;
        }
      }
      // stage in bucket order, write to the buckets' positions
      bool oob = false;
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        if (wofs + k * 32 < tile_n) {
          const uint32_t si = mcnt[(uint32_t)(key[k] >> MSHIFT)] + mr[k];
          if (si < (uint32_t)Ly::TILE)
            stage[si] = key[k];
          else
            oob = true;
        }
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < IPT; ++j) {
        const uint32_t i = j * BLOCK + tid;
        if (i < tile_n) {
          const K kk = stage[i];
          const uint64_t pos = (uint64_t)moff[(uint32_t)(kk >> MSHIFT)] + i;
          if (pos < n)
            kout[pos] = kk;
          else
            oob = true;
        }
      }
      if (oob) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
      zero_cnt();
      if (!res_grid_sync(bar, ++nbar, a.timeout_ns, ctl, a.host_err, &s_ok)) return finish();

      // ---- sort the segment in shared memory: warp sorts, then merges ---------------
      // (the segment is padded to whole runs with all-ones keys, which sort
      // last; only its first L keys are written back)
      const uint32_t seg_lo = s_seg[0], L = s_seg[1] - s_seg[0];
      if (s_seg[1] < s_seg[0] || L > 2u * Ly::TILE) {  // cannot happen with buckets <= TILE
        if (tid == 0) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
        return finish();
      }
      const uint32_t len = (L + RES_RUN - 1) & ~(uint32_t)(RES_RUN - 1);
      K* buf0 = stage;
      K* buf1 = stage + res_padded(Ly::STAGE_KEYS);
      for (uint32_t i = tid; i < len; i += BLOCK) buf0[res_pad(i)] = i < L ? __ldcg(kout + seg_lo + i) : ~K(0);
      __syncthreads();
      for (uint32_t run = warp; run * RES_RUN < len; run += Ly::WARPS) {
        K x[8];
        const uint32_t b = run * RES_RUN + lane * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = buf0[res_pad(b + i)];
        warp_sort256<K>(x);
#pragma unroll
        for (int i = 0; i < 8; ++i) buf0[res_pad(b + i)] = x[i];
      }
      __syncthreads();
      K* src = buf0;
      K* dst = buf1;
      for (uint32_t r = RES_RUN; r < len; r <<= 1) {
        if (len <= 8u * BLOCK)
          res_merge_level<K, BLOCK, 8>(src, dst, len, r);
        else
          res_merge_level<K, BLOCK, 16>(src, dst, len, r);
        __syncthreads();
        K* t = src;
        src = dst;
        dst = t;
      }
      for (uint32_t i = tid; i < L; i += BLOCK) kout[seg_lo + i] = from_ordered<K, XF>(src[res_pad(i)]);
      return finish();
    }
    // a bucket holds more than a tile: nothing was written, the LSD passes
    // below start from the keys still in registers
    zero_cnt();
    __syncthreads();
  }

  // ---- LSD passes ----------------------------------------------------------------
  bool moved = false;  // some pass has scattered: keys are no longer in input order
  uint32_t last_exec = P - 1;
  if (planned) last_exec = 31 - __clz(exec);
  for (int p = 0; p < P; ++p) {
    if (planned && !((exec >> p) & 1u)) continue;
    const int shift = p * RADIX_BITS;
    res_rank<K, IPT, true>(key, rank, IPT, wofs, tile_n, shift, !moved, wcnt, wrep);
    if (!planned) or_reduce(kor, kandn);
    __syncthreads();
    res_warp_starts<BLOCK>(sh, publisher(p, !planned));
    // (failure-path test: CTA 0 never arrives, so every other CTA's bounded
    // wait runs out and records DEV_ERR_TIMEOUT)
    if (a.test_skip_arrival && c == 0) return;
    if (!res_grid_sync(bar, ++nbar, a.timeout_ns, ctl, a.host_err, &s_ok)) return finish();
    if (!planned) {
      exec = plan_of();
      planned = true;
      if (exec == 0) {  // every key equal: the output is the input
        if (a.kout != a.kin) {
#pragma unroll
          for (int k = 0; k < IPT; ++k) {
            const uint32_t li = wofs + k * 32;
            if (li < tile_n) kout[tbase + li] = from_ordered<K, XF>(key[k]);
          }
        }
        return finish();
      }
      last_exec = 31 - __clz(exec);
      if (!((exec >> p) & 1u)) {  // this digit never varies: nothing moves in this pass
        zero_cnt();
        __syncthreads();
        continue;
      }
    }
    res_offsets<BLOCK, Ly::MAXG, Ly::MAXW>(sh, grp, a.counts, a.groups, p);
    res_scatter<K, XF, BLOCK, IPT, Ly::STAGE_KEYS, true>(sh, stage, key, rank, wofs, tile_n, shift, kout, n,
                                                          (uint32_t)p == last_exec, ctl);
    moved = true;
    if ((uint32_t)p == last_exec) break;
    zero_cnt();
    if (!res_grid_sync(bar, ++nbar, a.timeout_ns, ctl, a.host_err, &s_ok)) return finish();
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const uint32_t li = wofs + k * 32;
      key[k] = li < tile_n ? __ldcg(kout + tbase + li) : K(0);
    }
  }
  finish();
}

}  // namespace fs
