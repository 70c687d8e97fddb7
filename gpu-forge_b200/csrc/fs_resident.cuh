// fs_resident.cuh -- a whole keys-only LSD radix sort in one cooperative
// launch with every key held in registers, for the sizes where the chained
// launches of fs_kernels.cuh cost more than their kernels (up to a few
// million keys).
//
// CTA c owns positions [c*TILE, (c+1)*TILE) of the array (TILE = BLOCK*IPT),
// one CTA per SM, all resident.  Per executed digit pass:
//   1. rank its TILE keys (registers) by the digit: per-warp counters in
//      shared memory, shared atomics for the first executed pass (keys only:
//      order among equal keys is free), owner election + five ballots after;
//   2. publish the CTA's digit counts (plain stores) and add them to its
//      16-CTA group's sums (reductions in L2);
//   3. grid barrier;
//   4. output base of each digit: the digit totals (all group sums), the
//      group sums before this CTA's group and the counts of the CTAs before it
//      in its group -- at most 7 L2 loads a thread, all issued at once;
//   5. stage the tile in digit order in shared memory, write it coalesced;
//   6. grid barrier, then load the CTA's positions of the output again.
// The passes run in place in the output array: a pass's loads all happen
// before its first barrier and its stores after it.  The first pass's OR /
// AND words give every CTA the same plan (which digits vary) after the first
// barrier, so trivial passes cost nothing and the last executed pass applies
// the inverse order transform.
//
// Measured on one B200 (globaltimer stamps per phase, 2^20 u32 keys on 147
// CTAs): a barrier built from a generation word cost 2.2-3.9 us (four
// dependent L2 round trips), and one global OR per warp made the first
// barrier 6.6 us (4704 atomics on one word).  Here a barrier is one release
// reduction on a counter that only grows within a launch (the k-th barrier
// waits for k * gridDim.x arrivals) and the OR/AND words take one atomic per
// CTA.
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

// Accumulator set (32-bit words): [passes][groups][RADIX] group sums, then
// the OR and ~AND words of the ordered keys (lo, hi each) and the barrier
// counter, padded to 16 bytes.
__host__ __device__ constexpr uint32_t res_acc_words(int passes, uint32_t groups) {
  return (uint32_t)passes * RADIX * groups + 8u;
}

struct ResArgs {
  const void* kin;
  void* kout;         // may equal kin (in place)
  uint64_t n;         // 2 .. gridDim.x * TILE
  SortCtl* ctl;       // err
  uint32_t* counts;   // [passes][gridDim.x][RADIX], plain stores
  uint32_t* acc;      // this launch's accumulator set (zero on entry)
  uint32_t* acc_next; // the next launch's set: cleared here
  uint32_t acc_words; // words of a set (the largest layout any launch uses)
  uint32_t groups;    // group sums per pass in a set (>= ceil(gridDim.x / RES_GROUP))
  uint64_t timeout_ns;
  int* host_err;      // mapped page-locked word the host reads after the sort
  int test_skip_arrival;  // failure-path test: CTA 0 leaves before the first barrier
};

template <typename K, int BLOCK, int IPT>
struct ResLayout {
  static constexpr int WARPS = BLOCK / 32;
  static constexpr int TILE = BLOCK * IPT;
  static constexpr int SEG = 32 * IPT;
  static constexpr int Q = BLOCK / RADIX;  // threads per digit in the per-digit phases
  static constexpr int MAXG = ((RES_MAX_CTAS + RES_GROUP - 1) / RES_GROUP + Q - 1) / Q;  // group loads a thread
  static constexpr int MAXW = (RES_GROUP - 1 + Q - 1) / Q;  // in-group count loads a thread
  // dynamic shared memory: [warp digit counters | warp digit owners | staged keys]
  static constexpr size_t CNT_OFF = 0;
  static constexpr size_t REP_OFF = CNT_OFF + (size_t)WARPS * RADIX * 4;
  static constexpr size_t STAGE_OFF = REP_OFF + (size_t)WARPS * RADIX;
  static constexpr size_t BYTES = STAGE_OFF + (size_t)TILE * sizeof(K);
  static_assert(BLOCK % RADIX == 0 && WARPS % Q == 0, "whole warps per digit-thread group");
  static_assert(STAGE_OFF % 16 == 0, "staging alignment");
};

template <typename K, int XF, int BLOCK, int IPT>
__global__ void __launch_bounds__(BLOCK, 1) k_resident_sort(const ResArgs a) {
  using Ly = ResLayout<K, BLOCK, IPT>;
  constexpr int P = (int)sizeof(K);
  constexpr int Q = Ly::Q;
  constexpr int WPQ = Ly::WARPS / Q;  // warps per digit-thread group
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ uint32_t s_q[Q][RADIX];    // per-group partial sums
  __shared__ uint32_t s_q2[Q][RADIX];   // per-group partial digit totals
  __shared__ uint32_t s_tpart[RADIX];   // tile-local digit start within its warp of digits
  __shared__ uint32_t s_tstart[RADIX];  // tile-local start of each digit
  __shared__ uint32_t s_off[RADIX];     // global position - staging index, per digit
  __shared__ uint32_t s_wsum[RADIX / 32];
  __shared__ uint32_t s_or[4];
  __shared__ int s_ok;

  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const uint32_t c = blockIdx.x, G = gridDim.x;
  const uint64_t n = a.n;
  const uint64_t tbase = (uint64_t)c * Ly::TILE;
  const uint32_t tile_n = n - tbase < (uint64_t)Ly::TILE ? (uint32_t)(n - tbase) : (uint32_t)Ly::TILE;
  const uint32_t wofs = warp * Ly::SEG + lane;
  uint32_t* cnt = reinterpret_cast<uint32_t*>(dsm + Ly::CNT_OFF);
  uint32_t* wcnt = cnt + warp * RADIX;
  uint8_t* wrep = dsm + Ly::REP_OFF + warp * RADIX;
  K* stage = reinterpret_cast<K*>(dsm + Ly::STAGE_OFF);
  SortCtl* ctl = a.ctl;
  uint32_t* grp = a.acc;                                   // [P][groups][RADIX]
  uint32_t* orand = a.acc + (size_t)P * a.groups * RADIX;  // or lo, or hi, ~and lo, ~and hi
  unsigned* bar = orand + 4;
  unsigned nbar = 0;
  const uint32_t d_me = tid % RADIX, q_me = tid / RADIX;
  const uint32_t g_me = c / RES_GROUP, ngrp = (G + RES_GROUP - 1) / RES_GROUP;

  auto finish = [&]() {  // hand a device-side error to the host
    if (tid == 0) {
      const int e = ld_relaxed_s32(&ctl->err);
      if (e != 0) *(volatile int*)a.host_err = e;
    }
  };

  // clear the next launch's accumulators and this CTA's counters
  for (uint32_t i = c * BLOCK + tid; i < a.acc_words; i += G * BLOCK) a.acc_next[i] = 0;
  for (int i = tid; i < Ly::WARPS * RADIX; i += BLOCK) cnt[i] = 0;
  if (tid < 4) s_or[tid] = 0;

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
  K* kout = static_cast<K*>(a.kout);
  bool moved = false;           // some pass has scattered: keys are no longer in input order
  uint32_t exec = 0xffffffffu;  // passes that run (known after the first barrier)
  uint32_t last_exec = P - 1;

  for (int p = 0; p < P; ++p) {
    if (!((exec >> p) & 1u)) continue;
    const int shift = p * RADIX_BITS;
    auto digit = [&](K k) -> uint32_t { return (uint32_t)(k >> shift) & (RADIX - 1); };

    // ---- 1. warp-local ranks ------------------------------------------------------
    if (!moved) {
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        const bool valid = (wofs + k * 32) < tile_n;
        rank.set(k, valid ? atomicAdd(&wcnt[digit(key[k])], 1u) : 0u);
      }
    } else {
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        const bool valid = (wofs + k * 32) < tile_n;
        const uint32_t d = digit(key[k]);
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
    if (p == 0) {  // which digits vary across all keys: one shared OR per warp
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
    }
    __syncthreads();

    // ---- 2. CTA digit counts, warp prefixes, tile-local digit starts -------------
    {
      uint32_t sum = 0;
#pragma unroll
      for (int w = 0; w < WPQ; ++w) sum += cnt[(q_me * WPQ + w) * RADIX + d_me];
      s_q[q_me][d_me] = sum;
    }
    __syncthreads();
    {
      uint32_t run = 0, tot = 0;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const uint32_t v = s_q[q][d_me];
        if (q < (int)q_me) run += v;
        tot += v;
      }
      // exclusive prefix over the warps, per digit
#pragma unroll
      for (int w = 0; w < WPQ; ++w) {
        uint32_t* cw = &cnt[(q_me * WPQ + w) * RADIX + d_me];
        const uint32_t v = *cw;
        *cw = run;
        run += v;
      }
      if (tid < RADIX) {
        __stcg(&a.counts[((size_t)p * G + c) * RADIX + tid], tot);
        if (tot) atomicAdd(&grp[((size_t)p * a.groups + g_me) * RADIX + tid], tot);
        // tile-local digit starts: exclusive scan of tot over the digits
        uint32_t x = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
          if ((int)lane >= o) x += y;
        }
        if (lane == 31) s_wsum[warp] = x;
        s_tpart[tid] = x - tot;
      }
      if (p == 0 && tid < 4) {
        const uint32_t v = s_or[tid];
        if (v) atomicOr(&orand[tid], v);
      }
    }
    __syncthreads();
    {  // fold the tile-local digit start into the warp prefixes
      uint32_t ts = s_tpart[d_me];
      for (uint32_t w = 0; w < (d_me >> 5); ++w) ts += s_wsum[w];
      if (q_me == 0) s_tstart[d_me] = ts;
#pragma unroll
      for (int w = 0; w < WPQ; ++w) cnt[(q_me * WPQ + w) * RADIX + d_me] += ts;
    }

    // ---- 3. grid barrier: every CTA's counts are in ------------------------------
    // (failure-path test: CTA 0 never arrives, so every other CTA's bounded
    // wait runs out and records DEV_ERR_TIMEOUT)
    if (a.test_skip_arrival && c == 0) return;
    if (!res_grid_sync(bar, ++nbar, a.timeout_ns, ctl, a.host_err, &s_ok)) return finish();

    // ---- 4. output base of each digit: loads first, the plan meanwhile -------------
    uint32_t gv[Ly::MAXG], wv[Ly::MAXW];
    {
      const uint32_t* gp = grp + (size_t)p * a.groups * RADIX + d_me;
      const uint32_t* cp = a.counts + ((size_t)p * G + g_me * RES_GROUP) * RADIX + d_me;
      const uint32_t nw = c - g_me * RES_GROUP;
#pragma unroll
      for (int i = 0; i < Ly::MAXG; ++i) {
        const uint32_t g = q_me + i * Q;
        gv[i] = g < ngrp ? __ldcg(gp + (size_t)g * RADIX) : 0u;
      }
#pragma unroll
      for (int i = 0; i < Ly::MAXW; ++i) {
        const uint32_t j = q_me + i * Q;
        wv[i] = j < nw ? __ldcg(cp + (size_t)j * RADIX) : 0u;
      }
    }
    if (p == 0) {
      const unsigned long long o = ((unsigned long long)__ldcg(&orand[1]) << 32) | __ldcg(&orand[0]);
      const unsigned long long an = ((unsigned long long)__ldcg(&orand[3]) << 32) | __ldcg(&orand[2]);
      const unsigned long long varying = o & an;
      exec = 0;
#pragma unroll
      for (int pp = 0; pp < P; ++pp)
        if ((varying >> (RADIX_BITS * pp)) & (RADIX - 1)) exec |= 1u << pp;
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
      if (!(exec & 1u)) {  // digit 0 never varies: nothing moves in this pass
        for (int i = tid; i < Ly::WARPS * RADIX; i += BLOCK) cnt[i] = 0;
        __syncthreads();
        continue;
      }
    }
    {
      uint32_t tot = 0, pre = 0;
#pragma unroll
      for (int i = 0; i < Ly::MAXG; ++i) {
        tot += gv[i];
        if (q_me + i * Q < g_me) pre += gv[i];
      }
#pragma unroll
      for (int i = 0; i < Ly::MAXW; ++i) pre += wv[i];
      s_q[q_me][d_me] = pre;
      s_q2[q_me][d_me] = tot;
    }
    __syncthreads();
    if (tid < RADIX) {
      uint32_t tot = 0, pre = 0;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        tot += s_q2[q][tid];
        pre += s_q[q][tid];
      }
      uint32_t x = tot;  // digit starts: exclusive scan of the totals
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if ((int)lane >= o) x += y;
      }
      if (lane == 31) s_wsum[warp] = x;
      s_off[tid] = x - tot + pre - s_tstart[tid];
    }

    // ---- 5. stage in digit order, write coalesced ---------------------------------
    bool oob = false;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      if ((wofs + k * 32) < tile_n) {
        const uint32_t si = wcnt[digit(key[k])] + rank.get(k);
        if (si < (uint32_t)Ly::TILE)
          stage[si] = key[k];
        else
          oob = true;
      }
    }
    __syncthreads();
    if (tid < RADIX) {
      uint32_t add = 0;
      for (uint32_t w = 0; w < (tid >> 5); ++w) add += s_wsum[w];
      s_off[tid] += add;
    }
    __syncthreads();
    const bool xout = (uint32_t)p == last_exec;
    const uint64_t lastpos = n - 1;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const uint32_t i = j * BLOCK + tid;
      if (i < tile_n) {
        const K kk = stage[i];
        const uint64_t pos = (uint64_t)s_off[digit(kk)] + i;
        if (pos <= lastpos)
          kout[pos] = xout ? from_ordered<K, XF>(kk) : kk;
        else
          oob = true;
      }
    }
    if (oob) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
    moved = true;
    if ((uint32_t)p == last_exec) break;

    // ---- 6. grid barrier, then this CTA's positions of the output again -----------
    for (int i = tid; i < Ly::WARPS * RADIX; i += BLOCK) cnt[i] = 0;
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
