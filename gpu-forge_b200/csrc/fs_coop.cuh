// fs_coop.cuh -- a whole keys-only radix sort in one cooperative launch, for
// sizes where the 2 + 3P launches of the chained sort (fs_kernels.cuh) cost
// more than their kernels.  Measured on one B200, it wins for 32-bit keys up
// to 2^19 (58-65 us against 75 us a call) and loses beyond and for 64-bit
// keys, where a pass of one tile per CTA plus two grid barriers costs more
// than a chained pass; the sorter uses it only where it wins.
//
// One CTA per slice, every CTA resident at once (cooperative launch).  The
// phases of the chained sort run back to back inside the kernel, separated by
// a grid barrier instead of a kernel boundary:
//   count digit 0 + OR/AND of the ordered keys       | barrier
//   per executed pass i (digit p):
//     [i > 0 or p > 0: count digit p of the input    | barrier]
//     output offsets of this CTA's slice, from the digit totals, the partial
//     sums of 16-slice groups and the counts of the slices before it in its
//     group (at most 16 + 15 loads per digit, no scan kernel)
//     scatter the slice tile by tile (scatter_tile; the first executed pass
//     ranks with shared atomics, the others stably)  | barrier
//   copy-back when an in-place sort ended in the scratch buffer.
// Every CTA derives the same pass plan from the OR/AND words, so no plan
// phase is needed.  The grid barrier's wait is bounded: on timeout the
// waiting CTA records DEV_ERR_TIMEOUT (device word and the host's mapped
// error word) and returns.
#pragma once

#include "fs_kernels.cuh"

namespace fs {

constexpr int COOP_GROUP = 16;  // slices per partial-sum group

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct CoopArgs {
  const void* kin;
  void* kfinal;
  void* kother;   // n keys of scratch (never kfinal)
  uint64_t n;
  SortCtl* ctl;
  uint32_t* counts;  // [slices][RADIX]
  uint32_t* grp;     // [MAX_PASSES][groups][RADIX], zeroed before the launch
  Slices sl;
  uint32_t groups;
  uint64_t timeout_ns;
  int* host_err;  // mapped page-locked word the host reads after the sort
};

// Bounded grid barrier (all CTAs of the cooperative launch).  Thread 0 of each
// CTA publishes the CTA's writes (fence), arrives, and waits for the
// generation to change; the last to arrive resets the count and advances the
// generation.  false: the wait ran out (error recorded).
__device__ __forceinline__ bool coop_grid_sync(const CoopArgs& a, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    SortCtl* ctl = a.ctl;
    const unsigned gen = ld_acquire_u32(&ctl->bar_gen);
    __threadfence();
    if (atomicAdd(&ctl->bar_count, 1u) + 1 == gridDim.x) {
      atomicExch(&ctl->bar_count, 0u);
      st_release_u32(&ctl->bar_gen, gen + 1);
    } else {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_u32(&ctl->bar_gen) != gen) break;
        if ((i & 63u) == 0 && global_timer_ns() - t0 > a.timeout_ns) {
          atomicCAS(&ctl->err, 0, DEV_ERR_TIMEOUT);
          *(volatile int*)a.host_err = DEV_ERR_TIMEOUT;
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    *s_ok = ok && ld_relaxed_s32(&ctl->err) == 0;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Slice histogram of digit `shift` of keys [lo, hi) into counts[c][*], the
// group partial sums and the digit totals.  `xf`: the keys are the caller's
// (forward transform first).  Loads bypass L1: the input was written by other
// CTAs in the previous phase.
template <typename K, int XF, int BLOCK>
__device__ __forceinline__ void coop_count(const CoopArgs& a, const K* keys, bool xf, int pass, uint32_t c,
                                           uint64_t lo, uint64_t hi, uint32_t (*hw)[RADIX], bool orand,
                                           K& kor, K& kandn) {
  constexpr int WARPS = BLOCK / 32;
  uint32_t* h = hw[threadIdx.x >> 5];
  const RadixDigit dg{pass * RADIX_BITS};
  for (uint64_t i = lo + threadIdx.x; i < hi; i += BLOCK) {
    K x = __ldcg(keys + i);
    if (xf) x = to_ordered<K, XF>(x);
    if (orand) {
      kor |= x;
      kandn |= ~x;
    }
    atomicAdd(&h[dg(x, 0ull)], 1u);
  }
  __syncthreads();
  uint32_t* grp = a.grp + ((size_t)pass * a.groups + c / COOP_GROUP) * RADIX;
  for (int b = threadIdx.x; b < RADIX; b += BLOCK) {
    uint32_t v = 0;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      v += hw[w][b];
      hw[w][b] = 0;
    }
    a.counts[(size_t)c * RADIX + b] = v;
    if (v) {
      atomicAdd(&grp[b], v);
      atomicAdd(&a.ctl->hist[pass][b], (unsigned long long)v);
    }
  }
}

template <typename K, int XF, int BLOCK, int IPT>
__global__ void __launch_bounds__(BLOCK, 1) k_coop_sort(const CoopArgs a) {
  using Ly = ScatterLayout<K, false, BLOCK, IPT, false, RADIX>;
  constexpr int WARPS = BLOCK / 32;
  constexpr int P = (int)sizeof(K);
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ uint32_t hw[WARPS][RADIX];
  __shared__ uint32_t s_run[RADIX];
  __shared__ uint32_t s_off[RADIX];
  __shared__ uint32_t s_wsum[RADIX / 32 > WARPS ? RADIX / 32 : WARPS];
  __shared__ int s_ok;
  const uint32_t tid = threadIdx.x, c = blockIdx.x;
  const uint64_t n = a.n;
  const uint64_t lo = (uint64_t)c * a.sl.keys_per_slice;
  const uint64_t hi = lo + a.sl.keys_per_slice < n ? lo + a.sl.keys_per_slice : n;
  SortCtl* ctl = a.ctl;

  for (int i = tid; i < WARPS * RADIX; i += BLOCK) (&hw[0][0])[i] = 0;
  uint32_t* cnt = reinterpret_cast<uint32_t*>(dsm + Ly::CNT_OFF);
  for (int i = tid; i < Ly::WARPS * RADIX; i += BLOCK) cnt[i] = 0;
  __syncthreads();

  auto finish = [&]() {  // hand a device-side error to the host
    if (tid == 0) {
      const int e = ld_relaxed_s32(&ctl->err);
      if (e != 0) *(volatile int*)a.host_err = e;
    }
  };

  // ---- count digit 0 and which digits vary -------------------------------
  {
    K kor = 0, kandn = 0;
    coop_count<K, XF, BLOCK>(a, static_cast<const K*>(a.kin), XF != XF_NONE, 0, c, lo, hi, hw, true, kor, kandn);
    uint32_t lo_or = __reduce_or_sync(0xffffffffu, (uint32_t)kor);
    uint32_t lo_an = __reduce_or_sync(0xffffffffu, (uint32_t)kandn);
    uint32_t hi_or = 0, hi_an = 0xffffffffu;
    if constexpr (sizeof(K) == 8) {
      hi_or = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kor >> 32));
      hi_an = __reduce_or_sync(0xffffffffu, (uint32_t)((uint64_t)kandn >> 32));
    }
    if ((tid & 31) == 0) {
      atomicOr(&ctl->kor, ((unsigned long long)hi_or << 32) | lo_or);
      atomicOr(&ctl->kandn, ((unsigned long long)hi_an << 32) | lo_an);
    }
  }
  if (!coop_grid_sync(a, &s_ok)) return finish();

  // ---- plan: the same on every CTA ---------------------------------------
  const unsigned long long varying = __ldcg(&ctl->kor) & __ldcg(&ctl->kandn);
  uint32_t exec = 0;
  int m = 0;
#pragma unroll
  for (int p = 0; p < P; ++p)
    if ((varying >> (RADIX_BITS * p)) & (RADIX - 1)) {
      exec |= 1u << p;
      ++m;
    }
  const bool inplace = a.kin == a.kfinal;
  // executed passes alternate FINAL / OTHER; an in-place sort starts in
  // OTHER (pass 1 may not write what it reads) and, with an odd count,
  // ends there and copies back
  bool slot_final = inplace ? false : (m & 1) != 0;
  const void* kprev = a.kin;
  int i = 0;
  for (int p = 0; p < P; ++p) {
    if (!(exec & (1u << p))) continue;
    const K* kin = static_cast<const K*>(kprev);
    K* kout = static_cast<K*>(slot_final ? a.kfinal : a.kother);
    if (i > 0 || p > 0) {  // digit 0 of the caller's keys was counted above
      K unused0 = 0, unused1 = 0;
      coop_count<K, XF, BLOCK>(a, kin, i == 0 && XF != XF_NONE, p, c, lo, hi, hw, false, unused0, unused1);
      if (!coop_grid_sync(a, &s_ok)) return finish();
    }
    // output offsets of this slice: digit base + groups before + slices
    // before it in its group
    {
      const uint32_t d = tid;  // BLOCK == RADIX
      const uint32_t t = (uint32_t)__ldcg(&ctl->hist[p][d]);
      uint32_t x = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if ((int)(d & 31) >= o) x += y;
      }
      if ((d & 31) == 31) s_wsum[d >> 5] = x;
      __syncthreads();
      uint32_t run = x - t;
      for (uint32_t w = 0; w < (d >> 5); ++w) run += s_wsum[w];
      const uint32_t g = c / COOP_GROUP;
      const uint32_t* grp = a.grp + (size_t)p * a.groups * RADIX;
      for (uint32_t gg = 0; gg < g; ++gg) run += __ldcg(&grp[(size_t)gg * RADIX + d]);
      for (uint32_t cc = g * COOP_GROUP; cc < c; ++cc) run += __ldcg(&a.counts[(size_t)cc * RADIX + d]);
      s_run[d] = run;
      __syncthreads();
    }
    uint32_t flags = PD_EXEC | PD_WRITE_KEYS;
    if (i == 0) flags |= PD_XF_IN | PD_FIRST;
    if (i == m - 1) flags |= PD_XF_OUT;
    const RadixDigit dg{p * RADIX_BITS};
    for (uint64_t t0 = lo; t0 < hi; t0 += Ly::TILE) {
      const uint32_t tile_n = hi - t0 < (uint64_t)Ly::TILE ? (uint32_t)(hi - t0) : (uint32_t)Ly::TILE;
      if (tile_n == (uint32_t)Ly::TILE) {
        if (i == 0)
          scatter_tile<K, false, XF, BLOCK, IPT, true, false, true>(t0, tile_n, n, flags, kin, kout, nullptr, nullptr,
                                                                   dsm, dsm, s_run, s_off, s_wsum, ctl, dg, 0ull,
                                                                   nullptr, nullptr, nullptr);
        else
          scatter_tile<K, false, XF, BLOCK, IPT, true, false, false>(t0, tile_n, n, flags, kin, kout, nullptr,
                                                                    nullptr, dsm, dsm, s_run, s_off, s_wsum, ctl, dg,
                                                                    0ull, nullptr, nullptr, nullptr);
      } else {
        if (i == 0)
          scatter_tile<K, false, XF, BLOCK, IPT, false, false, true>(t0, tile_n, n, flags, kin, kout, nullptr,
                                                                    nullptr, dsm, dsm, s_run, s_off, s_wsum, ctl, dg,
                                                                    0ull, nullptr, nullptr, nullptr);
        else
          scatter_tile<K, false, XF, BLOCK, IPT, false, false, false>(t0, tile_n, n, flags, kin, kout, nullptr,
                                                                     nullptr, dsm, dsm, s_run, s_off, s_wsum, ctl, dg,
                                                                     0ull, nullptr, nullptr, nullptr);
      }
    }
    if (!coop_grid_sync(a, &s_ok)) return finish();
    kprev = kout;
    slot_final = !slot_final;
    ++i;
  }

  // ---- result where the caller wants it -----------------------------------
  const K* src = nullptr;
  if (m > 0 && kprev != a.kfinal) src = static_cast<const K*>(kprev);  // ended in OTHER
  if (m == 0 && !inplace) src = static_cast<const K*>(a.kin);          // nothing to sort: copy
  if (src) {
    K* dst = static_cast<K*>(a.kfinal);
    for (uint64_t j = lo + tid; j < hi; j += BLOCK) dst[j] = __ldcg(src + j);
  }
  finish();
}

}  // namespace fs
