// fs_kernels.cuh -- the sm_100a kernels of one sort:
//
//   k_upfront_hist   one read of the keys -> histograms of ALL digit passes
//   k_plan           exclusive bucket starts per pass, trivial-pass detection,
//                    device-side pass/buffer plan (1 CTA)
//   k_onesweep       one stable 8-bit LSD pass: warp-multisplit rank,
//                    decoupled lookback across tiles, shared-memory staging by
//                    digit, coalesced scatter; payload carried alongside
//   k_finalize       copy-back / iota when the plan needs it; error hand-off
//
// They replace the reference pipeline sort_msd_histogram -> sort_msd_prep ->
// sort_msd_atomic_scatter -> sort_inner_fused (+ sort_transform_*,
// sort_init_indices, sort_gather_values) in forge-sort shaders/sort.metal.
#pragma once

#include "fs_device.cuh"

#ifndef FS_ONESWEEP_MIN_BLOCKS
#define FS_ONESWEEP_MIN_BLOCKS 3
#endif

namespace fs {

// --------------------------------------------------------------------------
// Upfront histogram: every digit of every pass from one read of the keys.
// Replaces sort_msd_histogram (shaders/sort.metal:64-142), which counted only
// the most significant byte, and the per-bucket histograms that
// sort_inner_fused recomputed (sort.metal:378-769).
//
// Per key: P shared-memory increments.  When a whole warp shares the digit of
// a pass (skewed keys: small integers, Zipf, all-equal), lane 0 adds the warp
// count once instead of 32 conflicting atomics; the test costs one shuffle
// and one warp OR-reduction per key.
// --------------------------------------------------------------------------
template <typename K, int XF, int BLOCK>
__global__ void __launch_bounds__(BLOCK)
    k_upfront_hist(const K* __restrict__ keys, uint64_t n, SortCtl* __restrict__ ctl) {
  constexpr int P = (int)sizeof(K);
  __shared__ uint32_t h[P][RADIX];
  for (int i = threadIdx.x; i < P * RADIX; i += BLOCK) (&h[0][0])[i] = 0;
  __syncthreads();

  const uint32_t lane = threadIdx.x & 31;
  auto count = [&](K x, bool valid) {
    x = to_ordered<K, XF>(x);
    const uint32_t active = __ballot_sync(0xffffffffu, valid);
    if (!valid) return;
    // bits in which some active lane differs from the first active lane
    const int src = __ffs(active) - 1;
    const K x0 = __shfl_sync(active, x, src);
    const K diff = x ^ x0;
    uint32_t dlo = __reduce_or_sync(active, (uint32_t)diff);
    uint32_t dhi = 0;
    if constexpr (sizeof(K) == 8) dhi = __reduce_or_sync(active, (uint32_t)((uint64_t)diff >> 32));
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint32_t dbyte = (p < 4 ? (dlo >> (8 * p)) : (dhi >> (8 * (p - 4)))) & 0xffu;
      const uint32_t d = digit_of(x, RADIX_BITS * p);
      if (dbyte) {
        atomicAdd(&h[p][d], 1u);
      } else if (lane == (uint32_t)src) {
        atomicAdd(&h[p][d], (uint32_t)__popc(active));
      }
    }
  };

  // Loop bounds are tested on the warp's first index (the stride is a
  // multiple of 32), so whole warps iterate together and the warp-wide
  // shuffles and reductions above stay converged.
  const uint64_t stride = (uint64_t)gridDim.x * BLOCK;
  uint64_t wb = (uint64_t)blockIdx.x * BLOCK + (threadIdx.x & ~31u);
  // 4 independent loads in flight per thread
  for (; wb + 3 * stride + 32 <= n; wb += 4 * stride) {
    const uint64_t j = wb + lane;
    const K x0 = keys[j], x1 = keys[j + stride], x2 = keys[j + 2 * stride], x3 = keys[j + 3 * stride];
    count(x0, true);
    count(x1, true);
    count(x2, true);
    count(x3, true);
  }
  for (; wb < n; wb += stride) {
    const uint64_t j = wb + lane;
    const bool valid = j < n;
    count(valid ? keys[j] : K(0), valid);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < P * RADIX; b += BLOCK) {
    const uint32_t c = (&h[0][0])[b];
    if (c) atomicAdd(&(&ctl->hist[0][0])[b], (unsigned long long)c);
  }
}

// --------------------------------------------------------------------------
// Plan: per pass, exclusive scan of the digit counts -> global bucket starts;
// a pass in which one digit holds all n keys is the identity permutation and
// is skipped.  Then thread 0 routes the executed passes through the key and
// payload buffers so that the result lands where the caller wants it.
// Replaces sort_msd_prep (shaders/sort.metal:153-181).  Also zeroes the
// histogram and the tile counters for the next sort.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(RADIX) k_plan(SortCtl* __restrict__ ctl, PlanArgs a,
                                                uint32_t first_tile) {
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  __shared__ unsigned long long s_wsum[RADIX / 32];
  __shared__ int s_exec[MAX_PASSES];
  for (int p = 0; p < a.passes; ++p) {
    const unsigned long long c = ctl->hist[p][d];
    ctl->hist[p][d] = 0ull;
    unsigned long long x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_wsum[warp] = x;
    const int trivial = __syncthreads_or(c == a.n);
    unsigned long long pre = 0;
    for (int w = 0; w < warp; ++w) pre += s_wsum[w];
    ctl->base[p][d] = pre + x - c;
    if (d == 0) s_exec[p] = !trivial;
    __syncthreads();
  }
  if (d < MAX_PASSES) ctl->tile_counter[d] = first_tile;
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
      if (i == 1) f |= PD_XF_IN;
      if (i == 1 && a.has_vals && a.vin == nullptr) f |= PD_SYNTH_IDX;
      if (i == m) f |= PD_XF_OUT;
      if (a.write_keys || i < m) f |= PD_WRITE_KEYS;
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
// One stable LSD pass over digit `pass` (bits 8*pass .. 8*pass+7).
//
// Tile = BLOCK*IPT keys; warp w owns the contiguous segment
// [w*32*IPT, (w+1)*32*IPT) and holds item k of lane l at k*32 + l, so ranking
// items in (k, lane) order IS input order -> the pass is stable, which argsort
// and pairs need (the reference's atomic MSD scatter was not:
// shaders/sort.metal:267-283).
//
//   1. tile id from an atomic counter (so every tile we wait on is running)
//   2. coalesced load (+ forward transform on the first executed pass;
//      + index synthesis for argsort)
//   3. warp multisplit rank: __match_any_sync groups equal digits; the
//      highest lane of each group bumps the warp's shared counter
//   4. per digit: warp prefix, tile count, publish AGGREGATE, exclusive scan
//   5. decoupled lookback over earlier tiles' status words (bounded wait)
//   6. stage keys (and payload) in shared memory in digit order
//   7. coalesced scatter: consecutive staged keys of one digit go to
//      consecutive global positions (+ inverse transform on the last pass)
// --------------------------------------------------------------------------
template <typename K, bool VALS, int BLOCK, int IPT>
struct OnesweepCfg {
  static constexpr int WARPS = BLOCK / 32;
  static constexpr int TILE = BLOCK * IPT;
  static constexpr int SEG = 32 * IPT;
  static constexpr size_t STAGE_BYTES = (size_t)TILE * sizeof(K) + (VALS ? (size_t)TILE * 4 : 0);
  static constexpr size_t HIST_BYTES = (size_t)WARPS * RADIX * 4;
  static constexpr size_t DYN_SMEM = STAGE_BYTES > HIST_BYTES ? STAGE_BYTES : HIST_BYTES;
  static_assert(BLOCK >= RADIX && BLOCK % 32 == 0, "one thread per digit needed");
};

template <typename K, bool VALS, int XF, int BLOCK, int IPT, bool FULL>
__device__ __forceinline__ bool onesweep_tile(
    const uint32_t tile, const uint32_t tile_n, const uint64_t n, const int pass, const uint32_t flags,
    const K* __restrict__ kin, K* __restrict__ kout, const uint32_t* __restrict__ vin,
    uint32_t* __restrict__ vout, SortCtl* __restrict__ ctl, uint64_t* __restrict__ status,
    const uint32_t epoch, const uint64_t timeout_ns, uint32_t* whist, K* skeys, uint32_t* svals,
    uint32_t* s_start, uint32_t* s_off, uint32_t* s_wsum, int* s_abort) {
  using C = OnesweepCfg<K, VALS, BLOCK, IPT>;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int shift = pass * RADIX_BITS;
  const uint64_t tbase = (uint64_t)tile * C::TILE;
  const uint32_t wofs = warp * C::SEG + lane;

  // ---- 2. load -------------------------------------------------------------
  K key[IPT];
  uint32_t val[VALS ? IPT : 1];
  uint32_t rk[IPT];
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const uint32_t li = wofs + k * 32;
    key[k] = (FULL || li < tile_n) ? kin[tbase + li] : K(0);
  }
  if constexpr (XF != XF_NONE) {
    if (flags & PD_XF_IN) {
#pragma unroll
      for (int k = 0; k < IPT; ++k) key[k] = to_ordered<K, XF>(key[k]);
    }
  }
  if constexpr (VALS) {
    if (flags & PD_SYNTH_IDX) {
#pragma unroll
      for (int k = 0; k < IPT; ++k) val[k] = (uint32_t)(tbase + wofs + k * 32);
    } else {
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        const uint32_t li = wofs + k * 32;
        val[k] = (FULL || li < tile_n) ? vin[tbase + li] : 0u;
      }
    }
  }

  // ---- 3. warp multisplit rank --------------------------------------------
  uint32_t* wh = whist + warp * RADIX;
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const bool valid = FULL || (wofs + k * 32) < tile_n;
    const uint32_t d = digit_of(key[k], shift);
    const uint32_t peers = __match_any_sync(0xffffffffu, valid ? d : 0xffffffffu);
    uint32_t old = 0;
    if (valid) old = wh[d];
    __syncwarp();
    if (valid && lane == 31u - __clz(peers)) wh[d] = old + __popc(peers);
    __syncwarp();
    rk[k] = old + __popc(peers & lt_mask);
  }
  __syncthreads();

  // ---- 4. per-digit totals, warp prefixes, publish aggregate, scan ----------
  uint32_t cnt = 0;
  if (tid < RADIX) {
#pragma unroll
    for (int w = 0; w < C::WARPS; ++w) {
      const uint32_t c = whist[w * RADIX + tid];
      whist[w * RADIX + tid] = cnt;
      cnt += c;
    }
    st_relaxed_u64(status + (uint64_t)tile * RADIX + tid,
                   st_pack(epoch, tile ? ST_AGGREGATE : ST_INCLUSIVE, cnt));
  }
  uint32_t x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if ((int)lane >= o) x += y;
  }
  if (lane == 31 && tid < RADIX) s_wsum[warp] = x;
  __syncthreads();

  // ---- 5. decoupled lookback (one thread per digit) ------------------------
  if (tid < RADIX) {
    uint32_t pre = 0;
    for (uint32_t w = 0; w < warp; ++w) pre += s_wsum[w];
    const uint32_t start = pre + x - cnt;
    s_start[tid] = start;
    uint64_t excl = 0;
    bool ok = true;
    if (tile > 0) {
      const uint64_t* sp = status + (uint64_t)(tile - 1) * RADIX + tid;
      const uint32_t ep = epoch & ST_EPOCH_MASK;
      uint64_t t0 = 0;
      for (;;) {
        const uint64_t w = ld_relaxed_u64(sp);
        const uint32_t f = st_flag(w);
        if (f != ST_NOT_READY && st_epoch(w) == ep) {
          excl += st_value(w);
          if (f == ST_INCLUSIVE) break;
          sp -= RADIX;  // tile 0 always publishes INCLUSIVE, so this stops
        } else {
          const uint64_t now = global_timer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > timeout_ns || ld_relaxed_s32(&ctl->err) != 0) {
            if (atomicCAS(&ctl->err, 0, DEV_ERR_TIMEOUT) == 0) ctl->err_tile = tile;
            ok = false;
            break;
          }
        }
      }
      if (ok)
        st_relaxed_u64(status + (uint64_t)tile * RADIX + tid,
                       st_pack(epoch, ST_INCLUSIVE, excl + cnt));
    }
    if (!ok) *s_abort = 1;
    s_off[tid] = (uint32_t)(ctl->base[pass][tid] + excl) - start;
  }
  __syncthreads();
  if (*s_abort) return false;

  // ---- 6. stage in digit order ---------------------------------------------
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    if (FULL || (wofs + k * 32) < tile_n) {
      const uint32_t d = digit_of(key[k], shift);
      rk[k] += s_start[d] + wh[d];
    }
  }
  __syncthreads();  // whist and the staging area share memory
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    if (FULL || (wofs + k * 32) < tile_n) {
      skeys[rk[k]] = key[k];
      if constexpr (VALS) svals[rk[k]] = val[k];
    }
  }
  __syncthreads();

  // ---- 7. coalesced scatter ------------------------------------------------
  // Positions are checked against n: a wrong bucket offset records
  // DEV_ERR_BOUNDS and drops the write instead of touching foreign memory.
  const bool wkeys = (flags & PD_WRITE_KEYS) != 0;
  const bool xout = XF != XF_NONE && (flags & PD_XF_OUT);
  bool oob = false;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t i = j * BLOCK + tid;
    if (FULL || i < tile_n) {
      const K kk = skeys[i];
      const uint32_t pos = s_off[digit_of(kk, shift)] + i;
      if ((uint64_t)pos < n) {
        if (wkeys) kout[pos] = xout ? from_ordered<K, XF>(kk) : kk;
        if constexpr (VALS) vout[pos] = svals[i];
      } else {
        oob = true;
      }
    }
  }
  if (oob) atomicCAS(&ctl->err, 0, DEV_ERR_BOUNDS);
  __syncthreads();  // staging reads done before the next tile reuses smem
  return true;
}

template <typename K, bool VALS, int XF, int BLOCK, int IPT>
__global__ void __launch_bounds__(BLOCK, FS_ONESWEEP_MIN_BLOCKS)
    k_onesweep(SortCtl* __restrict__ ctl, const int pass, const uint64_t n,
               const uint32_t num_tiles, uint64_t* __restrict__ status, const uint32_t epoch,
               const uint64_t timeout_ns) {
  using C = OnesweepCfg<K, VALS, BLOCK, IPT>;
  extern __shared__ __align__(16) unsigned char dsm[];
  uint32_t* whist = reinterpret_cast<uint32_t*>(dsm);
  K* skeys = reinterpret_cast<K*>(dsm);
  uint32_t* svals = reinterpret_cast<uint32_t*>(dsm + (size_t)C::TILE * sizeof(K));
  __shared__ uint32_t s_start[RADIX];
  __shared__ uint32_t s_off[RADIX];
  __shared__ uint32_t s_wsum[C::WARPS];
  __shared__ uint32_t s_tile;
  __shared__ int s_abort;

  const PassDesc pd = ctl->pass[pass];
  if (!(pd.flags & PD_EXEC)) return;
  const K* kin = static_cast<const K*>(pd.kin);
  K* kout = static_cast<K*>(pd.kout);

  for (;;) {
    if (threadIdx.x == 0) {
      s_tile = atomicAdd(&ctl->tile_counter[pass], 1u);
      s_abort = ld_relaxed_s32(&ctl->err);
    }
    for (int i = threadIdx.x; i < C::WARPS * RADIX; i += BLOCK) whist[i] = 0;
    __syncthreads();
    const uint32_t tile = s_tile;
    if (tile >= num_tiles || s_abort) return;
    const uint64_t rem = n - (uint64_t)tile * C::TILE;
    const uint32_t tile_n = rem < (uint64_t)C::TILE ? (uint32_t)rem : (uint32_t)C::TILE;
    bool ok;
    if (tile_n == (uint32_t)C::TILE)
      ok = onesweep_tile<K, VALS, XF, BLOCK, IPT, true>(
          tile, tile_n, n, pass, pd.flags, kin, kout, pd.vin, pd.vout, ctl, status, epoch,
          timeout_ns, whist, skeys, svals, s_start, s_off, s_wsum, &s_abort);
    else
      ok = onesweep_tile<K, VALS, XF, BLOCK, IPT, false>(
          tile, tile_n, n, pass, pd.flags, kin, kout, pd.vin, pd.vout, ctl, status, epoch,
          timeout_ns, whist, skeys, svals, s_start, s_off, s_wsum, &s_abort);
    if (!ok) return;
  }
}

// --------------------------------------------------------------------------
// Finalize: copy-back for in-place sorts that ended in scratch, iota for an
// argsort whose keys were all equal; then hand any device error to the host
// (mapped pinned word; set-only, the host clears it) and re-arm ctl->err.
// --------------------------------------------------------------------------
template <typename K>
__global__ void __launch_bounds__(256)
    k_finalize(SortCtl* __restrict__ ctl, const uint64_t n, int* __restrict__ host_err) {
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
