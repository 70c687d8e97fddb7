// oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of forge-sort's results, used as the parity checker by
// tests/, by __graft_entry__.smoke(), and as the timed CPU baseline in
// bench.py.  The product (gpu-forge_b200/) never links or calls this.
//
// The reference (kavanaghpatrick/gpu-forge, crate metal-forge-compute/
// forge-sort) is Rust + Metal and cannot be built here (no cargo, no Metal).
// Its results are pinned by its own tests against Rust core's
// slice::sort_unstable / sort_by(f32::total_cmp) (tests/correctness_f32.rs:
// 115-212, correctness_f64.rs:110-180, src/lib.rs:3114-3143) and, for argsort
// and pairs, against a stable sort_by_key (required bit-exact here).  So:
//
//   keys     : sort the order-preserving image of each key (the bijection of
//              shaders/sort.metal:812-868, restated in to_ordered below) with
//              std::sort, map back.  Keys equal under total_cmp have equal
//              bits, so every correct sort yields this one bit pattern.
//   argsort  : std::stable_sort of indices by that image (ties by index).
//   pairs    : argsort, then gather keys and values.
//   radix    : an LSD radix sort restating the reference's GPU algorithm
//              (8-bit digits, counting sort per pass; src/lib.rs:285-592),
//              a second, independent path to the same answer.
//   par_sort : __gnu_parallel::sort, the stand-in for rayon
//              par_sort_unstable (forge-sort/benches/sort_benchmark.rs:177).
//
// Input generators restate BASELINE's seeded xorshift64 (Marsaglia 2003:
// x ^= x<<13; x ^= x>>7; x ^= x<<17; element i = state after i+1 steps from
// the seed; u32 = high half).  Because the step is linear over GF(2), the
// stream can start at any index via precomputed powers of its 64x64 bit
// matrix ("jump-ahead"), which lets OpenMP threads (and the GPU generator in
// the package) produce exactly the single sequential stream in parallel.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#include <omp.h>
#include <parallel/algorithm>

namespace {

inline uint64_t xs_step(uint64_t x) {
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  return x;
}

// jump[j][i] = column i of T^(2^j): the state reached in 2^j steps from e_i.
struct JumpTable {
  uint64_t col[64][64];
  JumpTable() {
    for (int i = 0; i < 64; ++i) col[0][i] = xs_step(1ull << i);
    for (int j = 1; j < 64; ++j)
      for (int i = 0; i < 64; ++i) col[j][i] = apply(j - 1, col[j - 1][i]);
  }
  uint64_t apply(int j, uint64_t x) const {
    uint64_t r = 0;
    while (x) {
      const int b = __builtin_ctzll(x);
      r ^= col[j][b];
      x &= x - 1;
    }
    return r;
  }
};
const JumpTable& jt() {
  static JumpTable t;
  return t;
}

// state after k steps from `seed`
uint64_t xs_jump(uint64_t seed, uint64_t k) {
  uint64_t x = seed;
  for (int j = 0; k; ++j, k >>= 1)
    if (k & 1) x = jt().apply(j, x);
  return x;
}

template <typename F>
void gen_parallel(uint64_t seed, uint64_t n, F emit) {
  // element i is produced from state after i+1 steps
#pragma omp parallel
  {
    const uint64_t nt = (uint64_t)omp_get_num_threads(), t = (uint64_t)omp_get_thread_num();
    const uint64_t lo = n * t / nt, hi = n * (t + 1) / nt;
    if (lo < hi) {
      uint64_t x = xs_jump(seed, lo);
      for (uint64_t i = lo; i < hi; ++i) {
        x = xs_step(x);
        emit(i, x);
      }
    }
  }
}

template <typename K> struct Bits;
template <> struct Bits<uint32_t> {
  using S = int32_t;
  static constexpr uint32_t SIGN = 0x80000000u;
};
template <> struct Bits<uint64_t> {
  using S = int64_t;
  static constexpr uint64_t SIGN = 0x8000000000000000ull;
};

// mode: 0 none (unsigned), 1 signed (flip sign bit), 2 float (FloatFlip)
template <typename K>
inline K to_ordered(K x, int mode) {
  if (mode == 1) return x ^ Bits<K>::SIGN;
  if (mode == 2) return (x & Bits<K>::SIGN) ? ~x : (x ^ Bits<K>::SIGN);
  return x;
}
template <typename K>
inline K from_ordered(K y, int mode) {
  if (mode == 1) return y ^ Bits<K>::SIGN;
  if (mode == 2) return (y & Bits<K>::SIGN) ? (y ^ Bits<K>::SIGN) : ~y;
  return y;
}

// dtype numbering = fs_dtype: 0 u32, 1 i32, 2 f32, 3 u64, 4 i64, 5 f64
inline int mode_of(int dtype) { return dtype % 3; }
inline bool wide(int dtype) { return dtype >= 3; }

template <typename K>
void sort_keys_t(K* k, uint64_t n, int mode) {
  for (uint64_t i = 0; i < n; ++i) k[i] = to_ordered(k[i], mode);
  std::sort(k, k + n);
  for (uint64_t i = 0; i < n; ++i) k[i] = from_ordered(k[i], mode);
}

template <typename K>
void par_sort_keys_t(K* k, uint64_t n, int mode, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
  for (uint64_t i = 0; i < n; ++i) k[i] = to_ordered(k[i], mode);
  __gnu_parallel::sort(k, k + n);
#pragma omp parallel for schedule(static)
  for (uint64_t i = 0; i < n; ++i) k[i] = from_ordered(k[i], mode);
}

template <typename K>
void argsort_t(const K* k, uint32_t* idx, uint64_t n, int mode) {
  std::vector<K> o(n);
  for (uint64_t i = 0; i < n; ++i) o[i] = to_ordered(k[i], mode);
  std::iota(idx, idx + n, 0u);
  std::stable_sort(idx, idx + n, [&](uint32_t a, uint32_t b) { return o[a] < o[b]; });
}

// Parallel stable argsort: sorting (ordered key, index) tuples with the
// index as the tie-break gives exactly the permutation of a stable
// sort_by_key, in any sort algorithm, so __gnu_parallel::sort may be used.
// 32-bit keys pack the tuple into one u64.  Lets full-size (2^24..2^28)
// argsort / pairs cases be checked bit-exactly in seconds.
template <typename K>
void par_argsort_t(const K* k, uint32_t* idx, uint64_t n, int mode, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
  if constexpr (sizeof(K) == 4) {
    std::vector<uint64_t> t(n);
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) t[i] = ((uint64_t)to_ordered(k[i], mode) << 32) | i;
    __gnu_parallel::sort(t.begin(), t.end());
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) idx[i] = (uint32_t)t[i];
  } else {
    struct KI {
      uint64_t k;
      uint32_t i;
      bool operator<(const KI& o) const { return k < o.k || (k == o.k && i < o.i); }
    };
    std::vector<KI> t(n);
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) t[i] = KI{to_ordered(k[i], mode), (uint32_t)i};
    __gnu_parallel::sort(t.begin(), t.end());
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) idx[i] = t[i].i;
  }
}

// LSD radix sort: P passes of 8-bit counting sort on the ordered image,
// payload carried.  Stable by construction.
template <typename K>
void radix_t(K* k, uint32_t* v, uint64_t n, int mode) {
  constexpr int P = sizeof(K);
  std::vector<K> a(n), b(n);
  std::vector<uint32_t> va, vb;
  if (v) {
    va.assign(v, v + n);
    vb.resize(n);
  }
  for (uint64_t i = 0; i < n; ++i) a[i] = to_ordered(k[i], mode);
  for (int p = 0; p < P; ++p) {
    uint64_t cnt[257] = {0};
    for (uint64_t i = 0; i < n; ++i) ++cnt[((a[i] >> (8 * p)) & 0xff) + 1];
    for (int d = 0; d < 256; ++d) cnt[d + 1] += cnt[d];
    for (uint64_t i = 0; i < n; ++i) {
      const uint64_t pos = cnt[(a[i] >> (8 * p)) & 0xff]++;
      b[pos] = a[i];
      if (v) vb[pos] = va[i];
    }
    a.swap(b);
    if (v) va.swap(vb);
  }
  for (uint64_t i = 0; i < n; ++i) k[i] = from_ordered(a[i], mode);
  if (v) std::memcpy(v, va.data(), n * 4);
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- generators
uint64_t orc_xs_jump(uint64_t seed, uint64_t k) { return xs_jump(seed, k); }

// Elements [start, start+n) of the u64 stream (full words).
void orc_gen_u64(uint64_t seed, uint64_t start, uint64_t n, uint64_t* out) {
  const uint64_t s0 = xs_jump(seed, start);
  gen_parallel(s0, n, [&](uint64_t i, uint64_t x) { out[i] = x; });
}

// Elements [start, start+n) of the u32 stream (high halves).
void orc_gen_u32(uint64_t seed, uint64_t start, uint64_t n, uint32_t* out) {
  const uint64_t s0 = xs_jump(seed, start);
  gen_parallel(s0, n, [&](uint64_t i, uint64_t x) { out[i] = (uint32_t)(x >> 32); });
}

// Skewed u32: element i uses word w = stream[i]; if (w & 0xffffffff) % 10 < 7
// the key is 0x40000000 + (high 20 bits of w), else the high 32 bits of w.
// (70 % of keys in one 2^20-wide range, 30 % uniform.)
void orc_gen_skew_u32(uint64_t seed, uint64_t start, uint64_t n, uint32_t* out) {
  const uint64_t s0 = xs_jump(seed, start);
  gen_parallel(s0, n, [&](uint64_t i, uint64_t w) {
    const uint32_t lo = (uint32_t)w;
    out[i] = (lo % 10u < 7u) ? 0x40000000u + (uint32_t)(w >> 44) : (uint32_t)(w >> 32);
  });
}

// f32 mix (16M config): element i uses two stream words a = s[2i], b = s[2i+1].
//   c = (a >> 32) % 100:  c < 80 -> N(0, 1e3) by Box-Muller from a, b
//                         c < 85 -> -0.0 or +0.0 (bit 0 of b)
//                         c < 90 -> -inf or +inf
//                         c < 95 -> subnormal, random sign, mantissa in [1, 2^23)
//                         else   -> small integer in [-16, 16]
void orc_gen_f32_mix(uint64_t seed, uint64_t n, uint32_t* out) {
  std::vector<uint64_t> w(2 * n);
  orc_gen_u64(seed, 0, 2 * n, w.data());
#pragma omp parallel for schedule(static)
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t a = w[2 * i], b = w[2 * i + 1];
    const uint32_t c = (uint32_t)(a >> 32) % 100u;
    uint32_t bits;
    if (c < 80) {
      const double u1 = ((double)((a & 0xffffffffull) + 1)) / 4294967297.0;  // (0,1)
      const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
      const double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
      const float f = (float)(z * 1000.0);
      std::memcpy(&bits, &f, 4);
    } else if (c < 85) {
      bits = (b & 1) ? 0x80000000u : 0u;
    } else if (c < 90) {
      bits = (b & 1) ? 0xff800000u : 0x7f800000u;
    } else if (c < 95) {
      uint32_t m = (uint32_t)(b >> 8) & 0x7fffffu;
      if (m == 0) m = 1;
      bits = ((b & 1) ? 0x80000000u : 0u) | m;
    } else {
      const float f = (float)((int)((b >> 16) % 33u) - 16);
      std::memcpy(&bits, &f, 4);
    }
    out[i] = bits;
  }
}

// f64 log-uniform magnitudes: element i uses word w = s[i]:
//   sign = bit 63, unbiased exponent = -996 + ((w >> 52) & 0x7ff) % 1992,
//   mantissa = low 52 bits.  Magnitudes span ~[1.5e-300, 6.7e299].
void orc_gen_f64_logu(uint64_t seed, uint64_t n, uint64_t* out) {
  gen_parallel(seed, n, [&](uint64_t i, uint64_t w) {
    const uint64_t sign = w & 0x8000000000000000ull;
    const uint64_t e = (uint64_t)(-996 + (int)(((w >> 52) & 0x7ff) % 1992u) + 1023);
    out[i] = sign | (e << 52) | (w & 0xfffffffffffffull);
  });
}

// Zipf(s) over `nvals` values: key = rank - 1 where P(rank = r) ~ r^-s.
// Inverse CDF (double) + binary search on u = (s[i] >> 11) * 2^-53.
void orc_gen_zipf_u32(uint64_t seed, uint64_t n, double s, uint32_t nvals, uint32_t* out) {
  std::vector<double> cdf(nvals);
  double acc = 0;
  for (uint32_t r = 1; r <= nvals; ++r) {
    acc += std::pow((double)r, -s);
    cdf[r - 1] = acc;
  }
  for (auto& c : cdf) c /= acc;
  cdf[nvals - 1] = 1.0;
  gen_parallel(seed, n, [&](uint64_t i, uint64_t w) {
    const double u = (double)(w >> 11) * (1.0 / 9007199254740992.0);
    out[i] = (uint32_t)(std::upper_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
  });
}

uint64_t orc_fnv1a64(const void* p, uint64_t bytes) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  uint64_t h = 0xcbf29ce484222325ull;
  for (uint64_t i = 0; i < bytes; ++i) {
    h ^= b[i];
    h *= 0x100000001b3ull;
  }
  return h;
}

// ---------------------------------------------------------------- transforms
uint32_t orc_to_ordered32(uint32_t x, int mode) { return to_ordered<uint32_t>(x, mode); }
uint32_t orc_from_ordered32(uint32_t y, int mode) { return from_ordered<uint32_t>(y, mode); }
uint64_t orc_to_ordered64(uint64_t x, int mode) { return to_ordered<uint64_t>(x, mode); }
uint64_t orc_from_ordered64(uint64_t y, int mode) { return from_ordered<uint64_t>(y, mode); }

// ---------------------------------------------------------------- oracles
void orc_sort_keys(int dtype, void* keys, uint64_t n) {
  if (wide(dtype))
    sort_keys_t(static_cast<uint64_t*>(keys), n, mode_of(dtype));
  else
    sort_keys_t(static_cast<uint32_t*>(keys), n, mode_of(dtype));
}

void orc_par_sort_keys(int dtype, void* keys, uint64_t n, int threads) {
  if (wide(dtype))
    par_sort_keys_t(static_cast<uint64_t*>(keys), n, mode_of(dtype), threads);
  else
    par_sort_keys_t(static_cast<uint32_t*>(keys), n, mode_of(dtype), threads);
}

void orc_argsort(int dtype, const void* keys, uint32_t* idx, uint64_t n) {
  if (wide(dtype))
    argsort_t(static_cast<const uint64_t*>(keys), idx, n, mode_of(dtype));
  else
    argsort_t(static_cast<const uint32_t*>(keys), idx, n, mode_of(dtype));
}

void orc_sort_pairs(int dtype, void* keys, uint32_t* vals, uint64_t n) {
  std::vector<uint32_t> idx(n), v(vals, vals + n);
  orc_argsort(dtype, keys, idx.data(), n);
  if (wide(dtype)) {
    uint64_t* k = static_cast<uint64_t*>(keys);
    std::vector<uint64_t> kk(k, k + n);
    for (uint64_t i = 0; i < n; ++i) {
      k[i] = kk[idx[i]];
      vals[i] = v[idx[i]];
    }
  } else {
    uint32_t* k = static_cast<uint32_t*>(keys);
    std::vector<uint32_t> kk(k, k + n);
    for (uint64_t i = 0; i < n; ++i) {
      k[i] = kk[idx[i]];
      vals[i] = v[idx[i]];
    }
  }
}

void orc_par_argsort(int dtype, const void* keys, uint32_t* idx, uint64_t n, int threads) {
  if (wide(dtype))
    par_argsort_t(static_cast<const uint64_t*>(keys), idx, n, mode_of(dtype), threads);
  else
    par_argsort_t(static_cast<const uint32_t*>(keys), idx, n, mode_of(dtype), threads);
}

// Stable pairs sort through the parallel argsort, then a parallel gather.
void orc_par_sort_pairs(int dtype, void* keys, uint32_t* vals, uint64_t n, int threads) {
  std::vector<uint32_t> idx(n), v(vals, vals + n);
  orc_par_argsort(dtype, keys, idx.data(), n, threads);
  if (wide(dtype)) {
    uint64_t* k = static_cast<uint64_t*>(keys);
    std::vector<uint64_t> kk(k, k + n);
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) {
      k[i] = kk[idx[i]];
      vals[i] = v[idx[i]];
    }
  } else {
    uint32_t* k = static_cast<uint32_t*>(keys);
    std::vector<uint32_t> kk(k, k + n);
#pragma omp parallel for schedule(static)
    for (uint64_t i = 0; i < n; ++i) {
      k[i] = kk[idx[i]];
      vals[i] = v[idx[i]];
    }
  }
}

// vals may be NULL (keys only)
void orc_radix_sort(int dtype, void* keys, uint32_t* vals, uint64_t n) {
  if (wide(dtype))
    radix_t(static_cast<uint64_t*>(keys), vals, n, mode_of(dtype));
  else
    radix_t(static_cast<uint32_t*>(keys), vals, n, mode_of(dtype));
}

int orc_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
