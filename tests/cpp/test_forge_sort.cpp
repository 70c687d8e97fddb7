// C++ tests of the forge_sort.hpp mirror, following the reference's own tests
// (metal-forge-compute/forge-sort/src/lib.rs:3019-3420 unit tests and
// tests/correctness*.rs, tests/regression.rs integration tests) case for case
// where a C++ caller can meet them.
//
//   test_forge_sort --cpu   tests that need no GPU (error strings, SortKey
//                           constants, DeviceNotFound without a device)
//   test_forge_sort         everything (needs a GPU)
//
// Expected results come from std::sort / std::stable_sort with the Rust
// total_cmp order for floats, on the host.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <numeric>
#include <string>
#include <vector>

#include "forge_runtime.hpp"
#include "forge_sort.hpp"

using forge_sort::GpuSorter;
using forge_sort::SortBuffer;
using forge_sort::SortError;
using forge_sort::SortKey;

namespace {

struct Case {
  const char* name;
  bool gpu;
  std::function<void()> fn;
};
std::vector<Case>& registry() {
  static std::vector<Case> r;
  return r;
}
struct Reg {
  Reg(const char* n, bool gpu, std::function<void()> f) { registry().push_back({n, gpu, std::move(f)}); }
};
#define CPU_TEST(name) \
  void name();         \
  Reg reg_##name(#name, false, name); \
  void name()
#define GPU_TEST(name) \
  void name();         \
  Reg reg_##name(#name, true, name); \
  void name()

struct Failure {
  std::string what;
};
#define CHECK(cond)                                                                      \
  do {                                                                                   \
    if (!(cond)) throw Failure{std::string(__FILE__ ":") + std::to_string(__LINE__) + ": " #cond}; \
  } while (0)

// Rust total_cmp as an unsigned key (FloatFlip of the bits).
uint32_t total_key(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
uint64_t total_key(double x) {
  uint64_t b;
  std::memcpy(&b, &x, 8);
  return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}
template <typename T>
auto order_key(T x) {
  if constexpr (std::is_floating_point_v<T>)
    return total_key(x);
  else
    return x;
}
template <typename T>
std::vector<T> sorted_copy(std::vector<T> v) {
  std::sort(v.begin(), v.end(), [](T a, T b) { return order_key(a) < order_key(b); });
  return v;
}
template <typename T>
std::vector<uint32_t> stable_argsort(const std::vector<T>& v) {
  std::vector<uint32_t> idx(v.size());
  std::iota(idx.begin(), idx.end(), 0u);
  std::stable_sort(idx.begin(), idx.end(), [&](uint32_t a, uint32_t b) { return order_key(v[a]) < order_key(v[b]); });
  return idx;
}
template <typename T>
bool same_bits(const std::vector<T>& a, const std::vector<T>& b) {
  return a.size() == b.size() && (a.empty() || std::memcmp(a.data(), b.data(), a.size() * sizeof(T)) == 0);
}

// xorshift64 stream (seeded), for the size sweeps
struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed ? seed : 1) {}
  uint64_t next() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
  }
};
std::vector<uint32_t> random_u32(size_t n, uint64_t seed) {
  Rng r(seed);
  std::vector<uint32_t> v(n);
  for (auto& x : v) x = (uint32_t)r.next();
  return v;
}

GpuSorter make() { return GpuSorter::create(); }

// ---- lib.rs unit tests ---------------------------------------------------------
CPU_TEST(test_sort_error_display) {
  CHECK(std::string(SortError::device_not_found().what()) == "no Metal GPU device found");
  CHECK(std::string(SortError::shader_compilation("test").what()) == "shader compilation failed: test");
  CHECK(std::string(SortError::gpu_execution("timeout").what()) == "GPU execution failed: timeout");
  const SortError e = SortError::length_mismatch(10, 5);
  CHECK(std::string(e.what()) == "length mismatch: keys=10, values=5");
  CHECK(e.kind() == SortError::Kind::LengthMismatch && e.keys() == 10 && e.values() == 5);
}

CPU_TEST(test_sort_key_consts) {
  static_assert(SortKey<uint32_t>::KEY_SIZE == 4 && !SortKey<uint32_t>::NEEDS_TRANSFORM && !SortKey<uint32_t>::IS_64BIT);
  static_assert(SortKey<uint32_t>::TRANSFORM_MODE_FORWARD == 0 && SortKey<uint32_t>::TRANSFORM_MODE_INVERSE == 0);
  static_assert(SortKey<int32_t>::KEY_SIZE == 4 && SortKey<int32_t>::NEEDS_TRANSFORM && !SortKey<int32_t>::IS_64BIT);
  static_assert(SortKey<int32_t>::TRANSFORM_MODE_FORWARD == 0 && SortKey<int32_t>::TRANSFORM_MODE_INVERSE == 0);
  static_assert(SortKey<float>::KEY_SIZE == 4 && SortKey<float>::NEEDS_TRANSFORM && !SortKey<float>::IS_64BIT);
  static_assert(SortKey<float>::TRANSFORM_MODE_FORWARD == 1 && SortKey<float>::TRANSFORM_MODE_INVERSE == 2);
  static_assert(SortKey<uint64_t>::KEY_SIZE == 8 && !SortKey<uint64_t>::NEEDS_TRANSFORM && SortKey<uint64_t>::IS_64BIT);
  static_assert(SortKey<int64_t>::KEY_SIZE == 8 && SortKey<int64_t>::NEEDS_TRANSFORM && SortKey<int64_t>::IS_64BIT);
  static_assert(SortKey<int64_t>::TRANSFORM_MODE_FORWARD == 0 && SortKey<int64_t>::TRANSFORM_MODE_INVERSE == 0);
  static_assert(SortKey<double>::KEY_SIZE == 8 && SortKey<double>::NEEDS_TRANSFORM && SortKey<double>::IS_64BIT);
  static_assert(SortKey<double>::TRANSFORM_MODE_FORWARD == 1 && SortKey<double>::TRANSFORM_MODE_INVERSE == 2);
}

// Without a visible device, create() reports DeviceNotFound (not a crash).
// Runs only in --cpu mode, where the caller hides every GPU.
CPU_TEST(test_no_device_is_device_not_found) {
  try {
    GpuSorter s = make();
    CHECK(false && "a sorter was created without a device");
  } catch (const SortError& e) {
    CHECK(e.kind() == SortError::Kind::DeviceNotFound);
    CHECK(std::string(e.what()) == "no Metal GPU device found");
  }
}

// The same for the multi-GPU sorter and the forge-runtime context (this
// also compiles the MultiGpuSorter templates for a caller's key type).
CPU_TEST(test_no_device_multi_and_context) {
  try {
    forge_sort::MultiGpuSorter mg({0, 1});
    std::vector<uint64_t> z(2, 0);
    std::vector<uint32_t*> k(2, nullptr), vo(2, nullptr);
    mg.sort_pairs<uint32_t>(k, {}, z, k, vo, z);
    mg.sort<uint32_t>(k, z, k, z);
    mg.sort_u32(k, z, k, z);
    std::vector<uint64_t*> k64(2, nullptr);
    mg.sort_u64(k64, z, k64, z);
    CHECK(false && "a multi-GPU sorter was created without a device");
  } catch (const SortError& e) {
    CHECK(e.kind() == SortError::Kind::DeviceNotFound);
  }
  try {
    auto ctx = forge_runtime::ForgeContext::create();
    CHECK(false && "a context was created without a device");
  } catch (const SortError& e) {
    CHECK(e.kind() == SortError::Kind::DeviceNotFound);
  }
}

GPU_TEST(test_sort_i32_basic) {
  auto s = make();
  std::vector<int32_t> d{5, -3, 0, std::numeric_limits<int32_t>::min(), std::numeric_limits<int32_t>::max(), -1, 1};
  auto want = sorted_copy(d);
  s.sort_i32(d);
  CHECK(d == want);
}

GPU_TEST(test_sort_f32_basic) {
  auto s = make();
  const float nan = std::numeric_limits<float>::quiet_NaN(), inf = std::numeric_limits<float>::infinity();
  std::vector<float> d{1.0f, nan, -0.0f, 0.0f, -inf, -1.0f, inf, -nan};
  auto want = sorted_copy(d);
  s.sort_f32(d);
  CHECK(same_bits(d, want));
}

GPU_TEST(test_argsort_u32_basic) {
  auto s = make();
  const std::vector<uint32_t> d{30, 10, 20};
  CHECK(s.argsort_u32(d) == (std::vector<uint32_t>{1, 2, 0}));
  CHECK(d == (std::vector<uint32_t>{30, 10, 20}));
}

GPU_TEST(test_argsort_empty_and_single) {
  auto s = make();
  CHECK(s.argsort_u32(std::vector<uint32_t>{}).empty());
  CHECK(s.argsort_i32(std::vector<int32_t>{}).empty());
  CHECK(s.argsort_f32(std::vector<float>{}).empty());
  CHECK(s.argsort_u64(std::vector<uint64_t>{}).empty());
  CHECK(s.argsort_u32(std::vector<uint32_t>{42}) == (std::vector<uint32_t>{0}));
  CHECK(s.argsort_u64(std::vector<uint64_t>{42}) == (std::vector<uint32_t>{0}));
}

GPU_TEST(test_argsort_i32_f32_basic) {
  auto s = make();
  CHECK(s.argsort_i32(std::vector<int32_t>{5, -3, 0, -1, 1}) == (std::vector<uint32_t>{1, 3, 2, 4, 0}));
  const std::vector<float> f{3.0f, 1.0f, 2.0f};
  CHECK(s.argsort_f32(f) == (std::vector<uint32_t>{1, 2, 0}));
  CHECK(f == (std::vector<float>{3.0f, 1.0f, 2.0f}));
}

GPU_TEST(test_sort_pairs_basic) {
  auto s = make();
  std::vector<uint32_t> k{3, 1, 2}, v{30, 10, 20};
  s.sort_pairs_u32(k, v);
  CHECK(k == (std::vector<uint32_t>{1, 2, 3}) && v == (std::vector<uint32_t>{10, 20, 30}));
  std::vector<int32_t> ki{5, -3, 0, -1, 1};
  std::vector<uint32_t> vi{50, 30, 0, 10, 10};
  s.sort_pairs_i32(ki, vi);
  CHECK(ki == (std::vector<int32_t>{-3, -1, 0, 1, 5}) && vi == (std::vector<uint32_t>{30, 10, 0, 10, 50}));
  std::vector<float> kf{3.0f, 1.0f, 2.0f};
  std::vector<uint32_t> vf{30, 10, 20};
  s.sort_pairs_f32(kf, vf);
  CHECK(same_bits(kf, std::vector<float>{1.0f, 2.0f, 3.0f}) && vf == (std::vector<uint32_t>{10, 20, 30}));
  std::vector<uint64_t> k64{30, 10, 20};
  std::vector<uint32_t> v64{300, 100, 200};
  s.sort_pairs_u64(k64, v64);
  CHECK(k64 == (std::vector<uint64_t>{10, 20, 30}) && v64 == (std::vector<uint32_t>{100, 200, 300}));
  std::vector<int64_t> ks{5, -3, 0};
  std::vector<uint32_t> vs{50, 30, 40};
  s.sort_pairs_i64(ks, vs);
  CHECK(ks == (std::vector<int64_t>{-3, 0, 5}) && vs == (std::vector<uint32_t>{30, 40, 50}));
}

GPU_TEST(test_sort_pairs_length_mismatch) {
  auto s = make();
  std::vector<uint32_t> k{1, 2, 3}, v{10, 20};
  try {
    s.sort_pairs_u32(k, v);
    CHECK(false && "expected LengthMismatch");
  } catch (const SortError& e) {
    CHECK(e.kind() == SortError::Kind::LengthMismatch && e.keys() == 3 && e.values() == 2);
    CHECK(std::string(e.what()) == "length mismatch: keys=3, values=2");
  }
}

GPU_TEST(test_sort_pairs_empty_and_single) {
  auto s = make();
  std::vector<uint32_t> k, v;
  s.sort_pairs_u32(k, v);
  CHECK(k.empty() && v.empty());
  std::vector<uint32_t> k1{42}, v1{100};
  s.sort_pairs_u32(k1, v1);
  CHECK(k1 == (std::vector<uint32_t>{42}) && v1 == (std::vector<uint32_t>{100}));
}

GPU_TEST(test_sort_64bit_basic) {
  auto s = make();
  std::vector<uint64_t> u{std::numeric_limits<uint64_t>::max(), 0, 1, std::numeric_limits<uint64_t>::max() - 1, 42};
  s.sort_u64(u);
  CHECK(u == (std::vector<uint64_t>{0, 1, 42, std::numeric_limits<uint64_t>::max() - 1,
                                    std::numeric_limits<uint64_t>::max()}));
  std::vector<int64_t> i{5, -3, 0, std::numeric_limits<int64_t>::min(), std::numeric_limits<int64_t>::max(), -1, 1};
  auto wi = sorted_copy(i);
  s.sort_i64(i);
  CHECK(i == wi);
  const double nan = std::numeric_limits<double>::quiet_NaN(), inf = std::numeric_limits<double>::infinity();
  std::vector<double> f{1.0, nan, -0.0, 0.0, -inf, -1.0, inf};
  auto wf = sorted_copy(f);
  s.sort_f64(f);
  CHECK(same_bits(f, wf));
  std::vector<uint64_t> e, one{42};
  s.sort_u64(e);
  s.sort_u64(one);
  CHECK(e.empty() && one == (std::vector<uint64_t>{42}));
  CHECK(s.argsort_u64(std::vector<uint64_t>{30, 10, 20}) == (std::vector<uint32_t>{1, 2, 0}));
  CHECK(s.argsort_i64(std::vector<int64_t>{5, -3, 0, -1, 1}) == (std::vector<uint32_t>{1, 3, 2, 4, 0}));
  CHECK(s.argsort_f64(std::vector<double>{3.0, 1.0, 2.0}) == (std::vector<uint32_t>{1, 2, 0}));
}

// ---- tests/correctness.rs ------------------------------------------------------
GPU_TEST(test_sort_sizes) {
  auto s = make();
  for (size_t n : {1000u, 4000u, 16000u, 64000u, 256000u, 1000000u, 4000000u}) {
    auto d = random_u32(n, 42 + n);
    auto want = sorted_copy(d);
    s.sort_u32(d);
    CHECK(d == want);
  }
}

GPU_TEST(test_patterns) {
  auto s = make();
  std::vector<uint32_t> z(100000, 0), same(100000, 7), pre(100000), rev(100000);
  std::iota(pre.begin(), pre.end(), 0u);
  for (size_t i = 0; i < rev.size(); ++i) rev[i] = (uint32_t)(rev.size() - i);
  for (auto* v : {&z, &same, &pre, &rev}) {
    auto want = sorted_copy(*v);
    s.sort_u32(*v);
    CHECK(*v == want);
  }
  for (size_t n : {4097u, 100u, 1u, 0u}) {  // non-tile-aligned, sub-tile, single, empty
    auto d = random_u32(n, 7);
    auto want = sorted_copy(d);
    s.sort_u32(d);
    CHECK(d == want);
  }
}

GPU_TEST(test_sort_buffer_roundtrip) {
  auto s = make();
  auto buf = s.alloc_sort_buffer<uint32_t>(1 << 20);
  CHECK(buf.capacity() == (1u << 20) && buf.is_empty());
  auto d = random_u32(1 << 20, 9);
  buf.copy_from_slice(d);
  s.sort_buffer(buf);
  CHECK(std::equal(buf.as_slice().begin(), buf.as_slice().end(), sorted_copy(d).begin()));
  // direct write through as_mut_slice, then set_len
  auto w = buf.as_mut_slice();
  for (size_t i = 0; i < 1000; ++i) w[i] = (uint32_t)(1000 - i);
  buf.set_len(1000);
  s.sort_buffer(buf);
  std::vector<uint32_t> out(1000);
  buf.copy_to_slice(out);
  for (size_t i = 0; i < 1000; ++i) CHECK(out[i] == i + 1);
  // interleave with a slice sort (the sorter's scratch is shared)
  auto d2 = random_u32(5000, 11);
  auto want2 = sorted_copy(d2);
  s.sort_u32(d2);
  CHECK(d2 == want2);
  bool threw = false;
  try {
    buf.set_len(buf.capacity() + 1);
  } catch (const std::length_error&) {
    threw = true;
  }
  CHECK(threw);
}

GPU_TEST(test_typed_buffers) {
  auto s = make();
  auto bf = s.alloc_sort_buffer<float>(3);
  bf.copy_from_slice(std::vector<float>{2.5f, -1.0f, 0.0f});
  s.sort_f32_buffer(bf);
  CHECK(same_bits(std::vector<float>(bf.as_slice().begin(), bf.as_slice().end()),
                  std::vector<float>{-1.0f, 0.0f, 2.5f}));
  auto bi = s.alloc_sort_buffer<int64_t>(4);
  bi.copy_from_slice(std::vector<int64_t>{3, -9, 0, -1});
  s.sort_i64_buffer(bi);
  CHECK(std::vector<int64_t>(bi.as_slice().begin(), bi.as_slice().end()) == (std::vector<int64_t>{-9, -1, 0, 3}));
  auto bd = s.alloc_sort_buffer<double>(3);
  bd.copy_from_slice(std::vector<double>{1e300, -1e-300, 0.5});
  s.sort_f64_buffer(bd);
  CHECK(std::vector<double>(bd.as_slice().begin(), bd.as_slice().end()) == (std::vector<double>{-1e-300, 0.5, 1e300}));
}

GPU_TEST(test_encode_sort) {
  auto s = make();
  auto buf = s.alloc_sort_buffer<uint32_t>(100000);
  auto d = random_u32(100000, 13);
  buf.copy_from_slice(d);
  s.encode_sort(nullptr, buf);
  s.synchronize();
  CHECK(std::equal(buf.as_slice().begin(), buf.as_slice().end(), sorted_copy(d).begin()));
}

// ---- tests/correctness_argsort.rs, correctness_sort_pairs.rs ----------------------
GPU_TEST(test_argsort_stable_and_unmodified) {
  auto s = make();
  std::vector<uint32_t> d = random_u32(1 << 20, 17);
  for (auto& x : d) x &= 0xffu;  // many ties: order among equals must be the input order
  const auto copy = d;
  CHECK(s.argsort_u32(d) == stable_argsort(d));
  CHECK(d == copy);
  std::vector<float> f(200000);
  Rng r(19);
  for (auto& x : f) x = (float)((int)(r.next() % 2001) - 1000) * 0.5f;
  f[5] = std::numeric_limits<float>::quiet_NaN();
  f[6] = -0.0f;
  CHECK(s.argsort_f32(f) == stable_argsort(f));
}

GPU_TEST(test_sort_pairs_stable) {
  auto s = make();
  std::vector<uint32_t> k = random_u32(1000000, 23), v(1000000);
  for (auto& x : k) x %= 1000u;
  std::iota(v.begin(), v.end(), 0u);
  const auto idx = stable_argsort(k);
  std::vector<uint32_t> wk(k.size()), wv(k.size());
  for (size_t i = 0; i < idx.size(); ++i) {
    wk[i] = k[idx[i]];
    wv[i] = v[idx[i]];
  }
  s.sort_pairs_u32(k, v);
  CHECK(k == wk && v == wv);
}

// ---- tests/regression.rs ---------------------------------------------------------
GPU_TEST(test_cross_type_interleave) {
  auto s = make();
  for (int round = 0; round < 3; ++round) {
    auto u = random_u32(30000, 100 + round);
    std::vector<int32_t> i(u.begin(), u.end());
    std::vector<float> f(u.size());
    for (size_t j = 0; j < u.size(); ++j) f[j] = (float)(int32_t)u[j] * 1e-3f;
    std::vector<uint64_t> w(u.size());
    for (size_t j = 0; j < u.size(); ++j) w[j] = ((uint64_t)u[j] << 32) | u[(j + 1) % u.size()];
    auto wu = sorted_copy(u);
    auto wi = sorted_copy(i);
    auto wf = sorted_copy(f);
    auto ww = sorted_copy(w);
    const auto ia = stable_argsort(f);
    s.sort_u32(u);
    s.sort_i32(i);
    CHECK(s.argsort_f32(f) == ia);
    s.sort_f32(f);
    s.sort_u64(w);
    CHECK(u == wu && i == wi && same_bits(f, wf) && w == ww);
  }
}

// ---- forge-runtime (forge-runtime/src, tests/pipeline_tests.rs) --------------
CPU_TEST(test_runtime_error_display) {
  using forge_runtime::GatherError;
  using forge_runtime::PipelineError;
  CHECK(std::string(GatherError::shader_compilation("x").what()) == "shader compilation failed: x");
  CHECK(std::string(GatherError::gpu_execution("x").what()) == "GPU execution failed: x");
  CHECK(std::string(PipelineError::command_buffer().what()) == "failed to create command buffer");
  CHECK(std::string(PipelineError::encoder().what()) == "failed to create compute encoder");
  CHECK(std::string(PipelineError::sort(SortError::gpu_execution("x")).what()) == "sort error: GPU execution failed: x");
}

// pipeline_tests.rs:172-210: sort 100K keys of a SortBuffer, then gather the
// first 100 in the same pipeline.
GPU_TEST(test_pipeline_sort_then_gather_100k) {
  auto ctx = forge_runtime::ForgeContext::create();
  auto sorter = GpuSorter::with_context(ctx.device(), ctx.queue());
  auto gather = forge_runtime::GpuGather::with_context(ctx.device(), ctx.queue());
  const auto data = random_u32(100000, 7);
  auto buf = sorter.alloc_sort_buffer<uint32_t>(data.size());
  buf.copy_from_slice(data);
  auto idx = ctx.alloc_buffer(100 * 4);
  for (uint32_t i = 0; i < 100; ++i) idx.as<uint32_t>()[i] = i;
  auto out = ctx.alloc_buffer(100 * 4);
  forge_runtime::Pipeline p(ctx);
  p.sort(sorter, buf);
  p.gather(gather, buf.device_ptr(), buf.len(), idx.device_ptr(), out.device_ptr(), 100, false);
  p.execute();
  const auto want = sorted_copy(data);
  CHECK(std::equal(want.begin(), want.begin() + 100, out.as<uint32_t>()));
  CHECK(std::equal(want.begin(), want.end(), buf.as_slice().begin()));
}

GPU_TEST(test_gather_u64_and_bounds) {
  auto ctx = forge_runtime::ForgeContext::create();
  auto g = forge_runtime::GpuGather::with_context(ctx.device(), ctx.queue());
  const uint32_t n = 1 << 16;
  auto src = ctx.alloc_buffer(n * 8);
  auto idx = ctx.alloc_buffer(n * 4);
  auto out = ctx.alloc_buffer(n * 8);
  const auto r = random_u32(n, 11);
  for (uint32_t i = 0; i < n; ++i) {
    src.as<uint64_t>()[i] = ((uint64_t)r[i] << 32) | i;
    idx.as<uint32_t>()[i] = r[i] % n;
  }
  g.gather_u64(src, idx, out, n);
  for (uint32_t i = 0; i < n; ++i) CHECK(out.as<uint64_t>()[i] == src.as<uint64_t>()[idx.as<uint32_t>()[i]]);
  idx.as<uint32_t>()[5] = n;  // one index past the source
  forge_runtime::Pipeline p(ctx);
  p.gather(g, src, idx, out, n, true);
  bool threw = false;
  try {
    p.execute();
  } catch (const forge_runtime::PipelineError& e) {
    threw = e.kind() == forge_runtime::PipelineError::Kind::GpuExecution;
  }
  CHECK(threw);
}

}  // namespace

int main(int argc, char** argv) {
  const bool cpu_only = argc > 1 && std::string(argv[1]) == "--cpu";
  int failed = 0, ran = 0;
  for (const Case& c : registry()) {
    if (cpu_only && c.gpu) continue;
    if (!cpu_only && !c.gpu && std::string(c.name).rfind("test_no_device", 0) == 0) continue;
    ++ran;
    try {
      c.fn();
      std::printf("ok   %s\n", c.name);
    } catch (const Failure& f) {
      ++failed;
      std::printf("FAIL %s: %s\n", c.name, f.what.c_str());
    } catch (const std::exception& e) {
      ++failed;
      std::printf("FAIL %s: exception: %s\n", c.name, e.what());
    }
  }
  std::printf("%d of %d passed\n", ran - failed, ran);
  return failed ? 1 : 0;
}
