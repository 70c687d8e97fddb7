// forge_sort.hpp -- the forge-sort GpuSorter / SortBuffer API in C++ over the
// libforgesort C ABI (include/forgesort.h).  Header-only; link -lforgesort.
//
// Mirrors metal-forge-compute/forge-sort/src/lib.rs of kavanaghpatrick/gpu-forge
// method for method: the same names, the same argument meaning, the same
// n <= 1 short-cuts and the same four error variants with the same Display
// strings.  Rust-to-C++ mapping:
//   Result<T, SortError>      -> T, or throws forge_sort::SortError
//   &mut [T] / &[T]           -> std::span<T> / std::span<const T>
//   Vec<u32>                  -> std::vector<uint32_t>
//   SortBuffer<T>             -> SortBuffer<T> (device memory + page-locked host
//                                mirror kept coherent lazily: sorts stay in
//                                HBM, host views copy back only what changed)
//   MTLDevice + command queue -> CUDA device ordinal + cudaStream_t (void*)
//   metal_buffer()            -> device_ptr()
// Sealed SortKey (lib.rs:15-88) -> SortKey<T>, defined for the six key types
// only, with the same constants.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <stdexcept>
#include <string>
#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

#include "forgesort.h"

namespace forge_sort {

// ---- SortError (lib.rs:94-104) ----------------------------------------------
class SortError : public std::runtime_error {
 public:
  enum class Kind { DeviceNotFound, ShaderCompilation, GpuExecution, LengthMismatch };

  static SortError device_not_found() { return SortError(Kind::DeviceNotFound, "no Metal GPU device found"); }
  static SortError shader_compilation(const std::string& m) {
    return SortError(Kind::ShaderCompilation, "shader compilation failed: " + m, m);
  }
  static SortError gpu_execution(const std::string& m) {
    return SortError(Kind::GpuExecution, "GPU execution failed: " + m, m);
  }
  static SortError length_mismatch(std::size_t keys, std::size_t values) {
    SortError e(Kind::LengthMismatch,
                "length mismatch: keys=" + std::to_string(keys) + ", values=" + std::to_string(values));
    e.keys_ = keys;
    e.values_ = values;
    return e;
  }

  Kind kind() const noexcept { return kind_; }
  const std::string& message() const noexcept { return msg_; }  // the variant's String payload
  std::size_t keys() const noexcept { return keys_; }           // LengthMismatch fields
  std::size_t values() const noexcept { return values_; }

 private:
  SortError(Kind k, const std::string& display, std::string msg = {})
      : std::runtime_error(display), kind_(k), msg_(std::move(msg)) {}
  Kind kind_;
  std::string msg_;
  std::size_t keys_ = 0, values_ = 0;
};

// Status codes that are not one of the four variants (invalid arguments) map
// to std::invalid_argument, as a Rust caller would have met a panic or a type
// error for them.
namespace detail {
inline void check(int rc, fs_sorter* h, std::size_t keys = 0, std::size_t values = 0) {
  if (rc == FS_OK) return;
  const char* t = fs_last_error(h);
  const std::string m = t ? t : "";
  switch (rc) {
    case FS_E_DEVICE_NOT_FOUND: throw SortError::device_not_found();
    case FS_E_KERNEL_IMAGE: throw SortError::shader_compilation(m);
    case FS_E_LENGTH_MISMATCH: throw SortError::length_mismatch(keys, values);
    case FS_E_INVALID: throw std::invalid_argument(m);
    default: throw SortError::gpu_execution(m);
  }
}
}  // namespace detail

// ---- SortKey (lib.rs:29-88) -------------------------------------------------
template <typename T>
struct SortKey;  // only the six key types below are sort keys

#define FORGE_SORT_KEY(T, DT, SIZE, XF, W64, FWD, INV)         \
  template <>                                                  \
  struct SortKey<T> {                                          \
    static constexpr int DTYPE = DT;                           \
    static constexpr std::size_t KEY_SIZE = SIZE;              \
    static constexpr bool NEEDS_TRANSFORM = XF;                \
    static constexpr bool IS_64BIT = W64;                      \
    static constexpr uint32_t TRANSFORM_MODE_FORWARD = FWD;    \
    static constexpr uint32_t TRANSFORM_MODE_INVERSE = INV;    \
  };
FORGE_SORT_KEY(uint32_t, FS_U32, 4, false, false, 0, 0)
FORGE_SORT_KEY(int32_t, FS_I32, 4, true, false, 0, 0)
FORGE_SORT_KEY(float, FS_F32, 4, true, false, 1, 2)
FORGE_SORT_KEY(uint64_t, FS_U64, 8, false, true, 0, 0)
FORGE_SORT_KEY(int64_t, FS_I64, 8, true, true, 0, 0)
FORGE_SORT_KEY(double, FS_F64, 8, true, true, 1, 2)
#undef FORGE_SORT_KEY

class GpuSorter;

// ---- SortBuffer<T> (lib.rs:160-281) -----------------------------------------
// Device memory plus a page-locked host mirror, kept coherent lazily by the
// library (fs_buffer_*): sorts stay in HBM; as_slice() copies back only what
// they changed; as_mut_slice() marks the device copy stale.  A span from
// as_mut_slice() is one host write session: take it again to write after a
// sort (Rust's borrow of &mut self ends the same way).
template <typename T>
class SortBuffer {
  static_assert(sizeof(SortKey<T>) > 0, "SortBuffer<T> needs a SortKey type");

 public:
  SortBuffer(SortBuffer&& o) noexcept { *this = std::move(o); }
  SortBuffer& operator=(SortBuffer&& o) noexcept {
    if (this != &o) {
      release();
      b_ = std::exchange(o.b_, nullptr);
      len_ = std::exchange(o.len_, 0);
      cap_ = std::exchange(o.cap_, 0);
    }
    return *this;
  }
  SortBuffer(const SortBuffer&) = delete;
  SortBuffer& operator=(const SortBuffer&) = delete;
  ~SortBuffer() { release(); }

  std::size_t len() const { return len_; }
  bool is_empty() const { return len_ == 0; }
  std::size_t capacity() const { return cap_; }

  // Writable view of all capacity() elements: write, then set_len().
  std::span<T> as_mut_slice() {
    detail::check(fs_buffer_host_write(b_), nullptr);
    return {host(), cap_};
  }
  // The first len() elements (the sorted result after a sort).
  std::span<const T> as_slice() const {
    detail::check(fs_buffer_host_read(b_), nullptr);
    return {host(), len_};
  }

  void set_len(std::size_t len) {
    if (len > cap_)
      throw std::length_error("len " + std::to_string(len) + " exceeds capacity " + std::to_string(cap_));
    len_ = len;
  }
  void copy_from_slice(std::span<const T> data) {
    if (data.size() > cap_)
      throw std::length_error("data len " + std::to_string(data.size()) + " exceeds capacity " +
                              std::to_string(cap_));
    detail::check(fs_buffer_host_write(b_), nullptr);
    if (!data.empty()) std::memcpy(host(), data.data(), data.size_bytes());
    len_ = data.size();
  }
  void copy_to_slice(std::span<T> dest) const {
    const std::size_t n = len_ < dest.size() ? len_ : dest.size();
    detail::check(fs_buffer_host_read(b_), nullptr);
    if (n) std::memcpy(dest.data(), host(), n * sizeof(T));
  }

  // Device address of element 0 (replaces metal_buffer()) for other device
  // code: the device copy is made current for len() elements and counted as
  // written, so a later host read waits for the device.
  void* device_ptr() const {
    detail::check(fs_buffer_device_use(b_, len_ * sizeof(T)), nullptr);
    return fs_buffer_device(b_);
  }
  // The library's buffer object (what the sorts take).
  fs_buffer* handle() const { return b_; }

  // Re-wrap a buffer object given up by into_raw_parts (owned again).
  static SortBuffer from_raw_parts(fs_buffer* b, std::size_t len, std::size_t capacity) {
    if (len > capacity)
      throw std::length_error("len " + std::to_string(len) + " exceeds capacity " + std::to_string(capacity));
    if (capacity * sizeof(T) > fs_buffer_bytes(b)) throw std::length_error("capacity exceeds the buffer's size");
    return SortBuffer(b, len, capacity);
  }
  // Give up ownership: (buffer object, len, capacity); fs_buffer_destroy frees it.
  std::tuple<fs_buffer*, std::size_t, std::size_t> into_raw_parts() && {
    return {std::exchange(b_, nullptr), std::exchange(len_, 0), std::exchange(cap_, 0)};
  }

 private:
  friend class GpuSorter;
  SortBuffer(fs_buffer* b, std::size_t len, std::size_t cap) : b_(b), len_(len), cap_(cap) {}
  T* host() const { return static_cast<T*>(fs_buffer_host(b_)); }
  void release() noexcept {
    if (b_) fs_buffer_destroy(b_);
    b_ = nullptr;
  }
  fs_buffer* b_ = nullptr;
  std::size_t len_ = 0, cap_ = 0;
};

// ---- GpuSorter (lib.rs:132-3015) ---------------------------------------------
class GpuSorter {
 public:
  // lib.rs:596 -- device 0, a private stream.
  static GpuSorter create() { return GpuSorter(0, nullptr); }
  // lib.rs:606 -- the caller's device and stream (a cudaStream_t).
  static GpuSorter with_context(int device, void* stream) { return GpuSorter(device, stream); }

  GpuSorter(GpuSorter&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
  GpuSorter& operator=(GpuSorter&& o) noexcept {
    if (this != &o) {
      if (h_) fs_destroy(h_);
      h_ = std::exchange(o.h_, nullptr);
    }
    return *this;
  }
  GpuSorter(const GpuSorter&) = delete;
  GpuSorter& operator=(const GpuSorter&) = delete;
  ~GpuSorter() {
    if (h_) fs_destroy(h_);
  }

  fs_sorter* handle() const { return h_; }
  void synchronize() { detail::check(fs_synchronize(h_), h_); }

  // -- zero-copy buffers (lib.rs:694-738, 1000-1117, 2301-2590) ----------------
  template <typename T>
  SortBuffer<T> alloc_sort_buffer(std::size_t capacity) {
    fs_buffer* b = nullptr;
    detail::check(fs_buffer_create(h_, (capacity ? capacity : 1) * sizeof(T), &b), h_);
    return SortBuffer<T>(b, 0, capacity);
  }
  void sort_buffer(const SortBuffer<uint32_t>& b) { sort_buf(b); }
  void sort_i32_buffer(const SortBuffer<int32_t>& b) { sort_buf(b); }
  void sort_f32_buffer(const SortBuffer<float>& b) { sort_buf(b); }
  void sort_u64_buffer(const SortBuffer<uint64_t>& b) { sort_buf(b); }
  void sort_i64_buffer(const SortBuffer<int64_t>& b) { sort_buf(b); }
  void sort_f64_buffer(const SortBuffer<double>& b) { sort_buf(b); }

  // lib.rs:749 -- enqueue an in-place u32 sort on `stream` (the sorter's own
  // stream when null) and return; the caller synchronises that stream before
  // reading the buffer.
  void encode_sort(void* stream, const SortBuffer<uint32_t>& b) {
    if (b.len() <= 1) return;
    if (stream) detail::check(fs_set_stream(h_, stream), h_);
    detail::check(fs_sort_buffer(h_, FS_U32, b.handle(), b.len(), 0), h_);
  }

  // -- host slices, in place (lib.rs:791-998, 2238-2485) ----------------------
  void sort_u32(std::span<uint32_t> d) { sort_host(d); }
  void sort_i32(std::span<int32_t> d) { sort_host(d); }
  void sort_f32(std::span<float> d) { sort_host(d); }
  void sort_u64(std::span<uint64_t> d) { sort_host(d); }
  void sort_i64(std::span<int64_t> d) { sort_host(d); }
  void sort_f64(std::span<double> d) { sort_host(d); }

  // -- argsort: stable permutation, input untouched (lib.rs:1675-1921, 2595-2825)
  std::vector<uint32_t> argsort_u32(std::span<const uint32_t> d) { return argsort_host(d); }
  std::vector<uint32_t> argsort_i32(std::span<const int32_t> d) { return argsort_host(d); }
  std::vector<uint32_t> argsort_f32(std::span<const float> d) { return argsort_host(d); }
  std::vector<uint32_t> argsort_u64(std::span<const uint64_t> d) { return argsort_host(d); }
  std::vector<uint32_t> argsort_i64(std::span<const int64_t> d) { return argsort_host(d); }
  std::vector<uint32_t> argsort_f64(std::span<const double> d) { return argsort_host(d); }

  // -- permutation apply (forge-runtime GpuGather): dst[i] = src[idx[i]] on device
  // memory, T a 4- or 8-byte element (no reference counterpart in forge-sort) --
  template <typename T>
  void gather_device(const T* src, uint64_t src_n, const uint32_t* idx, T* dst, uint64_t n) {
    static_assert(sizeof(T) == 4 || sizeof(T) == 8, "4- or 8-byte elements");
    detail::check(fs_gather(h_, (int)sizeof(T), src, src_n, idx, dst, n, 1), h_);
  }

  // -- stable key/value sort, u32 values (lib.rs:1923-2236, 2826-3015) --------
  void sort_pairs_u32(std::span<uint32_t> k, std::span<uint32_t> v) { pairs_host(k, v); }
  void sort_pairs_i32(std::span<int32_t> k, std::span<uint32_t> v) { pairs_host(k, v); }
  void sort_pairs_f32(std::span<float> k, std::span<uint32_t> v) { pairs_host(k, v); }
  void sort_pairs_u64(std::span<uint64_t> k, std::span<uint32_t> v) { pairs_host(k, v); }
  void sort_pairs_i64(std::span<int64_t> k, std::span<uint32_t> v) { pairs_host(k, v); }

 private:
  GpuSorter(int device, void* stream) {
    const int rc = fs_create(device, stream, &h_);
    if (rc != FS_OK) {
      h_ = nullptr;
      detail::check(rc, nullptr);
    }
  }

  template <typename T>
  void sort_buf(const SortBuffer<T>& b) {
    if (b.len() <= 1) return;
    detail::check(fs_sort_buffer(h_, SortKey<T>::DTYPE, b.handle(), b.len(), 1), h_);
  }
  template <typename T>
  void sort_host(std::span<T> d) {
    if (d.size() <= 1) return;
    detail::check(fs_host_sort_keys(h_, SortKey<T>::DTYPE, d.data(), d.size()), h_);
  }
  template <typename T>
  std::vector<uint32_t> argsort_host(std::span<const T> d) {
    if (d.empty()) return {};
    if (d.size() == 1) return {0u};
    std::vector<uint32_t> idx(d.size());
    detail::check(fs_host_argsort(h_, SortKey<T>::DTYPE, d.data(), idx.data(), d.size()), h_);
    return idx;
  }
  template <typename T>
  void pairs_host(std::span<T> k, std::span<uint32_t> v) {
    detail::check(fs_host_sort_pairs(h_, SortKey<T>::DTYPE, k.data(), k.size(), v.data(), v.size()), h_, k.size(),
                  v.size());
  }

  fs_sorter* h_ = nullptr;
};

// ---- MultiGpuSorter (no reference counterpart) ---------------------------------
// The sample sort over several GPUs of this process (fs_mg_*): shards in,
// pieces of the globally sorted sequence out, piece i on devices[i].
class MultiGpuSorter {
 public:
  explicit MultiGpuSorter(const std::vector<int>& devices) {
    const int rc = fs_mg_create(devices.data(), (int)devices.size(), &h_);
    if (rc != FS_OK) {
      h_ = nullptr;
      detail::check(rc, nullptr);
    }
    g_ = devices.size();
  }
  MultiGpuSorter(const MultiGpuSorter&) = delete;
  MultiGpuSorter& operator=(const MultiGpuSorter&) = delete;
  ~MultiGpuSorter() {
    if (h_) fs_mg_destroy(h_);
  }

  // shards[i]: device pointer on devices[i] with shard_n[i] keys of T;
  // out[i]: device pointer on devices[i] with room for out_cap[i] keys.
  // Returns the piece sizes.  Throws std::length_error (with the sizes
  // needed in `needed`) when a piece would not fit its out_cap.
  template <typename T>
  std::vector<uint64_t> sort(const std::vector<T*>& shards, const std::vector<uint64_t>& shard_n,
                             const std::vector<T*>& out, const std::vector<uint64_t>& out_cap,
                             std::vector<uint64_t>* needed = nullptr) {
    if (shards.size() != g_ || shard_n.size() != g_ || out.size() != g_ || out_cap.size() != g_)
      throw std::invalid_argument("one shard and one output per device");
    std::vector<void*> sp(shards.begin(), shards.end()), op(out.begin(), out.end());
    std::vector<uint64_t> out_n(g_);
    const int rc = fs_mg_sort_keys(h_, SortKey<T>::DTYPE, sp.data(), shard_n.data(), op.data(), out_cap.data(),
                                   out_n.data());
    if (rc == FS_E_INVALID) {
      bool over = false;
      for (size_t i = 0; i < g_; ++i) over = over || out_n[i] > out_cap[i];
      if (over) {
        if (needed) *needed = out_n;
        throw std::length_error(fs_mg_last_error(h_));
      }
    }
    if (rc != FS_OK) throw SortError::gpu_execution(fs_mg_last_error(h_));
    return out_n;
  }

  // The per-type names of the boundary.
  std::vector<uint64_t> sort_u32(const std::vector<uint32_t*>& shards, const std::vector<uint64_t>& shard_n,
                                 const std::vector<uint32_t*>& out, const std::vector<uint64_t>& out_cap,
                                 std::vector<uint64_t>* needed = nullptr) {
    return sort<uint32_t>(shards, shard_n, out, out_cap, needed);
  }
  std::vector<uint64_t> sort_u64(const std::vector<uint64_t*>& shards, const std::vector<uint64_t>& shard_n,
                                 const std::vector<uint64_t*>& out, const std::vector<uint64_t>& out_cap,
                                 std::vector<uint64_t>* needed = nullptr) {
    return sort<uint64_t>(shards, shard_n, out, out_cap, needed);
  }

  // The stable pairs form: vals[i] (device, shard_n[i] u32) travel with the
  // keys into out_vals[i] (room for out_cap[i]); with `vals` empty, every
  // key's global position is sent instead (an argsort).  Same sizing rule.
  template <typename T>
  std::vector<uint64_t> sort_pairs(const std::vector<T*>& shards, const std::vector<const uint32_t*>& vals,
                                   const std::vector<uint64_t>& shard_n, const std::vector<T*>& out,
                                   const std::vector<uint32_t*>& out_vals, const std::vector<uint64_t>& out_cap,
                                   std::vector<uint64_t>* needed = nullptr) {
    if (shards.size() != g_ || shard_n.size() != g_ || out.size() != g_ || out_cap.size() != g_ ||
        out_vals.size() != g_ || (!vals.empty() && vals.size() != g_))
      throw std::invalid_argument("one shard, value array and output per device");
    std::vector<void*> sp(shards.begin(), shards.end()), op(out.begin(), out.end());
    std::vector<uint64_t> out_n(g_);
    const int rc = fs_mg_sort_pairs(h_, SortKey<T>::DTYPE, sp.data(), vals.empty() ? nullptr : vals.data(),
                                    shard_n.data(), op.data(), out_vals.data(), out_cap.data(), out_n.data());
    if (rc == FS_E_INVALID) {
      bool over = false;
      for (size_t i = 0; i < g_; ++i) over = over || out_n[i] > out_cap[i];
      if (over) {
        if (needed) *needed = out_n;
        throw std::length_error(fs_mg_last_error(h_));
      }
      throw std::invalid_argument(fs_mg_last_error(h_));
    }
    if (rc != FS_OK) throw SortError::gpu_execution(fs_mg_last_error(h_));
    return out_n;
  }

 private:
  fs_mg* h_ = nullptr;
  size_t g_ = 0;
};

}  // namespace forge_sort
