// forge_runtime.hpp -- the sort side of gpu-forge's forge-runtime crate in C++
// over the libforgesort C ABI (include/forgesort.h).  Header-only; link
// -lforgesort.
//
// Mirrors metal-forge-compute/forge-runtime/src of kavanaghpatrick/gpu-forge:
//   ForgeContext (context.rs:16-55)  -> one CUDA device + one stream
//                                       (fs_stream_create), and alloc_buffer
//                                       backed by page-locked host memory
//   GpuGather    (gather.rs:27-140)  -> fs_gather: output[i] = source[idx[i]]
//   Pipeline     (pipeline.rs:56-140)-> stages enqueued on the context's
//                                       stream; execute() waits once
//   GatherError / PipelineError      -> exceptions with the same Display
//                                       strings
// The reference's one command buffer is the context's stream: stages run in
// submission order, each seeing the previous stage's writes.  Filter stages
// belong to forge-filter, which this build does not include.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "forge_sort.hpp"

namespace forge_runtime {

// ---- errors (gather.rs:17-24, pipeline.rs:41-54) -------------------------------
class GatherError : public std::runtime_error {
 public:
  enum class Kind { ShaderCompilation, GpuExecution };
  static GatherError shader_compilation(const std::string& m) {
    return GatherError(Kind::ShaderCompilation, "shader compilation failed: " + m);
  }
  static GatherError gpu_execution(const std::string& m) {
    return GatherError(Kind::GpuExecution, "GPU execution failed: " + m);
  }
  Kind kind() const noexcept { return kind_; }

 private:
  GatherError(Kind k, const std::string& d) : std::runtime_error(d), kind_(k) {}
  Kind kind_;
};

class PipelineError : public std::runtime_error {
 public:
  enum class Kind { CommandBuffer, Encoder, GpuExecution, Sort };
  static PipelineError command_buffer() { return PipelineError(Kind::CommandBuffer, "failed to create command buffer"); }
  static PipelineError encoder() { return PipelineError(Kind::Encoder, "failed to create compute encoder"); }
  static PipelineError gpu_execution(const std::string& m) {
    return PipelineError(Kind::GpuExecution, "GPU execution failed: " + m);
  }
  static PipelineError sort(const forge_sort::SortError& e) {
    return PipelineError(Kind::Sort, std::string("sort error: ") + e.what());
  }
  Kind kind() const noexcept { return kind_; }

 private:
  PipelineError(Kind k, const std::string& d) : std::runtime_error(d), kind_(k) {}
  Kind kind_;
};

class ForgeContext;

// A buffer from ForgeContext::alloc_buffer: page-locked host memory that the
// host reads and writes directly and the kernels reach through the same
// address (the discrete-GPU form of a StorageModeShared MTLBuffer).
class Buffer {
 public:
  Buffer(Buffer&& o) noexcept
      : owner_(std::exchange(o.owner_, nullptr)), p_(std::exchange(o.p_, nullptr)), bytes_(o.bytes_) {}
  Buffer& operator=(Buffer&& o) noexcept {
    if (this != &o) {
      release();
      owner_ = std::exchange(o.owner_, nullptr);
      p_ = std::exchange(o.p_, nullptr);
      bytes_ = o.bytes_;
    }
    return *this;
  }
  Buffer(const Buffer&) = delete;
  Buffer& operator=(const Buffer&) = delete;
  ~Buffer() { release(); }

  void* contents() const { return p_; }
  void* device_ptr() const { return p_; }
  std::size_t length() const { return bytes_; }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p_);
  }

 private:
  friend class ForgeContext;
  Buffer(fs_sorter* owner, void* p, std::size_t bytes) : owner_(owner), p_(p), bytes_(bytes) {}
  void release() {
    if (owner_ && p_) fs_free(owner_, p_);
    p_ = nullptr;
  }
  fs_sorter* owner_ = nullptr;
  void* p_ = nullptr;
  std::size_t bytes_ = 0;
};

// ---- ForgeContext (context.rs) ---------------------------------------------------
// Throws forge_sort::SortError (DeviceNotFound) without a CUDA device, where
// the reference panics.  Buffers from alloc_buffer must not outlive it.
class ForgeContext {
 public:
  static ForgeContext create(int device = 0) { return ForgeContext(device); }

  ForgeContext(ForgeContext&& o) noexcept
      : device_(o.device_), stream_(std::exchange(o.stream_, nullptr)), alloc_(std::exchange(o.alloc_, nullptr)) {}
  ForgeContext(const ForgeContext&) = delete;
  ForgeContext& operator=(const ForgeContext&) = delete;
  ForgeContext& operator=(ForgeContext&&) = delete;
  ~ForgeContext() {
    if (alloc_) fs_destroy(alloc_);
    if (stream_) fs_stream_destroy(stream_);
  }

  int device() const { return device_; }
  void* queue() const { return stream_; }  // a cudaStream_t

  Buffer alloc_buffer(std::size_t size) {
    void* p = nullptr;
    forge_sort::detail::check(fs_alloc(alloc_, size ? size : 1, 1, &p), alloc_);
    return Buffer(alloc_, p, size);
  }
  void synchronize() { forge_sort::detail::check(fs_stream_synchronize(stream_), nullptr); }

 private:
  explicit ForgeContext(int device) : device_(device) {
    forge_sort::detail::check(fs_stream_create(device, &stream_), nullptr);
    const int rc = fs_create(device, stream_, &alloc_);
    if (rc != FS_OK) {
      fs_stream_destroy(stream_);
      stream_ = nullptr;
      alloc_ = nullptr;
      forge_sort::detail::check(rc, nullptr);
    }
  }
  int device_ = 0;
  void* stream_ = nullptr;
  fs_sorter* alloc_ = nullptr;  // owns the alloc_buffer memory
};

// ---- GpuGather (gather.rs) ---------------------------------------------------------
// Every index is checked against the source length (source_len elements): an
// index past it is skipped and reported as GpuExecution when the work is
// waited for; the reference kernel has no such check.
class GpuGather {
 public:
  static GpuGather create() { return GpuGather(0, nullptr); }
  static GpuGather with_context(int device, void* queue) { return GpuGather(device, queue); }

  GpuGather(GpuGather&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
  GpuGather(const GpuGather&) = delete;
  GpuGather& operator=(const GpuGather&) = delete;
  GpuGather& operator=(GpuGather&&) = delete;
  ~GpuGather() {
    if (h_) fs_destroy(h_);
  }

  // gather.rs:77-117 -- enqueue on `stream` (this gather's stream when null).
  void encode_gather(void* stream, const void* source, uint64_t source_len, const void* indices, void* output,
                     uint32_t count, bool is_64bit) {
    if (stream) check(fs_set_stream(h_, stream));
    check(fs_gather(h_, is_64bit ? 8 : 4, source, source_len, static_cast<const uint32_t*>(indices), output, count,
                    0));
  }
  void encode_gather(void* stream, const Buffer& source, const Buffer& indices, Buffer& output, uint32_t count,
                     bool is_64bit) {
    encode_gather(stream, source.device_ptr(), source.length() / (is_64bit ? 8 : 4), indices.device_ptr(),
                  output.device_ptr(), count, is_64bit);
  }
  // gather.rs:119-140 -- wait for the result.
  void gather_u32(const Buffer& source, const Buffer& indices, Buffer& output, uint32_t count) {
    encode_gather(nullptr, source, indices, output, count, false);
    synchronize();
  }
  void gather_u64(const Buffer& source, const Buffer& indices, Buffer& output, uint32_t count) {
    encode_gather(nullptr, source, indices, output, count, true);
    synchronize();
  }
  void synchronize() { check(fs_synchronize(h_)); }

 private:
  GpuGather(int device, void* stream) {
    if (fs_create(device, stream, &h_) != FS_OK) {
      h_ = nullptr;
      throw GatherError::shader_compilation(fs_last_error(nullptr));
    }
  }
  void check(int rc) {
    if (rc == FS_OK) return;
    if (rc == FS_E_INVALID) throw std::invalid_argument(fs_last_error(h_));
    throw GatherError::gpu_execution(fs_last_error(h_));
  }
  fs_sorter* h_ = nullptr;
};

// ---- Pipeline (pipeline.rs) ----------------------------------------------------------
class Pipeline {
 public:
  explicit Pipeline(ForgeContext& ctx) : ctx_(&ctx) {
    if (!ctx.queue()) throw PipelineError::command_buffer();
  }
  static Pipeline create(ForgeContext& ctx) { return Pipeline(ctx); }

  // pipeline.rs:98-105 -- an in-place sort of a SortBuffer<u32>.
  void sort(forge_sort::GpuSorter& sorter, const forge_sort::SortBuffer<uint32_t>& buf) {
    try {
      sorter.encode_sort(ctx_->queue(), buf);
    } catch (const forge_sort::SortError& e) {
      throw PipelineError::sort(e);
    }
    sorters_.push_back(&sorter);
  }
  // pipeline.rs:107-122 -- output[i] = source[indices[i]].
  void gather(GpuGather& g, const Buffer& source, const Buffer& indices, Buffer& output, uint32_t count,
              bool is_64bit) {
    g.encode_gather(ctx_->queue(), source, indices, output, count, is_64bit);
    gathers_.push_back(&g);
  }
  void gather(GpuGather& g, const void* source, uint64_t source_len, const void* indices, void* output,
              uint32_t count, bool is_64bit) {
    g.encode_gather(ctx_->queue(), source, source_len, indices, output, count, is_64bit);
    gathers_.push_back(&g);
  }

  // pipeline.rs:124-139 -- wait once, then report the first device-side
  // failure a stage left behind.
  void execute() {
    std::string first;
    auto note = [&](const std::exception& e, const std::string& prefix) {
      if (!first.empty()) return;
      std::string w = e.what();
      first = w.rfind(prefix, 0) == 0 ? w.substr(prefix.size()) : w;
    };
    try {
      ctx_->synchronize();
    } catch (const std::exception& e) {
      note(e, "GPU execution failed: ");
    }
    for (auto* s : sorters_) try {
        s->synchronize();
      } catch (const std::exception& e) {
        note(e, "GPU execution failed: ");
      }
    for (auto* g : gathers_) try {
        g->synchronize();
      } catch (const std::exception& e) {
        note(e, "GPU execution failed: ");
      }
    sorters_.clear();
    gathers_.clear();
    if (!first.empty()) throw PipelineError::gpu_execution(first);
  }

 private:
  ForgeContext* ctx_;
  std::vector<forge_sort::GpuSorter*> sorters_;
  std::vector<GpuGather*> gathers_;
};

}  // namespace forge_runtime
