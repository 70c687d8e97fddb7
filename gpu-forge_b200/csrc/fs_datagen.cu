// fs_datagen.cu -- GPU generator of the seeded xorshift64 benchmark inputs
// (include/forgesort_bench.h).  Each thread jumps straight to the start of
// its run of elements with precomputed powers of the step's 64x64 GF(2)
// matrix, then steps sequentially; the output is bit-identical to one
// sequential xorshift64 stream.
#include "forgesort.h"
#include "forgesort_bench.h"

#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

namespace {

constexpr int RUN = 64;  // consecutive elements per thread

inline uint64_t xs_step_h(uint64_t x) {
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  return x;
}

__device__ __forceinline__ uint64_t xs_step(uint64_t x) {
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  return x;
}

// jump[j*64 + i] = column i of T^(2^j)
uint64_t* g_jump_dev[64] = {};
std::mutex g_mu;

uint64_t apply_h(const uint64_t* col, uint64_t x) {
  uint64_t r = 0;
  while (x) {
    r ^= col[__builtin_ctzll(x)];
    x &= x - 1;
  }
  return r;
}

int jump_table(int dev, const uint64_t** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= 64) return FS_E_INVALID;
  if (!g_jump_dev[dev]) {
    static uint64_t h[64 * 64];
    static bool built = false;
    if (!built) {
      for (int i = 0; i < 64; ++i) h[i] = xs_step_h(1ull << i);
      for (int j = 1; j < 64; ++j)
        for (int i = 0; i < 64; ++i) h[j * 64 + i] = apply_h(&h[(j - 1) * 64], h[(j - 1) * 64 + i]);
      built = true;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, sizeof h) != cudaSuccess) return FS_E_OOM;
    if (cudaMemcpy(p, h, sizeof h, cudaMemcpyHostToDevice) != cudaSuccess) return FS_E_GPU_EXECUTION;
    g_jump_dev[dev] = static_cast<uint64_t*>(p);
  }
  *out = g_jump_dev[dev];
  return FS_OK;
}

__device__ uint64_t jump(const uint64_t* __restrict__ tab, uint64_t x, uint64_t k) {
  for (int j = 0; k; ++j, k >>= 1) {
    if (k & 1) {
      const uint64_t* col = tab + j * 64;
      uint64_t r = 0, y = x;
      while (y) {
        r ^= __ldg(col + (__ffsll((long long)y) - 1));
        y &= y - 1;
      }
      x = r;
    }
  }
  return x;
}

__global__ void k_generate(const uint64_t* __restrict__ tab, int dist, uint64_t seed, uint64_t start,
                           uint64_t n, void* __restrict__ out) {
  const uint64_t runs = (n + RUN - 1) / RUN;
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < runs;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i0 = r * RUN;
    uint64_t x = jump(tab, seed, start + i0);  // state after (start+i0) steps
    const uint64_t m = n - i0 < RUN ? n - i0 : RUN;
    for (uint64_t t = 0; t < m; ++t) {
      x = xs_step(x);
      const uint64_t i = i0 + t;
      if (dist == FS_GEN_U64) {
        static_cast<uint64_t*>(out)[i] = x;
      } else if (dist == FS_GEN_U32) {
        static_cast<uint32_t*>(out)[i] = (uint32_t)(x >> 32);
      } else {
        const uint32_t lo = (uint32_t)x;
        static_cast<uint32_t*>(out)[i] = (lo % 10u < 7u) ? 0x40000000u + (uint32_t)(x >> 44) : (uint32_t)(x >> 32);
      }
    }
  }
}

}  // namespace

extern "C" int fs_generate(int dist, uint64_t seed, uint64_t start, uint64_t n, void* out, void* stream) {
  if (dist < FS_GEN_U32 || dist > FS_GEN_SKEW_U32 || (!out && n)) return FS_E_INVALID;
  if (n == 0) return FS_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FS_E_DEVICE_NOT_FOUND;
  const uint64_t* tab = nullptr;
  int rc = jump_table(dev, &tab);
  if (rc) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t runs = (n + RUN - 1) / RUN;
  uint64_t blocks = (runs + 255) / 256;
  if (blocks > (uint64_t)sms * 16) blocks = (uint64_t)sms * 16;
  k_generate<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(tab, dist, seed, start, n, out);
  return cudaGetLastError() == cudaSuccess ? FS_OK : FS_E_GPU_EXECUTION;
}
