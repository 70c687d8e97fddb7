// fs_multi.cu -- the sample sort over several GPUs of one process (the
// MultiGpuSorter of the C ABI: fs_mg_*).  The one-process-per-GPU form of the
// same algorithm lives in gpu-forge_b200/forge_sort/samplesort.py; both use
// the partition kernels of fs_sort.cu through the C ABI.
//
// Per call, with G devices holding shards of n_i keys:
//   1. samples: S keys at regular positions of every shard, as (ordered key,
//      global position, raw key) triples, gathered to the host; the host
//      picks the G-1 splitters (every S-th triple in (key, position) order;
//      the position breaks ties, so equal keys still split evenly);
//   2. count: fs_partition_count on every device -> the G x G send matrix;
//   3. dispatch: fs_partition_dispatch on every device writes each bucket
//      straight into its destination device's inbox (peer access over
//      NVLink, plain stores), at the offset the matrix gives;
//   4. local sort of every inbox into the caller's output buffer.
// fs_mg_sort_pairs carries a u32 per key (the caller's values, or each key's
// global position for an argsort) in a second region of every inbox and
// ends with a stable local pairs sort: keys reach an inbox in global-position
// order (lower devices first, each in input order), so equal keys end in
// global input order.
#include "forgesort.h"
#include "fs_device.cuh"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

using namespace fs;

namespace {

constexpr int MG_MAX = 16;                 // devices per fs_mg
constexpr uint32_t MG_SAMPLES = 8192;      // samples per shard

struct Sample {
  uint64_t ord, gpos, raw;
};

// Regular samples of one shard: element floor((j + 0.5) * m / S).
template <typename K, int XF>
__global__ void k_samples(const K* __restrict__ keys, uint64_t m, uint64_t gpos_base, uint32_t S,
                          Sample* __restrict__ out) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= S) return;
  uint64_t p = (uint64_t)(((double)j + 0.5) * ((double)m / (double)S));
  if (p >= m) p = m - 1;
  const K raw = keys[p];
  out[j] = Sample{(uint64_t)to_ordered<K, XF>(raw), gpos_base + p, (uint64_t)raw};
}

}  // namespace

struct fs_mg {
  int g = 0;
  int dev[MG_MAX] = {};
  fs_sorter* s[MG_MAX] = {};
  void* inbox[MG_MAX] = {};        // device memory on dev[i]
  uint64_t inbox_bytes = 0;        // every inbox has this capacity
  void* spl_keys[MG_MAX] = {};     // splitter raw keys / positions on dev[i]
  void* spl_gpos[MG_MAX] = {};
  Sample* samples_dev[MG_MAX] = {};
  Sample* samples_host = nullptr;  // pinned, G * MG_SAMPLES
  std::string err;
};

namespace {

int mg_fail(fs_mg* mg, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (mg) mg->err = buf;
  return code;
}

int mg_cuda(fs_mg* mg, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FS_OK;
  cudaGetLastError();
  const int code = e == cudaErrorMemoryAllocation ? FS_E_OOM : FS_E_GPU_EXECUTION;
  return mg_fail(mg, code, "%s: %s", what, cudaGetErrorString(e));
}

#define MG_CUDA(mg, call)                         \
  do {                                            \
    int rc_ = mg_cuda((mg), (call), #call);       \
    if (rc_) return rc_;                          \
  } while (0)

// Error of device i's sorter, as the fs_mg's error.
int mg_from(fs_mg* mg, int i, int rc) {
  if (rc == FS_OK) return FS_OK;
  const char* t = fs_last_error(mg->s[i]);
  mg->err = std::string("device ") + std::to_string(mg->dev[i]) + ": " + (t ? t : "");
  return rc;
}

// Run f(i) for every device on its own host thread; first failure wins.
template <typename F>
int each_device(fs_mg* mg, F&& f) {
  std::vector<int> rcs(mg->g, FS_OK);
  std::vector<std::thread> th;
  for (int i = 0; i < mg->g; ++i)
    th.emplace_back([&, i] {
      cudaSetDevice(mg->dev[i]);
      rcs[i] = f(i);
    });
  for (auto& t : th) t.join();
  for (int i = 0; i < mg->g; ++i)
    if (rcs[i]) return mg_from(mg, i, rcs[i]);
  return FS_OK;
}

template <typename K, int XF>
int mg_sort(fs_mg* mg, int dtype, void* const* shards, const uint32_t* const* vals, bool payload,
            const uint64_t* shard_n, void* const* out, uint32_t* const* out_vals, const uint64_t* out_cap,
            uint64_t* out_n) {
  const int G = mg->g;
  const uint32_t S = MG_SAMPLES;
  uint64_t base[MG_MAX + 1] = {};
  for (int i = 0; i < G; ++i) base[i + 1] = base[i] + shard_n[i];

  // 1. samples -> splitters (host)
  for (int i = 0; i < G; ++i) {
    MG_CUDA(mg, cudaSetDevice(mg->dev[i]));
    Sample* hs = mg->samples_host + (size_t)i * S;
    if (shard_n[i] == 0) {  // an empty shard sends the largest tuples (never picked unless most are empty)
      for (uint32_t j = 0; j < S; ++j) hs[j] = Sample{~0ull, ~0ull, 0};
      continue;
    }
    k_samples<K, XF><<<(S + 255) / 256, 256>>>(static_cast<const K*>(shards[i]), shard_n[i], base[i], S,
                                             mg->samples_dev[i]);
    MG_CUDA(mg, cudaGetLastError());
    MG_CUDA(mg, cudaMemcpy(hs, mg->samples_dev[i], (size_t)S * sizeof(Sample), cudaMemcpyDeviceToHost));
  }
  std::vector<Sample> all(mg->samples_host, mg->samples_host + (size_t)G * S);
  std::sort(all.begin(), all.end(), [](const Sample& a, const Sample& b) {
    return a.ord < b.ord || (a.ord == b.ord && a.gpos < b.gpos);
  });
  const int nsplit = G - 1;
  K spl_raw[MG_MAX];
  uint64_t spl_g[MG_MAX];
  for (int j = 1; j < G; ++j) {
    spl_raw[j - 1] = (K)all[(size_t)j * S].raw;
    spl_g[j - 1] = all[(size_t)j * S].gpos;
  }
  for (int i = 0; i < G && nsplit > 0; ++i) {
    MG_CUDA(mg, cudaSetDevice(mg->dev[i]));
    MG_CUDA(mg, cudaMemcpy(mg->spl_keys[i], spl_raw, (size_t)nsplit * sizeof(K), cudaMemcpyHostToDevice));
    MG_CUDA(mg, cudaMemcpy(mg->spl_gpos[i], spl_g, (size_t)nsplit * 8, cudaMemcpyHostToDevice));
  }

  // 2. bucket counts -> send matrix M[s][b]
  std::vector<uint64_t> M((size_t)G * G, 0);
  int rc = each_device(mg, [&](int i) {
    return fs_partition_count(mg->s[i], dtype, shards[i], shard_n[i], base[i], mg->spl_keys[i],
                              static_cast<const uint64_t*>(mg->spl_gpos[i]), nsplit, &M[(size_t)i * G]);
  });
  if (rc) return rc;
  uint64_t need = 0;
  bool fits = true;
  for (int b = 0; b < G; ++b) {
    uint64_t r = 0;
    for (int i = 0; i < G; ++i) r += M[(size_t)i * G + b];
    out_n[b] = r;
    need = std::max(need, r);
    if (r > out_cap[b]) fits = false;
  }
  if (!fits)
    return mg_fail(mg, FS_E_INVALID, "an output piece exceeds its capacity (out_n holds the sizes needed)");

  // inboxes: grow-only, one capacity for all devices; with a payload the
  // values follow the keys from a 256-byte boundary
  const uint64_t voff = payload ? (need * sizeof(K) + 255) / 256 * 256 : 0;
  const uint64_t need_bytes = payload ? voff + need * 4 : need * sizeof(K);
  if (need_bytes > mg->inbox_bytes) {
    const uint64_t cap = std::max<uint64_t>(need_bytes + need_bytes / 16, 1u << 20);
    for (int i = 0; i < G; ++i) {
      if (mg->inbox[i]) {
        rc = mg_from(mg, i, fs_free(mg->s[i], mg->inbox[i]));
        mg->inbox[i] = nullptr;
        if (rc) return rc;
      }
      if ((rc = mg_from(mg, i, fs_alloc(mg->s[i], cap, 0, &mg->inbox[i])))) return rc;
    }
    mg->inbox_bytes = cap;
  }

  // 3. dispatch: device i's bucket b goes to inbox b after the keys of lower devices
  for (int i = 0; i < G; ++i) {
    void* dst[MG_MAX];
    uint32_t* vdst[MG_MAX];
    for (int b = 0; b < G; ++b) {
      uint64_t start = 0;
      for (int s = 0; s < i; ++s) start += M[(size_t)s * G + b];
      dst[b] = static_cast<char*>(mg->inbox[b]) + start * sizeof(K);
      vdst[b] = reinterpret_cast<uint32_t*>(static_cast<char*>(mg->inbox[b]) + voff + start * 4);
    }
    MG_CUDA(mg, cudaSetDevice(mg->dev[i]));
    if (payload)
      rc = fs_partition_dispatch_pairs(mg->s[i], dtype, shards[i], vals ? vals[i] : nullptr, shard_n[i], base[i],
                                       mg->spl_keys[i], static_cast<const uint64_t*>(mg->spl_gpos[i]), nsplit, dst,
                                       vdst, 0);
    else
      rc = fs_partition_dispatch(mg->s[i], dtype, shards[i], shard_n[i], base[i], mg->spl_keys[i],
                                 static_cast<const uint64_t*>(mg->spl_gpos[i]), nsplit, dst, 0);
    if (rc) return mg_from(mg, i, rc);
  }
  // every inbox is complete once every device's dispatch is
  for (int i = 0; i < G; ++i)
    if ((rc = mg_from(mg, i, fs_synchronize(mg->s[i])))) return rc;

  // 4. local sorts, all devices at once
  for (int i = 0; i < G; ++i) {
    if (out_n[i] == 0) continue;
    MG_CUDA(mg, cudaSetDevice(mg->dev[i]));
    if (payload)
      rc = fs_sort_pairs_copy(mg->s[i], dtype, mg->inbox[i],
                              reinterpret_cast<const uint32_t*>(static_cast<char*>(mg->inbox[i]) + voff), out[i],
                              out_vals[i], out_n[i], 0);
    else
      rc = fs_sort_keys_copy(mg->s[i], dtype, mg->inbox[i], out[i], out_n[i], 0);
    if ((rc = mg_from(mg, i, rc))) return rc;
  }
  for (int i = 0; i < G; ++i)
    if ((rc = mg_from(mg, i, fs_synchronize(mg->s[i])))) return rc;
  return FS_OK;
}

}  // namespace

extern "C" {

int fs_mg_create(const int* devices, int g, fs_mg** out) {
  if (!out) return FS_E_INVALID;
  *out = nullptr;
  if (!devices || g < 1 || g > MG_MAX) return FS_E_INVALID;
  fs_mg* mg = new fs_mg();
  mg->g = g;
  auto bail = [&](int rc) {
    fs_mg_destroy(mg);
    return rc;
  };
  for (int i = 0; i < g; ++i) {
    mg->dev[i] = devices[i];
    for (int j = 0; j < i; ++j)
      if (devices[j] == devices[i]) return bail(FS_E_INVALID);
    const int rc = fs_create(devices[i], nullptr, &mg->s[i]);
    if (rc) return bail(rc);
  }
  // every device writes every other device's inbox: peer access both ways
  for (int i = 0; i < g; ++i) {
    if (cudaSetDevice(devices[i]) != cudaSuccess) return bail(FS_E_GPU_EXECUTION);
    for (int j = 0; j < g; ++j) {
      if (i == j) continue;
      int ok = 0;
      if (cudaDeviceCanAccessPeer(&ok, devices[i], devices[j]) != cudaSuccess || !ok) {
        cudaGetLastError();
        return bail(FS_E_DEVICE_NOT_FOUND);
      }
      const cudaError_t e = cudaDeviceEnablePeerAccess(devices[j], 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return bail(FS_E_GPU_EXECUTION);
      }
      cudaGetLastError();
    }
    if (cudaMalloc(&mg->spl_keys[i], MG_MAX * 8) != cudaSuccess ||
        cudaMalloc(&mg->spl_gpos[i], MG_MAX * 8) != cudaSuccess ||
        cudaMalloc(&mg->samples_dev[i], (size_t)MG_SAMPLES * sizeof(Sample)) != cudaSuccess) {
      cudaGetLastError();
      return bail(FS_E_OOM);
    }
  }
  if (cudaHostAlloc(&mg->samples_host, (size_t)g * MG_SAMPLES * sizeof(Sample), 0) != cudaSuccess) {
    cudaGetLastError();
    return bail(FS_E_OOM);
  }
  *out = mg;
  return FS_OK;
}

int fs_mg_destroy(fs_mg* mg) {
  if (!mg) return FS_OK;
  for (int i = 0; i < mg->g; ++i) {
    if (!mg->s[i]) continue;
    cudaSetDevice(mg->dev[i]);
    fs_synchronize(mg->s[i]);
    if (mg->inbox[i]) fs_free(mg->s[i], mg->inbox[i]);
    for (void* p : {mg->spl_keys[i], mg->spl_gpos[i], static_cast<void*>(mg->samples_dev[i])})
      if (p) cudaFree(p);
    fs_destroy(mg->s[i]);
  }
  if (mg->samples_host) cudaFreeHost(mg->samples_host);
  cudaGetLastError();
  delete mg;
  return FS_OK;
}

const char* fs_mg_last_error(const fs_mg* mg) { return mg ? mg->err.c_str() : ""; }

namespace {
int mg_entry(fs_mg* mg, int dtype, void* const* shards, const uint32_t* const* vals, bool payload,
             const uint64_t* shard_n, void* const* out, uint32_t* const* out_vals, const uint64_t* out_cap,
             uint64_t* out_n) {
  if (!mg) return FS_E_INVALID;
  if (dtype < FS_U32 || dtype > FS_F64) return mg_fail(mg, FS_E_INVALID, "unknown dtype %d", dtype);
  if (!shards || !shard_n || !out || !out_cap || !out_n || (payload && !out_vals))
    return mg_fail(mg, FS_E_INVALID, "NULL argument");
  uint64_t total = 0;
  for (int i = 0; i < mg->g; ++i) {
    if (shard_n[i] && !shards[i]) return mg_fail(mg, FS_E_INVALID, "shard %d is NULL", i);
    if (payload && vals && shard_n[i] && !vals[i]) return mg_fail(mg, FS_E_INVALID, "values of shard %d are NULL", i);
    total += shard_n[i];
  }
  for (int i = 0; i < mg->g; ++i) out_n[i] = 0;
  if (total == 0) return FS_OK;
  if (payload && !vals && total > (1ull << 32))
    return mg_fail(mg, FS_E_INVALID, "%llu keys: global positions past 2^32 do not fit u32",
                   (unsigned long long)total);
#define MG_CALL(K, XF) mg_sort<K, XF>(mg, dtype, shards, vals, payload, shard_n, out, out_vals, out_cap, out_n)
  switch (dtype) {
    case FS_U32: return MG_CALL(uint32_t, XF_NONE);
    case FS_I32: return MG_CALL(uint32_t, XF_SIGN);
    case FS_F32: return MG_CALL(uint32_t, XF_FLOAT);
    case FS_U64: return MG_CALL(uint64_t, XF_NONE);
    case FS_I64: return MG_CALL(uint64_t, XF_SIGN);
    default: return MG_CALL(uint64_t, XF_FLOAT);
  }
#undef MG_CALL
}
}  // namespace

int fs_mg_sort_keys(fs_mg* mg, int dtype, void* const* shards, const uint64_t* shard_n, void* const* out,
                    const uint64_t* out_cap, uint64_t* out_n) {
  return mg_entry(mg, dtype, shards, nullptr, false, shard_n, out, nullptr, out_cap, out_n);
}

int fs_mg_sort_pairs(fs_mg* mg, int dtype, void* const* shards, const uint32_t* const* vals,
                     const uint64_t* shard_n, void* const* out, uint32_t* const* out_vals, const uint64_t* out_cap,
                     uint64_t* out_n) {
  return mg_entry(mg, dtype, shards, vals, true, shard_n, out, out_vals, out_cap, out_n);
}

}  // extern "C"
