// Host-side runtime of the C ABI: error messages, dispatch counters, device
// queries and a small cache of TMA tensor maps.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.cuh"

namespace ss {

namespace {
thread_local std::string g_last_error;
std::mutex g_stats_mu;
std::map<std::string, long long> g_stats;
}  // namespace

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(SS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return SS_OK;
}

void count_dispatch(const char* name) {
  std::lock_guard<std::mutex> lk(g_stats_mu);
  g_stats[name] += 1;
}

namespace {
std::atomic<int*> g_error_sink{nullptr};
}  // namespace

int* error_sink() { return g_error_sink.load(std::memory_order_acquire); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int cached[64] = {0};
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

// ----------------------------------------------------------- tensor maps
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

struct MapKey {
  int dev, dtype;
  const void* base;
  uint64_t inner, rows, pairs, row_stride, pair_stride;
  uint32_t bi, br;
  bool operator<(const MapKey& o) const {
    return std::tie(dev, dtype, base, inner, rows, pairs, row_stride, pair_stride, bi, br) <
           std::tie(o.dev, o.dtype, o.base, o.inner, o.rows, o.pairs, o.row_stride,
                    o.pair_stride, o.bi, o.br);
  }
};
std::mutex g_map_mu;
std::map<MapKey, CUtensorMap*> g_maps;
}  // namespace

const CUtensorMap* tmap_3d_f16_sw128(const void* base, uint64_t inner, uint64_t rows,
                                     uint64_t pairs, uint64_t pair_stride_bytes,
                                     uint32_t box_inner, uint32_t box_rows) {
  return tmap_3d_sw128(base, SS_F16, inner, rows, pairs, inner * 2, pair_stride_bytes, box_inner,
                       box_rows);
}

const CUtensorMap* tmap_3d_sw128(const void* base, int dtype, uint64_t inner, uint64_t rows,
                                 uint64_t pairs, uint64_t row_stride_bytes,
                                 uint64_t pair_stride_bytes, uint32_t box_inner,
                                 uint32_t box_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{dev, dtype, base, inner, rows, pairs, row_stride_bytes, pair_stride_bytes,
             box_inner, box_rows};
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) return it->second;
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    fail(SS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    return nullptr;
  }
  if (g_maps.size() > 4096) {  // bound host memory for long-lived processes
    for (auto& kv : g_maps) delete kv.second;
    g_maps.clear();
  }
  auto* m = new CUtensorMap;
  cuuint64_t dims[3] = {inner, rows, pairs};
  cuuint64_t strides[2] = {row_stride_bytes, pair_stride_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == SS_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == SS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    delete m;
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", int(r));
    fail(SS_ERR_CUDA, buf);
    return nullptr;
  }
  g_maps[key] = m;
  return m;
}

}  // namespace ss

extern "C" {

int ss_abi_version(void) { return 101; }

const char* ss_last_error(void) { return ss::g_last_error.c_str(); }

int ss_device_sm_count(void) { return ss::sm_count(); }

int ss_set_error_sink(int* host_word) {
  if (!host_word) {
    ss::g_error_sink.store(nullptr, std::memory_order_release);
    return SS_OK;
  }
  void* dptr = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&dptr, host_word, 0);
  if (e != cudaSuccess || !dptr) {
    cudaGetLastError();
    return ss::fail(SS_ERR_BAD_ARG, std::string("ss_set_error_sink: not page-locked host memory "
                                                "visible to the device: ") + cudaGetErrorString(e));
  }
  ss::g_error_sink.store(static_cast<int*>(dptr), std::memory_order_release);
  return SS_OK;
}

int ss_kernel_stats(char* buf, size_t buf_len) {
  std::lock_guard<std::mutex> lk(ss::g_stats_mu);
  std::string s;
  for (auto& kv : ss::g_stats) s += kv.first + "=" + std::to_string(kv.second) + "\n";
  if (buf && buf_len) {
    size_t n = s.size() < buf_len - 1 ? s.size() : buf_len - 1;
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return static_cast<int>(s.size());
}

void ss_reset_kernel_stats(void) {
  std::lock_guard<std::mutex> lk(ss::g_stats_mu);
  ss::g_stats.clear();
}

}  // extern "C"
