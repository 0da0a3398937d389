// Host-side helpers: status strings, SM-count cache, tensor-map cache.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "lk_host.h"

#include <stdlib.h>

namespace lk {

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool pdl_enabled() {
  static int v = [] {
    const char* e = getenv("LITEKERN_PDL");
    return (e && atoi(e) == 0) ? 0 : 1;
  }();
  return v != 0;
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

namespace {

struct MapKey {
  const void* base;
  int64_t num_slots;
  int h_kv, d, dtype, box_slots, box_heads, dev;
  bool operator==(const MapKey& o) const {
    return base == o.base && num_slots == o.num_slots && h_kv == o.h_kv && d == o.d &&
           dtype == o.dtype && box_slots == o.box_slots && box_heads == o.box_heads &&
           dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.base);
    h ^= static_cast<size_t>(k.num_slots) * 0x9E3779B97F4A7C15ull;
    h ^= (static_cast<size_t>(k.h_kv) << 1) ^ (static_cast<size_t>(k.d) << 9) ^
         (static_cast<size_t>(k.dtype) << 20) ^ (static_cast<size_t>(k.box_slots) << 24) ^
         (static_cast<size_t>(k.box_heads) << 32) ^ (static_cast<size_t>(k.dev) << 40);
    return h;
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int load_encode() {
  if (g_encode) return LK_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return LK_ERR_DRIVER;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return LK_OK;
}

}  // namespace

int get_kv_tensor_map(CUtensorMap* out, const void* base, int64_t num_slots, int H_kv, int D,
                      int dtype, int box_slots, int box_heads) {
  if (dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) return LK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return LK_ERR_ALIGNMENT;
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{base, num_slots, H_kv, D, dtype, box_slots, box_heads, dev};
  std::lock_guard<std::mutex> lock(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return LK_OK;
  }
  int rc = load_encode();
  if (rc != LK_OK) return rc;
  const uint64_t esz = 2;
  // dims: (d, slot, head); the slot stride exceeds the head stride, which
  // is what puts each head's rows contiguously in shared memory.
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(num_slots),
                        static_cast<cuuint64_t>(H_kv)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(H_kv) * D * esz,
                           static_cast<cuuint64_t>(D) * esz};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_slots),
                       static_cast<cuuint32_t>(box_heads)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap map;
  CUresult r = g_encode(&map,
                        dtype == LK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return LK_ERR_DRIVER;
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, map);
  *out = map;
  return LK_OK;
}

}  // namespace lk

extern "C" int lk_version(void) { return 100; }

extern "C" const char* lk_status_string(int code) {
  switch (code) {
    case LK_OK: return "ok";
    case LK_ERR_INVALID_ARG: return "litekern: invalid argument";
    case LK_ERR_UNSUPPORTED: return "litekern: unsupported shape or dtype";
    case LK_ERR_ALIGNMENT: return "litekern: pointer or stride not 16-byte aligned";
    case LK_ERR_WORKSPACE: return "litekern: workspace missing, misaligned or too small";
    case LK_ERR_CUDA: return "litekern: CUDA launch error";
    case LK_ERR_DRIVER: return "litekern: tensor-map creation failed in the CUDA driver";
    case LK_ERR_TOO_LARGE:
      return "litekern: problem exceeds the static scratch of the allocation-free entry point";
    default: return "litekern: unknown status";
  }
}
