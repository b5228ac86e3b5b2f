// Library-wide C ABI helpers and host utilities: version, status strings, device-error
// collection, TMA tensor-map encoding (through the driver entry point, so the library
// links only the CUDA runtime) and the per-device SM count.
#include <mutex>

#include <atomic>

#include "common.cuh"

extern "C" int mes_elementwise_take_error(int* code);
extern "C" int mes_gemm_take_error(int* code);
extern "C" int mes_attention_take_error(int* code);

namespace mes_host {

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

namespace {
// Encoded tensor maps of this thread, direct-mapped by their arguments.  A forward pass asks
// for the same maps every time (the caching allocator hands back the same buffers), so most
// launches skip the encode.
struct MapKey {
  const void* base;
  uint64_t rows, cols, pitch;
  uint32_t box_rows, box_cols;
  int dtype, swizzle;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && pitch == o.pitch &&
           box_rows == o.box_rows && box_cols == o.box_cols && dtype == o.dtype &&
           swizzle == o.swizzle;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCacheSize = 512;
thread_local MapEntry t_map_cache[kMapCacheSize];

inline uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h;
}
}  // namespace

bool make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize,
                 uint64_t rows, uint64_t cols, uint64_t pitch_elems, uint32_t box_rows,
                 uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  const MapKey key{base, rows, cols, pitch_elems, box_rows, box_cols, (int)dtype, (int)swizzle};
  uint64_t h = mix(mix(mix(reinterpret_cast<uintptr_t>(base), rows), cols), pitch_elems);
  h = mix(mix(mix(h, box_rows), box_cols), ((uint64_t)dtype << 8) | (uint64_t)swizzle);
  MapEntry& e = t_map_cache[h % kMapCacheSize];
  if (e.valid && e.key == key) {
    *map = e.map;
    return true;
  }
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || rows == 0 || cols == 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * (uint64_t)esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  e.key = key;
  e.map = *map;
  e.valid = true;
  return true;
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
      c = 148;
    counts[dev] = c;
  }
  return counts[dev];
}

// SMs left to other kernels running concurrently with the persistent kernels (an NCCL
// collective overlapped on another stream): persistent grids use the rest, so that none of
// their CTAs - each of which owns a fixed share of the tiles - waits for an SM.
static std::atomic<int> g_sm_reserve{0};

int persistent_ctas() {
  const int c = sm_count() - g_sm_reserve.load(std::memory_order_relaxed);
  return c < 2 ? 2 : c;
}

}  // namespace mes_host

extern "C" int mes_set_sm_reserve(int sms) {
  if (sms < 0 || sms > 64) return MES_ERR_INVALID;
  mes_host::g_sm_reserve.store(sms, std::memory_order_relaxed);
  return MES_OK;
}

extern "C" int mes_version(void) { return 100; }

extern "C" const char* mes_status_string(int status) {
  switch (status) {
    case MES_OK: return "ok";
    case MES_ERR_INVALID: return "invalid argument or unsupported shape";
    case MES_ERR_ALIGN: return "pointer or pitch not aligned as required";
    case MES_ERR_CUDA: return "CUDA runtime or driver call failed";
    case MES_ERR_TIMEOUT: return "a device-side wait exceeded its limit";
    case MES_ERR_UNSUPPORTED: return "unsupported device or feature";
    default: return "unknown status";
  }
}

extern "C" int mes_take_device_error(int* code) {
  if (!code) return MES_ERR_INVALID;
  *code = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return MES_ERR_CUDA;
  int (*fns[3])(int*) = {mes_elementwise_take_error, mes_gemm_take_error, mes_attention_take_error};
  for (auto f : fns) {
    int c = 0;
    int st = f(&c);
    if (st != MES_OK) return st;
    if (c != 0 && *code == 0) *code = c;
  }
  return MES_OK;
}
