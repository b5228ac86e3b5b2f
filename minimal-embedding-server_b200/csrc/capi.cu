// Library-wide C ABI helpers and host utilities: version, status strings, device-error
// collection, TMA tensor-map encoding (through the driver entry point, so the library
// links only the CUDA runtime) and the per-device SM count.
#include <mutex>

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

bool make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize,
                 uint64_t rows, uint64_t cols, uint64_t pitch_elems, uint32_t box_rows,
                 uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || rows == 0 || cols == 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * (uint64_t)esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
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

}  // namespace mes_host

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
