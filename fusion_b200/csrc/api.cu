// Library-wide host plumbing: error strings, launch checks, SM count and the TMA
// tensor-map encoder (cuTensorMapEncodeTiled through cudaGetDriverEntryPoint).
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <set>
#include <tuple>

#include "host_util.h"

namespace fus {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return FUS_OK;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

int ensure_smem_attr(const void* fn, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;  // (kernel, device, bytes)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(fn, dev, bytes);
  if (done.count(key)) return FUS_OK;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "%s attr: %s", what, cudaGetErrorString(e));
  done.insert(key);
  return FUS_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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

int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                      uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FUS_E_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base) || (ld * 2) % 16)
    return set_error(FUS_E_INVALID, "tensor map: base and row pitch must be 16-byte aligned");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FUS_E_INVALID, "cuTensorMapEncodeTiled failed (%d): inner=%llu rows=%llu",
                     (int)r, (unsigned long long)inner, (unsigned long long)rows);
  return FUS_OK;
}

int make_tmap_store_2d(CUtensorMap* m, const void* base, bool f32, uint64_t inner, uint64_t rows,
                       uint64_t ld, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FUS_E_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const uint64_t es = f32 ? 4 : 2;
  if (!aligned16(base) || (ld * es) % 16 || (box_inner * es) % 16)
    return set_error(FUS_E_INVALID, "store tensor map: base, pitch and box must be 16-byte aligned");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FUS_E_INVALID, "cuTensorMapEncodeTiled (store) failed (%d)", (int)r);
  return FUS_OK;
}

}  // namespace fus

extern "C" int fus_version(void) { return 1; }
extern "C" const char* fus_last_error(void) { return fus::g_last_error; }
extern "C" int fus_num_sms(void) { return fus::num_sms(); }
