// Checkpoint ingest: FP8 (e4m3) block-scaled expert weights -> bf16.
//
// FP8 releases of DeepSeek-V3-style MoE checkpoints store each linear weight as e4m3
// with one fp32 `weight_scale_inv` per 128 x 128 block (value = fp8 * scale). The
// block's GEMMs run in bf16, so the weights are dequantised once at load:
//   dst[r, c] = bf16(float(src[r, c]) * scale[r / br, c / bc])
// One thread per 8 consecutive elements of a row (8-byte loads, 16-byte stores).
#include <cuda_fp8.h>

#include "common.cuh"
#include "host_util.h"

namespace fus {

__global__ void fp8_block_dequant_kernel(const uint8_t* __restrict__ src,
                                         const float* __restrict__ scale, long scale_ld,
                                         __nv_bfloat16* __restrict__ dst, long rows, int cols,
                                         int br, int bc) {
  const long nvec = rows * (long)(cols >> 3);
  for (long v = (long)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
       v += (long)gridDim.x * blockDim.x) {
    const long r = v / (cols >> 3);
    const int c = (int)(v - r * (cols >> 3)) * 8;
    const uint2 q = *reinterpret_cast<const uint2*>(src + r * cols + c);
    const float s = __ldg(scale + (r / br) * scale_ld + c / bc);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&q);
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      __nv_fp8_e4m3 x;
      x.__x = b[e];
      f[e] = static_cast<float>(x) * s;
    }
    *reinterpret_cast<uint4*>(dst + r * cols + c) = pack8(f);
  }
}

}  // namespace fus

using namespace fus;

extern "C" int fus_fp8_block_dequant(const void* src, const float* scale, long scale_ld,
                                     void* dst, long rows, int cols, int br, int bc,
                                     void* stream, int* status) {
  (void)status;
  if (!src || !scale || !dst || rows < 0 || cols <= 0 || cols % 8 || br < 1 || bc < 8 ||
      bc % 8 || scale_ld < (cols + bc - 1) / bc || ((uintptr_t)src & 7) || !aligned16(dst))
    return set_error(FUS_E_INVALID, "fp8_block_dequant: bad args");
  const long nvec = rows * (long)(cols / 8);
  if (nvec == 0) return FUS_OK;
  long grid = (nvec + 255) / 256;
  if (grid > (long)num_sms() * 16) grid = (long)num_sms() * 16;
  fp8_block_dequant_kernel<<<(int)grid, 256, 0, as_stream(stream)>>>(
      (const uint8_t*)src, scale, scale_ld, (__nv_bfloat16*)dst, rows, cols, br, bc);
  return check_launch("fp8_block_dequant");
}
