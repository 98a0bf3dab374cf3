// Per-row FP8 (e4m3) quantization of a weight matrix for the fp8-weight decode path.
//
// Row r of W [rows, cols] (fp16/bf16, pitch ld_src elements) becomes
//   scale[r] = absmax(W[r, :]) / 448          (448 = largest finite e4m3; 1 for an all-zero row)
//   q[r, c]  = RN_satfinite_e4m3(W[r, c] / scale[r])
// with IEEE fp32 division, so a CPU restatement reproduces every code and scale bit for bit.
// The fused kernel multiplies each output feature's fp32 sum by its row scale, which
// factors out of the K sum: y = sum_k x_k (q_k s) = s * sum_k x_k q_k.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/ffn_b200.h"

namespace ffnb200 {
namespace {

__device__ __forceinline__ float load_elem(const uint16_t* p, int bf16) {
  const uint16_t b = *p;
  return bf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
}

// One warp per row (grid-stride); pass 1 reduces |x|, pass 2 writes the codes.
__global__ void quantize_rows_e4m3(const uint16_t* __restrict__ src, int64_t ld_src, int bf16, int64_t rows,
                                   int64_t cols, uint8_t* __restrict__ dst, int64_t ld_dst, float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const uint16_t* row = src + r * ld_src;
    float amax = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(load_elem(row + c, bf16)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
    if (lane == 0) scales[r] = scale;
    uint8_t* out = dst + r * ld_dst;
    for (int64_t c = 2 * lane; c < cols; c += 64) {
      const float a = __fdiv_rn(load_elem(row + c, bf16), scale);
      const float b = c + 1 < cols ? __fdiv_rn(load_elem(row + c + 1, bf16), scale) : 0.0f;
      uint16_t q;  // first source -> upper byte: element c+1 high, element c low (memory order)
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(q) : "f"(b), "f"(a));
      out[c] = static_cast<uint8_t>(q & 0xFFu);
      if (c + 1 < cols) out[c + 1] = static_cast<uint8_t>(q >> 8);
    }
  }
}

}  // namespace
}  // namespace ffnb200

extern "C" int ffn_b200_quantize_fp8_rows(const void* src, int64_t ld_src, int32_t dtype, int64_t rows, int64_t cols,
                                          void* dst, int64_t ld_dst, float* scales, void* stream) {
  if (!src || !dst || !scales || rows <= 0 || cols <= 0 || ld_src < cols || ld_dst < cols) return FFN_B200_ERR_INVALID;
  if (dtype != FFN_B200_F16 && dtype != FFN_B200_BF16) return FFN_B200_ERR_INVALID;
  const int threads = 256;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 4096) blocks = 4096;
  ffnb200::quantize_rows_e4m3<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(src), ld_src, dtype == FFN_B200_BF16 ? 1 : 0, rows, cols, static_cast<uint8_t*>(dst),
      ld_dst, scales);
  if (cudaGetLastError() != cudaSuccess) return FFN_B200_ERR_CUDA;
  return FFN_B200_OK;
}
