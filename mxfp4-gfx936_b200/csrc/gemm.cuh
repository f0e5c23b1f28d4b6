// Shared pieces of the tcgen05 GEMM kernels: operand and epilogue modes, the
// tile constants and accumulator layout the pair kernel uses, and the
// epilogue helpers (weight loads of any dtype, 32-column row stores, the
// barrier drain used on the abort path).
#pragma once

#include "common.cuh"

namespace mx {

enum AMode : int { A_TMA = 0, A_GATHER = 1 };
enum BMode : int { B_DECODE = 0, B_TMA = 1 };
enum EpiMode : int { EPI_DENSE = 0, EPI_MOE = 1, EPI_GLU = 2 };

constexpr int kAccCols = 256;           // FP32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;  // two accumulators: epilogue of tile i overlaps tile i+1


__device__ __forceinline__ float load_weight(const void* w, int dtype, int64_t i) {
  if (dtype == MXFP4_DTYPE_F32) return static_cast<const float*>(w)[i];
  if (dtype == MXFP4_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
  return __half2float(static_cast<const __half*>(w)[i]);
}

__device__ __forceinline__ void store_row32(void* out_row, int dtype, const float (&v)[32], int ncols,
                                            bool vec) {
  if (dtype == MXFP4_DTYPE_F32) {
    float* o = static_cast<float*>(out_row);
    if (vec && ncols >= 32) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) o[i] = v[i];
    }
    return;
  }
  uint32_t p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    p[i] = dtype == MXFP4_DTYPE_BF16 ? f32x2_to_bf16x2(v[2 * i], v[2 * i + 1])
                                     : f32x2_to_f16x2(v[2 * i], v[2 * i + 1]);
  if (vec && ncols >= 32) {
    uint4* o = static_cast<uint4*>(out_row);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  } else {
    uint16_t* o = static_cast<uint16_t*>(out_row);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncols) o[i] = static_cast<uint16_t>((p[i >> 1] >> ((i & 1) * 16)) & 0xFFFF);
  }
}

__device__ __forceinline__ int out_esize(int dtype) { return dtype == MXFP4_DTYPE_F32 ? 4 : 2; }

// Bounded wait that ignores the abort flag (used to drain in-flight work).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      record_error(MXFP4_ERR_TIMEOUT);
      return;
    }
  }
}

}  // namespace mx
