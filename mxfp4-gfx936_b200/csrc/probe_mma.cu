// libmxfp4_b200_probe.so: the tensor-core rate probe behind the benchmark's
// FP4 (and cross-checking BF16) roofline denominators.  See
// include/mxfp4_b200_probe.h for the contract.
#include <string>

#include "gemm_w4a4.cuh"  // descriptors and MMA wrappers shared with the W4A4 GEMM
#include "mxfp4_b200_probe.h"

using namespace mx;

namespace {

constexpr int kProbeABytes = 128 * 128;            // 128 rows x 128 B (one 128B-swizzle atom column)
constexpr int kProbeBBytes = 256 * 128;            // 256 rows x 128 B
constexpr int kProbeSfBytes = 3 * 512;             // SFA chunk + two SFB chunks
constexpr uint32_t kProbeSfaCol = 256, kProbeSfbCol = 264;  // their TMEM columns, after the accumulator
constexpr int kProbeOffBar = kProbeABytes + kProbeBBytes + kProbeSfBytes;
constexpr int kProbeSmem = kProbeOffBar + 64 + 1024;
constexpr int64_t kProbeWaitNs = 10000000000LL;    // 10 s: the longest allowed probe runs ~0.1 s

__device__ __forceinline__ uint64_t probe_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

template <int KIND>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int iters) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a = smem;
  uint8_t* b = smem + kProbeABytes;
  uint8_t* sf = b + kProbeBBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kProbeOffBar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int warp = threadIdx.x >> 5;

  // operands: varied bit patterns (BF16 magnitudes below 2; any E2M1 code),
  // every scale factor 2^0, so the tensor cores see realistic data
  uint32_t* words = reinterpret_cast<uint32_t*>(smem);
  for (int i = threadIdx.x; i < (kProbeABytes + kProbeBBytes) / 4; i += blockDim.x) {
    uint32_t h = mix32(static_cast<uint32_t>(i) * 2654435761u + blockIdx.x);
    if (KIND == MXFP4_PROBE_BF16) h &= 0xBFFFBFFFu;
    words[i] = h;
  }
  for (int i = threadIdx.x; i < kProbeSfBytes / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sf)[i] = 0x7F7F7F7Fu;
  fence_proxy_async();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    const uint64_t adesc = desc_sw128(smem_u32(a));
    const uint64_t bdesc = desc_sw128(smem_u32(b));
    if (KIND == MXFP4_PROBE_MXF4) {
      tmem_cp_32x128b_warpx4(tmem + kProbeSfaCol, desc_sf_chunk(smem_u32(sf)));
      tmem_cp_32x128b_warpx4(tmem + kProbeSfbCol, desc_sf_chunk(smem_u32(sf + 512)));
      tmem_cp_32x128b_warpx4(tmem + kProbeSfbCol + 4, desc_sf_chunk(smem_u32(sf + 1024)));
      const uint32_t idesc = idesc_mxf4(128, 256);
      for (int i = 0; i < iters; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          umma_mxf4(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, tmem + kProbeSfaCol, tmem + kProbeSfbCol, (i | j) != 0);
    } else {
      const uint32_t idesc = idesc_f16(1, 128, 256);
      for (int i = 0; i < iters; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) umma_f16(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, (i | j) != 0);
    }
    umma_commit(bar);
    const uint64_t t0 = probe_ns();
    while (!mbar_try_wait(bar, 0)) {
      if (static_cast<int64_t>(probe_ns() - t0) > kProbeWaitNs) {
        record_error(MXFP4_ERR_TIMEOUT);
        break;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace

extern "C" int mxfp4_probe_mma_rate(int kind, int iters, float* ms, double* flops, void* stream) {
  if ((kind != MXFP4_PROBE_BF16 && kind != MXFP4_PROBE_MXF4) || iters < 1 || iters > 1000000 || !ms || !flops)
    return MXFP4_ERR_INVALID_ARGUMENT;
  int dev = 0;
  cudaDeviceProp prop;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return MXFP4_ERR_CUDA;
  if (prop.major != 10) return MXFP4_ERR_UNSUPPORTED_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = kind == MXFP4_PROBE_MXF4 ? mma_rate_kernel<MXFP4_PROBE_MXF4> : mma_rate_kernel<MXFP4_PROBE_BF16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem) != cudaSuccess)
    return MXFP4_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_status, &zero, sizeof(int)) != cudaSuccess) return MXFP4_ERR_CUDA;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return MXFP4_ERR_CUDA;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return MXFP4_ERR_CUDA;
  }
  cudaEventRecord(e0, s);
  kern<<<prop.multiProcessorCount, 128, kProbeSmem, s>>>(iters);
  cudaError_t err = cudaGetLastError();
  cudaEventRecord(e1, s);
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float elapsed = 0.0f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&elapsed, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (err != cudaSuccess) return MXFP4_ERR_CUDA;
  int status = 0;
  if (cudaMemcpyFromSymbol(&status, g_status, sizeof(int)) != cudaSuccess) return MXFP4_ERR_CUDA;
  if (status != 0) return status;
  const double k_per_mma = kind == MXFP4_PROBE_MXF4 ? 64.0 : 16.0;
  *ms = elapsed;
  *flops = static_cast<double>(prop.multiProcessorCount) * iters * 4 * 2.0 * 128 * 256 * k_per_mma;
  return MXFP4_OK;
}
