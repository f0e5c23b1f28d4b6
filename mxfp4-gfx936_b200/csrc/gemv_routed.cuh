// Routed GEMV: the routed op's and the MoE layer's GEMMs when there are few
// routes (decode batches).
//
// With a handful of routes per call every expert's weights serve one or two
// routes, so the tensor cores have almost nothing to multiply and the cost is
// reading and decoding the weights.  This kernel skips the routing pass and
// the routed-order copy: CTA (r, blk) takes route r = t * top_k + j, stages
// its activation row in shared memory, and each of its 8 warps computes one
// output of the route -- a weight row (GLU: the gate row and the up row of one
// intermediate column) of expert ids[r] against that row.  A lane takes the
// 32-value scale blocks b = lane, lane + 32, ... of the row: one 16-byte load
// of packed codes and one scale byte per block, the decode of the fused
// kernels (E2M1 -> BF16/FP16 times the E8M0 scale, exact), FP32 FMAs, then a
// butterfly sum over the lanes.  The result goes through the same epilogue
// chains as the grouped GEMMs: GLU bf16(bf16(silu(bf16 g)) * bf16 u); routed
// op: round, x a_scale, x b_scale[e], x route weight, each rounded to the
// output type (soft:487-494).  Routes to experts outside [0, E) are skipped
// (their rows of C are the zeros of C.zero_(); the MoE layer's combine skips
// them).
//
// The dot products are single FP32 reductions of the same exact products as
// the tensor-core paths, summed in another order, so results agree with them
// to FP32 rounding (well inside the BF16 output tolerance) and are
// deterministic; the op and the layer choose this kernel on the same route
// counts, so the layer equals the two-op composition bit for bit here too.
#pragma once

#include "elementwise.cuh"
#include "gemm_routed.cuh"
#include "gemm_small.cuh"

namespace mx {

constexpr int kMoeGemvMaxRoutes = 64;  // routes per call up to which the routed calls may use this kernel
constexpr int kMoeGemvWarps = 8;       // outputs (rows) per CTA

struct MoeGemvParams {
  int K;                      // reduction length (weights' K = activation columns)
  int rows;                   // outputs per route: GLU inter, plain N
  int num_experts;
  int top_k;                  // activation row of route r: r / top_k
  int num_routes;
  const void* x;              // activations (BF16 or FP16), row stride ldx elements
  int64_t ldx;
  const uint8_t* w;           // packed [E * w_rows_per_expert, K/2]
  int64_t w_rows_per_expert;
  int64_t ldw;                // bytes per weight row
  const uint8_t* w_scales;    // [E * w_rows_per_expert, K/32]
  int64_t lds;
  const void* ids;            // topk ids, route r at index r
  int ids_dtype;
  int glu_inter;              // GLU: the up row of column n is glu_inter + n
  void* out;                  // route r's outputs at out + r * ldo (elements of out_dtype)
  int64_t ldo;
  int out_dtype;
  const float* a_scale;       // routed op: NULL means 1 (and b_scale unused)
  const float* b_scale;
  const void* topk_w;         // route weights, route r at index r
  int w_dtype;
  int mul_w;
};

// One row's partial dot product over the lane's scale blocks.
template <bool FP16>
__device__ __forceinline__ float moe_gemv_row(const MoeGemvParams& p, int64_t wrow_idx, const uint8_t* xs, int lane) {
  float acc[kGemvMaxRows];
#pragma unroll
  for (int m = 0; m < kGemvMaxRows; ++m) acc[m] = 0.0f;
  const uint8_t* wrow = p.w + wrow_idx * p.ldw;
  const uint8_t* srow = p.w_scales + wrow_idx * p.lds;
  const int nblk = p.K / 32;
  for (int b = lane; b < nblk; b += 32) {
    const uint32_t code = __ldg(srow + b);
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(wrow + b * 16));
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 d;
      if (FP16) d = decode8_f16(qw[j], e8m0_to_f32(code));
      else d = decode8_bf16(qw[j], e8m0_to_bf16x2(code));
      const uint32_t w8[4] = {d.x, d.y, d.z, d.w};
      gemv_fma8<1, FP16>(acc, w8, xs, p.K * 2, b * 32 + 8 * j);
    }
  }
  float v = acc[0];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

template <int EPI, bool FP16>
__global__ void __launch_bounds__(32 * kMoeGemvWarps) mxfp4_moe_gemv_kernel(const MoeGemvParams p) {
  extern __shared__ __align__(16) uint8_t xs[];  // the route's activation row, K x 16-bit
  const int r = blockIdx.x;
  const int e = load_expert(p.ids, p.ids_dtype, r);
  if (e < 0 || e >= p.num_experts) return;  // uniform over the CTA
  const uint4* xrow = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) +
                                                     static_cast<int64_t>(r / p.top_k) * p.ldx * 2);
  for (int i = threadIdx.x; i < p.K / 8; i += blockDim.x) reinterpret_cast<uint4*>(xs)[i] = xrow[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.y * kMoeGemvWarps + (threadIdx.x >> 5);
  if (n >= p.rows) return;
  const int64_t base = static_cast<int64_t>(e) * p.w_rows_per_expert;
  if (EPI == EPI_GLU) {
    const float g = moe_gemv_row<false>(p, base + n, xs, lane);
    const float u = moe_gemv_row<false>(p, base + p.glu_inter + n, xs, lane);
    if (lane == 0) {
      const float gb = round_bf16(g), ub = round_bf16(u);
      const float h = round_bf16(gb / (1.0f + expf(-gb))) * ub;
      static_cast<__nv_bfloat16*>(p.out)[static_cast<int64_t>(r) * p.ldo + n] = __float2bfloat16_rn(h);
    }
  } else {
    float x = moe_gemv_row<FP16>(p, base + n, xs, lane);
    if (lane == 0) {
      const bool scales = p.a_scale != nullptr;
      const float asc = scales ? p.a_scale[0] : 1.0f;
      const float bsc = scales ? p.b_scale[e] : 1.0f;
      const float rw = p.mul_w ? load_weight(p.topk_w, p.w_dtype, r) : 1.0f;
      const int64_t o = static_cast<int64_t>(r) * p.ldo + n;
      if (p.out_dtype == MXFP4_DTYPE_F32) {
        if (scales) x = x * asc * bsc;
        if (p.mul_w) x = x * rw;
        static_cast<float*>(p.out)[o] = x;
      } else if (p.out_dtype == MXFP4_DTYPE_BF16) {
        x = rt_round<MXFP4_DTYPE_BF16>(x);
        if (scales) {
          x = rt_round<MXFP4_DTYPE_BF16>(x * asc);
          x = rt_round<MXFP4_DTYPE_BF16>(x * bsc);
        }
        if (p.mul_w) x = rt_round<MXFP4_DTYPE_BF16>(x * rw);
        static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(x);
      } else {
        x = rt_round<MXFP4_DTYPE_F16>(x);
        if (scales) {
          x = rt_round<MXFP4_DTYPE_F16>(x * asc);
          x = rt_round<MXFP4_DTYPE_F16>(x * bsc);
        }
        if (p.mul_w) x = rt_round<MXFP4_DTYPE_F16>(x * rw);
        static_cast<__half*>(p.out)[o] = __float2half_rn(x);
      }
    }
  }
}

}  // namespace mx
