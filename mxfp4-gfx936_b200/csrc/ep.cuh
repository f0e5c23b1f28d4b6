// Expert-parallel MoE layer across the GPUs of one node, one process per GPU,
// without NCCL and without a host round trip.  Rank r owns experts
// [r*E/G, (r+1)*E/G) and its own tokens.  Every rank's buffers below are
// mapped into every other rank (CUDA IPC), so these kernels read and write
// peers' memory directly over NVLink:
//   counts[G][E]   route counts: row s written by rank s into every rank
//   xr[cap, H]     owner's activations in routed order (every local expert
//                  padded to 32 rows), written by the sources' dispatch
//   wr[cap]        route weight of each xr row (FP32)
//   yr[cap, H]     owner's weighted down-projection rows, read back by the
//                  sources' combine
// Layer: count -> barrier -> plan (every rank derives every owner's block
// layout from the same count matrix) + stable local routing -> dispatch
// (push rows into the owners' xr) -> barrier -> gate_up and down GEMMs on the
// owner (the single-GPU routed kernels over the plan's route chunks, one
// route per row) -> barrier -> combine
// (pull the top_k rows of each token, FP32 sum in slot order: the single-GPU
// combine's order, so the result is bit-identical to the single-GPU layer).
#pragma once

#include "elementwise.cuh"
#include "gemm.cuh"

namespace mx {

constexpr int kEpMaxRanks = 8;
constexpr int kEpBlock = 32;       // padding of every local expert's rows for the routed tensor-memory GEMM
constexpr int kEpPairBlock = 256;  // ... for the CTA-pair GEMM (its M): many routes per expert
constexpr int kEpChunkRows = 256;  // a route chunk of the routed GEMM: at most 256 rows (its N)

struct EpPeers {
  void* p[kEpMaxRanks];
};

// Local per-expert route counts -> row `rank` of every rank's count matrix.
__global__ void __launch_bounds__(1024) ep_count_kernel(const void* __restrict__ ids, int ids_dtype, int64_t routes,
                                                        int num_experts, int rank, int world, EpPeers counts) {
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  // ids in batches of 8 per thread, all loads issued before the atomics: one
  // memory latency per batch instead of one per route
  constexpr int kBatch = 8;
  for (int64_t base = threadIdx.x; base < routes; base += static_cast<int64_t>(blockDim.x) * kBatch) {
    int e[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t r = base + static_cast<int64_t>(u) * blockDim.x;
      e[u] = r < routes ? load_expert(ids, ids_dtype, r) : -1;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (e[u] >= 0 && e[u] < num_experts) atomicAdd(&hist[e[u]], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < world * num_experts; i += blockDim.x) {
    const int j = i / num_experts, e = i % num_experts;
    static_cast<int32_t*>(counts.p[j])[rank * num_experts + e] = hist[e];
  }
}

// Exclusive scan over the 1024 threads of the block (one value per thread).
__device__ __forceinline__ int block_excl_scan_1024(int v, int* warp_tmp, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tmp[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int w = warp_tmp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= o) wi += y;
    }
    warp_tmp[lane] = wi - w;
    if (lane == 31) warp_tmp[32] = wi;
  }
  __syncthreads();
  const int r = incl - v + warp_tmp[wid];
  total = warp_tmp[32];
  __syncthreads();
  return r;
}

// One CTA of 1024 threads, thread e = global expert e.  From the complete
// count matrix: send_base[e] (first row of this rank's routes to expert e in
// the owner's xr), lstart[e] (first position of expert e in this rank's
// stable local order), and, for this rank as owner, the per-block local
// expert ids, the used length and the row ids of the down GEMM (row id =
// the row itself, pads = cap: not a route).
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t* __restrict__ counts, int num_experts, int world,
                                                       int rank, int32_t* __restrict__ send_base,
                                                       int32_t* __restrict__ lstart, int32_t* __restrict__ block_expert,
                                                       int32_t* __restrict__ num_post_padded, int32_t* __restrict__ rid,
                                                       int cap, int cap_blocks, int4* __restrict__ chunks,
                                                       int32_t* __restrict__ num_chunks, int blk) {
  __shared__ int warp_tmp[33];
  __shared__ int scan_nb[kMaxExperts];
  __shared__ int nb_s[kMaxExperts];
  __shared__ int tot_s[kMaxExperts];
  const int e = threadIdx.x;
  const int el = num_experts / world;
  int total = 0, below = 0, own = 0;
  if (e < num_experts) {
    for (int s = 0; s < world; ++s) {
      const int c = counts[s * num_experts + e];
      total += c;
      if (s < rank) below += c;
      if (s == rank) own = c;
    }
  }
  const int nb = (total + blk - 1) / blk;
  int t_nb, t_own;
  const int sc = block_excl_scan_1024(nb, warp_tmp, t_nb);
  const int ls = block_excl_scan_1024(own, warp_tmp, t_own);
  if (e < num_experts) {
    scan_nb[e] = sc;
    nb_s[e] = nb;
    tot_s[e] = total;
  }
  __syncthreads();
  if (e < num_experts) {
    const int first = (e / el) * el;  // the owner's first expert
    const int bstart = sc - scan_nb[first];
    send_base[e] = bstart * blk + below;
    lstart[e] = ls;
  }
  // owner side: this rank's experts [rank*el, rank*el + el)
  const int e0 = rank * el;
  const int used = (e0 + el - 1 < num_experts) ? scan_nb[e0 + el - 1] + nb_s[e0 + el - 1] - scan_nb[e0] : 0;
  if (threadIdx.x == 0) num_post_padded[0] = used * blk;
  for (int b = used + threadIdx.x; b < cap_blocks; b += blockDim.x) block_expert[b] = -1;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int x = wid; x < el; x += 32) {
    const int g = e0 + x;
    const int bstart = scan_nb[g] - scan_nb[e0];
    for (int b = lane; b < nb_s[g]; b += 32) block_expert[bstart + b] = x;
    const int base = bstart * blk;
    for (int i = lane; i < nb_s[g] * blk; i += 32) rid[base + i] = i < tot_s[g] ? base + i : cap;
  }
  // route chunks of the owner's experts for the routed GEMMs: {first row,
  // rows, local expert, 0}, at most kEpChunkRows rows each
  __syncthreads();
  const bool mine = e >= e0 && e < e0 + el;
  const int chunk_blocks = kEpChunkRows / blk;
  const int nc = mine ? (nb + chunk_blocks - 1) / chunk_blocks : 0;
  int t_nc;
  const int cb = block_excl_scan_1024(nc, warp_tmp, t_nc);
  if (threadIdx.x == 0) num_chunks[0] = t_nc;
  if (mine) {
    const int bstart = scan_nb[e] - scan_nb[e0];
    for (int i = 0; i < nc; ++i) {
      const int b0 = i * chunk_blocks;
      const int nbl = min(chunk_blocks, nb - b0);
      chunks[cb + i] = make_int4((bstart + b0) * blk, nbl * blk, e - e0, 0);
    }
  }
}

// One warp per position p of this rank's stable expert order: route i =
// sorted[p] of expert e goes to owner d = e / el at row send_base[e] + p -
// lstart[e]; the warp copies x[i / top_k] there (16 B per lane, whole rows)
// with the route weight, and records (d, row) for the combine.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const uint4* __restrict__ x, int64_t row_vecs,
                                                          const int32_t* __restrict__ sorted,
                                                          const int32_t* __restrict__ bexp,
                                                          const int32_t* __restrict__ num_valid,
                                                          const int32_t* __restrict__ send_base,
                                                          const int32_t* __restrict__ lstart, const void* tw,
                                                          int w_dtype, int top_k, int el, EpPeers xr, EpPeers wr,
                                                          int32_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int valid = num_valid[0];
  for (int64_t p = warp_id; p < valid; p += warps) {
    const int i = sorted[p];
    const int e = bexp[p];
    const int d = e / el;
    const int row = send_base[e] + static_cast<int>(p) - lstart[e];
    const uint4* src = x + static_cast<int64_t>(i / top_k) * row_vecs;
    uint4* out = static_cast<uint4*>(xr.p[d]) + static_cast<int64_t>(row) * row_vecs;
    // 8 loads in flight per lane before the (remote) stores
    for (int64_t v0 = lane; v0 < row_vecs; v0 += 32 * 8) {
      uint4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (v0 + 32 * u < row_vecs) buf[u] = src[v0 + 32 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (v0 + 32 * u < row_vecs) out[v0 + 32 * u] = buf[u];
    }
    if (lane == 0) {
      static_cast<float*>(wr.p[d])[row] = load_weight(tw, w_dtype, i);
      dst[i] = (d << 24) | row;
    }
  }
}

// out[t] = bf16(sum_j float(y_j)) over the token's top_k routes in slot order,
// y_j read from the owner's yr row recorded by the dispatch (dropped routes,
// dst = -1, contribute nothing).
__global__ void __launch_bounds__(256) ep_combine_kernel(const int32_t* __restrict__ dst, EpPeers yr,
                                                         __nv_bfloat16* __restrict__ out, int64_t num_tokens,
                                                         int top_k, int64_t hidden) {
  const int64_t vec_per_row = hidden / 8;
  const int64_t total = num_tokens * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row, v = i % vec_per_row;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    // slots in batches of 8: the route codes, then the rows, are loaded before
    // any sum; the sum runs in slot order
    for (int j0 = 0; j0 < top_k; j0 += 8) {
      int code[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) code[u] = j0 + u < top_k ? dst[t * top_k + j0 + u] : -1;
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        q[u] = make_uint4(0, 0, 0, 0);
        if (code[u] >= 0)
          q[u] = *(reinterpret_cast<const uint4*>(yr.p[code[u] >> 24]) +
                   static_cast<int64_t>(code[u] & 0xFFFFFF) * vec_per_row + v);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (code[u] < 0) continue;
        const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[2 * c] += __uint_as_float(w[c] << 16);
          acc[2 * c + 1] += __uint_as_float(w[c] & 0xFFFF0000u);
        }
      }
    }
    uint4 o;
    o.x = f32x2_to_bf16x2(acc[0], acc[1]);
    o.y = f32x2_to_bf16x2(acc[2], acc[3]);
    o.z = f32x2_to_bf16x2(acc[4], acc[5]);
    o.w = f32x2_to_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * hidden + v * 8) = o;
  }
}

}  // namespace mx
