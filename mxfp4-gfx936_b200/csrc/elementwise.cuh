// Bandwidth-bound kernels of the MXFP4 path:
//   K0  dequant        packed E2M1 + E8M0 -> F32 / BF16 / F16 (dequant_mxfp4, soft:277-307)
//   K4  routing        stable per-expert padded blocks (_make_routing, vllm:119-146)
//   K5  combine        sum over top-k routed rows (vllm:263-265)
//   --  cast           activation dtype conversion for the routed op (soft:473-475)
#pragma once

#include "common.cuh"

namespace mx {

// ---------------------------------------------------------------------------
// Dequant: a thread decodes one 32-bit packed word (8 values) per step, and
// the 32 lanes of a warp take 32 consecutive words, so every load (128 B of
// packed codes) and every store (512 B of BF16/FP16, 1 KB of FP32) of the warp
// is one contiguous segment.  Each thread walks 4 words spaced one warp-width
// apart per iteration for memory-level parallelism.
// ---------------------------------------------------------------------------
template <int OUT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ packed,
                                                      const uint8_t* __restrict__ scales,
                                                      void* __restrict__ out, int64_t num_blocks) {
  griddep_launch_dependents();  // the GEMM behind it may set up while this runs
  const int64_t num_words = num_blocks * 4;  // 4 words of 8 codes per 32-value scale block
  const uint32_t* words = reinterpret_cast<const uint32_t*>(packed);
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps_total = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp_global * 128; base < num_words; base += warps_total * 128) {
    uint32_t w[4], code[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t wi = base + lane + 32 * i;
      w[i] = wi < num_words ? __ldg(words + wi) : 0u;
      code[i] = wi < num_words ? __ldg(scales + (wi >> 2)) : 127u;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t wi = base + lane + 32 * i;
      if (wi >= num_words) break;
      if (OUT == MXFP4_DTYPE_BF16) {
        reinterpret_cast<uint4*>(out)[wi] = decode8_bf16(w[i], e8m0_to_bf16x2(code[i]));
      } else if (OUT == MXFP4_DTYPE_F16) {
        reinterpret_cast<uint4*>(out)[wi] = decode8_f16(w[i], e8m0_to_f32(code[i]));
      } else {
        const float sc = e8m0_to_f32(code[i]);
        uint32_t v[4];
        e2m1x8_to_bf16x8(w[i], v);
        float4* o = reinterpret_cast<float4*>(out) + 2 * wi;
        o[0] = make_float4(__uint_as_float(v[0] << 16) * sc, __uint_as_float(v[0] & 0xFFFF0000u) * sc,
                           __uint_as_float(v[1] << 16) * sc, __uint_as_float(v[1] & 0xFFFF0000u) * sc);
        o[1] = make_float4(__uint_as_float(v[2] << 16) * sc, __uint_as_float(v[2] & 0xFFFF0000u) * sc,
                           __uint_as_float(v[3] << 16) * sc, __uint_as_float(v[3] & 0xFFFF0000u) * sc);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// activation cast (A.to(C.dtype), soft:475): src dtype -> dst dtype, rounding.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) cast_kernel(const void* __restrict__ src, int src_dtype,
                                                   void* __restrict__ dst, int dst_dtype, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v;
    if (src_dtype == MXFP4_DTYPE_F32) v = static_cast<const float*>(src)[i];
    else if (src_dtype == MXFP4_DTYPE_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
    else v = __half2float(static_cast<const __half*>(src)[i]);
    if (dst_dtype == MXFP4_DTYPE_BF16) static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    else if (dst_dtype == MXFP4_DTYPE_F16) static_cast<__half*>(dst)[i] = __float2half_rn(v);
    else static_cast<float*>(dst)[i] = v;
  }
}

// Exact split of F16 / F32 activations into `parts` BF16 values whose sum is
// the input: hi = bf16(a), mid = bf16(a - hi), lo = bf16(a - hi - mid).  An F16
// value (11 significant bits) is hi + mid exactly; an F32 value (24 bits) is
// hi + mid + lo exactly unless its last bits lie below the BF16 subnormal
// range (|a| < 2^-109).  Each part times an exactly decoded BF16 weight is an
// exact FP32 product, so the FP32-output routed op computes the products of an
// FP32 matmul on the BF16 tensor cores.  Part r of row i lands in columns
// [r*k, (r+1)*k) of out row i (row stride parts*k); infinities and NaNs go
// whole into the first part.
__global__ void __launch_bounds__(256) split_bf16_kernel(const void* __restrict__ src, int src_dtype,
                                                         int64_t rows, int64_t k, int parts,
                                                         __nv_bfloat16* __restrict__ dst) {
  const int64_t n = rows * k;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = src_dtype == MXFP4_DTYPE_F32 ? static_cast<const float*>(src)[i]
                                                 : __half2float(static_cast<const __half*>(src)[i]);
    const int64_t r = i / k, c = i % k;
    __nv_bfloat16* row = dst + r * parts * k + c;
    const __nv_bfloat16 hi = __float2bfloat16_rn(a);
    float rem = isfinite(a) ? a - __bfloat162float(hi) : 0.0f;
    row[0] = hi;
    for (int q = 1; q < parts; ++q) {
      const __nv_bfloat16 part = __float2bfloat16_rn(rem);
      rem -= __bfloat162float(part);
      row[static_cast<int64_t>(q) * k] = part;
    }
  }
}

// ---------------------------------------------------------------------------
// K4 routing, three passes over the routes (stable counting sort):
//   pass 1 (route_count): each CTA takes a contiguous chunk of routes, ranks
//          every route among the earlier routes of the same expert in its
//          chunk (warp __match_any_sync + per-warp counts) and writes the
//          chunk histogram;
//   pass 2 (route_offsets): one CTA turns the [chunks x experts] histogram
//          into per-chunk bases, pads every expert to block_m, writes the
//          per-block expert ids, the pad entries and the used length;
//   pass 3 (route_scatter): every route lands at block_offset(e) + chunk
//          base + rank.
// No host synchronisation; everything stays on the stream.
// ---------------------------------------------------------------------------
constexpr int kRouteThreads = 512;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kMaxExperts = 1024;

__device__ __forceinline__ int load_expert(const void* ids, int ids_dtype, int64_t r) {
  return ids_dtype == MXFP4_DTYPE_I64 ? static_cast<int>(static_cast<const int64_t*>(ids)[r])
                                      : static_cast<const int32_t*>(ids)[r];
}

// smem: warp_cnt[kRouteWarps][E] ints.  rank_out[r] = rank in chunk; hist[c][e].
__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(
    const void* __restrict__ ids, int ids_dtype, int64_t num_routes, int num_experts,
    int expert_offset, int32_t* __restrict__ rank_out, int32_t* __restrict__ hist) {
  extern __shared__ int32_t warp_cnt[];  // [kRouteWarps][num_experts]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kRouteWarps * num_experts; i += blockDim.x) warp_cnt[i] = 0;
  __syncthreads();
  const int64_t r = blockIdx.x * static_cast<int64_t>(kRouteThreads) + threadIdx.x;
  int e = -1;
  if (r < num_routes) {
    e = load_expert(ids, ids_dtype, r) - expert_offset;
    if (e < 0 || e >= num_experts) e = -1;
  }
  const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
  const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank_in_warp == 0) warp_cnt[warp * num_experts + e] = __popc(peers);
  __syncthreads();
  // exclusive prefix over warps, per expert; chunk histogram
  for (int x = threadIdx.x; x < num_experts; x += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = warp_cnt[w * num_experts + x];
      warp_cnt[w * num_experts + x] = run;
      run += c;
    }
    hist[static_cast<int64_t>(blockIdx.x) * num_experts + x] = run;
  }
  __syncthreads();
  if (r < num_routes) rank_out[r] = e >= 0 ? warp_cnt[warp * num_experts + e] + rank_in_warp : -1;
}

// One CTA of 1024 threads (32 warps).  hist[c][e] -> per-chunk bases (in
// place: exclusive prefix over chunks per expert); blk_off[e] = first block of
// expert e (exclusive scan of the padded block counts); writes the per-block
// expert ids, the pad entries and the used length.  The histogram moves
// through shared memory in tiles of whole chunk rows (coalesced loads and
// stores, row stride E+1 so the column walks below are conflict-free); in a
// tile, warp w scans the chunk column of experts w, w+32, ... with its lanes
// on contiguous row ranges, carrying each expert's running total across tiles.
__device__ __forceinline__ int warp_excl_scan(int v, int lane, int& total) {
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  return incl - v;
}

constexpr int kOffsetsTileInts = 9216;  // 36 KB of counts per tile

// The routed layout from the per-expert route counts total_s[] (shared
// memory; one CTA of 1024 threads, every thread calls this): blk_off[e] and
// scan_s[e] = first block of expert e, the per-block expert ids, the pad
// entries of every expert's last block, the used length and, with rt_chunks,
// the chunk table.  Ends with scan_s valid for every thread.
__device__ __forceinline__ void route_layout(const int32_t* total_s, int32_t* scan_s, int32_t* warp_sums,
                                             int num_experts, int block_m, int64_t num_routes,
                                             int32_t* __restrict__ blk_off, int32_t* __restrict__ sorted_ids,
                                             int32_t* __restrict__ block_expert,
                                             int32_t* __restrict__ num_post_padded, int64_t capacity_blocks,
                                             int4* __restrict__ rt_chunks, int32_t* __restrict__ rt_num_chunks,
                                             int chunk_blocks) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  // exclusive scan of padded block counts over experts (E <= 1024: one per thread)
  const int e = threadIdx.x;
  const int nb = e < num_experts ? (total_s[e] + block_m - 1) / block_m : 0;
  int blocks_total;
  const int excl_in_warp = warp_excl_scan(nb, lane, blocks_total);
  if (lane == 0) warp_sums[wid] = blocks_total;
  __syncthreads();
  if (wid == 0) {
    int t;
    const int ex = warp_excl_scan(warp_sums[lane], lane, t);
    warp_sums[lane] = ex;  // exclusive over warps
    if (lane == 0) num_post_padded[0] = t * block_m;
  }
  __syncthreads();
  const int excl = excl_in_warp + warp_sums[wid];
  if (e < num_experts) {
    scan_s[e] = excl;
    blk_off[e] = excl;
  }
  __syncthreads();
  const int used_blocks = num_experts > 0 ? scan_s[num_experts - 1] +
                                                (total_s[num_experts - 1] + block_m - 1) / block_m
                                          : 0;
  for (int64_t b = used_blocks + threadIdx.x; b < capacity_blocks; b += blockDim.x) block_expert[b] = -1;
  // per-block expert ids and the pad entries of every expert's last block: warp per expert
  const int32_t pad = static_cast<int32_t>(num_routes);
  for (int x = wid; x < num_experts; x += 32) {
    const int cnt = total_s[x];
    const int nbx = (cnt + block_m - 1) / block_m;
    const int first = scan_s[x];
    for (int b = lane; b < nbx; b += 32) block_expert[first + b] = x;
    const int64_t base = static_cast<int64_t>(first) * block_m;
    for (int i = cnt + lane; i < nbx * block_m; i += 32) sorted_ids[base + i] = pad;
  }
  __syncthreads();
  if (rt_chunks == nullptr) return;  // uniform: every thread returns (scan_s is complete)
  // chunk table: exclusive scan of the per-expert chunk counts (one expert per thread)
  const int nc = e < num_experts ? (nb + chunk_blocks - 1) / chunk_blocks : 0;
  int chunks_total;
  const int cexcl_in_warp = warp_excl_scan(nc, lane, chunks_total);
  if (lane == 0) warp_sums[wid] = chunks_total;
  __syncthreads();
  if (wid == 0) {
    int t;
    const int ex = warp_excl_scan(warp_sums[lane], lane, t);
    warp_sums[lane] = ex;
    if (lane == 0) rt_num_chunks[0] = t;
  }
  __syncthreads();
  if (e < num_experts) {
    const int c0 = cexcl_in_warp + warp_sums[wid];
    for (int i = 0; i < nc; ++i) {
      const int b0 = i * chunk_blocks;
      const int nbl = min(chunk_blocks, nb - b0);
      rt_chunks[c0 + i] = make_int4((excl + b0) * block_m, nbl * block_m, e, 0);
    }
  }
  __syncthreads();
}

// Optional route chunks for the routed GEMMs (rt_chunks != nullptr): every
// expert's padded rows are cut into chunks of at most chunk_blocks blocks;
// chunk i of the table is int4 {first row, rows, expert, 0}, in expert order,
// and rt_num_chunks[0] holds their number.
__global__ void __launch_bounds__(1024) route_offsets_kernel(
    int32_t* __restrict__ hist, int num_chunks, int num_experts, int block_m, int64_t num_routes,
    int32_t* __restrict__ blk_off, int32_t* __restrict__ sorted_ids,
    int32_t* __restrict__ block_expert, int32_t* __restrict__ num_post_padded,
    int64_t capacity_blocks, int4* __restrict__ rt_chunks = nullptr, int32_t* __restrict__ rt_num_chunks = nullptr,
    int chunk_blocks = 1) {
  __shared__ int32_t tile[kOffsetsTileInts];
  __shared__ int32_t total_s[kMaxExperts];
  __shared__ int32_t scan_s[kMaxExperts];
  __shared__ int32_t warp_sums[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int ld = num_experts + 1;
  const int rows_per_tile = kOffsetsTileInts / ld > 0 ? kOffsetsTileInts / ld : 1;
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) total_s[e] = 0;
  for (int c0 = 0; c0 < num_chunks; c0 += rows_per_tile) {
    const int rows = min(rows_per_tile, num_chunks - c0);
    const int n = rows * num_experts;
    int32_t* g = hist + static_cast<int64_t>(c0) * num_experts;
    for (int i = threadIdx.x; i < n; i += blockDim.x) tile[(i / num_experts) * ld + i % num_experts] = g[i];
    __syncthreads();
    const int per = (rows + 31) / 32;
    const int r_beg = min(lane * per, rows), r_end = min(r_beg + per, rows);
    for (int e = wid; e < num_experts; e += 32) {
      int sum = 0;
      for (int r = r_beg; r < r_end; ++r) sum += tile[r * ld + e];
      int total;
      int run = warp_excl_scan(sum, lane, total) + total_s[e];
      for (int r = r_beg; r < r_end; ++r) {
        const int v = tile[r * ld + e];
        tile[r * ld + e] = run;
        run += v;
      }
      __syncwarp();
      if (lane == 0) total_s[e] += total;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) g[i] = tile[(i / num_experts) * ld + i % num_experts];
    __syncthreads();
  }
  __syncthreads();
  route_layout(total_s, scan_s, warp_sums, num_experts, block_m, num_routes, blk_off, sorted_ids, block_expert,
               num_post_padded, capacity_blocks, rt_chunks, rt_num_chunks, chunk_blocks);
}

__global__ void __launch_bounds__(kRouteThreads) route_scatter_kernel(
    const void* __restrict__ ids, int ids_dtype, int64_t num_routes, int num_experts,
    int expert_offset, int block_m, const int32_t* __restrict__ rank, const int32_t* __restrict__ hist,
    const int32_t* __restrict__ blk_off, int32_t* __restrict__ sorted_ids) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(kRouteThreads) + threadIdx.x;
  if (r >= num_routes) return;
  const int rk = rank[r];
  if (rk < 0) return;
  const int e = load_expert(ids, ids_dtype, r) - expert_offset;
  const int64_t pos = static_cast<int64_t>(blk_off[e]) * block_m +
                      hist[static_cast<int64_t>(blockIdx.x) * num_experts + e] + rk;
  sorted_ids[pos] = static_cast<int32_t>(r);
}

// Routing of up to kRouteSmallMax routes over up to kRouteSmallExperts experts
// in one CTA of 1024 threads (decode-sized calls): the stable ranks of
// route_count_kernel (a route per thread; __match_any_sync within the warp,
// exclusive prefix over the warps per expert), then route_layout, then the
// scatter of route_scatter_kernel.  Same metadata as the three-kernel path.
constexpr int kRouteSmallMax = 1024;
constexpr int kRouteSmallExperts = 256;
__global__ void __launch_bounds__(1024) route_small_kernel(
    const void* __restrict__ ids, int ids_dtype, int64_t num_routes, int num_experts, int expert_offset,
    int block_m, int32_t* __restrict__ blk_off, int32_t* __restrict__ sorted_ids,
    int32_t* __restrict__ block_expert, int32_t* __restrict__ num_post_padded, int64_t capacity_blocks,
    int4* __restrict__ rt_chunks, int32_t* __restrict__ rt_num_chunks, int chunk_blocks) {
  extern __shared__ int32_t warp_cnt[];  // [32][num_experts]
  __shared__ int32_t total_s[kMaxExperts];
  __shared__ int32_t scan_s[kMaxExperts];
  __shared__ int32_t warp_sums[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * num_experts; i += blockDim.x) warp_cnt[i] = 0;
  __syncthreads();
  const int r = threadIdx.x;
  int e = -1;
  if (r < num_routes) {
    e = load_expert(ids, ids_dtype, r) - expert_offset;
    if (e < 0 || e >= num_experts) e = -1;
  }
  const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
  const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank_in_warp == 0) warp_cnt[warp * num_experts + e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < num_experts; x += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = warp_cnt[w * num_experts + x];
      warp_cnt[w * num_experts + x] = run;
      run += c;
    }
    total_s[x] = run;
  }
  __syncthreads();
  route_layout(total_s, scan_s, warp_sums, num_experts, block_m, num_routes, blk_off, sorted_ids, block_expert,
               num_post_padded, capacity_blocks, rt_chunks, rt_num_chunks, chunk_blocks);
  if (e >= 0)
    sorted_ids[static_cast<int64_t>(scan_s[e]) * block_m + warp_cnt[warp * num_experts + e] + rank_in_warp] = r;
}

// ---------------------------------------------------------------------------
// Routed-order copy of the activations: xr[i] = x[sorted_ids[i] / top_k] for
// every used position i < num_post_padded[0] that holds a route; pad rows are
// left untouched (their GEMM rows are computed and discarded).  One warp per
// row, 16-byte vectors; the grouped GEMM then loads A tiles with TMA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint4* __restrict__ x, int64_t row_vecs,
                                                          const int32_t* __restrict__ sorted_ids,
                                                          const int32_t* __restrict__ num_post_padded,
                                                          int num_routes, int top_k, uint4* __restrict__ xr,
                                                          int64_t capacity) {
  const int64_t posted = num_post_padded[0];
  const int64_t used = posted < capacity ? posted : capacity;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); i < used; i += warps) {
    const int route = sorted_ids[i];
    if (route >= num_routes) continue;
    const uint4* src = x + static_cast<int64_t>(route / top_k) * row_vecs;
    uint4* dst = xr + i * row_vecs;
    for (int64_t v = lane; v < row_vecs; v += 32) dst[v] = src[v];
  }
}

// ---------------------------------------------------------------------------
// K5: out[t, :] = bf16( sum_j float(rows[t*top_k + j, :]) ), FP32 accumulation
// in j order.  8 columns (16 bytes) per thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) combine_topk_kernel(const __nv_bfloat16* __restrict__ rows,
                                                           __nv_bfloat16* __restrict__ out,
                                                           int64_t num_tokens, int top_k,
                                                           int64_t hidden, const void* __restrict__ ids,
                                                           int ids_dtype, int num_experts) {
  const int64_t vec_per_row = hidden / 8;
  const int64_t total = num_tokens * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row, v = i % vec_per_row;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    // slots in groups of eight: the group's ids, then its rows, are loaded
    // together (two memory round trips per group), then summed in slot order
    for (int j0 = 0; j0 < top_k; j0 += 8) {
      bool ok[8];
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        // a route to an expert outside [0, E) was not computed and contributes
        // zero, as its all-zero rows do in the reference composition
        const int e = j0 + u < top_k ? load_expert(ids, ids_dtype, t * top_k + j0 + u) : -1;
        ok[u] = e >= 0 && e < num_experts;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        q[u] = ok[u] ? *reinterpret_cast<const uint4*>(rows + ((t * top_k + j0 + u) * hidden) + v * 8)
                     : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (!ok[u]) continue;
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

// ---------------------------------------------------------------------------
// Router: per token, softmax over the experts' logits (FP32, max subtracted),
// the top_k largest probabilities in descending order (equal values: the lower
// expert first), optionally renormalised to sum to one.  This is the routing
// the vLLM adapter receives in topk_weights / topk_ids.  One warp per token;
// lane l holds the logits of experts l, l + 32, ... (E <= 32 * kRouterPerLane).
// ---------------------------------------------------------------------------
constexpr int kRouterPerLane = 8;  // E <= 256

__device__ __forceinline__ float load_logit(const void* p, int dtype, int64_t i) {
  if (dtype == MXFP4_DTYPE_F32) return static_cast<const float*>(p)[i];
  if (dtype == MXFP4_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__global__ void __launch_bounds__(256) router_kernel(const void* __restrict__ logits, int dtype, int64_t num_tokens,
                                                     int num_experts, int top_k, int renormalize,
                                                     float* __restrict__ w_out, int32_t* __restrict__ id_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; t < num_tokens; t += warps) {
    float v[kRouterPerLane];
#pragma unroll
    for (int j = 0; j < kRouterPerLane; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < num_experts ? load_logit(logits, dtype, t * num_experts + e) : -INFINITY;
    }
    float m = v[0];
#pragma unroll
    for (int j = 1; j < kRouterPerLane; ++j) m = fmaxf(m, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kRouterPerLane; ++j) {
      v[j] = lane + 32 * j < num_experts ? expf(v[j] - m) : 0.0f;
      sum += v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
#pragma unroll
    for (int j = 0; j < kRouterPerLane; ++j) v[j] = v[j] / sum;  // probabilities; 0 beyond E
    uint32_t taken = 0;
    float my_w = 0.0f;
    int my_id = 0;
    for (int r = 0; r < top_k; ++r) {
      float bv = -1.0f;
      int bi = 0x7FFFFFFF;
#pragma unroll
      for (int j = 0; j < kRouterPerLane; ++j) {
        const int e = lane + 32 * j;
        if (e < num_experts && !(taken & (1u << j)) && v[j] > bv) {
          bv = v[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      const bool found = bi < num_experts;  // false only when no candidate compares (NaN logits)
      if (found && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (lane == r) {
        my_w = found ? bv : 0.0f;
        my_id = found ? bi : -1;  // -1: no expert; the MoE ops drop such routes
      }
    }
    float sel = lane < top_k ? my_w : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sel += __shfl_xor_sync(0xFFFFFFFFu, sel, o);
    if (lane < top_k) {
      w_out[t * top_k + lane] = renormalize ? my_w / sel : my_w;
      id_out[t * top_k + lane] = my_id;
    }
  }
}

}  // namespace mx
