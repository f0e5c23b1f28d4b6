// Routed W4A16 grouped GEMM on CTA pairs with the decoded weights in tensor
// memory (the routed-MoE op's and the MoE layer's GEMMs).
//
// Operands are swapped with respect to the dense pair kernel: MMA M = 256
// weight rows of one expert (operand A, read from tensor memory, 128 rows per
// CTA), MMA N = up to 256 routes of that expert in routed order (operand B, a
// shared-memory tile loaded by TMA from the routed activation copy, half of
// the routes per CTA).  The routing pads every expert to 32 routes only, and a
// tile's N is its chunk's padded route count, so padded work is a few percent
// instead of the 1.5x of 256-route blocks.
//
// Weight path: TMA brings the packed E2M1 codes of a 64-K stage into a
// shared-memory ring; 16 decoder warps per CTA (4 per tensor-memory lane
// quarter, taking consecutive pairs of stages) read their rows' words, decode to
// BF16/FP16 pairs in registers, free the packed slot and store the pairs with
// tcgen05.st into a ring of tensor-memory slots (one lane per weight row, 32
// columns per stage).  The decoded weights never pass through shared memory.
//
// Work: tiles (route chunk c, weight block w), chunk-major, persistent over
// the clusters.  A chunk is at most 8 routing blocks of one expert
// (route_offsets_kernel's chunk table).  Weight block: plain = 256 consecutive
// output features (CTA r: [128 r, 128 r + 128)); GLU = 128 intermediate
// columns (CTA r: gate rows j0 + 64 r .. + 64 in lanes 0-63, the up rows of
// the same columns in lanes 64-127), so SiLU(gate) * up is formed inside one
// CTA.
//
// Epilogue (4 warps per CTA, one per tensor-memory lane quarter): the
// accumulator (lane = feature, column = route) is read in 32-column chunks;
// the routed op's rounding chain (compiled per output type, so each chunk is
// straight-line code) or, for GLU, the plain BF16 rounding of gate and up is
// applied in registers and the values are written transposed to a shared
// staging tile (route-major rows).  Once every column is read the accumulator
// is released to the MMA of the next tile; the staging rows then go to global
// memory as 16-byte vectors (GLU: all four warps form SiLU(gate) * up, eight
// independent columns per thread, on the way).
//
// Barriers (same shared offsets in both CTAs):
//   pfull[s]/pempty[s]  own CTA: packed ring, a group of pgroup stages per slot
//                       (one TMA per group / the decoder warps of its pairs)
//   xempty[s]           own CTA: route ring slot free (MMA commit, multicast)
//   ready[a]            leader: A slot a decoded in both CTAs (2 x 4 warps) and
//                       the stage's route tiles landed in both (each CTA's
//                       producer announces its bytes, its copies complete here)
//   aempty[a]           both: MMAs reading A slot a finished (multicast commit)
//   tfull / tempty      accumulator full (multicast commit) / drained (leader,
//                       2 x 4 epilogue warps)
// Every wait is bounded; on timeout the CTA aborts as the dense pair kernel does.
#pragma once

#include "gemm2.cuh"

namespace mx {

constexpr int kRtBlock = 32;              // routing block: padding granularity of every expert
constexpr int kRtChunkBlocks = 8;         // a tile's routes: at most 8 blocks = 256 (MMA N)
constexpr int kRtXSlots = 4;
constexpr int kRtPSlots = 4;              // packed ring: each slot holds a group of pgroup (2 or 4) stages
constexpr int kRtASlots = 8;              // tensor-memory A slots, 32 columns each, after the accumulator
constexpr int kRtDecodeWarps = 16;
constexpr int kRtThreads = 256 + 32 * kRtDecodeWarps;  // warps 0-3 control, 4-7 epilogue, 8-23 decoders
constexpr int kRtXBytes = 128 * 128;      // up to 128 route rows x 64 K (BF16), 128B swizzle
constexpr int kRtPBytes = 128 * 128;      // 128 weight rows x up to 4 stages x 64 K packed
constexpr int kRtStageOutBytes = 64 * 1024;
constexpr int kRtOffX = 0;
constexpr int kRtOffP = kRtOffX + kRtXSlots * kRtXBytes;
constexpr int kRtOffOut = kRtOffP + kRtPSlots * kRtPBytes;
constexpr int kRtOffRoute = kRtOffOut + kRtStageOutBytes;          // 256 route ids + 256 route weights
constexpr int kRtOffVote = kRtOffRoute + 256 * 8;                   // 4 epilogue warps' wait results
constexpr int kRtOffBar = kRtOffVote + 16;
constexpr int kRtNumBars = 2 * kRtPSlots + kRtXSlots + 2 * kRtASlots + 3;
constexpr int kRtOffMisc = kRtOffBar + kRtNumBars * 8;
constexpr int kRtSmemBytes = kRtOffMisc + 64 + 1024;
constexpr uint32_t kRtTmemCols = 512;     // accumulator [0, 256), A slots [256, 512)

struct RoutedParams {
  int N;                        // plain: output features; GLU: 2 * inter (weight rows per expert)
  int glu_inter;
  int K;                        // K of the routed activations (k_rep parts of the weights' K)
  int k_rep;
  int num_wblocks;              // plain: ceil(N / 256); GLU: ceil(inter / 128)
  int pgroup;                   // stages per packed TMA load (2 or 4; divides the weights' stage count)
  const uint8_t* w_scales;      // [E * N, Kw / 32]
  int64_t lds;
  int64_t w_rows_per_expert;
  const int4* chunks;           // {first routed row, rows, expert, 0}
  const int32_t* num_chunks;
  int max_chunks;
  const int32_t* sorted_ids;    // routed order (pad = num_routes)
  int num_routes;
  int top_k;
  void* out;                    // GLU: h [cap, ldo] in routed order; plain: C rows by route id
  int64_t ldo;
  int out_dtype;
  const float* a_scale;         // routed op: NULL means 1
  const float* b_scale;
  const void* topk_w;
  int w_dtype;
  int mul_w;
  int64_t c_stride_t, c_stride_j;
};

__device__ __forceinline__ void umma2_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Announce `bytes` of copies on a barrier given by its shared::cluster address
// (possibly in the peer CTA), counting as one arrival.
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(bytes)
               : "memory");
}
// 2-D tile load into this CTA's shared memory whose completion is signalled on
// a barrier of either CTA of the pair (shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.cta_group::2"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <int OUT>
__device__ __forceinline__ float rt_round(float x) {
  if (OUT == MXFP4_DTYPE_BF16) return round_bf16(x);
  if (OUT == MXFP4_DTYPE_F16) return round_f16(x);
  return x;
}

// One 32-route accumulator chunk of the routed op's epilogue for this
// thread's feature f: the rounding chain of soft:487-494 (round, x a_scale,
// x b_scale[e], x route weight, each rounded to the output type; FP32 output:
// FP32 products), written to the route-major staging tile.  Compiled per
// output type and chain shape, so the 32 elements are straight-line code.
template <int OUT, bool SCALES, bool MUL>
__device__ __forceinline__ void rt_plain_chunk(const uint32_t (&r)[32], uint8_t* stage, int jj0, int f, float asc,
                                               float bsc, const float* rw) {
#pragma unroll
  for (int i4 = 0; i4 < 32; i4 += 4) {
    float4 w4 = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    if (MUL) w4 = *reinterpret_cast<const float4*>(rw + i4);
    const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i4 + u;
      float x = __uint_as_float(r[i]);
      if (OUT == MXFP4_DTYPE_F32) {
        if (SCALES) x = x * asc * bsc;
        if (MUL) x = x * w[u];
        reinterpret_cast<float*>(stage)[(jj0 + i) * 128 + f] = x;
      } else {
        x = rt_round<OUT>(x);
        if (SCALES) {
          x = rt_round<OUT>(x * asc);
          x = rt_round<OUT>(x * bsc);
        }
        if (MUL) x = rt_round<OUT>(x * w[u]);
        reinterpret_cast<uint16_t*>(stage)[(jj0 + i) * 128 + f] =
            OUT == MXFP4_DTYPE_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(x)) : __half_as_ushort(__float2half_rn(x));
      }
    }
  }
}

template <int OUT>
__device__ __forceinline__ void rt_plain_chunk_any(const uint32_t (&r)[32], uint8_t* stage, int jj0, int f,
                                                   float asc, float bsc, const float* rw, bool scales, bool mul) {
  if (scales) {
    if (mul) rt_plain_chunk<OUT, true, true>(r, stage, jj0, f, asc, bsc, rw);
    else rt_plain_chunk<OUT, true, false>(r, stage, jj0, f, asc, bsc, rw);
  } else {
    if (mul) rt_plain_chunk<OUT, false, true>(r, stage, jj0, f, asc, bsc, rw);
    else rt_plain_chunk<OUT, false, false>(r, stage, jj0, f, asc, bsc, rw);
  }
}

// h = bf16(bf16(silu(bf16 g)) * bf16 u) for eight BF16 gate/up pairs (the
// reference composition's rounding points, vllm:240-265, F.silu's formula).
__device__ __forceinline__ uint4 rt_glu8(const uint4 g, const uint4 u) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
  float gg[8], uu[8], hh[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    gg[2 * i] = __uint_as_float(gw[i] << 16);
    gg[2 * i + 1] = __uint_as_float(gw[i] & 0xFFFF0000u);
    uu[2 * i] = __uint_as_float(uw[i] << 16);
    uu[2 * i + 1] = __uint_as_float(uw[i] & 0xFFFF0000u);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) hh[i] = round_bf16(gg[i] / (1.0f + expf(-gg[i]))) * uu[i];
  return make_uint4(f32x2_to_bf16x2(hh[0], hh[1]), f32x2_to_bf16x2(hh[2], hh[3]), f32x2_to_bf16x2(hh[4], hh[5]),
                    f32x2_to_bf16x2(hh[6], hh[7]));
}

// Weight row of local A row r (0..127) of this CTA for weight block wb of expert e.
template <int EPI>
__device__ __forceinline__ int64_t rt_weight_row(const RoutedParams& p, int e, int wb, uint32_t rank, int r,
                                                 bool& valid) {
  const int64_t base = static_cast<int64_t>(e) * p.w_rows_per_expert;
  if (EPI == EPI_GLU) {
    const int col = wb * 128 + static_cast<int>(rank) * 64 + (r & 63);
    valid = col < p.glu_inter;
    return base + (r < 64 ? col : p.glu_inter + col);
  }
  const int row = wb * 256 + static_cast<int>(rank) * 128 + r;
  valid = row < p.N;
  return base + row;
}

template <int EPI, bool FP16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kRtThreads, 1)
    mxfp4_routed_tmem_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x16,
                             const __grid_constant__ CUtensorMap tmap_x128, const RoutedParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRtOffBar);
  uint64_t* pfull = bars;
  uint64_t* pempty = pfull + kRtPSlots;
  uint64_t* xempty = pempty + kRtPSlots;
  uint64_t* ready = xempty + kRtXSlots;
  uint64_t* aempty = ready + kRtASlots;
  uint64_t* tfull = aempty + kRtASlots;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kRtOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kRtOffMisc + 4);
  int32_t* route_ids = reinterpret_cast<int32_t*>(smem + kRtOffRoute);
  float* route_w = reinterpret_cast<float*>(smem + kRtOffRoute + 256 * 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int KT = p.K / kP2BK;
  const int KTw = p.k_rep > 1 ? KT / p.k_rep : KT;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtPSlots; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 2 * p.pgroup);  // a pair's decoder warp of each lane quarter, pgroup / 2 pairs
    }
    for (int s = 0; s < kRtXSlots; ++s) mbar_init(&xempty[s], 1);
    for (int a = 0; a < kRtASlots; ++a) {
      // 4 decoder warps and the route-tile producer (expect_tx + its TMA bytes), in both CTAs
      mbar_init(&ready[a], 2 * 4 + 2);
      mbar_init(&aempty[a], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 8);  // 4 epilogue warps x 2 CTAs
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x16);
    prefetch_tmap(&tmap_x128);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, kRtTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_a = tmem_base + 256;
  constexpr int AS = kRtASlots, XS = kRtXSlots;
  int nch = p.num_chunks[0];
  nch = nch < p.max_chunks ? nch : p.max_chunks;
  const int num_tiles = nch * p.num_wblocks;

  if (warp == 0) {
    // ------------------------------------------------------------------ packed-weight producer
    // one TMA load (plain: 128 rows; GLU: the 64 gate and the 64 up rows) per
    // group of pgroup stages: each row's 32 * pgroup bytes land contiguously
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const int G = p.pgroup;
      const int gbytes = 128 * 32 * G;
      int gi = 0;
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        const int4 ch = p.chunks[t / p.num_wblocks];
        const int wb = t % p.num_wblocks;
        bool v;
        const int row_lo = static_cast<int>(rt_weight_row<EPI>(p, ch.z, wb, rank, 0, v));
        const int row_hi = static_cast<int>(rt_weight_row<EPI>(p, ch.z, wb, rank, 64, v));
        for (int kt = 0; kt < KT; kt += G, ++gi) {
          const int s = gi % kRtPSlots;
          const uint32_t ph = (gi / kRtPSlots) & 1;
          if (!mbar_wait(&pempty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&pfull[s], gbytes);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          uint8_t* dst = smem + kRtOffP + s * kRtPBytes;
          const int kx = (kt % KTw) * (kP2BK / 2);
          if (EPI == EPI_GLU) {
            tma_load_2d_hint(dst, &tmap_w, &pfull[s], kx, row_lo, pol_w);
            tma_load_2d_hint(dst + 64 * 32 * G, &tmap_w, &pfull[s], kx, row_hi, pol_w);
          } else {
            tma_load_2d_hint(dst, &tmap_w, &pfull[s], kx, row_lo, pol_w);
          }
        }
      }
      if (!ok || *abort_flag)
        for (int s = 0; s < kRtPSlots; ++s)
          if (armed & (1u << s)) mbar_drain(&pfull[s], (armed_par >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------------ route-tile producers
    // warp 2 takes the even stages, warp 3 the odd ones (two issuing threads).
    // Each load completes on the LEADER's ready barrier of its A slot
    // (.cta_group::2 bulk tensor copy), where this CTA first announced the bytes.
    if (lane == 0) {
      const uint32_t ready_leader = mapa_shared(smem_u32(ready), 0);
      const int par = warp - 2;
      int it = 0;
      bool ok = true, issued = false;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        const int4 ch = p.chunks[t / p.num_wblocks];
        const int half = ch.y >> 1;  // routes of this CTA (multiple of 16)
        const int row0 = ch.x + static_cast<int>(rank) * half;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          if ((it & 1) != par) continue;
          const int s = it % XS;
          const uint32_t ph = (it / XS) & 1;
          if (!mbar_wait(&xempty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          const uint32_t bar = ready_leader + (it % AS) * 8;
          mbar_arrive_expect_tx_cluster(bar, half * 128);
          uint8_t* dst = smem + kRtOffX + s * kRtXBytes;
          if (half == 128) {
            tma_load_2d_pair(dst, &tmap_x128, bar, kt * kP2BK, row0);
          } else {
            for (int i = 0; i < half / 16; ++i) tma_load_2d_pair(dst + i * 16 * 128, &tmap_x16, bar, kt * kP2BK, row0 + 16 * i);
          }
          issued = true;
        }
      }
      // an aborting CTA must not leave while its copies may still land in its
      // shared memory; their completion is tracked on the leader, so wait out
      // a bounded time far above any copy's latency
      if ((!ok || *abort_flag) && issued) {
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      int it = 0, tl = 0;
      bool ok = true, issued = false;
      // the next tile's route count is read one tile ahead (it sets the MMA's N)
      int n_next = cluster_id < num_tiles ? p.chunks[cluster_id / p.num_wblocks].y : 0;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++tl) {
        const int n_tile = n_next;
        if (t + num_clusters < num_tiles) n_next = p.chunks[(t + num_clusters) / p.num_wblocks].y;
        const uint32_t idesc = idesc_f16(FP16 ? 0 : 1, kP2BM, n_tile);
        if (!mbar_wait_cluster(tempty, (tl & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int a = it % AS, sx = it % XS;
          if (!mbar_wait_cluster(&ready[a], (it / AS) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bdesc = desc_sw128(smem_u32(smem + kRtOffX + sx * kRtXBytes));
          const uint32_t a_slot = tmem_a + a * 32;
#pragma unroll
          for (int k = 0; k < kP2BK / 16; ++k) umma2_f16_ta(tmem_base, a_slot + 8 * k, bdesc + 2 * k, idesc, (kt | k) != 0);
          umma2_commit_mc(&aempty[a], 0x3);
          umma2_commit_mc(&xempty[sx], 0x3);
          issued = true;
        }
        if (!ok) break;
        umma2_commit_mc(tfull, 0x3);
      }
      if (!ok && issued) {
        umma2_commit_mc(drain, 0x1);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ decoders -> tensor memory
    // warp 8 + dw: lane quarter q = dw % 4 (= warp % 4, the quarter it may
    // address) and group g = dw / 4.  Stages go to the quarter's four warps in
    // pairs (pair m = stages 2m, 2m + 1 to the warp with m % 4 == g): a warp
    // decodes both 64-K stages of its 32 rows per iteration, so eight stages
    // (the whole A ring) are in flight per quarter and each iteration's fixed
    // latency (barrier waits, tcgen05.st completion) covers two stages.
    const int dw = warp - 8;
    const int q = dw & 3, g = dw >> 2;
    const int r = q * 32 + lane;         // A row of this CTA = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t ready_leader = mapa_shared(smem_u32(ready), 0);
    const int total = num_tiles > cluster_id ? ((num_tiles - 1 - cluster_id) / num_clusters + 1) * KT : 0;
    // The scale codes of a pair (2 stages x 2 blocks of 32 K) are one aligned
    // 32-bit word of the row's scales (K is a multiple of 128).  Each pair's
    // word is loaded while the previous pair is decoded, so the load latency
    // is off the critical path; the chunk table is read only when the next
    // pair starts another tile.
    int next_tile = -1;
    const uint8_t* next_srow = p.w_scales;
    bool next_valid = false;
    auto scale_word = [&](int it) -> uint32_t {
      if (it >= total) return 0x7F7F7F7Fu;
      const int ts = it / KT, kt = it % KT;
      if (ts != next_tile) {
        next_tile = ts;
        const int t = cluster_id + ts * num_clusters;
        const int4 ch = p.chunks[t / p.num_wblocks];
        const int64_t grow = rt_weight_row<EPI>(p, ch.z, t % p.num_wblocks, rank, r, next_valid);
        next_srow = p.w_scales + (next_valid ? grow * p.lds : 0);
      }
      // rows past the expert's last feature read the first row's scales (their
      // products land in accumulator rows the epilogue drops); no select on
      // the loaded word, so nothing waits for it before its pair
      return ldg_nc_u32(next_srow + 2 * (kt % KTw));
    };
    uint32_t sc_next = scale_word(2 * g);
    for (int it0 = 2 * g; it0 < total; it0 += 8) {
      const uint32_t sc_pair = sc_next;
      sc_next = scale_word(it0 + 8);
      int nb = 0;  // stages of this pair (KT is even: the pair never straddles a tile)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int it = it0 + h;
        if (it >= total) break;
        const int gi = it / p.pgroup;  // packed group of this stage (both stages of a pair share it)
        const int sp = gi % kRtPSlots, a = it % AS;
        const uint32_t sc = sc_pair >> (16 * h);
        // warp-uniform waits: the tcgen05.st / wait::st below are .sync.aligned
        if (h == 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(&pfull[sp], (gi / kRtPSlots) & 1, abort_flag))) { nb = -1; break; }
        // rows of 32 * pgroup bytes, swizzled by the TMA (128B for 4 stages, 64B for 2): 16-byte chunk c
        // of row r sits at chunk c ^ (r % 8) resp. c ^ ((r / 2) % 4), so a warp's 32 rows spread over
        // all bank groups
        const uint32_t prow = smem_u32(smem + kRtOffP + sp * kRtPBytes) + r * 32 * p.pgroup;
        const uint32_t c0 = 2u * static_cast<uint32_t>(it % p.pgroup);
        const uint32_t sw = p.pgroup == 4 ? static_cast<uint32_t>(r & 7) : static_cast<uint32_t>((r >> 1) & 3);
        const uint4 q0 = ld_shared_v4(prow + ((c0 ^ sw) << 4));
        const uint4 q1 = ld_shared_v4(prow + (((c0 + 1) ^ sw) << 4));
        const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t code = (sc >> (8 * (i >> 2))) & 0xFF;  // words 0-3: first 32 K, 4-7: second
          uint4 d;
          if (FP16) d = decode8_f16(words[i], e8m0_to_f32(code));
          else d = decode8_bf16(words[i], e8m0_to_bf16x2(code));
          v[4 * i] = d.x;
          v[4 * i + 1] = d.y;
          v[4 * i + 2] = d.z;
          v[4 * i + 3] = d.w;
        }
        // after the pair's last words are used, the packed slot may be refilled
        if (h == 1 || it + 1 >= total) {
          asm volatile("" ::"r"(v[0]), "r"(v[31]));
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[sp]);
        }
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&aempty[a], ((it / AS) & 1) ^ 1, abort_flag))) { nb = -1; break; }
        tc_fence_after();
        tmem_st_32x32b_x32(tmem_a + lane_base + a * 32, v);
        ++nb;
      }
      if (nb < 0) break;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int h = 0; h < nb; ++h) mbar_arrive_cluster(ready_leader + ((it0 + h) % AS) * 8);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 4-7, both CTAs)
    const int q = warp & 3;
    const int etid = threadIdx.x - 128;  // 0..127
    const int f = q * 32 + lane;         // accumulator lane = A row of this CTA
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    const int esz = out_esize(p.out_dtype);
    uint8_t* stage = smem + kRtOffOut;
    volatile int* vote = reinterpret_cast<volatile int*>(smem + kRtOffVote);
    int tl = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters, ++tl) {
      const int4 ch = p.chunks[t / p.num_wblocks];
      const int wb = t % p.num_wblocks;
      const int n = ch.y;
      // the chunk's route ids and weights, once per tile
      named_bar_sync(1, 128);  // the previous tile's store phase is done with the staging tile
      for (int j = etid; j < n; j += 128) {
        const int sid = p.sorted_ids[ch.x + j];
        route_ids[j] = sid;
        route_w[j] = (EPI == EPI_MOE && p.mul_w && sid < p.num_routes) ? load_weight(p.topk_w, p.w_dtype, sid) : 1.0f;
      }
      // the accumulator wait, made uniform over the four epilogue warps: they
      // meet at named barriers below, so either all of them go on or none
      const bool got = __all_sync(0xFFFFFFFFu, mbar_wait_cluster(tfull, tl & 1, abort_flag));
      if (lane == 0) vote[q] = got ? 1 : 0;
      named_bar_sync(1, 128);
      if (!(vote[0] && vote[1] && vote[2] && vote[3])) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      if (EPI == EPI_GLU) {
        // phase A: the raw BF16 gate (lanes 0-63) and up (lanes 64-127) values
        // into the route-major staging tile [route][128]: the tile's 64 gate
        // columns, then its 64 up columns
        uint16_t* st16 = reinterpret_cast<uint16_t*>(stage);
        for (int c0 = 0; c0 < n; c0 += 32) {
          uint32_t r32[32];
          tmem_ld_32x32b_x32(tbase + c0, r32);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) st16[(c0 + i) * 128 + f] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r32[i])));
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (lane == 0) mbar_arrive_cluster(tempty_leader);  // the accumulator is free for the next tile
        // phase B: h[routed row ch.x + j][col0 + 8c .. + 8] for every route j and 8-column group c
        const int col0 = wb * 128 + static_cast<int>(rank) * 64;
        const int ncols = p.glu_inter - col0 < 64 ? p.glu_inter - col0 : 64;
        for (int i = etid; i < n * 8; i += 128) {
          const int j = i >> 3, c = i & 7;
          if (c * 8 >= ncols) continue;
          const uint32_t row = smem_u32(stage) + j * 256;
          const uint4 h8 = rt_glu8(ld_shared_v4(row + c * 16), ld_shared_v4(row + 128 + c * 16));
          uint8_t* dst = static_cast<uint8_t*>(p.out) + ((static_cast<int64_t>(ch.x) + j) * p.ldo + col0 + c * 8) * 2;
          if (c * 8 + 8 <= ncols) {
            *reinterpret_cast<uint4*>(dst) = h8;
          } else {
            const uint32_t hw[4] = {h8.x, h8.y, h8.z, h8.w};
            for (int b = 0; c * 8 + b < ncols; ++b)
              reinterpret_cast<uint16_t*>(dst)[b] = static_cast<uint16_t>(hw[b >> 1] >> ((b & 1) * 16));
          }
        }
      } else {
        // plain: rounding chain of the routed op (soft:487-494) per element,
        // rows scattered to C[t, j] / y[route]; staged in passes of as many
        // routes as the staging tile holds at this output size
        const int feat0 = wb * 256 + static_cast<int>(rank) * 128;
        const int nfeat = p.N - feat0 < 128 ? p.N - feat0 : 128;
        const bool scales = p.a_scale != nullptr;
        const float asc = scales ? p.a_scale[0] : 1.0f;
        const float bsc = scales ? p.b_scale[ch.z] : 1.0f;
        const bool mul = p.mul_w != 0;
        const int pass_routes = kRtStageOutBytes / (128 * esz);  // 256 (2-byte out) or 128 (F32)
        for (int pb = 0; pb < n; pb += pass_routes) {
          const int pe = n - pb < pass_routes ? n : pb + pass_routes;
          for (int c0 = pb; c0 < pe; c0 += 32) {
            uint32_t r32[32];
            tmem_ld_32x32b_x32(tbase + c0, r32);
            tmem_ld_wait();
            if (p.out_dtype == MXFP4_DTYPE_BF16)
              rt_plain_chunk_any<MXFP4_DTYPE_BF16>(r32, stage, c0 - pb, f, asc, bsc, route_w + c0, scales, mul);
            else if (p.out_dtype == MXFP4_DTYPE_F16)
              rt_plain_chunk_any<MXFP4_DTYPE_F16>(r32, stage, c0 - pb, f, asc, bsc, route_w + c0, scales, mul);
            else
              rt_plain_chunk_any<MXFP4_DTYPE_F32>(r32, stage, c0 - pb, f, asc, bsc, route_w + c0, scales, mul);
          }
          if (pe == n) {  // every column read: release the accumulator before the stores
            tc_fence_before();
            named_bar_sync(1, 128);
            if (lane == 0) mbar_arrive_cluster(tempty_leader);
          } else {
            named_bar_sync(1, 128);
          }
          const int rows = pe - pb;
          const int row_bytes = 128 * esz;
          const int vec_per_row = row_bytes / 16;
          for (int i = etid; i < rows * vec_per_row; i += 128) {
            const int jj = i / vec_per_row, c = i % vec_per_row;
            const int sid = route_ids[pb + jj];
            if (sid >= p.num_routes) continue;
            const int first = c * 16 / esz;  // first feature of this vector
            if (first >= nfeat) continue;
            const int64_t roff = static_cast<int64_t>(sid / p.top_k) * p.c_stride_t +
                                 static_cast<int64_t>(sid % p.top_k) * p.c_stride_j + feat0;
            uint8_t* dst = static_cast<uint8_t*>(p.out) + roff * esz + c * 16;
            const uint4 val = ld_shared_v4(smem_u32(stage + jj * row_bytes + c * 16));
            if (first + 16 / esz <= nfeat && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
              *reinterpret_cast<uint4*>(dst) = val;
            } else {
              const uint8_t* src = stage + jj * row_bytes + c * 16;
              for (int b = 0; b < 16 / esz && first + b < nfeat; ++b)
                for (int y = 0; y < esz; ++y) dst[b * esz + y] = src[b * esz + y];
            }
          }
          named_bar_sync(1, 128);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's TMEM and barriers stay alive until the leader is done
  tc_fence_after();
  if (warp == 1) tmem_dealloc2(tmem_base, kRtTmemCols);
}

}  // namespace mx
