// W4A16 GEMMs on CTA pairs (tcgen05 cta_group::2): a 256-row x bn-column
// output tile per cluster of two CTAs.  One template serves the dense linear
// (fused and safe modes), the routed MoE op and both passes of the MoE layer
// (256-row blocks of routes of one expert).
//
// CTA r of the pair stages rows [128r, 128r+128) of the A tile and rows
// [128r, 128r+128) of the B (weight) tile: each SM decodes and stores only half
// of the weight tile, and the pair's tensor cores read each half once.  The
// leader CTA (rank 0) issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16) from
// one thread; each CTA's tensor memory receives its own 128 accumulator rows.
//
// Synchronisation (all barriers sit at the same shared-memory offset in both
// CTAs):
//   full[s]    own CTA: its TMA loads (A half, packed weight half or BF16 half)
//   ready[s]   leader only: both CTAs' stage s is ready for the MMA -- one
//              arrival per decode warp of both CTAs (fused mode) or one per CTA
//              from a bridge thread that watched full[s] (safe mode)
//   empty[s]   both: MMAs reading stage s finished (multicast tcgen05.commit)
//   tfull[a]   both: accumulator a complete (multicast tcgen05.commit)
//   tempty[a]  leader only: both CTAs' epilogues drained accumulator a
// No TMA multicast is used: each CTA loads only its own half.
#pragma once

#include "gemm.cuh"

namespace mx {

constexpr int kP2BM = 256, kP2BN = 256, kP2BK = 64;  // pair tile
constexpr int kP2HalfRows = 128;
constexpr int kP2ABytes = kP2HalfRows * kP2BK * 2;    // 16 KB
constexpr int kP2BBytes = kP2HalfRows * kP2BK * 2;    // 16 KB
constexpr int kP2PBytes = kP2HalfRows * kP2BK / 2;    // 4 KB

// PEERS (dense all-gather): the epilogue stages each warp's 32 x 32 output
// chunk in shared memory (2 KB per epilogue warp) and stores whole 64-byte row
// segments locally, releases the accumulator, and hands the finished tile to
// four pusher warps, which copy its rows from the local output into every
// peer's buffer while the tensor cores work on the next tile.
template <int BMODE, int DECODE_WARPS, bool PEERS = false>
struct Pair2Cfg {
  static constexpr int kStages = (BMODE == B_DECODE && PEERS) ? 5 : 6;
  static constexpr int kDecodeWarps = BMODE == B_DECODE ? DECODE_WARPS : 0;
  // warps 0-3 control, 4-7 epilogue group 0, then the decoders, then epilogue
  // group 1, then (PEERS) the pushers
  static constexpr int kEpi1Warp = 8 + kDecodeWarps;
  static constexpr int kPushWarp = kEpi1Warp + 4;
  static constexpr int kThreads = 256 + 32 * kDecodeWarps + 128 + (PEERS ? 128 : 0);
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kP2ABytes;
  static constexpr int kOffP = kOffB + kStages * kP2BBytes;
  static constexpr int kOffOut = kOffP + (BMODE == B_DECODE ? kStages * kP2PBytes : 0);
  static constexpr int kOffBar = kOffOut + (PEERS ? 8 * 2048 : 0);
  // full, ready, empty per stage; tfull[2], tempty[2], drain; (PEERS) stored[2], pushed[2]
  static constexpr int kNumBars = 3 * kStages + 5 + (PEERS ? 4 : 0);
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}
// Arrive on a barrier given by its shared::cluster address (possibly in the
// peer CTA).  Default (.release.cta) semantics: a decoder orders its shared
// stores for the tensor cores with fence.proxy.async before arriving, which is
// what the MMA needs; a cluster-scope release here costs about 2x throughput.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      record_error(MXFP4_ERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at `bar`'s offset in every CTA of `mask` when all earlier
// tcgen05 operations of this thread complete.
__device__ __forceinline__ void umma2_commit_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

constexpr int kMaxPeers = 7;  // up to 8 ranks per node

struct PairParams {
  int M, N, K;                     // dense: rows of A; N: output columns (GLU: 2*inter); K: reduction
  int bn;                          // tile width: multiple of 32, <= 256 (each CTA holds bn/2 weight rows)
  int num_m_blocks, num_n_blocks;  // dense: ceil(M/256); routed: capacity blocks of 256 routes
  // routed A gather (A_GATHER): row of route r is A[r / top_k]
  const uint8_t* a_ptr;
  int64_t lda;                     // elements
  int a_row_offset;                // TMA row origin of A
  // weights
  const uint8_t* w_scales;         // [rows, K/32]
  int64_t lds;
  int64_t w_rows_per_expert;       // N (plain) or 2*inter (GLU)
  int glu_inter;
  // K of A is k_rep copies of the weights' K (0 or 1: one): A row =
  // [part 0 | part 1 | ...], every part multiplied by the same weights, so
  // the weight stages (packed tile and scale words) repeat every K/k_rep
  int k_rep;
  // routing
  const int32_t* sorted_ids;
  const int32_t* block_expert;
  const int32_t* num_post_padded;
  int num_routes;
  int top_k;
  // epilogue
  void* out;
  int64_t ldo;                     // elements (dense / GLU row stride)
  int out_dtype;
  const void* bias;
  const float* a_scale;            // routed op: NULL means 1
  const float* b_scale;
  const void* topk_w;
  int w_dtype;
  int mul_w;
  int64_t c_stride_t, c_stride_j;  // routed C row offset, elements
  int vec_ok;
  // dense all-gather epilogue: every output chunk is also stored, at the same
  // offset, into the buffers of num_peers other ranks (peer_out[j] is the
  // peer's mapping of its output over NVLink, already offset to this rank's
  // columns; ldo is the full row stride)
  int num_peers;
  void* peer_out[kMaxPeers];
  // optional NVLink multicast mapping of all ranks' outputs, offset like
  // peer_out: one multimem store reaches every rank (16-byte path only)
  void* mc_out;
};
using DenseParams = PairParams;

struct PairTile {
  int m_blk, n_blk, expert;
};

// Tile order.  Dense: row blocks fastest, so the clusters in flight share each
// weight tile through L2 and the activations (at most a few tens of MB) stay
// in L2 anyway.  Routed: column blocks fastest, so the (large) routed
// activation block is read from HBM once and reused from L2 by its column
// tiles, and the weights of an expert's consecutive route blocks are shared.
template <int EPI>
__device__ __forceinline__ PairTile pair_tile(const PairParams& p, int t, int nmb) {
  PairTile c;
  if (EPI == EPI_DENSE) {
    c.m_blk = t % nmb;
    c.n_blk = t / nmb;
  } else {
    c.m_blk = t / p.num_n_blocks;
    c.n_blk = t % p.num_n_blocks;
  }
  c.expert = EPI == EPI_DENSE ? 0 : p.block_expert[c.m_blk];
  return c;
}

// Weight row of local B row r (0..bn/2-1) of this CTA.  GLU: CTA 0 holds the
// gate rows and CTA 1 the up rows of the same bn/2 intermediate columns.
template <int EPI>
__device__ __forceinline__ int64_t pair_weight_row(const PairParams& p, const PairTile& c, uint32_t rank, int r,
                                                   bool& valid) {
  const int64_t base = static_cast<int64_t>(c.expert) * p.w_rows_per_expert;
  if (EPI == EPI_GLU) {
    const int col = c.n_blk * (p.bn / 2) + r;
    valid = col < p.glu_inter;
    return base + (rank == 0 ? col : p.glu_inter + col);
  }
  const int col = c.n_blk * p.bn + static_cast<int>(rank) * (p.bn / 2) + r;
  valid = col < p.N;
  return base + col;
}

// Rounding chain of the routed op for one 32-column chunk (soft:487-494),
// compiled per output dtype so the element loop has no dtype branches.
template <int OUT>
__device__ __forceinline__ void moe_chunk(float (&v)[32], float asc, float bsc, float rw, bool scales, bool mul) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float x = round_to(v[i], OUT);
    if (scales) {
      x = round_to(x * asc, OUT);
      x = round_to(x * bsc, OUT);
    }
    if (mul) x = round_to(x * rw, OUT);
    v[i] = x;
  }
}

// Epilogue of one tile for one thread: accumulator row r_local (its TMEM lane)
// of this CTA, 32-column chunks cc = grp, grp + 2, ... (two epilogue groups).
template <int EPI, bool PEERS = false>
__device__ __forceinline__ void pair_epilogue_tile(const PairParams& p, const PairTile& c, uint32_t tbase,
                                                   uint32_t rank, int r_local, int grp, int esz,
                                                   uint32_t stage = 0) {
  const int pos = c.m_blk * kP2BM + static_cast<int>(rank) * kP2HalfRows + r_local;  // row of the block
  if (EPI == EPI_DENSE) {
    const bool row_ok = pos < p.M;
    const int lane = r_local & 31;
    uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<int64_t>(row_ok ? pos : 0) * p.ldo * esz;
#pragma unroll 1
    for (int cc = grp; cc < p.bn / 32; cc += 2) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + cc * 32, r);
      tmem_ld_wait();
      const int col0 = c.n_blk * p.bn + cc * 32;
      if (col0 >= p.N) continue;  // warp-uniform
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (p.bias != nullptr) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int col = col0 + i < p.N ? col0 + i : p.N - 1;
          v[i] = round_to(round_to(v[i], p.out_dtype) + load_weight(p.bias, p.out_dtype, col), p.out_dtype);
        }
      }
      if constexpr (PEERS) {
        if (p.out_dtype != MXFP4_DTYPE_F32 && p.vec_ok && col0 + 32 <= p.N) {
          // stage the warp's 32 rows x 64 B, then store whole 64-byte row
          // segments (4 lanes per row, 8 rows per instruction) locally and to
          // every peer; chunk c of row r sits at c ^ ((r >> 1) & 3) (no bank conflicts)
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = p.out_dtype == MXFP4_DTYPE_BF16 ? f32x2_to_bf16x2(v[2 * i], v[2 * i + 1])
                                                    : f32x2_to_f16x2(v[2 * i], v[2 * i + 1]);
          const uint32_t xs = (lane >> 1) & 3;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            st_shared_v4(stage + lane * 64 + ((q4 ^ xs) << 4),
                         make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]));
          __syncwarp();
          const int row0 = pos - lane;  // first row of this warp
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + (lane >> 2);
            const int ch = lane & 3;
            const uint4 val = ld_shared_v4(stage + rr * 64 + ((ch ^ ((rr >> 1) & 3)) << 4));
            if (row0 + rr < p.M) {
              const int64_t off = (static_cast<int64_t>(row0 + rr) * p.ldo + col0 + ch * 8) * 2;
              *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + off) = val;
            }
          }
          __syncwarp();  // the next chunk reuses the staging area
          continue;
        }
      }
      if (!row_ok) continue;
      store_row32(orow + static_cast<int64_t>(col0) * esz, p.out_dtype, v, p.N - col0, p.vec_ok != 0);
    }
  } else if (EPI == EPI_MOE) {
    const int route = p.sorted_ids[pos];
    const bool row_ok = route < p.num_routes;
    const bool scales = p.a_scale != nullptr;
    const float asc = scales ? p.a_scale[0] : 1.0f;
    const float bsc = scales ? p.b_scale[c.expert] : 1.0f;
    const bool mul = p.mul_w != 0;
    const float rw = (row_ok && mul) ? load_weight(p.topk_w, p.w_dtype, route) : 1.0f;
    const int64_t roff = row_ok ? (static_cast<int64_t>(route / p.top_k) * p.c_stride_t +
                                   static_cast<int64_t>(route % p.top_k) * p.c_stride_j)
                                : 0;
    uint8_t* orow = static_cast<uint8_t*>(p.out) + roff * esz;
#pragma unroll 1
    for (int cc = grp; cc < p.bn / 32; cc += 2) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + cc * 32, r);
      tmem_ld_wait();
      const int col0 = c.n_blk * p.bn + cc * 32;
      if (row_ok && col0 < p.N) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (p.out_dtype == MXFP4_DTYPE_BF16) moe_chunk<MXFP4_DTYPE_BF16>(v, asc, bsc, rw, scales, mul);
        else if (p.out_dtype == MXFP4_DTYPE_F16) moe_chunk<MXFP4_DTYPE_F16>(v, asc, bsc, rw, scales, mul);
        else moe_chunk<MXFP4_DTYPE_F32>(v, asc, bsc, rw, scales, mul);
        store_row32(orow + static_cast<int64_t>(col0) * esz, p.out_dtype, v, p.N - col0, p.vec_ok != 0);
      }
    }
  } else {  // EPI_GLU: h = bf16(bf16(silu(bf16 g)) * bf16 u), written in routed order
    uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<int64_t>(pos) * p.ldo * 2;
#pragma unroll 1
    for (int cc = grp; cc < p.bn / 64; cc += 2) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(tbase + cc * 32, g);
      tmem_ld_32x32b_x32(tbase + p.bn / 2 + cc * 32, u);
      tmem_ld_wait();
      const int col0 = c.n_blk * (p.bn / 2) + cc * 32;
      if (col0 < p.glu_inter) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gg = round_bf16(__uint_as_float(g[i]));
          const float uu = round_bf16(__uint_as_float(u[i]));
          const float sg = round_bf16(gg / (1.0f + expf(-gg)));
          v[i] = round_bf16(sg * uu);
        }
        store_row32(orow + static_cast<int64_t>(col0) * 2, MXFP4_DTYPE_BF16, v, p.glu_inter - col0,
                    p.vec_ok != 0);
      }
    }
  }
}

// Pushers (PEERS): copy this CTA's rows [row0, row0 + 128) x columns
// [col0, col0 + width) of the finished tile from the local output (L2-hot,
// read past L1) into every peer buffer at the same offset; 128 threads, 16-byte
// vectors when the rows allow, four loads in flight per thread.
// One 16-byte store to a multicast address: NVSwitch writes it into every
// rank's buffer bound to the multicast object.
__device__ __forceinline__ void multimem_st_v4(void* mc_addr, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
               : "memory");
}

__device__ __forceinline__ void push_tile_rows(const PairParams& p, int row0, int col0, int width, int esz,
                                               int tid) {
  const int rows = p.M - row0 < 128 ? p.M - row0 : 128;
  if (rows <= 0 || width <= 0) return;
  const int64_t row_bytes = static_cast<int64_t>(width) * esz;
  const int64_t ld_bytes = p.ldo * esz;
  const uint8_t* src = static_cast<const uint8_t*>(p.out) + static_cast<int64_t>(row0) * ld_bytes +
                       static_cast<int64_t>(col0) * esz;
  const int64_t off0 = src - static_cast<const uint8_t*>(p.out);
  if (p.vec_ok && row_bytes % 16 == 0) {
    const int per_row = static_cast<int>(row_bytes / 16);
    const int total = rows * per_row;
    for (int base = tid; base < total; base += 4 * 128) {
      uint4 v[4];
      int64_t off[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * 128;
        off[u] = -1;
        if (i < total) {
          off[u] = static_cast<int64_t>(i / per_row) * ld_bytes + static_cast<int64_t>(i % per_row) * 16;
          v[u] = __ldcg(reinterpret_cast<const uint4*>(src + off[u]));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (off[u] >= 0) {
          if (p.mc_out != nullptr) {
            multimem_st_v4(static_cast<uint8_t*>(p.mc_out) + off0 + off[u], v[u]);
          } else {
#pragma unroll
            for (int j = 0; j < kMaxPeers; ++j)
              if (j < p.num_peers) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.peer_out[j]) + off0 + off[u]) = v[u];
          }
        }
    }
  } else {
    const int per_row = static_cast<int>(row_bytes / 2);
    const int total = rows * per_row;
    for (int i = tid; i < total; i += 128) {
      const int64_t off = static_cast<int64_t>(i / per_row) * ld_bytes + static_cast<int64_t>(i % per_row) * 2;
      const uint16_t v = __ldcg(reinterpret_cast<const unsigned short*>(src + off));
#pragma unroll
      for (int j = 0; j < kMaxPeers; ++j)
        if (j < p.num_peers) *reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(p.peer_out[j]) + off0 + off) = v;
    }
  }
}

template <int AMODE, int BMODE, int EPI, bool FP16, int DECODE_WARPS, bool PEERS = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Pair2Cfg<BMODE, DECODE_WARPS, PEERS>::kThreads, 1)
    mxfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const PairParams p) {
  static_assert(!PEERS || EPI == EPI_DENSE, "peer stores are a dense-epilogue feature");
  using Cfg = Pair2Cfg<BMODE, DECODE_WARPS, PEERS>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* ready = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* tfull = bars + 3 * S;
  uint64_t* tempty = bars + 3 * S + 2;
  uint64_t* drain = bars + 3 * S + 4;
  uint64_t* stored = bars + 3 * S + 5;  // PEERS only
  uint64_t* pushed = stored + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int KT = p.K / kP2BK;
  const int KTw = p.k_rep > 1 ? KT / p.k_rep : KT;  // weight stages per pass over the weights' K
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int half_rows = p.bn / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], AMODE == A_GATHER ? 33 : 1);
      mbar_init(&ready[s], BMODE == B_DECODE ? 2 * DECODE_WARPS : 2);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // 2 epilogue groups x 4 warps x 2 CTAs
    }
    mbar_init(drain, 1);
    if constexpr (PEERS) {
      for (int a = 0; a < 2; ++a) {
        mbar_init(&stored[a], 8);  // the 8 epilogue warps of this CTA
        mbar_init(&pushed[a], 4);  // the 4 pusher warps
      }
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (AMODE == A_TMA) prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  // launched right behind the weight decode (programmatic dependent launch):
  // the set-up above overlaps its tail, its output is read from here on
  griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  int nmb = p.num_m_blocks;
  if (EPI != EPI_DENSE) {
    const int used = p.num_post_padded[0] / kP2BM;
    nmb = used < nmb ? used : nmb;
  }
  const int num_tiles = nmb * p.num_n_blocks;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (both CTAs)
    // lane 0 issues the TMA loads; in gather mode all 32 lanes copy A rows
    const uint64_t pol_w = policy_evict_first();
    int it = 0;
    uint32_t armed = 0, armed_par = 0;
    bool ok = true;
    if (AMODE == A_GATHER || lane == 0)
    for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
      const PairTile c = pair_tile<EPI>(p, t, nmb);
      bool v0;
      const int brow = static_cast<int>(pair_weight_row<EPI>(p, c, rank, 0, v0));
      const int arow = p.a_row_offset + c.m_blk * kP2BM + static_cast<int>(rank) * kP2HalfRows;
      const uint8_t* gsrc[4];
      uint32_t gbytes[4];
      if (AMODE == A_GATHER) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = lane + 32 * i;
          const int route = p.sorted_ids[c.m_blk * kP2BM + static_cast<int>(rank) * kP2HalfRows + r];
          const int src_row = route < p.num_routes ? route / p.top_k : -1;
          gsrc[i] = p.a_ptr + (src_row >= 0 ? static_cast<int64_t>(src_row) * p.lda * 2 : 0);
          gbytes[i] = src_row >= 0 ? 16u : 0u;
        }
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (AMODE == A_GATHER || lane == 0) {
          if (!mbar_wait_cluster(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], (AMODE == A_TMA ? kP2ABytes : 0) +
                                              half_rows * (BMODE == B_DECODE ? kP2BK / 2 : kP2BK * 2));
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (AMODE == A_TMA) tma_load_2d(smem + Cfg::kOffA + s * kP2ABytes, &tmap_a, &full[s], kt * kP2BK, arow);
          if (BMODE == B_DECODE)
            tma_load_2d_hint(smem + Cfg::kOffP + s * kP2PBytes, &tmap_b, &full[s], (kt % KTw) * (kP2BK / 2), brow,
                             pol_w);
          else
            tma_load_2d_hint(smem + Cfg::kOffB + s * kP2BBytes, &tmap_b, &full[s], kt * kP2BK, brow, pol_w);
        }
        if (AMODE == A_GATHER) {
          const uint32_t abase = smem_u32(smem + Cfg::kOffA + s * kP2ABytes);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = lane + 32 * i;
            const uint8_t* src = gsrc[i] + static_cast<int64_t>(kt) * kP2BK * 2;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) cp_async_16(abase + r * 128 + ((ch ^ (r & 7)) << 4), src + ch * 16, gbytes[i]);
          }
          cp_async_arrive_noinc(&full[s]);
        }
      }
      if (AMODE == A_GATHER) __syncwarp();
    }
    if (!ok || *abort_flag) {
      if (AMODE == A_GATHER) cp_async_wait_all();
      if (lane == 0)
        for (int s = 0; s < S; ++s)
          if (armed & (1u << s)) mbar_drain(&full[s], (armed_par >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_f16(FP16 ? 0 : 1, kP2BM, p.bn);
      int it = 0, tl = 0;
      bool ok = true, issued = false;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++tl) {
        const int acc = tl & 1;
        if (!mbar_wait_cluster(&tempty[acc], ((tl >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait_cluster(&ready[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = desc_sw128(smem_u32(smem + Cfg::kOffA + s * kP2ABytes));
          const uint64_t bdesc = desc_sw128(smem_u32(smem + Cfg::kOffB + s * kP2BBytes));
#pragma unroll
          for (int k = 0; k < kP2BK / 16; ++k) umma2_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kt | k) != 0);
          umma2_commit_mc(&empty[s], 0x3);
          issued = true;
        }
        if (!ok) break;
        umma2_commit_mc(&tfull[acc], 0x3);
      }
      if (!ok && issued) {
        umma2_commit_mc(drain, 0x1);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp == 2 && BMODE == B_TMA) {
    // ------------------------------------------------------------------ bridge (safe mode)
    if (lane == 0) {
      const uint32_t ready_leader = mapa_shared(smem_u32(ready), 0);
      int it = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters)
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort_flag)) { ok = false; break; }
          mbar_arrive_cluster(ready_leader + s * 8);
        }
    }
    __syncwarp();
  } else if ((warp >= 4 && warp < 8) || (warp >= Cfg::kEpi1Warp && warp < Cfg::kEpi1Warp + 4)) {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    // two groups of four warps; warp w reads TMEM lane quarter w % 4 and group g
    // takes the 32-column chunks cc with cc % 2 == g
    const int q = warp & 3;
    const int grp = warp < 8 ? 0 : 1;
    const int r_local = q * 32 + lane;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    const int esz = out_esize(p.out_dtype);
    int tl = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters, ++tl) {
      const PairTile c = pair_tile<EPI>(p, t, nmb);
      const int acc = tl & 1;
      if (!mbar_wait_cluster(&tfull[acc], (tl >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kAccCols;
      pair_epilogue_tile<EPI, PEERS>(p, c, tbase, rank, r_local, grp, esz,
                                     smem_u32(smem + Cfg::kOffOut) + (grp * 4 + q) * 2048);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + acc * 8);
      if constexpr (PEERS) {
        // the tile's local rows are stored: hand them to the pushers (which must
        // be done with the tile two back, the last user of this barrier slot)
        if (!mbar_wait(&pushed[acc], ((tl >> 1) & 1) ^ 1, abort_flag)) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&stored[acc]);
      }
    }
  } else if (PEERS && warp >= Cfg::kPushWarp && warp < Cfg::kPushWarp + 4) {
    // ------------------------------------------------------------------ pushers (PEERS, both CTAs)
    if constexpr (PEERS) {
      const int tid = threadIdx.x - Cfg::kPushWarp * 32;
      const int esz = out_esize(p.out_dtype);
      int tl = 0;
      for (int t = cluster_id; t < num_tiles; t += num_clusters, ++tl) {
        const PairTile c = pair_tile<EPI>(p, t, nmb);
        const int acc = tl & 1;
        if (!mbar_wait(&stored[acc], (tl >> 1) & 1, abort_flag)) break;
        const int row0 = c.m_blk * kP2BM + static_cast<int>(rank) * kP2HalfRows;
        const int col0 = c.n_blk * p.bn;
        const int width = p.N - col0 < p.bn ? p.N - col0 : p.bn;
        push_tile_rows(p, row0, col0, width, esz, tid);
        __syncwarp();
        if (lane == 0) mbar_arrive(&pushed[acc]);
      }
    }
  } else if (warp >= 8 && warp < Cfg::kEpi1Warp) {
    // ------------------------------------------------------------------ decoders (both CTAs)
    if constexpr (BMODE == B_DECODE) {
      constexpr int kThreadsPerRow = (DECODE_WARPS * 32) / kP2HalfRows;  // 2 or 4
      constexpr int kChunks = 8 / kThreadsPerRow;                         // 16-byte output chunks per thread
      const int d = threadIdx.x - 256;
      const int r = d / kThreadsPerRow;   // weight row in this CTA's half
      const int part = d % kThreadsPerRow;
      const int j0 = part * kChunks;      // first chunk (8 K values each)
      const int blk_in_tile = j0 / 4;     // scale block (32 K) of this part within the 64-K stage
      const uint32_t ready_leader = mapa_shared(smem_u32(ready), 0);
      const bool row_live = r < half_rows;
      int it = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        const PairTile c = pair_tile<EPI>(p, t, nmb);
        bool valid;
        const int64_t grow = pair_weight_row<EPI>(p, c, rank, r, valid);
        valid = valid && row_live;
        const uint8_t* srow = p.w_scales + (valid ? grow * p.lds : 0);
        // one 32-bit scale word covers two 64-K stages; keep two words in flight.
        // The word sequence repeats every nwords words when A holds k_rep parts
        // (KTw is even: K is a multiple of 128).
        const int nwords = KTw / 2;
        const int nwords_all = KT / 2;
        uint32_t w0 = valid ? ldg_nc_u32(srow) : 0x7F7F7F7Fu;
        uint32_t w1 = (valid && nwords_all > 1) ? ldg_nc_u32(srow + 4 * (1 % nwords)) : 0x7F7F7F7Fu;
        uint32_t cur = 0;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          if ((kt & 1) == 0) {
            cur = w0;
            w0 = w1;
            const int nw = (kt >> 1) + 2;
            if (valid && nw < nwords_all) w1 = ldg_nc_u32(srow + 4 * (nw % nwords));
          }
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          if (row_live) {
            const uint32_t code = (cur >> (8 * ((kt & 1) * 2 + blk_in_tile))) & 0xFF;
            const uint32_t psrc = smem_u32(smem + Cfg::kOffP + s * kP2PBytes) + r * 32 + j0 * 4;
            const uint32_t bdst = smem_u32(smem + Cfg::kOffB + s * kP2BBytes) + r * 128;
            const uint32_t sw = r & 7;
            uint32_t w[kChunks];
            if constexpr (kChunks == 4) {
              const uint4 q4 = ld_shared_v4(psrc);
              w[0] = q4.x;
              w[1] = q4.y;
              w[2] = q4.z;
              w[3] = q4.w;
            } else {
              asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(psrc));
            }
            if (FP16) {
              const float f = e8m0_to_f32(code);
#pragma unroll
              for (int i = 0; i < kChunks; ++i) st_shared_v4(bdst + (((j0 + i) ^ sw) << 4), decode8_f16(w[i], f));
            } else {
              const uint32_t b = e8m0_to_bf16x2(code);
#pragma unroll
              for (int i = 0; i < kChunks; ++i) st_shared_v4(bdst + (((j0 + i) ^ sw) << 4), decode8_bf16(w[i], b));
            }
            fence_proxy_async();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(ready_leader + s * 8);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's TMEM and barriers stay alive until the leader is done
  tc_fence_after();
  if (warp == 1) tmem_dealloc2(tmem_base, kTmemCols);
}

}  // namespace mx
