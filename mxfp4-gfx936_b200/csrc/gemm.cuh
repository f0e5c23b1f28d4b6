// Warp-specialised tcgen05 GEMM with MXFP4 weight decode in the producer.
//
// One template serves the dense W4A16 linear (fused and safe modes) and the
// grouped GEMMs of the routed MoE op.  Per CTA tile: 128 rows of A x 256
// output columns, K in steps of 64; A and the weight operand B are staged in
// shared memory in the 128-byte-swizzled K-major layout tcgen05.mma reads,
// and the FP32 accumulator lives in tensor memory (two 256-column buffers so
// the epilogue of one tile overlaps the main loop of the next).
//
// Warp roles (persistent CTAs walk the same tile sequence):
//   warp 0      producer: TMA for A (or a cp.async row gather for routed A)
//               and for the packed weight bytes (or the BF16 weight tile in
//               safe mode)
//   warp 1      tensor-memory allocator and the single-thread MMA issuer
//   warps 4-7   epilogue: tcgen05.ld -> rounding chain -> global stores
//   warps 8-15  decoders (fused mode): packed E2M1 + E8M0 -> BF16/FP16 tile
//               in original K order, written straight into the swizzled
//               B stage that the MMA consumes
//
// Per stage s the barriers are: full[s] (operands landed), bready[s] (B tile
// decoded), empty[s] (MMAs reading stage s finished, via tcgen05.commit).
#pragma once

#include "common.cuh"

namespace mx {

enum AMode : int { A_TMA = 0, A_GATHER = 1 };
enum BMode : int { B_DECODE = 0, B_TMA = 1 };
enum EpiMode : int { EPI_DENSE = 0, EPI_MOE = 1, EPI_GLU = 2 };

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kPBytes = kBN * kBK / 2;  // 8 KB of packed codes
constexpr int kAccCols = kBN;           // FP32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kNumDecodeWarps = 8;

template <int BMODE>
struct GemmCfg {
  static constexpr int kStages = BMODE == B_DECODE ? 3 : 4;
  static constexpr int kThreads = BMODE == B_DECODE ? 512 : 256;
  static constexpr int kStageBytes = kABytes + kBBytes + (BMODE == B_DECODE ? kPBytes : 0);
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffP = kOffB + kStages * kBBytes;
  static constexpr int kOffBar = kOffP + (BMODE == B_DECODE ? kStages * kPBytes : 0);
  // full, bready, empty per stage + tfull[2], tempty[2], drain
  static constexpr int kNumBars = 3 * kStages + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
};

struct GemmParams {
  int M, N, K;                 // dense: A rows; all: output columns, reduction length
  int num_m_blocks;            // dense: ceil(M/128); MoE: capacity blocks
  int num_n_blocks;
  // routed A gather (A_GATHER): row of route r is A[r / top_k]
  const uint8_t* a_ptr;        // element bytes = 2
  int64_t lda;                 // elements
  int a_rows;                  // valid rows of A (tokens)
  int a_row_offset;            // dense TMA row origin
  // weights
  const uint8_t* w_scales;     // [rows, K/32]
  int64_t lds;                 // bytes per scale row
  int64_t w_rows_per_expert;   // N (plain) or 2*inter (GLU)
  int glu_inter;               // inter (GLU)
  // routing
  const int32_t* sorted_ids;
  const int32_t* block_expert;
  const int32_t* num_post_padded;
  int num_routes;
  int top_k;
  // epilogue
  void* out;
  int64_t ldo;                 // elements (dense / GLU row stride)
  int out_dtype;
  const void* bias;
  const float* a_scale;
  const float* b_scale;
  const void* topk_w;
  int w_dtype;
  int mul_w;
  int64_t c_stride_t, c_stride_j;  // MoE C row offset, elements
  int vec_ok;                  // 16-byte aligned output rows
};

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

struct TileCoord {
  int m_blk, n_blk, expert;
};

template <int EPI>
__device__ __forceinline__ TileCoord tile_coord(const GemmParams& p, int t, int nmb) {
  TileCoord c;
  c.m_blk = t % nmb;
  c.n_blk = t / nmb;
  c.expert = EPI == EPI_DENSE ? 0 : p.block_expert[c.m_blk];
  return c;
}

// Global weight row of B-tile row r (0..255).
template <int EPI>
__device__ __forceinline__ int64_t weight_row(const GemmParams& p, const TileCoord& c, int r,
                                              bool& valid) {
  if (EPI == EPI_GLU) {
    const int col = c.n_blk * (kBN / 2) + (r & (kBN / 2 - 1));
    valid = col < p.glu_inter;
    const int64_t base = static_cast<int64_t>(c.expert) * p.w_rows_per_expert;
    return base + (r < kBN / 2 ? col : p.glu_inter + col);
  }
  const int col = c.n_blk * kBN + r;
  valid = col < p.N;
  return static_cast<int64_t>(c.expert) * p.w_rows_per_expert + col;
}

template <int AMODE, int BMODE, int EPI, bool FP16>
__global__ void __launch_bounds__(GemmCfg<BMODE>::kThreads, 1)
    mxfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b, const GemmParams p) {
  using Cfg = GemmCfg<BMODE>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* bready = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* tfull = bars + 3 * S;
  uint64_t* tempty = bars + 3 * S + 2;
  uint64_t* drain = bars + 3 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KT = p.K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], AMODE == A_GATHER ? 33 : 1);
      mbar_init(&bready[s], kNumDecodeWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (AMODE == A_TMA) prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Number of tiles (MoE: from the device-side routing result).
  int nmb = p.num_m_blocks;
  if (EPI != EPI_DENSE) {
    const int used = p.num_post_padded[0] / kBM;
    nmb = used < nmb ? used : nmb;
  }
  const int num_tiles = nmb * p.num_n_blocks;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    int it = 0;
    uint32_t armed = 0, armed_par = 0;  // per-stage bit: armed at least once / parity of last arm
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const TileCoord c = tile_coord<EPI>(p, t, nmb);
      bool v0, v1;
      const int y0 = static_cast<int>(weight_row<EPI>(p, c, 0, v0));
      const int y1 = static_cast<int>(weight_row<EPI>(p, c, kBN / 2, v1));
      // routed A rows handled by this lane: r = lane + 32 i
      const uint8_t* arow[4];
      uint32_t abytes[4];
      if (AMODE == A_GATHER) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = lane + 32 * i;
          int src_row = -1;
          if (EPI == EPI_DENSE) {
            src_row = c.m_blk * kBM + r < p.a_rows ? c.m_blk * kBM + r : -1;
          } else {
            const int route = p.sorted_ids[c.m_blk * kBM + r];
            src_row = route < p.num_routes ? route / p.top_k : -1;
          }
          arow[i] = p.a_ptr + (src_row >= 0 ? static_cast<int64_t>(src_row) * p.lda * 2 : 0);
          abytes[i] = src_row >= 0 ? 16u : 0u;
        }
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (AMODE == A_GATHER || lane == 0) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        }
        if (lane == 0) {
          const uint32_t tx = (AMODE == A_TMA ? kABytes : 0) + (BMODE == B_DECODE ? kPBytes : kBBytes);
          mbar_arrive_expect_tx(&full[s], tx);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (AMODE == A_TMA)
            tma_load_2d(smem + Cfg::kOffA + s * kABytes, &tmap_a, &full[s], kt * kBK,
                        p.a_row_offset + c.m_blk * kBM);
          if (BMODE == B_DECODE) {
            uint8_t* pdst = smem + Cfg::kOffP + s * kPBytes;
            tma_load_2d_hint(pdst, &tmap_b, &full[s], kt * (kBK / 2), y0, pol_w);
            tma_load_2d_hint(pdst + kPBytes / 2, &tmap_b, &full[s], kt * (kBK / 2), y1, pol_w);
          } else {
            tma_load_2d_hint(smem + Cfg::kOffB + s * kBBytes, &tmap_b, &full[s], kt * kBK,
                             c.n_blk * kBN, pol_w);
          }
        }
        if (AMODE == A_GATHER) {
          const uint32_t abase = smem_u32(smem + Cfg::kOffA + s * kABytes);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = lane + 32 * i;
            const uint8_t* src = arow[i] + static_cast<int64_t>(kt) * kBK * 2;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              cp_async_16(abase + r * 128 + ((ch ^ (r & 7)) << 4), src + ch * 16, abytes[i]);
          }
          cp_async_arrive_noinc(&full[s]);
        }
      }
      __syncwarp();
    }
    if (!ok || *abort_flag) {
      if (AMODE == A_GATHER) cp_async_wait_all();
      if (lane == 0)
        for (int s = 0; s < S; ++s)
          if (armed & (1u << s)) mbar_drain(&full[s], (armed_par >> s) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(FP16 ? 0 : 1, kBM, kBN);
      int it = 0, tl = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tl) {
        const int acc = tl & 1;
        if (!mbar_wait(&tempty[acc], ((tl >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          uint64_t* ready = BMODE == B_DECODE ? &bready[s] : &full[s];
          if (!mbar_wait(ready, ph, abort_flag)) { ok = false; break; }
          if (AMODE == A_GATHER && BMODE == B_DECODE) {
            if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          }
          if (AMODE == A_GATHER) fence_proxy_async();
          tc_fence_after();
          const uint64_t adesc = desc_sw128(smem_u32(smem + Cfg::kOffA + s * kABytes));
          const uint64_t bdesc = desc_sw128(smem_u32(smem + Cfg::kOffB + s * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kt | k) != 0);
          umma_commit(&empty[s]);
          issued = true;
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter
    const int r_local = q * 32 + lane;      // row inside the tile
    int tl = 0;
    const int esz = out_esize(p.out_dtype);
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tl) {
      const TileCoord c = tile_coord<EPI>(p, t, nmb);
      const int acc = tl & 1;
      if (!mbar_wait(&tfull[acc], (tl >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kAccCols;

      if (EPI == EPI_DENSE) {
        const int row = c.m_blk * kBM + r_local;
        const bool row_ok = row < p.M;
        uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<int64_t>(row_ok ? row : 0) * p.ldo * esz;
#pragma unroll 1
        for (int cc = 0; cc < kBN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, r);
          tmem_ld_wait();
          const int col0 = c.n_blk * kBN + cc * 32;
          if (row_ok && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            if (p.bias != nullptr) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int col = col0 + i < p.N ? col0 + i : p.N - 1;
                v[i] = round_to(round_to(v[i], p.out_dtype) + load_weight(p.bias, p.out_dtype, col),
                                p.out_dtype);
              }
            }
            store_row32(orow + static_cast<int64_t>(col0) * esz, p.out_dtype, v, p.N - col0, p.vec_ok != 0);
          }
        }
      } else if (EPI == EPI_MOE) {
        const int route = p.sorted_ids[c.m_blk * kBM + r_local];
        const bool row_ok = route < p.num_routes;
        const float asc = p.a_scale != nullptr ? p.a_scale[0] : 1.0f;
        const float bsc = p.b_scale != nullptr ? p.b_scale[c.expert] : 1.0f;
        const float rw = (row_ok && p.mul_w) ? load_weight(p.topk_w, p.w_dtype, route) : 1.0f;
        const int64_t roff = row_ok ? (static_cast<int64_t>(route / p.top_k) * p.c_stride_t +
                                       static_cast<int64_t>(route % p.top_k) * p.c_stride_j)
                                    : 0;
        uint8_t* orow = static_cast<uint8_t*>(p.out) + roff * esz;
#pragma unroll 1
        for (int cc = 0; cc < kBN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, r);
          tmem_ld_wait();
          const int col0 = c.n_blk * kBN + cc * 32;
          if (row_ok && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float x = round_to(__uint_as_float(r[i]), p.out_dtype);
              x = round_to(x * asc, p.out_dtype);
              x = round_to(x * bsc, p.out_dtype);
              if (p.mul_w) x = round_to(x * rw, p.out_dtype);
              v[i] = x;
            }
            store_row32(orow + static_cast<int64_t>(col0) * esz, p.out_dtype, v, p.N - col0, p.vec_ok != 0);
          }
        }
      } else {  // EPI_GLU: h = bf16(bf16(silu(bf16 g)) * bf16 u), written in routed order
        const int pos = c.m_blk * kBM + r_local;
        uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<int64_t>(pos) * p.ldo * 2;
#pragma unroll 1
        for (int cc = 0; cc < kBN / 64; ++cc) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, g);
          tmem_ld_32x32b_x32(tbase + kBN / 2 + cc * 32, u);
          tmem_ld_wait();
          const int col0 = c.n_blk * (kBN / 2) + cc * 32;
          if (col0 < p.glu_inter) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float gg = round_bf16(__uint_as_float(g[i]));
              const float uu = round_bf16(__uint_as_float(u[i]));
              const float sg = round_bf16(gg / (1.0f + expf(-gg)));
              v[i] = round_bf16(sg * uu);
            }
            store_row32(orow + static_cast<int64_t>(col0) * 2, MXFP4_DTYPE_BF16, v,
                        p.glu_inter - col0, p.vec_ok != 0);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  } else if (BMODE == B_DECODE && warp >= 8) {
    // ------------------------------------------------------------------ decoders
    const int r = threadIdx.x - 256;  // B-tile row 0..255
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const TileCoord c = tile_coord<EPI>(p, t, nmb);
      bool valid;
      const int64_t wrow = weight_row<EPI>(p, c, r, valid);
      const uint8_t* srow = p.w_scales + (valid ? wrow * p.lds : 0);
      uint32_t nxt = valid ? ldg_nc_u32(srow) : 0x7F7F7F7Fu;
      uint32_t cur = 0;
      for (int kt = 0; kt < KT; ++kt, ++it) {
        if ((kt & 1) == 0) {
          cur = nxt;
          if (valid && kt + 2 < KT) nxt = ldg_nc_u32(srow + 4 * ((kt >> 1) + 1));
        }
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
        const uint32_t psrc = smem_u32(smem + Cfg::kOffP + s * kPBytes) + r * 32;
        const uint4 q0 = ld_shared_v4(psrc);
        const uint4 q1 = ld_shared_v4(psrc + 16);
        const uint32_t sh = (kt & 1) * 16;
        const uint32_t c0 = (cur >> sh) & 0xFF;
        const uint32_t c1 = (cur >> (sh + 8)) & 0xFF;
        const uint32_t bdst = smem_u32(smem + Cfg::kOffB + s * kBBytes) + r * 128;
        const uint32_t sw = r & 7;
        if (FP16) {
          const float f0 = e8m0_to_f32(c0), f1 = e8m0_to_f32(c1);
          st_shared_v4(bdst + ((0 ^ sw) << 4), decode8_f16(q0.x, f0));
          st_shared_v4(bdst + ((1 ^ sw) << 4), decode8_f16(q0.y, f0));
          st_shared_v4(bdst + ((2 ^ sw) << 4), decode8_f16(q0.z, f0));
          st_shared_v4(bdst + ((3 ^ sw) << 4), decode8_f16(q0.w, f0));
          st_shared_v4(bdst + ((4 ^ sw) << 4), decode8_f16(q1.x, f1));
          st_shared_v4(bdst + ((5 ^ sw) << 4), decode8_f16(q1.y, f1));
          st_shared_v4(bdst + ((6 ^ sw) << 4), decode8_f16(q1.z, f1));
          st_shared_v4(bdst + ((7 ^ sw) << 4), decode8_f16(q1.w, f1));
        } else {
          const uint32_t b0 = e8m0_to_bf16x2(c0), b1 = e8m0_to_bf16x2(c1);
          st_shared_v4(bdst + ((0 ^ sw) << 4), decode8_bf16(q0.x, b0));
          st_shared_v4(bdst + ((1 ^ sw) << 4), decode8_bf16(q0.y, b0));
          st_shared_v4(bdst + ((2 ^ sw) << 4), decode8_bf16(q0.z, b0));
          st_shared_v4(bdst + ((3 ^ sw) << 4), decode8_bf16(q0.w, b0));
          st_shared_v4(bdst + ((4 ^ sw) << 4), decode8_bf16(q1.x, b1));
          st_shared_v4(bdst + ((5 ^ sw) << 4), decode8_bf16(q1.y, b1));
          st_shared_v4(bdst + ((6 ^ sw) << 4), decode8_bf16(q1.z, b1));
          st_shared_v4(bdst + ((7 ^ sw) << 4), decode8_bf16(q1.w, b1));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace mx
