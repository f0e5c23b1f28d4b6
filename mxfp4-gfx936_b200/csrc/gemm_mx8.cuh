// Routed W4A16 grouped GEMM on the block-scaled tensor cores, without a
// weight decode (the routed-MoE op's and the MoE layer's GEMMs, BF16
// activations).
//
// The weights are MX-format already: E2M1 codes with one E8M0 scale per 32 K.
// tcgen05.mma.kind::mxf8f6f4.block_scale multiplies an E2M1 operand by an
// E4M3 operand, each with its own E8M0 scale per 32 K, with exact products and
// FP32 accumulation.  A BF16 activation has 8 significant bits; it is written
// as the sum of two E4M3 numbers (hi + lo), so the product with a weight is
// computed as two block-scaled MMAs into one accumulator and the packed codes
// go from HBM to the tensor core untouched (TMA with the 16U4_ALIGN16B type
// expands each 8-byte group of 16 codes to the 16-byte slot the MMA reads).
//
// Activation split (mx8_split_kernel), per 32-value block with e = the
// exponent of max|x|:
//   hi code   = e - 7 + 127            (block scale 2^(e-7): max|x| / scale in [128, 256))
//   x'        = x * 2^(7-e)            (exact)
//   hi        = RNE_e4m3(x')           (|x'| < 256; the E4M3 step there is 16)
//   lo code   = hi code - 5
//   lo        = RNE_e4m3((x' - hi) * 2^5)
// x' - hi is exact in FP32, at most 8 in magnitude, and a multiple of x's last
// bit, so it has at most 4 significant bits: lo is exact whenever it is at
// least the E4M3 subnormal step, i.e. for every element within 2^-14 of the
// block maximum.  Smaller elements lose at most 2^-22 of the block maximum.
// The sum over K then differs from the BF16 tensor-core GEMM only by that and
// by the FP32 summation order: well inside the BF16 output tolerance.
//
// Layout of the split activations: hi and lo [rows, K] bytes in routed order
// (K-major, TMA 128B-swizzled tiles of 32 rows x 128 K); E8M0 codes per route
// chunk in 512-byte pieces [chunk][K/128][512]: byte (j, kb) of the chunk's
// route j at (j % 32) * 16 + (j / 32) * 4 + kb, the layout tcgen05.cp
// .32x128b.warpx4 copies into tensor memory (the scale of B row j at column
// j / 32 of the scale region).

// Kernel: one CTA per SM, persistent over tiles (route chunk, weight block),
// chunk-major.  Swapped operands: MMA M = 128 weight rows of one expert
// (plain: 128 consecutive output features; GLU: 64 gate rows and the 64 up
// rows of the same intermediate columns), MMA N = the chunk's routes (a
// multiple of 32, at most BN).  K stages of 128:
//   warp 0   TMA producer: per group of stages one copy each of the weight
//            tile (unpacked E2M1), the hi and lo route tiles and the chunk's
//            hi and lo activation scales; the scales complete on their own
//            barrier (with the weight scales), so the scale writers start
//            while the tiles are still in flight
//   warp 2   weight-scale producer: the weights' scale words (one 32-bit word
//            = 4 codes per row and stage) by 4-byte cp.async into the
//            512-byte chunk layout
//   warps 8-11 scale writers, one per tensor-memory lane quarter: each
//            stage's weight and activation scales from shared memory into
//            the stage's tensor-memory region with tcgen05.st (the per-stage
//            scale copies kept off the MMA thread)
//   warp 1   MMA issuer: per 32 K one MMA over the hi and lo rows stacked
//            along N (32-route tiles) or two MMAs, hi and lo
//   warps 4-7 epilogue, one per tensor-memory lane quarter (the routed
//            kernels' epilogue: GLU, or the routed op's rounding chain)
// Two accumulators of BN columns alternate between tiles, so a tile's
// epilogue overlaps the next tile's MMAs.  Every wait is bounded; on a
// timeout the CTA records MXFP4_ERR_TIMEOUT and leaves after draining its
// copies.
#pragma once

#include "gemm_routed.cuh"
#include "gemm_w4a4.cuh"

namespace mx {

template <int BN>
struct Mx8Cfg {
  // stage slots of 128 K; the producer fills groups of G consecutive slots
  // (G = 4, 2 or 1, dividing both the slot count and K / 128) with one copy
  // per operand, so copies are few and large
  static constexpr int kSlots = BN == 128 ? 3 : 8;
  // accumulator pieces per tile, summed by the epilogue: 32-route tiles keep
  // even and odd K steps apart (independent MMA chains), each as hi then lo
  // columns: hi even, lo even, hi odd, lo odd, BN columns apart
  static constexpr int kAcc = BN == 32 ? 4 : 1;
  static_assert(kAcc * BN <= 128, "accumulator slot");
  static constexpr int kABytes = 128 * 128;          // 128 weight rows x 128 K (one byte per code in shared memory)
  static constexpr int kBBytes = BN * 128;           // BN routes x 128 K, E4M3 (hi; lo right after it)
  // 32-route tiles stack hi and lo along the MMA's N (one N = 64 MMA per
  // 32 K, the scales of both in one chunk: hi in column 0, lo in column 1);
  // 128-route tiles take two N = 128 MMAs (hi, lo) per 32 K
  static constexpr bool kStackHiLo = BN == 32;
  static constexpr int kSfaBytes = 512;
  static constexpr int kSfbBytes = 512;              // one route chunk (up to 128 routes)
  static constexpr int kOutBytes = BN * 128 * 2;     // staging: BN routes x 128 features, 16-bit outputs
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kSlots * kABytes;          // per slot: hi tile, lo tile
  static constexpr int kOffSfa = kOffB + kSlots * 2 * kBBytes;
  static constexpr int kOffSfb = kOffSfa + kSlots * kSfaBytes;    // per slot: hi chunk (+ lo chunk)
  static constexpr int kSfbSlot = kStackHiLo ? kSfbBytes : 2 * kSfbBytes;
  static constexpr int kOffOut = kOffSfb + kSlots * kSfbSlot;
  static constexpr int kOffRoute = kOffOut + kOutBytes;       // BN route ids + BN route weights
  static constexpr int kOffVote = kOffRoute + BN * 8;
  static constexpr int kOffBar = kOffVote + 16;
  static constexpr int kNumBars = 4 * kSlots + 5;
  static constexpr int kThreads = 384;  // warps 0-3 copies / MMA, 4-7 epilogue, 8-11 scale writers
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "mx8 kernel shared memory");
  static_assert(256 + kSlots * 12 <= 512, "mx8 scale regions in tensor memory");
};
// Tensor memory: two accumulator slots [0, 256); from column 256 one scale
// region per stage slot (weights 4, hi 4, lo 4 columns), so a stage's scale
// copy never waits for MMAs still reading another stage's scales.
constexpr uint32_t kMx8TmemCols = 512;
constexpr uint32_t kMx8SfCol = 256, kMx8SfRegion = 12;
constexpr int kMx8LoShift = 5;          // lo = (x' - hi) * 2^5, lo code = hi code - 5

struct Mx8Params {
  int group;                    // stages per copy group (divides K / 128 and the slot count)
  int N;                        // plain: output features; GLU: 2 * inter
  int glu_inter;
  int K;
  int num_wblocks;              // plain: ceil(N / 128); GLU: ceil(inter / 64)
  const uint8_t* w_scales;      // [E * rows, K / 32]
  int64_t lds;
  int64_t w_rows_per_expert;
  const uint8_t* sfh;           // activation scales [chunk][K/128][512]: hi (32-route tiles: hi and lo)
  const uint8_t* sfl;           // lo (128-route tiles)
  const int4* chunks;           // {first routed row, rows, expert, 0}
  const int32_t* num_chunks;
  int max_chunks;
  const int32_t* sorted_ids;
  int num_routes;
  int top_k;
  void* out;
  int64_t ldo;
  int out_dtype;
  const float* a_scale;
  const float* b_scale;
  const void* topk_w;
  int w_dtype;
  int mul_w;
  int64_t c_stride_t, c_stride_j;
};

// Instruction descriptor, kind::mxf8f6f4 block-scaled: A = E2M1 (format 5),
// B = E4M3 (format 0), E8M0 scales (bit 23), FP32 accumulate, K-major, K = 32.
__host__ __device__ constexpr uint32_t idesc_mx8(int m, int n) {
  return (5u << 7) | (0u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_mx8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// 3-D / 4-D tile loads (tensor maps whose outer dimension walks the 128-K
// stages, so one copy brings several stages).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 int z, int w, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Byte offset of the scale word (4 codes) of route j of chunk ci, K chunk c.
__host__ __device__ __forceinline__ int64_t mx8_sf_offset(int64_t ci, int kc, int c, int j) {
  return (ci * kc + c) * 512 + (j % 32) * 16 + (j / 32) * 4;
}

// Two floats -> two E4M3 codes (RNE, saturating), `a` in the low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}
// Two E4M3 codes (low byte first) -> two floats (exact).
__device__ __forceinline__ void e4m3x2_to_f32x2(uint32_t codes, float& a, float& b) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(codes)));
  a = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFF)));
  b = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 >> 16)));
}

// The hi/lo split of one 128-value piece held 4 values per lane (block =
// lane / 8): returns the lane's 4 hi and 4 lo codes and, in lanes 8b, block b's
// scale codes.
__device__ __forceinline__ void mx8_split_piece(uint2 raw, uint32_t& hi4, uint32_t& lo4, int& hc, int& lc) {
  const float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                      __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u)};
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a = __float_as_uint(v[i]) & 0x7FFFFFFFu;
    amax_bits = a > amax_bits ? a : amax_bits;
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    const uint32_t t = __shfl_xor_sync(0xFFFFFFFFu, amax_bits, o);
    amax_bits = t > amax_bits ? t : amax_bits;
  }
  // hi code = biased exponent of max|x| - 7 (>= 0); an all-zero block takes 127
  hc = amax_bits == 0 ? 127 : static_cast<int>(amax_bits >> 23) - 7;
  hc = hc < 0 ? 0 : (hc > 254 ? 254 : hc);
  const int sh = hc < kMx8LoShift ? hc : kMx8LoShift;
  lc = hc - sh;
  // 2^(127 - hc) (hc <= 253: a normal power of two; hc = 254: 2^-127)
  const float inv = __uint_as_float(hc <= 253 ? static_cast<uint32_t>(254 - hc) << 23 : 0x00400000u);
  const float up = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
  float xs[4], hv[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) xs[i] = v[i] * inv;
  const uint32_t h01 = f32x2_to_e4m3x2(xs[0], xs[1]);
  const uint32_t h23 = f32x2_to_e4m3x2(xs[2], xs[3]);
  e4m3x2_to_f32x2(h01, hv[0], hv[1]);
  e4m3x2_to_f32x2(h23, hv[2], hv[3]);
#pragma unroll
  for (int i = 0; i < 4; ++i) lo[i] = (xs[i] - hv[i]) * up;
  hi4 = h01 | (h23 << 16);
  lo4 = f32x2_to_e4m3x2(lo[0], lo[1]) | (f32x2_to_e4m3x2(lo[2], lo[3]) << 16);
}

// Split BF16 rows into E4M3 hi/lo codes and their E8M0 scales.  CTA per
// route chunk of the routing's chunk table (up to 128 rows), warp per row (32
// warps), up to sixteen 128-value pieces loaded at a time (lane l: values
// 4l..4l+3 of each piece).  GATHER: routed row r is activation row
// sorted[r] / top_k; otherwise row r of `x`.  Padding rows (sorted[r] >=
// num_routes) are skipped: a B row only reaches its own output column of the
// MMA, which the epilogue drops for padding, so whatever those rows and their
// scales hold never reaches a result.
constexpr int kMx8SplitBatch = 16;
constexpr int kMx8SplitThreads = 1024;
template <bool GATHER>
__global__ void __launch_bounds__(kMx8SplitThreads) mx8_split_kernel(const uint16_t* __restrict__ x, int64_t ldx, int K,
                                                         const int4* __restrict__ chunks,
                                                         const int32_t* __restrict__ num_chunks, int max_chunks,
                                                         const int32_t* __restrict__ sorted, int num_routes,
                                                         int top_k, uint8_t* __restrict__ xh,
                                                         uint8_t* __restrict__ xl, uint8_t* __restrict__ sfh,
                                                         uint8_t* __restrict__ sfl) {
  // sfl == sfh + 4: lo's scales in the chunk's next 32-row column (32-route chunks)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int nch = num_chunks[0];
  nch = nch < max_chunks ? nch : max_chunks;
  const int KC = K / 128;
  for (int ci = blockIdx.x; ci < nch; ci += gridDim.x) {
    const int4 ch = chunks[ci];
    for (int j = warp; j < ch.y; j += nwarps) {
      const int64_t r = static_cast<int64_t>(ch.x) + j;
      const int sid = sorted[r];
      if (sid >= num_routes) continue;  // padding (uniform over the warp)
      const int64_t src = GATHER ? sid / top_k : r;
      const uint16_t* xrow = x + src * ldx + 4 * lane;
      for (int c0 = 0; c0 < KC; c0 += kMx8SplitBatch) {
        uint2 raw[kMx8SplitBatch];
#pragma unroll
        for (int u = 0; u < kMx8SplitBatch; ++u)
          raw[u] = c0 + u < KC ? *reinterpret_cast<const uint2*>(xrow + (c0 + u) * 128) : make_uint2(0u, 0u);
#pragma unroll
        for (int u = 0; u < kMx8SplitBatch; ++u) {
          const int c = c0 + u;
          if (c >= KC) break;
          uint32_t hi4, lo4;
          int hc, lc;
          mx8_split_piece(raw[u], hi4, lo4, hc, lc);
          const int64_t off = r * K + c * 128 + 4 * lane;
          *reinterpret_cast<uint32_t*>(xh + off) = hi4;
          *reinterpret_cast<uint32_t*>(xl + off) = lo4;
          // scale words: block q's codes come from lane 8q
          uint32_t hw = 0, lw = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            hw |= (static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, hc, 8 * q)) & 0xFF) << (8 * q);
            lw |= (static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, lc, 8 * q)) & 0xFF) << (8 * q);
          }
          const int64_t so = mx8_sf_offset(ci, KC, c, j);
          if (lane == 0) *reinterpret_cast<uint32_t*>(sfh + so) = hw;
          if (lane == 1) *reinterpret_cast<uint32_t*>(sfl + so) = lw;
        }
      }
    }
  }
}

// Weight row of local A row r (0..127) for weight block wb of expert e.
template <int EPI>
__device__ __forceinline__ int64_t mx8_weight_row(const Mx8Params& p, int e, int wb, int r, bool& valid) {
  const int64_t base = static_cast<int64_t>(e) * p.w_rows_per_expert;
  if (EPI == EPI_GLU) {
    const int col = wb * 64 + (r & 63);
    valid = col < p.glu_inter;
    return base + (r < 64 ? col : p.glu_inter + col);
  }
  const int row = wb * 128 + r;
  valid = row < p.N;
  return base + row;
}

// 32 accumulator columns (routes c0..c0+31) of this warp's lane quarter, the
// sum of the tile's NACC accumulators (BN columns apart).
template <int NACC, int BN>
__device__ __forceinline__ void mx8_load_acc(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld_32x32b_x32(taddr, r);
  if (NACC > 1) {
    uint32_t t[32];
#pragma unroll
    for (int a = 1; a < NACC; ++a) {
      tmem_ld_32x32b_x32(taddr + a * BN, t);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(t[i]));
    }
  }
  tmem_ld_wait();
}

// Weight map (tmap_w) over the packed codes as 4-bit elements.  Plain: 3-D,
// dims {128 K, rows, K / 128 stages}, box {128, 128, group}.  GLU: 4-D, dims
// {128 K, rows, 2 halves (inter rows apart), K / 128 stages}, box
// {128, 64, 2, group}.  Either way a group of stages of the 128-row A tile
// (GLU: the 64 gate rows then the 64 up rows of the same columns) lands as
// [stage][128 rows][128 bytes].  Route maps over the E4M3 rows: 32-route tiles
// one 4-D map (tmap_xh), dims {128 K, rows, 2 parts (hi, lo), K / 128 stages},
// box {128, 32, 2, group}, landing as [stage][hi 32 rows, lo 32 rows];
// 128-route tiles 3-D maps of hi (tmap_xh) and lo (tmap_xl), dims
// {128 K, rows, K / 128 stages}, box {128, 32, 1}.
template <int EPI, int BN>
__global__ void __launch_bounds__(Mx8Cfg<BN>::kThreads, 1)
    mxfp4_routed_mx8_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_xh,
                            const __grid_constant__ CUtensorMap tmap_xl, const Mx8Params p) {
  using Cfg = Mx8Cfg<BN>;
  constexpr int S = Cfg::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;           // [S] (groups use the first S / G)
  uint64_t* empty = full + S;      // [S]
  uint64_t* tfull = empty + S;     // [2]
  uint64_t* tempty = tfull + 2;    // [2]
  uint64_t* drain = tempty + 2;
  uint64_t* sfready = drain + 1;   // [S]: a group's scales are in tensor memory (4 scale-writer warps)
  uint64_t* sffull = sfready + S;  // [S]: a group's weight and activation scales landed in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);
  int32_t* route_ids = reinterpret_cast<int32_t*>(smem + Cfg::kOffRoute);
  float* route_w = reinterpret_cast<float*>(smem + Cfg::kOffRoute + BN * 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = p.K / 128;
  const int G = p.group;
  const int NG = S / G;     // groups in the ring
  const int KG = KT / G;    // groups per tile
  // the copies' alignment rules (bulk copies: 16 bytes; scale words: 4 bytes),
  // the group shape and the 16-bit output the staging tile is sized for,
  // checked before any copy is issued; the host establishes them, so this only
  // guards against a caller that bypassed its checks
  if ((reinterpret_cast<uintptr_t>(p.sfh) & 15) != 0 || (!Cfg::kStackHiLo && (reinterpret_cast<uintptr_t>(p.sfl) & 15) != 0) ||
      (reinterpret_cast<uintptr_t>(p.w_scales) & 3) != 0 || (p.lds & 3) != 0 || (p.K & 127) != 0 ||
      p.out_dtype == MXFP4_DTYPE_F32 || G < 1 || S % G != 0 || KT % G != 0) {
    if (threadIdx.x == 0) record_error(MXFP4_ERR_INVALID_ARGUMENT);
    return;
  }

  if (threadIdx.x == 0) {
    for (int g = 0; g < S; ++g) {
      mbar_init(&full[g], 1);         // the TMA producer's expect_tx (weight and route tiles)
      mbar_init(&sffull[g], 1 + 32);  // its expect_tx (activation scales) + the scale warp's 32 cp.async arrivals
      mbar_init(&empty[g], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    for (int g = 0; g < S; ++g) mbar_init(&sfready[g], 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_xh);
    if (!Cfg::kStackHiLo) prefetch_tmap(&tmap_xl);  // unused (zero) with stacked hi/lo
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kMx8TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  int nch = p.num_chunks[0];
  nch = nch < p.max_chunks ? nch : p.max_chunks;
  const int num_tiles = nch * p.num_wblocks;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (lane 0)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int it = 0;
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int ci = t / p.num_wblocks;
        const int4 ch = p.chunks[ci];
        const int wb = t % p.num_wblocks;
        bool v;
        const int row0 = static_cast<int>(mx8_weight_row<EPI>(p, ch.z, wb, 0, v));
        const int nbox = ch.y / 32;  // one box when G > 1 (BN = 32)
        const uint32_t tx = G * (128 * 64 + 2 * ch.y * 128);
        const uint32_t tx_sf = G * Cfg::kSfbSlot;
        for (int kg = 0; kg < KG; ++kg, ++it) {
          const int g = it % NG;
          const uint32_t ph = (it / NG) & 1;
          if (!mbar_wait(&empty[g], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[g], tx);
          mbar_arrive_expect_tx(&sffull[g], tx_sf);
          armed |= 1u << g;
          armed_par = (armed_par & ~(1u << g)) | (ph << g);
          const int s0 = g * G, kt0 = kg * G;
          // the small scale copies first: the scale writers start on them while the tiles are in flight
          const int64_t sfo = (static_cast<int64_t>(ci) * KT + kt0) * 512;
          if (Cfg::kStackHiLo) {
            bulk_load(smem + Cfg::kOffSfb + s0 * Cfg::kSfbSlot, p.sfh + sfo, G * Cfg::kSfbBytes, &sffull[g]);
          } else {
            bulk_load(smem + Cfg::kOffSfb + s0 * Cfg::kSfbSlot, p.sfh + sfo, Cfg::kSfbBytes, &sffull[g]);
            bulk_load(smem + Cfg::kOffSfb + s0 * Cfg::kSfbSlot + Cfg::kSfbBytes, p.sfl + sfo, Cfg::kSfbBytes,
                      &sffull[g]);
          }
          if (EPI == EPI_GLU)
            tma_load_4d_hint(smem + Cfg::kOffA + s0 * Cfg::kABytes, &tmap_w, &full[g], 0, row0, 0, kt0, pol_w);
          else
            tma_load_3d_hint(smem + Cfg::kOffA + s0 * Cfg::kABytes, &tmap_w, &full[g], 0, row0, kt0, pol_w);
          uint8_t* bslot = smem + Cfg::kOffB + s0 * 2 * Cfg::kBBytes;
          if (Cfg::kStackHiLo) {
            // [stage][hi 32 rows, lo 32 rows] in one copy; the scales of both in one chunk per stage
            tma_load_4d(bslot, &tmap_xh, &full[g], 0, ch.x, 0, kt0);
          } else {
            for (int i = 0; i < nbox; ++i) {
              tma_load_3d(bslot + i * 32 * 128, &tmap_xh, &full[g], 0, ch.x + 32 * i, kt0);
              tma_load_3d(bslot + Cfg::kBBytes + i * 32 * 128, &tmap_xl, &full[g], 0, ch.x + 32 * i, kt0);
            }
          }
        }
      }
      if (!ok || *abort_flag)
        for (int g = 0; g < NG; ++g)
          if (armed & (1u << g)) {
            mbar_drain(&full[g], (armed_par >> g) & 1u);
            mbar_drain(&sffull[g], (armed_par >> g) & 1u);
          }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ weight-scale producer (whole warp)
    // copy j of a stage writes bytes [4 lane, 4 lane + 4) of the stage's
    // 512-byte chunk segment j (conflict-free): local row
    // r = 32 (lane % 4) + lane / 4 + 8 j; rows past the expert's last feature
    // read row 0's scales (their results are dropped)
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int4 ch = p.chunks[t / p.num_wblocks];
      const int wb = t % p.num_wblocks;
      bool v;
      const int64_t row0 = mx8_weight_row<EPI>(p, ch.z, wb, 0, v);
      const uint8_t* srow[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = 32 * (lane & 3) + (lane >> 2) + 8 * j;
        bool valid;
        const int64_t gr = mx8_weight_row<EPI>(p, ch.z, wb, r, valid);
        srow[j] = p.w_scales + (valid ? gr : row0) * p.lds;
      }
      for (int kg = 0; kg < KG; ++kg, ++it) {
        const int g = it % NG;
        const uint32_t ph = (it / NG) & 1;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[g], ph ^ 1, abort_flag))) { ok = false; break; }
        const uint32_t sfa = smem_u32(smem + Cfg::kOffSfa + g * G * Cfg::kSfaBytes) + 4 * lane;
        for (int st = 0; st < G; ++st) {
          const int kt = kg * G + st;
#pragma unroll
          for (int j = 0; j < 4; ++j) cp_async_4(sfa + st * Cfg::kSfaBytes + 128 * j, srow[j] + 4 * kt);
        }
        cp_async_arrive_noinc(&sffull[g]);
      }
    }
    cp_async_wait_all();
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, tl = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tl) {
        const int4 ch = p.chunks[t / p.num_wblocks];
        const uint32_t idesc0 = idesc_mx8(128, Cfg::kStackHiLo ? 2 * ch.y : ch.y);
        const int acc = tl & 1;
        if (!mbar_wait(&tempty[acc], ((tl >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 128;
        for (int kg = 0; kg < KG; ++kg, ++it) {
          const int g = it % NG;
          if (!mbar_wait(&full[g], (it / NG) & 1, abort_flag)) { ok = false; break; }
          // the group's scales, written into tensor memory by the scale-writer warps
          if (!mbar_wait(&sfready[g], (it / NG) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          for (int st = 0; st < G; ++st) {
            const int s = g * G + st;
            const int kt = kg * G + st;
            const uint32_t sf_t = tmem_base + kMx8SfCol + kMx8SfRegion * s;  // weights, hi, lo: 4 columns each
            const uint64_t adesc = desc_sw128(smem_u32(smem + Cfg::kOffA + s * Cfg::kABytes));
            const uint64_t bhdesc = desc_sw128(smem_u32(smem + Cfg::kOffB + s * 2 * Cfg::kBBytes));
            const uint64_t bldesc = desc_sw128(smem_u32(smem + Cfg::kOffB + s * 2 * Cfg::kBBytes + Cfg::kBBytes));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t sel = static_cast<uint32_t>(j) << 30;
              const uint32_t idesc = idesc0 | (static_cast<uint32_t>(j) << 29) | (static_cast<uint32_t>(j) << 4);
              if (Cfg::kStackHiLo) {
                // N = hi rows then lo rows: columns [0, 32) hi, [32, 64) lo of the even / odd K-step accumulator
                const uint32_t first = (kt == 0 && j < 2) ? 0u : 1u;
                umma_mx8(d_tmem + (j & 1) * 2 * BN, adesc + 2 * j, bhdesc + 2 * j, idesc, sf_t | sel, (sf_t + 4) | sel,
                         first);
              } else {
                umma_mx8(d_tmem, adesc + 2 * j, bhdesc + 2 * j, idesc, sf_t | sel, (sf_t + 4) | sel, (kt | j) != 0);
                umma_mx8(d_tmem, adesc + 2 * j, bldesc + 2 * j, idesc, sf_t | sel, (sf_t + 8) | sel, 1);
              }
            }
          }
          umma_commit(&empty[g]);
          issued = true;
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok && issued) {
        // the issued MMAs finish before the CTA (and its tensor memory) goes away
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ scale writers (warps 8-11)
    // Warp 8 + q writes lane quarter q of each stage's tensor-memory scale
    // region: lane i takes the 16 bytes of row i of the stage's weight-scale
    // chunk and of its activation-scale chunk(s) from shared memory (the
    // layout tcgen05.cp .32x128b.warpx4 would copy: column j = rows 32 j + i,
    // the same in all four quarters) and stores them with tcgen05.st.  The
    // slot's previous scales are free once its new scale copies have landed
    // (the producer and the scale warp refill a slot only after the MMAs that
    // read it completed).
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      bool ok = true;
      for (int kg = 0; kg < KG; ++kg, ++it) {
        const int g = it % NG;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sffull[g], (it / NG) & 1, abort_flag))) { ok = false; break; }
        for (int st = 0; st < G; ++st) {
          const int s = g * G + st;
          const uint32_t sf_t = tmem_base + lane_base + kMx8SfCol + kMx8SfRegion * s;
          const uint4 a = ld_shared_v4(smem_u32(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes) + 16 * lane);
          const uint32_t sfb = smem_u32(smem + Cfg::kOffSfb + s * Cfg::kSfbSlot) + 16 * lane;
          const uint4 b = ld_shared_v4(sfb);
          const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
          tmem_st_32x32b_x8(sf_t, v);
          if (!Cfg::kStackHiLo) {
            const uint4 c = ld_shared_v4(sfb + Cfg::kSfbBytes);
            const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
            tmem_st_32x32b_x4(sf_t + 8, w4);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfready[g]);
      }
      if (!ok) break;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp & 3;
    const int etid = threadIdx.x - 128;  // 0..127
    const int f = q * 32 + lane;         // accumulator lane = A row
    const int esz = out_esize(p.out_dtype);
    uint8_t* stage = smem + Cfg::kOffOut;
    volatile int* vote = reinterpret_cast<volatile int*>(smem + Cfg::kOffVote);
    int tl = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tl) {
      const int4 ch = p.chunks[t / p.num_wblocks];
      const int wb = t % p.num_wblocks;
      const int n = ch.y;
      const int acc = tl & 1;
      named_bar_sync(1, 128);  // the previous tile's store phase is done with the staging tile
      for (int j = etid; j < n; j += 128) {
        const int sid = p.sorted_ids[ch.x + j];
        route_ids[j] = sid;
        route_w[j] = (EPI == EPI_MOE && p.mul_w && sid < p.num_routes) ? load_weight(p.topk_w, p.w_dtype, sid) : 1.0f;
      }
      const bool got = __all_sync(0xFFFFFFFFu, mbar_wait(&tfull[acc], (tl >> 1) & 1, abort_flag));
      if (lane == 0) vote[q] = got ? 1 : 0;
      named_bar_sync(1, 128);
      if (!(vote[0] && vote[1] && vote[2] && vote[3])) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + acc * 128 + (static_cast<uint32_t>(q * 32) << 16);
      if (EPI == EPI_GLU) {
        uint16_t* st16 = reinterpret_cast<uint16_t*>(stage);
        for (int c0 = 0; c0 < n; c0 += 32) {
          uint32_t r32[32];
          mx8_load_acc<Cfg::kAcc, BN>(tbase + c0, r32);
#pragma unroll
          for (int i = 0; i < 32; ++i) st16[(c0 + i) * 128 + f] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r32[i])));
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (lane == 0) mbar_arrive(&tempty[acc]);
        const int col0 = wb * 64;
        const int ncols = p.glu_inter - col0 < 64 ? p.glu_inter - col0 : 64;
        for (int i = etid; i < n * 8; i += 128) {
          const int j = i >> 3, c = i & 7;
          if (c * 8 >= ncols) continue;
          if (route_ids[j] >= p.num_routes) continue;  // padding: the h split and the down GEMM drop its row
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
        const int feat0 = wb * 128;
        const int nfeat = p.N - feat0 < 128 ? p.N - feat0 : 128;
        const bool scales = p.a_scale != nullptr;
        const float asc = scales ? p.a_scale[0] : 1.0f;
        const float bsc = scales ? p.b_scale[ch.z] : 1.0f;
        const bool mul = p.mul_w != 0;
        for (int c0 = 0; c0 < n; c0 += 32) {
          uint32_t r32[32];
          mx8_load_acc<Cfg::kAcc, BN>(tbase + c0, r32);
          if (p.out_dtype == MXFP4_DTYPE_BF16)
            rt_plain_chunk_any<MXFP4_DTYPE_BF16>(r32, stage, c0, f, asc, bsc, route_w + c0, scales, mul);
          else
            rt_plain_chunk_any<MXFP4_DTYPE_F16>(r32, stage, c0, f, asc, bsc, route_w + c0, scales, mul);
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (lane == 0) mbar_arrive(&tempty[acc]);
        const int row_bytes = 128 * esz;
        const int vec_per_row = row_bytes / 16;
        for (int i = etid; i < n * vec_per_row; i += 128) {
          const int jj = i / vec_per_row, c = i % vec_per_row;
          const int sid = route_ids[jj];
          if (sid >= p.num_routes) continue;
          const int first = c * 16 / esz;
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
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kMx8TmemCols);
}

}  // namespace mx
