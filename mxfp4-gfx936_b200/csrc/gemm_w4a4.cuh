// W4A4: packed-MXFP4 activations x packed-MXFP4 weights on the block-scaled
// tensor cores (tcgen05.mma.kind::mxf4, UE8M0 scale per 32 K on both sides).
//
// Semantics: out = round(dequant(A) . dequant(B)^T) with FP32 accumulation,
// the reference's W4A4 result (soft:468-475 dequantises packed activations,
// then one matmul).  Every E2M1 x E2M1 product scaled by 2^(sa+sb-254) is exact
// in FP32, so only the accumulation order differs from the BF16 reference.
//
// Layout: both operands stay packed in HBM and reach shared memory by TMA in
// the 128-byte-swizzled K-major layout (one 128-byte row = 256 codes = one
// K stage).  The E8M0 scales are first rearranged (sf_block_kernel) into
// 512-byte chunks of 128 rows x 4 scale blocks, the layout tcgen05.cp copies
// into tensor memory: byte (r, kb) of a chunk sits at (r%32)*16 + (r/32)*4 + kb.
// Per stage four scale-writer warps (one per TMEM lane quarter) store the 2
// SFA chunks and 4 SFB chunks from shared memory into the stage's own TMEM
// scale region with tcgen05.st (lane i: row i of each chunk, the layout the
// .32x128b.warpx4 copy would produce), and the MMA thread issues only the four
// K=64 MMAs; as one tcgen05.cp per chunk from the MMA thread these copies set
// the kernel's pace.
#pragma once

#include "common.cuh"

namespace mx {

constexpr int kW4Stages = 4;
constexpr int kW4BM = 128, kW4BN = 256;
constexpr int kW4KStage = 256;                   // codes per stage (128 bytes per row)
constexpr int kW4ABytes = kW4BM * 128;           // 16 KB
constexpr int kW4BBytes = kW4BN * 128;           // 32 KB
constexpr int kW4SfaBytes = 2 * 512;             // 2 chunks x 128 rows
constexpr int kW4SfbBytes = 4 * 512;             // 2 row halves x 2 chunks
constexpr int kW4StageBytes = kW4ABytes + kW4BBytes + kW4SfaBytes + kW4SfbBytes;
constexpr int kW4OffBar = kW4Stages * kW4StageBytes;
constexpr int kW4SmemBytes = kW4OffBar + (3 * kW4Stages + 3) * 8 + 64 + 1024;
constexpr int kW4Threads = 384;                  // warps 0-1 copies / MMA, 4-7 epilogue, 8-11 scale writers
constexpr uint32_t kW4TmemCols = 512;            // accumulator 0..255, scale regions from 256
// scale region of stage slot s at column 256 + 24 s: SFA chunks c = 0, 1 at
// +4c, SFB chunk (c, row half h) at +8 + 8c + 4h
constexpr uint32_t kW4SfCol = 256, kW4SfRegion = 24;
static_assert(kW4SfCol + kW4Stages * kW4SfRegion <= kW4TmemCols, "W4A4 scale regions in tensor memory");

struct W4A4Params {
  int M, N, K;
  int num_m_blocks, num_n_blocks;
  const uint8_t* sfa_blk;   // [ceil(M/128)][K/128][512]
  const uint8_t* sfb_blk;   // [2*ceil(N/256)][K/128][512]
  void* out;
  int64_t ldo;
  int out_dtype;
  int vec_ok;
};

// E8M0 scales [rows, K/32] -> 512-byte tcgen05.cp chunks [rows/128][K/128][512].
// One thread per 32-bit word (4 consecutive scale blocks of one row).
__global__ void __launch_bounds__(256) sf_block_kernel(const uint8_t* __restrict__ src, int64_t lds, int rows,
                                                       int kchunks, int row_blocks, uint8_t* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(row_blocks) * 128 * kchunks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / kchunks;
    const int c = static_cast<int>(i % kchunks);
    uint32_t w = 0;
    if (r < rows) {
      const uint8_t* p = src + r * lds + 4 * c;
      w = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
          (static_cast<uint32_t>(p[3]) << 24);
    }
    const int64_t rb = r / 128;
    const int rr = static_cast<int>(r % 128);
    uint8_t* chunk = dst + ((rb * kchunks) + c) * 512;
    *reinterpret_cast<uint32_t*>(chunk + (rr % 32) * 16 + (rr / 32) * 4) = w;
  }
}

// Non-swizzled K-major descriptor over a 512-byte scale chunk: 32 rows of 16
// bytes, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t desc_sf_chunk(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(512 >> 4) << 16;   // LBO (single core matrix along K; unused)
  d |= static_cast<uint64_t>(128 >> 4) << 32;   // SBO: next 8 rows
  d |= static_cast<uint64_t>(1) << 46;          // version
  return d;                                     // layout 0 = no swizzle
}

// Instruction descriptor, kind::mxf4 block-scaled: E2M1 A/B (format 1),
// UE8M0 scales (bit 23), FP32 accumulate implied, K-major, dense K=64.
__host__ __device__ constexpr uint32_t idesc_mxf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__global__ void __launch_bounds__(kW4Threads, 1)
    mxfp4_w4a4_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const W4A4Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kW4OffBar);
  uint64_t* empty = full + kW4Stages;
  uint64_t* tfull = empty + kW4Stages;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tfull + 2;
  uint64_t* sfready = drain + 1;  // [kW4Stages]: a stage's scales are in TMEM (4 scale-writer warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sfready + kW4Stages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = (p.K + kW4KStage - 1) / kW4KStage;
  const int kchunks = p.K / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kW4Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 4);
    mbar_init(drain, 1);
    for (int s = 0; s < kW4Stages; ++s) mbar_init(&sfready[s], 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kW4TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m_blk = t % p.num_m_blocks, n_blk = t / p.num_m_blocks;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kW4Stages;
          const uint32_t ph = (it / kW4Stages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* st = smem + s * kW4StageBytes;
          // scale chunks of this stage: 2 (A rows) + 2 x 2 (B row halves); the
          // last stage of a K that is not a multiple of 256 has one chunk pair
          const int nch = (2 * kt + 2 <= kchunks) ? 2 : kchunks - 2 * kt;
          const uint32_t tx = kW4ABytes + kW4BBytes + 3u * nch * 512u;
          mbar_arrive_expect_tx(&full[s], tx);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          tma_load_2d(st, &tmap_a, &full[s], kt * 128, m_blk * kW4BM);
          tma_load_2d(st + kW4ABytes, &tmap_b, &full[s], kt * 128, n_blk * kW4BN);
          uint8_t* sfa = st + kW4ABytes + kW4BBytes;
          uint8_t* sfb = sfa + kW4SfaBytes;
          bulk_load(sfa, p.sfa_blk + (static_cast<int64_t>(m_blk) * kchunks + 2 * kt) * 512, nch * 512, &full[s]);
          for (int h = 0; h < 2; ++h)
            bulk_load(sfb + h * 1024, p.sfb_blk + (static_cast<int64_t>(2 * n_blk + h) * kchunks + 2 * kt) * 512,
                      nch * 512, &full[s]);
        }
      }
      if (!ok || *abort_flag)
        for (int s = 0; s < kW4Stages; ++s)
          if (armed & (1u << s)) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], (armed_par >> s) & 1u) && clock64() - t0 < kWaitCycles) {
            }
          }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc0 = idesc_mxf4(kW4BM, kW4BN);
      int it = 0, tl = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tl) {
        if (!mbar_wait(tempty, (tl & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kW4Stages;
          const uint32_t ph = (it / kW4Stages) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&sfready[s], ph, abort_flag)) { ok = false; break; }  // the stage's scales in TMEM
          tc_fence_after();
          uint8_t* st = smem + s * kW4StageBytes;
          const int nch = (2 * kt + 2 <= kchunks) ? 2 : kchunks - 2 * kt;
          const uint32_t sf_t = tmem_base + kW4SfCol + kW4SfRegion * s;
          const uint64_t adesc = desc_sw128(smem_u32(st));
          const uint64_t bdesc = desc_sw128(smem_u32(st + kW4ABytes));
          for (int j = 0; j < 2 * nch; ++j) {
            const uint32_t sf_id = (j & 1) * 2;
            const uint32_t c = j >> 1;
            const uint32_t sfa_t = (sf_t + 4 * c) | (sf_id << 30);
            const uint32_t sfb_t = (sf_t + 8 + 8 * c) | (sf_id << 30);
            const uint32_t idesc = idesc0 | (sf_id << 29) | (sf_id << 4);
            umma_mxf4(tmem_base, adesc + 2 * j, bdesc + 2 * j, idesc, sfa_t, sfb_t, (kt | j) != 0);
          }
          umma_commit(&empty[s]);
          issued = true;
        }
        if (!ok) break;
        umma_commit(tfull);
      }
      if (!ok && issued) {
        umma_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ scale writers (warps 8-11)
    // warp 8 + q stores lane quarter q of each stage's scale region: lane i
    // takes row i (16 bytes) of every scale chunk of the stage.  A slot's
    // region is free again once its next copies have landed: the producer
    // refills the slot only after the MMAs that read it completed.
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % kW4Stages;
        const uint32_t ph = (it / kW4Stages) & 1;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
        const uint32_t sfa = smem_u32(smem + s * kW4StageBytes + kW4ABytes + kW4BBytes) + 16 * lane;
        const uint32_t sfb = sfa + kW4SfaBytes;
        // chunks past K (a last stage of 128 K) hold stale bytes in columns no MMA reads
        const uint4 a0 = ld_shared_v4(sfa), a1 = ld_shared_v4(sfa + 512);
        const uint4 b00 = ld_shared_v4(sfb), b01 = ld_shared_v4(sfb + 1024);   // chunk 0, row halves 0 / 1
        const uint4 b10 = ld_shared_v4(sfb + 512), b11 = ld_shared_v4(sfb + 1536);  // chunk 1
        const uint32_t va[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t vb0[8] = {b00.x, b00.y, b00.z, b00.w, b01.x, b01.y, b01.z, b01.w};
        const uint32_t vb1[8] = {b10.x, b10.y, b10.z, b10.w, b11.x, b11.y, b11.z, b11.w};
        const uint32_t sf_t = tmem_base + lane_base + kW4SfCol + kW4SfRegion * s;
        tmem_st_32x32b_x8(sf_t, va);
        tmem_st_32x32b_x8(sf_t + 8, vb0);
        tmem_st_32x32b_x8(sf_t + 16, vb1);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfready[s]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    const int r_local = q * 32 + lane;
    const int esz = p.out_dtype == MXFP4_DTYPE_F32 ? 4 : 2;
    int tl = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tl) {
      const int m_blk = t % p.num_m_blocks, n_blk = t / p.num_m_blocks;
      if (!mbar_wait(tfull, tl & 1, abort_flag)) break;
      tc_fence_after();
      const int row = m_blk * kW4BM + r_local;
      const bool row_ok = row < p.M;
      uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<int64_t>(row_ok ? row : 0) * p.ldo * esz;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int cc = 0; cc < kW4BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + cc * 32, r);
        tmem_ld_wait();
        const int col0 = n_blk * kW4BN + cc * 32;
        if (row_ok && col0 < p.N) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          if (p.out_dtype == MXFP4_DTYPE_F32) {
            float* o = reinterpret_cast<float*>(orow) + col0;
            const int nc = p.N - col0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nc) o[i] = v[i];
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = p.out_dtype == MXFP4_DTYPE_BF16 ? f32x2_to_bf16x2(v[2 * i], v[2 * i + 1])
                                                      : f32x2_to_f16x2(v[2 * i], v[2 * i + 1]);
            uint16_t* o = reinterpret_cast<uint16_t*>(orow) + col0;
            if (p.vec_ok && p.N - col0 >= 32) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                reinterpret_cast<uint4*>(o)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            } else {
              const int nc = p.N - col0;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < nc) o[i] = static_cast<uint16_t>((pk[i >> 1] >> ((i & 1) * 16)) & 0xFFFF);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kW4TmemCols);
}

// ---------------------------------------------------------------------------
// OCP MXFP4 quantizer (the W4A4 configuration's rounding): per 32 values,
// q = fl32(max|x| / 6), e = floor(log2 q), scale code = clamp(e + 127, 0, 254)
// (0 for an all-zero block); element = RNE(x * 2^(127-code)) on the E2M1 grid,
// ties to the even code, saturated at 6; zero results carry no sign.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e2m1_rne_code(float v) {
  const float a = fabsf(v);
  const uint32_t mag = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) +
                       (a > 5.0f);
  return mag | ((mag != 0 && signbit(v)) ? 8u : 0u);
}

template <int IN>
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ x, int64_t ldx, int64_t rows,
                                                       int64_t k, uint8_t* __restrict__ packed,
                                                       uint8_t* __restrict__ scales) {
  const int64_t nb = k / 32;
  const int64_t total = rows * nb;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = b / nb, kb = b % nb;
    float v[32];
    if (IN == MXFP4_DTYPE_BF16) {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + r * ldx + kb * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 q = src[i];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
          v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
    } else {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(x) + r * ldx + kb * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q = src[i];
        v[4 * i] = q.x;
        v[4 * i + 1] = q.y;
        v[4 * i + 2] = q.z;
        v[4 * i + 3] = q.w;
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    uint32_t code = 0;
    if (amax > 0.0f) {
      const float q = __fdiv_rn(amax, 6.0f);
      const uint32_t bits = __float_as_uint(q);
      int e = static_cast<int>((bits >> 23) & 0xFF) - 127;
      if ((bits >> 23) == 0) e = (31 - __clz(static_cast<int>(bits))) - 149;  // subnormal q
      int c = e + 127;
      code = static_cast<uint32_t>(c < 0 ? 0 : (c > 254 ? 254 : c));
    }
    const float inv = __uint_as_float(code <= 253 ? (254u - code) << 23 : 0x00400000u);  // 2^(127-code)
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) w |= e2m1_rne_code(v[8 * i + j] * inv) << (4 * j);
      out[i] = w;
    }
    *reinterpret_cast<uint4*>(packed + r * (k / 2) + kb * 16) = make_uint4(out[0], out[1], out[2], out[3]);
    scales[r * nb + kb] = static_cast<uint8_t>(code);
  }
}

}  // namespace mx
