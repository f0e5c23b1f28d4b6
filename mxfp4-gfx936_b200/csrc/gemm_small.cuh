// Dense W4A16 linear for few tokens (M <= 256): the decode regime.
//
// With few rows of x, a 256x256 pair tile leaves most SMs idle while the few
// busy ones walk all of K.  This kernel swaps the operands and splits K:
//   * MMA M = 128 weight rows (the decoded E2M1 tile is operand A), MMA N =
//     the tokens padded to a multiple of 32 (x is operand B), D = W . x^T in
//     tensor memory, one lane per weight row;
//   * the KS CTAs of a thread-block cluster share one 128-row block of W and
//     take consecutive K ranges;
//   * each CTA writes its FP32 partial D to shared memory; after a cluster
//     barrier CTA c sums rows [c*128/KS, (c+1)*128/KS) of all KS partials
//     through distributed shared memory in rank order (deterministic), adds
//     the bias with the reference's two roundings and stores out[token][n].
// Safe mode uses the same kernel with the dequantised BF16 weight tile loaded
// by TMA, so fused and safe results stay bit-identical.
#pragma once

#include "gemm.cuh"

namespace mx {

constexpr int kSmRows = 128;            // weight rows per cluster (MMA M)
constexpr int kSmBK = 64;
constexpr int kSmWBytes = kSmRows * kSmBK * 2;   // 16 KB decoded / loaded weight tile
constexpr int kSmPBytes = kSmRows * kSmBK / 2;   // 4 KB packed codes
constexpr int kSmMaxStages = 4;

struct SmallParams {
  int M, N, K;
  int mp;                   // padded token count (MMA N): multiple of 32, <= 256
  int ks;                   // cluster size = K splits
  int stages;
  int stage_bytes;          // x tile + weight tile (+ packed tile)
  const uint8_t* w_scales;
  int64_t lds;
  void* out;
  int64_t ldo;
  int out_dtype;
  const void* bias;
};

// Partials are complete before the cluster barrier that precedes every read,
// so these loads need no ordering among themselves (no volatile, no clobber)
// and the compiler can keep several in flight.
__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t cluster_addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(cluster_addr));
  return v;
}
__device__ __forceinline__ uint32_t cluster_ctarank_sm() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_sm() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_sm(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}

constexpr int kSmDecodeWarps = 16;  // 4 threads per weight row, 16 K each per stage

template <int BMODE, bool FP16>
__global__ void __launch_bounds__(BMODE == B_DECODE ? 256 + 32 * kSmDecodeWarps : 256, 1)
    mxfp4_linear_small_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                              const SmallParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const int x_bytes = p.mp * 128;
  // per stage: [x tile (mp rows, SW128)][weight tile (128 rows, SW128)][packed (128 x 32 B)]
  const int data_bytes = S * p.stage_bytes;
  const int part_bytes = kSmRows * p.mp * 4;
  const int bar_off = ((data_bytes > part_bytes ? data_bytes : part_bytes) + 15) & ~15;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_off);
  uint64_t* bready = full + kSmMaxStages;
  uint64_t* empty = bready + kSmMaxStages;
  uint64_t* tfull = empty + kSmMaxStages;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* part = reinterpret_cast<float*>(smem);  // reused after the main loop: [mp tokens][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank_sm();
  const int n0 = blockIdx.y * kSmRows;
  const int KT = p.K / kSmBK;
  const int kt0 = static_cast<int>((static_cast<int64_t>(KT) * rank) / p.ks);
  const int kt1 = static_cast<int>((static_cast<int64_t>(KT) * (rank + 1)) / p.ks);
  const uint32_t tmem_cols = p.mp <= 32 ? 32 : (p.mp <= 64 ? 64 : (p.mp <= 128 ? 128 : 256));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kSmDecodeWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      const uint32_t tx = x_bytes + (BMODE == B_DECODE ? kSmPBytes : kSmWBytes);
      for (int kt = kt0, it = 0; kt < kt1; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        uint8_t* st = smem + s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | (ph << s);
        tma_load_2d(st, &tmap_x, &full[s], kt * kSmBK, 0);
        if (BMODE == B_DECODE)
          tma_load_2d(st + x_bytes + kSmWBytes, &tmap_w, &full[s], kt * (kSmBK / 2), n0);
        else
          tma_load_2d(st + x_bytes, &tmap_w, &full[s], kt * kSmBK, n0);
      }
      if (!ok || *abort_flag)
        for (int s = 0; s < S; ++s)
          if (armed & (1u << s)) mbar_drain(&full[s], (armed_par >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(FP16 ? 0 : 1, kSmRows, p.mp);
      bool ok = true, issued = false;
      for (int kt = kt0, it = 0; kt < kt1; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(BMODE == B_DECODE ? &bready[s] : &full[s], ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint8_t* st = smem + s * p.stage_bytes;
        const uint64_t adesc = desc_sw128(smem_u32(st + x_bytes));  // weights: MMA A (M = 128)
        const uint64_t bdesc = desc_sw128(smem_u32(st));            // x: MMA B (N = mp)
#pragma unroll
        for (int k = 0; k < kSmBK / 16; ++k) umma_f16(tmem_base, adesc + 2 * k, bdesc + 2 * k, idesc, (it | k) != 0);
        umma_commit(&empty[s]);
        issued = true;
      }
      if (ok) umma_commit(tfull);
      else if (issued) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp >= 8 && BMODE == B_DECODE) {
    // decoders: 4 threads per weight row, 2 chunks (16 K) each
    const int d = threadIdx.x - 256;
    const int r = d >> 2;
    const int part4 = d & 3;
    const int blk = part4 >> 1;     // scale block (32 K) within the 64-K stage
    const int grow = n0 + r;
    const bool valid = grow < p.N;
    const uint8_t* srow = p.w_scales + (valid ? static_cast<int64_t>(grow) * p.lds : 0) + blk;
    // scale byte of this thread's block for stages kt, kt+1, kt+2 in flight
    auto scale_at = [&](int kk) -> uint32_t { return (valid && kk < kt1) ? static_cast<uint32_t>(srow[2 * kk]) : 127u; };
    uint32_t c0 = scale_at(kt0), c1 = scale_at(kt0 + 1), c2 = scale_at(kt0 + 2);
    for (int kt = kt0, it = 0; kt < kt1; ++kt, ++it) {
      const int s = it % S;
      const uint32_t ph = (it / S) & 1;
      const uint32_t code = c0;
      c0 = c1;
      c1 = c2;
      c2 = scale_at(kt + 3);
      if (!mbar_wait(&full[s], ph, abort_flag)) break;
      uint8_t* st = smem + s * p.stage_bytes;
      uint32_t w0, w1;
      asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                   : "=r"(w0), "=r"(w1)
                   : "r"(smem_u32(st + x_bytes + kSmWBytes) + r * 32 + part4 * 8));
      const uint32_t bdst = smem_u32(st + x_bytes) + r * 128;
      const uint32_t sw = r & 7;
      const int j0 = part4 * 2;
      if (FP16) {
        const float f = e8m0_to_f32(code);
        st_shared_v4(bdst + (((j0 + 0) ^ sw) << 4), decode8_f16(w0, f));
        st_shared_v4(bdst + (((j0 + 1) ^ sw) << 4), decode8_f16(w1, f));
      } else {
        const uint32_t b = e8m0_to_bf16x2(code);
        st_shared_v4(bdst + (((j0 + 0) ^ sw) << 4), decode8_bf16(w0, b));
        st_shared_v4(bdst + (((j0 + 1) ^ sw) << 4), decode8_bf16(w1, b));
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[s]);
    }
  }

  // ---------------------------------------------------------------- partials
  if (warp >= 4 && warp < 8) {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool any = kt1 > kt0;
    if (any && mbar_wait(tfull, 0, abort_flag)) {
      tc_fence_after();
      for (int cc = 0; cc < p.mp / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + cc * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) part[(cc * 32 + i) * kSmRows + row] = __uint_as_float(v[i]);
      }
    } else {
      for (int c = 0; c < p.mp; ++c) part[c * kSmRows + row] = 0.0f;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_sm();  // every CTA's partial tile is in its shared memory
  tc_fence_after();

  // ---------------------------------------------------------------- reduction
  // CTA c owns rows [c*rows_per, ...) of the 128; a thread sums 4 consecutive
  // rows of one token over all KS partials (16-byte DSMEM reads, rank order).
  {
    const int rows_per = ((kSmRows + p.ks - 1) / p.ks + 3) & ~3;
    const int r_beg = static_cast<int>(rank) * rows_per;
    const int r_end = min(kSmRows, r_beg + rows_per);
    const int quads = r_end > r_beg ? (r_end - r_beg) / 4 : 0;
    const int esz = p.out_dtype == MXFP4_DTYPE_F32 ? 4 : 2;
    const uint32_t part_local = smem_u32(part);
    for (int i = threadIdx.x; i < quads * p.M; i += blockDim.x) {
      const int rr = r_beg + 4 * (i % quads);
      const int tok = i / quads;
      const uint32_t off = static_cast<uint32_t>((tok * kSmRows + rr) * 4);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int c = 0; c < p.ks; ++c) {
        const float4 v = ld_dsmem_v4(mapa_sm(part_local + off, c));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + rr + j;
        if (col >= p.N) continue;
        float v = round_to(a4[j], p.out_dtype);
        if (p.bias != nullptr) v = round_to(v + load_weight(p.bias, p.out_dtype, col), p.out_dtype);
        uint8_t* o = static_cast<uint8_t*>(p.out) + (static_cast<int64_t>(tok) * p.ldo + col) * esz;
        if (p.out_dtype == MXFP4_DTYPE_F32) *reinterpret_cast<float*>(o) = v;
        else if (p.out_dtype == MXFP4_DTYPE_BF16) *reinterpret_cast<__nv_bfloat16*>(o) = __float2bfloat16_rn(v);
        else *reinterpret_cast<__half*>(o) = __float2half_rn(v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_sm();  // peers finished reading this CTA's partials
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, tmem_cols);
}

// ---------------------------------------------------------------------------
// Fused few-token linear with the decoded weights in tensor memory.
//
// Same tiling, K split, MMA sequence and reduction as mxfp4_linear_small_kernel
// (so its results are the safe mode's bits), but the decoded weight tile never
// touches shared memory: decoder warps turn the packed codes they read from
// shared memory into BF16/FP16 pairs in registers and store them with
// tcgen05.st into a ring of tensor-memory slots (one lane per weight row, 32
// columns per 64-K stage), and the MMA reads operand A from there.  Three
// independent rings:
//   packed  [kTmPSlots]  TMA -> decoders; a slot is free once every decoder
//                        warp has read its words (before the MMA), so the
//                        producer runs up to kTmPSlots stages ahead;
//   x       [kTmXSlots]  TMA -> MMA (operand B), freed by the MMA's commit;
//   A       [kTmASlots]  decoders -> MMA in tensor memory, freed by commit.
// With 64-K stages and at most a few tens of stages per CTA, the packed ring
// holds a large part of the CTA's weight bytes in flight at once.
// ---------------------------------------------------------------------------
constexpr int kTmPSlots = 4;   // packed ring: each slot holds a group of 4 stages (one TMA load)
constexpr int kTmPGroup = 4;
constexpr int kTmPGroupBytes = kSmPBytes * kTmPGroup;  // 128 rows x 4 stages x 32 B
constexpr int kTmXSlots = 4;
constexpr int kTmASlots = 16;  // at most; a launch uses every tensor-memory column past the accumulator
constexpr int kTmDecodeWarps = 16;  // 4 warps per TMEM lane quarter, taking consecutive pairs of stages

__host__ __device__ constexpr int tm_small_acc_cols(int mp) {
  return mp <= 32 ? 32 : (mp <= 64 ? 64 : (mp <= 128 ? 128 : 256));
}
__host__ __device__ constexpr uint32_t tm_small_alloc_cols(int) { return 512u; }
__host__ __device__ constexpr int tm_small_a_slots(int mp) {
  return (512 - tm_small_acc_cols(mp)) / 32 < kTmASlots ? (512 - tm_small_acc_cols(mp)) / 32 : kTmASlots;
}

template <bool FP16>
__global__ void __launch_bounds__(256 + 32 * kTmDecodeWarps, 1)
    mxfp4_linear_small_tmem_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                                   const SmallParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int x_bytes = p.mp * 128;
  // [x ring][packed ring]; the partial tile reuses the start after the main loop
  const int x_off = 0;
  const int p_off = kTmXSlots * x_bytes;
  const int data_bytes = p_off + kTmPSlots * kTmPGroupBytes;
  const int part_bytes = kSmRows * p.mp * 4;
  const int bar_off = ((data_bytes > part_bytes ? data_bytes : part_bytes) + 15) & ~15;
  uint64_t* pfull = reinterpret_cast<uint64_t*>(smem + bar_off);
  uint64_t* pempty = pfull + kTmPSlots;
  uint64_t* xfull = pempty + kTmPSlots;
  uint64_t* xempty = xfull + kTmXSlots;
  uint64_t* aready = xempty + kTmXSlots;
  uint64_t* aempty = aready + kTmASlots;
  uint64_t* tfull = aempty + kTmASlots;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* part = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank_sm();
  const int n0 = blockIdx.y * kSmRows;
  const int KT = p.K / kSmBK;
  const int kt0 = static_cast<int>((static_cast<int64_t>(KT) * rank) / p.ks);
  const int kt1 = static_cast<int>((static_cast<int64_t>(KT) * (rank + 1)) / p.ks);
  const int nst = kt1 - kt0;
  const int acc_cols = tm_small_acc_cols(p.mp);
  const uint32_t alloc_cols = tm_small_alloc_cols(p.mp);
  const int AS = tm_small_a_slots(p.mp);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmPSlots; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 2 * kTmPGroup);  // a pair's decoder warp of each lane quarter, 2 pairs per group
    }
    for (int s = 0; s < kTmXSlots; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < kTmASlots; ++s) {
      mbar_init(&aready[s], 4);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, alloc_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_a = tmem_base + acc_cols;  // A slot i at columns [acc_cols + 32 i, +32)

  if (warp == 0) {
    // ---------------------------------------------------------- packed-weight producer
    // one TMA load per group of 4 stages (128 rows x 128 B)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int gi = 0; gi * kTmPGroup < nst; ++gi) {
        const int s = gi % kTmPSlots;
        const uint32_t ph = (gi / kTmPSlots) & 1;
        if (!mbar_wait(&pempty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&pfull[s], kTmPGroupBytes);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | (ph << s);
        tma_load_2d_hint(smem + p_off + s * kTmPGroupBytes, &tmap_w, &pfull[s], (kt0 + gi * kTmPGroup) * (kSmBK / 2),
                         n0, pol_w);
      }
      if (!ok || *abort_flag)
        for (int s = 0; s < kTmPSlots; ++s)
          if (armed & (1u << s)) mbar_drain(&pfull[s], (armed_par >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ---------------------------------------------------------- activation producers
    // warp 2 takes the even stages, warp 3 the odd ones (two issuing threads)
    if (lane == 0) {
      const int par = warp - 2;
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int it = par; it < nst; it += 2) {
        const int s = it % kTmXSlots;
        const uint32_t ph = (it / kTmXSlots) & 1;
        if (!mbar_wait(&xempty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&xfull[s], x_bytes);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | (ph << s);
        tma_load_2d(smem + x_off + s * x_bytes, &tmap_x, &xfull[s], (kt0 + it) * kSmBK, 0);
      }
      if (!ok || *abort_flag)
        for (int s = 0; s < kTmXSlots; ++s)
          if (armed & (1u << s)) mbar_drain(&xfull[s], (armed_par >> s) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(FP16 ? 0 : 1, kSmRows, p.mp);
      bool ok = true, issued = false;
      for (int it = 0; it < nst; ++it) {
        const int sa = it % AS, sx = it % kTmXSlots;
        if (!mbar_wait(&aready[sa], (it / AS) & 1, abort_flag)) { ok = false; break; }
        if (!mbar_wait(&xfull[sx], (it / kTmXSlots) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint64_t bdesc = desc_sw128(smem_u32(smem + x_off + sx * x_bytes));  // x: MMA B (N = mp)
        const uint32_t a_slot = tmem_a + sa * 32;
#pragma unroll
        for (int k = 0; k < kSmBK / 16; ++k) umma_f16_ta(tmem_base, a_slot + 8 * k, bdesc + 2 * k, idesc, (it | k) != 0);
        umma_commit(&aempty[sa]);
        umma_commit(&xempty[sx]);
        issued = true;
      }
      if (ok) umma_commit(tfull);
      else if (issued) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ---------------------------------------------------------- decoders -> tensor memory
    // warp 8 + dw: lane quarter q = dw % 4 (= warp % 4, the quarter it may
    // address) and group g = dw / 4.  Stages go to the quarter's four warps in
    // pairs (pair m = stages 2m, 2m + 1 to the warp with m % 4 == g), each
    // decoding both 64-K stages of its 32 rows into two 32-column A slots, so
    // eight stages are in flight per quarter.
    const int dw = warp - 8;
    const int q = dw & 3, g = dw >> 2;
    const int r = q * 32 + lane;  // weight row of the tile = TMEM lane
    const int grow = n0 + r;
    const bool valid = grow < p.N;
    // rows past N read row 0's scales (their products land in dropped accumulator rows)
    const uint8_t* srow = p.w_scales + (valid ? static_cast<int64_t>(grow) * p.lds : 0);
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // A pair's four scale codes are bytes 2kt .. 2kt+3 of the row: one aligned
    // word when kt is even, else the top half of the word at 2kt-2 and the
    // bottom half of the word at 2kt+2 (the word at 2kt-2 again when the pair
    // has no second stage).  The raw words are loaded one pair ahead and only
    // combined when the pair is decoded, so no instruction waits on the loads
    // before then.  Stages past the CTA's last re-read its last stage's words.
    auto scale_words = [&](int it) -> uint2 {
      const int kt = kt0 + (it < nst ? it : nst - 1);
      if ((kt & 1) == 0) {
        const uint32_t w = ldg_nc_u32(srow + 2 * kt);
        return make_uint2(w, w);
      }
      const uint8_t* hi = it + 1 < nst ? srow + 2 * kt + 2 : srow + 2 * kt - 2;
      return make_uint2(ldg_nc_u32(srow + 2 * kt - 2), ldg_nc_u32(hi));
    };
    auto pair_codes = [&](int it, uint2 w) -> uint32_t {
      return ((kt0 + it) & 1) == 0 ? w.x : __funnelshift_r(w.x, w.y, 16);
    };
    uint2 sc_next = scale_words(2 * g);
    for (int it0 = 2 * g; it0 < nst; it0 += 8) {
      const uint32_t sc_pair = pair_codes(it0, sc_next);
      sc_next = scale_words(it0 + 8);
      int nb = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int it = it0 + h;
        if (it >= nst) break;
        const int gi = it / kTmPGroup;  // packed group (both stages of a pair share it)
        const int sp = gi % kTmPSlots, sa = it % AS;
        const uint32_t sc = sc_pair >> (16 * h);
        // warp-uniform waits: the tcgen05.st / wait::st below are .sync.aligned
        if (h == 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(&pfull[sp], (gi / kTmPSlots) & 1, abort_flag))) { nb = -1; break; }
        // 128-byte rows, 128B-swizzled by the TMA: 16-byte chunk c of row r sits at chunk c ^ (r % 8),
        // so the 32 rows of a warp read from eight different bank groups
        const uint32_t prow = smem_u32(smem + p_off + sp * kTmPGroupBytes) + r * 32 * kTmPGroup;
        const uint32_t c0 = 2u * static_cast<uint32_t>(it % kTmPGroup), sw = static_cast<uint32_t>(r & 7);
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
        if (h == 1 || it + 1 >= nst) {
          asm volatile("" ::"r"(v[0]), "r"(v[31]));
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[sp]);
        }
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&aempty[sa], ((it / AS) & 1) ^ 1, abort_flag))) { nb = -1; break; }
        tc_fence_after();
        tmem_st_32x32b_x32(tmem_a + lane_base + sa * 32, v);
        ++nb;
      }
      if (nb < 0) break;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int h = 0; h < nb; ++h) mbar_arrive(&aready[(it0 + h) % AS]);
    }
  }

  // ---------------------------------------------------------------- partials
  if (warp >= 4 && warp < 8) {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    if (nst > 0 && mbar_wait(tfull, 0, abort_flag)) {
      tc_fence_after();
      for (int cc = 0; cc < p.mp / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + cc * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) part[(cc * 32 + i) * kSmRows + row] = __uint_as_float(v[i]);
      }
    } else {
      for (int c = 0; c < p.mp; ++c) part[c * kSmRows + row] = 0.0f;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_sm();  // every CTA's partial tile is in its shared memory
  tc_fence_after();

  // ---------------------------------------------------------------- reduction (as mxfp4_linear_small_kernel)
  {
    const int rows_per = ((kSmRows + p.ks - 1) / p.ks + 3) & ~3;
    const int r_beg = static_cast<int>(rank) * rows_per;
    const int r_end = min(kSmRows, r_beg + rows_per);
    const int quads = r_end > r_beg ? (r_end - r_beg) / 4 : 0;
    const int esz = p.out_dtype == MXFP4_DTYPE_F32 ? 4 : 2;
    const uint32_t part_local = smem_u32(part);
    for (int i = threadIdx.x; i < quads * p.M; i += blockDim.x) {
      const int rr = r_beg + 4 * (i % quads);
      const int tok = i / quads;
      const uint32_t off = static_cast<uint32_t>((tok * kSmRows + rr) * 4);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int c = 0; c < p.ks; ++c) {
        const float4 v = ld_dsmem_v4(mapa_sm(part_local + off, c));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + rr + j;
        if (col >= p.N) continue;
        float v = round_to(a4[j], p.out_dtype);
        if (p.bias != nullptr) v = round_to(v + load_weight(p.bias, p.out_dtype, col), p.out_dtype);
        uint8_t* o = static_cast<uint8_t*>(p.out) + (static_cast<int64_t>(tok) * p.ldo + col) * esz;
        if (p.out_dtype == MXFP4_DTYPE_F32) *reinterpret_cast<float*>(o) = v;
        else if (p.out_dtype == MXFP4_DTYPE_BF16) *reinterpret_cast<__nv_bfloat16*>(o) = __float2bfloat16_rn(v);
        else *reinterpret_cast<__half*>(o) = __float2half_rn(v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_sm();  // peers finished reading this CTA's partials
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, alloc_cols);
}

}  // namespace mx

namespace mx {

// ---------------------------------------------------------------------------
// One or two tokens: no tensor cores.  One warp owns a weight row: lane
// l takes the 32-value scale blocks l, l+32, ... (each step of the warp reads
// 512 contiguous packed bytes), decodes with the same exact BF16 decoder,
// multiplies by x in FP32 (each
// BF16 x BF16 product is exact in FP32) and the warp sums the lanes with
// shuffles.  Safe mode streams the dequantised BF16 row through the same lane
// and summation order, so fused and safe stay bit-identical.
// ---------------------------------------------------------------------------
constexpr int kGemvMaxRows = 2;  // accumulator slots (the host sends M <= 2 here)

struct GemvParams {
  int M, N, K;
  const void* x;           // [M, K] bf16/fp16, row stride ldx elements
  int64_t ldx;
  const uint8_t* w;        // fused: packed [N, K/2]; safe: dequantised [N, K] (x dtype)
  int64_t ldw;             // bytes per weight row
  const uint8_t* w_scales; // fused only
  int64_t lds;
  void* out;
  int64_t ldo;
  int out_dtype;
  const void* bias;
};

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float f16lo(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFF))); }
__device__ __forceinline__ float f16hi(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16))); }

// acc[m] += sum over 8 K values of x[m][k0..k0+7] * w8 (4 words of 16-bit values)
template <int MR, bool FP16>
__device__ __forceinline__ void gemv_fma8(float (&acc)[kGemvMaxRows], const uint32_t (&w8)[4], const uint8_t* xs,
                                          int kbytes_row, int k0) {
  float wf[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    wf[2 * i] = FP16 ? f16lo(w8[i]) : bf16lo(w8[i]);
    wf[2 * i + 1] = FP16 ? f16hi(w8[i]) : bf16hi(w8[i]);
  }
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * kbytes_row + k0 * 2);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[m] = fmaf(FP16 ? f16lo(xw[i]) : bf16lo(xw[i]), wf[2 * i], acc[m]);
      acc[m] = fmaf(FP16 ? f16hi(xw[i]) : bf16hi(xw[i]), wf[2 * i + 1], acc[m]);
    }
  }
}

template <int MR, int BMODE, bool FP16>
__global__ void __launch_bounds__(256) mxfp4_gemv_kernel(const GemvParams p) {
  extern __shared__ uint8_t xs[];  // x rows [MR][K] (16-bit)
  const int kbytes_row = p.K * 2;
  // stage x in shared memory (all warps of the CTA reuse it)
  for (int i = threadIdx.x; i < MR * (kbytes_row / 16); i += blockDim.x) {
    const int m = i / (kbytes_row / 16), v = i % (kbytes_row / 16);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (m < p.M) val = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) + m * p.ldx * 2)[v];
    reinterpret_cast<uint4*>(xs + m * kbytes_row)[v] = val;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int nblk = p.K / 32;  // 32-value scale blocks per row; lane l takes blocks l, l+32, ...
  for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < p.N; n += warps) {
    float acc[kGemvMaxRows];
#pragma unroll
    for (int m = 0; m < kGemvMaxRows; ++m) acc[m] = 0.0f;
    if (BMODE == B_DECODE) {
      const uint8_t* wrow = p.w + static_cast<int64_t>(n) * p.ldw;
      const uint8_t* srow = p.w_scales + static_cast<int64_t>(n) * p.lds;
      for (int b = lane; b < nblk; b += 32) {
        const uint32_t code = srow[b];
        const uint4 q = *reinterpret_cast<const uint4*>(wrow + b * 16);  // 32 codes, 16-byte aligned
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 d;
          if (FP16) d = decode8_f16(qw[j], e8m0_to_f32(code));
          else d = decode8_bf16(qw[j], e8m0_to_bf16x2(code));
          const uint32_t w8[4] = {d.x, d.y, d.z, d.w};
          gemv_fma8<MR, FP16>(acc, w8, xs, kbytes_row, b * 32 + 8 * j);
        }
      }
    } else {
      const uint8_t* wrow = p.w + static_cast<int64_t>(n) * p.ldw;
      for (int b = lane; b < nblk; b += 32) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 d = *reinterpret_cast<const uint4*>(wrow + b * 64 + j * 16);
          const uint32_t w8[4] = {d.x, d.y, d.z, d.w};
          gemv_fma8<MR, FP16>(acc, w8, xs, kbytes_row, b * 32 + 8 * j);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      acc[m] = v;
    }
    if (lane < MR && lane < p.M) {
      float v = 0.0f;
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m == lane) v = acc[m];
      v = round_to(v, p.out_dtype);
      if (p.bias != nullptr) v = round_to(v + load_weight(p.bias, p.out_dtype, n), p.out_dtype);
      uint8_t* o = static_cast<uint8_t*>(p.out) + (static_cast<int64_t>(lane) * p.ldo + n) * 2;
      if (p.out_dtype == MXFP4_DTYPE_BF16) *reinterpret_cast<__nv_bfloat16*>(o) = __float2bfloat16_rn(v);
      else *reinterpret_cast<__half*>(o) = __float2half_rn(v);
    }
  }
}

}  // namespace mx
