// Host side of libmxfp4_b200.so: argument validation, tensor-map encoding,
// workspace layout and kernel launches behind the C ABI in include/mxfp4_b200.h.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "elementwise.cuh"
#include "ep.cuh"
#include "gemm.cuh"
#include "gemm2.cuh"
#include "gemm_routed.cuh"
#include "gemm_small.cuh"
#include "gemm_w4a4.cuh"
#include "gemm_mx8.cuh"
#include "gemv_routed.cuh"

using namespace mx;

namespace {

thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

#define MX_CUDA(call)                                                                      \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return fail(MXFP4_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
  } while (0)

#define MX_CHECK(cond, msg)                                                                \
  do {                                                                                     \
    if (!(cond)) return fail(MXFP4_ERR_INVALID_ARGUMENT, msg);                             \
  } while (0)

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// --- device properties -----------------------------------------------------
struct DevInfo {
  int sms = 0;
  int major = 0, minor = 0;
  bool ok = false;
};

int current_device_info(DevInfo& info) {
  static std::mutex mu;
  static DevInfo cache[64];
  int dev = 0;
  MX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MXFP4_ERR_UNSUPPORTED_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev].ok) {
    cudaDeviceProp prop;
    MX_CUDA(cudaGetDeviceProperties(&prop, dev));
    cache[dev].sms = prop.multiProcessorCount;
    cache[dev].major = prop.major;
    cache[dev].minor = prop.minor;
    cache[dev].ok = true;
  }
  info = cache[dev];
  if (info.major != 10)
    return fail(MXFP4_ERR_UNSUPPORTED_DEVICE,
                "libmxfp4_b200 needs an sm_100 (B200) device, found sm_" +
                    std::to_string(info.major) + std::to_string(info.minor));
  return MXFP4_OK;
}

// --- tensor maps -----------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encoder(EncodeTiledFn& fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) cached = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (cached == nullptr)
    return fail(MXFP4_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  fn = cached;
  return MXFP4_OK;
}

// 2-D row-major tensor [rows, cols] of `esize`-byte elements, row pitch in bytes.
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize,
                uint64_t cols, uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols,
                uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc;
  if (int rc = get_encoder(enc)) return rc;
  if (!aligned(base, 16)) return fail(MXFP4_ERR_INVALID_ARGUMENT, "TMA operand must be 16-byte aligned");
  if (pitch_bytes % 16 != 0)
    return fail(MXFP4_ERR_INVALID_ARGUMENT, "TMA operand row pitch must be a multiple of 16 bytes");
  (void)esize;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MXFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return MXFP4_OK;
}

// Tiled tensor map of any rank (2..5): dims[0] innermost, strides in bytes
// for dims 1..rank-1 (any order).
int make_map_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc;
  if (int rc = get_encoder(enc)) return rc;
  if (!aligned(base, 16)) return fail(MXFP4_ERR_INVALID_ARGUMENT, "TMA operand must be 16-byte aligned");
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5];
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    if (i > 0) {
      if (strides[i - 1] % 16 != 0) return fail(MXFP4_ERR_INVALID_ARGUMENT, "TMA stride must be a multiple of 16 bytes");
      st[i - 1] = strides[i - 1];
    }
  }
  CUresult r = enc(map, dtype, rank, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MXFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return MXFP4_OK;
}

int elem_size(int dtype) {
  switch (dtype) {
    case MXFP4_DTYPE_F32: return 4;
    case MXFP4_DTYPE_BF16: return 2;
    case MXFP4_DTYPE_F16: return 2;
    case MXFP4_DTYPE_U8: return 1;
    case MXFP4_DTYPE_I32: return 4;
    case MXFP4_DTYPE_I64: return 8;
  }
  return 0;
}

struct PeerOut {
  int n = 0;
  void* p[kMaxPeers] = {};
  void* mc = nullptr;  // multicast mapping of all ranks' outputs (16-byte stores), or null
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int64_t kSmallMaxRows = 256;  // token counts served by the split-K few-token kernel
constexpr int64_t kGemvRows = 2;        // token counts served by the CUDA-core GEMV (measured crossover)

// --- GEMM launch ------------------------------------------------------------
int run_gather(const void* x, int64_t k_elems, const int32_t* sorted_ids, const int32_t* post, int64_t routes,
               int top_k, void* xr, int64_t cap, int sms, cudaStream_t stream) {
  const int64_t row_vecs = k_elems * 2 / 16;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((cap + 7) / 8, int64_t(sms) * 16)));
  gather_rows_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(x), row_vecs, sorted_ids, post,
                                               static_cast<int>(routes), top_k, static_cast<uint4*>(xr), cap);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

template <int AMODE, int BMODE, int EPI, bool FP16, int DW, bool PEERS = false>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const PairParams& p, int clusters,
                cudaStream_t stream, bool after_decode = false) {
  using Cfg = Pair2Cfg<BMODE, DW, PEERS>;
  auto kern = mxfp4_gemm_pair_kernel<AMODE, BMODE, EPI, FP16, DW, PEERS>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  });
  MX_CUDA(attr_err);
  if (!after_decode) {
    kern<<<2 * clusters, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p);
  } else {
    // programmatic dependent launch behind the weight decode: the GEMM's
    // set-up (barriers, tensor memory, cluster sync) overlaps the decode's
    // tail; the kernel waits for the decode's output before reading it
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MX_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
  }
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// Fused-decode GEMM on CTA pairs (dense, or routed over 256-route blocks).
template <int EPI>
int fused_pair_gemm(bool fp16, const CUtensorMap& ta, const CUtensorMap& tb, const PairParams& p, int clusters,
                    cudaStream_t stream) {
  if (fp16) return launch_pair<A_TMA, B_DECODE, EPI, true, 8>(ta, tb, p, clusters, stream);
  return launch_pair<A_TMA, B_DECODE, EPI, false, 8>(ta, tb, p, clusters, stream);
}

// Routed GEMM on CTA pairs over 256-route blocks (fused decode).
template <int AMODE, int EPI>
int routed_pair_gemm(bool fp16, const CUtensorMap& ta, const CUtensorMap& tb, const PairParams& p, int sms,
                     cudaStream_t stream) {
  static_assert(AMODE == A_TMA, "routed activations are copied to routed order and loaded by TMA");
  const int64_t tiles = static_cast<int64_t>(p.num_m_blocks) * p.num_n_blocks;
  const int clusters = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms / 2)));
  return fused_pair_gemm<EPI>(fp16, ta, tb, p, clusters, stream);
}

// Few-token linear (M <= 256): swap-AB, K split over a cluster of `ks` CTAs.
template <int BMODE, bool FP16>
int launch_small(const CUtensorMap& tx, const CUtensorMap& tw, const SmallParams& p, cudaStream_t stream) {
  auto kern = mxfp4_linear_small_kernel<BMODE, FP16>;
  const int data = p.stages * p.stage_bytes;
  const int part = kSmRows * p.mp * 4;
  const int smem = ((data > part ? data : part) + 15) / 16 * 16 + 3 * kSmMaxStages * 8 + 64 + 1024;
  MX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.ks, (p.N + kSmRows - 1) / kSmRows, 1);
  cfg.blockDim = dim3(BMODE == B_DECODE ? 256 + 32 * kSmDecodeWarps : 256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MX_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tw, p));
  return MXFP4_OK;
}

// Fused few-token linear with the decoded weights in tensor memory (the same
// K split, MMA order and reduction as launch_small's kernel).
template <bool FP16>
int launch_small_tmem(const CUtensorMap& tx, const CUtensorMap& tw, const SmallParams& p, cudaStream_t stream) {
  auto kern = mxfp4_linear_small_tmem_kernel<FP16>;
  const int data = kTmXSlots * p.mp * 128 + kTmPSlots * kTmPGroupBytes;
  const int part = kSmRows * p.mp * 4;
  const int bars = (2 * kTmPSlots + 2 * kTmXSlots + 2 * kTmASlots + 2) * 8;
  const int smem = ((data > part ? data : part) + 15) / 16 * 16 + bars + 64 + 1024;
  MX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.ks, (p.N + kSmRows - 1) / kSmRows, 1);
  cfg.blockDim = dim3(256 + 32 * kTmDecodeWarps, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MX_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tw, p));
  return MXFP4_OK;
}

template <int BMODE, bool FP16>
int launch_gemv(const GemvParams& g, int sms, cudaStream_t stream) {
  const int mr = g.M <= 1 ? 1 : 2;
  const size_t smem = static_cast<size_t>(mr) * g.K * 2;
  const int grid = static_cast<int>(std::min<int64_t>((g.N + 7) / 8, int64_t(sms) * 4));
  auto go = [&](auto kern) -> int {
    MX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    kern<<<grid, 256, smem, stream>>>(g);
    MX_CUDA(cudaGetLastError());
    return MXFP4_OK;
  };
  if (mr == 1) return go(mxfp4_gemv_kernel<1, BMODE, FP16>);
  return go(mxfp4_gemv_kernel<2, BMODE, FP16>);
}

// The kernels take one E8M0 scale per 32 K in row-major [rows, K/32] and read the
// scales as 32-bit words of four (128 K, two 64-code stages): K must be a positive
// multiple of 128.
int check_scales_layout(int64_t k) {
  if (k <= 0 || k % 128 != 0)
    return fail(MXFP4_ERR_INVALID_ARGUMENT, "logical K must be a positive multiple of 128, got " + std::to_string(k));
  return MXFP4_OK;
}

// --- routing ----------------------------------------------------------------
struct RouteWs {
  int32_t* rank;
  int32_t* hist;
  int32_t* blk_off;
};

size_t route_ws_bytes(int64_t num_routes, int num_experts) {
  const int64_t chunks = (num_routes + kRouteThreads - 1) / kRouteThreads;
  return align_up(sizeof(int32_t) * std::max<int64_t>(num_routes, 1), 256) +
         align_up(sizeof(int32_t) * std::max<int64_t>(chunks, 1) * num_experts, 256) +
         align_up(sizeof(int32_t) * num_experts, 256);
}

RouteWs carve_route_ws(uint8_t* ws, int64_t num_routes, int num_experts) {
  const int64_t chunks = (num_routes + kRouteThreads - 1) / kRouteThreads;
  RouteWs r;
  r.rank = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * std::max<int64_t>(num_routes, 1), 256);
  r.hist = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * std::max<int64_t>(chunks, 1) * num_experts, 256);
  r.blk_off = reinterpret_cast<int32_t*>(ws);
  return r;
}

// Rows of the padded routed layout, for any distribution of the routes: each
// expert that receives a route pads its last block by at most block_m - 1
// rows, and at most min(num_experts, num_routes) experts receive one.
int64_t route_capacity(int64_t num_routes, int num_experts, int block_m) {
  const int64_t used = std::min<int64_t>(num_experts, num_routes);
  const int64_t padded = num_routes + used * (block_m - 1);
  return (padded + block_m - 1) / block_m * block_m;
}

int run_route(const void* ids, int ids_dtype, int64_t num_routes, int num_experts,
              int expert_offset, int block_m, int32_t* sorted_ids, int32_t* block_expert,
              int32_t* post, int64_t capacity, uint8_t* ws, cudaStream_t stream,
              int4* rt_chunks = nullptr, int32_t* rt_num_chunks = nullptr, int chunk_blocks = kRtChunkBlocks) {
  RouteWs r = carve_route_ws(ws, num_routes, num_experts);
  if (num_routes <= kRouteSmallMax && num_experts <= kRouteSmallExperts) {
    // decode-sized calls: the whole routing in one CTA (one launch instead of three)
    const size_t smem_small = sizeof(int32_t) * 32 * num_experts;
    route_small_kernel<<<1, 1024, smem_small, stream>>>(ids, ids_dtype, num_routes, num_experts, expert_offset,
                                                        block_m, r.blk_off, sorted_ids, block_expert, post,
                                                        capacity / block_m, rt_chunks, rt_num_chunks, chunk_blocks);
    MX_CUDA(cudaGetLastError());
    return MXFP4_OK;
  }
  const int64_t chunks = std::max<int64_t>((num_routes + kRouteThreads - 1) / kRouteThreads, 1);
  const size_t smem = sizeof(int32_t) * kRouteWarps * num_experts;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(route_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    sizeof(int32_t) * kRouteWarps * kMaxExperts);
  });
  MX_CUDA(attr_err);
  if (num_routes > 0)
    route_count_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, smem, stream>>>(
        ids, ids_dtype, num_routes, num_experts, expert_offset, r.rank, r.hist);
  else
    MX_CUDA(cudaMemsetAsync(r.hist, 0, sizeof(int32_t) * num_experts, stream));
  MX_CUDA(cudaGetLastError());
  route_offsets_kernel<<<1, 1024, 0, stream>>>(r.hist, static_cast<int>(chunks), num_experts, block_m,
                                               num_routes, r.blk_off, sorted_ids, block_expert, post,
                                               capacity / block_m, rt_chunks, rt_num_chunks, chunk_blocks);
  MX_CUDA(cudaGetLastError());
  if (num_routes > 0)
    route_scatter_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, 0, stream>>>(
        ids, ids_dtype, num_routes, num_experts, expert_offset, block_m, r.rank, r.hist, r.blk_off,
        sorted_ids);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// --- routing of the routed GEMMs (32-route blocks, chunks of <= chunk_rows routes) ---
int64_t rt_max_chunks(int64_t routes, int num_experts, int chunk_rows) {
  const int64_t cap = route_capacity(routes, num_experts, kRtBlock);
  return cap / chunk_rows + std::min<int64_t>(num_experts, routes) + 1;
}

struct RtRouting {
  int64_t cap;         // padded routed rows
  int64_t max_chunks;
  int32_t* sorted;     // [cap]
  int32_t* block_expert;
  int32_t* post;
  int4* chunks;        // [max_chunks]
  int32_t* num_chunks;
  uint8_t* route_ws;
  int chunk_blocks;
};

size_t rt_routing_bytes(int64_t routes, int num_experts, int chunk_rows = kRtBlock * kRtChunkBlocks) {
  const int64_t cap = route_capacity(routes, num_experts, kRtBlock);
  return align_up(sizeof(int32_t) * std::max<int64_t>(cap, 1), 256) + align_up(sizeof(int32_t) * (cap / kRtBlock + 1), 256) +
         256 + align_up(sizeof(int4) * rt_max_chunks(routes, num_experts, chunk_rows), 256) + 256 +
         route_ws_bytes(routes, num_experts);
}

RtRouting carve_rt_routing(uint8_t*& ws, int64_t routes, int num_experts, int chunk_rows = kRtBlock * kRtChunkBlocks) {
  RtRouting r;
  r.cap = route_capacity(routes, num_experts, kRtBlock);
  r.max_chunks = rt_max_chunks(routes, num_experts, chunk_rows);
  r.chunk_blocks = chunk_rows / kRtBlock;
  r.sorted = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * std::max<int64_t>(r.cap, 1), 256);
  r.block_expert = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * (r.cap / kRtBlock + 1), 256);
  r.post = reinterpret_cast<int32_t*>(ws);
  ws += 256;
  r.chunks = reinterpret_cast<int4*>(ws);
  ws += align_up(sizeof(int4) * r.max_chunks, 256);
  r.num_chunks = reinterpret_cast<int32_t*>(ws);
  ws += 256;
  r.route_ws = ws;
  ws += route_ws_bytes(routes, num_experts);
  return r;
}

int run_rt_routing(const void* ids, int ids_dtype, int64_t routes, int num_experts, const RtRouting& r,
                   cudaStream_t s) {
  return run_route(ids, ids_dtype, routes, num_experts, 0, kRtBlock, r.sorted, r.block_expert, r.post, r.cap,
                   r.route_ws, s, r.chunks, r.num_chunks, r.chunk_blocks);
}

template <int EPI, bool FP16>
int launch_routed(const CUtensorMap& tw, const CUtensorMap& tx16, const CUtensorMap& tx128, const RoutedParams& p,
                  int sms, cudaStream_t stream) {
  auto kern = mxfp4_routed_tmem_kernel<EPI, FP16>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmemBytes);
  });
  MX_CUDA(attr_err);
  const int64_t tiles = static_cast<int64_t>(p.max_chunks) * p.num_wblocks;
  const int clusters = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms / 2)));
  kern<<<2 * clusters, kRtThreads, kRtSmemBytes, stream>>>(tw, tx16, tx128, p);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// Routed GEMV over (route, block of kMoeGemvWarps outputs).
template <int EPI, bool FP16>
int launch_moe_gemv(const MoeGemvParams& p, cudaStream_t stream) {
  MX_CHECK(aligned(p.x, 16) && (p.ldx * 2) % 16 == 0 && aligned(p.w, 16) && p.ldw % 16 == 0,
           "routed GEMV operands must be 16-byte aligned");
  if (p.num_routes == 0) return MXFP4_OK;
  auto kern = mxfp4_moe_gemv_kernel<EPI, FP16>;
  const int smem = p.K * 2;
  if (smem > 48 * 1024) MX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const dim3 grid(p.num_routes, (p.rows + kMoeGemvWarps - 1) / kMoeGemvWarps, 1);
  kern<<<grid, 32 * kMoeGemvWarps, smem, stream>>>(p);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// Stages per packed-weight TMA load of a routed GEMM: 4 when they divide the
// weights' 64-K stage count, else 2 (K is a multiple of 128).
int routed_pgroup(int64_t kw) { return (kw / kP2BK) % 4 == 0 ? 4 : 2; }

// The three tensor maps of a routed GEMM: packed weights [rows_total, kw/2]
// (boxes of pgroup stages x 128 rows, GLU: x 64 rows) and the routed
// activations [cap, ka] in 16-row and 128-row boxes.
int routed_maps(CUtensorMap* tw, CUtensorMap* tx16, CUtensorMap* tx128, const void* w, int64_t rows_total, int64_t kw,
                const void* xr, int64_t cap, int64_t ka, bool fp16, bool glu) {
  const CUtensorMapDataType xt = fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t box_bytes = static_cast<uint32_t>(routed_pgroup(kw) * (kP2BK / 2));
  if (int rc = make_map_2d(tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, kw / 2, rows_total, kw / 2, box_bytes,
                           glu ? 64 : 128, box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
    return rc;
  const uint64_t rows = static_cast<uint64_t>(std::max<int64_t>(cap, 1));
  if (int rc = make_map_2d(tx16, xr, xt, 2, ka, rows, ka * 2, kP2BK, 16, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  return make_map_2d(tx128, xr, xt, 2, ka, rows, ka * 2, kP2BK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

// --- routed GEMMs on the block-scaled tensor cores (gemm_mx8.cuh) -----------
// Route chunk of the mx8 kernel: 32 routes (7-stage ring) while the average
// expert receives fewer than kMx8WideRoutesPerExpert routes, else 128
// (3-stage ring; each weight tile serves up to 128 routes).
constexpr int64_t kMx8WideRoutesPerExpert = 48;
int mx8_bn(int64_t routes, int num_experts) {
  return routes >= kMx8WideRoutesPerExpert * static_cast<int64_t>(num_experts) ? 128 : 32;
}
// The weights reach shared memory by TMA of the 16U4_ALIGN16B type (32-byte
// aligned base) and their scale words by 4-byte cp.async.
bool mx8_weights_ok(const void* w, const void* w_scales) { return aligned(w, 32) && aligned(w_scales, 4); }

struct Mx8Act {
  uint8_t* xh;   // [rows, k] E4M3, routed order
  uint8_t* xl;
  uint8_t* sfh;  // [chunk][k/128][512] E8M0
  uint8_t* sfl;
};
// Bytes of the split activations: hi and lo rows, and the scale chunks --
// one array for 32-route chunks (lo's scales in the hi chunk's second column,
// sfl = sfh + 4), a hi and a lo array for 128-route chunks.
size_t mx8_act_bytes(int64_t rows, int64_t k, int64_t max_chunks, int bn) {
  rows = std::max<int64_t>(rows, 1);
  const size_t sb = align_up(static_cast<size_t>(std::max<int64_t>(max_chunks, 1)) * (k / 128) * 512, 256);
  return 2 * align_up(static_cast<size_t>(rows) * k, 256) + (bn == 32 ? 1 : 2) * sb;
}
Mx8Act carve_mx8_act(uint8_t*& ws, int64_t rows, int64_t k, int64_t max_chunks, int bn) {
  rows = std::max<int64_t>(rows, 1);
  Mx8Act a;
  const size_t xb = align_up(static_cast<size_t>(rows) * k, 256);
  const size_t sb = align_up(static_cast<size_t>(std::max<int64_t>(max_chunks, 1)) * (k / 128) * 512, 256);
  a.xh = ws;
  a.xl = ws + xb;
  a.sfh = ws + 2 * xb;
  a.sfl = bn == 32 ? a.sfh + 4 : ws + 2 * xb + sb;
  ws += 2 * xb + (bn == 32 ? 1 : 2) * sb;
  return a;
}

// Split BF16 rows into the mx8 operand, chunk by chunk of the routing's chunk
// table: gathered in routed order when `sorted` is given, else rows already
// in routed order; padding rows are skipped either way.
int run_mx8_split(const void* x, int64_t ldx, int64_t k, const RtRouting& rt, const int32_t* sorted, int64_t routes,
                  int top_k, const Mx8Act& a, int sms, cudaStream_t s) {
  if (rt.max_chunks <= 0) return MXFP4_OK;
  // a CTA per chunk (up to max_chunks; those past the routing's count exit)
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(rt.max_chunks, int64_t(sms) * 2)));
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  const int mc = static_cast<int>(rt.max_chunks);
  if (sorted)
    mx8_split_kernel<true><<<grid, kMx8SplitThreads, 0, s>>>(xs, ldx, static_cast<int>(k), rt.chunks, rt.num_chunks,
                                                             mc, sorted, static_cast<int>(routes), top_k, a.xh, a.xl,
                                                             a.sfh, a.sfl);
  else
    mx8_split_kernel<false><<<grid, kMx8SplitThreads, 0, s>>>(xs, ldx, static_cast<int>(k), rt.chunks, rt.num_chunks,
                                                              mc, rt.sorted, static_cast<int>(routes), 1, a.xh, a.xl,
                                                              a.sfh, a.sfl);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// Tensor maps of an mx8 GEMM (layouts at mxfp4_routed_mx8_kernel): the packed
// weights (every expert's rows) as 4-bit elements expanded to the MMA's
// 16-byte slots, groups of `group` 128-K stages per copy; hi and lo route
// tiles of 32 rows.
int mx8_maps(CUtensorMap* tw, CUtensorMap* txh, CUtensorMap* txl, const void* w, int64_t rows_total, int64_t k,
             const Mx8Act& a, int64_t rows, int64_t glu_inter, int group, int bn) {
  MX_CHECK(aligned(w, 32) && (k / 2) % 32 == 0, "mx8 weights must be 32-byte aligned with a 32-byte row pitch");
  const uint64_t kt = static_cast<uint64_t>(k / 128);
  const uint32_t g = static_cast<uint32_t>(group);
  if (glu_inter > 0) {
    const uint64_t dims[4] = {128, static_cast<uint64_t>(rows_total), 2, kt};
    const uint64_t strides[3] = {static_cast<uint64_t>(k / 2), static_cast<uint64_t>(glu_inter * (k / 2)), 64};
    const uint32_t box[4] = {128, 64, 2, g};
    if (int rc = make_map_nd(tw, w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 4, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    const uint64_t dims[3] = {128, static_cast<uint64_t>(rows_total), kt};
    const uint64_t strides[2] = {static_cast<uint64_t>(k / 2), 64};
    const uint32_t box[3] = {128, 128, g};
    if (int rc = make_map_nd(tw, w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  if (bn == 32) {
    // hi and lo as one tensor: the part dimension steps from xh to xl
    const uint64_t xdims[4] = {128, static_cast<uint64_t>(std::max<int64_t>(rows, 1)), 2, kt};
    const uint64_t xstrides[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(a.xl - a.xh), 128};
    const uint32_t xbox[4] = {128, 32, 2, g};
    *txl = {};
    return make_map_nd(txh, a.xh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, xdims, xstrides, xbox, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint64_t xdims[3] = {128, static_cast<uint64_t>(std::max<int64_t>(rows, 1)), kt};
  const uint64_t xstrides[2] = {static_cast<uint64_t>(k), 128};
  const uint32_t xbox[3] = {128, 32, g};
  if (int rc = make_map_nd(txh, a.xh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, xdims, xstrides, xbox, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  return make_map_nd(txl, a.xl, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, xdims, xstrides, xbox, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Stages per copy group: 4, 2 or 1, dividing K / 128 (32-route tiles; the
// 128-route kernel's 3 slots take one stage per copy).
int mx8_group(int bn, int64_t k) {
  if (bn == 128) return 1;
  const int64_t kt = k / 128;
  return kt % 4 == 0 ? 4 : (kt % 2 == 0 ? 2 : 1);
}

template <int EPI, int BN>
int launch_mx8_bn(const CUtensorMap& tw, const CUtensorMap& txh, const CUtensorMap& txl, const Mx8Params& p, int sms,
                  cudaStream_t stream) {
  auto kern = mxfp4_routed_mx8_kernel<EPI, BN>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Mx8Cfg<BN>::kSmemBytes);
  });
  MX_CUDA(attr_err);
  const int64_t tiles = static_cast<int64_t>(p.max_chunks) * p.num_wblocks;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms)));
  kern<<<grid, Mx8Cfg<BN>::kThreads, Mx8Cfg<BN>::kSmemBytes, stream>>>(tw, txh, txl, p);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}
template <int EPI>
int launch_mx8(int bn, const CUtensorMap& tw, const CUtensorMap& txh, const CUtensorMap& txl, const Mx8Params& p,
               int sms, cudaStream_t stream) {
  if (bn == 128) return launch_mx8_bn<EPI, 128>(tw, txh, txl, p, sms, stream);
  return launch_mx8_bn<EPI, 32>(tw, txh, txl, p, sms, stream);
}

}  // namespace

// ---------------------------------------------------------------------------
// Static scratch for mxfp4_fused_moe_noalloc.  Some callers cannot allocate
// device memory when they call into this library (a plugin host or graph
// executor that owns every buffer after initialisation, a fixed memory plan
// replayed under stream capture), so that entry point takes its routing
// scratch from this array instead of a caller workspace.  Every GPU that loads
// the library holds these bytes until the process exits.  In host code the
// array's name is only a host-side stand-in: its device address comes from
// cudaGetSymbolAddress, looked up once per device.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_noalloc_scratch for the current device; the first call
// on a device does the lookup (so it must not happen inside a stream capture).
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  MX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MXFP4_ERR_UNSUPPORTED_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MXFP4_ERR_CUDA, std::string("cudaGetSymbolAddress(g_noalloc_scratch): ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return MXFP4_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int mxfp4_abi_version(void) { return MXFP4_B200_ABI_VERSION; }

const char* mxfp4_last_error(void) { return t_last_error.c_str(); }

int mxfp4_device_supported(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return prop.major == 10 ? 1 : 0;
}

int mxfp4_device_status(int device, int clear) {
  int prev = 0;
  MX_CUDA(cudaGetDevice(&prev));
  MX_CUDA(cudaSetDevice(device));
  MX_CUDA(cudaDeviceSynchronize());
  int word = 0;
  MX_CUDA(cudaMemcpyFromSymbol(&word, g_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    MX_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)));
  }
  MX_CUDA(cudaSetDevice(prev));
  return word;
}

int mxfp4_dequant(const void* packed, const void* scales, void* out, int out_dtype, int64_t rows,
                  int64_t k, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(packed && scales && out, "null pointer");
  MX_CHECK(rows >= 0 && k >= 0 && k % 32 == 0, "logical K must be divisible by 32");
  MX_CHECK(out_dtype == MXFP4_DTYPE_F32 || out_dtype == MXFP4_DTYPE_BF16 || out_dtype == MXFP4_DTYPE_F16,
           "dequant output dtype must be F32, BF16 or F16");
  MX_CHECK(aligned(packed, 16) && aligned(out, 16), "packed and out must be 16-byte aligned");
  const int64_t nb = rows * (k / 32);
  if (nb == 0) return MXFP4_OK;
  const int grid = static_cast<int>(std::min<int64_t>((nb + 255) / 256, int64_t(info.sms) * 8));
  cudaStream_t s = as_stream(stream);
  if (out_dtype == MXFP4_DTYPE_BF16)
    dequant_kernel<MXFP4_DTYPE_BF16><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                          static_cast<const uint8_t*>(scales), out, nb);
  else if (out_dtype == MXFP4_DTYPE_F16)
    dequant_kernel<MXFP4_DTYPE_F16><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                         static_cast<const uint8_t*>(scales), out, nb);
  else
    dequant_kernel<MXFP4_DTYPE_F32><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(packed),
                                                         static_cast<const uint8_t*>(scales), out, nb);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

// Fused mode decodes inside the GEMM producer, once per 256-row block of x.
// From this many row blocks on, decoding each weight element once (the decode
// kernel into an L2-resident BF16 copy, then the TMA-fed pair GEMM) costs less
// time than re-decoding it per row block.  Measured on B200 at the config-1
// qkv shape with the weights cold in HBM (32 rotating weight sets, as a layer
// of a served model sees them): M = 1024 / 1280 (4 / 5 row blocks) 37.5 /
// 37.7 us decode-once against 43.0 / 44.9 us in the GEMM; at 2-3 row blocks the
// in-GEMM decode is ~4% faster.
constexpr int64_t kDecodeOnceRowBlocks = 4;

size_t mxfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int x_dtype, int mode) {
  (void)x_dtype;
  const bool decode_once = mode == MXFP4_LINEAR_FUSED && (m + kP2BM - 1) / kP2BM >= kDecodeOnceRowBlocks;
  if (mode != MXFP4_LINEAR_SAFE && !decode_once) return 0;
  return align_up(static_cast<size_t>(n) * k * 2, 256);
}

}  // extern "C"

namespace {

// Copy the [m, n] block at `out` (row stride ldo) into every peer buffer at the
// same offset: the all-gather of the few-token paths, whose kernels have no
// peer-store epilogue.
__global__ void __launch_bounds__(256) push_rows_kernel(const uint8_t* __restrict__ src, int64_t m,
                                                        int64_t row_bytes, int64_t ld_bytes, PeerOut peers) {
  const bool vec = (row_bytes % 16 == 0) && (ld_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0);
  const int64_t units = vec ? row_bytes / 16 : row_bytes / 2;
  const int64_t total = m * units;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / units, u = i % units;
    const int64_t off = r * ld_bytes + u * (vec ? 16 : 2);
    if (vec) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + off);
      if (peers.mc != nullptr) {
        multimem_st_v4(static_cast<uint8_t*>(peers.mc) + off, v);
      } else {
#pragma unroll
        for (int j = 0; j < kMaxPeers; ++j)
          if (j < peers.n) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(peers.p[j]) + off) = v;
      }
    } else {
      const uint16_t v = *reinterpret_cast<const uint16_t*>(src + off);
#pragma unroll
      for (int j = 0; j < kMaxPeers; ++j)
        if (j < peers.n) *reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(peers.p[j]) + off) = v;
    }
  }
}

// The dense linear.  `w_deq` (optional) holds the weights already decoded to
// x's dtype ([n, k], row pitch ldwd elements): the second launch of the safe
// and decode-once paths, callable on its own (mxfp4_linear_dequantized); then
// w_packed / w_scales are unused.
int linear_impl(const void* x, int x_dtype, int64_t ldx, const void* w_packed, int64_t ldw, const void* w_scales,
                int64_t lds, const void* bias, void* out, int64_t ldo, int64_t m, int64_t n, int64_t k, int mode,
                void* workspace, size_t workspace_bytes, void* stream, const PeerOut& peers,
                const void* w_deq = nullptr, int64_t ldwd = 0) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(x && out && (w_deq || (w_packed && w_scales)), "null pointer");
  MX_CHECK(x_dtype == MXFP4_DTYPE_BF16 || x_dtype == MXFP4_DTYPE_F16, "x must be BF16 or F16");
  MX_CHECK(mode == MXFP4_LINEAR_FUSED || mode == MXFP4_LINEAR_SAFE, "unknown linear mode");
  if (int rc = check_scales_layout(k)) return rc;
  MX_CHECK(m >= 0 && n > 0, "bad M/N");
  MX_CHECK(m < (int64_t(1) << 31) && n < (int64_t(1) << 31) && k < (int64_t(1) << 30), "dimension too large");
  MX_CHECK(ldx >= k && ldo >= n, "leading dimension too small");
  if (w_deq) {
    MX_CHECK(ldwd >= k && aligned(w_deq, 16) && (ldwd * 2) % 16 == 0,
             "dequantized weights need a 16-byte aligned base and row pitch >= k");
  } else {
    MX_CHECK(ldw >= k / 2 && lds >= k / 32, "leading dimension too small");
    MX_CHECK(aligned(w_scales, 4) && lds % 4 == 0, "scales must be 4-byte aligned rows");
  }
  if (m == 0) return MXFP4_OK;
  cudaStream_t s = as_stream(stream);
  auto push = [&](int rc) -> int {
    if (rc != MXFP4_OK || peers.n == 0 || m == 0) return rc;
    const int64_t esz = 2;
    const int64_t total = m * n;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 2047) / 2048, info.sms * 4)));
    push_rows_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(out), m, n * esz, ldo * esz, peers);
    MX_CUDA(cudaGetLastError());
    return MXFP4_OK;
  };
  // the explicit dequant of the safe path (soft:371-373) into the workspace;
  // afterwards `wd` / `ldwd` describe the decoded weights
  const void* wd = w_deq;
  auto dequant_into_workspace = [&]() -> int {
    const size_t need = align_up(static_cast<size_t>(n) * k * 2, 256);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(MXFP4_ERR_WORKSPACE, "safe linear needs " + std::to_string(need) + " workspace bytes");
    MX_CHECK(ldw == k / 2 && lds == k / 32, "safe mode needs contiguous packed weights and scales");
    if (int rc = mxfp4_dequant(w_packed, w_scales, workspace, x_dtype, n, k, stream)) return rc;
    wd = workspace;
    ldwd = k;
    return MXFP4_OK;
  };
  const bool fp16 = x_dtype == MXFP4_DTYPE_F16;
  const CUtensorMapDataType xt = fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;

  CUtensorMap ta, tb;
  if (m <= kGemvRows && static_cast<int64_t>(kGemvRows) * k * 2 <= 200 * 1024 && aligned(x, 16) &&
      (ldx * 2) % 16 == 0 && (wd != nullptr || (aligned(w_packed, 16) && ldw % 16 == 0))) {
    GemvParams g{};
    g.M = static_cast<int>(m);
    g.N = static_cast<int>(n);
    g.K = static_cast<int>(k);
    g.x = x;
    g.ldx = ldx;
    g.out = out;
    g.ldo = ldo;
    g.out_dtype = x_dtype;
    g.bias = bias;
    if (mode == MXFP4_LINEAR_FUSED && wd == nullptr) {
      g.w = static_cast<const uint8_t*>(w_packed);
      g.ldw = ldw;
      g.w_scales = static_cast<const uint8_t*>(w_scales);
      g.lds = lds;
      if (fp16) return push(launch_gemv<B_DECODE, true>(g, info.sms, s));
      return push(launch_gemv<B_DECODE, false>(g, info.sms, s));
    }
    if (wd == nullptr)
      if (int rc = dequant_into_workspace()) return rc;
    g.w = static_cast<const uint8_t*>(wd);
    g.ldw = ldwd * 2;
    if (fp16) return push(launch_gemv<B_TMA, true>(g, info.sms, s));
    return push(launch_gemv<B_TMA, false>(g, info.sms, s));
  }
  if (m <= kSmallMaxRows) {
    SmallParams q{};
    q.M = static_cast<int>(m);
    q.N = static_cast<int>(n);
    q.K = static_cast<int>(k);
    q.mp = static_cast<int>((m + 31) / 32 * 32);
    const int64_t row_blocks = (n + kSmRows - 1) / kSmRows;
    const int64_t kt = k / kSmBK;
    // the same stage layout (and so the same K split and summation order) in
    // both modes: fused and safe results stay bit-identical
    q.stage_bytes = q.mp * 128 + kSmWBytes + kSmPBytes;
    q.stages = static_cast<int>(std::max(2, std::min(kSmMaxStages, (200 * 1024) / q.stage_bytes)));
    // K splits: the largest cluster (<= 8) whose CTAs fit one CTA per SM
    int ks = 1;
    for (int c = 8; c >= 1; --c)
      if (row_blocks * c <= info.sms && c <= kt) { ks = c; break; }
    q.ks = ks;
    q.w_scales = static_cast<const uint8_t*>(w_scales);
    q.lds = lds;
    q.out = out;
    q.ldo = ldo;
    q.out_dtype = x_dtype;
    q.bias = bias;
    if (int rc = make_map_2d(&ta, x, xt, 2, k, m, ldx * 2, kSmBK, q.mp, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    if (mode == MXFP4_LINEAR_FUSED && wd == nullptr) {
      if (int rc = make_map_2d(&tb, w_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k / 2, n, ldw,
                               kTmPGroup * (kSmBK / 2), kSmRows, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
      if (fp16) return push(launch_small_tmem<true>(ta, tb, q, s));
      return push(launch_small_tmem<false>(ta, tb, q, s));
    }
    if (wd == nullptr)
      if (int rc = dequant_into_workspace()) return rc;
    if (int rc = make_map_2d(&tb, wd, xt, 2, k, n, ldwd * 2, kSmBK, kSmRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (fp16) return push(launch_small<B_TMA, true>(ta, tb, q, s));
    return push(launch_small<B_TMA, false>(ta, tb, q, s));
  }
  if (int rc = make_map_2d(&ta, x, xt, 2, k, m, ldx * 2, kP2BK, kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;

  PairParams p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.num_m_blocks = static_cast<int>((m + kP2BM - 1) / kP2BM);
  // pair tile width: the multiple of 32 (<= 256) that minimises rounds x width,
  // so the last round of persistent clusters is not mostly idle.  With peer
  // stores (the fused all-gather) only widths down to 64 that give every
  // cluster two or more tiles qualify: the pusher warps then send a cluster's
  // first tiles over NVLink while its tensor cores compute the next, instead
  // of every tile finishing in one round and the whole all-gather waiting for
  // the GEMM.
  {
    const int64_t clusters_max = std::max(1, info.sms / 2);
    const int min_bn = peers.n > 0 ? 64 : 128;
    int best_bn = peers.n > 0 ? 64 : 256;
    int64_t best_cost = -1;
    for (int bn = 256; bn >= min_bn; bn -= 32) {
      const int64_t tiles_bn = p.num_m_blocks * ((n + bn - 1) / bn);
      if (peers.n > 0 && tiles_bn < 2 * clusters_max) continue;
      const int64_t rounds = (tiles_bn + clusters_max - 1) / clusters_max;
      const int64_t cost = rounds * (bn + 64);  // + fixed per-tile cost of a narrower tile
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best_bn = bn;
      }
    }
    p.bn = best_bn;
  }
  p.num_n_blocks = static_cast<int>((n + p.bn - 1) / p.bn);
  p.w_scales = static_cast<const uint8_t*>(w_scales);
  p.w_rows_per_expert = n;
  p.lds = lds;
  p.out = out;
  p.ldo = ldo;
  p.out_dtype = x_dtype;
  p.bias = bias;
  p.vec_ok = aligned(out, 16) && (ldo * 2) % 16 == 0;
  p.num_peers = peers.n;
  for (int j = 0; j < kMaxPeers; ++j) p.peer_out[j] = j < peers.n ? peers.p[j] : nullptr;
  p.mc_out = peers.mc;
  if (peers.n > 0) {
    bool peers_aligned = true;
    for (int j = 0; j < peers.n; ++j) peers_aligned = peers_aligned && aligned(peers.p[j], 16);
    p.vec_ok = p.vec_ok && peers_aligned;
  }
  const int64_t tiles = static_cast<int64_t>(p.num_m_blocks) * p.num_n_blocks;
  const int clusters = static_cast<int>(std::min<int64_t>(tiles, info.sms / 2));

  const size_t once_bytes = align_up(static_cast<size_t>(n) * k * 2, 256);
  const bool decode_once = wd == nullptr && mode == MXFP4_LINEAR_FUSED && p.num_m_blocks >= kDecodeOnceRowBlocks &&
                           ldw == k / 2 && lds == k / 32 && workspace != nullptr && workspace_bytes >= once_bytes;
  if (wd == nullptr && mode == MXFP4_LINEAR_FUSED && !decode_once) {
    if (int rc = make_map_2d(&tb, w_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k / 2, n, ldw, kP2BK / 2,
                             p.bn / 2, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    if (peers.n > 0) {
      if (fp16) return launch_pair<A_TMA, B_DECODE, EPI_DENSE, true, 8, true>(ta, tb, p, clusters, s);
      return launch_pair<A_TMA, B_DECODE, EPI_DENSE, false, 8, true>(ta, tb, p, clusters, s);
    }
    return fused_pair_gemm<EPI_DENSE>(fp16, ta, tb, p, clusters, s);
  }
  // safe (and fused with many row blocks): dequant of W into the workspace, then the same MMA pipeline
  if (wd == nullptr)
    if (int rc = dequant_into_workspace()) return rc;
  if (int rc = make_map_2d(&tb, wd, xt, 2, k, n, ldwd * 2, kP2BK, p.bn / 2, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const bool after_decode = w_packed != nullptr && wd == workspace;  // the decode kernel just ran on this stream
  if (peers.n > 0) {
    if (fp16) return launch_pair<A_TMA, B_TMA, EPI_DENSE, true, 0, true>(ta, tb, p, clusters, s, after_decode);
    return launch_pair<A_TMA, B_TMA, EPI_DENSE, false, 0, true>(ta, tb, p, clusters, s, after_decode);
  }
  if (fp16) return launch_pair<A_TMA, B_TMA, EPI_DENSE, true, 0>(ta, tb, p, clusters, s, after_decode);
  return launch_pair<A_TMA, B_TMA, EPI_DENSE, false, 0>(ta, tb, p, clusters, s, after_decode);
}


// Device-side barrier over peer-mapped flag arrays (one warp): lane j signals
// rank j and waits for rank j's signal.  Every rank calls it the same number
// of times; the epoch is the local call count, kept on the device so the
// barrier works inside CUDA graphs.  A wait longer than `limit_ns` (global
// timer) records MXFP4_ERR_TIMEOUT and ends the kernel.
struct PeerFlags {
  int32_t* f[kMaxPeers + 1];  // flag array [world] of each rank
};

constexpr int64_t kBarrierLimitNs = 2000000000LL;  // default wait limit: 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void peer_barrier_kernel(PeerFlags flags, int rank, int world, int32_t* counter,
                                    int64_t limit_ns = kBarrierLimitNs) {
  const int lane = threadIdx.x;
  int epoch = 0;
  if (lane == 0) {
    epoch = *counter + 1;
    *counter = epoch;
  }
  epoch = __shfl_sync(0xFFFFFFFFu, epoch, 0);
  asm volatile("fence.acq_rel.sys;" ::: "memory");  // this rank's earlier (peer) stores before the signal
  if (lane < world) asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.f[lane] + rank), "r"(epoch) : "memory");
  if (lane < world) {
    const int32_t* mine = flags.f[rank] + lane;
    const uint64_t t0 = global_ns();
    while (true) {
      int32_t v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (v - epoch >= 0) break;
      if (static_cast<int64_t>(global_ns() - t0) > limit_ns) {
        record_error(MXFP4_ERR_TIMEOUT);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncwarp();
}

}  // namespace

extern "C" {

int mxfp4_linear_w4a16(const void* x, int x_dtype, int64_t ldx, const void* w_packed, int64_t ldw,
                       const void* w_scales, int64_t lds, const void* bias, void* out, int64_t ldo,
                       int64_t m, int64_t n, int64_t k, int mode, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return linear_impl(x, x_dtype, ldx, w_packed, ldw, w_scales, lds, bias, out, ldo, m, n, k, mode, workspace,
                     workspace_bytes, stream, PeerOut{});
}

int mxfp4_linear_dequantized(const void* x, int x_dtype, int64_t ldx, const void* w_deq, int64_t ldw,
                             const void* bias, void* out, int64_t ldo, int64_t m, int64_t n, int64_t k,
                             void* stream) {
  MX_CHECK(w_deq != nullptr, "null pointer");
  return linear_impl(x, x_dtype, ldx, nullptr, 0, nullptr, 0, bias, out, ldo, m, n, k, MXFP4_LINEAR_SAFE, nullptr, 0,
                     stream, PeerOut{}, w_deq, ldw);
}

int mxfp4_linear_w4a16_allgather(const void* x, int x_dtype, int64_t ldx, const void* w_packed, int64_t ldw,
                                 const void* w_scales, int64_t lds, const void* bias, void* out,
                                 void* const* peer_out, int num_peers, int64_t ldo, int64_t m, int64_t n,
                                 int64_t k, int mode, void* workspace, size_t workspace_bytes, void* stream) {
  MX_CHECK(num_peers >= 0 && num_peers <= kMaxPeers, "num_peers must be in [0, 7]");
  MX_CHECK(num_peers == 0 || peer_out != nullptr, "null peer_out");
  PeerOut peers{};
  peers.n = num_peers;
  for (int j = 0; j < num_peers; ++j) {
    MX_CHECK(peer_out[j] != nullptr, "null peer output pointer");
    peers.p[j] = peer_out[j];
  }
  return linear_impl(x, x_dtype, ldx, w_packed, ldw, w_scales, lds, bias, out, ldo, m, n, k, mode, workspace,
                     workspace_bytes, stream, peers);
}

int mxfp4_linear_w4a16_allgather_mc(const void* x, int x_dtype, int64_t ldx, const void* w_packed, int64_t ldw,
                                    const void* w_scales, int64_t lds, const void* bias, void* out,
                                    void* const* peer_out, int num_peers, void* out_mc, int64_t ldo, int64_t m,
                                    int64_t n, int64_t k, int mode, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  MX_CHECK(num_peers >= 1 && num_peers <= kMaxPeers, "num_peers must be in [1, 7]");
  MX_CHECK(peer_out != nullptr && out_mc != nullptr, "null peer_out or out_mc");
  MX_CHECK(reinterpret_cast<uintptr_t>(out_mc) % 16 == 0, "out_mc must be 16-byte aligned");
  PeerOut peers{};
  peers.n = num_peers;
  peers.mc = out_mc;
  for (int j = 0; j < num_peers; ++j) {
    MX_CHECK(peer_out[j] != nullptr, "null peer output pointer");
    peers.p[j] = peer_out[j];
  }
  return linear_impl(x, x_dtype, ldx, w_packed, ldw, w_scales, lds, bias, out, ldo, m, n, k, mode, workspace,
                     workspace_bytes, stream, peers);
}

int mxfp4_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(ptr != nullptr && handle != nullptr && bytes > 0, "bad ipc_alloc arguments");
  void* p = nullptr;
  MX_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(MXFP4_ERR_CUDA, std::string("ipc_alloc: ") + cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MXFP4_OK;
}

int mxfp4_ipc_open(const void* handle, void** ptr) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(ptr != nullptr && handle != nullptr, "bad ipc_open arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MX_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MXFP4_OK;
}

int mxfp4_ipc_close(void* ptr) {
  MX_CUDA(cudaIpcCloseMemHandle(ptr));
  return MXFP4_OK;
}

int mxfp4_ipc_free(void* ptr) {
  MX_CUDA(cudaFree(ptr));
  return MXFP4_OK;
}

int mxfp4_peer_barrier_timed(int32_t* const* flags, int rank, int world, int32_t* counter, int64_t timeout_us,
                             void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(world >= 1 && world <= kMaxPeers + 1 && rank >= 0 && rank < world, "bad rank/world");
  MX_CHECK(flags != nullptr && counter != nullptr, "null pointer");
  MX_CHECK(timeout_us >= 0 && timeout_us <= int64_t(60) * 1000 * 1000, "timeout_us must be in [0, 60 s]");
  PeerFlags f{};
  for (int j = 0; j < world; ++j) {
    MX_CHECK(flags[j] != nullptr && aligned(flags[j], 4), "flag arrays must be non-null and 4-byte aligned");
    f.f[j] = flags[j];
  }
  const int64_t limit_ns = timeout_us > 0 ? timeout_us * 1000 : kBarrierLimitNs;
  peer_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(f, rank, world, counter, limit_ns);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

int mxfp4_peer_barrier(int32_t* const* flags, int rank, int world, int32_t* counter, void* stream) {
  return mxfp4_peer_barrier_timed(flags, rank, world, counter, 0, stream);
}

int mxfp4_peer_barrier_reset(int32_t* local_flags, int world, int32_t* counter, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(world >= 1 && world <= kMaxPeers + 1, "bad world");
  MX_CHECK(local_flags != nullptr && counter != nullptr, "null pointer");
  cudaStream_t s = as_stream(stream);
  MX_CUDA(cudaMemsetAsync(local_flags, 0, sizeof(int32_t) * world, s));
  MX_CUDA(cudaMemsetAsync(counter, 0, sizeof(int32_t), s));
  return MXFP4_OK;
}

int mxfp4_moe_router(const void* logits, int logits_dtype, int64_t num_tokens, int num_experts, int top_k,
                     int renormalize, float* topk_weights, int32_t* topk_ids, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(logits_dtype == MXFP4_DTYPE_F32 || logits_dtype == MXFP4_DTYPE_BF16 || logits_dtype == MXFP4_DTYPE_F16,
           "router logits must be F32, BF16 or F16");
  MX_CHECK(num_tokens >= 0, "negative num_tokens");
  MX_CHECK(num_experts >= 1 && num_experts <= 32 * kRouterPerLane, "num_experts must be in [1, 256]");
  MX_CHECK(top_k >= 1 && top_k <= 32 && top_k <= num_experts, "top_k must be in [1, min(32, num_experts)]");
  if (num_tokens == 0) return MXFP4_OK;
  MX_CHECK(logits && topk_weights && topk_ids, "null pointer");
  const int64_t blocks = (num_tokens + 7) / 8;  // 8 warps, one token each
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(info.sms) * 16)));
  router_kernel<<<grid, 256, 0, as_stream(stream)>>>(logits, logits_dtype, num_tokens, num_experts, top_k,
                                                       renormalize, topk_weights, topk_ids);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

int64_t mxfp4_moe_route_capacity(int64_t num_routes, int num_experts, int block_m) {
  if (num_routes < 0 || num_experts <= 0 || block_m <= 0) return 0;
  return route_capacity(num_routes, num_experts, block_m);
}

size_t mxfp4_moe_route_workspace_size(int64_t num_routes, int num_experts) {
  return route_ws_bytes(num_routes, num_experts);
}

int mxfp4_moe_route(const void* topk_ids, int ids_dtype, int64_t num_tokens, int top_k,
                    int num_experts, int expert_offset, int block_m, int32_t* sorted_ids,
                    int32_t* block_expert, int32_t* num_post_padded, int64_t capacity,
                    void* workspace, size_t workspace_bytes, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(ids_dtype == MXFP4_DTYPE_I32 || ids_dtype == MXFP4_DTYPE_I64, "topk_ids must be I32 or I64");
  MX_CHECK(num_tokens >= 0 && top_k > 0, "bad num_tokens/top_k");
  MX_CHECK(num_experts > 0 && num_experts <= kMaxExperts, "num_experts must be in [1, 1024]");
  MX_CHECK(block_m > 0 && block_m <= 4096, "bad block_m");
  const int64_t routes = num_tokens * top_k;
  MX_CHECK(routes < (int64_t(1) << 31), "too many routes");
  MX_CHECK(sorted_ids && block_expert && num_post_padded && (routes == 0 || topk_ids), "null pointer");
  MX_CHECK(capacity >= route_capacity(routes, num_experts, block_m) && capacity % block_m == 0,
           "capacity smaller than mxfp4_moe_route_capacity()");
  if (workspace == nullptr || workspace_bytes < route_ws_bytes(routes, num_experts))
    return fail(MXFP4_ERR_WORKSPACE, "routing workspace too small");
  return run_route(topk_ids, ids_dtype, routes, num_experts, expert_offset, block_m, sorted_ids,
                   block_expert, num_post_padded, capacity, static_cast<uint8_t*>(workspace),
                   as_stream(stream));
}

}  // extern "C"

namespace {

// Tensor-core operand type of the routed op and how many BF16 parts each
// activation is split into.  C's dtype is the matmul dtype (soft:405):
//  - C BF16 / F16: A rounded to C's dtype (soft:475), one part;
//  - C F32: the products of an FP32 matmul.  BF16 and dequantised MXFP4
//    activations are exact in BF16 (one part); F16 activations are the exact
//    sum of two BF16 parts and F32 activations of three, each part multiplied
//    by the exactly decoded BF16 weights with FP32 accumulation.
struct MoeCompute {
  int dtype;  // BF16 or F16
  int parts;  // 1, 2 or 3
};

MoeCompute moe_compute(int a_dtype, int c_dtype) {
  if (c_dtype != MXFP4_DTYPE_F32) return {c_dtype, 1};
  if (a_dtype == MXFP4_DTYPE_F32) return {MXFP4_DTYPE_BF16, 3};
  if (a_dtype == MXFP4_DTYPE_F16) return {MXFP4_DTYPE_BF16, 2};
  return {MXFP4_DTYPE_BF16, 1};
}

// Which grouped GEMM a routed call runs on.  While experts receive few routes
// the tensor-memory decoder kernel (gemm_routed.cuh: 32-route padding, each
// expert's weights decoded once per chunk of up to 256 routes) wins; once the
// average expert receives kPairRoutesPerExpert routes the CTA-pair kernel over
// 256-route blocks (gemm2.cuh: shared-memory decode, two accumulators, the
// epilogue of one tile under the main loop of the next) is faster.  Both give
// the same bits: every output is the same single FP32 dot product of the same
// BF16 operands, rounded by the same epilogue chain.
constexpr int64_t kPairRoutesPerExpert = 128;
bool moe_pair_path(int64_t routes, int num_experts) {
  return routes >= kPairRoutesPerExpert * static_cast<int64_t>(num_experts);
}
// For decode batches the routed GEMV (gemv_routed.cuh) runs instead: no
// routing pass, no routed copy, each expert's weights read straight from HBM
// by the routes that use them.  Calls that can take the block-scaled grouped
// GEMM (`mx8`, below) use it up to kMoeGemvRoutesMx8 routes, the others up to
// kMoeGemvMaxRoutes (measured at the config-2 layer shape: T = 2 / 4 / 8 at
// top-8 take 38 / 67 / 123 us on the GEMV, 51 / 61 / 77 us on the block-scaled
// GEMM).  The op's FP32-precision mode with F16/F32 activations (split BF16
// parts) keeps the grouped GEMMs.
constexpr int64_t kMoeGemvRoutesMx8 = 24;
bool moe_gemv_path(int64_t routes, const MoeCompute& mc, bool mx8) {
  return routes <= (mx8 ? kMoeGemvRoutesMx8 : kMoeGemvMaxRoutes) && mc.parts == 1;
}
// Above that and below kPairRoutesPerExpert routes per expert, calls with a
// BF16 result run the block-scaled grouped GEMM (gemm_mx8.cuh) when the
// weights' alignment allows it: no weight decode.
bool mx8_dtypes(int c_dtype) { return c_dtype == MXFP4_DTYPE_BF16; }

// Routing of the pair path: 256-route blocks, no chunk table.
struct PairRouting {
  int64_t cap;
  int32_t* sorted;
  int32_t* block_expert;
  int32_t* post;
  uint8_t* route_ws;
};

size_t pair_routing_bytes(int64_t routes, int num_experts) {
  const int64_t cap = route_capacity(routes, num_experts, kP2BM);
  return align_up(sizeof(int32_t) * std::max<int64_t>(cap, 1), 256) + align_up(sizeof(int32_t) * (cap / kP2BM + 1), 256) +
         256 + route_ws_bytes(routes, num_experts);
}

PairRouting carve_pair_routing(uint8_t*& ws, int64_t routes, int num_experts) {
  PairRouting r;
  r.cap = route_capacity(routes, num_experts, kP2BM);
  r.sorted = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * std::max<int64_t>(r.cap, 1), 256);
  r.block_expert = reinterpret_cast<int32_t*>(ws);
  ws += align_up(sizeof(int32_t) * (r.cap / kP2BM + 1), 256);
  r.post = reinterpret_cast<int32_t*>(ws);
  ws += 256;
  r.route_ws = ws;
  ws += route_ws_bytes(routes, num_experts);
  return r;
}

// A converted to the operand dtype of the routed op (dequantised packed MXFP4,
// split BF16 parts, or a cast) into dst, or A itself.
int convert_activations(const void* A, int a_dtype, const void* a_mx_scale, const MoeCompute& mc, int64_t num_tokens,
                        int64_t k, void* dst, const DevInfo& info, cudaStream_t s, void* stream, const void*& a_eff) {
  a_eff = A;
  const int cdt = mc.dtype;
  if (a_dtype == MXFP4_DTYPE_U8) {
    if (int rc = mxfp4_dequant(A, a_mx_scale, dst, cdt, num_tokens, k, stream)) return rc;
    a_eff = dst;
  } else if (mc.parts > 1) {
    const int64_t cnt = num_tokens * k;
    const int grid = static_cast<int>(std::min<int64_t>((cnt + 255) / 256, int64_t(info.sms) * 8));
    split_bf16_kernel<<<grid, 256, 0, s>>>(A, a_dtype, num_tokens, k, mc.parts, reinterpret_cast<__nv_bfloat16*>(dst));
    MX_CUDA(cudaGetLastError());
    a_eff = dst;
  } else if (a_dtype != cdt) {
    const int64_t cnt = num_tokens * k;
    const int grid = static_cast<int>(std::min<int64_t>((cnt + 255) / 256, int64_t(info.sms) * 8));
    cast_kernel<<<grid, 256, 0, s>>>(A, a_dtype, dst, cdt, cnt);
    MX_CUDA(cudaGetLastError());
    a_eff = dst;
  }
  return MXFP4_OK;
}

}  // namespace

extern "C" {

// Workspace of the routed op: routing arrays and chunk table, routing
// scratch, converted A, activations in routed order.
size_t mxfp4_fused_moe_workspace_size(int64_t num_tokens, int top_k, int num_experts, int64_t n,
                                      int64_t k, int a_dtype, int c_dtype) {
  (void)n;
  const int64_t routes = num_tokens * top_k;
  const bool pair = moe_pair_path(routes, num_experts);
  const int64_t cap = route_capacity(routes, num_experts, pair ? kP2BM : kRtBlock);
  const MoeCompute mc = moe_compute(a_dtype, c_dtype);
  const int64_t ka = k * mc.parts;  // columns of the converted activations
  // sized as if the weights allow the block-scaled kernel; if they do not, the
  // GEMV that runs instead needs less
  if (moe_gemv_path(routes, mc, mx8_dtypes(c_dtype)))
    return a_dtype != mc.dtype ? align_up(static_cast<size_t>(num_tokens) * k * 2, 256) : 0;
  size_t b = pair ? pair_routing_bytes(routes, num_experts) : rt_routing_bytes(routes, num_experts);
  if (a_dtype != mc.dtype || mc.parts > 1) b += align_up(static_cast<size_t>(num_tokens) * ka * 2, 256);
  b += align_up(static_cast<size_t>(std::max<int64_t>(cap, 1)) * ka * 2, 256);  // activations in routed order
  if (mx8_dtypes(c_dtype) && !pair) {
    // the mx8 path (taken when the weights' alignment allows it): routing with
    // its chunk size, converted A, the split activations in routed order
    const int bn = mx8_bn(routes, num_experts);
    size_t m = rt_routing_bytes(routes, num_experts, bn);
    if (a_dtype != mc.dtype) m += align_up(static_cast<size_t>(num_tokens) * k * 2, 256);
    m += mx8_act_bytes(route_capacity(routes, num_experts, kRtBlock), k, rt_max_chunks(routes, num_experts, bn), bn);
    b = std::max(b, m);
  }
  return b;
}

int mxfp4_fused_moe(const void* A, int a_dtype, const void* a_mx_scale, const void* B,
                    const void* B_mx_scale, const float* a_scale, const float* b_scale,
                    const void* topk_weights, int w_dtype, const void* topk_ids, int ids_dtype,
                    void* C, int c_dtype, int64_t num_tokens, int top_k, int num_experts,
                    int64_t n, int64_t k, int mul_routed_weight, void* workspace,
                    size_t workspace_bytes, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  if (int rc = check_scales_layout(k)) return rc;
  MX_CHECK(A && B && B_mx_scale && a_scale && b_scale && topk_ids && C, "null pointer");
  MX_CHECK(c_dtype == MXFP4_DTYPE_F32 || c_dtype == MXFP4_DTYPE_BF16 || c_dtype == MXFP4_DTYPE_F16,
           "C must be F32, BF16 or F16");
  MX_CHECK(a_dtype == MXFP4_DTYPE_U8 || a_dtype == MXFP4_DTYPE_BF16 || a_dtype == MXFP4_DTYPE_F16 ||
               a_dtype == MXFP4_DTYPE_F32,
           "A must be U8 (packed MXFP4), BF16, F16 or F32");
  MX_CHECK(a_dtype != MXFP4_DTYPE_U8 || a_mx_scale != nullptr, "packed MXFP4 activations require A_mx_scale");
  MX_CHECK(!mul_routed_weight || topk_weights != nullptr, "route weights required");
  MX_CHECK(w_dtype == MXFP4_DTYPE_F32 || w_dtype == MXFP4_DTYPE_BF16 || w_dtype == MXFP4_DTYPE_F16,
           "topk_weights must be F32, BF16 or F16");
  MX_CHECK(num_tokens >= 0 && top_k > 0 && num_experts > 0 && num_experts <= kMaxExperts && n > 0,
           "bad sizes");
  MX_CHECK(num_tokens * top_k < (int64_t(1) << 31) && n < (int64_t(1) << 31), "dimension too large");
  MX_CHECK(k < (int64_t(1) << 30), "dimension too large");
  const MoeCompute mc = moe_compute(a_dtype, c_dtype);
  const int cdt = mc.dtype;
  const int64_t ka = k * mc.parts;  // K of the converted activations (k_rep parts)
  const size_t need = mxfp4_fused_moe_workspace_size(num_tokens, top_k, num_experts, n, k, a_dtype, c_dtype);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MXFP4_ERR_WORKSPACE, "fused MoE needs " + std::to_string(need) + " workspace bytes");
  cudaStream_t s = as_stream(stream);
  const int64_t routes = num_tokens * top_k;
  const int esz = elem_size(c_dtype);
  if (routes == 0) return MXFP4_OK;
  // C.zero_() (soft:476): routes to other experts stay zero
  MX_CUDA(cudaMemsetAsync(C, 0, static_cast<size_t>(routes) * n * esz, s));

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const bool mx8 = mx8_dtypes(c_dtype) && mx8_weights_ok(B, B_mx_scale);
  if (moe_gemv_path(routes, mc, mx8)) {
    const void* a_eff;
    if (int rc = convert_activations(A, a_dtype, a_mx_scale, mc, num_tokens, k, ws, info, s, stream, a_eff)) return rc;
    MoeGemvParams g{};
    g.K = static_cast<int>(k);
    g.rows = static_cast<int>(n);
    g.num_experts = num_experts;
    g.top_k = top_k;
    g.num_routes = static_cast<int>(routes);
    g.x = a_eff;
    g.ldx = k;
    g.w = static_cast<const uint8_t*>(B);
    g.w_rows_per_expert = n;
    g.ldw = k / 2;
    g.w_scales = static_cast<const uint8_t*>(B_mx_scale);
    g.lds = k / 32;
    g.ids = topk_ids;
    g.ids_dtype = ids_dtype;
    g.out = C;
    g.ldo = n;
    g.out_dtype = c_dtype;
    g.a_scale = a_scale;
    g.b_scale = b_scale;
    g.topk_w = topk_weights;
    g.w_dtype = w_dtype;
    g.mul_w = mul_routed_weight ? 1 : 0;
    if (cdt == MXFP4_DTYPE_F16) return launch_moe_gemv<EPI_MOE, true>(g, s);
    return launch_moe_gemv<EPI_MOE, false>(g, s);
  }
  if (mx8_dtypes(c_dtype) && !moe_pair_path(routes, num_experts) && mx8_weights_ok(B, B_mx_scale)) {
    const int bn = mx8_bn(routes, num_experts);
    const RtRouting rt = carve_rt_routing(ws, routes, num_experts, bn);
    const void* a_eff;
    if (int rc = convert_activations(A, a_dtype, a_mx_scale, mc, num_tokens, k, ws, info, s, stream, a_eff)) return rc;
    MX_CHECK(aligned(a_eff, 16), "A must be 16-byte aligned");
    if (a_eff != A) ws += align_up(static_cast<size_t>(num_tokens) * k * 2, 256);
    if (int rc = run_rt_routing(topk_ids, ids_dtype, routes, num_experts, rt, s)) return rc;
    const Mx8Act act = carve_mx8_act(ws, rt.cap, k, rt.max_chunks, bn);
    if (int rc = run_mx8_split(a_eff, k, k, rt, rt.sorted, routes, top_k, act, info.sms, s)) return rc;
    CUtensorMap tw, txh, txl;
    const int group = mx8_group(bn, k);
    if (int rc = mx8_maps(&tw, &txh, &txl, B, static_cast<int64_t>(num_experts) * n, k, act, rt.cap, 0, group, bn))
      return rc;
    Mx8Params p{};
    p.group = group;
    p.N = static_cast<int>(n);
    p.K = static_cast<int>(k);
    p.num_wblocks = static_cast<int>((n + 127) / 128);
    p.w_scales = static_cast<const uint8_t*>(B_mx_scale);
    p.lds = k / 32;
    p.w_rows_per_expert = n;
    p.sfh = act.sfh;
    p.sfl = act.sfl;
    p.chunks = rt.chunks;
    p.num_chunks = rt.num_chunks;
    p.max_chunks = static_cast<int>(rt.max_chunks);
    p.sorted_ids = rt.sorted;
    p.num_routes = static_cast<int>(routes);
    p.top_k = top_k;
    p.out = C;
    p.out_dtype = c_dtype;
    p.a_scale = a_scale;
    p.b_scale = b_scale;
    p.topk_w = topk_weights;
    p.w_dtype = w_dtype;
    p.mul_w = mul_routed_weight ? 1 : 0;
    p.c_stride_t = static_cast<int64_t>(top_k) * n;
    p.c_stride_j = n;
    return launch_mx8<EPI_MOE>(bn, tw, txh, txl, p, info.sms, s);
  }
  if (moe_pair_path(routes, num_experts)) {
    // many routes per expert: the pair kernel over 256-route blocks
    const PairRouting pr = carve_pair_routing(ws, routes, num_experts);
    const void* a_eff;
    if (int rc = convert_activations(A, a_dtype, a_mx_scale, mc, num_tokens, k, ws, info, s, stream, a_eff)) return rc;
    if (int rc = run_route(topk_ids, ids_dtype, routes, num_experts, 0, kP2BM, pr.sorted, pr.block_expert, pr.post,
                           pr.cap, pr.route_ws, s))
      return rc;
    MX_CHECK(aligned(a_eff, 16), "A must be 16-byte aligned");
    if (a_eff != A) ws += align_up(static_cast<size_t>(num_tokens) * ka * 2, 256);
    void* a_routed = ws;
    if (int rc = run_gather(a_eff, ka, pr.sorted, pr.post, routes, top_k, a_routed, pr.cap, info.sms, s)) return rc;
    CUtensorMap ta, tb;
    const CUtensorMapDataType at =
        cdt == MXFP4_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (int rc = make_map_2d(&ta, a_routed, at, 2, ka, pr.cap, ka * 2, kP2BK, kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = make_map_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k / 2, static_cast<uint64_t>(num_experts) * n,
                             k / 2, kP2BK / 2, kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    PairParams p{};
    p.N = static_cast<int>(n);
    p.K = static_cast<int>(ka);
    p.k_rep = mc.parts;
    p.bn = 256;
    p.num_m_blocks = static_cast<int>(pr.cap / kP2BM);
    p.num_n_blocks = static_cast<int>((n + p.bn - 1) / p.bn);
    p.a_ptr = static_cast<const uint8_t*>(a_eff);
    p.lda = ka;
    p.w_scales = static_cast<const uint8_t*>(B_mx_scale);
    p.lds = k / 32;
    p.w_rows_per_expert = n;
    p.sorted_ids = pr.sorted;
    p.block_expert = pr.block_expert;
    p.num_post_padded = pr.post;
    p.num_routes = static_cast<int>(routes);
    p.top_k = top_k;
    p.out = C;
    p.out_dtype = c_dtype;
    p.a_scale = a_scale;
    p.b_scale = b_scale;
    p.topk_w = topk_weights;
    p.w_dtype = w_dtype;
    p.mul_w = mul_routed_weight ? 1 : 0;
    p.c_stride_t = static_cast<int64_t>(top_k) * n;
    p.c_stride_j = n;
    p.vec_ok = aligned(C, 16) && (n * esz) % 16 == 0;
    return routed_pair_gemm<A_TMA, EPI_MOE>(cdt == MXFP4_DTYPE_F16, ta, tb, p, info.sms, s);
  }
  const RtRouting rt = carve_rt_routing(ws, routes, num_experts);
  const void* a_eff;
  if (int rc = convert_activations(A, a_dtype, a_mx_scale, mc, num_tokens, k, ws, info, s, stream, a_eff)) return rc;
  if (int rc = run_rt_routing(topk_ids, ids_dtype, routes, num_experts, rt, s)) return rc;
  MX_CHECK(aligned(a_eff, 16), "A must be 16-byte aligned");
  if (a_eff != A) ws += align_up(static_cast<size_t>(num_tokens) * ka * 2, 256);
  void* a_routed = ws;
  if (int rc = run_gather(a_eff, ka, rt.sorted, rt.post, routes, top_k, a_routed, rt.cap, info.sms, s)) return rc;

  CUtensorMap tw, tx16, tx128;
  if (int rc = routed_maps(&tw, &tx16, &tx128, B, static_cast<int64_t>(num_experts) * n, k, a_routed, rt.cap, ka,
                           cdt == MXFP4_DTYPE_F16, false))
    return rc;
  RoutedParams p{};
  p.pgroup = routed_pgroup(k);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(ka);
  p.k_rep = mc.parts;
  p.num_wblocks = static_cast<int>((n + 255) / 256);
  p.w_scales = static_cast<const uint8_t*>(B_mx_scale);
  p.lds = k / 32;
  p.w_rows_per_expert = n;
  p.chunks = rt.chunks;
  p.num_chunks = rt.num_chunks;
  p.max_chunks = static_cast<int>(rt.max_chunks);
  p.sorted_ids = rt.sorted;
  p.num_routes = static_cast<int>(routes);
  p.top_k = top_k;
  p.out = C;
  p.out_dtype = c_dtype;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.topk_w = topk_weights;
  p.w_dtype = w_dtype;
  p.mul_w = mul_routed_weight ? 1 : 0;
  p.c_stride_t = static_cast<int64_t>(top_k) * n;
  p.c_stride_j = n;
  if (cdt == MXFP4_DTYPE_F16) return launch_routed<EPI_MOE, true>(tw, tx16, tx128, p, info.sms, s);
  return launch_routed<EPI_MOE, false>(tw, tx16, tx128, p, info.sms, s);
}

// Same operation as mxfp4_fused_moe, with its scratch taken from the static
// g_noalloc_scratch array instead of a caller workspace: no cudaMalloc, no
// cudaFree, no allocating library call.  Requests whose scratch would exceed
// kNoAllocScratchBytes are rejected.  All calls share the array, so calls that
// overlap on the GPU race.  Nothing in it needs to start at zero: every byte
// that decides a result is written earlier in the same call (routing arrays,
// converted and routed activation rows); the padding rows of the routed copy
// keep whatever an earlier call left there, and the GEMM reads them but
// discards their results.
int mxfp4_fused_moe_noalloc(const void* A, int a_dtype, const void* a_mx_scale, const void* B,
                            const void* B_mx_scale, const float* a_scale, const float* b_scale,
                            const void* topk_weights, int w_dtype, const void* topk_ids, int ids_dtype,
                            void* C, int c_dtype, int64_t num_tokens, int top_k, int num_experts,
                            int64_t n, int64_t k, int mul_routed_weight, void* stream) {
  // the sizes and dtypes the workspace size depends on are checked first, so a
  // bad argument is reported as one and not as a scratch overflow
  MX_CHECK(num_tokens >= 0 && top_k > 0 && num_experts > 0 && num_experts <= kMaxExperts && n > 0,
           "bad sizes");
  MX_CHECK(num_tokens * top_k < (int64_t(1) << 31) && n < (int64_t(1) << 31), "dimension too large");
  if (int rc = check_scales_layout(k)) return rc;
  MX_CHECK(k < (int64_t(1) << 30), "dimension too large");
  MX_CHECK(c_dtype == MXFP4_DTYPE_F32 || c_dtype == MXFP4_DTYPE_BF16 || c_dtype == MXFP4_DTYPE_F16,
           "C must be F32, BF16 or F16");
  MX_CHECK(a_dtype == MXFP4_DTYPE_U8 || a_dtype == MXFP4_DTYPE_BF16 || a_dtype == MXFP4_DTYPE_F16 ||
               a_dtype == MXFP4_DTYPE_F32,
           "A must be U8 (packed MXFP4), BF16, F16 or F32");
  const size_t need = mxfp4_fused_moe_workspace_size(num_tokens, top_k, num_experts, n, k, a_dtype, c_dtype);
  if (need > kNoAllocScratchBytes)
    return fail(MXFP4_ERR_WORKSPACE, "mxfp4_fused_moe_noalloc needs " + std::to_string(need) +
                                         " scratch bytes, more than its static " +
                                         std::to_string(kNoAllocScratchBytes) +
                                         "-byte array; call mxfp4_fused_moe with a workspace instead");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return mxfp4_fused_moe(A, a_dtype, a_mx_scale, B, B_mx_scale, a_scale, b_scale, topk_weights, w_dtype,
                         topk_ids, ids_dtype, C, c_dtype, num_tokens, top_k, num_experts, n, k,
                         mul_routed_weight, scratch, kNoAllocScratchBytes, stream);
}

int mxfp4_quantize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t k, void* packed,
                   void* scales, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(x && packed && scales, "null pointer");
  MX_CHECK(x_dtype == MXFP4_DTYPE_BF16 || x_dtype == MXFP4_DTYPE_F32, "quantizer input must be BF16 or F32");
  MX_CHECK(rows >= 0 && k > 0 && k % 32 == 0 && ldx >= k, "K must be a positive multiple of 32");
  MX_CHECK(aligned(x, 16) && (ldx * elem_size(x_dtype)) % 16 == 0 && aligned(packed, 16),
           "quantizer operands must be 16-byte aligned");
  const int64_t nb = rows * (k / 32);
  if (nb == 0) return MXFP4_OK;
  const int grid = static_cast<int>(std::min<int64_t>((nb + 255) / 256, int64_t(info.sms) * 8));
  cudaStream_t s = as_stream(stream);
  if (x_dtype == MXFP4_DTYPE_BF16)
    quantize_kernel<MXFP4_DTYPE_BF16><<<grid, 256, 0, s>>>(x, ldx, rows, k, static_cast<uint8_t*>(packed),
                                                          static_cast<uint8_t*>(scales));
  else
    quantize_kernel<MXFP4_DTYPE_F32><<<grid, 256, 0, s>>>(x, ldx, rows, k, static_cast<uint8_t*>(packed),
                                                         static_cast<uint8_t*>(scales));
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

size_t mxfp4_gemm_w4a4_workspace_size(int64_t m, int64_t n, int64_t k) {
  const int64_t kch = k / 128;
  const int64_t mrb = (m + kW4BM - 1) / kW4BM;
  const int64_t nrb = 2 * ((n + kW4BN - 1) / kW4BN);
  return align_up(static_cast<size_t>(mrb * kch * 512), 256) + align_up(static_cast<size_t>(nrb * kch * 512), 256);
}

int mxfp4_gemm_w4a4(const void* a, const void* a_scales, const void* b, const void* b_scales, void* out,
                    int out_dtype, int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                    void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  if (int rc = check_scales_layout(k)) return rc;
  MX_CHECK(a && a_scales && b && b_scales && out, "null pointer");
  MX_CHECK(out_dtype == MXFP4_DTYPE_BF16 || out_dtype == MXFP4_DTYPE_F16 || out_dtype == MXFP4_DTYPE_F32,
           "W4A4 output must be BF16, F16 or F32");
  MX_CHECK(m >= 0 && n > 0 && m < (int64_t(1) << 31) && n < (int64_t(1) << 31), "bad M/N");
  const size_t need = mxfp4_gemm_w4a4_workspace_size(m, n, k);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MXFP4_ERR_WORKSPACE, "W4A4 GEMM needs " + std::to_string(need) + " workspace bytes");
  if (m == 0) return MXFP4_OK;
  cudaStream_t s = as_stream(stream);
  const int kch = static_cast<int>(k / 128);
  const int mrb = static_cast<int>((m + kW4BM - 1) / kW4BM);
  const int nrb = static_cast<int>(2 * ((n + kW4BN - 1) / kW4BN));
  uint8_t* sfa = static_cast<uint8_t*>(workspace);
  uint8_t* sfb = sfa + align_up(static_cast<size_t>(mrb) * kch * 512, 256);
  {
    const int64_t wa = static_cast<int64_t>(mrb) * 128 * kch, wb = static_cast<int64_t>(nrb) * 128 * kch;
    sf_block_kernel<<<static_cast<int>(std::min<int64_t>((wa + 255) / 256, info.sms * 8)), 256, 0, s>>>(
        static_cast<const uint8_t*>(a_scales), k / 32, static_cast<int>(m), kch, mrb, sfa);
    sf_block_kernel<<<static_cast<int>(std::min<int64_t>((wb + 255) / 256, info.sms * 8)), 256, 0, s>>>(
        static_cast<const uint8_t*>(b_scales), k / 32, static_cast<int>(n), kch, nrb, sfb);
    MX_CUDA(cudaGetLastError());
  }
  CUtensorMap ta, tb;
  if (int rc = make_map_2d(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k / 2, m, k / 2, 128, kW4BM,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = make_map_2d(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k / 2, n, k / 2, 128, kW4BN,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  W4A4Params p{};
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.num_m_blocks = mrb;
  p.num_n_blocks = static_cast<int>((n + kW4BN - 1) / kW4BN);
  p.sfa_blk = sfa;
  p.sfb_blk = sfb;
  p.out = out;
  p.ldo = n;
  p.out_dtype = out_dtype;
  p.vec_ok = aligned(out, 16) && (n * elem_size(out_dtype)) % 16 == 0;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(mxfp4_w4a4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kW4SmemBytes);
  });
  MX_CUDA(attr_err);
  const int64_t tiles = static_cast<int64_t>(p.num_m_blocks) * p.num_n_blocks;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, info.sms));
  mxfp4_w4a4_kernel<<<grid, kW4Threads, kW4SmemBytes, s>>>(ta, tb, p);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}

size_t mxfp4_moe_layer_workspace_size(int64_t num_tokens, int top_k, int num_experts, int64_t hidden,
                                      int64_t inter) {
  const int64_t routes = num_tokens * top_k;
  // routed GEMV: h and the weighted down rows, by route (sized as if the
  // weights allow the block-scaled kernel; the GEMV that runs instead if they
  // do not needs less than that kernel's workspace)
  if (routes <= kMoeGemvRoutesMx8)
    return align_up(static_cast<size_t>(routes) * inter * 2, 256) + align_up(static_cast<size_t>(routes) * hidden * 2, 256);
  const bool pair = moe_pair_path(routes, num_experts);
  const int64_t cap = std::max<int64_t>(route_capacity(routes, num_experts, pair ? kP2BM : kRtBlock), 1);
  size_t b = pair ? pair_routing_bytes(routes, num_experts) : rt_routing_bytes(routes, num_experts);
  b += align_up(static_cast<size_t>(cap) * inter * 2, 256);                           // h in routed order
  b += align_up(static_cast<size_t>(std::max<int64_t>(routes, 1)) * hidden * 2, 256);  // weighted down rows
  b += align_up(static_cast<size_t>(cap) * hidden * 2, 256);                          // x in routed order
  if (!pair) {
    // the mx8 path (taken when the weights' alignment allows it)
    const int bn = mx8_bn(routes, num_experts);
    const int64_t rcap = std::max<int64_t>(route_capacity(routes, num_experts, kRtBlock), 1);
    size_t m = rt_routing_bytes(routes, num_experts, bn);
    m += align_up(static_cast<size_t>(rcap) * inter * 2, 256);                          // h in routed order
    m += align_up(static_cast<size_t>(std::max<int64_t>(routes, 1)) * hidden * 2, 256);  // weighted down rows
    const int64_t mch = rt_max_chunks(routes, num_experts, bn);
    m += mx8_act_bytes(rcap, hidden, mch, bn) + mx8_act_bytes(rcap, inter, mch, bn);    // split x and h
    b = std::max(b, m);
  }
  return b;
}

int mxfp4_moe_layer(const void* x, const void* w13, const void* w13_scale, const void* w2,
                    const void* w2_scale, const void* topk_weights, int w_dtype,
                    const void* topk_ids, int ids_dtype, void* out, int64_t num_tokens, int top_k,
                    int num_experts, int64_t hidden, int64_t inter, void* workspace,
                    size_t workspace_bytes, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  MX_CHECK(x && w13 && w13_scale && w2 && w2_scale && topk_weights && topk_ids && out, "null pointer");
  MX_CHECK(hidden > 0 && hidden % 128 == 0, "hidden must be a positive multiple of 128");
  MX_CHECK(inter > 0 && inter % 128 == 0, "intermediate size must be a positive multiple of 128");
  MX_CHECK(num_tokens >= 0 && top_k > 0 && num_experts > 0 && num_experts <= kMaxExperts, "bad sizes");
  MX_CHECK(w_dtype == MXFP4_DTYPE_F32 || w_dtype == MXFP4_DTYPE_BF16 || w_dtype == MXFP4_DTYPE_F16,
           "topk_weights must be F32, BF16 or F16");
  MX_CHECK(ids_dtype == MXFP4_DTYPE_I32 || ids_dtype == MXFP4_DTYPE_I64, "topk_ids must be I32 or I64");
  MX_CHECK(aligned(x, 16) && aligned(out, 16), "x and out must be 16-byte aligned");
  const size_t need = mxfp4_moe_layer_workspace_size(num_tokens, top_k, num_experts, hidden, inter);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MXFP4_ERR_WORKSPACE, "MoE layer needs " + std::to_string(need) + " workspace bytes");
  cudaStream_t s = as_stream(stream);
  const int64_t routes = num_tokens * top_k;
  if (num_tokens == 0) return MXFP4_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* ybuf = nullptr;  // [routes, hidden]: the weighted down rows, by route id
  const bool mx8 = mx8_weights_ok(w13, w13_scale) && mx8_weights_ok(w2, w2_scale);
  if (routes <= (mx8 ? kMoeGemvRoutesMx8 : kMoeGemvMaxRoutes)) {
    // few routes: routed GEMVs straight from the token rows, h by route
    void* hbuf = ws;
    ws += align_up(static_cast<size_t>(routes) * inter * 2, 256);
    ybuf = ws;
    MoeGemvParams g{};
    g.K = static_cast<int>(hidden);
    g.rows = static_cast<int>(inter);
    g.num_experts = num_experts;
    g.top_k = top_k;
    g.num_routes = static_cast<int>(routes);
    g.x = x;
    g.ldx = hidden;
    g.w = static_cast<const uint8_t*>(w13);
    g.w_rows_per_expert = 2 * inter;
    g.ldw = hidden / 2;
    g.w_scales = static_cast<const uint8_t*>(w13_scale);
    g.lds = hidden / 32;
    g.ids = topk_ids;
    g.ids_dtype = ids_dtype;
    g.glu_inter = static_cast<int>(inter);
    g.out = hbuf;
    g.ldo = inter;
    g.out_dtype = MXFP4_DTYPE_BF16;
    if (int rc = launch_moe_gemv<EPI_GLU, false>(g, s)) return rc;
    MoeGemvParams d{};
    d.K = static_cast<int>(inter);
    d.rows = static_cast<int>(hidden);
    d.num_experts = num_experts;
    d.top_k = 1;
    d.num_routes = static_cast<int>(routes);
    d.x = hbuf;
    d.ldx = inter;
    d.w = static_cast<const uint8_t*>(w2);
    d.w_rows_per_expert = hidden;
    d.ldw = inter / 2;
    d.w_scales = static_cast<const uint8_t*>(w2_scale);
    d.lds = inter / 32;
    d.ids = topk_ids;
    d.ids_dtype = ids_dtype;
    d.out = ybuf;
    d.ldo = hidden;
    d.out_dtype = MXFP4_DTYPE_BF16;
    d.topk_w = topk_weights;
    d.w_dtype = w_dtype;
    d.mul_w = 1;
    if (int rc = launch_moe_gemv<EPI_MOE, false>(d, s)) return rc;
  } else if (!moe_pair_path(routes, num_experts) && mx8) {
    // block-scaled grouped GEMMs: x and h split into E4M3 hi/lo in routed order
    const int bn = mx8_bn(routes, num_experts);
    const RtRouting rt = carve_rt_routing(ws, routes, num_experts, bn);
    const int64_t cap = std::max<int64_t>(rt.cap, 1);
    void* hbuf = ws;
    ws += align_up(static_cast<size_t>(cap) * inter * 2, 256);
    ybuf = ws;
    ws += align_up(static_cast<size_t>(routes) * hidden * 2, 256);
    const Mx8Act ax = carve_mx8_act(ws, cap, hidden, rt.max_chunks, bn);
    const Mx8Act ah = carve_mx8_act(ws, cap, inter, rt.max_chunks, bn);
    if (int rc = run_rt_routing(topk_ids, ids_dtype, routes, num_experts, rt, s)) return rc;
    if (int rc = run_mx8_split(x, hidden, hidden, rt, rt.sorted, routes, top_k, ax, info.sms, s)) return rc;
    // gate_up with fused SiLU(gate) * up -> h [cap, inter] in routed order
    {
      CUtensorMap tw, txh, txl;
      const int group = mx8_group(bn, hidden);
      if (int rc = mx8_maps(&tw, &txh, &txl, w13, static_cast<int64_t>(num_experts) * 2 * inter, hidden, ax, cap, inter,
                            group, bn))
        return rc;
      Mx8Params p{};
      p.group = group;
      p.N = static_cast<int>(2 * inter);
      p.glu_inter = static_cast<int>(inter);
      p.K = static_cast<int>(hidden);
      p.num_wblocks = static_cast<int>((inter + 63) / 64);
      p.w_scales = static_cast<const uint8_t*>(w13_scale);
      p.lds = hidden / 32;
      p.w_rows_per_expert = 2 * inter;
      p.sfh = ax.sfh;
      p.sfl = ax.sfl;
      p.chunks = rt.chunks;
      p.num_chunks = rt.num_chunks;
      p.max_chunks = static_cast<int>(rt.max_chunks);
      p.sorted_ids = rt.sorted;
      p.num_routes = static_cast<int>(routes);
      p.top_k = top_k;
      p.out = hbuf;
      p.ldo = inter;
      p.out_dtype = MXFP4_DTYPE_BF16;
      if (int rc = launch_mx8<EPI_GLU>(bn, tw, txh, txl, p, info.sms, s)) return rc;
    }
    if (int rc = run_mx8_split(hbuf, inter, inter, rt, nullptr, routes, 1, ah, info.sms, s)) return rc;
    // down with route weights, scattered to y[route]
    {
      CUtensorMap tw, txh, txl;
      const int group = mx8_group(bn, inter);
      if (int rc = mx8_maps(&tw, &txh, &txl, w2, static_cast<int64_t>(num_experts) * hidden, inter, ah, cap, 0, group, bn))
        return rc;
      Mx8Params p{};
      p.group = group;
      p.N = static_cast<int>(hidden);
      p.K = static_cast<int>(inter);
      p.num_wblocks = static_cast<int>((hidden + 127) / 128);
      p.w_scales = static_cast<const uint8_t*>(w2_scale);
      p.lds = inter / 32;
      p.w_rows_per_expert = hidden;
      p.sfh = ah.sfh;
      p.sfl = ah.sfl;
      p.chunks = rt.chunks;
      p.num_chunks = rt.num_chunks;
      p.max_chunks = static_cast<int>(rt.max_chunks);
      p.sorted_ids = rt.sorted;
      p.num_routes = static_cast<int>(routes);
      p.top_k = 1;
      p.out = ybuf;
      p.out_dtype = MXFP4_DTYPE_BF16;
      p.topk_w = topk_weights;
      p.w_dtype = w_dtype;
      p.mul_w = 1;
      p.c_stride_t = hidden;
      p.c_stride_j = 0;
      if (int rc = launch_mx8<EPI_MOE>(bn, tw, txh, txl, p, info.sms, s)) return rc;
    }
  } else if (moe_pair_path(routes, num_experts)) {
    // many routes per expert: pair kernel over 256-route blocks
    const PairRouting pr = carve_pair_routing(ws, routes, num_experts);
    const int64_t cap = std::max<int64_t>(pr.cap, 1);
    void* hbuf = ws;
    ws += align_up(static_cast<size_t>(cap) * inter * 2, 256);
    ybuf = ws;
    ws += align_up(static_cast<size_t>(routes) * hidden * 2, 256);
    void* xbuf = ws;
    if (int rc = run_route(topk_ids, ids_dtype, routes, num_experts, 0, kP2BM, pr.sorted, pr.block_expert, pr.post,
                           pr.cap, pr.route_ws, s))
      return rc;
    if (int rc = run_gather(x, hidden, pr.sorted, pr.post, routes, top_k, xbuf, pr.cap, info.sms, s)) return rc;
    // gate_up with fused SiLU(gate) * up -> h [cap, inter] in routed order
    {
      CUtensorMap ta, tb;
      if (int rc = make_map_2d(&ta, xbuf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hidden, pr.cap, hidden * 2, kP2BK,
                               kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
      if (int rc = make_map_2d(&tb, w13, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, hidden / 2,
                               static_cast<uint64_t>(num_experts) * 2 * inter, hidden / 2, kP2BK / 2, kP2HalfRows,
                               CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
      PairParams p{};
      p.N = static_cast<int>(2 * inter);
      p.K = static_cast<int>(hidden);
      p.bn = 256;
      p.num_m_blocks = static_cast<int>(pr.cap / kP2BM);
      p.num_n_blocks = static_cast<int>((inter + p.bn / 2 - 1) / (p.bn / 2));
      p.a_ptr = static_cast<const uint8_t*>(x);
      p.lda = hidden;
      p.w_scales = static_cast<const uint8_t*>(w13_scale);
      p.lds = hidden / 32;
      p.w_rows_per_expert = 2 * inter;
      p.glu_inter = static_cast<int>(inter);
      p.sorted_ids = pr.sorted;
      p.block_expert = pr.block_expert;
      p.num_post_padded = pr.post;
      p.num_routes = static_cast<int>(routes);
      p.top_k = top_k;
      p.out = hbuf;
      p.ldo = inter;
      p.out_dtype = MXFP4_DTYPE_BF16;
      p.vec_ok = 1;
      if (int rc = routed_pair_gemm<A_TMA, EPI_GLU>(false, ta, tb, p, info.sms, s)) return rc;
    }
    // down with route weights, scattered to y[route]
    {
      CUtensorMap ta, tb;
      if (int rc = make_map_2d(&ta, hbuf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inter, pr.cap, inter * 2, kP2BK,
                               kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
      if (int rc = make_map_2d(&tb, w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inter / 2,
                               static_cast<uint64_t>(num_experts) * hidden, inter / 2, kP2BK / 2, kP2HalfRows,
                               CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
      PairParams p{};
      p.N = static_cast<int>(hidden);
      p.K = static_cast<int>(inter);
      p.bn = 256;
      p.num_m_blocks = static_cast<int>(pr.cap / kP2BM);
      p.num_n_blocks = static_cast<int>((hidden + p.bn - 1) / p.bn);
      p.w_scales = static_cast<const uint8_t*>(w2_scale);
      p.lds = inter / 32;
      p.w_rows_per_expert = hidden;
      p.sorted_ids = pr.sorted;
      p.block_expert = pr.block_expert;
      p.num_post_padded = pr.post;
      p.num_routes = static_cast<int>(routes);
      p.top_k = 1;
      p.out = ybuf;
      p.out_dtype = MXFP4_DTYPE_BF16;
      p.a_scale = nullptr;
      p.b_scale = nullptr;
      p.topk_w = topk_weights;
      p.w_dtype = w_dtype;
      p.mul_w = 1;
      p.c_stride_t = hidden;
      p.c_stride_j = 0;
      p.vec_ok = 1;
      if (int rc = routed_pair_gemm<A_TMA, EPI_MOE>(false, ta, tb, p, info.sms, s)) return rc;
    }
  } else {
    const RtRouting rt = carve_rt_routing(ws, routes, num_experts);
    const int64_t cap = std::max<int64_t>(rt.cap, 1);
    void* hbuf = ws;
    ws += align_up(static_cast<size_t>(cap) * inter * 2, 256);
    ybuf = ws;
    ws += align_up(static_cast<size_t>(routes) * hidden * 2, 256);
    void* xbuf = ws;
    if (int rc = run_rt_routing(topk_ids, ids_dtype, routes, num_experts, rt, s)) return rc;
    if (int rc = run_gather(x, hidden, rt.sorted, rt.post, routes, top_k, xbuf, rt.cap, info.sms, s)) return rc;
    // gate_up with fused SiLU(gate) * up -> h [cap, inter] in routed order
    {
      CUtensorMap tw, tx16, tx128;
      if (int rc = routed_maps(&tw, &tx16, &tx128, w13, static_cast<int64_t>(num_experts) * 2 * inter, hidden, xbuf,
                               cap, hidden, false, true))
        return rc;
      RoutedParams p{};
      p.pgroup = routed_pgroup(hidden);
      p.N = static_cast<int>(2 * inter);
      p.glu_inter = static_cast<int>(inter);
      p.K = static_cast<int>(hidden);
      p.num_wblocks = static_cast<int>((inter + 127) / 128);
      p.w_scales = static_cast<const uint8_t*>(w13_scale);
      p.lds = hidden / 32;
      p.w_rows_per_expert = 2 * inter;
      p.chunks = rt.chunks;
      p.num_chunks = rt.num_chunks;
      p.max_chunks = static_cast<int>(rt.max_chunks);
      p.sorted_ids = rt.sorted;
      p.num_routes = static_cast<int>(routes);
      p.top_k = top_k;
      p.out = hbuf;
      p.ldo = inter;
      p.out_dtype = MXFP4_DTYPE_BF16;
      if (int rc = launch_routed<EPI_GLU, false>(tw, tx16, tx128, p, info.sms, s)) return rc;
    }
    // down with route weights, scattered to y[route]
    {
      CUtensorMap tw, tx16, tx128;
      if (int rc = routed_maps(&tw, &tx16, &tx128, w2, static_cast<int64_t>(num_experts) * hidden, inter, hbuf, cap,
                               inter, false, false))
        return rc;
      RoutedParams p{};
      p.pgroup = routed_pgroup(inter);
      p.N = static_cast<int>(hidden);
      p.K = static_cast<int>(inter);
      p.num_wblocks = static_cast<int>((hidden + 255) / 256);
      p.w_scales = static_cast<const uint8_t*>(w2_scale);
      p.lds = inter / 32;
      p.w_rows_per_expert = hidden;
      p.chunks = rt.chunks;
      p.num_chunks = rt.num_chunks;
      p.max_chunks = static_cast<int>(rt.max_chunks);
      p.sorted_ids = rt.sorted;
      p.num_routes = static_cast<int>(routes);
      p.top_k = 1;
      p.out = ybuf;
      p.out_dtype = MXFP4_DTYPE_BF16;
      p.topk_w = topk_weights;
      p.w_dtype = w_dtype;
      p.mul_w = 1;
      p.c_stride_t = hidden;
      p.c_stride_j = 0;
      if (int rc = launch_routed<EPI_MOE, false>(tw, tx16, tx128, p, info.sms, s)) return rc;
    }
  }
  const int64_t vecs = num_tokens * (hidden / 8);
  const int grid = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, int64_t(info.sms) * 8));
  combine_topk_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(ybuf),
                                           static_cast<__nv_bfloat16*>(out), num_tokens, top_k, hidden, topk_ids,
                                           ids_dtype, num_experts);
  MX_CUDA(cudaGetLastError());
  return MXFP4_OK;
}


// ---------------------------------------------------------------------------
// Expert-parallel MoE layer (csrc/ep.cuh).
// ---------------------------------------------------------------------------
}  // extern "C"

namespace {
// Route chunks of an owner's received rows (all E experts bound the local ones).
int64_t ep_max_chunks(int64_t recv_capacity, int num_experts) {
  return recv_capacity / kEpChunkRows + num_experts + 1;
}
// Padding block of the owners' received rows, the same on every rank: the
// capacity from mxfp4_ep_moe_recv_capacity is at least 383 rows per local
// expert exactly when it was sized for 256-row blocks (>= 128 routes per
// local expert on average, the CTA-pair GEMM), and below that for 32-row
// blocks (the routed tensor-memory GEMM).
int ep_block_rows(int64_t recv_capacity, int el) {
  return recv_capacity >= static_cast<int64_t>(kPairRoutesPerExpert + kEpPairBlock - 1) * el ? kEpPairBlock : kEpBlock;
}

// The owner's two GEMMs on the CTA-pair kernel over 256-row blocks of the
// received rows (routed order, row ids = rows, pads = cap).
int ep_owner_pair_gemms(const void* xrow, const void* w13, const void* w13_scale, const void* w2, const void* w2_scale,
                        void* hbuf, void* yrow, const void* wrow, const int32_t* rid, const int32_t* block_expert,
                        const int32_t* post, int64_t cap, int cap_blocks, int el, int64_t hidden, int64_t inter, int sms,
                        cudaStream_t s) {
  {
    CUtensorMap ta, tb;
    if (int rc = make_map_2d(&ta, xrow, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hidden, cap, hidden * 2, kP2BK,
                             kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = make_map_2d(&tb, w13, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, hidden / 2,
                             static_cast<uint64_t>(el) * 2 * inter, hidden / 2, kP2BK / 2, kP2HalfRows,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    PairParams p{};
    p.N = static_cast<int>(2 * inter);
    p.K = static_cast<int>(hidden);
    p.bn = 256;
    p.num_m_blocks = cap_blocks;
    p.num_n_blocks = static_cast<int>((inter + p.bn / 2 - 1) / (p.bn / 2));
    p.w_scales = static_cast<const uint8_t*>(w13_scale);
    p.lds = hidden / 32;
    p.w_rows_per_expert = 2 * inter;
    p.glu_inter = static_cast<int>(inter);
    p.sorted_ids = rid;
    p.block_expert = block_expert;
    p.num_post_padded = post;
    p.num_routes = static_cast<int>(cap);
    p.top_k = 1;
    p.out = hbuf;
    p.ldo = inter;
    p.out_dtype = MXFP4_DTYPE_BF16;
    p.vec_ok = 1;
    if (int rc = routed_pair_gemm<A_TMA, EPI_GLU>(false, ta, tb, p, sms, s)) return rc;
  }
  CUtensorMap ta, tb;
  if (int rc = make_map_2d(&ta, hbuf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inter, cap, inter * 2, kP2BK, kP2HalfRows,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = make_map_2d(&tb, w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inter / 2, static_cast<uint64_t>(el) * hidden,
                           inter / 2, kP2BK / 2, kP2HalfRows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  PairParams p{};
  p.N = static_cast<int>(hidden);
  p.K = static_cast<int>(inter);
  p.bn = 256;
  p.num_m_blocks = cap_blocks;
  p.num_n_blocks = static_cast<int>((hidden + p.bn - 1) / p.bn);
  p.w_scales = static_cast<const uint8_t*>(w2_scale);
  p.lds = inter / 32;
  p.w_rows_per_expert = hidden;
  p.sorted_ids = rid;
  p.block_expert = block_expert;
  p.num_post_padded = post;
  p.num_routes = static_cast<int>(cap);
  p.top_k = 1;
  p.out = yrow;
  p.out_dtype = MXFP4_DTYPE_BF16;
  p.topk_w = wrow;
  p.w_dtype = MXFP4_DTYPE_F32;
  p.mul_w = 1;
  p.c_stride_t = hidden;
  p.c_stride_j = 0;
  p.vec_ok = 1;
  return routed_pair_gemm<A_TMA, EPI_MOE>(false, ta, tb, p, sms, s);
}

}  // namespace

extern "C" {

int64_t mxfp4_ep_moe_recv_capacity(int64_t max_tokens_per_rank, int top_k, int num_experts, int world) {
  if (max_tokens_per_rank < 0 || top_k <= 0 || num_experts <= 0 || world <= 0 || num_experts % world) return 0;
  const int64_t el = num_experts / world;
  const int64_t routes = static_cast<int64_t>(world) * max_tokens_per_rank * top_k;
  const int blk = routes >= kPairRoutesPerExpert * el ? kEpPairBlock : kEpBlock;
  const int64_t rows = routes + el * (blk - 1);
  return (rows + blk - 1) / blk * blk;
}

size_t mxfp4_ep_moe_workspace_size(int64_t num_tokens, int top_k, int num_experts, int64_t inter,
                                   int64_t recv_capacity) {
  const int64_t routes = num_tokens * top_k;
  size_t b = 0;
  b += align_up(sizeof(int32_t) * num_experts, 256) * 2;                  // send_base, lstart
  b += align_up(sizeof(int32_t) * (recv_capacity / kEpBlock + 1), 256);   // owner block experts
  b += 256;                                                               // owner used rows
  b += align_up(sizeof(int4) * ep_max_chunks(recv_capacity, num_experts), 256);  // owner route chunks
  b += 256;                                                               // number of chunks
  b += align_up(sizeof(int32_t) * std::max<int64_t>(recv_capacity, 1), 256);  // owner row ids
  b += align_up(sizeof(int32_t) * std::max<int64_t>(routes, 1), 256) * 3; // sorted, expert per position, dst
  b += 256;                                                               // valid routes
  b += route_ws_bytes(routes, num_experts);
  b += align_up(static_cast<size_t>(recv_capacity) * inter * 2, 256);     // h
  return b;
}

int mxfp4_ep_moe_layer(const void* x, const void* w13, const void* w13_scale, const void* w2, const void* w2_scale,
                       const void* topk_weights, int w_dtype, const void* topk_ids, int ids_dtype, void* out,
                       int64_t num_tokens, int top_k, int num_experts, int64_t hidden, int64_t inter, int rank,
                       int world, void* const* counts, void* const* xr, void* const* wr, void* const* yr,
                       int64_t recv_capacity, int32_t* const* flags, int32_t* counter, void* workspace,
                       size_t workspace_bytes, void* stream) {
  DevInfo info;
  if (int rc = current_device_info(info)) return rc;
  // a rank with no tokens still takes part (it owns experts and meets the
  // barriers): its token-side pointers may be null then
  MX_CHECK(w13 && w13_scale && w2 && w2_scale, "null pointer");
  MX_CHECK(num_tokens == 0 || (x && topk_weights && topk_ids && out), "null pointer");
  MX_CHECK(counts && xr && wr && yr && flags && counter, "null peer table");
  MX_CHECK(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world, "bad rank/world");
  MX_CHECK(num_experts > 0 && num_experts <= kMaxExperts && num_experts % world == 0,
           "num_experts must be in [1, 1024] and divide over the ranks");
  MX_CHECK(hidden > 0 && hidden % 128 == 0 && inter > 0 && inter % 128 == 0, "hidden/inter must be multiples of 128");
  MX_CHECK(num_tokens >= 0 && top_k > 0, "bad num_tokens/top_k");
  MX_CHECK(w_dtype == MXFP4_DTYPE_F32 || w_dtype == MXFP4_DTYPE_BF16 || w_dtype == MXFP4_DTYPE_F16,
           "topk_weights must be F32, BF16 or F16");
  MX_CHECK(ids_dtype == MXFP4_DTYPE_I32 || ids_dtype == MXFP4_DTYPE_I64, "topk_ids must be I32 or I64");
  MX_CHECK(aligned(x, 16) && aligned(out, 16), "x and out must be 16-byte aligned");
  const int blk = ep_block_rows(recv_capacity, num_experts / world);
  MX_CHECK(recv_capacity > 0 && recv_capacity % blk == 0 && recv_capacity < (int64_t(1) << 24),
           "recv_capacity must be a positive multiple of 32 (of 256 from 383 rows per local expert) below 2^24");
  const int64_t routes = num_tokens * top_k;
  MX_CHECK(static_cast<int64_t>(world) * routes + (num_experts / world) * (blk - 1) <= recv_capacity ||
               routes == 0,
           "recv_capacity too small for this many routes");
  const size_t need = mxfp4_ep_moe_workspace_size(num_tokens, top_k, num_experts, inter, recv_capacity);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MXFP4_ERR_WORKSPACE, "EP MoE layer needs " + std::to_string(need) + " workspace bytes");
  EpPeers pc{}, px{}, pw{}, py{};
  PeerFlags pf{};
  for (int j = 0; j < world; ++j) {
    MX_CHECK(counts[j] && xr[j] && wr[j] && yr[j] && flags[j], "null peer buffer");
    MX_CHECK(aligned(xr[j], 16) && aligned(yr[j], 16), "peer row buffers must be 16-byte aligned");
    pc.p[j] = counts[j];
    px.p[j] = xr[j];
    pw.p[j] = wr[j];
    py.p[j] = yr[j];
    pf.f[j] = flags[j];
  }
  cudaStream_t s = as_stream(stream);
  const int el = num_experts / world;
  const int64_t cap = recv_capacity;
  const int cap_blocks = static_cast<int>(cap / blk);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto take = [&](size_t bytes) {
    uint8_t* q = ws;
    ws += align_up(bytes, 256);
    return q;
  };
  int32_t* send_base = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * num_experts));
  int32_t* lstart = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * num_experts));
  int32_t* block_expert = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (cap_blocks + 1)));
  int32_t* post = reinterpret_cast<int32_t*>(take(256));
  const int64_t max_chunks = ep_max_chunks(cap, num_experts);
  int4* chunks = reinterpret_cast<int4*>(take(sizeof(int4) * max_chunks));
  int32_t* nchunks = reinterpret_cast<int32_t*>(take(256));
  int32_t* rid = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * cap));
  int32_t* sorted = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(routes, 1)));
  int32_t* bexp = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(routes, 1)));
  int32_t* dst = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(routes, 1)));
  int32_t* nvalid = reinterpret_cast<int32_t*>(take(256));
  uint8_t* route_ws = take(route_ws_bytes(routes, num_experts));
  void* hbuf = take(static_cast<size_t>(cap) * inter * 2);

  // 1. counts -> every rank; barrier
  ep_count_kernel<<<1, 1024, 0, s>>>(topk_ids, ids_dtype, routes, num_experts, rank, world, pc);
  MX_CUDA(cudaGetLastError());
  peer_barrier_kernel<<<1, 32, 0, s>>>(pf, rank, world, counter);
  MX_CUDA(cudaGetLastError());
  // 2. plan + stable local order; dispatch rows into the owners' xr; barrier
  ep_plan_kernel<<<1, 1024, 0, s>>>(static_cast<const int32_t*>(counts[rank]), num_experts, world, rank, send_base,
                                    lstart, block_expert, post, rid, static_cast<int>(cap), cap_blocks, chunks, nchunks,
                                    blk);
  MX_CUDA(cudaGetLastError());
  if (routes > 0) {
    if (int rc = run_route(topk_ids, ids_dtype, routes, num_experts, 0, 1, sorted, bexp, nvalid, routes, route_ws, s))
      return rc;
    MX_CUDA(cudaMemsetAsync(dst, 0xFF, sizeof(int32_t) * routes, s));
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((routes + 7) / 8, int64_t(info.sms) * 16)));
    ep_dispatch_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(x), hidden / 8, sorted, bexp, nvalid, send_base,
                                            lstart, topk_weights, w_dtype, top_k, el, px, pw, dst);
    MX_CUDA(cudaGetLastError());
  }
  peer_barrier_kernel<<<1, 32, 0, s>>>(pf, rank, world, counter);
  MX_CUDA(cudaGetLastError());
  // 3. owner: gate_up (fused SiLU * up) and down (route weight) over the received rows
  if (blk == kEpPairBlock) {
    if (int rc = ep_owner_pair_gemms(xr[rank], w13, w13_scale, w2, w2_scale, hbuf, yr[rank], wr[rank], rid,
                                     block_expert, post, cap, cap_blocks, el, hidden, inter, info.sms, s))
      return rc;
  } else {
  {
    CUtensorMap tw, tx16, tx128;
    if (int rc = routed_maps(&tw, &tx16, &tx128, w13, static_cast<int64_t>(el) * 2 * inter, hidden, xr[rank], cap,
                             hidden, false, true))
      return rc;
    RoutedParams p{};
    p.pgroup = routed_pgroup(hidden);
    p.N = static_cast<int>(2 * inter);
    p.glu_inter = static_cast<int>(inter);
    p.K = static_cast<int>(hidden);
    p.num_wblocks = static_cast<int>((inter + 127) / 128);
    p.w_scales = static_cast<const uint8_t*>(w13_scale);
    p.lds = hidden / 32;
    p.w_rows_per_expert = 2 * inter;
    p.chunks = chunks;
    p.num_chunks = nchunks;
    p.max_chunks = static_cast<int>(max_chunks);
    p.sorted_ids = rid;
    p.num_routes = static_cast<int>(cap);
    p.top_k = 1;
    p.out = hbuf;
    p.ldo = inter;
    p.out_dtype = MXFP4_DTYPE_BF16;
    if (int rc = launch_routed<EPI_GLU, false>(tw, tx16, tx128, p, info.sms, s)) return rc;
  }
  {
    CUtensorMap tw, tx16, tx128;
    if (int rc = routed_maps(&tw, &tx16, &tx128, w2, static_cast<int64_t>(el) * hidden, inter, hbuf, cap, inter, false,
                             false))
      return rc;
    RoutedParams p{};
    p.pgroup = routed_pgroup(inter);
    p.N = static_cast<int>(hidden);
    p.K = static_cast<int>(inter);
    p.num_wblocks = static_cast<int>((hidden + 255) / 256);
    p.w_scales = static_cast<const uint8_t*>(w2_scale);
    p.lds = inter / 32;
    p.w_rows_per_expert = hidden;
    p.chunks = chunks;
    p.num_chunks = nchunks;
    p.max_chunks = static_cast<int>(max_chunks);
    p.sorted_ids = rid;
    p.num_routes = static_cast<int>(cap);
    p.top_k = 1;
    p.out = yr[rank];
    p.out_dtype = MXFP4_DTYPE_BF16;
    p.topk_w = wr[rank];
    p.w_dtype = MXFP4_DTYPE_F32;
    p.mul_w = 1;
    p.c_stride_t = hidden;
    p.c_stride_j = 0;
    if (int rc = launch_routed<EPI_MOE, false>(tw, tx16, tx128, p, info.sms, s)) return rc;
  }
  }
  peer_barrier_kernel<<<1, 32, 0, s>>>(pf, rank, world, counter);
  MX_CUDA(cudaGetLastError());
  // 4. combine: pull the token's rows back from their owners
  if (num_tokens > 0) {
    const int64_t total = num_tokens * (hidden / 8);
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, int64_t(info.sms) * 8)));
    ep_combine_kernel<<<grid, 256, 0, s>>>(dst, py, static_cast<__nv_bfloat16*>(out), num_tokens, top_k, hidden);
    MX_CUDA(cudaGetLastError());
  }
  return MXFP4_OK;
}

}  // extern "C"
