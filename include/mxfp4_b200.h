/*
 * mxfp4_b200.h -- C ABI of libmxfp4_b200.so, the B200 (sm_100a) MXFP4 backend.
 *
 * This is the drop-in boundary for the operator surface of
 * lutianshu824/mxfp4-gfx936 (file "src/aiter/ops/triton/moe_op_mxfp4_soft.py",
 * cited below as soft:LINE, and the vLLM adapter
 * "integration/vllm/vllm_mxfp4_gfx936.py", cited as vllm:LINE).  The Python
 * operator module binds these symbols with ctypes; any other FFI can bind them
 * the same way.
 *
 * Conventions shared by every entry point:
 *  - All tensor arguments are device pointers owned by the caller; the library
 *    allocates no memory on the compute path.  Scratch space is passed as
 *    `workspace` and sized by the matching *_workspace_size() query.
 *  - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL is the
 *    legacy default stream) and runs asynchronously; no entry point
 *    synchronises the host on the compute path.
 *  - Matrices are row-major with an explicit leading dimension in ELEMENTS
 *    (bytes for uint8 tensors).  Packed MXFP4 holds two E2M1 codes per byte,
 *    the low nibble is the even K index; E8M0 scales are uint8, one per 32
 *    values along K, row-major [rows, K/32] (the swizzled AITER scale layout is
 *    rejected, soft:398-399).
 *  - Return value: MXFP4_OK or an MXFP4_ERR_* code; mxfp4_last_error() gives a
 *    message for the calling thread.  Nothing aborts or prints.
 */
#ifndef MXFP4_B200_H_
#define MXFP4_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXFP4_B200_ABI_VERSION 1

/* status codes */
#define MXFP4_OK 0
#define MXFP4_ERR_INVALID_ARGUMENT 1   /* bad shape, stride, alignment or null pointer */
#define MXFP4_ERR_UNSUPPORTED_DEVICE 2 /* not an sm_100 device */
#define MXFP4_ERR_CUDA 3               /* a CUDA runtime / driver call failed */
#define MXFP4_ERR_TIMEOUT 4            /* a device-side bounded wait expired */
#define MXFP4_ERR_WORKSPACE 5          /* workspace missing or too small */
#define MXFP4_ERR_UNSUPPORTED 6        /* valid request this backend does not implement */

/* element types */
#define MXFP4_DTYPE_F32 0
#define MXFP4_DTYPE_BF16 1
#define MXFP4_DTYPE_F16 2
#define MXFP4_DTYPE_U8 3
#define MXFP4_DTYPE_I32 4
#define MXFP4_DTYPE_I64 5

/* dense W4A16 execution modes (explicit backend selection, soft:45-49) */
#define MXFP4_LINEAR_FUSED 0 /* decode inside the GEMM producer (replaces soft:176-274) */
#define MXFP4_LINEAR_SAFE 1  /* explicit dequant into workspace, then the same GEMM (soft:371-373) */

/* Library ABI version (MXFP4_B200_ABI_VERSION). */
int mxfp4_abi_version(void);

/* Message for the last failing call made by this thread ("" if none). */
const char* mxfp4_last_error(void);

/* 1 if `device` is an sm_100 GPU this library can run on, else 0. */
int mxfp4_device_supported(int device);

/* Device status word written by kernels (MXFP4_OK or the first error code a
 * kernel recorded, e.g. MXFP4_ERR_TIMEOUT).  Synchronises `device`.  With
 * clear != 0 the word is reset to MXFP4_OK afterwards. */
int mxfp4_device_status(int device, int clear);

/* ------------------------------------------------------------------------ */
/* K0 -- dequantisation.  Replaces dequant_mxfp4 (soft:277-307).            */
/* out[r, k] = E2M1[code(r,k)] * 2^(scale(r, k/32) - 127), computed in FP32  */
/* and rounded to out_dtype (F32, BF16 or F16); scale code 255 gives NaN.    */
/* packed: [rows, k/2] u8 contiguous; scales: [rows, k/32] u8 contiguous;    */
/* out: [rows, k] contiguous.  k % 32 == 0.                                 */
int mxfp4_dequant(const void* packed, const void* scales, void* out, int out_dtype, int64_t rows,
                  int64_t k, void* stream);

/* ------------------------------------------------------------------------ */
/* K1 -- dense W4A16 linear.  Replaces linear_mxfp4_soft (soft:310-376),     */
/* including its Triton kernel (soft:176-274).                               */
/* out[m, n] = round(sum_k x[m,k] * W[n,k]) (+ bias[n], rounded again), with */
/* W = dequant(w_packed, w_scales) in x's dtype, FP32 accumulation in one    */
/* reduction per output.  x_dtype: BF16 or F16; out has x's dtype; bias is   */
/* NULL or a [n] vector of x's dtype.  k % 128 == 0.  ldx/ldo in elements,   */
/* ldw/lds in bytes (>= k/2, >= k/32).                                       */
size_t mxfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int x_dtype, int mode);
int mxfp4_linear_w4a16(const void* x, int x_dtype, int64_t ldx, const void* w_packed, int64_t ldw,
                       const void* w_scales, int64_t lds, const void* bias, void* out, int64_t ldo,
                       int64_t m, int64_t n, int64_t k, int mode, void* workspace,
                       size_t workspace_bytes, void* stream);

/* The matmul half of the safe path (soft:372-373) on weights already       */
/* decoded by mxfp4_dequant: out = round(x . w_deq^T) (+ bias), w_deq [n, k] */
/* in x's dtype with row pitch ldw ELEMENTS (16-byte aligned).  The same    */
/* kernels and summation order as mxfp4_linear_w4a16, so a dequant followed */
/* by this call gives that call's bits; it is also the second launch of a  */
/* decode-once fused linear, timed on its own by the benchmark.  No         */
/* workspace.                                                               */
int mxfp4_linear_dequantized(const void* x, int x_dtype, int64_t ldx, const void* w_deq, int64_t ldw,
                             const void* bias, void* out, int64_t ldo, int64_t m, int64_t n, int64_t k,
                             void* stream);

/* ------------------------------------------------------------------------ */
/* Quantizer -- BF16/F32 -> packed MXFP4 + E8M0 (the W4A4 configuration's   */
/* OCP rounding; the reference only has a test quantizer, test:28-60).       */
/* Per 32 values: q = fl32(max|x| / 6), scale code = clamp(floor(log2 q) +  */
/* 127, 0, 254) (0 for an all-zero block), element = RNE(x * 2^(127-code))   */
/* on the E2M1 grid, ties to the even code, saturated at +-6, zero unsigned. */
/* x: [rows, k] with row stride ldx elements; packed [rows, k/2];            */
/* scales [rows, k/32].  k % 32 == 0.                                       */
int mxfp4_quantize(const void* x, int x_dtype, int64_t ldx, int64_t rows, int64_t k, void* packed,
                   void* scales, void* stream);

/* ------------------------------------------------------------------------ */
/* K2 -- W4A4 GEMM on the block-scaled tensor cores (tcgen05 kind::mxf4).  */
/* Replaces the packed-activation branch of soft:468-475 (dequant A, dequant */
/* B, one matmul) and the native dot_scaled kernel of aiter:304-338:         */
/* out[m, n] = round(sum_k deq(A)[m,k] * deq(B)[n,k]), FP32 accumulation.    */
/* a: [m, k/2] u8, a_scales [m, k/32]; b: [n, k/2] u8, b_scales [n, k/32]; */
/* out [m, n] (BF16, F16 or F32); all contiguous; k % 128 == 0.              */
size_t mxfp4_gemm_w4a4_workspace_size(int64_t m, int64_t n, int64_t k);
int mxfp4_gemm_w4a4(const void* a, const void* a_scales, const void* b, const void* b_scales, void* out,
                    int out_dtype, int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                    void* stream);

/* MoE router: for each of num_tokens tokens, softmax (FP32) over the          */
/* num_experts logits [num_tokens, num_experts] (F32, BF16 or F16, dense),     */
/* then the top_k largest probabilities in descending order (equal values:     */
/* the lower expert first), renormalised to sum to one when renormalize != 0. */
/* Writes topk_weights [num_tokens, top_k] (F32) and topk_ids (I32).  This is  */
/* the routing vLLM computes before calling the reference adapter's            */
/* _moe_apply (vllm:233), which receives it as topk_weights / topk_ids; the    */
/* reference module has no router.  num_experts <= 256, top_k <= 32.           */
int mxfp4_moe_router(const void* logits, int logits_dtype, int64_t num_tokens, int num_experts,
                     int top_k, int renormalize, float* topk_weights, int32_t* topk_ids,
                     void* stream);

/* ------------------------------------------------------------------------ */
/* K4 -- device routing.  Replaces _make_routing (vllm:119-146) without its  */
/* host sync.  Route r = t*top_k + j of topk_ids[num_tokens, top_k] (I32 or  */
/* I64) goes to local expert e = id - expert_offset when 0 <= e <           */
/* num_experts, else it is dropped.  Output: sorted_ids [capacity] (route   */
/* ids grouped by expert in ascending expert order, ascending route id      */
/* inside an expert, each expert padded to a multiple of block_m with the    */
/* value num_tokens*top_k), block_expert [capacity/block_m] (expert of each  */
/* block, -1 after the last used block) and num_post_padded [1] (used       */
/* length).  capacity = mxfp4_moe_route_capacity(...).                       */
int64_t mxfp4_moe_route_capacity(int64_t num_routes, int num_experts, int block_m);
size_t mxfp4_moe_route_workspace_size(int64_t num_routes, int num_experts);
int mxfp4_moe_route(const void* topk_ids, int ids_dtype, int64_t num_tokens, int top_k,
                    int num_experts, int expert_offset, int block_m, int32_t* sorted_ids,
                    int32_t* block_expert, int32_t* num_post_padded, int64_t capacity,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* K3 -- routed MoE op.  Replaces fused_moe_mxfp4_soft (soft:379-494) and     */
/* its Triton kernel (soft:65-173).                                          */
/* C[t, j, :] = round(round(round(A'[t] . W[e]^T) * a_scale) * b_scale[e])    */
/* (then * topk_weights[t, j] and rounded again if mul_routed_weight) for    */
/* e = topk_ids[t, j] in [0, num_experts); other routes leave C[t, j, :] = 0.*/
/* A' = A in C's dtype, or dequant(A, a_mx_scale) when a_dtype is U8 (W4A4,  */
/* soft:468-475).  Rounding is to c_dtype (F32, BF16 or F16).  With C F32    */
/* the products are those of an FP32 matmul (soft:405): A is split exactly   */
/* into BF16 parts (one for BF16 or U8 A, two for F16, three for F32), each  */
/* part times the exactly decoded weights, FP32 accumulation.               */
/* A: [num_tokens, k] (a_dtype BF16/F16/F32, or U8 packed [num_tokens, k/2]  */
/* with a_mx_scale [num_tokens, k/32]); B: [num_experts, n, k/2] u8;         */
/* B_mx: [num_experts, n, k/32] u8; a_scale: 1 FP32; b_scale: [num_experts]  */
/* FP32; topk_weights: [num_tokens, top_k] (w_dtype F32/BF16/F16); topk_ids: */
/* [num_tokens, top_k] I32/I64; C: [num_tokens, top_k, n] contiguous.        */
/* All contiguous; k % 128 == 0.                                             */
size_t mxfp4_fused_moe_workspace_size(int64_t num_tokens, int top_k, int num_experts, int64_t n,
                                      int64_t k, int a_dtype, int c_dtype);
int mxfp4_fused_moe(const void* A, int a_dtype, const void* a_mx_scale, const void* B,
                    const void* B_mx_scale, const float* a_scale, const float* b_scale,
                    const void* topk_weights, int w_dtype, const void* topk_ids, int ids_dtype,
                    void* C, int c_dtype, int64_t num_tokens, int top_k, int num_experts,
                    int64_t n, int64_t k, int mul_routed_weight, void* workspace,
                    size_t workspace_bytes, void* stream);

/* No counterpart in the reference.  mxfp4_fused_moe for callers that cannot  */
/* allocate device memory at call time -- e.g. a plugin host or graph        */
/* executor that owns every buffer after initialisation, or a fixed memory   */
/* plan replayed under stream capture -- and so cannot provide `workspace`.  */
/* Same arguments and result as mxfp4_fused_moe without the workspace: the  */
/* scratch comes from an 8 MiB static device array of the library (held on  */
/* every GPU that loads it until exit).  A request needing more scratch than */
/* that (mxfp4_fused_moe_workspace_size() > 8 MiB) returns                   */
/* MXFP4_ERR_WORKSPACE.  While the routed GEMV runs (up to 24 routes with  */
/* BF16 C, 64 otherwise) the scratch is only A converted to the operand     */
/* dtype, none for BF16 A and C; above that it holds the routing and A in   */
/* routed order (BF16 C: split into two E4M3 parts with their scales),      */
/* every expert padded to 32 rows.  With BF16 A and C, 128 experts and      */
/* top-8 it takes up to 7 tokens at K = 2048 and 112 at K = 768             */
/* (decode-sized calls); bigger calls go to mxfp4_fused_moe with a          */
/* workspace.  Bad                                                          */
/* sizes or dtypes return MXFP4_ERR_INVALID_ARGUMENT before any sizing.      */
/* The first call on a device looks up the array's                          */
/* device address, so make it before any stream capture.  All calls share    */
/* the array: calls that overlap on the GPU (other streams, other host       */
/* threads) race and must be serialised by the caller.                      */
int mxfp4_fused_moe_noalloc(const void* A, int a_dtype, const void* a_mx_scale, const void* B,
                            const void* B_mx_scale, const float* a_scale, const float* b_scale,
                            const void* topk_weights, int w_dtype, const void* topk_ids, int ids_dtype,
                            void* C, int c_dtype, int64_t num_tokens, int top_k, int num_experts,
                            int64_t n, int64_t k, int mul_routed_weight, void* stream);

/* ------------------------------------------------------------------------ */
/* K3+K5 -- MoE layer.  Replaces _moe_apply (vllm:233-265) with the W4A16    */
/* MXFP4 experts: gate_up = x . W13[e]^T (gate = first `inter` rows), h =    */
/* bf16(bf16(silu(gate)) * up), y_r = bf16(bf16(h . W2[e]^T) * w_r) per      */
/* route, out[t] = bf16(sum_j y_(t*top_k+j)) with FP32 accumulation.        */
/* x: [num_tokens, hidden] BF16; w13: [E, 2*inter, hidden/2] u8 + scales    */
/* [E, 2*inter, hidden/32]; w2: [E, hidden, inter/2] u8 + scales            */
/* [E, hidden, inter/32]; topk_weights F32/BF16/F16 and topk_ids I32/I64     */
/* [num_tokens, top_k]; out: [num_tokens, hidden] BF16.  hidden % 128 == 0, */
/* inter % 128 == 0.                                                        */
size_t mxfp4_moe_layer_workspace_size(int64_t num_tokens, int top_k, int num_experts,
                                      int64_t hidden, int64_t inter);
int mxfp4_moe_layer(const void* x, const void* w13, const void* w13_scale, const void* w2,
                    const void* w2_scale, const void* topk_weights, int w_dtype,
                    const void* topk_ids, int ids_dtype, void* out, int64_t num_tokens,
                    int top_k, int num_experts, int64_t hidden, int64_t inter, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU dense linear (column-sharded).  No counterpart in the          */
/* reference; replaces the shard GEMM + NCCL all-gather pair.               */
/* mxfp4_linear_w4a16 whose output block is also written, from the GEMM     */
/* epilogue, into the buffers of up to 7 other ranks on this node: `out` is */
/* this rank's [m, n] column block inside its full [m, n * world] output    */
/* (row stride ldo elements), peer_out[j] the same block inside rank j's    */
/* output, mapped into this process (CUDA IPC over NVLink).  A host array   */
/* of num_peers device pointers, 16-byte aligned for the vector stores.     */
/* Arguments otherwise as mxfp4_linear_w4a16.  The peers' buffers hold the  */
/* block once every rank has passed mxfp4_peer_barrier after this call.     */
int mxfp4_linear_w4a16_allgather(const void* x, int x_dtype, int64_t ldx, const void* w_packed,
                                 int64_t ldw, const void* w_scales, int64_t lds, const void* bias,
                                 void* out, void* const* peer_out, int num_peers, int64_t ldo,
                                 int64_t m, int64_t n, int64_t k, int mode, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* The same with an NVLink multicast mapping of all ranks' outputs (NVSwitch */
/* multicast object, e.g. the multicast address of a torch symmetric-memory */
/* buffer), offset to this rank's block like peer_out.  Each 16-byte chunk  */
/* is stored once through out_mc and NVSwitch writes it into every rank's   */
/* buffer, so this GPU sends its block once instead of once per peer;       */
/* peer_out (num_peers >= 1) is still used for rows whose width or stride   */
/* is not a multiple of 16 bytes.  No counterpart in the reference.         */
int mxfp4_linear_w4a16_allgather_mc(const void* x, int x_dtype, int64_t ldx, const void* w_packed,
                                    int64_t ldw, const void* w_scales, int64_t lds, const void* bias,
                                    void* out, void* const* peer_out, int num_peers, void* out_mc,
                                    int64_t ldo, int64_t m, int64_t n, int64_t k, int mode,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Peer-mapped buffers for the multi-GPU paths (CUDA IPC; one process per   */
/* GPU on one node).  mxfp4_ipc_alloc: zero-filled device allocation of the  */
/* current device and its 64-byte IPC handle (written to `handle`).         */
/* mxfp4_ipc_open: maps another process's allocation into the current       */
/* device's context with peer access enabled; mxfp4_ipc_close unmaps it,    */
/* mxfp4_ipc_free releases a local allocation once every peer closed it.   */
int mxfp4_ipc_alloc(size_t bytes, void** ptr, void* handle);
int mxfp4_ipc_open(const void* handle, void** ptr);
int mxfp4_ipc_close(void* ptr);
int mxfp4_ipc_free(void* ptr);

/* Device-side barrier of `world` ranks (one kernel, one warp).  flags: a    */
/* host array of `world` device pointers, flags[j] = rank j's int32 flag    */
/* array [world] mapped into this process (flags[rank] is the local one);   */
/* all flag arrays start at zero.  counter: a local device int32, zero     */
/* before the first call, advanced by one per call.  Orders this rank's     */
/* earlier stores (including stores into peers' memory) before the signal.  */
/* Every rank makes the same sequence of calls.  A wait longer than 2 s     */
/* records MXFP4_ERR_TIMEOUT in the device status word and returns.         */
int mxfp4_peer_barrier(int32_t* const* flags, int rank, int world, int32_t* counter, void* stream);

/* The same barrier with its wait limit given in microseconds (0: 2 s; at   */
/* most 60 s).  No counterpart in the reference.                            */
int mxfp4_peer_barrier_timed(int32_t* const* flags, int rank, int world, int32_t* counter,
                             int64_t timeout_us, void* stream);

/* After a barrier recorded MXFP4_ERR_TIMEOUT the ranks' epochs disagree:    */
/* this rank's counter advanced while a peer's signal is missing, so later  */
/* barriers could pass early or keep timing out.  Reset before reuse, on    */
/* every rank: wait until no barrier kernel of any rank is running (each    */
/* rank synchronises its device, then a host-side barrier of the group),    */
/* call this to zero the local flag array [world] and the counter, wait for */
/* it on every rank (synchronise, host barrier again), then resume.  No     */
/* counterpart in the reference.                                            */
int mxfp4_peer_barrier_reset(int32_t* local_flags, int world, int32_t* counter, void* stream);

/* ------------------------------------------------------------------------ */
/* Expert-parallel MoE layer.  No counterpart in the reference;             */
/* replaces the NCCL all-to-all dispatch / local layer / all-to-all combine  */
/* of an expert-parallel _moe_apply (vllm:233-265).  Rank `rank` of `world`  */
/* (one process per GPU, one node) holds experts [rank*E/world, ...) as      */
/* w13[E/world, 2*inter, hidden/2] (+ scales) and w2[E/world, hidden,        */
/* inter/2] (+ scales), and its own num_tokens tokens with their global      */
/* topk_ids; `out` receives the same [num_tokens, hidden] rows the           */
/* single-GPU mxfp4_moe_layer gives for them, bit for bit.                   */
/* Peer tables (host arrays of `world` device pointers, entry j = rank j's   */
/* buffer mapped into this process, e.g. with mxfp4_ipc_open): counts       */
/* [world * E] int32; xr [recv_capacity, hidden] BF16; wr [recv_capacity]   */
/* F32; yr [recv_capacity, hidden] BF16; flags/counter as for               */
/* mxfp4_peer_barrier.  recv_capacity = mxfp4_ep_moe_recv_capacity() of the */
/* largest num_tokens of any rank.  Every rank calls it together (three    */
/* device barriers inside); no host synchronisation.                        */
int64_t mxfp4_ep_moe_recv_capacity(int64_t max_tokens_per_rank, int top_k, int num_experts, int world);
size_t mxfp4_ep_moe_workspace_size(int64_t num_tokens, int top_k, int num_experts, int64_t inter,
                                   int64_t recv_capacity);
int mxfp4_ep_moe_layer(const void* x, const void* w13, const void* w13_scale, const void* w2,
                       const void* w2_scale, const void* topk_weights, int w_dtype,
                       const void* topk_ids, int ids_dtype, void* out, int64_t num_tokens,
                       int top_k, int num_experts, int64_t hidden, int64_t inter, int rank, int world,
                       void* const* counts, void* const* xr, void* const* wr, void* const* yr,
                       int64_t recv_capacity, int32_t* const* flags, int32_t* counter,
                       void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXFP4_B200_H_ */
