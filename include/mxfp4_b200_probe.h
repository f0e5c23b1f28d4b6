/*
 * mxfp4_b200_probe.h -- C ABI of libmxfp4_b200_probe.so, the measurement probe
 * that gives the benchmark its tensor-core denominators on this machine.  It
 * is not part of the operator boundary and has no counterpart in the
 * reference.
 *
 * mxfp4_probe_mma_rate issues tcgen05 MMAs back to back from one thread per
 * CTA, one CTA per SM, on operands that stay in shared memory (no loads from
 * global memory in the timed loop), and reports the dense rate:
 *   kind MXFP4_PROBE_BF16: tcgen05.mma.cta_group::1.kind::f16, BF16 x BF16,
 *                          M = 128, N = 256, K = 16 per instruction;
 *   kind MXFP4_PROBE_MXF4: tcgen05.mma.cta_group::1.kind::mxf4.block_scale
 *                          .block32, E2M1 x E2M1 with UE8M0 scales from tensor
 *                          memory, M = 128, N = 256, K = 64 per instruction.
 * Every CTA issues `iters` x 4 instructions into one FP32 accumulator.  The
 * call synchronises the host (it times itself with CUDA events on `stream`)
 * and writes the elapsed milliseconds and the FLOPs executed (2*M*N*K per
 * instruction).  The only wait in the kernel is bounded.
 */
#ifndef MXFP4_B200_PROBE_H_
#define MXFP4_B200_PROBE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXFP4_PROBE_BF16 0
#define MXFP4_PROBE_MXF4 1

int mxfp4_probe_mma_rate(int kind, int iters, float* ms, double* flops, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXFP4_B200_PROBE_H_ */
