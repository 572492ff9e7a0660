/* probes.h - measurements of the B200 features the GEMM kernels are built around, and checks of the packed arithmetic
 * the encoder's row kernels use (libphonon2_probes.so, built beside the product library and loaded only by the bench's
 * probe workload, its large-M fractions and the tests). Each returns 0, or a negative code with a message in
 * p2cu_probes_last_error(). */
#ifndef P2_PROBES_H
#define P2_PROBES_H

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define P2PROBE_API __attribute__((visibility("default")))
#else
#define P2PROBE_API
#endif

P2PROBE_API const char *p2cu_probes_last_error(void);
/* The tcgen05 int8 MMA rate in MACs per second over all SMs, from shared-memory operands, one CTA per SM (pair = 0,
 * M = 128 per MMA) or on CTA pairs (pair != 0, M = 256); iters K = 128 steps per SM. */
P2PROBE_API int p2cu_probe_int8_mma(int pair, int iters, double *macs_per_s);
/* Tiled TMA load bytes per second per SM from an L2-resident matrix, boxes of box_rows 128-byte rows (8-256) issued by
 * `warps` warps (1-4) of each CTA, two boxes in flight per warp. */
P2PROBE_API int p2cu_probe_tma_load(int warps, int box_rows, double *bytes_per_s_per_sm);
/* The CTA-pair MMA stream (iters K = 128 steps per pair) over a ring of six 32 KB stages handed back through barriers
 * as in the pair GEMM, without copies: mode 0 no hand-back after the first round, mode 1 through a producer arrive and
 * the odd CTA's relay, mode 2 with the odd CTA arriving on the even CTA's barrier. */
P2PROBE_API int p2cu_probe_int8_ring(int mode, int iters, double *macs_per_s);
/* The encoder's packed fp32x2 arithmetic (numerics.cuh) against the scalar forms it replaces, bit for bit over every
 * input: mismatches[0] exp_poly against the rintf form, [1] exp_poly2, [2] swish2, [3] the packed FMA on hashed
 * operands, [4] rcp2_ge1 against __frcp_rn over [1, 2^126). All five are 0 on a correct build. */
P2PROBE_API int p2cu_probe_packed_math(unsigned long long *mismatches);

#ifdef __cplusplus
}
#endif

#endif /* P2_PROBES_H */
