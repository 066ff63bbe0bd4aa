/*
 * probe.h -- exports of libnerf_b200_l2probe.so, the benchmark's L2
 * microbenchmarks (not part of the product library libnerf_b200.so, and
 * with no counterpart in the reference).  They give the L2 peaks the
 * hash-grid kernels are measured against.  Both launch asynchronously on
 * `stream`; the caller times them with events.
 * read: `passes` sweeps of 16-byte loads over `bytes` of `buf` (16-byte
 *       aligned; `sink` >= 1024 words, written only to keep loads live).
 * red:  reps f16x2 reductions per thread (vec 0: 4-byte form, 1: 8-byte
 *       .v2, 2: 16-byte .v4) at hashed word indices of `buf` (16-byte
 *       aligned, `words` a power of two >= 4); *ops receives the number of
 *       reduction instructions issued.
 * gather: reps loads per thread (vec 0: 4-byte, 1: 8-byte aligned pair) at
 *       hashed word indices of `buf` (same rules as red; `sink` as in read);
 *       *ops receives the number of loads issued.
 */
#ifndef NERF_B200_PROBE_H
#define NERF_B200_PROBE_H

#include <stdint.h>

#include "nerf.h"

#ifdef __cplusplus
extern "C" {
#endif

NERF_API NerfStatus nerf_b200_probe_l2_read(const void* buf, uint64_t bytes, uint32_t passes, uint32_t* sink, void* stream);
NERF_API NerfStatus nerf_b200_probe_l2_red(void* buf, uint32_t words, uint32_t reps, uint32_t vec, uint64_t* ops,
                                           void* stream);
NERF_API NerfStatus nerf_b200_probe_l2_gather(const void* buf, uint32_t words, uint32_t reps, uint32_t vec, uint32_t* sink,
                                              uint64_t* ops, void* stream);

#ifdef __cplusplus
}
#endif

#endif
