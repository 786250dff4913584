// Allocation-free entry point of the fused reverse-SDE step.
//
// This entry point has no counterpart in the reference (verl-omni ships no native code); it exists for
// callers of this library that cannot allocate device memory: code running inside a custom allocator's
// callback (allocating there would re-enter the allocator), embedders that own a fixed memory budget and
// forbid cudaMalloc after start-up, and plain C hosts without a PyTorch caching allocator.  The caller
// passes every input and output; the per-block partial sums the kernel needs live in a fixed
// file-scope device array in sde.cu (VO_SDE_NOALLOC_MAX_PARTIALS floats, held by every GPU that
// loads the library until the process exits).
//
// Contract:
//   * all pointers are device pointers to contiguous fp32 data; x, v, mean_out, prev_out (and the
//     optional prev_in / noise) hold B * n floats; sigma, sigma_prev, logp_out, std_out hold B floats;
//   * prev_in != NULL: use it as the sample; prev_out may then be NULL, equal to prev_in, or a distinct
//     buffer, which receives a copy of prev_in (one device-to-device copy on `stream`).  Else
//     noise != NULL: prev = mean + scale * noise; else noise is drawn from Philox keyed by
//     (seed, row, offset);
//   * sde_type: 0 = sde, 1 = cps, 2 = dance_sde; want_logp / norm as in the allocating version;
//   * the first call on a device looks up the scratch array's device address (cudaGetSymbolAddress)
//     with that device current -- make that first call before any stream capture; the set-up is
//     guarded, so threads making their first calls at the same time are safe;
//   * the scratch array is shared by every call on a device and keeps the last call's contents;
//     every slot a call reads is written earlier in the same call, so nothing needs clearing, but
//     calls that overlap on the GPU (different streams, no ordering) race on it;
//   * returns 0 on success, -1 for bad arguments, -2 when B exceeds 65535 (one grid row per sample)
//     or B * (number of chunks) exceeds VO_SDE_NOALLOC_MAX_PARTIALS (the problem is too large for the
//     fixed scratch), otherwise a cudaError_t value.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define VO_SDE_NOALLOC_MAX_PARTIALS 65536

#ifdef __cplusplus
extern "C" {
#endif

int vo_sde_step_fwd_noalloc(const float* x, const float* v, const float* sigma, const float* sigma_prev,
                            const float* prev_in, const float* noise, float* prev_out, float* mean_out,
                            float* logp_out, float* std_out, int B, int64_t n, float sigma_max, float eta,
                            int sde_type, uint64_t seed, uint32_t offset, int want_logp, int norm,
                            cudaStream_t stream);

#ifdef __cplusplus
}
#endif
