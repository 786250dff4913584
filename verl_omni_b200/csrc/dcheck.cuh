// Optional device-side range checks for the sm_100a kernels of verl_omni_b200 (no torch dependency).
#pragma once

#include <cuda_runtime.h>

// Optional device-side checks (build with VO_DEVICE_CHECKS=1 in the environment; compiled out otherwise).
// VO_DCHECK(cond) evaluates to cond: a false check records the first failing source line of its file in a
// device word of that file, and the caller skips the guarded access (nothing traps, the context stays
// usable).  The host reads and clears the records with ext.device_check_status().
namespace vo {
using DcheckReader = unsigned long long (*)(bool reset);
void dcheck_register(const char* file, DcheckReader fn);
}  // namespace vo

#ifdef VO_DEVICE_CHECKS
static __device__ unsigned long long vo_dcheck_site_;  // one per source file (static linkage)
static unsigned long long vo_dcheck_read_(bool reset) {
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, vo_dcheck_site_, sizeof(v)) != cudaSuccess) return ~0ull;
  if (reset && v) {
    const unsigned long long z = 0;
    cudaMemcpyToSymbol(vo_dcheck_site_, &z, sizeof(z));
  }
  return v;
}
namespace {
struct VoDcheckRegistration {
  VoDcheckRegistration() { vo::dcheck_register(__BASE_FILE__, &vo_dcheck_read_); }
};
static VoDcheckRegistration vo_dcheck_registration_;
}  // namespace
__device__ __forceinline__ bool vo_dcheck_(bool ok, unsigned line) {
  if (!ok) atomicCAS(&vo_dcheck_site_, 0ull, (unsigned long long)line);
  return ok;
}
#define VO_DCHECK(cond) vo_dcheck_(static_cast<bool>(cond), __LINE__)
#else
#define VO_DCHECK(cond) (static_cast<bool>(cond))
#endif
