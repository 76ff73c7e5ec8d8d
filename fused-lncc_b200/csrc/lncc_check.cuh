// Range checks of the bounds-checked build (LNCC_CHECKED=1, `build.py --checked`), the stand-in on this
// platform for the reference's compute-sanitizer runs (reference tests/_sanitize2.py,
// tests/_sanitize_bf16.py). Every global and shared-memory access of the kernels names its element
// or byte range; in a checked build a range outside its array increments a device counter and the
// access is skipped (a load reads zero), so a bad index is reported without a trap. The host entry
// points of a checked build synchronise after their launches and return LNCC_ERR_CHECK when the
// counter grew. In the normal build every check is `true` and compiles away.
#pragma once

#include <stdint.h>

namespace lncc {

#ifdef LNCC_CHECKED
__device__ unsigned long long g_check_violations;

// [i, i + len) within [0, n)
__device__ __forceinline__ bool check_range(int64_t i, int64_t len, int64_t n) {
  const bool ok = i >= 0 && len >= 0 && i + len <= n;
  if (!ok) atomicAdd(&g_check_violations, 1ull);
  return ok;
}
// a shared-memory byte range [addr, addr + bytes) within the block's dynamic shared memory
__device__ __forceinline__ bool check_smem(uint32_t addr, uint32_t bytes, uint32_t base, uint32_t size) {
  const bool ok = addr >= base && addr + bytes <= base + size;
  if (!ok) atomicAdd(&g_check_violations, 1ull);
  return ok;
}
// the block's dynamic shared memory window (every kernel here keeps its buffers there)
__device__ __forceinline__ uint32_t dyn_smem_base() {
  extern __shared__ unsigned char lncc_dyn_smem[];
  return static_cast<uint32_t>(__cvta_generic_to_shared(lncc_dyn_smem));
}
__device__ __forceinline__ uint32_t dyn_smem_size() {
  uint32_t n;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(n));
  return n;
}
#define LNCC_IN(i, len, n) (::lncc::check_range(int64_t(i), int64_t(len), int64_t(n)))
// shared byte address (32-bit) or a generic pointer into shared memory
#define LNCC_IN_SMEM(addr, bytes) \
  (::lncc::check_smem(uint32_t(addr), uint32_t(bytes), ::lncc::dyn_smem_base(), ::lncc::dyn_smem_size()))
#define LNCC_IN_SMEM_PTR(ptr, bytes) \
  LNCC_IN_SMEM(static_cast<uint32_t>(__cvta_generic_to_shared(ptr)), bytes)
#else
#define LNCC_IN(i, len, n) true
#define LNCC_IN_SMEM(addr, bytes) true
#define LNCC_IN_SMEM_PTR(ptr, bytes) true
#endif

}  // namespace lncc
