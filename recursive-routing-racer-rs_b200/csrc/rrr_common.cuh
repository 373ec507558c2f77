// rrr_common.cuh — device helpers shared by the sm_100a kernels: bounded mbarrier waits,
// 1-D bulk copies (cp.async.bulk, no multicast), programmatic dependent launch controls,
// and the kernel error flag. Only sm_100a is targeted.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rrr_cuda.h"
#include "internal.h"

namespace rrr {

// Codes a kernel writes into the context's device error flag (rrr_check_device_error).
enum DeviceErr : int {
  kDevErrNone = 0,
  kDevErrFullTimeout = 1,   // a consumer gave up waiting for a bulk copy
  kDevErrEmptyTimeout = 2,  // the producer gave up waiting for consumers to free a stage
  kDevErrDrainTimeout = 3,  // copies still in flight at exit did not complete in time
  kDevErrCommTimeout = 5,   // an exchange gave up waiting for a peer rank's data
  kDevErrPosition = 6,      // a position outside the cache, or a token id outside the table
};

// A wait gives up after this many nanoseconds of %globaltimer (about one second) unless the
// context sets another limit (rrr_set_wait_limit); it then records an error and lets the
// kernel return instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
__device__ __forceinline__ uint64_t wait_limit_ns(const int* err) {
  if (!err) return kWaitLimitNs;
  const uint64_t v = *reinterpret_cast<const volatile unsigned long long*>(err + kWaitLimitSlot);
  return v ? v : kWaitLimitNs;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Tagged exchange words between ranks (peer memory over NVLink): value bits low, epoch of the
// step or call that stored them high. A naturally aligned 64-bit access is single-copy
// atomic, so a reader that sees the epoch sees the value stored with it: no fences, no
// separate flags. A vector access is a set of such 64-bit accesses.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ld_relaxed_sys_v2_u64(const unsigned long long* p,
                                                      unsigned long long& a,
                                                      unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Word p once its epoch is e (w: a value already loaded from p). Gives up after the
// context's wait limit: records kDevErrCommTimeout, clears ok and returns what it last read;
// once ok is false the caller's later words are not waited for.
__device__ __forceinline__ unsigned long long wait_tagged(const unsigned long long* p,
                                                          unsigned long long w, unsigned e,
                                                          bool& ok, int* err) {
  if ((unsigned)(w >> 32) == e || !ok) return w;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(err);
  for (int i = 0;; ++i) {
    w = ld_relaxed_sys_u64(p);
    if ((unsigned)(w >> 32) == e) return w;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > limit) {
      if (err) atomicCAS(err, 0, (int)kDevErrCommTimeout);
      ok = false;
      return w;
    }
  }
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
          smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep in hardware (up to hint_ns)
// until the phase completes instead of spinning on the issue slots.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete. Gives up after the context's wait limit
// (wait_limit_ns) times `limit_scale`: records `code` in *err (first error wins) and returns
// false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  int code, uint32_t limit_scale = 1) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(err) * limit_scale;
  while (true) {
    if (mbar_try_wait_hint(bar, parity, 100000u)) return true;
    if (globaltimer_ns() - t0 > limit) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared, completion counted in bytes on `bar`. dst, src and
// bytes must be multiples of 16. Plain (non-multicast) form: the source is always this
// GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Prefetch of a global range into L2 (no destination, no completion tracking). src and
// bytes must be multiples of 16. Prefetching lines that another grid is still writing is
// harmless: L2 stays coherent with those writes.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory to be visible /
// allow the next grid to start launching. No-ops when not launched with PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
  float f;
  asm("{ .reg .f16 h; mov.b16 h, %1; cvt.f32.f16 %0, h; }" : "=f"(f) : "h"((uint16_t)bits16));
  return f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace rrr

// Host-side launch helper: launch `kernel` with programmatic stream serialisation enabled
// (so the kernel may start while the previous one on the stream drains).
template <typename... KArgs, typename... Args>
static inline cudaError_t rrr_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                         size_t smem, cudaStream_t stream, bool pdl,
                                         Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
