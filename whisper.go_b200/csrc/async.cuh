// async.cuh — mbarrier handshakes and TMA / bulk copies (sm_100a) shared by
// the tensor-core GEMM and the attention kernels.
//
// Every wait is bounded: after WAIT_LIMIT tries or WAIT_NS nanoseconds it
// raises the CTA's abort flag, records `code` in the kernel family's error
// word (read by the host after a step) and returns false, so a kernel whose
// copies never land still ends and frees what it holds.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace wg {

constexpr uint32_t WAIT_LIMIT = 1u << 22;     // tries of one bounded wait
constexpr uint64_t WAIT_NS = 2000000000ull;   // and at most 2 s
constexpr uint32_t SUSPEND_NS = 100000;       // suspend-time hint of one try

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp is parked by the
// hardware until the phase completes (or the hint elapses) instead of
// spinning, so waiting warps do not take issue slots from the working warps
// of their SM sub-partition.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(SUSPEND_NS)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: false (abort flag raised, code recorded in *err) once the
// limits pass, or when another warp of the CTA has aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int code, int* err,
                                          uint64_t limit_ns = WAIT_NS) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < WAIT_LIMIT; i++) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > limit_ns) break;
  }
  *abort = 1;
  atomicCAS(err, 0, code);
  return false;
}
// Bounded wait that ignores the abort flag: used after an abort to let the
// copies still in flight land before the CTA exits.
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < WAIT_LIMIT; i++) {
    if (mbar_try(bar, parity)) return true;
    if (global_ns() - t0 > WAIT_NS) break;
  }
  return false;
}
// Waits for two barriers; both try_waits are issued before either result is
// used, so their latencies overlap.
__device__ __forceinline__ bool mbar_wait2(uint32_t bar_a, uint32_t par_a, uint32_t bar_b, uint32_t par_b,
                                           volatile int* abort, int code, int* err, uint64_t limit_ns = WAIT_NS) {
  bool da = false, db = false;
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < WAIT_LIMIT; i++) {
    uint32_t oa, ob;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%2], %3, %6;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 q, [%4], %5, %6;\n"
        " selp.u32 %0, 1, 0, p;\n selp.u32 %1, 1, 0, q;\n}\n"
        : "=r"(oa), "=r"(ob)
        : "r"(bar_a), "r"(par_a), "r"(bar_b), "r"(par_b), "r"(SUSPEND_NS)
        : "memory");
    da = da || oa != 0;
    db = db || ob != 0;
    if (da && db) return true;
    if (*abort) return false;
    if (i == 0) t0 = global_ns();
    else if (global_ns() - t0 > limit_ns) break;
  }
  *abort = 1;
  atomicCAS(err, 0, code | (da ? 0 : 0x10) | (db ? 0 : 0x20));
  return false;
}

// Linear bulk copy global -> shared (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Tiled tensor copies (the innermost coordinate x must be 16-byte aligned:
// every caller passes x = 0 or a multiple of 64 f16 elements).
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Host: the driver's cuTensorMapEncodeTiled, through the runtime's entry
// point query (no link dependency on libcuda). nullptr when unavailable.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();

}  // namespace wg
