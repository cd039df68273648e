// Shared device helpers for the mouse_core_b200 kernels (sm_100a only).
//
// Inline PTX wrappers for mbarriers, TMA tensor copies (no multicast: every
// load lands in the issuing CTA's own shared memory), ldmatrix and the
// m16n8k16 bf16 MMA, plus bounded waits that report a timeout through a
// device status word instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "mouse_core_b200 kernels target sm_100a (B200) only"
#endif

namespace mb {

// Status codes written to the device status word (see mb_device_status()).
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,   // consumer gave up waiting for a TMA stage
  kDevTimeoutEmpty = 2,  // producer gave up waiting for a free stage
  kDevBadPage = 3,       // block-table entry outside the page pool
  kDevBadSmem = 4,       // dynamic shared memory base not 1024-byte aligned
  kDevBadPair = 5,       // stored-dS pair index outside the scratch (inconsistent pair offsets)
  kDevTimeoutDrain = 6,  // a CTA's own copies or MMAs did not complete before it exited
  kDevBadIndex = 7,      // an embedding id outside its table (the token is left zero)
};

// The library is one translation unit (mouse_b200.cu), so the status word is
// defined here; every kernel reports through it.
__device__ int g_device_status = 0;

__device__ __forceinline__ void report(int code) { atomicCAS(&g_device_status, 0, code); }

// About two seconds at B200 clocks: long enough never to fire on a healthy
// pipeline, short enough that a broken one ends and the host sees a status.
constexpr long long kWaitCycles = 4000000000ll;

// Cycles a wait spins after its first failed test before it gives up; the
// host can change it (mb_set_wait_limit) to make a wait run out on purpose.
__device__ long long g_wait_limit = kWaitCycles;

// Limit of the waits that drain a CTA's own in-flight copies before it exits:
// those copies always complete, so this never depends on g_wait_limit.
constexpr long long kDrainCycles = kWaitCycles;

// Host side: launch set-up (a kernel's shared-memory attribute, an
// occupancy figure) is per device, so one-time caches of it are indexed by
// the current device's ordinal; -1 (no caching) outside [0, kMaxDevices).
constexpr int kMaxDevices = 64;
inline int device_slot() {
  int d = -1;
  return (cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < kMaxDevices) ? d : -1;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Dynamic shared memory is used from its base without padding (the kernels
// need nearly all 227 KB); the 128-byte-swizzled TMA boxes need the base
// 1024-byte aligned, which is checked before anything else runs.
__device__ __forceinline__ bool smem_base_aligned(const void* p) { return (smem_u32(p) & 1023u) == 0; }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ long long wait_limit() {
  return *reinterpret_cast<volatile long long*>(&g_wait_limit);
}

// Wait for the phase with the given parity to complete; false on timeout
// (after recording `code` in the device status word). The limit is checked
// before every retry, so a limit of 0 gives up right after the first failed
// test.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long limit = wait_limit();
  const long long t0 = clock64();
  while (true) {
    if (clock64() - t0 > limit) {
      report(code);
      return false;
    }
    if (mbar_try_wait(bar, parity)) return true;
  }
}

// As mbar_wait, for a wait off the critical path: the warp sleeps between
// polls, so it takes no issue slots or barrier-unit cycles from the warps
// doing the work it waits for.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long limit = wait_limit();
  const long long t0 = clock64();
  while (true) {
    if (clock64() - t0 > limit) {
      report(code);
      return false;
    }
    __nanosleep(256);
    if (mbar_try_wait(bar, parity)) return true;
  }
}

// As mbar_wait, but also gives up (without a new code) once `*abort` is set,
// and sets `*abort` itself when it times out, so the other warps of the CTA
// stop waiting too.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, int code, int* abort) {
  volatile int* ab = abort;
  if (mbar_try_wait(bar, parity)) return true;
  const long long limit = wait_limit();
  const long long t0 = clock64();
  while (true) {
    if (*ab) return false;
    if (clock64() - t0 > limit) {
      report(code);
      *ab = 1;
      return false;
    }
    if (mbar_try_wait(bar, parity)) return true;
  }
}

// Wait for a phase that this CTA's own in-flight copies complete (a TMA load
// it issued) before the CTA exits; bounded by kDrainCycles, not by the
// host-set limit.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kDrainCycles) {
      report(kDevTimeoutDrain);
      return;
    }
  }
}

// Every load a CTA issued into a ring of `stages` barriers lands before the
// CTA exits: load i of the `issued` went to barrier i % stages in phase
// (i / stages) & 1, and only the last `stages` can still be in flight (a slot
// is reloaded only after its previous phase completed). Each barrier's last
// phase is also the newest it will ever reach, so the wait is exact whether
// the pipeline finished or a wait of it ran out.
__device__ __forceinline__ void drain_ring(uint64_t* ring, int stages, int issued) {
  for (int i = issued > stages ? issued - stages : 0; i < issued; ++i)
    mbar_drain(&ring[i % stages], (uint32_t)(i / stages) & 1);
}

// ---------------------------------------------------------------- TMA
// 2-D tiled tensor load into this CTA's shared memory, completion counted in
// bytes on `bar`. Coordinates are in elements; x (innermost) must be a
// multiple of 16 bytes, which every caller guarantees by using x = 0 or 64.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (no multicast), completion
// counted in bytes on `bar`; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- warp MMA
__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a TMA box
// written with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, 1024-byte aligned).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// Named barrier over `nthreads` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over its `nthreads` threads: every
// thread gets the same answer, so a decision taken on it keeps them together.
__device__ __forceinline__ bool named_barrier_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mb
