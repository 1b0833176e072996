// Shared device/host helpers for the sm_100a int4/int8 weight-only GEMM library.
//
// Everything here is plain CUDA + inline PTX for sm_100a: mbarrier pipelines,
// TMA (cp.async.bulk.tensor) loads, Ampere-style cp.async with mbarrier
// completion, and the bounded waits every spin loop in this library uses.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "gfx906_b200.h"

namespace gfx {

// ---------------------------------------------------------------------------
// device-side error word: bounded waits that give up record a code here
// instead of hanging the GPU. Without relocatable device code every
// translation unit has its own copy; each kernel file exports a host reader
// (GFX_DEFINE_STATUS_READER) and gfx_device_status combines them.
// ---------------------------------------------------------------------------
static __device__ int g_device_error = 0;

#define GFX_DEFINE_STATUS_READER(name)                                        \
  int name(int clear) {                                                       \
    int v = 0;                                                                \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) \
      return -1;                                                              \
    if (clear && v) {                                                         \
      int zero = 0;                                                           \
      cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));                 \
    }                                                                         \
    return v;                                                                 \
  }

// Wall-clock budget of one bounded wait (ns). A healthy pipeline completes
// every wait in microseconds; this only ends waits that can never complete.
constexpr unsigned long long kWaitTimeoutNs = 2000ull * 1000ull * 1000ull;

enum DeviceErrorCode : int {
  kDevErrNone = 0,
  kDevErrFullBarrierTimeout = 1,
  kDevErrEmptyBarrierTimeout = 2,
  kDevErrMmaBarrierTimeout = 3,
  kDevErrEpilogueBarrierTimeout = 4,
  kDevErrClusterReduceTimeout = 5,
  kDevErrSelfTestTimeout = 6,  // gfx_selftest_wait_timeout: the expected outcome
  kDevErrPeerBarrierTimeout = 7,
};

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// Copy this translation unit's status word, if set, into `host_word`: one int
// of pinned, mapped host memory per device (host_status_word below), so that
// the host sees a wait that gave up before its next launch without a device
// synchronisation. Called on the failure paths only; a null word (host memory
// could not be mapped) skips it.
__device__ __forceinline__ void mirror_device_error(int* host_word) {
  if (host_word == nullptr) return;
  const int v = *(volatile int*)&g_device_error;
  if (v != 0) {
    *(volatile int*)host_word = v;
    __threadfence_system();
  }
}

// ---------------------------------------------------------------------------
// shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make barrier inits visible to the async proxy (TMA, tcgen05) and the cluster.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
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

// Bounded wait: returns false (and records `code`) once `timeout_ns` passes,
// or at once if another thread of the grid already recorded an error.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int code,
                                              unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0u) {
      if (*(volatile int*)&g_device_error != 0) return false;
      if (global_timer_ns() - t0 > timeout_ns) {
        record_device_error(code);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  return mbar_wait_for(bar, parity, code, kWaitTimeoutNs);
}

// ---------------------------------------------------------------------------
// thread-block clusters (CTA pairs)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster; release/acquire at cluster scope.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Store to distributed shared memory (a mapa'd shared::cluster address).
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Arrive with release at cluster scope on the barrier at the same offset in
// CTA `rank`: this thread's earlier stores, distributed shared memory
// included, are visible to a cluster-scope acquire of the completed phase.
__device__ __forceinline__ void mbar_arrive_release_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   mapa_shared(smem_u32(bar), rank))
               : "memory");
}

// Bounded wait with acquire at cluster scope (pairs with the arrive above).
__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity, int code) {
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((++spins & 255u) == 0u) {
      if (*(volatile int*)&g_device_error != 0) return false;
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        record_device_error(code);
        return false;
      }
    }
  }
}

// Arrive on the barrier at the same offset in CTA `rank` of the cluster
// (default .release.cta semantics: a cluster-scope release would wait for all
// of the thread's outstanding memory operations, global stores included).
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(mapa_shared(smem_u32(bar), rank)) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (tensor) and Ampere-style cp.async
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel of the
// stream is still running: pdl_wait() blocks until that kernel has completed
// and its memory is visible, so every read of data another kernel produced and
// every global write comes after it. pdl_trigger() lets the next kernel of the
// stream launch (its CTAs take SMs as this grid's CTAs retire). Both return at
// once when there is no such dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Prefetch one 2-D box of a tensor map into L2 (no shared memory, no barrier).
// Safe before pdl_wait(): L2 is the point of coherence, so a line fetched
// before the previous kernel's writes reach L2 is updated by those writes.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// 2-D tiled TMA load, completion counted on `bar` in bytes. c0 is the
// innermost coordinate (elements); c0 * elem_size must be 16-byte aligned.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 4-byte async copy global -> shared; src_bytes = 0 zero-fills (no read).
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// The mbarrier receives one arrival when all of this thread's prior cp.async
// copies have landed (the barrier's expected count must include it).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// explicit shared-window accesses (32-bit shared addresses): generic pointers
// into shared memory can compile to generic loads and stores, which take the
// L1TEX path (long-scoreboard latency) and split into extra wavefronts
// ---------------------------------------------------------------------------
__device__ __forceinline__ void sts128(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float lds_f16_as_f32(uint32_t addr) {
  unsigned short h;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr) : "memory");
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ---------------------------------------------------------------------------
// global loads / misc
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// d = (a & b) ^ c in one LOP3.
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

}  // namespace gfx

// ---------------------------------------------------------------------------
// host side helpers (defined in capi.cu)
// ---------------------------------------------------------------------------
namespace gfx {
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int sm_count(int device);
int current_device();
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
// Same, through a small per-device cache keyed on every argument: the weight
// maps of a model's layers are encoded once, not on every call.
int cached_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

// Host-visible status word of `dev` (a device-usable pointer into pinned,
// mapped host memory), or nullptr when that memory could not be mapped.
int* host_status_word(int dev);
// Its current value (a plain host read; no device synchronisation).
int host_status_read(int dev);
// Zero it; bumps the device's failure epoch when it was set.
void host_status_clear(int dev);
// Counts the failures cleared on `dev`; a cached scratch buffer whose split-K
// counters were last re-zeroed at an older epoch must re-zero them again.
unsigned failure_epoch(int dev);
// GFX_OK, or GFX_ERR_DEVICE (with a message) when `dev` reports a wait that
// gave up; then the first counter_bytes of `workspace` (the split-K arrival
// counters, if any) are re-zeroed on `stream` before returning.
int check_device_health(const char* fn, int dev, void* workspace, size_t counter_bytes, cudaStream_t stream);

// Argument checks shared by the GEMM entry points (messages name `fn`).
int check_gemm_common(const char* fn, const void* x, int x_dtype, const void* w, const void* ws, int scale_dtype,
                      void* y, int out_dtype, int M, int N, int K, int splits);
}  // namespace gfx
