// Shared device helpers for the okc_b200 kernels (sm_100a).
//
// * mbarrier rings with BOUNDED waits: every wait gives up after kWaitNs of %globaltimer
//   time, records OKC_DEVERR_TIMEOUT in the caller's error word and reports failure, so
//   no kernel here can spin forever.
// * 1-D bulk copies (cp.async.bulk, the TMA bulk engine) global -> shared, completing on
//   an mbarrier, with an L2 evict-first hint for data that is streamed exactly once.
// * warp-level mma.sync wrappers (bf16 m16n8k16, e4m3 m16n8k32) and small conversions.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdlib.h>
#include <utility>

#include "../../include/okc_b200.h"

namespace okc {

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s: far beyond any legal wait

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and sets
// OKC_DEVERR_TIMEOUT in *err) if it did not complete within kWaitNs.  With `abort` given, it
// also returns false (at once, or within 256 polls) once *abort is non-zero: a CTA whose other
// role gave up stops waiting for work that will never arrive.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          const volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  if (abort && *abort) return false;
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u) {
      if (abort && *abort) return false;
      if (globaltimer() - t0 > kWaitNs) {
        atomicOr(err, OKC_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) global -> shared,
// completing `bytes` transactions on `bar`.
// Same as bulk_g2s with the default L2 policy (for small, re-read data such as activations).
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------------------
// mma.sync wrappers.  Fragment layouts (PTX ISA, "Matrix fragments for mma.m16n8k16 /
// m16n8k32"), with g = lane / 4 and c = lane % 4:
//   A (16 x K, row): a0 (row g,   k-slots lo), a1 (row g+8, lo), a2 (row g, hi), a3 (row g+8, hi)
//   B (K x 8, col):  b0 (k-slots lo, col g), b1 (k-slots hi, col g)
//   C (16 x 8):      c0, c1 (row g, cols 2c, 2c+1), c2, c3 (row g+8, cols 2c, 2c+1)
// bf16/f16 k16: lo = {2c, 2c+1}, hi = {2c+8, 2c+9}.   e4m3 k32: lo = {4c..4c+3},
// hi = {16+4c..16+4c+3}.  Because a product sums over k, any bijection of k applied to
// A and B alike gives the same result; the kernels use that to load wide contiguous runs.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_e4m3_16832(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte permute (PRMT): result byte i = byte sel_i of the 8-byte value {b:a}.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Two floats -> two e4m3 bytes (x in the low byte), round-to-nearest-even, saturating.
__device__ __forceinline__ uint16_t f2_to_e4m3x2_sat(float x, float y) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(x, y), __NV_SATFINITE, __NV_E4M3);
}

// One float -> e4m3 byte, RNE, overflow -> NaN (the semantics of torch's .to(float8_e4m3fn)).
__device__ __forceinline__ uint8_t f_to_e4m3_nosat(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_NOSAT, __NV_E4M3);
}

__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&r);
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

}  // namespace okc

// Host-side helpers shared by the entry points.
// Programmatic dependent launch (PDL).  Every kernel lets its successor in the stream launch
// early (pdl_trigger at entry: the successor's blocks may then be scheduled as soon as all of
// this grid's blocks have started) and waits for its predecessor grid to complete, with its
// memory visible, before it touches global memory (pdl_wait).  pdl_wait returns at once when
// the kernel was launched without the attribute.  This hides the launch latency and the
// prologue (barrier init, TMEM allocation) of each kernel behind the tail of the previous one.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

namespace okc_host {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return OKC_OK;
  if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
    return OKC_ERR_DEVICE;
  return OKC_ERR_LAUNCH;
}

int num_sms();  // cached per device (defined in capi.cu)

// PDL on by default; OKC_PDL=0 launches every kernel with plain stream order.
inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("OKC_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Launches `kernel` with the programmatic-stream-serialization attribute (plus an optional
// cluster shape); returns an OKC status.
template <typename... KArgs, typename... Args>
inline int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                    dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_LAUNCH;
  }
  return launch_status();
}

}  // namespace okc_host
