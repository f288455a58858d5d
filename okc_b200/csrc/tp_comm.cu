// Tensor-parallel exchange of the decode layer over NVLink peer memory.
//
// The row-parallel O projection leaves every rank with an fp32 partial P_r [T, H]; the layer
// output is out = bf16(x + sum_r P_r), replicated on every rank.  tp_allreduce_kernel does that
// in ONE launch, reading and writing the peers' buffers directly (CUDA IPC mappings; every GPU
// of the box is a full-bandwidth NVSwitch peer):
//   1. entry: each rank publishes "my partial is complete" (epoch-tagged flag stored into every
//      peer's flag array, release at system scope) and waits for all peers' flags;
//   2. reduce-scatter + all-gather fused: rank r owns the r-th slice of the elements, sums the
//      W partials of that slice in rank order (the same fixed order on every rank, so the
//      replicated outputs are identical), adds the residual, rounds to bf16 and stores the
//      result into every rank's output buffer;
//   3. exit: the last CTA of the rank publishes "my stores are done" and waits for every peer's,
//      so when the kernel completes this rank's output buffer holds all slices.
// NVLink bytes per rank: (W-1)/W of the partial read (fp32) + (W-1)/W of the output written
// (bf16); at T = 128, H = 8192, W = 8: 3.5 MB in, 1.75 MB out.
// Every flag wait is bounded (2 s of %globaltimer): on expiry the kernel sets
// OKC_DEVERR_TIMEOUT in the error word and goes on, so a missing rank cannot hang the GPU.
// No TMA and no multicast: plain 16-byte peer loads and 8-byte peer stores.
#include <string.h>

#include "kernels.cuh"

namespace okc {

constexpr int kTpMaxRanks = 8;

struct TpArgs {
  const float* part[kTpMaxRanks];         // every rank's fp32 partial (this rank's is local)
  __nv_bfloat16* out[kTpMaxRanks];        // every rank's bf16 output buffer
  int* flags[kTpMaxRanks];                // every rank's flags: [0, W) entry, [8, 8 + W) exit
  const __nv_bfloat16* residual;          // local, replicated on every rank
  int* state;                             // local: [0] epoch of the last completed call, [1] CTAs done
  int* err;
  long long n;                            // elements of [T, H]
  int rank, world;
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *f >= epoch (bounded); false on timeout (error bit set).
__device__ bool wait_flag(const int* f, int epoch, int* err) {
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(f) < epoch) {
    if (globaltimer() - t0 > 2000000000ull) {
      atomicOr(err, OKC_DEVERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Signals `epoch` into slot `slot` of every rank's flag array: thread q < W stores to rank q,
// after one system-scope fence per storing thread (the fences run in parallel; with the
// preceding __syncthreads they order every prior write of the CTA before the flags).  A
// chain of release stores would instead serialise one NVLink round trip per peer.
__device__ __forceinline__ void signal_all(const TpArgs& a, int slot, int epoch) {
  if (threadIdx.x < (unsigned)a.world) {
    __threadfence_system();
    st_relaxed_sys(&a.flags[threadIdx.x][slot], epoch);
  }
}
// Thread q < W waits for rank q's flag in `base + q` of this rank's array; true if all arrived.
__device__ __forceinline__ bool wait_all(const TpArgs& a, int base, int epoch, int* s_ok) {
  if (threadIdx.x == 0) *s_ok = 1;
  __syncthreads();
  if (threadIdx.x < (unsigned)a.world)
    if (!wait_flag(&a.flags[a.rank][base + threadIdx.x], epoch, a.err)) *s_ok = 0;
  __syncthreads();
  return *s_ok != 0;
}

__global__ void __launch_bounds__(256) tp_allreduce_kernel(TpArgs a) {
  pdl_trigger();
  pdl_wait();  // this rank's partial (previous kernel) is complete and visible
  __shared__ int s_epoch, s_ok, s_last;
  if (threadIdx.x == 0) s_epoch = ld_acquire_sys(&a.state[0]) + 1;
  __syncthreads();
  const int epoch = s_epoch;
  if (blockIdx.x == 0) signal_all(a, a.rank, epoch);  // entry: "my partial is complete"
  if (wait_all(a, 0, epoch, &s_ok)) {
    const long long n4 = a.n >> 2;
    const long long per = (n4 + a.world - 1) / a.world;
    const long long lo = per * a.rank, hi = min(n4, lo + per);
    for (long long i = lo + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < hi;
         i += (long long)gridDim.x * blockDim.x) {
      float4 v[kTpMaxRanks];
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) v[q] = __ldcg(reinterpret_cast<const float4*>(a.part[q]) + i);
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) { s0 += v[q].x; s1 += v[q].y; s2 += v[q].z; s3 += v[q].w; }
      if (a.residual) {
        const uint2 rv = reinterpret_cast<const uint2*>(a.residual)[i];
        s0 += bf16_lo(rv.x); s1 += bf16_hi(rv.x); s2 += bf16_lo(rv.y); s3 += bf16_hi(rv.y);
      }
      const uint2 o = make_uint2(pack_bf16x2(s0, s1), pack_bf16x2(s2, s3));
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) reinterpret_cast<uint2*>(a.out[q])[i] = o;
    }
  }
  // exit: the last CTA of this rank tells the peers its stores are done and waits for theirs
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(&a.state[1], 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) a.state[1] = 0;
    signal_all(a, kTpMaxRanks + a.rank, epoch);
    wait_all(a, kTpMaxRanks, epoch, &s_ok);
    if (threadIdx.x == 0) st_release_sys(&a.state[0], epoch);
  }
}

}  // namespace okc

// ------------------------------------------------------------------------------ C ABI

extern "C" int okc_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return OKC_ERR_INVALID;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return OKC_ERR_DEVICE;
  }
  return OKC_OK;
}

extern "C" int okc_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? OKC_OK : OKC_ERR_DEVICE; }

extern "C" int okc_ipc_handle(const void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return OKC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  memcpy(handle_out, &h, sizeof(h));
  return OKC_OK;
}

extern "C" int okc_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return OKC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  return OKC_OK;
}

extern "C" int okc_ipc_close(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? OKC_OK : OKC_ERR_DEVICE;
}

extern "C" int okc_tp_allreduce_residual(const float* const* parts, void* const* outs, int* const* flags,
                                         const void* residual, int* state, int rank, int world,
                                         long long n, void* workspace, okc_stream_t stream) {
  if (world < 2 || world > okc::kTpMaxRanks || rank < 0 || rank >= world || n <= 0 || (n & 3) ||
      !parts || !outs || !flags || !state || !workspace)
    return OKC_ERR_INVALID;
  okc::TpArgs a = {};
  for (int q = 0; q < world; ++q) {
    if (!parts[q] || !outs[q] || !flags[q]) return OKC_ERR_INVALID;
    if (!okc_host::aligned16(parts[q]) || (reinterpret_cast<uintptr_t>(outs[q]) & 7)) return OKC_ERR_ALIGNMENT;
    a.part[q] = parts[q];
    a.out[q] = reinterpret_cast<__nv_bfloat16*>(outs[q]);
    a.flags[q] = flags[q];
  }
  if (reinterpret_cast<uintptr_t>(residual) & 7) return OKC_ERR_ALIGNMENT;
  a.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  a.state = state;
  a.err = reinterpret_cast<int*>(workspace);
  a.n = n;
  a.rank = rank;
  a.world = world;
  const long long per4 = ((n >> 2) + world - 1) / world;
  int blocks = (int)((per4 + 255) / 256);
  const int cap = 2 * okc_host::num_sms();
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return okc_host::launch_k(okc::tp_allreduce_kernel, dim3(blocks), dim3(256), 0,
                            reinterpret_cast<cudaStream_t>(stream), dim3(1), a);
}
