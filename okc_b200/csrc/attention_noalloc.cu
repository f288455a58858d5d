// Paged FP8 attention decode for callers that cannot allocate device memory.
//
// okc_attn_decode_fp8 needs a workspace for its split-KV partials (running max, running
// sum and unnormalised output of every (CTA, sequence) segment) that the caller allocates.
// Some callers cannot do that: code running inside a host framework whose allocator is off
// limits (for example a plugin that may only enqueue work on a stream it is handed), or a
// process that must not grow its device footprint after start-up.  This entry point keeps
// the partials in a fixed-size array that lives in the library itself, so the call needs no
// allocation at all.
//
// The array is a file-scope static __device__ buffer of kNoAllocScratchBytes (16 MiB).  Every
// GPU that loads this part of the library keeps it until the process exits.  It is shared
// by every call on that device and keeps the last call's contents; calls that can overlap
// on the GPU (different streams without ordering between them) race on it and must not be
// issued.  The partials need no clearing (each call writes every entry it later reads).  The
// error word at its start starts at zero (static device storage is zero-filled when the
// library's module loads), collects the OKC_DEVERR_* bits of every call on the device, and is
// read and cleared by okc_attn_decode_fp8_noalloc_error().  Requests whose partials do not fit
// are rejected with OKC_ERR_TOO_LARGE.
#include <mutex>

#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// The device address of g_attn_scratch on the current device.  The host-side name of the
// array is only a stand-in, so the address is looked up once per device (with that device
// current) and cached.  The lookup happens on the first call on each device; make that first
// call before capturing a stream into a CUDA graph.
void* scratch_on_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || !p) return nullptr;
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int okc_attn_decode_fp8_noalloc(const void* q, int ldq, const void* k_cache, const void* v_cache,
                                           const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                                           const float* k_scale, const float* v_scale, void* out, int ldo,
                                           int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                                           float sm_scale, int num_ctas, okc_stream_t stream) {
  if (num_ctas <= 0) num_ctas = okc_host::num_sms();
  const size_t need = okc_attn_decode_workspace_bytes(B, Hq, Hkv, D, num_ctas);
  if (need == 0) return OKC_ERR_INVALID;
  if (need > kNoAllocScratchBytes) return OKC_ERR_TOO_LARGE;
  void* scratch = scratch_on_current_device();
  if (!scratch) return OKC_ERR_DEVICE;
  return okc_attn_decode_fp8(q, ldq, k_cache, v_cache, page_table, table_ld, seq_lens, k_scale, v_scale, out,
                             ldo, B, Hq, Hkv, D, page_size, num_pages, sm_scale, num_ctas, scratch,
                             kNoAllocScratchBytes, stream);
}

// Reads and clears the error word of the no-alloc scratch on the current device, after the
// work already enqueued on `stream` (synchronises the stream).  The copy lands in a local
// variable, so this allocates nothing either.
extern "C" int okc_attn_decode_fp8_noalloc_error(okc_stream_t stream) {
  void* scratch = scratch_on_current_device();
  if (!scratch) return OKC_ERR_DEVICE;
  int word = 0;
  if (cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaMemsetAsync(scratch, 0, sizeof(int), stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_LAUNCH;
  }
  return word;
}
