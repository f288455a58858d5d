// Work partition shared by the paged-attention decode kernels (attention.cu: mma.sync consumer,
// attention_tc.cu: tcgen05 consumer) and the split-KV merge.
//
// A sequence b attends the cached tokens [lo_b, len_b) with len_b = seq_lens[b] and
// lo_b = max(0, len_b - window) for a sliding window (0 = the whole context): query token at
// position p attends (p - window, p], muse_prefill_layer/submission.py:169-171.  Its tokens are
// cut into units of TS tokens starting at origin_b = lo_b rounded down to `align` tokens (1 for
// the mma.sync kernel, the page size for the tcgen05 kernel, whose tiles start on a page);
// rows of a unit outside [lo_b, len_b) are masked.  Units of all sequences are numbered in
// order and split evenly over a persistent grid (stream-K): CTA c gets q or q+1 consecutive
// units, so ragged context lengths stay balanced.
//
// Speculative-verify blocks (q_len L tokens per request) are L "virtual" sequences per request,
// one per query token, each with its own visible length (position + 1) and the request's
// page-table row (virtual sequence v reads row v / q_per_seq).
#pragma once

#include "kernels.cuh"

namespace okc {

__host__ __device__ __forceinline__ void unit_range(int U, int C, int c, int& u0, int& u1) {
  const int q = U / C, r = U % C;
  u0 = c * q + (c < r ? c : r);
  u1 = u0 + q + (c < r ? 1 : 0);
}

__host__ __device__ __forceinline__ int cta_of_unit(int U, int C, int u) {
  const int q = U / C, r = U % C;
  const int big = r * (q + 1);
  return u < big ? u / (q + 1) : r + (u - big) / q;
}

__device__ __forceinline__ int seq_lo(int len, int window) {
  return window > 0 && len > window ? len - window : 0;
}

__device__ __forceinline__ int seq_origin(int len, int window, int align) {
  const int lo = seq_lo(len, window);
  return lo - lo % align;
}

// Exclusive prefix of per-sequence unit counts into prefix[0..B], by warp 0.
__device__ __forceinline__ void unit_prefix(const int32_t* seq_lens, int B, int TS, int window, int align,
                                            int* prefix) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      int len = b < B ? seq_lens[b] : 0;
      if (len < 0) len = 0;
      const int n = (len - seq_origin(len, window, align) + TS - 1) / TS;
      int v = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (b < B) prefix[b] = carry + v - n;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) prefix[B] = carry;
  }
}

__device__ __forceinline__ int find_seq(const int* prefix, int B, int u) {
  int lo = 0, hi = B - 1;  // largest b with prefix[b] <= u
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Launches the deterministic split-KV merge over the partials a decode kernel left in the
// workspace (units of TS tokens, NSUB sub-tiles per unit).
int launch_attn_merge(AttnArgs& a, int TS, int NSUB, int D, cudaStream_t stream);

// The tcgen05 decode kernel (attention_tc.cu): head_dim 128, page sizes 16..128, 2..8 KV heads,
// up to 8 query heads per KV head, selected with OKC_ATTN_TC=1; the mma.sync kernel
// (attention.cu) serves every shape and is the default.
bool attn_tc_eligible(const AttnArgs& a, int D, int Hkv);
int launch_attn_tc(AttnArgs& a, int Hkv, cudaStream_t stream);

}  // namespace okc
