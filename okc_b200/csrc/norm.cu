// RMSNorm over bf16 rows: y[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * g),
// g = w (plain weight) or 1 + w (Muse's zero-centred gain).  HBM-bound: 4*H bytes a row.
// Mirrors `_norm` muse_decode_layer/decode/boundaries.py:8-14 and `rms`/`gain`
// muse_prefill_layer/submission.py:89-96.
#include "common.cuh"

namespace okc {

constexpr int kNormMaxVec = 8;  // 16-byte vectors per thread: H <= 256 * 8 * 8 = 16384

// Single pass: the row stays in registers between the sum of squares and the scaling.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ y, int ldy, int H,
                                                      float eps, int unit_offset) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)t * ldx;
  __nv_bfloat16* yr = y + (size_t)t * ldy;
  __shared__ float red[8];
  uint4 v[kNormMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 8;
    v[j] = i < H ? *reinterpret_cast<const uint4*>(xr + i) : make_uint4(0, 0, 0, 0);
    const uint32_t wv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = bf16_lo(wv[k]), b = bf16_hi(wv[k]);
      ss += a * a + b * b;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 8;
    if (i >= H) break;
    const uint4 gw = *reinterpret_cast<const uint4*>(w + i);
    const uint32_t xv[4] = {v[j].x, v[j].y, v[j].z, v[j].w}, gv[4] = {gw.x, gw.y, gw.z, gw.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float g0 = bf16_lo(gv[k]), g1 = bf16_hi(gv[k]);
      if (unit_offset) { g0 += 1.f; g1 += 1.f; }
      o[k] = pack_bf16x2(bf16_lo(xv[k]) * inv * g0, bf16_hi(xv[k]) * inv * g1);
    }
    *reinterpret_cast<uint4*>(yr + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int launch_rmsnorm(const void* x, int ldx, const void* w, void* y, int ldy, int T, int H, float eps,
                   int unit_offset, cudaStream_t stream) {
  return okc_host::launch_k(rmsnorm_kernel, dim3(T), dim3(256), 0, stream, dim3(1),
                            reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                            reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<__nv_bfloat16*>(y), ldy,
                            H, eps, unit_offset);
}

}  // namespace okc
