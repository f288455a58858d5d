// RMSNorm over bf16 rows: y[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * g),
// g = w (plain weight) or 1 + w (Muse's zero-centred gain).  HBM-bound: 4*H bytes a row.
// Mirrors `_norm` muse_decode_layer/decode/boundaries.py:8-14 and `rms`/`gain`
// muse_prefill_layer/submission.py:89-96.
#include "common.cuh"

namespace okc {

constexpr int kNormMaxVec = 8;  // 16-byte vectors per thread: H <= 256 * 8 * 8 = 16384

// Single pass: the row stays in registers between the sum of squares and the scaling; the
// weight is loaded with the row, so its latency overlaps the row's instead of following the
// reduction.
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
  uint4 v[kNormMaxVec], gw[kNormMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 8;
    v[j] = i < H ? *reinterpret_cast<const uint4*>(xr + i) : make_uint4(0, 0, 0, 0);
    gw[j] = i < H ? *reinterpret_cast<const uint4*>(w + i) : make_uint4(0, 0, 0, 0);
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
    const uint32_t xv[4] = {v[j].x, v[j].y, v[j].z, v[j].w}, gv[4] = {gw[j].x, gw[j].y, gw[j].z, gw[j].w};
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

// Sum over the CTA (blockDim.x a multiple of 32, <= 1024); `red` holds a slot per warp.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  __syncthreads();  // red is reused by the next reduction
  return tot;
}

__device__ __forceinline__ float bf16_rn_f(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Muse's gated residual boundary (muse_decode_layer/decode/boundaries.py:17-37): the branch row
// (bf16; with post_w first scaled by 1 + post_w and rounded to bf16) is RMS-normalised with
// post_eps, the fp32 residual stream becomes alpha * stream + beta * branch, and the next block's
// input is hidden = bf16(stream' * rsqrt(mean(stream'^2) + pre_eps) * (1 + pre_w)), also stored
// unrounded in fp32 for the router when router_out is given.  Products and sums are rounded one
// at a time (the reference compiles this kernel with fp fusion off).  One CTA of 512 threads a
// row, the row in registers between the two reductions; stream_out may alias stream (a thread
// reads its stream elements, with pre_w, in the first pass, before it writes them).
constexpr int kBndVec = 4;  // 512 threads x 4 x 8 elements: H <= 16384

__global__ void __launch_bounds__(512) residual_boundary_kernel(
    const float* stream, const __nv_bfloat16* __restrict__ branch, int ldb, const float* __restrict__ alpha,
    const float* __restrict__ beta, const __nv_bfloat16* __restrict__ post_w,
    const __nv_bfloat16* __restrict__ pre_w, __nv_bfloat16* __restrict__ hidden, float* stream_out,
    float* __restrict__ router_out, int H, float post_eps, float pre_eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[16];
  const int t = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* br = branch + (size_t)t * ldb;
  const float* sr = stream + (size_t)t * H;
  float v[kBndVec][8];
  float4 sv[kBndVec][2];
  uint4 pre4[kBndVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kBndVec; ++j) {
    const int i = (j * 512 + tid) * 8;
    if (i >= H) break;
    const uint4 u4 = *reinterpret_cast<const uint4*>(br + i);
    // issued with the branch row: their latency overlaps its, not the reductions
    sv[j][0] = *reinterpret_cast<const float4*>(sr + i);
    sv[j][1] = *reinterpret_cast<const float4*>(sr + i + 4);
    pre4[j] = *reinterpret_cast<const uint4*>(pre_w + i);
    const uint32_t u[4] = {u4.x, u4.y, u4.z, u4.w};
    uint32_t pw[4] = {0u, 0u, 0u, 0u};
    if (post_w) {
      const uint4 p4 = *reinterpret_cast<const uint4*>(post_w + i);
      pw[0] = p4.x; pw[1] = p4.y; pw[2] = p4.z; pw[3] = p4.w;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float a = bf16_lo(u[k]), b = bf16_hi(u[k]);
      if (post_w) {
        a = bf16_rn_f(__fmul_rn(a, __fadd_rn(1.f, bf16_lo(pw[k]))));
        b = bf16_rn_f(__fmul_rn(b, __fadd_rn(1.f, bf16_hi(pw[k]))));
      }
      v[j][2 * k] = a;
      v[j][2 * k + 1] = b;
      ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
    }
  }
  const float inv_b = rsqrtf(block_sum(ss, red) / (float)H + post_eps);
  float* so = stream_out + (size_t)t * H;
  ss = 0.f;
#pragma unroll
  for (int j = 0; j < kBndVec; ++j) {
    const int i = (j * 512 + tid) * 8;
    if (i >= H) break;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 o = sv[j][h];
      const float4 al = *reinterpret_cast<const float4*>(alpha + i + 4 * h);
      const float4 be = *reinterpret_cast<const float4*>(beta + i + 4 * h);
      const float ov[4] = {o.x, o.y, o.z, o.w}, av[4] = {al.x, al.y, al.z, al.w}, bv[4] = {be.x, be.y, be.z, be.w};
      float r[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float nb = __fmul_rn(v[j][4 * h + k], inv_b);
        r[k] = __fadd_rn(__fmul_rn(av[k], ov[k]), __fmul_rn(bv[k], nb));
        v[j][4 * h + k] = r[k];
        ss = __fadd_rn(ss, __fmul_rn(r[k], r[k]));
      }
      *reinterpret_cast<float4*>(so + i + 4 * h) = make_float4(r[0], r[1], r[2], r[3]);
    }
  }
  const float inv_s = rsqrtf(block_sum(ss, red) / (float)H + pre_eps);
#pragma unroll
  for (int j = 0; j < kBndVec; ++j) {
    const int i = (j * 512 + tid) * 8;
    if (i >= H) break;
    const uint32_t pw[4] = {pre4[j].x, pre4[j].y, pre4[j].z, pre4[j].w};
    float h[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h[2 * k] = __fmul_rn(__fmul_rn(v[j][2 * k], inv_s), __fadd_rn(1.f, bf16_lo(pw[k])));
      h[2 * k + 1] = __fmul_rn(__fmul_rn(v[j][2 * k + 1], inv_s), __fadd_rn(1.f, bf16_hi(pw[k])));
    }
    uint4 o;
    o.x = pack_bf16x2(h[0], h[1]); o.y = pack_bf16x2(h[2], h[3]);
    o.z = pack_bf16x2(h[4], h[5]); o.w = pack_bf16x2(h[6], h[7]);
    *reinterpret_cast<uint4*>(hidden + (size_t)t * H + i) = o;
    if (router_out) {
      float4* r4 = reinterpret_cast<float4*>(router_out + (size_t)t * H + i);
      r4[0] = make_float4(h[0], h[1], h[2], h[3]);
      r4[1] = make_float4(h[4], h[5], h[6], h[7]);
    }
  }
}

int launch_residual_boundary(const float* stream_in, const void* branch, int ldb, const float* alpha,
                             const float* beta, const void* post_w, const void* pre_w, void* hidden,
                             float* stream_out, float* router_out, int T, int H, float post_eps, float pre_eps,
                             cudaStream_t stream) {
  return okc_host::launch_k(residual_boundary_kernel, dim3(T), dim3(512), 0, stream, dim3(1), stream_in,
                            reinterpret_cast<const __nv_bfloat16*>(branch), ldb, alpha, beta,
                            reinterpret_cast<const __nv_bfloat16*>(post_w),
                            reinterpret_cast<const __nv_bfloat16*>(pre_w), reinterpret_cast<__nv_bfloat16*>(hidden),
                            stream_out, router_out, H, post_eps, pre_eps);
}

int launch_rmsnorm(const void* x, int ldx, const void* w, void* y, int ldy, int T, int H, float eps,
                   int unit_offset, cudaStream_t stream) {
  return okc_host::launch_k(rmsnorm_kernel, dim3(T), dim3(256), 0, stream, dim3(1),
                            reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                            reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<__nv_bfloat16*>(y), ldy,
                            H, eps, unit_offset);
}

}  // namespace okc
