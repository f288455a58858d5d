// Skinny BF16 GEMM for decode projections: y[M,N] = x[M,K] · W[N,K]^T (+ residual).
//
// Roofline: HBM-bound on the weight stream (2*N*K bytes per call; x, y are < 1%).
// Design (B200):
//  * Each warp owns 16 weight rows; a CTA of 8 warps owns 128 rows and one K-slice.
//    Lane (g = lane/4, c = lane%4) loads rows g and g+8 of its 16 as 16-byte vectors
//    W[row][k0 + 8c .. k0 + 8c + 7] straight into mma.sync m16n8k16 A fragments.  The
//    K axis is permuted (k-slots {2c,2c+1} <-> physical {8c,8c+1} / {8c+4,8c+5}, slots
//    {2c+8,2c+9} <-> {8c+2,8c+3} / {8c+6,8c+7}); B (= x rows) uses the same permutation,
//    so the product is unchanged while every load is a full 16-byte vector with no
//    shared-memory round trip.  Tokens are the N=8 side of the MMA (MT tiles of 8).
//  * Split-K across S CTAs of one thread-block cluster (S <= 8).  Each CTA writes its
//    fp32 partial tile into its own shared memory; after a cluster barrier every CTA
//    reduces 1/S of the tile by reading all S partials through distributed shared memory
//    (fixed rank order -> deterministic), adds the optional residual, rounds once and
//    stores.  No global workspace, no atomics, no second launch.
// Mirrors muse_decode_layer/decode/projections.py:8-48 (GEMV, split-K partial GEMM and
// the partial reduction) and muse_bf16_proj/projection/kernels/{gemv,gemm,reduce}.py.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace okc {

constexpr int kSkinnyWarps = 8;
constexpr int kSkinnyRows = kSkinnyWarps * 16;  // rows per CTA
constexpr int kSkinnyUnroll = 4;                // 32-wide K chunks per batch of loads

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <int MT>
__global__ void __launch_bounds__(kSkinnyWarps * 32, 2)
    skinny_gemm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                       const __nv_bfloat16* __restrict__ w, int ldw, void* __restrict__ y,
                       int ldy, const __nv_bfloat16* __restrict__ residual, int M, int N, int K,
                       int splits, int chunks_per_split, int out_fp32) {
  constexpr int MTOK = MT * 8;
  constexpr int RED_LD = MTOK + 1;  // padded row of the partial tile (floats)
  extern __shared__ float red[];    // [kSkinnyRows][RED_LD] when splits > 1
  pdl_trigger();
  pdl_wait();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int split = splits > 1 ? (int)(blockIdx.x % splits) : 0;
  const int rb = blockIdx.x / splits;
  const int row0 = rb * kSkinnyRows + warp * 16;

  const int nchunks = (K + 31) >> 5;
  const int kc_begin = split * chunks_per_split;
  const int kc_end = min(nchunks, kc_begin + chunks_per_split);

  // Clamp out-of-range rows to a valid row: their loads stay in bounds and their
  // results are never stored.
  const int r_lo = min(row0 + g, N - 1), r_hi = min(row0 + g + 8, N - 1);
  const __nv_bfloat16* wlo = w + (size_t)r_lo * ldw + 8 * c;
  const __nv_bfloat16* whi = w + (size_t)r_hi * ldw + 8 * c;
  const __nv_bfloat16* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int m = 8 * t + g;
    xvalid[t] = m < M;
    xrow[t] = x + (size_t)(xvalid[t] ? m : 0) * ldx + 8 * c;
  }

  float acc[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  for (int kc = kc_begin; kc < kc_end; kc += kSkinnyUnroll) {
    uint4 a_lo[kSkinnyUnroll], a_hi[kSkinnyUnroll];
#pragma unroll
    for (int u = 0; u < kSkinnyUnroll; ++u) {
      const int k = (kc + u) * 32 + 8 * c;
      if (kc + u < kc_end && k < K) {
        a_lo[u] = ldg_stream(wlo + (size_t)(kc + u) * 32);
        a_hi[u] = ldg_stream(whi + (size_t)(kc + u) * 32);
      } else {
        a_lo[u] = make_uint4(0, 0, 0, 0);
        a_hi[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kSkinnyUnroll; ++u) {
      const int k = (kc + u) * 32 + 8 * c;
      const bool kin = (kc + u < kc_end) && k < K;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        uint4 b = make_uint4(0, 0, 0, 0);
        if (kin && xvalid[t]) b = __ldg(reinterpret_cast<const uint4*>(xrow[t] + (size_t)(kc + u) * 32));
        mma_bf16_16816(acc[t], a_lo[u].x, a_hi[u].x, a_lo[u].y, a_hi[u].y, b.x, b.y);
        mma_bf16_16816(acc[t], a_lo[u].z, a_hi[u].z, a_lo[u].w, a_hi[u].w, b.z, b.w);
      }
    }
  }

  if (splits == 1) {
    // Direct epilogue: rows (row0+g, row0+g+8), tokens (8t+2c, 8t+2c+1).
#pragma unroll
    for (int t = 0; t < MT; ++t) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int n = row0 + g + ((i >> 1) << 3);
        const int m = 8 * t + 2 * c + (i & 1);
        if (n < N && m < M) {
          float v = acc[t][i];
          if (residual) v += __bfloat162float(residual[(size_t)m * ldy + n]);
          if (out_fp32)
            reinterpret_cast<float*>(y)[(size_t)m * ldy + n] = v;
          else
            reinterpret_cast<__nv_bfloat16*>(y)[(size_t)m * ldy + n] = __float2bfloat16_rn(v);
        }
      }
    }
    return;
  }

  // Cluster split-K reduction through distributed shared memory.
#pragma unroll
  for (int t = 0; t < MT; ++t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int nl = warp * 16 + g + ((i >> 1) << 3);
      const int m = 8 * t + 2 * c + (i & 1);
      red[nl * RED_LD + m] = acc[t][i];
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int total = kSkinnyRows * MTOK;
  const int per = (total + splits - 1) / splits;
  const int e_begin = split * per, e_end = min(total, e_begin + per);
  for (int e = e_begin + (int)threadIdx.x; e < e_end; e += blockDim.x) {
    const int m = e / kSkinnyRows, nl = e % kSkinnyRows;
    const int n = rb * kSkinnyRows + nl;
    if (m >= M || n >= N) continue;
    float v = 0.f;
    for (int q = 0; q < splits; ++q) {
      const float* peer = cluster.map_shared_rank(red, q);
      v += peer[nl * RED_LD + m];
    }
    if (residual) v += __bfloat162float(residual[(size_t)m * ldy + n]);
    if (out_fp32)
      reinterpret_cast<float*>(y)[(size_t)m * ldy + n] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(y)[(size_t)m * ldy + n] = __float2bfloat16_rn(v);
  }
  cluster.sync();  // keep this CTA's partial alive until every peer has read it
}

template <int MT>
static int launch_skinny_mt(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                            const void* residual, int M, int N, int K, int out_fp32, int splits,
                            cudaStream_t stream) {
  const int row_blocks = (N + kSkinnyRows - 1) / kSkinnyRows;
  const int nchunks = (K + 31) / 32;
  if (splits <= 0) {
    static int blocks_per_sm = 0;
    if (blocks_per_sm == 0) {
      const size_t smem = (size_t)kSkinnyRows * (MT * 8 + 1) * sizeof(float);
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks_per_sm, skinny_gemm_kernel<MT>,
                                                    kSkinnyWarps * 32, smem);
      if (blocks_per_sm <= 0) blocks_per_sm = 1;
    }
    const int slots = okc_host::num_sms() * blocks_per_sm;
    splits = slots / row_blocks;
    if (splits < 1) splits = 1;
    if (splits > 8) splits = 8;
    // keep at least two 4-chunk batches per split
    while (splits > 1 && nchunks / splits < 2 * kSkinnyUnroll) --splits;
  }
  if (splits > 8 || splits < 1) return OKC_ERR_INVALID;
  const int cps = (nchunks + splits - 1) / splits;
  const size_t smem = splits > 1 ? (size_t)kSkinnyRows * (MT * 8 + 1) * sizeof(float) : 0;

  return okc_host::launch_k(skinny_gemm_kernel<MT>, dim3(row_blocks * splits), dim3(kSkinnyWarps * 32), smem,
                            stream, dim3(splits), reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                            reinterpret_cast<const __nv_bfloat16*>(w), ldw, y, ldy,
                            reinterpret_cast<const __nv_bfloat16*>(residual), M, N, K, splits, cps, out_fp32);
}

// M <= 64 per launch; larger M is issued as several 64-token passes by the caller.
int launch_skinny_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                       const void* residual, int M, int N, int K, int out_fp32, int splits,
                       cudaStream_t stream) {
  if (M <= 8)
    return launch_skinny_mt<1>(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32, splits, stream);
  if (M <= 16)
    return launch_skinny_mt<2>(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32, splits, stream);
  if (M <= 32)
    return launch_skinny_mt<4>(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32, splits, stream);
  if (M <= 64)
    return launch_skinny_mt<8>(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32, splits, stream);
  return OKC_ERR_INVALID;
}

}  // namespace okc
