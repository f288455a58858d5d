// W4A16 (NVFP4 E2M1 weights, bf16 activations) MoE decode: routing, token permutation,
// expert GEMVs and the weighted combine.
//
// route_kernel     logits = bf16(x · Wr^T) in a FIXED fp32 summation order (below), top-k
//                  over the bf16 logits (ties -> lower expert id), softmax weights.
//                  Lane l of the warp computing (t, e) accumulates, with fmaf from 0,
//                  x[256j + 8l + i] * w[e][256j + 8l + i] for j = 0.. (outer), i = 0..7
//                  (inner), then the 32 lanes combine by an xor butterfly (16, 8, 4, 2, 1).
//                  bf16 x bf16 products are exact in fp32, so the CPU oracle reproduces the
//                  logits bit for bit and the expert ids exactly.
// permute_kernel   per local expert, the pair ids p = t*topk + slot in ascending order
//                  (warp ballots over the pair list; deterministic), counts, offsets, tiles.
// gate_up_kernel   inter[p] = bf16(silu(bf16(gs * x·Wg)) * bf16(gs * x·Wu)) for the pairs of
//                  one expert; W13 rows streamed as 16-byte vectors of packed E2M1 codes,
//                  decoded in registers with cvt.rn.f16x2.e2m1x2 and scaled by the e4m3 block
//                  scale (e2m1 * e4m3 is exact in f16), f16 mma.sync m16n8k16 with fp32
//                  accumulate; the per-expert fp32 scale multiplies the accumulator.  Split-K
//                  over a thread-block cluster (DSMEM reduction) when few experts are active.
// down_kernel      y[p] = bf16(gs * inter[p] · W2^T), same decode.
// combine_kernel   out[t] = bf16(sum_slot w[t, slot] * y[t*topk + slot]) over local slots.
// Roofline: HBM, algorithmic bytes = (#experts hit) * (W13 + sf + W2 + sf) bytes + activations.
// Mirrors muse_moe_w4a16/submission.py:163-308 and muse_decode_layer/decode/nvfp4_gemv.py:9-75.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace okc {

// ---------------------------------------------------------------------------------------
// Routing
__global__ void __launch_bounds__(1024) route_kernel(const __nv_bfloat16* __restrict__ x,
                                                    const __nv_bfloat16* __restrict__ wr,
                                                    int32_t* __restrict__ ids, float* __restrict__ wts,
                                                    float* __restrict__ logits_out, int H, int E,
                                                    int topk, int renormalize) {
  extern __shared__ __align__(16) uint8_t rsm[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rsm);
  float* lg = reinterpret_cast<float*>(rsm + (size_t)H * 2);
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8)
    *reinterpret_cast<uint4*>(xs + i) = *reinterpret_cast<const uint4*>(x + (size_t)t * H + i);
  __syncthreads();
  const int nj = H / 256;
  const int nwarps = blockDim.x >> 5;
  for (int e = warp; e < E; e += nwarps) {
    const __nv_bfloat16* we = wr + (size_t)e * H;
    float acc = 0.f;
    for (int j0 = 0; j0 < nj; j0 += 8) {  // 8 row loads in flight before the first use
      uint4 wv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (j0 + q < nj) wv[q] = __ldg(reinterpret_cast<const uint4*>(we + 256 * (j0 + q) + 8 * lane));
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (j0 + q >= nj) break;
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + 256 * (j0 + q) + 8 * lane);
        const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          acc = fmaf(bf16_lo(xa[r]), bf16_lo(wa[r]), acc);
          acc = fmaf(bf16_hi(xa[r]), bf16_hi(wa[r]), acc);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) lg[e] = __bfloat162float(__float2bfloat16_rn(acc));
  }
  __syncthreads();
  if (warp != 0) return;
  if (logits_out)
    for (int e = lane; e < E; e += 32) logits_out[(size_t)t * E + e] = lg[e];
  // top-k by repeated (max value, min index) selection
  constexpr int kMaxPer = 8;  // E <= 256
  float v[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
  }
  float gmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) gmax = fmaxf(gmax, v[i]);
  gmax = warp_max(gmax);
  float chosen_val[16];
  int chosen_id[16];
  for (int s = 0; s < topk; ++s) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    chosen_val[s] = bv;
    chosen_id[s] = bi;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  float denom = 0.f;
  if (renormalize) {
    for (int s = 0; s < topk; ++s) denom += expf(chosen_val[s] - chosen_val[0]);
  } else {
    float part = 0.f;
    for (int e = lane; e < E; e += 32) part += expf(lg[e] - gmax);
    denom = warp_sum(part);
  }
  if (lane < topk) {
    float cv = 0.f;
    int ci = 0;
    for (int s = 0; s < topk; ++s)
      if (s == lane) { cv = chosen_val[s]; ci = chosen_id[s]; }
    const float ref = renormalize ? chosen_val[0] : gmax;
    ids[(size_t)t * topk + lane] = ci;
    wts[(size_t)t * topk + lane] = expf(cv - ref) / denom;
  }
}

// ---------------------------------------------------------------------------------------
// Permutation (single CTA of 1024 threads)
constexpr int kPermMaxPairs = 16384;
constexpr int kPermMaxExperts = 256;

__global__ void __launch_bounds__(1024) permute_kernel(const int32_t* __restrict__ ids, int n,
                                                       int expert_lo, int E, int bm,
                                                       int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ offsets,
                                                       int32_t* __restrict__ pairs,
                                                       int32_t* __restrict__ tiles, int max_tiles,
                                                       int* err) {
  __shared__ int16_t loc[kPermMaxPairs];
  __shared__ int cnt[kPermMaxExperts];
  __shared__ int off[kPermMaxExperts + 1];
  __shared__ int toff[kPermMaxExperts + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    const int e = ids[p] - expert_lo;
    loc[p] = (e >= 0 && e < E) ? (int16_t)e : (int16_t)-1;
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    int c = 0;
    for (int base = 0; base < n; base += 32) {
      const int p = base + lane;
      c += __popc(__ballot_sync(0xffffffffu, p < n && loc[p] == e));
    }
    if (lane == 0) cnt[e] = c;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0, tcarry = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int c = e < E ? cnt[e] : 0;
      const int nt = (c + bm - 1) / bm;
      int v = c, vt = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, v, o), at = __shfl_up_sync(0xffffffffu, vt, o);
        if (lane >= o) { v += a; vt += at; }
      }
      if (e < E) { off[e] = carry + v - c; toff[e] = tcarry + vt - nt; }
      carry += __shfl_sync(0xffffffffu, v, 31);
      tcarry += __shfl_sync(0xffffffffu, vt, 31);
    }
    if (lane == 0) { off[E] = carry; toff[E] = tcarry; }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    counts[e] = cnt[e];
    offsets[e] = off[e];
  }
  if (threadIdx.x == 0) {
    offsets[E] = off[E];
    const int total = toff[E];
    if (total > max_tiles && err) atomicOr(err, OKC_DEVERR_INDEX);
    tiles[0] = min(total, max_tiles);
  }
  for (int e = warp; e < E; e += nw) {
    int run = off[e];
    for (int base = 0; base < n; base += 32) {
      const int p = base + lane;
      const unsigned bal = __ballot_sync(0xffffffffu, p < n && loc[p] == e);
      if (p < n && loc[p] == e) pairs[run + __popc(bal & ((1u << lane) - 1u))] = p;
      run += __popc(bal);
    }
    const int nt = (cnt[e] + bm - 1) / bm;
    for (int j = lane; j < nt; j += 32) {
      const int ti = toff[e] + j;
      if (ti < max_tiles) tiles[1 + ti] = (e << 16) | (j * bm);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Expert GEMVs
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(r) : "r"(byte));
  return r;
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// e4m3 block scale -> f16x2 with both halves equal.
__device__ __forceinline__ uint32_t sf_to_h2(uint32_t sf_byte) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)sf_byte, __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.x << 16);
}

constexpr int kMoeWarps = 8;
constexpr int kMoeRows = kMoeWarps * 16;

// One warp-tile step over 128 K: rows (g, g+8) of one weight matrix, 16 bytes of codes each
// (k in [k0 + 32c, k0 + 32c + 32)), scales for the two 16-groups.  Produces A fragments for
// 8 k16 MMA steps: step s takes codes bytes 2s (slots lo) and 2s+1 (slots hi).
struct WTile {
  uint4 lo, hi;      // codes rows g, g+8
  uint32_t slo, shi; // 2 scale bytes rows g, g+8
};

__device__ __forceinline__ void load_wtile(WTile& t, const uint8_t* rlo, const uint8_t* rhi,
                                           const uint8_t* slo, const uint8_t* shi, int kbyte, int kgrp) {
  t.lo = __ldg(reinterpret_cast<const uint4*>(rlo + kbyte));
  t.hi = __ldg(reinterpret_cast<const uint4*>(rhi + kbyte));
  t.slo = *reinterpret_cast<const uint16_t*>(slo + kgrp);
  t.shi = *reinterpret_cast<const uint16_t*>(shi + kgrp);
}

__device__ __forceinline__ uint32_t code_byte(const uint4& v, int i) {
  const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (w >> (8 * (i & 3))) & 0xffu;
}

// GATED: inter = bf16(silu(g) * u) over rows [0, I) (gate) and [I, 2I) (up) of W13;
// else y rows of W2.  x16: f16 activations [rows][K] (K = H for GATED, I for down).
template <int MT, bool GATED>
__global__ void __launch_bounds__(kMoeWarps * 32) moe_expert_kernel(
    const __half* __restrict__ xin, const int32_t* __restrict__ counts,
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ pairs,
    const uint8_t* __restrict__ w, const uint8_t* __restrict__ sf, const float* __restrict__ gs,
    __half* __restrict__ inter_out, __nv_bfloat16* __restrict__ y_out, int topk, int K, int NR,
    int I, int splits, int expert_lo) {
  constexpr int MTOK = MT * 8;
  constexpr int RED_LD = 2 * MTOK + 1;
  extern __shared__ float mred[];  // [kMoeRows][RED_LD] when splits > 1
  const int e = blockIdx.y;
  const int n_e = counts[e];
  if (n_e == 0) return;  // uniform over the cluster (same expert)
  const int off = offsets[e];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int split = splits > 1 ? (int)(blockIdx.x % splits) : 0;
  const int rb = blockIdx.x / splits;
  const int r0 = rb * kMoeRows + warp * 16;  // output rows (gate index for GATED)
  const int rows_w = GATED ? 2 * I : NR;     // rows of the weight matrix
  const size_t wrow_bytes = (size_t)K / 2, srow_bytes = (size_t)K / 16;
  const uint8_t* we = w + (size_t)e * rows_w * wrow_bytes;
  const uint8_t* se = sf + (size_t)e * rows_w * srow_bytes;
  const float gsc = gs[e];
  const int nck = K / 128;
  const int cps = (nck + splits - 1) / splits;
  const int kc0 = split * cps, kc1 = min(nck, kc0 + cps);

  const int ra = min(r0 + g, NR - 1), rbw = min(r0 + g + 8, NR - 1);
  const uint8_t* wg_lo = we + (size_t)ra * wrow_bytes + 16 * c;
  const uint8_t* wg_hi = we + (size_t)rbw * wrow_bytes + 16 * c;
  const uint8_t* sg_lo = se + (size_t)ra * srow_bytes + 2 * c;
  const uint8_t* sg_hi = se + (size_t)rbw * srow_bytes + 2 * c;
  const uint8_t* wu_lo = wg_lo + (size_t)I * wrow_bytes;
  const uint8_t* wu_hi = wg_hi + (size_t)I * wrow_bytes;
  const uint8_t* su_lo = sg_lo + (size_t)I * srow_bytes;
  const uint8_t* su_hi = sg_hi + (size_t)I * srow_bytes;

  for (int pc = 0; pc < n_e; pc += MTOK) {
    const int ntile = min(MT, (n_e - pc + 7) / 8);
    const __half* xrow[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int i = pc + 8 * t + g;
      int row = 0;
      if (i < n_e) row = GATED ? pairs[off + i] / topk : off + i;
      xrow[t] = xin + (size_t)row * K + 32 * c;
    }
    float ag[MT][4], au[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int q = 0; q < 4; ++q) ag[t][q] = au[t][q] = 0.f;

    WTile tg, tu, ng, nu;
    if (kc0 < kc1) {
      load_wtile(tg, wg_lo, wg_hi, sg_lo, sg_hi, kc0 * 64, kc0 * 8);
      if (GATED) load_wtile(tu, wu_lo, wu_hi, su_lo, su_hi, kc0 * 64, kc0 * 8);
    }
    for (int kc = kc0; kc < kc1; ++kc) {
      if (kc + 1 < kc1) {  // next chunk's codes and scales in flight while this one computes
        load_wtile(ng, wg_lo, wg_hi, sg_lo, sg_hi, (kc + 1) * 64, (kc + 1) * 8);
        if (GATED) load_wtile(nu, wu_lo, wu_hi, su_lo, su_hi, (kc + 1) * 64, (kc + 1) * 8);
      }
      const uint32_t sgl[2] = {sf_to_h2(tg.slo & 0xff), sf_to_h2(tg.slo >> 8)};
      const uint32_t sgh[2] = {sf_to_h2(tg.shi & 0xff), sf_to_h2(tg.shi >> 8)};
      uint32_t sul[2] = {0, 0}, suh[2] = {0, 0};
      if (GATED) {
        sul[0] = sf_to_h2(tu.slo & 0xff); sul[1] = sf_to_h2(tu.slo >> 8);
        suh[0] = sf_to_h2(tu.shi & 0xff); suh[1] = sf_to_h2(tu.shi >> 8);
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int grp = s >> 2;
        const uint32_t a0 = hmul2u(e2m1x2_to_f16x2(code_byte(tg.lo, 2 * s)), sgl[grp]);
        const uint32_t a1 = hmul2u(e2m1x2_to_f16x2(code_byte(tg.hi, 2 * s)), sgh[grp]);
        const uint32_t a2 = hmul2u(e2m1x2_to_f16x2(code_byte(tg.lo, 2 * s + 1)), sgl[grp]);
        const uint32_t a3 = hmul2u(e2m1x2_to_f16x2(code_byte(tg.hi, 2 * s + 1)), sgh[grp]);
        uint32_t u0 = 0, u1 = 0, u2 = 0, u3 = 0;
        if (GATED) {
          u0 = hmul2u(e2m1x2_to_f16x2(code_byte(tu.lo, 2 * s)), sul[grp]);
          u1 = hmul2u(e2m1x2_to_f16x2(code_byte(tu.hi, 2 * s)), suh[grp]);
          u2 = hmul2u(e2m1x2_to_f16x2(code_byte(tu.lo, 2 * s + 1)), sul[grp]);
          u3 = hmul2u(e2m1x2_to_f16x2(code_byte(tu.hi, 2 * s + 1)), suh[grp]);
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if (t < ntile) {
            const uint2 xb = *reinterpret_cast<const uint2*>(xrow[t] + kc * 128 + 4 * s);
            mma_f16_16816(ag[t], a0, a1, a2, a3, xb.x, xb.y);
            if (GATED) mma_f16_16816(au[t], u0, u1, u2, u3, xb.x, xb.y);
          }
        }
      }
      tg = ng;
      if (GATED) tu = nu;
    }

    // epilogue: (optional) cluster reduction, then scale / round / activation / store
    auto finish = [&](int nl, int m, float vg, float vu) {
      const int r = rb * kMoeRows + nl;
      const int i = pc + m;
      if (r >= NR || i >= n_e) return;
      if (GATED) {
        const float hg = __bfloat162float(__float2bfloat16_rn(vg * gsc));
        const float hu = __bfloat162float(__float2bfloat16_rn(vu * gsc));
        const float a = hg / (1.f + expf(-hg)) * hu;
        inter_out[(size_t)(off + i) * I + r] = __float2half_rn(__bfloat162float(__float2bfloat16_rn(a)));
      } else {
        y_out[(size_t)pairs[off + i] * NR + r] = __float2bfloat16_rn(vg * gsc);
      }
    };
    if (splits == 1) {
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          finish(warp * 16 + g + ((q >> 1) << 3), 8 * t + 2 * c + (q & 1), ag[t][q], au[t][q]);
    } else {
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int nl = warp * 16 + g + ((q >> 1) << 3), m = 8 * t + 2 * c + (q & 1);
          mred[nl * RED_LD + m] = ag[t][q];
          mred[nl * RED_LD + MTOK + m] = au[t][q];
        }
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();
      const int total = kMoeRows * MTOK;
      const int per = (total + splits - 1) / splits;
      for (int idx = split * per + (int)threadIdx.x; idx < min(total, (split + 1) * per); idx += blockDim.x) {
        const int m = idx / kMoeRows, nl = idx % kMoeRows;
        float vg = 0.f, vu = 0.f;
        for (int q = 0; q < splits; ++q) {
          const float* peer = cluster.map_shared_rank(mred, q);
          vg += peer[nl * RED_LD + m];
          vu += peer[nl * RED_LD + MTOK + m];
        }
        finish(nl, m, vg, vu);
      }
      cluster.sync();
    }
  }
}

__global__ void __launch_bounds__(256) to_f16_kernel(const __nv_bfloat16* __restrict__ x,
                                                     __half* __restrict__ y, size_t n) {
  for (size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 8; i < n;
       i += (size_t)gridDim.x * blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + i);
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 h = __floats2half2_rn(bf16_lo(a[k]), bf16_hi(a[k]));
      o[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(y + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(64) combine_kernel(const __nv_bfloat16* __restrict__ y,
                                                     const int32_t* __restrict__ ids,
                                                     const float* __restrict__ wts,
                                                     __nv_bfloat16* __restrict__ out, int topk, int H,
                                                     int expert_lo, int E) {
  // grid (T, H / 512): 64 threads x 8 elements (one 16-byte load per slot)
  const int t = blockIdx.x;
  const int d = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (d >= H) return;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < topk; ++s) {
    const int e = ids[(size_t)t * topk + s] - expert_lo;
    if (e < 0 || e >= E) continue;  // slots routed to other ranks were never written
    const float wv = wts[(size_t)t * topk + s];
    const uint4 v = *reinterpret_cast<const uint4*>(y + ((size_t)t * topk + s) * H + d);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      a[2 * k] = fmaf(wv, bf16_lo(u[k]), a[2 * k]);
      a[2 * k + 1] = fmaf(wv, bf16_hi(u[k]), a[2 * k + 1]);
    }
  }
  uint4 o;
  o.x = pack_bf16x2(a[0], a[1]); o.y = pack_bf16x2(a[2], a[3]);
  o.z = pack_bf16x2(a[4], a[5]); o.w = pack_bf16x2(a[6], a[7]);
  *reinterpret_cast<uint4*>(out + (size_t)t * H + d) = o;
}

// ---------------------------------------------------------------------------------------
int launch_moe_route(const void* x, const void* wr, int32_t* ids, float* wts, float* logits,
                     int T, int H, int E, int topk, int renormalize, cudaStream_t stream) {
  const size_t smem = (size_t)H * 2 + (size_t)E * 4;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  route_kernel<<<T, 1024, smem, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                         reinterpret_cast<const __nv_bfloat16*>(wr), ids, wts, logits,
                                         H, E, topk, renormalize);
  return okc_host::launch_status();
}

int launch_moe_permute(const int32_t* ids, int n, int expert_lo, int E, int bm, int32_t* counts,
                       int32_t* offsets, int32_t* pairs, int32_t* tiles, int max_tiles, int* err,
                       cudaStream_t stream) {
  permute_kernel<<<1, 1024, 0, stream>>>(ids, n, expert_lo, E, bm, counts, offsets, pairs, tiles,
                                         max_tiles, err);
  return okc_host::launch_status();
}

template <int MT, bool GATED>
static int launch_expert_t(const __half* xin, const int32_t* counts, const int32_t* offsets,
                           const int32_t* pairs, const void* w, const void* sf, const float* gs,
                           __half* inter, __nv_bfloat16* y, int topk, int K, int NR, int I,
                           int E, int splits, int expert_lo, cudaStream_t stream) {
  const int row_blocks = (NR + kMoeRows - 1) / kMoeRows;
  const size_t smem = splits > 1 ? (size_t)kMoeRows * (2 * MT * 8 + 1) * sizeof(float) : 0;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(moe_expert_kernel<MT, GATED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)((size_t)kMoeRows * (2 * MT * 8 + 1) * sizeof(float)));
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_blocks * splits, E, 1);
  cfg.blockDim = dim3(kMoeWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, moe_expert_kernel<MT, GATED>, xin, counts, offsets, pairs,
                     reinterpret_cast<const uint8_t*>(w), reinterpret_cast<const uint8_t*>(sf), gs,
                     inter, y, topk, K, NR, I, splits, expert_lo);
  return okc_host::launch_status();
}

template <bool GATED>
static int launch_expert(int T, const __half* xin, const int32_t* counts, const int32_t* offsets,
                         const int32_t* pairs, const void* w, const void* sf, const float* gs,
                         __half* inter, __nv_bfloat16* y, int topk, int K, int NR, int I, int E,
                         int splits, int expert_lo, cudaStream_t stream) {
  if (T <= 8)
    return launch_expert_t<1, GATED>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I,
                                     E, splits, expert_lo, stream);
  if (T <= 16)
    return launch_expert_t<2, GATED>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I,
                                     E, splits, expert_lo, stream);
  if (T <= 32)
    return launch_expert_t<4, GATED>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I,
                                     E, splits, expert_lo, stream);
  return launch_expert_t<8, GATED>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I,
                                   E, splits, expert_lo, stream);
}

size_t moe_experts_ws_bytes(int T, int topk, int H, int I) {
  const size_t npairs = (size_t)T * topk;
  size_t b = 256;
  b += ((size_t)T * H * 2 + 255) / 256 * 256;        // x in f16
  b += (npairs * I * 2 + 255) / 256 * 256;            // inter f16 (compact order)
  b += (npairs * H * 2 + 255) / 256 * 256;            // y bf16 (by pair id)
  return b;
}

int launch_moe_experts(const void* x, const int32_t* ids, const float* wts, const int32_t* counts,
                       const int32_t* offsets, const int32_t* pairs, const void* w13,
                       const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                       const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                       int E, void* ws, cudaStream_t stream) {
  uint8_t* base = reinterpret_cast<uint8_t*>(ws) + 256;
  __half* xh = reinterpret_cast<__half*>(base);
  base += ((size_t)T * H * 2 + 255) / 256 * 256;
  __half* inter = reinterpret_cast<__half*>(base);
  base += ((size_t)T * topk * I * 2 + 255) / 256 * 256;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(base);
  const size_t n = (size_t)T * H;
  int blocks = (int)((n / 8 + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  to_f16_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), xh, n);
  int st = okc_host::launch_status();
  if (st) return st;
  // Few active experts (small T): split K over a cluster so that all SMs stream weights.
  const int sp1 = T <= 4 ? 4 : (T <= 16 ? 2 : 1);
  st = launch_expert<true>(T, xh, counts, offsets, pairs, w13, w13_sf, w13_gs, inter, nullptr, topk, H,
                           I, I, E, sp1, expert_lo, stream);
  if (st) return st;
  const int sp2 = T <= 4 ? 2 : 1;
  st = launch_expert<false>(T, inter, counts, offsets, pairs, w2, w2_sf, w2_gs, nullptr, y, topk, I, H,
                            I, E, sp2, expert_lo, stream);
  if (st) return st;
  combine_kernel<<<dim3(T, (H + 511) / 512), 64, 0, stream>>>(y, ids, wts, reinterpret_cast<__nv_bfloat16*>(out),
                                                               topk, H, expert_lo, E);
  return okc_host::launch_status();
}

}  // namespace okc
