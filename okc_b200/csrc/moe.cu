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
// combine_postnorm_kernel  the same with Muse's post-expert RMSNorm of each slot first.
// Roofline: HBM, algorithmic bytes = (#experts hit) * (W13 + sf + W2 + sf) bytes + activations.
// Mirrors muse_moe_w4a16/submission.py:163-308 and muse_decode_layer/decode/nvfp4_gemv.py:9-75.
#include <cooperative_groups.h>
#include <stdlib.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace okc {

// ---------------------------------------------------------------------------------------
// Routing
// Top-k of one token's logits lg[0..E) by one warp: repeated (max value, min index) selection,
// softmax over the chosen logits (renormalize) or the full-softmax probabilities of the
// chosen experts; logits_out row written when given.
__device__ void route_topk_warp(const float* lg, int t, int E, int topk, int renormalize, int32_t* ids,
                                float* wts, float* logits_out, int lane) {
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
  route_topk_warp(lg, t, E, topk, renormalize, ids, wts, logits_out, lane);
}

// ---------------------------------------------------------------------------------------
// Permutation (single CTA of 1024 threads)
constexpr int kPermMaxPairs = 16384;
constexpr int kPermMaxExperts = 256;

// O(n) work: warp w owns the pairs [w * per, (w + 1) * per) in 32-pair chunks.  Pass 1 counts the
// warp's pairs per expert (__match_any_sync; the lowest lane of each expert group adds the group's
// size); an exclusive prefix over the warps per expert, then over the experts, gives each
// (warp, expert) its first output slot; pass 2 walks the same chunks in order and writes each
// pair at that slot + its rank among the chunk's earlier pairs of its expert, so every expert's
// list comes out in ascending pair order.
__global__ void __launch_bounds__(1024) permute_kernel(const int32_t* __restrict__ ids, int n,
                                                       int expert_lo, int E, int bm,
                                                       int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ offsets,
                                                       int32_t* __restrict__ pairs,
                                                       int32_t* __restrict__ tiles, int max_tiles,
                                                       int* err) {
  __shared__ int16_t wcnt[32][kPermMaxExperts];  // per (warp, expert): count, then first slot in the expert
  __shared__ int cnt[kPermMaxExperts];
  __shared__ int off[kPermMaxExperts + 1];
  __shared__ int toff[kPermMaxExperts + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wcnt[i / E][i % E] = 0;
  __syncthreads();
  const int per = (n + 31) / 32;
  const int p0 = warp * per, p1 = min(n, p0 + per);
  auto expert_of = [&](int q) {
    if (q >= p1) return -1;
    const int v = ids[q] - expert_lo;
    return (v >= 0 && v < E) ? v : -1;
  };
  for (int base = p0; base < p1; base += 32) {
    const int e = expert_of(base + lane);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) wcnt[warp][e] += (int16_t)__popc(peers);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wcnt[w][e];
      wcnt[w][e] = (int16_t)run;
      run += c;
    }
    cnt[e] = run;
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
  for (int base = p0; base < p1; base += 32) {
    const int q = base + lane;
    const int e = expert_of(q);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) pairs[off[e] + wcnt[warp][e] + __popc(peers & ((1u << lane) - 1u))] = q;
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) wcnt[warp][e] += (int16_t)__popc(peers);
    __syncwarp();
  }
  for (int e = warp; e < E; e += 32) {
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

// One 32-bit word of packed codes (8 values, bytes b0..b3) -> four f16x2 (byte i -> hi, lo pair).
__device__ __forceinline__ void e2m1_word_to_f16x2(uint32_t w, uint32_t& h0, uint32_t& h1, uint32_t& h2, uint32_t& h3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
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
__global__ void __launch_bounds__(kMoeWarps * 32, 1) moe_expert_kernel(
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
        const bool odd = s & 1;
        uint32_t q0, q1, q2, q3, r0, r1, r2, r3;
        e2m1_word_to_f16x2((&tg.lo.x)[s >> 1], q0, q1, q2, q3);
        e2m1_word_to_f16x2((&tg.hi.x)[s >> 1], r0, r1, r2, r3);
        const uint32_t a0 = hmul2u(odd ? q2 : q0, sgl[grp]);
        const uint32_t a1 = hmul2u(odd ? r2 : r0, sgh[grp]);
        const uint32_t a2 = hmul2u(odd ? q3 : q1, sgl[grp]);
        const uint32_t a3 = hmul2u(odd ? r3 : r1, sgh[grp]);
        uint32_t u0 = 0, u1 = 0, u2 = 0, u3 = 0;
        if (GATED) {
          e2m1_word_to_f16x2((&tu.lo.x)[s >> 1], q0, q1, q2, q3);
          e2m1_word_to_f16x2((&tu.hi.x)[s >> 1], r0, r1, r2, r3);
          u0 = hmul2u(odd ? q2 : q0, sul[grp]);
          u1 = hmul2u(odd ? r2 : r0, suh[grp]);
          u2 = hmul2u(odd ? q3 : q1, sul[grp]);
          u3 = hmul2u(odd ? r3 : r1, suh[grp]);
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

// ---------------------------------------------------------------------------------------
// Pipelined expert kernel.  A unit = RT*16 consecutive output rows of one active expert over the
// full K: for GATED the gate rows [r0, r0 + RT*16) and the up rows I + [r0, ...), each one
// contiguous span of codes and one of scales in HBM, moved by cp.async.bulk (1 or 2 matrices x
// (codes + scales)) into an NS-deep shared-memory ring by warp 8.  Warps 0..7 = RT m-tiles x WK
// K-slices: each decodes its rows' codes from shared memory (cvt.rn.f16x2.e2m1x2, x e4m3 scale)
// and runs f16 mma.sync against the expert's token rows of x (L1/L2); the WK partial sums meet in
// shared memory, are scaled by gs, rounded, activated (GATED: silu(g) * u) and stored.
// Persistent grid: every CTA derives the active-expert list from `counts` and takes an equal
// contiguous range of units, so only experts that received tokens are streamed.
template <bool GATED, int RT, int WK, int MT, int NS>
struct MoeCfg {
  static constexpr int ROWS = RT * 16;
  static constexpr int MATS = GATED ? 2 : 1;
  static constexpr int MTOK = MT * 8;
};

template <bool GATED, int RT, int WK, int MT, int NS>
__global__ void __launch_bounds__(288, 1) moe_pipe_kernel(
    const __half* __restrict__ xin, const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ pairs, const uint8_t* __restrict__ w, const uint8_t* __restrict__ sf,
    const float* __restrict__ gs, __half* __restrict__ inter_out, __nv_bfloat16* __restrict__ y_out, int topk,
    int K, int NR, int I, int E, int* err) {
  using C = MoeCfg<GATED, RT, WK, MT, NS>;
  extern __shared__ __align__(128) uint8_t msm[];
  const int code_row = K / 2, sf_row = K / 16;
  const int mat_bytes = C::ROWS * (code_row + sf_row);          // codes then scales of one matrix
  const int stage_bytes = (C::MATS * mat_bytes + 127) / 128 * 128;
  uint8_t* stages = msm;
  float* red = reinterpret_cast<float*>(msm + (size_t)NS * stage_bytes);  // [8 warps][ROWS/RT=16][MTOK][2]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 8 * 16 * C::MTOK * 2);
  uint64_t* empty = full + NS;
  int* act = reinterpret_cast<int*>(empty + NS);  // [E + 1]: active expert list, act[E] = count
  volatile int* abort_flag = act + E + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {  // ordered list of experts with tokens
    int base = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool on = e < E && counts[e] > 0;
      const unsigned bal = __ballot_sync(0xffffffffu, on);
      if (on) act[base + __popc(bal & ((1u << lane) - 1u))] = e;
      base += __popc(bal);
    }
    if (lane == 0) act[E] = base;
  }
  __syncthreads();
  const int rb_per_expert = NR / C::ROWS;
  const int U = act[E] * rb_per_expert;
  const int q = U / (int)gridDim.x, r = U % (int)gridDim.x;
  const int u0 = blockIdx.x * q + min((int)blockIdx.x, r);
  const int u1 = u0 + q + ((int)blockIdx.x < r ? 1 : 0);
  if (u0 >= u1) return;
  const int rows_w = GATED ? 2 * I : NR;

  if (warp == 8) {
    // ------------------------------- producer -------------------------------
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    for (int u = u0; u < u1; ++u) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u, err) && !*abort_flag;
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) { *abort_flag = 1; break; }
      const int e = act[u / rb_per_expert];
      const int r0 = (u % rb_per_expert) * C::ROWS;
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)(C::MATS * mat_bytes));
      __syncwarp();
      uint8_t* dst = stages + (size_t)stage * stage_bytes;
      if (lane < 2 * C::MATS) {
        const int m = lane >> 1, part = lane & 1;  // (matrix, codes|scales)
        const size_t row = (size_t)e * rows_w + r0 + (m ? I : 0);
        const uint8_t* src = part == 0 ? w + row * code_row : sf + row * sf_row;
        const uint32_t bytes = (uint32_t)(C::ROWS * (part == 0 ? code_row : sf_row));
        uint8_t* d = dst + m * mat_bytes + (part == 0 ? 0 : C::ROWS * code_row);
        bulk_g2s(d, src, bytes, &full[stage], pol);
      }
      ++issued;
      if (++stage == NS) { stage = 0; phase ^= 1u; }
    }
    if (lane == 0) {  // make sure this warp's copies have landed before leaving
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < min(issued, NS); ++i) {
        if (--s < 0) { s = NS - 1; ph ^= 1u; }
        if (!mbar_wait(&full[s], ph, err)) break;
      }
    }
    return;
  }

  // -------------------------------- consumers --------------------------------
  const int g = lane >> 2, c = lane & 3;
  const int mt = warp / WK, ks = warp % WK;       // m-tile of the unit, K slice
  const int kslice = K / WK;                      // multiple of 128
  const int nck = kslice / 128;
  int stage = 0;
  uint32_t phase = 0;
  for (int u = u0; u < u1; ++u) {
    const int e = act[u / rb_per_expert];
    const int r0 = (u % rb_per_expert) * C::ROWS;
    const int n_e = counts[e], off = offsets[e];
    const float gsc = gs[e];
    // No early return: after a timed-out wait this warp skips the math but still takes every
    // named barrier below (their count depends only on n_e, the same for all 8 warps).
    const bool ok = *abort_flag ? false : mbar_wait(&full[stage], phase, err);
    const bool skip = !__all_sync(0xffffffffu, ok);
    if (skip) *abort_flag = 1;
    const uint8_t* sbase = stages + (size_t)stage * stage_bytes;
    for (int pc = 0; pc < n_e; pc += C::MTOK) {
      const int ntile = min(MT, (n_e - pc + 7) / 8);
      const __half* xrow[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int i = pc + 8 * t + g;
        int xr = 0;
        if (i < n_e) xr = GATED ? pairs[off + i] / topk : off + i;
        xrow[t] = xin + (size_t)xr * K + ks * kslice + 32 * c;
      }
      float ag[MT][4], au[MT][4];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int z = 0; z < 4; ++z) ag[t][z] = au[t][z] = 0.f;
      // x fragments of a whole 128-chunk (8 MMA steps) come in one batch of 16-byte loads; with
      // MT <= 2 the next chunk's batch is in flight while this chunk computes.
      constexpr bool kPrefetch = MT <= 2;
      uint4 xcur[MT][4], xnext[MT][4];
      auto load_x = [&](uint4 (&dst)[MT][4], int ck) {
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[t][v] = t < ntile ? *reinterpret_cast<const uint4*>(xrow[t] + ck * 128 + 8 * v)
                                  : make_uint4(0, 0, 0, 0);
      };
      if (!skip && nck > 0) load_x(xcur, 0);
      for (int ck = 0; ck < (skip ? 0 : nck); ++ck) {
        const int kb = ks * kslice + ck * 128;   // first k of this 128-chunk
        if (kPrefetch && ck + 1 < nck) load_x(xnext, ck + 1);
        uint4 clo[C::MATS], chi[C::MATS];
        uint32_t slo[C::MATS], shi[C::MATS];
#pragma unroll
        for (int m = 0; m < C::MATS; ++m) {
          const uint8_t* cb = sbase + m * mat_bytes;
          const uint8_t* sb = cb + C::ROWS * code_row;
          const int rl = mt * 16 + g;
          clo[m] = *reinterpret_cast<const uint4*>(cb + (size_t)rl * code_row + kb / 2 + 16 * c);
          chi[m] = *reinterpret_cast<const uint4*>(cb + (size_t)(rl + 8) * code_row + kb / 2 + 16 * c);
          slo[m] = *reinterpret_cast<const uint16_t*>(sb + (size_t)rl * sf_row + kb / 16 + 2 * c);
          shi[m] = *reinterpret_cast<const uint16_t*>(sb + (size_t)(rl + 8) * sf_row + kb / 16 + 2 * c);
        }
        uint32_t sl[C::MATS][2], sh[C::MATS][2];
#pragma unroll
        for (int m = 0; m < C::MATS; ++m) {
          sl[m][0] = sf_to_h2(slo[m] & 0xff); sl[m][1] = sf_to_h2(slo[m] >> 8);
          sh[m][0] = sf_to_h2(shi[m] & 0xff); sh[m][1] = sf_to_h2(shi[m] >> 8);
        }
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8) {
          const int grp = s8 >> 2;
          uint32_t a[C::MATS][4];
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) {
            // word s8/2 of each row holds steps s8 (bytes 0,1) and s8+1 (bytes 2,3)
            const uint32_t wl = (&clo[m].x)[s8 >> 1], wh = (&chi[m].x)[s8 >> 1];
            uint32_t l0, l1, l2, l3, u0_, u1_, u2_, u3_;
            e2m1_word_to_f16x2(wl, l0, l1, l2, l3);
            e2m1_word_to_f16x2(wh, u0_, u1_, u2_, u3_);
            const bool odd = s8 & 1;
            a[m][0] = hmul2u(odd ? l2 : l0, sl[m][grp]);
            a[m][1] = hmul2u(odd ? u2_ : u0_, sh[m][grp]);
            a[m][2] = hmul2u(odd ? l3 : l1, sl[m][grp]);
            a[m][3] = hmul2u(odd ? u3_ : u1_, sh[m][grp]);
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            if (t < ntile) {
              const uint4 xq = xcur[t][s8 >> 1];  // halves 8*(s8/2) .. +7 of this thread's 32
              const uint32_t b0 = (s8 & 1) ? xq.z : xq.x, b1 = (s8 & 1) ? xq.w : xq.y;
              mma_f16_16816(ag[t], a[0][0], a[0][1], a[0][2], a[0][3], b0, b1);
              if (GATED) mma_f16_16816(au[t], a[C::MATS - 1][0], a[C::MATS - 1][1], a[C::MATS - 1][2],
                                       a[C::MATS - 1][3], b0, b1);
            }
          }
        }
        if (ck + 1 < nck) {
          if (kPrefetch) {
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
              for (int v = 0; v < 4; ++v) xcur[t][v] = xnext[t][v];
          } else {
            load_x(xcur, ck + 1);
          }
        }
      }
      // K-slice partials -> shared memory -> the ks == 0 warp of each m-tile finishes
      float* myred = red + ((size_t)warp * 16) * C::MTOK * 2;
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          const int rr = g + ((z >> 1) << 3), mm = 8 * t + 2 * c + (z & 1);
          myred[(rr * C::MTOK + mm) * 2] = ag[t][z];
          myred[(rr * C::MTOK + mm) * 2 + 1] = au[t][z];
        }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (ks == 0 && !skip) {
        for (int idx = lane; idx < 16 * C::MTOK; idx += 32) {
          const int rr = idx / C::MTOK, mm = idx % C::MTOK;
          const int i = pc + mm;
          if (i >= n_e) continue;
          float vg = 0.f, vu = 0.f;
          for (int kw = 0; kw < WK; ++kw) {
            const float* o = red + ((size_t)(mt * WK + kw) * 16 + rr) * C::MTOK * 2 + mm * 2;
            vg += o[0];
            vu += o[1];
          }
          const int rowo = r0 + mt * 16 + rr;
          if (GATED) {
            const float hg = __bfloat162float(__float2bfloat16_rn(vg * gsc));
            const float hu = __bfloat162float(__float2bfloat16_rn(vu * gsc));
            const float act_v = hg / (1.f + expf(-hg)) * hu;
            inter_out[(size_t)(off + i) * I + rowo] = __float2half_rn(__bfloat162float(__float2bfloat16_rn(act_v)));
          } else {
            y_out[(size_t)pairs[off + i] * NR + rowo] = __float2bfloat16_rn(vg * gsc);
          }
        }
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");  // red is reused by the next pair chunk
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == NS) { stage = 0; phase ^= 1u; }
  }
}

template <bool GATED, int RT, int WK, int MT, int NS>
static int launch_moe_pipe_t(const __half* xin, const int32_t* counts, const int32_t* offsets, const int32_t* pairs,
                             const void* w, const void* sf, const float* gs, __half* inter, __nv_bfloat16* y,
                             int topk, int K, int NR, int I, int E, int* err, cudaStream_t stream) {
  using C = MoeCfg<GATED, RT, WK, MT, NS>;
  const int mat_bytes = C::ROWS * (K / 2 + K / 16);
  const int stage_bytes = (C::MATS * mat_bytes + 127) / 128 * 128;
  const size_t smem = (size_t)NS * stage_bytes + 8 * 16 * C::MTOK * 2 * 4 + 2 * NS * 8 + (size_t)(E + 2) * 4;
  if (smem > 232448) return OKC_ERR_INVALID;
  static size_t configured = 0;
  if (smem > configured) {
    if (cudaFuncSetAttribute(moe_pipe_kernel<GATED, RT, WK, MT, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = smem;
  }
  const int grid = okc_host::num_sms();
  moe_pipe_kernel<GATED, RT, WK, MT, NS><<<grid, 288, smem, stream>>>(
      xin, counts, offsets, pairs, reinterpret_cast<const uint8_t*>(w), reinterpret_cast<const uint8_t*>(sf), gs,
      inter, y, topk, K, NR, I, E, err);
  return okc_host::launch_status();
}

// GATED: unit = 16 rows x (gate + up), warps split K in 8 (K % 1024 == 0).  Down: unit = 32 rows,
// 2 m-tiles x 4 K slices (K % 512 == 0).  MT from the token count (a chunk of 8*MT pairs per pass).
template <bool GATED>
static int launch_moe_pipe(int T, const __half* xin, const int32_t* counts, const int32_t* offsets,
                           const int32_t* pairs, const void* w, const void* sf, const float* gs, __half* inter,
                           __nv_bfloat16* y, int topk, int K, int NR, int I, int E, int* err, cudaStream_t stream) {
  if (GATED) {
    if (T <= 8) return launch_moe_pipe_t<true, 1, 8, 1, 2>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
    if (T <= 16) return launch_moe_pipe_t<true, 1, 8, 2, 2>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
    return launch_moe_pipe_t<true, 1, 8, 4, 2>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
  }
  if (T <= 8) return launch_moe_pipe_t<false, 2, 4, 1, 4>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
  if (T <= 16) return launch_moe_pipe_t<false, 2, 4, 2, 4>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
  return launch_moe_pipe_t<false, 2, 4, 4, 4>(xin, counts, offsets, pairs, w, sf, gs, inter, y, topk, K, NR, I, E, err, stream);
}

// ---------------------------------------------------------------------------------------
// Row-owning expert kernel (T <= 64).  A unit = ROWS weight rows of one active expert over the
// full K; its K is streamed in stages of KC = 512: per stage one 2-D TMA box of codes
// [ROWS][256 B] and one of scales [ROWS][32 B] per matrix (16 KB + 2 KB), into a 5-deep ring.
// Warp w owns 16 MMA rows of the unit for the whole K, so its fp32 accumulators finish the
// rows with no cross-warp reduction and no block barrier:
//   GATED: MMA rows 0-7 = gate rows 8w..8w+7, rows 8-15 = the same up rows (one MMA yields
//          both halves of SwiGLU), ROWS = 64;
//   down:  MMA rows = weight rows 16w..16w+15, ROWS = 128.
// Tokens: all of the expert's pairs (<= 64) in tiles of 8, x read from L2 per 128-K chunk.
template <bool GATED, int MTMAX>
struct MoeRowCfg {
  static constexpr int KC = 512;
  static constexpr int ROWS = GATED ? 64 : 128;
  static constexpr int MATS = GATED ? 2 : 1;
  static constexpr int CODE_BOX = ROWS * KC / 2;
  static constexpr int SF_BOX = ROWS * KC / 16;
  static constexpr int WBYTES = MATS * (CODE_BOX + SF_BOX);  // 36 KB of weights
  // The first XR token rows' x for this K chunk ride along in the stage (bulk copies of 1 KB,
  // rows padded to 1040 B so the 8 rows of a fragment load fall in distinct banks); tokens
  // beyond XR are read from L2.
  static constexpr int XR = MTMAX >= 2 ? 16 : 8;
  static constexpr int XROW = KC * 2 + 16;
  static constexpr int STAGE = WBYTES + XR * XROW;
  static constexpr int NS = 196608 / STAGE > 5 ? 5 : 196608 / STAGE;
};

__device__ __forceinline__ void tma_load_2d_u8(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

template <bool GATED, int MTMAX>
__global__ void __launch_bounds__(288, 1) moe_rows_kernel(
    const __grid_constant__ CUtensorMap cmap, const __grid_constant__ CUtensorMap smap,
    const __half* __restrict__ xin, const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ pairs, const float* __restrict__ gs, __half* __restrict__ inter_out,
    __nv_bfloat16* __restrict__ y_out, int topk, int K, int NR, int I, int E, int* err) {
  using C = MoeRowCfg<GATED, MTMAX>;
  extern __shared__ __align__(128) uint8_t msm_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(msm_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + (size_t)C::NS * C::STAGE);
  uint64_t* empty = full + C::NS;
  int* act = reinterpret_cast<int*>(empty + C::NS);  // [E + 1]
  volatile int* abort_flag = act + E + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  pdl_wait();
  if (warp == 0) {  // ordered list of experts with tokens
    int base = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool on = e < E && counts[e] > 0;
      const unsigned bal = __ballot_sync(0xffffffffu, on);
      if (on) act[base + __popc(bal & ((1u << lane) - 1u))] = e;
      base += __popc(bal);
    }
    if (lane == 0) act[E] = base;
  }
  __syncthreads();
  const int rows_w = GATED ? 2 * I : NR;           // rows of one expert in the tensor maps
  const int nrb = (GATED ? I : NR) / C::ROWS;      // row blocks per expert
  const int nkc = K / C::KC;
  const int U = act[E] * nrb;
  const int q = U / (int)gridDim.x, r = U % (int)gridDim.x;
  const int u0 = blockIdx.x * q + min((int)blockIdx.x, r);
  const int u1 = u0 + q + ((int)blockIdx.x < r ? 1 : 0);
  if (u0 >= u1) return;

  if (warp == 8) {
    // ------------------------------- producer -------------------------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int u = u0; u < u1 && !*abort_flag; ++u) {
        const int e = act[u / nrb];
        const int y0 = e * rows_w + (u % nrb) * C::ROWS;
        const int nx = min(counts[e], C::XR), off = offsets[e];
        for (int kc = 0; kc < nkc; ++kc) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1u, err)) { *abort_flag = 1; break; }
          mbar_arrive_expect_tx(&full[stage], (uint32_t)(C::WBYTES + nx * C::KC * 2));
          uint8_t* dst = stages + (size_t)stage * C::STAGE;
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) {
            uint8_t* d = dst + m * (C::CODE_BOX + C::SF_BOX);
            const int yy = y0 + (m ? I : 0);
            tma_load_2d_u8(d, &cmap, kc * (C::KC / 2), yy, &full[stage], pol);
            tma_load_2d_u8(d + C::CODE_BOX, &smap, kc * (C::KC / 16), yy, &full[stage], pol);
          }
          for (int i = 0; i < nx; ++i) {  // x rows of the first XR pairs, this K chunk (L2-resident)
            const int xr = GATED ? pairs[off + i] / topk : off + i;
            bulk_g2s_plain(dst + C::WBYTES + i * C::XROW, xin + (size_t)xr * K + kc * C::KC, C::KC * 2, &full[stage]);
          }
          ++issued;
          if (++stage == C::NS) { stage = 0; phase ^= 1u; }
        }
      }
      int s = stage;  // make sure the copies issued have landed before leaving
      uint32_t ph = phase;
      for (int i = 0; i < min(issued, C::NS); ++i) {
        if (--s < 0) { s = C::NS - 1; ph ^= 1u; }
        if (!mbar_wait(&full[s], ph, err)) break;
      }
    }
    return;
  }

  // -------------------------------- consumers --------------------------------
  const int g = lane >> 2, c = lane & 3;
  // shared-memory rows of this lane: "lo" feeds MMA row g, "hi" MMA row g + 8
  const int row_lo = GATED ? 8 * warp + g : 16 * warp + g;
  const int row_hi = GATED ? 8 * warp + g : 16 * warp + 8 + g;
  const int mat_hi = GATED ? 1 : 0;
  int stage = 0;
  uint32_t phase = 0;
  for (int u = u0; u < u1; ++u) {
    const int e = act[u / nrb];
    const int rb = u % nrb;
    const int n_e = min(counts[e], 8 * MTMAX), off = offsets[e];
    const int ntile = (n_e + 7) >> 3;
    const float gsc = gs[e];
    const __half* xrow[MTMAX];
#pragma unroll
    for (int t = 0; t < MTMAX; ++t) {
      const int i = 8 * t + g;
      int xr = 0;
      if (i < n_e) xr = GATED ? pairs[off + i] / topk : off + i;
      xrow[t] = xin + (size_t)xr * K + 32 * c;
    }
    // NACC independent accumulators per token tile (k16 step s feeds acc[t][s % NACC]) so that
    // consecutive MMAs do not wait on each other; they are summed in a fixed order at the end.
    constexpr int NACC = MTMAX <= 2 ? 4 : 2;
    float acc[MTMAX][NACC][4];
#pragma unroll
    for (int t = 0; t < MTMAX; ++t)
#pragma unroll
      for (int q = 0; q < NACC; ++q) acc[t][q][0] = acc[t][q][1] = acc[t][q][2] = acc[t][q][3] = 0.f;
    bool ok = true;
    for (int kc = 0; kc < nkc; ++kc) {
      ok = ok && !*abort_flag && mbar_wait(&full[stage], phase, err);
      if (__all_sync(0xffffffffu, ok)) {
        const uint8_t* sb = stages + (size_t)stage * C::STAGE;
        const uint8_t* clo_b = sb + (size_t)row_lo * (C::KC / 2);
        const uint8_t* chi_b = sb + mat_hi * (C::CODE_BOX + C::SF_BOX) + (size_t)row_hi * (C::KC / 2);
        const uint8_t* slo_b = sb + C::CODE_BOX + (size_t)row_lo * (C::KC / 16);
        const uint8_t* shi_b = sb + mat_hi * (C::CODE_BOX + C::SF_BOX) + C::CODE_BOX + (size_t)row_hi * (C::KC / 16);
        const uint8_t* xs_b = sb + C::WBYTES + g * C::XROW + 64 * c;  // token row g (+8 per tile)
#pragma unroll 1
        for (int sub = 0; sub < C::KC / 128; ++sub) {
          const int kl = sub * 128;            // k within the stage
          const int kb = kc * C::KC + kl;      // absolute k
          uint4 xq[2][4];                       // x of token tiles t and t+1 (double buffer)
          auto load_x = [&](uint4 (&dst)[4], int t) {
            if (8 * t < C::XR) {  // staged with the weights
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = *reinterpret_cast<const uint4*>(xs_b + 8 * t * C::XROW + kl * 2 + 16 * v);
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = *reinterpret_cast<const uint4*>(xrow[t] + kb + 8 * v);
            }
          };
          load_x(xq[0], 0);
          if (MTMAX > 1 && ntile > 1) load_x(xq[1], 1);
          const uint4 cl = *reinterpret_cast<const uint4*>(clo_b + kl / 2 + 16 * c);
          const uint4 ch = *reinterpret_cast<const uint4*>(chi_b + kl / 2 + 16 * c);
          const uint32_t sl16 = *reinterpret_cast<const uint16_t*>(slo_b + kl / 16 + 2 * c);
          const uint32_t sh16 = *reinterpret_cast<const uint16_t*>(shi_b + kl / 16 + 2 * c);
          const uint32_t sl[2] = {sf_to_h2(sl16 & 0xff), sf_to_h2(sl16 >> 8)};
          const uint32_t sh[2] = {sf_to_h2(sh16 & 0xff), sf_to_h2(sh16 >> 8)};
          uint32_t a[8][4];  // A fragments of the 8 k16 steps of this 128 chunk
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {  // word wi of each row: steps 2wi (bytes 0,1) and 2wi+1 (bytes 2,3)
            uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
            e2m1_word_to_f16x2((&cl.x)[wi], l0, l1, l2, l3);
            e2m1_word_to_f16x2((&ch.x)[wi], h0, h1, h2, h3);
            const int grp = wi >> 1;
            a[2 * wi][0] = hmul2u(l0, sl[grp]);
            a[2 * wi][1] = hmul2u(h0, sh[grp]);
            a[2 * wi][2] = hmul2u(l1, sl[grp]);
            a[2 * wi][3] = hmul2u(h1, sh[grp]);
            a[2 * wi + 1][0] = hmul2u(l2, sl[grp]);
            a[2 * wi + 1][1] = hmul2u(h2, sh[grp]);
            a[2 * wi + 1][2] = hmul2u(l3, sl[grp]);
            a[2 * wi + 1][3] = hmul2u(h3, sh[grp]);
          }
#pragma unroll
          for (int t = 0; t < MTMAX; ++t) {
            if (t < ntile) {
              const uint4* xt = xq[t & 1];
#pragma unroll
              for (int s8 = 0; s8 < 8; ++s8) {
                const uint4 v = xt[s8 >> 1];
                const uint32_t b0 = (s8 & 1) ? v.z : v.x, b1 = (s8 & 1) ? v.w : v.y;
                mma_f16_16816(acc[t][s8 % NACC], a[s8][0], a[s8][1], a[s8][2], a[s8][3], b0, b1);
              }
              if (t + 2 < ntile) load_x(xq[t & 1], t + 2);
            }
          }
        }
      } else {
        ok = false;
        if (lane == 0) *abort_flag = 1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == C::NS) { stage = 0; phase ^= 1u; }
    }
    if (!ok) continue;
    // finish the warp's rows: fragment (g, c) holds tokens 2c, 2c+1 of each tile, rows g / g+8
#pragma unroll
    for (int t = 0; t < MTMAX; ++t) {
      if (t >= ntile) break;
#pragma unroll
      for (int q = 1; q < NACC; ++q)
#pragma unroll
        for (int z = 0; z < 4; ++z) acc[t][0][z] += acc[t][q][z];
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int i = 8 * t + 2 * c + e2;
        if (i >= n_e) continue;
        if (GATED) {
          const float hg = __bfloat162float(__float2bfloat16_rn(acc[t][0][e2] * gsc));
          const float hu = __bfloat162float(__float2bfloat16_rn(acc[t][0][2 + e2] * gsc));
          const float act_v = hg / (1.f + expf(-hg)) * hu;
          inter_out[(size_t)(off + i) * I + rb * C::ROWS + 8 * warp + g] =
              __float2half_rn(__bfloat162float(__float2bfloat16_rn(act_v)));
        } else {
          __nv_bfloat16* yr = y_out + (size_t)pairs[off + i] * NR + rb * C::ROWS + 16 * warp + g;
          yr[0] = __float2bfloat16_rn(acc[t][0][e2] * gsc);
          yr[8] = __float2bfloat16_rn(acc[t][0][2 + e2] * gsc);
        }
      }
    }
  }
}

static bool make_u8_map(CUtensorMap* m, const void* base, long long inner, long long rows, int box_x, int box_y) {
  auto fn = tensor_map_encoder();
  if (!fn || !okc_host::aligned16(base) || inner % 16 || rows <= 0 || rows >= (1LL << 31)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Shapes the row-owning kernel takes: K a multiple of 512, whole row blocks, <= 64 tokens.
static bool moe_rows_ok(int T, int H, int I) {
  return T <= 64 && H % 512 == 0 && I % 512 == 0 && I % MoeRowCfg<true, 1>::ROWS == 0 &&
         H % MoeRowCfg<false, 1>::ROWS == 0 && tensor_map_encoder() != nullptr;
}

template <bool GATED, int MTMAX>
static int launch_moe_rows_t(const void* w, const void* sf, int E, const __half* xin, const int32_t* counts,
                             const int32_t* offsets, const int32_t* pairs, const float* gs, __half* inter,
                             __nv_bfloat16* y, int topk, int K, int NR, int I, int* err, cudaStream_t stream) {
  using C = MoeRowCfg<GATED, MTMAX>;
  const long long rows = (long long)E * (GATED ? 2 * I : NR);
  CUtensorMap cm, sm;
  if (!make_u8_map(&cm, w, K / 2, rows, C::KC / 2, C::ROWS) || !make_u8_map(&sm, sf, K / 16, rows, C::KC / 16, C::ROWS))
    return OKC_ERR_INVALID;
  const size_t smem = 128 + (size_t)C::NS * C::STAGE + 2 * C::NS * 8 + (size_t)(E + 2) * 4;
  if (smem > 232448) return OKC_ERR_INVALID;
  static size_t configured = 0;
  if (smem > configured) {
    if (cudaFuncSetAttribute(moe_rows_kernel<GATED, MTMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = smem;
  }
  return okc_host::launch_k(moe_rows_kernel<GATED, MTMAX>, dim3(okc_host::num_sms()), dim3(288), smem, stream,
                            dim3(1), cm, sm, xin, counts, offsets, pairs, gs, inter, y, topk, K, NR, I, E, err);
}

template <bool GATED>
static int launch_moe_rows(int T, const void* w, const void* sf, int E, const __half* xin, const int32_t* counts,
                           const int32_t* offsets, const int32_t* pairs, const float* gs, __half* inter,
                           __nv_bfloat16* y, int topk, int K, int NR, int I, int* err, cudaStream_t stream) {
  if (T <= 8) return launch_moe_rows_t<GATED, 1>(w, sf, E, xin, counts, offsets, pairs, gs, inter, y, topk, K, NR, I, err, stream);
  if (T <= 16) return launch_moe_rows_t<GATED, 2>(w, sf, E, xin, counts, offsets, pairs, gs, inter, y, topk, K, NR, I, err, stream);
  if (T <= 32) return launch_moe_rows_t<GATED, 4>(w, sf, E, xin, counts, offsets, pairs, gs, inter, y, topk, K, NR, I, err, stream);
  return launch_moe_rows_t<GATED, 8>(w, sf, E, xin, counts, offsets, pairs, gs, inter, y, topk, K, NR, I, err, stream);
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
                                                     void* __restrict__ out, int topk, int H,
                                                     int expert_lo, int E, int out_fp32) {
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
  if (out_fp32) {  // this rank's share of an expert-parallel sum, reduced across ranks later
    float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * H + d);
    o4[0] = make_float4(a[0], a[1], a[2], a[3]);
    o4[1] = make_float4(a[4], a[5], a[6], a[7]);
    return;
  }
  uint4 o;
  o.x = pack_bf16x2(a[0], a[1]); o.y = pack_bf16x2(a[2], a[3]);
  o.z = pack_bf16x2(a[4], a[5]); o.w = pack_bf16x2(a[6], a[7]);
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * H + d) = o;
}

__device__ __forceinline__ float bf16_rn(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Post-expert RMSNorm and weighted sum (muse_moe_w4a16/submission.py:295-308): per local slot
// scaled = bf16(y * gain) (gain = 1 + post_norm_w, fp32), inv = rsqrt(sum(scaled^2) / H + eps),
// out[t] = sum over local slots of (w * inv) * scaled.  One CTA of 256 threads per token, H <= 8192
// (four 16-byte vectors a thread), topk <= 16.  Pass 1 reduces every slot's sum of squares; pass 2
// re-reads the slot rows, just written by the down projection and still in L2.
constexpr int kPostVec = 4;

__global__ void __launch_bounds__(256) combine_postnorm_kernel(const __nv_bfloat16* __restrict__ y,
                                                               const int32_t* __restrict__ ids,
                                                               const float* __restrict__ wts,
                                                               const float* __restrict__ gain,
                                                               void* __restrict__ out, int topk, int H,
                                                               int expert_lo, int E, float eps, int out_fp32) {
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float red[8][16];
  __shared__ float coef[16];
  float g[kPostVec][8];
#pragma unroll
  for (int j = 0; j < kPostVec; ++j) {
    const int i = (j * 256 + tid) * 8;
    if (i < H) {
      const float4 a = *reinterpret_cast<const float4*>(gain + i);
      const float4 b = *reinterpret_cast<const float4*>(gain + i + 4);
      g[j][0] = a.x; g[j][1] = a.y; g[j][2] = a.z; g[j][3] = a.w;
      g[j][4] = b.x; g[j][5] = b.y; g[j][6] = b.z; g[j][7] = b.w;
    }
  }
  for (int s = 0; s < topk; ++s) {
    const int e = ids[(size_t)t * topk + s] - expert_lo;
    float p = 0.f;
    if (e >= 0 && e < E) {  // slots routed to other ranks were never written
      const __nv_bfloat16* row = y + ((size_t)t * topk + s) * H;
#pragma unroll
      for (int j = 0; j < kPostVec; ++j) {
        const int i = (j * 256 + tid) * 8;
        if (i >= H) break;
        const uint4 v = *reinterpret_cast<const uint4*>(row + i);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a = bf16_rn(__fmul_rn(bf16_lo(u[k]), g[j][2 * k]));
          const float b = bf16_rn(__fmul_rn(bf16_hi(u[k]), g[j][2 * k + 1]));
          p = fmaf(a, a, p);
          p = fmaf(b, b, p);
        }
      }
    }
    p = warp_sum(p);
    if (lane == 0) red[warp][s] = p;
  }
  __syncthreads();
  if (tid < topk) {
    const int e = ids[(size_t)t * topk + tid] - expert_lo;
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w][tid];
    coef[tid] = (e >= 0 && e < E) ? wts[(size_t)t * topk + tid] * rsqrtf(tot / (float)H + eps) : 0.f;
  }
  __syncthreads();
  float acc[kPostVec][8];
#pragma unroll
  for (int j = 0; j < kPostVec; ++j)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[j][k] = 0.f;
  for (int s = 0; s < topk; ++s) {
    const int e = ids[(size_t)t * topk + s] - expert_lo;
    if (e < 0 || e >= E) continue;
    const float c = coef[s];
    const __nv_bfloat16* row = y + ((size_t)t * topk + s) * H;
#pragma unroll
    for (int j = 0; j < kPostVec; ++j) {
      const int i = (j * 256 + tid) * 8;
      if (i >= H) break;
      const uint4 v = *reinterpret_cast<const uint4*>(row + i);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[j][2 * k] = fmaf(bf16_rn(__fmul_rn(bf16_lo(u[k]), g[j][2 * k])), c, acc[j][2 * k]);
        acc[j][2 * k + 1] = fmaf(bf16_rn(__fmul_rn(bf16_hi(u[k]), g[j][2 * k + 1])), c, acc[j][2 * k + 1]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kPostVec; ++j) {
    const int i = (j * 256 + tid) * 8;
    if (i >= H) break;
    if (out_fp32) {  // this rank's share of an expert-parallel sum
      float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * H + i);
      o4[0] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
      o4[1] = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
    } else {
      uint4 o;
      o.x = pack_bf16x2(acc[j][0], acc[j][1]); o.y = pack_bf16x2(acc[j][2], acc[j][3]);
      o.z = pack_bf16x2(acc[j][4], acc[j][5]); o.w = pack_bf16x2(acc[j][6], acc[j][7]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * H + i) = o;
    }
  }
}

static int launch_combine(const __nv_bfloat16* y, const int32_t* ids, const float* wts, const float* gain,
                          float eps, void* out, int T, int topk, int H, int expert_lo, int E, int out_fp32,
                          cudaStream_t stream) {
  if (gain)
    combine_postnorm_kernel<<<T, 256, 0, stream>>>(y, ids, wts, gain, out, topk, H, expert_lo, E, eps, out_fp32);
  else
    combine_kernel<<<dim3(T, (H + 511) / 512), 64, 0, stream>>>(y, ids, wts, out, topk, H, expert_lo, E, out_fp32);
  return okc_host::launch_status();
}


int launch_moe_route(const void* x, const void* wr, int32_t* ids, float* wts, float* logits,
                     int T, int H, int E, int topk, int renormalize, cudaStream_t stream) {
  // One CTA per token.  (An 8-CTA cluster per 8 tokens sharing router rows through distributed
  // shared memory measured slower at T = 8..256 on B200: 12.6-24.5 vs 10.3-20.3 us.)
  const size_t smem = (size_t)H * 2 + (size_t)E * 4;
  if (smem > 232448) return OKC_ERR_INVALID;
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    if (cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = smem;
  }
  route_kernel<<<T, 1024, smem, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                         reinterpret_cast<const __nv_bfloat16*>(wr), ids, wts, logits,
                                         H, E, topk, renormalize);
  return okc_host::launch_status();
}

// Muse routing (muse_prefill_layer/submission.py:179-184, FusedMuseSparkRouting with
// route_scale 1, router_output_multiplier 0.1767766952966369, division eps 1e-15): one warp per
// token; score = sigmoid(logit * scale) in fp32; the top-k of score + bias (the bias only
// chooses; ties -> lower expert id); weight = score / (sum of the chosen scores + eps) *
// route_scale.  With `lo` the logit is lo-added first (logits[t][e] + lo[t][e]: the two halves of
// the fp32 router split into bf16 hi and lo parts, high += low as the reference's `_gemm`).
__global__ void __launch_bounds__(256) route_sigmoid_kernel(const float* __restrict__ logits, int ld,
                                                            const float* __restrict__ lo,
                                                            const float* __restrict__ bias, int32_t* __restrict__ ids,
                                                            float* __restrict__ wts, float* __restrict__ logits_out,
                                                            int T, int E, int topk, float scale, float eps,
                                                            float route_scale) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  constexpr int kMaxPer = 8;  // E <= 256
  float sc[kMaxPer], key[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    sc[i] = 0.f;
    key[i] = -INFINITY;
    if (e < E) {
      float z = logits[(size_t)t * ld + e];
      if (lo) z += lo[(size_t)t * ld + e];
      if (logits_out) logits_out[(size_t)t * E + e] = z;
      sc[i] = 1.f / (1.f + expf(-(z * scale)));
      key[i] = bias ? sc[i] + bias[e] : sc[i];
    }
  }
  float chosen = 0.f, sum = 0.f;
  int cid = 0;
  for (int s = 0; s < topk; ++s) {
    float bv = -INFINITY, bs = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (key[i] > bv || (key[i] == bv && e < bi))) { bv = key[i]; bi = e; bs = sc[i]; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; bs = os; }
    }
    sum += bs;  // in selection order, the same on every lane
    if (lane == s) { chosen = bs; cid = bi; }
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (lane + 32 * i == bi) key[i] = -INFINITY;
  }
  if (lane < topk) {
    ids[(size_t)t * topk + lane] = cid;
    wts[(size_t)t * topk + lane] = chosen / (sum + eps) * route_scale;
  }
}

int launch_route_sigmoid(const float* logits, int ld, const float* lo, const float* bias, int32_t* ids, float* wts,
                         float* logits_out, int T, int E, int topk, float scale, float eps, float route_scale,
                         cudaStream_t stream) {
  return okc_host::launch_k(route_sigmoid_kernel, dim3((T + 7) / 8), dim3(256), 0, stream, dim3(1), logits, ld, lo,
                            bias, ids, wts, logits_out, T, E, topk, scale, eps, route_scale);
}

// out[t][e] = y[t][e] + y[t][E + e]: the fp32 router logits from the GEMM of x with the stacked
// bf16 hi / lo halves of the router (two independent fp32 accumulations, then high += low).
__global__ void __launch_bounds__(256) add_halves_kernel(const float* __restrict__ y, float* __restrict__ out,
                                                         int ldo, int T, int E) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * E) return;
  const int t = i / E, e = i - t * E;
  out[(size_t)t * ldo + e] = y[(size_t)t * 2 * E + e] + y[(size_t)t * 2 * E + E + e];
}

int launch_add_halves(const float* y, float* out, int ldo, int T, int E, cudaStream_t stream) {
  return okc_host::launch_k(add_halves_kernel, dim3((T * E + 255) / 256), dim3(256), 0, stream, dim3(1), y, out, ldo,
                            T, E);
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
  b += (npairs * H * 2 + 255) / 256 * 256;            // x in f16: per token, or gathered per pair
  b += (npairs * I * 2 + 255) / 256 * 256;            // inter f16 (compact order)
  b += (npairs * H * 2 + 255) / 256 * 256;            // y bf16 (by pair id)
  b += (npairs * 4 + 255) / 256 * 256;                // per-pair activation scales (gate/up)
  b += (npairs * I * 2 + 255) / 256 * 256;            // inter as scaled f16 (tcgen05 down GEMM)
  b += (npairs * 4 + 255) / 256 * 256;                // its per-pair scales
  return b;
}

// The tcgen05 expert kernels (moe_tc.cu) from this many tokens on; OKC_MOE_TC=0/1 forces
// either family (tuning and tests).
constexpr int kMoeTcMinT = 16;

static int moe_tc_choice(int T) {
  const char* e = getenv("OKC_MOE_TC");
  if (e && (e[0] == '0' || e[0] == '1')) return e[0] - '0';
  return T >= kMoeTcMinT ? 1 : 0;
}

int launch_moe_experts(const void* x, const int32_t* ids, const float* wts, const int32_t* counts,
                       const int32_t* offsets, const int32_t* pairs, const void* w13,
                       const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                       const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                       int E, void* ws, cudaStream_t stream, int out_fp32, const float* post_gain,
                       float post_eps) {
  const size_t npairs = (size_t)T * topk;
  uint8_t* base = reinterpret_cast<uint8_t*>(ws) + 256;
  __half* xh = reinterpret_cast<__half*>(base);
  base += (npairs * H * 2 + 255) / 256 * 256;
  __half* inter = reinterpret_cast<__half*>(base);
  base += (npairs * I * 2 + 255) / 256 * 256;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(base);
  base += (npairs * H * 2 + 255) / 256 * 256;
  float* rs = reinterpret_cast<float*>(base);
  base += (npairs * 4 + 255) / 256 * 256;
  __half* inter_h = reinterpret_cast<__half*>(base);
  base += (npairs * I * 2 + 255) / 256 * 256;
  float* rs2 = reinterpret_cast<float*>(base);
  int* err = reinterpret_cast<int*>(ws);
  int st;
  if (moe_tc_choice(T) && moe_tc_ok(H, I, E)) {
    __nv_bfloat16* inter_b = reinterpret_cast<__nv_bfloat16*>(inter);
    st = launch_moe_rows_f16(x, pairs, offsets, E, topk, H, (int)npairs, xh, rs, stream);
    if (st) return st;
    st = launch_moe_tc<true>(w13, w13_sf, E, xh, (int)npairs, rs, counts, offsets, pairs, w13_gs, inter_b, nullptr,
                             H, I, I, err, stream);
    if (st) return st;
    st = launch_moe_rows_f16(inter_b, pairs, offsets, E, 0, I, (int)npairs, inter_h, rs2, stream);
    if (st) return st;
    st = launch_moe_tc<false>(w2, w2_sf, E, inter_h, (int)npairs, rs2, counts, offsets, pairs, w2_gs, nullptr, y,
                              I, H, I, err, stream);
    if (st) return st;
    return launch_combine(y, ids, wts, post_gain, post_eps, out, T, topk, H, expert_lo, E, out_fp32, stream);
  }
  const size_t n = (size_t)T * H;
  int blocks = (int)((n / 8 + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  to_f16_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), xh, n);
  st = okc_host::launch_status();
  if (st) return st;
  const int pipe_env = getenv("OKC_MOE_PIPE") ? atoi(getenv("OKC_MOE_PIPE")) : 2;
  if (pipe_env == 2 && moe_rows_ok(T, H, I)) {
    st = launch_moe_rows<true>(T, w13, w13_sf, E, xh, counts, offsets, pairs, w13_gs, inter, nullptr, topk, H, I, I,
                               err, stream);
    if (st) return st;
    st = launch_moe_rows<false>(T, w2, w2_sf, E, inter, counts, offsets, pairs, w2_gs, nullptr, y, topk, I, H, I,
                                err, stream);
    if (st) return st;
    return launch_combine(y, ids, wts, post_gain, post_eps, out, T, topk, H, expert_lo, E, out_fp32, stream);
  }
  // Measured on B200: the pipelined kernel wins up to 64 tokens, the per-expert kernel above.
  const bool pipe_ok = pipe_env && T <= 64 && H % 1024 == 0 && I % 512 == 0 && I % 16 == 0 && H % 32 == 0 &&
                       (size_t)16 * 2 * (H / 2 + H / 16) * 2 < 200000;
  if (pipe_ok) {
    st = launch_moe_pipe<true>(T, xh, counts, offsets, pairs, w13, w13_sf, w13_gs, inter, nullptr, topk, H, I, I, E,
                               err, stream);
    if (st) return st;
    st = launch_moe_pipe<false>(T, inter, counts, offsets, pairs, w2, w2_sf, w2_gs, nullptr, y, topk, I, H, I, E,
                                err, stream);
    if (st) return st;
  } else {
    // Few active experts (small T): split K over a cluster so that all SMs stream weights.
    const int sp1 = T <= 4 ? 4 : (T <= 16 ? 2 : 1);
    st = launch_expert<true>(T, xh, counts, offsets, pairs, w13, w13_sf, w13_gs, inter, nullptr, topk, H,
                             I, I, E, sp1, expert_lo, stream);
    if (st) return st;
    const int sp2 = T <= 4 ? 2 : 1;
    st = launch_expert<false>(T, inter, counts, offsets, pairs, w2, w2_sf, w2_gs, nullptr, y, topk, I, H,
                              I, E, sp2, expert_lo, stream);
    if (st) return st;
  }
  return launch_combine(y, ids, wts, post_gain, post_eps, out, T, topk, H, expert_lo, E, out_fp32, stream);
}

}  // namespace okc
