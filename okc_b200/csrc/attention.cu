// Paged FP8-KV attention decode (q_len = 1) and the fused RoPE + FP8 KV-append.
//
// KV cache layout (the reference's, muse_decode_layer/decode/spec.py:48-49):
//   k_cache / v_cache  e4m3 [num_pages][P][Hkv][D]   (one token row = Hkv*D bytes)
// so a run of tokens of one page is ONE contiguous span holding every KV head.
//
// attn_decode_kernel (roofline: HBM, algorithmic bytes = sum_b len_b * Hkv * D * 2):
//  * Work = all sequences' tokens cut into "units" of TS = 32 * 8/Hkv tokens; the units
//    are split evenly over a persistent grid (stream-K), so ragged context lengths stay
//    balanced.  A CTA that crosses a sequence boundary flushes a partial (m, l, acc).
//  * Warp 8 is the producer: per unit it looks up the page table and issues one
//    cp.async.bulk per (page, K|V) span into a 3-stage shared-memory ring (mbarrier
//    complete_tx), with an L2 evict-first hint (the cache is streamed once).
//  * Warps 0..7 are consumers: warp w attends KV head w % Hkv over the 32-token sub-tile
//    w / Hkv of each unit.  QK^T and PV run as e4m3 mma.sync m16n8k32 directly on the
//    cache bytes (no per-element dequant): the query rows are carried as two e4m3 terms
//    q ~= (q1 + q2/16) * 2^-a (a per row), which fill the 16 MMA rows (8 query heads x 2
//    terms) and keep ~8 significant bits, the precision of the bf16 query; likewise the
//    probabilities p ~= (p1 + p2/16) / 256.  k_scale / v_scale / sm_scale are applied in
//    fp32 to the scores and to the merged output.  Online softmax in fp32 (exp2 domain).
//  * K fragments are 16-byte shared loads (K-axis permutation, see common.cuh); V
//    fragments are 16-byte loads of 4 token rows, transposed 4x4 in registers with PRMT.
// attn_merge_kernel: deterministic log-sum-exp merge of the partials of each sequence.
//
// Mirrors muse_attention_decode/submission.py:100-351 (tile loop, online softmax,
// split partials and merge) and muse_prefill_layer/submission.py:137-176 (semantics).
#include "attention_common.cuh"

namespace okc {

template <int D, int HKV>
struct AttnCfg {
  static constexpr int NSUB = 8 / HKV;          // 32-token sub-tiles per unit
  static constexpr int TS = 32 * NSUB;          // tokens per unit (stage)
  static constexpr int ROW = HKV * D;           // bytes per token row
  static constexpr int KV_BYTES = TS * ROW;     // bytes of K (or V) per stage
  static constexpr int STAGE = 2 * KV_BYTES;
  static constexpr int NS = (196608 / STAGE) > 4 ? 4 : (196608 / STAGE);
  static constexpr int RL = D / 8;              // bytes per K run / V run per lane
  static constexpr int KSTEPS = D / 32;         // k32 MMA steps over the head dim
  static constexpr int DB = D / 8;              // n8 blocks over the head dim (PV)
  static constexpr int THREADS = 9 * 32;
};


// 4x4 byte transpose: out_i = (w0.byte_i, w1.byte_i, w2.byte_i, w3.byte_i).
__device__ __forceinline__ void transpose4x4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                             uint32_t& o0, uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  const uint32_t t0 = prmt(w0, w1, 0x5140), t1 = prmt(w2, w3, 0x5140);
  const uint32_t t2 = prmt(w0, w1, 0x7362), t3 = prmt(w2, w3, 0x7362);
  o0 = prmt(t0, t1, 0x5410);
  o1 = prmt(t0, t1, 0x7632);
  o2 = prmt(t2, t3, 0x5410);
  o3 = prmt(t2, t3, 0x7632);
}

// RL bytes (8, 16 or 32) of one token row from shared memory as 32-bit words, 8/16-byte loads.
template <int RL>
__device__ __forceinline__ void ld_run(const uint8_t* p, uint32_t (&w)[RL / 4]) {
  if constexpr (RL == 8) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    w[0] = x.x; w[1] = x.y;
  } else {
#pragma unroll
    for (int i = 0; i < RL / 16; ++i) {
      const uint4 x = *reinterpret_cast<const uint4*>(p + 16 * i);
      w[4 * i] = x.x; w[4 * i + 1] = x.y; w[4 * i + 2] = x.z; w[4 * i + 3] = x.w;
    }
  }
}

// TMA gather of 4 rows of a 2-D map (row indices r0..r3, x = 0) into 4 consecutive rows at dst.
// The map's box is one row high.  Rows outside the map (a bad page id) read zeros.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, const int (&r)[4], uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile::gather4.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

// The kernel body; G4 compiles the TMA gather4 page fetch in (attn_decode_g4_kernel, maps
// given), else the producer only issues bulk copies (attn_decode_kernel): an instantiation with
// the gather code measured ~1.5x slower on 16 KB pages that never take it (C4: 382 vs 248 us).
template <int D, int HKV, bool G4>
__device__ __forceinline__ void attn_decode_body(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                                 const AttnArgs& a) {
  using C = AttnCfg<D, HKV>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NS * C::STAGE);
  uint64_t* empty = full + C::NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::NS);
  int* prefix = const_cast<int*>(abort_flag) + 4;

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
  unit_prefix(a.seq_lens, a.B, C::TS, a.window, 1, prefix);
  __syncthreads();
  if (blockIdx.x == 0)  // for the merge kernel
    for (int i = threadIdx.x; i <= a.B; i += blockDim.x) a.ws_prefix[i] = prefix[i];

  const int U = prefix[a.B];
  int u0, u1;
  unit_range(U, a.num_ctas, blockIdx.x, u0, u1);
  if (u0 >= u1) return;

  if (warp == 8) {
    // ------------------------------- producer -------------------------------------
    // The page-table entries of unit u+1 are loaded (lane sg: the unit's sg-th page span)
    // while unit u waits for its ring slot, so the lookup latency is off the critical path.
    const uint64_t pol = l2_evict_first_policy();
    struct Span { int row, t0, t_end, p_first, nseg, page; };
    auto lookup = [&](int u, int bb) {
      Span f;
      const int len = a.seq_lens[bb];
      f.row = bb / a.q_per_seq;
      f.t0 = seq_origin(len, a.window, 1) + (u - prefix[bb]) * C::TS;
      f.t_end = min(len, f.t0 + C::TS);
      f.p_first = f.t0 / a.P;
      f.nseg = (f.t_end - 1) / a.P - f.p_first + 1;
      const int lp = f.p_first + lane;
      f.page = (lane < f.nseg && lp < a.table_ld) ? a.page_table[(size_t)f.row * a.table_ld + lp] : -1;
      return f;
    };
    auto page_of = [&](const Span& f, int sg) {
      if (sg < 32) return f.page;  // (lane == sg)
      const int lp = f.p_first + sg;
      return lp < a.table_ld ? a.page_table[(size_t)f.row * a.table_ld + lp] : -1;
    };
    int b = find_seq(prefix, a.B, u0);
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    Span nxt = lookup(u0, b);
    for (int u = u0; u < u1; ++u) {
      if (*abort_flag) break;
      const Span cur = nxt;
      if (u + 1 < u1) {
        while (prefix[b + 1] <= u + 1) ++b;
        nxt = lookup(u + 1, b);
      }
      uint32_t my_bytes = 0;
      for (int sg = lane; sg < cur.nseg; sg += 32) {
        const int lp = cur.p_first + sg;
        const int page = page_of(cur, sg);
        const int lo = max(cur.t0, lp * a.P), hi = min(cur.t_end, (lp + 1) * a.P);
        if (page >= 0 && page < a.num_pages) my_bytes += 2u * (uint32_t)(hi - lo) * C::ROW;
        else atomicOr(a.err, OKC_DEVERR_PAGE);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) my_bytes += __shfl_xor_sync(0xffffffffu, my_bytes, o);
      // Small pages (one or two 2 KB rows: one or two KV heads of 16 tokens; or a whole page
      // below 2 KB, e.g. one token at page size 1), units starting on a page: TMA gather4
      // fetches 4 rows per instruction, where a bulk copy per page pays the copy engine's fixed
      // cost per copy (measured: 2 KB pages 5.4 vs 4.0 TB/s over 148 SMs; 128-byte pages are
      // bound by that cost at ~0.4 TB/s).  The row count is padded to a multiple of 4 with the
      // last row (the extra tokens are masked).
      const int g4_rows = (G4 && a.g4_rpp > 0) ? cur.nseg * a.g4_rpp : 0;
      const int g4_ops = (g4_rows + 3) >> 2;
      if (g4_rows) my_bytes = (uint32_t)g4_ops * 4u * (uint32_t)a.g4_rb * 2u;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u, a.err);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) { *abort_flag = 1; break; }
      if (lane == 0) {
        if (my_bytes) mbar_arrive_expect_tx(&full[stage], my_bytes);
        else mbar_arrive(&full[stage]);
      }
      __syncwarp();
      uint8_t* sk = stages + (size_t)stage * C::STAGE;
      uint8_t* sv = sk + C::KV_BYTES;
      // op o (lane o % 32, pass o / 32, warp-uniform passes for the shuffles) gathers rows
      // 4o .. 4o + 3; segments past the first 32 read their page id from the table
      for (int o0 = 0; o0 < g4_ops; o0 += 32) {
        const int o = o0 + lane;
        int rid[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = min(4 * o + i, g4_rows - 1);
          const int sg = r / a.g4_rpp;
          const int sh = __shfl_sync(0xffffffffu, cur.page, sg & 31);
          const int pg = sg < 32 ? sh : page_of(cur, sg);
          rid[i] = (pg >= 0 && pg < a.num_pages) ? pg * a.g4_rpp + r % a.g4_rpp : -1;
        }
        if (o < g4_ops) {
          tma_gather4(sk + (size_t)o * 4 * a.g4_rb, kmap, rid, &full[stage], pol);
          tma_gather4(sv + (size_t)o * 4 * a.g4_rb, vmap, rid, &full[stage], pol);
        }
      }
      for (int sg = lane; sg < cur.nseg && !g4_rows; sg += 32) {
        const int lp = cur.p_first + sg;
        const int page = page_of(cur, sg);
        if (page < 0 || page >= a.num_pages) continue;
        const int lo = max(cur.t0, lp * a.P), hi = min(cur.t_end, (lp + 1) * a.P);
        const size_t src = ((size_t)page * a.P + (lo - lp * a.P)) * C::ROW;
        const uint32_t bytes = (uint32_t)(hi - lo) * C::ROW;
        const int dst = (lo - cur.t0) * C::ROW;
        bulk_g2s(sk + dst, a.k_cache + src, bytes, &full[stage], pol);
        bulk_g2s(sv + dst, a.v_cache + src, bytes, &full[stage], pol);
      }
      ++issued;
      if (++stage == C::NS) { stage = 0; phase ^= 1u; }
    }
    // Before leaving, make sure the copies this warp issued have landed (bounded).
    if (lane == 0) {
      const int n = min(issued, C::NS);
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < n; ++i) {
        if (--s < 0) { s = C::NS - 1; ph ^= 1u; }
        if (!mbar_wait(&full[s], ph, a.err)) break;
      }
    }
    return;
  }

  // --------------------------------- consumers ------------------------------------
  const int h = warp % HKV, sub = warp / HKV;
  const int g = lane >> 2, c = lane & 3;
  const float ksc = a.k_scale[h];
  const int hq = h * a.G + g;
  const bool row_ok = g < a.G;

  uint32_t q1lo[C::KSTEPS], q2lo[C::KSTEPS], q1hi[C::KSTEPS], q2hi[C::KSTEPS];
  float qf = 0.f;  // 2^-a * k_scale * sm_scale * log2(e)
  float m = -INFINITY, l = 0.f;
  float acc[C::DB][4];

  auto load_q = [&](int b) {
    float v0[C::RL], v1[C::RL];
    float amax = 0.f;
    if (row_ok) {
      const __nv_bfloat16* qr = a.q + (size_t)b * a.ldq + (size_t)hq * D;
#pragma unroll
      for (int i = 0; i < C::RL; i += 8) {
        const uint4 r0 = *reinterpret_cast<const uint4*>(qr + C::RL * c + i);
        const uint4 r1 = *reinterpret_cast<const uint4*>(qr + D / 2 + C::RL * c + i);
        const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w}, w1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v0[i + 2 * k] = bf16_lo(w0[k]);
          v0[i + 2 * k + 1] = bf16_hi(w0[k]);
          v1[i + 2 * k] = bf16_lo(w1[k]);
          v1[i + 2 * k + 1] = bf16_hi(w1[k]);
        }
      }
#pragma unroll
      for (int i = 0; i < C::RL; ++i) amax = fmaxf(amax, fmaxf(fabsf(v0[i]), fabsf(v1[i])));
    } else {
#pragma unroll
      for (int i = 0; i < C::RL; ++i) v0[i] = v1[i] = 0.f;
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // 2^ea with amax * 2^ea in [128, 256): the e4m3 terms keep their full precision
    int ea = 0;
    if (amax > 0.f) ea = 7 - (int)((__float_as_uint(amax) >> 23) & 0xff) + 127;
    const float up = __uint_as_float((uint32_t)(127 + ea) << 23);
    const float down = __uint_as_float((uint32_t)(127 - ea) << 23);
    qf = down * ksc * a.sm_scale_log2;
#pragma unroll
    for (int s = 0; s < C::KSTEPS; ++s) {
      uint32_t w1a = 0, w2a = 0, w1b = 0, w2b = 0;
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int i = 4 * s + 2 * pr;
        const float x0 = v0[i] * up, x1 = v0[i + 1] * up;
        const float y0 = v1[i] * up, y1 = v1[i + 1] * up;
        const uint16_t hx = f2_to_e4m3x2_sat(x0, x1), hy = f2_to_e4m3x2_sat(y0, y1);
        const __half2 bx = __half2(__nv_cvt_fp8x2_to_halfraw2(hx, __NV_E4M3));
        const __half2 by = __half2(__nv_cvt_fp8x2_to_halfraw2(hy, __NV_E4M3));
        const uint16_t lx = f2_to_e4m3x2_sat((x0 - __low2float(bx)) * 16.f, (x1 - __high2float(bx)) * 16.f);
        const uint16_t ly = f2_to_e4m3x2_sat((y0 - __low2float(by)) * 16.f, (y1 - __high2float(by)) * 16.f);
        w1a |= (uint32_t)hx << (16 * pr);
        w2a |= (uint32_t)lx << (16 * pr);
        w1b |= (uint32_t)hy << (16 * pr);
        w2b |= (uint32_t)ly << (16 * pr);
      }
      q1lo[s] = w1a; q2lo[s] = w2a; q1hi[s] = w1b; q2hi[s] = w2b;
    }
    m = -INFINITY;
    l = 0.f;
#pragma unroll
    for (int i = 0; i < C::DB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  };

  auto flush = [&](int b) {
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (!row_ok) return;
    const int slot = blockIdx.x + b;
    const size_t rowi = ((size_t)slot * C::NSUB + sub) * a.Hq + hq;
    if (c == 0) {
      a.ws_ml[rowi * 2] = m;
      a.ws_ml[rowi * 2 + 1] = l;
    }
    float* dst = a.ws_acc + rowi * D + 2 * c * C::RL;
    constexpr float kInv = 1.f / 256.f, kLo = 1.f / 4096.f;
#pragma unroll
    for (int i = 0; i < C::RL; i += 4) {
      float4 o0, o1;
      o0.x = acc[i][0] * kInv + acc[i][2] * kLo;
      o0.y = acc[i + 1][0] * kInv + acc[i + 1][2] * kLo;
      o0.z = acc[i + 2][0] * kInv + acc[i + 2][2] * kLo;
      o0.w = acc[i + 3][0] * kInv + acc[i + 3][2] * kLo;
      o1.x = acc[i][1] * kInv + acc[i][3] * kLo;
      o1.y = acc[i + 1][1] * kInv + acc[i + 1][3] * kLo;
      o1.z = acc[i + 2][1] * kInv + acc[i + 2][3] * kLo;
      o1.w = acc[i + 3][1] * kInv + acc[i + 3][3] * kLo;
      *reinterpret_cast<float4*>(dst + i) = o0;
      *reinterpret_cast<float4*>(dst + C::RL + i) = o1;
    }
  };

  int b = find_seq(prefix, a.B, u0);
  int cur_b = -1;
  int stage = 0;
  uint32_t phase = 0;
  for (int u = u0; u < u1; ++u) {
    while (prefix[b + 1] <= u) ++b;
    if (b != cur_b) {
      if (cur_b >= 0) flush(cur_b);
      load_q(b);
      cur_b = b;
    }
    const int len = a.seq_lens[b];
    const int tb = seq_origin(len, a.window, 1) + (u - prefix[b]) * C::TS + sub * 32;
    const int valid = min(32, max(0, len - tb));

    bool ok = mbar_wait(&full[stage], phase, a.err);
    if (!__all_sync(0xffffffffu, ok)) { *abort_flag = 1; return; }

    if (valid > 0) {
      const uint8_t* sk = stages + (size_t)stage * C::STAGE + (size_t)(sub * 32) * C::ROW + h * D;
      const uint8_t* sv = sk + C::KV_BYTES;
      // ---- S = Q K^T over 32 tokens: 4 n8 blocks, k-steps interleaved across blocks ----
      float S[4][4];
      uint32_t kr0[4][C::KSTEPS], kr1[4][C::KSTEPS];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.f;
        const int tok = 16 * (j >> 1) + 4 * (g >> 1) + 2 * (j & 1) + (g & 1);
        const uint8_t* kr = sk + (size_t)tok * C::ROW + C::RL * c;
        if constexpr (D == 128) {
          const uint4 x0 = *reinterpret_cast<const uint4*>(kr);
          const uint4 x1 = *reinterpret_cast<const uint4*>(kr + 64);
          kr0[j][0] = x0.x; kr0[j][1] = x0.y; kr0[j][2] = x0.z; kr0[j][3] = x0.w;
          kr1[j][0] = x1.x; kr1[j][1] = x1.y; kr1[j][2] = x1.z; kr1[j][3] = x1.w;
        } else {
          const uint2 x0 = *reinterpret_cast<const uint2*>(kr);
          const uint2 x1 = *reinterpret_cast<const uint2*>(kr + 32);
          kr0[j][0] = x0.x; kr0[j][1] = x0.y;
          kr1[j][0] = x1.x; kr1[j][1] = x1.y;
        }
      }
#pragma unroll
      for (int s2 = 0; s2 < C::KSTEPS; ++s2)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_e4m3_16832(S[j], q1lo[s2], q2lo[s2], q1hi[s2], q2hi[s2], kr0[j][s2], kr1[j][s2]);
      constexpr int VW = C::RL / 4;  // 32-bit words per V run
      uint32_t vlw[4][VW], vhw[4][VW];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ld_run<C::RL>(sv + (size_t)(4 * c + u) * C::ROW + C::RL * g, vlw[u]);
        ld_run<C::RL>(sv + (size_t)(16 + 4 * c + u) * C::ROW + C::RL * g, vhw[u]);
      }
      // ---- online softmax (log2 domain), rows g (q1 part) + g+8 (q2 part) ----
      float sc[4][2];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tok = 16 * (j >> 1) + 4 * c + 2 * (j & 1) + e;
          float v = (S[j][e] + S[j][2 + e] * 0.0625f) * qf;
          if (valid < 32) v = tok < valid ? v : -INFINITY;  // warp-uniform: tail tiles only
          sc[j][e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = fast_exp2(m - m_use);
      m = m_new;
      float p[4][2];
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          p[j][e] = fast_exp2(sc[j][e] - m_use);
          ps += p[j][e];
        }
      }
      l = l * alpha + ps;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int i = 0; i < C::DB; ++i) {
          acc[i][0] *= alpha; acc[i][1] *= alpha; acc[i][2] *= alpha; acc[i][3] *= alpha;
        }
      }
      // ---- P as two e4m3 terms: p*256 ~= p1 + p2/16, formed in f16x2 arithmetic (p*256 is in
      // [0, 256]: its f16 rounding, 2^-11, is far below the ~2^-8 of the two-term form; the
      // residual x - p1 is exact in f16) ----
      uint16_t t1[4], t2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 xh = __floats2half2_rn(p[j][0] * 256.f, p[j][1] * 256.f);
        t1[j] = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(xh), __NV_SATFINITE, __NV_E4M3);
        const __half2 bk = __half2(__nv_cvt_fp8x2_to_halfraw2(t1[j], __NV_E4M3));
        const __half2 r = __hmul2(__hsub2(xh, bk), __float2half2_rn(16.f));
        t2[j] = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(r), __NV_SATFINITE, __NV_E4M3);
      }
      // a0 (p1, tokens 4c..), a1 (p2), a2 (p1, 16+4c..), a3 (p2): j = 0,1 -> a0/a1, j = 2,3 -> a2/a3
      const uint32_t pa[4] = {(uint32_t)t1[0] | ((uint32_t)t1[1] << 16), (uint32_t)t2[0] | ((uint32_t)t2[1] << 16),
                              (uint32_t)t1[2] | ((uint32_t)t1[3] << 16), (uint32_t)t2[2] | ((uint32_t)t2[3] << 16)};
      // ---- O += P V: V rows (4c+u) and (16+4c+u), columns [RL*g, RL*g + RL) ----
      const bool tail = valid < 32;
      uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
      if (tail) {
        mlo = 0; mhi = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (4 * c + u < valid) mlo |= 0xffu << (8 * u);
          if (16 + 4 * c + u < valid) mhi |= 0xffu << (8 * u);
        }
      }
#pragma unroll
      for (int k = 0; k < VW; ++k) {  // one 4-byte column group (4 d-blocks) at a time
        uint32_t b0[4], b1[4];
        transpose4x4(vlw[0][k], vlw[1][k], vlw[2][k], vlw[3][k], b0[0], b0[1], b0[2], b0[3]);
        transpose4x4(vhw[0][k], vhw[1][k], vhw[2][k], vhw[3][k], b1[0], b1[1], b1[2], b1[3]);
        if (tail) {
#pragma unroll
          for (int i = 0; i < 4; ++i) { b0[i] &= mlo; b1[i] &= mhi; }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          mma_e4m3_16832(acc[4 * k + i], pa[0], pa[1], pa[2], pa[3], b0[i], b1[i]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == C::NS) { stage = 0; phase ^= 1u; }
  }
  if (cur_b >= 0) flush(cur_b);
}

// ---------------------------------------------------------------------------------------
// Merge of one (sequence b, query head hq): out = v_scale[h] * sum_parts 2^(m_i - M) acc_i /
// sum_parts 2^(m_i - M) l_i over the split-KV partials of the CTAs that covered b (units
// [uf, ul] of U over C CTAs; NSUB sub-tiles per unit).  S warps share a (b, hq): warp s folds
// the contiguous part range s of S (merge_fold, lane owning D/32 consecutive d), then warp 0
// combines the folds in split order (merge_store).  Parts are read in a fixed order and through
// L2 (they may come from other SMs of the running grid), so the result does not depend on which
// CTA finished first.  S = 4 where units hold >= 4 sub-tiles (1-2 KV heads: with one KV head a
// sequence has ~24 parts, which one warp reads in three dependent round trips; the merge took
// ~10 of ~62 us at 128 sequences, 4 warps take it to ~57 us); S = 1 otherwise (8 KV heads: 2-3
// parts per sequence, where the 4-warp form measured 268 vs 248 us for C4).

__device__ void merge_fold(const AttnArgs& a, int b, int hq, int U, int uf, int ul, int NSUB, int D, int lane,
                           int s, int S, float& M, float& L, float (&o)[4]) {
  const int per = D / 32;  // 4 (D = 128) or 2 (D = 64)
  o[0] = o[1] = o[2] = o[3] = 0.f;
  L = 0.f;
  M = -INFINITY;
  if (ul < uf) return;
  const int cf = cta_of_unit(U, a.num_ctas, uf), cl = cta_of_unit(U, a.num_ctas, ul);
  const int nparts = (cl - cf + 1) * NSUB;
  const int q0 = nparts * s / S, q1 = nparts * (s + 1) / S;
  auto row_of = [&](int p) { return ((size_t)(cf + p / NSUB + b) * NSUB + p % NSUB) * a.Hq + hq; };
  // Batches of 8 parts: the (m, l) of part p0 + i sit in lane i, and the 8 parts' slices of acc
  // are loaded in the same round, so one batch costs one memory round trip.  A running maximum
  // carries the log-sum-exp across batches.
  for (int p0 = q0; p0 < q1; p0 += 8) {
    const int n = min(8, q1 - p0);
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < n) ml = __ldcg(reinterpret_cast<const float2*>(a.ws_ml + row_of(p0 + lane) * 2));
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n) {
        const float* src = a.ws_acc + row_of(p0 + i) * D + lane * per;
        if (per == 4) v[i] = __ldcg(reinterpret_cast<const float4*>(src));
        else { const float2 t = __ldcg(reinterpret_cast<const float2*>(src)); v[i].x = t.x; v[i].y = t.y; }
      }
    }
    const float Mn = fmaxf(M, warp_max(ml.x));
    if (Mn == -INFINITY) continue;  // nothing attended yet
    if (M != -INFINITY && M != Mn) {
      const float r = exp2f(M - Mn);
      L *= r;
      o[0] *= r; o[1] *= r; o[2] *= r; o[3] *= r;
    }
    M = Mn;
    const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
    L += w * ml.y;  // per lane; summed over the warp at the end
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float wi = __shfl_sync(0xffffffffu, w, i);
      o[0] += wi * v[i].x; o[1] += wi * v[i].y; o[2] += wi * v[i].z; o[3] += wi * v[i].w;
    }
  }
  L = warp_sum(L);
}

// out[b][hq] = o / L * v_scale (then Muse's rms(o) * sigmoid(gate) when a.gate), as bf16.
__device__ void merge_store(const AttnArgs& a, int b, int hq, int D, int lane, float L, float (&o)[4]) {
  const int per = D / 32;
  __nv_bfloat16* dst = a.out + (size_t)b * a.ldo + (size_t)hq * D + lane * per;
  const float scale = L > 0.f ? a.v_scale[hq / a.G] / L : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] *= scale;
  if (a.gate) {
    // Muse output gate (muse_prefill_layer/submission.py:176): rms(o) * sigmoid(gate), per head
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += i < per ? o[i] * o[i] : 0.f;
    const float inv = rsqrtf(warp_sum(ss) / (float)D + a.out_eps);
    const __nv_bfloat16* g = a.gate + (size_t)b * a.ld_gate + (size_t)hq * D + lane * per;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= per) break;
      const float gv = __bfloat162float(g[i]);
      o[i] = o[i] * inv * (1.f / (1.f + expf(-gv)));
    }
  }
  if (per == 4) {
    uint2 r;
    r.x = pack_bf16x2(o[0], o[1]);
    r.y = pack_bf16x2(o[2], o[3]);
    *reinterpret_cast<uint2*>(dst) = r;
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(o[0], o[1]);
  }
}

template <int D, int HKV>
__global__ void __launch_bounds__(AttnCfg<D, HKV>::THREADS, 1) attn_decode_kernel(AttnArgs a) {
  attn_decode_body<D, HKV, false>(nullptr, nullptr, a);
}

template <int D, int HKV>
__global__ void __launch_bounds__(AttnCfg<D, HKV>::THREADS, 1) attn_decode_g4_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
  attn_decode_body<D, HKV, true>(&kmap, &vmap, a);
}

// The merge kernel: one warp per (sequence, query head), after the whole decode grid.
template <int S>
__global__ void __launch_bounds__(256 * S) attn_merge_kernel(AttnArgs a, int TS, int NSUB, int D) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = warp / S, s = warp % S;
  const int hq = blockIdx.y * 8 + hl;
  const bool on = hq < a.Hq;
  float M = -INFINITY, L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  if (on) merge_fold(a, b, hq, a.ws_prefix[a.B], a.ws_prefix[b], a.ws_prefix[b + 1] - 1, NSUB, D, lane, s, S, M, L, o);
  if constexpr (S == 1) {
    if (on) merge_store(a, b, hq, D, lane, L, o);
    return;
  }
  __shared__ float fold[8][S][6][32];  // per head of the CTA and split: M, L, o[0..3]
  fold[hl][s][0][lane] = M;
  fold[hl][s][1][lane] = L;
#pragma unroll
  for (int i = 0; i < 4; ++i) fold[hl][s][2 + i][lane] = o[i];
  __syncthreads();
  if (!on || s != 0) return;
  float Ma = -INFINITY;
#pragma unroll
  for (int t = 0; t < S; ++t) Ma = fmaxf(Ma, fold[hl][t][0][lane]);
  float La = 0.f, oa[4] = {0.f, 0.f, 0.f, 0.f};
  if (Ma != -INFINITY) {
#pragma unroll
    for (int t = 0; t < S; ++t) {  // split order: deterministic
      const float Mt = fold[hl][t][0][lane];
      const float w = Mt == -INFINITY ? 0.f : exp2f(Mt - Ma);
      La += w * fold[hl][t][1][lane];
#pragma unroll
      for (int i = 0; i < 4; ++i) oa[i] += w * fold[hl][t][2 + i][lane];
    }
  }
  merge_store(a, b, hq, D, lane, La, oa);
}

// ---------------------------------------------------------------------------------------
// RoPE + FP8 KV-append.  grid (B, chunks): each thread owns 8 consecutive elements (4 pairs,
// one 16-byte load) of the token's q | k | v row; sin/cos are computed once per token.
__global__ void __launch_bounds__(256) rope_append_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ldqkv, const int64_t* __restrict__ positions,
    const int32_t* __restrict__ page_table, int table_ld, int max_pages,
    const float* __restrict__ inv_freq, const float* __restrict__ k_scale,
    const float* __restrict__ v_scale, __nv_bfloat16* __restrict__ q_out,
    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache, int64_t* __restrict__ slots_out,
    int Hq, int Hkv, int D, int P, long long num_pages, float q_scale, int qk_norm, float norm_eps, int* err) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const long long pos = positions[b];
  const long long lp = pos / P;
  long long slot = -1;
  if (pos >= 0 && lp < max_pages) {
    const int page = page_table[(size_t)b * table_ld + lp];
    if (page >= 0 && page < num_pages) slot = (long long)page * P + pos % P;
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    if (slot < 0) atomicOr(err, OKC_DEVERR_PAGE);
    if (slots_out) slots_out[b] = slot;
  }
  const int half = D / 2;
  __shared__ float sin_s[256], cos_s[256];  // D <= 512: the angles depend on (pos, pair) only
  if (inv_freq) {
    const float posf = (float)pos;
    for (int i = threadIdx.x; i < half; i += blockDim.x) sincosf(__fmul_rn(posf, inv_freq[i]), &sin_s[i], &cos_s[i]);
  }
  __syncthreads();
  const int e0 = (blockIdx.y * blockDim.x + threadIdx.x) * 8;  // first element of this thread
  const int total = (Hq + 2 * Hkv) * D;
  const bool active = e0 < total;
  const int head = e0 / D, d0 = e0 - head * D;  // D % 8 == 0: the 8 elements share one head
  float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (active) {
    const uint4 raw = *reinterpret_cast<const uint4*>(qkv + (size_t)b * ldqkv + e0);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) { x[2 * k] = bf16_lo(w[k]); x[2 * k + 1] = bf16_hi(w[k]); }
  }
  const bool is_v = head >= Hq + Hkv;
  if (qk_norm) {
    // Muse's per-head RMSNorm of q and k (muse_prefill_layer/submission.py:144-145): the D/8
    // threads of a head are consecutive lanes of one warp, reduced with xor shuffles.
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += x[k] * x[k];
    for (int o = 1; o < D / 8; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (!is_v) {
      const float inv = rsqrtf(ss / (float)D + norm_eps);
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] *= inv;
    }
  }
  if (!active) return;
  if (inv_freq && !is_v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = d0 / 2 + k;
      const float sn = sin_s[i], cs = cos_s[i];
      const float y0 = __fsub_rn(__fmul_rn(x[2 * k], cs), __fmul_rn(x[2 * k + 1], sn));
      const float y1 = __fadd_rn(__fmul_rn(x[2 * k], sn), __fmul_rn(x[2 * k + 1], cs));
      x[2 * k] = y0;
      x[2 * k + 1] = y1;
    }
  }
  if (head < Hq) {
    if (q_scale != 1.f) {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] *= q_scale;  // the query scale factor before bf16
    }
    uint4 o;
    o.x = pack_bf16x2(x[0], x[1]); o.y = pack_bf16x2(x[2], x[3]);
    o.z = pack_bf16x2(x[4], x[5]); o.w = pack_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(q_out + ((size_t)b * Hq + head) * D + d0) = o;
  } else if (slot >= 0) {
    const int h = is_v ? head - Hq - Hkv : head - Hq;
    const float sc = is_v ? v_scale[h] : k_scale[h];
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      lo |= (uint32_t)f_to_e4m3_nosat(__fdiv_rn(x[k], sc)) << (8 * k);
      hi |= (uint32_t)f_to_e4m3_nosat(__fdiv_rn(x[4 + k], sc)) << (8 * k);
    }
    uint8_t* cache = is_v ? v_cache : k_cache;
    *reinterpret_cast<uint2*>(cache + ((size_t)slot * Hkv + h) * D + d0) = make_uint2(lo, hi);
  }
}

// ---------------------------------------------------------------------------------------
// A 2-D map over the cache as rows of rb bytes (rb / 8 x u64; rb a multiple of 16, <= 2048),
// one-row box: the gather4 source.
static bool g4_map(CUtensorMap* m, const void* base, long long rows, int rb) {
  auto fn = tensor_map_encoder();
  if (!fn || !okc_host::aligned16(base) || rb % 16 || rb > 2048 || rb <= 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)(rb / 8), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)rb};
  cuuint32_t box[2] = {(cuuint32_t)(rb / 8), 1};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, int HKV>
static int launch_attn_t(AttnArgs& a, cudaStream_t stream) {
  using C = AttnCfg<D, HKV>;
  const size_t smem = (size_t)C::NS * C::STAGE + 2 * C::NS * sizeof(uint64_t) + 16 +
                      (size_t)(a.B + 1) * sizeof(int);
  static size_t configured = 0;  // largest dynamic smem size set so far for this instance
  if (smem > 232448) return OKC_ERR_INVALID;  // 227 KB per block on sm_100
  if (smem > configured) {
    if (cudaFuncSetAttribute(attn_decode_kernel<D, HKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_g4_kernel<D, HKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = smem;
  }
  // TMA gather4 maps when a page is below 2 KB (a multiple of 16 bytes: one gather row each) and
  // units start on a page (always so for one-token pages, whatever the window).  Pages of one or
  // two 2 KB rows gather as well, but measured no faster than bulk copies in the kernel instance
  // without the gather code (1 KV head: 64.4 vs 65.2 us; 2 heads: 103 vs 86 us), so they take
  // that instance; one-token pages of 128 bytes gather at 2x the bulk rate (155 vs 297 us).
  CUtensorMap km{}, vm{};
  a.g4_rpp = 0;
  a.g4_rb = 0;
  const long long pb = (long long)a.P * C::ROW;
  const int rb = (pb < 2048 && pb % 16 == 0) ? (int)pb : 0;
  if (rb && (a.window == 0 || a.P == 1) && C::TS % a.P == 0 && C::KV_BYTES % (4 * rb) == 0 &&
      !getenv("OKC_ATTN_NO_GATHER")) {
    const long long rows = a.num_pages * (pb / rb);
    if (rows < (1LL << 31) && g4_map(&km, a.k_cache, rows, rb) && g4_map(&vm, a.v_cache, rows, rb)) {
      a.g4_rpp = (int)(pb / rb);
      a.g4_rb = rb;
    }
  }
  int st = a.g4_rpp > 0
               ? okc_host::launch_k(attn_decode_g4_kernel<D, HKV>, dim3(a.num_ctas), dim3(C::THREADS), smem, stream,
                                    dim3(1), km, vm, a)
               : okc_host::launch_k(attn_decode_kernel<D, HKV>, dim3(a.num_ctas), dim3(C::THREADS), smem, stream,
                                    dim3(1), a);
  if (st) return st;
  return launch_attn_merge(a, C::TS, C::NSUB, D, stream);
}

int launch_attn_merge(AttnArgs& a, int TS, int NSUB, int D, cudaStream_t stream) {
  if (NSUB >= 4)
    return okc_host::launch_k(attn_merge_kernel<4>, dim3(a.B, (a.Hq + 7) / 8), dim3(1024), 0, stream, dim3(1), a, TS,
                              NSUB, D);
  return okc_host::launch_k(attn_merge_kernel<1>, dim3(a.B, (a.Hq + 7) / 8), dim3(256), 0, stream, dim3(1), a, TS,
                            NSUB, D);
}

int launch_attn_decode(AttnArgs& a, int D, int Hkv, cudaStream_t stream) {
  if (attn_tc_eligible(a, D, Hkv)) return launch_attn_tc(a, Hkv, stream);
  if (D == 128) {
    switch (Hkv) {
      case 1: return launch_attn_t<128, 1>(a, stream);
      case 2: return launch_attn_t<128, 2>(a, stream);
      case 4: return launch_attn_t<128, 4>(a, stream);
      case 8: return launch_attn_t<128, 8>(a, stream);
    }
  } else if (D == 64) {
    switch (Hkv) {
      case 1: return launch_attn_t<64, 1>(a, stream);
      case 2: return launch_attn_t<64, 2>(a, stream);
      case 4: return launch_attn_t<64, 4>(a, stream);
      case 8: return launch_attn_t<64, 8>(a, stream);
    }
  }
  return OKC_ERR_INVALID;
}

int launch_rope_append(const void* qkv, int ldqkv, const int64_t* positions,
                       const int32_t* page_table, int table_ld, int max_pages,
                       const float* inv_freq, const float* k_scale, const float* v_scale,
                       void* q_out, void* k_cache, void* v_cache, int64_t* slots_out, int B,
                       int Hq, int Hkv, int D, int P, long long num_pages, float q_scale, int qk_norm,
                       float norm_eps, int* err, cudaStream_t stream) {
  const int chunks = ((Hq + 2 * Hkv) * D / 8 + 255) / 256;
  return okc_host::launch_k(rope_append_kernel, dim3(B, chunks), dim3(256), 0, stream, dim3(1),
      reinterpret_cast<const __nv_bfloat16*>(qkv), ldqkv, positions, page_table, table_ld, max_pages,
      inv_freq, k_scale, v_scale, reinterpret_cast<__nv_bfloat16*>(q_out),
      reinterpret_cast<uint8_t*>(k_cache), reinterpret_cast<uint8_t*>(v_cache), slots_out, Hq, Hkv,
      D, P, num_pages, q_scale, qk_norm, norm_eps, err);
}

}  // namespace okc
