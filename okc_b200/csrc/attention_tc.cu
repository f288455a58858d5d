// Paged FP8-KV attention decode on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract and split-KV partials as attn_decode_kernel (attention.cu), for head_dim 128,
// page sizes 16, 32 and 64, 4 or 8 KV heads and up to 8 query heads per KV head.  Selected with
// OKC_ATTN_TC=1.
//
//  * attn_q8_kernel turns every query row into two e4m3 terms q ~= (q1 + q2/16) * 2^-a (a per
//    row; the precision of the bf16 query) laid out as the MMA's B operand (per KV head 16 rows
//    x 128 B, 128-byte swizzle), plus the per-row scale 2^-a * k_scale * sm_scale * log2(e).
//  * Units are 64-token tiles of a sequence, split evenly over a persistent grid (stream-K).
//    An "item" is one KV-head pair of a unit: 64 tokens x 2 heads = 128 rows, the MMA's M.
//    Warp 0 (producer) loads an item with one 4-D TMA box per page (P tokens x 2 heads x 128 B)
//    from the cache [pages][P][Hkv][128]: the rows land as [page][head][token] in a 128-byte-
//    swizzled tile.  K and V have separate rings of 6 slots (192 KB together), and K is issued
//    two items ahead of V, since K is consumed at once while V waits for the softmax.
//  * Warp 1 (one thread) issues tcgen05.mma kind::f8f6f4 with fp32 accumulators in TMEM:
//      S[row, c] = K[row, :] . Q[c, :]        M = 128 rows, N = 32 (2 heads x 16), K = 128
//      O[d, c]  += V[row, d] . P[row, c]      M = 128 (d), N = 32, K = 128 rows
//    The rows mix two heads, so Q (both heads' 16 rows) and P (a row's 16 bytes in its own
//    head's column block, zeros in the other) are block diagonal: an MMA reads each KV byte
//    once and the unused products are multiplied by zero.  P carries p * 256 ~= p1 + p2/16.
//    At a sequence change it copies the next Q in (after its MMAs on the previous Q are done).
//  * Warps 2..9 are two softmax warpgroups taking alternate items (one TMEM row per thread):
//    scores, tile maximum per (head, query row) over the 128 rows (warp transpose-reduction
//    plus one shared-memory barrier), running maxima, per-thread partial sums of p, O rescale
//    in TMEM when a maximum rises, P.  O is double-buffered by sequence, so the flush of a
//    finished sequence's split-KV partial overlaps the next sequence's first item.
// Every wait is bounded (mbar_wait); on expiry the kernel stops issuing work, sets
// OKC_DEVERR_TIMEOUT, waits (bounded) for its own copies and MMAs, frees TMEM and returns.
//
// Roofline: HBM; algorithmic bytes = sum_b len_b * Hkv * 128 * 2 (the KV cache streamed once).
// Mirrors the tile loop / online softmax / split partials of muse_attention_decode/
// submission.py:100-351 and the semantics of muse_prefill_layer/submission.py:137-176.
#include "attention_common.cuh"
#include "tcgen05.cuh"

namespace okc {

template <int HKV>
struct TcAttnCfg {
  static constexpr int D = 128;
  static constexpr int TILE = 64;                  // tokens per unit
  static constexpr int ROWS = 128;                 // rows per item: TILE tokens x 2 heads
  static constexpr int NGRP = HKV / 2;             // head pairs (items) per unit: 4 or 2
  static constexpr int GPW = NGRP / 2;             // items of a unit per softmax warpgroup
  static constexpr int SLOT = ROWS * D;            // 16 KB: K (or V) of one item
  static constexpr int NS = 6;                     // slots per ring
  static constexpr int RING = 2 * NS * SLOT;       // 192 KB: a K ring and a V ring
  static constexpr int AHEAD = 2;                  // K issued this many items before V
  static constexpr int Q_BYTES = HKV * 16 * D;     // [head][16 rows][128 B], SW128 K-major
  static constexpr int P_NBLK = ROWS * 16;         // one head's column block of P: [row][16 B]
  static constexpr int P_WG = 2 * P_NBLK;          // P of one warpgroup (two column blocks)
  static constexpr int P_BYTES = 2 * P_WG;
  static constexpr int S_COLS = 32;                // S of one item (per warpgroup)
  static constexpr int O_COL0 = 2 * S_COLS;        // O: [sequence parity][head][16]
  static constexpr int O_COLS = HKV * 16;
  static constexpr int USED_COLS = O_COL0 + 2 * O_COLS;
  static constexpr int TMEM_COLS = USED_COLS <= 128 ? 128 : USED_COLS <= 256 ? 256 : 512;
  // small shared arrays after the P buffers
  static constexpr int QF_OFF = 0;                         // float [2][HKV][8]: query scales by sequence parity
  static constexpr int RED_OFF = QF_OFF + 2 * HKV * 8 * 4; // float [2 wg][2][4][16]: tile maxima per warp
  static constexpr int FL_OFF = RED_OFF + 2 * 2 * 4 * 16 * 4;  // float [2 wg][4][GPW * 16]: l sums
  static constexpr int M_OFF = FL_OFF + 2 * 4 * GPW * 16 * 4;  // float [NGRP][2][16]: running maxima
  static constexpr int BAR_OFF = M_OFF + NGRP * 2 * 16 * 4;
  static constexpr int NBARS = 4 * NS + 2 + 2 + 2 + 2 + 1 + 1 + 1;
  static constexpr int MISC = BAR_OFF + NBARS * 8 + 16;    // + TMEM slot, abort flag
  static constexpr int BODY = RING + Q_BYTES + P_BYTES + MISC;
  static constexpr int THREADS = 320;              // producer, MMA, two softmax warpgroups
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// kind::f8f6f4 instruction descriptor: D f32, A/B e4m3, M = 128, N = 32, majors as given.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int a_mn_major, int b_mn_major) {
  return (1u << 4) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(32 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// Shared-memory descriptor without swizzle (core matrices of 8 rows x 16 B stored as 128
// contiguous bytes): leading offset between core matrices along K, stride offset along M/N.
__device__ __forceinline__ uint64_t umma_desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}

__device__ __forceinline__ void umma_e4m3(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Named barrier `id` over the 128 threads of one softmax warpgroup.
__device__ __forceinline__ void wg_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// Maximum over the 128 threads of a softmax warpgroup of each of 16 values; every thread gets
// all 16 results.  Within a warp a transpose-reduction halves the values per lane each round
// (a lane keeps one half and trades the other with its partner), so lane l ends with value
// idx(l) reduced over the warp; the four warps meet in shared memory behind one barrier (the
// buffer alternates between consecutive calls, so no second barrier is needed).
__device__ __forceinline__ void wg_max16(float (&v)[16], float* red, int wq, int lane, int bar_id) {
  float w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = v[i];
  int idx = 0;
#pragma unroll
  for (int o = 16, n = 16; o >= 2; o >>= 1, n >>= 1) {
    const int h = n / 2;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < h) {
        const float send = up ? w[i] : w[i + h];
        const float keep = up ? w[i + h] : w[i];
        w[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    }
    if (up) idx += h;
  }
  w[0] = fmaxf(w[0], __shfl_xor_sync(0xffffffffu, w[0], 1));
  if ((lane & 1) == 0) red[wq * 16 + idx] = w[0];
  wg_bar(bar_id);
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 a0 = *reinterpret_cast<const float4*>(red + i), a1 = *reinterpret_cast<const float4*>(red + 16 + i);
    const float4 a2 = *reinterpret_cast<const float4*>(red + 32 + i), a3 = *reinterpret_cast<const float4*>(red + 48 + i);
    v[i] = fmaxf(fmaxf(a0.x, a1.x), fmaxf(a2.x, a3.x));
    v[i + 1] = fmaxf(fmaxf(a0.y, a1.y), fmaxf(a2.y, a3.y));
    v[i + 2] = fmaxf(fmaxf(a0.z, a1.z), fmaxf(a2.z, a3.z));
    v[i + 3] = fmaxf(fmaxf(a0.w, a1.w), fmaxf(a2.w, a3.w));
  }
}

// ---------------------------------------------------------------------------------------
// Two-term e4m3 queries.  grid (B), block (128): thread (h, r) = (tid / 16, tid % 16) writes row
// r of KV head h's 16 rows (r < 8: first term of query head h*G + r; r >= 8: second term of
// query head h*G + r - 8; rows of query heads >= G are zero) as 128 swizzled bytes, and for
// r < 8 the row's scale.
__global__ void __launch_bounds__(128) attn_q8_kernel(AttnArgs a, int hkv) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, h = threadIdx.x >> 4, r = threadIdx.x & 15, rr = r & 7;
  if (h >= hkv) return;
  uint8_t* dst = a.ws_q8 + ((size_t)b * hkv + h) * 2048 + (r >> 3) * 1024 + rr * 128;
  float qscale = 0.f;
  if (rr < a.G) {
    const uint4* src = reinterpret_cast<const uint4*>(a.q + (size_t)b * a.ldq + (size_t)(h * a.G + rr) * 128);
    uint4 x[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) x[c] = src[c];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint32_t xw[4] = {x[c].x, x[c].y, x[c].z, x[c].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(xw[k])), fabsf(bf16_hi(xw[k]))));
    }
    int ea = 0;  // amax * 2^ea in [128, 256): both e4m3 terms keep their full precision
    if (amax > 0.f) ea = 7 - (int)((__float_as_uint(amax) >> 23) & 0xff) + 127;
    const float up = __uint_as_float((uint32_t)(127 + ea) << 23);
    qscale = __uint_as_float((uint32_t)(127 - ea) << 23) * a.k_scale[h] * a.sm_scale_log2;
#pragma unroll
    for (int c = 0; c < 8; ++c) {  // 16 elements -> one 16-byte chunk
      const uint32_t xw[8] = {x[2 * c].x, x[2 * c].y, x[2 * c].z, x[2 * c].w,
                              x[2 * c + 1].x, x[2 * c + 1].y, x[2 * c + 1].z, x[2 * c + 1].w};
      uint32_t out[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t wv = 0;
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const uint32_t rw = xw[2 * k + pr];
          const float y0 = bf16_lo(rw) * up, y1 = bf16_hi(rw) * up;
          const uint16_t t1 = f2_to_e4m3x2_sat(y0, y1);
          uint16_t o = t1;
          if (r >= 8) {
            const __half2 bk = __half2(__nv_cvt_fp8x2_to_halfraw2(t1, __NV_E4M3));
            o = f2_to_e4m3x2_sat((y0 - __low2float(bk)) * 16.f, (y1 - __high2float(bk)) * 16.f);
          }
          wv |= (uint32_t)o << (16 * pr);
        }
        out[k] = wv;
      }
      *reinterpret_cast<uint4*>(dst + ((c ^ rr) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + (c << 4)) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (r < 8) a.ws_qf[((size_t)b * hkv + h) * 8 + r] = qscale;
}

// ---------------------------------------------------------------------------------------
template <int HKV>
__global__ void __launch_bounds__(320, 1) attn_tc_kernel(const __grid_constant__ CUtensorMap map_k,
                                                         const __grid_constant__ CUtensorMap map_v, AttnArgs a) {
  using C = TcAttnCfg<HKV>;
  constexpr int NGRP = C::NGRP, GPW = C::GPW, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_k = smem;
  uint8_t* ring_v = smem + NS * C::SLOT;
  uint8_t* qs = smem + C::RING;
  uint8_t* ps = qs + C::Q_BYTES;
  uint8_t* misc = ps + C::P_BYTES;
  float* qf_all = reinterpret_cast<float*>(misc + C::QF_OFF);
  float* red_all = reinterpret_cast<float*>(misc + C::RED_OFF);
  float* fl_all = reinterpret_cast<float*>(misc + C::FL_OFF);
  float* msh = reinterpret_cast<float*>(misc + C::M_OFF);
  uint64_t* full_k = reinterpret_cast<uint64_t*>(misc + C::BAR_OFF);
  uint64_t* empty_k = full_k + NS;
  uint64_t* full_v = empty_k + NS;
  uint64_t* empty_v = full_v + NS;
  uint64_t* s_full = empty_v + NS;  // [2]: S of the item of softmax warpgroup w = item & 1
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_full = pv_done + 2;   // Q and the query scales of the next sequence have landed
  uint64_t* q_free = q_full + 1;    // the MMAs on the previous Q are done
  uint64_t* mma_done = q_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* prefix = reinterpret_cast<int*>(smem_raw + (C::BODY + 1024));  // [B + 1]
  int* lens = prefix + a.B + 1;                                         // [B] context lengths

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_k[s], 1);
      mbar_init(&empty_k[s], 1);
      mbar_init(&full_v[s], 1);
      mbar_init(&empty_v[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // P's off-diagonal column blocks stay zero for the whole kernel (a row's head never changes)
  for (int i = threadIdx.x; i < C::P_BYTES / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(ps)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_async_smem();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  unit_prefix(a.seq_lens, a.B, C::TILE, a.window, a.P, prefix);
  for (int i = threadIdx.x; i < a.B; i += blockDim.x) lens[i] = max(0, a.seq_lens[i]);
  __syncthreads();
  if (blockIdx.x == 0)  // for the merge kernel
    for (int i = threadIdx.x; i <= a.B; i += blockDim.x) a.ws_prefix[i] = prefix[i];

  const int U = prefix[a.B];
  int u0, u1;
  unit_range(U, a.num_ctas, blockIdx.x, u0, u1);
  const int nK = (u1 - u0) * NGRP;  // items (K and V each)

  if (nK > 0 && warp == 0) {
    // ------------------------------------ producer ------------------------------------
    // Issue order: K(t), then V(t - AHEAD); each ring waits for its own released slot.  The
    // items of a unit share its pages: lane l holds the unit's l-th page id, looked up once,
    // and the next unit's ids are loaded while the current unit is being issued.
    const uint64_t pol = l2_evict_first_policy();
    const int ppt = C::TILE / a.P;  // pages per unit (<= 4)
    const uint32_t box_bytes = (uint32_t)a.P * 2 * 128;
    struct Unit { int npg, page; };
    int bl = find_seq(prefix, a.B, u0);
    auto lookup = [&](int u) -> Unit {  // units are looked up in increasing order
      Unit r{0, -1};
      if (u >= u1) return r;
      while (prefix[bl + 1] <= u) ++bl;
      const int len = lens[bl];
      const int t0 = seq_origin(len, a.window, a.P) + (u - prefix[bl]) * C::TILE;
      const int t1 = min(len, t0 + C::TILE);
      r.npg = min(ppt, (t1 - t0 + a.P - 1) / a.P);
      const int lp = t0 / a.P + lane;
      const int row = bl / a.q_per_seq;
      r.page = (lane < r.npg && lp < a.table_ld) ? __ldg(a.page_table + (size_t)row * a.table_ld + lp) : -1;
      return r;
    };
    static_assert(C::AHEAD <= NGRP, "V must trail K by at most one unit");
    Unit uk = lookup(u0), unext = lookup(u0 + 1), uprev = uk;  // K's unit, the next, the previous
    int uk_id = u0, nk = 0, nv = 0;
    auto issue = [&](int kk, int isv, const Unit& un) -> bool {
      const int g = kk % NGRP;
      const bool ok_page = un.page >= 0 && un.page < a.num_pages;
      if (lane < un.npg && !ok_page && isv == 0 && g == 0) atomicOr(a.err, OKC_DEVERR_PAGE);
      const uint32_t nbox = __popc(__ballot_sync(0xffffffffu, lane < un.npg && ok_page));
      const int slot = kk % NS;
      uint64_t* fb = isv ? &full_v[slot] : &full_k[slot];
      uint64_t* eb = isv ? &empty_v[slot] : &empty_k[slot];
      bool ok = true;
      if (lane == 0) ok = mbar_wait(eb, ((uint32_t)(kk / NS) & 1u) ^ 1u, a.err, abort_flag);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) return false;
      if (lane == 0) {
        if (nbox) mbar_arrive_expect_tx(fb, nbox * box_bytes);
        else mbar_arrive(fb);
      }
      __syncwarp();
      if (lane < un.npg && ok_page)
        tma_load_4d((isv ? ring_v : ring_k) + (size_t)slot * C::SLOT + (size_t)lane * box_bytes,
                    isv ? &map_v : &map_k, 0, 0, 2 * g, un.page, fb, pol);
      return true;
    };
    for (int t = 0; t < nK + C::AHEAD; ++t) {
      if (t < nK) {
        const int u = u0 + t / NGRP;
        if (u != uk_id) {  // K moves to the next unit; prefetch the one after it
          uprev = uk;
          uk = unext;
          uk_id = u;
          unext = lookup(u + 1);
        }
        if (!issue(t, 0, uk)) { *abort_flag = 1; break; }
        ++nk;
      }
      if (t >= C::AHEAD) {
        const int j = t - C::AHEAD;
        if (!issue(j, 1, (u0 + j / NGRP) == uk_id ? uk : uprev)) { *abort_flag = 1; break; }
        ++nv;
      }
    }
    // no copy may land after this CTA's shared memory is released
    if (lane == 0) {
      for (int i = max(0, nk - NS); i < nk; ++i)
        if (!mbar_wait(&full_k[i % NS], (uint32_t)(i / NS) & 1u, a.err)) break;
      for (int i = max(0, nv - NS); i < nv; ++i)
        if (!mbar_wait(&full_v[i % NS], (uint32_t)(i / NS) & 1u, a.err)) break;
    }
  } else if (nK > 0 && warp == 1) {
    // ------------------------------------ MMA issuer ----------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_e4m3(0, 0), idesc_pv = umma_idesc_e4m3(1, 1);
      const uint32_t q_bytes = HKV * 2048, qf_bytes = HKV * 32;
      int bq = find_seq(prefix, a.B, u0), bp = bq, cur = -1, nq = 0, np = -1, pcur = -1;
      int pv_next = 0;  // next item whose PV is to be issued
      // O += V^T P^T for item j into the O buffer of its sequence (np: the sequence's index
      // among the sequences this CTA works on; empty sequences have no units and are skipped)
      auto issue_pv = [&](int j) -> bool {
        const int u = u0 + j / NGRP, g = j % NGRP;
        while (prefix[bp + 1] <= u) ++bp;
        if (bp != pcur) {
          ++np;
          pcur = bp;
        }
        const bool reset = (u == u0) || (u == prefix[bp]);
        const int slot = j % NS, pb = j & 1;
        if (!mbar_wait(&full_v[slot], (uint32_t)(j / NS) & 1u, a.err, abort_flag)) return false;
        if (!mbar_wait(&p_full[pb], (uint32_t)(j >> 1) & 1u, a.err, abort_flag)) return false;
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem_u32(ring_v + (size_t)slot * C::SLOT));
        const uint64_t db = umma_desc_noswz(smem_u32(ps + pb * C::P_WG), 128, C::P_NBLK);
        const uint32_t dcol = C::O_COL0 + (np & 1) * C::O_COLS + g * 32;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)  // 32 rows per step: 4096 B of V, 512 B of P
          umma_e4m3(tmem + dcol, da + 256 * ks, db + 32 * ks, idesc_pv, (ks > 0 || !reset) ? 1u : 0u);
        umma_commit(&pv_done[pb]);
        umma_commit(&empty_v[slot]);
        return true;
      };
      for (int kk = 0; kk < nK && !*abort_flag; ++kk) {
        const int u = u0 + kk / NGRP, g = kk % NGRP;
        while (prefix[bq + 1] <= u) ++bq;
        if (bq != cur) {
          // next sequence: finish the previous item's PV, let every MMA on the old Q complete,
          // then copy the new Q and its scales in
          if (pv_next < kk) {
            if (!issue_pv(pv_next)) { *abort_flag = 1; break; }
            ++pv_next;
          }
          umma_commit(q_free);
          if (!mbar_wait(q_free, (uint32_t)nq & 1u, a.err, abort_flag)) { *abort_flag = 1; break; }
          mbar_arrive_expect_tx(q_full, q_bytes + qf_bytes);
          bulk_g2s_plain(qs, a.ws_q8 + (size_t)bq * q_bytes, q_bytes, q_full);
          bulk_g2s_plain(qf_all + (nq & 1) * HKV * 8, a.ws_qf + (size_t)bq * HKV * 8, qf_bytes, q_full);
          if (!mbar_wait(q_full, (uint32_t)nq & 1u, a.err, abort_flag)) { *abort_flag = 1; break; }
          ++nq;
          cur = bq;
        }
        // S(kk) = K Q^T into the S buffer of warpgroup kk & 1
        const int slot = kk % NS, sb = kk & 1;
        if (!mbar_wait(&full_k[slot], (uint32_t)(kk / NS) & 1u, a.err, abort_flag)) { *abort_flag = 1; break; }
        if (kk >= 2 && !mbar_wait(&s_free[sb], (uint32_t)((kk - 2) >> 1) & 1u, a.err, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem_u32(ring_k + (size_t)slot * C::SLOT));
        const uint64_t db = umma_desc_sw128(smem_u32(qs + g * 2 * 2048));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_e4m3(tmem + sb * C::S_COLS, da + 2 * ks, db + 2 * ks, idesc_qk, ks > 0 ? 1u : 0u);
        umma_commit(&s_full[sb]);
        umma_commit(&empty_k[slot]);
        // then the PV of the previous item
        if (pv_next < kk) {
          if (!issue_pv(pv_next)) { *abort_flag = 1; break; }
          ++pv_next;
        }
      }
      while (!*abort_flag && pv_next < nK) {
        if (!issue_pv(pv_next)) { *abort_flag = 1; break; }
        ++pv_next;
      }
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, a.err);
    }
  } else if (nK > 0) {
    // --------------------------- softmax / correction / flush ---------------------------
    // Warpgroup w (warps 2 + 4w .. 5 + 4w) takes the items kk with kk & 1 == w: the head pairs
    // g with g & 1 == w of every unit, with their own S and P buffers.  A bounded wait that
    // expires sets the abort flag; the loop then runs on without waiting (every later wait
    // returns at once), so every thread of the warpgroup still meets every barrier.
    const int w = (warp - 2) >> 2;
    const int bar_id = 1 + w;
    const int wq = warp & 3;                    // TMEM lane quarter of this warp
    const int row = wq * 32 + lane;             // item row of S, d row of O
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const int G = a.G;
    const int hh = (row / a.P) & 1;             // this row's head within the pair
    const int rtok = (row / (2 * a.P)) * a.P + row % a.P;  // this row's token within the unit
    float* red = red_all + w * 128;
    float* flr = fl_all + w * 4 * GPW * 16;
    uint8_t* pw = ps + w * C::P_WG + hh * C::P_NBLK + row * 16;  // this row's P bytes
    // Per-thread partial sums of p (this row's head in each of the warpgroup's pairs); the
    // running maxima (equal in every thread) live in msh [pair][unit parity][head][row]: item
    // (u, g) reads what item (u - 1, g) wrote after its barrier and writes the other half after
    // its own, so readers and writers never overlap.
    float l_part[GPW][8];
    int b = find_seq(prefix, a.B, u0), cur = -1, nseq = 0, nit = 0;
    int kk_last = -1;       // this warpgroup's last item handed to the MMA warp
    int par_last = 0;       // unit parity of the current sequence's last unit
    int pend = -1, pend_par = 0, pend_obuf = 0;  // a finished sequence whose partial is not yet written
    const float* qf = qf_all;

    // Writes the split-KV partial of sequence bb (this warpgroup's heads) from O buffer obuf,
    // the maxima of unit parity par and the l sums in flr.  Needs the sequence's PVs done.
    auto flush = [&](int bb, int par, int obuf) {
      tc_fence_after();
      const size_t slot = (size_t)blockIdx.x + bb;
#pragma unroll
      for (int gl = 0; gl < GPW; ++gl) {
        const int g = 2 * gl + w;
        float o[32];
        tmem_ld32(tmem + lane_base + C::O_COL0 + obuf * C::O_COLS + g * 32, o);
#pragma unroll
        for (int hp = 0; hp < 2; ++hp)
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            if (r < G) {
              const size_t rowi = slot * a.Hq + (2 * g + hp) * G + r;
              a.ws_acc[rowi * 128 + row] = o[hp * 16 + r] * (1.f / 256.f) + o[hp * 16 + 8 + r] * (1.f / 4096.f);
            }
          }
      }
      if (row < GPW * 16) {
        const int gl = row >> 4, i = row & 15, hp = i >> 3, r = i & 7;
        const int g = 2 * gl + w;
        if (r < G) {
          const float mv = msh[(g * 2 + par) * 16 + i];
          const float lv = flr[gl * 16 + i] + flr[GPW * 16 + gl * 16 + i] + flr[2 * GPW * 16 + gl * 16 + i] +
                           flr[3 * GPW * 16 + gl * 16 + i];
          const size_t rowi = slot * a.Hq + (2 * g + hp) * G + r;
          a.ws_ml[rowi * 2] = mv;
          a.ws_ml[rowi * 2 + 1] = lv;
        }
      }
    };
    // l sums of the finished sequence into flr: per (pair, head, row), per warp (after every
    // thread has finished reading flr for the previous flush)
    auto reduce_l = [&]() {
      wg_bar(bar_id);
#pragma unroll
      for (int gl = 0; gl < GPW; ++gl)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float s = warp_sum((i >> 3) == hh ? l_part[gl][i & 7] : 0.f);
          if (lane == 0) flr[wq * GPW * 16 + gl * 16 + i] = s;
        }
    };

    for (int u = u0; u < u1; ++u) {
      while (prefix[b + 1] <= u) ++b;
      const bool first = (u == u0) || (u == prefix[b]);
      if (b != cur) {
        if (cur >= 0) {  // the previous sequence's partial is written during this unit
          reduce_l();
          pend = cur;
          pend_par = par_last;
          pend_obuf = (nseq - 1) & 1;
        }
        qf = qf_all + (nseq & 1) * HKV * 8;
        if (!mbar_wait(q_full, (uint32_t)nseq & 1u, a.err, abort_flag)) *abort_flag = 1;
        ++nseq;
#pragma unroll
        for (int gl = 0; gl < GPW; ++gl)
#pragma unroll
          for (int r = 0; r < 8; ++r) l_part[gl][r] = 0.f;
        cur = b;
      }
      const int len = lens[b];
      const int lo = seq_lo(len, a.window);
      const int t0 = seq_origin(len, a.window, a.P) + (u - prefix[b]) * C::TILE;
      const int tok = t0 + rtok;
      const bool valid = tok >= lo && tok < len;
      const bool tail = t0 + C::TILE > len;
      const int par = (u - u0) & 1;
      par_last = par;
#pragma unroll
      for (int gl = 0; gl < GPW; ++gl) {
        const int g = 2 * gl + w;
        const int kk = (u - u0) * NGRP + g;  // kk & 1 == w
        if (!mbar_wait(&s_full[w], (uint32_t)(kk >> 1) & 1u, a.err, abort_flag)) *abort_flag = 1;
        tc_fence_after();
        float S[32];
        tmem_ld32(tmem + lane_base + w * C::S_COLS, S);
        // scores of this row's head, log2 domain: (S1 + S2/16) * 2^-a * k_scale * sm_scale * log2(e)
        const float* qfh = qf + (2 * g + hh) * 8;
        float v16[16];
        float s[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float s1 = hh ? S[16 + r] : S[r];
          const float s2 = hh ? S[24 + r] : S[8 + r];
          s[r] = (valid && r < G) ? (s1 + s2 * 0.0625f) * qfh[r] : -INFINITY;
          v16[r] = hh ? -INFINITY : s[r];
          v16[8 + r] = hh ? s[r] : -INFINITY;
        }
        // S may be overwritten now; the query scales of this sequence have been read
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[w]);
        wg_max16(v16, red + (nit & 1) * 64, wq, lane, bar_id);  // v16 = tile maxima of both heads
        ++nit;
        float alpha[16], muse[16];
        bool rescale = false;
        const float* mprev = msh + (g * 2 + (par ^ 1)) * 16;
        float* mnext = msh + (g * 2 + par) * 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float mold = first ? -INFINITY : mprev[i];
          const float mn = fmaxf(mold, v16[i]);
          muse[i] = mn == -INFINITY ? 0.f : mn;
          alpha[i] = fast_exp2(mold - muse[i]);
          if ((i & 7) < G && alpha[i] != 1.f) rescale = true;
          if (row == i) mnext[i] = mn;
        }
        rescale = rescale && !first;  // the first tile of a sequence resets O instead
        // P[w] is free and this pair's O is current once this warpgroup's previous item is done
        if (kk >= 2) {
          if (!mbar_wait(&pv_done[w], (uint32_t)((kk - 2) >> 1) & 1u, a.err, abort_flag)) *abort_flag = 1;
          tc_fence_after();
        }
        if (pend >= 0) {  // the finished sequence's PVs are done now: write its partial
          flush(pend, pend_par, pend_obuf);  // flr was written before this item's barrier
          pend = -1;
        }
        if (rescale) {
          float o[32];
          const uint32_t ta = tmem + lane_base + C::O_COL0 + ((nseq - 1) & 1) * C::O_COLS + g * 32;
          tmem_ld32(ta, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = (i >> 3) * 16 + (i & 7);
            o[c] *= alpha[i];
            o[c + 8] *= alpha[i];
          }
          tmem_st32(ta, o);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        // probabilities, partial sums, and P as two e4m3 terms (p * 256 ~= p1 + p2 / 16)
        {
          uint32_t w1[2] = {0u, 0u}, w2[2] = {0u, 0u};
#pragma unroll
          for (int r = 0; r < 8; r += 2) {
            const float a0 = hh ? alpha[8 + r] : alpha[r], a1 = hh ? alpha[9 + r] : alpha[r + 1];
            const float m0 = hh ? muse[8 + r] : muse[r], m1 = hh ? muse[9 + r] : muse[r + 1];
            const float p0 = (r < G && valid) ? fast_exp2(s[r] - m0) : 0.f;
            const float p1 = (r + 1 < G && valid) ? fast_exp2(s[r + 1] - m1) : 0.f;
            l_part[gl][r] = l_part[gl][r] * a0 + p0;
            l_part[gl][r + 1] = l_part[gl][r + 1] * a1 + p1;
            const __half2 xh = __floats2half2_rn(p0 * 256.f, p1 * 256.f);
            const uint16_t t1 = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(xh), __NV_SATFINITE, __NV_E4M3);
            const __half2 bk = __half2(__nv_cvt_fp8x2_to_halfraw2(t1, __NV_E4M3));
            const __half2 rs = __hmul2(__hsub2(xh, bk), __float2half2_rn(16.f));
            const uint16_t t2 = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(rs), __NV_SATFINITE, __NV_E4M3);
            w1[r >> 2] |= (uint32_t)t1 << (16 * ((r >> 1) & 1));
            w2[r >> 2] |= (uint32_t)t2 << (16 * ((r >> 1) & 1));
          }
          *reinterpret_cast<uint4*>(pw) = make_uint4(w1[0], w1[1], w2[0], w2[1]);
        }
        if (tail) {
          // rows past the context hold stale or unwritten cache bytes: zero this item's V rows
          // there (after its copy landed) so that 0 * NaN cannot reach the accumulator
          const int slot = kk % NS;
          if (!mbar_wait(&full_v[slot], (uint32_t)(kk / NS) & 1u, a.err, abort_flag)) *abort_flag = 1;
          if (tok >= len) {
            uint4* vr = reinterpret_cast<uint4*>(ring_v + (size_t)slot * C::SLOT + row * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) vr[c] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[w]);
        kk_last = kk;
      }
    }
    if (cur >= 0) {
      if (!mbar_wait(&pv_done[w], (uint32_t)(kk_last >> 1) & 1u, a.err, abort_flag)) *abort_flag = 1;
      reduce_l();
      wg_bar(bar_id);
      flush(cur, par_last, (nseq - 1) & 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------------------
// Host side.  The tensor maps view a cache [pages][P][Hkv][128] e4m3 as 4-D (d, token, head,
// page) with byte strides (Hkv*128, 128, P*Hkv*128); a box is one page of a pair of heads,
// landing as [head][P tokens][128 B].
static bool make_kv_map(CUtensorMap* m, const void* base, int hkv, int P, long long pages) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[4] = {128, (cuuint64_t)P, (cuuint64_t)hkv, (cuuint64_t)pages};
  cuuint64_t strides[3] = {(cuuint64_t)hkv * 128, 128, (cuuint64_t)P * hkv * 128};
  cuuint32_t box[4] = {128, (cuuint32_t)P, 2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HKV>
static size_t tc_attn_smem(int B) {
  return (size_t)TcAttnCfg<HKV>::BODY + 1024 + (size_t)(2 * B + 1) * sizeof(int);
}

size_t attn_q8_ws_bytes(int B, int Hkv) { return (size_t)B * Hkv * (2048 + 32); }

bool attn_tc_eligible(const AttnArgs& a, int D, int Hkv) {
  // OKC_ATTN_TC=1 selects this kernel where it applies; otherwise the mma.sync kernel serves
  // every shape (read per call, so tests can compare the two kernels in one process)
  const char* e = getenv("OKC_ATTN_TC");
  if (!(e && e[0] == '1') || D != 128 || a.G > 8 || a.B > 2048 || !(Hkv == 4 || Hkv == 8)) return false;
  if (!(a.P == 16 || a.P == 32 || a.P == 64) || a.num_pages >= (1ll << 31) || !a.ws_q8 || !a.ws_qf) return false;
  if (tensor_map_encoder() == nullptr) return false;
  return (Hkv == 8 ? tc_attn_smem<8>(a.B) : tc_attn_smem<4>(a.B)) <= 232448;
}

template <int HKV>
static int launch_attn_tc_t(AttnArgs& a, cudaStream_t stream) {
  CUtensorMap mk, mv;
  if (!make_kv_map(&mk, a.k_cache, HKV, a.P, a.num_pages) || !make_kv_map(&mv, a.v_cache, HKV, a.P, a.num_pages))
    return OKC_ERR_INVALID;
  const size_t smem = tc_attn_smem<HKV>(a.B);
  static size_t configured = 0;
  if (smem > configured) {
    if (cudaFuncSetAttribute(attn_tc_kernel<HKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = smem;
  }
  int st = okc_host::launch_k(attn_q8_kernel, dim3(a.B), dim3(128), 0, stream, dim3(1), a, HKV);
  if (st) return st;
  st = okc_host::launch_k(attn_tc_kernel<HKV>, dim3(a.num_ctas), dim3(TcAttnCfg<HKV>::THREADS), smem, stream,
                          dim3(1), mk, mv, a);
  if (st) return st;
  return launch_attn_merge(a, TcAttnCfg<HKV>::TILE, 1, 128, stream);
}

int launch_attn_tc(AttnArgs& a, int Hkv, cudaStream_t stream) {
  switch (Hkv) {
    case 4: return launch_attn_tc_t<4>(a, stream);
    case 8: return launch_attn_tc_t<8>(a, stream);
  }
  return OKC_ERR_INVALID;
}

}  // namespace okc
