// tcgen05 (5th-generation tensor core) BF16 GEMM for projections of 33..256 tokens:
// y[M,N] = x[M,K] · W[N,K]^T (+ residual), fp32 accumulate in tensor memory (TMEM).
//
// Roofline: HBM on the weight stream at decode token counts (2*N*K bytes; the arithmetic
// intensity is M flop/byte, far below the ~250 flop/byte ridge of B200).
// Design (B200):
//  * swap-AB: the weight tile is the MMA's 128-row A operand, the tokens are its N side
//    (BN = 64/128/256), so one CTA tile covers 128 weight rows x all tokens and the weight
//    matrix is read exactly once.
//  * warp 0 (one thread) streams K-tiles of W [128 x 64] and x [BN x 64] with 2-D TMA loads
//    (SWIZZLE_128B, the canonical K-major UMMA layout) into a STAGES-deep mbarrier ring;
//    warp 1 (one thread) issues tcgen05.mma kind::f16 (K = 16 per instruction) with the
//    accumulator in TMEM and frees each stage with tcgen05.commit;
//  * persistent stream-K grid (one CTA per SM): the (tile, K-block) units are split evenly
//    over the CTAs, so every SM streams the same number of bytes whatever N and K are;
//  * 4 epilogue warps drain the double-buffered TMEM accumulator with tcgen05.ld (warp w owns
//    TMEM lanes 32(w%4)..+31 = weight rows) while the next segment's MMAs run.  A tile that
//    one CTA covers whole is written directly; a split tile leaves one fp32 partial slot per
//    contributing CTA, and tc_reduce_kernel (all SMs, launched as a programmatic dependent of
//    the GEMM) sums each tile's slots in slot order (deterministic).  A last-arriver fixup
//    inside the GEMM put up to 4 x 64 KB of L2 reads on one SM at the end of the stream
//    (11-13 us on B200 with the HBM still saturated); spread over every SM it takes ~2 us.
// Every mbarrier wait is bounded (common.cuh); TMEM is always released before exit.
// Mirrors the M >= 32 tensor-core path of muse_bf16_proj/projection/kernels/{tma,
// hopper_ws}.py and muse_decode_layer/decode/projections.py:75-77 (there: cuBLAS / wgmma).
#include <cudaTypedefs.h>
#include <stdlib.h>

#include "kernels.cuh"
#include "tcgen05.cuh"

namespace okc {

// Optional epilogue of the QKV projection: interleaved RoPE on the q and k columns, q to
// bf16 [M][Hq][D], k and v quantised to e4m3 into the paged caches at slot(token) (the work of
// rope_append_kernel, fused so the bf16 qkv never goes to HBM).  Output column n = head*D + d
// with heads [0, Hq) = q, [Hq, Hq + Hkv) = k, [Hq + Hkv, Hq + 2 Hkv) = v.
struct TcRopeEpi {
  const int64_t* positions;
  const int32_t* page_table;
  int table_ld, max_pages;
  const float* inv_freq;
  const float* k_scale;
  const float* v_scale;
  __nv_bfloat16* q_out;
  uint8_t* k_cache;
  uint8_t* v_cache;
  int64_t* slots_out;
  int Hq, Hkv, D, P;
  long long num_pages;
  float q_scale;
};

struct TcParams {
  int M, N, K, ldy, out_fp32, tiles;
  void* y;
  const __nv_bfloat16* residual;
  int* err;
  float* part;    // stream-K partial slots [ctas + tiles][BN][128] (workspace)
  int rope_on;    // 1: every tile goes through tc_reduce_kernel, which applies `rope`
  TcRopeEpi rope;
};

template <int BN, int STAGES, int KS = 1>
struct TcCfg {
  static constexpr int A_BOX = TC_BM * TC_BK * 2;  // one 128 x 64 W box
  static constexpr int B_BOX = BN * TC_BK * 2;     // one BN x 64 x box
  static constexpr int A_BYTES = A_BOX * KS;       // KS adjacent K boxes per stage
  static constexpr int B_BYTES = B_BOX * KS;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BODY = STAGE * STAGES;
  static constexpr int SMEM = 1024 + BODY + 256;  // alignment slack + body + barriers
  static constexpr int TMEM_COLS = 2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512));
};

__host__ __device__ __forceinline__ void sk_range(int U, int C, int c, int& u0, int& u1) {
  const int q = U / C, r = U % C;
  u0 = c * q + (c < r ? c : r);
  u1 = u0 + q + (c < r ? 1 : 0);
}
__host__ __device__ __forceinline__ int sk_owner(int U, int C, int u) {
  const int q = U / C, r = U % C;
  const int big = r * (q + 1);
  return u < big ? u / (q + 1) : r + (u - big) / q;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Persistent stream-K: the (tile, K-block) units of the whole GEMM are split evenly over the
// grid; a CTA's consecutive units form at most a few segments, one per weight tile it touches.
// Warp 0: TMA producer.  Warp 1: MMA issuer (double-buffered TMEM accumulator).  Warps 2..5:
// epilogue (TMEM lane quarter = warp % 4).  A segment that covers its whole tile stores y
// directly; otherwise it stores an fp32 partial (m-major, coalesced) into slot (CTA + tile).
template <int BN, int STAGES, int KS>
__global__ void __launch_bounds__(192) tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_w,
                                                         const __grid_constant__ CUtensorMap tma_x,
                                                         TcParams p) {
  using C = TcCfg<BN, STAGES, KS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator buffer ready for the epilogue
  uint64_t* acce = accf + 2;        // [2] accumulator buffer drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the dependent reduce kernel may launch now: it waits for this grid before reading
  pdl_trigger();
  const int nkb = (p.K + TC_BK * KS - 1) / (TC_BK * KS);  // stages (units) per tile
  const int U = p.tiles * nkb;
  int u0, u1;
  sk_range(U, gridDim.x, blockIdx.x, u0, u1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // barriers and TMEM are set up; the inputs are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------- TMA producer ----------------------------
      int issued = 0;
      for (int u = u0; u < u1; ++u, ++issued) {
        const int s = issued % STAGES;
        const uint32_t ph = (uint32_t)(issued / STAGES) & 1u;
        if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u, p.err)) { *abort_flag = 1; break; }
        const int tile = u / nkb, kb = u - tile * nkb;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        uint8_t* sa = smem + s * C::STAGE;
#pragma unroll
        for (int i = 0; i < KS; ++i) {  // adjacent K boxes back to back: longer DRAM bursts per row
          tma_load_2d(sa + i * C::A_BOX, &tma_w, (kb * KS + i) * TC_BK, tile * TC_BM, &full[s]);
          tma_load_2d(sa + C::A_BYTES + i * C::B_BOX, &tma_x, (kb * KS + i) * TC_BK, 0, &full[s]);
        }
      }
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        if (!mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, p.err)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------- MMA issuer -------------------------------
      const uint32_t idesc = umma_idesc_bf16(BN);
      int done = 0, seg = 0;
      bool first = true;
      for (int u = u0; u < u1; ++u, ++done) {
        const int tile = u / nkb, kb = u - tile * nkb;
        const int buf = seg & 1;
        if (u == u0 || kb == 0) {  // a new segment: wait until the epilogue freed this buffer
          if (*abort_flag || !mbar_wait(&acce[buf], ((uint32_t)(seg >> 1) & 1u) ^ 1u, p.err)) {
            *abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          first = true;
        }
        const int s = done % STAGES;
        if (*abort_flag || !mbar_wait(&full[s], (uint32_t)(done / STAGES) & 1u, p.err)) { *abort_flag = 1; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sa = smem_u32(smem + s * C::STAGE);
#pragma unroll
        for (int i = 0; i < KS; ++i) {
          const uint64_t da = umma_desc_sw128(sa + i * C::A_BOX), db = umma_desc_sw128(sa + C::A_BYTES + i * C::B_BOX);
#pragma unroll
          for (int j = 0; j < TC_BK / 16; ++j)
            umma_bf16(tmem + buf * BN, da + 2 * j, db + 2 * j, idesc, (first && i == 0 && j == 0) ? 0u : 1u);
        }
        first = false;
        umma_commit(&empty[s]);
        if (u == u1 - 1 || kb == nkb - 1) {  // segment complete: hand the buffer to the epilogue
          umma_commit(&accf[buf]);
          ++seg;
        }
      }
      // on abort, release every epilogue wait that can still be pending
      if (*abort_flag)
        for (int i = 0; i < 2; ++i) umma_commit(&accf[i]);
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;  // TMEM lane = weight row within the tile
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    int seg = 0;
    for (int u = u0; u < u1; ++seg) {
      const int tile = u / nkb, kb_first = u - tile * nkb;
      const int seg_end = min(u1, (tile + 1) * nkb);
      const bool whole = kb_first == 0 && seg_end == (tile + 1) * nkb && !p.rope_on;
      const int buf = seg & 1;
      const bool ok = mbar_wait(&accf[buf], (uint32_t)(seg >> 1) & 1u, p.err) && !*abort_flag;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int n = tile * TC_BM + row;
      const uint32_t taddr = tmem + lane_base + buf * BN;
      if (whole) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          if (!ok || n >= p.N) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c0 + j;
            if (m >= p.M) break;
            float r = v[j];
            if (p.residual) r += __bfloat162float(p.residual[(size_t)m * p.ldy + n]);
            if (p.out_fp32)
              reinterpret_cast<float*>(p.y)[(size_t)m * p.ldy + n] = r;
            else
              reinterpret_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] = __float2bfloat16_rn(r);
          }
        }
      } else {
        float* mine = p.part + (size_t)(blockIdx.x + tile) * BN * TC_BM;  // [m][row] for this slot
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) mine[(size_t)(c0 + j) * TC_BM + row] = v[j];
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);  // the MMA warp may reuse this buffer now
      u = seg_end;
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// RoPE + FP8 KV-append of 4 consecutive projection outputs (token m, columns n4..n4+3, one
// head: D % 4 == 0), in the arithmetic of rope_append_kernel (sincosf of pos * inv_freq, RN
// fp32 rotation, q * q_scale -> bf16, k|v / scale -> e4m3 RN, NaN on overflow).  rope_prep
// runs before the partial sums are loaded (its page-table reads and sincosf overlap them).
struct RopeCtx {
  long long slot;
  float sn[2], cs[2];
  int head, d0;
  bool is_v;
};

__device__ __forceinline__ RopeCtx rope_prep(const TcRopeEpi& e, int m, int n4, int* err) {
  RopeCtx c;
  const long long pos = e.positions[m];
  const long long lp = pos / e.P;
  c.slot = -1;
  if (pos >= 0 && lp < e.max_pages) {
    const int page = e.page_table[(size_t)m * e.table_ld + lp];
    if (page >= 0 && page < e.num_pages) c.slot = (long long)page * e.P + pos % e.P;
  }
  if (n4 == 0) {  // once per token
    if (c.slot < 0) atomicOr(err, OKC_DEVERR_PAGE);
    if (e.slots_out) e.slots_out[m] = c.slot;
  }
  c.head = n4 / e.D;
  c.d0 = n4 - c.head * e.D;
  c.is_v = c.head >= e.Hq + e.Hkv;
  c.sn[0] = c.sn[1] = 0.f;
  c.cs[0] = c.cs[1] = 1.f;
  if (e.inv_freq && !c.is_v) {
    const float posf = (float)pos;
#pragma unroll
    for (int k = 0; k < 2; ++k) sincosf(__fmul_rn(posf, e.inv_freq[c.d0 / 2 + k]), &c.sn[k], &c.cs[k]);
  }
  return c;
}

__device__ __forceinline__ void rope_apply(const TcRopeEpi& e, const RopeCtx& c, int m, float (&x)[4]) {
  if (e.inv_freq && !c.is_v) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float y0 = __fsub_rn(__fmul_rn(x[2 * k], c.cs[k]), __fmul_rn(x[2 * k + 1], c.sn[k]));
      const float y1 = __fadd_rn(__fmul_rn(x[2 * k], c.sn[k]), __fmul_rn(x[2 * k + 1], c.cs[k]));
      x[2 * k] = y0;
      x[2 * k + 1] = y1;
    }
  }
  if (c.head < e.Hq) {
    if (e.q_scale != 1.f) {
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] *= e.q_scale;
    }
    *reinterpret_cast<uint2*>(e.q_out + ((size_t)m * e.Hq + c.head) * e.D + c.d0) =
        make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
  } else if (c.slot >= 0) {
    const int h = c.is_v ? c.head - e.Hq - e.Hkv : c.head - e.Hq;
    const float sc = c.is_v ? e.v_scale[h] : e.k_scale[h];
    uint32_t v = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) v |= (uint32_t)f_to_e4m3_nosat(__fdiv_rn(x[k], sc)) << (8 * k);
    uint8_t* cache = c.is_v ? e.v_cache : e.k_cache;
    *reinterpret_cast<uint32_t*>(cache + ((size_t)c.slot * e.Hkv + h) * e.D + c.d0) = v;
  }
}

// Split-tile reduction: y[m, tile*128 + r] = sum over the tile's slots (in slot order) of the
// partials (+ residual).  Block (x, tile) covers tokens [8x, 8x + 8) x 128 rows; thread t owns 4
// consecutive rows of one token (float4 loads, all slots' loads issued before the sum).
template <int BN>
__global__ void __launch_bounds__(256) tc_reduce_kernel(TcParams p, int U, int C, int nkb) {
  pdl_trigger();
  pdl_wait();  // the GEMM grid is complete and its partials visible
  const int tile = blockIdx.y;
  const int c_first = sk_owner(U, C, tile * nkb), c_last = sk_owner(U, C, (tile + 1) * nkb - 1);
  if (c_first == c_last && !p.rope_on) return;  // one CTA covered the tile: written directly
  const int m = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (m >= p.M) return;
  const int r4 = 4 * (threadIdx.x & 31);
  const int n4 = tile * TC_BM + r4;
  const int nslot = c_last - c_first + 1;
  const float* base = p.part + (size_t)(c_first + tile) * BN * TC_BM + (size_t)m * TC_BM + r4;
  const size_t slot_stride = (size_t)BN * TC_BM;
  RopeCtx rc;
  if (p.rope_on && n4 < p.N) rc = rope_prep(p.rope, m, n4, p.err);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
  for (int q0 = 0; q0 < nslot; q0 += 8) {
    float4 t4[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      t4[i] = q0 + i < nslot ? __ldcg(reinterpret_cast<const float4*>(base + (q0 + i) * slot_stride))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) { acc.x += t4[i].x; acc.y += t4[i].y; acc.z += t4[i].z; acc.w += t4[i].w; }
  }
  float r[4] = {acc.x, acc.y, acc.z, acc.w};
  if (p.rope_on) {
    // the unfused path rounds the projection to bf16 before RoPE: do the same
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __bfloat162float(__float2bfloat16_rn(r[j]));
    if (n4 < p.N) rope_apply(p.rope, rc, m, r);
    return;
  }
  const size_t o = (size_t)m * p.ldy + n4;
  if (n4 + 3 < p.N && (o & 3) == 0) {
    if (p.residual) {
      const uint2 rv = *reinterpret_cast<const uint2*>(p.residual + o);
      r[0] += bf16_lo(rv.x); r[1] += bf16_hi(rv.x); r[2] += bf16_lo(rv.y); r[3] += bf16_hi(rv.y);
    }
    if (p.out_fp32)
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.y) + o) = make_float4(r[0], r[1], r[2], r[3]);
    else
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.y) + o) =
          make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (n4 + j >= p.N) break;
      float rv = r[j];
      if (p.residual) rv += __bfloat162float(p.residual[o + j]);
      if (p.out_fp32)
        reinterpret_cast<float*>(p.y)[o + j] = rv;
      else
        reinterpret_cast<__nv_bfloat16*>(p.y)[o + j] = __float2bfloat16_rn(rv);
    }
  }
}

// ------------------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool tc_make_map(CUtensorMap* m, const void* base, int inner, int rows, int ld, int box_rows) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_gemm_supported(int M, int N, int K, int ldx, int ldw) {
  return M >= 1 && M <= 256 && N >= 1 && K >= 16 && K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 &&
         tensor_map_encoder() != nullptr;
}

struct TcPlan {
  int bn, tiles, nkb, ctas, per_sm, ks;
};

// Variant: "1" = one CTA per SM with 64-wide K stages, "2" = two CTAs per SM, "w" (default) =
// one CTA per SM with two adjacent 64-wide K boxes per stage (256-byte DRAM bursts per row).
// OKC_TC_VARIANT selects another one for tuning sweeps.
static char tc_variant() {
  static char v = 0;
  if (!v) {
    const char* e = getenv("OKC_TC_VARIANT");
    v = (e && (e[0] == '1' || e[0] == '2' || e[0] == 'w')) ? e[0] : 'w';
  }
  return v;
}

// Persistent grid of (CTAs per SM) x SMs; at most one CTA per (tile, K block) unit.
static TcPlan tc_plan(int M, int N, int K) {
  TcPlan pl;
  pl.bn = M <= 64 ? 64 : (M <= 128 ? 128 : 256);
  const char v = pl.bn == 256 ? '1' : tc_variant();
  pl.per_sm = v == '2' ? 2 : 1;
  pl.ks = v == 'w' ? 2 : 1;
  pl.tiles = (N + TC_BM - 1) / TC_BM;
  pl.nkb = (K + TC_BK * pl.ks - 1) / (TC_BK * pl.ks);
  const long long units = (long long)pl.tiles * pl.nkb;
  long long slots = (long long)okc_host::num_sms() * pl.per_sm;
  static int cap = -1;  // OKC_TC_MAX_CTAS: grid cap for tuning sweeps (0 = none)
  if (cap < 0) {
    const char* e = getenv("OKC_TC_MAX_CTAS");
    cap = e ? atoi(e) : 0;
  }
  if (cap > 0 && slots > cap) slots = cap;
  // Few tiles (small N): split each tile over at most 8 CTAs; wider splits cost more partial
  // traffic and reduce work than they gain (N = 1280, K = 8192, M = 128 on B200: 2 CTAs per
  // tile 24.2 us, 4: 15.2, 8: 11.4, 16: 12.5, no cap: 12.7).
  static int split = -1;  // OKC_TC_SPLIT: CTAs per tile cap for tuning sweeps (default 8)
  if (split < 0) {
    const char* e = getenv("OKC_TC_SPLIT");
    split = e ? atoi(e) : 8;
  }
  if (split > 0 && slots > (long long)split * pl.tiles) slots = (long long)split * pl.tiles;
  pl.ctas = (int)(units < slots ? units : slots);
  return pl;
}

// Workspace: [kTcCounterBytes reserved][fp32 partial slots: (ctas + tiles) x BN x 128].
constexpr size_t kTcCounterBytes = 16384;  // reserved (N <= 524288: 4096 tiles of 128 rows)

size_t tc_gemm_ws_bytes(int M, int N, int K) {
  if (M < 1 || M > 256 || N < 1 || K < 1) return 0;
  const TcPlan pl = tc_plan(M, N, K);
  return kTcCounterBytes + (size_t)(pl.ctas + pl.tiles) * pl.bn * TC_BM * 4;
}

template <int BN, int STAGES, int KS = 1>
static int launch_tc_t(const void* x, int ldx, const void* w, int ldw, TcParams& p, const TcPlan& pl,
                       void* ws, size_t ws_bytes, cudaStream_t stream) {
  using C = TcCfg<BN, STAGES, KS>;
  CUtensorMap mw, mx;
  if (!tc_make_map(&mw, w, p.K, p.N, ldw, TC_BM) || !tc_make_map(&mx, x, p.K, p.M, ldx, BN)) return OKC_ERR_INVALID;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<BN, STAGES, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = true;
  }
  const size_t part_bytes = (size_t)(pl.ctas + pl.tiles) * BN * TC_BM * 4;
  if (!ws || ws_bytes < kTcCounterBytes + part_bytes || (size_t)pl.tiles * 4 > kTcCounterBytes)
    return OKC_ERR_WORKSPACE;  // (the tile-count bound keeps the documented N limit)
  p.tiles = pl.tiles;
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kTcCounterBytes);
  int st = okc_host::launch_k(tc_gemm_kernel<BN, STAGES, KS>, dim3(pl.ctas), dim3(192), C::SMEM, stream, dim3(1),
                              mw, mx, p);
  if (st) return st;
  // Reduce of the split tiles, as a programmatic dependent launch: its blocks may be scheduled
  // while the GEMM drains and wait in griddepcontrol.wait until the GEMM grid has completed.
  if ((long long)pl.tiles * pl.nkb <= pl.ctas && pl.nkb == 1 && !p.rope_on) return OKC_OK;  // no split tile
  const int U = pl.tiles * pl.nkb;
  return okc_host::launch_k(tc_reduce_kernel<BN>, dim3((unsigned)((min(p.M, BN) + 7) / 8), (unsigned)pl.tiles),
                            dim3(256), 0, stream, dim3(1), p, U, pl.ctas, pl.nkb);
}

int launch_tc_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, const void* residual, int M,
                   int N, int K, int out_fp32, void* ws, size_t ws_bytes, cudaStream_t stream,
                   const TcRopeArgs* rope) {
  TcParams p = {};
  p.rope_on = rope != nullptr;
  if (rope) {
    p.rope.positions = rope->positions;
    p.rope.page_table = rope->page_table;
    p.rope.table_ld = rope->table_ld;
    p.rope.max_pages = rope->max_pages;
    p.rope.inv_freq = rope->inv_freq;
    p.rope.k_scale = rope->k_scale;
    p.rope.v_scale = rope->v_scale;
    p.rope.q_out = reinterpret_cast<__nv_bfloat16*>(rope->q_out);
    p.rope.k_cache = reinterpret_cast<uint8_t*>(rope->k_cache);
    p.rope.v_cache = reinterpret_cast<uint8_t*>(rope->v_cache);
    p.rope.slots_out = rope->slots_out;
    p.rope.Hq = rope->Hq;
    p.rope.Hkv = rope->Hkv;
    p.rope.D = rope->D;
    p.rope.P = rope->P;
    p.rope.num_pages = rope->num_pages;
    p.rope.q_scale = rope->q_scale;
  }
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldy = ldy;
  p.out_fp32 = out_fp32;
  p.y = y;
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.err = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) - 256);  // the caller's error word
  const TcPlan pl = tc_plan(M, N, K);
  if (pl.bn == 64) {
    if (pl.ks == 2) return launch_tc_t<64, 4, 2>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
    return pl.per_sm == 2 ? launch_tc_t<64, 4>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream)
                          : launch_tc_t<64, 8>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
  }
  if (pl.bn == 128) {
    if (pl.ks == 2) return launch_tc_t<128, 3, 2>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
    return pl.per_sm == 2 ? launch_tc_t<128, 3>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream)
                          : launch_tc_t<128, 6>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
  }
  return launch_tc_t<256, 4>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
}

}  // namespace okc
