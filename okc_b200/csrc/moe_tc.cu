// NVFP4 (W4A16) expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), for MoE steps
// whose experts see more than a few tokens (the row-owning mma.sync kernel in moe.cu serves the
// few-token decode steps).  Same contract as the moe.cu expert kernels
// (muse_moe_w4a16/submission.py:163-248): gate/up h = bf16(acc * gs), inter = bf16(silu(g) * u),
// down y = bf16(acc * gs), fp32 accumulation.
//
//  * moe_rows_f16_kernel turns bf16 activation rows into f16 rows scaled by 2^s_j, s_j chosen per
//    row so that its largest magnitude lands in [2^14, 2^15): every bf16 value of the row is then
//    exact in f16 (no overflow; only values below 2^-28 of the row maximum reach f16 subnormals),
//    and the epilogue multiplies by rs[j] = 2^-s_j.  Since the dequantised weights (e2m1 x e4m3,
//    at most 5 significant bits) are exact in f16 too, the f16 MMAs form exactly the products a
//    bf16 MMA of the reference's operands would.  Before the gate/up GEMM it gathers the local
//    (token, slot) pairs expert-major (row j = x[pairs[j] / topk]); before the down GEMM it
//    converts the bf16 intermediate rows.
//  * The dequantised weights never touch shared memory: they are the MMA's A operand in tensor
//    memory (lane = weight row, column c = the f16 pair of K 2c, 2c+1), written by tcgen05.st
//    from the registers that decoded them.  Shared memory only carries the packed codes (one
//    TMA write, one read) and the activation tiles, so its bandwidth is not the limit; per 64
//    K the tensor pipe then needs 4 MMAs (M = 128 weight rows, N = the chunk's pairs, K = 16),
//    issued from one thread at ~50 cycles each.
//  * A unit = (active expert, chunk of <= NT of its pairs, 128 weight rows: 64 gate + the same 64
//    up rows (GATED) or 128 down rows) over the full K.  Units of all experts are split evenly
//    over a persistent grid (one CTA per SM).
//  * Warp 0 streams the unit's packed codes and e4m3 scales with 2-D TMA boxes (256 K per stage:
//    one 128-byte row of codes per weight row, 128-byte swizzle, plus 16 scale bytes a row) into
//    the raw ring (8 stages at NT = 32, 6 at NT = 64).  Warp 2 loads the stage's activation tiles
//    (4 boxes of 64 K x 16/32/64 rows, f16, 128-byte swizzle) into the activation ring, one slot
//    deeper than the A slots (MtCfg below).
//  * Warps 3..10 dequantise, two per TMEM lane quarter (one per 128-K half of a stage), lane =
//    one weight row: the stage's codes and scales into registers (the raw slot is freed there),
//    cvt.rn.f16x2.e2m1x2, x the e4m3 group scale in f16 (exact), tcgen05.st into the stage's A
//    slot (128 columns; 3 slots at NT = 32, 2 at NT = 64), tcgen05.wait::st, tcgen05.fence,
//    mbarrier arrive (warp 3's arrival also waits for the stage's activation tiles).
//    f16 rather than bf16 because the e2m1 -> f16x2 conversion is one instruction; the same
//    product in bf16 takes about four more integer operations per pair.
//  * Two issuer threads (warps 1 and 15, on different SM sub-partitions; four at NT = 32): issuer
//    h issues the 8 MMAs of K half h of each stage into its own double-buffered TMEM accumulator and frees the
//    stage (A slot and activation slot) with one tcgen05.commit (the stage's done barrier counts
//    both).  At NT = 32 four threads (warps 1, 15, 16, 18) issue a K quarter each.  Measured:
//    issuing half the MMAs (a timing-only variant) takes 10-15 % off the expert time, four
//    issuers instead of two only 2-3 %, and ncu counts the tensor pipe active ~22 % of the
//    time: a cost per MMA that neither the issuing threads nor the pipe's busy cycles show
//    (the A operand read from TMEM is the remaining suspect) paces a stage.  One thread waits
//    ~50 cycles per MMA it issues; two threads issue concurrently (measured), which doubles the
//    MMA rate.  For GATED the A rows are ordered so that each 32-lane quarter holds 16 gate rows
//    and the same 16 up rows: lanes l and l + 16 of an epilogue warp hold g and u of one column.
//  * Warps 11..14 drain TMEM (tcgen05.ld 32x32b), add the two issuers' accumulators, apply the
//    row scale and gs, and store inter (bf16, compact pair order) or y (bf16, the pair's row).
// Every wait is bounded (mbar_wait); on expiry a role sets the abort flag, the others stop at
// their next wait, copies and MMAs in flight are waited for (bounded), TMEM is freed.
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace okc {

constexpr int kMtKC = 256;                         // K per stage
constexpr int kMtCodes = 128 * (kMtKC / 2);        // 16 KB of codes per raw stage
constexpr int kMtRawBytes = kMtCodes + 128 * (kMtKC / 16);  // + 2 KB of scales
static_assert(kMtRawBytes % 1024 == 0, "1024-aligned tiles");

// NT = pairs per unit (the MMA's N): 32 while the experts see few tokens, 64 beyond.  TMEM holds
// 2 issuers x 2 accumulator buffers of NT columns (0 .. 4 NT) and after them the NS A slots (128
// columns each: NT = 32: 3, NT = 64: 2).  The stage ring has three parts of different depths:
//  * RAW raw stages (packed codes + scales, 18 KB): a dequantising warp frees its stage as soon
//    as it holds the stage's codes in registers, so a slot is held for the copy's latency only
//    (~3 us under a full weight stream) and RAW stages keep RAW x 18 KB in flight per SM;
//  * NA activation slots (NA = NS + 1), loaded ahead of the A slot they pair with: an activation
//    copy (an L2 hit) takes ~1.5 us to land behind the weight stream;
//  * NS A slots in TMEM (the dequantised weights).
// Stage q's MMAs complete on sdone[q % NA], which frees activation slot q % NA and A slot q % NS.
template <int NT_>
struct MtCfg {
  static constexpr int NT = NT_;
  // MMA-issuing threads: 4 at NT = 32 (one per SM sub-partition, each a K quarter of a stage;
  // their 4 x 2 accumulators fit beside 2 A slots), 2 at NT = 64 (K halves)
  static constexpr int NI = NT == 32 ? 4 : 2;
  static constexpr int THREADS = (NI == 4 ? 19 : 16) * 32;  // NI = 4: issuers on warps 1, 15, 16, 18
  static constexpr int ACOL = 2 * NI * NT;                // first A-slot column
  static constexpr int NS = (512 - ACOL) / 128;           // A slots
  static constexpr int NA = NS + 1;                       // activation slots
  static constexpr int ATOM = NT * 128;                   // <= NT pairs x 64 K f16
  static constexpr int ACT = 4 * ATOM;                    // a stage's activation tiles
  static constexpr int RAW_FIT = (232448 - 1024 - NA * ACT - 5120) / kMtRawBytes;
  static constexpr int RAW = RAW_FIT > 8 ? 8 : RAW_FIT;   // NT = 32: 8, NT = 64: 6
  static constexpr int BODY = RAW * kMtRawBytes + NA * ACT;
  static constexpr int BARS = 2 * RAW + NS + 2 * NA + 2 + 2 + 1;
  static constexpr int SMEM = 1024 + BODY + BARS * 8 + 16 + (2 * 257 + 2 * 256) * 4;
  static_assert(ATOM % 1024 == 0, "1024-aligned tiles");
  static_assert(SMEM <= 232448, "shared memory");
  static_assert(ACOL + NS * 128 <= 512 && NS >= 2 && NA >= NS && RAW >= 4, "rings");
};

__device__ __forceinline__ void mt_tma_u8(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D (TMEM) (+)= A (TMEM: lane = row, column = f16 pair along K) x B (shared memory descriptor)^T.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}

// One word of packed codes (bytes b0..b3 = K pairs (2i, 2i+1), low nibble first) -> four f16x2.
__device__ __forceinline__ uint4 mt_e2m1_word(uint32_t w) {
  uint4 r;
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "r"(w));
  return r;
}

__device__ __forceinline__ uint32_t mt_hmul2(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Two e4m3 scale bytes -> f16x2 of each one duplicated: (s0, s0), (s1, s1).
__device__ __forceinline__ void mt_scales2(uint32_t two, uint32_t& d0, uint32_t& d1) {
  uint32_t h;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(h) : "r"(two));
  d0 = prmt(h, 0u, 0x1010u);
  d1 = prmt(h, 0u, 0x3232u);
}

__device__ __forceinline__ void mt_tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

struct MtUnit {
  int e, rb, row0, n;  // expert, weight-row block, first compact pair row, pairs (<= 64)
};

// Unit u: active expert i with upre[i] <= u < upre[i+1], then chunk-major, row block minor.
__device__ __forceinline__ MtUnit mt_unit(const int* act, const int* upre, const int* cnt, const int* off,
                                          int nact, int nrb, int u, int nt) {
  int lo = 0, hi = nact - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (upre[mid] <= u) lo = mid; else hi = mid - 1;
  }
  MtUnit t;
  const int v = u - upre[lo];
  const int ch = v / nrb;
  t.e = act[lo];
  t.rb = v - ch * nrb;
  t.row0 = off[t.e] + ch * nt;
  t.n = min(nt, cnt[t.e] - ch * nt);
  return t;
}

template <bool GATED, int NT>
__global__ void __launch_bounds__(MtCfg<NT>::THREADS, 1) moe_tc_kernel(
    const __grid_constant__ CUtensorMap cmap, const __grid_constant__ CUtensorMap smap,
    const __grid_constant__ CUtensorMap a16, const __grid_constant__ CUtensorMap a32,
    const __grid_constant__ CUtensorMap a64, const int32_t* __restrict__ counts,
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ pairs, const float* __restrict__ gs,
    const float* __restrict__ rs, __nv_bfloat16* __restrict__ inter_out, __nv_bfloat16* __restrict__ y_out, int K,
    int NR, int I, int E, int* err) {
  using C = MtCfg<NT>;
  extern __shared__ uint8_t mt_raw_smem[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mt_raw_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* rawr = base;
  uint8_t* actt = rawr + C::RAW * kMtRawBytes;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(actt + C::NA * C::ACT);
  uint64_t* raw_empty = raw_full + C::RAW;
  uint64_t* sfull = raw_empty + C::RAW;  // [NS] A slot q % NS written (8 dequantising warps)
  uint64_t* afull = sfull + C::NS;       // [NA] activation tiles of stage q landed
  uint64_t* sdone = afull + C::NA;       // [NA] stage q's MMAs completed (both issuers' commits)
  uint64_t* acc_full = sdone + C::NA;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* act = reinterpret_cast<int*>(tmem_slot + 4);  // [257] active experts, [256] = count
  int* upre = act + 257;                             // [257] unit prefix over active experts
  int* cnt = upre + 257;                             // [256] counts
  int* off = cnt + 256;                              // [256] offsets

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_w = GATED ? 2 * I : NR;
  const int nrb = GATED ? I / 64 : NR / 128;
  const int nk = K / kMtKC;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::RAW; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 8); }
    for (int i = 0; i < C::NS; ++i) mbar_init(&sfull[i], 8);
    for (int i = 0; i < C::NA; ++i) { mbar_init(&afull[i], 1); mbar_init(&sdone[i], C::NI); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], C::NI); mbar_init(&acc_empty[i], 4); }
    mbar_init(drain, C::NI);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  pdl_wait();
  if (warp == 0) {  // active experts and their unit prefix
    int carry = 0, ncarry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? counts[e] : 0;
      if (e < E) { cnt[e] = c; off[e] = offsets[e]; }
      const bool on = c > 0;
      const unsigned bal = __ballot_sync(0xffffffffu, on);
      const int nu = on ? ((c + C::NT - 1) / C::NT) * nrb : 0;
      int v = nu;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (on) {
        const int i = ncarry + __popc(bal & ((1u << lane) - 1u));
        act[i] = e;
        upre[i] = carry + v - nu;
      }
      carry += __shfl_sync(0xffffffffu, v, 31);
      ncarry += __popc(bal);
    }
    if (lane == 0) { act[256] = ncarry; upre[ncarry] = carry; }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int nact = act[256];
  const int U = nact > 0 ? upre[nact] : 0;
  int u0, u1;
  {
    const int q = U / (int)gridDim.x, r = U % (int)gridDim.x, c = blockIdx.x;
    u0 = c * q + min(c, r);
    u1 = u0 + q + (c < r ? 1 : 0);
  }

  if (warp == 0) {
    // ------------------------------ weight producer ------------------------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t r = 0;
      for (int u = u0; u < u1 && !*abort_flag; ++u) {
        const MtUnit t = mt_unit(act, upre, cnt, off, nact, nrb, u, C::NT);
        const int wrow = t.e * rows_w + t.rb * (GATED ? 64 : 128);
        for (int ks = 0; ks < nk; ++ks, ++r) {
          const int s = (int)(r % C::RAW);
          if (!mbar_wait(&raw_empty[s], ((r / C::RAW) & 1u) ^ 1u, err, abort_flag)) { *abort_flag = 1; break; }
          mbar_arrive_expect_tx(&raw_full[s], kMtRawBytes);
          uint8_t* d = rawr + s * kMtRawBytes;
          if (GATED) {  // raw rows 0-63: gate rows, 64-127: the same up rows
            mt_tma_u8(d, &cmap, ks * (kMtKC / 2), wrow, &raw_full[s], pol);
            mt_tma_u8(d + kMtCodes / 2, &cmap, ks * (kMtKC / 2), wrow + I, &raw_full[s], pol);
            mt_tma_u8(d + kMtCodes, &smap, ks * (kMtKC / 16), wrow, &raw_full[s], pol);
            mt_tma_u8(d + kMtCodes + 64 * 16, &smap, ks * (kMtKC / 16), wrow + I, &raw_full[s], pol);
          } else {
            mt_tma_u8(d, &cmap, ks * (kMtKC / 2), wrow, &raw_full[s], pol);
            mt_tma_u8(d + kMtCodes, &smap, ks * (kMtKC / 16), wrow, &raw_full[s], pol);
          }
        }
      }
      for (uint32_t i = r > (uint32_t)C::RAW ? r - C::RAW : 0u; i < r; ++i)  // copies in flight land
        if (!mbar_wait(&raw_full[i % C::RAW], (i / C::RAW) & 1u, err)) break;
    }
  } else if (warp == 2) {
    // ---------------------------- activation producer ----------------------------
    if (lane == 0) {
      uint32_t q = 0;
      bool ok = true;
      for (int u = u0; u < u1 && ok && !*abort_flag; ++u) {
        const MtUnit t = mt_unit(act, upre, cnt, off, nact, nrb, u, C::NT);
        const int box = t.n <= 16 ? 16 : (t.n <= 32 ? 32 : 64);
        const CUtensorMap* map = box == 16 ? &a16 : (box == 32 ? &a32 : &a64);
        for (int ks = 0; ks < nk; ++ks, ++q) {
          const int s = (int)(q % C::NA);
          if (!mbar_wait(&sdone[s], ((q / C::NA) & 1u) ^ 1u, err, abort_flag)) { *abort_flag = 1; ok = false; break; }
          mbar_arrive_expect_tx(&afull[s], (uint32_t)box * 128u * 4u);
          uint8_t* d = actt + s * C::ACT;
#pragma unroll
          for (int j = 0; j < 4; ++j) tma_load_2d(d + j * C::ATOM, map, ks * kMtKC + 64 * j, t.row0, &afull[s]);
        }
      }
      // the copies issued land before the CTA can leave
      for (uint32_t i = q > (uint32_t)C::NA ? q - C::NA : 0u; i < q; ++i)
        if (!mbar_wait(&afull[i % C::NA], (i / C::NA) & 1u, err)) break;
    }
  } else if (warp == 1 || warp == 15 || (C::NI == 4 && (warp == 16 || warp == 18))) {
    // ---------------------------------- MMA issuers ---------------------------------
    // Issuer h (warps 1, 15, 16, 18: h = 0, 1, 2, 3) takes the K slice h (of NI) of every stage
    // into its own accumulator; one thread issuing kind::f16 MMAs waits ~50-76 cycles per
    // instruction, and threads on different SM sub-partitions issue concurrently (measured at
    // full rate each for up to 4).
    if (lane == 0) {
      const int h = warp == 1 ? 0 : (warp == 15 ? 1 : (warp == 16 ? 2 : 3));
      uint32_t q = 0;
      int ui = 0;
      bool ok = true;
      for (int u = u0; u < u1 && ok; ++u, ++ui) {
        const MtUnit t = mt_unit(act, upre, cnt, off, nact, nrb, u, C::NT);
        const uint32_t idesc = umma_idesc_f16((t.n + 15) & ~15);
        const int buf = ui & 1;
        if (!mbar_wait(&acc_empty[buf], ((uint32_t)(ui >> 1) & 1u) ^ 1u, err, abort_flag)) { ok = false; break; }
        for (int ks = 0; ks < nk; ++ks, ++q) {
          const int s = (int)(q % C::NS), sx = (int)(q % C::NA);
          // sfull[s] completes only after the stage's activation tiles landed (warp 3 waits for them)
          if (!mbar_wait(&sfull[s], (q / C::NS) & 1u, err, abort_flag)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(actt + sx * C::ACT + (4 / C::NI) * h * C::ATOM);
          const uint32_t ta = tmem + C::ACOL + (uint32_t)s * 128u + (128u / C::NI) * h;
#pragma unroll
          for (int k16 = 0; k16 < 16 / C::NI; ++k16) {
            const uint64_t db = umma_desc_sw128(sa + (k16 >> 2) * C::ATOM) + 2 * (k16 & 3);
            umma_f16_ts(tmem + 2 * C::NT * h + buf * C::NT, ta + 8 * k16, db, idesc, (ks | k16) ? 1u : 0u);
          }
          umma_commit(&sdone[sx]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(&acc_full[0]);
        umma_commit(&acc_full[1]);
      }
      umma_commit(drain);  // arrives once every MMA issued above has completed
      mbar_wait(drain, 0u, err);
    }
  } else if (warp >= 3 && warp <= 10) {
    // -------------------------------- dequantisation --------------------------------
    const int qd = warp & 3, half = (warp - 3) >> 2;
    const int m = 32 * qd + lane;  // A row = TMEM lane
    const int rho = GATED ? (lane < 16 ? 16 * qd + lane : 64 + 16 * qd + lane - 16) : m;  // raw row
    const int sw = rho & 7;
    const uint32_t tbase = tmem + ((uint32_t)(32 * qd) << 16) + C::ACOL + 64u * half;
    uint32_t q = 0;
    bool ok = true;
    for (int u = u0; u < u1 && ok; ++u) {
      for (int ks = 0; ks < nk; ++ks, ++q) {
        const int sr = (int)(q % C::RAW), s = (int)(q % C::NS);
        if (!mbar_wait(&raw_full[sr], (q / C::RAW) & 1u, err, abort_flag)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        // the stage's codes and scales into registers, then the raw slot is free again
        const uint8_t* rw = rawr + sr * kMtRawBytes;
        const uint8_t* crow = rw + rho * 128;
        const uint2 sc8 = *reinterpret_cast<const uint2*>(rw + kMtCodes + rho * 16 + 8 * half);
        uint4 cw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) cw[i] = *reinterpret_cast<const uint4*>(crow + (((4 * half + i) ^ sw) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[sr]);
        // A slot s is free once stage q - NS's MMAs completed (sdone of that stage; the phase
        // after it needs stage q - NS + NA >= q, not yet written, so the parity is unambiguous)
        if (q >= (uint32_t)C::NS &&
            !mbar_wait(&sdone[(q - C::NS) % C::NA], ((q - C::NS) / C::NA) & 1u, err, abort_flag)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint32_t sd[8];
        mt_scales2(sc8.x & 0xffffu, sd[0], sd[1]);
        mt_scales2(sc8.x >> 16, sd[2], sd[3]);
        mt_scales2(sc8.y & 0xffffu, sd[4], sd[5]);
        mt_scales2(sc8.y >> 16, sd[6], sd[7]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // 16 code bytes = K [128 half + 32 i, + 32), scale groups 2i, 2i+1
          const uint4 c = cw[i];
          const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
          uint32_t o[16];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t sj = sd[2 * i + (wi >> 1)];
            const uint4 h = mt_e2m1_word(wv[wi]);
            o[4 * wi + 0] = mt_hmul2(h.x, sj);
            o[4 * wi + 1] = mt_hmul2(h.y, sj);
            o[4 * wi + 2] = mt_hmul2(h.z, sj);
            o[4 * wi + 3] = mt_hmul2(h.w, sj);
          }
          mt_tmem_st16(tbase + (uint32_t)s * 128u + 16u * i, o);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          // one of the 8 arrivals waits for the stage's activation tiles, so the MMA issuers wait
          // on one barrier per stage (afull's next phase needs this stage's MMAs: unambiguous)
          if (warp == 3 && !mbar_wait(&afull[q % C::NA], (q / C::NA) & 1u, err, abort_flag)) *abort_flag = 1;
          mbar_arrive(&sfull[s]);
        }
      }
    }
  } else if (warp >= 11 && warp <= 14) {
    // ------------------------------------ epilogue ------------------------------------
    const int q4 = warp & 3;
    const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
    int ui = 0;
    for (int u = u0; u < u1; ++u, ++ui) {
      const MtUnit t = mt_unit(act, upre, cnt, off, nact, nrb, u, C::NT);
      const int buf = ui & 1;
      if (!mbar_wait(&acc_full[buf], (uint32_t)(ui >> 1) & 1u, err, abort_flag) || *abort_flag) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const float gsc = gs[t.e];
      const uint32_t taddr = tmem + lane_base + buf * C::NT;
      for (int c0 = 0; c0 < t.n; c0 += 16) {
        float v[16], v1[16];
        tmem_ld16(taddr + c0, v);  // issuer 0's K slices of the stages
#pragma unroll
        for (int h = 1; h < C::NI; ++h) {  // + the other issuers' slices
          tmem_ld16(taddr + 2 * C::NT * h + c0, v1);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) v[jj] += v1[jj];
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = c0 + jj;
          if (j >= t.n) break;
          const float acc = v[jj] * rs[t.row0 + j];  // exact: a power of two
          if (GATED) {
            const float h = __bfloat162float(__float2bfloat16_rn(acc * gsc));
            const float up = __shfl_down_sync(0xffffffffu, h, 16);
            if (lane < 16)
              inter_out[(size_t)(t.row0 + j) * I + t.rb * 64 + 16 * q4 + lane] =
                  __float2bfloat16_rn(h / (1.f + expf(-h)) * up);
          } else {
            y_out[(size_t)pairs[t.row0 + j] * NR + t.rb * 128 + 32 * q4 + lane] = __float2bfloat16_rn(acc * gsc);
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// dst[j] = f16(src[r_j] * 2^s_j), rs[j] = 2^-s_j for the local pairs j < offsets[E], with
// r_j = pairs[j] / topk (gather, topk > 0) or j (topk == 0); one warp per row: a pass for the row
// maximum, a second (L1-resident) pass to scale, convert and store.
__global__ void __launch_bounds__(256) moe_rows_f16_kernel(const __nv_bfloat16* __restrict__ src,
                                                           const int32_t* __restrict__ pairs,
                                                           const int32_t* __restrict__ offsets, int E, int topk,
                                                           int K, __half* __restrict__ dst, float* __restrict__ rs) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int n = offsets[E];
  for (int j = blockIdx.x * 8 + (threadIdx.x >> 5); j < n; j += gridDim.x * 8) {
    const __nv_bfloat16* xr = src + (size_t)(topk > 0 ? pairs[j] / topk : j) * K;
    float amax = 0.f;
    for (int k = lane * 8; k < K; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(w[h])), fabsf(bf16_hi(w[h]))));
    }
    amax = warp_max(amax);
    // s = 14 - floor(log2 amax), clamped so that both 2^s and 2^-s are normal floats
    int s = 0;
    if (amax > 0.f) {
      const int e2 = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127;
      s = min(100, max(-113, 14 - e2));
    }
    const float up = __uint_as_float((uint32_t)(127 + s) << 23);
    if (lane == 0) rs[j] = __uint_as_float((uint32_t)(127 - s) << 23);
    __half* gr = dst + (size_t)j * K;
    for (int k = lane * 8; k < K; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        __half2 p = __floats2half2_rn(bf16_lo(w[h]) * up, bf16_hi(w[h]) * up);
        o[h] = *reinterpret_cast<uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(gr + k) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

static bool mt_u8_map(CUtensorMap* m, const void* base, long long inner, long long rows, int box_x, int box_y,
                      bool swizzle) {
  auto fn = tensor_map_encoder();
  if (!fn || !okc_host::aligned16(base) || inner % 16 || rows <= 0 || rows >= (1LL << 31)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool mt_f16_map(CUtensorMap* m, const void* base, long long inner, long long rows, int box_rows) {
  auto fn = tensor_map_encoder();
  if (!fn || !okc_host::aligned16(base) || inner % 64 || rows <= 0 || rows >= (1LL << 31)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool moe_tc_ok(int H, int I, int E) {
  return H % kMtKC == 0 && I % kMtKC == 0 && I % 64 == 0 && H % 128 == 0 && H <= 8192 && E <= 256 &&
         tensor_map_encoder() != nullptr;
}

int launch_moe_rows_f16(const void* src, const int32_t* pairs, const int32_t* offsets, int E, int topk, int K,
                        int max_rows, __half* dst, float* rs, cudaStream_t stream) {
  int blocks = (max_rows + 7) / 8;
  const int cap = 4 * okc_host::num_sms();
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return okc_host::launch_k(moe_rows_f16_kernel, dim3(blocks), dim3(256), 0, stream, dim3(1),
                            reinterpret_cast<const __nv_bfloat16*>(src), pairs, offsets, E, topk, K, dst, rs);
}

template <bool GATED, int NT>
static int launch_moe_tc_nt(const CUtensorMap& cm, const CUtensorMap& sm, const CUtensorMap& m16,
                            const CUtensorMap& m32, const CUtensorMap& m64, const int32_t* counts,
                            const int32_t* offsets, const int32_t* pairs, const float* gs, const float* rs,
                            __nv_bfloat16* inter, __nv_bfloat16* y, int K, int NR, int I, int E, int* err,
                            cudaStream_t stream) {
  using C = MtCfg<NT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(moe_tc_kernel<GATED, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = true;
  }
  return okc_host::launch_k(moe_tc_kernel<GATED, NT>, dim3(okc_host::num_sms()), dim3(C::THREADS), C::SMEM, stream,
                            dim3(1), cm, sm, m16, m32, m64, counts, offsets, pairs, gs, rs, inter, y, K, NR, I, E,
                            err);
}

// GATED: act = xg [rows][K = H], weights W13, out inter; else act = inter as f16 [rows][K = I],
// weights W2, out y.  rs: the activation rows' scales.
template <bool GATED>
int launch_moe_tc(const void* w, const void* sf, int E, const __half* act, int rows, const float* rs,
                  const int32_t* counts, const int32_t* offsets, const int32_t* pairs, const float* gs,
                  __nv_bfloat16* inter, __nv_bfloat16* y, int K, int NR, int I, int* err, cudaStream_t stream) {
  const long long wrows = (long long)E * (GATED ? 2 * I : NR);
  const int box_rows = GATED ? 64 : 128;
  CUtensorMap cm, sm, m16, m32, m64;
  if (!mt_u8_map(&cm, w, K / 2, wrows, kMtKC / 2, box_rows, true) ||
      !mt_u8_map(&sm, sf, K / 16, wrows, kMtKC / 16, box_rows, false) || !mt_f16_map(&m16, act, K, rows, 16) ||
      !mt_f16_map(&m32, act, K, rows, 32) || !mt_f16_map(&m64, act, K, rows, 64))
    return OKC_ERR_INVALID;
  // chunks of <= 32 pairs (3 A slots, 8 raw stages) while the experts see few tokens each, 64 beyond
  if (rows <= 8 * 128)
    return launch_moe_tc_nt<GATED, 32>(cm, sm, m16, m32, m64, counts, offsets, pairs, gs, rs, inter, y, K, NR, I, E,
                                       err, stream);
  return launch_moe_tc_nt<GATED, 64>(cm, sm, m16, m32, m64, counts, offsets, pairs, gs, rs, inter, y, K, NR, I, E,
                                     err, stream);
}

template int launch_moe_tc<true>(const void*, const void*, int, const __half*, int, const float*, const int32_t*,
                                 const int32_t*, const int32_t*, const float*, __nv_bfloat16*, __nv_bfloat16*, int,
                                 int, int, int*, cudaStream_t);
template int launch_moe_tc<false>(const void*, const void*, int, const __half*, int, const float*, const int32_t*,
                                  const int32_t*, const int32_t*, const float*, __nv_bfloat16*, __nv_bfloat16*, int,
                                  int, int, int*, cudaStream_t);

}  // namespace okc
