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
//  * all 4 warps drain TMEM with tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = weight
//    rows) and store y; with split-K every split stores an fp32 partial tile and the last
//    CTA of the tile to arrive (self-resetting counter) sums them in split order
//    (deterministic) — no thread-block clusters, so all CTAs of the grid stay co-resident.
// Every mbarrier wait is bounded (common.cuh); TMEM is always released before exit.
// Mirrors the M >= 32 tensor-core path of muse_bf16_proj/projection/kernels/{tma,
// hopper_ws}.py and muse_decode_layer/decode/projections.py:75-77 (there: cuBLAS / wgmma).
#include <cudaTypedefs.h>

#include "kernels.cuh"

namespace okc {

constexpr int TC_BM = 128;  // weight rows per tile (MMA M)
constexpr int TC_BK = 64;   // K elements per stage (128 bytes: one swizzle atom row)

struct TcParams {
  int M, N, K, ldy, out_fp32, splits, kb_per_split;
  void* y;
  const __nv_bfloat16* residual;
  int* err;
  float* part;    // split-K partial tiles [tiles][splits][128][BN] (workspace)
  int* counters;  // per-tile arrival counters, zero between calls (the last arriver resets)
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor, K-major SWIZZLE_128B: 8-row groups 1024 B apart (SBO),
// LBO unused (1), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int STAGES>
struct TcCfg {
  static constexpr int A_BYTES = TC_BM * TC_BK * 2;
  static constexpr int B_BYTES = BN * TC_BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BODY = STAGE * STAGES;
  static constexpr int SMEM = 1024 + BODY + 256;  // alignment slack + body + barriers
  static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(128, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_w,
                                                         const __grid_constant__ CUtensorMap tma_x,
                                                         TcParams p) {
  using C = TcCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = p.splits > 1 ? (int)(blockIdx.x % p.splits) : 0;
  const int tile = blockIdx.x / p.splits;
  const int n0 = tile * TC_BM;
  const int nkb = (p.K + TC_BK - 1) / TC_BK;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(nkb, kb0 + p.kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
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

  if (warp == 0 && lane == 0) {
    // ---------------------------- TMA producer ----------------------------
    int issued = 0;
    for (int kb = kb0; kb < kb1; ++kb, ++issued) {
      const int s = issued % STAGES;
      const uint32_t ph = (uint32_t)(issued / STAGES) & 1u;
      if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u, p.err)) { *abort_flag = 1; break; }
      mbar_arrive_expect_tx(&full[s], C::STAGE);
      uint8_t* sa = smem + s * C::STAGE;
      tma_load_2d(sa, &tma_w, kb * TC_BK, n0, &full[s]);
      tma_load_2d(sa + C::A_BYTES, &tma_x, kb * TC_BK, 0, &full[s]);
    }
    // make sure this thread's last loads have landed before anyone can leave
    for (int i = max(0, issued - STAGES); i < issued; ++i)
      if (!mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, p.err)) break;
  } else if (warp == 1 && lane == 0) {
    // ---------------------------- MMA issuer -------------------------------
    const uint32_t idesc = umma_idesc_bf16(BN);
    int done = 0;
    for (int kb = kb0; kb < kb1; ++kb, ++done) {
      const int s = done % STAGES;
      const uint32_t ph = (uint32_t)(done / STAGES) & 1u;
      if (*abort_flag || !mbar_wait(&full[s], ph, p.err)) { *abort_flag = 1; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = smem_u32(smem + s * C::STAGE);
      const uint64_t da = umma_desc_sw128(sa), db = umma_desc_sw128(sa + C::A_BYTES);
#pragma unroll
      for (int j = 0; j < TC_BK / 16; ++j)  // +32 bytes per K=16 step inside the swizzle atom
        umma_bf16(tmem, da + 2 * j, db + 2 * j, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(accf);  // fires when every MMA above has completed
  }
  __syncwarp();

  // ------------------------------ epilogue --------------------------------
  const bool ok = mbar_wait(accf, 0, p.err);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const int row = warp * 32 + lane;  // TMEM lane = weight row within the tile
  const int n = n0 + row;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  const bool empty_split = kb1 <= kb0;

  if (p.splits == 1) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (!ok || n >= p.N) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = c0 + j;
        if (m >= p.M) break;
        float r = empty_split ? 0.f : v[j];
        if (p.residual) r += __bfloat162float(p.residual[(size_t)m * p.ldy + n]);
        if (p.out_fp32)
          reinterpret_cast<float*>(p.y)[(size_t)m * p.ldy + n] = r;
        else
          reinterpret_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] = __float2bfloat16_rn(r);
      }
    }
  } else {
    // Split-K: every split stores its fp32 partial tile; the last CTA of the tile to arrive
    // (self-resetting counter) sums the partials in split order — deterministic — and stores y.
    float* mine = p.part + ((size_t)tile * p.splits + split) * TC_BM * BN + (size_t)row * BN;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(mine + c0 + j) =
            empty_split ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
    __threadfence();
    __syncthreads();
    int* last = reinterpret_cast<int*>(const_cast<int*>(abort_flag)) + 1;
    if (threadIdx.x == 0) *last = atomicAdd(&p.counters[tile], 1) == p.splits - 1;
    __syncthreads();
    if (*last) {
      __threadfence();
      const int mv = min(p.M, BN);
      const float* base = p.part + (size_t)tile * p.splits * TC_BM * BN + (size_t)row * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < mv; c0 += 4) {
        float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < p.splits; ++q) {
          const float4 t4 = __ldcg(reinterpret_cast<const float4*>(base + (size_t)q * TC_BM * BN + c0));
          acc4.x += t4.x; acc4.y += t4.y; acc4.z += t4.z; acc4.w += t4.w;
        }
        const float r4[4] = {acc4.x, acc4.y, acc4.z, acc4.w};
        if (!ok || n >= p.N) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = c0 + j;
          if (m >= mv) break;
          float r = r4[j];
          if (p.residual) r += __bfloat162float(p.residual[(size_t)m * p.ldy + n]);
          if (p.out_fp32)
            reinterpret_cast<float*>(p.y)[(size_t)m * p.ldy + n] = r;
          else
            reinterpret_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] = __float2bfloat16_rn(r);
        }
      }
      if (threadIdx.x == 0) p.counters[tile] = 0;
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ------------------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

static bool make_map(CUtensorMap* m, const void* base, int inner, int rows, int ld, int box_rows) {
  auto fn = encode_fn();
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
         encode_fn() != nullptr;
}

struct TcPlan {
  int bn, ctas_per_sm, tiles, nkb, splits, kb_per_split;
};

// Split K so that tiles x splits fills the resident CTA slots of every SM (all CTAs co-resident).
static TcPlan tc_plan(int M, int N, int K) {
  TcPlan pl;
  pl.bn = M <= 64 ? 64 : (M <= 128 ? 128 : 256);
  pl.ctas_per_sm = pl.bn <= 128 ? 2 : 1;
  pl.tiles = (N + TC_BM - 1) / TC_BM;
  pl.nkb = (K + TC_BK - 1) / TC_BK;
  int s = okc_host::num_sms() * pl.ctas_per_sm / pl.tiles;
  s = s < 1 ? 1 : (s > 16 ? 16 : s);
  while (s > 1 && pl.nkb / s < 2) --s;
  int kbps = (pl.nkb + s - 1) / s;
  while (s > 1 && (s - 1) * kbps >= pl.nkb) {  // every split owns at least one K block
    --s;
    kbps = (pl.nkb + s - 1) / s;
  }
  pl.splits = s;
  pl.kb_per_split = kbps;
  return pl;
}

// Workspace: [kTcCounterBytes of per-tile counters at a FIXED offset, so that they stay zero
// from call to call whatever the shape][fp32 partial tiles].
constexpr size_t kTcCounterBytes = 16384;  // 4096 tiles of 128 rows: N <= 524288

size_t tc_gemm_ws_bytes(int M, int N, int K) {
  if (M < 1 || M > 256 || N < 1 || K < 1) return 0;
  const TcPlan pl = tc_plan(M, N, K);
  if (pl.splits == 1) return 0;
  return kTcCounterBytes + (size_t)pl.tiles * pl.splits * TC_BM * pl.bn * 4;
}

template <int BN, int STAGES>
static int launch_tc_t(const void* x, int ldx, const void* w, int ldw, TcParams& p, const TcPlan& pl,
                       void* ws, size_t ws_bytes, cudaStream_t stream) {
  using C = TcCfg<BN, STAGES>;
  CUtensorMap mw, mx;
  if (!make_map(&mw, w, p.K, p.N, ldw, TC_BM) || !make_map(&mx, x, p.K, p.M, ldx, BN)) return OKC_ERR_INVALID;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM) != cudaSuccess)
      return OKC_ERR_LAUNCH;
    configured = true;
  }
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.part = nullptr;
  p.counters = nullptr;
  if (pl.splits > 1) {
    const size_t part_bytes = (size_t)pl.tiles * pl.splits * TC_BM * BN * 4;
    if (!ws || ws_bytes < kTcCounterBytes + part_bytes || (size_t)pl.tiles * 4 > kTcCounterBytes)
      return OKC_ERR_WORKSPACE;
    p.counters = reinterpret_cast<int*>(ws);
    p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kTcCounterBytes);
  }
  tc_gemm_kernel<BN, STAGES><<<pl.tiles * pl.splits, 128, C::SMEM, stream>>>(mw, mx, p);
  return okc_host::launch_status();
}

int launch_tc_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, const void* residual, int M,
                   int N, int K, int out_fp32, void* ws, size_t ws_bytes, cudaStream_t stream) {
  TcParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldy = ldy;
  p.out_fp32 = out_fp32;
  p.y = y;
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.err = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) - 256);  // the caller's error word
  const TcPlan pl = tc_plan(M, N, K);
  if (pl.bn == 64) return launch_tc_t<64, 4>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
  if (pl.bn == 128) return launch_tc_t<128, 3>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
  return launch_tc_t<256, 4>(x, ldx, w, ldw, p, pl, ws, ws_bytes, stream);
}

}  // namespace okc
