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
//    rows) and store y; with split-K the S CTAs of a cluster reduce their partial tiles
//    through distributed shared memory in a fixed order (deterministic, no workspace).
// Every mbarrier wait is bounded (common.cuh); TMEM is always released before exit.
// Mirrors the M >= 32 tensor-core path of muse_bf16_proj/projection/kernels/{tma,
// hopper_ws}.py and muse_decode_layer/decode/projections.py:75-77 (there: cuBLAS / wgmma).
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace okc {

constexpr int TC_BM = 128;  // weight rows per tile (MMA M)
constexpr int TC_BK = 64;   // K elements per stage (128 bytes: one swizzle atom row)

struct TcParams {
  int M, N, K, ldy, out_fp32, splits, kb_per_split;
  void* y;
  const __nv_bfloat16* residual;
  int* err;
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
  static constexpr int RED_LD = BN + 1;
  static constexpr int RED_BYTES = TC_BM * RED_LD * 4;
  static constexpr int PIPE = STAGE * STAGES;
  static constexpr int BODY = PIPE > RED_BYTES ? PIPE : RED_BYTES;
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
    float* red = reinterpret_cast<float*>(smem);  // pipeline buffers are idle now
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) red[row * C::RED_LD + c0 + j] = empty_split ? 0.f : v[j];
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int mv = min(p.M, BN);
    const int total = TC_BM * mv;
    const int per = (total + p.splits - 1) / p.splits;
    const int e1 = min(total, (split + 1) * per);
    for (int e = split * per + (int)threadIdx.x; e < e1; e += blockDim.x) {
      const int m = e / TC_BM, nl = e % TC_BM;
      const int nn = n0 + nl;
      if (nn >= p.N) continue;
      float r = 0.f;
      for (int q = 0; q < p.splits; ++q) r += cluster.map_shared_rank(red, q)[nl * C::RED_LD + m];
      if (p.residual) r += __bfloat162float(p.residual[(size_t)m * p.ldy + nn]);
      if (p.out_fp32)
        reinterpret_cast<float*>(p.y)[(size_t)m * p.ldy + nn] = r;
      else
        reinterpret_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + nn] = __float2bfloat16_rn(r);
    }
    cluster.sync();
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

size_t tc_gemm_ws_bytes(int, int, int) { return 0; }

template <int BN, int STAGES>
static int launch_tc_t(const void* x, int ldx, const void* w, int ldw, TcParams& p, cudaStream_t stream,
                       int ctas_per_sm) {
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
  const int tiles = (p.N + TC_BM - 1) / TC_BM;
  const int nkb = (p.K + TC_BK - 1) / TC_BK;
  int splits = okc_host::num_sms() * ctas_per_sm / tiles;
  splits = splits < 1 ? 1 : (splits > 8 ? 8 : splits);
  while (splits > 1 && nkb / splits < 2) --splits;
  p.splits = splits;
  p.kb_per_split = (nkb + splits - 1) / splits;
  // every split must own at least one K block
  while (p.splits > 1 && (p.splits - 1) * p.kb_per_split >= nkb) {
    --p.splits;
    p.kb_per_split = (nkb + p.splits - 1) / p.splits;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * p.splits, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, STAGES>, mw, mx, p);
  return okc_host::launch_status();
}

int launch_tc_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, const void* residual, int M,
                   int N, int K, int out_fp32, void* ws, size_t, cudaStream_t stream) {
  TcParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldy = ldy;
  p.out_fp32 = out_fp32;
  p.y = y;
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.err = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) - 256);  // the caller's error word
  if (M <= 64) return launch_tc_t<64, 4>(x, ldx, w, ldw, p, stream, 2);
  if (M <= 128) return launch_tc_t<128, 3>(x, ldx, w, ldw, p, stream, 2);
  if (M <= 256) return launch_tc_t<256, 4>(x, ldx, w, ldw, p, stream, 1);
  return OKC_ERR_INVALID;
}

}  // namespace okc
