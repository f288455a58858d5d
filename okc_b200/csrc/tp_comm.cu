// Tensor-parallel exchange of the decode layer over NVLink peer memory.
//
// The row-parallel O projection leaves every rank with an fp32 partial P_r [T, H]; the layer
// output is out = bf16(x + sum_r P_r), replicated on every rank.  Two kernels do that, reading
// and writing the peers' buffers directly (CUDA IPC mappings; every GPU of the box is a
// full-bandwidth NVSwitch peer):
//   * tp_oproj_kernel: the O projection itself (tcgen05) fused with the exchange: each tile's
//     partial is pushed to its owner rank as soon as its accumulator is done;
//   * tp_allreduce_kernel: the exchange alone, for a partial that is already in HBM (the
//     expert-parallel MoE shares, and shapes the fused kernel does not take).
//
// Synchronisation is per CTA: CTA c of a rank only ever waits for CTA c of the other ranks
// (the grids are identical on every rank), with one flag word per (CTA, source rank) and one
// call epoch per CTA in `state`.  A signal is a release: the CTA's threads finish their stores,
// meet at a barrier, and one thread issues fence.acq_rel.sys followed by relaxed system-scope
// stores of the epoch into the peers' flag words (a fence.sc.sys, a fence per peer, or a chain
// of release stores costs more).  A wait is an acquire load loop on the local flag word.  There is no grid-wide barrier, no atomic counter and no "last CTA".
// Every wait is bounded (2 s of %globaltimer): on expiry the kernel sets OKC_DEVERR_TIMEOUT in
// the error word and goes on, so a missing rank cannot hang the GPU.
// No TMA multicast; the only TMA sources are this GPU's own buffers.
#include <string.h>

#include "kernels.cuh"
#include "tcgen05.cuh"

namespace okc {

// Payload pushed in place of a partial whose accumulation did not complete (quiet NaN).
constexpr float kTpPoison = __builtin_nanf("");

constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxCtas = 512;                     // per kernel: sizes the state and flag words
constexpr int kTpStateExchange = 0;                 // state[0, 512): tp_allreduce_kernel CTA epochs
constexpr int kTpStateOproj = kTpMaxCtas;           // state[512, 1024): tp_oproj_kernel CTA epochs
static_assert(OKC_TP_STATE_WORDS >= 2 * kTpMaxCtas, "state words");
static_assert(OKC_TP_EXCHANGE_FLAG_WORDS >= 2 * kTpMaxCtas * kTpMaxRanks, "exchange flag words");

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Waits until *f >= epoch (bounded); false on timeout (error bit set).
__device__ bool wait_flag(const int* f, int epoch, int* err) {
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(f) < epoch) {
    if (globaltimer() - t0 > kWaitNs) {
      atomicOr(err, OKC_DEVERR_TIMEOUT);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// After a barrier over the CTA's storing threads: thread 0 issues ONE system-scope release
// fence and then publishes `epoch` into word `slot` of every other rank's flag array (relaxed
// stores after the fence: they do not wait for one another).  Concurrent system fences are
// expensive (each waits for the SM's outstanding NVLink stores), so a CTA issues one per signal.
__device__ __forceinline__ void tp_signal(int* const* flags, int t, int world, int rank, int slot, int epoch) {
  if (t == 0) {
    fence_acq_rel_sys();
    for (int q = 0; q < world; ++q)
      if (q != rank) st_relaxed_sys(&flags[q][slot], epoch);
  }
}
// Thread q < W (q != rank) waits for word `base + q` of this rank's flag array; false on timeout.
__device__ __forceinline__ bool tp_wait(int* const* flags, int t, int world, int rank, int base, int epoch,
                                        int* err) {
  if (t < world && t != rank) return wait_flag(&flags[rank][base + t], epoch, err);
  return true;
}

// Optional phase trace (OKC_TP_TRACE=1): %globaltimer stamps of CTA 0, kept for its last 4
// calls: stamps[kernel][epoch % 4][phase] (64-bit ns; 16 phases).
constexpr int kTpTraceOffset = 256;  // bytes into the workspace (after the error word)
__device__ __forceinline__ void tp_stamp(unsigned long long* st, int epoch, int phase, unsigned long long t) {
  if (st) st[(epoch & 3) * 16 + phase] = t;
}

// ------------------------------------------------------------------------------ exchange
//
// tp_allreduce_kernel: rank r owns the r-th slice of the elements; CTA c of rank r
//   1. entry: tells CTA c of every rank "my partial is complete" and waits for theirs;
//   2. sums its grid-stride share of slice r over the W partials in rank order (the same
//      fixed order on every rank, so the replicated outputs are identical), adds the residual,
//      rounds to bf16 and stores the result into every rank's output;
//   3. exit: tells CTA c of every rank "my stores into you are done" and waits for theirs, so
//      when the grid completes this rank's output holds every slice.
// NVLink bytes per rank: (W-1)/W of the partial read (fp32) + (W-1)/W of the output written
// (bf16); at T = 128, H = 8192, W = 8: 3.5 MB in, 1.75 MB out.
struct TpArgs {
  const float* part[kTpMaxRanks];         // every rank's fp32 partial (this rank's is local)
  __nv_bfloat16* out[kTpMaxRanks];        // every rank's bf16 output buffer
  int* flags[kTpMaxRanks];                // every rank's flags: [c*8 + q] entry, [4096 + c*8 + q] exit
  const __nv_bfloat16* residual;          // local, replicated on every rank
  int* state;                             // local CTA epochs (OKC_TP_STATE_WORDS)
  int* err;
  long long n;                            // elements of [T, H]
  int rank, world;
  unsigned long long* stamps;             // phase trace or null
};

constexpr int kTpExitBase = kTpMaxCtas * kTpMaxRanks;

__global__ void __launch_bounds__(256) tp_allreduce_kernel(TpArgs a) {
  const unsigned long long t_entry = globaltimer();
  pdl_trigger();
  pdl_wait();  // this rank's partial (previous kernel) is complete and visible
  __shared__ int s_epoch, s_ok;
  const int c = blockIdx.x, t = threadIdx.x;
  if (t == 0) {
    s_epoch = a.state[kTpStateExchange + c] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int epoch = s_epoch;
  unsigned long long* const st0 = (a.stamps && c == 0 && t == 0) ? a.stamps : nullptr;
  tp_stamp(st0, epoch, 0, t_entry);
  tp_stamp(st0, epoch, 1, globaltimer());
  tp_signal(a.flags, t, a.world, a.rank, c * kTpMaxRanks + a.rank, epoch);  // entry
  tp_stamp(st0, epoch, 2, globaltimer());
  if (!tp_wait(a.flags, t, a.world, a.rank, c * kTpMaxRanks, epoch, a.err)) s_ok = 0;
  __syncthreads();
  tp_stamp(st0, epoch, 3, globaltimer());
  if (s_ok) {
    const long long n4 = a.n >> 2;
    const long long per = (n4 + a.world - 1) / a.world;
    const long long lo = per * a.rank, hi = min(n4, lo + per);
    for (long long i = lo + c * (long long)blockDim.x + t; i < hi; i += (long long)gridDim.x * blockDim.x) {
      float4 v[kTpMaxRanks];
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) v[q] = __ldcg(reinterpret_cast<const float4*>(a.part[q]) + i);
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) { s0 += v[q].x; s1 += v[q].y; s2 += v[q].z; s3 += v[q].w; }
      if (a.residual) {
        const uint2 rv = reinterpret_cast<const uint2*>(a.residual)[i];
        s0 += bf16_lo(rv.x); s1 += bf16_hi(rv.x); s2 += bf16_lo(rv.y); s3 += bf16_hi(rv.y);
      }
      const uint2 o = make_uint2(pack_bf16x2(s0, s1), pack_bf16x2(s2, s3));
#pragma unroll
      for (int q = 0; q < kTpMaxRanks; ++q)
        if (q < a.world) reinterpret_cast<uint2*>(a.out[q])[i] = o;
    }
  }
  __syncthreads();
  tp_stamp(st0, epoch, 4, globaltimer());
  tp_signal(a.flags, t, a.world, a.rank, kTpExitBase + c * kTpMaxRanks + a.rank, epoch);  // exit
  tp_stamp(st0, epoch, 5, globaltimer());
  tp_wait(a.flags, t, a.world, a.rank, kTpExitBase + c * kTpMaxRanks, epoch, a.err);
  tp_stamp(st0, epoch, 6, globaltimer());
  if (t == 0) a.state[kTpStateExchange + c] = epoch;  // read by this CTA index's next call
}

// ------------------------------------------------------------------------------ fused O projection
//
// tp_oproj_kernel: the row-parallel O projection and the exchange in ONE kernel.
// out_r = bf16(residual + sum_q x_q · W_q^T) on every rank r, where rank q holds the
// attention output x_q [M, K] of its heads and the matching columns W_q [N, K] of the O weight.
//   * tensor cores: a CTA pair (thread-block cluster of S = 2) owns one 128-row weight tile and
//     splits its K range; each CTA streams its half of the K tiles with 2-D TMA into a
//     SWIZZLE_128B ring and accumulates with tcgen05.mma in tensor memory (as tc_gemm_kernel);
//   * split-K over distributed shared memory: each CTA finishes one token half of the tile;
//     it drains the other half of its accumulator straight into its partner's shared memory,
//     and after one cluster barrier adds its own half to the partner's there (fixed order);
//   * reduce-scatter by pushing: the finished half, staged in shared memory, is cut into W
//     slices of `sl` tokens; slice s goes to rank s as 16-byte fp32 stores into receive slot
//     [cta][this rank], then the flag word (cta, this rank) is raised in rank s; the slice this
//     rank owns never leaves shared memory;
//   * all-gather: the CTA waits for the W - 1 flags of its own slice (raised by the same CTA
//     index on the other ranks), sums the W partials in rank order, adds the residual, rounds
//     once to bf16 and stores 16-byte rows into every rank's output;
//   * exit: the CTA tells the same CTA index on every rank "my stores into you are done" and
//     waits for theirs, so the output is complete on this rank when the grid ends.
// There is no fp32 partial in HBM, no separate split-K reduce and no load from a peer (all
// peer traffic is stores).  No entry barrier is needed: a rank pushes into a peer only after
// its own stream reached this call (its pdl_wait), and it writes a peer's output only after
// that peer's push flag for this call arrived, so nothing a peer still reads from the previous
// call is overwritten; a receive slot of the previous call was consumed before its CTA's exit
// signal.  Cross-GPU waits are on CTAs of the same index on the other GPUs; the host checks
// that the whole grid is co-resident.
// The weight tiles of the first stages are requested before griddepcontrol.wait (the weight is
// never written by an earlier kernel), so their latency hides under the previous kernel's tail.
template <int BN, int STAGES, int KS, int S>
struct TpCfg {
  static constexpr int A_BOX = TC_BM * TC_BK * 2;
  static constexpr int B_BOX = BN * TC_BK * 2;
  static constexpr int A_BYTES = A_BOX * KS;
  static constexpr int B_BYTES = B_BOX * KS;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BODY = STAGE * STAGES;
  static constexpr int HALF = BN / S;            // tokens this CTA finishes
  static constexpr int XCHG = HALF * TC_BM * 4;  // [HALF][128] fp32: partner's partial, then the sum
  static constexpr int SMEM = 1024 + BODY + XCHG + 256;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};

struct TpGemmArgs {
  float* recv[kTpMaxRanks];               // every rank's receive slots [ctas][W][sl][128] fp32
  __nv_bfloat16* out[kTpMaxRanks];        // every rank's output [M][ldo] bf16
  int* flags[kTpMaxRanks];                // every rank's flags: [cta*W + q] push, [ctas*W + cta*W + q] exit
  const __nv_bfloat16* residual;          // local [M][ldo] (nullable)
  int* state;                             // local CTA epochs (OKC_TP_STATE_WORDS)
  int* err;
  int M, N, K, ldo;
  int rank, world, sl, ctas;
  unsigned long long* stamps;             // phase trace or null
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tp_epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, int STAGES, int KS, int S>
__global__ void __launch_bounds__(192, 1) tp_oproj_kernel(const __grid_constant__ CUtensorMap tma_w,
                                                         const __grid_constant__ CUtensorMap tma_x,
                                                         TpGemmArgs a) {
  using C = TpCfg<BN, STAGES, KS, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stage = reinterpret_cast<float*>(smem + C::BODY);  // [HALF][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY + C::XCHG);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_epoch, s_ok;
  __shared__ unsigned long long s_tacc;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  const int part = S > 1 ? (int)cluster_ctarank() : 0;  // K half and token half of this CTA
  const int tile = S > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int cta = tile * S + part;  // the same (tile, part) has the same index on every rank
  const int nkb = (a.K + TC_BK * KS - 1) / (TC_BK * KS);
  const int u0 = nkb * part / S, u1 = nkb * (part + 1) / S;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf[0], 1);
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

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------- TMA producer ----------------------------
      const int pre = min(STAGES, u1 - u0);
      for (int i = 0; i < pre; ++i) {  // weight boxes of the first stages: before the wait
        mbar_arrive_expect_tx(&full[i], C::STAGE);
        for (int k = 0; k < KS; ++k)
          tma_load_2d(smem + i * C::STAGE + k * C::A_BOX, &tma_w, ((u0 + i) * KS + k) * TC_BK, tile * TC_BM,
                      &full[i]);
      }
      pdl_wait();  // x (the attention output) is complete from here on
      for (int i = 0; i < pre; ++i)
        for (int k = 0; k < KS; ++k)
          tma_load_2d(smem + i * C::STAGE + C::A_BYTES + k * C::B_BOX, &tma_x, ((u0 + i) * KS + k) * TC_BK, 0,
                      &full[i]);
      int issued = pre;
      for (int u = u0 + pre; u < u1; ++u, ++issued) {
        const int st = issued % STAGES;
        const uint32_t ph = (uint32_t)(issued / STAGES) & 1u;
        if (*abort_flag || !mbar_wait(&empty[st], ph ^ 1u, a.err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&full[st], C::STAGE);
        uint8_t* sa = smem + st * C::STAGE;
        for (int k = 0; k < KS; ++k) {
          tma_load_2d(sa + k * C::A_BOX, &tma_w, (u * KS + k) * TC_BK, tile * TC_BM, &full[st]);
          tma_load_2d(sa + C::A_BYTES + k * C::B_BOX, &tma_x, (u * KS + k) * TC_BK, 0, &full[st]);
        }
      }
      // drain: no TMA write may land after this CTA's shared memory is released
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        if (!mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, a.err)) break;
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      // ---------------------------- MMA issuer -------------------------------
      const uint32_t idesc = umma_idesc_bf16(BN);
      for (int i = 0; i < u1 - u0; ++i) {
        const int st = i % STAGES;
        if (*abort_flag || !mbar_wait(&full[st], (uint32_t)(i / STAGES) & 1u, a.err)) { *abort_flag = 1; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sa = smem_u32(smem + st * C::STAGE);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          const uint64_t da = umma_desc_sw128(sa + k * C::A_BOX), db = umma_desc_sw128(sa + C::A_BYTES + k * C::B_BOX);
#pragma unroll
          for (int j = 0; j < TC_BK / 16; ++j)
            umma_bf16(tmem, da + 2 * j, db + 2 * j, idesc, (i == 0 && k == 0 && j == 0) ? 0u : 1u);
        }
        umma_commit(&empty[st]);
      }
      umma_commit(&accf[0]);  // also after an abort: the epilogue must not wait in vain
    }
  } else {
    const unsigned long long t_entry = globaltimer();
    pdl_wait();
    if (threadIdx.x == 64) {
      s_epoch = a.state[kTpStateOproj + cta] + 1;
      s_ok = 1;
      if (a.stamps && cta == 0) {
        tp_stamp(a.stamps, s_epoch, 0, t_entry);
        tp_stamp(a.stamps, s_epoch, 1, globaltimer());
      }
    }
    // ------------------- epilogue part 1: the partner's token half -------------------
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const bool ok = mbar_wait(&accf[0], 0, a.err) && !*abort_flag;
    if (!ok) *abort_flag = 1;  // read again by every epilogue thread in part 2
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x == 64) s_tacc = globaltimer();
    if (S > 1) {
      const uint32_t dst = mapa_shared(smem_u32(stage), (uint32_t)(part ^ 1));
      const int c_other = (part ^ 1) * C::HALF;
#pragma unroll 1
      for (int c0 = 0; c0 < C::HALF; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + lane_base + c_other + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) st_cluster_f32(dst + (uint32_t)(((c0 + j) * TC_BM + row) * 4), ok ? v[j] : kTpPoison);
      }
    }
  }
  __syncwarp();
  if (S > 1) cluster_sync_all();  // every CTA's half has landed in its partner

  if (warp >= 2) {
    const int et = threadIdx.x - 64;  // 0..127
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int W = a.world, sl = a.sl, rank = a.rank;
    tp_epi_bar();  // s_epoch visible
    const int epoch = s_epoch;
    unsigned long long* const st0 = (a.stamps && cta == 0 && et == 0) ? a.stamps : nullptr;
    tp_stamp(st0, epoch, 2, s_tacc);
    tp_stamp(st0, epoch, 3, globaltimer());
    // ---------- epilogue part 2: finish the own half in shared memory, push the slices ----------
    // An expired wait anywhere in this CTA (loads, MMAs, accumulator) leaves the accumulator
    // incomplete: the slices are then pushed as NaN, so the peers (whose own error words stay
    // clear) produce visibly invalid rows for this tile instead of a silently wrong sum, and
    // nobody waits for flags that are never raised.
    const int c_own = part * C::HALF;
    const bool acc_ok = !*abort_flag;
#pragma unroll 1
    for (int c0 = 0; c0 < C::HALF; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + lane_base + c_own + c0, v);
      if (!acc_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = kTpPoison;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float* sp = stage + (c0 + j) * TC_BM + row;
        *sp = S > 1 ? (part == 0 ? v[j] + *sp : *sp + v[j]) : v[j];
      }
    }
    tp_epi_bar();
    tp_stamp(st0, epoch, 4, globaltimer());
    for (int s = 0; s < W; ++s) {
      if (s == rank || c_own + s * sl >= a.M) continue;  // own slice stays; empty slices are skipped
      const float4* src = reinterpret_cast<const float4*>(stage + s * sl * TC_BM);
      float4* dst = reinterpret_cast<float4*>(a.recv[s] + (size_t)(cta * W + rank) * sl * TC_BM);
      for (int e = et; e < sl * (TC_BM / 4); e += 128) dst[e] = src[e];
    }
    tp_epi_bar();
    tp_stamp(st0, epoch, 5, globaltimer());
    tp_signal(a.flags, et, W, rank, cta * W + rank, epoch);
    tp_stamp(st0, epoch, 6, globaltimer());
    // ------------- epilogue part 3: reduce this rank's slice, all-gather it -------------
    if (!tp_wait(a.flags, et, W, rank, cta * W, epoch, a.err)) s_ok = 0;
    tp_epi_bar();
    tp_stamp(st0, epoch, 7, globaltimer());
    if (s_ok) {
      const float* slots = a.recv[rank] + (size_t)cta * W * sl * TC_BM;  // [W][sl][128]
      const float* own = stage + rank * sl * TC_BM;                      // [sl][128]
      for (int e = et; e < sl * 16; e += 128) {
        const int mo = e >> 4, r8 = (e & 15) * 8;
        const int m = c_own + rank * sl + mo, n8 = tile * TC_BM + r8;
        if (m >= a.M || n8 >= a.N) continue;
        float4 v[2 * kTpMaxRanks];
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
          if (q < W) {
            if (q == rank) {
              const float4* src = reinterpret_cast<const float4*>(own + mo * TC_BM + r8);
              v[2 * q] = src[0];
              v[2 * q + 1] = src[1];
            } else {
              const float4* src = reinterpret_cast<const float4*>(slots + ((size_t)q * sl + mo) * TC_BM + r8);
              v[2 * q] = __ldcg(src);
              v[2 * q + 1] = __ldcg(src + 1);
            }
          }
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
          if (q < W) {
            acc[0] += v[2 * q].x; acc[1] += v[2 * q].y; acc[2] += v[2 * q].z; acc[3] += v[2 * q].w;
            acc[4] += v[2 * q + 1].x; acc[5] += v[2 * q + 1].y; acc[6] += v[2 * q + 1].z; acc[7] += v[2 * q + 1].w;
          }
        const size_t o = (size_t)m * a.ldo + n8;
        if (a.residual) {
          const uint4 rv = *reinterpret_cast<const uint4*>(a.residual + o);
          acc[0] += bf16_lo(rv.x); acc[1] += bf16_hi(rv.x); acc[2] += bf16_lo(rv.y); acc[3] += bf16_hi(rv.y);
          acc[4] += bf16_lo(rv.z); acc[5] += bf16_hi(rv.z); acc[6] += bf16_lo(rv.w); acc[7] += bf16_hi(rv.w);
        }
        const uint4 ov = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                    pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
#pragma unroll
        for (int q = 0; q < kTpMaxRanks; ++q)
          if (q < W) *reinterpret_cast<uint4*>(a.out[q] + o) = ov;
      }
    }
    // ------------- exit: the same CTA index of every rank has stored into us -------------
    tp_epi_bar();
    tp_stamp(st0, epoch, 8, globaltimer());
    const int xb = a.ctas * W;
    tp_signal(a.flags, et, W, rank, xb + cta * W + rank, epoch);
    tp_stamp(st0, epoch, 9, globaltimer());
    tp_wait(a.flags, et, W, rank, xb + cta * W, epoch, a.err);
    tp_stamp(st0, epoch, 10, globaltimer());
    if (et == 0) a.state[kTpStateOproj + cta] = epoch;  // read by this CTA index's next call
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// Host plan of tp_oproj_kernel: BN = 64 (M <= 64) or 128 (M <= 128) tokens; S = 2 CTAs per
// weight tile when the pairs fit on the GPU at once, else 1; sl = BN / S / W tokens per slice.
struct TpPlan {
  int bn, s, tiles, ctas, sl;
};

template <int BN, int STAGES, int KS, int S>
static int tp_kernel_fits(int ctas) {
  using C = TpCfg<BN, STAGES, KS, S>;
  static int max_ctas = -1;  // co-resident CTAs of this instantiation (per process: one device type)
  if (max_ctas < 0) {
    if (cudaFuncSetAttribute(tp_oproj_kernel<BN, STAGES, KS, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM) != cudaSuccess) {
      cudaGetLastError();
      max_ctas = 0;
    } else if (S > 1) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S * okc_host::num_sms());
      cfg.blockDim = dim3(192);
      cfg.dynamicSmemBytes = C::SMEM;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = S;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, tp_oproj_kernel<BN, STAGES, KS, S>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
      }
      max_ctas = clusters * S;
    } else {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tp_oproj_kernel<BN, STAGES, KS, S>, 192,
                                                        C::SMEM) != cudaSuccess) {
        cudaGetLastError();
        per_sm = 0;
      }
      max_ctas = per_sm * okc_host::num_sms();
    }
  }
  return ctas <= max_ctas && ctas <= kTpMaxCtas;
}

// tp_oproj stage shapes: BN = 64 -> 4 stages of 2 K boxes (48 KB each); BN = 128 -> 3 (64 KB),
// or 2 when one CTA finishes all 128 tokens (its 64 KB staging buffer takes the third).
#define OKC_TP_CFG_64 64, 4, 2
#define OKC_TP_CFG_128 128, 3, 2
#define OKC_TP_CFG_128_S1 128, 2, 2

static bool tp_plan(int M, int N, int K, int world, TpPlan& pl) {
  if (M < 1 || M > 128 || N < 8 || N % 8 || K < 16 || K % 8 || world < 2 || world > kTpMaxRanks) return false;
  pl.bn = M <= 64 ? 64 : 128;
  pl.tiles = (N + TC_BM - 1) / TC_BM;
  const int nkb = (K + TC_BK * 2 - 1) / (TC_BK * 2);
  for (int s = 2; s >= 1; --s) {
    if (s == 2 && nkb < 2) continue;
    if ((pl.bn / s) % world) continue;
    const int ctas = pl.tiles * s;
    bool fits;
    if (pl.bn == 64)
      fits = s == 2 ? tp_kernel_fits<OKC_TP_CFG_64, 2>(ctas) : tp_kernel_fits<OKC_TP_CFG_64, 1>(ctas);
    else
      fits = s == 2 ? tp_kernel_fits<OKC_TP_CFG_128, 2>(ctas) : tp_kernel_fits<OKC_TP_CFG_128_S1, 1>(ctas);
    if (!fits) continue;
    pl.s = s;
    pl.ctas = ctas;
    pl.sl = pl.bn / s / world;
    return true;
  }
  return false;
}

template <int BN, int STAGES, int KS, int S>
static int launch_tp_oproj_t(const CUtensorMap& mw, const CUtensorMap& mx, const TpGemmArgs& a, cudaStream_t stream) {
  using C = TpCfg<BN, STAGES, KS, S>;
  return okc_host::launch_k(tp_oproj_kernel<BN, STAGES, KS, S>, dim3(a.ctas), dim3(192), C::SMEM, stream, dim3(S),
                            mw, mx, a);
}

}  // namespace okc

// ------------------------------------------------------------------------------ C ABI

static unsigned long long* tp_trace_stamps(void* workspace, int kernel) {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("OKC_TP_TRACE");
    on = (e && e[0] == '1') ? 1 : 0;
  }
  return on ? reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(workspace) + okc::kTpTraceOffset) +
                  kernel * 64
            : nullptr;
}

extern "C" int okc_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return OKC_ERR_INVALID;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return OKC_ERR_DEVICE;
  }
  return OKC_OK;
}

extern "C" int okc_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? OKC_OK : OKC_ERR_DEVICE; }

extern "C" int okc_ipc_handle(const void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return OKC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  memcpy(handle_out, &h, sizeof(h));
  return OKC_OK;
}

extern "C" int okc_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return OKC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return OKC_ERR_DEVICE;
  }
  return OKC_OK;
}

extern "C" int okc_ipc_close(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? OKC_OK : OKC_ERR_DEVICE;
}

extern "C" int okc_tp_allreduce_residual(const float* const* parts, void* const* outs, int* const* flags,
                                         const void* residual, int* state, int rank, int world,
                                         long long n, void* workspace, okc_stream_t stream) {
  if (world < 2 || world > okc::kTpMaxRanks || rank < 0 || rank >= world || n <= 0 || (n & 3) ||
      !parts || !outs || !flags || !state || !workspace)
    return OKC_ERR_INVALID;
  okc::TpArgs a = {};
  for (int q = 0; q < world; ++q) {
    if (!parts[q] || !outs[q] || !flags[q]) return OKC_ERR_INVALID;
    if (!okc_host::aligned16(parts[q]) || (reinterpret_cast<uintptr_t>(outs[q]) & 7)) return OKC_ERR_ALIGNMENT;
    a.part[q] = parts[q];
    a.out[q] = reinterpret_cast<__nv_bfloat16*>(outs[q]);
    a.flags[q] = flags[q];
  }
  if (reinterpret_cast<uintptr_t>(residual) & 7) return OKC_ERR_ALIGNMENT;
  a.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  a.state = state;
  a.err = reinterpret_cast<int*>(workspace);
  a.n = n;
  a.rank = rank;
  a.world = world;
  a.stamps = tp_trace_stamps(workspace, 0);
  // The grid must be the same on every rank (CTA c waits for CTA c of the peers): it depends
  // only on n, world and the SM count of the (identical) GPUs.
  const long long per4 = ((n >> 2) + world - 1) / world;
  int blocks = (int)((per4 + 255) / 256);
  int cap = 2 * okc_host::num_sms();
  if (cap > okc::kTpMaxCtas) cap = okc::kTpMaxCtas;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return okc_host::launch_k(okc::tp_allreduce_kernel, dim3(blocks), dim3(256), 0,
                            reinterpret_cast<cudaStream_t>(stream), dim3(1), a);
}

extern "C" int okc_tp_oproj_plan(int M, int N, int K, int world, size_t* recv_bytes, int* flag_words) {
  okc::TpPlan pl;
  if (!okc::tp_plan(M, N, K, world, pl)) return OKC_ERR_INVALID;
  if (recv_bytes) *recv_bytes = (size_t)pl.ctas * world * pl.sl * okc::TC_BM * sizeof(float);
  if (flag_words) *flag_words = 2 * pl.ctas * world;
  return OKC_OK;
}

extern "C" int okc_tp_oproj_allreduce_residual(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                                               float* const* recv, void* const* outs, int* const* flags,
                                               const void* residual, int ldo, int* state, int rank, int world,
                                               void* workspace, okc_stream_t stream) {
  okc::TpPlan pl;
  if (!x || !w || !recv || !outs || !flags || !state || !workspace || rank < 0 || rank >= world ||
      ldx < K || ldw < K || ldo < N || !okc::tp_plan(M, N, K, world, pl))
    return OKC_ERR_INVALID;
  if (!okc_host::aligned16(x) || !okc_host::aligned16(w) || ldx % 8 || ldw % 8 || ldo % 8 ||
      !okc_host::aligned16(residual))
    return OKC_ERR_ALIGNMENT;
  okc::TpGemmArgs a = {};
  for (int q = 0; q < world; ++q) {
    if (!recv[q] || !outs[q] || !flags[q]) return OKC_ERR_INVALID;
    if (!okc_host::aligned16(recv[q]) || !okc_host::aligned16(outs[q])) return OKC_ERR_ALIGNMENT;
    a.recv[q] = recv[q];
    a.out[q] = reinterpret_cast<__nv_bfloat16*>(outs[q]);
    a.flags[q] = flags[q];
  }
  a.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  a.state = state;
  a.err = reinterpret_cast<int*>(workspace);
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldo = ldo;
  a.rank = rank;
  a.world = world;
  a.sl = pl.sl;
  a.ctas = pl.ctas;
  a.stamps = tp_trace_stamps(workspace, 1);
  CUtensorMap mw, mx;
  if (!okc::tc_make_map(&mw, w, K, N, ldw, okc::TC_BM) || !okc::tc_make_map(&mx, x, K, M, ldx, pl.bn))
    return OKC_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pl.bn == 64)
    return pl.s == 2 ? okc::launch_tp_oproj_t<OKC_TP_CFG_64, 2>(mw, mx, a, st)
                     : okc::launch_tp_oproj_t<OKC_TP_CFG_64, 1>(mw, mx, a, st);
  return pl.s == 2 ? okc::launch_tp_oproj_t<OKC_TP_CFG_128, 2>(mw, mx, a, st)
                   : okc::launch_tp_oproj_t<OKC_TP_CFG_128_S1, 1>(mw, mx, a, st);
}
