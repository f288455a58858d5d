// Paged FP8 attention for prefill blocks: the L new tokens of a request attend its cache
// (positions <= their own, inside the sliding window when one is set) with the block's own
// keys already appended — muse_prefill_layer/submission.py:137-176 (`attention`) for
// q_len 200-16384.  The decode kernel serves one query row per token and reads a token's whole
// span for each; here one CTA takes 8 consecutive tokens of a request x the G query heads of
// one KV head (64 query rows, 4 warps of 16) and streams the request's keys in tiles of 64
// positions once for all of them.
//
// Roofline: compute on the CUDA-core tensor path at these sizes (per 64-key tile and CTA:
// 64 x 64 x D x 2 MACs for QK and PV against 64 x D x 2 bytes from L2); the cache itself is
// read from HBM once per request and KV head and served from L2 to the CTAs of its tokens.
//
//  * Operands in f16: e4m3 cache values and bf16 query values are exact in f16 (the query rows
//    are first scaled by a power of two so that their largest magnitude is below 2^14), P is
//    rounded to f16 (2^-11 relative); accumulation in fp32 (mma.sync m16n8k16 f16 -> f32).
//  * Tile loads: 128 threads fetch the 64 positions' K and V rows of this KV head (one page-table
//    lookup per position; a position outside the table or past the CTA's last token reads
//    zeros and is masked), convert e4m3 -> f16 and store K as [key][d] and V transposed as
//    [d][key] in shared memory, padded so the fragment loads are conflict-free.
//  * Online softmax in the log2 domain per query row; a row's mask is its token's position
//    (causal) and the window.  Epilogue: o / l * v_scale, then (with a gate) Muse's per-head
//    RMSNorm times sigmoid(gate), bf16.
#include "kernels.cuh"

namespace okc {

namespace {

constexpr int kPfTok = 8;     // tokens per CTA
constexpr int kPfKeys = 64;   // key positions per tile
constexpr int kPfThreads = 128;

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two e4m3 bytes (low byte first) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two) {
  uint32_t h;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(h) : "r"(two));
  return h;
}

struct PfArgs {
  const __nv_bfloat16* q;  // [T][Hq][D] (row stride ldq elements)
  int ldq;
  const uint8_t* k_cache;  // e4m3 [num_pages][P][Hkv][D]
  const uint8_t* v_cache;
  const int32_t* page_table;  // [B][table_ld], max_pages valid columns
  int table_ld, max_pages;
  const int64_t* positions;  // [T] = [B][L]
  const float* k_scale;      // [Hkv]
  const float* v_scale;
  const __nv_bfloat16* gate;  // [T][ld_gate] or nullptr
  int ld_gate;
  __nv_bfloat16* out;  // [T][ldo]
  int ldo;
  int B, L, Hq, Hkv, G, P, window;
  long long num_pages;
  float sm_scale_log2;  // sm_scale * log2(e)
  float out_eps;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(PfArgs a) {
  constexpr int KS = D / 16;    // k16 steps over d (QK)
  constexpr int ND = D / 8;     // n8 blocks over d (PV)
  constexpr int KP = D + 8;     // K row pitch (f16): conflict-free 32-bit fragment loads
  constexpr int VP = kPfKeys + 8;  // Vt row pitch (f16)
  __shared__ __align__(16) __half Ks[kPfKeys * KP];
  __shared__ __align__(16) __half Vt[D * VP];
  __shared__ int tile_page[kPfKeys];

  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.z, h = blockIdx.y;
  const int t0 = blockIdx.x * kPfTok;  // first token of the CTA inside the request's block
  if (t0 >= a.L) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  // this thread's two query rows: (token ta, head g) and (token tb, head g)
  const int ta = t0 + 2 * warp, tb = ta + 1;
  const bool va = ta < a.L && g < a.G, vb = tb < a.L && g < a.G;
  const long long pa = va ? a.positions[(size_t)b * a.L + ta] : -1;
  const long long pb = vb ? a.positions[(size_t)b * a.L + tb] : -1;
  const int hq = h * a.G + g;

  // ---- query fragments (rows ta/tb x head g), scaled by 2^-sa / 2^-sb (exact) into f16 ----
  float qa[D / 4], qb[D / 4];  // this thread's 2 elements per 8-wide group: d = 8 j + 2 c + {0, 1}
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    float2 x = make_float2(0.f, 0.f), y = make_float2(0.f, 0.f);
    if (va) x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
              a.q + (size_t)(b * a.L + ta) * a.ldq + (size_t)hq * D + 8 * j + 2 * c));
    if (vb) y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
              a.q + (size_t)(b * a.L + tb) * a.ldq + (size_t)hq * D + 8 * j + 2 * c));
    qa[2 * j] = x.x; qa[2 * j + 1] = x.y;
    qb[2 * j] = y.x; qb[2 * j + 1] = y.y;
  }
  float ma = 0.f, mb = 0.f;
#pragma unroll
  for (int i = 0; i < D / 4; ++i) { ma = fmaxf(ma, fabsf(qa[i])); mb = fmaxf(mb, fabsf(qb[i])); }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  }
  // 2^s with the row maximum below 2^14 after the scale (|q| in [2^-100, 2^100] assumed)
  auto pow2_down = [](float m) {
    int s = 0;
    if (m > 0.f) s = max(0, (int)((__float_as_uint(m) >> 23) & 0xff) - 127 - 13);
    return s;
  };
  const int sa = pow2_down(ma), sb = pow2_down(mb);
  const float da = __uint_as_float((uint32_t)(127 - sa) << 23), db = __uint_as_float((uint32_t)(127 - sb) << 23);
  uint32_t qf[KS][4];
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    qf[k][0] = pack_h2(qa[4 * k] * da, qa[4 * k + 1] * da);      // row g (ta), d = 16k + 2c
    qf[k][1] = pack_h2(qb[4 * k] * db, qb[4 * k + 1] * db);      // row g+8 (tb)
    qf[k][2] = pack_h2(qa[4 * k + 2] * da, qa[4 * k + 3] * da);  // row g, d = 16k + 8 + 2c
    qf[k][3] = pack_h2(qb[4 * k + 2] * db, qb[4 * k + 3] * db);
  }
  const float ks = a.k_scale[h] * a.sm_scale_log2;
  const float fa = ks * __uint_as_float((uint32_t)(127 + sa) << 23);  // undo the query scale
  const float fb = ks * __uint_as_float((uint32_t)(127 + sb) << 23);

  // ---- key range of the CTA: [lo, hi] over its tokens' visible spans ----
  const int tl = min(a.L, t0 + kPfTok) - 1;
  const long long p_first = a.positions[(size_t)b * a.L + t0];
  const long long p_last = a.positions[(size_t)b * a.L + tl];
  long long lo = 0;
  if (a.window > 0) lo = max(0ll, p_first - a.window + 1);
  const long long hi = p_last;

  float o_acc[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o_acc[n][0] = o_acc[n][1] = o_acc[n][2] = o_acc[n][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  for (long long kv0 = lo; kv0 <= hi; kv0 += kPfKeys) {
    // ---- tile load: K [key][d], V^T [d][key] in f16 ----
    __syncthreads();  // the previous tile's fragments are consumed
    if (threadIdx.x < kPfKeys) {
      const long long pos = kv0 + threadIdx.x;
      int page = -1;
      if (pos <= hi) {
        const long long lp = pos / a.P;
        if (lp < a.max_pages) page = a.page_table[(size_t)b * a.table_ld + lp];
        if (page < 0 || page >= a.num_pages) {
          atomicOr(a.err, OKC_DEVERR_PAGE);
          page = -1;
        }
      }
      tile_page[threadIdx.x] = page;
    }
    __syncthreads();
    {
      const int key = threadIdx.x >> 1, part = threadIdx.x & 1;  // 2 threads per position: D/2 bytes each
      const int page = tile_page[key];
      const long long pos = kv0 + key;
      uint4 kr[D / 32], vr[D / 32];
#pragma unroll
      for (int i = 0; i < D / 32; ++i) kr[i] = vr[i] = make_uint4(0u, 0u, 0u, 0u);
      if (page >= 0) {
        const size_t row = (((size_t)page * a.P + (size_t)(pos % a.P)) * a.Hkv + h) * D + part * (D / 2);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
          kr[i] = *reinterpret_cast<const uint4*>(a.k_cache + row + 16 * i);
          vr[i] = *reinterpret_cast<const uint4*>(a.v_cache + row + 16 * i);
        }
      }
#pragma unroll
      for (int i = 0; i < D / 32; ++i) {
        const uint32_t kw[4] = {kr[i].x, kr[i].y, kr[i].z, kr[i].w};
        const uint32_t vw[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int d0 = part * (D / 2) + 16 * i + 4 * w;  // 4 values: d0 .. d0 + 3
          const uint32_t k01 = e4m3x2_to_h2(kw[w] & 0xffffu), k23 = e4m3x2_to_h2(kw[w] >> 16);
          *reinterpret_cast<uint2*>(&Ks[key * KP + d0]) = make_uint2(k01, k23);
          const uint32_t v01 = e4m3x2_to_h2(vw[w] & 0xffffu), v23 = e4m3x2_to_h2(vw[w] >> 16);
          Vt[(d0 + 0) * VP + key] = __ushort_as_half((unsigned short)(v01 & 0xffffu));
          Vt[(d0 + 1) * VP + key] = __ushort_as_half((unsigned short)(v01 >> 16));
          Vt[(d0 + 2) * VP + key] = __ushort_as_half((unsigned short)(v23 & 0xffffu));
          Vt[(d0 + 3) * VP + key] = __ushort_as_half((unsigned short)(v23 >> 16));
        }
      }
    }
    __syncthreads();

    // ---- S = Q K^T: 16 rows x 64 keys per warp (8 n8 blocks) ----
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&Ks[(8 * n + g) * KP + 16 * k + 2 * c]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&Ks[(8 * n + g) * KP + 16 * k + 8 + 2 * c]);
        mma_f16_16816(s[n], qf[k], b0, b1);
      }
    }
    // ---- mask, online softmax (log2 domain) ----
    float tmax_a = -INFINITY, tmax_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const long long kp = kv0 + 8 * n + 2 * c + e;
        const bool ok_a = va && kp <= pa && (a.window <= 0 || kp > pa - a.window);
        const bool ok_b = vb && kp <= pb && (a.window <= 0 || kp > pb - a.window);
        s[n][e] = ok_a ? s[n][e] * fa : -INFINITY;
        s[n][2 + e] = ok_b ? s[n][2 + e] * fb : -INFINITY;
        tmax_a = fmaxf(tmax_a, s[n][e]);
        tmax_b = fmaxf(tmax_b, s[n][2 + e]);
      }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      tmax_a = fmaxf(tmax_a, __shfl_xor_sync(0xffffffffu, tmax_a, o));
      tmax_b = fmaxf(tmax_b, __shfl_xor_sync(0xffffffffu, tmax_b, o));
    }
    const float nm_a = fmaxf(m_a, tmax_a), nm_b = fmaxf(m_b, tmax_b);
    // a row with nothing visible yet keeps a finite subtraction origin
    const float oa = nm_a == -INFINITY ? 0.f : nm_a, ob = nm_b == -INFINITY ? 0.f : nm_b;
    const float ra = exp2f(m_a - oa), rb = exp2f(m_b - ob);  // exp2(-inf) = 0 for a fresh row
    m_a = nm_a;
    m_b = nm_b;
    float rs_a = 0.f, rs_b = 0.f;
    uint32_t pf[4][4];  // P as the A operand of PV: k16 step j = keys 16 j .. 16 j + 15
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - oa), p1 = exp2f(s[n][1] - oa);
      const float p2 = exp2f(s[n][2] - ob), p3 = exp2f(s[n][3] - ob);
      rs_a += p0 + p1;
      rs_b += p2 + p3;
      pf[n >> 1][(n & 1) * 2 + 0] = pack_h2(p0, p1);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_h2(p2, p3);
    }
    l_a = l_a * ra + rs_a;
    l_b = l_b * rb + rs_b;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      o_acc[n][0] *= ra; o_acc[n][1] *= ra;
      o_acc[n][2] *= rb; o_acc[n][3] *= rb;
    }
    // ---- O += P V: V^T rows are d, columns keys ----
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int n = 0; n < ND; ++n) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&Vt[(8 * n + g) * VP + 16 * j + 2 * c]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&Vt[(8 * n + g) * VP + 16 * j + 8 + 2 * c]);
        mma_f16_16816(o_acc[n], pf[j], b0, b1);
      }
    }
  }

  // ---- epilogue: o / l * v_scale, then rms(o) * sigmoid(gate) per head (with a gate) ----
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o);
  }
  const float vs = a.v_scale[h];
  const float ia = l_a > 0.f ? vs / l_a : 0.f, ib = l_b > 0.f ? vs / l_b : 0.f;
  float ss_a = 0.f, ss_b = 0.f;
#pragma unroll
  for (int n = 0; n < ND; ++n) {
    o_acc[n][0] *= ia; o_acc[n][1] *= ia;
    o_acc[n][2] *= ib; o_acc[n][3] *= ib;
    ss_a += o_acc[n][0] * o_acc[n][0] + o_acc[n][1] * o_acc[n][1];
    ss_b += o_acc[n][2] * o_acc[n][2] + o_acc[n][3] * o_acc[n][3];
  }
  if (a.gate) {
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      ss_a += __shfl_xor_sync(0xffffffffu, ss_a, o);
      ss_b += __shfl_xor_sync(0xffffffffu, ss_b, o);
    }
    const float na = rsqrtf(ss_a / (float)D + a.out_eps), nb = rsqrtf(ss_b / (float)D + a.out_eps);
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      const int d = 8 * n + 2 * c;
      if (va) {
        const float2 gv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
            a.gate + (size_t)(b * a.L + ta) * a.ld_gate + (size_t)hq * D + d));
        o_acc[n][0] = o_acc[n][0] * na * (1.f / (1.f + expf(-gv.x)));
        o_acc[n][1] = o_acc[n][1] * na * (1.f / (1.f + expf(-gv.y)));
      }
      if (vb) {
        const float2 gv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
            a.gate + (size_t)(b * a.L + tb) * a.ld_gate + (size_t)hq * D + d));
        o_acc[n][2] = o_acc[n][2] * nb * (1.f / (1.f + expf(-gv.x)));
        o_acc[n][3] = o_acc[n][3] * nb * (1.f / (1.f + expf(-gv.y)));
      }
    }
  }
#pragma unroll
  for (int n = 0; n < ND; ++n) {
    const int d = 8 * n + 2 * c;
    if (va)
      *reinterpret_cast<__nv_bfloat162*>(a.out + (size_t)(b * a.L + ta) * a.ldo + (size_t)hq * D + d) =
          __floats2bfloat162_rn(o_acc[n][0], o_acc[n][1]);
    if (vb)
      *reinterpret_cast<__nv_bfloat162*>(a.out + (size_t)(b * a.L + tb) * a.ldo + (size_t)hq * D + d) =
          __floats2bfloat162_rn(o_acc[n][2], o_acc[n][3]);
  }
}

}  // namespace

int launch_attn_prefill(const void* q, int ldq, const void* k_cache, const void* v_cache, const int32_t* page_table,
                        int table_ld, int max_pages, const int64_t* positions, const float* k_scale,
                        const float* v_scale, const void* gate, int ld_gate, void* out, int ldo, int B, int L, int Hq,
                        int Hkv, int D, int page_size, long long num_pages, float sm_scale, int window, float out_eps,
                        int* err, cudaStream_t stream) {
  PfArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.ldq = ldq;
  a.k_cache = reinterpret_cast<const uint8_t*>(k_cache);
  a.v_cache = reinterpret_cast<const uint8_t*>(v_cache);
  a.page_table = page_table;
  a.table_ld = table_ld;
  a.max_pages = max_pages;
  a.positions = positions;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  a.ld_gate = ld_gate;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.B = B;
  a.L = L;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.P = page_size;
  a.window = window;
  a.num_pages = num_pages;
  a.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  a.out_eps = out_eps;
  a.err = err;
  const dim3 grid((L + kPfTok - 1) / kPfTok, Hkv, B);
  if (D == 64) return okc_host::launch_k(attn_prefill_kernel<64>, grid, dim3(kPfThreads), 0, stream, dim3(1), a);
  if (D == 128) return okc_host::launch_k(attn_prefill_kernel<128>, grid, dim3(kPfThreads), 0, stream, dim3(1), a);
  return OKC_ERR_INVALID;
}

}  // namespace okc
