// extern "C" entry points of libokc_b200.so: argument validation, workspace carving and
// kernel-family dispatch.  Declarations and contracts: include/okc_b200.h.
#include <mutex>

#include "common.cuh"

#include "kernels.cuh"

namespace okc_host {
int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}
}  // namespace okc_host

using okc_host::aligned16;

extern "C" {

const char* okc_version(void) { return "okc_b200 0.1 sm_100a"; }

int okc_read_device_error(const void* workspace, okc_stream_t stream) {
  if (!workspace) return OKC_ERR_INVALID;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return OKC_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return OKC_ERR_LAUNCH;
  if (cudaMemset(const_cast<void*>(workspace), 0, sizeof(int)) != cudaSuccess) return OKC_ERR_LAUNCH;
  return v;
}

// ------------------------------------------------------------------------------ GEMM
size_t okc_gemm_bf16_workspace_bytes(int M, int N, int K) {
  size_t tc = okc::tc_gemm_ws_bytes(M > 256 ? 256 : M, N, K);  // M > 256 runs in 256-row blocks
  return 256 + tc;
}

int okc_gemm_bf16_ex(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                     const void* residual, int M, int N, int K, int out_fp32, int family, int splits,
                     void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  if (!x || !w || !y || M <= 0 || N <= 0 || K <= 0) return OKC_ERR_INVALID;
  if (K % 8 || ldx % 8 || ldw % 8 || ldx < K || ldw < K || ldy < N) return OKC_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w)) return OKC_ERR_ALIGNMENT;
  const uintptr_t ya = reinterpret_cast<uintptr_t>(y), ra = reinterpret_cast<uintptr_t>(residual);
  if ((ya & (out_fp32 ? 3u : 1u)) || (ra & 1u)) return OKC_ERR_ALIGNMENT;
  if (M > 256 && family != 1) {
    // prefill token counts: 256-row blocks through the tcgen05 path (a block's weight tiles are
    // re-read from L2 by the next block); a tail of <= 32 rows takes the skinny kernel
    const size_t esz = out_fp32 ? 4 : 2;
    for (int m0 = 0; m0 < M; m0 += 256) {
      const int mm = M - m0 < 256 ? M - m0 : 256;
      const void* rs = residual ? reinterpret_cast<const uint8_t*>(residual) + (size_t)m0 * ldy * 2 : nullptr;
      const int st = okc_gemm_bf16_ex(reinterpret_cast<const uint8_t*>(x) + (size_t)m0 * ldx * 2, ldx, w, ldw,
                                      reinterpret_cast<uint8_t*>(y) + (size_t)m0 * ldy * esz, ldy, rs, mm, N, K,
                                      out_fp32, family == 2 && mm > 32 ? 2 : 0, splits, workspace,
                                      workspace_bytes, stream);
      if (st) return st;
    }
    return OKC_OK;
  }
  if (family == 0) family = (M > 32 && okc::tc_gemm_supported(M, N, K, ldx, ldw) && ldy % 8 == 0) ? 2 : 1;
  if (family == 2) {
    if (!okc::tc_gemm_supported(M, N, K, ldx, ldw)) return OKC_ERR_INVALID;
    if (!workspace || workspace_bytes < okc_gemm_bf16_workspace_bytes(M, N, K)) return OKC_ERR_WORKSPACE;
    return okc::launch_tc_gemm(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32,
                               reinterpret_cast<uint8_t*>(workspace) + 256, workspace_bytes - 256,
                               stream);
  }
  if (family != 1) return OKC_ERR_INVALID;
  // skinny kernel: 64 tokens per pass
  const size_t esz = out_fp32 ? 4 : 2;
  for (int m0 = 0; m0 < M; m0 += 64) {
    const int mm = M - m0 < 64 ? M - m0 : 64;
    const void* xs = reinterpret_cast<const uint8_t*>(x) + (size_t)m0 * ldx * 2;
    void* ys = reinterpret_cast<uint8_t*>(y) + (size_t)m0 * ldy * esz;
    const void* rs = residual ? reinterpret_cast<const uint8_t*>(residual) + (size_t)m0 * ldy * 2 : nullptr;
    const int st = okc::launch_skinny_gemm(xs, ldx, w, ldw, ys, ldy, rs, mm, N, K, out_fp32, splits, stream);
    if (st) return st;
  }
  return OKC_OK;
}

int okc_gemm_bf16(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                  const void* residual, int M, int N, int K, int out_fp32, void* workspace,
                  size_t workspace_bytes, okc_stream_t stream) {
  return okc_gemm_bf16_ex(x, ldx, w, ldw, y, ldy, residual, M, N, K, out_fp32, 0, 0, workspace,
                          workspace_bytes, stream);
}

// --------------------------------------------------------------------------- RMSNorm
int okc_rmsnorm_bf16(const void* x, int ldx, const void* w, void* y, int ldy, int T, int H, float eps,
                     int unit_offset, okc_stream_t stream) {
  if (!x || !w || !y || T <= 0 || H <= 0 || H % 8 || H > 16384 || ldx % 8 || ldy % 8) return OKC_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return OKC_ERR_ALIGNMENT;
  return okc::launch_rmsnorm(x, ldx, w, y, ldy, T, H, eps, unit_offset, stream);
}

int okc_residual_boundary(const float* stream_in, const void* branch, int ld_branch, const float* alpha,
                          const float* beta, const void* post_w, const void* pre_w, void* hidden, float* stream_out,
                          float* router_out, int T, int H, float post_eps, float pre_eps, okc_stream_t stream) {
  if (!stream_in || !branch || !alpha || !beta || !pre_w || !hidden || !stream_out || T <= 0 || H <= 0 ||
      H % 8 || H > 16384 || ld_branch < H || ld_branch % 8)
    return OKC_ERR_INVALID;
  if (!aligned16(stream_in) || !aligned16(branch) || !aligned16(alpha) || !aligned16(beta) || !aligned16(pre_w) ||
      !aligned16(hidden) || !aligned16(stream_out) || (post_w && !aligned16(post_w)) ||
      (router_out && !aligned16(router_out)))
    return OKC_ERR_ALIGNMENT;
  return okc::launch_residual_boundary(stream_in, branch, ld_branch, alpha, beta, post_w, pre_w, hidden, stream_out,
                                       router_out, T, H, post_eps, pre_eps, stream);
}

// --------------------------------------------------------------- prefill attention
int okc_attn_prefill_fp8(const void* q, int ldq, const void* k_cache, const void* v_cache, const int32_t* page_table,
                         int table_ld, int max_pages, const int64_t* positions, const float* k_scale,
                         const float* v_scale, const void* gate, int ld_gate, float out_eps, void* out, int ldo,
                         int B, int L, int Hq, int Hkv, int D, int page_size, int64_t num_pages, float sm_scale,
                         int window, void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  if (!q || !k_cache || !v_cache || !page_table || !positions || !k_scale || !v_scale || !out) return OKC_ERR_INVALID;
  if (B <= 0 || L <= 0 || (long long)B * L >= (1LL << 31) || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8) return OKC_ERR_INVALID;
  if (!(D == 64 || D == 128) || page_size <= 0 || num_pages <= 0 || max_pages <= 0 || table_ld < max_pages ||
      window < 0)
    return OKC_ERR_INVALID;
  if (ldq < Hq * D || ldq % 8 || ldo < Hq * D || ldo % 2 || (gate && (ld_gate < Hq * D || ld_gate % 2)))
    return OKC_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (gate && (reinterpret_cast<uintptr_t>(gate) & 3)))
    return OKC_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < 256) return OKC_ERR_WORKSPACE;
  return okc::launch_attn_prefill(q, ldq, k_cache, v_cache, page_table, table_ld, max_pages, positions, k_scale,
                                  v_scale, gate, ld_gate, out, ldo, B, L, Hq, Hkv, D, page_size, num_pages, sm_scale,
                                  window, out_eps, reinterpret_cast<int*>(workspace), stream);
}

// ------------------------------------------------------------------- RoPE + append
int okc_rope_kv_append_ex(const void* qkv, int ldqkv, const int64_t* positions, const int32_t* page_table,
                          int table_ld, int max_pages, const float* inv_freq, const float* k_scale,
                          const float* v_scale, void* q_out, void* k_cache, void* v_cache, int64_t* slots_out,
                          int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages, float q_scale,
                          int qk_norm, float norm_eps, void* workspace, size_t workspace_bytes,
                          okc_stream_t stream) {
  if (!qkv || !positions || !page_table || !k_scale || !v_scale || !q_out || !k_cache || !v_cache)
    return OKC_ERR_INVALID;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2 || page_size <= 0 || num_pages <= 0 ||
      max_pages <= 0 || (table_ld != 0 && table_ld < max_pages) || table_ld < 0 || ldqkv < (Hq + 2 * Hkv) * D ||
      ldqkv % 8 || D % 8 || D > 512)
    return OKC_ERR_INVALID;
  if (qk_norm && (D > 256 || (D & (D - 1)))) return OKC_ERR_INVALID;  // a head's lanes fit one warp
  if (!aligned16(qkv) || !aligned16(q_out) || (reinterpret_cast<uintptr_t>(k_cache) & 7) ||
      (reinterpret_cast<uintptr_t>(v_cache) & 7))
    return OKC_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < 256) return OKC_ERR_WORKSPACE;
  return okc::launch_rope_append(qkv, ldqkv, positions, page_table, table_ld, max_pages, inv_freq, k_scale,
                                 v_scale, q_out, k_cache, v_cache, slots_out, B, Hq, Hkv, D, page_size,
                                 num_pages, q_scale, qk_norm, norm_eps, reinterpret_cast<int*>(workspace),
                                 stream);
}

int okc_rope_kv_append(const void* qkv, int ldqkv, const int64_t* positions, const int32_t* page_table,
                       int table_ld, int max_pages, const float* inv_freq, const float* k_scale,
                       const float* v_scale, void* q_out, void* k_cache, void* v_cache,
                       int64_t* slots_out, int B, int Hq, int Hkv, int D, int page_size,
                       int64_t num_pages, void* workspace, size_t workspace_bytes,
                       okc_stream_t stream) {
  return okc_rope_kv_append_ex(qkv, ldqkv, positions, page_table, table_ld, max_pages, inv_freq, k_scale,
                               v_scale, q_out, k_cache, v_cache, slots_out, B, Hq, Hkv, D, page_size, num_pages,
                               1.0f, 0, 0.0f, workspace, workspace_bytes, stream);
}

int okc_gemm_bf16_rope_kv_append(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                                 const int64_t* positions, const int32_t* page_table, int table_ld,
                                 int max_pages, const float* inv_freq, const float* k_scale,
                                 const float* v_scale, void* q_out, void* k_cache, void* v_cache,
                                 int64_t* slots_out, int Hq, int Hkv, int D, int page_size,
                                 int64_t num_pages, float q_scale, void* workspace, size_t workspace_bytes,
                                 okc_stream_t stream) {
  if (!x || !w || !positions || !page_table || !k_scale || !v_scale || !q_out || !k_cache || !v_cache)
    return OKC_ERR_INVALID;
  if (M <= 0 || M > 256 || K <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 8 || D > 512 || page_size <= 0 ||
      num_pages <= 0 || table_ld <= 0 || max_pages <= 0 || N != (Hq + 2 * Hkv) * D)
    return OKC_ERR_INVALID;
  if (K % 8 || ldx % 8 || ldw % 8 || ldx < K || ldw < K) return OKC_ERR_INVALID;
  if (!okc::tc_gemm_supported(M, N, K, ldx, ldw)) return OKC_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w) || (reinterpret_cast<uintptr_t>(q_out) & 7) ||
      (reinterpret_cast<uintptr_t>(k_cache) & 3) || (reinterpret_cast<uintptr_t>(v_cache) & 3))
    return OKC_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < okc_gemm_bf16_workspace_bytes(M, N, K)) return OKC_ERR_WORKSPACE;
  okc::TcRopeArgs r;
  r.positions = positions;
  r.page_table = page_table;
  r.table_ld = table_ld;
  r.max_pages = max_pages;
  r.inv_freq = inv_freq;
  r.k_scale = k_scale;
  r.v_scale = v_scale;
  r.q_out = q_out;
  r.k_cache = k_cache;
  r.v_cache = v_cache;
  r.slots_out = slots_out;
  r.Hq = Hq;
  r.Hkv = Hkv;
  r.D = D;
  r.P = page_size;
  r.num_pages = num_pages;
  r.q_scale = q_scale;
  // y is not written (every output goes through the epilogue); pass the q buffer as a
  // placeholder with a row stride of N.
  return okc::launch_tc_gemm(x, ldx, w, ldw, q_out, N, nullptr, M, N, K, 0,
                             reinterpret_cast<uint8_t*>(workspace) + 256, workspace_bytes - 256, stream, &r);
}

// ------------------------------------------------------------------------ attention
// Workspace of the decode kernels: [error word | (m, l) partials | output partials | unit
// prefix | two-term e4m3 queries + scales].

size_t okc_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int num_ctas) {
  if (num_ctas <= 0) num_ctas = okc_host::num_sms();
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0) return 0;
  const size_t nsub = Hkv >= 8 ? 1 : 8 / Hkv;
  const size_t rows = (size_t)(num_ctas + B) * nsub * Hq;
  return 256 + ((rows * 2 * 4 + 255) / 256) * 256 + ((rows * D * 4 + 255) / 256) * 256 +
         (((size_t)B + 1) * 4 + 255) / 256 * 256 + (okc::attn_q8_ws_bytes(B, Hkv) + 255) / 256 * 256;
}

int okc_attn_decode_fp8_ex(const void* q, int ldq, const void* k_cache, const void* v_cache,
                           const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                           const float* k_scale, const float* v_scale, void* out, int ldo, int B, int Hq,
                           int Hkv, int D, int page_size, int64_t num_pages, float sm_scale, int num_ctas,
                           int window, int q_per_seq, const void* gate, int ld_gate, float out_eps,
                           void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  if (gate && (ld_gate < Hq * D || (reinterpret_cast<uintptr_t>(gate) & 1))) return OKC_ERR_INVALID;
  if (!q || !k_cache || !v_cache || !page_table || !seq_lens || !k_scale || !v_scale || !out)
    return OKC_ERR_INVALID;
  if (B <= 0 || B > 4096 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8 || table_ld <= 0 || num_pages <= 0)
    return OKC_ERR_INVALID;
  if (window < 0 || q_per_seq <= 0 || B % q_per_seq) return OKC_ERR_INVALID;
  if (!(D == 64 || D == 128) || !(Hkv == 1 || Hkv == 2 || Hkv == 4 || Hkv == 8)) return OKC_ERR_INVALID;
  if (page_size <= 0 || !((32 % page_size) == 0 || (page_size % 32) == 0)) return OKC_ERR_INVALID;
  if (ldq % 8 || ldo % 8 || ldq < Hq * D || ldo < Hq * D) return OKC_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return OKC_ERR_ALIGNMENT;
  if (num_ctas <= 0) num_ctas = okc_host::num_sms();
  const size_t need = okc_attn_decode_workspace_bytes(B, Hq, Hkv, D, num_ctas);
  if (!workspace || workspace_bytes < need) return OKC_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return OKC_ERR_ALIGNMENT;
  const size_t nsub = Hkv >= 8 ? 1 : 8 / Hkv;
  const size_t rows = (size_t)(num_ctas + B) * nsub * Hq;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  okc::AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.ldq = ldq;
  a.k_cache = reinterpret_cast<const uint8_t*>(k_cache);
  a.v_cache = reinterpret_cast<const uint8_t*>(v_cache);
  a.page_table = page_table;
  a.table_ld = table_ld;
  a.seq_lens = seq_lens;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.err = reinterpret_cast<int*>(ws);
  a.ws_ml = reinterpret_cast<float*>(ws + 256);
  a.ws_acc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.ws_ml) + ((rows * 2 * 4 + 255) / 256) * 256);
  a.ws_prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a.ws_acc) + ((rows * D * 4 + 255) / 256) * 256);
  a.ws_q8 = reinterpret_cast<uint8_t*>(a.ws_prefix) + (((size_t)B + 1) * 4 + 255) / 256 * 256;
  a.ws_qf = reinterpret_cast<float*>(a.ws_q8 + (size_t)B * Hkv * 2048);
  a.B = B;
  a.Hq = Hq;
  a.G = Hq / Hkv;
  a.P = page_size;
  a.num_pages = num_pages;
  a.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  a.num_ctas = num_ctas;
  a.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  a.ld_gate = ld_gate;
  a.out_eps = out_eps;
  a.window = window;
  a.q_per_seq = q_per_seq;
  a.g4_rpp = 0;
  a.g4_rb = 0;
  return okc::launch_attn_decode(a, D, Hkv, stream);
}

int okc_attn_decode_fp8_gated(const void* q, int ldq, const void* k_cache, const void* v_cache,
                              const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                              const float* k_scale, const float* v_scale, void* out, int ldo, int B, int Hq,
                              int Hkv, int D, int page_size, int64_t num_pages, float sm_scale, int num_ctas,
                              const void* gate, int ld_gate, float out_eps, void* workspace,
                              size_t workspace_bytes, okc_stream_t stream) {
  return okc_attn_decode_fp8_ex(q, ldq, k_cache, v_cache, page_table, table_ld, seq_lens, k_scale, v_scale, out,
                                ldo, B, Hq, Hkv, D, page_size, num_pages, sm_scale, num_ctas, 0, 1, gate, ld_gate,
                                out_eps, workspace, workspace_bytes, stream);
}

int okc_attn_decode_fp8(const void* q, int ldq, const void* k_cache, const void* v_cache,
                        const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                        const float* k_scale, const float* v_scale, void* out, int ldo, int B, int Hq,
                        int Hkv, int D, int page_size, int64_t num_pages, float sm_scale, int num_ctas,
                        void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  return okc_attn_decode_fp8_gated(q, ldq, k_cache, v_cache, page_table, table_ld, seq_lens, k_scale, v_scale,
                                   out, ldo, B, Hq, Hkv, D, page_size, num_pages, sm_scale, num_ctas, nullptr, 0,
                                   0.0f, workspace, workspace_bytes, stream);
}

// ------------------------------------------------------------------------------ MoE
int okc_moe_route(const void* x, const void* wr, int32_t* ids, float* weights, float* logits_out, int T,
                  int H, int E, int topk, int renormalize, okc_stream_t stream) {
  if (!x || !wr || !ids || !weights || T <= 0 || H <= 0 || H % 256 || E <= 0 || E > 256 || topk <= 0 ||
      topk > 16 || topk > E)
    return OKC_ERR_INVALID;
  if (!aligned16(x) || !aligned16(wr)) return OKC_ERR_ALIGNMENT;
  return okc::launch_moe_route(x, wr, ids, weights, logits_out, T, H, E, topk, renormalize, stream);
}

int okc_moe_route_sigmoid(const float* logits, int ld, const float* logits_lo, const float* bias, int32_t* ids,
                          float* weights, float* logits_out, int T, int E, int topk, float logit_scale,
                          float score_eps, float route_scale, okc_stream_t stream) {
  if (!logits || !ids || !weights || T <= 0 || E <= 0 || E > 256 || topk <= 0 || topk > 32 || topk > E || ld < E)
    return OKC_ERR_INVALID;
  return okc::launch_route_sigmoid(logits, ld, logits_lo, bias, ids, weights, logits_out, T, E, topk, logit_scale,
                                   score_eps, route_scale, stream);
}

size_t okc_router_logits_workspace_bytes(int T, int E, int K) {
  return okc_gemm_bf16_workspace_bytes(T, 2 * E, K) + ((size_t)T * 2 * E * 4 + 255) / 256 * 256;
}

int okc_router_logits(const void* x, int ldx, const void* w_hilo, float* logits, int ldl, int T, int E, int K,
                      void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  if (!x || !w_hilo || !logits || T <= 0 || E <= 0 || K <= 0 || ldl < E) return OKC_ERR_INVALID;
  if (!workspace || workspace_bytes < okc_router_logits_workspace_bytes(T, E, K)) return OKC_ERR_WORKSPACE;
  const size_t gws = okc_gemm_bf16_workspace_bytes(T, 2 * E, K);
  float* y = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + gws);
  int st = okc_gemm_bf16_ex(x, ldx, w_hilo, K, y, 2 * E, nullptr, T, 2 * E, K, 1, 0, 0, workspace, gws, stream);
  if (st) return st;
  return okc::launch_add_halves(y, logits, ldl, T, E, stream);
}

int okc_moe_permute(const int32_t* ids, int T, int topk, int expert_lo, int E_local, int bm,
                    int32_t* counts, int32_t* offsets, int32_t* pairs, int32_t* tiles, int max_tiles,
                    okc_stream_t stream) {
  if (!ids || !counts || !offsets || !pairs || !tiles || T <= 0 || topk <= 0 || E_local <= 0 ||
      E_local > 256 || bm <= 0 || max_tiles < 0 || (long long)T * topk > 16384)
    return OKC_ERR_INVALID;
  // tiles[0] is clamped to max_tiles; a caller that sizes max_tiles as
  // min(E_local, T*topk) + ceil(T*topk / bm) can never overflow the table.
  return okc::launch_moe_permute(ids, T * topk, expert_lo, E_local, bm, counts, offsets, pairs, tiles,
                                 max_tiles, nullptr, stream);
}

size_t okc_moe_experts_workspace_bytes(int T, int topk, int H, int I) {
  return okc::moe_experts_ws_bytes(T, topk, H, I);
}

int okc_moe_experts_w4a16(const void* x, const int32_t* ids, const float* weights, const int32_t* counts,
                          const int32_t* offsets, const int32_t* pairs, const void* w13,
                          const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                          const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                          int E_local, void* workspace, size_t workspace_bytes, okc_stream_t stream) {
  return okc_moe_experts_w4a16_ex(x, ids, weights, counts, offsets, pairs, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs,
                                  out, T, topk, H, I, expert_lo, E_local, 0, workspace, workspace_bytes, stream);
}

int okc_moe_experts_w4a16_ex(const void* x, const int32_t* ids, const float* weights, const int32_t* counts,
                             const int32_t* offsets, const int32_t* pairs, const void* w13,
                             const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                             const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                             int E_local, int out_fp32, void* workspace, size_t workspace_bytes,
                             okc_stream_t stream) {
  return okc_moe_experts_w4a16_post(x, ids, weights, counts, offsets, pairs, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs,
                                    out, T, topk, H, I, expert_lo, E_local, out_fp32, nullptr, 0.0f, workspace,
                                    workspace_bytes, stream);
}

int okc_moe_experts_w4a16_post(const void* x, const int32_t* ids, const float* weights, const int32_t* counts,
                               const int32_t* offsets, const int32_t* pairs, const void* w13,
                               const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                               const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                               int E_local, int out_fp32, const float* post_gain, float post_eps, void* workspace,
                               size_t workspace_bytes, okc_stream_t stream) {
  if (post_gain && (H > 8192 || topk > 16)) return OKC_ERR_INVALID;
  if (post_gain && !aligned16(post_gain)) return OKC_ERR_ALIGNMENT;
  if (!x || !ids || !weights || !counts || !offsets || !pairs || !w13 || !w13_sf || !w13_gs || !w2 ||
      !w2_sf || !w2_gs || !out)
    return OKC_ERR_INVALID;
  if (T <= 0 || topk <= 0 || H % 256 || I % 128 || H <= 0 || I <= 0 || E_local <= 0) return OKC_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w13) || !aligned16(w2) || !aligned16(out)) return OKC_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < okc::moe_experts_ws_bytes(T, topk, H, I)) return OKC_ERR_WORKSPACE;
  return okc::launch_moe_experts(x, ids, weights, counts, offsets, pairs, w13, w13_sf, w13_gs, w2, w2_sf,
                                 w2_gs, out, T, topk, H, I, expert_lo, E_local, workspace, stream, out_fp32,
                                 post_gain, post_eps);
}


// ------------------------------------------------------------------ contract short names
int okc_gemv_bf16(const void* x, const void* w, void* y, int M, int N, int K, int ldw, void* scratch,
                  okc_stream_t stream) {
  if (!scratch) return OKC_ERR_WORKSPACE;
  return okc_gemm_bf16_ex(x, K, w, ldw, y, N, nullptr, M, N, K, 0, 0, 0, scratch,
                          okc_gemm_bf16_workspace_bytes(M, N, K), stream);
}

int okc_kv_append_rope(const void* qkv, int ldqkv, const int64_t* positions, const int32_t* page_table,
                       int table_ld, int max_pages, const float* inv_freq, const float* k_scale,
                       const float* v_scale, void* q_out, void* k_cache, void* v_cache, int64_t* slots_out,
                       int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages, void* workspace,
                       size_t workspace_bytes, okc_stream_t stream) {
  return okc_rope_kv_append(qkv, ldqkv, positions, page_table, table_ld, max_pages, inv_freq, k_scale, v_scale,
                            q_out, k_cache, v_cache, slots_out, B, Hq, Hkv, D, page_size, num_pages, workspace,
                            workspace_bytes, stream);
}

int okc_moe_w4a16(const void* x, const int32_t* ids, const float* weights, const int32_t* counts,
                  const int32_t* offsets, const int32_t* pairs, const void* w13, const void* w13_sf,
                  const float* w13_gs, const void* w2, const void* w2_sf, const float* w2_gs, void* out, int T,
                  int topk, int H, int I, int expert_lo, int E_local, void* workspace, size_t workspace_bytes,
                  okc_stream_t stream) {
  return okc_moe_experts_w4a16(x, ids, weights, counts, offsets, pairs, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs,
                               out, T, topk, H, I, expert_lo, E_local, workspace, workspace_bytes, stream);
}

int okc_rmsnorm(const void* x, const void* w, void* y, int T, int H, float eps, okc_stream_t stream) {
  return okc_rmsnorm_bf16(x, H, w, y, H, T, H, eps, 0, stream);
}

}  // extern "C"
