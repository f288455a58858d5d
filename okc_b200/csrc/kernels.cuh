// Internal launcher declarations shared by the entry points (capi.cu) and the kernels.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace okc {

struct AttnArgs {
  const __nv_bfloat16* q;
  int ldq;
  const uint8_t* k_cache;
  const uint8_t* v_cache;
  const int32_t* page_table;
  int table_ld;
  const int32_t* seq_lens;
  const float* k_scale;
  const float* v_scale;
  __nv_bfloat16* out;
  int ldo;
  float* ws_ml;   // [slots][NSUB][Hq][2]: running max (log2 units), running sum
  float* ws_acc;  // [slots][NSUB][Hq][D]: unnormalised output
  int* ws_prefix; // [B + 1]: unit prefix of the sequences (written by the attention kernel for the merge)
  int* err;
  int B, Hq, G, P;
  long long num_pages;
  float sm_scale_log2;
  int num_ctas;
  const __nv_bfloat16* gate;  // optional output gate (Muse): out = rms(o) * sigmoid(gate)
  int ld_gate;
  float out_eps;
  int window;     // sliding window in tokens (0: the whole context)
  int q_per_seq;  // query tokens per request (verify blocks): sequence b reads table row b / q_per_seq
  uint8_t* ws_q8; // [B][Hkv][16][128] two-term e4m3 queries (tcgen05 kernel)
  float* ws_qf;   // [B][Hkv][8] their per-row scales
  int g4_rpp;     // > 0: pages are fetched with TMA gather4 as this many rows each (mma.sync kernel)
  int g4_rb;      // the gather rows' bytes: 2048, or a whole page smaller than 2 KB
};
size_t attn_q8_ws_bytes(int B, int Hkv);

// cuTensorMapEncodeTiled from the driver (nullptr when unavailable); cached.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

int launch_skinny_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                       const void* residual, int M, int N, int K, int out_fp32, int splits,
                       cudaStream_t stream);
// RoPE + FP8 KV-append fused into the QKV projection's epilogue (tcgen05 path).
struct TcRopeArgs {
  const int64_t* positions;
  const int32_t* page_table;
  int table_ld, max_pages;
  const float* inv_freq;
  const float* k_scale;
  const float* v_scale;
  void* q_out;
  void* k_cache;
  void* v_cache;
  int64_t* slots_out;
  int Hq, Hkv, D, P;
  long long num_pages;
  float q_scale;
};
int launch_tc_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                   const void* residual, int M, int N, int K, int out_fp32, void* ws, size_t ws_bytes,
                   cudaStream_t stream, const TcRopeArgs* rope = nullptr);
size_t tc_gemm_ws_bytes(int M, int N, int K);
bool tc_gemm_supported(int M, int N, int K, int ldx, int ldw);
int launch_rmsnorm(const void* x, int ldx, const void* w, void* y, int ldy, int T, int H, float eps,
                   int unit_offset, cudaStream_t stream);
int launch_residual_boundary(const float* stream_in, const void* branch, int ldb, const float* alpha,
                             const float* beta, const void* post_w, const void* pre_w, void* hidden,
                             float* stream_out, float* router_out, int T, int H, float post_eps, float pre_eps,
                             cudaStream_t stream);
int launch_attn_decode(AttnArgs& a, int D, int Hkv, cudaStream_t stream);
int launch_attn_prefill(const void* q, int ldq, const void* k_cache, const void* v_cache, const int32_t* page_table,
                        int table_ld, int max_pages, const int64_t* positions, const float* k_scale,
                        const float* v_scale, const void* gate, int ld_gate, void* out, int ldo, int B, int L, int Hq,
                        int Hkv, int D, int page_size, long long num_pages, float sm_scale, int window, float out_eps,
                        int* err, cudaStream_t stream);
int launch_rope_append(const void* qkv, int ldqkv, const int64_t* positions,
                       const int32_t* page_table, int table_ld, int max_pages, const float* inv_freq,
                       const float* k_scale, const float* v_scale, void* q_out, void* k_cache,
                       void* v_cache, int64_t* slots_out, int B, int Hq, int Hkv, int D, int P,
                       long long num_pages, float q_scale, int qk_norm, float norm_eps, int* err,
                       cudaStream_t stream);
int launch_moe_route(const void* x, const void* wr, int32_t* ids, float* wts, float* logits, int T,
                     int H, int E, int topk, int renormalize, cudaStream_t stream);
int launch_moe_permute(const int32_t* ids, int n, int expert_lo, int E, int bm, int32_t* counts,
                       int32_t* offsets, int32_t* pairs, int32_t* tiles, int max_tiles, int* err,
                       cudaStream_t stream);
size_t moe_experts_ws_bytes(int T, int topk, int H, int I);
int launch_route_sigmoid(const float* logits, int ld, const float* lo, const float* bias, int32_t* ids, float* wts,
                         float* logits_out, int T, int E, int topk, float scale, float eps, float route_scale,
                         cudaStream_t stream);
int launch_add_halves(const float* y, float* out, int ldo, int T, int E, cudaStream_t stream);
bool moe_tc_ok(int H, int I, int E);
int launch_moe_rows_f16(const void* src, const int32_t* pairs, const int32_t* offsets, int E, int topk, int K,
                        int max_rows, __half* dst, float* rs, cudaStream_t stream);
template <bool GATED>
int launch_moe_tc(const void* w, const void* sf, int E, const __half* act, int rows, const float* rs,
                  const int32_t* counts, const int32_t* offsets, const int32_t* pairs, const float* gs,
                  __nv_bfloat16* inter, __nv_bfloat16* y, int K, int NR, int I, int* err, cudaStream_t stream);
int launch_moe_experts(const void* x, const int32_t* ids, const float* wts, const int32_t* counts,
                       const int32_t* offsets, const int32_t* pairs, const void* w13,
                       const void* w13_sf, const float* w13_gs, const void* w2, const void* w2_sf,
                       const float* w2_gs, void* out, int T, int topk, int H, int I, int expert_lo,
                       int E, void* ws, cudaStream_t stream, int out_fp32 = 0,
                       const float* post_gain = nullptr, float post_eps = 1e-8f);

}  // namespace okc
