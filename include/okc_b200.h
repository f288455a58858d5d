/*
 * okc_b200 — C ABI of the B200 (sm_100a) decode-step kernels.
 *
 * Every entry point takes raw device pointers, explicit sizes and a CUDA stream,
 * enqueues its kernels on that stream and returns at once (no host synchronisation,
 * so every call can be captured in a CUDA graph).  Return value: OKC_OK or a negative
 * OKC_ERR_* code; a call that returns an error enqueued nothing that writes outputs.
 * No entry point allocates memory: scratch ("workspace") is passed in by the caller,
 * sized by the matching *_workspace_bytes() query, and must be zero-filled once
 * before its first use (it keeps its own state self-consistent across calls).
 *
 * Device-side errors (a bad page id, a device wait that timed out) cannot be
 * returned synchronously; kernels OR an OKC_DEVERR_* bit into the 32-bit error word
 * at the start of the workspace.  okc_read_device_error() reads and clears it.
 *
 * Tensor layouts are row-major and dense unless a leading dimension says otherwise.
 * Element types: bf16 = IEEE bfloat16, e4m3 = OCP FP8 E4M3 (float8_e4m3fn),
 * e2m1 = OCP FP4 E2M1 packed two per byte (low nibble = even element).
 */
#ifndef OKC_B200_H
#define OKC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* okc_stream_t; /* == cudaStream_t */

enum {
  OKC_OK = 0,
  OKC_ERR_INVALID = -1,     /* bad size, null pointer or unsupported shape */
  OKC_ERR_ALIGNMENT = -2,   /* a pointer or leading dimension breaks 16-byte alignment */
  OKC_ERR_WORKSPACE = -3,   /* workspace too small */
  OKC_ERR_LAUNCH = -4,      /* the CUDA launch itself failed */
  OKC_ERR_DEVICE = -5,      /* no sm_100 device / kernel image */
  OKC_ERR_TOO_LARGE = -6,   /* the request needs more than the fixed scratch of a no-alloc entry point */
};

enum {
  OKC_DEVERR_TIMEOUT = 1,   /* a bounded device wait (mbarrier) gave up */
  OKC_DEVERR_PAGE = 2,      /* a page-table entry outside [0, num_pages) was skipped */
  OKC_DEVERR_INDEX = 4,     /* an expert id or slot outside its range was skipped */
};

/* Library version string, e.g. "okc_b200 0.1 sm_100a". */
const char* okc_version(void);

/* Reads the device error word at the start of `workspace` (synchronises `stream`),
 * clears it, and returns it (0 = no error, else OKC_DEVERR_* bits; <0 = CUDA error). */
int okc_read_device_error(const void* workspace, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Projection: y[M,N] = x[M,K] · W[N,K]^T (+ residual[M,N]), bf16 in, fp32 accumulate.
 * Replaces the projection dispatch of muse_decode_layer/decode/projections.py:50-77
 * (`_project`: M=1 `_gemv` :8-15, split-K `_small_gemm` :18-39 + `_reduce_projection`
 * :42-48) and muse_bf16_proj/projection/runtime.py:80-220 (`run_config`).
 * Picks the split-K skinny kernel (M <= 32, cluster/DSMEM split-K reduction) or the
 * tcgen05 kernel (M >= 33) itself; M > 256 (prefill) runs as 256-row blocks of the tcgen05
 * kernel (the workspace covers one block).  out_fp32 != 0 writes fp32 y (a row-parallel partial
 * that an all-reduce sums), else bf16.  residual (bf16, may be NULL) is added to the
 * fp32 accumulator before the single rounding.  K must be a multiple of 8, ldx/ldw
 * multiples of 8 elements, x and w 16-byte aligned (y and residual element-aligned).
 * ---------------------------------------------------------------------------------- */
size_t okc_gemm_bf16_workspace_bytes(int M, int N, int K);
int okc_gemm_bf16(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                  const void* residual, int M, int N, int K, int out_fp32,
                  void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* Forces one kernel family (0 = auto, 1 = skinny split-K, 2 = tcgen05) and, for the
 * skinny family, a split count (0 = auto).  Exposed for tests and tuning sweeps. */
int okc_gemm_bf16_ex(const void* x, int ldx, const void* w, int ldw, void* y, int ldy,
                     const void* residual, int M, int N, int K, int out_fp32,
                     int family, int splits,
                     void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * RMSNorm: y[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * g), g = w or (1 + w).
 * Replaces `_norm` muse_decode_layer/decode/boundaries.py:8-14 and `rms`/`gain`
 * muse_prefill_layer/submission.py:89-96.  x bf16 [T,H] (ldx), w bf16 [H], H <= 16384.
 * ---------------------------------------------------------------------------------- */
int okc_rmsnorm_bf16(const void* x, int ldx, const void* w, void* y, int ldy, int T, int H,
                     float eps, int unit_offset, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Gated residual boundary between a layer's branches.  Replaces `_boundary` /
 * `_residual_boundary` of muse_decode_layer/decode/boundaries.py:17-50 (the stream update of
 * muse_prefill_layer/submission.py:205-215).  Per row t:
 *   b       = branch[t] (bf16, row stride ld_branch); with post_w != NULL first
 *             b = bf16(b * (1 + post_w))  (the final, post-FFN boundary);
 *   b       = b * rsqrt(mean(b^2) + post_eps)                    (the reference: 1e-8);
 *   stream' = alpha * stream_in[t] + beta * b                    (fp32, stream_out[t]);
 *   hidden  = bf16(stream' * rsqrt(mean(stream'^2) + pre_eps) * (1 + pre_w))  (1e-5);
 *   router_out[t] = the same hidden unrounded, fp32 (skipped when router_out is NULL).
 * stream fp32 [T,H] contiguous (stream_out may equal stream_in), alpha/beta fp32 [H], post_w /
 * pre_w bf16 [H], hidden bf16 [T,H]; H % 8 == 0, H <= 16384, every pointer 16-byte aligned.
 * Each product and sum is rounded on its own (no fused multiply-add), as the reference
 * compiles it.
 * ---------------------------------------------------------------------------------- */
int okc_residual_boundary(const float* stream_in, const void* branch, int ld_branch,
                          const float* alpha, const float* beta, const void* post_w,
                          const void* pre_w, void* hidden, float* stream_out, float* router_out,
                          int T, int H, float post_eps, float pre_eps, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * QKV projection with the RoPE + FP8 KV-append fused into its epilogue (the tcgen05 path,
 * M <= 256): qkv = x · W^T (fp32 accumulate, rounded to bf16 as the unfused path does), then
 * exactly okc_rope_kv_append_ex's arithmetic with qk_norm = 0: q (rotated, x q_scale) to
 * bf16 q_out [M][Hq][D], k (rotated) and v quantised e4m3 into k_cache / v_cache at
 * slot = page_table[m][pos/P]*P + pos%P, slots_out[m] (may be NULL).  N = (Hq + 2 Hkv) * D,
 * D % 8 == 0.  The bf16 qkv never goes to memory.  Workspace as okc_gemm_bf16_workspace_bytes.
 * Replaces the QKV projection + `_qkv_norm_store` pair of muse_decode_layer/decode/
 * projections.py:75-77 and decode/attention.py:13-37 for the plain (no QK-norm) layer.
 * ---------------------------------------------------------------------------------- */
int okc_gemm_bf16_rope_kv_append(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                                 const int64_t* positions, const int32_t* page_table, int table_ld,
                                 int max_pages, const float* inv_freq, const float* k_scale,
                                 const float* v_scale, void* q_out, void* k_cache, void* v_cache,
                                 int64_t* slots_out, int Hq, int Hkv, int D, int page_size,
                                 int64_t num_pages, float q_scale, void* workspace, size_t workspace_bytes,
                                 okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * RoPE + FP8 KV-append (one decode token per sequence, q_len = 1).
 * Replaces `_qkv_norm_store` muse_decode_layer/decode/attention.py:13-37, the append of
 * muse_attention_decode/submission.py:283-305 and the cache write of
 * muse_prefill_layer/submission.py:155-156.
 * qkv: bf16 [B, ldqkv] holding q (Hq*D) | k (Hkv*D) | v (Hkv*D) per row.
 * positions: int64 [B] (the new token's position = cached length).  page_table int32
 * [B, max_pages] (ld = table_ld; table_ld 0: every row reads table row 0, e.g. a block of
 * one request's tokens).  Slot = page_table[b][pos / P] * P + pos % P.
 * Writes q_out bf16 [B, Hq, D] (rotated), k_cache/v_cache e4m3 [num_pages, P, Hkv, D] at
 * the slot (k rotated, / k_scale[h]; v / v_scale[h]; RNE, overflow -> NaN like torch),
 * and slots_out int64 [B] (may be NULL).  inv_freq fp32 [D/2] (NULL = no RoPE).  D % 8 == 0,
 * D <= 512, ldqkv % 8 == 0, qkv / q_out 16-byte aligned, caches 8-byte aligned.
 * ---------------------------------------------------------------------------------- */
int okc_rope_kv_append(const void* qkv, int ldqkv, const int64_t* positions,
                       const int32_t* page_table, int table_ld, int max_pages,
                       const float* inv_freq, const float* k_scale, const float* v_scale,
                       void* q_out, void* k_cache, void* v_cache, int64_t* slots_out,
                       int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                       void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* okc_rope_kv_append plus Muse's query/key treatment (the reference problem's own semantics,
 * muse_prefill_layer/submission.py:141-147 and muse_attention_decode/submission.py:57-69,252-257):
 * qk_norm != 0 applies a per-head RMSNorm without weight (eps norm_eps) to q and k before RoPE,
 * and q is multiplied by q_scale (the qk_scale_factor) before its bf16 rounding.  With
 * q_scale = 1, qk_norm = 0 it is okc_rope_kv_append.  qk_norm needs D a power of two <= 256. */
int okc_rope_kv_append_ex(const void* qkv, int ldqkv, const int64_t* positions,
                          const int32_t* page_table, int table_ld, int max_pages,
                          const float* inv_freq, const float* k_scale, const float* v_scale,
                          void* q_out, void* k_cache, void* v_cache, int64_t* slots_out,
                          int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                          float q_scale, int qk_norm, float norm_eps,
                          void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Paged FP8 attention for prefill blocks: B requests of L new tokens each (rows b*L .. b*L+L-1
 * of q / positions / out, their K/V already appended), each token attending the positions
 * p <= its own (and p > own - window when window > 0) of its request's cache.  Replaces
 * `attention` of muse_prefill_layer/submission.py:137-176 for q_len 200-16384 (after its
 * cache write): q bf16 [B*L][ldq] (Hq heads of D, the scaled and rounded queries), caches e4m3
 * [num_pages, P, Hkv, D] with per-head fp32 scales, page_table int32 [B][table_ld] (max_pages
 * valid columns), positions int64 [B*L].  out bf16 [B*L][ldo] = softmax(q k^T * sm_scale) v,
 * or with gate (bf16 [B*L][ld_gate], may be NULL) rms(o) * sigmoid(gate) per head (eps out_eps).
 * D 64 or 128, Hq / Hkv <= 8.  Workspace >= 256 bytes, its first int the device error word
 * (OKC_DEVERR_PAGE for a page id outside the pool; those positions read zeros).
 * ---------------------------------------------------------------------------------- */
int okc_attn_prefill_fp8(const void* q, int ldq, const void* k_cache, const void* v_cache,
                         const int32_t* page_table, int table_ld, int max_pages, const int64_t* positions,
                         const float* k_scale, const float* v_scale, const void* gate, int ld_gate,
                         float out_eps, void* out, int ldo, int B, int L, int Hq, int Hkv, int D,
                         int page_size, int64_t num_pages, float sm_scale, int window,
                         void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Paged FP8 attention decode (q_len = 1), split-KV with a log-sum-exp merge.
 * Replaces `_fused_attn` muse_attention_decode/submission.py:191-351 (its cached-context
 * splits and two-level merge), `_attention_parts`/`_attention_finish`
 * muse_decode_layer/decode/attention.py:40-113, and the attention of
 * muse_prefill_layer/submission.py:158-176 (GQA grouping q.view(B, Hkv, G, D)).
 * q bf16 [B, Hq, D] (ldq = row stride in elements); caches e4m3 [num_pages, P, Hkv, D];
 * page_table int32 [B, table_ld]; seq_lens int32 [B] = keys to attend per sequence;
 * k_scale/v_scale fp32 [Hkv]; out bf16 [B, Hq, D] (ldo).  out = softmax(q·K^T * sm_scale)
 * · V with K = e4m3 * k_scale[h], V = e4m3 * v_scale[h].  Supported: D in {64, 128},
 * Hkv in {1, 2, 4, 8}, G = Hq/Hkv <= 8, P dividing 32 or a multiple of 32.
 * ---------------------------------------------------------------------------------- */
size_t okc_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int num_ctas);
int okc_attn_decode_fp8(const void* q, int ldq, const void* k_cache, const void* v_cache,
                        const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                        const float* k_scale, const float* v_scale, void* out, int ldo,
                        int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                        float sm_scale, int num_ctas,
                        void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* okc_attn_decode_fp8 followed by Muse's output gate (muse_prefill_layer/submission.py:176;
 * `_epilogue` muse_attention_decode/submission.py:366-383): out = bf16(rms(o) * sigmoid(gate))
 * with a per-head RMSNorm of the fp32 attention output o (eps out_eps).  gate bf16 [B, Hq*D]
 * with row stride ld_gate (the gate columns of the fused projection output).  gate = NULL
 * gives okc_attn_decode_fp8. */
int okc_attn_decode_fp8_gated(const void* q, int ldq, const void* k_cache, const void* v_cache,
                              const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                              const float* k_scale, const float* v_scale, void* out, int ldo,
                              int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                              float sm_scale, int num_ctas, const void* gate, int ld_gate,
                              float out_eps, void* workspace, size_t workspace_bytes,
                              okc_stream_t stream);

/* okc_attn_decode_fp8_gated with Muse's sliding-window layers and speculative-verify blocks
 * (muse_attention_decode/submission.py:191-351, 409-439; the mask of
 * muse_prefill_layer/submission.py:169-171): a query at position p attends the cached
 * positions (p - window, p] (window = 0: [0, p]).  A verify block of q_per_seq query tokens per
 * request is passed as q_per_seq consecutive rows of q / out / seq_lens per request, row i
 * of request r having seq_lens = (its position + 1) and reading page-table row r (so B is
 * requests * q_per_seq and page_table has B / q_per_seq rows).  window = 0 and q_per_seq = 1
 * give okc_attn_decode_fp8_gated. */
int okc_attn_decode_fp8_ex(const void* q, int ldq, const void* k_cache, const void* v_cache,
                           const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                           const float* k_scale, const float* v_scale, void* out, int ldo,
                           int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                           float sm_scale, int num_ctas, int window, int q_per_seq,
                           const void* gate, int ld_gate, float out_eps,
                           void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* Same computation as okc_attn_decode_fp8, for callers that cannot allocate device memory
 * (no counterpart in the reference, whose operators allocate their scratch per call).  The
 * split-KV partials live in a fixed 16 MiB array inside the library, so the caller passes only
 * inputs and outputs.  A request whose partials need more than that (okc_attn_decode_workspace_
 * bytes(B, Hq, Hkv, D, num_ctas) > 16 MiB) returns OKC_ERR_TOO_LARGE.  The array is shared by
 * every call on a device and keeps the last call's contents: calls that may overlap on the GPU
 * (streams without ordering between them) race and must not be issued.  The first call on each
 * device looks up the array's device address (with that device current); make it before any
 * stream capture.  Device-side problems (a page id outside [0, num_pages) is skipped, not
 * read) OR their OKC_DEVERR_* bits into an error word kept beside the array, which collects
 * every call's bits until okc_attn_decode_fp8_noalloc_error() reads and clears it. */
int okc_attn_decode_fp8_noalloc(const void* q, int ldq, const void* k_cache, const void* v_cache,
                                const int32_t* page_table, int table_ld, const int32_t* seq_lens,
                                const float* k_scale, const float* v_scale, void* out, int ldo,
                                int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                                float sm_scale, int num_ctas, okc_stream_t stream);

/* Reads and clears the device error word of okc_attn_decode_fp8_noalloc on the current device
 * once the work enqueued on `stream` is done (synchronises the stream; allocates nothing).
 * Returns 0 (no error) or OKC_DEVERR_* bits, or a negative OKC_ERR_* code.  Like the entry
 * point it belongs to, it has no counterpart in the reference. */
int okc_attn_decode_fp8_noalloc_error(okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * MoE routing: logits = bf16(x · Wr^T) (fp32 sums in a fixed order: lane l of a warp sums
 * elements 256j + 8l + i over j then i, then an xor butterfly over the 32 lanes, so
 * the logits are reproducible bit for bit on the CPU),
 * ids = top-k of the logits (ties -> lower expert id), weights = softmax over the
 * chosen logits (renormalize != 0) or the full-softmax probabilities of the chosen
 * experts (renormalize == 0).  x bf16 [T,H], wr bf16 [E,H]; ids int32 [T,k];
 * weights fp32 [T,k]; logits_out fp32 [T,E] (may be NULL).  E <= 256, k <= 16.
 * Replaces `route` muse_prefill_layer/submission.py:179-184 and the routing call of
 * muse_decode_layer/decode/runtime.py:55-63 (softmax top-k of the bf16 logits).
 * ---------------------------------------------------------------------------------- */
/* ------------------------------------------------------------------------------------
 * Muse routing: score = sigmoid((logits[t][e] (+ logits_lo[t][e] when given)) * logit_scale),
 * ids = top-k of score + bias[e] (bias may be NULL; it only chooses; ties -> lower id),
 * weights = score / (sum of the chosen scores + score_eps) * route_scale.  logits fp32 [T][ld];
 * logits_out fp32 [T][E] (the summed logits; may be NULL).  E <= 256, topk <= 32.  Replaces
 * `route` of muse_prefill_layer/submission.py:179-184 and FusedMuseSparkRouting as
 * muse_decode_layer/decode/runtime.py:30-32,63 configures it (logit_scale 0.1767766952966369,
 * score_eps 1e-15, route_scale 1).
 * ---------------------------------------------------------------------------------- */
int okc_moe_route_sigmoid(const float* logits, int ld, const float* logits_lo, const float* bias,
                          int32_t* ids, float* weights, float* logits_out, int T, int E, int topk,
                          float logit_scale, float score_eps, float route_scale, okc_stream_t stream);

/* FP32 router projection through bf16 halves: w_hilo bf16 [2E][K] holds hi = bf16(router) in
 * rows 0..E-1 and lo = bf16(router - hi) in rows E..2E-1 (the reference's prepare,
 * muse_bf16_proj/projection/runtime.py:42-47); logits[t][e] = x·hi[e] + x·lo[e], two
 * independent fp32 accumulations summed at the end (`_gemm` ROUTER,
 * muse_bf16_proj/projection/kernels/gemm.py:8-39).  x bf16 [T][ldx]; logits fp32 [T][ldl]. */
size_t okc_router_logits_workspace_bytes(int T, int E, int K);
int okc_router_logits(const void* x, int ldx, const void* w_hilo, float* logits, int ldl, int T, int E,
                      int K, void* workspace, size_t workspace_bytes, okc_stream_t stream);

int okc_moe_route(const void* x, const void* wr, int32_t* ids, float* weights,
                  float* logits_out, int T, int H, int E, int topk, int renormalize,
                  okc_stream_t stream);

/* Token permutation: per expert, the pair ids p = t*topk + slot routed to it, ascending.
 * Replaces `_route` muse_moe_w4a16/submission.py:274-291 and `moe_align_block_size`
 * (muse_decode_layer/decode/experts.py:80).  ids int32 [T*topk] (values outside
 * [expert_lo, expert_lo + E_local) are not local and are skipped).  Outputs:
 * counts int32 [E_local], offsets int32 [E_local + 1] (exclusive prefix of counts),
 * pairs int32 [T*topk] (expert-major, ascending p inside each expert),
 * tiles int32 [1 + max_tiles]: tiles[0] = number of (expert, first row) tiles of `bm`
 * pairs, then (expert << 16 | first) per tile.  T*topk <= 65536. */
int okc_moe_permute(const int32_t* ids, int T, int topk, int expert_lo, int E_local, int bm,
                    int32_t* counts, int32_t* offsets, int32_t* pairs, int32_t* tiles,
                    int max_tiles, okc_stream_t stream);

/* W4A16 experts: for each local expert e and each pair p routed to it,
 *   h = x[p / topk] · W13[e]^T  (W13 e2m1 [E, 2I, H/2], sf e4m3 [E, 2I, H/16], gs fp32 [E])
 *   inter[p] = bf16( silu(bf16(h[:I])) * bf16(h[I:]) )
 *   y[p] = bf16( inter[p] · W2[e]^T )  (W2 e2m1 [E, H, I/2], sf [E, H, I/16], gs [E])
 * and out[t] = bf16( sum_slot weights[t, slot] * y[t*topk + slot] ) over local slots.
 * Weight element = e2m1 * sf (exact in bf16) with gs applied to the fp32 accumulator.
 * Replaces `_expert_gemm` + `_finalize` muse_moe_w4a16/submission.py:163-308 and
 * `_nvfp4_gate_up`/`_nvfp4_down` muse_decode_layer/decode/nvfp4_gemv.py:21-75.
 * Needs the okc_moe_permute outputs.  inter/y are scratch inside `workspace`.
 * H multiple of 256, I multiple of 128. */
size_t okc_moe_experts_workspace_bytes(int T, int topk, int H, int I);
int okc_moe_experts_w4a16(const void* x, const int32_t* ids, const float* weights,
                          const int32_t* counts, const int32_t* offsets, const int32_t* pairs,
                          const void* w13, const void* w13_sf, const float* w13_gs,
                          const void* w2, const void* w2_sf, const float* w2_gs,
                          void* out, int T, int topk, int H, int I, int expert_lo, int E_local,
                          void* workspace, size_t workspace_bytes, okc_stream_t stream);
/* Same, with out_fp32 != 0: out is fp32 [T,H] and holds this rank's unrounded share of the
 * sum (expert parallelism: the ranks' shares are summed by okc_tp_allreduce_residual). */
int okc_moe_experts_w4a16_ex(const void* x, const int32_t* ids, const float* weights,
                             const int32_t* counts, const int32_t* offsets, const int32_t* pairs,
                             const void* w13, const void* w13_sf, const float* w13_gs,
                             const void* w2, const void* w2_sf, const float* w2_gs,
                             void* out, int T, int topk, int H, int I, int expert_lo, int E_local,
                             int out_fp32, void* workspace, size_t workspace_bytes, okc_stream_t stream);

/* Same, with Muse's post-expert RMSNorm (`_finalize`, muse_moe_w4a16/submission.py:295-308):
 * with post_gain != NULL (fp32 [H] = 1 + post_norm_w, as the reference's prepare stores it)
 * each local slot is first scaled = bf16(y * post_gain) and normalised by
 * rsqrt(mean(scaled^2) + post_eps) (the reference: 1e-8), then weighted and summed.
 * post_gain needs H <= 8192 and topk <= 16; NULL gives okc_moe_experts_w4a16_ex. */
int okc_moe_experts_w4a16_post(const void* x, const int32_t* ids, const float* weights,
                               const int32_t* counts, const int32_t* offsets, const int32_t* pairs,
                               const void* w13, const void* w13_sf, const float* w13_gs,
                               const void* w2, const void* w2_sf, const float* w2_gs,
                               void* out, int T, int topk, int H, int I, int expert_lo, int E_local,
                               int out_fp32, const float* post_gain, float post_eps, void* workspace,
                               size_t workspace_bytes, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Tensor-parallel exchange over NVLink peer memory (multi-GPU layer step).  No reference
 * counterpart: the reference runs the layer on one GPU.  Replaces the NCCL all-reduce of the
 * row-parallel O-projection partials followed by the residual add (the multi-GPU contract
 * of the decode layer: column-parallel QKV, row-parallel O, all-reduce after O).
 *
 * okc_ipc_alloc / okc_ipc_free: a zero-filled device buffer of its own cudaMalloc
 * allocation (so that its IPC handle maps exactly that buffer).  okc_ipc_handle writes the
 * 64-byte cudaIpcMemHandle_t of such a buffer; okc_ipc_open maps a peer's handle (peer
 * access enabled lazily); okc_ipc_close unmaps it.
 *
 * okc_tp_allreduce_residual: out_r = bf16(residual + sum_q parts[q]) on every rank r
 * (residual may be NULL: out_r = bf16(sum_q parts[q])).
 * parts[q] (fp32 [n]), outs[q] (bf16 [n]) and flags[q] (int [OKC_TP_EXCHANGE_FLAG_WORDS],
 * zero-filled) are HOST arrays of `world` device pointers: this rank's own buffers at index
 * `rank`, the peers' mapped buffers elsewhere.  state: this rank's int [OKC_TP_STATE_WORDS]
 * (zero-filled), private to one exchange group and shared by its calls of both exchange
 * entry points.  Every rank calls it in the same order on its own stream.  Rank r sums
 * the r-th slice of the elements in rank order and stores it into every rank's output;
 * the call completes on a rank when all slices have arrived there.  Synchronisation is per
 * CTA (CTA c waits only for CTA c of the other ranks).  Flag waits are bounded (2 s): on
 * expiry OKC_DEVERR_TIMEOUT is set in the workspace error word.  The workspace holds at
 * least 4096 bytes (error word; optional phase trace at byte 256, OKC_TP_TRACE=1).
 * n multiple of 4; world 2..8; parts 16-byte aligned, outs and residual 8-byte aligned. */
#define OKC_TP_STATE_WORDS 1024
#define OKC_TP_EXCHANGE_FLAG_WORDS 8192
int okc_ipc_alloc(size_t bytes, void** ptr);
int okc_ipc_free(void* ptr);
int okc_ipc_handle(const void* ptr, void* handle_out);
int okc_ipc_open(const void* handle, void** ptr);
int okc_ipc_close(void* ptr);
int okc_tp_allreduce_residual(const float* const* parts, void* const* outs, int* const* flags,
                              const void* residual, int* state, int rank, int world,
                              long long n, void* workspace, okc_stream_t stream);

/* okc_tp_oproj_allreduce_residual: the row-parallel O projection fused with the exchange
 * above, in one tcgen05 kernel: out_r = bf16(residual + sum_q x_q · W_q^T) on every rank r,
 * x_q bf16 [M, K] (row stride ldx) and W_q bf16 [N, K] (row stride ldw) being rank q's
 * attention output and O-weight columns; out and residual bf16 [M, N] with row stride ldo.
 * Each CTA pair splits one 128-row weight tile's K range (partial sums meet in distributed
 * shared memory), pushes each token slice of the tile as fp32 into the owning rank's receive
 * buffer over NVLink, and the owner sums the ranks' slices in rank order, adds the residual
 * and stores bf16 into every rank's output.  recv[q], outs[q], flags[q] are HOST arrays of
 * `world` device pointers (own buffers at `rank`, mapped peer buffers elsewhere): recv of
 * okc_tp_oproj_plan's recv_bytes, flags of its flag_words ints (zero-filled, not shared with
 * okc_tp_allreduce_residual's flag words).  state: the exchange group's int
 * [OKC_TP_STATE_WORDS].  Same ordering, per-CTA synchronisation and timeout rules as
 * okc_tp_allreduce_residual.  M 1..128, N multiple of 8, K multiple of 8, world 2..8 with
 * 64 (M <= 64: 32) divisible by world; 16-byte aligned pointers.  OKC_ERR_INVALID when the
 * shape is outside that range or the grid cannot be co-resident on this GPU.
 * okc_tp_oproj_plan: OKC_OK and the buffer sizes when the shape is supported. */
int okc_tp_oproj_plan(int M, int N, int K, int world, size_t* recv_bytes, int* flag_words);
int okc_tp_oproj_allreduce_residual(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                                    float* const* recv, void* const* outs, int* const* flags,
                                    const void* residual, int ldo, int* state, int rank, int world,
                                    void* workspace, okc_stream_t stream);

/* ------------------------------------------------------------------------------------
 * The short names of the decode-path contract (the C-ABI list the drop-in boundary
 * names), as thin forms of the entry points above:
 *   okc_gemv_bf16       = okc_gemm_bf16 with contiguous x [M,K], W [N,K], y [M,N] (bf16,
 *                         no residual); `scratch` must hold okc_gemm_bf16_workspace_bytes(M,N,K)
 *                         bytes, zero-filled once;
 *   okc_kv_append_rope  = okc_rope_kv_append;
 *   okc_moe_w4a16       = okc_moe_experts_w4a16;
 *   okc_rmsnorm         = okc_rmsnorm_bf16 with plain weight (no unit offset).
 * ---------------------------------------------------------------------------------- */
int okc_gemv_bf16(const void* x, const void* w, void* y, int M, int N, int K, int ldw, void* scratch,
                  okc_stream_t stream);
int okc_kv_append_rope(const void* qkv, int ldqkv, const int64_t* positions,
                       const int32_t* page_table, int table_ld, int max_pages,
                       const float* inv_freq, const float* k_scale, const float* v_scale,
                       void* q_out, void* k_cache, void* v_cache, int64_t* slots_out,
                       int B, int Hq, int Hkv, int D, int page_size, int64_t num_pages,
                       void* workspace, size_t workspace_bytes, okc_stream_t stream);
int okc_moe_w4a16(const void* x, const int32_t* ids, const float* weights,
                  const int32_t* counts, const int32_t* offsets, const int32_t* pairs,
                  const void* w13, const void* w13_sf, const float* w13_gs,
                  const void* w2, const void* w2_sf, const float* w2_gs,
                  void* out, int T, int topk, int H, int I, int expert_lo, int E_local,
                  void* workspace, size_t workspace_bytes, okc_stream_t stream);
int okc_rmsnorm(const void* x, const void* w, void* y, int T, int H, float eps, okc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OKC_B200_H */
