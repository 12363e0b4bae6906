/*
 * ds_kernels.h — C ABI of libds_kernels_sm100.so, the B200 (sm_100a) implementation of
 * DeepSeek-V2-Lite's MoE layer and MLA projection hot path.
 *
 * Every compute entry point takes raw device pointers, plain sizes and a CUDA stream passed
 * as `void*` (a cudaStream_t; NULL = legacy default stream) and allocates no device memory:
 * scratch is passed in by the caller as (workspace, workspace_bytes), sized by the matching
 * *_workspace_size() query.  (The one allocating call is ds_ep_alloc, which creates the
 * expert-parallel segment once.)  All launches are asynchronous on `stream` and nothing in
 * the compute entry points synchronises with the host.
 *
 * Return value: DS_OK (0) or a DS_ERR_* code.  ds_last_error() returns a message for the
 * last failure on the calling host thread.  Device-side failures (a bounded wait that ran
 * out) are recorded in a per-device status word read by ds_get_device_status().
 *
 * Each declaration cites the reference interface it replaces (paths inside the reference
 * project sahan974/DeepSeek-V2-Lite-CUDA).  Differences from the reference launchers:
 *   - int status instead of `throw std::runtime_error`;
 *   - expert offsets are DEVICE pointers (the reference GEMMs take a host array);
 *   - scratch is caller-provided (the reference scan cudaMalloc's per call);
 *   - routing/dispatch are deterministic: experts per token in descending logit order
 *     (ties -> lower expert index); slots within an expert in ascending token order.
 */
#ifndef DS_KERNELS_H
#define DS_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DS_API __attribute__((visibility("default")))
#else
#define DS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DS_OK 0
#define DS_ERR_INVALID_ARG 1   /* bad shape / null pointer / misaligned pointer          */
#define DS_ERR_UNSUPPORTED 2   /* valid arguments this build does not handle              */
#define DS_ERR_CUDA 3          /* a CUDA runtime call failed                              */
#define DS_ERR_TIMEOUT 4       /* device status: a bounded on-device wait ran out         */
#define DS_ERR_WORKSPACE 5     /* workspace pointer null or smaller than required         */

/* Message for the last failing call on this host thread ("" if none). */
DS_API const char* ds_last_error(void);

/* Library / build identification, e.g. "ds_kernels sm_100a 0.1". */
DS_API const char* ds_version(void);

/* Device status word: *status receives DS_OK or DS_ERR_TIMEOUT (set by a kernel whose
 * bounded wait ran out).  Synchronises the device.  ds_clear_device_status() resets it. */
DS_API int ds_get_device_status(int* status);
DS_API int ds_clear_device_status(void);

/* Replaces run_hello (src/kernels/hello.cu:11-21, bindings.cu:187-189): prints one line
 * from a kernel; toolchain smoke test only. */
DS_API int ds_run_hello(void* stream);

/* ---------------------------------------------------------------------------------------
 * K1 routing.  Replaces launch_moe_routing (src/kernels/include/moe/routing.h:27-36,
 * src/kernels/moe/routing.cu:230-260) and moe_routing_forward (routing.cu:266-301).
 * logits f32 [num_tokens, num_experts] -> topk_indices i32 [num_tokens, top_k] (descending
 * logit, ties -> lower index), topk_weights f32 [num_tokens, top_k] (softmax values, no
 * renormalisation), expert_counts i32 [num_experts] (zeroed and filled here).
 * num_experts <= 64, 1 <= top_k <= min(8, num_experts). */
DS_API int ds_moe_routing(const float* logits, int32_t* topk_indices, float* topk_weights,
                   int32_t* expert_counts, int num_tokens, int num_experts, int top_k,
                   void* stream);

/* ---------------------------------------------------------------------------------------
 * K2 scan.  Replaces launch_moe_scan (src/kernels/include/moe/scan.h:31-36,
 * src/kernels/moe/scan.cu:33-75) and moe_scan_forward (scan.cu:86-130).
 * expert_offsets[i] = sum(expert_counts[0..i-1]); expert_offsets[num_experts] = total.
 * No host synchronisation, no allocation.  num_experts >= 1. */
DS_API int ds_moe_scan(const int32_t* expert_counts, int32_t* expert_offsets, int num_experts,
                void* stream);

/* ---------------------------------------------------------------------------------------
 * K3 dispatch.  Replaces launch_moe_dispatch (src/kernels/include/moe/dispatch.h:44-57,
 * src/kernels/moe/dispatch.cu:106-139) and moe_dispatch_forward (dispatch.cu:156-218).
 * Row for (token t, pick j) with expert e = topk_indices[t, j]:
 *   slot = expert_offsets[e] + #{t' < t routed to e}
 * dispatched[slot] = input[t]; token_map[slot] = t; dispatched_weights[slot] = w[t, j].
 * Deterministic (the reference claims slots with atomics).  hidden_size % 8 == 0.
 * The reference's expert_cursor scratch is replaced by `workspace`. */
DS_API size_t ds_moe_dispatch_workspace_size(int num_tokens, int num_experts, int top_k);
DS_API int ds_moe_dispatch(const void* input_bf16, const int32_t* topk_indices,
                    const float* topk_weights, const int32_t* expert_offsets,
                    void* dispatched_bf16, int32_t* token_map, float* dispatched_weights,
                    int num_tokens, int hidden_size, int num_experts, int top_k,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free dispatch (no counterpart in the reference).  Same arguments, outputs and
 * ordering as ds_moe_dispatch, minus the workspace: for callers that cannot allocate device
 * memory where they call this (a serving loop that keeps the CUDA allocator off its hot
 * path, a binding that only holds plain pointers, code running while other work is being
 * captured into a CUDA graph).  Its scratch is one fixed 2.5 MiB array in this library's
 * device memory, reserved on every GPU that loads the library until the process exits.
 * Limit: num_tokens <= DS_NOALLOC_MAX_TOKENS (else DS_ERR_UNSUPPORTED, nothing launched),
 * num_experts <= 64, top_k <= 8.  All calls on a device share that array: calls that may
 * overlap on the GPU (unordered streams, several host threads) race and corrupt each
 * other's results, so order them on one stream.  The first call on each device looks up
 * the array's address (one-time set-up); make it before any stream capture begins.  The
 * stream must belong to the current device (another device's stream: DS_ERR_UNSUPPORTED). */
#define DS_NOALLOC_MAX_TOKENS 65536
DS_API int ds_moe_dispatch_noalloc(const void* input_bf16, const int32_t* topk_indices,
                                   const float* topk_weights, const int32_t* expert_offsets,
                                   void* dispatched_bf16, int32_t* token_map,
                                   float* dispatched_weights, int num_tokens, int hidden_size,
                                   int num_experts, int top_k, void* stream);

/* ---------------------------------------------------------------------------------------
 * K7 combine.  Replaces launch_moe_combine (src/kernels/include/moe/combine.h:41-49; a
 * throwing stub at combine.cu:80-93) and moe_combine_forward (combine.cu:107-176).
 * final[t] = bf16( sum over slots s with token_map[s] == t, in ascending s, of
 *                  f32(expert_output[s]) * dispatched_weights[s] ),   0 for tokens with
 * no slot.  token_map may hold any multiplicity; entries outside [0, num_tokens) are
 * ignored.  Deterministic (the reference accumulates with f32 atomics). */
DS_API size_t ds_moe_combine_workspace_size(int total_slots, int num_tokens);
DS_API int ds_moe_combine(const void* expert_output_bf16, const int32_t* token_map,
                   const float* dispatched_weights, void* final_output_bf16,
                   int total_slots, int hidden_size, int num_tokens,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * K5 swiglu.  Replaces launch_swiglu (src/kernels/include/moe/swiglu.h:26-32,
 * src/kernels/moe/swiglu.cu:114-130) and swiglu_forward (swiglu.cu:142-170).
 * out[r, j] = bf16( f32(bf16(silu(f32 in[r, j]))) * f32 in[r, j + I] ): the rounding
 * sequence of the reference model's bf16 F.silu(gate) * up (src/reference/moe.py:19); the
 * reference kernel rounds once (swiglu.cu:96-104), at most one bf16 ulp apart.  I even. */
DS_API int ds_swiglu(const void* input_bf16, void* output_bf16, int total_tokens,
              int intermediate_size, void* stream);

/* ---------------------------------------------------------------------------------------
 * K4 grouped GEMM1.  Replaces launch_moe_gemm1 (src/kernels/include/moe/gemm1.h:25-34,
 * src/kernels/moe/gemm1.cu:84-155) and moe_gemm1_forward (gemm1.cu:167-227).
 * For each expert e: out[off[e]:off[e+1]] = dispatched[off[e]:off[e+1]] @ packed_w1[e]^T.
 * packed_w1 bf16 [num_experts, 2I, H] (gate rows then up rows), out bf16 [S, 2I].
 * expert_offsets is a DEVICE pointer [num_experts+1].  Rows outside [off[0], off[E]) are
 * zeroed.  tcgen05/TMEM tensor cores.  H % 8 == 0, I % 128 == 0. */
DS_API int ds_moe_gemm1(const void* dispatched_bf16, const void* packed_w1_bf16,
                 const int32_t* expert_offsets, void* gemm1_out_bf16, int total_slots,
                 int num_experts, int hidden_size, int double_intermed, void* stream);

/* New (additive) op: GEMM1 with the SwiGLU epilogue fused: out bf16 [S, I] equals
 * ds_swiglu(ds_moe_gemm1(...)) except that the gate/up values are not rounded to bf16
 * before the activation. */
DS_API int ds_moe_gemm1_swiglu(const void* dispatched_bf16, const void* packed_w1_bf16,
                        const int32_t* expert_offsets, void* swiglu_out_bf16,
                        int total_slots, int num_experts, int hidden_size,
                        int double_intermed, void* stream);

/* Tiling of the tcgen05 grouped GEMM behind ds_moe_gemm1/2, ds_kv_upproj and the layer
 * (additive; no reference counterpart): 0 = one CTA per 128 x 256 tile, 1 = CTA pairs
 * (2-CTA clusters, cta_group::2 MMAs) on 256 x 256 tiles for every plain / SwiGLU launch,
 * -1 = automatic (pairs when a launch's groups average at least 2048 rows).  The default comes
 * from the DS_GEMM_PAIR environment variable (unset: -1).  Other values only query.
 * Returns the previous mode.  Process-wide; results are identical in every mode. */
DS_API int ds_gemm_pair_mode(int mode);

/* ---------------------------------------------------------------------------------------
 * K6 grouped GEMM2.  Replaces launch_moe_gemm2 (src/kernels/include/moe/gemm2.h:25-34,
 * src/kernels/moe/gemm2.cu:75-124) and moe_gemm2_forward (gemm2.cu:136-195).
 * For each expert e: out[off[e]:off[e+1]] = swiglu_out[...] @ w2[e]^T.
 * w2 bf16 [num_experts, H, I], out bf16 [S, H].  I % 8 == 0, H % 256 == 0. */
DS_API int ds_moe_gemm2(const void* swiglu_out_bf16, const void* w2_bf16,
                 const int32_t* expert_offsets, void* gemm2_out_bf16, int total_slots,
                 int num_experts, int intermediate_size, int hidden_size, void* stream);

/* ---------------------------------------------------------------------------------------
 * K8 RMSNorm.  Replaces launch_rms_norm (src/kernels/include/mla/rms_norm.h:27-35,
 * src/kernels/mla/rms_norm.cu:126-144) and rms_norm_forward (rms_norm.cu:158-192).
 * out[r] = bf16( weight * x[r] * rsqrt(mean(x[r]^2) + eps) ), f32 weight.  hidden even.
 * in_stride / out_stride are row strides in elements (hidden_size for contiguous rows). */
DS_API int ds_rms_norm(const void* input_bf16, const float* weight, void* output_bf16, int rows,
                int hidden_size, float eps, void* stream);
DS_API int ds_rms_norm_strided(const void* input_bf16, int64_t in_stride, const float* weight,
                        void* output_bf16, int64_t out_stride, int rows, int hidden_size,
                        float eps, void* stream);

/* Decoder-layer glue around the MoE layer (additive op; the residual adds and pre-norms of
 * src/reference/decoder_layer.py:123-139 with RMSNorm of src/reference/mla.py:59-64):
 *   sum_out[r] = bf16(residual[r] + input[r]),
 *   normed_out[r] = bf16( weight * sum_out[r] * rsqrt(mean(sum_out[r]^2) + eps) ),
 * statistics in f32 over the rounded sum, one pass over both inputs.  Contiguous rows,
 * hidden_size a multiple of 8 and at most 2048, 16-byte aligned pointers. */
DS_API int ds_rms_norm_residual(const void* input_bf16, const void* residual_bf16,
                                const float* weight, void* sum_out_bf16, void* normed_out_bf16,
                                int rows, int hidden_size, float eps, void* stream);

/* ---------------------------------------------------------------------------------------
 * K9 kv up-projection.  Replaces launch_kv_upproj (src/kernels/include/mla/kv_upproj.h:
 * 30-38, src/kernels/mla/kv_upproj.cu:77-119) and kv_upproj_forward (kv_upproj.cu:
 * 133-178): out bf16 [rows, out_dim] = normed bf16 [rows, K] @ weight bf16 [out_dim, K]^T.
 * tcgen05/TMEM tensor cores.  K % 8 == 0, out_dim % 256 == 0. */
DS_API int ds_kv_upproj(const void* normed_kv_bf16, const void* weight_bf16, void* kv_up_bf16,
                 int rows, int kv_lora_rank, int out_dim, void* stream);

/* ---------------------------------------------------------------------------------------
 * K10 RoPE.  Replaces launch_rope (src/kernels/include/mla/rope.h:33-41,
 * src/kernels/mla/rope.cu:101-119) and rope_forward (rope.cu:139-207), in one launch for
 * q and k.  q_pe [bsz, heads, seq, D], k_pe [bsz, 1, seq, D], cos/sin [bsz, 1, seq, D]
 * (pre-indexed by position; broadcast over heads by index, not copied).  For k < D/2:
 *   out[k]       = x[2k]   * cos[k]       - x[2k+1] * sin[k]
 *   out[k + D/2] = x[2k+1] * cos[k + D/2] + x[2k]   * sin[k + D/2]      (f32, one rounding)
 * D even. */
DS_API int ds_rope(const void* q_pe_bf16, const void* k_pe_bf16, const void* cos_bf16,
            const void* sin_bf16, void* q_out_bf16, void* k_out_bf16, int bsz, int heads,
            int seq, int rope_dim, void* stream);

/* ---------------------------------------------------------------------------------------
 * MLA attention (config 3): the causal attention core and the whole MLA forward of
 * DeepSeekMLA (src/reference/mla.py:295-393: q_proj, kv_a_proj_with_mqa, kv_a_layernorm,
 * kv_b_proj, YaRN/plain RoPE on the 64-wide parts, softmax(q k^T * scale) v with 192-wide
 * q/k and 128-wide v heads, o_proj).  The reference has no kernel for this part (its
 * src/kernels/mla/ covers rms_norm, kv_upproj and rope only).
 *
 * ds_mla_attention: qkv bf16 [batch*seq, qkv_ld] holds per token the heads' q (192 each:
 * 128 nope then 64 RoPE-rotated), then the 512-wide latent, then the 64-wide rotated k_pe;
 * kv bf16 [batch*seq, heads*256] holds per head 128 k_nope then 128 v; out bf16
 * [batch*seq, heads*128] (head h in columns h*128 ..).  Causal; seq % 8 == 0.  v is read in
 * place; workspace (ds_mla_attention_workspace_size bytes, 4-byte aligned) holds the counter
 * from which the persistent kernel's CTAs take their (batch, head, q tile) work items; it is
 * zeroed on `stream` before the launch, so calls on different streams need different
 * workspaces. */
DS_API size_t ds_mla_attention_workspace_size(int batch, int seq, int heads);
DS_API int ds_mla_attention(const void* qkv_bf16, int qkv_ld, const void* kv_bf16,
                            void* out_bf16, int batch, int seq, int heads, float softmax_scale,
                            void* workspace, size_t workspace_bytes, void* stream);
/* ds_mla_forward: x bf16 [batch*seq, hidden]; w_qkv_a bf16 [heads*192 + 576, hidden] =
 * q_proj.weight rows then kv_a_proj_with_mqa.weight rows; kv_norm_weight f32 [512];
 * w_kv_b bf16 [heads*256, 512]; w_o bf16 [hidden, heads*128]; cos/sin bf16 [positions, 64]
 * tables (the module's cos_cached/sin_cached); positions int32 [batch*seq] or NULL
 * (position = index within the sequence); out bf16 [batch*seq, hidden].  `events`: NULL or
 * DS_MLA_NUM_EVENTS handles recorded before the first kernel and after each phase (qkv
 * projection, latent RMSNorm, kv_b projection, RoPE, attention, o_proj). */
#define DS_MLA_NUM_EVENTS 7
DS_API size_t ds_mla_forward_workspace_size(int batch, int seq, int hidden, int heads);
DS_API int ds_mla_forward(const void* x_bf16, const void* w_qkv_a_bf16,
                          const float* kv_norm_weight, const void* w_kv_b_bf16,
                          const void* w_o_bf16, const void* cos_bf16, const void* sin_bf16,
                          const int32_t* positions, void* out_bf16, int batch, int seq,
                          int hidden, int heads, float eps, float softmax_scale,
                          void* workspace, size_t workspace_bytes, void** events,
                          void* stream);

/* ds_mla_prefill: ds_mla_forward over a prompt (positions 0 .. seq-1) that also writes the
 * prompt's raw latents and raw k_pe into a latent KV cache (the layout of
 * src/kernels/mla_cache.py:29-219: latent bf16 [batch, max_seq, 512], k_pe bf16
 * [batch, max_seq, 64]) together with the cache's two side arrays (rstd f32
 * [batch, max_seq], k_pe_rot bf16 [batch, max_seq, 64]; see ds_mla_cache_append). */
DS_API int ds_mla_prefill(const void* x_bf16, const void* w_qkv_a_bf16,
                          const float* kv_norm_weight, const void* w_kv_b_bf16,
                          const void* w_o_bf16, const void* cos_bf16, const void* sin_bf16,
                          void* out_bf16, int batch, int seq, int hidden, int heads, float eps,
                          float softmax_scale, void* cache_latent_bf16, void* cache_kpe_bf16,
                          float* cache_rstd, void* cache_kpe_rot_bf16, int max_seq, int pos0,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * MLA decode over the latent KV cache (config 4; the cache of src/kernels/mla_cache.py:29-219
 * and the attention of src/reference/mla.py:295-393 for one new token per sequence; the
 * reference has no decode kernel).
 *
 * ds_mla_cache_append: tokens pos0 .. pos0+new_tokens-1 of each of `batch` sequences; token i
 * of sequence b reads its latent (512) at latent + (b*src_rows_per_seq + i)*latent_ld and its
 * raw k_pe (64) at kpe + (...)*kpe_ld.  Writes the raw values into the cache (copy_raw != 0;
 * 0 refreshes only the side arrays of tokens already in it), and the side arrays the decode
 * attention reads: rstd = rsqrt(mean(latent^2) + eps) and k_pe rotated at its position with
 * the bf16 cos/sin [positions, 64] tables.
 *
 * ds_mla_decode_step: one token per sequence, heads == 16.  x bf16 [batch, hidden];
 * w_dec bf16 [16*512 + 16*64 + 512 + 64, hidden] = the absorbed query weights (per head
 * diag(g) W_uk_h^T W_q_nope_h, g the latent norm weight), the q_pe rows of q_proj, and
 * kv_a_proj_with_mqa; w_out bf16 [hidden, 16*512] = per head W_o_h W_uv_h diag(g).  Appends
 * the token at position cache_len, attends over positions 0 .. cache_len, writes out bf16
 * [batch, hidden].  cache_len_dev: NULL, or a device int32 holding the cached length; the
 * kernels then read the position from it (cache_len is only checked against max_seq), and
 * the step adds 1 to it after its attention — so a captured CUDA graph of the step replays
 * at successive positions.  `events`: NULL or DS_MLA_DECODE_NUM_EVENTS handles (projection,
 * append + query, attention, output projection). */
DS_API int ds_mla_cache_append(const void* latent_bf16, int latent_ld, const void* kpe_bf16,
                               int kpe_ld, int src_rows_per_seq, int batch, int new_tokens,
                               int pos0, int max_seq, int copy_raw, void* cache_latent_bf16,
                               void* cache_kpe_bf16, float* cache_rstd, void* cache_kpe_rot_bf16,
                               const void* cos_bf16, const void* sin_bf16, float eps,
                               void* stream);
#define DS_MLA_DECODE_NUM_EVENTS 5
DS_API size_t ds_mla_decode_workspace_size(int batch, int max_seq, int hidden);
DS_API int ds_mla_decode_step(const void* x_bf16, const void* w_dec_bf16, const void* w_out_bf16,
                              const void* cos_bf16, const void* sin_bf16,
                              void* cache_latent_bf16, void* cache_kpe_bf16, float* cache_rstd,
                              void* cache_kpe_rot_bf16, int batch, int max_seq, int cache_len,
                              int32_t* cache_len_dev, int hidden, int heads, float eps,
                              float softmax_scale, void* out_bf16, void* workspace,
                              size_t workspace_bytes, void** events, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused MoE layer (new, additive; the pipeline of src/kernels/moe_fused.py:118-154 plus the
 * shared expert of src/reference/moe.py:72-74,106-107 that the reference pipeline drops).
 * router_logits f32 [T, E] (x @ gate^T in f32), x bf16 [T, H], packed_w1 bf16 [E, 2I, H],
 * w2 bf16 [E, H, I], shared_w1 bf16 [2*Is, H] (gate rows then up rows) and shared_w2 bf16
 * [H, Is] or both NULL (no shared expert), out bf16 [T, H].
 * `events`: NULL, or DS_LAYER_NUM_EVENTS cudaEvent_t handles recorded on `stream` before
 * the first kernel and after each phase (routing, plan, dispatch, gemm1, gemm2, shared1,
 * shared2, combine) for per-kernel timing. */
#define DS_LAYER_NUM_EVENTS 9
DS_API size_t ds_moe_layer_workspace_size(int num_tokens, int hidden_size, int num_experts,
                                   int top_k, int intermediate_size,
                                   int shared_intermediate_size);
/* Where a layer forward leaves its routing inside the workspace (new, additive; the
 * reference pipeline returns it from moe_routing, src/kernels/moe_fused.py:131-134): byte
 * offsets of topk_indices int32 [T, k], topk_weights f32 [T, k] and slot_of int32 [T, k]
 * (the dispatch slot of each (token, pick)), valid after the forward until the next call
 * that uses the same workspace. */
DS_API int ds_moe_layer_workspace_routing(int num_tokens, int hidden_size, int num_experts,
                                          int top_k, int intermediate_size,
                                          int shared_intermediate_size, size_t* idx_offset,
                                          size_t* weights_offset, size_t* slot_of_offset);
DS_API int ds_moe_layer_forward(const float* router_logits, const void* x_bf16,
                         const void* packed_w1_bf16, const void* w2_bf16,
                         const void* shared_w1_bf16, const void* shared_w2_bf16,
                         void* out_bf16, int num_tokens, int hidden_size, int num_experts,
                         int top_k, int intermediate_size, int shared_intermediate_size,
                         void* workspace, size_t workspace_bytes, void** events,
                         void* stream);

/* ---------------------------------------------------------------------------------------
 * Layer stages (new, additive).  The fused layer above is these stages back to back; they
 * are exported so a caller can put a collective between them (expert parallelism:
 * route_dispatch -> all-to-all -> ep_plan + gather_rows -> expert_mlp -> all-to-all ->
 * combine_slots).  Pipeline of src/kernels/moe_fused.py:118-154 split at its data exchanges.
 *
 * ds_moe_route_dispatch: routing (as ds_moe_routing) + expert offsets [E+1] + deterministic
 *   dispatch (as ds_moe_dispatch) of x into expert-major `dispatched` [T*k, H]; slot_of[t, j]
 *   is the dispatched row of (token t, pick j). */
DS_API size_t ds_moe_route_dispatch_workspace_size(int num_tokens, int num_experts, int top_k);
DS_API int ds_moe_route_dispatch(const float* router_logits, const void* x_bf16, int num_tokens,
                                 int hidden_size, int num_experts, int top_k,
                                 int32_t* topk_indices, float* topk_weights,
                                 int32_t* expert_offsets, int32_t* slot_of, int32_t* token_map,
                                 void* dispatched_bf16, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ds_moe_router: router logits x @ gate^T with f32 accuracy on the tensor cores (the f32
 *   gate is pre-split by ds_router_weight_split into bf16 hi/mid/lo parts that sum to it;
 *   the GEMM writes per-K-slice partial accumulators into `workspace`, the routing kernel
 *   sums them), then the top-k of ds_moe_routing.  Replaces the f32 F.linear + moe_routing
 *   pair of src/kernels/moe_fused.py:131-137.  logits_out f32 [T, E] may be NULL.
 * ds_router_weight_split: gate f32 [E, H] -> w_split bf16 [256, H] (rows e, 64+e, 128+e). */
DS_API int ds_router_weight_split(const float* gate_weight, int num_experts, int hidden_size,
                                  void* w_split_bf16, void* stream);
DS_API size_t ds_moe_router_workspace_size(int num_tokens);
DS_API int ds_moe_router(const void* x_bf16, const void* w_split_bf16, int num_tokens,
                         int hidden_size, int num_experts, int top_k, int32_t* topk_indices,
                         float* topk_weights, float* logits_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ds_moe_dispatch_routed: ds_moe_route_dispatch for routing that is already computed
 *   (topk_indices/weights [T, k]); workspace size as ds_moe_route_dispatch_workspace_size. */
DS_API int ds_moe_dispatch_routed(const int32_t* topk_indices, const float* topk_weights,
                                  const void* x_bf16, int num_tokens, int hidden_size,
                                  int num_experts, int top_k, int32_t* expert_offsets,
                                  int32_t* slot_of, int32_t* token_map, void* dispatched_bf16,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* ds_moe_expert_mlp: for each group g (rows [off[g], off[g+1]) of `rows`), down(silu(gate x)
 *   * up x) with the group's weights (packed_w1 [G, 2I, H], w2 [G, H, I]); h [R, I] is
 *   scratch; output row i goes to out[out_row_map ? out_row_map[i] : i].  max_ctas caps the
 *   GEMM grid (0 = one CTA per SM) to leave SMs to work that must run concurrently. */
DS_API int ds_moe_expert_mlp(const void* rows_bf16, int num_rows, const int32_t* group_offsets,
                             int num_groups, const void* packed_w1_bf16, const void* w2_bf16,
                             int hidden_size, int intermediate_size, void* h_bf16,
                             void* out_bf16, const int32_t* out_row_map, int max_ctas,
                             void* stream);

/* ds_dense_mlp: one SwiGLU MLP over all rows (the shared expert, src/reference/moe.py:72-74):
 *   w1 [2I, H] (gate rows then up rows), w2 [H, I], h [R, I] scratch; max_ctas as above. */
DS_API int ds_dense_mlp(const void* x_bf16, int num_rows, const void* w1_bf16,
                        const void* w2_bf16, int hidden_size, int intermediate_size,
                        void* h_bf16, void* out_bf16, int max_ctas, void* stream);
/* ds_dense_mlp with a caller workspace (ds_dense_mlp_workspace_size; 0 bytes when no split
 * is needed): for few rows (decode) the GEMMs split K over the SMs, f32 partials in the
 * workspace reduced through the same epilogues. */
DS_API size_t ds_dense_mlp_workspace_size(int num_rows, int hidden_size, int intermediate_size);
DS_API int ds_dense_mlp_ws(const void* x_bf16, int num_rows, const void* w1_bf16,
                           const void* w2_bf16, int hidden_size, int intermediate_size,
                           void* h_bf16, void* out_bf16, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ds_dense_gemm1_swiglu / ds_dense_gemm2: the two halves of ds_dense_mlp as separate
 *   launches (h = silu(x gate^T) * (x up^T); out = h w2^T), so each can overlap a different
 *   exchange; max_ctas as above. */
DS_API int ds_dense_gemm1_swiglu(const void* x_bf16, int num_rows, const void* w1_bf16,
                                 int hidden_size, int intermediate_size, void* h_bf16,
                                 int max_ctas, void* stream);
DS_API int ds_dense_gemm2(const void* h_bf16, int num_rows, const void* w2_bf16,
                          int intermediate_size, int hidden_size, void* out_bf16, int max_ctas,
                          void* stream);

/* ds_moe_combine_slots: out[t] = bf16( sum_j w[t,j] * expert_out[slot_of[t,j]] (ascending
 *   slot) + shared_out[t] ) ; shared_out may be NULL. */
DS_API int ds_moe_combine_slots(const void* expert_out_bf16, const int32_t* slot_of,
                                const float* topk_weights, int top_k,
                                const void* shared_out_bf16, void* out_bf16, int num_tokens,
                                int hidden_size, void* stream);

/* ds_ep_plan: receive side of the expert-parallel all-to-all.  recv_counts[s*El + e] = rows
 *   source rank s sent for local expert e; received rows are source-major.  Writes
 *   expert_offsets [El+1] of the expert-major order and row_map [recv_rows]: expert-major
 *   row i is source-major row row_map[i] (use it to gather the GEMM input and as the GEMM2
 *   out_row_map so results land back in source-major order). */
DS_API size_t ds_ep_plan_workspace_size(int num_ranks, int local_experts);
DS_API int ds_ep_plan(const int32_t* recv_counts, int num_ranks, int local_experts,
                      int recv_rows, int32_t* expert_offsets, int32_t* row_map,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ds_gather_rows: dst[i] = src[row_map[i]] for bf16 rows of hidden_size. */
DS_API int ds_gather_rows(const void* src_bf16, const int32_t* row_map, int num_rows,
                          int hidden_size, void* dst_bf16, void* stream);

/* Fused layer from the tokens: ds_moe_router (f32-accurate tensor-core router + top-k)
 * followed by the pipeline of ds_moe_layer_forward.  router_w_split from
 * ds_router_weight_split; logits_out f32 [T, E] may be NULL; workspace size as
 * ds_moe_layer_workspace_size; events as ds_moe_layer_forward (phase 0 = router + ranks). */
DS_API int ds_moe_layer_forward_from_x(const void* x_bf16, const void* router_w_split_bf16,
                                       float* logits_out, const void* packed_w1_bf16,
                                       const void* w2_bf16, const void* shared_w1_bf16,
                                       const void* shared_w2_bf16, void* out_bf16,
                                       int num_tokens, int hidden_size, int num_experts,
                                       int top_k, int intermediate_size,
                                       int shared_intermediate_size, void* workspace,
                                       size_t workspace_bytes, void** events, void* stream);

/* ---------------------------------------------------------------------------------------
 * Expert parallelism over NVLink peer memory (additive: the reference is single-GPU; this is
 * its fused pipeline, src/kernels/moe_fused.py:118-154, with experts partitioned
 * contiguously over `world` ranks, one process per GPU).  Each rank allocates one symmetric
 * segment with ds_ep_alloc(ds_ep_symmetric_size(...)), exports it with ds_ep_ipc_handle,
 * and maps every other rank's segment with ds_ep_ipc_open; sym_bases[r] is rank r's
 * segment as seen from this process (its own pointer at [rank]).  No host synchronisation
 * and no collective library call on the data path: the count exchange, row transfer and
 * result return run inside the plan, dispatch, GEMM2 and combine kernels, ordered by
 * per-forward flags in the segments.  Every cross-GPU wait is bounded by timeout_ms; a
 * wait that runs out sets the device status to DS_ERR_TIMEOUT (read it with
 * ds_get_device_status), the ranks behind it time out in turn, and the segments must be
 * re-created before the next forward. */
#define DS_EP_IPC_HANDLE_BYTES 64
#define DS_EP_NUM_EVENTS 7

DS_API int ds_ep_symmetric_size(int max_tokens, int hidden_size, int num_experts, int top_k,
                                int world, size_t* bytes);
/* cudaMalloc + zero fill (the flags start at zero); ds_ep_free releases it. */
DS_API int ds_ep_alloc(size_t bytes, void** ptr);
DS_API int ds_ep_free(void* ptr);
DS_API int ds_ep_ipc_handle(void* ptr, void* handle_out /* DS_EP_IPC_HANDLE_BYTES */);
DS_API int ds_ep_ipc_open(const void* handle, void** ptr);
DS_API int ds_ep_ipc_close(void* ptr);
DS_API size_t ds_ep_layer_workspace_size(int max_tokens, int hidden_size, int num_experts,
                                         int top_k, int intermediate_size,
                                         int shared_intermediate_size, int world);
/* One expert-parallel MoE layer forward of this rank's num_tokens (0 allowed; every rank
 * must call it for every forward, with epoch = 1, 2, 3, ...).  w1_local [El*2I, H] and
 * w2_local [El*H, I] hold experts [rank*El, (rank+1)*El) in the prepacked layout; router,
 * shared expert, logits_out and out as ds_moe_layer_forward_from_x.  The shared expert's
 * GEMM1 runs on an internal second stream beside the routing and the dispatch (forked from
 * and joined back into `stream` with events; one forward at a time per device).  events: NULL or
 * DS_EP_NUM_EVENTS handles bracketing route | plan+count exchange | dispatch+send |
 * routed GEMM1 | GEMM2 (+shared, return) | combine. */
DS_API int ds_ep_layer_forward(const void* x_bf16, int num_tokens,
                               const void* router_w_split_bf16, float* logits_out,
                               const void* w1_local_bf16, const void* w2_local_bf16,
                               const void* shared_w1_bf16, const void* shared_w2_bf16,
                               void* out_bf16, int hidden_size, int num_experts, int top_k,
                               int intermediate_size, int shared_intermediate_size, int rank,
                               int world, int max_tokens, void* const* sym_bases, int epoch,
                               int timeout_ms, void* workspace, size_t workspace_bytes,
                               void** events, void* stream);

/* ---------------------------------------------------------------------------------------
 * Failure-detection probe (no reference counterpart): launches one CTA that waits on an
 * mbarrier nothing arrives on, through the same bounded-wait routine the GEMM pipeline
 * uses, with a limit of `timeout_cycles` SM clock cycles.  The wait runs out, the kernel
 * sets the device status to DS_ERR_TIMEOUT and returns; the context stays usable. */
DS_API int ds_debug_wait_probe(long long timeout_cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DS_KERNELS_H */
