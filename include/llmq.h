/*
 * llmq.h -- C ABI of the B200 (sm_100a) quantized-matmul hot path of
 * llm_mojo (GPT-2 124M inference with pluggable weight formats).
 *
 * Plain pointers and sizes only. "dev" pointers are CUDA device memory of
 * the context's device; "host" pointers are borrowed for the duration of the
 * call. Every function returns an llmq_status; llmq_last_error() gives the
 * message of the last failure on a context. Handles are owned by the caller
 * and released with the matching *_free. One context serves one host thread
 * and one device; its calls are issued on the context's stream.
 */
#ifndef LLMQ_H
#define LLMQ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int llmq_status;
#define LLMQ_OK 0
#define LLMQ_ERR_INVALID 1     /* bad argument or shape (the reference raises or aborts) */
#define LLMQ_ERR_CUDA 2        /* a CUDA call failed */
#define LLMQ_ERR_NOMEM 3       /* device or host allocation failed */
#define LLMQ_ERR_TIMEOUT 4     /* a bounded device-side wait gave up */
#define LLMQ_ERR_UNSUPPORTED 5 /* format or path not available */

typedef struct llmq_ctx llmq_ctx;
typedef struct llmq_weight llmq_weight;
typedef struct llmq_kv llmq_kv;
typedef struct llmq_model llmq_model;

/* linear() epilogue flags: kernels.mojo:38-48 store_out[RESID, GELU], BIAS. */
#define LLMQ_BIAS 1
#define LLMQ_GELU 2
#define LLMQ_RESID 4

/* KV cache kinds: kvcache.mojo QuantKV[8] (float attention) and
 * int_attention.mojo IntAttnKV (integer attention). */
#define LLMQ_KV_QUANT8 1
#define LLMQ_KV_INTATTN 2
#define LLMQ_KV_F32 3  /* DenseKV[float32] (kvcache.mojo:153-246) */
#define LLMQ_KV_BF16 4 /* DenseKV[bfloat16] */

/* ---- context ------------------------------------------------------------ */
/* No reference counterpart (the reference runs in-process on the CPU). */
llmq_status llmq_init(int device, llmq_ctx **out);
llmq_status llmq_destroy(llmq_ctx *ctx);
const char *llmq_last_error(const llmq_ctx *ctx);
/* Issue the context's work on `cuda_stream` (a cudaStream_t); NULL restores
 * the context's own stream. */
llmq_status llmq_set_stream(llmq_ctx *ctx, void *cuda_stream);
llmq_status llmq_sync(llmq_ctx *ctx);

/* ---- weight formats ------------------------------------------------------ */
/* Replaces QuantMatrix.from_f32 (tensor.mojo:333-383): the reference's RTN
 * affine quantizer, on the host. src is [rows, cols] row-major float32;
 * reduce_rows=1 stores the transpose (layer matrices, [IN, OUT] -> [OUT, IN]),
 * 0 stores src as is (wte, [V, C]). group 0 = per channel. a16 with bits 4
 * and group 32 selects the BLOCKED decode layout (tensor.mojo:277-288,
 * nibble_at :385-404). codes: n*k*bits/8 bytes, scale (float16 bits) and zp:
 * n*(k/group) each, n = reduce_rows ? cols : rows, k the other. */
llmq_status llmq_quantize_affine(const float *src_host, int rows, int cols, int reduce_rows, int bits, int group,
                                 int sym, int a16, uint8_t *codes_host, uint16_t *scale_host, uint8_t *zp_host);

/* Uploads a QuantMatrix[bits, group, sym, a16] in its stored layout
 * (tensor.mojo:302-307: codes, float16 scale, u8 zero point per group), as
 * restore (tensor.mojo:645-656) takes it. rows = outputs, cols = the
 * reduction axis; group 0 = per channel. */
llmq_status llmq_weight_create_affine(llmq_ctx *ctx, int bits, int group, int sym, int a16, int rows, int cols,
                                      const uint8_t *codes_host, const uint16_t *scale_host,
                                      const uint8_t *zp_host, llmq_weight **out);
/* Uploads a GGUFMatrix (gguf.mojo:344-512): `rows` rows of `cols` values in
 * ggml block type ggml_type (0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 8 Q8_0, 12 Q4_K,
 * 13 Q5_K, 14 Q6_K), as stored in the file: rows * (cols / block) blocks. */
llmq_status llmq_weight_create_gguf(llmq_ctx *ctx, int ggml_type, const void *blocks_host, int rows, int cols,
                                    llmq_weight **out);
/* Uploads a DenseMatrix[dtype] (tensor.mojo:150-227), [rows, cols] row-major
 * as the reference stores it ([IN, OUT] layer matrices, [V, C] wte). */
#define LLMQ_DENSE_F32 0
#define LLMQ_DENSE_F16 1
#define LLMQ_DENSE_BF16 2
llmq_status llmq_weight_create_dense(llmq_ctx *ctx, int dtype, const void *data_host, int rows, int cols,
                                     llmq_weight **out);
/* WeightMatrix.free (tensor.mojo:658-661). */
llmq_status llmq_weight_free(llmq_weight *w);
/* WeightMatrix.nbytes (tensor.mojo:629-632): codes + 3 bytes per group. */
long long llmq_weight_nbytes(const llmq_weight *w);

/* ---- kernels (device pointers) ------------------------------------------ */
/* Replaces kernels.linear (kernels.mojo:655-673): out[T, OUT] (+)=
 * act(x[T, IN] @ w + b), with the kernel for w's format:
 *  - ACT16 affine: matmul_rows_a16 (:419-509); T == 1 is the decode path
 *    (dot_row_i16 via linear_team, :774-816), T > 1 the tile path (tile_i16,
 *    :512-573; rows_i16 for OUT % 32);
 *  - other affine and GGUF formats: matmul_rows (:285-349), one token;
 *  - dense [IN, OUT]: gemv (:132-176) split in llmq_set_dense_parts parts,
 *    one token.
 * Unbuilt combinations return LLMQ_ERR_UNSUPPORTED. */
llmq_status llmq_linear(llmq_ctx *ctx, const llmq_weight *w, const float *x_dev, const float *bias_dev,
                        float *out_dev, int T, int IN, int OUT, int flags);
/* Replaces head (kernels.mojo:676-690): logits[T, V] = h[T, C] @ w[V, C]^T
 * with the head kernel for w's format (head_i16 for GGUF Q8_0 / Q6_K,
 * matmul_rows_a16 for ACT16, lm_head / lm_head_rows for dense,
 * matmul_rows otherwise). */
llmq_status llmq_head(llmq_ctx *ctx, const llmq_weight *w, const float *h_dev, float *logits_dev, int T, int C,
                      int V);
/* The number of parts the dense gemv splits its reduction into (the
 * reference's thread count, kernels.mojo:141-142 / :828-834; default 4).
 * Results depend on it, as the reference's do. */
llmq_status llmq_set_dense_parts(llmq_ctx *ctx, int nparts);
/* Replaces head (kernels.mojo:676-690) + argmax (gpt2t.mojo:792-797) for one
 * token: logits[V] = h[C] @ w^T (logits_dev may be NULL) and the first index
 * of the largest logit into *argmax_dev. */
llmq_status llmq_head_argmax(llmq_ctx *ctx, const llmq_weight *w, const float *h_dev, float *logits_dev,
                             int *argmax_dev);
/* No counterpart in the reference: llmq_head_argmax without any device
 * allocation, for callers that cannot allocate while they run (a serving
 * process whose pool holds the device's memory, or a host that must not meet
 * the device-wide synchronisation of cudaMalloc / cudaFree). Same arguments
 * and results as llmq_head_argmax. Its scratch is a fixed 16 KiB device
 * array, one per device, with room for LLMQ_NOALLOC_MAX_PARTS per-CTA
 * partials; a weight whose gemv grid needs more returns LLMQ_ERR_INVALID
 * (on B200 the grid is at most 8 CTAs per SM, 1184). The first call on each
 * device looks up the array's address and should come before any stream
 * capture. Calls on one device that overlap in time (other streams, other
 * contexts, other host threads) race on the array: order them. */
#define LLMQ_NOALLOC_MAX_PARTS 1920
llmq_status llmq_head_argmax_noalloc(llmq_ctx *ctx, const llmq_weight *w, const float *h_dev, float *logits_dev,
                                     int *argmax_dev);
/* Limit, in SM clock cycles, of each device-side wait of the persistent and
 * cluster decode kernels and of the row GEMVs (GGUF and dense formats);
 * 0 restores the default (4e9 cycles, about 2 s). A wait that runs out
 * makes the kernel record an error, wait for its own copies in flight (a
 * separate, long bound) and return; the call that synchronises next
 * reports LLMQ_ERR_TIMEOUT. No counterpart in the reference (its waits are
 * host spin loops); this is the hook the timeout tests use. */
llmq_status llmq_set_wait_limit(llmq_ctx *ctx, long long cycles);
/* Which kernel runs the several-token (T > 1) A16 matmuls of llmq_linear /
 * llmq_head (tile_i16, kernels.mojo:512-573): AUTO (the tcgen05 split-int8
 * GEMM from 16 tokens on, where the shape allows), CUDA_CORE (dp tiles), or
 * TCGEN05 (the GEMM whenever the shape allows). Results are identical; no
 * counterpart in the reference, which has one CPU kernel. */
#define LLMQ_PREFILL_AUTO 0
#define LLMQ_PREFILL_CUDA_CORE 1
#define LLMQ_PREFILL_TCGEN05 2
llmq_status llmq_set_prefill_kernel(llmq_ctx *ctx, int kind);
/* Replaces layernorm (kernels.mojo:179-197), eps 1e-5. */
llmq_status llmq_layernorm(llmq_ctx *ctx, float *out_dev, const float *x_dev, const float *w_dev,
                           const float *b_dev, int T, int C);
/* Replaces quantize_rows (kernels.mojo:400-416). */
llmq_status llmq_quantize_rows(llmq_ctx *ctx, const float *x_dev, int T, int IN, int16_t *xq_dev, float *sx_dev);
/* The int32 lane sums of dot_row_i16 (tensor.mojo:518-577) for input x[IN]
 * after quantize_rows: lanes_dev[OUT][units][16], units = IN/256 for the
 * BLOCKED layout (sums of x*u before the zero point), else IN/group (sums of
 * x*(u - zp)). For bit-exact parity checks of the integer accumulators. */
llmq_status llmq_debug_lane_sums(llmq_ctx *ctx, const llmq_weight *w, const float *x_dev, int32_t *lanes_dev);

/* ---- KV cache (kvcache.mojo:31-87 KVCache) ------------------------------ */
/* KVCache.create. kind LLMQ_KV_QUANT8, LLMQ_KV_INTATTN, LLMQ_KV_F32 or
 * LLMQ_KV_BF16 (the dense caches attend with the several-token kernel for
 * every token count). */
llmq_status llmq_kv_create(llmq_ctx *ctx, int kind, int n_layer, int max_t, int n_head, int head_dim,
                           llmq_kv **out);
llmq_status llmq_kv_free(llmq_kv *kv);
/* KVCache.store for T tokens: the key and value of qkv row t ([T, 3C],
 * columns C.. and 2C..) at position pos0 + t of `layer`. */
llmq_status llmq_kv_store(llmq_ctx *ctx, llmq_kv *kv, int layer, int pos0, int T, const float *qkv_dev);
/* KVCache.attend (kvcache.mojo:62-79): out[T, C] for T tokens at pos0.. */
llmq_status llmq_kv_attend(llmq_ctx *ctx, llmq_kv *kv, float *out_dev, const float *qkv_dev, int layer, int T,
                           int pos0);
/* Copies the cache's storage to the host (codes and scales as the format
 * lays them out; QuantKV[8]: k, v int8 [L][max_t][H][hd], ks, vs float
 * [L][max_t][H]). Any pointer may be NULL. For tests. */
llmq_status llmq_kv_read(llmq_ctx *ctx, const llmq_kv *kv, void *k_host, void *v_host, void *ks_host,
                         void *vs_host);

/* ---- model (gpt2t.mojo:198-572 Model) ------------------------------------ */
/* Model[W, E, KV] from 4*n_layer layer matrices (per layer: attn.c_attn,
 * attn.c_proj, mlp.c_fc, mlp.c_proj, gpt2t.mojo:84-96), the tied wte/head
 * matrix and the float32 parameters in Model.small order (per layer
 * ln_1.w, ln_1.b, c_attn.b, c_proj.b, ln_2.w, ln_2.b, c_fc.b, mlp.c_proj.b,
 * then wpe [1024][768], ln_f.w, ln_f.b; gpt2t.mojo:255-267). The matrices
 * stay owned by the caller and must outlive the model. */
llmq_status llmq_model_create(llmq_ctx *ctx, int n_layer, llmq_weight *const *mats, const llmq_weight *head,
                              const float *small_host, int kv_kind, int max_t, llmq_model **out);
llmq_status llmq_model_free(llmq_model *m);
/* Model.forward (gpt2t.mojo:329-342): tokens at positions pos0.., logits of
 * the last token into logits_dev (may be NULL) and its argmax into
 * *argmax_host (may be NULL). */
llmq_status llmq_model_forward(llmq_ctx *ctx, llmq_model *m, const int *tokens_host, int T, int pos0,
                               float *logits_dev, int *argmax_host);
/* Model.forward_all (gpt2t.mojo:449-459): logits_dev[T, V] for every
 * position of tokens (from position 0). */
llmq_status llmq_model_forward_all(llmq_ctx *ctx, llmq_model *m, const int *tokens_host, int T,
                                   float *logits_dev);
/* Greedy generate (gpt2t.mojo:942-980, without the stop at EOT): forward
 * the prompt, then `steps` argmaxes with a decode step between consecutive
 * ones; ids into out_ids_host[steps]. Each decode step is one CUDA graph
 * launch. */
llmq_status llmq_generate(llmq_ctx *ctx, llmq_model *m, const int *prompt_host, int n_prompt, int steps,
                          int *out_ids_host);
/* generate with device-resident prompt and ids, asynchronous on the
 * context's stream (no host synchronisation): the same steps as
 * llmq_generate. */
llmq_status llmq_generate_async(llmq_ctx *ctx, llmq_model *m, const int *prompt_dev, int n_prompt, int steps,
                                int *ids_dev);

/* ---- sampling (gpt2t.mojo:775-834) ---- */
/* Rng(seed) (gpt2t.mojo:775-781): the xorshift64* state seed *
 * 0x9E3779B97F4A7C15 + 1, wrapping. */
unsigned long long llmq_rng_init(long long seed);
/* top_k (gpt2t.mojo:800-815): ids of the k largest of logits_dev[0, V) in
 * descending order, an equal logit ordered by the lower id first; k <= 0 or
 * k >= V gives all V. Writes min(k, V) ids (V for k <= 0) to ids_dev.
 * Asynchronous on the context's stream. V <= 2^24. */
llmq_status llmq_top_k(llmq_ctx *ctx, const float *logits_dev, int V, int k, int *ids_dev);
/* sample (gpt2t.mojo:818-834): temperature <= 0 is the argmax (first index
 * of the largest logit; *rng_dev untouched); otherwise one draw from the top
 * k (k <= 0: all V) with weights exp((logit - max) / temperature), summed in
 * order in float32, advancing the device Rng state *rng_dev. The id goes to
 * *id_dev. Asynchronous on the context's stream. V <= 2^24. */
llmq_status llmq_sample(llmq_ctx *ctx, const float *logits_dev, int V, float temperature, int k,
                        unsigned long long *rng_dev, int *id_dev);
/* generate (gpt2t.mojo:965-980) with sample in place of the argmax, without
 * the stop at EOT: `steps` ids into out_ids_host; *rng_state (host) is the
 * Rng state, read before and written back after. temperature <= 0 is
 * llmq_generate. The draws run on the device after each head; in
 * LLMQ_MODE_PERSISTENT each decode step is one launch of the persistent
 * kernel, otherwise a CUDA graph launch (or eager in LLMQ_MODE_EAGER). */
llmq_status llmq_generate_sampled(llmq_ctx *ctx, llmq_model *m, const int *prompt_host, int n_prompt, int steps,
                                  float temperature, int k, unsigned long long *rng_state, int *out_ids_host);
/* Per-operation timers of the persistent decode kernel, as the reference's
 * --profile (gpt2t.mojo:121-142, print_profile :461-483): with profiling on,
 * CTA 0 (which also runs head 0's attention) and CTA grid/2 add the SM
 * cycles of each phase of every step to 2 x 20 counters, in this order:
 * embed, QKV wait, QKV (LN1 + quantize + GEMV), attention (KV store +
 * attend), PROJ wait, PROJ, FC wait, FC (LN2 + GEMV + GELU), FCPROJ wait,
 * FCPROJ, head wait, head (LN_f + GEMV), argmax, ring-slot waits (also
 * inside the phases), steps, then inside the phases: LayerNorm, quantize,
 * integer dots, float epilogue. profile_read copies them (n >= 40). */
llmq_status llmq_model_profile(llmq_ctx *ctx, llmq_model *m, int enable);
llmq_status llmq_model_profile_read(llmq_ctx *ctx, llmq_model *m, long long *cycles_host, int n, int reset);
/* Waits for the context's stream and reports a bounded device-side wait of
 * the model's persistent kernel that gave up (LLMQ_ERR_TIMEOUT). */
llmq_status llmq_model_check(llmq_ctx *ctx, llmq_model *m);
/* The cudaStream_t the context issues its work on. */
void *llmq_stream(const llmq_ctx *ctx);
/* How decode steps run (replacing the reference's per-token thread team,
 * team.mojo:36-82, and gpt2t.mojo:350-447's single parallel region):
 * LLMQ_MODE_PERSISTENT (default when the formats allow it: int4-g32 A16
 * layers, a per-channel int8 A16 head, QuantKV[8] or IntAttnKV) runs a whole
 * generation as one persistent kernel over all SMs that exchange activations
 * through global memory; LLMQ_MODE_CLUSTER (768-wide, 12-head models with
 * QuantKV[8]) runs it as one launch of 16-CTA thread-block clusters, the
 * layers inside one cluster exchanging through distributed shared memory;
 * LLMQ_MODE_GRAPH replays each step as a captured CUDA graph of one-token
 * kernels; LLMQ_MODE_EAGER launches those kernels one by one. All give the
 * same ids and logits. Returns LLMQ_ERR_UNSUPPORTED if the model cannot run
 * `mode`. */
#define LLMQ_MODE_EAGER 0
#define LLMQ_MODE_GRAPH 1
#define LLMQ_MODE_PERSISTENT 2
#define LLMQ_MODE_CLUSTER 3
llmq_status llmq_model_set_mode(llmq_model *m, int mode);
int llmq_model_mode(const llmq_model *m);

/* ---- saved weights and GGUF files ------------------------------------------ */
/* Replaces save_model (gpt2t.mojo:617-643): writes the model's weights, as
 * converted, to path in the reference's saved-model layout (serialize.mojo
 * encoding: 8-byte little-endian integers, length-prefixed strings): magic,
 * version 1, the layer and head format names, the head, the 48 layer
 * matrices (WeightMatrix.save), then the float32 tensors. 12-layer models
 * with affine or dense weights. */
llmq_status llmq_model_save(llmq_ctx *ctx, const llmq_model *m, const char *path);
/* Replaces load_saved (gpt2t.mojo:667-698): a model from a file written by
 * llmq_model_save or by the reference's --save, with the cache kv_kind and
 * max_t positions. The model owns its weights (freed by llmq_model_free). */
llmq_status llmq_model_load(llmq_ctx *ctx, const char *path, int kv_kind, int max_t, llmq_model **out);
/* Replaces load_gguf (gpt2t.mojo:728-760) with GGUFFile (gguf.mojo:519-636):
 * a llama.cpp GGUF file of GPT-2 124M, its matrices used as stored (tied
 * token_embd head), the small tensors float32. The model owns its weights. */
llmq_status llmq_model_load_gguf(llmq_ctx *ctx, const char *path, int kv_kind, int max_t, llmq_model **out);

/* ---- perplexity harness ---------------------------------------------------- */
/* Replaces score_rows (gpt2t.mojo:1042-1097) for rows [r0, r1) of a window's
 * logits ([rows][V], device): stats_dev[k * stride + (r - r0)] in float64 for
 * k = 0 NLL (-log p(target), log_sum_exp as gpt2t.mojo:1030-1039), 1 NLL
 * under base_dev (the float32 model's logits; may be NULL), 2 top-1
 * agreement, 3 KL(base || model) in nats, 4 max and 5 sum of |logit
 * differences|. targets_dev[r] is row r's next token. */
llmq_status llmq_score_rows(llmq_ctx *ctx, const float *logits_dev, const float *base_dev, const int *targets_dev, int V,
                            int r0, int r1, double *stats_dev, int stride);

/* ---- batched greedy decode (independent sequences) ----------------------- */
/* No counterpart in the reference, which decodes one sequence at a time
 * (generate, gpt2t.mojo:942-980). State for the greedy decode of up to
 * max_seqs independent sequences with prompts of up to max_prompt tokens,
 * each with its own QuantKV[8] cache of the model's max_t positions. The
 * model must use the QuantKV[8] cache. */
typedef struct llmq_batch llmq_batch;
llmq_status llmq_batch_create(llmq_ctx *ctx, llmq_model *m, int max_seqs, int max_prompt, llmq_batch **out);
llmq_status llmq_batch_free(llmq_batch *b);
/* Which kernel runs the batched one-token matmuls (the layers' BLOCKED
 * int4-g32 rows and the per-channel int8 head; dot_row_i16 per sequence,
 * tensor.mojo:522-566): AUTO (the lane-mode tcgen05 GEMM from 16 sequences
 * on), CUDA_CORE (the dp2a batched GEMVs) or TCGEN05 (the GEMM for any
 * count). Results are identical; no counterpart in the reference, which
 * decodes one sequence at a time. */
#define LLMQ_BATCH_AUTO 0
#define LLMQ_BATCH_CUDA_CORE 1
#define LLMQ_BATCH_TCGEN05 2
llmq_status llmq_batch_set_kernel(llmq_batch *b, int kind);
/* generate (gpt2t.mojo:942-980, without the stop at EOT) for B sequences at
 * once: prompts [B][n_prompt] and out_ids [B][steps] on the host. Each
 * sequence's ids are those of llmq_generate on that sequence alone: its
 * prompt runs through the several-token path, its later tokens through the
 * one-token arithmetic. */
llmq_status llmq_batch_generate(llmq_ctx *ctx, llmq_batch *b, const int *prompts, int B, int n_prompt, int steps,
                                int *out_ids);
/* The same with device prompts and device ids, enqueued on the context's
 * stream without synchronising (for timing with inputs already in HBM). */
llmq_status llmq_batch_generate_async(llmq_ctx *ctx, llmq_batch *b, const int *prompts_dev, int B, int n_prompt,
                                      int steps, int *ids_dev);

#ifdef __cplusplus
}
#endif

#endif /* LLMQ_H */
