/* qwen3_b200.h -- C ABI of the B200 (sm_100a) Qwen3 4-bit decode library.
 *
 * Drop-in boundary for base-mlx's decode hot path.  Every entry point replaces
 * one piece of the Rust crate base-mlx-core (paths relative to the
 * flakerimi/base-mlx project root):
 *
 *   qw_model_load            Architecture::load / Qwen3::load      model.rs:36-43, model/qwen3.rs:194-295
 *   qw_model_init_random     (benchmark helper: seeded random-init weights in the same layout)
 *   qw_cache_new             Architecture::new_cache / KvCache::new model.rs:45-51, model/qwen3.rs:127-129
 *   qw_cache_reset           ArchitectureCache::reset              model.rs:88-96, model/qwen3.rs:130-134
 *   qw_cache_truncate        ArchitectureCache::truncate           model.rs:98-106, model/qwen3.rs:150-161
 *   qw_forward               Architecture::forward / forward_multi model.rs:53-80, model/qwen3.rs:297-312
 *   qw_kv_slice_update       mlx_ext::slice_update on a cache tensor mlx_ext.rs:36-64
 *   qw_quantized_matmul      mlx_rs::ops::quantized_matmul(transpose=true, 64, 4) model/qwen3.rs:30-41
 *   qw_generate_greedy       LoadedModel::generate_text (greedy)   engine.rs:149-201
 *   qw_generate_sampled      LoadedModel::generate_text, temperature/top-p pick_next engine.rs:149-201,203-263
 *   qw_sample_topp           LoadedModel::pick_next on one logits row (device)         engine.rs:195-263
 *   qw_spec_generate         speculative::generate                 speculative.rs:57-286
 *   qw_check_compatible      speculative::check_compatible         speculative.rs:40-54
 *
 * Conventions
 *   - every function returns an int status: QW_OK (0) or a negative QW_ERR_*
 *     code; qw_last_error() copies the thread's last error message.  The codes
 *     map onto the crate's Error enum (error.rs:6-32): QW_ERR_MODEL_LOAD ->
 *     Error::ModelLoad, QW_ERR_INVALID_CONFIG -> Error::InvalidConfig, every
 *     other code -> Error::Inference.
 *   - handles are opaque and owned by the library; one handle is used by one
 *     thread at a time (the crate serialises requests behind a Mutex,
 *     base-mlx-server/src/state.rs:18-27).
 *   - token ids are uint32; logits are bf16 bit patterns (uint16).
 *   - pointers named *_host are host memory; qw_quantized_matmul takes device
 *     pointers (it stands in for an op on MLX arrays that already live on the GPU).
 *   - there is no CPU fallback: without a usable sm_100 GPU every compute call
 *     fails with QW_ERR_CUDA.
 */
#ifndef QWEN3_B200_H
#define QWEN3_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QW_API __attribute__((visibility("default")))
#else
#define QW_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QW_OK 0
#define QW_ERR_INVALID_ARG -1     /* bad pointer / size / shape */
#define QW_ERR_INVALID_CONFIG -2  /* Error::InvalidConfig */
#define QW_ERR_MODEL_LOAD -3      /* Error::ModelLoad (missing / unmapped tensors, io) */
#define QW_ERR_INFERENCE -4       /* Error::Inference */
#define QW_ERR_KV_EXHAUSTED -5    /* Error::Inference("KV cache exhausted ...") qwen3.rs:423-428 */
#define QW_ERR_CUDA -6            /* CUDA runtime error or no usable GPU */
#define QW_ERR_UNSUPPORTED -7     /* e.g. bits != 4, group_size != 64, model_type != qwen3 */
#define QW_ERR_DEVICE_FLAG -8     /* a kernel raised its device-side error flag */

typedef struct qw_model qw_model;
typedef struct qw_cache qw_cache;

typedef struct qw_model_info {
    int32_t num_layers, hidden, intermediate, num_heads, num_kv_heads, head_dim;
    int32_t vocab, tied_embeddings, tp_rank, tp_size;
    float rms_eps, rope_theta;
    uint64_t weight_bytes;  /* device bytes of this rank's quantized weights + norms */
} qw_model_info;

typedef struct qw_gen_stats {
    int32_t prompt_tokens;
    int32_t completion_tokens; /* counts a terminating EOS, as GenerationResult does (engine.rs:178) */
    int32_t finish_reason;     /* 0 = "length", 1 = "stop" */
    int32_t pad;
    double prefill_ms, decode_ms; /* device time (CUDA events) */
} qw_gen_stats;

typedef struct qw_spec_stats {
    int32_t iters, proposed, accepted, completion_tokens;
    int32_t finish_reason, pad;
    double prefill_ms, total_ms;         /* device time of the whole call */
    double draft_ms_mean, verify_ms_mean, accept_ms_mean; /* speculative.rs:242-264 */
} qw_spec_stats;

/* Copy the calling thread's last error message (NUL-terminated, truncated to len). */
QW_API int qw_last_error(char* buf, size_t len);

/* Library build / runtime version string. */
QW_API int qw_version(char* buf, size_t len);

/* ---- models ---------------------------------------------------------- */

/* Load an MLX-format Qwen3 checkpoint directory (config.json + *.safetensors).
 * tp_rank/tp_size select this rank's shard of a tensor-parallel split (1 = whole model). */
QW_API int qw_model_load(const char* dir, int device, int tp_rank, int tp_size, qw_model** out);

/* Seeded random-init model with the tensors of `config_json` (a config.json
 * string), generated on the device: N(0,0.02) weights quantized affine 4-bit
 * g64; norm_mode 0 = norm weights 1.0, 1 = bf16(1 + N(0,0.1)). */
QW_API int qw_model_init_random(const char* config_json, uint64_t seed, int norm_mode, int device,
                                int tp_rank, int tp_size, qw_model** out);

/* Frees the model and every cache still attached to it. */
QW_API int qw_model_free(qw_model* m);
QW_API int qw_model_info_get(const qw_model* m, qw_model_info* out);

/* Copy one named tensor of this rank (MLX name, e.g. "model.layers.0.mlp.up_proj.scales")
 * to host memory.  bytes must equal the tensor's size. */
QW_API int qw_model_export_tensor(const qw_model* m, const char* name, void* dst_host, size_t bytes);

/* The CUDA stream the model's work runs on (cudaStream_t as void*). */
QW_API int qw_model_stream(const qw_model* m, void** stream_out);

/* Tensor parallel (no reference counterpart: base-mlx has no distributed path).
 * qw_tp_unique_id writes a fresh NCCL unique id (128 bytes) for rank 0 to share
 * with the other ranks (any host channel: torch.distributed, a file, MPI). */
QW_API int qw_tp_unique_id(void* out, size_t bytes);

/* Tensor parallel: attach an NCCL communicator (ncclUniqueId bytes, 128) to a
 * model loaded with tp_size > 1.  Must be called on every rank before forward. */
QW_API int qw_model_tp_attach(qw_model* m, const void* nccl_unique_id, int rank, int size);

/* Tensor parallelism without a library collective on the decode path: each
 * rank allocates an exchange block and returns its CUDA IPC handle (64 bytes)
 * with qw_tp_exchange_handle; after the ranks have shared their handles over
 * the host (rank order, size x 64 bytes), qw_tp_exchange_open maps every
 * peer's block.  With QW_TP_PUSH=1 set at open time the o_proj / down_proj
 * reductions of steps of up to 8 rows then run over peer memory: the GEMV
 * stores its fp32 partial rows into
 * every rank's block and raises an epoch flag there, one small kernel per rank
 * waits for the flags (bounded), sums the partials in rank order and adds them
 * to the residual (NCCL keeps the prefill reductions and the lm_head argmax).
 * Measured slightly slower than NCCL on Qwen3-32B decode at 2 and 4 GPUs, so
 * NCCL is the default.  No reference counterpart. */
QW_API int qw_tp_exchange_handle(qw_model* m, void* handle_out, size_t bytes);
QW_API int qw_tp_exchange_open(qw_model* m, const void* handles, size_t bytes);

QW_API int qw_check_compatible(const qw_model* target, const qw_model* draft);

/* ---- KV cache --------------------------------------------------------- */

QW_API int qw_cache_new(qw_model* m, int max_pos, qw_cache** out);
QW_API int qw_cache_free(qw_cache* c);
QW_API int qw_cache_reset(qw_cache* c);
/* Roll back to the first new_len positions (no-op when already shorter). */
QW_API int qw_cache_truncate(qw_cache* c, int new_len);
QW_API int qw_cache_len(const qw_cache* c, int* out);

/* cache[layer].{k|v}[:, start:stop, :] = update_host ([kv_heads_local, stop-start, head_dim] bf16). */
QW_API int qw_kv_slice_update(qw_cache* c, int layer, int which_v, const uint16_t* update_host,
                              int start, int stop);
/* Read cache[layer].{k|v}[:, start:stop, :] back to the host. */
QW_API int qw_kv_read(const qw_cache* c, int layer, int which_v, uint16_t* dst_host, int start, int stop);

/* ---- forward ------------------------------------------------------------ */

/* Run `n` tokens through the model at the cache's current length and extend it.
 * all_rows = 0 -> Architecture::forward (last row), 1 -> forward_multi (every row).
 * logits_out_host (optional) receives bf16 logits [rows, vocab_local];
 * argmax_out_host (optional) receives the argmax of each returned row. */
QW_API int qw_forward(qw_model* m, qw_cache* c, const uint32_t* ids_host, int n, int all_rows,
                      uint16_t* logits_out_host, uint32_t* argmax_out_host);

/* Diagnostics (no reference counterpart; an MLX caller can inspect any
 * intermediate array): Architecture::forward of `n` tokens that also copies
 * the residual stream after the embedding and after every layer to
 * residual_out_host (bf16 [num_layers + 1][n][hidden]), the residual after
 * every layer's attention block to mid_out_host (optional, bf16
 * [num_layers][n][hidden]) and every layer's attention output (the o_proj
 * input) to attn_out_host (optional, bf16 [num_layers][n][heads * head_dim]).
 * Same decode / prefill path as qw_forward; allocates and frees a device
 * buffer for the copies. */
QW_API int qw_forward_trace(qw_model* m, qw_cache* c, const uint32_t* ids_host, int n, uint16_t* residual_out_host,
                            uint16_t* mid_out_host, uint16_t* attn_out_host, uint16_t* logits_out_host,
                            uint32_t* argmax_out_host);

/* Diagnostics: timing stamps of the last persistent decode-step launch, when
 * the model was created with the environment variable QW_MK_PROFILE set
 * (otherwise *written = 0).  Layout: uint64 globaltimer ns
 * [cta][phase][16], 514 phases per CTA (phase 5l + {0..4} = layer l's q|k|v,
 * attention, o_proj, gate|up, down_proj; 5L = lm_head; slot k = 0 phase
 * barrier passed, 1 staging done, 2 first weight stage ready, 3 own weight
 * loop done, 4 all warps done, 5 epilogue done, 6 arriving, 8 / 9 weight loop
 * entered / left by warp 0; attention items use slots 1-7 for their steps).
 * No reference counterpart. */
QW_API int qw_debug_decode_stamps(const qw_model* m, void* dst_host, size_t bytes, size_t* written);

/* ---- generation --------------------------------------------------------- */

/* Greedy generation (temperature 0).  out_host receives up to max_new ids (a
 * terminating EOS is not written); *n_out = ids written.  eos == NULL uses the
 * model config's eos ids (or 151645/151643 when the config has none). */
QW_API int qw_generate_greedy(qw_model* m, const uint32_t* prompt_host, int n_prompt, int max_new,
                              const uint32_t* eos, int n_eos, uint32_t* out_host, int* n_out,
                              qw_gen_stats* stats);

/* Speculative sampling (temperature > 0): the reference falls back to plain
 * sampled decoding there (speculative.rs:65-69); this runs the rejection rule
 * on the device over the sampled pick's distributions (engine.rs:203-263:
 * softmax of logits / temperature, top-p nucleus).  The first token and each
 * of the k drafted tokens per iteration are drawn like qw_generate_sampled;
 * drafted token i is accepted with probability min(1, P_target / P_draft) of
 * that token; at the first rejection the emitted token is drawn from
 * max(0, P_target - P_draft), after k acceptances from the target's next row,
 * so every token follows the target's distribution.  Draws come from the
 * counter-based generator seeded by `seed` (iteration t, slot i: draft pick
 * 64t + i, acceptance 64t + 16 + i, residual / bonus 64t + 32; first token
 * 2^40).  temperature <= 0 runs qw_spec_generate's greedy loop.  Target and
 * draft must hold the whole vocabulary (no vocabulary-parallel lm_head). */
QW_API int qw_spec_generate_sampled(qw_model* target, qw_model* draft, const uint32_t* prompt_host, int n_prompt,
                                    int max_new, int k, float temperature, float top_p, uint64_t seed,
                                    const uint32_t* eos, int n_eos, uint32_t* out_host, int* n_out,
                                    qw_spec_stats* stats);

/* Batched greedy generation (benchmark config 5 at batch 8; the reference
 * serves one request at a time, model.rs:21-108, so this has no single
 * reference counterpart: it is generate_text's greedy loop, engine.rs:149-201,
 * for nseq independent requests at once).  nseq (1..8) prompts, concatenated
 * in prompts_host with lengths n_prompt[nseq], each decoded in its own cache
 * caches[nseq] (distinct, of this model; reset to the prompt first).  Every
 * decode step carries all nseq sequences through the weights once; each
 * sequence's tokens equal its batch-1 greedy run.  out_host is [nseq][max_new]
 * (row stride max_new), n_out[b] = ids written for sequence b (a terminating
 * EOS is not written); stats: prompt / completion tokens summed over the
 * batch, prefill_ms of all prompts, decode_ms of the batched loop. */
QW_API int qw_generate_greedy_batch(qw_model* m, qw_cache* const* caches, int nseq, const uint32_t* prompts_host,
                                    const int* n_prompt, int max_new, const uint32_t* eos, int n_eos,
                                    uint32_t* out_host, int* n_out, qw_gen_stats* stats);

/* One batched decode step: token ids_host[b] of sequence b at caches[b]'s next
 * position (nseq 1..8, distinct caches); logits_out_host [nseq][vocab] bf16
 * (may be NULL) and argmax_out_host [nseq] (may be NULL).  Each cache grows
 * by one position. */
QW_API int qw_forward_batch(qw_model* m, qw_cache* const* caches, int nseq, const uint32_t* ids_host,
                            uint16_t* logits_out_host, uint32_t* argmax_out_host);

/* Greedy speculative decoding: k drafted tokens per iteration, one (k+1)-row
 * target verify, on-device accept and rollback.  k = 3 reproduces the
 * reference loop (SPEC_K = 4).  With forced_seq != NULL and force_p > 0 each
 * drafted token is replaced, with probability force_p, by forced_seq[pos]
 * (the plain-greedy target sequence) -- the benchmark's acceptance control. */
QW_API int qw_spec_generate(qw_model* target, qw_model* draft, const uint32_t* prompt_host, int n_prompt,
                            int max_new, int k, float force_p, uint64_t seed,
                            const uint32_t* forced_seq_host, int n_forced, const uint32_t* eos, int n_eos,
                            uint32_t* out_host, int* n_out, qw_spec_stats* stats);

/* Sampled generation (engine.rs:149-263 with SamplingParams temperature,
 * top_p, seed; top_k and repetition_penalty are not read by the reference's
 * pick_next either).  temperature <= 0 is greedy, as in the reference.  Each
 * pick draws u = top 24 bits of splitmix64(seed ^ splitmix64(i)) / 2^24 with i
 * the number of tokens already picked, or i = 0 for every pick when
 * same_draw_each_token != 0 (the reference seeds a fresh generator from the
 * same seed at every token, so it reuses one draw).  Outputs as in
 * qw_generate_greedy.  Needs the whole vocabulary on the rank (no untied
 * vocab-parallel lm_head). */
QW_API int qw_generate_sampled(qw_model* m, const uint32_t* prompt_host, int n_prompt, int max_new,
                               float temperature, float top_p, uint64_t seed, int same_draw_each_token,
                               const uint32_t* eos, int n_eos, uint32_t* out_host, int* n_out, qw_gen_stats* stats);

/* One pick from a device bf16 logits row of `vocab` entries with the draw
 * counter `counter` (same generator as qw_generate_sampled); *token_out
 * (device int32).  `scratch` is a device buffer of QW_SAMPLE_SCRATCH_BYTES(vocab)
 * bytes, zero before its first use, that the call leaves ready for the next
 * one (its head is the control block of the grid the pick runs on); calls that
 * share a scratch buffer must not overlap on the GPU.  logits and scratch must
 * be 16-byte aligned.  stream may be NULL. */
#define QW_SAMPLE_SCRATCH_BYTES(vocab) (16384u + 4u * (size_t)(vocab))
QW_API int qw_sample_topp(const void* logits, int vocab, float temperature, float top_p, uint64_t seed,
                          uint64_t counter, void* scratch, int32_t* token_out, void* stream);

/* ---- standalone op ----------------------------------------------------- */

/* y[M,N] (bf16) = x[M,K] (bf16) . dequant(W)^T with W uint32 [N,K/8],
 * scales/biases bf16 [N,K/64]; device pointers; stream may be NULL (default
 * stream).  Only group_size 64 and bits 4 are supported.  At M <= 8 the kernel
 * is launched so that it may start while the previous kernel on the stream
 * drains; it then only prefetches into L2 until that kernel has completed, so
 * operands that kernel writes are read correctly.  The weights' tensor-map
 * descriptors are cached per (w, scales, biases, N, K). */
QW_API int qw_quantized_matmul(const void* x, const void* w, const void* scales, const void* biases,
                               void* y, int M, int N, int K, int group_size, int bits, void* stream);

/* ---- standalone op without workspace ------------------------------------ */

/* Scratch of qw_quantized_matmul_argmax_static: 131072 per-CTA maxima of
 * 8 bytes (1 MiB) in a static device array of the library. */
#define QW_STATIC_AMAX_SLOTS 131072

/* Greedy logits head that allocates no memory: y[M,N] (bf16, optional) =
 * x[M,K] . dequant(W)^T as in qw_quantized_matmul, plus argmax_dev[m] (int32,
 * device) = the lowest index of row m's largest bf16 logit.  No counterpart in
 * the reference (mlx-rs allocates every intermediate through MLX's allocator);
 * it serves callers that cannot allocate device memory on the call: a host
 * whose device memory is fully reserved up front (weights, KV arena), or one
 * that must not synchronise the device, which cudaMalloc/cudaFree can do.
 *   - Its per-CTA maxima live in a file-scope device array of
 *     QW_STATIC_AMAX_SLOTS slots; M (1..8) * ceil(N / 16) must not exceed it,
 *     otherwise QW_ERR_INVALID_ARG with the sizes in the message
 *     (Qwen3's 151936-entry vocabulary uses 75968 slots at M = 8).
 *   - K is bounded by the GEMV's shared-memory staging of a whole 16-row
 *     slab: up to 17984 at M = 1, 10304 at M = 5, 7808 at M = 8; a longer
 *     row is QW_ERR_INVALID_ARG with K and M in the message.
 *   - The first call on each device (that device current) looks the array's
 *     address up once; make that first call before any stream capture.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine.
 *   - Calls that overlap on the GPU on one device (two streams, two host
 *     threads) share the array and race; serialise them.
 * Only group_size 64 and bits 4 are supported. */
QW_API int qw_quantized_matmul_argmax_static(const void* x, const void* w, const void* scales,
                                             const void* biases, void* y_or_null, int* argmax_dev, int M,
                                             int N, int K, int group_size, int bits, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QWEN3_B200_H */
