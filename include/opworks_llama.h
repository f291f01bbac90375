/* C ABI of the OpWorks-B200 Llama runtime (libopworks_llama.so).
 *
 * The first eleven entry points are the ones OpWorks' src/llama_c_api.cu
 * exports (same names, signatures, return values and error convention:
 * guarded calls return -1 / NULL, copy at most err_len - 1 bytes of the
 * message plus a NUL into `err`, and set a thread-local message readable with
 * opw_llama_last_error()). Sessions must be destroyed before their model.
 * prefill / decode_step block until the next token is on the host.
 *
 * The opw_llama_batch_* / *_ex / set_device entry points are new API: a
 * batched engine (many sequences per forward over a paged KV cache, CUDA
 * graph per batch size, device-side greedy or top-p sampling).
 */
#ifndef OPWORKS_LLAMA_H
#define OPWORKS_LLAMA_H

#include <stdint.h>

/* Only the C ABI is exported; the libraries are built with hidden default
 * visibility so two of them (or the reference's library) can share a process. */
#ifndef OPW_API
#define OPW_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* --- OpWorks interface (src/llama_c_api.cu:54-159) --- */

/* replaces opw_llama_load (src/llama_c_api.cu:57-73): float32 or bfloat16 pack */
OPW_API void *opw_llama_load(const char *pack_path, char *err, int err_len);
/* replaces opw_llama_free (src/llama_c_api.cu:75) */
OPW_API void opw_llama_free(void *model);
/* replaces opw_llama_create_session (src/llama_c_api.cu:77-91); max_seq_len in (0, 8192] */
OPW_API void *opw_llama_create_session(void *model, int max_seq_len, char *err, int err_len);
/* replaces opw_llama_destroy_session (src/llama_c_api.cu:93) */
OPW_API void opw_llama_destroy_session(void *session);
/* replaces opw_llama_reset_session (src/llama_c_api.cu:95-102) */
OPW_API int opw_llama_reset_session(void *session, char *err, int err_len);
/* replaces opw_llama_prefill (src/llama_c_api.cu:105-116): first greedy token or -1 */
OPW_API int opw_llama_prefill(void *session, const int32_t *tokens, int n, char *err, int err_len);
/* replaces opw_llama_decode_step (src/llama_c_api.cu:119-126): next greedy token or -1 */
OPW_API int opw_llama_decode_step(void *session, int32_t prev_token, char *err, int err_len);
/* replaces opw_llama_is_eos (src/llama_c_api.cu:129-136): 1, 0 or -1 */
OPW_API int opw_llama_is_eos(void *session, int32_t token, char *err, int err_len);
/* replaces opw_llama_last_logits (src/llama_c_api.cu:139-149): n must be vocab_size */
OPW_API int opw_llama_last_logits(void *session, float *out, int n, char *err, int err_len);
/* replaces opw_llama_vocab_size (src/llama_c_api.cu:151-154); not guarded, as in OpWorks */
OPW_API int opw_llama_vocab_size(void *session);
/* replaces opw_llama_last_error (src/llama_c_api.cu:156) */
OPW_API const char *opw_llama_last_error(void);

/* --- extensions (no counterpart in OpWorks) --- */

/* Select the CUDA device used by subsequent loads on this thread. */
OPW_API int opw_llama_set_device(int device);
/* Load keeping only some weight precisions: bit 1 = 16-bit (fast path: fp16
 * words for float32 packs, or bf16 with OPWORKS_FAST_WEIGHTS=bf16; the pack's
 * bf16 words for bfloat16 packs), 2 = fp32 (accurate GEMV), 4 = tf32 hi/lo
 * (accurate GEMM); 0 = default.
 * max_positions sizes the RoPE table (>= the longest session). */
OPW_API void *opw_llama_load_ex(const char *pack_path, unsigned weight_sets, int max_positions, char *err, int err_len);
/* Model hyper-parameters: out[0..7] = layers, hidden, intermediate, q heads,
 * kv heads, head dim, vocab, device. */
OPW_API int opw_llama_model_info(void *model, int32_t *out8, char *err, int err_len);

/* Batched engine: max_batch sequences (slots) of up to max_seq_len tokens
 * each over one paged KV cache. precision: 0 = accurate (fp32), 1 = fast
 * (16-bit weights and two-term 16-bit GEMM activations, fp32 residual / KV /
 * softmax).
 * prefill_rows: prefill chunk size (0 = max_seq_len). */
OPW_API void *opw_llama_create_batch(void *model, int max_batch, int max_seq_len, int precision, int prefill_rows, char *err,
                             int err_len);
OPW_API void opw_llama_destroy_batch(void *batch);
/* Tensor parallelism (extension): opw_llama_nccl_unique_id writes a 128-byte
 * NCCL communicator id (one rank creates it and shares it with the others);
 * opw_llama_create_batch_tp creates this rank's fast-path engine of a
 * tp_world-way tensor-parallel group (one process per GPU, every rank loads
 * the full model): rank r owns query heads [r qh / tp_world, ...), the
 * matching KV heads and MLP columns [r I / tp_world, ...), and the ranks sum
 * the o and down projections with one NCCL all-reduce each per layer. Every
 * rank must make the same calls with the same arguments (prefill, decode),
 * and returns the same tokens. Requires libnccl.so.2. */
OPW_API int opw_llama_nccl_unique_id(char *out128, char *err, int err_len);
OPW_API void *opw_llama_create_batch_tp(void *model, int max_batch, int max_seq_len, int prefill_rows, int tp_rank,
                                        int tp_world, const char *nccl_id, char *err, int err_len);
/* Fused peer-to-peer reduction of a tensor-parallel batch (extension; one
 * GPU per rank, peers reachable over NVLink): opw_llama_batch_tp_ipc_handle
 * writes 128 bytes (CUDA IPC handles of this rank's receive buffer and
 * arrival counters); after every rank has them, each calls
 * opw_llama_batch_tp_open_peers with the world's handles concatenated in rank
 * order (world x 128 bytes). From then on the o and down projections store
 * their partial tiles into every rank's receive buffer from the GEMM
 * epilogue and one kernel per projection sums them in rank order, instead of
 * an NCCL all-reduce (environment OPWORKS_TP_P2P=0 keeps NCCL). */
OPW_API int opw_llama_batch_tp_ipc_handle(void *batch, char *out128, char *err, int err_len);
OPW_API int opw_llama_batch_tp_open_peers(void *batch, const char *handles, char *err, int err_len);
/* The shard plan of tensor-parallel rank `rank` of `world` (pure host
 * arithmetic; include/models/tp_plan.cuh): cfg5 = hidden, intermediate, q
 * heads, kv heads, head dim; out12 = this rank's q heads, kv heads, MLP
 * columns, first QKV rows of its q / k / v heads, q rows, kv rows, first O
 * input column, first interleaved gate/up row, gate/up rows, first down input
 * column. Returns 0, or -1 when the model does not shard `world` ways. */
OPW_API int opw_llama_tp_shard(const int32_t *cfg5, int rank, int world, int64_t *out12, char *err, int err_len);
/* Frees the slot's KV blocks; the slot starts empty. */
OPW_API int opw_llama_batch_reset(void *batch, int slot, char *err, int err_len);
/* Current token count of a slot, or -1. */
OPW_API int opw_llama_batch_length(void *batch, int slot);
/* Appends n prompt tokens to `slot` and returns the next token sampled from
 * the last position: temperature <= 0 -> greedy argmax; otherwise top-p with
 * the uniform `uniform` when >= 0, else a counter-based draw from (seed, 0). */
OPW_API int opw_llama_batch_prefill(void *batch, int slot, const int32_t *tokens, int n, float temperature, float top_p,
                            double uniform, uint64_t seed, char *err, int err_len);
/* One decode step for n slots: prev_tokens[i] is appended to slots[i] and
 * out_tokens[i] receives the next token. temperature / top_p / uniforms /
 * seeds / steps may be NULL (greedy; counter RNG at step 0). Returns 0 / -1. */
OPW_API int opw_llama_batch_decode(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                           const float *temperature, const float *top_p, const double *uniforms,
                           const uint64_t *seeds, const int32_t *steps, int32_t *out_tokens, char *err, int err_len);
/* `steps` decode steps for n slots with no host round trip per step (the
 * host-sync-free multi-step decode the reference's blocking decode_step,
 * include/models/llama.cuh:118-134, does not have): the sampled tokens are
 * fed back on the device and KV blocks for all steps are reserved up front.
 * out_tokens[k * n + i] = row i's token of step k, or -1 after the row
 * emitted eos_id (eos_id < 0: none); out_counts[i] = tokens row i produced up
 * to and including its eos. uniforms, when given, is [steps][n] (one uniform
 * per step); the other arrays are as in opw_llama_batch_decode. The tokens
 * equal those of `steps` single-step calls with the same arguments. */
OPW_API int opw_llama_batch_decode_multi(void *batch, int n, const int32_t *slots, const int32_t *prev_tokens,
                                         const float *temperature, const float *top_p, const double *uniforms,
                                         const uint64_t *seeds, const int32_t *steps0, int steps, int eos_id,
                                         int32_t *out_tokens, int32_t *out_counts, char *err, int err_len);
/* Logits (vocab_size floats) of row `row` of the last step. */
OPW_API int opw_llama_batch_logits(void *batch, int row, float *out, int n, char *err, int err_len);

/* KV-cache inspection (extension; the reference's contiguous cache needs
 * none, include/runtime/kv_cache.cuh:11-35 there). The pool holds 16-token
 * blocks; a per-slot block table maps logical to physical blocks.
 * opw_llama_batch_kv_blocks: physical block ids of `slot` as the kernels see
 * them (the device copy of the table); writes min(count, cap) ids, returns
 * the count or -1.
 * opw_llama_batch_kv_read: K (post-RoPE) and V of positions [pos0, pos0 + n)
 * of `slot` in `layer`, gathered through the device block table, as
 * [n][kv_heads][head_dim] floats each; positions may run up to the end of the
 * slot's last mapped block. Returns 0 / -1.
 * opw_llama_batch_kv_pool: raw physical blocks [block0, block0 + nblocks) of
 * `layer`, [block][kv_heads][16][head_dim] floats each for K and V; returns
 * the pool's block count (nblocks = 0 only asks for it) or -1. */
OPW_API int opw_llama_batch_kv_blocks(void *batch, int slot, int32_t *out, int cap, char *err, int err_len);
OPW_API int opw_llama_batch_kv_read(void *batch, int slot, int layer, int pos0, int n, float *k_out, float *v_out,
                                    char *err, int err_len);
OPW_API int opw_llama_batch_kv_pool(void *batch, int layer, int block0, int nblocks, float *k_out, float *v_out,
                                    char *err, int err_len);

/* The engine's CUDA stream (cudaStream_t), e.g. to record timing events. */
OPW_API void *opw_llama_batch_stream(void *batch);
/* Bytes copied host->device and device->host around one decode step of n
 * rows: out2[0] = h2d, out2[1] = d2h. */
OPW_API int opw_llama_batch_io_bytes(void *batch, int n, int64_t *out2);
/* Per-kernel device time of the last decode step of n rows (re-run eagerly
 * `iters` times with CUDA events between launch groups; lengths are not
 * advanced). Writes up to max_kernels entries: ms_per_step[i],
 * launches_per_step[i] and a NUL-terminated label of at most 31 characters
 * at labels + 32 * i. Returns the number of entries, or -1. */
OPW_API int opw_llama_batch_profile(void *batch, int n, int iters, float *ms_per_step, int32_t *launches_per_step,
                            char *labels, int max_kernels, char *err, int err_len);

#ifdef __cplusplus
}
#endif

#endif /* OPWORKS_LLAMA_H */
