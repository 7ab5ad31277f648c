/*
 * b200ops.h -- C-ABI of libb200ops.so, the sm_100a kernels behind the
 * tensor-parallel Qwen3 decoder forward path of nano-vllm-diy.
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise; tensors are
 *     bf16 ("void*"), int32 (block tables, cu_seqlens, slot mapping) or int64
 *     (token ids, positions) as documented per argument.
 *   - Strides are in ELEMENTS between consecutive rows (tokens).
 *   - Calls launch on `stream` and return immediately; nothing is allocated
 *     and nothing synchronises, so every call can be captured in a CUDA graph.
 *   - Return value: B200_OK (0) or a negative status; b200_last_error()
 *     returns the message of the calling thread's last failure.
 *   - Kernels never trap.  Out-of-range slot / block-table entries and
 *     timed-out waits set bits of a per-device error word instead, readable
 *     with b200_device_error() (which synchronises the device).
 *
 * Reference interfaces are cited as path:line inside DestineG/nano-vllm-diy.
 */
#ifndef B200OPS_H_
#define B200OPS_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ABI_VERSION 1

#define B200_OK 0
#define B200_ERR_INVALID (-1)     /* bad shape, stride, alignment or null pointer */
#define B200_ERR_UNSUPPORTED (-2) /* shape outside what the kernels implement */
#define B200_ERR_CUDA (-3)        /* a CUDA runtime / driver call failed */
#define B200_ERR_WORKSPACE (-4)   /* caller-provided workspace too small */
#define B200_ERR_PEER (-5)        /* tensor-parallel communicator not set up */

/* device error word bits (b200_device_error) */
#define B200_DEVERR_MBAR_TIMEOUT 1u
#define B200_DEVERR_PEER_TIMEOUT 2u
#define B200_DEVERR_BAD_INDEX 4u

typedef struct CUstream_st* b200_stream_t; /* == cudaStream_t */

const char* b200_last_error(void);
int b200_version(void);

/* Kernels launched by this library from the host so far (a CUDA-graph
 * capture counts each captured launch once; replays are not counted). */
unsigned long long b200_launch_count(void);

/* Reads the device error word of the current device; clears it when `clear`
 * is non-zero.  Synchronous.  After a timeout bit (a bounded wait gave up),
 * zero the first b200_attention_workspace_bytes(0, 0, 1) bytes of the
 * attention workspace and the first 4096 bytes of the GEMM workspace before
 * the next call: the kernel that gave up can leave counters behind. */
int b200_device_error(unsigned* out, int clear);

/* ------------------------------------------------------------------------
 * Linear layers
 * ------------------------------------------------------------------------ */

/* Workspace bytes b200_linear / b200_linear_silu_and_mul use: the split-K
 * flags and fp32 partial tiles of the persistent SM-pair GEMM (4 KiB +
 * 128 KiB per SM, the same for every shape).  The workspace must be
 * zero-filled before its first use; every call leaves it reusable. */
int b200_linear_workspace_bytes(int T, int N, int K, size_t* bytes);

/* Host-side check of the SM-pair GEMM's work split (no counterpart in the
 * reference; no CUDA call): plans `tiles` output tiles of `num_kb` 64-wide K
 * blocks over at most `max_pairs` SM pairs (grouped schedule allowed when
 * `grouped` is non-zero), walks every pair's segments with the iterator the
 * kernel uses, and returns the number of violations: (tile, K block) units
 * not covered exactly once, malformed segments, group members out of place,
 * flag words outside the workspace's flag area.  0 = the schedule partitions
 * the work.  Negative status on bad arguments. */
int b200_gemm_schedule_check(long long tiles, int num_kb, int max_pairs, int grouped);

/* y[T, N] = x[T, K] * w[N, K]^T (+ bias[N]), bf16 in/out, fp32 accumulate,
 * tcgen05 tensor cores.  Replaces F.linear in
 *   src/layers/linear.py:74-75   ColumnParallelLinear.forward
 *   src/layers/linear.py:169-170 RowParallelLinear.forward (per-rank part)
 *   src/layers/llm_head.py:64    ParallelLMHead.forward
 * K, ldx and ldw must be multiples of 8; x and w 16-byte aligned.
 * With a workspace of b200_linear_workspace_bytes() bytes (zeroed once,
 * 16-byte aligned) the GEMM runs on the persistent SM-pair kernel
 * (tcgen05.mma.cta_group::2; grouped split-K, stream-K or cluster split-K
 * schedule) where that is faster; with NULL it runs on the single-SM kernel.  Concurrent
 * calls must not share one workspace. */
int b200_linear(const void* x, long long ldx, const void* w, long long ldw, const void* bias,
                void* y, long long ldy, int T, int N, int K, void* workspace, size_t ws_bytes,
                b200_stream_t stream);

/* y[T, I] = silu(x * w[:I]^T) * (x * w[I:]^T): the gate_up projection with
 * SiLU-and-mul in its epilogue.  Replaces
 *   src/models/qwen3.py:119-121 (gate_up_proj -> act_fn) =
 *   src/layers/linear.py:74-75 + src/layers/activation.py:6-10.
 * w is [2I, K] with rows [gate ; up] exactly as MergedColumnParallelLinear
 * stores them (src/layers/linear.py:89-102).  I must be a multiple of 64
 * (B200_ERR_UNSUPPORTED otherwise); workspace as for b200_linear. */
int b200_linear_silu_and_mul(const void* x, long long ldx, const void* w, long long ldw, void* y,
                             long long ldy, int T, int I, int K, void* workspace, size_t ws_bytes,
                             b200_stream_t stream);

/* RMSNorm (+ residual add) and the projection that consumes it, in one call:
 *   s = x (+ residual) in fp32; residual_out = bf16(s)  (only with residual)
 *   xn = bf16(norm_weight * (s / sqrt(mean(s^2) + eps)))   [T, K], row stride ldxn
 *   y = xn * w^T (silu = 0: w [N, K], y [T, N]) or the gate_up projection
 *       with SiLU-and-mul (silu = 1: w [N = 2I, K], y [T, I]).
 * Replaces src/models/qwen3.py:162-168 (input_layernorm -> self_attn's
 * qkv_proj, post_attention_layernorm -> mlp's gate_up_proj) =
 * src/layers/layernorm.py:10-28 followed by src/layers/linear.py:74-75.
 * By default the rms_norm kernel runs first, then the GEMM.  With the
 * environment variable B200_FUSE_NORM=1, and when the GEMM runs on the
 * persistent SM-pair kernel with every CTA resident, the norm rows are
 * computed inside the GEMM launch instead (a grid barrier before its first
 * activation loads, the weight loads already in flight; measured slower in
 * the decode step).  Either way xn and residual_out hold the results.
 * K <= 8192; workspace as for b200_linear (its flag words also hold the
 * grid barrier). */
int b200_rmsnorm_linear(const void* x, long long ldx, const void* residual, void* residual_out,
                        const void* norm_weight, float eps, void* xn, long long ldxn, const void* w,
                        long long ldw, void* y, long long ldy, int T, int N, int K, int silu,
                        void* workspace, size_t ws_bytes, b200_stream_t stream);

/* RowParallelLinear at tp > 1 in one launch: y = sum over ranks of
 * bf16(x_r * w_r^T (+ bias on rank 0)), the all-reduce of
 * src/layers/linear.py:169-173 (torch.distributed.all_reduce after F.linear)
 * fused into the GEMM epilogue over NVLink peer memory.  Every rank calls it
 * with the same shapes and the same `one_shot`; stage / out / flags / done
 * are arrays of `world` device pointers giving each rank's address of its
 * symmetric buffers (rank r's own entry at index r), zero before the first
 * call:
 *   one_shot == 0 (two-shot: the rows of every CTA position are split among
 *   the ranks; each rank's CTA gathers and reduces its share and writes it
 *   into every rank's output; 2 (world-1)/world of the output bytes cross
 *   NVLink per rank):
 *     stage[r]: bf16 [world][stage_rows][ldo]; out[r]: bf16 [stage_rows][ldo]
 *     flags[r], done[r]: uint32 [max_positions] (left zero by every call)
 *   one_shot != 0 (every rank pushes its partial to every rank and reduces
 *   its own copy: one NVLink hop, world - 1 times the output bytes):
 *     stage[r]: bf16 [2][world][stage_rows][ldo]; out[r] as above
 *     flags[r]: uint32 [2][max_positions]; done[r]: uint32 [2] call counters
 * The reduced y is in out[rank] (rows [0, T), columns [0, N)) when the
 * launch completes on this rank's stream.  Returns B200_ERR_UNSUPPORTED
 * without launching when the CTAs of the launch could not all be resident
 * at once (the owner ranks wait on peer CTAs) or the sizes exceed the
 * buffers; the caller then runs b200_linear + a collective.  Waits on peer
 * flags are bounded (1 s) and set B200_DEVERR_PEER_TIMEOUT. */
int b200_linear_allreduce(const void* x, long long ldx, const void* w, long long ldw,
                          const void* bias, int T, int N, int K, int rank, int world,
                          void* const* stage, void* const* out, void* const* flags,
                          void* const* done, long long stage_rows, long long ldo,
                          long long max_positions, int one_shot, b200_stream_t stream);

/* Whether b200_linear_allreduce would launch (T, N, K) at `world` ranks with
 * these buffer sizes (*supported = 1) or refuse it with B200_ERR_UNSUPPORTED
 * (*supported = 0; b200_last_error() gives the reason).  Launches nothing.
 * The answer depends only on the shapes, the sizes and the device type, so
 * ranks of one job on identical GPUs agree; callers still agree on it with a
 * collective before choosing between the fused path and
 * b200_linear + torch.distributed.all_reduce (src/layers/linear.py:169-173),
 * so that no rank takes the other path. */
int b200_linear_allreduce_supported(int T, int N, int K, int world, long long stage_rows,
                                    long long ldo, long long max_positions, int* supported);

/* CUDA IPC helpers for the symmetric buffers: export the allocation that
 * holds `ptr` (64-byte handle + offset of ptr inside it), map a peer's
 * export into this process, and unmap it. */
int b200_ipc_export(const void* ptr, void* handle, unsigned long long* offset);
int b200_ipc_import(const void* handle, unsigned long long offset, void** ptr);
int b200_ipc_close(void* ptr, unsigned long long offset);

/* ------------------------------------------------------------------------
 * Normalisation, RoPE, activation
 * ------------------------------------------------------------------------ */

/* RMSNorm over rows of `dim` (multiple of 8, <= 8192).
 * residual == NULL: out = bf16(w * (x / sqrt(mean(x^2) + eps)))
 *   -> src/layers/layernorm.py:10-16 RMSNorm.normal_forward
 * residual != NULL: s = x + residual (fp32); residual_out = bf16(s);
 *   out = bf16(w * (s / sqrt(mean(s^2) + eps)))
 *   -> src/layers/layernorm.py:18-28 RMSNorm.residual_forward
 * residual and residual_out are contiguous [rows, dim]; they may alias. */
int b200_rms_norm(const void* x, long long x_stride, const void* residual, const void* weight,
                  void* out, long long out_stride, void* residual_out, int rows, int dim,
                  float eps, b200_stream_t stream);

/* Per token: q heads -> RMSNorm(q_norm_w) -> RoPE -> q_out;
 * k heads -> RMSNorm(k_norm_w) -> RoPE -> k_out and k_cache[slot];
 * v heads -> v_out and v_cache[slot].  head_dim is 128.
 * Replaces src/models/qwen3.py:81-89 (split, q_norm/k_norm, rotary_emb)
 * together with the cache write of src/layers/attention.py:86-88.
 *  - q_norm_w / k_norm_w NULL: no q/k norm (attention_bias models,
 *    src/models/qwen3.py:85).
 *  - v_in NULL: RoPE only (src/layers/pos_embedding.py:30-52 RoPE.forward).
 *  - k_cache NULL: no cache write; otherwise slot_mapping[t] == -1 skips t.
 *  - cos_sin: fp32 [max_pos, 128] = [cos | sin] table of
 *    src/layers/pos_embedding.py:6-18; positions: int64 [T].
 *  - k_out / v_out may be NULL. */
int b200_qk_norm_rope_store(const void* q_in, long long q_in_stride, const void* k_in,
                            long long k_in_stride, const void* v_in, long long v_in_stride, int T,
                            int Hq, int Hkv, const void* q_norm_w, const void* k_norm_w, float eps,
                            const float* cos_sin, long long max_pos, const long long* positions,
                            const int* slot_mapping, void* k_cache, void* v_cache,
                            long long num_slots, void* q_out, void* k_out, void* v_out,
                            b200_stream_t stream);

/* out[T, I] = silu(x[:, :I]) * x[:, I:].
 * Replaces src/layers/activation.py:6-10 SiluAndMul.forward. */
int b200_silu_and_mul(const void* x, long long x_stride, void* out, long long out_stride, int T,
                      int I, b200_stream_t stream);

/* ------------------------------------------------------------------------
 * KV cache and attention
 * ------------------------------------------------------------------------ */

/* k_cache.view(-1, D)[slot_mapping[i]] = key[i] (and value), slot -1 skipped,
 * 16-byte vector copies; slot_mapping is int32 [T]; num_slots bounds the
 * cache rows (num_blocks * block_size).
 * Replaces src/layers/attention.py:36-61 store_kvcache (Triton kernel
 * store_kvcache_kernel, src/layers/attention.py:10-34). */
int b200_store_kvcache(const void* key, long long key_stride, const void* value,
                       long long value_stride, void* k_cache, void* v_cache,
                       const int* slot_mapping, int T, int D, long long num_slots,
                       b200_stream_t stream);

/* Workspace of b200_paged_attention's decode path for up to `max_seqs`
 * sequences of up to `max_seqlen_k` keys. */
int b200_attention_workspace_bytes(int max_seqs, int max_seqlen_k, int Hq, size_t* bytes);

/* Causal (bottom-right aligned) varlen GQA attention, head_dim 128.
 * Replaces src/layers/attention.py:93-104 (flash_attn_varlen_func with
 * cu_seqlens_q/k, max_seqlen_q/k, softmax_scale, causal=True, block_table).
 *  - q: num_q_rows token rows of Hq x 128, q_stride elements apart.
 *  - block_tables != NULL: K/V from the paged cache [num_blocks, page, Hkv,
 *    128] (int32 block_tables: B rows of bt_width entries, bt_stride apart,
 *    -1 padded; a key past the row's width or in a -1 block is read as zero
 *    and flags B200_DEVERR_BAD_INDEX);
 *    block_tables == NULL: K/V from contiguous k / v rows cu_seqlens_k[b]+j.
 *  - cu_seqlens_q / cu_seqlens_k: int32 [B + 1] on the device; sequences
 *    with q length <= 0 (CUDA-graph padding) are skipped.
 *  - max_seqlen_q == 1 with a block table (B <= 1024, Hkv <= 64, Hq/Hkv <= 8,
 *    page a multiple of 256) takes the split-KV decode kernel and needs
 *    `workspace` (b200_attention_workspace_bytes).  Its first 256 KiB + 256
 *    bytes hold work-queue words and per-(sequence, kv head) completion
 *    counters that must be zero before the first call and are zero again
 *    after every call; the rest is per-call scratch (split-KV partials).  The
 *    kernel is launched cooperatively (its merges wait, bounded, on items
 *    that other CTAs compute).  Calls that share a
 *    workspace must not overlap on the GPU. */
int b200_paged_attention(const void* q, long long q_stride, int num_q_rows, const void* k,
                         long long k_stride,
                         const void* v, long long v_stride, const void* k_cache,
                         const void* v_cache, long long num_slots, const int* block_tables,
                         int bt_stride, int bt_width, const int* cu_seqlens_q, const int* cu_seqlens_k, int B,
                         int max_seqlen_q, int max_seqlen_k, int Hq, int Hkv, int page,
                         float softmax_scale, void* out, long long out_stride, void* workspace,
                         size_t ws_bytes, b200_stream_t stream);

/* Allocation-free variant of the decode path of b200_paged_attention (every
 * sequence has query length 1, K/V from the paged cache): the same kernel,
 * with its scratch in a fixed 32 MiB array inside the library instead of a
 * caller workspace.  No counterpart in the reference: it is for callers that
 * cannot allocate device memory -- hosts that reach this library through a
 * foreign-function boundary with device memory owned elsewhere, or serving
 * loops that must not call cudaMalloc (it may synchronise the device and
 * cannot be recorded into a CUDA graph).
 *  - Limits: B <= 1024, Hkv <= 64, Hq / Hkv <= 8, page a multiple of 256, and
 *    256 KiB + 256 + B * ceil(max_seqlen_k / 512) * Hq * 520 bytes must fit the
 *    32 MiB array (e.g. 250 sequences of 4096 keys with 32 heads); larger
 *    problems return B200_ERR_WORKSPACE without launching anything.
 *  - The first call on a device looks up the array's device address; make
 *    that first call before any CUDA-graph capture.
 *  - Every call clears the array's counters on `stream` and then uses it, so
 *    calls on different streams that overlap on the GPU race with each
 *    other; serialise them.
 *  - Allocates nothing (no cudaMalloc / cudaFree); the array stays resident on
 *    every GPU that loaded the library until the process exits. */
int b200_paged_decode_attention_static(const void* q, long long q_stride, int num_q_rows,
                                       const void* k_cache, const void* v_cache,
                                       long long num_slots, const int* block_tables,
                                       int bt_stride, int bt_width, const int* cu_seqlens_q,
                                       const int* cu_seqlens_k, int B, int max_seqlen_k, int Hq,
                                       int Hkv, int page, float softmax_scale, void* out,
                                       long long out_stride, b200_stream_t stream);

/* Attention metadata of one step from per-sequence values, the expansion of
 * src/engine/model_runner.py:174-233 (ModelRunner.prepare_seqs) done on the
 * device.  seq_info = int32 [3][B]: start = min(num_cached_tokens, len - 1),
 * num_scheduled_tokens, and the length of the sequence's block table (0 for
 * none, as in warm-up).  block_tables = int32 [B][bt_stride], -1 padded
 * (bt_stride 0: no sequence has a table).  Writes cu_seqlens_q / _k [B + 1]
 * (prefix sums of the query lengths and of end = start + length),
 * context_lens [B] = end, positions int64 [T] = start .. end - 1 per
 * sequence, and slot_mapping int32 for the tokens of the sequences that have
 * a table (block_table[p / page] * page + p % page, in token order; a block
 * missing from the table gives -1 and B200_DEVERR_BAD_INDEX). */
int b200_step_metadata(const int* seq_info, const int* block_tables, int bt_stride, int B, int page,
                       long long* positions, int* slot_mapping, int* cu_seqlens_q, int* cu_seqlens_k,
                       int* context_lens, b200_stream_t stream);

/* ------------------------------------------------------------------------
 * Vocabulary
 * ------------------------------------------------------------------------ */

/* out[t] = weight[ids[t] - vocab_start] if vocab_start <= ids[t] < vocab_end
 * else 0 (int64 ids).  The local half of src/layers/llm_head.py:38-49
 * VocabParallelEmbedding.forward (the all_reduce stays in NCCL). */
int b200_embedding(const long long* ids, const void* weight, void* out, int T, int H,
                   long long vocab_start, long long vocab_end, b200_stream_t stream);

/* Vocabulary-parallel embedding whose all-reduce is done as a scatter over
 * NVLink: replaces src/layers/llm_head.py:38-49 (masked F.embedding of this
 * rank's shard + dist.all_reduce).  Every rank calls it with the same ids;
 * rank `rank` writes the rows of the ids in [vocab_start, vocab_end) into
 * out[dst] of every rank dst (rows [0, T), row stride ld_out elements), and
 * rank 0 also writes the zero rows of ids outside [0, vocab_size).  The last
 * CTA signals the peers through flags[*] and waits (bounded) until every
 * rank's rows have arrived, so out[rank] is complete when the launch
 * completes.  out / flags are arrays of `world` addresses (this rank's view
 * of each rank's buffer, its own at index rank); flags[r] points at rank r's
 * uint32 [2][8] flag words and `state` at this rank's own uint32 [4] words
 * (call epochs and a CTA counter), all zero before the first call.  world 1:
 * the plain masked lookup into out[0]. */
int b200_embedding_exchange(const long long* ids, const void* weight, int T, int H,
                            long long vocab_start, long long vocab_end, long long vocab_size,
                            int rank, int world, void* const* out, long long ld_out,
                            void* const* flags, void* state, b200_stream_t stream);

/* Token selection on this rank's vocabulary shard: keys[r] = the packed
 * (score, global index) of row r's best column, where score = logit (greedy,
 * temperatures == NULL) or logit / T_r - ln(max(E, 1e-10)) with E ~ Exp(1)
 * taken from `noise` ([rows][noise_stride] fp32) or, when noise == NULL,
 * drawn by Philox-4x32-10 keyed by (seed, row, global column, offset).  The
 * maximum of the keys over the shards selects the same token as
 * src/layers/sampler.py:4-17 (softmax(logits / T) / E, argmax) over the
 * gathered logits of src/layers/llm_head.py:65-68 (lowest index on ties),
 * so no logits need to be gathered.  One CTA per row. */
int b200_select_tokens_partial(const void* logits, long long stride, int rows, int V,
                               long long vocab_start, const float* temperatures, const float* noise,
                               long long noise_stride, unsigned long long seed,
                               unsigned long long offset, long long* keys, b200_stream_t stream);

/* tokens[r] = the token of the maximum of keys[r] over the `world` ranks:
 * every rank pushes its keys into key_slots[*] (int64 [2][world][max_rows]
 * per rank), one signal round through flags[*] (as for
 * b200_embedding_exchange, the other word), bounded wait, maximum per row.
 * rows <= max_rows.  world 1: tokens straight from the keys (any rows). */
int b200_select_tokens_exchange(const long long* keys, int rows, int rank, int world,
                                void* const* key_slots, void* const* flags, void* state,
                                long long max_rows, long long* tokens, b200_stream_t stream);

/* out[r] = argmax(logits[r, :V]) (first maximum), int64.  Greedy selection
 * over the logits returned by src/layers/llm_head.py:60-69. */
int b200_argmax(const void* logits, long long stride, int rows, int V, long long* out,
                b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200OPS_H_ */
