/*
 * b200_attn.h — C ABI of the B200 (sm_100a) attention hot path of nano-vLLM.
 *
 * Every entry point that launches work takes plain device pointers, element
 * strides and sizes, enqueues its kernels on the caller's CUDA stream (a
 * `cudaStream_t` passed as `void*`), never synchronises the host, never
 * allocates device memory and never reads device data on the host.  That
 * makes each call capturable in a CUDA graph, which is how nano-vLLM runs
 * decode (nanovllm/engine/model_runner.py:222-257).  The diagnostic readers
 * (b200_workspace_error, b200_paged_attention_noalloc_error,
 * b200_varlen_prefill_error, b200_oproj_allreduce_error, b200_allreduce_error) synchronise the
 * stream they are given.
 *
 * Every wait inside a kernel is bounded (1 s).  One that runs out sets a bit
 * of the call's device-side error word and the kernel returns; the results of
 * that call are then undefined.  Bits: 1 a pipeline stage was never filled,
 * 2 a stage was never released, 4 copies in flight did not complete before
 * exit, 8 a barrier among the kernel's own warps ran out.
 *
 * Return value: B200_OK or one of the error codes below.  The text of the
 * last error of the calling host thread is available from b200_last_error().
 * Argument checks mirror the `assert`s of the reference launcher
 * (nanovllm/layers/attention.py:36-39); a failed check launches nothing.
 *
 * Tensor conventions (all row-major, element strides):
 *   token rows  : [N, H, D] with the head dimension contiguous and the head
 *                 stride equal to D; the token stride is passed explicitly so
 *                 that the strided `v` view produced by the fused QKV
 *                 projection (nanovllm/models/qwen3.py:79-82) is accepted.
 *   KV cache    : one layer of nano-vLLM's cache, [num_blocks, block_size,
 *                 Hkv, D] contiguous (model_runner.py:113-120).
 *   block table : int32 [batch, block_table_stride], entries past a
 *                 sequence's last block are never read (model_runner.py:125).
 */
#ifndef B200_ATTN_H
#define B200_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum b200_status {
    B200_OK = 0,
    B200_ERR_ARG = 1,         /* argument check failed (reference: AssertionError) */
    B200_ERR_UNSUPPORTED = 2, /* shape or dtype outside what the kernels implement */
    B200_ERR_WORKSPACE = 3,   /* workspace missing, misaligned or too small */
    B200_ERR_CUDA = 4         /* the CUDA runtime or driver reported an error */
};

enum b200_dtype { B200_F16 = 0, B200_BF16 = 1, B200_F32 = 2 };

/* Message of the last failed call on this host thread ("" if none). */
B200_API const char* b200_last_error(void);

/* Bumped whenever a signature below changes (2: b200_oproj_allreduce takes its
 * split-K workspace and low-latency slots; the epoch moved to the device;
 * 3: b200_varlen_prefill takes a workspace for its dynamic scheduler). */
#define B200_ABI_VERSION 3
B200_API int32_t b200_abi_version(void);

/*
 * KV-cache scatter.  Replaces nanovllm/layers/attention.py:33-40
 * (`store_kvcache`, Triton kernel at :10-30):
 *     k_cache.view(-1, Hkv*D)[slot_mapping[t]] = key[t]   (same for value)
 * for every token t with slot_mapping[t] != -1.  Rows whose slot lies outside
 * [0, num_slots) are skipped as well (the reference would write out of
 * bounds).  Non-negative slots must be unique within one call, as in the
 * reference.  elem_bytes is 2 (bf16/fp16) or 4 (fp32); the copy is bitwise.
 */
B200_API int32_t b200_store_kvcache(const void* key, int64_t key_stride,
                           const void* value, int64_t value_stride,
                           void* k_cache, void* v_cache,
                           const int32_t* slot_mapping, int32_t num_tokens,
                           int32_t num_kv_heads, int32_t head_dim,
                           int64_t num_slots, int32_t elem_bytes, void* stream);

/*
 * Fused q/k RMSNorm + rotary embedding + KV-cache scatter for Qwen3 layers.
 * Replaces, in one pass over the fused QKV projection output `qkv`
 * ([num_tokens, (Hq + 2 Hkv) * D], token stride qkv_stride):
 *     q = q_norm(q); k = k_norm(k)           nanovllm/models/qwen3.py:82-84
 *                                            (RMSNorm, nanovllm/layers/layernorm.py:16-26)
 *     q, k = rotary_emb(positions, q, k)     qwen3.py:85 (layers/rotary_embedding.py:6-14, 37-48)
 *     store_kvcache(k, v, k_cache, v_cache, slot_mapping)   layers/attention.py:60-63
 * Rounding follows the reference's eager order: RMSNorm in fp32, rounded to
 * the model dtype, times the weight (rounded); RoPE in fp32 on the rounded
 * normalised values, rounded.  cos_sin is the model's cos_sin_cache,
 * [max_position, D] fp32 with cos in the first D/2 columns and sin in the
 * rest; positions (int64) are clamped to [0, max_position).
 * Outputs: q_out [num_tokens, Hq, D] (token stride q_out_stride); k_out
 * [num_tokens, Hkv, D] or NULL; the rotated k and the unchanged v rows go to
 * k_cache / v_cache [num_slots, Hkv, D] at slot_mapping[t] (NULL caches: no
 * store; slots of -1 or outside the cache are skipped).  All rows 8-byte
 * aligned (cos_sin 16-byte); D == 128; dtype bf16 or fp16.
 */
B200_API int32_t b200_qk_norm_rope_store(void* q_out, int64_t q_out_stride,
                                void* k_out, int64_t k_out_stride,
                                const void* qkv, int64_t qkv_stride,
                                const int64_t* positions,
                                const void* q_weight, const void* k_weight, float eps,
                                const float* cos_sin, int32_t max_position,
                                void* k_cache, void* v_cache,
                                const int32_t* slot_mapping, int64_t num_slots,
                                int32_t num_tokens, int32_t num_heads, int32_t num_kv_heads,
                                int32_t head_dim, int32_t dtype, void* stream);

/*
 * Fused sampler.  Replaces nanovllm/layers/sampler.py:7-12
 *     token[b] = argmax_j softmax(logits[b] / T[b])_j / clamp_min(E[b, j], 1e-10)
 * computed as argmax_j (logits[b, j] / T[b] - log E[b, j]) (the softmax only
 * rescales a row), one pass over the logits.  E is the caller's noise
 * [batch, V] fp32 (row stride noise_stride; e.g. the reference's own
 * exponential_ draw), or, with noise == NULL, Exp(1) samples -log(U) with U
 * from Philox-4x32-10: counter (j / 4, b, offset_lo, offset_hi), key
 * (seed_lo, seed_hi), output word j % 4, U = ((bits >> 8) + 0.5) * 2^-24 —
 * the same (seed, offset) gives the same tokens on any grid.  Ties go to the
 * smallest index (torch.argmax).
 * logits [batch, V] (row stride row_stride, dtype bf16 / fp16 / fp32);
 * temperatures [batch] fp32 (> 0, as SamplingParams asserts);
 * out_tokens [batch] int64 (torch.argmax's dtype).
 * workspace: b200_sample_workspace_size(batch) bytes, 16-byte aligned.
 */
B200_API size_t b200_sample_workspace_size(int32_t batch);

B200_API int32_t b200_sample(int64_t* out_tokens, const void* logits, int64_t row_stride, int32_t dtype,
                    const float* temperatures, int32_t batch, int32_t vocab_size,
                    const float* noise, int64_t noise_stride, uint64_t seed, uint64_t offset,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode-step metadata on the device.  Replaces the per-sequence host loops
 * of nanovllm/engine/model_runner.py:167-193 (prepare_decode,
 * prepare_block_tables, prepare_sample).  `packed` is a device int32 buffer
 * (one host-to-device copy per step): [batch] lengths, [batch] last tokens,
 * [batch] temperatures (fp32 bits), [batch + 1] offsets into `flat`, then
 * `flat` = every block id of the batch, sequence after sequence.  Writes
 *   input_ids[b] = last token, positions[b] = len - 1 (int64);
 *   context_lens[b] = len, slot_mapping[b] = block_table[-1] * block_size +
 *   (len - (num_blocks - 1) * block_size) - 1 (int32);
 *   block_tables[b, j] = block_table[j] or -1 past the sequence's blocks,
 *   [batch, max_blocks] int32 (max_blocks = the batch's longest table);
 *   temperatures[b] (fp32).
 * The host must give offsets that stay inside `flat` (the kernel trusts them).
 */
B200_API int32_t b200_decode_metadata(const int32_t* packed, int32_t batch, int32_t max_blocks,
                             int32_t block_size, int64_t* input_ids, int64_t* positions,
                             int32_t* slot_mapping, int32_t* context_lens, int32_t* block_tables,
                             float* temperatures, void* stream);

/*
 * Row-parallel output projection fused with its all-reduce over peer memory.
 * Replaces RowParallelLinear.forward of the attention output projection
 * (nanovllm/layers/linear.py:152-156, called at nanovllm/models/qwen3.py:87):
 *     y = F.linear(a, w)   (a [M, K] this rank's shard, w [N, K]; bf16)
 *     dist.all_reduce(y)
 * One launch per rank: tcgen05 GEMM units (128 x 256 tiles, split along K
 * when there are fewer tiles than SMs, split partials summed in fp32 in split
 * order) are rounded to bf16 and stored straight into every rank's slot
 * buffer (plain stores over NVLink), announced with system-scope release
 * flags; then every rank sums the ranks' partials from its own slot buffer
 * (fp32, rank order, so all ranks get the same bits) into out [M, N] (row
 * stride ldo).
 * slots[r] / flags[r]: device arrays of every rank's buffers, mapped into this
 * process (e.g. CUDA symmetric memory): slots [2][world][slot_rows][N] bf16,
 * ll_slots[r] (may be NULL): every rank's low-latency slots, uint32
 * [2][world][ll_rows][N] zeroed once, used by split calls with M <= ll_rows
 * (<= 128): each 8-byte word carries two bf16 values and the call's epoch, so
 * readers poll the data itself instead of flags.  world <= 8.
 * flags uint32 [max_units * world + 2] zeroed once before the first call.  The
 * call's epoch lives in the flag words, so the launch may be captured in a
 * CUDA graph; every rank makes the same calls in the same order.  workspace:
 * b200_oproj_allreduce_workspace_size() bytes of this rank's memory, zeroed
 * once (NULL disables the K split).  max_units >= the tile count
 * ceil(M/128) * N/256; the K split never makes more units than max_units.
 * N % 256 == 0, K % 64 == 0, M <= slot_rows; a, w 16-byte aligned with
 * strides that are multiples of 8 elements.  Bounded waits set the error word
 * read by b200_oproj_allreduce_error (results of that call undefined).
 */
B200_API int32_t b200_oproj_allreduce(void* out, int64_t ldo, const void* a, int64_t lda,
                             const void* w, int64_t ldw, int32_t M, int32_t N, int32_t K,
                             void* const* slots, int32_t slot_rows,
                             uint32_t* const* ll_slots, int32_t ll_rows,
                             uint32_t* const* flags, int32_t max_units,
                             void* workspace, int64_t workspace_bytes,
                             int32_t rank, int32_t world, void* stream);

B200_API int64_t b200_oproj_allreduce_workspace_size(void);

B200_API int32_t b200_oproj_allreduce_error(void* stream, int32_t* flag);

/*
 * All-reduce (sum) of a bf16 vector over the ranks of a tensor-parallel group
 * through memory every rank maps (plain loads and stores over NVLink, no
 * multicast).  Replaces the NCCL call that ends a row-parallel layer
 * (nanovllm/layers/linear.py:155, dist.all_reduce(y)) for decode-sized
 * tensors.  Two shots: each rank reduces one slice of the vector over every
 * rank's copy (fp32, rank order, one rounding to bf16) and stores it into
 * every rank's result slot, so all ranks get the same bits.
 * in / out: n bf16 values of this rank, 16-byte aligned (out may be in);
 * n % 8 == 0.  bufs[r]: device array of every rank's slot buffer of buf_elems
 * bf16 values (a multiple of 16, >= 2 n): the input slot is its first half,
 * the result slot its second; in == this rank's input slot skips the copy in,
 * out == its result slot the copy out.  in and out may each be either slot's
 * start or memory outside the slot buffer, no other place inside it.  flags[r]: every rank's b200_allreduce_flag_words()
 * uint32 words, zeroed once before the first call.  world <= 8.  The call's
 * epoch lives in the flag words, so the launch may be captured in a CUDA graph;
 * every rank makes the same calls in the same order.  Bounded waits set the
 * error word read by b200_allreduce_error (results of that call undefined).
 */
B200_API int32_t b200_allreduce_bf16(void* out, const void* in, int64_t n, void* const* bufs,
                            int64_t buf_elems, uint32_t* const* flags, int32_t rank,
                            int32_t world, void* stream);

B200_API int64_t b200_allreduce_flag_words(void);

B200_API int32_t b200_allreduce_error(void* stream, int32_t* flag);

/*
 * Paged multi-query attention over the KV cache: decode (query_len == 1)
 * and speculative verify (query_len == k+1).  Replaces the decode call of
 * nanovllm/layers/attention.py:71-74:
 *     flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
 *                             cache_seqlens=context_lens,
 *                             block_table=block_tables,
 *                             softmax_scale=scale, causal=True)
 * q   : [batch, query_len, Hq, D], token stride q_stride_token (a multiple
 *       of 8 elements), 16-byte aligned
 * out : [batch, query_len, Hq, D] contiguous, 16-byte aligned, dtype of q
 * context_lens[b] counts every cached token of sequence b including its
 * query_len new ones; query j of sequence b sees cache positions
 * p <= context_lens[b] - query_len + j (causal, bottom-right aligned).
 * Rows with context_lens[b] <= 0 (CUDA-graph padding) get a zero output.
 * kv head of query head h is h / (Hq / Hkv) (GQA).
 * workspace: b200_paged_attention_workspace_size() bytes, 256-byte aligned,
 * zero-filled once before the first call; every call leaves its control
 * region zeroed again.  Calls sharing a workspace must not overlap on the GPU.
 * Constraints: D == 128, dtype bf16 or fp16, block_size % 128 == 0,
 * batch <= 2048, query_len * (Hq / Hkv) <= 16, softmax_scale positive and
 * finite (B200_ERR_ARG otherwise).
 */
B200_API size_t b200_paged_attention_workspace_size(int32_t max_items, int32_t query_len,
                                           int32_t group_size, int32_t head_dim);

B200_API int32_t b200_paged_attention(void* out, const void* q, int64_t q_stride_token,
                             const void* k_cache, const void* v_cache,
                             int32_t num_blocks, int32_t block_size,
                             const int32_t* block_tables, int32_t block_table_stride,
                             const int32_t* context_lens, int32_t batch,
                             int32_t query_len, int32_t num_heads,
                             int32_t num_kv_heads, int32_t head_dim,
                             float softmax_scale, int32_t dtype,
                             void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * Allocation-free variant of b200_paged_attention; no counterpart in the
 * reference (which always has PyTorch's allocator at hand).  For callers that
 * cannot allocate device memory on the execution path -- runtimes whose own
 * allocator owns the device heap and gives plugins no workspace, plugin hosts
 * that forbid cudaMalloc there, code that must not risk cudaMalloc/cudaFree's
 * implicit device synchronisation.  Same arguments and results as
 * b200_paged_attention without the workspace: the split-K scratch is a 32 MiB
 * array inside the library that every GPU loading the library holds until the
 * process exits.  Limit: batch * num_kv_heads <= 8192 and at most
 * (32 MiB - 33 KiB) / (query_len * Hq/Hkv * 516 B) work items; larger calls
 * return B200_ERR_WORKSPACE.  The first call on a device looks up the array's
 * device address (make it before any stream capture); the lookup is repeated
 * in any other CUDA context of that device (a driver-API context, the new
 * primary context after cudaDeviceReset).  Calls share the array: each clears
 * the control words it needs (the error word included), and calls that
 * overlap on the GPU race, so serialise them.
 */
B200_API int32_t b200_paged_attention_noalloc(void* out, const void* q, int64_t q_stride_token,
                                     const void* k_cache, const void* v_cache,
                                     int32_t num_blocks, int32_t block_size,
                                     const int32_t* block_tables, int32_t block_table_stride,
                                     const int32_t* context_lens, int32_t batch,
                                     int32_t query_len, int32_t num_heads,
                                     int32_t num_kv_heads, int32_t head_dim,
                                     float softmax_scale, int32_t dtype, void* stream);

/*
 * Copies the workspace's device-side error word to *flag (synchronously on
 * `stream`).  Non-zero means a bounded wait inside a kernel gave up; the
 * results of that call are undefined.  For tests and diagnostics only.
 */
B200_API int32_t b200_workspace_error(const void* workspace, void* stream, int32_t* flag);

/*
 * Copies the device-side error word of the latest b200_paged_attention_noalloc
 * call on the current device (it lives in the library's built-in scratch) to
 * *flag, synchronously on `stream`; the bits are those listed at the top of
 * this file.  No counterpart in the reference.  For tests and diagnostics.
 */
B200_API int32_t b200_paged_attention_noalloc_error(void* stream, int32_t* flag);

/*
 * Test hook, no counterpart in the reference: the next `launches`
 * paged-attention launches (either entry point) made by the calling host
 * thread run with an idle producer warp that issues no loads, and with every
 * wait limited to wait_limit_ns (1 us .. 1 s).  The consumer warps' first wait
 * then runs out, the call's error word gets bit 1 and the kernel returns (the
 * output is undefined); nothing faults and later calls run normally.  Lets a
 * test check that a wait that runs out is reported to the host.
 */
B200_API int32_t b200_testing_idle_producer(int32_t launches, int64_t wait_limit_ns);

/*
 * Causal varlen prefill attention, optionally over the paged cache (prefix
 * caching / chunked prefill).  Replaces nanovllm/layers/attention.py:64-70:
 *     flash_attn_varlen_func(q, k, v, cu_seqlens_q=..., cu_seqlens_k=...,
 *                            max_seqlen_q=..., max_seqlen_k=...,
 *                            softmax_scale=scale, causal=True,
 *                            block_table=block_tables)
 * q/out : [total_q, Hq, D] (out contiguous, 16-byte aligned); total_q and
 *         total_k_rows are the row counts of the q and k/v buffers (the TMA
 *         descriptors never reach past them)
 * Without a block table k/v are packed token rows [total_k, Hkv, D] and the
 * keys of sequence s are rows cu_seqlens_k[s] .. cu_seqlens_k[s+1]-1.
 * With a block table k/v are the layer's caches [num_blocks, block_size,
 * Hkv, D] and key position p of sequence s lives in block
 * block_tables[s][p / block_size].  Query i of a sequence with Lq queries and
 * Lk keys sees key positions p <= i + Lk - Lq (bottom-right causal mask).
 * workspace: b200_varlen_prefill_workspace_size() bytes, 256-byte aligned,
 * zero-filled once before the first call (it holds the work counter that the
 * CTAs claim query tiles from; every call leaves it zeroed again).  Calls
 * sharing a workspace must not overlap on the GPU.
 * Constraints: D == 128, dtype bf16 or fp16, block_size % 128 == 0.
 */
B200_API size_t b200_varlen_prefill_workspace_size(void);

B200_API int32_t b200_varlen_prefill(void* out, const void* q, int64_t q_stride_token,
                            const void* k, int64_t k_stride_token,
                            const void* v, int64_t v_stride_token,
                            const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                            int32_t num_seqs, int32_t total_q,
                            int32_t max_seqlen_q, int32_t max_seqlen_k,
                            int32_t total_k_rows,
                            const int32_t* block_tables, int32_t block_table_stride,
                            int32_t block_size,
                            int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                            float softmax_scale, int32_t dtype,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * Copies the prefill kernels' device-side error word to *flag after
 * synchronising `stream`; non-zero means a bounded wait inside the kernel gave
 * up (results of that call undefined).  For tests and diagnostics only.
 */
B200_API int32_t b200_varlen_prefill_error(void* stream, int32_t* flag);

/*
 * Speculative-decoding acceptance sampling (standard rejection scheme):
 * for draft position i = 0..k-1 with draft token x_i, accept when
 *     u_i < min(1, p_i(x_i) / q_i(x_i))
 * with p = softmax(target_logits / T), q = softmax(draft_logits / T); at the
 * first rejection sample from normalise(max(p_i - q_i, 0)), and when all k
 * drafts are accepted sample a bonus token from p_k.  Sampling uses the
 * uniform uniform_sample[b] through a fixed-order inverse CDF, so that
 * results are reproducible bit for bit.  The reference engine has no
 * speculative path; this op has no counterpart there.
 * target_logits [batch, k+1, V], draft_logits [batch, k, V] fp32;
 * draft_tokens, uniform_accept [batch, k]; uniform_sample [batch];
 * temperatures [batch] or NULL (T = 1).
 * out_tokens [batch, k+1] int32 (accepted drafts, then the sampled token,
 * then -1), out_num_tokens [batch] = accepted + 1.
 */
B200_API size_t b200_spec_accept_workspace_size(int32_t batch, int32_t num_draft, int32_t vocab_size);

B200_API int32_t b200_spec_accept(int32_t* out_tokens, int32_t* out_num_tokens,
                         const float* target_logits, const float* draft_logits,
                         const int32_t* draft_tokens, const float* uniform_accept,
                         const float* uniform_sample, const float* temperatures,
                         int32_t batch, int32_t num_draft, int32_t vocab_size,
                         void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_ATTN_H */
