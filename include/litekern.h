/*
 * litekern.h - C ABI of liblitekern.so, the sm_100a kernels for litevllm's
 * per-step hot path: paged KV-cache store, paged decode attention, chunked
 * prefill attention over paged context, and the vocab-wide sampler.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless stated otherwise. The library
 *     allocates no device memory; the caller owns every buffer, including the
 *     workspaces.
 *   - Calls are asynchronous and stream-ordered on `stream` (a cudaStream_t,
 *     NULL = legacy default stream). No entry point synchronises the host.
 *   - The device that owns the buffers must be current on the calling thread.
 *   - Return value: LK_OK (0) or a negative LK_ERR_* code; lk_status_string()
 *     turns it into text. Invalid arguments are rejected before any launch.
 *   - dtype codes: LK_DTYPE_F32 / LK_DTYPE_F16 / LK_DTYPE_BF16.
 *   - Tensor layouts follow litevllm (reference paths relative to the
 *     lxy-alexander/lite-vllm project root):
 *       k_cache / v_cache : [num_blocks, block_size, num_kv_heads, head_dim],
 *                           contiguous (litevllm/cache/kv_cache.py:41-47)
 *       slot_mapping      : int64 [num_tokens]  (engine/model_runner.py:237)
 *       block_tables      : int32 [B, max_blocks], zero padded
 *                           (engine/model_runner.py:243-247)
 *       context_lens      : int32 [B], including the token written this step
 *                           (engine/model_runner.py:230, :248-250)
 */
#ifndef LITEKERN_H
#define LITEKERN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LK_OK 0
#define LK_ERR_INVALID_ARG (-1)
#define LK_ERR_UNSUPPORTED (-2)
#define LK_ERR_ALIGNMENT (-3)
#define LK_ERR_WORKSPACE (-4)
#define LK_ERR_CUDA (-5)
#define LK_ERR_DRIVER (-6)
#define LK_ERR_TOO_LARGE (-7)

#define LK_DTYPE_F32 0
#define LK_DTYPE_F16 1
#define LK_DTYPE_BF16 2

/* Bits the kernels OR into a caller-provided device status word. */
#define LK_STATUS_SLOT_OOB 1       /* slot_mapping entry >= num_slots or < -1 */
#define LK_STATUS_BLOCK_OOB 2      /* block table entry outside [0, num_blocks) */
#define LK_STATUS_WAIT_TIMEOUT 4   /* a bounded mbarrier wait gave up */
#define LK_STATUS_CTX_OOB 8        /* context_len larger than the block table */
#define LK_STATUS_TOKEN_OOB 16     /* a past token id outside [-V, V) */

/* Library version (major*10000 + minor*100 + patch). */
int lk_version(void);

/* Human-readable text for an LK_* return code. Never NULL. */
const char* lk_status_string(int code);

/*
 * KV-cache store. Replaces the advanced-index scatter in
 * litevllm/layers/attention.py:79-84 (Attention.forward) and its twin
 * PagedAttention.write_to_cache, litevllm/layers/attention.py:18-33:
 *     key_cache[slot // bs, slot % bs] = key[t];  value_cache[...] = value[t]
 * key/value: [num_tokens, num_kv_heads, head_dim] with head stride head_dim,
 * unit element stride and a token stride given in elements. A slot of -1 is
 * skipped (padding); any other slot outside [0, num_slots) is skipped and
 * flagged with LK_STATUS_SLOT_OOB in *status (status may be NULL).
 * Bit-exact copy; duplicate slots in one call are unspecified (as in torch).
 */
int lk_store_kv(const void* key, const void* value, void* k_cache, void* v_cache,
                const int64_t* slot_mapping, int32_t num_tokens,
                int32_t num_kv_heads, int32_t head_dim,
                int64_t key_token_stride, int64_t value_token_stride,
                int64_t num_slots, int32_t dtype, int32_t* status, void* stream);

/*
 * Paged decode attention. Replaces Attention._decode_fast,
 * litevllm/layers/attention.py:91-139:
 *   out[b,h,:] = softmax_s(scale * q[b,h] . k[b,s,h/G]) @ v[b,s,h/G],
 *   s < context_lens[b], G = H / H_kv.
 * q / out: [B, H, D] (token stride q_token_stride / out_token_stride elements,
 * head stride D). The split kernel takes dtype F16 or BF16, D = 128,
 * block_size a multiple of 16 and G <= 8; other shapes (fp32, other head dims
 * or block sizes, larger G) run lk_paged_attention_generic's kernel, which
 * ignores num_splits: it needs the workspace's status word (at least 4
 * bytes) and splits long contexts across CTAs when the workspace also holds
 * their partials (lk_paged_attention_generic_workspace_bytes() bytes give
 * the full split count; a smaller workspace gives fewer splits). A
 * context_len of 0 yields NaN rows, like the reference's softmax over an all
 * -inf row.
 * num_splits: a positive value runs the split-KV kernel with that many
 * splits per sequence; 0 picks the split count lk_paged_decode_num_splits
 * returns; -1 runs the persistent stage-balanced kernel (one CTA per SM, the
 * (sequence, 16-token stage) space cut into equal contiguous ranges, partial
 * sequences merged by the last CTA to finish them). workspace: at least
 * lk_paged_decode_workspace_bytes(B, H, H_kv, D, num_splits) bytes, 256-byte
 * aligned, zero-filled before its first use; its counter region sits at a
 * fixed offset and every completed call leaves it zero again, so one
 * workspace serves consecutive calls of any shape on one stream. Calls that
 * overlap on the GPU must not share a workspace. B * (H_kv / 8) <= 65536.
 * With num_splits >= 1 the call launches two kernels: a one-CTA ordering
 * kernel writes the (sequence, split) units longest first into the workspace
 * (8 bytes per unit), and the decode kernel's CTA i takes unit i.
 */
int lk_paged_decode_num_splits(int32_t B, int32_t H_kv, int32_t max_blocks_per_seq,
                               int32_t block_size);
size_t lk_paged_decode_workspace_bytes(int32_t B, int32_t H, int32_t H_kv, int32_t D,
                                       int32_t num_splits);
int lk_paged_decode(void* out, int64_t out_token_stride,
                    const void* q, int64_t q_token_stride,
                    const void* k_cache, const void* v_cache, int64_t num_blocks,
                    const int32_t* block_tables, int64_t block_table_stride,
                    const int32_t* context_lens,
                    int32_t B, int32_t H, int32_t H_kv, int32_t D,
                    int32_t block_size, int32_t max_blocks_per_seq, float scale,
                    int32_t num_splits, void* workspace, size_t workspace_bytes,
                    int32_t dtype, void* stream);

/*
 * Decode for a batch whose rows all begin with the same prefix_tokens tokens
 * (block_tables[b][0 .. prefix_tokens / block_size) equal to row 0's, as the
 * reference's PrefixCache hands out shared blocks): the same result as
 * lk_paged_decode (it restates Attention._decode_fast, attention.py:91-139),
 * computed as the prefix part once for all rows -- every row's G query heads
 * of a KV head against the prefix keys on the tensor cores, in key ranges --
 * plus each row's own suffix on the split decode kernel, merged by log-sum-exp.
 * No counterpart in the reference (its decode re-reads the shared blocks per
 * row). Requires context_lens[b] >= prefix_tokens (a shorter row sets
 * LK_STATUS_CTX_OOB in the workspace status word), prefix_tokens a multiple of
 * block_size, G in {1, 2, 4, 8}. workspace: at least
 * lk_paged_decode_shared_prefix_workspace_bytes(...) bytes, 256-byte aligned,
 * zero-filled before first use (the same reuse rules as lk_paged_decode).
 * Launches three kernels on `stream`: the suffix units' ordering, the prefix
 * (once for all rows, on the tensor cores) and the suffix decode, which runs
 * beside the prefix kernel and waits for it only to merge its partials. Their
 * counters live in the workspace; nothing is allocated.
 */
size_t lk_paged_decode_shared_prefix_workspace_bytes(int32_t B, int32_t H, int32_t H_kv,
                                                      int32_t D, int32_t max_blocks_per_seq,
                                                      int32_t block_size, int32_t prefix_tokens);
int lk_paged_decode_shared_prefix(void* out, int64_t out_token_stride,
                                  const void* q, int64_t q_token_stride,
                                  const void* k_cache, const void* v_cache, int64_t num_blocks,
                                  const int32_t* block_tables, int64_t block_table_stride,
                                  const int32_t* context_lens,
                                  int32_t B, int32_t H, int32_t H_kv, int32_t D,
                                  int32_t block_size, int32_t max_blocks_per_seq, float scale,
                                  int32_t prefix_tokens, void* workspace, size_t workspace_bytes,
                                  int32_t dtype, void* stream);

/*
 * Read back the status word the last decode call left in its workspace
 * (host copy; synchronises `stream`). Returns LK_STATUS_* bits or a negative
 * LK_ERR_* code.
 */
int lk_paged_decode_status(const void* workspace, void* stream);

/*
 * Chunked-prefill attention over prior paged context. The reference only has
 * Attention._prefill (litevllm/layers/attention.py:141-151: causal SDPA over
 * the new tokens, one sequence per call); this generalises it. Sequence b has
 * q_len = cu_seqlens_q[b+1] - cu_seqlens_q[b] query tokens (rows
 * cu_seqlens_q[b].. of q/out, [T, H, D]) at absolute positions
 * prior .. prior+q_len-1, prior = context_lens[b] - q_len; query i attends key
 * positions j <= prior + i. With block_tables != NULL, keys and values (prior
 * and the chunk's own, already stored) come from the paged cache. With
 * block_tables == NULL, k_cache / v_cache are the contiguous [T, H_kv, D] keys
 * and values of the chunk (context_lens may then be NULL, meaning prior = 0):
 * this is exactly the reference's _prefill. The tensor-core kernel takes
 * dtype F16 or BF16, D = 128, G in {1,2,4,8} and (paged mode) block_size a
 * multiple of 16; other shapes run lk_paged_attention_generic.
 * status (may be NULL) receives LK_STATUS_* bits.
 */
int lk_paged_prefill(void* out, const void* q, int64_t q_token_stride,
                     const void* k_cache, const void* v_cache, int64_t num_blocks,
                     const int32_t* block_tables, int64_t block_table_stride,
                     const int32_t* cu_seqlens_q, const int32_t* context_lens,
                     int32_t num_seqs, int32_t max_q_len,
                     int32_t H, int32_t H_kv, int32_t D, int32_t block_size,
                     float scale, int32_t dtype, int32_t* status, void* stream);

/*
 * Generic paged attention on the CUDA cores, for the shapes the tuned kernels
 * do not take: fp32 / f16 / bf16 storage, D in {32, 64, 96, 128, 256}, any
 * block_size, G = H / H_kv up to 32. lk_paged_decode and lk_paged_prefill(_ws)
 * call it themselves for such shapes (fp32 models, head_dim 64 Llamas, 8-slot
 * blocks); it is exported so that a caller may also pick it directly. It
 * restates the reference's Attention._decode_fast
 * (litevllm/layers/attention.py:91-139) and Attention._prefill (:141-151) with
 * the prior-context generalisation of lk_paged_prefill: query token i of
 * sequence b (rows cu_seqlens_q[b].. of q / out) sits at position
 * prior + i, prior = context_lens[b] - q_len, and attends keys j <= prior + i.
 * cu_seqlens_q == NULL means decode: one query per sequence (row b,
 * max_q_len 1) at position context_lens[b] - 1, and block_tables is then
 * required. block_tables == NULL means contiguous keys ([T, H_kv, D], key j of
 * sequence b at row cu_seqlens_q[b] + j, prior 0; num_blocks = T).
 * max_blocks_per_seq > 0 bounds context_lens (larger ones are clamped and
 * flagged LK_STATUS_CTX_OOB); 0 = no bound. Out-of-range block ids read
 * zeros and set LK_STATUS_BLOCK_OOB in *status (may be NULL). Scores, softmax
 * and the PV sum are fp32; a row with no keys (context 0) is NaN. No
 * workspace, no allocation; one launch (one CTA per KV head, query tile and
 * sequence; lk_paged_decode adds split-KV for this kernel).
 */
/*
 * Workspace bytes with which lk_paged_decode splits a decode that takes the
 * generic kernel at its full split count (about 512 keys per split, at most
 * 64 splits; partials of (max, sum) and D fp32 per row, head and split). No
 * counterpart in the reference.
 */
size_t lk_paged_attention_generic_workspace_bytes(int32_t B, int32_t H, int32_t D,
                                                  int32_t max_blocks_per_seq,
                                                  int32_t block_size);
int lk_paged_attention_generic(void* out, int64_t out_token_stride,
                               const void* q, int64_t q_token_stride,
                               const void* k_cache, const void* v_cache, int64_t num_blocks,
                               const int32_t* block_tables, int64_t block_table_stride,
                               const int32_t* cu_seqlens_q, const int32_t* context_lens,
                               int32_t num_seqs, int32_t max_q_len,
                               int32_t H, int32_t H_kv, int32_t D, int32_t block_size,
                               int32_t max_blocks_per_seq, float scale, int32_t dtype,
                               int32_t* status, void* stream);

/*
 * lk_paged_prefill with a caller-owned workspace (same arguments and results;
 * workspace NULL = lk_paged_prefill). The workspace (256-byte aligned, at
 * least lk_paged_prefill_workspace_bytes() for key splits, any size from
 * 197 KiB for the plan alone; no zero-fill needed, the planning kernel clears
 * what it uses) holds the launch's work plan — (sequence, query tile) pairs
 * ordered most key tiles first — and lets the tail of a launch with at most
 * four waves of work items cut its longest late items into two key-range
 * pieces, merged exactly in a fixed order (fp32 partials), so the last wave
 * is made of shorter items. One workspace per stream. Without a workspace the
 * plan lives in a small buffer the library keeps per (device, stream) and no
 * item is cut.
 */
size_t lk_paged_prefill_workspace_bytes(void);
int lk_paged_prefill_ws(void* out, const void* q, int64_t q_token_stride,
                        const void* k_cache, const void* v_cache, int64_t num_blocks,
                        const int32_t* block_tables, int64_t block_table_stride,
                        const int32_t* cu_seqlens_q, const int32_t* context_lens,
                        int32_t num_seqs, int32_t max_q_len,
                        int32_t H, int32_t H_kv, int32_t D, int32_t block_size,
                        float scale, int32_t dtype, void* workspace, size_t workspace_bytes,
                        int32_t* status, void* stream);

/*
 * Vocab-wide sampler. Replaces Sampler.sample's greedy path
 * (litevllm/layers/sampler.py:174-175 -> _argmax_kernel :60-84) and its
 * temperature path (:178, :187: softmax(logits / T) then torch.multinomial)
 * with a single pass per row:
 *   temperatures[b] == 0 (or temperatures == NULL): argmax_v float(logits[b,v])
 *   otherwise: argmax_v  float(logits[b,v]) / T_b + g[b,v]   (Gumbel-max)
 * with IEEE fp32 division and addition; ties go to the lowest index; a NaN key
 * beats every number (torch.argmax semantics). g is read from `noise`
 * ([B, noise_ld] fp32) when non-NULL, else generated in-kernel as
 * g = -ln(-ln(u)), u from Philox4x32-10 keyed by (seed, offset, b, v), the
 * logarithms from hardware base-2 logarithms (within 5e-7 relative of exact);
 * noise_dump ([B, V] fp32, optional) receives the generated g.
 * logits: [B, V] with row stride ld elements, dtype F32, F16 or BF16.
 * out_ids: int64 [B]. workspace: lk_sample_workspace_bytes(B, V) bytes,
 * 256-byte aligned, zero-filled before first use (the counter region sits at a
 * fixed offset and every call leaves it zero again, whatever B and V).
 */
size_t lk_sample_workspace_bytes(int32_t B, int32_t V);
int lk_sample(int64_t* out_ids, const void* logits, int32_t B, int32_t V, int64_t ld,
              const float* temperatures, const float* noise, int64_t noise_ld,
              uint64_t seed, uint64_t offset, float* noise_dump,
              void* workspace, size_t workspace_bytes, int32_t dtype, void* stream);

/*
 * probs[b, :] = softmax(float(logits[b, :]) / temperatures[b]) in fp32, for the
 * top-k / top-p path of Sampler.sample (replaces _triton_softmax_temp,
 * litevllm/layers/sampler.py:127-144, including vocabularies > 65536 where the
 * reference falls back to F.softmax).
 */
/*
 * Block copies for copy-on-write forks and swaps. Replaces the per-block,
 * per-layer copy_ loops of KVCache.swap_in / swap_out
 * (litevllm/cache/kv_cache.py:74-102) and serves SchedulerOutput.blocks_to_copy
 * (litevllm/engine/scheduler.py:25-27): for every pair p and layer l,
 *   dst[l][mapping[p][1]] = src[l][mapping[p][0]]   (K and V).
 * src_cache_ptrs / dst_cache_ptrs: device arrays of 2 * num_layers addresses
 * (K of layer 0, V of layer 0, K of layer 1, ...); an address may point to
 * pinned host memory (unified addressing) for swaps. block_mapping: device
 * int64 [num_pairs, 2] (src, dst). block_bytes = block_size * H_kv * D * elem.
 * Pairs outside [0, num_blocks) are skipped and flagged LK_STATUS_BLOCK_OOB in
 * *status (may be NULL). Destination blocks must be distinct.
 */
int lk_copy_blocks(const uint64_t* src_cache_ptrs, const uint64_t* dst_cache_ptrs,
                   int32_t num_layers, const int64_t* block_mapping, int32_t num_pairs,
                   int64_t block_bytes, int64_t src_num_blocks, int64_t dst_num_blocks,
                   int32_t* status, void* stream);

/*
 * Fused q/k RMSNorm + rotary embedding + KV-cache store, the steps between the
 * projections and attention in Qwen3Attention.forward
 * (litevllm/models/qwen3.py:76-92; LlamaAttention without the norm):
 * LlamaRMSNorm (models/llama.py:18-27) when a weight is given, then the
 * half-split rotation of apply_rotary_emb (layers/rotary_emb.py:104-117) with
 * the caller's fp32 cos / sin tables ([max_pos, D/2], the RotaryEmbedding
 * cos_cached / sin_cached buffers) at positions[t]; q is rotated in place
 * ([T, H, D]); k is rotated and stored with v into slot slot_mapping[t] of the
 * caches (slot_mapping NULL: q / k only, no store; -1: skip), and written to
 * k_out ([T, H_kv, D], token stride k_out_token_stride; may be k itself) when
 * k_out is not NULL, for attention over the new tokens only (the reference's
 * _prefill reads the rotated k directly). D = 128, dtype
 * F16 or BF16, rounding points as in the reference (16-bit after the norm
 * and after the weight, fp32 rotation, 16-bit store).
 */
int lk_rope_store_kv(void* q, int64_t q_token_stride, const void* k, int64_t k_token_stride,
                     const void* v, int64_t v_token_stride, void* k_out,
                     int64_t k_out_token_stride, void* k_cache, void* v_cache,
                     int64_t num_slots, const int64_t* slot_mapping, const int64_t* positions,
                     const float* cos_cache, const float* sin_cache, int64_t max_pos,
                     const void* q_norm_weight, const void* k_norm_weight, float eps,
                     int32_t num_tokens, int32_t H, int32_t H_kv, int32_t D, int32_t dtype,
                     int32_t* status, void* stream);

/*
 * Device address of pinned (page-locked) host memory, for the swap pointer
 * tables of lk_copy_blocks. No counterpart in the reference (its swaps are
 * torch copy_ calls). Returns LK_ERR_INVALID_ARG for memory that is not
 * pinned, so a kernel is never given an unmapped host address.
 */
int lk_host_device_pointer(const void* host_ptr, uint64_t* device_ptr);

/*
 * Sampling with top-k / top-p filters, fused. Replaces the filtered branch of
 * Sampler.sample (litevllm/layers/sampler.py:178-187 with _apply_top_k_top_p,
 * :204-225: softmax(x / T), zero p below the k-th largest, drop tokens whose
 * preceding sorted mass exceeds top_p, renormalise, draw) with a Gumbel-max
 * draw over the kept tokens (same distribution; bit-exact given the noise).
 * Per row: temperatures[b] (0 = greedy, filters ignored), top_k[b] (<= 0 or
 * NULL: off), top_p[b] (>= 1 or NULL: off). Noise as for lk_sample (given
 * tensor, or Philox keyed by seed / offset / row / index). Logits F32, F16
 * or BF16 ([B, V], row stride ld); tokens with equal logits are kept or
 * dropped together; with F32 logits the top-k survivors also include every
 * token whose probability equals the k-th largest (distinct fp32 logits can
 * round to one probability, and the reference keeps them all). No workspace.
 */
int lk_sample_filtered(int64_t* out_ids, const void* logits, int32_t B, int32_t V, int64_t ld,
                       const float* temperatures, const int32_t* top_k, const float* top_p,
                       const float* noise, int64_t noise_ld, uint64_t seed, uint64_t offset,
                       int32_t dtype, void* stream);

/*
 * Self-test of the bounded-wait failure path (no counterpart in the
 * reference): a kernel waits on an mbarrier that nothing arrives on, gives up
 * after timeout_ns (at most 100 ms), sets LK_STATUS_WAIT_TIMEOUT in *status
 * and returns. Faults nothing; the context stays usable.
 */
int lk_selftest_wait_timeout(int32_t* status, uint64_t timeout_ns, void* stream);

/*
 * Self-tests of two pieces of the in-kernel-noise sampler (no counterpart in
 * the reference). lk_selftest_sampler_div writes out[j * n + i] = x[i] /
 * temps[j] as the sampler computes it (Markstein's correction of x * RN(1/T),
 * IEEE division for out-of-range inputs); a caller compares it with IEEE
 * fp32 division. lk_selftest_gumbel writes the Gumbel noise the sampler
 * derives from each 32-bit Philox word bits[i].
 */
int lk_selftest_sampler_div(float* out, const float* x, int32_t n, const float* temps, int32_t nt,
                            void* stream);
int lk_selftest_gumbel(float* out, const uint32_t* bits, int32_t n, void* stream);

/*
 * Tensor-core issue-rate self-test (no counterpart in the reference): one CTA
 * per SM issues n_mma back-to-back tcgen05.mma (bf16, fp32 accumulator in
 * TMEM, M = 128; shape 0: A and B in shared memory, N = 128; 1: N = 256;
 * 2: A in TMEM, N = 128; 3: A in TMEM and B N-major, the P.V form, N = 128;
 * 4: A in shared memory and B N-major, N = 128; 5: as 0 with B in the
 * 32-byte swizzle; 6: as 0 with A and B in the 32-byte swizzle; 7: as 1 with B
 * in the 32-byte swizzle; 8-15: shapes 0-7 with consecutive MMAs rotating
 * over independent accumulators, 4 for N = 128 with A in shared memory, else 2)
 * and writes the SM cycles from first issue to
 * completion to cycles[cta] (gridDim = number of SMs), -1 and
 * LK_STATUS_WAIT_TIMEOUT in *status if the completion wait (100 ms) ran out.
 */
int lk_selftest_mma_rate(int32_t n_mma, int32_t shape, int64_t* cycles, int32_t* status,
                         void* stream);

/*
 * Allocation-free variant of lk_sample. It has no counterpart in the
 * reference. It is for callers that cannot call cudaMalloc at the point where
 * they sample: code running while another component owns the allocator
 * (a caching allocator mid-reconfiguration, an arena that must not grow),
 * hosts that forbid device allocation after start-up, and plugins handed only
 * input and output buffers. Instead of a caller workspace it uses a
 * file-scope 160 KiB __device__ scratch array that every GPU which loads this
 * library holds until the process exits; the call itself allocates and frees
 * nothing. Limits: B <= 8192 rows and B * chunks <= 16384, where chunks is
 * the vocabulary split of the call (greedy and noise-tensor rows: at most
 * 6 * SMs / B, and 1 for V <= 2048; in-kernel-noise rows lengthen their
 * chunks to stay within the limit), so every B <= 8192 fits on a 148-SM
 * B200; larger problems return LK_ERR_TOO_LARGE before any launch.
 * The first call on each device looks up the array's device address with
 * that device current (cudaGetSymbolAddress) and keeps it for the life of the
 * process; make that first call before any stream capture. The kept address
 * does not survive cudaDeviceReset on that device (a new context places the
 * array elsewhere): do not call this entry point after resetting a device. Every call shares the one array: calls that overlap on
 * the GPU (other streams, other threads) race and must be serialised by the
 * caller. Each call clears the counters it uses, so an earlier aborted call
 * leaves nothing behind. Arguments and results are those of lk_sample.
 */
int lk_sample_noalloc(int64_t* out_ids, const void* logits, int32_t B, int32_t V, int64_t ld,
                      const float* temperatures, const float* noise, int64_t noise_ld,
                      uint64_t seed, uint64_t offset, float* noise_dump, int32_t dtype,
                      void* stream);

/*
 * Repetition penalty in place, replacing _apply_repetition_penalty
 * (litevllm/layers/sampler.py:190-201) as Sampler.sample applies it
 * (:168-171, on a clone of the logits): for each row b with
 * penalties[b] != 1, every distinct id among past_token_ids[b, 0..L) (int64,
 * row stride past_ld; negative ids index from the end of the row) gets
 * s > 0 ? s / penalty : s * penalty, computed in fp32 and rounded once to the
 * logits dtype (fp32, f16, bf16; [B, V], row stride ld). Ids outside
 * [-V, V) are skipped and flagged LK_STATUS_TOKEN_OOB in *status (may be
 * NULL); the reference raises IndexError for them.
 */
int lk_repetition_penalty(void* logits, int32_t B, int32_t V, int64_t ld,
                          const int64_t* past_token_ids, int64_t past_ld, int32_t L,
                          const float* penalties, int32_t* status, int32_t dtype,
                          void* stream);

int lk_softmax_temp(float* probs, int64_t probs_ld, const void* logits, int32_t B,
                    int32_t V, int64_t ld, const float* temperatures, int32_t dtype,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LITEKERN_H */
