/*
 * nqt.h - C ABI of the B200 (sm_100a) attention + sampler + planner hot path
 * for Qwen3-TTS serving (talker and code-predictor decoders).
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * plus a cudaStream_t passed as `void*`.  Nothing here allocates device
 * memory, synchronises the stream or reads device memory on the host, so
 * every call can be recorded into a CUDA graph with static pointers.
 *
 * Return value: NQT_OK (0) or a negative NQT_ERR_* code for an argument or
 * capacity error detected on the host before any launch.  Errors that only
 * the device can see (a page id outside the pool, an exhausted page pool, a
 * bounded wait that ran out) are OR-ed as NQT_DEV_* bits into the caller's
 * device `status` word, which the host reads whenever it chooses.
 *
 * Tensor layouts follow the reference engine (nari-labs/nari-qwen3-tts,
 * src/nari_qwen3_tts/...):
 *   - paged KV layer view  [total_pages, 2, page_size, num_kv_heads, head_dim]
 *     (kind 0 = K, kind 1 = V), executor/talker_kv.py:336-340
 *   - metadata: paged_kv_indptr i32 [B+1], paged_kv_indices i32 [nnz],
 *     paged_kv_last_page_len i32 [B], qo_indptr i32 [B+1] (prefill),
 *     position_ids / write_pages / write_offsets i64 [tokens],
 *     executor/talker_kv.py:15-25, 403-480
 */
#ifndef NQT_H_
#define NQT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* host-side return codes */
#define NQT_OK 0
#define NQT_ERR_ARG (-1)         /* invalid pointer, shape, stride or dtype */
#define NQT_ERR_CUDA (-2)        /* a CUDA runtime/driver call failed */
#define NQT_ERR_CAPACITY (-3)    /* a static capacity (workspace, vocab) is too small */
#define NQT_ERR_UNSUPPORTED (-4) /* a valid shape this build has no kernel for */

/* device-side status bits (OR-ed into *status) */
#define NQT_DEV_BAD_PAGE 0x1      /* page id outside [0, total_pages); read as zeros */
#define NQT_DEV_TIMEOUT 0x2       /* a bounded mbarrier wait gave up */
#define NQT_DEV_KV_EXHAUSTED 0x4  /* planner: not enough free pages, nothing reserved */
#define NQT_DEV_BAD_SLOT 0x8      /* planner: request slot outside the table */
#define NQT_DEV_TABLE_FULL 0x10   /* planner: a request outgrew its page-table row */
#define NQT_DEV_CAPACITY 0x20     /* metadata outgrew a static buffer */
#define NQT_DEV_BAD_TOKEN 0x40    /* a token id outside [0, vocab); its row is left unchanged */

/* nqt_decode_attention_ex flags */
#define NQT_DECODE_OVERLAP_KV_WRITE 0x1 /* see nqt_decode_attention_ex */
#define NQT_DECODE_SHORT_WAIT 0x2       /* test only: see nqt_decode_attention_ex */

/* element types */
#define NQT_BF16 0
#define NQT_F16 1
#define NQT_F32 2

/* Version of this ABI; bumped on any signature change. */
int nqt_abi_version(void);

/* Last CUDA error string seen by this library on the calling thread. */
const char* nqt_last_error(void);

/*
 * Paired QK RMSNorm + RoPE with the paged K/V write, in place on q and k.
 * Replaces paired_qk_norm_rope_paged_cache_ (model/kernels.py:94-160,
 * kernel :15-91): per (token, head) fp32 RMSNorm over head_dim, times the
 * norm weight, rounded to the element type, then non-interleaved RoPE with
 * inv_freq = theta^(-2i/D); rotated K and raw V are stored into
 * layer_cache[write_pages[t], kind, write_offsets[t], h, :].
 * q/k/v: [tokens, heads, head_dim] with the given token/head strides
 * (elements) and unit stride along head_dim.  bf16 only.
 */
int nqt_qk_norm_rope_paged_kv_write(
    void* q, int64_t q_stride_tok, int64_t q_stride_head,
    void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head,
    const void* q_weight, const void* k_weight,
    const int64_t* position_ids, const int64_t* write_pages, const int64_t* write_offsets,
    void* layer_cache, int total_pages, int page_size,
    int tokens, int num_qo_heads, int num_kv_heads, int head_dim,
    float eps, float rope_theta, int dtype,
    int32_t* status, void* stream);

/*
 * Dense (code-predictor) QK RMSNorm + RoPE, optionally writing K/V into a
 * dense per-row cache at cache_position.  Replaces paired_qk_norm_rope_
 * (round_to_input=1, k_cache == NULL) and paired_qk_norm_rope_dense_cache_
 * (round_to_input=0, caches given), model/kernels.py:163-405.
 * k_cache/v_cache: [tokens, capacity, num_kv_heads, head_dim] with strides
 * (row, position, head) in elements.
 */
int nqt_qk_norm_rope_dense(
    void* q, int64_t q_stride_tok, int64_t q_stride_head,
    void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head,
    const void* q_weight, const void* k_weight,
    const int64_t* positions, int64_t positions_stride,
    void* k_cache, void* v_cache, int64_t cache_stride_row, int64_t cache_stride_pos,
    int64_t cache_stride_head, int cache_position,
    int tokens, int num_qo_heads, int num_kv_heads, int head_dim,
    float eps, float rope_theta, int round_to_input, int dtype,
    int32_t* status, void* stream);

/*
 * Workspace bytes that nqt_decode_plan / nqt_decode_attention need for a
 * capture of `batch_capacity` rows.  The caller owns the buffer (the
 * binding's uint8 workspace, executor/talker_kv.py:80-82).
 */
size_t nqt_decode_workspace_bytes(int batch_capacity, int num_qo_heads, int head_dim);

/*
 * Split-KV partition of a decode (or prefill) batch, built on the device
 * from paged_kv_indptr alone: no host round trip, CUDA-graph safe.  Takes
 * the place of BatchDecodeWithPagedKVCacheWrapper.plan
 * (executor/talker_kv.py:289-298), which needs host indptr.
 */
int nqt_decode_plan(
    const int32_t* kv_indptr, const int32_t* last_page_len, int batch, int batch_capacity,
    int page_size, int num_qo_heads, int head_dim,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Paged GQA decode attention (one query per row), split-KV with TMA page
 * gathers into shared memory; split rows are combined by LSE inside the
 * same launch (the last covering CTA finishes them).  Replaces
 * BatchDecodeWithPagedKVCacheWrapper.run (executor/talker_kv.py:305-306).
 * q/out: [batch, num_qo_heads, head_dim] bf16 with token/head strides.
 * layer_cache: contiguous [total_pages, 2, page_size, num_kv_heads, head_dim]
 * bf16.  page_size must be a multiple of 16; head_dim 64 or 128;
 * num_qo_heads / num_kv_heads <= 8; num_kv_heads <= 8.
 * The workspace must hold a plan made by nqt_decode_plan for the same
 * kv_indptr and batch.
 */
int nqt_decode_attention(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    const void* layer_cache, int total_pages, int page_size,
    const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* last_page_len,
    int batch, int batch_capacity, int num_qo_heads, int num_kv_heads, int head_dim,
    float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    void* workspace, size_t workspace_bytes,
    int32_t* status, void* stream);

/*
 * nqt_decode_attention with launch flags; flags = 0 is nqt_decode_attention.
 * Same reference interface (BatchDecodeWithPagedKVCacheWrapper.run,
 * executor/talker_kv.py:305-306), called right after the layer's K/V write
 * (attend, executor/talker_kv.py:104-130, writes K/V at :116, then runs
 * the wrapper).
 * NQT_DECODE_OVERLAP_KV_WRITE: the kernel may start while the kernel before
 * it on the stream is still running, and reads the plan in the workspace,
 * kv_indptr, kv_indices, last_page_len and every KV tile except each row's
 * last 16-token tile before that kernel has finished; q, each row's last
 * tile and all of its writes wait for it.  Pass it only when the previous
 * kernel writes none of the former, e.g. when it is
 * nqt_qk_norm_rope_paged_kv_write of one decode token per row (that token
 * lies in its row's last tile), or another decode launch on the same plan.
 * NQT_DECODE_SHORT_WAIT (for tests of the failure path only): every wait of
 * the launch's TMA pipeline gives up at once instead of after 2 s, so the
 * launch reports NQT_DEV_TIMEOUT and its output is undefined.  A launch
 * whose wait gave up still settles its split-KV fix-up state and waits for
 * its own copies in flight before exiting, so the next launch on the same
 * plan is correct.
 */
int nqt_decode_attention_ex(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    const void* layer_cache, int total_pages, int page_size,
    const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* last_page_len,
    int batch, int batch_capacity, int num_qo_heads, int num_kv_heads, int head_dim,
    float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    void* workspace, size_t workspace_bytes, int flags,
    int32_t* status, void* stream);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference:
 * it is the same split-KV decode as nqt_decode_attention (plan included),
 * for callers that cannot allocate device memory and so cannot provide a
 * workspace - e.g. a host whose device memory is owned by another runtime's
 * allocator, or a loader that only passes pointers to buffers it already
 * holds.  Its scratch (plan + split partials) is one fixed array inside the
 * library, nqt_decode_noalloc_scratch_bytes() bytes (about 5.1 MB), held on
 * every GPU that loads the library until the process exits.
 * Limits: batch <= 1024, num_qo_heads <= 32, num_qo_heads * head_dim <= 2048;
 * larger shapes return NQT_ERR_CAPACITY (see nqt_last_error).
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make it before any
 * stream capture.  The looked-up address belongs to the device's primary
 * context: after a cudaDeviceReset of that device, do not call this entry
 * point on it again in the same process.  All calls share the array: calls that may overlap on
 * the GPU (other streams or threads on the same device) race and must be
 * serialised by the caller.  Inputs, outputs and status as in
 * nqt_decode_attention.
 */
int nqt_decode_attention_noalloc(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    const void* layer_cache, int total_pages, int page_size,
    const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* last_page_len,
    int batch, int num_qo_heads, int num_kv_heads, int head_dim, float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    int32_t* status, void* stream);

/* Size of the fixed scratch array behind nqt_decode_attention_noalloc. */
size_t nqt_decode_noalloc_scratch_bytes(void);

/*
 * Ragged causal prefill attention over paged KV.  Query rows of sequence b
 * are tokens [qo_indptr[b], qo_indptr[b+1]) and are the last qo_len
 * positions of that sequence's KV, so query i sees KV positions
 * <= kv_len - qo_len + i.  Replaces BatchPrefillWithPagedKVCacheWrapper.run
 * (executor/talker_kv.py:225-226, causal=True).
 * out needs 4-byte alignment and even strides.  With head_dim 128, a 16-byte
 * aligned out whose strides are multiples of 8 elements lets every full
 * 128-row query tile leave through one TMA store (the fast path); any other
 * accepted layout is written with 4-byte stores.
 */
int nqt_prefill_attention(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    const void* layer_cache, int total_pages, int page_size,
    const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
    const int32_t* last_page_len,
    int batch, int total_q_tokens, int num_qo_heads, int num_kv_heads, int head_dim,
    float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    int32_t* status, void* stream);

/*
 * Code-predictor decode step, fused: QK RMSNorm + RoPE of the new token
 * (no rounding before RoPE), K/V write into the dense cache at
 * cache_position, then one-query GQA attention over positions
 * [0, cache_position].  Replaces paired_qk_norm_rope_dense_cache_ followed
 * by decode_attn_nhd_short_cache (model/kernels.py:335-520 as called from
 * model/components.py:309-345).  q is rotated in place (bf16), like the
 * reference.  k_cache/v_cache as in nqt_qk_norm_rope_dense.
 */
int nqt_cp_decode_attention(
    void* q, int64_t q_stride_tok, int64_t q_stride_head,
    void* k, int64_t k_stride_tok, int64_t k_stride_head,
    const void* v, int64_t v_stride_tok, int64_t v_stride_head,
    const void* q_weight, const void* k_weight,
    const int64_t* positions, int64_t positions_stride,
    void* k_cache, void* v_cache, int64_t cache_stride_row, int64_t cache_stride_pos,
    int64_t cache_stride_head, int cache_capacity, int cache_position,
    int rows, int num_qo_heads, int num_kv_heads, int head_dim,
    float eps, float rope_theta, float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    int32_t* status, void* stream);

/*
 * Short-cache one-query attention over positions [0, cache_length) of a
 * dense cache.  Replaces decode_attn_nhd_short_cache (model/kernels.py:466-520).
 */
int nqt_cp_short_attention(
    const void* q, int64_t q_stride_tok, int64_t q_stride_head,
    const void* k_cache, const void* v_cache, int64_t cache_stride_row,
    int64_t cache_stride_pos, int64_t cache_stride_head, int cache_length,
    int rows, int num_qo_heads, int num_kv_heads, int head_dim, float sm_scale,
    void* out, int64_t out_stride_tok, int64_t out_stride_head,
    int32_t* status, void* stream);

/*
 * Fused logits sampler, one CTA per row: repetition penalty on the seen
 * mask, greedy argmax when temperature == 0, otherwise x / T, top-k
 * (k <= 0 means the whole vocabulary), softmax over the top-k values,
 * top-p (drop ranks whose exclusive cumulative mass exceeds top_p),
 * renormalise, then an exponential-race draw argmax(p_i / E_i) with
 * E_i = -log(U_i) and U_i from Philox4x32-10 keyed by (seed, offset, rank):
 * the draw depends only on the row's own (seed, offset), never its batch
 * position.  Semantics follow sample_logits_stateless
 * (model/sampling.py:127-225, _cpu_sample_row :68-95); replaces
 * sample_talker_cuda_graph (executor/sampling.py:156-198, plus the seen
 * scatter at executor/talker.py:373 when update_seen != 0),
 * sample_logits_cuda_graph (:201-239) and sample_code_predictor_cuda_graph
 * (:305-336).
 *   logits [rows, vocab] (bf16/f16/f32, row stride in elements);
 *   temperature f32 [rows]; top_k i32 [rows]; top_p f32 [rows];
 *   seed i64 [rows]; offset i64 [rows] (element stride offset_stride);
 *   repetition_penalty f32 [rows] or NULL; seen u8/bool [rows, vocab] or NULL;
 *   round_scaled_to_input: round x / T to the logits type (what torch does
 *   for a half-precision row without a seen mask);
 *   tokens_out i64 [rows];
 *   probs_out f32 [rows, vocab] or NULL: filtered, renormalised probabilities
 *   in rank order (zeros past the kept ranks); ids_out i32 [rows, vocab] or
 *   NULL: token id of each rank.
 */
int nqt_sample_rows(
    const void* logits, int logits_dtype, int64_t logits_stride, int rows, int vocab,
    const float* temperature, const int32_t* top_k, const float* top_p,
    const int64_t* seed, const int64_t* offset, int64_t offset_stride,
    const float* repetition_penalty, uint8_t* seen, int64_t seen_stride, int update_seen,
    int round_scaled_to_input,
    int64_t* tokens_out, float* probs_out, int32_t* ids_out,
    int32_t* status, void* stream);

/*
 * Parity entry of nqt_sample_rows: identical, except the exponential noise
 * E_i of rank i is read from noise[row * noise_stride + i] instead of being
 * generated.  With E drawn from torch's CPU generator seeded like
 * _cpu_sample_row (model/sampling.py:89-94), argmax(p / E) equals
 * torch.multinomial(p, 1) there, so sampled ids can be compared exactly.
 */
int nqt_sample_rows_noise(
    const void* logits, int logits_dtype, int64_t logits_stride, int rows, int vocab,
    const float* temperature, const int32_t* top_k, const float* top_p,
    const float* noise, int64_t noise_stride,
    const float* repetition_penalty, uint8_t* seen, int64_t seen_stride, int update_seen,
    int round_scaled_to_input,
    int64_t* tokens_out, float* probs_out, int32_t* ids_out,
    int32_t* status, void* stream);

/*
 * GPU planner state: one device-resident page pool per GPU.
 *   free_bitmap u32 [ceil(total_pages/32)]  bit set = page free;
 *   seq_len i32 [slots], pos_start i32 [slots], n_pages i32 [slots],
 *   page_table i32 [slots, max_pages_per_slot].
 * Allocation order is the reference allocator's: lowest free page first,
 * rows in order (executor/cache.py:135-184).
 */
size_t nqt_planner_state_bytes(int total_pages, int slots, int max_pages_per_slot);

/* Reset the planner state: every page free except the scratch pages, which
 * are claimed as the `scratch_count` lowest pages (executor/cache.py:103-112). */
int nqt_planner_init(void* state, int total_pages, int slots, int max_pages_per_slot,
                     int scratch_count, void* stream);

/*
 * One planning step for the rows of the next batch, entirely on the device.
 * Replaces PagedTalkerKV._metadata + PagedKVAllocator.reserve
 * (executor/talker_kv.py:403-480, executor/cache.py:135-184).
 *   row_slot i32 [capture_rows] (slot of row r, or -1 for padding rows);
 *   row_advance i32 [capture_rows] (tokens appended by row r);
 *   scratch_pages i32 [scratch_count].
 * Writes the step's metadata into the binding's static buffers
 * (qo_indptr may be NULL for decode) and the proposed page lists into
 * `pending` (i32 [capture_rows, max_pages_per_slot + 1]) for a later commit.
 * When the pool cannot cover the step, NQT_DEV_KV_EXHAUSTED is set and no
 * page is reserved, like KVAllocationError (executor/cache.py:155-158).
 * If `decode_workspace` is not NULL the split-KV plan of nqt_decode_plan is
 * built in the same call.  With position_ids, write_pages and write_offsets
 * all NULL the step only reserves pages and writes the row-level metadata
 * (admitting a request whose KV is filled elsewhere); token_capacity is then
 * ignored.
 */
int nqt_plan_step(
    void* state, int total_pages, int slots, int max_pages_per_slot, int page_size,
    const int32_t* row_slot, const int32_t* row_advance, int capture_rows, int token_capacity,
    const int32_t* scratch_pages, int scratch_count, int prefill,
    int32_t* qo_indptr, int32_t* kv_indptr, int32_t* kv_indices, int kv_indices_capacity,
    int32_t* last_page_len, int64_t* position_ids, int64_t* write_pages, int64_t* write_offsets,
    int32_t* pending,
    void* decode_workspace, size_t decode_workspace_bytes, int num_qo_heads, int head_dim,
    int32_t* status, void* stream);

/*
 * Publish (row_publish[r] != 0) or discard the pending reservation of each
 * real row of the last nqt_plan_step: publish advances seq_len/pos_start
 * and adopts the proposed pages; discard returns the new pages to the pool.
 * Mirrors PendingKVPublication.publish/discard (executor/cache.py:77-83,
 * 186-212).  Each committed row's pending entry is marked consumed, so a
 * second commit of the same plan changes nothing (the reference raises
 * StaleKVPublicationError there).
 */
int nqt_plan_commit(
    void* state, int total_pages, int slots, int max_pages_per_slot,
    const int32_t* row_slot, const int32_t* row_advance, const int32_t* row_publish,
    int capture_rows, int32_t* pending, int32_t* status, void* stream);

/*
 * Release every page of the listed slots and reset them to empty
 * (remove_request, executor/cache.py:127-133).  slot_list i32 [count].
 */
int nqt_plan_release(
    void* state, int total_pages, int slots, int max_pages_per_slot,
    const int32_t* slot_list, int count, int32_t* status, void* stream);

/*
 * Install an existing page list for one slot (state import: a request
 * whose KV was written elsewhere, or a benchmark's scattered pages).  The
 * pages are marked used.  pages i32 [n_pages] in sequence order.
 */
int nqt_plan_import(
    void* state, int total_pages, int slots, int max_pages_per_slot,
    int slot, const int32_t* pages, int n_pages, int seq_len, int pos_start,
    int32_t* status, void* stream);

/*
 * Talker layer glue (one launch each, fp32 math, bf16/f16 storage).
 * nqt_rmsnorm replaces flashinfer.norm.rmsnorm at model/layers.py:80-100;
 * nqt_fused_add_rmsnorm replaces flashinfer.norm.fused_add_rmsnorm at
 * model/layers.py:42-77 (residual <- x + residual; x <- rmsnorm(residual) * w,
 * both in place); nqt_silu_and_mul replaces flashinfer.activation.silu_and_mul
 * at model/layers.py:28-39 (out = silu(gate) * up, gate_up = [gate | up]).
 * Rows are contiguous in hidden / 2d; strides in elements.
 */
int nqt_rmsnorm(const void* x, int64_t x_stride, const void* weight, void* out, int64_t out_stride,
                int rows, int hidden, float eps, int dtype, void* stream);
int nqt_fused_add_rmsnorm(void* x, void* residual, const void* weight, int rows, int hidden, float eps,
                          int dtype, void* stream);
int nqt_silu_and_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                     int rows, int d, int dtype, void* stream);

/*
 * Decoder projection Y[m, n] = X[m, k] . W[n, k]^T (bf16, fp32 accumulate;
 * nn.Linear weight layout), a weight-streaming tcgen05 GEMM for m <= 256.
 * Replaces the torch/cuBLAS projections of the decoder layers
 * (model/layers.py:195-270 and model/components.py:300-356, the CP
 * small_to_mtp_projection and lm heads at executor/code_predictor.py:221)
 * and the sm90-only fused gate/up path (executor/optimizations.py:22-47).
 *
 * nqt_gemm_pack_weight lays W out once (at load time) as contiguous 16 KB
 * tiles [n / 128][k / 64][128 rows x 64] in the MMA's 128-byte-swizzled
 * order; packed holds n * k bf16.  interleave_gate_up = 1 packs a gate_up
 * weight [gate (n/2 rows) | up (n/2 rows)] as blocks [gate 64 | up 64] for
 * epilogue 2.
 *
 * nqt_gemm_bf16 on a packed weight:
 *   epilogue 0  Y = bf16(acc)
 *   epilogue 1  Y = bf16(acc + bias[n])
 *   epilogue 2  (weight packed with interleave_gate_up) Y[m, f] =
 *               silu(g) * up, g and up rounded to bf16 (the gate_up GEMM
 *               followed by nqt_silu_and_mul); Y is [m, n / 2].
 * 1 <= m <= 256, n % 128 == 0, k % 64 == 0; x and the packed weight
 * 16-byte aligned, ldx (elements) a multiple of 8.  split = CTAs (one
 * thread-block cluster) that share each 128-row tile's K and sum their fp32
 * partials through distributed shared memory, 1..8; 0 picks the largest
 * power of two that keeps the grid within one CTA per SM.  No workspace:
 * calls on different streams may overlap.  Launched with programmatic
 * stream serialization (the weight copies start before the previous kernel
 * has finished).
 */
int nqt_gemm_pack_weight(const void* w, int64_t ldw, int n, int k, int interleave_gate_up, void* packed,
                         void* stream);
int nqt_gemm_bf16(const void* x, int64_t ldx, const void* w_packed, void* y, int64_t ldy, const void* bias,
                  int m, int n, int k, int epilogue, int split, int32_t* status, void* stream);

/*
 * Code-predictor frame glue after codebook g's tokens are sampled, one launch for the six torch ops of the
 * whole-frame loop (executor/code_predictor.py:160-235; the next step's input norm,
 * model/components.py:254-258).  Per row: frames[row * frames_stride] = token;
 * codec_sum[row] = bf16(codec_sum[row] + codec_emb[token]) (accumulate != 0) or codec_emb[token];
 * when proj_emb is given, residual[row] = proj_emb[token] and h[row] = bf16(rmsnorm(residual[row]) * ln)
 * (the nqt_rmsnorm arithmetic).  codec_emb [vocab, talker_hidden], proj_emb [vocab, hidden], rows
 * contiguous, bf16, 16-byte aligned; hidden <= 4096.  Tokens outside [0, vocab) set NQT_DEV_BAD_TOKEN.
 */
int nqt_cp_codec_step(const int64_t* tokens, int rows, int64_t* frames, int64_t frames_stride,
                      const void* codec_emb, int vocab, int talker_hidden, void* codec_sum, int accumulate,
                      const void* proj_emb, const void* ln, int hidden, float eps, void* residual, void* h,
                      int dtype, int32_t* status, void* stream);

/*
 * FP8 (e4m3) block-scaled gate/up projection.  The reference's production
 * executor requires it for every talker layer (executor/build.py:73,
 * executor/optimizations.py:22-47), on a path that only starts on sm90.
 *
 * nqt_fp8_quantize_weight_blocks replaces quantize_fp8_weight_blocks
 * (model/layers.py:11-25): per 128 x 128 block of the bf16 weight [n, k],
 * s = 2^ceil(log2(max(amax, 1e-4) / 448)) and q = e4m3(w / s).  Outputs in
 * the reference's layout: q [n, k] row-major (ldq bytes), scale f32
 * [n / 128, k / 128].  n, k multiples of 128.
 *
 * nqt_fp8_quantize_rows is the activation rule of the reference's GEMM on a
 * bf16 input (model/layers.py:242-256, flashinfer fp8_blockscale_gemm_sm90:
 * per token per 128-element block, f = 448 / amax or 1 when amax = 0,
 * q = e4m3(x * f), scale = 1 / f).  q [m, k] (ldq bytes); scale f32
 * K-block-major: scale[b * ld_scale + row], ld_scale >= m.
 *
 * nqt_fused_add_rmsnorm_fp8 is nqt_fused_add_rmsnorm (bf16) whose output row
 * is quantised by that rule into q / scale (same layouts); the bf16 normed
 * row is also written to x when write_x != 0.  hidden % 128 == 0.
 *
 * nqt_gemm_fp8_pack_weight lays q out once as 16 KB units [n / 128][k / 128]
 * [128 rows x 128 B] in the MMA's swizzled order (interleave_gate_up: unit
 * rows in 32-row groups [gate 16 | up 16], so unit t holds gate and up rows
 * 64 t .. 64 t + 63 of a weight [gate (n/2 rows) | up (n/2 rows)]).
 *
 * nqt_gemm_fp8: Y = sum over K blocks b of (Xq_b . Wq_b^T) * xscale[b, row] *
 * wscale[weight row / 128, b] (fp32), epilogue 0 (Y = bf16) or 2 (packed with
 * interleave_gate_up: Y[m, f] = silu(bf16 g) * bf16 up, Y is [m, n / 2]).
 * wscale is the quantiser's [n / 128, k / 128] table in the unpacked row
 * order.  m >= 1 (chunks of up to 128 tokens), n % 128 == 0 (n % 256 with
 * interleave_gate_up), k % 128 == 0; xq and the packed weight 16-byte
 * aligned, ldxq a multiple of 16.  split bits 0-7: CTAs that share each
 * tile's K, 1..8, 0 = automatic (every SM streams about the same number of
 * K blocks); bits 8-11: K blocks per copy stage, 0 = automatic.  A split
 * sums its fp32 partials through `workspace` (256-byte aligned, at least
 * nqt_gemm_fp8_workspace_bytes for the same m, n, k and split; none is needed
 * when that is 0): zero it once before the first call; every launch returns
 * its tickets to zero.  A workspace's tickets are laid out for one (m, n, k,
 * split): give each shape its own workspace (or zero it before another
 * shape uses it), and run one launch at a time per workspace.  Launched with
 * programmatic stream serialization.
 */
int nqt_fp8_quantize_weight_blocks(const void* w, int64_t ldw, int n, int k, void* q, int64_t ldq, float* scale,
                                   void* stream);
int nqt_fp8_quantize_rows(const void* x, int64_t ldx, int m, int k, void* q, int64_t ldq, float* scale,
                          int64_t ld_scale, void* stream);
int nqt_fused_add_rmsnorm_fp8(void* x, void* residual, const void* weight, int rows, int hidden, float eps, void* q,
                              int64_t ldq, float* scale, int64_t ld_scale, int write_x, int dtype, void* stream);
int nqt_gemm_fp8_pack_weight(const void* q, int64_t ldq, int n, int k, int interleave_gate_up, void* packed,
                             void* stream);
int nqt_gemm_fp8_workspace_bytes(int m, int n, int k, int split, int64_t* bytes);
int nqt_gemm_fp8(const void* xq, int64_t ldxq, const float* xscale, int64_t ld_xscale, const void* w_packed,
                 const float* wscale, void* y, int64_t ldy, int m, int n, int k, int epilogue,
                 int interleave_gate_up, int split, void* workspace, int64_t workspace_bytes, int32_t* status,
                 void* stream);

/*
 * Device-side request control of a talker step (no host staging before a captured step, no per-row
 * host read after it).  Per-request state lives in a slot table on the device; rows name their slot
 * (row_slot[r] < 0 marks a padding row).  Distinct rows must name distinct slots.
 *
 * nqt_step_stage gathers each row's sampler parameters from its slot - it replaces the pinned host
 * staging of TalkerExecutor._stage_sampling_rows (executor/talker.py:527-563, padding rows take its
 * defaults: temperature 0, top_k 1, top_p 1, penalty 1, seed 0, offset 0) - and, when suppress_eos is
 * given, the row's EOS-suppression flag step < eos_from (engine/input_builder.py:60-70: eos_from is
 * INT32_MAX while EOS is suppressed indefinitely, else max(2, token_count - 1) for a terminal
 * continuation, else 2).  slot_penalty and penalty are both given or both NULL.
 */
int nqt_step_stage(
    const int32_t* row_slot, int rows, int slots,
    const float* slot_temperature, const int32_t* slot_top_k, const float* slot_top_p,
    const float* slot_penalty, const int64_t* slot_seed, const int64_t* slot_offset,
    const int32_t* slot_step, const int32_t* slot_eos_from,
    float* temperature, int32_t* top_k, float* top_p, float* penalty, int64_t* seed, int64_t* offset,
    uint8_t* suppress_eos, int32_t* status, void* stream);

/*
 * The codec head's suppress mask, in place on logits [rows, vocab] (stride logits_stride elements):
 * columns >= codec_vocab become -inf except eos_id, and eos_id becomes -inf on rows with
 * suppress_eos[r] != 0 (Qwen3TTSTalkerExecutor.forward_logits, executor/talker.py:170-183, 241-243).
 * eos_id < 0: no EOS column.  suppress_eos may be NULL (no row suppressed).
 */
int nqt_talker_logits_mask(void* logits, int dtype, int64_t logits_stride, int rows, int vocab, int codec_vocab,
                           int eos_id, const uint8_t* suppress_eos, void* stream);

/*
 * The decode completion rule of SynthesisPipeline (engine/pipeline.py:583-609) on the device, which
 * replaces its per-row host read tokens[i].item(): reached_limit = step + 1 >= max_tokens;
 * eos = tokens[r] == eos_id on a row whose EOS is not suppressed (step < eos_from) and that has not
 * reached the limit; terminal[r] = eos || reached_limit.  Then each live row's slot advances: step + 1
 * and offset + offset_stride (TALKER_FRAME_OFFSET_STRIDE = 512, executor/talker.py:606).
 * n_terminal (optional) is incremented once per terminal row.
 */
int nqt_step_finish(const int32_t* row_slot, int rows, int slots, const int64_t* tokens, int eos_id,
                    int32_t* slot_step, const int32_t* slot_max_tokens, const int32_t* slot_eos_from,
                    int64_t* slot_offset, int64_t offset_stride, uint8_t* terminal, int32_t* n_terminal,
                    int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NQT_H_ */
