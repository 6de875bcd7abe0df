/*
 * nslg_b200.h -- C ABI of the B200 (sm_100a) kernels behind NanoSLG's per-layer
 * attention path.
 *
 * Every entry point takes raw device pointers (nslg_plan_decode_host: host arrays for
 * its inputs), element strides and sizes, plus the cudaStream_t to launch on (passed as
 * void*), and returns an int status (NSLG_OK == 0).  On a non-zero status
 * nslg_last_error() returns a message for the calling thread.  Apart from
 * nslg_ipc_alloc, whose job it is, no entry point allocates device memory: scratch
 * space is passed in by the caller (see nslg_decode_workspace_bytes), with one
 * exception, nslg_paged_decode_noalloc, whose scratch is a fixed
 * NSLG_NOALLOC_SCRATCH_BYTES __device__ array compiled into the library (held on every
 * GPU that loads it); nslg_plan_decode_host keeps pinned host staging of its own.
 *
 * Errors that can only be seen on the device (a page id outside the pool, a write
 * slot outside the pool, a position outside the RoPE table) never trap: the kernel
 * skips the access and ORs an NSLG_DEV_* bit into *dev_status (when dev_status is not
 * NULL).  The caller reads it whenever it chooses to synchronise.
 *
 * Layouts follow the reference (nanoslg/kv_cache.py):
 *   KV pool, one layer:  [num_pages, page_size, num_kv_heads, head_dim]  ("NHD",
 *                        kv_cache.py:384-392, PagePool.k[layer] / PagePool.v[layer])
 *   CSR page list:       kv_indptr[B+1], kv_indices[kv_indptr[B]],
 *                        kv_last_page_len[B]  (kv_cache.py:598-615, the arrays the
 *                        reference hands to FlashInfer's plan())
 */
#ifndef NSLG_B200_H
#define NSLG_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types (the reference runs float32, bfloat16 and float16 activations,
 * worker.py:22-26) */
#define NSLG_DTYPE_F32 0
#define NSLG_DTYPE_BF16 1
#define NSLG_DTYPE_F16 2

/* host-side status codes */
#define NSLG_OK 0
#define NSLG_ERR_ARG 1         /* invalid argument: null pointer, bad size or stride    */
#define NSLG_ERR_UNSUPPORTED 2 /* shape / dtype combination this build does not cover  */
#define NSLG_ERR_CUDA 3        /* a CUDA runtime call failed (message has the details)  */
#define NSLG_ERR_WORKSPACE 4   /* workspace smaller than nslg_decode_workspace_bytes()  */

/* device-side status bits (ORed into *dev_status) */
#define NSLG_DEV_BAD_PAGE 1u     /* kv_indices entry outside [0, num_pages)            */
#define NSLG_DEV_BAD_SLOT 2u     /* write location outside the pool                    */
#define NSLG_DEV_BAD_POSITION 4u /* RoPE position outside the cos/sin table            */
#define NSLG_DEV_WAIT_TIMEOUT 8u /* a bounded pipeline wait gave up (kernel returned)  */
#define NSLG_DEV_BAD_PLAN 16u    /* plan input outside the block tables / plan buffer   */

/* Library version string. */
const char* nslg_version(void);

/* Message for the last non-OK status returned on this thread ("" if none). */
const char* nslg_last_error(void);

/* Fused rotary embedding + paged KV append.
 *
 * Replaces the reference's RoPE on q and k (models.py:99-103, apply_rotary_emb at
 * models.py:69-83: rotate-half, cos/sin cast to the activation type) followed by the
 * KV write of attend() (kv_cache.py:661-674 paged, kv_cache.py:302-310 contiguous).
 *
 *   q[t, h, :]  at q + t*q_stride + h*head_dim   (t < num_tokens, h < num_qo_heads)
 *   k, v        likewise with k_stride / v_stride and num_kv_heads
 *   q_out       contiguous [num_tokens, num_qo_heads, head_dim]: rotated q
 *   positions   [num_tokens] int32 row of cos/sin for each token; NULL = no rotation
 *   cos_table, sin_table  fp32 [table_rows, head_dim] (models.py:37-66 layout)
 *   write_loc   [num_tokens] int32 page*page_size + slot; < 0 = token not written
 *   pool_k, pool_v        one layer of the pool, pool_slots = num_pages*page_size rows
 *                         of [num_kv_heads, head_dim]; receive rotated k and plain v.
 * head_dim must be even and a multiple of 16 (bf16) / 8 (fp32); rows 16-byte aligned.
 */
int nslg_rope_kv_append(int dtype, int num_tokens, int num_qo_heads, int num_kv_heads,
                        int head_dim, const void* q, int64_t q_stride, const void* k,
                        int64_t k_stride, const void* v, int64_t v_stride, void* q_out,
                        const int32_t* positions, const float* cos_table,
                        const float* sin_table, int64_t table_rows,
                        const int32_t* write_loc, void* pool_k, void* pool_v,
                        int64_t pool_slots, uint32_t* dev_status, void* stream);

/* Bytes of scratch nslg_paged_decode needs for this batch / head count / head_dim on
 * the current device.  The workspace must be zeroed before its first use (cudaMemset);
 * the kernel keeps per-CTA arrival counts at its head and leaves them zero after every
 * call, so a workspace kept from call to call (any batch, head count or head_dim that
 * fits) needs no further zeroing.  Do not share it between calls that may overlap on
 * the GPU. */
int64_t nslg_decode_workspace_bytes(int batch, int num_qo_heads, int head_dim);

/* Batched paged decode attention: one query token per sequence.
 *
 * Replaces FlashInferCacheContext.attend's decode branch (kv_cache.py:648-651,
 * BatchDecodeWithPagedKVCacheWrapper.run over the CSR built at kv_cache.py:598-621)
 * and ContiguousCacheContext.attend's SDPA for S == 1 (kv_cache.py:312-322).
 *
 *   q[b, h, :]   at q + b*q_stride + h*head_dim    [batch, num_qo_heads, head_dim]
 *   out[b, h, :] at out + b*out_stride + h*head_dim
 *   out = softmax(sm_scale * q . K^T) V over the kv_len(b) tokens of sequence b,
 *   kv_len(b) = (kv_indptr[b+1]-kv_indptr[b]-1)*page_size + kv_last_page_len[b].
 * GQA: query head h reads kv head h / (num_qo_heads / num_kv_heads).
 * Sequences with no pages produce zeros.
 * One kernel launch: sequences split across CTAs are combined by the last CTA to finish
 * its share (arrival counts in the workspace), with no second kernel.
 * Launched with programmatic dependent launch: it may start while the kernel before it
 * on the stream runs, if that kernel allows its dependents to launch early (the library's
 * KV-append, RMSNorm and SwiGLU kernels do). It reads q and the pool only after that
 * kernel has finished, but the CSR arrays (kv_indptr, kv_indices, kv_last_page_len)
 * before: they must be written by work that finished before that kernel started (the
 * planner's kernels never allow an early launch, so a plan followed directly by this
 * call is always safe).
 */
int nslg_paged_decode(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                      int head_dim, int page_size, const void* q, int64_t q_stride,
                      void* out, int64_t out_stride, const void* pool_k,
                      const void* pool_v, int64_t num_pages, const int32_t* kv_indptr,
                      const int32_t* kv_indices, const int32_t* kv_last_page_len,
                      float sm_scale, void* workspace, int64_t workspace_bytes,
                      uint32_t* dev_status, void* stream);

/* Decode attention of a small batch split by kv head as well as by pages: sequence
 * b * num_kv_heads + h is kv head h of sequence b with its group of num_qo_heads /
 * num_kv_heads query heads, so batch 1 spreads over many more CTAs without more partials
 * per query head. The page list comes from nslg_split_heads_plan (v_indptr, v_indices,
 * v_last_page_len, built once per step from the plan's CSR). q and out are contiguous
 * [batch, num_qo_heads, head_dim]; the pool, scale, workspace and status as in
 * nslg_paged_decode (the workspace sized for batch * num_kv_heads sequences of the group
 * size: nslg_decode_workspace_bytes(batch * num_kv_heads, group, head_dim)). The same
 * attention as nslg_paged_decode with the plain CSR, within fp32 rounding of the merge
 * order. No counterpart in the reference (it is a work split of the decode of
 * kv_cache.py:639-651); NSLG_ERR_UNSUPPORTED off the tensor-core path or for one kv
 * head. */
int nslg_paged_decode_split_heads(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                                  int head_dim, int page_size, const void* q, void* out,
                                  const void* pool_k, const void* pool_v, int64_t num_pages,
                                  const int32_t* v_indptr, const int32_t* v_indices,
                                  const int32_t* v_last_page_len, float sm_scale,
                                  void* workspace, int64_t workspace_bytes,
                                  uint32_t* dev_status, void* stream);

/* The page list of nslg_paged_decode_split_heads from a decode plan's CSR (kv_indptr
 * [batch + 1], kv_indices, kv_last_page_len [batch], device arrays): v_indptr
 * [batch * num_kv_heads + 1], v_indices [num_kv_heads * kv_indptr[batch] <=
 * max_v_indices] (page * num_kv_heads + h), v_last_page_len [batch * num_kv_heads]. One
 * launch, graph-capturable; a page list longer than max_v_indices sets NSLG_DEV_BAD_PLAN.
 * No counterpart in the reference. */
int nslg_split_heads_plan(int batch, int num_kv_heads, const int32_t* kv_indptr,
                          const int32_t* kv_indices, const int32_t* kv_last_page_len,
                          int32_t* v_indptr, int32_t* v_indices, int32_t* v_last_page_len,
                          int64_t max_v_indices, int64_t num_pages, uint32_t* dev_status,
                          void* stream);

/* The decode step of CacheContext.attend in one call: the new token's k and v of each
 * sequence appended to the pool at write_loc (nslg_rope_kv_append without rotation, q
 * and k already rotated as attend() receives them), then nslg_paged_decode over the
 * sequences' pages, the new token included. Arguments as in those two calls; k and v are
 * [batch, num_kv_heads, head_dim] rows with strides k_stride / v_stride. Replaces the
 * decode branch of FlashInferCacheContext.attend (kv_cache.py:639-651: _write_kv, then
 * the decode wrapper's run). */
int nslg_append_paged_decode(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                             int head_dim, int page_size, const void* q, int64_t q_stride,
                             const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                             const int32_t* write_loc, void* out, int64_t out_stride,
                             void* pool_k, void* pool_v, int64_t num_pages,
                             const int32_t* kv_indptr, const int32_t* kv_indices,
                             const int32_t* kv_last_page_len, float sm_scale, void* workspace,
                             int64_t workspace_bytes, uint32_t* dev_status, void* stream);

/* Scratch size of nslg_paged_decode_noalloc: a fixed device array inside the library. */
#define NSLG_NOALLOC_SCRATCH_BYTES (8ll << 20)

/* nslg_paged_decode for callers that cannot allocate device memory.
 *
 * No counterpart in the reference (NanoSLG always lets FlashInfer use a workspace it
 * allocated). For callers with no device allocator of their own -- a serving process
 * that gave nearly all HBM to its KV page pool and runs on a fixed budget, a host
 * program in another language binding this ABI, a decode loop that cannot take the
 * synchronisation of cudaMalloc/cudaFree. Same arguments and result as
 * nslg_paged_decode minus the workspace: the split-KV partials go to a fixed
 * NSLG_NOALLOC_SCRATCH_BYTES array compiled into the library, which every GPU that loads
 * the library holds until the process exits (zeroed at load, and the arrival counts at
 * its head are left zero by every call). Batches whose scratch
 * ((batch + #SMs) * num_qo_heads * (head_dim + 1) * 4 bytes, plus 1 KiB) exceeds it are
 * rejected with NSLG_ERR_WORKSPACE. The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress) with that device current; make it before any stream capture.
 * The address is kept with the CUDA context it belongs to: the first call in another
 * context (after cudaDeviceReset, or in a context the caller created) looks it up again
 * and must also come before any capture.
 * All calls on a device share the array, so calls that overlap on the GPU race: order
 * them. Allocates and frees nothing. */
int nslg_paged_decode_noalloc(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                              int head_dim, int page_size, const void* q, int64_t q_stride,
                              void* out, int64_t out_stride, const void* pool_k,
                              const void* pool_v, int64_t num_pages, const int32_t* kv_indptr,
                              const int32_t* kv_indices, const int32_t* kv_last_page_len,
                              float sm_scale, uint32_t* dev_status, void* stream);

/* Batched paged prefill / extend attention with a causal mask.
 *
 * Replaces FlashInferCacheContext.attend's prefill branch (kv_cache.py:652-655,
 * BatchPrefillWithPagedKVCacheWrapper.run with causal=True, planned at
 * kv_cache.py:622-632) together with _pack_q/_unpack (kv_cache.py:676-691), and the
 * masked SDPA of ContiguousCacheContext.attend (kv_cache.py:312-322 with the mask of
 * _build_causal_mask, kv_cache.py:192-224).
 *
 * Sequence b has qo_len(b) = qo_indptr[b+1]-qo_indptr[b] new query rows; its rows live
 * at q + (q_row_start[b] + i)*q_stride (i < qo_len(b)), or at qo_indptr[b] + i when
 * q_row_start is NULL; outputs at the same rows of out.  Row i sits at absolute
 * position kv_len(b) - qo_len(b) + i and, when causal != 0, attends to kv positions
 * <= that position (the reference's kpos <= start + i  and  kpos < seq_len).
 * q and out hold q_rows rows (the extent of the TMA view of q; rows past it read as
 * zero). max_qo_len bounds qo_len(b). bf16 with head_dim 128, page_size 16 and a GQA
 * group (num_qo_heads / num_kv_heads) that divides 128 runs on tcgen05 tensor cores;
 * other shapes and fp32 run on CUDA cores.
 */
int nslg_paged_prefill(int dtype, int batch, int num_qo_heads, int num_kv_heads,
                       int head_dim, int page_size, const void* q, int64_t q_stride,
                       int64_t q_rows, void* out, int64_t out_stride, const int32_t* qo_indptr,
                       const int32_t* q_row_start, int max_qo_len, const void* pool_k,
                       const void* pool_v, int64_t num_pages, const int32_t* kv_indptr,
                       const int32_t* kv_indices, const int32_t* kv_last_page_len,
                       float sm_scale, int causal, uint32_t* dev_status, void* stream);

/* Fused residual add + RMSNorm.
 *
 * Replaces RMSNorm.forward (models.py:31-34: fp32 statistics, normalised value rounded
 * to the activation type, then multiplied by the weight) and the residual adds around
 * it (models.py:169-172).
 *   residual == NULL:  out = rmsnorm(x) * weight
 *   residual != NULL:  residual = x + residual (rounded to dtype, in place);
 *                      out = rmsnorm(residual) * weight
 * x, residual, out: [rows, hidden] with row strides x_stride / residual_stride /
 * out_stride (elements); weight: [hidden].
 */
int nslg_rmsnorm_residual(int dtype, int rows, int hidden, const void* x,
                          int64_t x_stride, void* residual, int64_t residual_stride,
                          const void* weight, void* out, int64_t out_stride, float eps,
                          void* stream);

/* SwiGLU activation on a fused gate|up projection output.
 *
 * Replaces F.silu(gate_proj(x)) * up_proj(x) (models.py:156-157) when the gate and up
 * weights are stacked into one GEMM: gate_up is [rows, 2*inter] (gate in columns
 * [0, inter), up in [inter, 2*inter)) with row stride gate_up_stride; out [rows, inter]
 * with row stride out_stride receives silu(gate) * up, each op rounded to dtype as in
 * the reference.
 */
int nslg_silu_mul(int dtype, int rows, int inter, const void* gate_up, int64_t gate_up_stride,
                  void* out, int64_t out_stride, void* stream);

/* Linear layer of a decode step on the tcgen05 tensor cores:
 *   y[rows, out_features] = x[rows, in_features] . weight[out_features, in_features]^T
 * bf16 or fp16 (x, weight and y of one type), fp32 accumulation, rounded once.
 *
 * Replaces F.linear in ColumnParallelLinear / RowParallelLinear (tp_layers.py:28-158,
 * and the q|k|v and gate|up projections stacked into one weight each) and the LM head
 * (tp_layers.py:210-234) for forwards of 1 <= rows <= 256 (decode steps); larger
 * forwards stay cuBLAS GEMMs. in_features must be a multiple of 64; x and weight rows
 * 16-byte aligned (strides in elements). Needs no workspace: a split of the in_features
 * sum across CTAs is reduced on chip, within a thread-block cluster. */
int nslg_linear(int dtype, int rows, int out_features, int in_features, const void* x,
                int64_t x_stride, const void* weight, int64_t w_stride, void* y,
                int64_t y_stride, uint32_t* dev_status, void* stream);

/* The MLP's gate|up product and its SwiGLU in one kernel (nslg_linear's tcgen05 path):
 *   out[rows, inter] = silu(x . gate^T) * (x . up^T)
 * with gate_up = [gate; up], 2 * inter rows of w_stride elements (gate rows first),
 * rounded as the reference does (models.py:156-157: each product rounded to the
 * activation type, silu rounded, the product rounded) -- the same values as
 * nslg_linear followed by nslg_silu_mul, without the [rows, 2 * inter] intermediate or
 * the second kernel. Replaces F.silu(gate_proj(x)) * up_proj(x) (models.py:156-157,
 * gate_proj / up_proj being ColumnParallelLinear, tp_layers.py:28-91) for decode
 * batches. Same operand rules as nslg_linear; returns NSLG_ERR_UNSUPPORTED where the
 * shape's split of the in_features sum would not fit the kernel's on-chip reduction
 * (then call the two kernels). */
int nslg_linear_swiglu(int dtype, int rows, int inter, int in_features, const void* x,
                       int64_t x_stride, const void* gate_up, int64_t w_stride, void* out,
                       int64_t out_stride, uint32_t* dev_status, void* stream);

/* The attention's q|k|v product followed by nslg_rope_kv_append, in one kernel
 * (nslg_linear's tcgen05 path; head_dim 128, where one 128-row tile of the stacked
 * weight is one head): w_qkv = [q; k; v] weight, (num_qo_heads + 2 * num_kv_heads) * 128
 * rows of w_stride elements; the products are rounded to the activation type and then
 * rotated (q into q_out, contiguous [rows, num_qo_heads, 128]; k into the pool slot
 * write_loc[m]) or copied (v into the pool slot), exactly as nslg_rope_kv_append does
 * with the same positions, tables, write_loc and pool arguments (their meaning and
 * device-status reports are that function's). Replaces the q/k/v projections
 * (models.py:136-138, ColumnParallelLinear, tp_layers.py:28-91) and the RoPE + KV write
 * that follow them (models.py:99-103, kv_cache.py:661-674) for decode batches. Returns
 * NSLG_ERR_UNSUPPORTED for another head_dim, or where the shape's split of the
 * in_features sum would not fit the kernel's on-chip reduction (then call nslg_linear
 * and nslg_rope_kv_append). */
int nslg_linear_rope_append(int dtype, int rows, int num_qo_heads, int num_kv_heads,
                            int head_dim, int in_features, const void* x, int64_t x_stride,
                            const void* w_qkv, int64_t w_stride, void* q_out,
                            const int32_t* positions, const float* cos_table,
                            const float* sin_table, int64_t table_rows,
                            const int32_t* write_loc, void* pool_k, void* pool_v,
                            int64_t pool_slots, uint32_t* dev_status, void* stream);

/* Greedy sampling: for each of `rows` rows of logits x (cols entries, row stride
 * x_stride elements), the maximum (out_val[r], fp32; out_val may be NULL) and the index
 * of its first occurrence plus index_offset (out_idx[r]), ordered as torch.argmax: NaN
 * above every number, ties to the lowest index. Replaces logits.argmax(-1) of the
 * greedy decode on the all-gathered LM-head logits (tp_layers.py:89); a vocab-parallel
 * head calls it on its shard with index_offset = the shard's first vocabulary id. */
int nslg_argmax_rows(int dtype, int rows, int cols, const void* x, int64_t x_stride,
                     int64_t index_offset, float* out_val, int64_t* out_idx, void* stream);

/* Device-side plan of a decode step (every sequence adds one token).
 *
 * Replaces the per-forward plan of FlashInferCacheContext.__init__ and
 * _plan_flashinfer (kv_cache.py:547-632) for decode steps: the host keeps the page
 * bookkeeping and the block tables, and mirrors the tables into device memory
 * (block_tables: bt_rows rows of bt_stride int32 page ids, one row per sequence "slot").
 *   slots[b]     row of sequence b;  starts[b]  its token count before the step
 *   updates      num_updates triples (slot, index, page id) written into the tables first
 *                (pages added or copied on write since the last step)
 * Outputs, all int32 device arrays, with the host plan's values:
 *   positions[b] = starts[b];  write_loc[b] = page * page_size + starts[b] % page_size of
 *   the page holding position starts[b];  kv_indptr[B+1], kv_indices (<= max_indices
 *   entries), kv_last_page_len[B] of the sequences' first ceil((starts[b]+1)/page_size)
 *   pages;  qo_indptr[b] = b (B+1 entries);  q_row_start[b] = b.
 * Entries outside the tables or a page list longer than max_indices set
 * NSLG_DEV_BAD_PLAN in *dev_status. batch <= 4096.
 */
int nslg_plan_decode(int batch, int page_size, const int32_t* slots, const int32_t* starts,
                     int num_updates, const int32_t* updates, int32_t* block_tables,
                     int64_t bt_stride, int64_t bt_rows, int32_t* positions, int32_t* write_loc,
                     int32_t* kv_indptr, int32_t* kv_last_page_len, int32_t* qo_indptr,
                     int32_t* q_row_start, int32_t* kv_indices, int64_t max_indices,
                     uint32_t* dev_status, void* stream);

/* Zeroes whole pages of a KV pool tensor [layers, num_pages, page elements]
 * (page_bytes bytes per page and layer): every layer of pages[0 .. n). Replaces the
 * page zeroing of PagePool.alloc (kv_cache.py:411), done once per forward for the pages
 * allocated since the last one. */
int nslg_zero_pages(const int32_t* pages, int num_pages_to_zero, void* pool, int64_t layers,
                    int64_t num_pages, int64_t page_bytes, uint32_t* dev_status, void* stream);

/* One decode step's planning from HOST arrays in a single call: nslg_zero_pages of
 * zero_pages[0 .. num_zero) on both pools (pool_k, pool_v; skipped when num_zero == 0),
 * then nslg_plan_decode. slots, starts, updates and zero_pages are host memory, read
 * before the call returns (the caller may reuse them at once): up to 128 sequences, 192
 * updates and 96 pages to zero they travel in the kernel launch's parameters, larger
 * steps are copied into pinned, device-mapped staging owned by the library, which the
 * kernels read. The plan goes to one
 * device array `plan` laid out as
 *   positions[B] | write_loc[B] | kv_indptr[B+1] | kv_last_page_len[B] | qo_indptr[B+1] |
 *   q_row_start[B] | kv_indices[max_indices]
 * (offsets 0, B, 2B, 3B+1, 4B+1, 5B+2, 6B+2 int32 entries). The staging is a ring of
 * slots per device, a slot reused only after the kernels of its earlier call finished.
 * Not capturable in a CUDA graph (NSLG_ERR_UNSUPPORTED during capture). Replaces the
 * decode-step plan of FlashInferCacheContext.__init__ + _plan_flashinfer
 * (kv_cache.py:547-632) and the page zeroing of PagePool.alloc (kv_cache.py:411). */
int nslg_plan_decode_host(int batch, int page_size, const int32_t* slots, const int32_t* starts,
                          int num_updates, const int32_t* updates, int num_zero,
                          const int32_t* zero_pages, void* pool_k, void* pool_v, int64_t layers,
                          int64_t num_pages, int64_t page_bytes, int32_t* block_tables,
                          int64_t bt_stride, int64_t bt_rows, int32_t* plan,
                          int64_t max_indices, uint32_t* dev_status, void* stream);

/* ---------------------------------------------------------------- tensor parallel */

#define NSLG_IPC_HANDLE_BYTES 64   /* cudaIpcMemHandle_t                                 */
#define NSLG_TP_MAX_WORLD 8
#define NSLG_TP_COUNTER_BYTES 1024 /* per-rank call counters of nslg_tp_allreduce_rmsnorm */

/* Device memory that peers in other processes can map (CUDA IPC, no multicast).
 * nslg_ipc_alloc: cudaMalloc of `bytes` on the current device, zeroed, and its
 *   NSLG_IPC_HANDLE_BYTES-byte handle in handle_out (to be sent to the peers);
 * nslg_ipc_open: maps a peer's handle into this process (peer access over NVLink);
 * nslg_ipc_close / nslg_ipc_free: undo open / alloc.
 * Replaces nothing in the reference (whose only collective path is NCCL through
 * parallel.py:167-184); it sets up the memory nslg_tp_allreduce_rmsnorm writes.
 */
int nslg_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle_out);
int nslg_ipc_open(const void* handle, void** dev_ptr);
int nslg_ipc_close(void* dev_ptr);
int nslg_ipc_free(void* dev_ptr);

/* Tensor-parallel all-reduce of a RowParallelLinear output fused with the residual add
 * and the RMSNorm that follow it, over peer memory.
 *
 * Replaces RowParallelLinear.forward's all-reduce (tp_layers.py:148-158, through
 * all_reduce_tp, parallel.py:167-172) together with the block's `h = x + attn` /
 * `h + mlp` and the next RMSNorm (models.py:169-172, 25-34), for one TP group of
 * `world` ranks (one process per GPU), this process being `rank`:
 *   sum            = sum over ranks of partial[row]   (fp32, rank order, rounded once)
 *   residual[row] <- round(residual[row] + sum)       (in place)
 *   out[row]       = weight * round(residual[row] * rsqrt(mean(residual[row]^2) + eps))
 *                    (skipped when weight == NULL: the caller wants the residual only)
 * partial, residual, out: [rows, hidden] (row strides in elements, rows 16-byte aligned,
 *   hidden * element size <= 16 KiB).
 * stage_bufs: HOST array of `world` device pointers, entry i = rank i's stage buffer
 *   (stage_bytes each, the same on every rank, >= 4 * world * rows * hidden * element
 *   size), from nslg_ipc_alloc: entry `rank` is this process's own allocation, the
 *   others its nslg_ipc_open mappings of the peers'. Peers write into it.
 * counters: this rank's NSLG_TP_COUNTER_BYTES of zeroed device memory, kept between
 *   calls (private to the rank).
 * Every rank must make the same sequence of calls (the counters pair them; the launch
 * may be captured in a CUDA graph). A wait on a peer gives up after timeout_ns, sets
 * NSLG_DEV_WAIT_TIMEOUT in *dev_status and leaves that call's rows unwritten.
 */
int nslg_tp_allreduce_rmsnorm(int dtype, int rows, int hidden, int world, int rank,
                              const void* partial, int64_t partial_stride,
                              void* const* stage_bufs, int64_t stage_bytes, void* counters,
                              void* residual, int64_t residual_stride, const void* weight,
                              void* out, int64_t out_stride, float eps, int64_t timeout_ns,
                              uint32_t* dev_status, void* stream);

/* nslg_tp_allreduce_rmsnorm for every rank of a TP group at once, all on the current
 * GPU: rank r's partial, counters, residual and out are entry r of the HOST arrays
 * partials / counters / residuals / outs, and stage_bufs[r] its stage buffer. One
 * cooperative launch holds the ranks' blocks side by side, so the ranks wait on one
 * another inside one grid (it fails with NSLG_ERR_CUDA if they cannot all be resident,
 * instead of waiting). Same protocol, same one-shot / two-shot choice, same results as
 * `world` processes each calling nslg_tp_allreduce_rmsnorm; for checking the exchange on
 * a machine with one GPU. No counterpart in the reference. */
int nslg_tp_allreduce_rmsnorm_emulated(int dtype, int rows, int hidden, int world,
                                       const void* const* partials, int64_t partial_stride,
                                       void* const* stage_bufs, int64_t stage_bytes,
                                       void* const* counters, void* const* residuals,
                                       int64_t residual_stride, const void* weight,
                                       void* const* outs, int64_t out_stride, float eps,
                                       int64_t timeout_ns, uint32_t* dev_status, void* stream);

/* The RowParallel product and its collective in one kernel: nslg_linear (y = x . W^T,
 * `rows` <= 256 rows, y the caller's [rows, out_features] with 16-byte aligned rows) that
 * also stores y's rows, packed with the reduction's call numbers, into every peer's stage
 * buffer over NVLink as soon as each tile is final -- the one-shot push that
 * nslg_tp_allreduce_rmsnorm would otherwise do after the product.  y stays this rank's
 * partial (the reduction reads it).  Arguments after y_stride as in
 * nslg_tp_allreduce_rmsnorm (out_features is its `hidden`); counters are only read.  Must
 * be followed on the same stream, before any other reduction call of the group, by
 * nslg_tp_reduce_pushed_rmsnorm on the same y, rows and buffers.  Replaces
 * RowParallelLinear.forward's F.linear + all-reduce (tp_layers.py:148-158,
 * parallel.py:167-172) for decode steps. */
int nslg_linear_tp_push(int dtype, int rows, int out_features, int in_features, const void* x,
                        int64_t x_stride, const void* weight, int64_t w_stride, void* y,
                        int64_t y_stride, int world, int rank, void* const* stage_bufs,
                        int64_t stage_bytes, const void* counters, uint32_t* dev_status,
                        void* stream);

/* nslg_tp_allreduce_rmsnorm without its push: the partial rows were already pushed by
 * nslg_linear_tp_push (always the one-shot layout). Same arguments and results. */
int nslg_tp_reduce_pushed_rmsnorm(int dtype, int rows, int hidden, int world, int rank,
                                  const void* partial, int64_t partial_stride,
                                  void* const* stage_bufs, int64_t stage_bytes,
                                  void* counters, void* residual, int64_t residual_stride,
                                  const void* weight, void* out, int64_t out_stride, float eps,
                                  int64_t timeout_ns, uint32_t* dev_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NSLG_B200_H */
