/*
 * kessie_capi.h -- C ABI of libkessie_cuda.so (B200 / sm_100a).
 *
 * Drop-in replacement for the native boundary of the KeSSie fog-attention
 * path.  The five legacy launchers keep the exact argument lists of the
 * reference's extern "C" HIP launchers so that kessie_hip_ctypes.KeSSieKernels
 * (kessie_hip_ctypes.py:65-114) binds them unchanged; the library is also
 * published under the reference's file name build/libkessie_hip.so.
 *
 * Conventions
 *   - Every pointer is a device pointer owned by the caller (PyTorch tensor
 *     storage); the library allocates no device memory, except on explicit
 *     request through kessie_cp_exchange_alloc (the context-parallel
 *     exchange buffer, which must be cudaMalloc'd to be shared over CUDA
 *     IPC).  Scratch memory is passed in as `workspace` and sized by the
 *     matching *_workspace_size().
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream),
 *     the value of torch.cuda.Stream.cuda_stream.  All calls are asynchronous
 *     on that stream.
 *   - Legacy launchers return void (ctypes restype=None, as in the
 *     reference); their failures are recorded and readable through
 *     kessie_get_last_error().  _v2 entry points return a status:
 *     0 = ok, >0 = argument / unsupported-shape error (nothing launched),
 *     <0 = CUDA launch error.  No entry point calls exit() or abort().
 *   - Device-detected faults (page id out of range, a bounded wait that ran
 *     out) do not trap: the kernel skips the access, records a code in the
 *     library's device status word and returns; kessie_read_device_status()
 *     reads and clears it.
 *   - Strides are in ELEMENTS; head_dim is always the contiguous dimension.
 *   - The library caches, per device, the addresses of its own device
 *     variables (the status word, the allocation-free decode's scratch) and
 *     launch settings (kernels' shared-memory limits, occupancy): do not use
 *     it on a device after cudaDeviceReset of that device.
 *   - Positions are int32; page tables are int32; page_valid is int8.
 */
#ifndef KESSIE_CAPI_H
#define KESSIE_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of the _v2 entry points. */
#define KESSIE_DTYPE_F16  0
#define KESSIE_DTYPE_BF16 1
#define KESSIE_DTYPE_F32  2

/* Host-side status codes. */
#define KESSIE_OK               0
#define KESSIE_ERR_ARG          1   /* bad pointer / size / stride            */
#define KESSIE_ERR_UNSUPPORTED  2   /* shape or dtype this build does not run */
#define KESSIE_ERR_WORKSPACE    3   /* workspace missing or too small          */
#define KESSIE_ERR_CUDA        -1   /* CUDA runtime / launch error             */

/* Device status bits (kessie_read_device_status). */
#define KESSIE_DEV_BAD_PAGE_ID  0x1 /* a page id outside [0, num_pages) was skipped */
#define KESSIE_DEV_WAIT_TIMEOUT 0x2 /* a bounded pipeline wait gave up              */
#define KESSIE_DEV_BAD_ARG      0x4 /* a per-sequence argument was out of range     */

/* ------------------------------------------------------------------------- */
/* Library status                                                            */
/* ------------------------------------------------------------------------- */

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len) and returns the last status code (0 if none).
 * No reference counterpart: the reference launchers report nothing
 * (kessie_kernels_v2.hip:749,823 print to stderr only). */
int kessie_get_last_error(char* buf, int len);

/* Library version string, e.g. "kessie_b200 0.1 sm_100a". */
const char* kessie_version(void);

/* Synchronises `stream`, then returns the current device's status word (an
 * OR of KESSIE_DEV_* bits) and clears it.  Returns <0 on a CUDA error. */
int kessie_read_device_status(void* stream);

/* No reference counterpart (the reference launches nothing programmatically).
 * The library's registry of programmatic launches, open to callers that
 * launch their own programmatic dependents (griddepcontrol) on a stream that
 * this library also launches on.  The library's f16/bf16 decodes, page
 * gathers, RoPE remaps, fused inserts and tiered updates are programmatic
 * dependent launches that may read their inputs before their
 * griddepcontrol.wait when the previous programmatic launch on the same
 * (device, stream) wrote none of them; the registry keeps that launch's
 * written byte ranges.  A caller that launches such a kernel of its own
 * records it here just before the launch:
 *   writes: nwrites [lo, hi) byte-address pairs (2 * nwrites values); more
 *     than 8 non-empty ranges record "everything" (and that claim gets 0);
 *   *may_read_early = 1 when none of the previous record's ranges overlaps
 *     the nreads pairs in `reads` (the new launch may read them before its
 *     wait), else 0;
 *   merge = 1 and delay_ns: for a launch that signals its dependents before
 *     its own griddepcontrol.wait -- its record keeps the previous record's
 *     ranges (that launch may still run when the next one starts), and
 *     delay_ns bounds how long its dependents can then sit in
 *     griddepcontrol.wait;
 *   prev_delay_ns (nullable) receives the previous record's bound; when it
 *     is NULL a non-zero bound gives *may_read_early = 0.
 * Issue the launch before any other claim on the same stream.  Returns
 * KESSIE_OK or KESSIE_ERR_ARG. */
int kessie_launch_registry_claim(void* stream, const uint64_t* reads, int nreads, const uint64_t* writes,
                                 int nwrites, uint64_t delay_ns, int merge, uint64_t* prev_delay_ns,
                                 int* may_read_early);

/* ------------------------------------------------------------------------- */
/* Legacy launchers -- identical argument lists to the reference             */
/* ------------------------------------------------------------------------- */

/* Replaces launch_kessie_windowed_attn (kessie_kernels_v2.hip:716-751).
 * Q,K,V,O: fp16 [B,H,N,D] contiguous, D in {64,128}.  Causal and/or sliding
 * window W (0 <= i-j < W) exactly as kessie_hip_kernels.py:577-588. */
void launch_kessie_windowed_attn(const void* Q, const void* K, const void* V, void* O,
                                 float sm_scale, int batch_size, int num_heads, int seq_len,
                                 int head_dim, int window_size, int is_causal, void* stream);

/* Replaces launch_kessie_fused_fog_attn (kessie_kernels_v2.hip:788-825).
 * As above with fog_weights: fp32 [N]; O = softmax(mask(QK^T s)) (V * w),
 * the semantics of kessie_fused_fog_attention_ref (kessie_hip_kernels.py:591-593). */
void launch_kessie_fused_fog_attn(const void* Q, const void* K, const void* V, void* O,
                                  const void* fog_weights, float sm_scale, int batch_size,
                                  int num_heads, int seq_len, int head_dim, int window_size,
                                  int is_causal, void* stream);

/* Replaces launch_kessie_page_evict (kessie_kernels_v2.hip:753-764): for each
 * page, valid==1 && pos < evict_before_pos -> valid=0 and *evict_count += 1.
 * page_valid int8 [P], page_positions int32 [P], evict_count int32 [1]. */
void launch_kessie_page_evict(void* page_valid, const void* page_positions, void* evict_count,
                              int evict_before_pos, int num_pages, void* stream);

/* Replaces launch_kessie_page_insert (kessie_kernels_v2.hip:766-782).
 * kv_cache fp16 [max_pages, page_size, 2, H, D]; new_keys/new_values fp16
 * [T, H, D]; token t -> page target_page_ids[t/page_size], slot t%page_size;
 * first token of each page sets page_valid=1, page_positions=conv_pos+t.
 * Page ids outside [0,max_pages) are skipped (as kessie_kernels_v2.hip:441). */
void launch_kessie_page_insert(void* kv_cache, const void* new_keys, const void* new_values,
                               const void* target_page_ids, void* page_valid, void* page_positions,
                               int conv_pos, int num_tokens, int num_heads, int head_dim,
                               int page_size, int max_pages, void* stream);

/* Replaces launch_kessie_rope_remap (kessie_kernels_v2.hip:827-842).
 * In-place rotate-half re-rotation of fp16 K [T, H, 2*half_dim] from
 * orig_positions to target_positions (int32 [T]). */
void launch_kessie_rope_remap(void* k_data, const void* orig_positions,
                              const void* target_positions, float rope_theta,
                              int num_tokens, int num_heads, int half_dim, void* stream);

/* ------------------------------------------------------------------------- */
/* _v2 entry points (dtype-generic, strided, paged, status-returning)        */
/* ------------------------------------------------------------------------- */

/* RoPE remap, any dtype, strided K (token_stride, head_stride in elements,
 * head_dim contiguous).  Same math as kessie_hip_kernels.py:596-606 /
 * kessie_kernels_v2.hip:670-707; the frequency table 1/theta^(d/half) is
 * computed once on the host in float64 and rounded to fp32 (bit-identical to
 * the reference's torch table at theta 1e4 and 5e5).  With 16-byte aligned
 * rows it is a programmatic dependent launch, like kessie_page_gather_v2: its
 * rows and positions may be copied in before the previous kernel on the
 * stream completes when the last such launch of this library there wrote none
 * of them; it writes only after that kernel completes.  The same holds for
 * kessie_page_insert_v2 with orig_positions (rows, positions and page ids
 * read early; cache rows and page metadata written after). */
int kessie_rope_remap_v2(void* k_data, int dtype, int num_tokens, int num_heads, int head_dim,
                         int64_t token_stride, int64_t head_stride,
                         const int32_t* orig_positions, const int32_t* target_positions,
                         float rope_theta, void* stream);

/* Device eviction with ORDERED compaction of the freed page ids.
 * Replaces KeSSiePagedKVCache.evict_before (kessie_hip_kernels.py:526-540)
 * whose Python loop does one device sync per page.
 *   - valid==1 && pos < evict_before_pos -> valid = 0 (kessie_kernels_v2.hip:403-406)
 *   - freed set = pages with page_allocated[p]==1 && valid[p]==0 after the
 *     update (the reference's "page_valid==0 and not in free_pages");
 *     their page_allocated is cleared.  With page_allocated == NULL the
 *     freed set is the pages evicted by this call.
 *   - freed_ids[0..*freed_count) = freed page ids in ascending order (the
 *     append order of the reference's scan).  freed_ids may be NULL.
 * workspace: kessie_page_evict_workspace_size(num_pages) bytes. */
size_t kessie_page_evict_workspace_size(int num_pages);
int kessie_page_evict_v2(int8_t* page_valid, const int32_t* page_positions, int8_t* page_allocated,
                         int num_pages, int evict_before_pos, int32_t* freed_count,
                         int32_t* freed_ids, void* workspace, size_t workspace_bytes, void* stream);

/* Ordered list of pages with page_valid != 0 (the torch.nonzero of
 * KeSSiePagedKVCache.get_layer_kv, kessie_hip_kernels.py:559).
 * Uses the same workspace size as kessie_page_evict_v2. */
int kessie_page_list_valid_v2(const int8_t* page_valid, int num_pages, int32_t* count,
                              int32_t* ids, void* workspace, size_t workspace_bytes, void* stream);

/* Fused page insert + RoPE remap.  Replaces launch_kessie_page_insert
 * (kessie_kernels_v2.hip:766-782) + launch_kessie_rope_remap for the recall
 * path and KeSSiePagedKVCache.insert_probe_kv's per-page copies
 * (kessie_hip_kernels.py:548-554).
 * kv_cache: [.., page_size, .., H, D] addressed by page/token/kv/head strides
 * (covers [P][ps][2][H][D] and vLLM's [2][P][ps][H][D]).  new_keys /
 * new_values: [T, H, D] with src_token_stride / src_head_stride.
 * When orig_positions != NULL, K is re-rotated from orig_positions[t] to
 * target_positions[t] (or conv_pos + t when target_positions == NULL).
 * page_valid / page_positions may be NULL (no metadata update). */
int kessie_page_insert_v2(void* kv_cache, int dtype, int64_t page_stride, int64_t token_stride,
                          int64_t kv_stride, int64_t head_stride, int max_pages, int page_size,
                          const void* new_keys, const void* new_values, int64_t src_token_stride,
                          int64_t src_head_stride, int num_tokens, int num_heads, int head_dim,
                          const int32_t* target_page_ids, int8_t* page_valid,
                          int32_t* page_positions, int conv_pos, const int32_t* orig_positions,
                          const int32_t* target_positions, float rope_theta, void* stream);

/* Page gather: out_keys / out_values [n*page_size, H, D] contiguous from the
 * pages page_ids[0..n) in that order -- KeSSiePagedKVCache.get_layer_kv
 * (kessie_hip_kernels.py:558-564) and the connector's block copies
 * (kessie_kv_connector.py:419-428, 467-479).  Ids outside [0,max_pages)
 * produce zero rows and set KESSIE_DEV_BAD_PAGE_ID.  Either output may be
 * NULL (gather only K or only V).  With rows of H*D contiguous elements the
 * gather is a programmatic dependent launch, like kessie_tiered_update_v2:
 * its first page loads may start before the previous kernel on the stream
 * completes when the last such launch of this library on that stream wrote
 * none of the cache or page-id bytes it reads; it writes only after that
 * kernel completes.  A kernel that writes the cache or the ids must not be
 * launched with a programmatic dependency that triggers before its writes. */
int kessie_page_gather_v2(const void* kv_cache, int dtype, int64_t page_stride,
                          int64_t token_stride, int64_t kv_stride, int64_t head_stride,
                          int max_pages, int page_size, const int32_t* page_ids, int num_gather,
                          int num_heads, int head_dim, void* out_keys, void* out_values,
                          void* stream);

/* Fog weight vector fp32 [seq_len]: 1, then (j/max(cs-1,1))^fog_alpha for
 * j < clear_start when fog_alpha > 0 and clear_start > 0.  Replaces
 * kessie_build_fog_weights (kessie_hip_kernels.py:403-413); the caller
 * passes clear_start = int(seq_len * (1.0 - fog_start)) computed on the host. */
int kessie_build_fog_weights_v2(float* out, int seq_len, int clear_start, float fog_alpha,
                                void* stream);

/* Paged fog decode (one query token per sequence), split-KV over the page
 * table, GQA.  New entry point: the reference has no paged / GQA / decode
 * kernel; its semantics are kessie_fused_fog_attention_ref
 * (kessie_hip_kernels.py:577-593) evaluated at the query row.
 *   q [B, Hq, D] (q_stride_b, q_stride_h); K and V pages at k_cache /
 *   v_cache with shared page/token/head strides; block_table [B, *]
 *   (block_table_stride); seq_lens [B] local keys; kv_pos_offset [B]
 *   (nullable: 0) global position of local key 0; q_positions [B]
 *   (nullable: offset + len - 1) query position.
 *   Mask: key j (global) visible iff j <= q_pos and, when window_size > 0,
 *   q_pos - j < window_size.
 *   Fog on V: w(j) = (j / max(cs-1,1))^fog_alpha for j < cs = clear_start[b]
 *   (global), else 1 (kessie_hip_kernels.py:408-412); clear_start NULL or
 *   fog_alpha <= 0 means no fog; fog_weights (nullable, fp32 indexed by
 *   global position) overrides the formula.
 *   out [B, Hq, D] (dtype) and/or out_partial fp32 [B, Hq, D+2] holding
 *   (O/l, m, l) with m in natural-log units of the scaled scores -- the
 *   triple merged across context-parallel shards by kessie_lse_combine_v2.
 *   D in {64, 128}; dtype f16, bf16 or f32; Hq % Hkv == 0; Hq/Hkv <= 16.
 *   f32 (q, caches and out all fp32) runs every product in fp32 on the CUDA
 *   cores, for the reference's fp32 path at its 1e-4 bar; the additive-bias
 *   and context-parallel forms below take f16 / bf16 only.
 * workspace: kessie_paged_fog_decode_workspace_size(...) bytes.
 * f16 / bf16 decodes are programmatic dependent launches: when the last such
 * launch of this library on the same (device, stream) wrote none of q, the
 * caches, the block table, the length arrays or a bias's recall bitmap (and
 * no fog_weights array is passed), the q and page loads may start before the previous kernel on
 * the stream completes; everything is written only after it completes.  A
 * kernel that writes those inputs must not be launched with a programmatic
 * dependency that triggers before its writes. */
size_t kessie_paged_fog_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                              int head_dim, int max_seq_len, int page_size);
int kessie_paged_fog_decode_v2(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                               const void* k_cache, const void* v_cache, int64_t page_stride,
                               int64_t token_stride, int64_t head_stride, int num_pages,
                               int page_size, const int32_t* block_table,
                               int64_t block_table_stride, const int32_t* seq_lens,
                               const int32_t* kv_pos_offset, const int32_t* q_positions,
                               const int32_t* clear_start, float fog_alpha,
                               const float* fog_weights, int window_size, float sm_scale,
                               int batch, int num_q_heads, int num_kv_heads, int head_dim,
                               int max_seq_len, int dtype, void* out, float* out_partial,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Dense fog attention, any GQA ratio: q/out [B, Hq, N, D], k/v [B, Hkv, N, D]
 * contiguous (f16, bf16 or f32; f32 runs the fp32 CUDA-core decode once per
 * query row), optional fog_weights fp32 [N].  The _v2 form of
 * launch_kessie_fused_fog_attn / launch_kessie_windowed_attn
 * (kessie_hip_kernels.py:367-440, semantics :577-593). */
int kessie_fog_attention_v2(const void* q, const void* k, const void* v, void* out, int dtype,
                            const float* fog_weights, float sm_scale, int batch, int num_q_heads,
                            int num_kv_heads, int seq_len, int head_dim, int window_size,
                            int is_causal, void* stream);

/* Chunked prefill over a paged KV cache.  New entry point (the reference has
 * no paged prefill); semantics kessie_hip_kernels.py:577-593 with a query
 * offset: query i of sequence b sits at absolute position q_start[b] + i
 * (q_start NULL: kv_lens[b] - num_q_tokens, i.e. the chunk is the last
 * num_q_tokens keys of the cache) and attends to keys j < kv_lens[b] with
 * j <= pos (is_causal) and pos - j < window_size (window_size > 0).
 * Fog: clear_start[b] / fog_alpha as in the decode, or fog_weights
 * [B, fog_weights_stride_b] fp32 by key position.
 * q [B, T, Hq, D] and out [B, T, Hq, D] with explicit strides. */
int kessie_paged_fog_prefill_v2(const void* q, int64_t q_stride_b, int64_t q_stride_t,
                                int64_t q_stride_h, const void* k_cache, const void* v_cache,
                                int64_t page_stride, int64_t token_stride, int64_t head_stride,
                                int num_pages, int page_size, const int32_t* block_table,
                                int64_t block_table_stride, const int32_t* kv_lens,
                                const int32_t* q_start, const int32_t* clear_start,
                                float fog_alpha, const float* fog_weights,
                                int64_t fog_weights_stride_b, int window_size, int is_causal,
                                float sm_scale, int batch, int num_q_tokens, int num_q_heads,
                                int num_kv_heads, int head_dim, int dtype, void* out,
                                int64_t o_stride_b, int64_t o_stride_t, int64_t o_stride_h,
                                void* stream);

/* kessie_paged_fog_decode_v2 with a phase mask.  The split merge runs inside
 * the decode kernel, so bit 0 (1 or 3) launches the one kernel that writes
 * out / out_partial, and phases = 2 only checks the arguments.  Kept for
 * callers written against the earlier two-launch form.
 * The workspace needs no initialisation: its per-group arrival counters
 * carry a per-launch tag, so contents left by any earlier use are ignored. */
int kessie_paged_fog_decode_ex_v2(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                  const void* k_cache, const void* v_cache, int64_t page_stride,
                                  int64_t token_stride, int64_t head_stride, int num_pages,
                                  int page_size, const int32_t* block_table,
                                  int64_t block_table_stride, const int32_t* seq_lens,
                                  const int32_t* kv_pos_offset, const int32_t* q_positions,
                                  const int32_t* clear_start, float fog_alpha,
                                  const float* fog_weights, int window_size, float sm_scale,
                                  int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                  int max_seq_len, int dtype, void* out, float* out_partial,
                                  void* workspace, size_t workspace_bytes, int phases,
                                  void* stream);

/* Size of the scratch array built into the library for
 * kessie_paged_fog_decode_noalloc_v2 (16 MiB per GPU that loads the library). */
#define KESSIE_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)

/* Paged fog decode for callers that cannot allocate device memory.
 * No counterpart in the reference.  Same arguments and results as
 * kessie_paged_fog_decode_v2 except that there is no workspace argument: the
 * split-KV scratch is a fixed KESSIE_NOALLOC_SCRATCH_BYTES array inside the
 * library, so code whose device allocator is fixed or owned by another
 * runtime can still decode.  Allocates nothing (no cudaMalloc / cudaFree).
 *   - Shapes whose scratch (kessie_paged_fog_decode_workspace_size) exceeds
 *     the array are rejected with KESSIE_ERR_WORKSPACE and a message.
 *   - The first call on each device looks the array's address up
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     The address is cached for the life of the process: do not call this
 *     entry point on a device after cudaDeviceReset of that device.
 *   - Every call uses the same array: calls that can overlap on the GPU race
 *     and must be ordered by the caller.  Leftover contents from a previous
 *     call are never read. */
int kessie_paged_fog_decode_noalloc_v2(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                       const void* k_cache, const void* v_cache,
                                       int64_t page_stride, int64_t token_stride,
                                       int64_t head_stride, int num_pages, int page_size,
                                       const int32_t* block_table, int64_t block_table_stride,
                                       const int32_t* seq_lens, const int32_t* kv_pos_offset,
                                       const int32_t* q_positions, const int32_t* clear_start,
                                       float fog_alpha, const float* fog_weights, int window_size,
                                       float sm_scale, int batch, int num_q_heads,
                                       int num_kv_heads, int head_dim, int max_seq_len, int dtype,
                                       void* out, float* out_partial, void* stream);

/* kessie_paged_fog_prefill_v2 with a staging workspace: the visible keys of
 * every sequence (kv_lens[b] <= max_kv_len) are first gathered from the pages
 * into workspace as head-major [B][Hkv][kv][D] K and V, so the tensor-core
 * kernel streams 128-token tiles from contiguous memory.  Same results as the
 * unstaged call.  workspace: kessie_paged_fog_prefill_workspace_size() bytes;
 * NULL workspace runs the unstaged kernel. */
size_t kessie_paged_fog_prefill_workspace_size(int batch, int num_kv_heads, int head_dim,
                                               int max_kv_len);
int kessie_paged_fog_prefill_ex_v2(const void* q, int64_t q_stride_b, int64_t q_stride_t,
                                   int64_t q_stride_h, const void* k_cache, const void* v_cache,
                                   int64_t page_stride, int64_t token_stride, int64_t head_stride,
                                   int num_pages, int page_size, const int32_t* block_table,
                                   int64_t block_table_stride, const int32_t* kv_lens,
                                   const int32_t* q_start, const int32_t* clear_start,
                                   float fog_alpha, const float* fog_weights,
                                   int64_t fog_weights_stride_b, int window_size, int is_causal,
                                   float sm_scale, int batch, int num_q_tokens, int num_q_heads,
                                   int num_kv_heads, int head_dim, int dtype, void* out,
                                   int64_t o_stride_b, int64_t o_stride_t, int64_t o_stride_h,
                                   int max_kv_len, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Log-sum-exp merge of S partial triples [S][rows][D+2] (split_stride
 * elements apart) -> out [rows, D] (out_dtype) and/or out_partial
 * [rows, D+2].  Used for the context-parallel combine after the NCCL
 * all-gather.  New entry point (the reference has no split-KV path). */
int kessie_lse_combine_v2(const float* partials, int num_splits, int64_t split_stride, int rows,
                          int head_dim, void* out, int out_dtype, float* out_partial,
                          void* stream);

/* ---------------------------------------------------------------------------
 * Additive fog bias of the vLLM attention path.  The reference computes it in
 * _FogCache._compute_into (kessie_attention.py:114-139) and hands it to vLLM
 * as attn_bias, which vLLM's attention ignores; here it is applied inside the
 * attention kernels, added to the scaled scores:
 *   fb = int(kv_len * (1.0 - fog_start))                      (per sequence)
 *   bias(j) = -fog_alpha * (1 - j/fb)^2 for j < fb, else 0;
 *   bias(j) = recall_boost where bit j of recall_bits is set (overrides).
 * The value of every step is rounded to `dtype` as the reference's torch ops
 * on a buffer of that dtype round it (KESSIE_DTYPE_F32 / BF16 / F16).
 * A null kessie_fog_bias pointer, or fog_alpha <= 0 with no recall bits,
 * means no bias. */
typedef struct kessie_fog_bias {
    float fog_alpha;
    double fog_start;
    float recall_boost;
    const uint32_t* recall_bits;   /* device bitmap over key positions, nullable */
    int recall_nbits;
    int dtype;
} kessie_fog_bias;

/* The reference's bias buffer: out[j] = bias(j) for j < kv_len, in out_dtype
 * (the (1, 1, 1, kv_len) tensor _FogCache.get_fog_bias returns). */
int kessie_build_fog_bias_v2(void* out, int out_dtype, int kv_len, const kessie_fog_bias* bias,
                             void* stream);

/* kessie_paged_fog_prefill_ex_v2 with the additive fog bias on the scores
 * instead of the V fog (the vLLM attention path): the bias of sequence b uses
 * kv_len = kv_lens[b] and key positions j < kv_lens[b]. */
int kessie_paged_fog_prefill_biased_v2(const void* q, int64_t q_stride_b, int64_t q_stride_t,
                                       int64_t q_stride_h, const void* k_cache, const void* v_cache,
                                       int64_t page_stride, int64_t token_stride, int64_t head_stride,
                                       int num_pages, int page_size, const int32_t* block_table,
                                       int64_t block_table_stride, const int32_t* kv_lens,
                                       const int32_t* q_start, int window_size, int is_causal,
                                       float sm_scale, int batch, int num_q_tokens, int num_q_heads,
                                       int num_kv_heads, int head_dim, int dtype,
                                       const kessie_fog_bias* bias, void* out, int64_t o_stride_b,
                                       int64_t o_stride_t, int64_t o_stride_h, int max_kv_len,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* kessie_paged_fog_decode_v2 with the additive fog bias on the scores; the
 * bias of sequence b uses kv_len = q_positions[b] + 1 (the query is the last
 * token) and global key positions. */
int kessie_paged_fog_decode_biased_v2(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                      const void* k_cache, const void* v_cache,
                                      int64_t page_stride, int64_t token_stride,
                                      int64_t head_stride, int num_pages, int page_size,
                                      const int32_t* block_table, int64_t block_table_stride,
                                      const int32_t* seq_lens, const int32_t* kv_pos_offset,
                                      const int32_t* q_positions, const int32_t* clear_start,
                                      float fog_alpha, const float* fog_weights, int window_size,
                                      float sm_scale, int batch, int num_q_heads,
                                      int num_kv_heads, int head_dim, int max_seq_len, int dtype,
                                      const kessie_fog_bias* bias, void* out, float* out_partial,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Conversation-index query: cosine similarity of one fp32 query [dim] against
 * an fp32 index [num_rows, dim] (row-major, 16-byte aligned, dim % 4 == 0),
 * as _kessie_index_query_kernel (kessie_hip_kernels.py:343-360):
 *   sim_i = (q / sqrt(|q|^2 + 1e-8)) . (x_i / sqrt(|x_i|^2 + 1e-8))
 * (normalize_rows = 0: the rows are already normalised, VectorIndex style,
 * kessie_exp3.py:69-81, and only the query is normalised).  Optional outputs:
 * sims [num_rows]; the top_k (<= 32) rows by similarity, descending, ties to
 * the lower row index (top_idx -1 / top_scores -FLT_MAX past num_rows).
 * workspace: kessie_index_query_workspace_size(num_rows, top_k) bytes. */
size_t kessie_index_query_workspace_size(int num_rows, int top_k);
int kessie_index_query_v2(const float* query, const float* index, int num_rows, int dim,
                          int normalize_rows, float* sims, int top_k, int32_t* top_idx,
                          float* top_scores, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ---------------------------------------------------------------------------
 * HF tiered KV cache (KeSSieCache, kessie_exp3.py:342-627) on per-layer stores
 * [B, H, cap, D] (dtype elements, live tokens at [lo, hi) of the cap axis).
 *
 * kessie_tiered_update_v2 replaces KeSSieCache.update (:425-450): appends the
 * T new tokens k_new / v_new [B, H, T, D] (element strides b, h, t; head_dim
 * contiguous; K and V share the strides) at [hi, hi + T) and, when the
 * reference's _compute_fog_mask (:415-423) gives a mask for S = hi + T - lo
 * (fog_alpha > 0, fc = S - max(1, int(S * fog_start)) > 0), writes
 *   v_fog[b, h, s, :] = dtype(float(v[b, h, lo + s, :]) * w(s)),
 *   w(s) = max((s / max(fc - 1, 1)) ^ fog_alpha, 0.01) for s < fc, else 1
 * into v_fog, contiguous [B, H, S, D]; with no mask v_fog is not touched.
 * Needs hi + T <= cap, D * element size a multiple of 16, 16-byte aligned
 * buffers.  The update is a programmatic dependent launch: it may start while
 * the previous kernel on the stream drains.  When the last tiered update
 * launched on the same (device, stream) by this process wrote none of this V
 * store, the live-V loads start before that kernel completes; new tokens are
 * read, and everything is written, only after it completes.  So the stores
 * belong to this library: a kernel that writes them must not be launched with
 * a programmatic dependency that triggers before its own writes.
 *
 * kessie_strided_pack_v2 replaces the per-layer slicing copies of
 * evict_if_needed / recall_from_cpu (:452-533): for every store m of
 * num_stores, store_bases[m] = device address of (row 0, token t0) and
 * store_pitch_bytes[m] = bytes between its rows (cap * D * element size),
 * rows_per_store rows (B * H) of `tokens` tokens of row_bytes (D * element
 * size, a multiple of 16) are copied to (unpack = 0) or from (unpack = 1) a
 * contiguous staging [num_stores][rows_per_store][tokens][row_bytes].
 * store_bases and store_pitch_bytes are DEVICE arrays. */
int kessie_tiered_update_v2(void* k_store, void* v_store, long long cap, long long lo, long long hi,
                            const void* k_new, const void* v_new, long long new_stride_b,
                            long long new_stride_h, long long new_stride_t, int B, int H, int T, int D,
                            int dtype, void* v_fog, float fog_alpha, double fog_start, void* stream);
int kessie_strided_pack_v2(const unsigned long long* store_bases, const long long* store_pitch_bytes,
                           int num_stores, int rows_per_store, long long tokens, int row_bytes,
                           void* staging, int unpack, void* stream);

/* ---------------------------------------------------------------------------
 * Context-parallel decode over NVLink peer memory (no counterpart in the
 * reference, which has no multi-GPU attention path).  Each of the `world`
 * ranks (one GPU each, one node, world <= 8) holds a contiguous position
 * range of every sequence (kv_pos_offset = global position of local key 0).
 * Every rank allocates one exchange buffer and maps the others':
 *   kessie_cp_exchange_bytes(world, B, Hq, Hkv, D) -> size
 *   kessie_cp_exchange_alloc(size, &ptr, handle)    cudaMalloc, zero-fill,
 *                                                   IPC handle (64 bytes)
 *   (all-gather the handles over the caller's process group)
 *   kessie_cp_exchange_open(peer_handle, &peer_ptr) for every other rank
 *   kessie_cp_exchange_close(peer_ptr) / kessie_cp_exchange_free(ptr) at the
 *   end, after every rank has finished its last step.
 * A step, kessie_paged_fog_decode_cp_v2 with exchange_buffers[r] = rank r's
 * buffer as mapped in this process (this rank's own at [rank]):
 *   phases bit 0: the decode kernel over the local shard; the CTA that
 *     completes a (seq, kv_head) group stores the group's merged rows into
 *     every rank's buffer over NVLink as self-validating (value, epoch)
 *     8-byte words -- no fence or flag, so the decode never waits;
 *   phases bit 1: a combine kernel that polls this rank's own buffer until
 *     every rank's words of a row carry the epoch (at most wait_timeout_ns,
 *     then KESSIE_DEV_WAIT_TIMEOUT in the device status word and zero rows)
 *     and writes out [B, Hq, D] and/or out_partial [B, Hq, D+2] (same triple
 *     as kessie_paged_fog_decode_v2).  With both bits the combine is a
 *     programmatic dependent launch of the decode.  The combine lets the
 *     next launch on the stream start at once (the next step's decode then
 *     reads ahead while this step finishes; the library keeps the decode's
 *     and the combine's written ranges for that decision).
 * All ranks call it with the same shapes and the same epoch; epoch starts at
 * 1 and goes up by one per step (consecutive steps alternate between two
 * slots of the buffer, so keep the parity alternating across any wrap).
 * Only the combine waits, and only on memory of its own GPU. */
#define KESSIE_IPC_HANDLE_BYTES 64
size_t kessie_cp_exchange_bytes(int world, int batch, int num_q_heads, int num_kv_heads,
                                int head_dim);
int kessie_cp_exchange_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
int kessie_cp_exchange_open(const void* ipc_handle, void** dev_ptr);
int kessie_cp_exchange_close(void* dev_ptr);
int kessie_cp_exchange_free(void* dev_ptr);
/* Phase bit 1 of kessie_paged_fog_decode_cp_v2 on its own (needs only the
 * exchange arguments and the shapes). */
int kessie_cp_combine_v2(void* const* exchange_buffers, int rank, int world, uint32_t epoch,
                         int64_t wait_timeout_ns, int batch, int num_q_heads, int num_kv_heads,
                         int head_dim, int dtype, void* out, float* out_partial, void* stream);
int kessie_paged_fog_decode_cp_v2(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                  const void* k_cache, const void* v_cache, int64_t page_stride,
                                  int64_t token_stride, int64_t head_stride, int num_pages,
                                  int page_size, const int32_t* block_table,
                                  int64_t block_table_stride, const int32_t* seq_lens,
                                  const int32_t* kv_pos_offset, const int32_t* q_positions,
                                  const int32_t* clear_start, float fog_alpha,
                                  const float* fog_weights, int window_size, float sm_scale,
                                  int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                  int max_seq_len, int dtype, void* const* exchange_buffers,
                                  int rank, int world, uint32_t epoch, int64_t wait_timeout_ns,
                                  void* out, float* out_partial, void* workspace,
                                  size_t workspace_bytes, int phases, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KESSIE_CAPI_H */
