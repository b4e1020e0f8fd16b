/*
 * kvcache.h — C ABI of libkvcache.so, the B200 (sm_100a) KV-cache decode path.
 *
 * This library replaces the hot-path entry points of gfx1150-inference's pybind11
 * `matmul_module` (src/python_bindings/bindings.cpp) and the HIP launchers behind
 * them (src/kernels/attention.h).  Every function:
 *   - takes plain pointers and sizes (no torch / numpy types),
 *   - returns an int status (KVC_OK == 0), with a human-readable message available
 *     from kvc_last_error() on the calling thread,
 *   - maps the reference's C++ exception classes onto status codes:
 *       std::invalid_argument -> KVC_ERR_INVALID_ARG   (Python ValueError)
 *       std::out_of_range     -> KVC_ERR_OUT_OF_RANGE  (Python IndexError)
 *       std::runtime_error    -> KVC_ERR_RUNTIME / KVC_ERR_CUDA / KVC_ERR_DEVICE
 *                                                      (Python RuntimeError)
 *
 * Two families of entry points exist:
 *   1. Reference-compatible process-wide pool ("kvc_cache_*", "kvc_gqa_attention*"):
 *      same arguments, same validation order and same semantics as the reference's
 *      DeviceKVCachePool singleton and its launchers.  Host-buffer variants copy in
 *      and out like the reference; the *_device variant takes device pointers and a
 *      cudaStream_t (passed as void*).
 *   2. Handle-based paged pool for batched decode ("kvc_pool_*", "kvc_plan_*",
 *      "kvc_append", "kvc_decode*", "kvc_gather"): many sequences, block tables of
 *      fixed-size pages, one KV-head shard per GPU.  Device pointers + stream.
 *   3. Host-streamed offload ("kvc_offload_*"): the --offload-kv-cpu / --kv-mmap-dir
 *      modes.  KV lives in host memory; each call streams one layer to the GPU on a
 *      copy stream, double-buffered, while the previous layer's attention runs.
 *
 * Numerics (all attention entry points): fp16 / bf16 / fp32 KV storage, fp32
 * accumulation, online softmax, scores = (q . k) * scale with `scale` used exactly
 * as given (0.0 gives all-equal scores, as in the reference kernel
 * src/kernels/attention.hip:99), causal bound min(kv_len, start_pos + m + 1)
 * (attention.hip:75), and an all-zero output row when no position is attended
 * (attention.hip:115).
 */
#ifndef KVCACHE_H
#define KVCACHE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KVC_API __attribute__((visibility("default")))
#else
#define KVC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define KVC_OK 0
#define KVC_ERR_INVALID_ARG 1   /* reference: std::invalid_argument */
#define KVC_ERR_OUT_OF_RANGE 2  /* reference: std::out_of_range */
#define KVC_ERR_RUNTIME 3       /* reference: std::runtime_error (e.g. pool missing) */
#define KVC_ERR_CUDA 4          /* reference: HIP_CHECK -> std::runtime_error */
#define KVC_ERR_DEVICE 5        /* a kernel reported a bad page id or a wait limit */
#define KVC_ERR_TIMEOUT 6       /* a host-side wait ran past its limit */

/* ---- storage types --------------------------------------------------------- */
#define KVC_DTYPE_F16 0
#define KVC_DTYPE_BF16 1
#define KVC_DTYPE_F32 2

/* device error codes written by kernels (kvc_device_error) */
#define KVC_DEVERR_NONE 0u
#define KVC_DEVERR_BAD_PAGE 1u        /* block table entry outside [0, num_pages), or past the row's width */
#define KVC_DEVERR_WAIT_LIMIT 2u      /* an mbarrier wait gave up after its limit */
#define KVC_DEVERR_BAD_POSITION 3u    /* append position outside the block table */

/* Library ABI version (bumped on any signature change). */
KVC_API int kvc_version(void);

/* Message for the last failing call on this thread ("" if none). */
KVC_API const char* kvc_last_error(void);

/* Read (and optionally clear) the device-side error word of `device`.
 * *code receives one of KVC_DEVERR_*, *info an auxiliary value (e.g. the bad page). */
KVC_API int kvc_device_error(int device, int clear, uint32_t* code, uint32_t* info);

/* Number of streaming multiprocessors of `device` (grid sizing helper). */
KVC_API int kvc_device_sm_count(int device, int* out);

/* No counterpart in the reference (its HIP calls block without a limit).  Limit,
 * in seconds, of every wait of the host for the library's own GPU work: the end
 * of a host-buffer call, a plan upload, the offload engine's copies.  A wait that
 * runs out returns KVC_ERR_TIMEOUT; the call's work may still be queued, so
 * synchronise its stream before reusing its buffers.  Default 60 s; (0, 86400]. */
KVC_API int kvc_set_host_wait_limit(double seconds);

/* No counterpart in the reference.  Host-side fault injection for tests: after
 * `skip` further calls at `site` succeed, the next `count` fail the way the CUDA
 * call would (device / page-locked allocations: cudaErrorMemoryAllocation;
 * page-locking caller memory: cudaErrorNotPermitted; a host wait: its limit runs
 * out at once).  Nothing reaches the GPU.  count 0 disarms the site. */
#define KVC_FAULT_DEVICE_ALLOC 1   /* cudaMalloc of pools, scratch, staging */
#define KVC_FAULT_HOST_ALLOC 2     /* cudaHostAlloc of page-locked staging */
#define KVC_FAULT_HOST_REGISTER 3  /* cudaHostRegister of caller memory (offload) */
#define KVC_FAULT_WAIT 4           /* bounded host waits */
KVC_API int kvc_test_inject_failure(int site, int skip, int count);

/* ==== 1. Reference-compatible process-wide pool ============================ */

/* Replaces init_device_kv_cache_fp16 (src/kernels/attention.h:27-32,
 * attention.hip:286-296) behind matmul_module.kv_cache_init
 * (src/python_bindings/bindings.cpp:468-472).  Allocates (or grows) the fp16
 * pool for one sequence of up to max_seq_len positions in every layer.  Like the
 * reference, memory is only reallocated when the new size exceeds the capacity
 * and pool contents are not zeroed.  Fails with KVC_ERR_INVALID_ARG unless all
 * dimensions are positive. */
KVC_API int kvc_cache_init(int num_layers, int max_seq_len, int num_kv_heads, int head_dim);

/* Extension of kvc_cache_init: storage dtype (KVC_DTYPE_*) and page size in
 * positions (a multiple of 16; 0 selects 16). */
KVC_API int kvc_cache_init_ex(int num_layers, int max_seq_len, int num_kv_heads, int head_dim,
                      int dtype, int page_size);

/* Replaces free_device_kv_cache_fp16 (attention.h:35, attention.hip:298-300)
 * behind matmul_module.kv_cache_free (bindings.cpp:474-478). */
KVC_API int kvc_cache_free(void);

/* Storage dtype of the process-wide pool, or -1 if none is allocated. */
KVC_API int kvc_cache_dtype(void);

/* Replaces launch_gqa_attention_cached_fp16 (attention.h:41-54,
 * attention.hip:302-374) behind matmul_module.gqa_attention_cached
 * (bindings.cpp:480-514).  Host buffers in the pool's dtype:
 *   h_Q (q_len, num_heads, head_dim), h_K_new / h_V_new (q_len, num_kv_heads,
 *   head_dim), h_Out (q_len, num_heads, head_dim).
 * Appends the q_len new rows at (layer_idx, start_pos) and attends over
 * [0, start_pos + q_len).  Validation order and status codes follow
 * attention.hip:316-329. */
KVC_API int kvc_gqa_attention_cached(const void* h_Q, const void* h_K_new, const void* h_V_new,
                             void* h_Out, int layer_idx, int q_len, int start_pos,
                             int num_heads, int num_kv_heads, int head_dim, float scale,
                             int causal);

/* Replaces launch_gqa_attention_cached_fp16_device (attention.h:59-72,
 * attention.hip:376-440): device pointers, work enqueued on `stream`
 * (a cudaStream_t; NULL = legacy default stream), no host synchronisation. */
KVC_API int kvc_gqa_attention_cached_device(const void* d_Q, const void* d_K_new,
                                    const void* d_V_new, void* d_Out, int layer_idx,
                                    int q_len, int start_pos, int num_heads,
                                    int num_kv_heads, int head_dim, float scale,
                                    int causal, void* stream);

/* Replaces launch_gqa_attention_fp16 (attention.h:10-23, attention.hip:228-284)
 * behind matmul_module.gqa_attention (bindings.cpp:414-447): full K/V for one
 * layer in host memory, token-major (kv_len, num_kv_heads, head_dim), fp16.
 * Same validation as attention.hip:242-247. */
KVC_API int kvc_gqa_attention(const void* h_Q, const void* h_K, const void* h_V, void* h_Out,
                      int q_len, int kv_len, int num_heads, int num_kv_heads,
                      int head_dim, int start_pos, float scale, int causal);

/* kvc_gqa_attention with an explicit storage dtype (KVC_DTYPE_*). */
KVC_API int kvc_gqa_attention_ex(const void* h_Q, const void* h_K, const void* h_V, void* h_Out,
                         int q_len, int kv_len, int num_heads, int num_kv_heads,
                         int head_dim, int start_pos, float scale, int causal,
                         int dtype);

/* Copy positions [start, start+count) of `layer_idx` out of the process-wide pool
 * into host buffers laid out like the reference pool, (count, num_kv_heads,
 * head_dim).  No reference counterpart: it exists so pool contents can be
 * compared bit for bit with the reference's host-mode append (kv_cache.py:222-225). */
KVC_API int kvc_cache_gather(int layer_idx, int start, int count, void* h_K_out, void* h_V_out);

/* ==== 2. Paged pool for batched decode ==================================== */

typedef struct kvc_pool kvc_pool_t;
typedef struct kvc_plan kvc_plan_t;

/* Create a paged pool on `device`: for every layer, num_pages pages, each holding
 * page_size positions of num_kv_heads heads.  Storage is head-major inside a page
 * (one contiguous page_size x head_dim block per head).  No reference counterpart
 * beyond DeviceKVCachePool (attention.hip:168-214), which is the one-sequence,
 * unpaged special case. */
KVC_API int kvc_pool_create(int num_layers, int num_pages, int page_size, int num_kv_heads,
                    int head_dim, int dtype, int device, kvc_pool_t** out);
KVC_API int kvc_pool_destroy(kvc_pool_t* pool);

/* Device base addresses and sizes of the pool (for tests and diagnostics). */
KVC_API int kvc_pool_info(const kvc_pool_t* pool, void** k_base, void** v_base,
                  size_t* bytes_per_layer, size_t* bytes_per_page_head);

/* Fill pages [page_begin, page_end) of layers [layer_begin, layer_end) with
 * seeded N(0, stddev^2) values (synthetic benchmark data), on `stream`. */
KVC_API int kvc_pool_fill_normal(kvc_pool_t* pool, int layer_begin, int layer_end, int page_begin,
                         int page_end, uint64_t seed, float stddev, void* stream);

/* Append n token rows.  d_k_new / d_v_new: (n, num_kv_heads, head_dim) in the
 * pool dtype.  Row i goes to sequence d_rows[i] (a block-table row; NULL means
 * row 0 for every i) at position d_positions[i].  d_block_tables: int32
 * (n_rows, bt_stride) page ids.  The fused, vectorised replacement of the
 * reference's two blocking row copies (attention.hip:336-341, :410-415). */
KVC_API int kvc_append(kvc_pool_t* pool, int layer, const void* d_k_new, const void* d_v_new,
               const int32_t* d_block_tables, int bt_stride, const int32_t* d_rows,
               const int32_t* d_positions, int n, void* stream);

/* A decode plan: the split-K work list for one batch of queries, reused by every
 * layer of a step.  The split of a query depends only on its context length. */
KVC_API int kvc_plan_create(kvc_plan_t** out);
KVC_API int kvc_plan_destroy(kvc_plan_t* plan);

/* Build the plan on the host and upload it on `stream`.  Query i reads the block
 * table row h_rows[i] (NULL: row i) over positions [0, h_ctx_lens[i]).  The
 * queries' q rows are (num_heads, head_dim) at index i of the q buffer. */
KVC_API int kvc_plan_decode(kvc_plan_t* plan, const kvc_pool_t* pool, const int32_t* h_rows,
                    const int32_t* h_ctx_lens, int n_queries, int num_heads,
                    void* stream);

/* The split length (positions) kvc_plan_decode chooses for a batch on a GPU
 * with sm_count SMs: 512, or the one-wave length its cost model estimates
 * faster (KVC_SPLIT_TOKENS, when set, overrides the plan but not this query).
 * Host only; no counterpart in the reference. */
KVC_API int kvc_plan_split_tokens(const int32_t* h_ctx_lens, int n_queries, int num_heads,
                                  int num_kv_heads, int page_size, int sm_count, int* out);

/* The whole split partition kvc_plan_decode (and kvc_decode_noalloc) gives a batch
 * on a GPU with sm_count SMs, computed on the host: *split_tokens_out = the split
 * length, splits_out[i] (n_queries entries; may be NULL) = query i's splits,
 * including any full split the tail refinement cut into quarters, and
 * *n_splits_out = their sum, the split slots a plan's partials take (each
 * num_heads x (head_dim + 2) floats).  Unlike kvc_plan_split_tokens it follows the
 * KVC_SPLIT_TOKENS / KVC_TAIL_REFINE overrides, as the plan does.  Host only; no
 * counterpart in the reference. */
KVC_API int kvc_plan_split_counts(const int32_t* h_ctx_lens, int n_queries, int num_heads,
                                  int num_kv_heads, int page_size, int sm_count,
                                  int* split_tokens_out, int32_t* splits_out, int* n_splits_out);

/* Plan flags.  KVC_PLAN_KV_STABLE: the block tables and KV pages the plan reads
 * are not written by the kernel launched immediately before each decode on the
 * stream (e.g. they change only through host copies or earlier steps), so the
 * decode kernel may start streaming KV pages before that kernel's results are
 * visible (programmatic dependent launch).  Without it, the kernel waits first. */
#define KVC_PLAN_KV_STABLE 1
/* KVC_PLAN_GRAPH: decode launches of this plan may be captured in a CUDA graph
 * and replayed after the plan is rebuilt for other contexts (a decode loop whose
 * contexts grow by one position per step).  The kernels then read the plan's
 * counts from its device buffers, the decode grid spans every SM, the merge grid
 * has room for every query and head, and the plan keeps its device buffers (and
 * their layout) across rebuilds, growing them with headroom when a rebuild needs
 * more.  A rebuild that had to move them, or that changes the query count, head
 * count or pool, advances kvc_plan_generation: captured launches are then stale
 * and must be captured again.  Set the flag before the first build. */
#define KVC_PLAN_GRAPH 2
KVC_API int kvc_plan_set_flags(kvc_plan_t* plan, int flags);
/* The plan's layout generation (see KVC_PLAN_GRAPH).  No counterpart in the reference. */
KVC_API int kvc_plan_generation(const kvc_plan_t* plan, uint64_t* out);

/* Of the last plan: split items, work units (item x KV head x q-head chunk: one CTA
 * each in the CUDA-core kernel, handed out to the warps of the persistent
 * tensor-core kernel) and bytes of split scratch. */
KVC_API int kvc_plan_info(const kvc_plan_t* plan, int* n_items, int* n_ctas, size_t* scratch_bytes);

/* Split-K GQA decode attention for one layer.  d_q, d_out: (n_queries,
 * num_heads, head_dim) in the pool dtype.  Replaces gqa_online_softmax_kernel
 * (attention.hip:35-123) for a batch of queries over a paged pool. */
KVC_API int kvc_decode(kvc_pool_t* pool, const kvc_plan_t* plan, int layer, const void* d_q,
               void* d_out, const int32_t* d_block_tables, int bt_stride, float scale,
               void* stream);

/* Fused decode step for one layer on device buffers: appends row i of
 * d_k_new / d_v_new ((n_queries, num_kv_heads, head_dim)) at position
 * ctx_len[i]-1 of the query's block-table row (the plan's context lengths
 * include the new token), then runs kvc_decode.  The batched counterpart of
 * launch_gqa_attention_cached_fp16_device (attention.hip:376-440). */
KVC_API int kvc_append_decode(kvc_pool_t* pool, const kvc_plan_t* plan, int layer, const void* d_q,
                      const void* d_k_new, const void* d_v_new, void* d_out,
                      const int32_t* d_block_tables, int bt_stride, float scale, void* stream);

/* Reference-facing batched call with HOST buffers: copies h_q, h_k_new, h_v_new
 * to the device, appends and attends like kvc_append_decode, copies the result
 * to h_out and waits for it, like launch_gqa_attention_cached_fp16
 * (attention.hip:302-374) but for a batch of sequences. */
KVC_API int kvc_decode_host(kvc_pool_t* pool, const kvc_plan_t* plan, int layer, const void* h_q,
                    const void* h_k_new, const void* h_v_new, void* h_out,
                    const int32_t* d_block_tables, int bt_stride, float scale, void* stream);

/* No counterpart in the reference.  kvc_decode for callers that cannot allocate
 * device memory (runtimes that own every device allocation through their own
 * arena, plugins that may not call cudaMalloc).  The caller passes one layer's K
 * and V pages (the pool's layout, e.g. kvc_pool_info's base + layer *
 * bytes_per_layer), int32 block tables (query i uses row i), HOST context
 * lengths, q and out; the plan and the split partials live in a fixed 16 MiB
 * device array inside the library that every GPU loading it holds until the
 * process exits.  No cudaMalloc / cudaFree or other allocating routine is called.
 * fp16/bf16 pages, head_dim in {32,64,96,128,160,192,256}, page_size a multiple
 * of 16; at most 4096 queries, 16384 splits and 65536 work units, and the plan +
 * partials must fit 16 MiB: larger requests fail with KVC_ERR_INVALID_ARG.  The
 * split partition is kvc_plan_decode's for the same batch.  Every call looks up
 * the array's device address on the current device (cudaGetSymbolAddress), so a
 * call after cudaDeviceReset uses the array's new address.  All calls on a
 * device share its array, and each call overwrites it, so calls whose kernels
 * overlap on that GPU (for example on two streams) race: serialise them on one
 * stream.  The plan is staged through pageable host memory, so a call first
 * waits for the work already queued on its stream, and a call on a stream that
 * is being captured returns KVC_ERR_INVALID_ARG without enqueuing anything. */
KVC_API int kvc_decode_noalloc(const void* d_k_layer, const void* d_v_layer, int num_pages,
                               int page_size, int num_kv_heads, int head_dim, int dtype,
                               const int32_t* d_block_tables, int bt_stride,
                               const int32_t* h_ctx_lens, int n_queries, int num_heads,
                               const void* d_q, void* d_out, float scale, void* stream);

/* Copy positions [start, start+count) of block-table row `row` in `layer` into
 * device buffers (count, num_kv_heads, head_dim) on `stream`. */
KVC_API int kvc_gather(kvc_pool_t* pool, int layer, const int32_t* d_block_tables, int bt_stride,
               int row, int start, int count, void* d_k_out, void* d_v_out, void* stream);

/* ---- rotary position embedding ------------------------------------------------ */

/* The reference's `rope` (bindings.cpp:392-412, rope.hip:21-55 and :154-200) on
 * host fp16 arrays (seq_len, num_heads, head_dim), synchronous: the pair (i0, i1)
 * of every head of token t rotated by (pos_offset + t) / freq_base^(2i/head_dim),
 * i0 = 2i, i1 = 2i + 1, or i0 = i, i1 = i + head_dim/2 when neox != 0; fp32
 * math, fp16 result.  head_dim must be a positive even number <= 256. */
KVC_API int kvc_rope_host(const void* h_x, void* h_out, int seq_len, int num_heads, int head_dim,
                          int pos_offset, float freq_base, int neox);
/* The same on device buffers (fp16, bf16 or fp32 by `dtype`) on `stream`;
 * token t's position is d_positions[t] (int32, device) or, when d_positions is
 * null, pos_offset + t.  No counterpart in the reference for the per-token
 * positions (a batch of sequences each at its own position). */
KVC_API int kvc_rope(const void* d_x, void* d_out, int n_tokens, int num_heads, int head_dim,
                     const int32_t* d_positions, int pos_offset, float freq_base, int neox,
                     int dtype, void* stream);
/* kvc_append_decode with q and the new K rows rotated first, each query at its
 * plan position (ctx - 1): the rope + append + attend of one decode step
 * (layer.py:291-298 followed by kv_cache.py:240-256) as one launch chain.  The
 * rotation runs as a programmatic dependent ahead of the decode, which streams
 * KV meanwhile.  d_q / d_k_new are read, not modified. */
KVC_API int kvc_append_decode_rope(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                                   const void* d_q, const void* d_k_new, const void* d_v_new,
                                   void* d_out, const int32_t* d_block_tables, int bt_stride,
                                   float scale, float freq_base, int neox, void* stream);

/* ==== 3. Host-streamed offload (--offload-kv-cpu / --kv-mmap-dir) ========== */

typedef struct kvc_offload kvc_offload_t;

/* Page-locked host memory for the offload pools. */
KVC_API int kvc_host_alloc(size_t bytes, void** out);
KVC_API int kvc_host_free(void* ptr);

#define KVC_OFFLOAD_PINNED 1   /* h_k / h_v came from kvc_host_alloc */
#define KVC_OFFLOAD_REGISTER 2 /* try cudaHostRegister on h_k / h_v */

/* Attach host KV pools laid out as the reference's host arrays,
 * (num_layers, max_seq_len, num_kv_heads, head_dim) (src/kv_cache.py:97, :133-135
 * and the mmap arrays of :100-132).  The caller keeps ownership of h_k / h_v.
 * When the memory is neither pinned nor registrable, copies go through pinned
 * bounce buffers.  device < 0 selects the calling thread's current device. */
KVC_API int kvc_offload_create(void* h_k, void* h_v, int num_layers, int max_seq_len,
                       int num_kv_heads, int head_dim, int dtype, int flags, int device,
                       kvc_offload_t** out);
KVC_API int kvc_offload_destroy(kvc_offload_t* off);

/* Offload-mode attend, the replacement of KVCacheManager.attend's offload branch
 * (src/kv_cache.py:219-239) plus launch_gqa_attention_fp16 (attention.hip:228-284):
 * writes the q_len new rows into the host pools at (layer_idx, start_pos) (or,
 * when h_K_new and h_V_new are both null, takes them as written there already,
 * which is what KVCacheManager's own host append does before it calls
 * gqa_attention), makes rows [0, start_pos+q_len) of the layer resident on the
 * GPU (reusing the copy prefetched during the previous call for the rows below
 * start_pos, which are the cached history), attends, copies h_Out back, and
 * starts prefetching the next layer.  Results are bit-identical to the
 * GPU-resident pool's for the same inputs. */
KVC_API int kvc_offload_attend(kvc_offload_t* off, const void* h_Q, const void* h_K_new,
                       const void* h_V_new, void* h_Out, int layer_idx, int q_len,
                       int start_pos, int num_heads, float scale, int causal);

/* Discard prefetched layers (call after the host pools were written elsewhere). */
KVC_API int kvc_offload_invalidate(kvc_offload_t* off);

/* Cumulative host-to-device bytes and copy-engine time (ms) of the streamed
 * layers, and how many attend calls found their layer already prefetched. */
KVC_API int kvc_offload_stats(const kvc_offload_t* off, double* h2d_bytes, double* h2d_ms,
                      int64_t* prefetch_hits, int64_t* attend_calls);

/* No counterpart in the reference.  Keep an HBM mirror of as many layers as
 * `budget_bytes` of device memory holds (layers 0 .. n-1, *n_layers = n; 0
 * releases it).  The host pools stay the source of truth: an attend on a
 * mirrored layer appends on the host as before, uploads only the rows the
 * mirror lacks (the appended ones in decode; the whole layer on its first use
 * or after kvc_offload_invalidate) and attends on the mirror, bit-identical to
 * the streamed and resident paths; the other layers are streamed as before.
 * For a B200, whose HBM holds what a smaller GPU had to offload. */
KVC_API int kvc_offload_set_mirror(kvc_offload_t* off, size_t budget_bytes, int* n_layers);
/* Mirrored layers and the bytes uploaded into the mirror so far. */
KVC_API int kvc_offload_mirror_stats(const kvc_offload_t* off, int* n_layers,
                                     double* uploaded_bytes);

/* ==== 4. Head exchange across the GPUs of one node ========================
 * No counterpart in the reference (it runs on one GPU).  When the KV heads of
 * each layer are split over `world` GPUs (one process per GPU, rank r holding
 * KV heads [r*Hkv/world, (r+1)*Hkv/world) and their q-heads), every rank needs
 * all heads of the attention output.  kvc_append_decode_xchg runs the fused
 * append + decode on this rank's heads; its merge kernel stores every output
 * row straight into exchange slot `slot` of EVERY rank over NVLink (peer
 * stores), and a one-warp kernel behind it publishes a per-call epoch on every
 * rank and waits until all ranks have published it.  When the call's work has run on
 * `stream`, slot `slot` of this rank holds (n_queries, total_heads, head_dim)
 * outputs of all ranks.  All ranks must make the same sequence of calls (same
 * slots, same plans' query counts).  A slot may be rewritten by a peer from the
 * second following call on, so consume a slot on `stream` before the next
 * call, or rotate at least two slots.  A rank that never arrives makes the wait
 * give up after the wait limit (default 2 s): the device error word then holds
 * KVC_DEVERR_WAIT_LIMIT with info 0x10000 + the missing rank. */

typedef struct kvc_xchg kvc_xchg_t;

#define KVC_XCHG_HANDLE_BYTES 64

/* This rank's exchange buffer: n_slots slots of slot_bytes (a CUDA IPC
 * allocation on `device`). */
KVC_API int kvc_xchg_create(int device, int rank, int world, size_t slot_bytes, int n_slots,
                            kvc_xchg_t** out);
/* KVC_XCHG_HANDLE_BYTES bytes that let the other ranks map this buffer. */
KVC_API int kvc_xchg_handle(const kvc_xchg_t* x, void* handle_out);
/* Map every rank's buffer: `handles` holds world handles in rank order (this
 * rank's own entry is ignored). */
KVC_API int kvc_xchg_connect(kvc_xchg_t* x, const void* handles);
/* Alternative to kvc_xchg_connect for hosts that map peer memory themselves:
 * the device address of every rank's exchange buffer in this process, in rank
 * order, peer_bases[rank] being this rank's own (kvc_xchg_base). */
KVC_API int kvc_xchg_connect_ptrs(kvc_xchg_t* x, void* const* peer_bases);
KVC_API int kvc_xchg_base(const kvc_xchg_t* x, void** d_base);
/* Device address of slot `slot` of this rank's buffer. */
KVC_API int kvc_xchg_slot(const kvc_xchg_t* x, int slot, void** d_ptr);
/* Limit of the wait for the other ranks, in seconds (0, 60]. */
KVC_API int kvc_xchg_set_wait_limit(kvc_xchg_t* x, double seconds);
KVC_API int kvc_xchg_destroy(kvc_xchg_t* x);
/* kvc_append_decode with the outputs exchanged: this rank's q-heads are heads
 * [head_offset, head_offset + plan's num_heads) of total_heads.  d_k_new and
 * d_v_new may both be null (decode without an append).  fp16/bf16 pools with
 * the tensor-core head dims only. */
KVC_API int kvc_append_decode_xchg(kvc_pool_t* pool, const kvc_plan_t* plan, int layer,
                                   const void* d_q, const void* d_k_new, const void* d_v_new,
                                   kvc_xchg_t* x, int slot, int total_heads, int head_offset,
                                   const int32_t* d_block_tables, int bt_stride, float scale,
                                   void* stream);

/* ==== 5. Layer pipeline over the process-wide pool ========================== */

/* Weight storage types: the GGML type ids forward_layer_cached takes
 * (bindings.cpp:518-557).  A weight is (n, k) row-major; each row is k / per
 * blocks: F16 (per 1, 2 bytes), Q4_0 (32, 18), Q8_0 (32, 34), Q4_K (256, 144),
 * Q6_K (256, 210), the block layouts of gguf_parser.py:374-590. */
#define KVC_WTYPE_F16 1
#define KVC_WTYPE_Q4_0 2
#define KVC_WTYPE_Q8_0 8
#define KVC_WTYPE_Q4_K 12
#define KVC_WTYPE_Q6_K 14

/* Bytes of an (n, k) weight of w_type (the size rule of check_weight_buffer,
 * bindings.cpp:518-557); KVC_ERR_INVALID_ARG for an unknown type or a k the
 * type's block does not divide. */
KVC_API int kvc_weight_bytes(int w_type, int n, int k, size_t* out);

/* d_out (m, n) = d_x (m, k) · Wᵀ on the device, fp16 activations, fp32 sums,
 * fp16 out: the projections of project_on_device (attention.hip:572-599 ⇒
 * launch_matmul_fp16_nt_device / launch_matmul_q4_0_device / ..._q8_0 / ..._q4_k
 * / ..._q6_k).  k a multiple of 32 and n of 16; d_x and d_w 16-byte aligned. */
KVC_API int kvc_linear(const void* d_x, int m, int k, const void* d_w, int w_type, int n,
                       void* d_out, void* stream);
/* d_out (m, n) = silu(x · Wgateᵀ) · (x · Wupᵀ), both products rounded to fp16
 * first (attention.hip:684-686 with launch_swiglu_fp16_device, mlp.hip:18-31). */
KVC_API int kvc_linear_swiglu(const void* d_x, int m, int k, const void* d_w_gate,
                              const void* d_w_up, int w_type, int n, void* d_out, void* stream);
/* d_out (m, n) = d_res + fp16(x · Wᵀ) (attention.hip:687-689: the down projection
 * and launch_residual_add_fp16_device).  d_out may alias d_res. */
KVC_API int kvc_linear_residual(const void* d_x, int m, int k, const void* d_w, int w_type, int n,
                                const void* d_res, void* d_out, void* stream);
/* RMSNorm of each row of d_x (m, k): x / sqrt(mean(x²) + eps) · w (rmsnorm.hip:23-74).
 * With d_res: h = fp16(x + res) is written to d_h_out and normalised instead
 * (rmsnorm.hip:79-140).  fp16 throughout. */
KVC_API int kvc_rmsnorm(const void* d_x, const void* d_res, void* d_h_out, const void* d_w,
                        void* d_out, int m, int k, float eps, void* stream);

/* Replaces launch_forward_layer_cached_fp16 (attention.h:77-105,
 * attention.hip:603-695) behind matmul_module.forward_layer_cached
 * (bindings.cpp:562-627): one transformer layer for seq_len tokens at positions
 * pos_offset.. on the process-wide fp16 pool, with the reference's argument order.
 * Host buffers: x_in / x_out (seq_len, hidden_size), the two norm weights
 * (hidden_size), and the seven weights of the given types (q, k, v: (H·D | Hkv·D,
 * hidden); o: (hidden, H·D); gate, up: (intermediate, hidden); down: (hidden,
 * intermediate)).  Like the reference, the activations and all weights are copied
 * to the device on every call and the result back before it returns.  The pool
 * receives the rotated K rows and the V rows at (layer_idx, pos_offset..). */
KVC_API int kvc_forward_layer_cached(
    const void* h_x_in, void* h_x_out, const void* h_attn_norm_w, const void* h_wq, int wq_type,
    const void* h_wk, int wk_type, const void* h_wv, int wv_type, const void* h_wo, int wo_type,
    const void* h_ffn_norm_w, const void* h_wgate, int wgate_type, const void* h_wup,
    int wup_type, const void* h_wdown, int wdown_type, int layer_idx, int seq_len, int pos_offset,
    int hidden_size, int intermediate_size, int num_heads, int num_kv_heads, int head_dim,
    float rms_norm_eps, float rope_freq_base, int rope_neox, float scale);

/* kvc_forward_layer_cached on device buffers (weights resident in HBM), work
 * enqueued on `stream`, no host synchronisation.  x_out may alias x_in. */
KVC_API int kvc_forward_layer_cached_device(
    const void* d_x_in, void* d_x_out, const void* d_attn_norm_w, const void* d_wq, int wq_type,
    const void* d_wk, int wk_type, const void* d_wv, int wv_type, const void* d_wo, int wo_type,
    const void* d_ffn_norm_w, const void* d_wgate, int wgate_type, const void* d_wup,
    int wup_type, const void* d_wdown, int wdown_type, int layer_idx, int seq_len, int pos_offset,
    int hidden_size, int intermediate_size, int num_heads, int num_kv_heads, int head_dim,
    float rms_norm_eps, float rope_freq_base, int rope_neox, float scale, void* stream);

/* One decode step of one layer for a BATCH of sequences on a paged pool: the
 * batched counterpart of kvc_forward_layer_cached_device, for the decode loop of
 * generate_batch_ids (src/inference.py:435-447), which the reference runs one
 * sequence at a time through forward_layer_cached (attention.hip:603-695).
 * Token i of d_x_in / d_x_out ((n, hidden_size) fp16, n = the plan's query
 * count) is the new token of query i of `plan` (kvc_plan_decode): it is rotated
 * at position ctx_i - 1, its K/V row is appended there in block-table row
 * rows[i], and it attends over positions [0, ctx_i).  Head counts come from the
 * plan (q-heads) and the fp16 pool (KV heads, head_dim); weights as in
 * kvc_forward_layer_cached.  The activations live in a workspace of the plan, so
 * calls sharing a plan must be ordered on one stream.  x_out may alias x_in. */
KVC_API int kvc_forward_layer_paged(
    kvc_pool_t* pool, const kvc_plan_t* plan, int layer_idx, const void* d_x_in, void* d_x_out,
    const void* d_attn_norm_w, const void* d_wq, int wq_type, const void* d_wk, int wk_type,
    const void* d_wv, int wv_type, const void* d_wo, int wo_type, const void* d_ffn_norm_w,
    const void* d_wgate, int wgate_type, const void* d_wup, int wup_type, const void* d_wdown,
    int wdown_type, const int32_t* d_block_tables, int bt_stride, int hidden_size,
    int intermediate_size, float rms_norm_eps, float rope_freq_base, int rope_neox, float scale,
    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVCACHE_H */
