/*
 * aoh.h -- C ABI of libaoh.so, the B200 (sm_100a) head-mixed attention runtime
 * and effective-rank head classifier.
 *
 * Plain C: every pointer is either a host pointer or a caller-owned CUDA device
 * pointer (stated per argument); sizes are in elements unless named *_bytes;
 * streams are cudaStream_t passed as void*.  Every entry point returns an
 * aoh_status; on failure aoh_last_error() returns a message for the calling
 * thread.  No exception crosses this boundary.
 *
 * Tensor layouts (row-major, contiguous): q and out (batch, q_len, num_q_heads,
 * head_dim); k_new and v_new (batch, q_len, num_kv_heads, head_dim) -- the
 * reference's (bsz, q_len, heads, head_dim) projection views before
 * .transpose(1, 2), with RoPE already applied (eval/efficiency/
 * benchmark_llama31.py:204-209).  Heads are in ORIGINAL order: the library is
 * label-driven and needs no offline weight reordering
 * (eval/efficiency/reorder_weights.py:19-60 is not required).
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the reference project root).
 */
#ifndef AOH_H_
#define AOH_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AOH_ABI_VERSION 1

#if defined(__GNUC__)
#define AOH_API __attribute__((visibility("default")))
#else
#define AOH_API
#endif

typedef enum {
  AOH_OK = 0,
  AOH_ERR_INVALID_ARGUMENT = 1, /* reference: ValueError (benchmark_llama31.py:257-265, classifier.py:41-42) */
  AOH_ERR_OUT_OF_PAGES = 2,     /* reference: torch.OutOfMemoryError (benchmark_llama31.py:398) */
  AOH_ERR_CUDA = 3,             /* a CUDA runtime call failed */
  AOH_ERR_UNSUPPORTED = 4,      /* shape/dtype outside what the kernels implement */
  AOH_ERR_STATE = 5,            /* reference: RuntimeError (classifier.py:143-144) */
  AOH_ERR_DEVICE_CHECK = 6      /* a device-side bounds check or bounded wait tripped */
} aoh_status;

typedef enum { AOH_F32 = 0, AOH_BF16 = 1 } aoh_dtype;

typedef void* aoh_stream; /* cudaStream_t */

/* ABI version of the loaded library (AOH_ABI_VERSION it was built with). */
AOH_API int aoh_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
AOH_API const char* aoh_last_error(void);

/* ------------------------------------------------------------------------- */
/* Paged KV cache                                                            */
/* Replaces AoHKVCache (eval/efficiency/benchmark_llama31.py:135-184;        */
/* benchmark_qwen.py:144-193): per-layer full KV for retrieval heads, sink + */
/* recent KV for streaming heads (compress_stream, attention_utils.py:23-42).*/
/* Here every (layer, sequence, KV head) "unit" owns a list of fixed-size    */
/* pages in one device pool; retrieval units grow page by page, streaming    */
/* units own ceil(sink/page) sink pages plus a ring of ceil(recent/page)     */
/* pages and never more.                                                     */
/* ------------------------------------------------------------------------- */

typedef struct aoh_kv_cache aoh_kv_cache;

typedef struct {
  int32_t num_layers;
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;     /* must be 128 */
  int32_t page_size;    /* must be 16 */
  int32_t dtype;        /* aoh_dtype */
  int32_t sink_size;    /* >= 0; reference default 128 */
  int32_t recent_size;  /* >= 0; reference default 256 */
  int32_t max_context;  /* tokens per sequence a retrieval unit may hold */
  int32_t num_pages;    /* pages in the pool */
  const uint8_t* labels; /* host, (num_layers, num_kv_heads): 1 = retrieval, 0 = streaming */
  const uint8_t* owned;  /* host, (num_layers, batch, num_kv_heads): 1 = stored here; NULL = all */
} aoh_kv_config;

/* AoHKVCache.__init__ (benchmark_llama31.py:136-151) + patch_aoh_model's label
 * validation (:256-266).  Host bookkeeping only; no device memory is touched. */
AOH_API int aoh_kv_create(const aoh_kv_config* cfg, aoh_kv_cache** out);
AOH_API void aoh_kv_destroy(aoh_kv_cache* cache);

/* Device buffers the caller must allocate for aoh_kv_bind. */
AOH_API int aoh_kv_buffer_sizes(const aoh_kv_cache* cache, int64_t* pool_bytes, int64_t* table_bytes);

/* Bind caller-owned device memory (pool: pool_bytes, 1024-byte aligned;
 * tables: table_bytes, 16-byte aligned) and upload the block tables.
 * Streaming units receive their sink and ring pages here. */
AOH_API int aoh_kv_bind(aoh_kv_cache* cache, void* pool, void* tables, aoh_stream stream);

/* Give every retrieval unit of sequence `seq` (-1 = all sequences) the pages
 * for positions [0, n_tokens).  Host-side; call aoh_kv_sync before the next
 * kernel that reads the new pages.  AOH_ERR_OUT_OF_PAGES leaves the cache
 * consistent (pages granted so far stay granted). */
AOH_API int aoh_kv_reserve(aoh_kv_cache* cache, int32_t seq, int32_t n_tokens);

/* Return all pages of sequence `seq` (-1 = all) to the pool; sequences are
 * then empty (positions restart at 0). Streaming pages are kept. */
AOH_API int aoh_kv_release(aoh_kv_cache* cache, int32_t seq);

/* Upload block-table entries changed since the last sync (stream-ordered). */
AOH_API int aoh_kv_sync(aoh_kv_cache* cache, aoh_stream stream);

/* Pages currently free in the pool. */
AOH_API int32_t aoh_kv_free_pages(const aoh_kv_cache* cache);

/* Host copy of one unit's page list (for inspection and tests). */
AOH_API int aoh_kv_unit_pages(const aoh_kv_cache* cache, int32_t layer, int32_t seq, int32_t kv_head,
                      int32_t* pages, int32_t capacity, int32_t* n_pages);

/* Where `position` of unit (layer, seq, kv_head) is stored, given past_len
 * cached tokens: *page (pool page id) and *slot (0..15), both -1 if the
 * position is not held (evicted from a streaming head, not yet cached, or the
 * unit is not stored here).  Page layout in the pool:
 *   f32 (16 KB):  row-major [kv: 0 = K, 1 = V][slot: 16][dim: 128];
 *   bf16 (8 KB):  [half h: dims 64h..64h+63][kv][slot][128 bytes], the 16-byte
 *                 chunk c of a row stored at chunk c ^ (slot & 7) -- the 128-byte
 *                 swizzle the tensor-core kernels read directly. */
AOH_API int aoh_kv_locate(const aoh_kv_cache* cache, int32_t layer, int32_t seq, int32_t kv_head,
                          int32_t position, int32_t past_len, int32_t* page, int32_t* slot);

/* Read and clear the device-side check word (bounds checks, bounded waits);
 * synchronizes `stream`. *flags == 0 means no check tripped.  Bit 1: a
 * block-table entry outside the pool (the page was skipped); bit 2: a bounded
 * wait gave up (250 ms for a CTA's own pipeline, 1 s for a peer's gather
 * flag) -- until this call clears the bit, later launches give up at their
 * first slow wait too, and their results are void.  On bit 2 this call also
 * re-zeroes the ticket counters the library owns (prefill scratch, the
 * allocation-free decode scratch); a caller-owned decode workspace must be
 * re-zeroed by the caller before its next use. */
AOH_API int aoh_kv_device_status(aoh_kv_cache* cache, int32_t* flags, aoh_stream stream);

/* ------------------------------------------------------------------------- */
/* Attention: attend over (cached keys + this call's keys), then append.     */
/* Replaces the patched forward's attention core (make_aoh_forward,          */
/* benchmark_llama31.py:218-250; benchmark_qwen.py:235-267):                 */
/*   retrieval heads -> eager_attention (:123-132), causal iff q_len > 1,    */
/*   streaming heads -> streaming_attention (attention_utils.py:92-119),     */
/*   then AoHKVCache.append_layer (:171-184).                                */
/* past_len is the reference's kv_cache.kv_seq_len (all sequences equal).    */
/* Positions [0, past_len + q_len) must be reserved (aoh_kv_reserve + sync). */
/* ------------------------------------------------------------------------- */

/* Device-resident sequence length, for decode steps replayed from a CUDA
 * graph: aoh_kv_set_length writes it, aoh_kv_advance adds to it (one tiny
 * kernel each, stream-ordered, capturable), and aoh_attn_decode reads it when
 * called with past_len = AOH_PAST_LEN_DEVICE.  The host keeps a copy of the
 * expected value to size kernel launches; pages for every length the device
 * will reach must be reserved and synced beforehand. */
#define AOH_PAST_LEN_DEVICE (-1)
AOH_API int aoh_kv_set_length(aoh_kv_cache* cache, int32_t length, aoh_stream stream);
AOH_API int aoh_kv_advance(aoh_kv_cache* cache, int32_t n, aoh_stream stream);
/* enabled = 0: aoh_attn_decode / aoh_attn_decode_noalloc attend without
 * appending the new token (a dry run) until re-enabled; default 1.  For the
 * uncaptured first launch before capturing a decode step at the same position:
 * an append there would already overwrite a streaming head's ring slot that
 * the captured step still attends (its oldest window row). */
AOH_API int aoh_kv_set_decode_append(aoh_kv_cache* cache, int32_t enabled);

/* Upper bound of the workspace aoh_attn_decode needs (bytes). */
AOH_API size_t aoh_decode_workspace_bytes(const aoh_kv_cache* cache);

/* Decode step (q_len = 1): split-KV over the paged cache, combine, append.
 * past_len may be AOH_PAST_LEN_DEVICE (bf16 caches).  workspace: caller-owned
 * device memory of aoh_decode_workspace_bytes(), zero-filled once before its
 * first use; calls sharing a workspace must be ordered on one stream (the
 * kernel starts early under programmatic dependent launch and waits for the
 * previous kernel before touching q, outputs or the workspace). */
AOH_API int aoh_attn_decode(aoh_kv_cache* cache, int32_t layer, int32_t past_len, const void* q,
                    const void* k_new, const void* v_new, void* out, void* workspace,
                    size_t workspace_bytes, aoh_stream stream);

/* aoh_attn_decode without a workspace argument (past_len may be
 * AOH_PAST_LEN_DEVICE, as for aoh_attn_decode), for callers that cannot
 * allocate device memory: plugin hosts that hand an op only its input and
 * output buffers and own every allocation themselves, and runtimes that may
 * not allocate after start-up (fixed memory budgets, allocators that are not
 * reachable from the calling layer).  No counterpart in the reference, whose
 * eager path allocates new tensors on every call.
 *
 * The split-KV scratch is a static device array inside libaoh.so: 274,432
 * bytes (tickets for 256 units + 64 cluster partials), held on every GPU that
 * loads the library until the process exits.  bf16 caches only; a layer whose
 * plan would need more than 256 (sequence, KV head) units or more than 64
 * cluster partials is rejected with AOH_ERR_UNSUPPORTED (a one-wave plan on a
 * 148-SM B200 needs at most 45).  The first call on a device looks up the
 * array's device address and zeroes its tickets on `stream` -- make that first
 * call outside any stream capture.  Every call shares the array and it keeps
 * the last call's contents: calls that overlap on the GPU (two streams, two
 * caches at once) race; order them on one stream.  Allocates nothing: no
 * cudaMalloc, no cudaFree, no allocating library routine. */
AOH_API int aoh_attn_decode_noalloc(aoh_kv_cache* cache, int32_t layer, int32_t past_len, const void* q,
                                    const void* k_new, const void* v_new, void* out, aoh_stream stream);

/* Prefill chunk (any q_len >= 1): causal attention for retrieval heads,
 * sink + window for streaming heads, then append.  bf16 caches: one kernel
 * attends and appends; when a chunk has too few row blocks to fill the GPU,
 * retrieval heads are split over key ranges whose partials (each range's
 * normalised output in bf16, its max and sum in fp32) are combined on the
 * GPU.  The kernel's scratch (ticket counters, partials) belongs to the
 * cache, is allocated by the first call and grows (a growing call
 * synchronises `stream` and must not be inside a stream capture), and is
 * freed by aoh_kv_destroy. */
AOH_API int aoh_attn_prefill(aoh_kv_cache* cache, int32_t layer, int32_t past_len, int32_t q_len,
                     const void* q, const void* k_new, const void* v_new, void* out,
                     aoh_stream stream);

/* The prefill of the decoding-simulation ("flash") protocol: replaces the
 * prefill branch of aoh_flash_attention (eval/efficiency/attention_utils.py:
 * 45-89, driven by flash_prefill in eval/results/run_longbench.py:119-139).
 * The prompt goes in one call over an empty cache (past_len must be 0):
 * every head -- streaming heads too -- attends causally to the whole prompt,
 * then each unit keeps what its label says (retrieval: every row; streaming:
 * the sink and the latest window rows, the reference's trim).  Decode steps of
 * the protocol are aoh_attn_decode (the same arithmetic as the eager path for
 * q_len = 1).  bf16 caches only; AOH_ERR_UNSUPPORTED for past_len != 0. */
AOH_API int aoh_attn_prefill_flash(aoh_kv_cache* cache, int32_t layer, int32_t past_len, int32_t q_len,
                                   const void* q, const void* k_new, const void* v_new, void* out,
                                   aoh_stream stream);

/* Query/key preparation of the patched forward in one kernel: replaces the
 * q_norm / k_norm (Qwen3's per-head RMSNorm) and apply_rotary_pos_emb steps
 * of make_aoh_forward (eval/efficiency/benchmark_qwen.py:216-226,
 * benchmark_llama31.py:204-209).  bf16 device tensors: q (batch, q_len,
 * num_q_heads, 128), k (batch, q_len, num_kv_heads, 128) -- the projections'
 * views --, cos / sin (batch, q_len, 128) as the model's rotary embedding
 * returns them; q_norm_weight / k_norm_weight (128) or both NULL (no norm);
 * eps the norms' epsilon.  Writes the rotated q_out / k_out (same shapes,
 * contiguous, not aliasing the inputs): the attention entry points' q and
 * k_new.  The rotation is bit-exact to the bf16 torch ops; a normed value may
 * differ by one bf16 ulp (the mean square is summed in another order). */
AOH_API int aoh_rope_qk(const void* q, const void* k, const void* cos, const void* sin, const void* q_norm_weight,
                        const void* k_norm_weight, float eps, int32_t batch, int32_t q_len, int32_t num_q_heads,
                        int32_t num_kv_heads, int32_t head_dim, void* q_out, void* k_out, aoh_stream stream);

/* AoHKVCache.append_layer alone (benchmark_llama31.py:171-184): write q_len
 * new tokens at positions past_len.. into every unit of `layer`. */
AOH_API int aoh_kv_append(aoh_kv_cache* cache, int32_t layer, int32_t past_len, int32_t q_len,
                  const void* k_new, const void* v_new, aoh_stream stream);

/* ------------------------------------------------------------------------- */
/* Effective-rank classifier                                                 */
/* Replaces compute_all_eff_ranks / compute_eff_rank                         */
/* (aoh/effective_rank.py:27-142): per (query head h, KV group h / GRP) the  */
/* spectrum of C = (W_Q W_Q^T)(W_K W_K^T), turned into an effective rank.    */
/* ------------------------------------------------------------------------- */

/* wq: device (num_layers, num_q_heads * head_dim, d_model) -- q_proj.weight per layer;
 * wk: device (num_layers, num_kv_heads * head_dim, d_model) -- k_proj.weight;
 * dtype: AOH_BF16 or AOH_F32 (the reference upcasts either to float32,
 * aoh/weight_extract.py:105-111);
 * eff_ranks_out: device f64 (num_layers, num_q_heads), each value rounded to
 * float32 as the reference stores float(fp32) (effective_rank.py:85);
 * binary != 0 uses sign(W) (compute_gram_matrix_binary, :45-59).
 * workspace: device memory of aoh_classify_workspace_bytes(). */
AOH_API size_t aoh_classify_workspace_bytes(int32_t num_layers, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim);
AOH_API int aoh_classify_eff_ranks(const void* wq, const void* wk, int32_t dtype, int32_t num_layers, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, int32_t d_model, int32_t binary,
                           double* eff_ranks_out, void* workspace, size_t workspace_bytes,
                           aoh_stream stream);

/* ------------------------------------------------------------------------- */
/* Multi-GPU partition (no counterpart in the reference, which only places   */
/* whole layers with device_map="sequential", benchmark_llama31.py:354-374): */
/* per layer, longest-processing-time greedy assignment of the (sequence,    */
/* KV head) units to ranks by touched KV tokens.                             */
/* ------------------------------------------------------------------------- */

/* labels: host (num_layers, num_kv_heads); owner_out: host (num_layers, batch,
 * num_kv_heads) rank ids; cost of a unit = context + 1 for retrieval,
 * min(context, sink + recent) + 1 for streaming. */
AOH_API int aoh_partition(const uint8_t* labels, int32_t num_layers, int32_t batch, int32_t num_kv_heads,
                  int32_t context, int32_t sink_size, int32_t recent_size, int32_t n_ranks,
                  int32_t* owner_out);

/* ------------------------------------------------------------------------- */
/* Output gather over NVLink (no counterpart in the reference).              */
/* One process per GPU of one node; each rank decodes the units it owns      */
/* (aoh_partition) and the decode kernel itself stores every finished unit's */
/* output rows into the output region of every rank.  aoh_gather_wait, after */
/* the decode of the layer, publishes this rank's units (a flag per (layer, */
/* unit) in every rank's flag array) and returns (on the GPU) once all units */
/* of the layer have arrived here: every rank calls it for every layer.      */
/* ------------------------------------------------------------------------- */

#define AOH_IPC_HANDLE_BYTES 64

/* Device memory (zero-filled) that the other processes of the node can map:
 * *dev_ptr is usable here, ipc_handle (AOH_IPC_HANDLE_BYTES) is passed to
 * them.  Freed with aoh_shared_free. */
AOH_API int aoh_shared_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
AOH_API int aoh_shared_free(void* dev_ptr);
/* Map another process's aoh_shared_alloc region on the current device;
 * unmapped with aoh_shared_close. */
AOH_API int aoh_shared_open(const void* ipc_handle, void** dev_ptr);
AOH_API int aoh_shared_close(void* dev_ptr);

/* Attach the gather to a bf16 cache (n_ranks <= 8; n_ranks = 0 detaches).
 * out_regions[r]: rank r's output region as mapped in this process
 * (out_regions[rank] is this rank's own), each out_bytes long, laid out alike
 * on every rank; flag_arrays[r]: rank r's flag array as mapped here, int32
 * (num_layers * batch * num_kv_heads), zero-filled before the first step.
 * While attached, aoh_attn_decode needs its `out` inside the own region and
 * writes the same offsets in every region. */
AOH_API int aoh_kv_set_peers(aoh_kv_cache* cache, int32_t n_ranks, int32_t rank, void* const* out_regions,
                             size_t out_bytes, int32_t* const* flag_arrays);
/* Stream-ordered, after this rank's aoh_attn_decode of `layer`: publishes the
 * units this rank owns (flag = position + 1 in every rank's flag array, after
 * a system-scope fence), then waits until every (sequence, KV head) unit of
 * `layer` decoded at position past_len (or the device length,
 * AOH_PAST_LEN_DEVICE) has been stored here by its owner.  The wait is
 * bounded: a missing peer sets the cache's device check word
 * (aoh_kv_device_status) instead of hanging. */
AOH_API int aoh_gather_wait(aoh_kv_cache* cache, int32_t layer, int32_t past_len, aoh_stream stream);

/* ------------------------------------------------------------------------- */
/* Diagnostics (no counterpart in the reference): one building block of the  */
/* kernels on caller-given device data, for tests.                           */
/* ------------------------------------------------------------------------- */

/* out[i] = 2^x[i] as the prefill softmax computes it on the FMA pipe (a cubic
 * on the fraction, the integer part added to the exponent; x in [-126, 8]);
 * x and out: device float32 arrays of n elements. */
AOH_API int aoh_diag_exp2_poly(const float* x, float* out, int32_t n, aoh_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* AOH_H_ */
