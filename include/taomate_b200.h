/*
 * taomate_b200: C ABI of the B200 (sm_100a) kernels for TaoMate's causal-LTX
 * streaming attention step.
 *
 * All pointers are device pointers owned by the caller (PyTorch's caching
 * allocator in the Python host layer); the library never frees them and never
 * keeps them past the call.  `stream` is a cudaStream_t passed as void*; all
 * work is stream-ordered and no entry point synchronises the host, except
 * tm_device_error().  Every entry point returns a tm_status; on error
 * tm_last_error() gives a one-line message (thread-local).
 *
 * Reference paths below are relative to the TaoLiveAIGC/TaoMate source tree.
 */
#ifndef TAOMATE_B200_H
#define TAOMATE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define TM_API __attribute__((visibility("default")))
#else
#define TM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  TM_OK = 0,
  TM_ERR_INVALID_ARGUMENT = 1, /* shape, size or count out of range */
  TM_ERR_ALIGNMENT = 2,        /* pointer or stride misaligned for vector / TMA access */
  TM_ERR_UNSUPPORTED = 3,      /* head dim or dtype that is not built */
  TM_ERR_CUDA = 4,             /* CUDA runtime / driver call failed */
  TM_ERR_DEVICE = 5            /* a kernel's bounded wait ran out (device error flag) */
} tm_status;

enum { TM_DTYPE_BF16 = 0, TM_DTYPE_F32 = 1 };

/* Version of this ABI (incremented on any signature change).  No counterpart
 * in the reference (library housekeeping). */
TM_API int tm_abi_version(void);

/* Message of the last failed call on this thread ("" if none).
 * No counterpart in the reference: the Python layer raises it as the
 * reference's exception types. */
TM_API const char* tm_last_error(void);

/*
 * No counterpart in the reference (its torch ops have no device-side waits).
 * Read and clear the device-side error flag of the current device.  Blocks
 * until all prior work on the device has finished.  *code_out receives 0 when
 * no kernel reported an error, 1 when an attention kernel's bounded pipeline
 * wait ran out, 2 when a peer flag wait (tm_peer_wait / tm_peer_exchange) did.
 */
TM_API int tm_device_error(int* code_out);

/*
 * A1. SPLIT-mode RoPE cos/sin tables for one batch row.
 * Replaces causal_precompute_freqs_cis (ltx_causal/rope/causal_rope.py:139-357,
 * called at ltx_causal/transformer/kv_cache.py:2911-3027) for rope_type=SPLIT.
 *   grid: n_pos (1 or 3) latent extents: (F, H, W) video, (F,) audio / temporal.
 *   theta: effective base (the caller applies NTK scaling, causal_rope.py:199-246).
 *   max_pos: n_pos normalisers (20, 2048, 2048 for video).
 *   repeat_per_frame: >1 expands each temporal position to that many tokens
 *     (cross-modal PE expansion at kv_cache.py:2973-2983); 1 otherwise.
 * Output layout: [num_heads, T, dim / 2 / num_heads], T = prod(grid) * repeat,
 * dtype out_dtype (bf16 or fp32).  Angles are formed in fp32 in the
 * reference's operation order; cos/sin in full-precision fp32.
 */
TM_API int tm_rope_tables_split(void* cos_out, void* sin_out, int out_dtype, int n_pos,
                         const int64_t* grid, int dim, int num_heads, double theta,
                         const double* max_pos, int64_t start_frame, int is_audio,
                         int64_t repeat_per_frame, void* stream);

/*
 * A2+A3. Fused q/k RMSNorm (over the full H*D inner dim) + split RoPE, with
 * the Ulysses seq->head send-buffer layout applied on the store.
 * Replaces attn.q_norm / attn.k_norm (nn.RMSNorm, causal_attention.py:105-106,
 * applied at kv_cache.py:1406-1407) followed by attn._apply_rope ->
 * apply_split_rotary_emb (causal_attention.py:326, causal_rope.py:102-132),
 * and the pack permute of _seq_to_head (taomate/runtime_support/parallel/
 * all_to_all.py:139-140).
 *   x:   [B, L, H*D] bf16 (token rows; row/batch strides in elements).
 *   out: element (b, l, h, d) is stored at
 *        out + g*out_group_stride + b*out_batch_stride + l*out_row_stride
 *            + (h mod H/sp_size)*D + d,   g = h / (H/sp_size),
 *        i.e. [B, L, H, D] for sp_size 1 and an all-to-all send buffer with
 *        one head group per destination rank otherwise.
 *   norm_weight: [H*D] bf16, or NULL for no RMSNorm.
 *   cos/sin: [B, H, L, D/2] bf16 with the given strides, or NULL for no RoPE
 *   (a job with neither is a pure layout copy, used for V).
 * Up to 4 jobs (q, k, v) run in one launch.  D in {64, 128};
 * H*D in {256, 512, 1024, 2048, 4096}.  Rows must be 16-byte aligned.
 */
typedef struct {
  const void* x;
  void* out;
  const void* norm_weight;
  const void* cos;
  const void* sin;
  int64_t x_batch_stride, x_row_stride;
  int64_t out_group_stride, out_batch_stride, out_row_stride;
  int64_t pe_batch_stride, pe_head_stride, pe_row_stride;
  int64_t L;
} tm_norm_rope_job;

TM_API int tm_norm_rope(const tm_norm_rope_job* jobs, int n_jobs, int B, int H, int D, float eps,
                 int sp_size, void* stream);

/*
 * A2+A3+A4. tm_norm_rope whose head group g (the heads rank g owns after the
 * seq->head exchange) is stored group_delta[g] bytes away from the job's
 * output address: with every rank's receive buffer mapped into this process
 * (tm_peer_open) the exchange happens in the kernel's own stores over NVLink
 * (_seq_to_head, all_to_all.py:125-151).  Offsets 16-byte aligned, sp_size <= 8.
 */
TM_API int tm_norm_rope_peer(const tm_norm_rope_job* jobs, int n_jobs, int B, int H, int D,
                 float eps, int sp_size, const int64_t* group_delta, void* stream);

/*
 * A4/A8. NVLink peer memory for the fused Ulysses exchanges (no counterpart
 * function in the reference, which calls torch.distributed.all_to_all_single,
 * all_to_all.py:125-173).
 *   tm_peer_alloc   device buffer (cleared) and its 64-byte CUDA IPC handle;
 *   tm_peer_open    map another rank's buffer (same box) into this process;
 *   tm_peer_close / tm_peer_free  undo them;
 *   tm_peer_flag_bytes  size of a rank's flag buffer (flags, then this rank's
 *                   epoch counters at byte tm_peer_flag_bytes() - 64);
 *   tm_peer_signal  after this rank's stores: publish its next epoch of
 *                   `slot` (0..3) in every rank's flag buffer (peer_flags[i] =
 *                   rank i's flag buffer as mapped here);
 *   tm_peer_wait    stream-ordered wait until every rank published that epoch;
 *                   gives up after the wait limit (2 s unless set below) and
 *                   records device error 2 (tm_device_error) instead of hanging;
 *   tm_peer_exchange  tm_peer_signal then tm_peer_wait in one kernel launch
 *                   (flags = this rank's own flag buffer);
 *   tm_peer_set_wait_limit  limit, in ns, of the waits launched after the
 *                   call (<= 0: back to the 2 s default); returns the old
 *                   limit.  A wait that runs out advances its epoch counter
 *                   like one that succeeded, so the next wait of that slot
 *                   waits for the following epoch.
 * At most 8 ranks.  Plain peer stores and loads; no multicast.
 */
TM_API int tm_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
TM_API int tm_peer_free(void* ptr);
TM_API int tm_peer_open(const void* ipc_handle, void** peer_ptr);
TM_API int tm_peer_close(void* peer_ptr);
TM_API int64_t tm_peer_flag_bytes(void);
TM_API int tm_peer_signal(void* const* peer_flags, int n_ranks, int rank, void* counters, int slot,
                   void* stream);
TM_API int tm_peer_wait(const void* flags, int n_ranks, void* counters, int slot, void* stream);
TM_API int tm_peer_exchange(void* const* peer_flags, int n_ranks, int rank, const void* flags,
                     void* counters, int slot, void* stream);
TM_API int64_t tm_peer_set_wait_limit(int64_t ns);

/*
 * A6/A11/A12. Row-span copies for the KV slot arena: commit-time append of a
 * chunk's K/V into a slot, compaction on eviction and materialisation of a
 * slot list into a contiguous [B, L, H, D] tensor.
 * Replaces the torch.cat of _cat_cache (kv_cache.py:394-398, 2642-2654) and
 * the per-field slicing of _slice_cache / _slice_tensor
 * (taomate/inference/cache.py:28-56).
 * Each span copies `rows` rows of `row_bytes` bytes (strides in bytes).
 * row_bytes, strides and pointers must be multiples of 16.  Up to 64 spans.
 */
typedef struct {
  const void* src;
  void* dst;
  int64_t rows;
  int64_t src_row_stride;
  int64_t dst_row_stride;
} tm_copy_span;

TM_API int tm_copy_rows(const tm_copy_span* spans, int n_spans, int64_t row_bytes, void* stream);

/*
 * A4/A8/A13. Rank-5 strided copy with a contiguous innermost dimension: the
 * layout permutes around the Ulysses all-to-all (_seq_to_head / _head_to_seq,
 * all_to_all.py:125-173; cp_utils._all_to_all_swap, ltx_causal/parallel/
 * cp_utils.py:272-345) and the SP pad/split (sp_utils.py:25-55).
 * sizes[4] is the contiguous dimension, in elements of elem_bytes; strides in
 * elements.  sizes[4] * elem_bytes must be a multiple of 16.
 */
TM_API int tm_strided_copy5(const void* src, void* dst, const int64_t* sizes,
                     const int64_t* src_strides, const int64_t* dst_strides, int elem_bytes,
                     void* stream);

/*
 * Block elementwise ops around the attention (f4): gated residual update,
 * RMSNorm / LayerNorm and the AdaLN modulation in one pass over each token
 * row.  Replaces, in block_forward_with_cache (ltx_causal/transformer/
 * kv_cache.py:2145-2654):
 *   rms_norm(x) * (1 + scale) + shift   (kv_cache.py:2200-2201, 2514-2525, 2604-2606)
 *   x + out * gate                      (kv_cache.py:2217, 2566, 2579, 2610)
 * with (shift, scale, gate) = table[i] + timestep[..., i, :] from
 * CausalAVTransformerBlock.get_ada_values / get_av_ca_ada_values
 * (ltx_causal/transformer/causal_block.py:434-478), and the LayerNorm +
 * modulation of CausalLTXModel._process_output (causal_model.py:568-598).
 *
 * tm_ada_source: value of parameter p at column c for token row (b, t) =
 *   table[p * D + c] + ts[b * ts_batch_stride + ((t + ts_row_offset) /
 *   ts_row_div) * ts_row_stride + p * D + c]      (either pointer may be NULL).
 * ts_row_div = tokens per frame reads per-frame parameter rows (the
 * reference's per-token expansion, kv_cache.py:2970, is not needed); 1 reads
 * per-token rows.
 *
 * tm_residual_norm, per row (b, t) of [B, L, D] bf16 tensors:
 *   r = x + y * gate[gate_index]   (y NULL: r = x; gate NULL or index < 0: no gate)
 *   x_out = r                      (when x_out is given; may alias x)
 *   n = (r - mean) / sqrt(var + eps)  for norm_kind 1 (LayerNorm, no affine),
 *       r / sqrt(mean(r^2) + eps)      for norm_kind 0 (RMSNorm, no weight),
 *   outs[k] = n * (1 + scale) + shift (scale_index < 0: n), k < n_outs <= 2.
 * fp32 arithmetic, one rounding per stored value; the norm reads the rounded
 * residual.  D a multiple of 256, at most 8192; pointers 16-byte aligned,
 * strides (elements) multiples of 8.
 */
typedef struct {
  const void* table;
  const void* ts;
  int64_t ts_batch_stride, ts_row_stride;
  int32_t ts_row_div, ts_row_offset;
} tm_ada_source;

typedef struct {
  void* out;
  int64_t batch_stride, row_stride;
  tm_ada_source mod;
  int32_t scale_index, shift_index;
} tm_norm_output;

TM_API int tm_residual_norm(const void* x, int64_t x_batch_stride, int64_t x_row_stride,
                     const void* y, int64_t y_batch_stride, int64_t y_row_stride,
                     const tm_ada_source* gate, int gate_index, void* x_out,
                     int64_t x_out_batch_stride, int64_t x_out_row_stride,
                     const tm_norm_output* outs, int n_outs, int norm_kind, int B, int L, int D,
                     float eps, void* stream);

/*
 * In-place tanh-approximate GELU over n bf16 values (n a multiple of 8,
 * 16-byte aligned): the activation of the FFN's first linear, GELUApprox
 * (ltx_causal/transformer/compat.py:40, gelu(proj(x), approximate="tanh")).
 */
TM_API int tm_gelu_tanh(void* x, int64_t n, void* stream);

/*
 * A7. Flash attention of a query chunk over a KV visibility list, on
 * tcgen05 tensor cores (TMA-fed tiles, fp32 accumulators in TMEM, online
 * softmax in registers).  Replaces the cache concat + SDPA of
 * attention_with_cache (kv_cache.py:1486-1531) ->
 * standard_attention_forward (ltx_causal/attention/flex_attention_utils.py:
 * 225-276, F.scaled_dot_product_attention without mask).
 *
 * The visible key set is the ordered list of spans; each span names a source
 * (TM_KV_SOURCE_CACHE: the slot arena k_cache/v_cache; TM_KV_SOURCE_NEW: the
 * chunk's own k_new/v_new) and a row range in it.  The anchor + rolling
 * window + current-chunk visibility is evaluated per key tile in the kernel;
 * no mask and no concatenated K/V are materialised.
 *   q, out: [B, Lq, H, D] bf16.  k_cache, v_cache, k_new, v_new: [B, rows, H, D] bf16.
 *   Heads contiguous (head stride D); batch / row strides in elements,
 *   multiples of 8 (16 bytes).  D in {64, 128}; total visible keys <= 24576.
 */
enum { TM_KV_SOURCE_CACHE = 0, TM_KV_SOURCE_NEW = 1 };

typedef struct {
  int32_t source;
  int32_t row_start;
  int32_t rows;
} tm_kv_span;

TM_API int tm_attention_fwd(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                     const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                     int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                     const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                     int64_t new_rows, const tm_kv_span* spans, int n_spans, void* out,
                     int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H,
                     int D, float scale, void* stream);

/*
 * A7, same contract as tm_attention_fwd plus a caller-owned device workspace.
 * When the query chunk has too few (head, query tile) pairs to occupy every
 * SM (few heads per GPU under sequence parallelism, or a short chunk such as
 * V2A's 25 audio queries against the video keys), the kernel divides each
 * query tile's key tiles into ranges, one CTA each, writes normalised fp32
 * partial outputs with their (max, sum) into the workspace and merges them
 * in a second kernel.  workspace_bytes below what the best partition needs
 * only limits the partition (0 / NULL never splits a key range).  The
 * workspace is 16-byte aligned, not read before it is written, and must not
 * be shared by calls that overlap on the GPU.  Same reference interface as
 * tm_attention_fwd (flex_attention_utils.py:225-276).
 */
TM_API int tm_attention_fwd_ws(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                     const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                     int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                     const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                     int64_t new_rows, const tm_kv_span* spans, int n_spans, void* out,
                     int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H,
                     int D, float scale, void* workspace, int64_t workspace_bytes,
                     void* stream);

/*
 * No counterpart in the reference (torch SDPA allocates its own scratch).
 * Workspace bytes tm_attention_fwd_ws uses for these shapes on the current
 * device (0: no key-range split).  visible_keys = total rows of all spans.
 */
TM_API int64_t tm_attention_workspace_bytes(int B, int Lq, int H, int D, int64_t visible_keys);

/*
 * No counterpart in the reference: describes this library's launch.
 *
 * The work partition tm_attention_fwd / _ws / _noalloc choose for these
 * shapes on the current device, with `workspace_bytes` of workspace and the
 * visible keys in one span (each extra span can add one key tile):
 *   *mode       0: pair CTAs (two 128-row query tiles of a head share every
 *                  key tile), the odd tile of a head in a split CTA;
 *               1: split CTAs (one query tile; the two softmax lanes take
 *                  alternate key tiles), *kv_splits key ranges per query tile
 *                  merged by a second pass when > 1;
 *               2: pair CTAs, the odd tiles of heads h and h + 1 in one CTA
 *                  (one head per softmax lane);
 *   *kv_splits  key ranges per query tile (1 unless mode 1);
 *   *ctas       CTAs that do work (one per SM at a time).
 * Host arithmetic only: no device memory is touched.
 */
TM_API int tm_attention_plan(int B, int Lq, int H, int D, int64_t visible_keys,
                             int64_t workspace_bytes, int* mode, int* kv_splits, int* ctas);

/*
 * Options of tm_attention_fwd_ext (zero-initialise, then set what is used):
 *   device_tiles     key-tile table in device memory (tm_attention_tiles
 *                    layout), as tm_attention_fwd_dev_tiles; NULL: from spans
 *   workspace, _bytes  key-range split scratch, as tm_attention_fwd_ws
 *   rows_per_rank    0: `out` holds all Lq rows.  > 0: the fused head->seq
 *                    exchange of Ulysses parallelism: query row r is stored in
 *                    rank r / rows_per_rank's output buffer at local row
 *                    r % rows_per_rank (at most 8 ranks)
 *   head_base        head index of this call's head 0 within an output row
 *                    (out_row_stride >= (head_base + H) * D)
 *   out_delta[i]     bytes from `out` to rank i's output buffer, mapped into
 *                    this process (tm_peer_open); 0 for this rank
 *   gate_logits      optional [B, Lq, H] bf16 logits (head stride 1, strides in
 *                    elements): each output row of head h is multiplied by
 *                    2 * sigmoid(logit) before it is stored — the per-head gate
 *                    of kv_cache.py:1691-1697 fused into the epilogue
 *   parts, _bytes    export partial results instead of storing `out` (which
 *                    may then be NULL; placement, gate and workspace are
 *                    ignored): the visible keys are divided into part_splits
 *                    ranges, and for each range the normalised fp32 output
 *                    and its (max * log2 scale, sum) go to `parts` in the
 *                    tm_attention_partial_bytes layout.  Several GPUs that
 *                    each attend over their own share of the keys gather
 *                    their parts and merge them with tm_attention_combine.
 *   part_splits      key ranges of an export (1 .. visible key tiles);
 *                    tm_attention_partial_splits suggests one
 * Replaces the attention + head->seq all-to-all of attention_with_cache
 * (kv_cache.py:1531-1538, all_to_all.py:154-173); with `parts`, the
 * attention + both exchanges of V2A under sequence parallelism
 * (kv_cache.py:1432-1462, 1535-1538), where the keys are split by rank.
 */
typedef struct {
  const void* device_tiles;
  void* workspace;
  int64_t workspace_bytes;
  int32_t rows_per_rank;
  int32_t head_base;
  int64_t out_delta[8];
  const void* gate_logits;
  int64_t gate_batch_stride;
  int64_t gate_row_stride;
  void* parts;
  int64_t parts_bytes;
  int32_t part_splits;
  int32_t reserved;
} tm_attention_ext;

/*
 * No counterpart in the reference (it moves the V2A keys, not partial
 * results, between GPUs).
 * Bytes of one export of tm_attention_fwd_ext `parts` with `splits` key
 * ranges: [splits][B][Lq][H][D] fp32 normalised outputs, then, at the next
 * 256-byte boundary, [splits][B][Lq][H] float2 (max * log2 scale, sum).
 */
TM_API int64_t tm_attention_partial_bytes(int B, int Lq, int H, int D, int splits);

/*
 * No counterpart in the reference (as for tm_attention_partial_bytes).
 * Key ranges for an export over `visible_keys` keys that keep every SM busy
 * (the kernel's own work-partition cost model), >= 1.
 */
TM_API int tm_attention_partial_splits(int B, int Lq, int H, int D, int64_t visible_keys);

/*
 * Merge n_groups exports of `splits` key ranges each (group g at byte offset
 * g * group_bytes from `parts`, 16-byte aligned, group_bytes >=
 * tm_attention_partial_bytes) into out [B, Lq, H, D] bf16 (strides in
 * elements, multiples of 8), as one softmax over all their keys; with
 * gate_logits, each row of head h is multiplied by 2 * sigmoid(logit) as in
 * tm_attention_fwd_ext.  The merge order is fixed (group-major), so GPUs
 * that merge the same gathered bytes store the same bits.  Reference
 * interface: the V2A output of kv_cache.py:1531-1538 after its head->seq
 * exchange.
 */
TM_API int tm_attention_combine(const void* parts, int n_groups, int64_t group_bytes, int splits,
                     int B, int Lq, int H, int D, void* out, int64_t out_batch_stride,
                     int64_t out_row_stride, const void* gate_logits, int64_t gate_batch_stride,
                     int64_t gate_row_stride, void* stream);

TM_API int tm_attention_fwd_ext(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                     const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                     int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                     const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                     int64_t new_rows, const tm_kv_span* spans, int n_spans, void* out,
                     int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H,
                     int D, float scale, const tm_attention_ext* ext, void* stream);

/*
 * No counterpart in the reference (it concatenates the cache instead,
 * kv_cache.py:1486-1492).
 * The key-tile list the attention kernel walks for a span list: n_tiles pairs
 * (source << 30 | first row, valid rows), 64 keys per tile, in span order.
 * Validates the spans as tm_attention_fwd does.  Used to refresh the device
 * tile table of tm_attention_fwd_dev_tiles between CUDA-graph replays.
 */
TM_API int tm_attention_tiles(const tm_kv_span* spans, int n_spans, int64_t cache_rows,
                     int64_t new_rows, int32_t* tiles_out, int max_tiles, int* n_tiles);

/*
 * tm_attention_fwd_ws whose kernel reads its key-tile list from device memory
 * (device_tiles, 16-byte aligned, in the tm_attention_tiles layout) instead of
 * from its launch parameters.  `spans` fixes the tile count and the work
 * partition at launch; the table may be rewritten before each replay of a
 * captured graph as long as it keeps that tile count and each tile's source
 * (both sources' pointers, when given, stay mapped).  Same reference
 * interface as tm_attention_fwd (flex_attention_utils.py:225-276): it replaces
 * the per-block cache concat of attention_with_cache (kv_cache.py:1486-1492)
 * in a replayed forward.
 */
TM_API int tm_attention_fwd_dev_tiles(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                     const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                     int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                     const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                     int64_t new_rows, const tm_kv_span* spans, int n_spans,
                     const void* device_tiles, void* out, int64_t out_batch_stride,
                     int64_t out_row_stride, int B, int Lq, int H, int D, float scale,
                     void* workspace, int64_t workspace_bytes, void* stream);

/*
 * No counterpart in the reference: an addition of this library.
 *
 * tm_attention_fwd_ws for callers that cannot allocate device memory: a
 * host program that embeds this library in a runtime owning every byte of
 * the GPU (memory reserved up front, no allocator offered to plugins), or a
 * latency-critical path where cudaMalloc's implicit synchronisation is not
 * allowed.  The caller still passes q, K/V and out; the key-range split's
 * scratch is a fixed 16 MiB array in the library's own device memory, which
 * every GPU that loads the library keeps until the process exits.  Shapes
 * whose split needs more are rejected with TM_ERR_INVALID_ARGUMENT before
 * anything is launched (the need is that of the partition the launch would
 * choose; for one span it equals tm_attention_workspace_bytes).
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other threads) race on it.  Serialise them.
 *   - Nothing has to be cleared between calls: each call writes every
 *     scratch row it reads.
 */
TM_API int tm_attention_fwd_noalloc(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                     const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                     int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                     const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                     int64_t new_rows, const tm_kv_span* spans, int n_spans, void* out,
                     int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H,
                     int D, float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TAOMATE_B200_H */
