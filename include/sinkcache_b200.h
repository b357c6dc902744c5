/*
 * sinkcache_b200.h -- C ABI of the B200 (sm_100a) attention-sink KV-cache decode path.
 *
 * The library replaces the GPU work of the sinkcache package (buttaRahul/Attention_sinks):
 *   - the per-layer append of new K/V rows     (src/sinkcache/cache.py:159-160)
 *   - the in-place eviction + RoPE re-rotation (src/sinkcache/kernels.py:24-73, cache.py:129-147)
 *   - split-K GQA decode attention             (src/sinkcache/decode_attention.py:29-130)
 *   - and a fused decode step doing all three in one pass over the cache.
 *
 * Conventions
 *   - Every tensor is described by plain pointers, sizes and element strides.  The last
 *     dimension (head_dim) is always contiguous.  Cache buffers additionally need their
 *     rows (slots) contiguous: stride between slots == head_dim.
 *   - Cache buffers are [batch, heads_kv, slots, head_dim] (the layout SinkLayer._alloc
 *     creates, cache.py:97-104): K in k_dtype (float32 by default), V in the model dtype.
 *   - All launches go to `stream` (a cudaStream_t passed as void*); nothing synchronises,
 *     nothing allocates.  Scratch memory ("workspace") is owned by the caller; its size
 *     comes from sink_workspace_bytes().  Every launch is CUDA-graph capturable.
 *   - Return value: 0 on success, a negative SINK_E* code for a rejected argument, or a
 *     positive cudaError_t from the launch.  sink_strerror() describes any code.
 *   - The device workspace starts with a 256-byte header holding a 32-bit status word, zero
 *     when the workspace is first used.  A kernel whose bounded wait for a bulk copy runs
 *     out sets a SINK_STATUS_* bit there instead of hanging; sink_read_status() returns and
 *     clears it.
 */
#ifndef SINKCACHE_B200_H
#define SINKCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SINK_ABI_VERSION 1

/* element types */
#define SINK_DTYPE_F32 0
#define SINK_DTYPE_BF16 1
#define SINK_DTYPE_F16 2

/* argument errors (negative return codes) */
#define SINK_OK 0
#define SINK_EINVAL (-1)      /* a size or index out of range */
#define SINK_EDTYPE (-2)      /* unsupported dtype combination */
#define SINK_EHEADDIM (-3)    /* head_dim not in {64, 128, 256} */
#define SINK_EGROUP (-4)      /* heads_q / heads_kv not an integer in [1, 8] */
#define SINK_ELAYOUT (-5)     /* slots not contiguous, or a pointer not 16-byte aligned */
#define SINK_EWORKSPACE (-6)  /* workspace missing or smaller than sink_workspace_bytes() */
#define SINK_EDEVICE (-7)     /* no usable CUDA device */
#define SINK_ESCRATCH (-8)    /* needs more than the static scratch of sink_decode_attention_noalloc */

/* status bits written by kernels into the workspace status word */
#define SINK_STATUS_WAIT_TIMEOUT 1

/* operations, for sink_workspace_bytes() */
#define SINK_OP_APPEND 0
#define SINK_OP_EVICT 1
#define SINK_OP_ATTEND 2
#define SINK_OP_FUSED_STEP 3

/* One layer's K/V cache buffers: [batch, heads_kv, slots, head_dim] each. */
typedef struct sink_kv_buffers {
  void* k;
  void* v;
  int32_t k_dtype;
  int32_t v_dtype;
  int32_t batch;
  int32_t heads_kv;
  int32_t slots;     /* allocated rows per (batch, head) */
  int32_t head_dim;
  int64_t k_stride_b; /* element strides of the batch and head dimensions */
  int64_t k_stride_h;
  int64_t v_stride_b;
  int64_t v_stride_h;
} sink_kv_buffers_t;

/* A [batch, heads, n, head_dim] tensor with a unit last stride (k/v of a new chunk, q, out). */
typedef struct sink_rows {
  void* data;
  int32_t dtype;
  int32_t heads;
  int32_t n;
  int32_t pad_;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
} sink_rows_t;

/* Library ABI version (SINK_ABI_VERSION). */
int32_t sink_abi_version(void);

/*
 * Kernel launches this library has issued in the calling process so far (every successful
 * launch of every entry point; replays of a CUDA graph that captured them are not counted).
 * For benchmarks and tests: the difference across a region is the number of this library's
 * kernels launched inside it.  No counterpart in the reference.
 */
uint64_t sink_launch_count(void);

/* Human-readable text for any return code of this library (negative or cudaError_t). */
const char* sink_strerror(int32_t code);

/*
 * Bytes of device workspace that `op` needs for these shapes (0 if none).  `num_sms` is the
 * device's multiprocessor count (cudaDevAttrMultiProcessorCount); the launch uses the same
 * count, so size the workspace for the device it will run on.  `rows` is the number of
 * attended cache rows for SINK_OP_ATTEND and SINK_OP_FUSED_STEP (after the append).
 * Pure host arithmetic: callable without a GPU.
 */
size_t sink_workspace_bytes(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q,
                            int32_t head_dim, int32_t k_dtype, int32_t v_dtype, int32_t rows,
                            int32_t n_sink, int32_t window, int32_t drop, int32_t num_sms);

/*
 * Split plan the launch will use (for tests and profiling): number of splits per
 * (batch, head) pair, rows per split, rows per pipeline chunk, pipeline stages, dynamic
 * shared memory per CTA, and CTAs per thread-block cluster (`splits` when every split of a
 * pair runs in one cluster and the step is a single launch, else 1).  Pure host
 * arithmetic.  Returns 0 or SINK_E*.
 */
int32_t sink_plan(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q, int32_t head_dim,
                  int32_t k_dtype, int32_t v_dtype, int32_t rows, int32_t n_sink, int32_t window,
                  int32_t drop, int32_t num_sms, int32_t* splits, int32_t* rows_per_split,
                  int32_t* chunk_rows, int32_t* stages, int32_t* smem_bytes,
                  int32_t* cluster_ctas);

/* launch modes reported by sink_plan_launch() */
#define SINK_LAUNCH_SPLIT 0      /* one CTA per split; halo pre-pass and combine launches as needed */
#define SINK_LAUNCH_CLUSTER 1    /* every split of a pair in one thread-block cluster: one launch */
#define SINK_LAUNCH_TENSOR 2     /* the tensor-core attention kernel (16-bit K, head_dim 128) */

/*
 * How the plan of sink_plan() is launched (for tests and profiling): *mode is one of
 * SINK_LAUNCH_*, *ctas the CTAs of the main kernel's grid (the tensor-core launch is
 * persistent: one CTA per SM at most).  Same arguments as sink_plan; pure host arithmetic.
 * No counterpart in the reference.  Returns 0 or SINK_E*.
 */
int32_t sink_plan_launch(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q,
                         int32_t head_dim, int32_t k_dtype, int32_t v_dtype, int32_t rows,
                         int32_t n_sink, int32_t window, int32_t drop, int32_t num_sms,
                         int32_t* mode, int32_t* ctas);

/*
 * Append: kv[:, :, row:row+n] = (k_new, v_new)  (k converted to k_dtype exactly, or rounded
 * to nearest-even when k_dtype is narrower).
 * Replaces SinkLayer.update's `self._kbuf[:, :, self.length:end].copy_(key_states)` and the
 * matching V copy (cache.py:159-160).  k_new/v_new: model dtype == kv->v_dtype, n rows.
 */
int32_t sink_append(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                    const sink_rows_t* v_new, int32_t row, void* stream);

/*
 * Eviction with re-rotation, in place, for every (batch, head):
 *   K[s : s+W] = rope(K[s+drop : s+drop+W], -drop)   (fp32 math, one rounding to k_dtype)
 *   V[s : s+W] = V[s+drop : s+drop+W]
 * with s = n_sink, W = window.  cos/sin are the float32 [head_dim] tables for the angle -drop
 * (rope_cos_sin(-drop, inv_freq), HF half-split layout, both halves equal); ignored when
 * rotate == 0 (shift only: the rerotate_keys=False ablation).  Rows [0, s) are untouched.
 * Needs s + W + drop <= slots.  drop == 0 is a no-op.
 * Replaces shift_window_ (kernels.py:59-73) as called by SinkLayer._evict_pending
 * (cache.py:134-137), and the PyTorch branch of the same method (cache.py:138-143).
 */
int32_t sink_evict_rerotate(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                            int32_t drop, const float* cos_tab, const float* sin_tab,
                            int32_t rotate, void* workspace, size_t workspace_bytes,
                            void* stream);

/*
 * sink_evict_rerotate that also writes every window row's final key, rounded to the value
 * type, into k_copy rows [n_sink, n_sink + window) (k_copy: [batch, heads_kv, >= n_sink +
 * window, head_dim] in v_dtype, rows contiguous and 16-byte aligned) -- in the same pass over
 * the cache.  With drop == 0 nothing moves and the launch only writes the copy.
 * Replaces, for a multi-token step, the model-dtype key copy SinkLayer.update returns
 * (`self._kbuf[:, :, :end].to(self.dtype)`, cache.py:163) for the window rows: the copy no
 * longer costs a separate read of the float32 keys.  The caller copies the sink rows and the
 * appended rows itself.
 */
int32_t sink_evict_rerotate_keycopy(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                                    int32_t drop, const float* cos_tab, const float* sin_tab,
                                    int32_t rotate, const sink_rows_t* k_copy, void* workspace,
                                    size_t workspace_bytes, void* stream);

/*
 * Decode attention for one query token per sequence over the first `rows` cache rows:
 *   out[b, 0, hq, :] = softmax(q[b, hq] . K[b, hq / G, :rows]^T * scale) @ V[b, hq / G, :rows]
 * with G = q->heads / heads_kv (grouped-query attention, HF repeat_kv head order).
 * q: [batch, heads_q, 1, head_dim] in the model dtype; out: [batch, 1, heads_q, head_dim]
 * in the model dtype, given by pointer and its batch / head element strides.
 * K may be float32 (read directly, no bf16 copy) or the model dtype.
 * `mask` (optional, may be NULL): one byte per (batch, row), row r attended iff nonzero,
 * rows contiguous, batch stride `mask_stride_b` bytes (0 to share one row across the batch)
 * -- the boolean [B, 1, 1, rows] mask an SDPA-style backend receives for a one-token query.
 * Replaces flash_decode (decode_attention.py:102-130): split-K partials + a combine pass.
 */
int32_t sink_decode_attention(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows,
                              float scale, const uint8_t* mask, int64_t mask_stride_b,
                              void* out, int64_t out_stride_b, int64_t out_stride_h,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * One fused decode step of a sink layer, q_len == 1:
 *   1. pending eviction of `drop` rows with re-rotation (as sink_evict_rerotate; drop may be 0)
 *   2. append of (k_new, v_new) at row `append_row` (== n_sink + window when drop > 0)
 *   3. decode attention of q over rows [0, append_row] of the updated cache
 * in one pass over the cache: every window row is read once, re-rotated in registers,
 * written back once and consumed by the attention in the same CTA.  `mask` as for
 * sink_decode_attention, over rows [0, append_row] (masked rows are still evicted and
 * re-rotated; they only drop out of the attention).
 * Replaces SinkLayer.update (cache.py:151-165) followed by decode_attention_forward
 * (decode_attention.py:136-143) for a one-token step; the cache contents afterwards are
 * those SinkLayer.update leaves, without the bf16 key copy of cache.py:163.
 */
int32_t sink_fused_decode_step(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                               const sink_rows_t* v_new, const sink_rows_t* q,
                               int32_t n_sink, int32_t window, int32_t drop,
                               int32_t append_row, const float* cos_tab, const float* sin_tab,
                               int32_t rotate, float scale, const uint8_t* mask,
                               int64_t mask_stride_b, void* out, int64_t out_stride_b,
                               int64_t out_stride_h, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Copy the workspace status word to *status (synchronises `stream`) and clear it. */
int32_t sink_read_status(void* workspace, void* stream, int32_t* status);

/*
 * One-time set-up of the current device: opts the kernels into their shared-memory sizes
 * and cluster sizes, asks the device how many clusters of the tensor-core attention kernel
 * it holds at once (which decides, at launch, whether a split attention merges its
 * partials inside clusters), and looks up the driver's tensor-map encoder.  These calls
 * cannot be made inside a CUDA
 * stream capture, so call this once per device before capturing any launch of this
 * library into a graph (every entry point also runs it on its first use).  No counterpart
 * in the reference (its Triton kernels compile on first use instead).
 */
int32_t sink_prepare_device(void);

/*
 * Ring-buffer cache (SinkLayerV2, src/sinkcache/cache_v2.py:59-248).  Window keys stay at the
 * rotation the model gave them (absolute positions); only the region -- the sinks and any
 * pinned tokens -- is re-rotated, from stored originals, to sit just before the window.
 * The layer's buffers are a ring of window + 1 slots followed by the region slots:
 *   kv: [batch, heads_kv, window + 1 + region_cap, head_dim], K and V in the model dtype
 * (k_dtype == v_dtype).  The token at absolute position p >= n_sink sits in ring slot
 * (p - n_sink) mod (window + 1).
 *
 * Place step:
 *   - (k_new, v_new) [batch, heads_kv, 1, head_dim], optional (both or neither): written to
 *     ring slot (t - n_sink) mod (window + 1);
 *   - region_keys [batch, heads_kv, >= R, head_dim], rows 0..R-1 at their original rotations,
 *     region_pos (device int64 [>= R]) their original positions: row j is rotated to
 *     position ws - R + j, ws = max(min(t, n_sink), t - window), into region_out rows
 *     0..R-1 (NULL: the kv rows window+1 .. window+R).  Angles in fp64, cos/sin rounded to
 *     fp32, fp32 math, one rounding to k_dtype; inv_freq (device fp64 [rot_half]) covers the
 *     first 2 * rot_half dims (HF half-split layout), the rest pass through;
 *   - position (optional): device int64[2] = {t, 0}.  t is read on the device and advanced
 *     by one when the step ends, so a CUDA graph of the step serves every later token; the
 *     second word is an arrival counter that must be 0 between calls.  NULL: t = t_host,
 *     nothing advanced.
 * Replaces the device work of SinkLayerV2._decode_step (cache_v2.py:171-176: the slot
 * index_copy_, the region copy of _rotate_region (:101-116) and _t_dev.add_(1)), and
 * _rotate_region alone (region_out, no new token) for _general_step / kept() (:192, :234).
 */
int32_t sink_v2_place(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                      const sink_rows_t* v_new, const sink_rows_t* region_keys,
                      const int64_t* region_pos, int32_t region_len,
                      const sink_rows_t* region_out, int64_t* position, int64_t t_host,
                      int32_t n_sink, int32_t window, const double* inv_freq,
                      int32_t rot_half, void* stream);

/*
 * One steady-state decode step of a ring-buffer layer fused with its attention: the place
 * step with (k_new, v_new) and `position`, then decode attention of q [batch, heads_q, 1,
 * head_dim] over the window + 1 + R rows (ring, then region) -- as sink_decode_attention,
 * with its mask convention over those rows.  Workspace: sink_workspace_bytes(SINK_OP_ATTEND,
 * ..., rows = window + 1 + R, ...).  On the tensor-core path (16-bit K and V, head_dim 128)
 * the place work runs inside the attention kernel, in two warps of each CTA on the rows of
 * its own split items while the pipeline loads the other chunks, so the step is one launch
 * (plus the split combine when the splits do not merge inside their clusters); otherwise
 * the place kernel runs first.  Replaces SinkLayerV2._decode_step (cache_v2.py:167-181)
 * followed by decode_attention_forward over the views it returns (decode_attention.py:136-143).
 */
int32_t sink_v2_decode_step(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                            const sink_rows_t* v_new, const sink_rows_t* region_keys,
                            const int64_t* region_pos, int32_t region_len, int64_t* position,
                            int32_t n_sink, int32_t window, const double* inv_freq,
                            int32_t rot_half, const sink_rows_t* q, float scale,
                            const uint8_t* mask, int64_t mask_stride_b, void* out,
                            int64_t out_stride_b, int64_t out_stride_h, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Failure-detection test hook; no counterpart in the reference (which records only
 * out-of-memory failures).  Arms the NEXT launch of the stream kernel in this process -- the
 * kernel behind sink_evict_rerotate, sink_fused_decode_step, and sink_decode_attention over
 * float32 keys or head_dim 64/256 -- so that every CTA leaves its row chunk `chunk` (0 = the
 * first of its split) unissued: no copy and no arrival, so the wait for that chunk runs
 * out after `polls` polls (each of that launch's waits is bounded by `polls`).  The CTAs then
 * wait for the copies they did issue, store nothing further, and set
 * SINK_STATUS_WAIT_TIMEOUT in the workspace status word; the context stays usable.  CTAs
 * whose split has no chunk `chunk` run normally.  A launch that fails this way leaves an
 * in-place eviction partly applied, so the caller restores the buffers (a read-only
 * attention leaves them untouched).  Returns 0, or SINK_EINVAL for chunk < 0 or polls < 1.
 */
int32_t sink_debug_fail_next_wait(int32_t chunk, int32_t polls);

/*
 * Test hook for the cluster fallback: clusters >= 0 is taken as the number of clusters the
 * device can hold at once for every clustered stream launch of the process (a clustered plan
 * needs one per (batch, head) pair in one wave; with fewer -- 0: none can be placed -- it runs
 * as the split launch: halo pre-pass, stream kernel, combine, with the same splits); -1 (the
 * default) asks the device (cudaOccupancyMaxActiveClusters, once per kernel and cluster size,
 * outside stream capture).  Launches nothing.  Returns 0, or SINK_EINVAL for clusters < -1.
 */
int32_t sink_debug_cluster_capacity(int32_t clusters);

/*
 * The rows a ring-buffer layer's multi-token step attends over, in the reference's order
 * [region (R rows), window by position, chunk (n rows)], gathered into out_k / out_v
 * ([batch, heads_kv, >= R + (hi - lo) + n, head_dim], rows 16-byte aligned):
 *   - rows [0, R): out_v gets the region's value rows (kv rows window + 1 ..); out_k is left
 *     for sink_v2_place with region_out = those rows (the rotated region keys);
 *   - rows [R, R + hi - lo): positions lo .. hi - 1 (>= n_sink, at most window + 1 of them)
 *     from their ring slots (p - n_sink) mod (window + 1);
 *   - the rest: the chunk's rows k_new / v_new (both or neither).
 * kv: K and V in the model dtype.  16-byte copies, one launch for both tensors.
 * Replaces the index_select / cat gathers of SinkLayerV2._general_step and kept()
 * (src/sinkcache/cache_v2.py:189-193, 229-234).
 */
int32_t sink_v2_gather(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                       int32_t region_len, int64_t lo, int64_t hi, const sink_rows_t* k_new,
                       const sink_rows_t* v_new, const sink_rows_t* out_k, const sink_rows_t* out_v,
                       void* stream);

/* Size of the static device scratch behind sink_decode_attention_noalloc: 16 MiB. */
#define SINK_NOALLOC_SCRATCH_BYTES (16u << 20)

/*
 * sink_decode_attention without a caller-provided workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory -- a binding from a
 * foreign runtime that has no device allocator of its own (a C or FFI host outside
 * PyTorch), or a decode loop that must not call cudaMalloc / cudaFree because those
 * synchronise the device and stall the stream.  Same arguments and results as
 * sink_decode_attention minus the workspace; the split partials live instead in a
 * file-scope 16 MiB device array (SINK_NOALLOC_SCRATCH_BYTES) that every GPU which loads
 * the library holds until the process exits (on a B200 it holds, e.g., 16 streams of a
 * 32K-slot Qwen3 layer).
 *   - Each device's copy of the array is looked up once (cudaGetSymbolAddress, with the
 *     device current) by sink_prepare_device(), or else by the first call on that device;
 *     either must happen before any stream capture.
 *   - The arguments are checked exactly as sink_decode_attention checks them (same error
 *     codes, nothing launched); then a request whose scratch
 *     (sink_workspace_bytes(SINK_OP_ATTEND, ...)) exceeds the array returns SINK_ESCRATCH
 *     and launches nothing.
 *   - All calls share the one array and each call leaves its partials there: calls that can
 *     overlap on the GPU (different streams, different host threads) race and must be
 *     serialised by the caller.  Each call clears the array's status word first; the
 *     bounded-wait status is not reported through this entry point.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
int32_t sink_decode_attention_noalloc(const sink_rows_t* q, const sink_kv_buffers_t* kv,
                                      int32_t rows, float scale, const uint8_t* mask,
                                      int64_t mask_stride_b, void* out, int64_t out_stride_b,
                                      int64_t out_stride_h, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SINKCACHE_B200_H */
