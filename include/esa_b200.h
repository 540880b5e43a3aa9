/*
 * esa_b200.h -- C ABI of the B200-native elastic sparse attention library
 * (libesa_b200.so).  Plain pointers and sizes only; every buffer is device
 * memory owned by the caller; no entry point allocates device memory.  All
 * launches go to the stream passed in (a cudaStream_t, NULL = legacy default
 * stream) and are asynchronous.  Functions return ESA_OK (0) or a negative
 * code; esa_last_error() gives the message of the last failure on the
 * calling thread.
 *
 * Tensor convention: an attention operand of logical shape [B, H, L, D] is
 * described by esa_tensor_t {data, stride_b, stride_h, stride_s} with strides
 * in elements and the D axis contiguous.  Base pointers and the three strides
 * (times the element size) must be multiples of 16 bytes.
 *
 * Reference interfaces replaced (HighCWu/elastic-sparse-attention,
 * elastic_sparse_attention.py):
 *   esa_pattern          _create_elastic_sparse_indices          :470-535
 *                        + _get_prepared_indices_and_mask slicing :574-590, :600-615
 *   esa_forward          ElasticSparseAttentionFunction.forward  :241-297
 *                        (Triton kernel, IS_BWD=False            :117-166)
 *   esa_backward         ElasticSparseAttentionFunction.backward :300-339
 *                        (Triton kernel, IS_BWD=True             :169-233)
 */
#ifndef ESA_B200_H
#define ESA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ESA_OK 0
#define ESA_ERR_INVALID (-1)     /* bad argument, shape, stride or alignment */
#define ESA_ERR_UNSUPPORTED (-2) /* dtype / head_dim combination not built */
#define ESA_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define ESA_ERR_WORKSPACE (-4)   /* workspace smaller than esa_backward_workspace_size */

typedef enum {
  ESA_DTYPE_F32 = 0,
  ESA_DTYPE_BF16 = 1,
  ESA_DTYPE_F16 = 2
} esa_dtype_t;

typedef struct {
  void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_s;
} esa_tensor_t;

/*
 * One attention call.  Mirrors the reference module's arguments:
 *   num_heads / num_kv_heads / head_dim / attention_length / layer_idx /
 *   num_hidden_layers  -- ElasticSparseAttention.__init__ (:375-386)
 *   q_len, kv_len      -- query_states.shape[2], key_states.shape[2]
 *   rows               -- cache_position (:602-608) as device int64 [q_len],
 *                         or NULL: query row j is position row_offset + j
 *                         (the reference slices rows [:q_len], i.e. offset 0).
 *                         esa_forward reads a negative entry as kv_len + entry
 *                         (torch indexing of the reference's [:kv_len] slice,
 *                         :607-608); an entry outside [-kv_len, kv_len) gets
 *                         an output row of zeros and sets
 *                         ESA_DEVERR_QUERY_RANGE (no host round trip checks
 *                         it).  esa_backward expects entries in [0, kv_len).
 *   kv_offset, kv_rows -- the k/v (and dk/dv) buffers hold positions
 *                         [kv_offset, kv_offset + kv_rows); for a plain call
 *                         kv_offset = 0 and kv_rows = kv_len
 *   scale              -- softmax scale, the reference uses head_dim ** -0.5
 *   dropout_p          -- probability of dropping a softmax weight (the
 *                         reference's naive/dense paths in training, :674,
 *                         :721); 0 disables.  The keep mask is a function of
 *                         (dropout_seed, batch, head, position, slot), so the
 *                         backward reproduces it from the same problem.
 *   weights            -- optional output of esa_forward: the softmax weights
 *                         after dropout, input dtype, contiguous
 *                         [B, num_heads, q_len, attn_length] (the reference's
 *                         naive attn_weights, :673-680); NULL = not written
 *   probs              -- optional float32 [B, num_heads, attn_length, q_len]
 *                         (slot-major, contiguous, 16-byte aligned): when
 *                         esa_forward_writes_probs(problem) is 1, esa_forward
 *                         writes the normalised softmax probabilities there
 *                         and esa_backward, given the same buffer, reads them
 *                         instead of recomputing the scores (one gather pass
 *                         less).  NULL = the backward recomputes them.
 *   head_offset,       -- the call's num_heads query heads are heads
 *   pattern_heads         [head_offset, head_offset + num_heads) of a layer
 *                         whose pattern is defined over pattern_heads query
 *                         heads (the module's num_attention_heads, :375-386;
 *                         the head weight is t = (head_offset + h) /
 *                         (pattern_heads - 1), :515-516).  0 / 0 = the call
 *                         holds every head.  This lets a caller split one
 *                         layer's heads over GPUs or launches; num_kv_heads
 *                         are then the K/V heads of those query heads.
 *   key_plan,          -- optional device buffer filled by esa_key_plan_build
 *   key_plan_bytes        for this problem (same pattern, shapes and offsets;
 *                         key_plan_bytes = esa_key_plan_size(problem)): the
 *                         backward's key side then reads its precomputed user
 *                         lists instead of searching the pattern.  NULL / 0 =
 *                         no plan.  A plan built for another problem is
 *                         rejected (ESA_ERR_INVALID when its size differs,
 *                         else ESA_DEVERR_PLAN and dk / dv left unwritten).
 */
typedef struct {
  int32_t dtype;
  int32_t batch;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t attn_length;
  int32_t layer_idx;
  int32_t num_hidden_layers;
  int64_t q_len;
  int64_t kv_len;
  int64_t kv_offset;
  int64_t kv_rows;
  int64_t row_offset;
  const int64_t* rows;
  float scale;
  int32_t flags;   /* ESA_FLAG_* bits, 0 by default */
  float dropout_p;
  int32_t head_offset;
  uint64_t dropout_seed;
  void* weights;
  void* probs;
  int32_t pattern_heads;
  int32_t reserved;   /* 0 */
  const void* key_plan;
  uint64_t key_plan_bytes;
} esa_problem_t;

/* flags: run every layer on the CUDA-core gather kernels, also where the
 * tensor-core sliding-window kernel would apply (for cross-checking paths). */
#define ESA_FLAG_GATHER_ONLY 1
/* flags: esa_backward writes dk and dv as float32 (their esa_tensor_t strides
 * in float elements) whatever the input dtype: the unrounded sums, for a
 * caller that adds partial key gradients of several calls (the sequence
 * split adds the partial dK / dV that other ranks' queries produce for its
 * keys) and rounds once. */
#define ESA_FLAG_F32_DKV 2

/* Bits of the per-device error word that kernels set instead of faulting
 * (read and reset with esa_device_errors). */
#define ESA_DEVERR_KV_RANGE 1     /* a computed key row fell outside the k/v buffer
                                     (kv_offset / kv_rows too small); masked */
#define ESA_DEVERR_TIMEOUT 2      /* a bounded wait of the tensor-core kernel gave
                                     up; its tile was not written */
#define ESA_DEVERR_QUERY_RANGE 4  /* a rows[] entry outside [-kv_len, kv_len);
                                     its output row is zero */
#define ESA_DEVERR_PLAN 8         /* esa_backward was given a key plan built for
                                     another problem; dk / dv not written */

/* Library version, e.g. 130 for 0.1.3 (110 added head_offset / pattern_heads
 * to esa_problem_t, the launch trace and the gather probe; 120 the key plan:
 * key_plan / key_plan_bytes in esa_problem_t, esa_key_plan_size / _build;
 * 130 esa_copy_rows). */
int esa_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* esa_last_error(void);

/*
 * 1 if esa_forward, for this problem, runs the kernel that writes `probs`
 * (and esa_backward can use them), 0 if not, negative on an invalid problem.
 * No reference counterpart: the reference recomputes the scores in its
 * backward (:169-233) from the saved row statistics L and M.
 */
int esa_forward_writes_probs(const esa_problem_t* problem);

/*
 * Error bits (ESA_DEVERR_*) recorded by kernels on the current device since
 * the last reset, as of the work queued on `stream` so far: copies the word
 * to *flags after that work, resets it when clear != 0, and synchronises
 * `stream`.  The reference has no counterpart (its kernels have no error
 * channel; an out-of-range cache_position there is an indexing failure).
 */
int esa_device_errors(int32_t clear, int32_t* flags, void* stream);

/*
 * Pattern buffers, bit-exact with the reference: idx/mask int64 [H, n_rows, w]
 * for the query positions rows[r] (device int64, or row_offset + r when rows
 * is NULL).  clamp_len > 0 clamps indices to [0, clamp_len - 1] as
 * _triton_forward does (:615); clamp_len <= 0 gives the raw module buffers
 * sparse_attention_indices / sparse_causal_mask (:465-468, :532-535).
 * Replaces _create_elastic_sparse_indices (:470-535).
 */
int esa_pattern(int32_t num_heads, int32_t attn_length, int32_t layer_idx,
                int32_t num_hidden_layers, int64_t n_rows, const int64_t* rows,
                int64_t row_offset, int64_t clamp_len, int64_t* idx, int64_t* mask,
                void* stream);

/*
 * Counts (head, row, slot) where the raw slot index decreases from query
 * position r - 1 to r, r < seq_len, and adds the count to *d_count (device
 * uint64, caller zeroes it).  Zero is the precondition of esa_backward's
 * key-side enumeration; the library's Python module checks it once per
 * pattern.  No reference counterpart (the reference backward uses atomics).
 */
int esa_pattern_audit(int32_t num_heads, int32_t attn_length, int32_t layer_idx,
                      int32_t num_hidden_layers, int64_t seq_len,
                      unsigned long long* d_count, void* stream);

/*
 * Forward.  q [B, Hq, q_len, D], k/v [B, Hkv, kv_rows, D], o [B, Hq, q_len, D]
 * (any strides per the tensor convention; the Python module passes an o laid
 * out as [B, q_len, Hq, D] so that its final reshape is free), lse float32
 * [B, Hq, q_len] contiguous: base-2 log-sum-exp of the scaled scores
 * (replaces the reference's separate L and M outputs, :255-257, :165-166).
 * Replaces ElasticSparseAttentionFunction.forward (:241-297).
 */
int esa_forward(const esa_problem_t* prob, esa_tensor_t q, esa_tensor_t k, esa_tensor_t v,
                esa_tensor_t o, float* lse, void* stream);

/* Bytes of workspace esa_backward needs for this problem. */
size_t esa_backward_workspace_size(const esa_problem_t* prob);

/*
 * Key plan (no reference counterpart: the reference keeps its index buffers
 * [H, max_seq_len, w] from construction, :454-468; this is the transposed,
 * key-ordered form the backward's key side needs).  It depends only on the
 * pattern, shapes and offsets of the problem (not on batch size or data), so
 * a caller builds it once and passes it (problem.key_plan) to every backward
 * of that layer.
 *   esa_key_plan_size   bytes of the plan; 0 when this problem's key side
 *                       takes no plan (sliding-window layers, fp32, head_dim
 *                       other than 64 / 128, explicit rows, more than 2^23
 *                       query rows)
 *   esa_key_plan_build  fills a device buffer of that size (256-byte aligned)
 *                       on `stream`
 */
size_t esa_key_plan_size(const esa_problem_t* prob);
int esa_key_plan_build(const esa_problem_t* prob, void* plan, size_t plan_bytes, void* stream);

/*
 * Backward.  Takes the forward's o and lse and the upstream gradient dout
 * (all [B, Hq, q_len, D]); writes dq [B, Hq, q_len, D] and dk/dv
 * [B, Hkv, kv_rows, D], fully (no zero-initialisation needed, no atomics).
 * When rows != NULL the key side needs the positions sorted ascending:
 * pass sorted_rows (device int64 [q_len], ascending) and row_perm (device
 * int64 [q_len], sorted slot -> query row), or NULL for both when rows is
 * already sorted.  workspace: device memory of esa_backward_workspace_size()
 * bytes, 256-byte aligned.
 * Replaces ElasticSparseAttentionFunction.backward (:300-339).
 */
int esa_backward(const esa_problem_t* prob, esa_tensor_t q, esa_tensor_t k, esa_tensor_t v,
                 esa_tensor_t o, const float* lse, esa_tensor_t dout, esa_tensor_t dq,
                 esa_tensor_t dk, esa_tensor_t dv, const int64_t* sorted_rows,
                 const int64_t* row_perm, void* workspace, size_t workspace_bytes,
                 void* stream);

/*
 * Launch trace (measurement aid; no reference counterpart).  While enabled,
 * every kernel the library launches is bracketed by two CUDA events recorded
 * on its stream, so a caller can attribute device time to the library's
 * kernels without a profiler.  esa_trace_enable(1) clears the records and
 * starts recording, esa_trace_enable(0) stops (records are kept);
 * esa_trace_count() is the number of records; esa_trace_read(i, &name, &ms)
 * waits for record i and gives its kernel's name and elapsed milliseconds.
 * Recording creates CUDA events (no device memory) and is off by default.
 */
int esa_trace_enable(int32_t on);
int esa_trace_count(void);
int esa_trace_read(int32_t i, const char** name, float* ms);

/*
 * Gather probe (measurement aid; no reference counterpart): loads, without
 * arithmetic, the K and V rows the slot-major tile forward would read for
 * `prob` (16-bit data, head_dim 64 / 128, w <= 64; same grid, same order),
 * B * num_heads * q_len * attn_length rows of each, and folds them into an
 * xor checksum written to *sink (device uint32) only if it equals a fixed
 * improbable value, so that the loads are not optimised away.  mode:
 *   ESA_PROBE_PATTERN    the elastic pattern's rows (the tile kernels' stream)
 *   ESA_PROBE_L2_RANDOM  the same number of rows, uniformly random over the
 *                        KV head's kv_rows (one KV head at a time: L2-resident)
 *   ESA_PROBE_L1_WINDOW  the same number of rows, random within 64 rows per
 *                        CTA (K and V: 32 KB at D = 128, L1-resident)
 *   ESA_PROBE_L2_STREAM  the same number of rows, each pair's slots reading
 *                        consecutive rows and no row read twice by a CTA
 *                        (runs of rows from L2 with no L1 reuse, the access
 *                        pattern of the key side's user rows)
 * The elapsed time gives the achievable row-gather bandwidth of each level.
 */
#define ESA_PROBE_PATTERN 0
#define ESA_PROBE_L2_RANDOM 1
#define ESA_PROBE_L1_WINDOW 2
#define ESA_PROBE_L2_STREAM 3
int esa_probe_gather(int32_t mode, const esa_problem_t* prob, esa_tensor_t k, esa_tensor_t v,
                     uint32_t* sink, void* stream);

/*
 * Strided row copy (no reference counterpart: the reference runs on one
 * device).  The sequence split keeps each KV-head group's K / V rows and its
 * fp32 partial dK / dV in [rows, B, heads, D] buffers, while its callers hold
 * [B, S, H, D] tensors; this moves rows between the two layouts on `stream`.
 * A row is row_elems contiguous elements; row (i0, i1, i2), 0 <= ik <
 * count[k], starts at element sum ik * src_stride[k] of src and sum ik *
 * dst_stride[k] of dst.  dtypes: src and dst both BF16 or both F16 (a copy),
 * or src F32 and dst BF16 / F16 (rounded to nearest even).  row_elems must be
 * a positive multiple of 8; src, dst and every stride must be 16-byte
 * aligned.  The rows of dst must not overlap each other or src.
 */
typedef struct {
  const void* src;
  void* dst;
  int32_t src_dtype;
  int32_t dst_dtype;
  int64_t row_elems;
  int64_t count[3];
  int64_t src_stride[3];
  int64_t dst_stride[3];
} esa_rows_t;
int esa_copy_rows(const esa_rows_t* rows, void* stream);

/* Size of the workspace array built into the library for esa_backward_noalloc. */
#define ESA_NOALLOC_WORKSPACE_BYTES (16u * 1024u * 1024u)

/*
 * esa_backward_noalloc -- esa_backward for callers that cannot allocate device
 * memory, e.g. a plugin running inside a host application that owns every GPU
 * allocation, or a serving loop that must not allocate once it is running.
 * It takes the same arguments as esa_backward minus the workspace, and uses an
 * array of ESA_NOALLOC_WORKSPACE_BYTES (16 MiB) compiled into the library
 * instead; it calls no cudaMalloc, cudaFree or other allocating routine.  No
 * counterpart in the reference (its backward allocates dq/dk/dv with torch).
 *
 * Limit: a problem whose esa_backward_workspace_size() exceeds 16 MiB is
 * rejected with ESA_ERR_WORKSPACE (the workspace is B * num_heads *
 * attention_length * q_len * 8 bytes, plus 8 * B * num_kv_heads * kv_rows *
 * head_dim bytes with GQA: e.g. 8 heads, w=64, 2048 query rows fit).
 * Set-up: the first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it; make that
 * first call before any stream capture.  Call with the tensors' device current.
 * Sharing: every call on a device uses the same array and leaves its contents
 * behind; calls that overlap on the GPU (other streams, other threads) race
 * and corrupt each other's gradients, so serialise them.  Nothing needs
 * clearing: each call writes every workspace byte before reading it.
 */
int esa_backward_noalloc(const esa_problem_t* prob, esa_tensor_t q, esa_tensor_t k,
                         esa_tensor_t v, esa_tensor_t o, const float* lse, esa_tensor_t dout,
                         esa_tensor_t dq, esa_tensor_t dk, esa_tensor_t dv,
                         const int64_t* sorted_rows, const int64_t* row_perm, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ESA_B200_H */
