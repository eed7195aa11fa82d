/*
 * torque_b200.h — C ABI of libtorque_b200.so, the B200 (sm_100a) packed-KV
 * decode path of torque-mlx.
 *
 * Every entry point takes plain device pointers and sizes, is ordered on the
 * CUDA stream it is given (NULL = legacy default stream), allocates nothing,
 * and returns 0 (TQ_OK) or a negative TQ_E_* status.  Argument errors are
 * detected on the host before any launch.  No entry point keeps mutable global
 * state, so separate host threads may call it on separate streams.
 *
 * Data formats (identical to the reference):
 *   - a head vector of d = 64|128|256 scalars is rotated by Pi = D1 H D2 / sqrt(d)
 *     (signs_left = D1, signs_right = D2; rotation.py:51-106),
 *   - each rotated scalar becomes the index of the nearest centroid of a sorted
 *     2^bits-entry fp32 codebook, ties to the lower index (quantization.py:120-125),
 *   - indices are packed LSB-first, code i at bit i*bits of the vector, into
 *     W = ceil(d*bits/32) uint32 words (quantization.py:156-201),
 *   - a cache slab is [groups, capacity, W] words with groups = (seq, layer,
 *     kv_head) flattened; the reference's [layers, kv_heads, seq, W] slab
 *     (layout.py:34-35) is the batch-1 case.
 *
 * Reference citations are path:line inside the cbun/torque-mlx project.
 */
#ifndef TORQUE_B200_H
#define TORQUE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tq_stream_t; /* same type as cudaStream_t */

enum tq_status {
  TQ_OK = 0,
  TQ_E_BITS = -1,      /* bits not in {2,3,4}           -> ValueError (quantization.py:16-18) */
  TQ_E_HEAD_DIM = -2,  /* head_dim not in {64,128,256}  -> ValueError (rotation.py:14-16)     */
  TQ_E_SHAPE = -3,     /* inconsistent sizes            -> ValueError (mlx_ops.py:351-357)   */
  TQ_E_CUDA = -4,      /* a CUDA call failed            -> RuntimeError                      */
  TQ_E_TIMEOUT = -5,   /* a bounded device wait gave up -> RuntimeError                      */
  TQ_E_WORKSPACE = -6, /* workspace missing/too small   -> RuntimeError                      */
  TQ_E_ARG = -7,       /* null pointer / bad enum value -> ValueError                        */
  TQ_E_SCRATCH_LIMIT = -8 /* needs more than the built-in decode scratch -> ValueError        */
};

enum tq_dtype { TQ_F32 = 0, TQ_F16 = 1, TQ_BF16 = 2 };

enum tq_decode_mode {
  TQ_DECODE_AUTO = 0,   /* tensor-core kernel when group_size >= 2, else exact */
  TQ_DECODE_EXACT = 1,  /* fp32 CUDA-core kernel, centroids and query in fp32  */
  TQ_DECODE_TENSOR = 2  /* mma.sync kernel, fp16 centroids/query/probabilities, fp32 accumulate */
};

/* ABI version of this header (bumped on any signature change). */
int tq_abi_version(void);
/* Human-readable text for a tq_status value. */
const char* tq_status_string(int status);
/* cudaError_t of the most recent TQ_E_CUDA on the calling thread. */
int tq_last_cuda_error(void);

/* ---------------------------------------------------------------------------
 * Primitives
 * ------------------------------------------------------------------------- */

/* y[r] = signs_second * H(signs_first * x[r]) / f32(sqrt(d)) for rows r; fp32 out.
 * Forward rotation: first = signs_right, second = signs_left (RotationSpec.apply,
 * rotation.py:88-94); inverse: first = signs_left, second = signs_right
 * (RotationSpec.inverse, rotation.py:96-102).  Bit-exact with numpy. */
int tq_rotate(const void* x, int x_dtype, float* y, int64_t rows, int head_dim,
              const float* signs_first, const float* signs_second, tq_stream_t stream);

/* codes[i] = argmin_k |x[i] - centroids[k]| (fp32, first index on ties).
 * Replaces quantize (quantization.py:120-125) and the boundary-count
 * quantize_mlx (quantization.py:139-148) of the MLX path. */
int tq_quantize(const float* x, uint8_t* codes, int64_t n, const float* centroids, int bits,
                tq_stream_t stream);

/* words[r, :] = LSB-first packing of codes[r, 0:count] (pack_indices /
 * pack_indices_batched, quantization.py:156-201).  words is [rows, ceil(count*bits/32)]. */
int tq_pack(const uint8_t* codes, uint32_t* words, int64_t rows, int count, int bits,
            tq_stream_t stream);

/* codes[r, 0:count] from words[r, :] (unpack_indices, quantization.py:272-290). */
int tq_unpack(const uint32_t* words, uint8_t* codes, int64_t rows, int count, int bits,
              tq_stream_t stream);

/* out[r, 0:d] = centroids[unpack(words[r])] — dequantize(unpack_indices(...))
 * as used by TorqueKVCache.export_dequantized (cache.py:189-214). */
int tq_dequantize_packed(const uint32_t* words, float* out, int64_t rows, int head_dim, int bits,
                         const float* centroids, tq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Append: rotate + quantize + pack straight into a cache slab
 * ------------------------------------------------------------------------- */

/* For group g in [0, groups) and token t in [0, tokens):
 *   pos = (start_pos ? start_pos[g / groups_per_seq] : 0) + pos_offset + t
 *   k_slab[g*group_stride_words + pos*W + 0:W] = pack(quantize(Pi k[g, t, :], cent_k))
 * and the same for v with cent_v when v != NULL.  k, v are contiguous
 * [groups, tokens, head_dim] in x_dtype.  rotate = 0 skips Pi (input already
 * rotated, as quantize_and_pack_rows_dual_metal expects).  Rows whose pos falls
 * outside [0, capacity) are not written.
 * Replaces TorqueKVCache.append's per-head loop (cache.py:78-96),
 * TorqueKVCacheMLX._append_packed_tokens (cache_mlx.py:396-418) and
 * quantize_and_pack_rows[_dual]_metal (mlx_ops.py:342-412). */
int tq_append_kv(const void* k, const void* v, int x_dtype, int64_t groups, int tokens,
                 int head_dim, int bits, const float* signs_left, const float* signs_right,
                 int rotate, const float* cent_k, const float* cent_v, uint32_t* k_slab,
                 uint32_t* v_slab, int64_t group_stride_words, int64_t capacity,
                 const int32_t* start_pos, int groups_per_seq, int64_t pos_offset,
                 tq_stream_t stream);

/* words_a[r, :] = pack(count_k(values_a[r, i] > boundaries_a[k])) for rows r of
 * already-rotated fp32 values [rows, head_dim], and the same for the b set
 * when values_b != NULL: the boundary-count quantizer of the MLX path
 * (quantize_mlx, quantization.py:139-148) fused with LSB-first packing.
 * boundaries_* hold 2^bits - 1 fp32 midpoints (codebook_boundaries,
 * quantization.py:128-136).  Replaces quantize_and_pack_rows_metal and
 * quantize_and_pack_rows_dual_metal (mlx_ops.py:342-412).  A value exactly on
 * a boundary takes the lower code, which can differ from tq_quantize's
 * nearest-centroid rule at exact midpoints (as the reference's two rules do). */
int tq_quantize_pack_boundaries(const float* values_a, const float* values_b, int64_t rows, int head_dim,
                                int bits, const float* boundaries_a, const float* boundaries_b,
                                uint32_t* words_a, uint32_t* words_b, tq_stream_t stream);

/* start_pos[i] += delta for i in [0, n): advances device-resident sequence
 * lengths after an append without a host round trip. */
int tq_lengths_add(int32_t* lengths, int n, int delta, tq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Decode attention over packed codes
 * ------------------------------------------------------------------------- */

/* Bytes of workspace tq_decode needs for these sizes (on the current device:
 * the split plan follows its SM count and the kernel's occupancy).  For
 * TQ_DECODE_AUTO the figure covers both kernels, because slabs that are not
 * 16-byte aligned (or a unit stride that is not a multiple of 4 words) make
 * AUTO run the exact kernel, whose plan can need more. */
int tq_decode_workspace_size(int64_t units, int group_size, int head_dim, int bits, int64_t max_len,
                             int mode, size_t* bytes);

/* Grouped-query decode attention (q_len = 1) straight on packed codes.
 *
 * units = (seq, layer, kv_head) triples; unit u reads
 *   k_slab/v_slab + u*unit_stride_words, tokens [0, n_u) with
 *   n_u = (lengths ? lengths[u / units_per_seq] : 0) + len_offset, clamped to max_len.
 * query is [units*group_size, head_dim] fp32 (query head h*G + g of unit u's
 * layer and seq attends kv head h, cache_mlx.py:706-722).  rotate_query = 1
 * applies Pi to the query first (cache.py:109); otherwise it is taken as rotated.
 * out[u*G + g] = softmax(scale * q . K^T) V over the dequantized codes,
 * optionally rotated back by Pi^T (inverse_rotate_output = 1, cache.py:131-134).
 * lse (nullable) receives the natural-log sum-exp of the scaled scores
 * (-inf for an empty sequence, whose output is 0 as in reference.py:40-41).
 * Replaces TorqueKVCache.decode (cache.py:98-140), TorqueKVCacheMLX.decode_mlx
 * (cache_mlx.py:173-234) and decode_packed_attention[_split_batched]
 * (mlx_ops.py:571-595, 663-692). */
int tq_decode(const float* query, int rotate_query, const float* signs_left,
              const float* signs_right, const uint32_t* k_slab, const uint32_t* v_slab,
              int64_t unit_stride_words, const int32_t* lengths, int units_per_seq,
              int64_t len_offset, int64_t max_len, int64_t units, int group_size, int head_dim,
              int bits, const float* cent_k, const float* cent_v, float scale, float* out,
              float* lse, int inverse_rotate_output, int mode, void* workspace,
              size_t workspace_bytes, tq_stream_t stream);

/* Chunked-prefill attention over packed codes: the last q_tokens tokens of
 * each unit (already appended) are also queries, causally.  query is
 * [units, q_tokens, group_size, head_dim] fp32 (token-major); row (t, g) of
 * unit u attends positions [0, n_u - q_tokens + t + 1), with n_u as in
 * tq_decode (lengths + len_offset, clamped to max_len).  out / lse have the
 * query's row layout.  q_tokens * group_size <= 16 per call (a longer chunk is
 * attended by successive calls, with len_offset moving the chunk's end).
 * Runs on the tensor-core kernel; workspace as tq_decode_workspace_size with
 * group_size = q_tokens * group_size and TQ_DECODE_TENSOR.
 * Replaces the prefill attention of the reference's chunked-prefill loop
 * (qwen_mlx.py:829-845, where it is dense attention over fresh K/V): here the
 * chunk attends the packed cache, prefix and chunk alike. */
int tq_decode_causal(const float* query, int rotate_query, const float* signs_left, const float* signs_right,
                     const uint32_t* k_slab, const uint32_t* v_slab, int64_t unit_stride_words,
                     const int32_t* lengths, int units_per_seq, int64_t len_offset, int64_t max_len, int64_t units,
                     int q_tokens, int group_size, int head_dim, int bits, const float* cent_k,
                     const float* cent_v, float scale, float* out, float* lse, int inverse_rotate_output,
                     void* workspace, size_t workspace_bytes, tq_stream_t stream);

/* One decode step with its append fused in: for every unit u of sequence
 * s = u / units_per_seq, row u of new_k / new_v ([units, head_dim] in kv_dtype)
 * is rotated (rotate_k / rotate_v), quantized with cent_k / cent_v and packed
 * at position lengths[s] of the unit's slab rows, then the query attends
 * tokens [0, lengths[s] + 1) exactly as tq_decode with len_offset = 1.  With
 * advance = 1, lengths[s] += 1 once the step is complete (append + decode);
 * with advance = 0 the lengths stay, which is the append-then-attend
 * semantics of decode_mlx_with_current (cache_mlx.py:236-302): the token is
 * written at the next position and attended but not counted, so a later
 * append of the same token leaves the same cache.
 * On the tensor-core path the CTA whose token chunk holds the new position
 * packs the token itself before it loads its tiles, so a step is two kernel
 * launches (decode + split merge) instead of four.  The caller guarantees
 * lengths[s] + 1 <= max_len (rows past max_len are neither written nor
 * attended) and the usual tq_decode workspace.
 * Replaces the TorqueKVCacheMLX.append_many_mlx + decode_mlx pair of one
 * generation step (cache_mlx.py:151-234) and decode_mlx_with_current. */
int tq_decode_append(const void* new_k, const void* new_v, int kv_dtype, int rotate_k, int rotate_v,
                     int advance, const float* query, int rotate_query, const float* signs_left,
                     const float* signs_right, uint32_t* k_slab, uint32_t* v_slab,
                     int64_t unit_stride_words, int32_t* lengths, int units_per_seq, int64_t max_len,
                     int64_t units, int group_size, int head_dim, int bits, const float* cent_k,
                     const float* cent_v, float scale, float* out, float* lse,
                     int inverse_rotate_output, int mode, void* workspace, size_t workspace_bytes,
                     tq_stream_t stream);

/* Allocation-free variant of tq_decode.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory (or must not at this point):
 * code that runs inside a memory pool or allocator it does not own, a host
 * language binding with no handle on the CUDA allocator, or a serving loop
 * whose memory budget is fixed once at start-up.  Same arguments and result as
 * tq_decode without the workspace pair: the split-K partials go to a scratch
 * array compiled into the library, TQ_DECODE_STATIC_SCRATCH_BYTES (16 MiB) per
 * GPU, which every GPU that loads the library holds until the process exits.
 *  - A decode whose plan needs more scratch than that (tq_decode_workspace_size
 *    reports the need) returns TQ_E_SCRATCH_LIMIT and launches nothing.
 *  - The scratch need is that of the plan the call really runs: with
 *    TQ_DECODE_AUTO and unaligned slabs that is the exact kernel's plan.
 *  - The first call on a device looks up that device's copy of the array
 *    (with the device current); make that first call outside any CUDA stream
 *    capture.  The address is kept per device index for the life of the
 *    process, so the entry point serves the device's primary context only:
 *    after cudaDeviceReset, or under a context the caller created itself, the
 *    kept address is no longer valid.
 *  - Every call on a device shares the one array.  Calls whose kernels may run
 *    at the same time on the GPU (different streams without ordering between
 *    them) race on it and give wrong results; order them on one stream.
 *  - Nothing in the array needs to start at zero: each call overwrites every
 *    partial it later reads.
 *  - It calls no allocator (no cudaMalloc / cudaFree). */
#define TQ_DECODE_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int tq_decode_static(const float* query, int rotate_query, const float* signs_left,
                     const float* signs_right, const uint32_t* k_slab, const uint32_t* v_slab,
                     int64_t unit_stride_words, const int32_t* lengths, int units_per_seq,
                     int64_t len_offset, int64_t max_len, int64_t units, int group_size,
                     int head_dim, int bits, const float* cent_k, const float* cent_v, float scale,
                     float* out, float* lse, int inverse_rotate_output, int mode,
                     tq_stream_t stream);

/* Merge P normalised partial attentions over disjoint key sets (the sequence
 * shards of a multi-GPU decode):
 *   LSE = logsumexp_p lse[p, r];  out[r] = sum_p exp(lse[p, r] - LSE) outs[p, r, :]
 * outs [parts, rows, head_dim], lses [parts, rows]; lse_out nullable;
 * inverse_rotate applies Pi^T to the merged row.  New in this build: the
 * reference runs on one device only (no counterpart). */
int tq_lse_merge(const float* outs, const float* lses, int parts, int64_t rows, int head_dim,
                 float* out, float* lse_out, int inverse_rotate, const float* signs_left,
                 const float* signs_right, tq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence-shard decode across GPUs (one process per GPU).  New in this build:
 * the reference runs on one device only (no counterpart).
 *
 * Each rank holds a share of one long sequence's tokens.  Every rank owns one
 * exchange buffer (tq_exchange_alloc, zero-filled) and maps every other
 * rank's buffer through its CUDA IPC handle (tq_exchange_open); the handles
 * travel over the host process group.  tq_decode_exchange then decodes the
 * rank's tokens and, in the launch that merges its split partials, stores the
 * rank's normalised partial and lse into every rank's buffer over NVLink,
 * publishes them with a system-scope flag per (rank, row), waits for the
 * other ranks' flags (each wait bounded by timeout_ns, measured with the GPU
 * global timer) and merges the world's partials by log-sum-exp.  Two kernel
 * launches per step, no host round trip and no library collective; a step can
 * be captured in a CUDA graph.  A wait that gives up writes TQ_E_TIMEOUT to
 * *status (device int32, never cleared by the library), leaves NaN rows and
 * returns; the host reads *status between steps.
 * ------------------------------------------------------------------------- */

#define TQ_IPC_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer for world ranks and rows query rows. */
int tq_exchange_buffer_bytes(int head_dim, int world, int64_t rows, size_t* bytes);
/* cudaMalloc + zero-fill `bytes` on the current device; *ptr gets the buffer,
 * ipc_handle (TQ_IPC_HANDLE_BYTES) its CUDA IPC handle.  Set-up only. */
int tq_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another process's exchange buffer from its IPC handle (peer access is
 * enabled lazily).  Set-up only. */
int tq_exchange_open(const void* ipc_handle, void** ptr);
/* Unmap a buffer mapped by tq_exchange_open / free one from tq_exchange_alloc. */
int tq_exchange_close(void* ptr);
int tq_exchange_free(void* ptr);

/* One sequence-shard decode step on this rank.  Arguments as tq_decode_append
 * (new_k == NULL: no token is appended on this rank; then new_v must be NULL
 * and advance 0, and len_offset is tq_decode's), plus:
 *   exchange_bufs  device array of `world` buffer pointers, [rank] = own buffer
 *   rank, world    this rank and the rank count (world <= 16)
 *   epoch          device int32[rows], zero at start, advanced by each step
 *                  (the same number of steps on every rank)
 *   timeout_ns     bound of each wait for a peer
 *   status         device int32 that receives TQ_E_TIMEOUT on a timeout
 * out / lse receive the merged rows over all ranks' tokens (lse natural-log). */
int tq_decode_exchange(const void* new_k, const void* new_v, int kv_dtype, int rotate_k, int rotate_v,
                       int advance, const float* query, int rotate_query, const float* signs_left,
                       const float* signs_right, uint32_t* k_slab, uint32_t* v_slab, int64_t unit_stride_words,
                       int32_t* lengths, int units_per_seq, int64_t len_offset, int64_t max_len, int64_t units,
                       int group_size, int head_dim, int bits, const float* cent_k, const float* cent_v,
                       float scale, float* out, float* lse, int inverse_rotate_output, int mode, void* workspace,
                       size_t workspace_bytes, float* const* exchange_bufs, int rank, int world, int32_t* epoch,
                       int64_t timeout_ns, int32_t* status, tq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Decoder glue for the end-to-end generation step (benchmark config 5, a 28-layer GQA decoder).  No
 * counterpart in the reference's C surface: these replace the PyTorch
 * elementwise ops around the KV step of the example decoder (the reference
 * runs the same ops as MLX graph nodes in its Qwen adapter,
 * families/qwen_mlx.py).  bf16 tensors, fp32 math, bf16 rounding where the
 * PyTorch ops round.
 * ------------------------------------------------------------------------- */

/* y[r] = bf16(bf16(x[r] * rsqrt(mean(x[r]^2) + eps)) * weight) for rows r of n
 * (n even; 4-byte aligned pointers). */
int tq_rmsnorm(const void* x, const void* weight, float eps, int64_t rows, int n, void* y, tq_stream_t stream);

/* RoPE (interleaved pairs (2i, 2i+1), angle table rows at *position) on the
 * q and k heads of one fused row qkv = [q_heads | kv_heads | kv_heads] x
 * head_dim (bf16): q_out gets the bf16-rounded q in fp32, k_out the k heads
 * in bf16.  cos/sin tables are [positions, head_dim/2] fp32; position is a
 * device int64 (so a captured graph follows it). */
int tq_rope_qk(const void* qkv, const float* cos_table, const float* sin_table, const int64_t* position,
               int q_heads, int kv_heads, int head_dim, float* q_out, void* k_out, tq_stream_t stream);

/* y[r, j] = bf16(bf16(silu(g)) * u) with g = gate_up[r, j], u = gate_up[r, f + j]. */
int tq_silu_mul(const void* gate_up, int64_t rows, int f, void* y, tq_stream_t stream);

/* One-token linear layer: y[i] = bf16(sum_j weight[i, j] x'[j] (+ residual[i]))
 * for weight [n, k] bf16 (16-byte aligned, k a multiple of 256, k <= 8192),
 * fp32 accumulation, where x' is built from x by x_mode:
 *   0  x' = x (bf16 [k])
 *   1  x' = bf16(x) (fp32 [k])
 *   2  x' = tq_rmsnorm(x, norm_weight, eps) (bf16 [k])
 *   3  x' = tq_silu_mul(x) (bf16 [2k] = [gate | up])
 * residual (nullable) is bf16 [n], added in fp32 before the one rounding. */
int tq_gemv(const void* weight, const void* x, int x_mode, const void* norm_weight, float eps,
            const void* residual, void* y, int n, int k, tq_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TORQUE_B200_H */
