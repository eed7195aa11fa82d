// Per-token append path: structured-Hadamard rotation fused with the nearest-
// centroid quantizer and LSB-first bit packing, written straight into the
// cache slab.  Also the stand-alone primitives (rotate, quantize, pack,
// unpack, dequantize) and the ABI bookkeeping entry points.
//
// Layout: one warp owns one head vector; lane l holds elements j*32 + l
// (j < d/32), so global loads and the packed-word stores are coalesced and
// the Hadamard butterflies are shuffles (span < 32) or register pairs.
#include "tq_common.cuh"

#include <stdio.h>

namespace tq {

static thread_local int g_last_cuda_error = 0;
void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

constexpr int kAppendWarps = 8;  // rows per CTA

// ---------------------------------------------------------------------------
// rotate + quantize + pack one row per warp into the slab.
// ---------------------------------------------------------------------------
// Each warp takes kAppendRows consecutive rows and issues all their loads
// before any math, so several rows' reads are in flight per warp.
constexpr int kAppendRows = 4;

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(kAppendWarps * 32)
append_pack_kernel(const T* __restrict__ k, const T* __restrict__ v, int64_t groups, int tokens,
                   const float* __restrict__ signs_left, const float* __restrict__ signs_right,
                   int rotate, const float* __restrict__ cent_k, const float* __restrict__ cent_v,
                   uint32_t* __restrict__ k_slab, uint32_t* __restrict__ v_slab,
                   int64_t group_stride, int64_t capacity, const int32_t* __restrict__ start_pos,
                   int groups_per_seq, int64_t pos_offset) {
  constexpr int E = D / 32;
  constexpr int W = D * BITS / 32;
  constexpr int L = 1 << BITS;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * kAppendWarps + (threadIdx.x >> 5)) * kAppendRows;
  const int64_t rows = groups * (int64_t)tokens;
  if (row0 >= rows) return;
  const int which = blockIdx.y;  // 0 = K, 1 = V
  const T* x = which ? v : k;
  const float* cent = which ? cent_v : cent_k;
  uint32_t* slab = which ? v_slab : k_slab;

  float val[kAppendRows][E];
#pragma unroll
  for (int r = 0; r < kAppendRows; ++r) {
    const int64_t row = row0 + r;
    const T* src = x + (row < rows ? row : row0) * D;
#pragma unroll
    for (int j = 0; j < E; ++j) val[r][j] = to_f32(src[j * 32 + lane]);
  }
  float c[L];
#pragma unroll
  for (int i = 0; i < L; ++i) c[i] = __ldg(cent + i);

#pragma unroll
  for (int r = 0; r < kAppendRows; ++r) {
    const int64_t row = row0 + r;
    if (row >= rows) break;
    const int64_t g = row / tokens;
    const int t = (int)(row - g * tokens);
    int64_t pos = pos_offset + t;
    if (start_pos) pos += start_pos[g / groups_per_seq];
    if (pos < 0 || pos >= capacity) continue;  // warp-uniform
    if (rotate) warp_rotate<D>(val[r], lane, signs_right, signs_left);
    warp_pack_row<D, BITS>(val[r], lane, c, slab + g * group_stride + pos * W);
  }
}

// Boundary-count quantize + pack of already-rotated fp32 rows, one row per
// warp: code = number of boundaries b[k] with x > b[k] (the MLX path's rule,
// quantization.py:139-148 and the append-pack kernels of mlx_ops.py:257-339),
// then the same LSB-first packing as the cache.  blockIdx.y selects the
// (values, boundaries, words) set: 0 = a, 1 = b.
template <int D, int BITS>
__global__ void __launch_bounds__(kAppendWarps * 32)
boundary_pack_kernel(const float* __restrict__ xa, const float* __restrict__ xb, int64_t rows,
                     const float* __restrict__ ba, const float* __restrict__ bb, uint32_t* __restrict__ wa,
                     uint32_t* __restrict__ wb) {
  constexpr int E = D / 32;
  constexpr int W = D * BITS / 32;
  constexpr int NB = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool second = blockIdx.y == 1;
  const float* x = (second ? xb : xa) + row * D;
  const float* bnd = second ? bb : ba;
  float b[NB];
#pragma unroll
  for (int k = 0; k < NB; ++k) b[k] = __ldg(bnd + k);
  uint32_t code[E];
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const float v = x[j * 32 + lane];
    uint32_t c = 0;
#pragma unroll
    for (int k = 0; k < NB; ++k) c += v > b[k] ? 1u : 0u;
    code[j] = c;
  }
  warp_pack_codes<D, BITS>(code, lane, (second ? wb : wa) + row * W);
}

template <int D>
static void launch_boundary_pack(int bits, const float* xa, const float* xb, int64_t rows, const float* ba,
                                 const float* bb, uint32_t* wa, uint32_t* wb, cudaStream_t st) {
  dim3 grid((unsigned)((rows + kAppendWarps - 1) / kAppendWarps), xb ? 2 : 1);
  if (bits == 2) boundary_pack_kernel<D, 2><<<grid, kAppendWarps * 32, 0, st>>>(xa, xb, rows, ba, bb, wa, wb);
  else if (bits == 3) boundary_pack_kernel<D, 3><<<grid, kAppendWarps * 32, 0, st>>>(xa, xb, rows, ba, bb, wa, wb);
  else boundary_pack_kernel<D, 4><<<grid, kAppendWarps * 32, 0, st>>>(xa, xb, rows, ba, bb, wa, wb);
}

// rotation only (RotationSpec.apply / inverse)
template <int D, typename T>
__global__ void __launch_bounds__(256)
rotate_kernel(const T* __restrict__ x, float* __restrict__ y, int64_t rows,
              const float* __restrict__ first, const float* __restrict__ second) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float val[E];
#pragma unroll
  for (int j = 0; j < E; ++j) val[j] = to_f32(x[row * D + j * 32 + lane]);
  warp_rotate<D>(val, lane, first, second);
#pragma unroll
  for (int j = 0; j < E; ++j) y[row * D + j * 32 + lane] = val[j];
}

template <int BITS>
__global__ void quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ codes, int64_t n,
                                const float* __restrict__ centroids) {
  float c[1 << BITS];
#pragma unroll
  for (int i = 0; i < (1 << BITS); ++i) c[i] = __ldg(centroids + i);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    codes[i] = (uint8_t)nearest_code<BITS>(x[i], c);
}

// one thread per output word: OR in every code that overlaps it
__global__ void pack_kernel(const uint8_t* __restrict__ codes, uint32_t* __restrict__ words,
                            int64_t rows, int count, int bits) {
  const int W = (count * bits + 31) / 32;
  const int64_t total = rows * W;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / W;
    const int w = (int)(idx - r * W);
    const uint8_t* c = codes + r * count;
    const int lo_bit = 32 * w, hi_bit = lo_bit + 32;
    int first = lo_bit / bits;
    if (first > 0) --first;  // the code before may spill into this word
    uint32_t word = 0;
    for (int i = first; i < count && i * bits < hi_bit; ++i) {
      if (i * bits + bits <= lo_bit) continue;
      const int sh = i * bits - lo_bit;
      const uint32_t val = c[i] & ((1u << bits) - 1u);
      if (sh >= 0) word |= val << sh;
      else word |= val >> (-sh);
    }
    words[idx] = word;
  }
}

__global__ void unpack_kernel(const uint32_t* __restrict__ words, uint8_t* __restrict__ codes,
                              int64_t rows, int count, int bits, const float* __restrict__ cent,
                              float* __restrict__ deq) {
  const int W = (count * bits + 31) / 32;
  const int64_t total = rows * count;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / count;
    const int i = (int)(idx - r * count);
    const uint32_t* w = words + r * W;
    const int bit = i * bits, wi = bit >> 5, sh = bit & 31;
    uint32_t val = w[wi] >> sh;
    if (sh + bits > 32) val |= w[wi + 1] << (32 - sh);
    val &= mask;
    if (codes) codes[idx] = (uint8_t)val;
    if (deq) deq[idx] = __ldg(cent + val);
  }
}

__global__ void lengths_add_kernel(int32_t* lengths, int n, int delta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) lengths[i] += delta;
}

inline int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  return (int)(b < 1 ? 1 : b);
}

template <int D, int BITS, typename T>
static void launch_append(const void* k, const void* v, int64_t groups, int tokens,
                          const float* sl, const float* sr, int rotate, const float* ck,
                          const float* cv, uint32_t* ks, uint32_t* vs, int64_t gstride,
                          int64_t capacity, const int32_t* start, int gps, int64_t off,
                          cudaStream_t st) {
  const int64_t rows = groups * (int64_t)tokens;
  const int64_t per_cta = (int64_t)kAppendWarps * kAppendRows;
  dim3 grid((unsigned)((rows + per_cta - 1) / per_cta), v ? 2 : 1);
  append_pack_kernel<D, BITS, T><<<grid, kAppendWarps * 32, 0, st>>>(
      (const T*)k, (const T*)v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity,
      start, gps, off);
}

template <int D, typename T>
static void launch_append_b(int bits, const void* k, const void* v, int64_t groups, int tokens,
                            const float* sl, const float* sr, int rotate, const float* ck,
                            const float* cv, uint32_t* ks, uint32_t* vs, int64_t gstride,
                            int64_t capacity, const int32_t* start, int gps, int64_t off,
                            cudaStream_t st) {
  if (bits == 2) launch_append<D, 2, T>(k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
  else if (bits == 3) launch_append<D, 3, T>(k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
  else launch_append<D, 4, T>(k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
}

template <typename T>
static void launch_append_d(int d, int bits, const void* k, const void* v, int64_t groups,
                            int tokens, const float* sl, const float* sr, int rotate,
                            const float* ck, const float* cv, uint32_t* ks, uint32_t* vs,
                            int64_t gstride, int64_t capacity, const int32_t* start, int gps,
                            int64_t off, cudaStream_t st) {
  if (d == 64) launch_append_b<64, T>(bits, k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
  else if (d == 128) launch_append_b<128, T>(bits, k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
  else launch_append_b<256, T>(bits, k, v, groups, tokens, sl, sr, rotate, ck, cv, ks, vs, gstride, capacity, start, gps, off, st);
}

template <typename T>
static void launch_rotate(int d, const void* x, float* y, int64_t rows, const float* a,
                          const float* b, cudaStream_t st) {
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (d == 64) rotate_kernel<64, T><<<grid, 256, 0, st>>>((const T*)x, y, rows, a, b);
  else if (d == 128) rotate_kernel<128, T><<<grid, 256, 0, st>>>((const T*)x, y, rows, a, b);
  else rotate_kernel<256, T><<<grid, 256, 0, st>>>((const T*)x, y, rows, a, b);
}

}  // namespace tq

using namespace tq;

extern "C" {

int tq_abi_version(void) { return 1; }

const char* tq_status_string(int s) {
  switch (s) {
    case TQ_OK: return "ok";
    case TQ_E_BITS: return "unsupported bit width (expected 2, 3 or 4)";
    case TQ_E_HEAD_DIM: return "unsupported head dimension (expected 64, 128 or 256)";
    case TQ_E_SHAPE: return "inconsistent sizes";
    case TQ_E_CUDA: return "CUDA error";
    case TQ_E_TIMEOUT: return "device wait timed out";
    case TQ_E_WORKSPACE: return "workspace missing or too small";
    case TQ_E_ARG: return "invalid argument";
    case TQ_E_SCRATCH_LIMIT: return "decode needs more scratch than the library's built-in 16 MiB (use tq_decode with a workspace)";
    default: return "unknown status";
  }
}

int tq_last_cuda_error(void) { return g_last_cuda_error; }

int tq_rotate(const void* x, int x_dtype, float* y, int64_t rows, int head_dim,
              const float* signs_first, const float* signs_second, tq_stream_t stream) {
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (rows < 0) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!x || !y || !signs_first || !signs_second) return TQ_E_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (x_dtype == TQ_F32) launch_rotate<float>(head_dim, x, y, rows, signs_first, signs_second, st);
  else if (x_dtype == TQ_F16) launch_rotate<__half>(head_dim, x, y, rows, signs_first, signs_second, st);
  else if (x_dtype == TQ_BF16) launch_rotate<__nv_bfloat16>(head_dim, x, y, rows, signs_first, signs_second, st);
  else return TQ_E_ARG;
  return launch_status();
}

int tq_quantize(const float* x, uint8_t* codes, int64_t n, const float* centroids, int bits,
                tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (n < 0) return TQ_E_SHAPE;
  if (n == 0) return TQ_OK;
  if (!x || !codes || !centroids) return TQ_E_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int grid = grid_for(n, 256);
  if (bits == 2) quantize_kernel<2><<<grid, 256, 0, st>>>(x, codes, n, centroids);
  else if (bits == 3) quantize_kernel<3><<<grid, 256, 0, st>>>(x, codes, n, centroids);
  else quantize_kernel<4><<<grid, 256, 0, st>>>(x, codes, n, centroids);
  return launch_status();
}

int tq_pack(const uint8_t* codes, uint32_t* words, int64_t rows, int count, int bits,
            tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (rows < 0 || count < 0) return TQ_E_SHAPE;
  if (rows == 0 || count == 0) return TQ_OK;
  if (!codes || !words) return TQ_E_ARG;
  const int64_t total = rows * (int64_t)words_for(count, bits);
  pack_kernel<<<grid_for(total, 256), 256, 0, (cudaStream_t)stream>>>(codes, words, rows, count, bits);
  return launch_status();
}

int tq_unpack(const uint32_t* words, uint8_t* codes, int64_t rows, int count, int bits,
              tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (rows < 0 || count < 0) return TQ_E_SHAPE;
  if (rows == 0 || count == 0) return TQ_OK;
  if (!codes || !words) return TQ_E_ARG;
  unpack_kernel<<<grid_for(rows * (int64_t)count, 256), 256, 0, (cudaStream_t)stream>>>(
      words, codes, rows, count, bits, nullptr, nullptr);
  return launch_status();
}

int tq_dequantize_packed(const uint32_t* words, float* out, int64_t rows, int head_dim, int bits,
                         const float* centroids, tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (rows < 0) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!words || !out || !centroids) return TQ_E_ARG;
  unpack_kernel<<<grid_for(rows * (int64_t)head_dim, 256), 256, 0, (cudaStream_t)stream>>>(
      words, nullptr, rows, head_dim, bits, centroids, out);
  return launch_status();
}

int tq_append_kv(const void* k, const void* v, int x_dtype, int64_t groups, int tokens,
                 int head_dim, int bits, const float* signs_left, const float* signs_right,
                 int rotate, const float* cent_k, const float* cent_v, uint32_t* k_slab,
                 uint32_t* v_slab, int64_t group_stride_words, int64_t capacity,
                 const int32_t* start_pos, int groups_per_seq, int64_t pos_offset,
                 tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (groups < 0 || tokens < 0 || capacity < 0) return TQ_E_SHAPE;
  if (groups == 0 || tokens == 0) return TQ_OK;
  if (!k || !cent_k || !k_slab) return TQ_E_ARG;
  if (v && (!cent_v || !v_slab)) return TQ_E_ARG;
  if (rotate && (!signs_left || !signs_right)) return TQ_E_ARG;
  if (start_pos && groups_per_seq <= 0) return TQ_E_ARG;
  const int W = words_for(head_dim, bits);
  if (group_stride_words < capacity * W) return TQ_E_SHAPE;
  if (!start_pos && (pos_offset < 0 || pos_offset + tokens > capacity)) return TQ_E_SHAPE;
  cudaStream_t st = (cudaStream_t)stream;
  if (x_dtype == TQ_F32)
    launch_append_d<float>(head_dim, bits, k, v, groups, tokens, signs_left, signs_right, rotate, cent_k, cent_v, k_slab, v_slab, group_stride_words, capacity, start_pos, groups_per_seq, pos_offset, st);
  else if (x_dtype == TQ_F16)
    launch_append_d<__half>(head_dim, bits, k, v, groups, tokens, signs_left, signs_right, rotate, cent_k, cent_v, k_slab, v_slab, group_stride_words, capacity, start_pos, groups_per_seq, pos_offset, st);
  else if (x_dtype == TQ_BF16)
    launch_append_d<__nv_bfloat16>(head_dim, bits, k, v, groups, tokens, signs_left, signs_right, rotate, cent_k, cent_v, k_slab, v_slab, group_stride_words, capacity, start_pos, groups_per_seq, pos_offset, st);
  else
    return TQ_E_ARG;
  return launch_status();
}

int tq_quantize_pack_boundaries(const float* values_a, const float* values_b, int64_t rows, int head_dim,
                                int bits, const float* boundaries_a, const float* boundaries_b,
                                uint32_t* words_a, uint32_t* words_b, tq_stream_t stream) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (rows < 0) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!values_a || !boundaries_a || !words_a) return TQ_E_ARG;
  if (values_b && (!boundaries_b || !words_b)) return TQ_E_ARG;
  if (rows > (int64_t)65535 * 65535 * kAppendWarps) return TQ_E_SHAPE;
  cudaStream_t st = (cudaStream_t)stream;
  if (head_dim == 64) launch_boundary_pack<64>(bits, values_a, values_b, rows, boundaries_a, boundaries_b, words_a, words_b, st);
  else if (head_dim == 128) launch_boundary_pack<128>(bits, values_a, values_b, rows, boundaries_a, boundaries_b, words_a, words_b, st);
  else launch_boundary_pack<256>(bits, values_a, values_b, rows, boundaries_a, boundaries_b, words_a, words_b, st);
  return launch_status();
}

int tq_lengths_add(int32_t* lengths, int n, int delta, tq_stream_t stream) {
  if (n < 0) return TQ_E_SHAPE;
  if (n == 0) return TQ_OK;
  if (!lengths) return TQ_E_ARG;
  lengths_add_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(lengths, n, delta);
  return launch_status();
}

}  // extern "C"
