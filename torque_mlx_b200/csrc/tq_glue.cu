// Decoder glue around the packed-KV step (benchmark config 5, a 28-layer GQA decoder): the per-token
// elementwise work of a pre-norm GQA decoder layer, one launch per op, in the
// op order and roundings of the PyTorch code it replaces (fp32 math, bf16
// results), so a CUDA-graph step is a dozen launches per layer instead of
// about fifty small PyTorch kernels.
//
//   tq_rmsnorm  y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)
//   tq_rope_qk  q, k of the fused qkv row rotated by RoPE (interleaved pairs)
//               at a device-resident position; q out in fp32 (of its bf16
//               value), k out in bf16
//   tq_silu_mul y = bf16(bf16(silu(g)) * u) for the gate/up halves of a row
#include "tq_common.cuh"

#include <math.h>

namespace tq {

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int T>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < T / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
    if (lane == 0) red[0] = s;
  }
  __syncthreads();
  return red[0];
}

constexpr int kGlueThreads = 256;

// one CTA per row; n a multiple of 2 (bf16x2 loads)
__global__ void __launch_bounds__(kGlueThreads)
rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, float eps, int n,
               __nv_bfloat16* __restrict__ y) {
  __shared__ float red[kGlueThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + row * n);
  const __nv_bfloat162* wr = reinterpret_cast<const __nv_bfloat162*>(w);
  __nv_bfloat162* yr = reinterpret_cast<__nv_bfloat162*>(y + row * n);
  float ss = 0.f;
  for (int i = threadIdx.x; i < n / 2; i += kGlueThreads) {
    const float2 v = __bfloat1622float2(xr[i]);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
  }
  const float total = block_sum<kGlueThreads>(ss, red);
  const float inv = rsqrtf(total / (float)n + eps);
  for (int i = threadIdx.x; i < n / 2; i += kGlueThreads) {
    const float2 v = __bfloat1622float2(xr[i]);
    const float2 g = __bfloat1622float2(wr[i]);
    yr[i] = __floats2bfloat162_rn(__fmul_rn(bf16_round(__fmul_rn(v.x, inv)), g.x),
                                  __fmul_rn(bf16_round(__fmul_rn(v.y, inv)), g.y));
  }
}

// qkv row = [q heads | k heads | v heads] x d (bf16); pairs (2i, 2i+1) of a
// head rotate by angle pos * inv_freq[i] with cos/sin tables [positions, d/2].
__global__ void __launch_bounds__(kGlueThreads)
rope_qk_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
               const float* __restrict__ sin_t, const int64_t* __restrict__ pos, int hq, int hkv, int d,
               float* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out) {
  const int half = d / 2;
  const int64_t p = *pos;
  const float* c = cos_t + p * half;
  const float* s = sin_t + p * half;
  const int pairs = (hq + hkv) * half;
  for (int idx = blockIdx.x * kGlueThreads + threadIdx.x; idx < pairs; idx += gridDim.x * kGlueThreads) {
    const int head = idx / half, i = idx - head * half;
    const __nv_bfloat162 v2 = reinterpret_cast<const __nv_bfloat162*>(qkv + (int64_t)head * d)[i];
    const float x1 = __bfloat162float(v2.x), x2 = __bfloat162float(v2.y);
    const float ci = c[i], si = s[i];
    // separate roundings (no fma contraction), as the elementwise PyTorch ops do
    const float r1 = bf16_round(__fsub_rn(__fmul_rn(x1, ci), __fmul_rn(x2, si)));
    const float r2 = bf16_round(__fadd_rn(__fmul_rn(x1, si), __fmul_rn(x2, ci)));
    if (head < hq) {
      q_out[(int64_t)head * d + 2 * i] = r1;
      q_out[(int64_t)head * d + 2 * i + 1] = r2;
    } else {
      reinterpret_cast<__nv_bfloat162*>(k_out + (int64_t)(head - hq) * d)[i] = __floats2bfloat162_rn(r1, r2);
    }
  }
}

// gu row = [gate (f) | up (f)] (bf16) -> y row (f)
__global__ void __launch_bounds__(kGlueThreads)
silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int f, int64_t rows, __nv_bfloat16* __restrict__ y) {
  const int64_t total = rows * f;
  for (int64_t idx = (int64_t)blockIdx.x * kGlueThreads + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * kGlueThreads) {
    const int64_t r = idx / f, j = idx - r * f;
    const float g = __bfloat162float(gu[r * 2 * f + j]);
    const float u = __bfloat162float(gu[r * 2 * f + f + j]);
    const float act = bf16_round(g / (1.f + expf(-g)));
    y[idx] = __float2bfloat16_rn(__fmul_rn(act, u));
  }
}

}  // namespace tq

using namespace tq;

extern "C" {

int tq_rmsnorm(const void* x, const void* weight, float eps, int64_t rows, int n, void* y, tq_stream_t stream) {
  if (rows < 0 || n <= 0 || (n & 1)) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!x || !weight || !y) return TQ_E_ARG;
  if ((uintptr_t)x % 4 || (uintptr_t)weight % 4 || (uintptr_t)y % 4) return TQ_E_SHAPE;
  rmsnorm_kernel<<<(unsigned)rows, kGlueThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, eps, n, (__nv_bfloat16*)y);
  return launch_status();
}

int tq_rope_qk(const void* qkv, const float* cos_table, const float* sin_table, const int64_t* position,
               int q_heads, int kv_heads, int head_dim, float* q_out, void* k_out, tq_stream_t stream) {
  if (q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || (head_dim & 1)) return TQ_E_SHAPE;
  if (!qkv || !cos_table || !sin_table || !position || !q_out || !k_out) return TQ_E_ARG;
  if ((uintptr_t)qkv % 4 || (uintptr_t)k_out % 4) return TQ_E_SHAPE;
  const int pairs = (q_heads + kv_heads) * head_dim / 2;
  const unsigned grid = (unsigned)((pairs + kGlueThreads - 1) / kGlueThreads);
  rope_qk_kernel<<<grid, kGlueThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, cos_table, sin_table, position, q_heads, kv_heads, head_dim, q_out,
      (__nv_bfloat16*)k_out);
  return launch_status();
}

int tq_silu_mul(const void* gate_up, int64_t rows, int f, void* y, tq_stream_t stream) {
  if (rows < 0 || f <= 0) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!gate_up || !y) return TQ_E_ARG;
  const int64_t total = rows * f;
  int64_t grid = (total + kGlueThreads - 1) / kGlueThreads;
  if (grid > 148 * 16) grid = 148 * 16;
  silu_mul_kernel<<<(unsigned)grid, kGlueThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)gate_up, f, rows, (__nv_bfloat16*)y);
  return launch_status();
}

}  // extern "C"
