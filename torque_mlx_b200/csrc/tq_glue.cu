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


// ---------------------------------------------------------------------------
// GEMV for one token: y[n] = bf16(sum_k W[n, k] x[k] (+ residual[n])), W the
// [N, K] bf16 weight of a linear layer (PyTorch layout), fp32 accumulation.
// The input vector is built once per CTA in shared memory (as the bf16
// values the separate PyTorch ops would produce) by one of four prologues:
//   kGemvBf16   x as given (bf16)
//   kGemvF32    bf16(x) of an fp32 vector (the attention output)
//   kGemvRms    rmsnorm(x, norm_w, eps) of a bf16 vector
//   kGemvSilu   bf16(bf16(silu(g)) * u) of a [g | u] bf16 row (K = f)
// The weight stream is the whole cost: a group of wpr warps takes two rows
// at a time, each warp a contiguous slice of k with 16-byte loads (8 weights
// a lane, four chunks of both rows issued before the math).  wpr (1..8)
// grows for short outputs so that every SM streams.
// ---------------------------------------------------------------------------
enum GemvInput { kGemvBf16 = 0, kGemvF32 = 1, kGemvRms = 2, kGemvSilu = 3 };
constexpr int kGemvThreads = 512;
constexpr int kGemvMaxK = 8192;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& w, float (&f)[8]) {
  const uint32_t r[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(r[i] << 16);
    f[2 * i + 1] = __uint_as_float(r[i] & 0xffff0000u);
  }
}

template <int MODE>
__global__ void __launch_bounds__(kGemvThreads)
gemv_kernel(const __nv_bfloat16* __restrict__ W, const void* __restrict__ x, const __nv_bfloat16* __restrict__ norm_w,
            float eps, const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ y, int N, int K,
            int wpr) {
  extern __shared__ __align__(16) __nv_bfloat16 xs[];  // [K]
  __shared__ float red[kGemvThreads / 32];
  __shared__ float part_s[2 * (kGemvThreads / 32)];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunks = K / 256;  // 16-byte chunks a lane takes per row (K multiple of 256)
  const int groups = (kGemvThreads / 32) / wpr;
  const int g = warp / wpr, part = warp - g * wpr;
  const int c_lo = part * chunks / wpr, c_hi = (part + 1) * chunks / wpr;

  // The weights depend on no earlier kernel: pull this warp's first row pair
  // into L2 before waiting for the previous kernel (programmatic dependent
  // launch) and building the input vector.
  {
    const int n0 = blockIdx.x * groups * 2 + 2 * g;
    for (int r = n0; r < n0 + 2 && r < N; ++r)
      for (int c = c_lo; c < c_hi; ++c)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(W + (int64_t)r * K + (int64_t)(c * 32 + lane) * 8));
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- prologue: the input vector as bf16 in shared memory ----
  if (MODE == kGemvRms) {
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
    float ss = 0.f;
    for (int k = tid; k < K; k += kGemvThreads) {
      const float v = __bfloat162float(xb[k]);
      ss = fmaf(v, v, ss);
    }
    const float inv = rsqrtf(block_sum<kGemvThreads>(ss, red) / (float)K + eps);
    for (int k = tid; k < K; k += kGemvThreads)
      xs[k] = __float2bfloat16_rn(
          __fmul_rn(bf16_round(__fmul_rn(__bfloat162float(xb[k]), inv)), __bfloat162float(norm_w[k])));
  } else if (MODE == kGemvSilu) {
    const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(x);
    for (int k = tid; k < K; k += kGemvThreads) {
      const float g = __bfloat162float(gu[k]), u = __bfloat162float(gu[K + k]);
      xs[k] = __float2bfloat16_rn(__fmul_rn(bf16_round(g / (1.f + expf(-g))), u));
    }
  } else if (MODE == kGemvF32) {
    const float* xf = reinterpret_cast<const float*>(x);
    for (int k = tid; k < K; k += kGemvThreads) xs[k] = __float2bfloat16_rn(xf[k]);
  } else {
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
    for (int k = tid; k < K; k += kGemvThreads) xs[k] = xb[k];
  }
  __syncthreads();
  // the next kernel may start its own prologue-free part (weight prefetch)
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- rows: a group of wpr warps takes two rows, each warp a slice of k ----
  const uint4* xv = reinterpret_cast<const uint4*>(xs);
  for (int base = blockIdx.x * groups * 2; base < N; base += gridDim.x * groups * 2) {  // uniform per CTA
    const int n0 = base + 2 * g;
    const bool one = n0 < N, two = n0 + 1 < N;
    float a0 = 0.f, a1 = 0.f;
    if (one) {
      const uint4* w0 = reinterpret_cast<const uint4*>(W + (int64_t)n0 * K);
      const uint4* w1 = reinterpret_cast<const uint4*>(W + (int64_t)(two ? n0 + 1 : n0) * K);
      int c = c_lo;
      for (; c + 4 <= c_hi; c += 4) {
        uint4 r0[4], r1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          r0[i] = __ldcs(w0 + (c + i) * 32 + lane);
          r1[i] = __ldcs(w1 + (c + i) * 32 + lane);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float xf[8], f0[8], f1[8];
          bf16x8_to_f32(xv[(c + i) * 32 + lane], xf);
          bf16x8_to_f32(r0[i], f0);
          bf16x8_to_f32(r1[i], f1);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            a0 = fmaf(f0[j], xf[j], a0);
            a1 = fmaf(f1[j], xf[j], a1);
          }
        }
      }
      for (; c < c_hi; ++c) {
        const uint4 r0 = __ldcs(w0 + c * 32 + lane), r1 = __ldcs(w1 + c * 32 + lane);
        float xf[8], f0[8], f1[8];
        bf16x8_to_f32(xv[c * 32 + lane], xf);
        bf16x8_to_f32(r0, f0);
        bf16x8_to_f32(r1, f1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          a0 = fmaf(f0[j], xf[j], a0);
          a1 = fmaf(f1[j], xf[j], a1);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a0 += __shfl_xor_sync(FULL, a0, o);
      a1 += __shfl_xor_sync(FULL, a1, o);
    }
    if (wpr > 1) {  // the group's slices meet in shared memory
      if (lane == 0) {
        part_s[2 * warp] = a0;
        part_s[2 * warp + 1] = a1;
      }
      __syncthreads();
      if (part == 0) {
        a0 = a1 = 0.f;
        for (int q = 0; q < wpr; ++q) {
          a0 += part_s[2 * (warp + q)];
          a1 += part_s[2 * (warp + q) + 1];
        }
      }
      __syncthreads();
    }
    if (one && part == 0 && lane == 0) {
      if (residual) {
        a0 += __bfloat162float(residual[n0]);
        if (two) a1 += __bfloat162float(residual[n0 + 1]);
      }
      y[n0] = __float2bfloat16_rn(a0);
      if (two) y[n0 + 1] = __float2bfloat16_rn(a1);
    }
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

int tq_gemv(const void* weight, const void* x, int x_mode, const void* norm_weight, float eps,
            const void* residual, void* y, int n, int k, tq_stream_t stream) {
  if (n <= 0 || k <= 0 || k % 256 || k > kGemvMaxK) return TQ_E_SHAPE;
  if (x_mode < kGemvBf16 || x_mode > kGemvSilu) return TQ_E_ARG;
  if (!weight || !x || !y || (x_mode == kGemvRms && !norm_weight)) return TQ_E_ARG;
  if ((uintptr_t)weight % 16) return TQ_E_SHAPE;
  // SMs and resident CTAs per SM (the same for every mode: one kernel body)
  static int sms = 0, per_sm = 1;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel<kGemvRms>, kGemvThreads,
                                                      (size_t)kGemvMaxK * sizeof(__nv_bfloat16)) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
  }
  const size_t smem = (size_t)k * sizeof(__nv_bfloat16);
  // warps per row pair: the smallest power of two that fills the resident wave
  int wpr = 1;
  while (wpr < 8 && wpr * 2 <= k / 256 && (int64_t)n * wpr < (int64_t)per_sm * sms * 2 * (kGemvThreads / 32)) wpr *= 2;
  const int rows_per_cta = 2 * (kGemvThreads / 32) / wpr;
  // one resident wave: every CTA builds the input vector once and streams
  // row groups grid-stride, the same number of rounds for every CTA (a grid
  // of all resident slots would leave most of them idle in a last partial
  // round)
  const int tasks = (n + rows_per_cta - 1) / rows_per_cta;
  const int slots = per_sm * sms;
  const int rounds = (tasks + slots - 1) / slots;
  const int grid = (tasks + rounds - 1) / rounds;
  cudaStream_t st = (cudaStream_t)stream;
  const __nv_bfloat16* w = (const __nv_bfloat16*)weight;
  const __nv_bfloat16* nw = (const __nv_bfloat16*)norm_weight;
  const __nv_bfloat16* res = (const __nv_bfloat16*)residual;
  __nv_bfloat16* out = (__nv_bfloat16*)y;
  // programmatic dependent launch: the kernel may be scheduled while the
  // previous kernel in the stream finishes; it waits (griddepcontrol.wait)
  // before touching anything that kernel wrote
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const void* xp = x;
  cudaError_t e;
  switch (x_mode) {
    case kGemvBf16: e = cudaLaunchKernelEx(&cfg, gemv_kernel<kGemvBf16>, w, xp, nw, eps, res, out, n, k, wpr); break;
    case kGemvF32: e = cudaLaunchKernelEx(&cfg, gemv_kernel<kGemvF32>, w, xp, nw, eps, res, out, n, k, wpr); break;
    case kGemvRms: e = cudaLaunchKernelEx(&cfg, gemv_kernel<kGemvRms>, w, xp, nw, eps, res, out, n, k, wpr); break;
    default: e = cudaLaunchKernelEx(&cfg, gemv_kernel<kGemvSilu>, w, xp, nw, eps, res, out, n, k, wpr); break;
  }
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return TQ_E_CUDA;
  }
  return launch_status();
}

}  // extern "C"
