// Shared device helpers for the packed-KV kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/torque_b200.h"

namespace tq {

// Optional step timeline for development builds (-DTQ_TRACE): thread 0 of a
// CTA records %globaltimer at fixed points into a per-file device array.
#ifdef TQ_TRACE
#define TQ_STAMP(arr, idx)                                                 \
  do {                                                                     \
    if (threadIdx.x == 0) {                                                \
      unsigned long long t_;                                               \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));               \
      arr[idx] = t_;                                                       \
    }                                                                      \
  } while (0)
#else
#define TQ_STAMP(arr, idx) do { } while (0)
#endif


constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------
// host-side status plumbing
// ---------------------------------------------------------------------------
void set_last_cuda_error(cudaError_t e);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return TQ_E_CUDA;
  }
  return TQ_OK;
}

inline bool valid_bits(int b) { return b == 2 || b == 3 || b == 4; }
inline bool valid_head_dim(int d) { return d == 64 || d == 128 || d == 256; }
inline int words_for(int count, int bits) { return (count * bits + 31) / 32; }

// f32(sqrt(d)) exactly as numpy rounds it (a C++ double literal converted to
// float rounds to nearest, like np.float32(math.sqrt(d))).
template <int D> struct SqrtD;
template <> struct SqrtD<64>  { static constexpr float v = 8.0f; };
template <> struct SqrtD<128> { static constexpr float v = (float)11.313708498984761; };
template <> struct SqrtD<256> { static constexpr float v = 16.0f; };

// ---------------------------------------------------------------------------
// element loads
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ---------------------------------------------------------------------------
// Walsh-Hadamard butterfly network across one warp.
//
// A d-vector lives in a warp as v[j] = x[j*32 + lane], j < d/32.  Stages run
// in the order span = 1, 2, 4, ..., d/2 and each maps the pair
// (x[i], x[i+span]) (bit `span` of i clear) to (a + b, a - b) in fp32, which
// is the exact operation sequence of the reference's numpy transform, so the
// result is bit-identical.  Spans < 32 cross lanes (shuffle), larger spans
// pair registers of the same lane.
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void warp_fwht(float (&v)[D / 32], int lane) {
  constexpr int E = D / 32;
#pragma unroll
  for (int span = 1; span < 32; span <<= 1) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      float other = __shfl_xor_sync(FULL, v[j], span);
      v[j] = (lane & span) ? __fsub_rn(other, v[j]) : __fadd_rn(v[j], other);
    }
  }
#pragma unroll
  for (int s = 1; s < E; s <<= 1) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      if ((j & s) == 0) {
        float a = v[j], b = v[j + s];
        v[j] = __fadd_rn(a, b);
        v[j + s] = __fsub_rn(a, b);
      }
    }
  }
}

// y = second * H(first * x) / f32(sqrt(d)), IEEE division (no reciprocal).
template <int D>
__device__ __forceinline__ void warp_rotate(float (&v)[D / 32], int lane, const float* first,
                                            const float* second) {
  constexpr int E = D / 32;
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = __fmul_rn(v[j], __ldg(first + j * 32 + lane));
  warp_fwht<D>(v, lane);
#pragma unroll
  for (int j = 0; j < E; ++j)
    v[j] = __fmul_rn(__fdiv_rn(v[j], SqrtD<D>::v), __ldg(second + j * 32 + lane));
}

// The same rotation with the sign vectors already in registers (loaded by
// load_signs ahead of time, so their latency overlaps other work).
template <int D>
__device__ __forceinline__ void load_signs(float (&s)[D / 32], const float* p, int lane) {
#pragma unroll
  for (int j = 0; j < D / 32; ++j) s[j] = __ldg(p + j * 32 + lane);
}

template <int D>
__device__ __forceinline__ void warp_rotate_regs(float (&v)[D / 32], int lane, const float (&first)[D / 32],
                                                 const float (&second)[D / 32]) {
  constexpr int E = D / 32;
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = __fmul_rn(v[j], first[j]);
  warp_fwht<D>(v, lane);
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = __fmul_rn(__fdiv_rn(v[j], SqrtD<D>::v), second[j]);
}

// argmin_k |x - c[k]| over fp32 rounded distances, first index on ties.
template <int BITS>
__device__ __forceinline__ uint32_t nearest_code(float x, const float (&c)[1 << BITS]) {
  uint32_t best = 0;
  float bd = fabsf(__fsub_rn(x, c[0]));
#pragma unroll
  for (int k = 1; k < (1 << BITS); ++k) {
    float dk = fabsf(__fsub_rn(x, c[k]));
    if (dk < bd) { bd = dk; best = (uint32_t)k; }
  }
  return best;
}

// Store the W = D*BITS/32 packed words of a warp-resident row of codes
// (code[j] = code of element j*32 + lane) to dst, LSB-first: code i at bit
// i*BITS.  The 32 codes of register j fill words j*BITS .. j*BITS + BITS-1;
// lane j*BITS + q assembles word q of group j with one warp OR-reduction and
// lanes 0..W-1 store.
template <int D, int BITS>
__device__ __forceinline__ void warp_pack_codes(const uint32_t (&code)[D / 32], int lane, uint32_t* dst) {
  constexpr int E = D / 32;
  constexpr int W = D * BITS / 32;
  uint32_t out_word = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
#pragma unroll
    for (int q = 0; q < BITS; ++q) {
      const int shift = BITS * lane - 32 * q;
      uint32_t part = 0;
      if (shift >= 0 && shift < 32) part = code[j] << shift;
      else if (shift < 0 && shift > -BITS) part = code[j] >> (-shift);
      const uint32_t word = __reduce_or_sync(FULL, part);
      if (lane == j * BITS + q) out_word = word;
    }
  }
  if (lane < W) dst[lane] = out_word;
}

// Quantize a warp-resident row (v[j] = x[j*32 + lane]) against the codebook
// c (nearest centroid) and store its packed words to dst.
template <int D, int BITS>
__device__ __forceinline__ void warp_pack_row(const float (&v)[D / 32], int lane, const float (&c)[1 << BITS],
                                              uint32_t* dst) {
  uint32_t code[D / 32];
#pragma unroll
  for (int j = 0; j < D / 32; ++j) code[j] = nearest_code<BITS>(v[j], c);
  warp_pack_codes<D, BITS>(code, lane, dst);
}

// Element i of a row of the given dtype (TQ_F32 / TQ_F16 / TQ_BF16).
__device__ __forceinline__ float load_as_f32(const void* x, int dtype, int64_t i) {
  if (dtype == TQ_F16) return __half2float(reinterpret_cast<const __half*>(x)[i]);
  if (dtype == TQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  return reinterpret_cast<const float*>(x)[i];
}

// Extract code `i` of a packed vector (LSB-first, may straddle two words).
template <int BITS>
__device__ __forceinline__ uint32_t code_at(const uint32_t* w, int i) {
  const int bit = i * BITS;
  const int wi = bit >> 5, sh = bit & 31;
  uint32_t v = w[wi] >> sh;
  if (sh + BITS > 32) v |= w[wi + 1] << (32 - sh);
  return v & ((1u << BITS) - 1u);
}

}  // namespace tq
