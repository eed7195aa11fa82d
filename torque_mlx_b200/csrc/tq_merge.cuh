// Split-K merge of one query row: the partials (o_i un-normalised, m_i in
// log2 units, l_i) of the row's parts become
//     M = max m_i,  w_i = 2^(m_i - M),  L = sum w_i l_i,  o = sum w_i o_i / L
// and, optionally, the inverse rotation; lse = (M + log2 L) ln 2.
//
// One CTA of T threads merges one row; the thread count is a template
// parameter so rows with many parts (long single sequences split over every
// SM) get more loads in flight.  The function starts and ends with a barrier
// so calls can follow each other.
#pragma once

#include "tq_common.cuh"

namespace tq {

constexpr int kMergeMaxParts = 1024;  // parts weighed in shared memory per row
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Shared memory a merge_row call needs (floats): weights, per-slice sums,
// per-warp reduction slots and the two row scalars.
template <int D, int T>
struct MergeSmem {
  static constexpr int SLICES = T / D;  // threads per output dim (parts split between them)
  static constexpr int FLOATS = 2 * kMergeMaxParts + T + T / 32 + 2;
};

// part row layout: [nparts][D + 2] = (o[0..D), m, l), read through L2
// (ld.global.cg: every partial is read once).  One global round trip: each
// thread issues the loads of its parts' (m, l) and, at the same time, of the
// first kPrefetch o values it will weigh; the weights are formed in shared
// memory once the row max is known, and only rows with more parts than the
// prefetch covers go back to global memory for the rest.
// Prefetch depth: enough o values per thread that a row of up to ~80 parts
// (a long sequence split over every SM) needs a single round trip.
template <int SLICES>
constexpr int merge_prefetch() { return SLICES >= 4 ? 20 : 32; }

template <int D, int T>
__device__ __forceinline__ void merge_row(const float* __restrict__ base, int nparts, float* __restrict__ out_row,
                                          float* lse_row, int inverse_rotate, const float* signs_left,
                                          const float* signs_right, float* smem) {
  static_assert(T % D == 0 || D % T == 0, "thread count and head dim must nest");
  static_assert(T >= D, "one thread per output dim at least");
  constexpr int E = D / 32;
  constexpr int NWARP = T / 32;
  constexpr int SLICES = MergeSmem<D, T>::SLICES;
  constexpr int kMergePrefetch = merge_prefetch<SLICES>();
  float* w_s = smem;                         // [kMergeMaxParts] m_i, then the weights
  float* acc_s = w_s + kMergeMaxParts;       // [SLICES][D]
  float* red = acc_s + T;                    // [NWARP]
  float* row_s = red + NWARP;                // M, L
  float* l_s = row_s + 2;                    // [kMergeMaxParts] l_i
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int np = nparts < kMergeMaxParts ? nparts : kMergeMaxParts;
  const int dim = tid % D, slice = tid / D;
  __syncthreads();  // smem may still be in use by the caller
  // warp 0 applies the inverse rotation at the end: its signs load now
  float sg_a[E], sg_b[E];
  if (inverse_rotate && warp == 0) {
    load_signs<D>(sg_a, signs_left, lane);
    load_signs<D>(sg_b, signs_right, lane);
  }

  // 1) loads in flight together: (m, l) of parts tid, tid + T, ... and the o
  //    values of parts slice, slice + SLICES, ... (the first kPrefetch)
  float ov[kMergePrefetch];
#pragma unroll
  for (int k = 0; k < kMergePrefetch; ++k) {
    const int i = slice + k * SLICES;
    ov[k] = i < np ? __ldcg(base + (int64_t)i * (D + 2) + dim) : 0.f;
  }
  float M = -INFINITY;
  for (int i = tid; i < np; i += T) {
    const float* pp = base + i * (int64_t)(D + 2);
    const float mi = __ldcg(pp + D), li = __ldcg(pp + D + 1);
    const bool seen = li > 0.f;
    w_s[i] = seen ? mi : -INFINITY;
    l_s[i] = li;
    if (seen) M = fmaxf(M, mi);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  // every warp reduces the per-warp maxima itself (no serial pass, no extra barrier)
  M = lane < NWARP ? red[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
  // 2) weights from shared memory, and the denominator
  float L = 0.f;
  for (int i = tid; i < np; i += T) {
    const float mi = w_s[i];
    const float w = (mi == -INFINITY || M == -INFINITY) ? 0.f : exp2f(mi - M);
    w_s[i] = w;
    L += l_s[i] * w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
  __syncthreads();  // every warp has read red[] and w_s is complete
  if (lane == 0) red[warp] = L;
  // 3) weighted sum over the prefetched values, then any remaining parts
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int k = 0; k < kMergePrefetch; k += 2) {
    const int i = slice + k * SLICES;
    if (i < np) a0 = fmaf(ov[k], w_s[i], a0);
    if (i + SLICES < np) a1 = fmaf(ov[k + 1], w_s[i + SLICES], a1);
  }
  {
    int i = slice + kMergePrefetch * SLICES;
    float a2 = 0.f, a3 = 0.f;
    for (; i + SLICES < np; i += 2 * SLICES) {
      a2 = fmaf(__ldcg(base + (int64_t)i * (D + 2) + dim), w_s[i], a2);
      a3 = fmaf(__ldcg(base + (int64_t)(i + SLICES) * (D + 2) + dim), w_s[i + SLICES], a3);
    }
    if (i < np) a2 = fmaf(__ldcg(base + (int64_t)i * (D + 2) + dim), w_s[i], a2);
    a0 += a2;
    a1 += a3;
  }
  acc_s[slice * D + dim] = a0 + a1;
  __syncthreads();
  if (warp == 0) {
    float Lsum = lane < NWARP ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) Lsum += __shfl_xor_sync(FULL, Lsum, o);
    float v[E];
#pragma unroll
    for (int j = 0; j < E; ++j) {
      float a = 0.f;
#pragma unroll
      for (int sl = 0; sl < SLICES; ++sl) a += acc_s[sl * D + j * 32 + lane];
      v[j] = M == -INFINITY ? 0.f : a / Lsum;
    }
    if (inverse_rotate) warp_rotate_regs<D>(v, lane, sg_a, sg_b);
#pragma unroll
    for (int j = 0; j < E; ++j) out_row[j * 32 + lane] = v[j];
    if (lse_row && lane == 0) *lse_row = (M == -INFINITY) ? -INFINITY : (M + log2f(Lsum)) * kLn2;
  }
  __syncthreads();
}


}  // namespace tq
