// Sequence-shard exchange fused with the split merge (multi-GPU decode of one
// long sequence whose tokens are spread over the ranks).
//
// One CTA per query row.  It
//   1. merges the row's local split partials (o, m, l) into this rank's
//      normalised partial (o_r, lse_r)  (merge_row, tq_merge.cuh);
//   2. stores [o_r | lse_r] into slot [parity][rank][row] of EVERY rank's
//      exchange buffer over NVLink (plain peer stores, cudaIpc mappings), then
//      publishes it with a system-scope release store of the step's epoch to
//      flag [rank][row] of each buffer;
//   3. waits (acquire loads, bounded by %globaltimer) until every rank's flag
//      for this row in its own buffer has reached the epoch;
//   4. merges the world's partials by log-sum-exp, rotates back by Pi^T if
//      asked, and writes the row and its lse.
// The epoch of a row is a per-rank device counter (one per row, owned by that
// row's CTA), so a captured step replays without host arguments.  Slots are
// double-buffered by epoch parity: a rank can be at most one step ahead of a
// peer (it cannot finish step e+1 before the peer has published e+1, which
// the peer does only after its step e), so the slot a peer may be writing is
// never the one being read.
//
// Exchange buffer of one rank (floats, 16-byte aligned):
//   data  [2][world][rows][D + 4]   (o[0..D), lse, pad)
//   flags [world][rows] uint32      (after the data)
#pragma once

#include "tq_common.cuh"
#include "tq_merge.cuh"

namespace tq {

constexpr int kExchangeMaxWorld = 16;

__host__ __device__ constexpr int64_t exchange_row_floats(int D) { return D + 4; }

__host__ __device__ inline int64_t exchange_data_floats(int D, int world, int64_t rows) {
  return 2 * (int64_t)world * rows * exchange_row_floats(D);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ExchangeParams {
  float* const* bufs;     // [world] exchange buffers (index rank = this rank's own), device array
  int rank, world;
  int32_t* epoch;         // [rows] this rank's step counters
  int64_t timeout_ns;     // bound of each wait
  int32_t* status;        // set to TQ_E_TIMEOUT when a wait gives up (never cleared here)
};

template <int D, int T>
__global__ void __launch_bounds__(T)
exchange_merge_kernel(const float* __restrict__ part, int nparts, int64_t rows, ExchangeParams x,
                      float* __restrict__ out, float* __restrict__ lse, int inverse_rotate,
                      const float* __restrict__ signs_left, const float* __restrict__ signs_right,
                      int32_t* __restrict__ advance, int64_t advance_n) {
  constexpr int E = D / 32;
  constexpr int64_t RF = exchange_row_floats(D);
  __shared__ float sm[MergeSmem<D, T>::FLOATS];
  __shared__ int s_ok;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid's partials are complete
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const uint32_t e = (uint32_t)x.epoch[row] + 1u;
  const int par = (int)(e & 1u);
  float* own = x.bufs[x.rank];
  const int64_t data = exchange_data_floats(D, x.world, rows);

  // 1. this rank's partial into its own slot
  float* mine = own + ((par * (int64_t)x.world + x.rank) * rows + row) * RF;
  merge_row<D, T>(part + row * nparts * (int64_t)(D + 2), nparts, mine, mine + D, 0, nullptr, nullptr, sm);
  // (merge_row ends with a barrier: the slot is complete and visible in the CTA)

  // 2. warp 0 copies it to every peer, makes its stores visible system-wide
  //    and publishes (the other warps go straight to the wait)
  if (tid < 32) {
    for (int p = 0; p < x.world; ++p) {
      if (p == x.rank) continue;
      float* dst = x.bufs[p] + ((par * (int64_t)x.world + x.rank) * rows + row) * RF;
      for (int i = tid; i < D + 1; i += 32) dst[i] = mine[i];
    }
    if (x.world > 1) __threadfence_system();
    __syncwarp();
    if (tid < x.world) {
      uint32_t* flags = reinterpret_cast<uint32_t*>(x.bufs[tid] + data);
      st_release_sys(flags + (int64_t)x.rank * rows + row, e);
    }
  }

  // 3. wait for every rank's slot in this buffer (bounded)
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < x.world) {
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(own + data) + (int64_t)tid * rows + row;
    const uint64_t t0 = global_timer_ns();
    // (int32_t)(v - e) >= 0: the flag reached e (epochs are compared modulo 2^32)
    while ((int32_t)(ld_acquire_sys(flag) - e) < 0) {
      if ((int64_t)(global_timer_ns() - t0) > x.timeout_ns) {
        s_ok = 0;
        atomicExch(x.status, TQ_E_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();

  // 4. log-sum-exp merge of the world's partials (warp 0)
  if (tid < 32) {
    const int lane = tid;
    float v[E];
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = 0.f;
    float M = -INFINITY, tot = 0.f;
    if (s_ok) {
      const float* base = own + (par * (int64_t)x.world * rows + row) * RF;
      for (int r = 0; r < x.world; ++r) M = fmaxf(M, __ldcv(base + (int64_t)r * rows * RF + D));
      if (M != -INFINITY) {
        for (int r = 0; r < x.world; ++r) {
          const float* o = base + (int64_t)r * rows * RF;
          const float s = __ldcv(o + D);
          if (s == -INFINITY) continue;
          const float w = expf(s - M);
          tot += w;
#pragma unroll
          for (int j = 0; j < E; ++j) v[j] = fmaf(__ldcv(o + j * 32 + lane), w, v[j]);
        }
        const float inv = 1.f / tot;
#pragma unroll
        for (int j = 0; j < E; ++j) v[j] *= inv;
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = __int_as_float(0x7fc00000);  // NaN: a peer never arrived
    }
    if (inverse_rotate) warp_rotate<D>(v, lane, signs_left, signs_right);
#pragma unroll
    for (int j = 0; j < E; ++j) out[row * D + j * 32 + lane] = v[j];
    if (lse && lane == 0) lse[row] = (!s_ok || M == -INFINITY) ? -INFINITY : M + logf(tot);
    if (lane == 0) x.epoch[row] = (int32_t)e;
  }
  if (advance && row == 0)
    for (int64_t i = tid; i < advance_n; i += T) advance[i] += 1;
}

}  // namespace tq
