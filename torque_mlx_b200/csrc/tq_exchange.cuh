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

#ifdef TQ_TRACE
static __device__ unsigned long long g_trace_mrg[4096 * 4];
#define TQ_MSTAMP(k) TQ_STAMP(g_trace_mrg, (blockIdx.x % 4096) * 4 + (k))
#else
#define TQ_MSTAMP(k) do { } while (0)
#endif

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
  constexpr int NWARP = T / 32;
  constexpr int64_t RF = exchange_row_floats(D);
  __shared__ float sm[MergeSmem<D, T>::FLOATS];
  __shared__ float xs[kExchangeMaxWorld * (D + 1)];  // every rank's [o | lse] for this row
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  TQ_MSTAMP(0);
  // the next step's decode grid may be scheduled now (it waits for this grid)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid's partials are complete
  TQ_MSTAMP(1);
  const int64_t row = blockIdx.x;
  const uint32_t e = (uint32_t)x.epoch[row] + 1u;
  const int par = (int)(e & 1u);
  float* own = x.bufs[x.rank];
  const int64_t data = exchange_data_floats(D, x.world, rows);
  float* slot0 = own + (par * (int64_t)x.world * rows + row) * RF;  // rank r's slot: slot0 + r * rows * RF

  // 1. this rank's partial into its own slot
  float* mine = slot0 + (int64_t)x.rank * rows * RF;
  merge_row<D, T>(part + row * nparts * (int64_t)(D + 2), nparts, mine, mine + D, 0, nullptr, nullptr, sm);
  // (merge_row ends with a barrier: the slot is complete and visible in the CTA)

  // warp 0 applies the inverse rotation at the end: its signs load now, in
  // flight during the exchange
  float sg_a[E], sg_b[E];
  if (inverse_rotate && warp == 0) {
    load_signs<D>(sg_a, signs_left, lane);
    load_signs<D>(sg_b, signs_right, lane);
  }
  if (tid == 0) s_ok = 1;
  if (x.world > 1) {
    // 2. warp p copies the slot to peer p (one warp per peer, all at once),
    //    makes its stores visible system-wide; after a barrier one thread
    //    per rank publishes the epoch to that rank's flag of this row
    for (int pr = warp; pr < x.world; pr += NWARP) {
      if (pr == x.rank) continue;
      float* dst = x.bufs[pr] + ((par * (int64_t)x.world + x.rank) * rows + row) * RF;
      for (int i = lane; i < D + 1; i += 32) dst[i] = __ldcg(mine + i);
      __threadfence_system();
    }
    __syncthreads();
    if (tid < x.world) {
      uint32_t* flags = reinterpret_cast<uint32_t*>(x.bufs[tid] + data);
      st_release_sys(flags + (int64_t)x.rank * rows + row, e);
    }
    TQ_MSTAMP(2);
    // 3. wait for every peer's slot in this buffer (bounded)
    if (tid < x.world && tid != x.rank) {
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
  }
  __syncthreads();

  // 4. every rank's row into shared memory in one round trip (warp r reads
  //    rank r), then warp 0 merges them by log-sum-exp
  if (s_ok) {
    for (int r = warp; r < x.world; r += NWARP) {
      const float* o = slot0 + (int64_t)r * rows * RF;
      for (int i = lane; i < D + 1; i += 32) xs[r * (D + 1) + i] = __ldcg(o + i);
    }
  }
  __syncthreads();
  if (warp == 0) {
    float v[E];
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = 0.f;
    float M = -INFINITY, tot = 0.f;
    if (s_ok) {
      const float sl = lane < x.world ? xs[lane * (D + 1) + D] : -INFINITY;
      M = sl;
#pragma unroll
      for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
      if (M != -INFINITY) {
        const float wl = sl == -INFINITY ? 0.f : expf(sl - M);
        for (int r = 0; r < x.world; ++r) {
          const float w = __shfl_sync(FULL, wl, r);
          tot += w;
          if (w == 0.f) continue;
#pragma unroll
          for (int j = 0; j < E; ++j) v[j] = fmaf(xs[r * (D + 1) + j * 32 + lane], w, v[j]);
        }
        const float inv = 1.f / tot;
#pragma unroll
        for (int j = 0; j < E; ++j) v[j] *= inv;
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = __int_as_float(0x7fc00000);  // NaN: a peer never arrived
    }
    if (inverse_rotate) warp_rotate_regs<D>(v, lane, sg_a, sg_b);
#pragma unroll
    for (int j = 0; j < E; ++j) out[row * D + j * 32 + lane] = v[j];
    if (lse && lane == 0) lse[row] = (!s_ok || M == -INFINITY) ? -INFINITY : M + logf(tot);
    if (lane == 0) x.epoch[row] = (int32_t)e;
  }
  if (advance && row == 0)
    for (int64_t i = tid; i < advance_n; i += T) advance[i] += 1;
  TQ_MSTAMP(3);
}

}  // namespace tq
