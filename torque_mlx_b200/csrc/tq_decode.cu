// Packed-code decode attention (q_len = 1, grouped queries) and the
// log-sum-exp merges.
//
// Split-K ("flash-decoding") structure: the grid is (splits, units); a CTA
// streams one contiguous token chunk of one (seq, layer, kv_head) unit and
// serves all G query heads of that kv head from the same code bytes.  Each
// warp leaves an online-softmax partial (o, m, l) in the workspace; a merge
// kernel combines the partials of a query row, normalises, optionally
// rotates the row back by Pi^T and emits the log-sum-exp.
//
// Two compute variants share that skeleton:
//   * exact  — fp32 CUDA-core math with fp32 centroids and query;
//   * tensor — mma.sync m16n8k16 with fp16 operands (see tq_decode_mma.cuh).
#include "tq_common.cuh"
#include "tq_decode_mma.cuh"  // DecodeParams, kMma*
#include "tq_merge.cuh"
#include "tq_exchange.cuh"

#include <math.h>
#include <mutex>

namespace tq {

constexpr int kExactWarps = 4;

// ---------------------------------------------------------------------------
// exact fp32 kernel
//   score phase: lane = token of a 32-token tile, loop over dims;
//   value phase: lane = dims {lane + 32 i}, loop over the tile's tokens.
// ---------------------------------------------------------------------------
template <int D, int BITS, int GM>
__global__ void __launch_bounds__(kExactWarps * 32)
decode_exact_kernel(DecodeParams p) {
  constexpr int W = D * BITS / 32;
  constexpr int E = D / 32;
  constexpr int L = 1 << BITS;
  __shared__ float q_s[GM][D];
  __shared__ uint32_t tile_s[kExactWarps][32][W + 1];
  __shared__ float p_s[kExactWarps][32][GM];
  __shared__ float ck_s[L], cv_s[L];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u = blockIdx.y;
  const int split = blockIdx.x;
  const int G = p.G;

  if (threadIdx.x < L) {
    ck_s[threadIdx.x] = p.cent_k[threadIdx.x];
    cv_s[threadIdx.x] = p.cent_v[threadIdx.x];
  }
  for (int g = warp; g < GM; g += kExactWarps) {
    float v[E];
    if (g < G) {
      const float* q = p.query + (u * G + g) * D;
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = q[j * 32 + lane];
      if (p.rotate_query) warp_rotate<D>(v, lane, p.signs_right, p.signs_left);
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < E; ++j) q_s[g][j * 32 + lane] = v[j];
  }
  __syncthreads();

  const int64_t n = unit_length(p, u);
  const int64_t c0 = (int64_t)split * p.chunk;
  const int64_t c1 = min(c0 + (int64_t)p.chunk, n);
  const uint32_t* kbase = p.k_slab + u * p.unit_stride;
  const uint32_t* vbase = p.v_slab + u * p.unit_stride;

  float m[GM], l[GM], acc[GM][E];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) acc[g][i] = 0.f;
  }

  for (int64_t t0 = c0 + warp * 32; t0 < c1; t0 += kExactWarps * 32) {
    const int nt = (int)min((int64_t)32, c1 - t0);
    // ---- stage K words of the tile (coalesced) ----
    for (int i = lane; i < nt * W; i += 32) tile_s[warp][i / W][i % W] = kbase[(t0 + i / W) * W + i % W];
    __syncwarp();
    float s[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) s[g] = 0.f;
    if (lane < nt) {
      uint32_t r[W + 1];
#pragma unroll
      for (int w = 0; w < W; ++w) r[w] = tile_s[warp][lane][w];
      r[W] = 0;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const float c = ck_s[code_at<BITS>(r, d)];
#pragma unroll
        for (int g = 0; g < GM; ++g) s[g] = fmaf(q_s[g][d], c, s[g]);
      }
    }
    // ---- online softmax over the tile ----
    float alpha[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float sc = lane < nt ? s[g] * p.scale_log2 : -INFINITY;
      float tm = sc;
#pragma unroll
      for (int o = 16; o; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, o));
      const float mn = fmaxf(m[g], tm);
      alpha[g] = exp2f(m[g] - mn);  // m = -inf on the first tile -> 0
      const float pr = lane < nt ? exp2f(sc - mn) : 0.f;
      float ps = pr;
#pragma unroll
      for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(FULL, ps, o);
      l[g] = l[g] * alpha[g] + ps;
      m[g] = mn;
      p_s[warp][lane][g] = pr;
    }
    __syncwarp();
    // ---- stage V words, accumulate P.V ----
    for (int i = lane; i < nt * W; i += 32) tile_s[warp][i / W][i % W] = vbase[(t0 + i / W) * W + i % W];
    __syncwarp();
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
      for (int i = 0; i < E; ++i) acc[g][i] *= alpha[g];
    for (int t = 0; t < nt; ++t) {
      const uint32_t* row = tile_s[warp][t];
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int dim = lane + 32 * i;
        const int bit = dim * BITS, wi = bit >> 5, sh = bit & 31;
        uint32_t cv = row[wi] >> sh;
        if (sh + BITS > 32) cv |= row[wi + 1] << (32 - sh);
        const float c = cv_s[cv & (L - 1)];
#pragma unroll
        for (int g = 0; g < GM; ++g) acc[g][i] = fmaf(p_s[warp][t][g], c, acc[g][i]);
      }
    }
    __syncwarp();
  }

  // ---- this warp's partial ----
  const int nparts = p.splits * kExactWarps;
  const int part = split * kExactWarps + warp;
  for (int g = 0; g < G && g < GM; ++g) {
    float* dst = p.part + ((u * G + g) * nparts + part) * (int64_t)(D + 2);
#pragma unroll
    for (int i = 0; i < E; ++i) dst[lane + 32 * i] = acc[g][i];
    if (lane == 0) {
      dst[D] = m[g];
      dst[D + 1] = l[g];
    }
  }
}

// ---------------------------------------------------------------------------
// merge the split partials (o unnormalised, m in log2 units, l) of each query
// row; optional inverse rotation.  One CTA per row: its warps take the parts
// round-robin, so rows with many splits (long single sequences) merge in
// parallel instead of one warp walking every part.
// ---------------------------------------------------------------------------
// Rows with many parts (a few long units split over every SM) merge with
// 1024 threads a row, so each thread walks few parts; rows with a handful of
// parts (batched decode) with 256.
constexpr int kMergeWarps = 8;
constexpr int kMergeWarpsWide = 32;
constexpr int kMergeWideParts = 64;

// advance (nullable): lengths[0..advance_n) += 1 once the step's decode is
// complete (tq_decode_append), so the lengths the decode read stay put while
// it runs.
template <int D, int T>
__global__ void __launch_bounds__(T)
merge_partials_kernel(const float* __restrict__ part, int nparts, int64_t rows,
                      float* __restrict__ out, float* __restrict__ lse, int inverse_rotate,
                      const float* __restrict__ signs_left, const float* __restrict__ signs_right,
                      int32_t* __restrict__ advance, int64_t advance_n) {
  __shared__ float sm[MergeSmem<D, T>::FLOATS];
  // launched as a programmatic dependent of the decode kernel: wait for its
  // whole grid (and its memory) before reading a partial
  TQ_MSTAMP(0);
  // the next step's decode grid may be scheduled now; it waits for this grid
  // to complete before it reads or writes global memory
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  TQ_MSTAMP(1);
  const int64_t row = blockIdx.x;
  merge_row<D, T>(part + row * nparts * (int64_t)(D + 2), nparts, out + row * D, lse ? lse + row : nullptr,
                  inverse_rotate, signs_left, signs_right, sm);
  TQ_MSTAMP(2);
  if (advance && row == 0)
    for (int64_t i = threadIdx.x; i < advance_n; i += T) advance[i] += 1;
  TQ_MSTAMP(3);
}

// ---------------------------------------------------------------------------
// merge normalised parts with natural-log lse (multi-GPU sequence shards)
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256)
lse_merge_kernel(const float* __restrict__ outs, const float* __restrict__ lses, int parts,
                 int64_t rows, float* __restrict__ out, float* __restrict__ lse_out,
                 int inverse_rotate, const float* __restrict__ signs_left,
                 const float* __restrict__ signs_right) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float M = -INFINITY;
  for (int i = lane; i < parts; i += 32) M = fmaxf(M, lses[i * rows + row]);
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = 0.f;
  float tot = 0.f;
  if (M != -INFINITY) {
    for (int i = 0; i < parts; ++i) {
      const float s = lses[i * rows + row];
      if (s == -INFINITY) continue;
      const float w = expf(s - M);
      tot += w;
      const float* o = outs + (i * rows + row) * (int64_t)D;
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = fmaf(o[j * 32 + lane], w, v[j]);
    }
    const float inv = 1.f / tot;
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] *= inv;
  }
  if (inverse_rotate) warp_rotate<D>(v, lane, signs_left, signs_right);
#pragma unroll
  for (int j = 0; j < E; ++j) out[row * D + j * 32 + lane] = v[j];
  if (lse_out && lane == 0) lse_out[row] = (M == -INFINITY) ? -INFINITY : M + logf(tot);
}

// ---------------------------------------------------------------------------
// host-side planning
// ---------------------------------------------------------------------------
struct Plan {
  int mode;       // resolved: exact or tensor
  int nw;        // warps per CTA (tensor kernel)
  int chunk;      // tokens per CTA
  int splits;     // CTAs per unit
  int warps;      // partials per CTA
  size_t bytes;   // workspace
};

// The tensor-core kernel reads 16-byte blocks of the slabs: it needs both
// slabs 16-byte aligned and a unit stride of whole 16-byte blocks.
static bool slabs_aligned(const void* k_slab, const void* v_slab, int64_t unit_stride_words) {
  return ((uintptr_t)k_slab % 16 == 0) && ((uintptr_t)v_slab % 16 == 0) && (unit_stride_words % 4 == 0);
}

static int resolve_mode(int mode, int G) {
  if (mode == TQ_DECODE_AUTO) return G >= 2 ? TQ_DECODE_TENSOR : TQ_DECODE_EXACT;
  return mode;
}

static int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) {
    cudaGetLastError();
    sms = 148;  // B200
  }
  return sms;
}

// Split planning.  Few units (long single sequences): one full wave of
// resident CTAs, so every SM streams and each CTA's fixed cost (tables,
// query rotation, merge) is paid once.  Many units (batched decode): about
// four waves, so ragged lengths balance across SMs.
static Plan make_plan(int64_t units, int G, int D, int bits, int64_t max_len, int mode) {
  Plan pl;
  pl.mode = resolve_mode(mode, G);
  pl.warps = pl.mode == TQ_DECODE_TENSOR ? 1 : kExactWarps;  // partials per CTA
  const int sms = sm_count();
  // d <= 128: 16-warp CTAs (one per SM, the pair tables built once per SM)
  // for batched decode (at least two units per SM) and for a few long units
  // (at most SMs/8, each split over >= 8 SMs); in between, 8-warp CTAs (two
  // per SM) spread the units over more SMs.
  // Short caches (< 4096 tokens) with few units stay on 8-warp CTAs: each
  // split is then one or two tiles a warp and the wider CTA's table build and
  // merge do not pay (measured on the 28-layer decoder's ~1K-token layers).
  const bool wide_ok = pl.mode == TQ_DECODE_TENSOR && D <= 128;
  const bool batched = units >= 2 * (int64_t)sms;
  pl.nw = (wide_ok && (batched || (units * 8 <= (int64_t)sms && max_len >= 4096))) ? kMmaWarpsWide : kMmaWarps;
  const int tile = pl.mode == TQ_DECODE_TENSOR ? pl.nw * 16 : kExactWarps * 32;
  const int per_sm = pl.mode == TQ_DECODE_TENSOR ? mma_blocks_per_sm(D, bits, G, pl.nw) : 4;
  const int64_t wave = (int64_t)sms * per_sm;
  const int64_t len = max_len < 1 ? 1 : max_len;
  const int64_t uu = units < 1 ? 1 : units;
  // few units: as many splits as keep every unit's CTAs inside one wave
  // (rounding up would leave a nearly empty second wave); many units: about
  // four waves of CTAs so the ragged tails even out
  int64_t splits = uu < wave ? wave / uu : (4 * wave + uu - 1) / uu;
  // (a single-split plan - one tile range per unit - writes its rows from
  // the decode kernel; fewer, longer splits were measured slower than the
  // merge launch they save)
  const int64_t max_splits = (len + tile - 1) / tile;
  if (splits > max_splits) splits = max_splits;
  if (splits * pl.warps > kMergeMaxParts) splits = kMergeMaxParts / pl.warps;  // merge weighs parts in smem
  if (splits < 1) splits = 1;
  int64_t chunk = (len + splits - 1) / splits;
  chunk = (chunk + tile - 1) / tile * tile;
  pl.chunk = (int)chunk;
  pl.splits = (int)((len + chunk - 1) / chunk);
  pl.bytes = (size_t)units * G * pl.splits * pl.warps * (size_t)(D + 2) * sizeof(float);
  return pl;
}

template <int D, int BITS>
static void launch_exact(const DecodeParams& p, cudaStream_t st) {
  dim3 grid(p.splits, (unsigned)p.units);
  if (p.G <= 1) decode_exact_kernel<D, BITS, 1><<<grid, kExactWarps * 32, 0, st>>>(p);
  else if (p.G <= 2) decode_exact_kernel<D, BITS, 2><<<grid, kExactWarps * 32, 0, st>>>(p);
  else if (p.G <= 4) decode_exact_kernel<D, BITS, 4><<<grid, kExactWarps * 32, 0, st>>>(p);
  else if (p.G <= 8) decode_exact_kernel<D, BITS, 8><<<grid, kExactWarps * 32, 0, st>>>(p);
  else decode_exact_kernel<D, BITS, 16><<<grid, kExactWarps * 32, 0, st>>>(p);
}

template <int D>
static void launch_decode_d(int bits, int mode, const DecodeParams& p, cudaStream_t st) {
  if (mode == TQ_DECODE_TENSOR) {
    launch_mma_dispatch(D, bits, p, st);
  } else {
    if (bits == 2) launch_exact<D, 2>(p, st);
    else if (bits == 3) launch_exact<D, 3>(p, st);
    else launch_exact<D, 4>(p, st);
  }
}

// The merge launches as a programmatic dependent of the decode kernel
// (griddepcontrol): its CTAs are scheduled as the decode CTAs retire instead
// of after the whole grid has drained, and each waits for the decode grid's
// completion before reading a partial.
template <typename... KArgs, typename... Args>
static void launch_dependent(void (*kernel)(KArgs...), unsigned grid, unsigned block, cudaStream_t st,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int D>
static void launch_merge(const float* part, int nparts, int64_t rows, float* out, float* lse,
                         int inv, const float* sl, const float* sr, int32_t* adv, int64_t adv_n,
                         cudaStream_t st) {
  if (nparts >= kMergeWideParts)
    launch_dependent(merge_partials_kernel<D, kMergeWarpsWide * 32>, (unsigned)rows, kMergeWarpsWide * 32, st,
                     part, nparts, rows, out, lse, inv, sl, sr, adv, adv_n);
  else
    launch_dependent(merge_partials_kernel<D, kMergeWarps * 32>, (unsigned)rows, kMergeWarps * 32, st,
                     part, nparts, rows, out, lse, inv, sl, sr, adv, adv_n);
}

template <int D>
static void launch_exchange(const float* part, int nparts, int64_t rows, const ExchangeParams& x, float* out,
                            float* lse, int inv, const float* sl, const float* sr, int32_t* adv, int64_t adv_n,
                            cudaStream_t st) {
  if (nparts >= kMergeWideParts)
    launch_dependent(exchange_merge_kernel<D, kMergeWarpsWide * 32>, (unsigned)rows, kMergeWarpsWide * 32, st,
                     part, nparts, rows, x, out, lse, inv, sl, sr, adv, adv_n);
  else
    launch_dependent(exchange_merge_kernel<D, kMergeWarps * 32>, (unsigned)rows, kMergeWarps * 32, st,
                     part, nparts, rows, x, out, lse, inv, sl, sr, adv, adv_n);
}

// The new token of a fused append-and-decode step (tq_decode_append).
struct StepAppend {
  const void* k;
  const void* v;
  int dtype;
  int rotate_k, rotate_v;
  int32_t* lengths;  // writable lengths (advanced by the merge when advance != 0)
  int advance;
};

}  // namespace tq

using namespace tq;

extern "C" {

int tq_decode_workspace_size(int64_t units, int group_size, int head_dim, int bits, int64_t max_len,
                             int mode, size_t* bytes) {
  if (!bytes) return TQ_E_ARG;
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (units < 0 || group_size < 1 || group_size > 16 || max_len < 0) return TQ_E_SHAPE;
  if (mode < TQ_DECODE_AUTO || mode > TQ_DECODE_TENSOR) return TQ_E_ARG;
  size_t need = make_plan(units, group_size, head_dim, bits, max_len, mode).bytes;
  // AUTO takes the exact kernel when the slabs are not 16-byte aligned (the
  // pointers are not known here), so it reports enough for either plan.
  if (mode == TQ_DECODE_AUTO) {
    const size_t exact = make_plan(units, group_size, head_dim, bits, max_len, TQ_DECODE_EXACT).bytes;
    if (exact > need) need = exact;
  }
  *bytes = need;
  return TQ_OK;
}

}  // extern "C"

namespace tq {

static int decode_core(const float* query, int rotate_query, const float* signs_left,
                       const float* signs_right, const uint32_t* k_slab, const uint32_t* v_slab,
                       int64_t unit_stride_words, const int32_t* lengths, int units_per_seq,
                       int64_t len_offset, int64_t max_len, int64_t units, int group_size, int head_dim,
                       int bits, const float* cent_k, const float* cent_v, float scale, float* out,
                       float* lse, int inverse_rotate_output, int mode, void* workspace,
                       size_t workspace_bytes, tq_stream_t stream, const StepAppend* app,
                       const ExchangeParams* xch = nullptr, int q_tokens = 1) {
  if (!valid_bits(bits)) return TQ_E_BITS;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (units < 0 || group_size < 1 || group_size > 16 || max_len < 0) return TQ_E_SHAPE;
  if (mode < TQ_DECODE_AUTO || mode > TQ_DECODE_TENSOR) return TQ_E_ARG;
  if (units == 0) return TQ_OK;
  if (!query || !k_slab || !v_slab || !cent_k || !cent_v || !out) return TQ_E_ARG;
  if ((rotate_query || inverse_rotate_output) && (!signs_left || !signs_right)) return TQ_E_ARG;
  if (lengths && units_per_seq <= 0) return TQ_E_ARG;
  const int W = words_for(head_dim, bits);
  if (unit_stride_words < max_len * W) return TQ_E_SHAPE;
  // the bulk-copy engine needs 16-byte aligned rows of whole 16-byte blocks
  if (!slabs_aligned(k_slab, v_slab, unit_stride_words)) {
    if (mode == TQ_DECODE_TENSOR) return TQ_E_SHAPE;
    mode = TQ_DECODE_EXACT;
  }
  if (q_tokens > 1) {
    if (mode == TQ_DECODE_EXACT) return TQ_E_ARG;  // the causal chunk runs on the tensor-core kernel
    mode = TQ_DECODE_TENSOR;
  }
  const Plan pl = make_plan(units, group_size, head_dim, bits, max_len, mode);
  if (!workspace || workspace_bytes < pl.bytes) return TQ_E_WORKSPACE;
  if (units > 65535) return TQ_E_SHAPE;  // grid.y limit

  DecodeParams p;
  p.query = query;
  p.rotate_query = rotate_query;
  p.signs_left = signs_left;
  p.signs_right = signs_right;
  p.k_slab = k_slab;
  p.v_slab = v_slab;
  p.unit_stride = unit_stride_words;
  p.lengths = lengths;
  p.units_per_seq = units_per_seq;
  p.len_offset = len_offset;
  p.max_len = max_len;
  p.units = units;
  p.G = group_size;
  p.cent_k = cent_k;
  p.cent_v = cent_v;
  p.scale_log2 = scale * kLog2e;
  p.chunk = pl.chunk;
  p.nw = pl.nw;
  p.splits = pl.splits;
  p.part = (float*)workspace;
  p.new_k = p.new_v = nullptr;
  p.new_dtype = TQ_F32;
  p.rotate_new_k = p.rotate_new_v = 0;
  p.k_slab_w = p.v_slab_w = nullptr;
  // a single-split tensor plan writes the final rows from the decode kernel
  const bool direct = pl.mode == TQ_DECODE_TENSOR && pl.splits == 1 && !xch;
  p.out = direct ? out : nullptr;
  p.lse = direct ? lse : nullptr;
  p.inverse_rotate = inverse_rotate_output;
  p.q_tokens = q_tokens;
  p.heads = group_size / (q_tokens > 0 ? q_tokens : 1);

  cudaStream_t st = (cudaStream_t)stream;
  if (app) {
    if (pl.mode == TQ_DECODE_TENSOR) {
      // packed inside the decode kernel by the CTA that owns the position
      p.new_k = app->k;
      p.new_v = app->v;
      p.new_dtype = app->dtype;
      p.rotate_new_k = app->rotate_k;
      p.rotate_new_v = app->rotate_v;
      p.k_slab_w = const_cast<uint32_t*>(k_slab);
      p.v_slab_w = const_cast<uint32_t*>(v_slab);
    } else {
      // the exact kernel reads the token through the append kernel's output
      uint32_t* ks = const_cast<uint32_t*>(k_slab);
      uint32_t* vs = const_cast<uint32_t*>(v_slab);
      int s0 = app->rotate_k == app->rotate_v
                   ? tq_append_kv(app->k, app->v, app->dtype, units, 1, head_dim, bits, signs_left, signs_right,
                                  app->rotate_k, cent_k, cent_v, ks, vs, unit_stride_words, max_len, lengths,
                                  units_per_seq, len_offset - 1, stream)
                   : tq_append_kv(app->k, nullptr, app->dtype, units, 1, head_dim, bits, signs_left, signs_right,
                                  app->rotate_k, cent_k, cent_v, ks, vs, unit_stride_words, max_len, lengths,
                                  units_per_seq, len_offset - 1, stream);
      if (s0 == TQ_OK && app->rotate_k != app->rotate_v)
        s0 = tq_append_kv(app->v, nullptr, app->dtype, units, 1, head_dim, bits, signs_left, signs_right,
                          app->rotate_v, cent_v, cent_v, vs, vs, unit_stride_words, max_len, lengths,
                          units_per_seq, len_offset - 1, stream);
      if (s0 != TQ_OK) return s0;
    }
  }
  if (head_dim == 64) launch_decode_d<64>(bits, pl.mode, p, st);
  else if (head_dim == 128) launch_decode_d<128>(bits, pl.mode, p, st);
  else launch_decode_d<256>(bits, pl.mode, p, st);
  int s = launch_status();
  if (s != TQ_OK) return s;

  int32_t* adv = (app && app->advance) ? app->lengths : nullptr;
  const int64_t adv_n = units / (units_per_seq > 0 ? units_per_seq : 1);
  if (direct) return adv ? tq_lengths_add(adv, (int)adv_n, 1, stream) : TQ_OK;
  const int nparts = pl.splits * pl.warps;
  const int64_t rows = units * group_size;
  if (xch) {
    if (head_dim == 64) launch_exchange<64>(p.part, nparts, rows, *xch, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
    else if (head_dim == 128) launch_exchange<128>(p.part, nparts, rows, *xch, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
    else launch_exchange<256>(p.part, nparts, rows, *xch, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
    return launch_status();
  }
  if (head_dim == 64) launch_merge<64>(p.part, nparts, rows, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
  else if (head_dim == 128) launch_merge<128>(p.part, nparts, rows, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
  else launch_merge<256>(p.part, nparts, rows, out, lse, inverse_rotate_output, signs_left, signs_right, adv, adv_n, st);
  return launch_status();
}

}  // namespace tq

extern "C" {

int tq_decode(const float* query, int rotate_query, const float* signs_left,
              const float* signs_right, const uint32_t* k_slab, const uint32_t* v_slab,
              int64_t unit_stride_words, const int32_t* lengths, int units_per_seq,
              int64_t len_offset, int64_t max_len, int64_t units, int group_size, int head_dim,
              int bits, const float* cent_k, const float* cent_v, float scale, float* out,
              float* lse, int inverse_rotate_output, int mode, void* workspace,
              size_t workspace_bytes, tq_stream_t stream) {
  return decode_core(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                     units_per_seq, len_offset, max_len, units, group_size, head_dim, bits, cent_k, cent_v, scale,
                     out, lse, inverse_rotate_output, mode, workspace, workspace_bytes, stream, nullptr);
}

int tq_decode_append(const void* new_k, const void* new_v, int kv_dtype, int rotate_k, int rotate_v,
                     int advance, const float* query, int rotate_query, const float* signs_left,
                     const float* signs_right, uint32_t* k_slab, uint32_t* v_slab,
                     int64_t unit_stride_words, int32_t* lengths, int units_per_seq, int64_t max_len,
                     int64_t units, int group_size, int head_dim, int bits, const float* cent_k,
                     const float* cent_v, float scale, float* out, float* lse,
                     int inverse_rotate_output, int mode, void* workspace, size_t workspace_bytes,
                     tq_stream_t stream) {
  if (!new_k || !new_v || !lengths) return TQ_E_ARG;
  if (kv_dtype != TQ_F32 && kv_dtype != TQ_F16 && kv_dtype != TQ_BF16) return TQ_E_ARG;
  if ((rotate_k || rotate_v) && (!signs_left || !signs_right)) return TQ_E_ARG;
  StepAppend app{new_k, new_v, kv_dtype, rotate_k, rotate_v, lengths, advance};
  return decode_core(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                     units_per_seq, 1, max_len, units, group_size, head_dim, bits, cent_k, cent_v, scale, out, lse,
                     inverse_rotate_output, mode, workspace, workspace_bytes, stream, &app);
}

int tq_exchange_buffer_bytes(int head_dim, int world, int64_t rows, size_t* bytes) {
  if (!bytes) return TQ_E_ARG;
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (world < 1 || world > kExchangeMaxWorld || rows < 0) return TQ_E_SHAPE;
  const size_t data = (size_t)exchange_data_floats(head_dim, world, rows) * sizeof(float);
  const size_t flags = ((size_t)world * rows * sizeof(uint32_t) + 15) / 16 * 16;
  *bytes = data + flags;
  return TQ_OK;
}

int tq_decode_exchange(const void* new_k, const void* new_v, int kv_dtype, int rotate_k, int rotate_v,
                       int advance, const float* query, int rotate_query, const float* signs_left,
                       const float* signs_right, uint32_t* k_slab, uint32_t* v_slab, int64_t unit_stride_words,
                       int32_t* lengths, int units_per_seq, int64_t len_offset, int64_t max_len, int64_t units,
                       int group_size, int head_dim, int bits, const float* cent_k, const float* cent_v,
                       float scale, float* out, float* lse, int inverse_rotate_output, int mode, void* workspace,
                       size_t workspace_bytes, float* const* exchange_bufs, int rank, int world, int32_t* epoch,
                       int64_t timeout_ns, int32_t* status, tq_stream_t stream) {
  if (!exchange_bufs || !epoch || !status) return TQ_E_ARG;
  if (world < 1 || world > kExchangeMaxWorld || rank < 0 || rank >= world) return TQ_E_ARG;
  if (timeout_ns <= 0) return TQ_E_ARG;
  if (units > 0x7fffffff / 16) return TQ_E_SHAPE;
  ExchangeParams x{exchange_bufs, rank, world, epoch, timeout_ns, status};
  if (!new_k) {
    if (new_v || advance) return TQ_E_ARG;
    return decode_core(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                       units_per_seq, len_offset, max_len, units, group_size, head_dim, bits, cent_k, cent_v, scale,
                       out, lse, inverse_rotate_output, mode, workspace, workspace_bytes, stream, nullptr, &x);
  }
  if (!new_v || !lengths || len_offset != 1) return TQ_E_ARG;
  if (kv_dtype != TQ_F32 && kv_dtype != TQ_F16 && kv_dtype != TQ_BF16) return TQ_E_ARG;
  if ((rotate_k || rotate_v) && (!signs_left || !signs_right)) return TQ_E_ARG;
  StepAppend app{new_k, new_v, kv_dtype, rotate_k, rotate_v, lengths, advance};
  return decode_core(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                     units_per_seq, 1, max_len, units, group_size, head_dim, bits, cent_k, cent_v, scale, out, lse,
                     inverse_rotate_output, mode, workspace, workspace_bytes, stream, &app, &x);
}

int tq_decode_causal(const float* query, int rotate_query, const float* signs_left, const float* signs_right,
                     const uint32_t* k_slab, const uint32_t* v_slab, int64_t unit_stride_words,
                     const int32_t* lengths, int units_per_seq, int64_t len_offset, int64_t max_len, int64_t units,
                     int q_tokens, int group_size, int head_dim, int bits, const float* cent_k,
                     const float* cent_v, float scale, float* out, float* lse, int inverse_rotate_output,
                     void* workspace, size_t workspace_bytes, tq_stream_t stream) {
  if (q_tokens < 1 || group_size < 1 || q_tokens * group_size > 16) return TQ_E_SHAPE;
  return decode_core(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                     units_per_seq, len_offset, max_len, units, q_tokens * group_size, head_dim, bits, cent_k, cent_v,
                     scale, out, lse, inverse_rotate_output, TQ_DECODE_TENSOR, workspace, workspace_bytes, stream,
                     nullptr, nullptr, q_tokens);
}

int tq_lse_merge(const float* outs, const float* lses, int parts, int64_t rows, int head_dim,
                 float* out, float* lse_out, int inverse_rotate, const float* signs_left,
                 const float* signs_right, tq_stream_t stream) {
  if (!valid_head_dim(head_dim)) return TQ_E_HEAD_DIM;
  if (parts < 1 || rows < 0) return TQ_E_SHAPE;
  if (rows == 0) return TQ_OK;
  if (!outs || !lses || !out) return TQ_E_ARG;
  if (inverse_rotate && (!signs_left || !signs_right)) return TQ_E_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (head_dim == 64) lse_merge_kernel<64><<<grid, 256, 0, st>>>(outs, lses, parts, rows, out, lse_out, inverse_rotate, signs_left, signs_right);
  else if (head_dim == 128) lse_merge_kernel<128><<<grid, 256, 0, st>>>(outs, lses, parts, rows, out, lse_out, inverse_rotate, signs_left, signs_right);
  else lse_merge_kernel<256><<<grid, 256, 0, st>>>(outs, lses, parts, rows, out, lse_out, inverse_rotate, signs_left, signs_right);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free decode: the split partials live in a scratch array compiled
// into this library instead of a caller-provided workspace.
// ---------------------------------------------------------------------------
}  // extern "C"

namespace tq {

// One copy per GPU that loads the library, alive until the process exits.
static __device__ __align__(256) unsigned char g_decode_scratch[TQ_DECODE_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices];  // device address of g_decode_scratch, per device
static std::mutex g_scratch_mutex;

// Device address of this device's scratch.  In host code the array's name is
// only a host-side stand-in, so the real address is looked up once per device
// (with that device current) and cached.
static int scratch_for_current_device(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return TQ_E_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return TQ_E_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p) {
      set_last_cuda_error(e);
      return TQ_E_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return TQ_OK;
}

}  // namespace tq

extern "C" {

int tq_decode_static(const float* query, int rotate_query, const float* signs_left,
                     const float* signs_right, const uint32_t* k_slab, const uint32_t* v_slab,
                     int64_t unit_stride_words, const int32_t* lengths, int units_per_seq,
                     int64_t len_offset, int64_t max_len, int64_t units, int group_size,
                     int head_dim, int bits, const float* cent_k, const float* cent_v, float scale,
                     float* out, float* lse, int inverse_rotate_output, int mode,
                     tq_stream_t stream) {
  // size the plan decode_core will run: unaligned slabs take the exact kernel
  int eff = mode;
  if (mode == TQ_DECODE_AUTO && k_slab && v_slab && !slabs_aligned(k_slab, v_slab, unit_stride_words))
    eff = TQ_DECODE_EXACT;
  size_t need = 0;
  int s = tq_decode_workspace_size(units, group_size, head_dim, bits, max_len, eff, &need);
  if (s != TQ_OK) return s;
  if (eff == TQ_DECODE_AUTO)  // aligned: the resolved plan alone
    need = make_plan(units, group_size, head_dim, bits, max_len, mode).bytes;
  if (need > TQ_DECODE_STATIC_SCRATCH_BYTES) return TQ_E_SCRATCH_LIMIT;
  void* scratch = nullptr;
  s = scratch_for_current_device(&scratch);
  if (s != TQ_OK) return s;
  return tq_decode(query, rotate_query, signs_left, signs_right, k_slab, v_slab, unit_stride_words, lengths,
                   units_per_seq, len_offset, max_len, units, group_size, head_dim, bits, cent_k, cent_v, scale,
                   out, lse, inverse_rotate_output, mode, scratch, TQ_DECODE_STATIC_SCRATCH_BYTES, stream);
}

}  // extern "C"

#ifdef TQ_TRACE
// Development builds only: copy the merge kernels' step timeline to the host.
extern "C" int tq_trace_read_merge(void* host, size_t bytes) {
  const size_t n = bytes < sizeof(tq::g_trace_mrg) ? bytes : sizeof(tq::g_trace_mrg);
  return cudaMemcpyFromSymbol(host, tq::g_trace_mrg, n) == cudaSuccess ? 0 : -1;
}
#endif
