// Tensor-core packed decode attention (sm_100a, mma.sync m16n8k16 f16 -> f32).
//
// Grid (splits, units); a CTA takes one token chunk of one (seq, layer,
// kv_head) unit and gives each of its NW warps a contiguous sub-range, so the
// warps run independent software pipelines (no barrier in the token loop).
//
//  * Codes stream HBM -> registers with coalesced vector loads (a warp load
//    instruction covers whole token rows); the next 16-token tile is loaded
//    while the current one is computed (two register sets, ping-pong).
//  * A code pair (two b-bit indices) becomes a half2 of centroids with ONE
//    32-bit shared-memory load from a pair table: entry e holds
//    (c[e & (2^b-1)], c[e >> b]).  Every lane owns a private copy of the K and
//    V tables in its own bank (see lut_off), so lookups never conflict
//    whatever the codes are.
//  * scores  S[t, g] = K[t, :] . Qs[g, :]  as M = 16 tokens, N = 8 heads,
//    K = 16 dims per mma.  Lane (r = lane/4, c = lane%4) takes the contiguous
//    run of d/4 dims [c*d/4, (c+1)*d/4) of its two token rows, so every code
//    is loaded once; the query fragments use the same dim permutation (a sum
//    over dims does not depend on its order).
//  * values  O^T[dim, g] = V^T[dim, t] . P^T[t, g]  as M = 16 dims, N = 8
//    heads, K = 16 tokens.  Lane r owns the run of d/8 dims [r*d/8, (r+1)*d/8);
//    the codes of tokens t and t+1 at one dim are interleaved in registers
//    (mask + funnel shift) into the same pair index.
//  * online softmax in base 2 (scale folded into the query) with a lazy
//    reference max: probabilities are exp2(s - m) with m shared by the lanes of
//    a head; m is only raised (shuffle max + rescale) when a score exceeds it
//    by more than 8, so p <= 256 stays exact in fp16 and most tiles need no
//    cross-lane reduction.  P.V uses P rounded to fp16, the denominator sums
//    the fp32 values.  The C->B fragment transpose of P is movmatrix.
//  * the warps' accumulators are merged through shared memory (fragment
//    slabs, read back conflict-free); one partial (o, m, l) per query row and
//    split goes to the split-merge kernel.
#pragma once

#include "tq_common.cuh"
#include "tq_merge.cuh"  // kLn2

namespace tq {

#ifdef TQ_TRACE
constexpr int kTraceCtas = 8192;
static __device__ unsigned long long g_trace_dec[kTraceCtas * 8];
#define TQ_DSTAMP(k) TQ_STAMP(g_trace_dec, ((blockIdx.y * gridDim.x + blockIdx.x) % kTraceCtas) * 8 + (k))
#else
#define TQ_DSTAMP(k) do { } while (0)
#endif

struct DecodeParams {
  const float* query;
  const float* signs_left;
  const float* signs_right;
  int rotate_query;
  const uint32_t* k_slab;
  const uint32_t* v_slab;
  int64_t unit_stride;   // words between units
  const int32_t* lengths;
  int units_per_seq;
  int64_t len_offset;
  int64_t max_len;
  int64_t units;
  int G;
  const float* cent_k;
  const float* cent_v;
  float scale_log2;      // softmax scale * log2(e)
  int chunk;             // tokens per CTA
  int nw;                // warps per CTA of the tensor-core kernel (kMmaWarps or kMmaWarpsWide)
  int splits;            // CTAs per unit
  float* part;           // [units*G, splits*(partials per CTA), D+2]
  // fused append of one new token per unit (tq_decode_append); new_k == null: none.
  // Row u of new_k / new_v is packed at position n_u - 1 of unit u, where
  // n_u = lengths[seq] + len_offset before clamping (len_offset = 1).
  const void* new_k;
  const void* new_v;
  int new_dtype;         // tq_dtype of new_k / new_v
  int rotate_new_k;
  int rotate_new_v;
  uint32_t* k_slab_w;    // writable views of k_slab / v_slab
  uint32_t* v_slab_w;
  // single-split plans: the CTA writes the final rows itself (no merge kernel)
  float* out;            // [units*G, D], null: partials to `part`
  float* lse;            // [units*G] or null
  int inverse_rotate;
  // causal chunk attention (tq_decode_causal): the unit's last q_tokens
  // tokens are also queries; query row g is token g / heads of the chunk and
  // attends positions < n - q_tokens + g / heads + 1.  q_tokens <= 1: decode.
  int q_tokens;
  int heads;
};

// Length of unit u before clamping to max_len.
__device__ __forceinline__ int64_t unit_length_raw(const DecodeParams& p, int64_t u) {
  int64_t n = p.len_offset;
  if (p.lengths) n += p.lengths[u / p.units_per_seq];
  return n;
}

// Pack unit u's new K (which = 0) or V (which = 1) row at position pos with
// one warp: load, optional rotation, nearest centroid, LSB-first packing -
// the append kernel's row path.
template <int D, int BITS>
__device__ __forceinline__ void append_new_row(const DecodeParams& p, int64_t u, int64_t pos, int which, int lane) {
  constexpr int E = D / 32;
  constexpr int W = D * BITS / 32;
  const void* src = which ? p.new_v : p.new_k;
  const float* cent = which ? p.cent_v : p.cent_k;
  float c[1 << BITS];
#pragma unroll
  for (int i = 0; i < (1 << BITS); ++i) c[i] = __ldg(cent + i);
  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = load_as_f32(src, p.new_dtype, u * D + j * 32 + lane);
  if (which ? p.rotate_new_v : p.rotate_new_k) warp_rotate<D>(v, lane, p.signs_right, p.signs_left);
  warp_pack_row<D, BITS>(v, lane, c, (which ? p.v_slab_w : p.k_slab_w) + u * p.unit_stride + pos * W);
}

__device__ __forceinline__ int64_t unit_length(const DecodeParams& p, int64_t u) {
  int64_t n = p.len_offset;
  if (p.lengths) n += p.lengths[u / p.units_per_seq];
  if (n > p.max_len) n = p.max_len;
  return n < 0 ? 0 : n;
}

// Warps per CTA: 16 (one CTA per SM, the tables built once for 16 warps) for
// batched decode and for a few long units; 8 (two CTAs per SM) in between
// and for d = 256.
constexpr int kMmaWarps = 8;
constexpr int kMmaWarpsWide = 16;
constexpr float kLazyMaxSlack = 8.f;              // log2 headroom before the max is raised

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 tile held in mma C-fragment order (lane (r, c) holds
// row r, cols 2c, 2c+1) so that lane (r, c) holds rows 2c, 2c+1 of column r.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Pair tables: K and V entries interleave with a 256-byte stride per entry,
// K entry e of lane l at byte e*256 + 4l and V entry e at byte e*256 + 128 + 4l,
// so one offset serves both tables and every lane reads its own bank.  Entries
// are indexed by a whole byte: the low 2b bits are the code pair, any higher
// bits are ignored (the entry is repeated for them).
//
// A pair field of 2b bits starts at an even bit of the run.  Copies of the
// run shifted right by 0, 2, 4 and 6 bits (funnel shifts, built once per run)
// put every field at the start of a byte of one copy, so a single byte
// permute yields the byte offset e*256 + 4*lane for any field.
template <int N>
__device__ __forceinline__ void shifted_copies(const uint32_t (&r)[N], uint32_t (&c)[4][N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    c[0][i] = r[i];
#pragma unroll
    for (int k = 1; k < 4; ++k) c[k][i] = i + 1 < N ? __funnelshift_r(r[i], r[i + 1], 2 * k) : (r[i] >> (2 * k));
  }
}

template <int N>
__device__ __forceinline__ uint32_t lut_off(const uint32_t (&c)[4][N], int bit, uint32_t lane4) {
  const int k = bit & 7;          // even for every pair field
  const int aligned = bit - k;    // byte-aligned start in copy k/2
  // result bytes: [lane4, field byte, 0, 0]; selector nibbles index bytes of {word, lane4}
  return __byte_perm(c[k >> 1][aligned >> 5], lane4, 0x5504u | ((uint32_t)((aligned >> 3) & 3) << 4));
}

constexpr uint32_t kLutVOffset = 128;  // V entry follows the K entry inside a 256-byte row

__device__ __forceinline__ uint32_t lut_ld(const uint32_t* lut, uint32_t byte_off) {
  return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(lut) + byte_off);
}

// Raw words of the NB-bit run that starts at bit `start` (< 32) of `row`
// (W words per token row, global memory).  Word-aligned runs use the widest
// vector load their alignment allows.  Unaligned runs load the words they
// touch (never past the row) and are shifted into place by align_run() when
// they are used, so a prefetch never waits for its own data.
template <int NB>
struct Run {
  static constexpr int NW = (NB + 31) / 32;
  static constexpr bool ALIGNED = (NB & 31) == 0;
  static constexpr int RAW = ALIGNED ? NW : NW + 1;
};

// Code words are streamed once, so they are read through L2 only
// (ld.global.cg); that path is also coherent with the in-kernel append of
// the step's new token, whose words the same CTA reads after a barrier.
template <typename T>
__device__ __forceinline__ T load_code(const T* p) {
#if defined(TQ_CODE_LOADS_NC)
  return __ldg(p);
#else
  return __ldcg(p);
#endif
}

template <bool SMEM, typename T>
__device__ __forceinline__ T ld_run(const T* p) {
  if constexpr (SMEM) return *p;
  else return load_code(p);
}

// Whether any of the COUNT lane runs of NB bits (lane k starts at bit k*NB)
// reaches one word past its first NW words; when none can, the tail load and
// its branch are dropped at compile time (3-bit d128 V runs, for one).
template <int NB, int COUNT>
constexpr bool may_tail() {
  for (int k = 0; k < COUNT; ++k)
    if (((k * NB) & 31) + NB > 32 * Run<NB>::NW) return true;
  return false;
}

template <int NB, int W, bool SMEM = false, bool TAIL = true>
__device__ __forceinline__ void load_raw(uint32_t (&raw)[Run<NB>::RAW], const uint32_t* row, int start) {
  constexpr int NW = Run<NB>::NW;
  if constexpr (Run<NB>::ALIGNED) {
    constexpr int VEC = (NW % 4 == 0 && W % 4 == 0) ? 4 : (NW % 2 == 0 && W % 2 == 0) ? 2 : 1;
#pragma unroll
    for (int i = 0; i < NW; i += VEC) {
      if constexpr (VEC == 4) {
        const uint4 v = ld_run<SMEM>(reinterpret_cast<const uint4*>(row + i));
        raw[i] = v.x; raw[i + 1] = v.y; raw[i + 2] = v.z; raw[i + 3] = v.w;
      } else if constexpr (VEC == 2) {
        const uint2 v = ld_run<SMEM>(reinterpret_cast<const uint2*>(row + i));
        raw[i] = v.x; raw[i + 1] = v.y;
      } else {
        raw[i] = ld_run<SMEM>(row + i);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < NW; ++i) raw[i] = ld_run<SMEM>(row + i);
    raw[NW] = 0u;
    if constexpr (TAIL) {
      if (start + NB > 32 * NW) raw[NW] = ld_run<SMEM>(row + NW);  // the run reaches one more word
    }
  }
}

// Run bits LSB-aligned in r[0..NW-1], r[NW] = 0.
template <int NB>
__device__ __forceinline__ void align_run(uint32_t (&r)[Run<NB>::NW + 1], const uint32_t (&raw)[Run<NB>::RAW],
                                          int start) {
  constexpr int NW = Run<NB>::NW;
  if constexpr (Run<NB>::ALIGNED) {
#pragma unroll
    for (int i = 0; i < NW; ++i) r[i] = raw[i];
  } else {
#pragma unroll
    for (int i = 0; i < NW; ++i) r[i] = __funnelshift_r(raw[i], raw[i + 1], start);
  }
  r[NW] = 0;
}

// Bit j of the interleave mask is set iff (j mod 2b) < b: the low half of a
// 2b-bit field that starts at a multiple of 2b.
template <int BITS>
__host__ __device__ constexpr uint32_t pair_mask(int word) {
  uint32_t m = 0;
  for (int t = 0; t < 32; ++t)
    if (((32 * word + t) % (2 * BITS)) < BITS) m |= 1u << t;
  return m;
}

// Interleave the runs of token t (A) and t+1 (B): field k (2b bits at bit
// 2b*k) of ev = code_t(2k) | code_t+1(2k) << b, of od the same at run
// position 2k+1.  Funnel shifts carry across words, so fields that straddle a
// word edge (3-bit) come out whole.  Bits past the run are don't-care.
template <int BITS, int NR>
__device__ __forceinline__ void pair_tokens(const uint32_t* A, const uint32_t* B, uint32_t* ev, uint32_t* od) {
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const uint32_t m = pair_mask<BITS>(i);
    const uint32_t b_up = i == 0 ? (B[0] << BITS) : __funnelshift_l(B[i - 1], B[i], BITS);
    const uint32_t a_dn = i + 1 < NR ? __funnelshift_r(A[i], A[i + 1], BITS) : (A[i] >> BITS);
    ev[i] = (A[i] & m) | (b_up & ~m);
    od[i] = (a_dn & m) | (B[i] & ~m);
  }
}

// ---------------------------------------------------------------------------
// configuration
// ---------------------------------------------------------------------------
template <int D, int BITS, int NT, int NW = kMmaWarps>
struct MmaCfg {
  static constexpr int W = D * BITS / 32;     // words per token
  static constexpr int NP = 256;              // pair-table entries (indexed by a byte)
  static constexpr int LUT_WORDS = NP * 64;   // K + V tables, 256 B per entry (one copy per lane each)
  static constexpr int RUNK = D / 4 * BITS;   // K bits per lane
  static constexpr int RUNV = D / 8 * BITS;   // V bits per lane
  static constexpr int RK = Run<RUNK>::NW + 1;
  static constexpr int RV = Run<RUNV>::NW + 1;
  static constexpr int KB = D / 16;           // k-blocks (score) = m-blocks (value)
  static constexpr int GM = 8 * NT;           // padded group size
  static constexpr int FRAG = NT * KB * 4 * 32;  // accumulator words of one warp
  static constexpr size_t MAIN_BYTES = (size_t)LUT_WORDS * 4 + (size_t)GM * D * 4;
  static constexpr size_t MERGE_BYTES =
      ((size_t)NW * FRAG + 3 * NW * GM + 2 * GM) * 4;
  static constexpr size_t DIRECT_BYTES = MERGE_BYTES + (size_t)GM * D * 4;  // + the normalised rows
  static constexpr size_t SMEM_BYTES = MAIN_BYTES > DIRECT_BYTES ? MAIN_BYTES : DIRECT_BYTES;
};

// Per-warp staging ring: each warp streams its token range through STAGES
// slots of one 16-token tile of K and V words, filled by the bulk-copy
// engine (cp.async.bulk global -> shared, completion counted on one mbarrier
// per slot).  Several tiles per warp are in flight while the warp computes,
// without holding them in registers.  The ring follows the tables and the
// query rows; the barriers follow the ring.  STAGES is the largest count
// (at most 4) that fits the CTA's share of the SM's shared memory: all of it
// for one CTA per SM, half for two.
#ifndef TQ_RING_TILES
#define TQ_RING_TILES 2
#endif
template <int D, int BITS, int NT, int NW>
struct RingCfg {
  using C = MmaCfg<D, BITS, NT, NW>;
  static constexpr size_t BUDGET = (NW == 16 || D == 256) ? 225 * 1024 : 112 * 1024;
  static constexpr size_t RING_OFF = (C::MAIN_BYTES + 127) / 128 * 128;
  static constexpr size_t fit(int tiles) {
    return (BUDGET - RING_OFF - (size_t)NW * 4 * 8) / ((size_t)NW * 2 * tiles * 16 * C::W * 4);
  }
  // tiles per stage: two (one wait, one refill and one pair of copies per 32
  // tokens) when two such stages fit, else one
  static constexpr int TILES = (TQ_RING_TILES >= 2 && fit(2) >= 2) ? 2 : 1;
  static constexpr int TILE_WORDS = TILES * 16 * C::W;            // one stage of one of K / V
  static constexpr size_t STAGE_BYTES = 2 * (size_t)TILE_WORDS * 4;
  static constexpr size_t FIT = fit(TILES);
  static constexpr int STAGES = FIT > 4 ? 4 : (int)FIT;
  static_assert(FIT >= 2, "staging ring needs two slots per warp");
  static constexpr size_t BAR_OFF = RING_OFF + (size_t)NW * STAGES * STAGE_BYTES;
  static constexpr size_t RING_TOTAL = BAR_OFF + (size_t)NW * STAGES * 8;
  static constexpr size_t SMEM_BYTES = RING_TOTAL > C::DIRECT_BYTES ? RING_TOTAL : C::DIRECT_BYTES;
};

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Wait until the barrier's phase with this parity has completed.  Each
// try_wait suspends the warp in hardware until the phase completes or the
// 100 us hint runs out, so a waiting warp issues almost nothing; after about
// a second of attempts it gives up (false) instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t it = 0; it < 10000u; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(100000u)
        : "memory");
    if (done) return true;
  }
  return false;
}

// One bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this GPU's global memory into this CTA's shared memory, completing on
// `bar`.  No multicast: the destination is the issuing CTA only.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Raw code words of one 16-token tile of a lane.
template <int D, int BITS>
struct TileRegs {
  static constexpr int KR = Run<MmaCfg<D, BITS, 1>::RUNK>::RAW;
  static constexpr int VR = Run<MmaCfg<D, BITS, 1>::RUNV>::RAW;
  uint32_t k0[KR], k1[KR];  // token rows r, r+8
  uint32_t va[VR], vb[VR];  // tokens 2c, 2c+1
  uint32_t vc[VR], vd[VR];  // tokens 2c+8, 2c+9
};

// Per-lane load plan, fixed for the whole token loop: the lane reads K token
// rows r and r+8 at bit offset c*RUNK and V rows 2c, 2c+1, 2c+8, 2c+9 at bit
// offset r*RUNV of each row.
struct LanePlan {
  int k_row, v_row;    // word offsets of the lane's first K / V run within a tile
  int k_word, v_word;  // word offset of the run inside a token row
  int k_bit, v_bit;    // bit offset of the run inside its first word
};

template <int D, int BITS>
__device__ __forceinline__ void load_tile(TileRegs<D, BITS>& t, const uint32_t* kt, const uint32_t* vt,
                                          const LanePlan& lp) {
  using C = MmaCfg<D, BITS, 1>;
  constexpr int W = C::W;
  load_raw<C::RUNK, W>(t.k0, kt + lp.k_row, lp.k_bit);
  load_raw<C::RUNK, W>(t.k1, kt + lp.k_row + 8 * W, lp.k_bit);
  load_raw<C::RUNV, W>(t.va, vt + lp.v_row, lp.v_bit);
  load_raw<C::RUNV, W>(t.vb, vt + lp.v_row + W, lp.v_bit);
  load_raw<C::RUNV, W>(t.vc, vt + lp.v_row + 8 * W, lp.v_bit);
  load_raw<C::RUNV, W>(t.vd, vt + lp.v_row + 9 * W, lp.v_bit);
}

// The same lane runs, read from a 16-token tile staged in shared memory.
template <int D, int BITS>
__device__ __forceinline__ void load_tile_smem(TileRegs<D, BITS>& t, const uint32_t* kt, const uint32_t* vt,
                                               const LanePlan& lp) {
  using C = MmaCfg<D, BITS, 1>;
  constexpr int W = C::W;
  constexpr bool TK = may_tail<C::RUNK, 4>(), TV = may_tail<C::RUNV, 8>();
  load_raw<C::RUNK, W, true, TK>(t.k0, kt + lp.k_row, lp.k_bit);
  load_raw<C::RUNK, W, true, TK>(t.k1, kt + lp.k_row + 8 * W, lp.k_bit);
  load_raw<C::RUNV, W, true, TV>(t.va, vt + lp.v_row, lp.v_bit);
  load_raw<C::RUNV, W, true, TV>(t.vb, vt + lp.v_row + W, lp.v_bit);
  load_raw<C::RUNV, W, true, TV>(t.vc, vt + lp.v_row + 8 * W, lp.v_bit);
  load_raw<C::RUNV, W, true, TV>(t.vd, vt + lp.v_row + 9 * W, lp.v_bit);
}

// Tile that runs past the unit's last token: rows are clamped to `last`
// (relative to the tile start) so no load leaves the unit.
template <int D, int BITS>
__device__ __forceinline__ void load_tile_clamped(TileRegs<D, BITS>& t, const uint32_t* kt, const uint32_t* vt,
                                                  int last, int gr, int tq, const LanePlan& lp) {
  using C = MmaCfg<D, BITS, 1>;
  constexpr int W = C::W;
  auto row = [&](int r) { return (r < last ? r : last) * W; };
  load_raw<C::RUNK, W>(t.k0, kt + row(gr) + lp.k_word, lp.k_bit);
  load_raw<C::RUNK, W>(t.k1, kt + row(gr + 8) + lp.k_word, lp.k_bit);
  load_raw<C::RUNV, W>(t.va, vt + row(2 * tq) + lp.v_word, lp.v_bit);
  load_raw<C::RUNV, W>(t.vb, vt + row(2 * tq + 1) + lp.v_word, lp.v_bit);
  load_raw<C::RUNV, W>(t.vc, vt + row(2 * tq + 8) + lp.v_word, lp.v_bit);
  load_raw<C::RUNV, W>(t.vd, vt + row(2 * tq + 9) + lp.v_word, lp.v_bit);
}

// One 16-token tile of a warp: scores, online softmax, P.V into the warp's
// accumulators (o, reference max, threshold, row sums).
template <int D, int BITS, int NT>
__device__ __forceinline__ void tile_math(const TileRegs<D, BITS>& t, int valid, const uint32_t* lut,
                                          const LanePlan& lp, uint32_t lane4, int gr, int tq,
                                          const uint32_t (&qf)[NT][D / 16][2], float (&o)[NT][D / 16][4],
                                          float (&mref)[NT][2], float (&mthr)[NT][2], float (&lrow)[NT][2],
                                          int64_t causal_lim0 = 0, int64_t tpos = -1, int heads = 1) {
  using C = MmaCfg<D, BITS, NT>;
  constexpr int KB = C::KB;
  constexpr int PB = 2 * BITS;
    // ---------------- scores S[t, g] (two independent accumulator chains) ----------------
    float sc[NT][4], sd[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = sd[nt][e] = 0.f;
    uint32_t k0[C::RK], k1[C::RK];
    align_run<C::RUNK>(k0, t.k0, lp.k_bit);
    align_run<C::RUNK>(k1, t.k1, lp.k_bit);
    uint32_t kc0[4][C::RK], kc1[4][C::RK];
    shifted_copies(k0, kc0);
    shifted_copies(k1, kc1);
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
      const uint32_t a0 = lut_ld(lut, lut_off(kc0, (2 * kb) * PB, lane4));
      const uint32_t a1 = lut_ld(lut, lut_off(kc1, (2 * kb) * PB, lane4));
      const uint32_t a2 = lut_ld(lut, lut_off(kc0, (2 * kb + 1) * PB, lane4));
      const uint32_t a3 = lut_ld(lut, lut_off(kc1, (2 * kb + 1) * PB, lane4));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (kb & 1) mma_f16(sd[nt], a0, a1, a2, a3, qf[nt][kb][0], qf[nt][kb][1]);
        else mma_f16(sc[nt], a0, a1, a2, a3, qf[nt][kb][0], qf[nt][kb][1]);
      }
    }
    // ---------------- online softmax with a lazy reference max ----------------
    bool raise = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] += sd[nt][e];
    if (valid < 16) {  // only the last tile of a range is partial
      const bool v0 = gr < valid, v1 = gr + 8 < valid;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (!((e < 2) ? v0 : v1)) sc[nt][e] = -INFINITY;
    }
    if (tpos >= 0 && tpos + 16 > causal_lim0) {  // tile reaches the causal chunk
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int g = nt * 8 + 2 * tq + (e & 1);
          const int64_t pos = tpos + gr + ((e < 2) ? 0 : 8);
          if (pos >= causal_lim0 + g / heads) sc[nt][e] = -INFINITY;
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) raise |= sc[nt][e] > mthr[nt][e & 1];
    if (__any_sync(FULL, raise)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float tm = fmaxf(sc[nt][e], sc[nt][2 + e]);
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 4));
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 8));
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 16));
          const float mn = fmaxf(mref[nt][e], tm);
          const float alpha = mn == -INFINITY ? 0.f : fast_exp2(mref[nt][e] - mn);  // -inf -> 0
          mref[nt][e] = mn;
          mthr[nt][e] = mn + kLazyMaxSlack;
          lrow[nt][e] *= alpha;
#pragma unroll
          for (int kb = 0; kb < KB; ++kb) {
            o[nt][kb][e] *= alpha;
            o[nt][kb][2 + e] *= alpha;
          }
        }
    }
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float p0 = fast_exp2(sc[nt][0] - mref[nt][0]), p1 = fast_exp2(sc[nt][1] - mref[nt][1]);
      float p2 = fast_exp2(sc[nt][2] - mref[nt][0]), p3 = fast_exp2(sc[nt][3] - mref[nt][1]);
      if (tpos >= 0) {  // causal: a head may not have seen any position yet (max still -inf)
        p0 = sc[nt][0] == -INFINITY ? 0.f : p0;
        p1 = sc[nt][1] == -INFINITY ? 0.f : p1;
        p2 = sc[nt][2] == -INFINITY ? 0.f : p2;
        p3 = sc[nt][3] == -INFINITY ? 0.f : p3;
      }
      const __half2 lo = __floats2half2_rn(p0, p1);
      const __half2 hi = __floats2half2_rn(p2, p3);
      lrow[nt][0] += p0 + p2;
      lrow[nt][1] += p1 + p3;
      pb[nt][0] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&lo));  // tokens 2c, 2c+1 of head r
      pb[nt][1] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&hi));  // tokens 2c+8, 2c+9
    }
    // ---------------- values O^T[dim, g] ----------------
    constexpr int NR = Run<C::RUNV>::NW;
    uint32_t va[C::RV], vb[C::RV], vc[C::RV], vd[C::RV];
    align_run<C::RUNV>(va, t.va, lp.v_bit);
    align_run<C::RUNV>(vb, t.vb, lp.v_bit);
    align_run<C::RUNV>(vc, t.vc, lp.v_bit);
    align_run<C::RUNV>(vd, t.vd, lp.v_bit);
    uint32_t ea[C::RV], oa[C::RV], ec[C::RV], oc[C::RV];
    pair_tokens<BITS, NR>(va, vb, ea, oa);
    pair_tokens<BITS, NR>(vc, vd, ec, oc);
    ea[NR] = oa[NR] = ec[NR] = oc[NR] = 0;
    // m-block mb: run code 2mb (row r) and 2mb+1 (row r+8) = field mb of ev / od
    uint32_t ca[4][C::RV], cb[4][C::RV], cc[4][C::RV], cd[4][C::RV];
    shifted_copies(ea, ca);
    shifted_copies(oa, cb);
    shifted_copies(ec, cc);
    shifted_copies(oc, cd);
#pragma unroll
    for (int mb = 0; mb < KB; ++mb) {
      const uint32_t a0 = lut_ld(lut, lut_off(ca, mb * PB, lane4) + kLutVOffset);
      const uint32_t a1 = lut_ld(lut, lut_off(cb, mb * PB, lane4) + kLutVOffset);
      const uint32_t a2 = lut_ld(lut, lut_off(cc, mb * PB, lane4) + kLutVOffset);
      const uint32_t a3 = lut_ld(lut, lut_off(cd, mb * PB, lane4) + kLutVOffset);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_f16(o[nt][mb], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
    }
}

// d = 256 tiles need more registers (one 8-warp CTA per SM); smaller heads run
// two 8-warp CTAs or one 16-warp CTA per SM (128 registers a thread either way).
template <int D, int NW>
constexpr int mma_min_blocks() { return (D == 256 || NW == kMmaWarpsWide) ? 1 : 2; }

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int D, int BITS, int NT, int NW>
__global__ void __launch_bounds__(NW * 32, mma_min_blocks<D, NW>())
decode_mma_kernel(DecodeParams p) {
  using C = MmaCfg<D, BITS, NT, NW>;
  constexpr int E = D / 32;
  constexpr int KB = C::KB;
  constexpr int GM = C::GM;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_fail;  // a staging copy never completed: the CTA's rows become NaN
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem);      // interleaved K/V pair tables
  float* q_s = reinterpret_cast<float*>(lut + C::LUT_WORDS);  // [GM][D]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gr = lane >> 2, tq = lane & 3;
  if (tid == 0) s_fail = 0;  // published by the table barrier below
  TQ_DSTAMP(0);
  // The grid is launched as a programmatic dependent of the previous kernel
  // on the stream (the previous step's split merge): wait for that grid and
  // its memory before reading the lengths, queries or slabs, or writing the
  // partials it may still be reading.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  TQ_DSTAMP(1);
  const int64_t u = blockIdx.y;
  const int split = blockIdx.x;
  const int G = p.G;

  const int64_t n = unit_length(p, u);
  const int64_t c0 = (int64_t)split * p.chunk;
  const int64_t c1 = min(c0 + (int64_t)p.chunk, n);
  // the CTA's real token range is shared evenly (in 16-token tiles) by its
  // warps, so a short last split of a ragged sequence still uses every warp
  const int64_t tiles = c1 > c0 ? (c1 - c0 + 15) / 16 : 0;
  const int64_t per_warp = (tiles + NW - 1) / NW * 16;
  const int64_t w0 = min(c0 + warp * per_warp, max(c1, c0));
  const int64_t w1 = min(w0 + per_warp, c1);
  const uint32_t* kbase = p.k_slab + u * p.unit_stride;
  const uint32_t* vbase = p.v_slab + u * p.unit_stride;

  // lane load plan and the first tile (in flight while the tables are built)
  LanePlan lp;
  lp.k_word = (tq * C::RUNK) >> 5;
  lp.k_bit = (tq * C::RUNK) & 31;
  lp.v_word = (gr * C::RUNV) >> 5;
  lp.v_bit = (gr * C::RUNV) & 31;
  lp.k_row = gr * C::W + lp.k_word;
  lp.v_row = 2 * tq * C::W + lp.v_word;
  // ---- staging ring of this warp: S slots of [K tile | V tile] words ----
  using RC = RingCfg<D, BITS, NT, NW>;
  constexpr int S = RC::STAGES;
  constexpr int TW = RC::TILE_WORDS;
  uint32_t* ring = reinterpret_cast<uint32_t*>(smem + RC::RING_OFF) + (size_t)warp * S * 2 * TW;
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(smem + RC::BAR_OFF) + (uint32_t)(warp * S * 8);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < S; ++i) mbar_init(bar0 + 8 * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const int64_t cap_rows = p.unit_stride / C::W;  // rows of the unit that may be read
  const int ntiles = w1 > w0 ? (int)((w1 - w0 + 15) / 16) : 0;
  constexpr int TPS = RC::TILES;
  constexpr int ROWS = TPS * 16;                   // token rows per stage
  const int nstages = (ntiles + TPS - 1) / TPS;
  // tile i of the warp's range -> slot i % S.  Tiles start at multiples of 16
  // tokens, so both copies start on 16-byte boundaries; a whole tile is
  // copied when the unit's storage holds its 16 rows (rows past the length
  // are masked by the softmax), else the lanes copy the rows that exist.
  auto issue = [&](int i) {
    const int slot = i % S;
    const int64_t t0 = w0 + ROWS * (int64_t)i;
    const uint32_t bar = bar0 + 8 * slot;
    if (t0 + ROWS <= cap_rows) {
      if (lane == 0) {
        mbar_expect_tx(bar, 2 * TW * 4);
        bulk_g2s(ring_s + slot * 2 * TW * 4, kbase + t0 * C::W, TW * 4, bar);
        bulk_g2s(ring_s + (slot * 2 + 1) * TW * 4, vbase + t0 * C::W, TW * 4, bar);
      }
    } else {
      const int words = (int)min((int64_t)ROWS, cap_rows - t0) * C::W;
      uint32_t* kd = ring + slot * 2 * TW;
      for (int w = lane; w < TW; w += 32) {
        kd[w] = w < words ? __ldcg(kbase + t0 * C::W + w) : 0u;
        kd[TW + w] = w < words ? __ldcg(vbase + t0 * C::W + w) : 0u;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    }
  };
  // fused append: the CTA whose chunk holds the new token packs it first
  if (p.new_k) {
    const int64_t raw_n = unit_length_raw(p, u);
    const int64_t pos = raw_n - 1;
    if (raw_n >= 1 && raw_n <= p.max_len && pos >= c0 && pos < c0 + p.chunk) {
      if (warp < 2) append_new_row<D, BITS>(p, u, pos, warp, lane);
      // the new words were written through the generic proxy; the bulk copies
      // that read them are async-proxy operations
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncthreads();
      TQ_DSTAMP(7);
    }
  }
  for (int i = 0; i < S && i < nstages; ++i) issue(i);  // in flight while the tables are built
  TQ_DSTAMP(2);

  // ---- pair tables: entry e = half2(c[e & m], c[e >> b]), one copy per lane ----
  // 16-byte store idx covers entry idx / 16: K copies in its first 8 stores,
  // V copies in the last 8.  Consecutive threads write consecutive 16 bytes,
  // so the stores are free of bank conflicts.
  {
    constexpr int MASK = (1 << BITS) - 1;
    for (int idx = tid; idx < C::NP * 16; idx += NW * 32) {
      const int e = idx >> 4;
      const float* cent = (idx & 15) < 8 ? p.cent_k : p.cent_v;
      const uint32_t h = pack_half2(__ldg(cent + (e & MASK)), __ldg(cent + ((e >> BITS) & MASK)));
      reinterpret_cast<uint4*>(lut)[idx] = make_uint4(h, h, h, h);
    }
  }
  // ---- query rows: rotate (exact fp32), fold the scale in base 2 ----
  for (int g = warp; g < GM; g += NW) {
    float v[E];
    if (g < G) {
      const float* q = p.query + (u * G + g) * D;
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = __ldg(q + j * 32 + lane);
      if (p.rotate_query) warp_rotate<D>(v, lane, p.signs_right, p.signs_left);
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < E; ++j) q_s[g * D + j * 32 + lane] = v[j] * p.scale_log2;
  }
  __syncthreads();
  TQ_DSTAMP(3);

  // B fragments of the score mma: lane (r, c) holds head r (+8 nt) at dims
  // c*D/4 + 4kb + {0,1} and {2,3}, the same permutation as the K runs.
  uint32_t qf[NT][KB][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
      const float* qr = q_s + (nt * 8 + gr) * D + tq * (D / 4) + 4 * kb;
      qf[nt][kb][0] = pack_half2(qr[0], qr[1]);
      qf[nt][kb][1] = pack_half2(qr[2], qr[3]);
    }

  float o[NT][KB][4];  // O^T accumulators: m-block kb, n-tile nt
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kb = 0; kb < KB; ++kb)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][kb][e] = 0.f;
  float mref[NT][2], mthr[NT][2], lrow[NT][2];  // reference max (uniform over a head's 8 lanes), + slack, row sums
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mref[nt][0] = mref[nt][1] = -INFINITY;
    mthr[nt][0] = mthr[nt][1] = -INFINITY;
    lrow[nt][0] = lrow[nt][1] = 0.f;
  }
  const uint32_t lane4 = (uint32_t)lane * 4u;

  // token loop: wait for slot i % S, compute, refill the slot with tile i + S
  bool stalled = false;
  int i = 0;
  // rounds of S stages, unrolled so every slot address is a constant offset
  for (; i < nstages; i += S) {
#pragma unroll
    for (int slot = 0; slot < S; ++slot) {
      const int st = i + slot;
      if (st >= nstages) break;
      if (!mbar_wait(bar0 + 8 * slot, (uint32_t)(st / S) & 1u)) {
        stalled = true;
        break;
      }
#pragma unroll
      for (int sub = 0; sub < TPS; ++sub) {
        const int64_t t0 = w0 + ROWS * (int64_t)st + 16 * sub;
        if (sub > 0 && t0 >= w1) break;
        TileRegs<D, BITS> t;
        load_tile_smem<D, BITS>(t, ring + slot * 2 * TW + sub * 16 * C::W,
                                ring + slot * 2 * TW + TW + sub * 16 * C::W, lp);
        if (p.q_tokens > 1)
          tile_math<D, BITS, NT>(t, (int)min((int64_t)16, w1 - t0), lut, lp, lane4, gr, tq, qf, o, mref, mthr, lrow,
                                 n - p.q_tokens + 1, t0, p.heads);
        else
          tile_math<D, BITS, NT>(t, (int)min((int64_t)16, w1 - t0), lut, lp, lane4, gr, tq, qf, o, mref, mthr, lrow);
      }
      __syncwarp();  // every lane has read the slot before it is refilled
      if (st + S < nstages) issue(st + S);
    }
    if (stalled) break;
  }
  if (stalled) {
    // a copy never completed: wait (bounded) for the ones still in flight so
    // none lands after the CTA's shared memory is reused, and poison the rows
    for (int j = i; j < nstages && j < i + 2 * S; ++j) mbar_wait(bar0 + 8 * (j % S), (uint32_t)(j / S) & 1u);
    s_fail = 1;
  }

  TQ_DSTAMP(4);
  // the split-merge grid may be scheduled as CTAs reach this point
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // ---- merge the warps of this CTA through shared memory (reusing the tables) ----
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float lv = lrow[nt][e];
      lv += __shfl_xor_sync(FULL, lv, 4);
      lv += __shfl_xor_sync(FULL, lv, 8);
      lv += __shfl_xor_sync(FULL, lv, 16);
      lrow[nt][e] = lv;
    }
  __syncthreads();  // all warps are done with the tables
  float* frag = reinterpret_cast<float*>(smem);       // [NW][FRAG] accumulators in fragment order
  float* red_m = frag + NW * C::FRAG;          // [NW][GM]
  float* red_l = red_m + NW * GM;              // [NW][GM]
  float* scale = red_l + NW * GM;              // [NW][GM]
  float* fin_m = scale + NW * GM;              // [GM]
  float* fin_l = fin_m + GM;                          // [GM]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int mb = 0; mb < KB; ++mb)
#pragma unroll
      for (int e = 0; e < 4; ++e) frag[warp * C::FRAG + ((nt * KB + mb) * 4 + e) * 32 + lane] = o[nt][mb][e];
  if (gr == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool seen = lrow[nt][e] > 0.f;
        red_m[warp * GM + nt * 8 + 2 * tq + e] = seen ? mref[nt][e] : -INFINITY;
        red_l[warp * GM + nt * 8 + 2 * tq + e] = lrow[nt][e];
      }
  }
  __syncthreads();
  if (tid < GM) {
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, red_m[w * GM + tid]);
    float L = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float mw = red_m[w * GM + tid];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      scale[w * GM + tid] = f;
      L += red_l[w * GM + tid] * f;
    }
    fin_m[tid] = s_fail ? 0.f : M;
    fin_l[tid] = s_fail ? 1.f : L;
  }
  __syncthreads();
  TQ_DSTAMP(5);
  const float poison = s_fail ? __int_as_float(0x7fc00000) : 0.f;
  float* rows = fin_l + GM;  // [GM][D] normalised rows (single-split plans)
  // element i of a warp's fragment slab = (nt, mb, e, lane) -> (head, dim)
  for (int i = tid; i < C::FRAG; i += NW * 32) {
    const int ln = i & 31, e = (i >> 5) & 3, blk = i >> 7;
    const int nt = blk / KB, mb = blk % KB;
    const int g = nt * 8 + 2 * (ln & 3) + (e & 1);
    if (g >= G) continue;
    const int dim = (ln >> 2) * (D / 8) + 2 * mb + (e >> 1);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc = fmaf(frag[w * C::FRAG + i], scale[w * GM + g], acc);
    acc += poison;
    if (p.out) rows[g * D + dim] = fin_l[g] > 0.f ? acc / fin_l[g] : 0.f;
    else p.part[((u * G + g) * (int64_t)p.splits + split) * (D + 2) + dim] = acc;
  }
  if (p.out) {
    // one split: the unit's rows are final (normalised, optionally rotated back)
    __syncthreads();
    for (int g = warp; g < G; g += NW) {
      float v[E];
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = rows[g * D + j * 32 + lane];
      if (p.inverse_rotate) warp_rotate<D>(v, lane, p.signs_left, p.signs_right);
      float* o = p.out + (u * G + g) * D;
#pragma unroll
      for (int j = 0; j < E; ++j) o[j * 32 + lane] = v[j];
      if (p.lse && lane == 0)
        p.lse[u * G + g] = (fin_l[g] > 0.f) ? (fin_m[g] + log2f(fin_l[g])) * kLn2 : -INFINITY;
    }
    TQ_DSTAMP(6);
    return;
  }
  if (tid < G && tid < GM) {
    float* dst = p.part + ((u * G + tid) * (int64_t)p.splits + split) * (D + 2);
    dst[D] = fin_m[tid];
    dst[D + 1] = fin_l[tid];
  }
  TQ_DSTAMP(6);
}

// Launches the tensor-core kernel for (D, BITS) (tq_decode_mma.cu).
void launch_mma_dispatch(int D, int bits, const DecodeParams& p, cudaStream_t st);
// Resident CTAs per SM of the tensor-core kernel for (D, BITS, G, warps per CTA).
int mma_blocks_per_sm(int D, int bits, int G, int nw);

}  // namespace tq
