// Tensor-core packed decode attention (sm_100a, mma.sync m16n8k16 f16 -> f32).
//
// Per CTA: one token chunk of one (seq, layer, kv_head) unit, NW warps.
//
//  * K/V code bytes are streamed HBM -> shared memory by the bulk-copy engine
//    (cp.async.bulk, completion on an mbarrier) through a ring of RS stages of
//    NW*16 tokens each, so loads stay in flight while warps compute.
//  * A code pair (two b-bit indices, 2b bits) is turned into a half2 of
//    centroids by ONE 32-bit shared load from a pair table: entry e holds
//    (c[e & (2^b-1)], c[e >> b]).  Every lane has its own copy of the table in
//    its own bank (entry e of lane l at word e*32 + l), so lookups never
//    conflict whatever the codes are.
//  * scores:  S[t, g] = K[t, :] . Qs[g, :]   as M = 16 tokens, N = 8 query
//    heads, K = 16 dims per mma.  Lane (r = lane/4, c = lane%4) takes the
//    contiguous run of d/4 dims [c*d/4, (c+1)*d/4) for its two token rows, so
//    it reads whole words and no code is read twice; the query fragments use
//    the same dim permutation (a sum over dims does not depend on its order).
//  * values:  O^T[dim, g] = V^T[dim, t] . P^T[t, g]  as M = 16 dims,
//    N = 8 heads, K = 16 tokens.  Lane r owns the run of d/8 dims
//    [r*d/8, (r+1)*d/8); the two codes of consecutive tokens at one dim are
//    interleaved in registers (SWAR for 2/4 bits) into the same pair index.
//  * online softmax in fp32 (base-2, scale folded into the query), the
//    probabilities are rounded to fp16 once and used for both P.V and the
//    denominator, so the weights of a row sum to one.
//  * the NW warps of a CTA are merged in shared memory and one partial
//    (o, m, l) per query row is written for the split merge kernel.
#pragma once

#include "tq_common.cuh"

namespace tq {

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
  int splits;            // CTAs per unit
  float* part;           // [units*G, splits*(warps per partial), D+2]
  int* err;              // bounded-wait failure flag (nullable)
};

__device__ __forceinline__ int64_t unit_length(const DecodeParams& p, int64_t u) {
  int64_t n = p.len_offset;
  if (p.lengths) n += p.lengths[u / p.units_per_seq];
  if (n > p.max_len) n = p.max_len;
  return n < 0 ? 0 : n;
}

constexpr int kMmaWarps = 8;                  // warps per CTA
constexpr int kMmaTokensPerCta = kMmaWarps * 16;  // tokens per stage
constexpr int kMmaStages = 3;                 // ring depth

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier + bulk copy + mma
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bounded wait on phase `parity`; returns false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Plain (non-multicast) bulk copy global -> own shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// `n` consecutive bits of a register run starting at static bit `bit`.
template <int N>
__device__ __forceinline__ uint32_t run_bits(const uint32_t* r, int bit) {
  const int w = bit >> 5, s = bit & 31;
  uint32_t v = (s + N > 32) ? __funnelshift_r(r[w], r[w + 1], s) : (r[w] >> s);
  return v & ((1u << N) - 1u);
}

// Load `NB` bits starting at (runtime) bit `start` of a shared-memory word row
// into registers r[0..], LSB-aligned.  When the run is word-aligned for every
// lane this is a plain vector of loads.
template <int NB>
__device__ __forceinline__ void load_run(uint32_t (&r)[(NB + 31) / 32 + 1], const uint32_t* row,
                                         int start) {
  constexpr int NW = (NB + 31) / 32;
  if ((NB & 31) == 0) {
    const uint32_t* src = row + (start >> 5);
#pragma unroll
    for (int i = 0; i < NW; ++i) r[i] = src[i];
    r[NW] = 0;
  } else {
    const int w0 = start >> 5, sh = start & 31;
    uint32_t tmp[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) tmp[i] = row[w0 + i];
#pragma unroll
    for (int i = 0; i < NW; ++i) r[i] = __funnelshift_r(tmp[i], tmp[i + 1], sh);
    r[NW] = 0;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int D, int BITS, int NT>
struct MmaCfg {
  static constexpr int W = D * BITS / 32;               // words per token
  static constexpr int NP = 1 << (2 * BITS);            // pair-table entries
  static constexpr int LUT_WORDS = NP * 32;             // per table
  static constexpr int STAGE_TOK = kMmaTokensPerCta;
  static constexpr int STAGE_WORDS = STAGE_TOK * W + 4;  // +16 B pad for run over-read
  static constexpr int RUNK = D / 4 * BITS;             // bits per lane, K
  static constexpr int RUNV = D / 8 * BITS;             // bits per lane, V
  static constexpr int KB = D / 16;                     // k-blocks (score) = m-blocks (value)
  static constexpr int GM = 8 * NT;                     // padded group size
  static constexpr size_t SMEM_BYTES =
      (size_t)(2 * LUT_WORDS + 2 * kMmaStages * STAGE_WORDS) * 4 +
      (size_t)GM * D * 4 /* rotated queries */ + (size_t)kMmaWarps * GM * 16 * 2 /* P tiles */ +
      kMmaStages * 8 /* mbarriers */ + 64;
};

template <int D, int BITS, int NT>
__global__ void __launch_bounds__(kMmaWarps * 32, 1)
decode_mma_kernel(DecodeParams p) {
  using C = MmaCfg<D, BITS, NT>;
  constexpr int W = C::W;
  constexpr int E = D / 32;
  constexpr int KB = C::KB;
  constexpr int GM = C::GM;
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* lut_k = reinterpret_cast<uint32_t*>(smem);
  uint32_t* lut_v = lut_k + C::LUT_WORDS;
  uint32_t* ring_k = lut_v + C::LUT_WORDS;                  // [RS][STAGE_WORDS]
  uint32_t* ring_v = ring_k + kMmaStages * C::STAGE_WORDS;  // [RS][STAGE_WORDS]
  float* q_s = reinterpret_cast<float*>(ring_v + kMmaStages * C::STAGE_WORDS);         // [GM][D]
  __half* p_tiles = reinterpret_cast<__half*>(q_s + GM * D);                            // [NW][GM][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_tiles + kMmaWarps * GM * 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int64_t u = blockIdx.y;
  const int split = blockIdx.x;
  const int G = p.G;

  const int64_t n = unit_length(p, u);
  const int64_t c0 = (int64_t)split * p.chunk;
  const int64_t c1 = min(c0 + (int64_t)p.chunk, n);
  const int nstages = c1 > c0 ? (int)((c1 - c0 + C::STAGE_TOK - 1) / C::STAGE_TOK) : 0;
  const uint32_t* kbase = p.k_slab + u * p.unit_stride;
  const uint32_t* vbase = p.v_slab + u * p.unit_stride;

  // ---- producer prologue: barriers + first RS stages ----
  auto issue = [&](int s) {
    const int slot = s % kMmaStages;
    const int64_t t0 = c0 + (int64_t)s * C::STAGE_TOK;
    const int ntok = (int)min((int64_t)C::STAGE_TOK, c1 - t0);
    const uint32_t bytes = (uint32_t)ntok * W * 4;
    const uint32_t bulk = bytes & ~15u;
    uint32_t* dk = ring_k + slot * C::STAGE_WORDS;
    uint32_t* dv = ring_v + slot * C::STAGE_WORDS;
    const uint32_t* sk = kbase + t0 * W;
    const uint32_t* sv = vbase + t0 * W;
    if (bulk) {
      mbar_expect_tx(&bars[slot], 2 * bulk);
      bulk_g2s(dk, sk, bulk, &bars[slot]);
      bulk_g2s(dv, sv, bulk, &bars[slot]);
    } else {
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bars[slot])) : "memory");
    }
    if (bytes != bulk) {  // ragged tail (< 16 B) of 24-byte rows: plain copies
      for (uint32_t w = bulk / 4; w < bytes / 4; ++w) {
        dk[w] = __ldg(sk + w);
        dv[w] = __ldg(sv + w);
      }
    }
  };
  if (tid == 0) {
    for (int s = 0; s < kMmaStages; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int s = 0; s < kMmaStages && s < nstages; ++s) issue(s);
  }

  // ---- pair tables (per-lane copies) ----
  {
    constexpr int MASK = (1 << BITS) - 1;
    for (int i = tid; i < C::LUT_WORDS; i += kMmaWarps * 32) {
      const int e = i >> 5;
      lut_k[i] = pack_half2(__ldg(p.cent_k + (e & MASK)), __ldg(p.cent_k + (e >> BITS)));
      lut_v[i] = pack_half2(__ldg(p.cent_v + (e & MASK)), __ldg(p.cent_v + (e >> BITS)));
    }
  }

  // ---- query rows: rotate (exact fp32, as the append path), fold the
  //      softmax scale in base 2, stage in shared memory ----
  for (int g = warp; g < GM; g += kMmaWarps) {
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

  // B fragments of the score mma: lane (r, c) holds head r (+8 nt) at the
  // dims c*D/4 + 4kb + {0,1} and {2,3}, the same permutation as the K runs.
  uint32_t qf[NT][KB][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kb = 0; kb < KB; ++kb) {
      const float* qr = q_s + (nt * 8 + gr) * D + tq * (D / 4) + 4 * kb;
      qf[nt][kb][0] = pack_half2(qr[0], qr[1]);
      qf[nt][kb][1] = pack_half2(qr[2], qr[3]);
    }

  // ---- main loop ----
  float o[NT][KB][4];   // O^T accumulators: m-block kb, n-tile nt
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kb = 0; kb < KB; ++kb)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][kb][e] = 0.f;
  float mrow[NT][2], lrow[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mrow[nt][0] = mrow[nt][1] = -INFINITY;
    lrow[nt][0] = lrow[nt][1] = 0.f;
  }

  const uint32_t lut_k_lane = smem_u32(lut_k) + lane * 4;
  const uint32_t lut_v_lane = smem_u32(lut_v) + lane * 4;
  __half* ptile = p_tiles + warp * GM * 16;
  bool ok = true;

  for (int s = 0; s < nstages; ++s) {
    const int slot = s % kMmaStages;
    if (!mbar_wait(&bars[slot], (uint32_t)((s / kMmaStages) & 1))) ok = false;
    const int64_t tile0 = c0 + (int64_t)s * C::STAGE_TOK + warp * 16;
    const int valid = (int)max((int64_t)0, min((int64_t)16, c1 - tile0));
    if (valid > 0 && ok) {
      const uint32_t* ks = ring_k + slot * C::STAGE_WORDS + warp * 16 * W;
      const uint32_t* vs = ring_v + slot * C::STAGE_WORDS + warp * 16 * W;
      // ---------------- scores ----------------
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
      {
        uint32_t r0[(C::RUNK + 31) / 32 + 1], r1[(C::RUNK + 31) / 32 + 1];
        load_run<C::RUNK>(r0, ks + gr * W, tq * C::RUNK);
        load_run<C::RUNK>(r1, ks + (gr + 8) * W, tq * C::RUNK);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          const uint32_t pa0 = run_bits<2 * BITS>(r0, (2 * kb) * 2 * BITS);
          const uint32_t pa1 = run_bits<2 * BITS>(r1, (2 * kb) * 2 * BITS);
          const uint32_t pa2 = run_bits<2 * BITS>(r0, (2 * kb + 1) * 2 * BITS);
          const uint32_t pa3 = run_bits<2 * BITS>(r1, (2 * kb + 1) * 2 * BITS);
          const uint32_t a0 = lds32(lut_k_lane + (pa0 << 7));
          const uint32_t a1 = lds32(lut_k_lane + (pa1 << 7));
          const uint32_t a2 = lds32(lut_k_lane + (pa2 << 7));
          const uint32_t a3 = lds32(lut_k_lane + (pa3 << 7));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma16816(sc[nt], a0, a1, a2, a3, qf[nt][kb][0], qf[nt][kb][1]);
        }
      }
      // ---------------- online softmax ----------------
      const bool v0 = gr < valid, v1 = gr + 8 < valid;
      float alpha[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float s0 = v0 ? sc[nt][e] : -INFINITY;
          float s1 = v1 ? sc[nt][2 + e] : -INFINITY;
          float tm = fmaxf(s0, s1);
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 4));
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 8));
          tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 16));
          const float mn = fmaxf(mrow[nt][e], tm);
          alpha[nt][e] = exp2f(mrow[nt][e] - mn);
          mrow[nt][e] = mn;
          const __half h0 = __float2half_rn(exp2f(s0 - mn));
          const __half h1 = __float2half_rn(exp2f(s1 - mn));
          lrow[nt][e] = lrow[nt][e] * alpha[nt][e] + (__half2float(h0) + __half2float(h1));
          // P^T tile for the value mma: ptile[g][token]
          ptile[(nt * 8 + 2 * tq + e) * 16 + gr] = h0;
          ptile[(nt * 8 + 2 * tq + e) * 16 + gr + 8] = h1;
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          o[nt][kb][0] *= alpha[nt][0];
          o[nt][kb][1] *= alpha[nt][1];
          o[nt][kb][2] *= alpha[nt][0];
          o[nt][kb][3] *= alpha[nt][1];
        }
      __syncwarp();
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        pb[nt][0] = *reinterpret_cast<const uint32_t*>(ptile + (nt * 8 + gr) * 16 + 2 * tq);
        pb[nt][1] = *reinterpret_cast<const uint32_t*>(ptile + (nt * 8 + gr) * 16 + 2 * tq + 8);
      }
      // ---------------- values ----------------
      {
        constexpr int RW = (C::RUNV + 31) / 32 + 1;
        uint32_t ra[RW], rb[RW], rc[RW], rd[RW];  // tokens 2tq, 2tq+1, 2tq+8, 2tq+9
        load_run<C::RUNV>(ra, vs + (2 * tq) * W, gr * C::RUNV);
        load_run<C::RUNV>(rb, vs + (2 * tq + 1) * W, gr * C::RUNV);
        load_run<C::RUNV>(rc, vs + (2 * tq + 8) * W, gr * C::RUNV);
        load_run<C::RUNV>(rd, vs + (2 * tq + 9) * W, gr * C::RUNV);
        // m-block mb uses run codes 2mb (row gr) and 2mb+1 (row gr+8)
#pragma unroll
        for (int mb = 0; mb < KB; ++mb) {
          uint32_t i0, i1, i2, i3;
          if constexpr (BITS == 4) {
            const int wj = (2 * mb) / 8, by = mb % 4;
            const uint32_t A = ra[wj], B = rb[wj], Cc = rc[wj], Dd = rd[wj];
            const uint32_t ev01 = (A & 0x0F0F0F0Fu) | ((B << 4) & 0xF0F0F0F0u);
            const uint32_t od01 = ((A >> 4) & 0x0F0F0F0Fu) | (B & 0xF0F0F0F0u);
            const uint32_t ev89 = (Cc & 0x0F0F0F0Fu) | ((Dd << 4) & 0xF0F0F0F0u);
            const uint32_t od89 = ((Cc >> 4) & 0x0F0F0F0Fu) | (Dd & 0xF0F0F0F0u);
            i0 = (ev01 >> (8 * by)) & 0xFFu;
            i1 = (od01 >> (8 * by)) & 0xFFu;
            i2 = (ev89 >> (8 * by)) & 0xFFu;
            i3 = (od89 >> (8 * by)) & 0xFFu;
          } else if constexpr (BITS == 2) {
            const int wj = (2 * mb) / 16, nb = mb % 8;
            const uint32_t A = ra[wj], B = rb[wj], Cc = rc[wj], Dd = rd[wj];
            const uint32_t ev01 = (A & 0x33333333u) | ((B << 2) & 0xCCCCCCCCu);
            const uint32_t od01 = ((A >> 2) & 0x33333333u) | (B & 0xCCCCCCCCu);
            const uint32_t ev89 = (Cc & 0x33333333u) | ((Dd << 2) & 0xCCCCCCCCu);
            const uint32_t od89 = ((Cc >> 2) & 0x33333333u) | (Dd & 0xCCCCCCCCu);
            i0 = (ev01 >> (4 * nb)) & 0xFu;
            i1 = (od01 >> (4 * nb)) & 0xFu;
            i2 = (ev89 >> (4 * nb)) & 0xFu;
            i3 = (od89 >> (4 * nb)) & 0xFu;
          } else {
            const int be = (2 * mb) * BITS, bo = (2 * mb + 1) * BITS;
            i0 = run_bits<BITS>(ra, be) | (run_bits<BITS>(rb, be) << BITS);
            i1 = run_bits<BITS>(ra, bo) | (run_bits<BITS>(rb, bo) << BITS);
            i2 = run_bits<BITS>(rc, be) | (run_bits<BITS>(rd, be) << BITS);
            i3 = run_bits<BITS>(rc, bo) | (run_bits<BITS>(rd, bo) << BITS);
          }
          const uint32_t a0 = lds32(lut_v_lane + (i0 << 7));
          const uint32_t a1 = lds32(lut_v_lane + (i1 << 7));
          const uint32_t a2 = lds32(lut_v_lane + (i2 << 7));
          const uint32_t a3 = lds32(lut_v_lane + (i3 << 7));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma16816(o[nt][mb], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
        }
      }
    }
    __syncthreads();  // every warp is done with this slot
    if (tid == 0 && s + kMmaStages < nstages) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(s + kMmaStages);
    }
  }
  if (!ok && p.err && lane == 0) atomicExch(p.err, TQ_E_TIMEOUT);

  // ---- merge the warps of this CTA in shared memory (reuse the ring) ----
  float* red_o = reinterpret_cast<float*>(ring_k);  // [GM][D]
  float* red_m = red_o + GM * D;                    // [NW][GM]
  float* red_l = red_m + kMmaWarps * GM;            // [NW][GM]
  float* fin_m = red_l + kMmaWarps * GM;            // [GM]
  // full l per column: reduce lane partials across gr
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
  for (int i = tid; i < GM * D; i += kMmaWarps * 32) red_o[i] = 0.f;
  if (gr == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        red_m[warp * GM + nt * 8 + 2 * tq + e] = mrow[nt][e];
        red_l[warp * GM + nt * 8 + 2 * tq + e] = lrow[nt][e];
      }
  }
  __syncthreads();
  if (tid < GM) {
    float M = -INFINITY;
    for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, red_m[w * GM + tid]);
    fin_m[tid] = M;
  }
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float f[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float M = fin_m[nt * 8 + 2 * tq + e];
      f[e] = (mrow[nt][e] == -INFINITY) ? 0.f : exp2f(mrow[nt][e] - M);
    }
#pragma unroll
    for (int mb = 0; mb < KB; ++mb) {
      const int dlo = gr * (D / 8) + 2 * mb;  // row gr; row gr+8 -> dlo + 1
      const int g0 = nt * 8 + 2 * tq;
      atomicAdd(&red_o[g0 * D + dlo], o[nt][mb][0] * f[0]);
      atomicAdd(&red_o[(g0 + 1) * D + dlo], o[nt][mb][1] * f[1]);
      atomicAdd(&red_o[g0 * D + dlo + 1], o[nt][mb][2] * f[0]);
      atomicAdd(&red_o[(g0 + 1) * D + dlo + 1], o[nt][mb][3] * f[1]);
    }
  }
  __syncthreads();
  for (int g = warp; g < G && g < GM; g += kMmaWarps) {
    const float M = fin_m[g];
    float Ls = 0.f;
    for (int w = 0; w < kMmaWarps; ++w) {
      const float mw = red_m[w * GM + g];
      if (mw != -INFINITY) Ls += red_l[w * GM + g] * exp2f(mw - M);
    }
    float* dst = p.part + ((u * G + g) * (int64_t)p.splits + split) * (D + 2);
    for (int i = lane; i < D; i += 32) dst[i] = red_o[g * D + i];
    if (lane == 0) {
      dst[D] = M;
      dst[D + 1] = Ls;
    }
  }
}

// Launches the tensor-core kernel for (D, BITS) (tq_decode_mma.cu).
void launch_mma_dispatch(int D, int bits, const DecodeParams& p, cudaStream_t st);

}  // namespace tq
