// Q4 weight streaming engine shared by gemv_q, ffn_fused and the decode-batch
// gemm.  HBM-bound: each weight byte is read exactly once per launch.
//
// GPU weight layout ("unit layout").  A Q4 matrix of N rows x K columns is cut
// into units of 16 rows x 64 columns; unit (r, kt) sits at byte offset
// (r*KT + kt) * 576 and holds
//   bytes [0, 512)   nibbles: lane L (g = L/4, t4 = L%4) owns bytes [16L, 16L+16),
//                    one 32-bit word per 16-column chunk j (0..3).  Word bits:
//                    [0:4) u(g, c)   [4:8) u(g+8, c)   [8:12) u(g, c+8)   [12:16) u(g+8, c+8)
//                    [16:20) u(g, c+1) [20:24) u(g+8,c+1) [24:28) u(g,c+9) [28:32) u(g+8,c+9)
//                    with c = 16j + 2*t4 and u = q + 8 (offset binary).  Masking a word
//                    with 0x000F000F after shifts of 0/4/8/12 yields exactly the four
//                    bf16x2 registers of an m16n8k16 A fragment.
//   bytes [512, 576) block scales: for g = 0..7, four bf16 at 512 + 8g:
//                    S(g, blk0), S(g, blk1), S(g+8, blk0), S(g+8, blk1).
// Algorithmic content is 18 B per 32 weights; the layout adds no padding beyond
// rounding N up to 16 and K up to 64.
//
// Dequantization reproduces the reference's w = bf16_rn(float(q) * scale)
// (tools/ref/gemv_q.py:32-37) bit for bit:
//  * fast path: a nibble u placed in the low bits of a bf16 half is the
//    subnormal u * 2^-133.  With the stored scale S = s * 2^(133 - je) and
//    C = -8 * s * 2^-je, fma.rn.bf16x2(u*2^-133, S, C) = rn((u - 8) * s * 2^-je)
//    = bf16_rn(q*s) * 2^-je exactly (one rounding, power-of-two scaling); the
//    epilogue multiplies by 2^je.  je is chosen per matrix at load time so
//    that no scaled scale overflows and no product becomes subnormal.
//  * generic path (any finite scales): OR the nibble into 128.0 (0x4300),
//    subtract 136 (exact), multiply by s (one rounding).
// The products w * x are then accumulated in fp32 on the tensor cores
// (mma.sync m16n8k16, bf16 x bf16 products are exact).  An fp32 activation x is
// split into x_hi = bf16(x) and x_lo = bf16(x - x_hi), fed as two B columns,
// and recombined in fp32 (residual < 2^-17 |x|).
#pragma once

#include "common.cuh"

namespace alv {

constexpr int kUnitBytes = 576;
constexpr int kUnitNibBytes = 512;
constexpr int kTileRows = 16;
constexpr int kTileCols = 64;

struct Q4Mat {
  const uint8_t* units;  // RT*KT units of kUnitBytes
  uint32_t RT;           // row tiles of 16 rows
  uint32_t KT;           // k tiles of 64 columns
  uint32_t fast;         // 1: subnormal-magic dequant; 0: generic
  float scale_mul;       // 2^je (fast) or 1 (generic)
};

// Contiguous split of U units over W warps: warp w owns [start(w), start(w+1)).
// W must be min(#warps, U) so that every participating warp owns >= 1 unit
// (the fixup counts contributors as a contiguous warp interval).
__device__ __forceinline__ uint64_t range_start(uint64_t w, uint64_t U, uint64_t W) {
  return w * U / W;
}
// Participating warps for U units of a matrix with KT k tiles: every warp
// owns >= 1 unit, and >= ceil(KT/16) units so that no row tile is split over
// more than ~16 warps (the split-K fixup gathers one partial per contributor).
__host__ __device__ __forceinline__ uint64_t effective_warps(uint64_t Wtot, uint64_t U, uint64_t KT) {
  const uint64_t min_units = (KT + 15) / 16;
  uint64_t w = U / (min_units ? min_units : 1);
  if (w < 1) w = 1;
  return w < Wtot ? w : Wtot;
}
// Participating warp index of warp `warp` of CTA `cta`: warp-major over CTAs,
// so a small problem spreads over all SMs.
__device__ __forceinline__ uint32_t participant_index(uint32_t cta, uint32_t warp, uint32_t nctas) {
  return warp * nctas + cta;
}
// The warp whose range contains unit u.
__device__ __forceinline__ uint32_t warp_of_unit(uint64_t u, uint64_t U, uint64_t W) {
  return static_cast<uint32_t>(((u + 1) * W - 1) / U);
}

// ---------------------------------------------------------------------------
// Dequantize one 32-bit nibble word into the four bf16x2 A-fragment registers.
// S*/C* are bf16x2 broadcasts of the scale (and -8*scale) for rows g and g+8.
// ---------------------------------------------------------------------------
template <bool FAST>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t Sg, uint32_t Cg, uint32_t Sg8,
                                             uint32_t Cg8, uint32_t (&a)[4]) {
  const uint32_t m = 0x000F000Fu;
  const uint32_t p0 = w & m, p1 = (w >> 4) & m, p2 = (w >> 8) & m, p3 = (w >> 12) & m;
  if (FAST) {
    a[0] = bf2_fma(p0, Sg, Cg);
    a[1] = bf2_fma(p1, Sg8, Cg8);
    a[2] = bf2_fma(p2, Sg, Cg);
    a[3] = bf2_fma(p3, Sg8, Cg8);
  } else {
    const uint32_t magic = 0x43004300u;   // bf16x2 (128, 128)
    const uint32_t m136 = 0x43084308u;    // bf16x2 (136, 136)
    a[0] = bf2_mul(bf2_sub(p0 | magic, m136), Sg);
    a[1] = bf2_mul(bf2_sub(p1 | magic, m136), Sg8);
    a[2] = bf2_mul(bf2_sub(p2 | magic, m136), Sg);
    a[3] = bf2_mul(bf2_sub(p3 | magic, m136), Sg8);
  }
}

// bf16x2 (-2^-130, -2^-130): multiplying a fast-path stored scale by it gives -8*s*2^-je.
constexpr uint32_t kNeg8Sub = 0x80088008u;

// ---------------------------------------------------------------------------
// x staging: B-fragment layout in shared memory.
// For k tile kt, column n and lane quad t4, 32 contiguous bytes hold the four
// chunks' fragments: at ((kt*NCOLS + n)*4 + t4)*32 + j*8 the uint2 {b0, b1} with
//   b0 = bf16x2(col_n[k0], col_n[k0+1]), b1 = bf16x2(col_n[k0+8], col_n[k0+9]),
//   k0 = 64*kt + 16*j + 2*t4,
// so one lane fetches a unit's fragments with two 128-bit loads.  Column n is
// token n (bf16 x) or token n/2, hi (n even) / lo (n odd) part (fp32 x).
// ---------------------------------------------------------------------------
template <int NCOLS, bool SPLIT, class Src>
__device__ void stage_frags(uint8_t* xs, uint32_t KT, const Src& src) {
  constexpr int BATCH = 8;  // entries per thread per pass: all loads in flight together
  const uint32_t total = KT * 4 * NCOLS * 4;
  for (uint32_t base = 0; base < total; base += blockDim.x * BATCH) {
    float v[BATCH][4];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const uint32_t e = base + u * blockDim.x + threadIdx.x;
      const uint32_t j = e & 3, t4 = (e >> 2) & 3, n = (e >> 4) % NCOLS, kt = (e >> 4) / NCOLS;
      const uint32_t tok = SPLIT ? (n >> 1) : n;
      const uint32_t k0 = kt * 64 + j * 16 + 2 * t4;
      if (e < total) {
        src.pair(tok, k0, v[u][0], v[u][1]);       // 0 outside [0, ntok) x [0, K)
        src.pair(tok, k0 + 8, v[u][2], v[u][3]);
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const uint32_t e = base + u * blockDim.x + threadIdx.x;
      if (e >= total) continue;
      const bool lo = SPLIT && (((e >> 4) % NCOLS) & 1);
      uint16_t h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = v[u][i];
        h[i] = bf16_bits_rn(lo ? (x - bf16_round(x)) : x);
      }
      uint2 w;
      w.x = pack_bf2(h[0], h[1]);
      w.y = pack_bf2(h[2], h[3]);
      *reinterpret_cast<uint2*>(xs + static_cast<size_t>(e) * 8) = w;
    }
  }
}

// Shared-memory bytes of the staged fragments for KT k tiles.
__host__ __device__ constexpr size_t frag_bytes(uint32_t KT, int ncols) {
  return static_cast<size_t>(KT) * 128 * ncols;
}

// ---------------------------------------------------------------------------
// Per-warp ring filled by the TMA engine.  The warp's work list is up to two
// contiguous unit ranges (segment 0 then segment 1, e.g. FFN gate/up then
// down); stages hold UPS consecutive list units and may straddle the two
// segments.  All bookkeeping is incremental 32-bit arithmetic.
// ---------------------------------------------------------------------------
template <int UPS>
struct WarpRing {
  static constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  uint8_t* ring;            // nst * kStageBytes (shared)
  uint64_t* bars;           // nst mbarriers (shared)
  uint64_t policy;
  uint32_t nst;             // number of stages
  // producer (lane 0 issues; every lane keeps the same counters)
  const uint8_t* p_src;     // source of the next unit to issue
  const uint8_t* seg1;      // first unit of segment 1
  const uint8_t* seg0_end;  // one past the last unit of each segment
  const uint8_t* seg1_end;
  uint32_t* status;         // device status word (bounds violations)
  uint32_t p_left0;         // units of segment 0 not yet issued
  uint32_t p_left;          // units not yet issued
  uint32_t p_stage;         // stage the next group goes to
  // consumer
  uint32_t stage, phase;    // current stage and its parity
  uint32_t slot;            // units consumed in the current stage
  uint32_t c_left;          // units not yet consumed

  __device__ void setup(const uint8_t* s0, uint32_t c0, const uint8_t* s1, uint32_t c1) {
    p_src = c0 ? s0 : s1;
    seg1 = s1;
    seg0_end = s0 + static_cast<size_t>(c0) * kUnitBytes;
    seg1_end = s1 + static_cast<size_t>(c1) * kUnitBytes;
    p_left0 = c0;
    p_left = c0 + c1;
    c_left = c0 + c1;
    p_stage = stage = phase = slot = 0;
  }
  // lane 0: copy the next min(UPS, p_left) list units into stage p_stage.
  // Every copy is checked against the end of its segment; a copy that would
  // leave it is not issued and reported (the consumer's wait then times out).
  __device__ __forceinline__ void issue_next() {
    const uint32_t n = p_left < UPS ? p_left : UPS;
    uint8_t* dst = ring + p_stage * kStageBytes;
    uint64_t* bar = &bars[p_stage];
    if (n <= p_left0 || p_left0 == 0) {
      const uint8_t* end = p_left0 ? seg0_end : seg1_end;
      if (p_src + n * kUnitBytes > end) {
        atomicOr(status, kStatusBadLaunch);
        return;
      }
      mbar_arrive_expect_tx(bar, n * kUnitBytes);
      bulk_g2s(dst, p_src, n * kUnitBytes, bar, policy);
    } else {  // the group straddles the end of segment 0
      if (p_src + p_left0 * kUnitBytes > seg0_end || seg1 + (n - p_left0) * kUnitBytes > seg1_end) {
        atomicOr(status, kStatusBadLaunch);
        return;
      }
      mbar_arrive_expect_tx(bar, n * kUnitBytes);
      bulk_g2s(dst, p_src, p_left0 * kUnitBytes, bar, policy);
      bulk_g2s(dst + p_left0 * kUnitBytes, seg1, (n - p_left0) * kUnitBytes, bar, policy);
    }
  }
  // every lane: advance the producer counters past one issued group
  __device__ __forceinline__ void advance_producer() {
    const uint32_t n = p_left < UPS ? p_left : UPS;
    if (n < p_left0) {          // still inside segment 0
      p_src += n * kUnitBytes;
      p_left0 -= n;
    } else if (p_left0 > 0) {   // reached or crossed the end of segment 0
      p_src = seg1 + (n - p_left0) * kUnitBytes;
      p_left0 = 0;
    } else {                    // inside segment 1
      p_src += n * kUnitBytes;
    }
    p_left -= n;
    if (++p_stage == nst) p_stage = 0;
  }
  __device__ void init_and_prime(int lane) {
    if (lane == 0) {
      for (uint32_t s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    for (uint32_t s = 0; s < nst && p_left; ++s) {
      if (lane == 0) issue_next();
      advance_producer();
    }
    __syncwarp();
  }
  __device__ __forceinline__ bool wait_stage() {  // warp-uniform result
    return __all_sync(0xffffffffu, mbar_wait_bounded(&bars[stage], phase)) != 0;
  }
  __device__ __forceinline__ const uint8_t* unit_ptr() const {
    return ring + stage * kStageBytes + slot * kUnitBytes;
  }
  // Units left in the current stage (its group holds min(UPS, units left at
  // the group's start) units).
  __device__ __forceinline__ uint32_t stage_left() const {
    const uint32_t at_start = c_left + slot;
    return (at_start < UPS ? at_start : UPS) - slot;
  }
  // Consume `n` units of the current stage; refill the stage once finished.
  // The refill overwrites data this warp already read into registers and used,
  // so no proxy fence is needed (only generic-proxy writes need one).
  __device__ __forceinline__ void consume(uint32_t n, int lane) {
    c_left -= n;
    slot += n;
    if (slot == UPS || c_left == 0) {
      __syncwarp();
      if (p_left) {
        if (lane == 0) issue_next();
        advance_producer();
      }
      slot = 0;
      if (++stage == nst) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  // After an error: wait (bounded) for every stage that was issued and not
  // yet consumed, starting with the current one.
  __device__ void drain() {
    const uint32_t issued_not_consumed_units = c_left + slot - p_left;
    uint32_t groups = (issued_not_consumed_units + UPS - 1) / UPS;
    uint32_t s = stage, ph = phase;
    for (; groups; --groups) {
      (void)mbar_wait_bounded(&bars[s], ph);
      if (++s == nst) {
        s = 0;
        ph ^= 1;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Accumulate one unit.  acc[grp][parity][4] holds the C fragments for column
// group grp (8 columns each); even/odd chunks use separate accumulators to
// shorten the MMA dependency chain.
// ---------------------------------------------------------------------------
template <int NCOLS, bool FAST>
struct UnitMath {
  static constexpr int NGRP = NCOLS > 8 ? 2 : 1;

  // xl: this lane's fragment base, xs + (n*4 + t4)*32 with n its B column.
  __device__ __forceinline__ static void run(const uint8_t* ubuf, const uint8_t* xl, uint32_t kt, int lane,
                                             float (&acc)[NGRP][2][4]) {
    const int g = lane >> 2;
    const uint4 nib = lds128(ubuf + lane * 16);
    const uint2 sc = lds64(ubuf + kUnitNibBytes + g * 8);
    uint4 xf[NGRP][2];
#pragma unroll
    for (int grp = 0; grp < NGRP; ++grp) {
      const uint8_t* xk = xl + static_cast<size_t>(kt) * (NCOLS * 128) + grp * (8 * 128);
      xf[grp][0] = lds128(xk);
      xf[grp][1] = lds128(xk + 16);
    }
    uint32_t S[2][2], C[2][2];  // [block][row g / row g+8]
    S[0][0] = bf2_bcast(sc.x, 0);
    S[1][0] = bf2_bcast(sc.x, 1);
    S[0][1] = bf2_bcast(sc.y, 0);
    S[1][1] = bf2_bcast(sc.y, 1);
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int h = 0; h < 2; ++h) C[b][h] = FAST ? bf2_mul(S[b][h], kNeg8Sub) : 0u;
    const uint32_t words[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = j >> 1;
      uint32_t a[4];
      dequant_word<FAST>(words[j], S[b][0], C[b][0], S[b][1], C[b][1], a);
#pragma unroll
      for (int grp = 0; grp < NGRP; ++grp) {
        const uint4& v = xf[grp][j >> 1];
        const uint32_t b0 = (j & 1) ? v.z : v.x;
        const uint32_t b1 = (j & 1) ? v.w : v.y;
        mma_16816(acc[grp][j & 1], a[0], a[1], a[2], a[3], b0, b1);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Split-K fixup scratch.  A row tile covered by several warps is reduced by
// the last contributor (acq_rel arrival counter) summing every contributor's
// partial in warp order, so results are deterministic for a given grid.
// ---------------------------------------------------------------------------
struct Fixup {
  float* ws;          // [Wtot][2 slots][ntok][16]
  uint32_t* cnt;      // [RT] arrival counters, zero between launches
};

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Per-lane token values after a row tile.  Lane (g, t4) owns output columns
// 8*grp + 2*t4 + {0,1}: one token (hi + lo parts) when SPLIT, else two tokens.
template <int NCOLS, bool SPLIT>
struct LaneVals {
  static constexpr int NGRP = NCOLS > 8 ? 2 : 1;
  static constexpr int T = SPLIT ? NGRP : 2 * NGRP;
  float vg[T], vg8[T];
  __device__ __forceinline__ static int tok_of(int i, int t4) {
    return SPLIT ? 4 * i + t4 : 8 * (i >> 1) + 2 * t4 + (i & 1);
  }
  __device__ __forceinline__ void load(const float (&acc)[NGRP][2][4]) {
#pragma unroll
    for (int grp = 0; grp < NGRP; ++grp) {
      float v[2][2];  // [e][h]
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int h = 0; h < 2; ++h) v[e][h] = acc[grp][0][2 * h + e] + acc[grp][1][2 * h + e];
      if (SPLIT) {
        vg[grp] = v[0][0] + v[1][0];
        vg8[grp] = v[0][1] + v[1][1];
      } else {
        vg[2 * grp] = v[0][0];
        vg8[2 * grp] = v[0][1];
        vg[2 * grp + 1] = v[1][0];
        vg8[2 * grp + 1] = v[1][1];
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Finish a row tile: apply epi directly when this warp covered the whole tile,
// else publish the partial and let the last contributor reduce in warp order.
// ---------------------------------------------------------------------------
template <int NCOLS, bool SPLIT, class Epi>
__device__ __forceinline__ void flush_tile(const float (&acc)[(NCOLS > 8 ? 2 : 1)][2][4], bool whole, uint32_t r,
                                        uint32_t first_row, uint32_t KT, uint64_t U, uint32_t W,
                                        const Fixup& fx, uint32_t gw, int ntok, const Epi& epi) {
  using LV = LaneVals<NCOLS, SPLIT>;
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  LV lv;
  lv.load(acc);
  if (whole) {
#pragma unroll
    for (int i = 0; i < LV::T; ++i) {
      const int tok = LV::tok_of(i, t4);
      if (tok < ntok) epi.apply(r, g, tok, lv.vg[i], lv.vg8[i]);
    }
    return;
  }
  const uint32_t w_lo = warp_of_unit(static_cast<uint64_t>(r) * KT, U, W);
  const uint32_t w_hi = warp_of_unit((static_cast<uint64_t>(r) + 1) * KT - 1, U, W);
  const int slotw = (r == first_row) ? 0 : 1;
  const size_t slot_floats = static_cast<size_t>(ntok) * 16;
  float* mine = fx.ws + (static_cast<size_t>(gw) * 2 + slotw) * slot_floats;
#pragma unroll
  for (int i = 0; i < LV::T; ++i) {
    const int tok = LV::tok_of(i, t4);
    if (tok < ntok) {
      mine[tok * 16 + g] = lv.vg[i];
      mine[tok * 16 + g + 8] = lv.vg8[i];
    }
  }
  __syncwarp();
  uint32_t old = 0;
  if (lane == 0) old = atom_add_acq_rel_gpu(&fx.cnt[r], 1u);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != w_hi - w_lo) return;
  // Gather the contributors' partials CB at a time (independent loads in
  // flight), then add them in warp order.
  constexpr int CB = 8 / LV::T;
  float sg[LV::T], sg8[LV::T];
#pragma unroll
  for (int i = 0; i < LV::T; ++i) sg[i] = sg8[i] = 0.f;
  for (uint32_t w0 = w_lo; w0 <= w_hi; w0 += CB) {
    float pg[CB][LV::T], pg8[CB][LV::T];
#pragma unroll
    for (int c = 0; c < CB; ++c) {
      const uint32_t w = w0 + c;
      if (w > w_hi) continue;
      const uint32_t wfirst = static_cast<uint32_t>(range_start(w, U, W) / KT);
      const int ws = (r == wfirst) ? 0 : 1;
      const float* src = fx.ws + (static_cast<size_t>(w) * 2 + ws) * slot_floats;
#pragma unroll
      for (int i = 0; i < LV::T; ++i) {
        const int tok = LV::tok_of(i, t4);
        pg[c][i] = tok < ntok ? __ldcg(src + tok * 16 + g) : 0.f;
        pg8[c][i] = tok < ntok ? __ldcg(src + tok * 16 + g + 8) : 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < CB; ++c) {
      if (w0 + c > w_hi) continue;
#pragma unroll
      for (int i = 0; i < LV::T; ++i) {
        sg[i] += pg[c][i];
        sg8[i] += pg8[c][i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < LV::T; ++i) {
    const int tok = LV::tok_of(i, t4);
    if (tok < ntok) epi.apply(r, g, tok, sg[i], sg8[i]);
  }
  if (lane == 0) fx.cnt[r] = 0;
}

// ---------------------------------------------------------------------------
// Consume the unit range [u0, u1) of matrix m from the warp's ring, applying
// epi to every finished row tile.  Returns false on a timed-out copy (after
// draining the ring).  W = participating warps for this matrix.
// ---------------------------------------------------------------------------
template <int NCOLS, bool SPLIT, bool FAST, int UPS, class Epi>
__device__ bool consume_range(WarpRing<UPS>& ring, const Q4Mat& m, uint32_t u0, uint32_t u1,
                              const uint8_t* xs, const Fixup& fx, uint32_t gw, uint32_t W, int ntok,
                              const Epi& epi, uint32_t* status) {
  constexpr int NGRP = NCOLS > 8 ? 2 : 1;
  if (u0 >= u1) return true;
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const uint32_t KT = m.KT;
  const uint64_t U = static_cast<uint64_t>(m.RT) * KT;
  const uint32_t n_lane = NCOLS >= 8 ? g : (g & (NCOLS - 1));
  const uint8_t* xl = xs + (n_lane * 4 + t4) * 32;
  const uint32_t first_row = u0 / KT;
  uint32_t r = first_row;
  uint32_t kt = u0 - r * KT;
  uint32_t seg_kt0 = kt;  // k tile where the current row segment started
  uint32_t left = u1 - u0;
  float acc[NGRP][2][4];
#pragma unroll
  for (int a = 0; a < NGRP; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
  while (left) {
    if (ring.slot == 0 && !ring.wait_stage()) {
      if (lane == 0) atomicOr(status, kStatusMbarTimeout);
      ring.drain();
      return false;
    }
    const uint32_t sl = ring.stage_left();
    const uint32_t take = sl < left ? sl : left;
    const uint8_t* sp = ring.unit_ptr();
    if (take == UPS && kt + UPS < KT) {
      // Common case: a full stage inside one row tile -- straight-line code so
      // the UPS units' dequant and MMA chains interleave.
#pragma unroll
      for (int s = 0; s < UPS; ++s) UnitMath<NCOLS, FAST>::run(sp + s * kUnitBytes, xl, kt + s, lane, acc);
      kt += UPS;
      ring.consume(take, lane);
      left -= take;
      continue;
    }
#pragma unroll
    for (int s = 0; s < UPS; ++s) {
      if (static_cast<uint32_t>(s) < take) {
        UnitMath<NCOLS, FAST>::run(sp + s * kUnitBytes, xl, kt, lane, acc);
        if (++kt == KT) {
          flush_tile<NCOLS, SPLIT>(acc, seg_kt0 == 0, r, first_row, KT, U, W, fx, gw, ntok, epi);
#pragma unroll
          for (int a = 0; a < NGRP; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
          ++r;
          kt = seg_kt0 = 0;
        }
      }
    }
    ring.consume(take, lane);
    left -= take;
  }
  if (kt != seg_kt0) flush_tile<NCOLS, SPLIT>(acc, false, r, first_row, KT, U, W, fx, gw, ntok, epi);
  return true;
}

}  // namespace alv
