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
constexpr int kConsumerWarps = 15;  // + 1 producer warp = 16 warps, 4 per SM sub-partition

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
// Called by the consumer threads (threads [0, NTHR)) only.
template <int NCOLS, bool SPLIT, class Src>
__device__ void stage_frags(uint8_t* xs, uint32_t KT, const Src& src) {
  constexpr int BATCH = 8;  // entries per thread per pass: all loads in flight together
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  const uint32_t total = KT * 4 * NCOLS * 4;
  for (uint32_t base = 0; base < total; base += NTHR * BATCH) {
    float v[BATCH][4];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const uint32_t e = base + u * NTHR + threadIdx.x;
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
      const uint32_t e = base + u * NTHR + threadIdx.x;
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
// Warp-specialized unit rings.  Each consumer warp of a CTA owns a ring of
// nst stages of UPS units; one more warp (the producer) fills them with
// 1-D bulk copies through the TMA engine.  Per stage: `full` (producer
// arrive.expect_tx, completed by the copy) and `empty` (consumer lane 0
// arrives after the stage's data has been read and used).  A consumer's work
// list is up to two contiguous unit ranges (segment 0 then segment 1, e.g.
// FFN gate/up then down); a stage may straddle them.
// ---------------------------------------------------------------------------

// Work list of one consumer warp.
struct WorkList {
  const uint8_t* s0;   // first unit of segment 0
  const uint8_t* s1;   // first unit of segment 1
  uint32_t c0, c1;     // units in each segment
};

template <int UPS>
struct RingShape {
  static constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  // [rings: consumers x nst x stage][full: consumers x nst][empty: consumers x nst]
  __host__ __device__ static constexpr size_t smem_bytes(uint32_t nst) {
    return static_cast<size_t>(kConsumerWarps) * nst * (kStageBytes + 16);
  }
  __device__ static uint8_t* ring(uint8_t* smem, uint32_t nst, int c) {
    return smem + static_cast<size_t>(c) * nst * kStageBytes;
  }
  __device__ static uint64_t* full(uint8_t* smem, uint32_t nst, int c) {
    return reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kConsumerWarps) * nst * kStageBytes) + c * nst;
  }
  __device__ static uint64_t* empty(uint8_t* smem, uint32_t nst, int c) {
    return full(smem, nst, c) + kConsumerWarps * nst;
  }
  // All threads: initialize every barrier, then the caller syncs the CTA.
  __device__ static void init_barriers(uint8_t* smem, uint32_t nst) {
    uint64_t* f = full(smem, nst, 0);
    for (uint32_t i = threadIdx.x; i < 2u * kConsumerWarps * nst; i += blockDim.x) mbar_init(&f[i], 1);
    fence_mbar_init();
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Consumer side.
template <int UPS>
struct ConsumerRing {
  static constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  uint32_t ring_saddr;      // shared address of this warp's ring
  uint64_t* full;
  uint64_t* empty;
  uint32_t nst;
  uint32_t stage, phase;    // current stage and the parity of its next fill
  uint32_t slot;            // units consumed in the current stage
  uint32_t c_left;          // units not yet consumed

  __device__ void setup(uint8_t* smem, uint32_t nst_, int c, uint32_t total) {
    nst = nst_;
    ring_saddr = smem_u32(RingShape<UPS>::ring(smem, nst, c));
    full = RingShape<UPS>::full(smem, nst, c);
    empty = RingShape<UPS>::empty(smem, nst, c);
    stage = phase = slot = 0;
    c_left = total;
  }
  __device__ __forceinline__ bool wait_full() {  // warp-uniform result
    return __all_sync(0xffffffffu, mbar_wait_bounded(&full[stage], phase)) != 0;
  }
  __device__ __forceinline__ uint32_t unit_saddr() const {
    return ring_saddr + stage * kStageBytes + slot * kUnitBytes;
  }
  // Units left in the current stage (its group holds min(UPS, units left at
  // the group's start) units).
  __device__ __forceinline__ uint32_t stage_left() const {
    const uint32_t at_start = c_left + slot;
    return (at_start < UPS ? at_start : UPS) - slot;
  }
  // Consume n units of the current stage; hand a finished stage back.  The
  // stage's data has been read into registers and used, so the producer may
  // overwrite it (reads need no proxy fence).
  __device__ __forceinline__ void consume(uint32_t n, int lane) {
    c_left -= n;
    slot += n;
    if (slot == UPS || c_left == 0) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      slot = 0;
      if (++stage == nst) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  // Error path: keep the protocol moving without computing, so the producer
  // can finish and no copy is left in flight; stop if a copy never lands.
  __device__ void drain(int lane) {
    while (c_left) {
      if (slot == 0 && !wait_full()) return;
      consume(stage_left(), lane);
    }
  }
};

// Producer warp: lane c < kConsumerWarps feeds consumer warp c.  Non-blocking round
// robin: a lane issues its next group when the target stage is empty; the
// warp sleeps briefly when no lane made progress.  A lane that sees no
// progress for kWaitTimeoutNs records a timeout and stops.
template <int UPS>
__device__ void produce(uint8_t* smem, uint32_t nst, const WorkList& wl, uint64_t policy, uint32_t* status) {
  constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  const int lane = threadIdx.x & 31;
  const bool mine = lane < kConsumerWarps;
  uint8_t* ring = mine ? RingShape<UPS>::ring(smem, nst, lane) : nullptr;
  uint64_t* full = mine ? RingShape<UPS>::full(smem, nst, lane) : nullptr;
  uint64_t* empty = mine ? RingShape<UPS>::empty(smem, nst, lane) : nullptr;
  const uint8_t* seg0_end = wl.s0 + static_cast<size_t>(wl.c0) * kUnitBytes;
  const uint8_t* seg1_end = wl.s1 + static_cast<size_t>(wl.c1) * kUnitBytes;
  const uint8_t* src = wl.c0 ? wl.s0 : wl.s1;
  uint32_t left0 = wl.c0;
  uint32_t left = mine ? wl.c0 + wl.c1 : 0;
  uint32_t g = 0, pstage = 0, round = 0;  // group, its stage, and g / nst
  unsigned long long last = globaltimer_ns();
  while (__any_sync(0xffffffffu, left != 0)) {
    bool progress = false;
    if (left) {
      const bool ready = round == 0 || mbar_try_wait(&empty[pstage], (round - 1) & 1);
      if (ready) {
        const uint32_t n = left < UPS ? left : UPS;
        uint8_t* dst = ring + pstage * kStageBytes;
        bool ok;
        if (n <= left0 || left0 == 0) {
          ok = src + static_cast<size_t>(n) * kUnitBytes <= (left0 ? seg0_end : seg1_end);
          if (ok) {
            mbar_arrive_expect_tx(&full[pstage], n * kUnitBytes);
            bulk_g2s(dst, src, n * kUnitBytes, &full[pstage], policy);
          }
        } else {  // the group straddles the end of segment 0
          ok = src + static_cast<size_t>(left0) * kUnitBytes <= seg0_end &&
               wl.s1 + static_cast<size_t>(n - left0) * kUnitBytes <= seg1_end;
          if (ok) {
            mbar_arrive_expect_tx(&full[pstage], n * kUnitBytes);
            bulk_g2s(dst, src, left0 * kUnitBytes, &full[pstage], policy);
            bulk_g2s(dst + left0 * kUnitBytes, wl.s1, (n - left0) * kUnitBytes, &full[pstage], policy);
          }
        }
        if (!ok) {  // a copy would leave its segment: report, stop this lane
          atomicOr(status, kStatusBadLaunch);
          left = 0;
        } else {
          if (n < left0) {
            src += static_cast<size_t>(n) * kUnitBytes;
            left0 -= n;
          } else if (left0 > 0) {
            src = wl.s1 + static_cast<size_t>(n - left0) * kUnitBytes;
            left0 = 0;
          } else {
            src += static_cast<size_t>(n) * kUnitBytes;
          }
          left -= n;
          ++g;
          if (++pstage == nst) {
            pstage = 0;
            ++round;
          }
          progress = true;
          last = globaltimer_ns();
        }
      } else if (globaltimer_ns() - last > kWaitTimeoutNs) {
        atomicOr(status, kStatusMbarTimeout);
        left = 0;
      }
    }
    if (!__any_sync(0xffffffffu, progress)) __nanosleep(128);
  }
}

// Barrier 2 (all 16 warps): the producer waits there until the consumers have
// staged their activations, so those few latency-critical loads are not
// queued behind the weight stream.
__device__ __forceinline__ void producer_wait_release() {
  asm volatile("bar.sync 2, %0;" ::"n"((kConsumerWarps + 1) * 32) : "memory");
}
__device__ __forceinline__ void consumers_release_producer() {
  asm volatile("bar.arrive 2, %0;" ::"n"((kConsumerWarps + 1) * 32) : "memory");
}

// Named barrier and AND-reduction over the consumer warps only (the producer
// warp runs free).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}
__device__ __forceinline__ bool consumers_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kConsumerWarps * 32)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// Accumulate one unit.  acc[grp][parity][4] holds the C fragments for column
// group grp (8 columns each); even/odd chunks use separate accumulators to
// shorten the MMA dependency chain.
// ---------------------------------------------------------------------------
template <int NCOLS, bool FAST>
struct UnitMath {
  static constexpr int NGRP = NCOLS > 8 ? 2 : 1;
  static constexpr int kXStride = NCOLS * 128;  // fragment bytes per k tile

  // Core: nibble word, scale pair and fragments already in registers.
  __device__ __forceinline__ static void math(const uint4& nib, const uint2& sc, const uint4 (&xf)[NGRP][2],
                                              float (&acc)[NGRP][2][4]) {
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

  // Unit S of a stage: nib_base = stage + lane*16, sc_base = stage + 512 + g*8,
  // x_base = this lane's fragments of the stage's first k tile.
  template <int S>
  __device__ __forceinline__ static void at(uint32_t nib_base, uint32_t sc_base, uint32_t x_base,
                                            float (&acc)[NGRP][2][4]) {
    const uint4 nib = lds128_at<S * kUnitBytes>(nib_base);
    const uint2 sc = lds64_at<S * kUnitBytes>(sc_base);
    uint4 xf[NGRP][2];
    xf[0][0] = lds128_at<S * kXStride>(x_base);
    xf[0][1] = lds128_at<S * kXStride + 16>(x_base);
    if constexpr (NGRP > 1) {
      xf[NGRP - 1][0] = lds128_at<S * kXStride + 1024>(x_base);
      xf[NGRP - 1][1] = lds128_at<S * kXStride + 1024 + 16>(x_base);
    }
    math(nib, sc, xf, acc);
  }

  // Generic form (runtime unit address and k tile; shared-space addresses).
  __device__ __forceinline__ static void run_saddr(uint32_t u, uint32_t x_saddr, uint32_t kt, int lane,
                                                   float (&acc)[NGRP][2][4]) {
    const int g = lane >> 2;
    at<0>(u + lane * 16, u + kUnitNibBytes + g * 8, x_saddr + kt * kXStride, acc);
  }
};

// Straight-line run of units S..UPS-1 of a full stage.
template <int NCOLS, bool FAST, int S, int UPS>
struct StageUnroll {
  __device__ __forceinline__ static void go(uint32_t nib_base, uint32_t sc_base, uint32_t x_base,
                                            float (&acc)[NCOLS > 8 ? 2 : 1][2][4]) {
    UnitMath<NCOLS, FAST>::template at<S>(nib_base, sc_base, x_base, acc);
    StageUnroll<NCOLS, FAST, S + 1, UPS>::go(nib_base, sc_base, x_base, acc);
  }
};
template <int NCOLS, bool FAST, int UPS>
struct StageUnroll<NCOLS, FAST, UPS, UPS> {
  __device__ __forceinline__ static void go(uint32_t, uint32_t, uint32_t, float (&)[NCOLS > 8 ? 2 : 1][2][4]) {}
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
  constexpr int CB = 16 / LV::T;
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
__device__ bool consume_range(ConsumerRing<UPS>& ring, const Q4Mat& m, uint32_t u0, uint32_t u1,
                              const uint8_t* xs, const Fixup& fx, uint32_t gw, uint32_t W, int ntok,
                              const Epi& epi, uint32_t* status) {
  constexpr int NGRP = NCOLS > 8 ? 2 : 1;
  if (u0 >= u1) return true;
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const uint32_t KT = m.KT;
  const uint64_t U = static_cast<uint64_t>(m.RT) * KT;
  const uint32_t n_lane = NCOLS >= 8 ? g : (g & (NCOLS - 1));
  const uint8_t* xl = xs + (n_lane * 4 + t4) * 32;
  const uint32_t x_saddr = smem_u32(xl);
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
    if (ring.slot == 0 && !ring.wait_full()) {
      if (lane == 0) atomicOr(status, kStatusMbarTimeout);
      return false;
    }
    const uint32_t sl = ring.stage_left();
    const uint32_t take = sl < left ? sl : left;
    const uint32_t su = ring.unit_saddr();
    if (take == UPS && kt + UPS < KT) {
      // Common case: a full stage inside one row tile -- straight-line code so
      // the UPS units' dequant and MMA chains interleave; all shared-memory
      // offsets are immediates.
      StageUnroll<NCOLS, FAST, 0, UPS>::go(su + lane * 16, su + kUnitNibBytes + g * 8,
                                           x_saddr + kt * UnitMath<NCOLS, FAST>::kXStride, acc);
      kt += UPS;
      ring.consume(take, lane);
      left -= take;
      continue;
    }
#pragma unroll
    for (int s = 0; s < UPS; ++s) {
      if (static_cast<uint32_t>(s) < take) {
        UnitMath<NCOLS, FAST>::run_saddr(su + s * kUnitBytes, x_saddr, kt, lane, acc);
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
