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
// Units per ring stage (one bulk-copy group).
#ifndef ALV_UNITS_PER_STAGE
#define ALV_UNITS_PER_STAGE 8
#endif

// Warps per CTA (one CTA per SM), each streaming its own unit range.
#ifndef ALV_WARPS
#define ALV_WARPS 16
#endif
constexpr int kConsumerWarps = ALV_WARPS;
constexpr uint32_t kWarpsPerCtaS = kConsumerWarps;

struct Q4Mat {
  const uint8_t* units;  // RT*KT units of kUnitBytes
  uint32_t RT;           // row tiles of 16 rows
  uint32_t KT;           // k tiles of 64 columns
  uint32_t fast;         // 1: subnormal-magic dequant; 0: generic
  float scale_mul;       // 2^je (fast) or 1 (generic)
};

// Round-down division of 32-bit numerators by a divisor d >= 1 fixed at
// launch: one multiply-high, an add, a subtract and two shifts instead of the
// software division loop (Granlund and Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994, section 4): with l = ceil(log2 d)
// and m = floor(2^32 (2^l - d) / d) + 1, t = mulhi(m, n) gives
// n / d = (t + ((n - t) >> min(l, 1))) >> max(l - 1, 0).  Built on the host.
struct FastDiv {
  uint32_t d, m, s1, s2;
  __host__ static FastDiv make(uint32_t d) {
    FastDiv f{};
    f.d = d ? d : 1;
    uint32_t l = 0;
    while ((uint64_t{1} << l) < f.d) ++l;
    f.m = static_cast<uint32_t>((uint64_t{1} << 32) * ((uint64_t{1} << l) - f.d) / f.d + 1);
    f.s1 = l < 1 ? l : 1;
    f.s2 = l > 1 ? l - 1 : 0;
    return f;
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#ifdef __CUDA_ARCH__
    const uint32_t t = __umulhi(m, n);
#else
    const uint32_t t = static_cast<uint32_t>((static_cast<uint64_t>(m) * n) >> 32);
#endif
    return (t + ((n - t) >> s1)) >> s2;
  }
};

// How a matrix's RT x KT units are split over the grid: CTA c owns one
// contiguous unit range and its warps split that range.  Row-aligned when
// asked for (`row_aligned`: the FFN's gate/up matrices, whose split-K
// reduction then never leaves the CTA) or when every CTA can take whole row
// tiles at < 1/32 imbalance (then no row tile spans two CTAs and the split-K
// reduction stays in shared memory); otherwise unit-balanced: W
// participating warps numbered CTA-major, warp gw owning
// [floor(gw U / W), floor((gw + 1) U / W)), W chosen so that every warp owns
// >= 1 and >= ceil(KT / 16) units.  A row-aligned split of RT < nctas row
// tiles leaves CTAs without work.
//
// Built on the host for the launch's grid (every divisor fixed then, so the
// device side is 32-bit multiply-high arithmetic: the kernels evaluate these
// at their start and in every split-K reduction, on the critical path).
// Limits (checked by make): U < 2^28 units, RT < 2^24 row tiles.
struct Partition {
  uint32_t RT, KT, nctas, aligned;
  uint32_t U, W;        // units; participating warps (unit-balanced)
  uint32_t qUW, rUW;    // U / W and U % W
  float invU;           // 1 / U, for the warp-of-unit estimate
  FastDiv kt, nct, wd;  // division by KT, nctas and W

  __host__ static bool fits(uint64_t RT, uint64_t KT) { return RT < (1u << 24) && RT * KT < (1u << 28); }
  __host__ static Partition make(uint32_t RT, uint32_t KT, uint32_t nctas, bool row_aligned = false) {
    Partition p{};
    p.RT = RT;
    p.KT = KT;
    p.nctas = nctas;
    p.U = RT * KT;
    const uint64_t per = (static_cast<uint64_t>(RT) + nctas - 1) / nctas;
    p.aligned = row_aligned || (RT >= nctas && per * nctas * 32 <= static_cast<uint64_t>(RT) * 33);
    const uint32_t min_units = (KT + 15) / 16;
    uint64_t w = p.U / (min_units ? min_units : 1);
    if (w < 1) w = 1;
    const uint64_t wtot = static_cast<uint64_t>(nctas) * kWarpsPerCtaS;
    p.W = static_cast<uint32_t>(w < wtot ? w : wtot);
    p.qUW = p.U / p.W;
    p.rUW = p.U % p.W;
    p.invU = p.U ? 1.0f / static_cast<float>(p.U) : 0.f;
    p.kt = FastDiv::make(KT);
    p.nct = FastDiv::make(nctas);
    p.wd = FastDiv::make(p.W);
    return p;
  }
  // First unit of warp gw of the unit-balanced split: floor(gw U / W), as
  // gw (U / W) + (gw (U % W)) / W (gw (U % W) < W^2 < 2^32).
  __host__ __device__ __forceinline__ uint32_t range_start(uint32_t gw) const { return gw * qUW + wd.div(gw * rUW); }
  // First unit of CTA c (c = nctas gives U).
  __host__ __device__ __forceinline__ uint32_t cta_begin(uint32_t c) const {
    if (aligned) return nct.div(c * RT) * KT;
    const uint32_t gw = c * kWarpsPerCtaS;
    return range_start(gw < W ? gw : W);
  }
  // Units [u0, u1) of warp w of CTA c (possibly empty).
  __host__ __device__ __forceinline__ void warp_range(uint32_t c, uint32_t w, uint32_t& u0, uint32_t& u1) const {
    if (aligned) {
      const uint32_t c0 = cta_begin(c), len = cta_begin(c + 1) - c0;
      u0 = c0 + len * w / kWarpsPerCtaS;
      u1 = c0 + len * (w + 1) / kWarpsPerCtaS;
      return;
    }
    const uint32_t gw = c * kWarpsPerCtaS + w;
    if (gw >= W) {
      u0 = u1 = U;
      return;
    }
    u0 = range_start(gw);
    u1 = range_start(gw + 1);
  }
  // The warp whose range holds unit u (unit-balanced): the gw with
  // range_start(gw) <= u < range_start(gw + 1), i.e. floor(((u + 1) W - 1) / U);
  // a float estimate corrected exactly with 64-bit products.
  __host__ __device__ __forceinline__ uint32_t warp_of_unit(uint32_t u) const {
    const uint64_t n = static_cast<uint64_t>(u + 1) * W - 1;
    uint32_t q = static_cast<uint32_t>(static_cast<float>(n) * invU);
    if (q >= W) q = W - 1;
    while (q > 0 && static_cast<uint64_t>(q) * U > n) --q;
    while (q + 1 < W && static_cast<uint64_t>(q + 1) * U <= n) ++q;
    return q;
  }
  // CTA holding unit u (unit-balanced partitions only).
  __host__ __device__ __forceinline__ uint32_t cta_of_unit(uint32_t u) const { return warp_of_unit(u) / kWarpsPerCtaS; }
};

// ---------------------------------------------------------------------------
// Dequantize one 32-bit nibble word into the four bf16x2 A-fragment registers.
// S*/C* are bf16x2 broadcasts of the scale (and -8*scale) for rows g and g+8;
// S16g8 is the fast-path scale of row g+8 times 2^-4.
//
// Fast path: bits 0-7 of a bf16 half, read as an integer v, encode the value
// v * 2^-133 whether bit 7 (the exponent's lowest bit) is set or not, so a
// nibble masked in place at bits 0-3 is u * 2^-133 and one at bits 4-7 is
// 16u * 2^-133.  The first pairs with S, the second with S/16 (an exact
// power-of-two rescale), and one shift by 8 brings the upper two nibbles down:
// one shift and four masks per word instead of three shifts and four masks.
// ---------------------------------------------------------------------------
template <bool FAST>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t Sg, uint32_t Cg, uint32_t Sg8, uint32_t Cg8,
                                             uint32_t S16g8, uint32_t (&a)[4]) {
  const uint32_t m = 0x000F000Fu;
  if (FAST) {
    const uint32_t w8 = w >> 8;
    a[0] = bf2_fma(w & m, Sg, Cg);
    a[1] = bf2_fma(w & (m << 4), S16g8, Cg8);
    a[2] = bf2_fma(w8 & m, Sg, Cg);
    a[3] = bf2_fma(w8 & (m << 4), S16g8, Cg8);
  } else {
    const uint32_t p0 = w & m, p1 = (w >> 4) & m, p2 = (w >> 8) & m, p3 = (w >> 12) & m;
    const uint32_t magic = 0x43004300u;   // bf16x2 (128, 128)
    const uint32_t m136 = 0x43084308u;    // bf16x2 (136, 136)
    a[0] = bf2_mul(bf2_sub(p0 | magic, m136), Sg);
    a[1] = bf2_mul(bf2_sub(p1 | magic, m136), Sg8);
    a[2] = bf2_mul(bf2_sub(p2 | magic, m136), Sg);
    a[3] = bf2_mul(bf2_sub(p3 | magic, m136), Sg8);
  }
}

// bf16x2 (2^-4, 2^-4)
constexpr uint32_t kPow2m4 = 0x3D803D80u;

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
// Per-warp unit rings.  Each warp of a CTA owns a ring of nst stages of UPS
// units in shared memory, filled by 1-D bulk copies through the TMA engine
// (one `full` mbarrier per stage: arrive.expect_tx, completed by the copies).
// The warp refills its own ring: when it has used a stage, its lane 0 issues
// the copies of the group nst groups ahead into that stage, so nst groups
// are always in flight and no warp spends issue slots polling.  A warp's
// work is a sequence of contiguous unit ranges (segments: e.g. FFN gate/up
// then down, layer after layer); groups of UPS units are cut from the
// concatenated sequence, so a stage may span segment ends.
// ---------------------------------------------------------------------------

// A warp's work is a sequence of segments: contiguous unit ranges of one
// matrix.  get(i, ...) gives segment i's first unit, its length, the matrix's
// k tiles per row tile (KT) and the k tile the segment starts at.

// Work of one warp as two segments (segment 0 then segment 1).
struct WorkList {
  const uint8_t* s0;   // first unit of segment 0
  const uint8_t* s1;   // first unit of segment 1
  uint32_t c0, c1;     // units in each segment
  uint32_t kt0, kt1;   // k tile of each segment's first unit
  uint32_t KT0, KT1;   // k tiles per row tile of each segment's matrix
  __device__ uint32_t nseg() const { return 2; }
  __device__ void get(uint32_t i, const uint8_t*& base, uint32_t& n, uint32_t& KT, uint32_t& kt) const {
    base = i ? s1 : s0;
    n = i ? c1 : c0;
    KT = i ? KT1 : KT0;
    kt = i ? kt1 : kt0;
  }
};

// Per-layer weights of a fused FFN stack.
struct LayerW {
  const uint8_t* gu;   // gate/up units of the layer
  const uint8_t* dn;   // down units
  float gu_mul, dn_mul;  // dequant epilogue multipliers (2^je, or 1)
  uint32_t pad[2];
};

// Work of one warp over a whole FFN stack: layer l contributes gate/up units
// [a0, a0+na) then down units [b0, b0+nb).
struct StackWork {
  const LayerW* layers;
  uint32_t L, a0, na, b0, nb;
  uint32_t KTA, KTB;   // k tiles per row tile of gate/up and of down
  uint32_t kta, ktb;   // k tile of unit a0 (a0 % KTA) and of unit b0
  __device__ uint32_t nseg() const { return 2 * L; }
  __device__ void get(uint32_t i, const uint8_t*& base, uint32_t& n, uint32_t& KT, uint32_t& kt) const {
    const LayerW* lw = layers + (i >> 1);
    if (i & 1) {
      base = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&lw->dn))) +
             static_cast<size_t>(b0) * kUnitBytes;
      n = nb;
      KT = KTB;
      kt = ktb;
    } else {
      base = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&lw->gu))) +
             static_cast<size_t>(a0) * kUnitBytes;
      n = na;
      KT = KTA;
      kt = kta;
    }
  }
};

// [rings: warps x nst x stage][full barriers: warps x nst], padded to 128
// bytes so whatever follows keeps 16-byte (vector / bulk copy) alignment.
template <int UPS>
struct RingShape {
  static constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  __host__ __device__ static constexpr size_t smem_bytes(uint32_t nst) {
    return (static_cast<size_t>(kConsumerWarps) * nst * (kStageBytes + 8) + 127) / 128 * 128;
  }
  __device__ static uint8_t* ring(uint8_t* smem, uint32_t nst, int c) {
    return smem + static_cast<size_t>(c) * nst * kStageBytes;
  }
  __device__ static uint64_t* full(uint8_t* smem, uint32_t nst, int c) {
    return reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kConsumerWarps) * nst * kStageBytes) + c * nst;
  }
  // All threads: initialize every barrier, then the caller syncs the CTA.
  __device__ static void init_barriers(uint8_t* smem, uint32_t nst) {
    uint64_t* f = full(smem, nst, 0);
    for (uint32_t i = threadIdx.x; i < kConsumerWarps * nst; i += blockDim.x) mbar_init(&f[i], 1);
    fence_mbar_init();
  }
  // One warp: initialize its own ring's barriers (no CTA-wide sync needed
  // before the warp issues its first copies).
  __device__ static void init_warp_barriers(uint8_t* smem, uint32_t nst, int c) {
    uint64_t* f = full(smem, nst, c);
    const uint32_t lane = threadIdx.x & 31;
    if (lane < nst) mbar_init(&f[lane], 1);
    fence_mbar_init();
    __syncwarp();
  }
};

// Lane 0 only (pred): arm `bar` for `bytes` and start one bulk copy of them.
__device__ __forceinline__ void lane0_arm_and_copy(bool pred, uint32_t bar, uint32_t bytes, uint32_t dst,
                                                   const void* src, uint64_t policy) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %0, 0;\n\t"
      "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n\t"
      "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%3], [%4], %2, [%1], %5;\n\t}" ::"r"(static_cast<uint32_t>(pred)),
      "r"(bar), "r"(bytes), "r"(dst), "l"(src), "l"(policy)
      : "memory");
}

// Copy cursor: position in the warp's segment sequence.
struct Cursor {
  const uint8_t* src;   // next unit to copy
  uint32_t seg_left;    // units of the current segment not yet copied
  uint32_t row_left;    // units until the current row tile ends
  uint32_t KT;          // k tiles per row tile of the current segment
  uint32_t si;          // segments entered so far
};

// Rare path of a refill: step to the next non-empty segment.
template <class Seq>
__device__ __noinline__ Cursor next_segment(Cursor c, const Seq* seq) {
  const Seq sq = *seq;
  const uint32_t nseg = sq.nseg();
  while (c.seg_left == 0 && c.si < nseg) {
    uint32_t kt;
    sq.get(c.si++, c.src, c.seg_left, c.KT, kt);
    c.row_left = c.KT - kt;
  }
  return c;
}

// One warp's ring.  Groups are cut at segment and row-tile ends, so a stage
// always holds units of one row tile of one matrix: min(UPS, units to the
// row tile's end, units left in the segment).  The consumer derives the same
// size from its own position.  The copy cursor lives in registers and is
// advanced by all lanes alike (uniform control flow); lane 0 alone issues the
// copies.
template <int UPS, class Seq>
struct ConsumerRing {
  static constexpr uint32_t kStageBytes = UPS * kUnitBytes;
  uint32_t ring_saddr;      // shared address of this warp's ring
  uint32_t full_saddr;      // shared address of this warp's full[0]
  uint32_t nst;
  uint32_t stage, phase;    // current stage and the parity of its next fill
  uint32_t inflight;        // groups copied and not yet released
  uint32_t cp_left;         // units of the sequence not yet copied
  uint32_t primed;          // stages issued by setup()
  Cursor cur;
  const Seq* seq;           // this warp's work sequence (shared memory)

  // total = units of the whole sequence.  Issues the copies of the first
  // `first` stages (all of them by default; all lanes call).  A kernel that
  // must read something latency-critical right after it starts (its input
  // vector) primes one stage, reads its input while only that much of its own
  // weight stream is queued ahead of it, then calls fill_rest().
  __device__ void setup(uint8_t* smem, uint32_t nst_, int c, uint32_t total, const Seq* seq_, uint32_t first = ~0u) {
    nst = nst_;
    ring_saddr = smem_u32(RingShape<UPS>::ring(smem, nst, c));
    full_saddr = smem_u32(RingShape<UPS>::full(smem, nst, c));
    stage = phase = inflight = 0;
    cp_left = total;
    cur = Cursor{nullptr, 0, 0, 1, 0};
    seq = seq_;
    primed = first < nst ? first : nst;
    for (uint32_t s = 0; s < primed; ++s) refill(s);
  }
  // Issue the stages setup() held back (before the first release()).
  __device__ __forceinline__ void fill_rest() {
    for (uint32_t s = primed; s < nst; ++s) refill(s);
    primed = nst;
  }
  // Copy the next group into stage s (a single bulk copy).  The stage's
  // previous contents were loaded into registers and consumed by the warp's
  // earlier instructions, so the copy cannot overwrite data still needed.
  __device__ __forceinline__ void refill(uint32_t s) {
    if (cp_left == 0) return;
    if (cur.seg_left == 0) cur = next_segment(cur, seq);
    uint32_t n = cur.seg_left < cur.row_left ? cur.seg_left : cur.row_left;
    if (n > UPS) n = UPS;
    if (n == 0) return;  // cannot happen (cp_left counts the segments); the wait for it times out
    lane0_arm_and_copy((threadIdx.x & 31) == 0, full_saddr + s * 8, n * kUnitBytes, ring_saddr + s * kStageBytes,
                       cur.src, l2_policy_evict_first());
    cur.src += static_cast<size_t>(n) * kUnitBytes;
    cur.seg_left -= n;
    cur.row_left -= n;
    if (cur.row_left == 0) cur.row_left = cur.KT;
    cp_left -= n;
    ++inflight;
  }
  __device__ __forceinline__ bool wait_full() {  // warp-uniform result
    return __all_sync(0xffffffffu, mbar_wait_bounded_s(full_saddr + stage * 8, phase)) != 0;
  }
  __device__ __forceinline__ uint32_t stage_saddr() const { return ring_saddr + stage * kStageBytes; }
  // The current stage has been used: refill it with the group nst ahead and
  // move on.
  __device__ __forceinline__ void release() {
    __syncwarp();
    --inflight;
    refill(stage);
    if (++stage == nst) {
      stage = 0;
      phase ^= 1;
    }
  }
  // Error path: let every copy in flight land (bounded), issue no more.
  __device__ void drain() {
    while (inflight) {
      if (!wait_full()) return;
      --inflight;
      if (++stage == nst) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
};

// Named barrier and AND-reduction over the CTA's warps (barrier 1).
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
    uint32_t S16[2];  // row g+8 scales times 2^-4 (the nibbles at bits 4-7)
#pragma unroll
    for (int b = 0; b < 2; ++b) S16[b] = FAST ? bf2_mul(S[b][1], kPow2m4) : 0u;
    const uint32_t words[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = j >> 1;
      uint32_t a[4];
      dequant_word<FAST>(words[j], S[b][0], C[b][0], S[b][1], C[b][1], S16[b], a);
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

// Units per straight-line run in the consumer's inner loop (a divisor of the
// stage size): longer runs interleave more independent work, shorter ones
// keep the loop's instructions resident in the instruction cache.
#ifndef ALV_STAGE_UNROLL
#define ALV_STAGE_UNROLL ALV_UNITS_PER_STAGE
#endif
constexpr int kStageUnroll = ALV_STAGE_UNROLL;

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
// Split-K scratch.  A row tile split between warps of one CTA is reduced in
// shared memory once the CTA's warps are done (warp partials summed in warp
// order); a row tile split between CTAs is then finished by the last CTA to
// arrive (acq_rel arrival counter), CTA partials summed in CTA order.  Fixed
// orders: results are deterministic for a given grid.
// ---------------------------------------------------------------------------
struct Fixup {
  float* ws;          // global: [nctas][2 slots][ntok][16] CTA partials
  uint32_t* cnt;      // global: [RT] arrival counters, zero between launches
  float* part;        // shared: [warps][2 slots][ntok][16] warp partials
};

// Shared-memory bytes of the warp partials.
__host__ __device__ constexpr size_t part_bytes(int ntok) {
  return static_cast<size_t>(kConsumerWarps) * 2 * ntok * 16 * sizeof(float);
}

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
// Finish a row tile: apply epi directly when this warp covered the whole
// tile, else park the partial for cta_fixup.
// ---------------------------------------------------------------------------
template <int NCOLS, bool SPLIT, class Epi>
__device__ __forceinline__ void flush_tile(const float (&acc)[(NCOLS > 8 ? 2 : 1)][2][4], bool whole, uint32_t r,
                                        uint32_t first_row, const Fixup& fx, int ntok, const Epi& epi) {
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
  // Partial row tile: park it in this warp's shared slot (0: the range's
  // first row, 1: its last row); cta_fixup reduces it after the phase.
  const int slotw = (r == first_row) ? 0 : 1;
  float* mine = fx.part + (static_cast<size_t>(threadIdx.x >> 5) * 2 + slotw) * ntok * 16;
#pragma unroll
  for (int i = 0; i < LV::T; ++i) {
    const int tok = LV::tok_of(i, t4);
    if (tok < ntok) {
      mine[tok * 16 + g] = lv.vg[i];
      mine[tok * 16 + g + 8] = lv.vg8[i];
    }
  }
}

// ---------------------------------------------------------------------------
// After every warp of the CTA finished its range: reduce the row tiles that
// were split between warps (shared memory, warp order) and apply epi to the
// ones inside the CTA's range.  Row tiles shared with other CTAs (unit-
// balanced partitions only) get a CTA partial in fx.ws; unless DEFER, the
// last CTA to arrive (acq_rel counter) sums them in CTA order and applies
// epi.  With DEFER the partials are left for the consumer of the result to
// sum after the next grid barrier (the FFN stack's next glue).  All warps of
// the CTA call this (it syncs them).
// ---------------------------------------------------------------------------
template <bool DEFER = false, class Epi>
__device__ void cta_fixup(const Partition& pt, const uint32_t* wr, const Fixup& fx, int ntok, const Epi& epi) {
  // wr[4 * w + 0 / 1]: unit range [u0, u1) of warp w of this CTA (shared memory)
  consumers_sync();  // every warp's partials are in shared memory
  const uint32_t KT = pt.KT, c = blockIdx.x;
  const uint32_t c0 = pt.cta_begin(c), c1 = pt.cta_begin(c + 1);
  if (c0 >= c1) return;
  const uint32_t r_lo = pt.kt.div(c0), r_hi = pt.kt.div(c1 - 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t slot_floats = static_cast<size_t>(ntok) * 16;
  // Lane w holds warp w's range and the row its slot 0 belongs to, so the
  // contributors of a row tile are one ballot and every partial load of an
  // element is in flight at once (a loop over the warps would pay one
  // shared-memory round trip per warp and step).
  const uint32_t lu0 = lane < kConsumerWarps ? wr[4 * lane] : 0u;
  const uint32_t lu1 = lane < kConsumerWarps ? wr[4 * lane + 1] : 0u;
  const uint32_t lrow0 = pt.kt.div(lu0);
  for (uint32_t r = r_lo + warp; r <= r_hi; r += kWarpsPerCtaS) {
    const uint32_t rb = r * KT, re = rb + KT;
    const uint32_t ib = rb > c0 ? rb : c0, ie = re < c1 ? re : c1;  // this CTA's part of the row tile
    const bool inside = rb >= c0 && re <= c1;
    // Contributing warps (contiguous): non-empty ranges that meet [ib, ie).
    const uint32_t meets = __ballot_sync(0xffffffffu, lu0 < lu1 && lu0 < ie && lu1 > ib);
    if (!meets) continue;
    const bool whole = __shfl_sync(0xffffffffu, lu0 <= rb && lu1 >= re, 31 - __clz(meets));
    if (inside && __popc(meets) == 1 && whole) continue;  // one warp held the whole tile: applied already
    const uint32_t slot1 = __ballot_sync(0xffffffffu, r != lrow0);  // warp w parked row r in its slot 1
    const int cslot = (r == r_lo) ? 0 : 1;
    float* cpart = fx.ws + (static_cast<size_t>(c) * 2 + cslot) * slot_floats;
    for (uint32_t e = lane; e < 8u * ntok; e += 32) {
      const int g = e & 7, tok = e >> 3;
      float pg[kConsumerWarps], pg8[kConsumerWarps];
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        pg[w] = pg8[w] = 0.f;
        if ((meets >> w) & 1u) {
          const float* src = fx.part + (static_cast<size_t>(w) * 2 + ((slot1 >> w) & 1u)) * slot_floats;
          pg[w] = src[tok * 16 + g];
          pg8[w] = src[tok * 16 + g + 8];
        }
      }
      float vg = 0.f, vg8 = 0.f;  // warp order
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w)
        if ((meets >> w) & 1u) {
          vg += pg[w];
          vg8 += pg8[w];
        }
      if (inside) {
        epi.apply(r, g, tok, vg, vg8);
      } else if constexpr (DEFER) {  // the epilogue may pre-scale parked partials
        cpart[tok * 16 + g] = epi.park(vg);
        cpart[tok * 16 + g + 8] = epi.park(vg8);
      } else {
        cpart[tok * 16 + g] = vg;
        cpart[tok * 16 + g + 8] = vg8;
      }
    }
    if (inside || DEFER) continue;
    // Shared with other CTAs: publish, count, and the last CTA finishes.
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(&fx.cnt[r], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    const uint32_t cta_lo = pt.cta_of_unit(rb), cta_hi = pt.cta_of_unit(re - 1);
    if (old != cta_hi - cta_lo) continue;
    __threadfence();  // every lane reads the other CTAs' partials after the count
    for (uint32_t e = lane; e < 8u * ntok; e += 32) {
      const int g = e & 7, tok = e >> 3;
      float vg = 0.f, vg8 = 0.f;
      for (uint32_t cc = cta_lo; cc <= cta_hi; ++cc) {
        const uint32_t cfirst = pt.kt.div(pt.cta_begin(cc));
        const float* src = fx.ws + (static_cast<size_t>(cc) * 2 + (r == cfirst ? 0 : 1)) * slot_floats;
        vg += __ldcg(src + tok * 16 + g);
        vg8 += __ldcg(src + tok * 16 + g + 8);
      }
      epi.apply(r, g, tok, vg, vg8);
    }
    if (lane == 0) fx.cnt[r] = 0;
  }
}

// ---------------------------------------------------------------------------
// Consume the unit range [u0, u1) of matrix m from the warp's ring, applying
// epi to every row tile the warp holds whole and parking the partial ones for
// cta_fixup.  Returns false on a timed-out copy.
// ---------------------------------------------------------------------------
template <int NCOLS, bool SPLIT, bool FAST, int UPS, class Seq, class Epi>
__device__ bool consume_range(ConsumerRing<UPS, Seq>& ring, const Q4Mat& m, uint32_t u0, uint32_t u1,
                              const uint8_t* xs, const Fixup& fx, int ntok, const Epi& epi, uint32_t* status) {
  constexpr int NGRP = NCOLS > 8 ? 2 : 1;
  if (u0 >= u1) return true;
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const uint32_t KT = m.KT;
  const uint32_t n_lane = NCOLS >= 8 ? g : (g & (NCOLS - 1));
  const uint32_t x_saddr = smem_u32(xs + (n_lane * 4 + t4) * 32);
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
    if (!ring.wait_full()) {
      if (lane == 0) atomicOr(status, kStatusMbarTimeout);
      return false;
    }
    const uint32_t su = ring.stage_saddr();
    // This stage's group: the units up to the row tile's end, at most UPS.
    uint32_t n = KT - kt;
    if (n > UPS) n = UPS;
    if (n > left) n = left;
    if (n == UPS) {
      // Common case: a full stage -- straight-line runs of kStageUnroll units
      // so their dequant and MMA chains interleave, with immediate
      // shared-memory offsets inside a run.
#pragma unroll 1
      for (uint32_t q = 0; q < UPS; q += kStageUnroll) {
        const uint32_t uq = su + q * kUnitBytes;
        StageUnroll<NCOLS, FAST, 0, kStageUnroll>::go(uq + lane * 16, uq + kUnitNibBytes + g * 8,
                                                      x_saddr + (kt + q) * UnitMath<NCOLS, FAST>::kXStride, acc);
      }
    } else {
#pragma unroll 1
      for (uint32_t s = 0; s < n; ++s)
        UnitMath<NCOLS, FAST>::run_saddr(su + s * kUnitBytes, x_saddr, kt + s, lane, acc);
    }
    ring.release();
    kt += n;
    left -= n;
    if (kt == KT) {
      flush_tile<NCOLS, SPLIT>(acc, seg_kt0 == 0, r, first_row, fx, ntok, epi);
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
  if (kt != seg_kt0) flush_tile<NCOLS, SPLIT>(acc, false, r, first_row, fx, ntok, epi);
  return true;
}

}  // namespace alv
