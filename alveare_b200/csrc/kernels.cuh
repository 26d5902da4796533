// Device kernels of the Q4 decode hot path: gemv (decode / decode-batch), the
// fused FFN, the FFN-stack layer glue and the one-launch FFN stack, with their
// epilogues and grid barriers.  Host launchers live in gemv.cu, ffn.cu and
// stack.cu; the load-time kernels in loadtime.cuh.
#pragma once

#include <climits>

#include "common.cuh"
#include "stream.cuh"

namespace alv {

constexpr int kWarpsPerCta = kConsumerWarps;  // warps per CTA, each streaming its own unit range

// ===========================================================================
// Activation sources / epilogues
// ===========================================================================
struct XSrc {  // (ntok, K) activations, fp32 or bf16, row stride ld
  const void* x;
  int bf16;
  int ntok;
  uint32_t K;
  uint32_t ld;
  // Values at (tok, k) and (tok, k+1), k even; zero outside [0, ntok) x [0, K).
  // K is a multiple of 32, so k < K implies k + 1 < K.
  __device__ __forceinline__ void pair(uint32_t tok, uint32_t k, float& a, float& b) const {
    if (static_cast<int>(tok) >= ntok || k >= K) {
      a = b = 0.f;
      return;
    }
    const uint64_t i = static_cast<uint64_t>(tok) * ld + k;
    if (bf16) {
      const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(static_cast<const uint16_t*>(x) + i));
      a = bf16_bits_to_f32(w & 0xFFFF);
      b = bf16_bits_to_f32(w >> 16);
    } else {
      const float2 f = __ldg(reinterpret_cast<const float2*>(static_cast<const float*>(x) + i));
      a = f.x;
      b = f.y;
    }
  }
};

struct SmemSrc {  // staged activations in shared memory: float[ntok][K]
  const float* v;
  int ntok;
  uint32_t K;
  __device__ __forceinline__ void pair(uint32_t tok, uint32_t k, float& a, float& b) const {
    if (static_cast<int>(tok) >= ntok || k >= K) {
      a = b = 0.f;
      return;
    }
    a = v[static_cast<uint64_t>(tok) * K + k];
    b = v[static_cast<uint64_t>(tok) * K + k + 1];
  }
};

struct ActSrc {  // FFN intermediate written by other CTAs: read through L2
  const uint16_t* act;
  int ntok;
  uint32_t I;
  uint32_t ld;
  __device__ __forceinline__ void pair(uint32_t tok, uint32_t k, float& a, float& b) const {
    if (static_cast<int>(tok) >= ntok || k >= I) {
      a = b = 0.f;
      return;
    }
    const uint32_t w = __ldcg(reinterpret_cast<const unsigned int*>(act + static_cast<uint64_t>(tok) * ld + k));
    a = bf16_bits_to_f32(w & 0xFFFF);
    b = bf16_bits_to_f32(w >> 16);
  }
};

struct RowsEpi {  // y[tok, row] = v * scale_mul (fp32 and/or bf16)
  float* y32;
  uint16_t* y16;
  uint32_t N;
  uint32_t ld;
  float sm;
  __device__ __forceinline__ void put(int tok, uint32_t row, float v) const {
    if (row >= N) return;
    const uint64_t i = static_cast<uint64_t>(tok) * ld + row;
    v *= sm;
    if (y32) y32[i] = v;
    if (y16) y16[i] = bf16_bits_rn(v);
  }
  __device__ __forceinline__ void apply(uint32_t r, int g, int tok, float vg, float vg8) const {
    put(tok, r * 16 + g, vg);
    put(tok, r * 16 + g + 8, vg8);
  }
};

// GeGLU exactly as runtime/py/model.py:690-693 evaluates it under numpy
// promotion: float32 cubic term, float64 from the sqrt(2/pi) factor on,
// float64 -> float32 before the bf16 cast.
__device__ __forceinline__ float geglu_ref(float g, float u) {
  const float g3 = __fmul_rn(__fmul_rn(g, g), g);                 // exact for bf16 g
  const float inner = __fadd_rn(g, __fmul_rn(0x1.6e4e26p-5f, g3));  // g + 0.044715f * g^3
  const double t = tanh(0x1.9884533d43651p-1 * static_cast<double>(inner));  // np.sqrt(2/np.pi)
  const double gelu = static_cast<double>(__fmul_rn(0.5f, g)) * (1.0 + t);
  return static_cast<float>(gelu * static_cast<double>(u));
}

// A float whose bf16 rounding equals that of geglu_ref(g, u), mostly in
// float32: 0.5 g (1 + tanh z) = g / (1 + exp(-2z)), z = sqrt(2/pi) * inner,
// has no cancellation and stays within ~1e-6 relative of the float64 value
// for |z| <= 9 (expf: 2 ulp; the rest: four float32 roundings).  That result
// is kept when it lies more than 256 float32 ulps (1.5e-5 relative) from a
// bf16 rounding midpoint, so the float64 value and its float32 rounding fall
// on the same side of every midpoint; otherwise (and for |z| > 9, where
// float64 1 + tanh(z) itself cancels, or a zero / non-normal result) it
// returns geglu_ref.
__device__ __forceinline__ float geglu_act(float g, float u) {
  const float g3 = __fmul_rn(__fmul_rn(g, g), g);
  const float inner = __fadd_rn(g, __fmul_rn(0x1.6e4e26p-5f, g3));
  const float z = 0x1.988454p-1f * inner;
  if (fabsf(z) <= 9.0f) {
    const float y = __fdiv_rn(g, 1.0f + expf(-2.0f * z)) * u;
    const uint32_t b = __float_as_uint(y), e = (b >> 23) & 0xFFu;
    const int lo = static_cast<int>(b & 0xFFFFu) - 0x8000;
    if (e != 0u && e != 0xFFu && (lo > 256 || lo < -256)) return y;
  }
  return geglu_ref(g, u);
}

// SwiGLU as runtime/py/model.py:857-859 (float32 throughout).
__device__ __forceinline__ float swiglu_ref(float g, float u) {
  const float e = static_cast<float>(exp(-static_cast<double>(g)));  // correctly rounded expf
  const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
  return __fmul_rn(__fmul_rn(g, s), u);
}


// Byte offset of value (column n, k) in the B-fragment layout (stage_frags).
__device__ __forceinline__ uint32_t frag_offset(uint32_t ncols, uint32_t n, uint32_t k) {
  const uint32_t kt = k >> 6, r = k & 63, j = r >> 4, c = r & 15;
  const uint32_t t4 = (c & 7) >> 1, reg = c >> 3, half = c & 1;
  return ((kt * ncols + n) * 4 + t4) * 32 + j * 8 + reg * 4 + half * 2;
}

struct GateUpEpi {  // tile rows 0-7 gate, 8-15 up of the same 8 intermediate indices
  uint8_t* act;     // fragment-order act for the down projection (ncb columns)
  uint32_t I;
  uint32_t ncb;
  float sm;
  int fn;
  __device__ __forceinline__ void apply(uint32_t r, int g, int tok, float vg, float vg8) const {
    const uint32_t i = r * 8 + g;
    if (i >= I) return;
    const float gate = bf16_round(vg * sm), up = bf16_round(vg8 * sm);
    const float a = fn == 0 ? geglu_act(gate, up) : swiglu_ref(gate, up);
    *reinterpret_cast<uint16_t*>(act + frag_offset(ncb, static_cast<uint32_t>(tok), i)) = bf16_bits_rn(a);
  }
};

// ===========================================================================
// Grid-wide barrier (sense by generation counter), bounded wait.
// ===========================================================================
struct GridBar {
  unsigned long long count;  // monotonically increasing arrivals (never wraps)
};

// floor(n / d) for a counter n < 2^50 and d >= 1: a double-precision
// estimate (relative error below 2^-51, so within one of the quotient)
// corrected with integer products -- a few instructions where a 64-bit
// integer division is a long software sequence on the barrier's critical path.
__device__ __forceinline__ unsigned long long div_counter(unsigned long long n, uint32_t d) {
  unsigned long long q = static_cast<unsigned long long>(__dmul_rn(static_cast<double>(n), __drcp_rn(static_cast<double>(d))));
  if (q * d > n) --q;
  if ((q + 1) * d <= n) ++q;
  return q;
}

// Grid barrier: the k-th use of the barrier by a launch completes when the
// monotonic counter reaches base + k * nblocks.  The arrival is a
// fire-and-forget release reduction and the target is known in advance, so
// a CTA pays one poll round trip, not an atomic's return trip plus the poll.
// Correct across launches because every launch uses it a whole number of
// times with the same grid, so the counter always resumes at a multiple of
// nblocks.  `base` is the counter's value at launch, read once before
// the first arrival (grid_base); `epoch` counts this launch's barriers.
__device__ __forceinline__ unsigned long long grid_base(GridBar* gb, uint32_t nblocks) {
  // At most nblocks - 1 arrivals of this launch can precede the read (the
  // first barrier needs every CTA), and launches start at multiples of nblocks.
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(&gb->count) : "memory");
  return div_counter(v, nblocks) * nblocks;
}
inline __device__ bool grid_barrier_epoch(GridBar* gb, uint32_t nblocks, unsigned long long base, uint32_t epoch,
                                   uint32_t* status) {
  consumers_sync();
  int ok = 1;
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(&gb->count) : "memory");
    const unsigned long long target = base + static_cast<unsigned long long>(epoch) * nblocks;
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(&gb->count) : "memory");
    if (v < target) {
      const unsigned long long t0 = globaltimer_ns();
      while (true) {
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(&gb->count) : "memory");
        if (v >= target) break;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(status, kStatusGridTimeout);
          ok = 0;
          break;
        }
      }
    }
  }
  return consumers_and(ok != 0);
}

// Exchange step of a tensor-parallel FFN stack (ranks on distinct GPUs, one
// launch each), after the rank's own grid barrier: CTA 0 -- which the grid
// barrier ordered after every local CTA's pushes -- issues one system-scope
// release (fence.acq_rel.sys) and adds 1 to every rank's counter, its own
// included; every CTA then polls its own counter (system-scope acquire) for
// base + epoch * world.  One system fence per rank and exchange, not one per
// CTA.  `base` is the own counter at launch rounded down to a multiple of
// world: before this launch's CTA 0 signals (which needs every local CTA past
// the first grid barrier, so after each CTA read its base) at most the
// other ranks' world - 1 first-exchange signals can have landed.
__device__ __forceinline__ unsigned long long peer_base(const uint8_t* own, uint32_t world) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(own) : "memory");
  return div_counter(v, world) * world;
}
inline __device__ bool peer_exchange(uint8_t* const* xr, uint32_t world, uint32_t rank, unsigned long long base,
                              uint32_t epoch, uint32_t* status) {
  int ok = 1;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (uint32_t q = 0; q < world; ++q)
        asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(xr[q]) : "memory");
    }
    const unsigned long long target = base + static_cast<unsigned long long>(epoch) * world;
    const uint8_t* own = xr[rank];
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(own) : "memory");
    if (v < target) {
      const unsigned long long t0 = globaltimer_ns();
      while (true) {
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(own) : "memory");
        if (v >= target) break;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(status, kStatusPeerTimeout);
          ok = 0;
          break;
        }
      }
    }
  }
  return consumers_and(ok != 0);
}


// Sum over the consumer threads (all of them get the result) through `red`
// (>= 16 floats).  One named barrier: consecutive calls must alternate
// between two such buffers (a call's buffer is rewritten two calls later,
// after the intervening call's barrier, when every thread has read it).
// Fixed order, so every CTA computes the identical value.
inline __device__ float consumers_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  consumers_sync();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) s += red[i];
  return s;
}

// Single-CTA block sum for the finalize kernel (blockDim.x threads).
inline __device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  __syncthreads();
  return s;
}

// ===========================================================================
// gemv: persistent, one CTA per SM, stream-K over units.
// ===========================================================================
struct GemvParams {
  Q4Mat m;
  Partition pt;  // the launch's split of m's units (host-built for the grid)
  XSrc x;
  RowsEpi epi;
  Fixup fx;
  uint32_t* status;
  uint32_t nst;    // ring stages per warp
  uint32_t first;  // stages requested before x is staged (the rest after)
  unsigned long long* trace;  // optional: [gridDim.x][16] phase timestamps (ns)
};

constexpr int kUnitsPerStage = ALV_UNITS_PER_STAGE;
static_assert(kUnitsPerStage % kStageUnroll == 0, "the unroll length must divide the stage");
constexpr int kThreadsPerCta = kConsumerWarps * 32;
using Shape = RingShape<kUnitsPerStage>;

__host__ __device__ constexpr size_t ring_smem_bytes(uint32_t nst) { return Shape::smem_bytes(nst); }
static_assert(ring_smem_bytes(1) % 128 == 0 && ring_smem_bytes(2) % 128 == 0 && ring_smem_bytes(3) % 128 == 0,
              "what follows the rings must stay 16-byte aligned");
static_assert(part_bytes(1) % 128 == 0, "what follows the warp partials must stay 16-byte aligned");
// Shared layout of every streaming kernel: [rings][warp partials][kernel's own].
__host__ __device__ constexpr size_t base_smem_bytes(uint32_t nst, int ntok) {
  return ring_smem_bytes(nst) + part_bytes(ntok);
}

// Phase timestamps of one gemv CTA (thread 0): 0 start, 1 weights requested,
// 2 predecessor finished (griddepcontrol.wait returned), 3 x staged, 4 warp
// 0's units consumed, 5 split-K reduction done.
__device__ __forceinline__ void gemv_mark(unsigned long long* trace, int i) {
  if (trace && threadIdx.x == 0) trace[blockIdx.x * 16 + i] = globaltimer_ns();
}

template <int NCOLS, bool SPLIT, bool FAST>
__global__ void __launch_bounds__(kThreadsPerCta, 1) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ WorkList wl[kConsumerWarps];
  __shared__ uint32_t wr[kConsumerWarps][4];  // per warp: unit range [u0, u1)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Partition& pt = p.pt;
  gemv_mark(p.trace, 0);
  // Each warp starts its own weight stream as soon as it can: its ring's
  // barriers, range and work list are its own (the CTA syncs before it
  // stages x, which every warp reads).
  Shape::init_warp_barriers(smem, p.nst, warp);
  uint32_t u0, u1;
  pt.warp_range(blockIdx.x, warp, u0, u1);
  if (lane == 0) {
    wl[warp] = WorkList{p.m.units + static_cast<size_t>(u0) * kUnitBytes, p.m.units, u1 - u0, 0,
                        u0 - pt.kt.div(u0) * p.m.KT, 0, p.m.KT, 1};
    wr[warp][0] = u0;
    wr[warp][1] = u1;
  }
  __syncwarp();
  ConsumerRing<kUnitsPerStage, WorkList> ring;
  ring.setup(smem, p.nst, warp, u1 - u0, &wl[warp], p.first);  // weights start streaming
  pdl_trigger();
  Fixup fx = p.fx;
  fx.part = reinterpret_cast<float*>(smem + ring_smem_bytes(p.nst));
  uint8_t* xs = smem + base_smem_bytes(p.nst, p.x.ntok);
  gemv_mark(p.trace, 1);
  pdl_wait();  // x, y and the split-K workspace belong to the stream's order from here
  gemv_mark(p.trace, 2);
  stage_frags<NCOLS, SPLIT>(xs, p.m.KT, p.x);
  ring.fill_rest();
  consumers_sync();
  gemv_mark(p.trace, 3);
  if (!consume_range<NCOLS, SPLIT, FAST>(ring, p.m, u0, u1, xs, fx, p.x.ntok, p.epi, p.status))
    ring.drain();
  gemv_mark(p.trace, 4);
  cta_fixup(pt, &wr[0][0], fx, p.x.ntok, p.epi);
  gemv_mark(p.trace, 5);
}

// ===========================================================================
// Fused FFN: phase A (gate/up interleaved, activation epilogue -> act),
// grid barrier, phase B (down projection).  The per-warp ring prefetches
// phase-B weights while phase A finishes and the barrier is pending.
// ===========================================================================
struct FfnParams {
  Q4Mat gu;
  Q4Mat dn;
  Partition ptA, ptB;   // gate/up (row-aligned) and down splits, host-built for the grid
  uint32_t H;
  uint32_t I;
  int fn;
  int ntok;
  XSrc x;               // plain input (glue == 0)
  int glue;             // 1: x is the bf16 residual stream, norms/residual fused
  const uint16_t* x_in;
  const float* down_in;
  uint16_t* x_out;
  float eps;
  uint32_t first;       // ring stages requested before the inputs are staged (the rest after)
  RowsEpi out;          // down projection output
  uint8_t* act;         // scratch: act in B-fragment order, frag_bytes(dn.KT, NT) bytes
  Fixup fxA, fxB;
  GridBar* bar;
  uint32_t* status;
  uint32_t nst;  // ring stages per warp
  unsigned long long* trace;  // optional: [gridDim.x][16] phase timestamps (ns)
  int glue_tma;          // glue inputs 16-byte aligned: fetch them with bulk copies
};

// Phase timestamps of one CTA (thread 0): 0 start, 1 prologue staged, 2 phase A
// done (all warps), 3 grid barrier passed, 4 act staged, 5 phase B done.
__device__ __forceinline__ void trace_mark(unsigned long long* trace, int i) {
  if (trace && threadIdx.x == 0) trace[blockIdx.x * 16 + i] = globaltimer_ns();
}

// ---------------------------------------------------------------------------
// Layer glue: the residual update and pre-norm around each FFN call of the
// decode loop (runtime/py/model.py:782-806, runtime/cpp/src/model.cpp:404),
// per token
//   x  = bf16(x_in + bf16(rmsnorm(bf16(d))))   when a down vector d is given
//   xn = bf16(rmsnorm(x))                       when PRE
// with unit-weight rmsnorm v / sqrt(mean(v*v) + eps), the mean dividing the
// float32 sum by H like np.mean.  Consumer thread t owns the groups of eight
// consecutive values g = t + k * T (T consumer threads, k < GK) and holds
// them in registers, so every load of a token is in flight at once; sums are
// reduced in a fixed order, so every caller and every CTA computes identical
// values.  H <= 8 * T * GK.
// ---------------------------------------------------------------------------
constexpr int kGlueRegs = 16;
constexpr int kMaxRanks = 8;  // tensor-parallel ranks of one FFN stack

// Loaders: value of token tok at index h, flat index i = tok * H + h.
// 8 consecutive values at flat index i (a multiple of 8): one 16-byte access
// when the address allows it (shared or global memory alike).
__device__ __forceinline__ bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }
__device__ __forceinline__ void unpack8(const uint4& w, float (&v)[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    v[2 * t] = bf16_bits_to_f32(ws[t] & 0xFFFFu);
    v[2 * t + 1] = bf16_bits_to_f32(ws[t] >> 16);
  }
}

struct Bf16In {   // bf16 values in memory written before the launch (or shared)
  const uint16_t* p;
  __device__ __forceinline__ float operator()(uint32_t, uint32_t, size_t i) const { return bf16_bits_to_f32(p[i]); }
  __device__ __forceinline__ void load8(size_t i, float (&v)[8]) const {
    const uint16_t* q = p + i;
    if (al16(q)) {
      unpack8(*reinterpret_cast<const uint4*>(q), v);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = bf16_bits_to_f32(q[t]);
    }
  }
};
struct F32In {    // fp32 values in memory written before the launch (or shared)
  const float* p;
  __device__ __forceinline__ float operator()(uint32_t, uint32_t, size_t i) const { return p[i]; }
  __device__ __forceinline__ void load(uint32_t, uint32_t, size_t i, float& a, float& b, uint32_t& how) const {
    a = p[i];
    b = 0.f;
    how = 0;
  }
  __device__ __forceinline__ float combine(float a, float, uint32_t) const { return a; }
  __device__ __forceinline__ void load8(uint32_t, uint32_t, size_t i, float (&v)[8]) const {
    const float* q = p + i;
    if (al16(q)) {
      const float4 a = *reinterpret_cast<const float4*>(q), b = *reinterpret_cast<const float4*>(q + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = q[t];
    }
  }
};
// The down projection of the previous stack layer as the glue reads it
// (token tok, index h, flat i = tok*H + h): a row tile held by one CTA is
// final in `down`; a row tile split between CTAs was left as CTA partials
// (cta_fixup<true>) that are summed here in CTA order and scaled, exactly as
// the last CTA to arrive would have done.  split[r] = element offsets in ws
// of the first two CTAs' partials of row tile r (x = ~0: not split), or
// y = ~0 with x = the first CTA when the tile spans three or more CTAs.
struct DownIn {
  const float* down;
  const float* ws;          // CTA partials: [CTA][2 slots][ntok][16]
  const uint2* split;       // per row tile, see above
  const uint32_t* cfirst;   // per CTA: its first row tile
  const uint32_t* span;     // per row tile: first CTA | last CTA << 16
  uint32_t slot_floats;
  float sm;
  // Two passes, so a thread's loads are all in flight before any is used:
  // load() issues them, combine() adds and scales.
  __device__ __forceinline__ void load(uint32_t tok, uint32_t h, size_t i, float& a, float& b, uint32_t& how) const {
    const uint32_t r = h >> 4;
    const uint2 o = split[r];
    const uint32_t e = tok * 16 + (h & 15);
    if (o.x == ~0u) {
      a = __ldcg(down + i);
      b = 0.f;
      how = 0;
    } else if (o.y != ~0u) {
      a = __ldcg(ws + o.x + e);
      b = __ldcg(ws + o.y + e);
      how = 1;
    } else {  // a row tile over three or more CTAs (small problems)
      const uint32_t sp = span[r];
      float v = 0.f;
      for (uint32_t c = sp & 0xFFFFu; c <= (sp >> 16); ++c)
        v += __ldcg(ws + (static_cast<size_t>(c) * 2 + (r == cfirst[c] ? 0 : 1)) * slot_floats + e);
      a = v;
      b = 0.f;
      how = 2;
    }
  }
  __device__ __forceinline__ float combine(float a, float b, uint32_t how) const {
    return how == 0 ? a : (how == 1 ? (a + b) * sm : a * sm);
  }
  // Elements h..h+7 (h a multiple of 8: one row tile, one half of it),
  // combined as above.
  __device__ __forceinline__ void load8(uint32_t tok, uint32_t h, size_t i, float (&v)[8]) const {
    const uint32_t r = h >> 4;
    const uint2 o = split[r];
    const uint32_t e = tok * 16 + (h & 15);
    auto ld8 = [](const float* q, float (&w)[8]) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(q)), b = __ldcg(reinterpret_cast<const float4*>(q + 4));
      w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    };
    if (o.x == ~0u) {
      ld8(down + i, v);
    } else if (o.y != ~0u) {
      float a[8], b[8];
      ld8(ws + o.x + e, a);
      ld8(ws + o.y + e, b);
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = (a[t] + b[t]) * sm;
    } else {  // a row tile over three or more CTAs (small problems)
      const uint32_t sp = span[r];
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = 0.f;
      for (uint32_t c = sp & 0xFFFFu; c <= (sp >> 16); ++c) {
        float a[8];
        ld8(ws + (static_cast<size_t>(c) * 2 + (r == cfirst[c] ? 0 : 1)) * slot_floats + e, a);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] += a[t];
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] *= sm;
    }
  }
};
struct NoIn {
  __device__ __forceinline__ void load(uint32_t, uint32_t, size_t, float& a, float& b, uint32_t& how) const {
    a = b = 0.f;
    how = 0;
  }
  __device__ __forceinline__ float combine(float a, float, uint32_t) const { return a; }
  __device__ __forceinline__ void load8(uint32_t, uint32_t, size_t, float (&v)[8]) const {
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = 0.f;
  }
};
struct Bf16Out {  // null: no output
  uint16_t* p;
  __device__ __forceinline__ void operator()(size_t i, float v) const {
    if (p) p[i] = bf16_bits_rn(v);
  }
  __device__ __forceinline__ void store8(size_t i, const float (&v)[8]) const {
    if (!p) return;
    uint16_t* q = p + i;
    if (al16(q)) {
      uint4 w;
      w.x = pack_bf2(bf16_bits_rn(v[0]), bf16_bits_rn(v[1]));
      w.y = pack_bf2(bf16_bits_rn(v[2]), bf16_bits_rn(v[3]));
      w.z = pack_bf2(bf16_bits_rn(v[4]), bf16_bits_rn(v[5]));
      w.w = pack_bf2(bf16_bits_rn(v[6]), bf16_bits_rn(v[7]));
      *reinterpret_cast<uint4*>(q) = w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) q[t] = bf16_bits_rn(v[t]);
    }
  }
};

// Where xn (PRE) goes: straight into the B-fragment layout of the next
// phase (frag: nc columns, kpad = 64 * k tiles; every position outside
// [0, ntok) x [0, H) is zeroed), or as fp32 (holding bf16 values) into
// tmp[ntok][H].
struct XnOut {
  float* tmp;
  uint8_t* frag;
  uint32_t nc, kpad;
};

// Copy `bytes` (a multiple of 16) from global memory (through L2) into
// shared memory with the consumer threads, 16 bytes per thread and step.
// (Holding several loads in registers before the stores makes the stack
// kernel spill.)
__device__ __forceinline__ void stage_from_l2(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
  constexpr uint32_t NTHR = kConsumerWarps * 32, STEP = NTHR * 16;
  for (uint32_t o = threadIdx.x * 16; o < bytes; o += STEP)
    *reinterpret_cast<uint4*>(dst + o) = __ldcg(reinterpret_cast<const uint4*>(src + o));
}

template <int GK, bool PRE, bool HAS_D, class XL, class DL, class XO>
__device__ void glue_tokens(int ntok, uint32_t H, float eps, const XL& xl, const DL& dl, const XO& xo,
                            const XnOut& xn_out, float* red, unsigned long long* tr) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  static_assert(kConsumerWarps <= 16, "consumers_sum buffers hold 16 partials");
  const float hf = static_cast<float>(H);
  const uint32_t G = H / 8;  // groups of 8 consecutive values; thread t owns groups t + k * NTHR
  // consumers_sum alternates between red[0..15] and red[16..31]; the caller's
  // barrier before the glue orders this glue's first use after the last one
  // of the previous glue.
  int rs = 0;
  for (int tok = 0; tok < ntok; ++tok) {
    const size_t base = static_cast<size_t>(tok) * H;
    // All loads of the token in flight before any is used.
    float xv[GK][8], dv[GK][8];
#pragma unroll
    for (int k = 0; k < GK; ++k) {
      const uint32_t g = threadIdx.x + k * NTHR;
#pragma unroll
      for (int t = 0; t < 8; ++t) xv[k][t] = dv[k][t] = 0.f;
      if (g < G) {
        xl.load8(base + 8 * g, xv[k]);
        if (HAS_D) dl.load8(static_cast<uint32_t>(tok), 8 * g, base + 8 * g, dv[k]);
      }
    }
    if (tok == 0) trace_mark(tr, 9);
    if (HAS_D) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < GK; ++k)
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          dv[k][t] = bf16_round(dv[k][t]);
          ss = fmaf(dv[k][t], dv[k][t], ss);
        }
      ss = consumers_sum(ss, red + 16 * (rs++ & 1));
      if (tok == 0) trace_mark(tr, 10);
      const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, hf), eps)));
#pragma unroll
      for (int k = 0; k < GK; ++k)
#pragma unroll
        for (int t = 0; t < 8; ++t) xv[k][t] = bf16_round(xv[k][t] + bf16_round(dv[k][t] * inv));
    }
#pragma unroll
    for (int k = 0; k < GK; ++k) {
      const uint32_t g = threadIdx.x + k * NTHR;
      if (g < G) xo.store8(base + 8 * g, xv[k]);
    }
    if (PRE) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < GK; ++k)
#pragma unroll
        for (int t = 0; t < 8; ++t) ss = fmaf(xv[k][t], xv[k][t], ss);
      ss = consumers_sum(ss, red + 16 * (rs++ & 1));
      if (tok == 0) trace_mark(tr, 11);
      const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, hf), eps)));
#pragma unroll
      for (int k = 0; k < GK; ++k) {
        const uint32_t g = threadIdx.x + k * NTHR;
        if (g >= G) continue;
        const uint32_t h = 8 * g;
        float xn[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) xn[t] = bf16_round(xv[k][t] * inv);
        if (xn_out.frag) {
          // values h + 2i, h + 2i + 1 share one 32-bit word; the four words
          // of a group sit 32 bytes apart (fragment lane quads t4 = i)
          uint8_t* f = xn_out.frag + frag_offset(xn_out.nc, static_cast<uint32_t>(tok), h);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint32_t*>(f + 32 * i) = pack_bf2(bf16_bits_rn(xn[2 * i]), bf16_bits_rn(xn[2 * i + 1]));
        } else {
#pragma unroll
          for (int t = 0; t < 8; ++t) xn_out.tmp[base + h + t] = xn[t];
        }
      }
    }
  }
  if (PRE && xn_out.frag) {  // zero padding: k in [H, kpad) and columns [ntok, nc)
    const uint32_t pad_k = xn_out.kpad - H;
    for (uint32_t e = threadIdx.x; e < pad_k * xn_out.nc; e += NTHR) {
      const uint32_t n = e % xn_out.nc, k = H + e / xn_out.nc;
      *reinterpret_cast<uint16_t*>(xn_out.frag + frag_offset(xn_out.nc, n, k)) = 0;
    }
    const uint32_t extra = xn_out.nc - static_cast<uint32_t>(ntok);
    for (uint32_t e = threadIdx.x; e < H * extra; e += NTHR) {
      const uint32_t n = ntok + e % extra, k = e / extra;
      *reinterpret_cast<uint16_t*>(xn_out.frag + frag_offset(xn_out.nc, n, k)) = 0;
    }
  }
  trace_mark(tr, 12);
  consumers_sync();
}

// Groups of 8 per thread chosen from H at run time (one covers H <= 3840).
// tr: optional phase stamps [9] down loaded, [10] its norm reduced, [11] x's
// norm reduced, [12] xn written (first token).
template <bool PRE, bool HAS_D, class XL, class DL, class XO>
__device__ __forceinline__ void glue(int ntok, uint32_t H, float eps, const XL& xl, const DL& dl, const XO& xo,
                                     const XnOut& xn_out, float* red, unsigned long long* tr = nullptr) {
  if (H <= 8u * kConsumerWarps * 32)
    glue_tokens<1, PRE, HAS_D>(ntok, H, eps, xl, dl, xo, xn_out, red, tr);
  else
    glue_tokens<kGlueRegs / 8, PRE, HAS_D>(ntok, H, eps, xl, dl, xo, xn_out, red, tr);
}

template <int NT, bool SPLIT, bool FAST>
__global__ void __launch_bounds__(kThreadsPerCta, 1) ffn_kernel(const FfnParams p) {
  constexpr int NCA = SPLIT ? 2 * NT : NT;
  constexpr int NCB = NT;
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Partition& ptA = p.ptA;
  const Partition& ptB = p.ptB;
  __shared__ WorkList wl[kConsumerWarps];
  __shared__ uint32_t wr[kConsumerWarps][4];  // per warp: gate/up [u0, u1), down [u0, u1)
  Shape::init_warp_barriers(smem, p.nst, warp);
  uint32_t a0, a1, b0, b1;
  ptA.warp_range(blockIdx.x, warp, a0, a1);
  ptB.warp_range(blockIdx.x, warp, b0, b1);
  if (lane == 0) {
    wl[warp] = WorkList{p.gu.units + static_cast<size_t>(a0) * kUnitBytes,
                        p.dn.units + static_cast<size_t>(b0) * kUnitBytes, a1 - a0, b1 - b0,
                        a0 - ptA.kt.div(a0) * p.gu.KT, b0 - ptB.kt.div(b0) * p.dn.KT, p.gu.KT, p.dn.KT};
    wr[warp][0] = a0;
    wr[warp][1] = a1;
    wr[warp][2] = b0;
    wr[warp][3] = b1;
  }
  // Shared layout after the rings and warp partials:
  // [xs frags][red][tmp ntok*H f32][x_in raw][down_in raw][xbar]
  Fixup fxA = p.fxA, fxB = p.fxB;
  fxA.part = fxB.part = reinterpret_cast<float*>(smem + ring_smem_bytes(p.nst));
  uint8_t* xs = smem + base_smem_bytes(p.nst, p.ntok);
  const size_t xs_bytes_a = frag_bytes(p.gu.KT, NCA);
  const size_t xs_bytes_b = frag_bytes(p.dn.KT, NCB);
  const size_t xs_bytes = xs_bytes_a > xs_bytes_b ? xs_bytes_a : xs_bytes_b;
  float* red = reinterpret_cast<float*>(xs + xs_bytes);
  float* tmp = red + 32;
  const size_t glue_vals = p.glue ? static_cast<size_t>(p.ntok) * p.H : 0;
  uint16_t* xraw = reinterpret_cast<uint16_t*>(tmp + glue_vals);
  float* draw = reinterpret_cast<float*>(xraw + (p.glue_tma ? glue_vals : 0));
  uint64_t* xbar = reinterpret_cast<uint64_t*>(draw + (p.glue_tma && p.down_in ? glue_vals : 0));
  const bool tma_in = p.glue && p.glue_tma;
  if (tma_in && threadIdx.x == 0) {
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Each warp starts its weight stream (its ring, range and work list are its
  // own) while the previous kernel in the stream may still be finishing; the
  // layer inputs, the split-K workspace and the barrier counter are touched
  // only after griddepcontrol.wait.  Large FFNs request one stage per warp
  // first, so the inputs do not queue behind the whole weight stream.
  ConsumerRing<kUnitsPerStage, WorkList> ring;
  ring.setup(smem, p.nst, warp, (a1 - a0) + (b1 - b0), &wl[warp], p.first);
  pdl_trigger();
  pdl_wait();
  const unsigned long long bar_base = threadIdx.x == 0 ? grid_base(p.bar, gridDim.x) : 0ull;
  __syncthreads();  // xbar initialized
  if (tma_in && threadIdx.x == 0) {
    const uint64_t pol = l2_policy_evict_first();
    const uint32_t xb = static_cast<uint32_t>(glue_vals * 2), db = p.down_in ? static_cast<uint32_t>(glue_vals * 4) : 0;
    mbar_arrive_expect_tx(xbar, xb + db);
    bulk_g2s(xraw, p.x_in, xb, xbar, pol);
    if (db) bulk_g2s(draw, p.down_in, db, xbar, pol);
  }
  trace_mark(p.trace, 0);

  // The act padding (k in [I, 64*dn.KT)) must read as zero in phase B.
  if (blockIdx.x == 0) {
    const uint32_t kpad = p.dn.KT * 64;
    for (uint32_t e = threadIdx.x; e < (kpad - p.I) * NCB; e += NTHR) {
      const uint32_t n = e % NCB, k = p.I + e / NCB;
      *reinterpret_cast<uint16_t*>(p.act + frag_offset(NCB, n, k)) = 0;
    }
  }
  bool in_ok = true;
  if (p.glue) {
    if (tma_in) in_ok = consumers_and(mbar_wait_bounded(xbar, 0));
    if (!in_ok && threadIdx.x == 0) atomicOr(p.status, kStatusMbarTimeout);
    trace_mark(p.trace, 6);
    const Bf16Out xo{blockIdx.x == 0 ? p.x_out : nullptr};
    const Bf16In xl{tma_in ? xraw : p.x_in};
    const XnOut xn{nullptr, xs, static_cast<uint32_t>(NCA), p.gu.KT * 64};
    if (p.down_in)
      glue<true, true>(p.ntok, p.H, p.eps, xl, F32In{tma_in ? draw : p.down_in}, xo, xn, red);
    else
      glue<true, false>(p.ntok, p.H, p.eps, xl, NoIn{}, xo, xn, red);
    trace_mark(p.trace, 7);
  } else {
    stage_frags<NCA, SPLIT>(xs, p.gu.KT, p.x);
  }
  ring.fill_rest();
  consumers_sync();
  trace_mark(p.trace, 1);

  GateUpEpi ge{p.act, p.I, NCB, p.gu.scale_mul, p.fn};
  const bool ok = consume_range<NCA, SPLIT, FAST>(ring, p.gu, a0, a1, xs, fxA, p.ntok, ge, p.status);
  cta_fixup(ptA, &wr[0][0], fxA, p.ntok, ge);
  if (p.trace) {
    consumers_sync();
    trace_mark(p.trace, 2);
  }
  const bool bar_ok = grid_barrier_epoch(p.bar, gridDim.x, bar_base, 1, p.status);
  trace_mark(p.trace, 3);
  if (!bar_ok || !consumers_and(ok)) {
    ring.drain();
    return;
  }
  // act is already in fragment order: stage it with 16-byte copies through L2.
  stage_from_l2(xs, p.act, static_cast<uint32_t>(xs_bytes_b));
  consumers_sync();
  trace_mark(p.trace, 4);
  if (!consume_range<NCB, false, FAST>(ring, p.dn, b0, b1, xs, fxB, p.ntok, p.out, p.status))
    ring.drain();
  cta_fixup(ptB, &wr[0][2], fxB, p.ntok, p.out);
  if (p.trace) {
    consumers_sync();
    trace_mark(p.trace, 5);
  }
}

// ===========================================================================
// Whole FFN stack in one persistent launch: for l = 0..L-1
//   glue (x += rmsnorm(down_{l-1}); xn = rmsnorm(x)) -> phase A (gate/up +
//   activation -> act) -> grid barrier -> phase B (down -> down_l) -> grid
//   barrier,
// then the last residual x += rmsnorm(down_{L-1}) -> out.  Each warp's ring
// runs through every layer's weights back to back, so nst groups stay in
// flight while the warps run the glue and wait at the barriers.  The residual
// stream stays in shared memory (every CTA holds the identical copy); only
// down (H fp32 per token) and act cross CTAs, through L2.  Each step's
// arithmetic and reduction order equal the per-layer ffn_kernel chain, so
// the two paths agree bit for bit.
// ===========================================================================
struct StackParams {
  const LayerW* layers;
  uint32_t L;
  Q4Mat gu, dn;           // per-layer shapes (RT, KT); units / scale_mul come from layers
  Partition ptA, ptB;     // gate/up (row-aligned) and down splits, host-built for the grid
  uint32_t H, I;
  int fn;
  int ntok;
  float eps;
  const uint16_t* x_in;   // [ntok][H] bf16 stack input
  uint16_t* out;          // [ntok][H] bf16 stack output
  float* down;            // [ntok][H] fp32: a layer's down projection
  uint8_t* act;           // [dn.KT*64][ntok] bf16 intermediate, B-fragment order
  Fixup fxA, fxB;
  GridBar* bar;
  uint32_t* status;
  uint32_t nst;
  unsigned long long* trace;  // optional: phase stamps of layer 1
  float* probe;               // optional: [ntok][H] fp32 down projection of the last layer
  // Tensor parallelism (ffn_stack_kernel<..., TP = true>): rank `rank` of
  // `world` holds an I-slice of every layer.  xr[q] is rank q's exchange
  // region as mapped on this GPU (xr[rank] is this GPU's own):
  //   [peer-barrier counter u64 @0][slots @kXHeader: parity x world x xslot floats]
  // Slot (parity, q) of every region holds rank q's down output of the
  // layers of that parity: [whole rows: ntok x H][CTA partials @xws_off].
  uint32_t world, rank;
  uint8_t* xr[kMaxRanks];
  uint32_t xslot, xws_off;
};

// Exchange region header: the peer-barrier counter, padded.
constexpr size_t kXHeader = 256;

// Epilogue of either stack phase: gate/up -> activation into act (phase A),
// or down rows into the fp32 down vector (phase B).
struct StackEpi {
  bool down_phase;
  uint8_t* act;
  float* down;
  uint32_t I, H, ncb;
  float sm;
  int fn;
  float pmul;  // parked CTA partials are stored times pmul (1, or sm when the sum is taken across ranks)
  __device__ __forceinline__ float park(float v) const { return v * pmul; }
  __device__ __forceinline__ void apply(uint32_t r, int g, int tok, float vg, float vg8) const {
    if (down_phase) {
      RowsEpi{down, nullptr, H, H, sm}.apply(r, g, tok, vg, vg8);
    } else {
      GateUpEpi{act, I, ncb, sm, fn}.apply(r, g, tok, vg, vg8);
    }
  }
};

// Shared layout after the rings: [xs region][red 32 f][xres ntok*H bf16].
// The xs region holds phase B's fragments, or phase A's fragments followed by
// the glue's xn (tmp, fp32).
__host__ __device__ inline size_t stack_xs_region(uint32_t KTA, uint32_t KTB, int nc, uint32_t H, int ntok) {
  const size_t b = frag_bytes(KTB, nc);
  const size_t a = frag_bytes(KTA, nc) + static_cast<size_t>(ntok) * H * 4;
  return ((b > a ? b : a) + 15) / 16 * 16;
}
// [...][xres][down row splits: dn.RT uint2][row spans: dn.RT u32][CTA first rows: #CTAs u32]
__host__ __device__ inline size_t stack_tables_offset(uint32_t nst, uint32_t KTA, uint32_t KTB, int nc, uint32_t H,
                                                      int ntok) {
  return (base_smem_bytes(nst, ntok) + stack_xs_region(KTA, KTB, nc, H, ntok) + 128 +
          static_cast<size_t>(ntok) * H * 2 + 15) / 16 * 16;
}
__host__ __device__ inline size_t stack_smem_bytes(uint32_t nst, uint32_t KTA, uint32_t KTB, int nc, uint32_t H,
                                                   int ntok, uint32_t RTB, uint32_t nctas) {
  return stack_tables_offset(nst, KTA, KTB, nc, H, ntok) + (static_cast<size_t>(RTB) * 3 + nctas) * 4;
}

// Slot (parity, owner) of rank `region`'s exchange region (TP stacks).
__device__ __forceinline__ float* xslot_ptr(const StackParams& p, uint32_t region, uint32_t par, uint32_t owner) {
  return reinterpret_cast<float*>(p.xr[region] + kXHeader) + (static_cast<size_t>(par) * p.world + owner) * p.xslot;
}

// Tensor parallelism: copy what this CTA wrote into its own rank's slot --
// its whole down rows [row0, row1) and its two CTA-partial slots -- to the
// same offsets of every peer's slot (plain stores over NVLink, consecutive
// threads on consecutive floats).
inline __device__ void push_down(const StackParams& p, uint32_t par, uint32_t row0, uint32_t row1) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  consumers_sync();  // every warp's rows and partials are written
  const float* src = xslot_ptr(p, p.rank, par, p.rank);
  const uint32_t H = p.H, ntok = static_cast<uint32_t>(p.ntok);
  const uint32_t h0 = min(row0 * 16, H), h1 = min(row1 * 16, H), nr = h1 - h0;
  const uint32_t sf = ntok * 16, n_rows = nr * ntok, n = n_rows + 2 * sf;
  for (uint32_t e = threadIdx.x; e < n; e += NTHR) {
    size_t off;
    if (e < n_rows) {
      const uint32_t tok = e / nr;
      off = static_cast<size_t>(tok) * H + h0 + (e - tok * nr);
    } else {
      off = p.xws_off + static_cast<size_t>(blockIdx.x) * 2 * sf + (e - n_rows);
    }
    const float v = __ldcg(src + off);
    for (uint32_t q = 0; q < p.world; ++q)
      if (q != p.rank) xslot_ptr(p, q, par, p.rank)[off] = v;
  }
}

// Tensor parallelism with a row-aligned down partition (every down row whole
// in one CTA, so a rank's slot holds whole rows only): dsum[e] = the ranks'
// values of element e summed in rank order, as tp_gather computes it, but
// with one 16-byte load per rank and group of four elements, and the loads
// of four ranks for two groups per thread in flight together.
__device__ __forceinline__ void tp_gather_rows(const StackParams& p, uint32_t par, float* dsum) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  constexpr int WG = 4;      // ranks per batch
  constexpr int kQuads = 2;  // element quads per thread per pass
  const uint32_t W = p.world, nquads = static_cast<uint32_t>(p.ntok) * p.H / 4;
  for (uint32_t base = 0; base < nquads; base += NTHR * kQuads) {
    float4 acc[kQuads];
    for (uint32_t q0 = 0; q0 < W; q0 += WG) {
      float4 a[kQuads][WG];
#pragma unroll
      for (int i = 0; i < kQuads; ++i)
#pragma unroll
        for (int qq = 0; qq < WG; ++qq) {
          const uint32_t quad = base + i * NTHR + threadIdx.x;
          a[i][qq] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (q0 + qq < W && quad < nquads)
            a[i][qq] = __ldcg(reinterpret_cast<const float4*>(xslot_ptr(p, p.rank, par, q0 + qq) + 4 * quad));
        }
#pragma unroll
      for (int i = 0; i < kQuads; ++i)
#pragma unroll
        for (int qq = 0; qq < WG; ++qq) {
          const uint32_t q = q0 + qq;
          if (q >= W) continue;
          if (q == 0) {
            acc[i] = a[i][qq];
          } else {
            acc[i].x += a[i][qq].x;
            acc[i].y += a[i][qq].y;
            acc[i].z += a[i][qq].z;
            acc[i].w += a[i][qq].w;
          }
        }
    }
#pragma unroll
    for (int i = 0; i < kQuads; ++i) {
      const uint32_t quad = base + i * NTHR + threadIdx.x;
      if (quad < nquads) *reinterpret_cast<float4*>(dsum + 4 * quad) = acc[i];
    }
  }
  consumers_sync();
}

// Tensor parallelism: sum the ranks' partial down projections of the
// previous layer (their slots in this GPU's exchange region, complete after
// the peer barrier) into dsum (fp32 [ntok][H], before the glue's bf16
// rounding), every element as the one-GPU glue reads it -- each rank's
// whole-row value or its CTA partials (pre-scaled) summed in CTA order, the
// ranks summed in rank order.  Memory-level parallelism is what matters:
// a thread owns kQuads groups of four consecutive elements (16-byte loads)
// and issues the loads of all of them, for two ranks at a time, before it
// adds anything (more in flight makes the kernel spill around the call).
static __device__ __noinline__ void tp_gather(const StackParams& p, uint32_t par, const uint2* split,
                                       const uint32_t* cfirst, const uint32_t* span, float* dsum) {
  if (p.ptB.aligned) {  // whole rows only: one load per rank and element
    tp_gather_rows(p, par, dsum);
    return;
  }
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  constexpr int WG = 2;      // ranks per batch
  constexpr int kQuads = 1;  // element quads per thread per pass
  const uint32_t H = p.H, ntok = static_cast<uint32_t>(p.ntok), W = p.world;
  const uint32_t nquads = ntok * H / 4, sf = ntok * 16;
  for (uint32_t base = 0; base < nquads; base += NTHR * kQuads) {
    uint32_t eq[kQuads], rq[kQuads], elq[kQuads];
    uint2 oq[kQuads];
    float4 acc[kQuads];
#pragma unroll
    for (int i = 0; i < kQuads; ++i) {
      const uint32_t q = base + i * NTHR + threadIdx.x;
      eq[i] = 4 * q;
      const uint32_t tok = q < nquads ? eq[i] / H : 0, h = eq[i] - tok * H;
      rq[i] = h >> 4;
      oq[i] = q < nquads ? split[rq[i]] : make_uint2(~0u, ~0u);
      elq[i] = tok * 16 + (h & 15);
      acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (uint32_t q0 = 0; q0 < W; q0 += WG) {
      float4 a[kQuads][WG], b[kQuads][WG];
#pragma unroll
      for (int i = 0; i < kQuads; ++i)
#pragma unroll
        for (int qq = 0; qq < WG; ++qq) {
          a[i][qq] = b[i][qq] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (q0 + qq >= W || base + i * NTHR + threadIdx.x >= nquads) continue;
          const float* d = xslot_ptr(p, p.rank, par, q0 + qq);
          const uint2 o = oq[i];
          if (o.x == ~0u) {
            a[i][qq] = __ldcg(reinterpret_cast<const float4*>(d + eq[i]));
          } else if (o.y != ~0u) {
            a[i][qq] = __ldcg(reinterpret_cast<const float4*>(d + p.xws_off + o.x + elq[i]));
            b[i][qq] = __ldcg(reinterpret_cast<const float4*>(d + p.xws_off + o.y + elq[i]));
          } else {  // a row tile over three or more CTAs (small problems)
            const uint32_t sp = span[rq[i]];
            for (uint32_t c = sp & 0xFFFFu; c <= (sp >> 16); ++c) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(
                  d + p.xws_off + (static_cast<size_t>(c) * 2 + (rq[i] == cfirst[c] ? 0 : 1)) * sf + elq[i]));
              a[i][qq].x += v.x;
              a[i][qq].y += v.y;
              a[i][qq].z += v.z;
              a[i][qq].w += v.w;
            }
          }
        }
#pragma unroll
      for (int i = 0; i < kQuads; ++i) {
        const bool two = oq[i].x != ~0u && oq[i].y != ~0u;
#pragma unroll
        for (int qq = 0; qq < WG; ++qq) {
          const uint32_t q = q0 + qq;
          if (q >= W) continue;
          const float4 t = two ? make_float4(a[i][qq].x + b[i][qq].x, a[i][qq].y + b[i][qq].y,
                                             a[i][qq].z + b[i][qq].z, a[i][qq].w + b[i][qq].w)
                               : a[i][qq];
          if (q == 0) {
            acc[i] = t;
          } else {
            acc[i].x += t.x;
            acc[i].y += t.y;
            acc[i].z += t.z;
            acc[i].w += t.w;
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kQuads; ++i)
      if (base + i * NTHR + threadIdx.x < nquads) *reinterpret_cast<float4*>(dsum + eq[i]) = acc[i];
  }
  consumers_sync();
}

// The last layer's down projection as the final glue read it (fp32, summed
// over CTAs and, with tensor parallelism, over ranks): a test probe.
template <class DL>
__device__ void write_probe(float* probe, int ntok, uint32_t H, const DL& dl) {
  const uint32_t n = static_cast<uint32_t>(ntok) * H;
  for (uint32_t e = threadIdx.x; e < n; e += kConsumerWarps * 32) {
    const uint32_t tok = e / H, h = e - tok * H;
    float a, b;
    uint32_t how;
    dl.load(tok, h, e, a, b, how);
    probe[e] = dl.combine(a, b, how);
  }
}

// TP = true: one rank of a tensor-parallel stack (see StackParams).  Phase B
// writes this rank's partial down projection into its own exchange slot and
// pushes it to every peer; after the rank's grid barrier the ranks meet in
// peer_exchange, and the next glue sums the ranks' slots in rank order.  The
// slots alternate between two parities by the global count of exchanges, so
// a rank that runs ahead writes the other parity from the one its peers
// still read.
template <int NT, bool FAST, bool TP>
__global__ void __launch_bounds__(kThreadsPerCta, 1) ffn_stack_kernel(const __grid_constant__ StackParams p) {
  constexpr int NC = NT;  // bf16 activations: one fragment column per token
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t wk[kConsumerWarps][4];  // per warp: a0 a1 b0 b1
  __shared__ StackWork sw[kConsumerWarps];
  __shared__ unsigned long long xbase_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Partition& ptA = p.ptA;
  const Partition& ptB = p.ptB;
  Shape::init_barriers(smem, p.nst);
  const unsigned long long bar_base = threadIdx.x == 0 ? grid_base(p.bar, gridDim.x) : 0ull;
  if (TP && threadIdx.x == 0) xbase_s = peer_base(p.xr[p.rank], p.world);
  if (lane == 0) {
    uint32_t* w = wk[warp];
    ptA.warp_range(blockIdx.x, warp, w[0], w[1]);
    ptB.warp_range(blockIdx.x, warp, w[2], w[3]);
    sw[warp] = StackWork{p.layers, p.L, w[0], w[1] - w[0], w[2], w[3] - w[2], p.gu.KT, p.dn.KT,
                         w[0] - ptA.kt.div(w[0]) * p.gu.KT, w[2] - ptB.kt.div(w[2]) * p.dn.KT};
  }
  // Down row tiles -> the CTAs holding them (one CTA: `down` has the row;
  // several: the glue sums their partials), and each CTA's first row tile.
  uint2* split = reinterpret_cast<uint2*>(smem + stack_tables_offset(p.nst, p.gu.KT, p.dn.KT, NC, p.H, p.ntok));
  uint32_t* span = reinterpret_cast<uint32_t*>(split + p.dn.RT);
  uint32_t* cfirst = span + p.dn.RT;
  for (uint32_t r = threadIdx.x; r < p.dn.RT; r += blockDim.x) {
    const uint32_t rb = r * p.dn.KT;
    span[r] = ptB.aligned ? 0u : (ptB.cta_of_unit(rb) | (ptB.cta_of_unit(rb + p.dn.KT - 1) << 16));
  }
  for (uint32_t c = threadIdx.x; c < gridDim.x; c += blockDim.x) cfirst[c] = ptB.kt.div(ptB.cta_begin(c));
  __syncthreads();
  for (uint32_t r = threadIdx.x; r < p.dn.RT; r += blockDim.x) {
    const uint32_t clo = span[r] & 0xFFFFu, chi = span[r] >> 16;
    const uint32_t sf = static_cast<uint32_t>(p.ntok) * 16;
    uint2 o = make_uint2(~0u, ~0u);
    if (chi == clo + 1) {
      o.x = (clo * 2 + (r == cfirst[clo] ? 0 : 1)) * sf;
      o.y = (chi * 2 + (r == cfirst[chi] ? 0 : 1)) * sf;
    } else if (chi > clo + 1) {
      o.x = clo;
    }
    split[r] = o;
  }
  __syncthreads();
  // TP: this CTA's whole down rows [prow0, prow1) (pushed to the peers), and
  // the parity of layer 0's exchange slots.
  uint32_t prow0 = 0, prow1 = 0, xpar0 = 0;
  unsigned long long xbase = 0;
  if (TP) {
    const uint32_t c0 = ptB.cta_begin(blockIdx.x), c1 = ptB.cta_begin(blockIdx.x + 1);
    prow0 = ptB.kt.div(c0 + p.dn.KT - 1);
    prow1 = ptB.kt.div(c1);
    if (prow1 < prow0) prow1 = prow0;
    xbase = xbase_s;
    xpar0 = static_cast<uint32_t>(div_counter(xbase, p.world)) & 1u;
  }
  const uint32_t* my = wk[warp];
  ConsumerRing<kUnitsPerStage, StackWork> ring;
  ring.setup(smem, p.nst, warp, p.L * ((my[1] - my[0]) + (my[3] - my[2])), &sw[warp]);
  // The previous layer's down projection as the glue reads it.
  auto down_in = [&](uint32_t l) {
    return DownIn{p.down, p.fxB.ws, split, cfirst, span, static_cast<uint32_t>(p.ntok) * 16,
                  __ldg(&p.layers[l].dn_mul)};
  };
  // The act padding (k in [I, 64*dn.KT)) must read as zero in phase B.
  if (blockIdx.x == 0) {
    const uint32_t kpad = p.dn.KT * 64;
    for (uint32_t e = threadIdx.x; e < (kpad - p.I) * NC; e += NTHR) {
      const uint32_t n = e % NC, k = p.I + e / NC;
      *reinterpret_cast<uint16_t*>(p.act + frag_offset(NC, n, k)) = 0;
    }
  }
#pragma unroll 1
  for (uint32_t i = 0; i < 2 * p.L; ++i) {
    const uint32_t l = i >> 1;
    const bool B = i & 1;
    uint8_t* xs = smem + base_smem_bytes(p.nst, p.ntok);
    unsigned long long* tr = (l == 1) ? p.trace : nullptr;
    float* bdown = TP ? xslot_ptr(p, p.rank, (xpar0 + l) & 1u, p.rank) : p.down;
    if (!B) {
      float* red = reinterpret_cast<float*>(xs + stack_xs_region(p.gu.KT, p.dn.KT, NC, p.H, p.ntok));
      uint16_t* xres = reinterpret_cast<uint16_t*>(red + 32);  // the residual stream (bf16)
      trace_mark(tr, 0);
      const XnOut xn{nullptr, xs, static_cast<uint32_t>(NC), p.gu.KT * 64};
      if (l == 0) {
        glue<true, false>(p.ntok, p.H, p.eps, Bf16In{p.x_in}, NoIn{}, Bf16Out{xres}, xn, red);
      } else if constexpr (TP) {
        float* dsum = reinterpret_cast<float*>(xs + frag_bytes(p.gu.KT, NC));  // after the x fragments
        tp_gather(p, (xpar0 + l - 1) & 1u, split, cfirst, span, dsum);
        glue<true, true>(p.ntok, p.H, p.eps, Bf16In{xres}, F32In{dsum}, Bf16Out{xres}, xn, red, tr);
      } else {
        glue<true, true>(p.ntok, p.H, p.eps, Bf16In{xres}, down_in(l - 1), Bf16Out{xres}, xn, red, tr);
      }
    } else {
      stage_from_l2(xs, p.act, static_cast<uint32_t>(frag_bytes(p.dn.KT, NC)));
    }
    consumers_sync();
    trace_mark(tr, B ? 4 : 1);
    const float sm = B ? __ldg(&p.layers[l].dn_mul) : __ldg(&p.layers[l].gu_mul);
    const StackEpi epi{B, p.act, bdown, p.I, p.H, NC, sm, p.fn, TP ? sm : 1.0f};
    Fixup fx = B ? p.fxB : p.fxA;
    if (TP && B) fx.ws = bdown + p.xws_off;
    fx.part = reinterpret_cast<float*>(smem + ring_smem_bytes(p.nst));
    const bool ok = consume_range<NC, false, FAST>(ring, B ? p.dn : p.gu, my[B ? 2 : 0], my[B ? 3 : 1], xs, fx,
                                                   p.ntok, epi, p.status);
    if (tr) {
      consumers_sync();
      trace_mark(tr, B ? 8 : 7);
    }
    if (B)
      cta_fixup<true>(ptB, &wk[0][2], fx, p.ntok, epi);  // rows shared between CTAs: summed by the next glue
    else
      cta_fixup(ptA, &wk[0][0], fx, p.ntok, epi);
    if (TP && B) push_down(p, (xpar0 + l) & 1u, prow0, prow1);
    if (tr) {
      consumers_sync();
      trace_mark(tr, B ? 5 : 2);
    }
    bool bar_ok = grid_barrier_epoch(p.bar, gridDim.x, bar_base, i + 1, p.status);
    if (TP && B && bar_ok) bar_ok = peer_exchange(p.xr, p.world, p.rank, xbase, l + 1, p.status);
    if (!bar_ok || !consumers_and(ok)) {
      ring.drain();
      return;
    }
    trace_mark(tr, B ? 6 : 3);
  }
  if (blockIdx.x == 0) {
    float* red = reinterpret_cast<float*>(smem + base_smem_bytes(p.nst, p.ntok) +
                                          stack_xs_region(p.gu.KT, p.dn.KT, NC, p.H, p.ntok));
    const Bf16In xl{reinterpret_cast<uint16_t*>(red + 32)};
    if constexpr (TP) {
      float* dsum = reinterpret_cast<float*>(smem + base_smem_bytes(p.nst, p.ntok) + frag_bytes(p.gu.KT, NC));
      tp_gather(p, (xpar0 + p.L - 1) & 1u, split, cfirst, span, dsum);
      glue<false, true>(p.ntok, p.H, p.eps, xl, F32In{dsum}, Bf16Out{p.out}, XnOut{}, red);
      if (p.probe)
        for (uint32_t e = threadIdx.x; e < static_cast<uint32_t>(p.ntok) * p.H; e += NTHR) p.probe[e] = dsum[e];
    } else {
      glue<false, true>(p.ntok, p.H, p.eps, xl, down_in(p.L - 1), Bf16Out{p.out}, XnOut{}, red);
      if (p.probe) write_probe(p.probe, p.ntok, p.H, down_in(p.L - 1));
    }
  }
}

}  // namespace alv
