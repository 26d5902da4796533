// One-launch Llama decode step: every layer's RMSNorm, QKV projection, RoPE,
// KV-cache append, GQA attention, O projection, residuals, SwiGLU FFN, then
// the LM head and the greedy argmax, in one persistent kernel of one CTA per
// SM separated by grid barriers.  The Q4 weights of the whole step (~700 MB
// for Llama-3.2-1B) stream through the same per-warp bulk-copy rings as the
// FFN stack, so the next projection's weights are already in flight while a
// phase's reduction, barrier and glue run; the step costs one launch instead
// of about a hundred.
//
// The arithmetic is the separate-kernel step's (decode.cuh, gemv_kernel,
// ffn_kernel) operation for operation: the same unit partitions and split-K
// orders, the same bf16 rounding points, RMSNorm sums in the order of a
// 1024-thread CTA and attention on 256 threads in the order of
// attention_kernel.  Its logits are therefore bit-identical to that path
// (runtime/py/model.py:821-934 for the reference's CPU step).
#pragma once

#include <cuda_fp16.h>

#include "decode.cuh"
#include "kernels.cuh"

namespace alv {

// Batched prefill: act[b][i] = bf16(swiglu(gate, up)) from the gate/up
// projection of the interleaved matrix (rows 16r..16r+7 gate, 16r+8..16r+15
// up of intermediate indices 8r..8r+7), gate and up bf16 as the FFN's
// epilogue rounds them (model.py:689-698 for SwiGLU).
__global__ void __launch_bounds__(256) swiglu_rows_kernel(const uint16_t* __restrict__ gu, int I,
                                                          uint16_t* __restrict__ act) {
  const int b = blockIdx.y;
  const uint16_t* row = gu + static_cast<size_t>(b) * 2 * I;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < I; i += gridDim.x * blockDim.x) {
    const int r = i >> 3, g = i & 7;
    const float gate = bf16_bits_to_f32(row[r * 16 + g]), up = bf16_bits_to_f32(row[r * 16 + 8 + g]);
    act[static_cast<size_t>(b) * I + i] = bf16_bits_rn(swiglu_ref(gate, up));
  }
}

// The position the next decode step consumes, after a batched prefill.
__global__ void set_pos_kernel(DecodeState* st, int pos) {
  if (threadIdx.x == 0) st->pos = pos;
}

// Per-layer weights: 0 [q|k|v], 1 o, 2 gate/up (interleaved), 3 down.
struct LlamaLayerW {
  const uint8_t* mat[4];
  float mul[4];  // dequant epilogue multipliers (2^je, or 1)
};

// Work of one warp over a whole step: segment 4l + k is matrix k of layer l,
// segment 4L the LM head.  The warp owns units [u0[k], u0[k] + n[k]) of
// matrix k in every layer (the layers share shapes and partitions).
struct LlamaWork {
  const LlamaLayerW* layers;
  const uint8_t* lm;
  uint32_t count;  // segments: 4L, plus 1 with the LM head
  uint32_t L4;
  uint32_t u0[5], n[5], KT[5], kt0[5];
  __device__ uint32_t nseg() const { return count; }
  __device__ void get(uint32_t i, const uint8_t*& base, uint32_t& cnt, uint32_t& kt_per_row, uint32_t& kt) const {
    const uint32_t k = i < L4 ? (i & 3u) : 4u;
    const uint8_t* m =
        k == 4 ? lm
               : reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(&layers[i >> 2].mat[k])));
    base = m + static_cast<size_t>(u0[k]) * kUnitBytes;
    cnt = n[k];
    kt_per_row = KT[k];
    kt = kt0[k];
  }
};

constexpr int kLlamaMats = 5;         // qkv, o, gate/up, down, LM head
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnChunk = 128;       // cached V rows staged in shared memory at a time

struct LlamaStepParams {
  const LlamaLayerW* layers;
  const uint8_t* lm;
  float lm_mul;
  uint32_t L;
  Q4Mat mat[kLlamaMats];            // shapes (RT, KT) of each kind
  Partition pt[kLlamaMats];         // the separate-kernel step's splits, for this grid
  uint32_t H, I, nq, nkv, hd, max_seq, V;
  float eps;
  double attn_scale;
  int logits;                       // LM head + argmax (else only the position advances)
  const uint16_t* emb;              // f16 [V][H]
  const float* norms;               // [2L + 1][H]
  const uint16_t* rope;             // bf16 [max_seq][2 hd]
  uint16_t* kcache;                 // bf16 [L][nkv][max_seq][hd]
  uint16_t* vcache;
  DecodeState* state;
  int* tokens;
  int* pred;
  uint16_t* qkvb;                   // bf16 [nq + 2 nkv][hd]... as rows of the qkv projection
  uint16_t* attn;                   // bf16 [nq * hd]
  uint16_t* proj;                   // bf16 [H]: O projection
  uint16_t* logit16;                // bf16 [V]
  uint8_t* act;                     // SwiGLU output, B-fragment order
  float* down;                      // fp32 [H]: down rows held by one CTA (scaled)
  float* dws;                       // down rows shared between CTAs: CTA partials
  Fixup fx;                         // split-K scratch of the other projections (ws, counters)
  float* cand_v;                    // [#CTAs] argmax candidates
  int* cand_i;
  GridBar* bar;
  uint32_t* status;
  uint32_t nst;
  unsigned long long* trace;        // optional: phase stamps of layer 1
};

// Dynamic shared memory after the rings and warp partials.  The attention
// area (q, the position's k and v, partial sums, scores, two V chunks)
// shares its space with the B-fragment area xs: attention runs between the
// qkv projection, whose fragments are consumed, and the O staging.
struct LlamaSmem {
  size_t xs, attn, xres, nw, red, tables, end;
};
__host__ __device__ inline size_t attn_floats(uint32_t hd, uint32_t max_seq) {
  return (static_cast<size_t>(3 * hd + kAttnThreads + max_seq) + 3) / 4 * 4;
}
__host__ __device__ inline LlamaSmem llama_smem(uint32_t nst, uint32_t kt_max, uint32_t H, uint32_t hd,
                                                uint32_t max_seq, uint32_t dn_rt, uint32_t nctas) {
  LlamaSmem s;
  s.xs = base_smem_bytes(nst, 1);
  s.attn = s.xs;
  const size_t frag = (frag_bytes(kt_max, 1) + 15) / 16 * 16;
  const size_t attn = attn_floats(hd, max_seq) * 4 + static_cast<size_t>(2) * kAttnChunk * hd * 2;
  s.xres = s.xs + (frag > attn ? frag : attn);
  s.nw = s.xres + (static_cast<size_t>(H) * 4 + 15) / 16 * 16;
  s.red = s.nw + (static_cast<size_t>(H) * 4 + 15) / 16 * 16;
  s.tables = s.red + 64 * 4;
  s.end = s.tables + (static_cast<size_t>(dn_rt) * 3 + nctas) * 4;
  return s;
}

// 16-byte asynchronous copies global -> shared of `n` rows of `hd` bf16
// (thread t of the 256 attention threads copies vectors t, t + 256, ...).
__device__ __forceinline__ void attn_copy_rows(uint16_t* dst, const uint16_t* src, uint32_t n, uint32_t hd) {
  const uint32_t nvec = n * (hd / 8);
  for (uint32_t e = threadIdx.x; e < nvec; e += kAttnThreads)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + 8 * e)), "l"(src + 8 * e)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Sum of x[h]^2 over h < H in the order of rmsnorm_store on a 1024-thread
// CTA: virtual thread t sums h = t, t + 1024, ... in sequence; a warp's 32
// virtual threads by the xor tree; the 32 virtual warps in order.  Real
// warp w plays virtual warps w, w + W, w + 2W (W consumer warps).
__device__ __forceinline__ float llama_sumsq(const float* x, uint32_t H, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int vw = warp; vw < 32; vw += kConsumerWarps) {
    float ss = 0.f;
    for (uint32_t h = static_cast<uint32_t>(vw * 32 + lane); h < H; h += kDecodeThreads)
      ss = __fadd_rn(ss, __fmul_rn(x[h], x[h]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[vw] = ss;
  }
  consumers_sync();
  float s = 0.f;
  for (int i = 0; i < 32; ++i) s += red[i];
  return s;
}

// Start copying a norm weight vector (H floats, 16-byte aligned) into shared
// memory (cp.async, no registers held), at the start of a glue, so that its
// latency overlaps the residual's loads; llama_norm_frag waits for it.
__device__ __forceinline__ void load_norm_w(float* dst, const float* __restrict__ w, uint32_t H) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  for (uint32_t k = 4 * threadIdx.x; k < H; k += 4 * NTHR)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + k)), "l"(w + k) : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// xn = bf16((x * inv) * w) into the B-fragment layout of a KT-tile matrix
// (one column; k in [H, 64 KT) zero), inv = 1 / sqrt(mean(x^2) + eps); w is
// the shared-memory copy load_norm_w started.
__device__ __forceinline__ void llama_norm_frag(const float* x, uint32_t H, const float* w, float eps, uint8_t* xs,
                                                uint32_t KT, float* red) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  asm volatile("cp.async.wait_all;" ::: "memory");
  const float ss = llama_sumsq(x, H, red);  // (its barrier also publishes every thread's copies of w)
  const float var = __fdiv_rn(ss, static_cast<float>(H));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const uint32_t kpad = KT * 64;
  for (uint32_t k = 2 * threadIdx.x; k < kpad; k += 2 * NTHR) {
    uint32_t word = 0;
    if (k < H) {
      const uint16_t a = bf16_bits_rn(__fmul_rn(__fmul_rn(x[k], inv), w[k]));
      const uint16_t b = k + 1 < H ? bf16_bits_rn(__fmul_rn(__fmul_rn(x[k + 1], inv), w[k + 1])) : 0;
      word = pack_bf2(a, b);
    }
    *reinterpret_cast<uint32_t*>(xs + frag_offset(1, 0, k)) = word;
  }
  consumers_sync();
}

// x += a bf16 vector written earlier in this launch (the O projection),
// every load in flight before the adds: x = bf16(x + v).
__device__ __forceinline__ void llama_add_bf16(float* x, const uint16_t* v, uint32_t H) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  constexpr int kPairs = 4;  // pairs per thread per pass: one pass for hidden <= 4096 with 16 warps
  for (uint32_t k0 = 2 * threadIdx.x; k0 < H; k0 += 2 * NTHR * kPairs) {
    uint32_t w[kPairs];
#pragma unroll
    for (int j = 0; j < kPairs; ++j) {
      const uint32_t k = k0 + 2 * NTHR * j;
      w[j] = k < H ? __ldcg(reinterpret_cast<const unsigned int*>(v + k)) : 0u;
    }
#pragma unroll
    for (int j = 0; j < kPairs; ++j) {
      const uint32_t k = k0 + 2 * NTHR * j;
      if (k < H) {
        x[k] = bf16_round(__fadd_rn(x[k], bf16_bits_to_f32(w[j] & 0xFFFFu)));
        x[k + 1] = bf16_round(__fadd_rn(x[k + 1], bf16_bits_to_f32(w[j] >> 16)));
      }
    }
  }
  consumers_sync();
}

// A bf16 vector written earlier in this launch, into the B-fragment layout
// (k in [K, 64 KT) zero).  Loads bypass L1: other SMs wrote the data.
__device__ __forceinline__ void llama_stage_bf16(const uint16_t* src, uint32_t K, uint8_t* xs, uint32_t KT) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  const uint32_t kpad = KT * 64;
  for (uint32_t k = 2 * threadIdx.x; k < kpad; k += 2 * NTHR) {
    uint32_t word = 0;
    if (k + 1 < K) {
      word = __ldcg(reinterpret_cast<const unsigned int*>(src + k));
    } else if (k < K) {
      word = __ldcg(reinterpret_cast<const unsigned short*>(src + k));
    }
    *reinterpret_cast<uint32_t*>(xs + frag_offset(1, 0, k)) = word;
  }
  consumers_sync();
}

// Named barrier of the 256 attention threads (barrier 2).
__device__ __forceinline__ void attn_sync() { asm volatile("bar.sync 2, %0;" ::"n"(kAttnThreads) : "memory"); }

__device__ __forceinline__ float attn_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  attn_sync();
  if (lane == 0) red[warp] = v;
  attn_sync();
  float s = 0.f;
  for (int i = 0; i < kAttnWarps; ++i) s += red[i];
  return s;
}
__device__ __forceinline__ float attn_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  attn_sync();
  if (lane == 0) red[warp] = v;
  attn_sync();
  float s = red[0];
  for (int i = 1; i < kAttnWarps; ++i) s = fmaxf(s, red[i]);
  return s;
}

// RoPE, KV append and attention of query head `head` (threads [0, 256) of
// its CTA), as rope_cache_kernel + attention_kernel compute them.  The
// position's own K and V are used from registers/shared memory (the cache
// gets them from the group's first head, for later steps), so no barrier
// separates the append from the reads.
// Out of line: its own register budget (inlined into the step kernel, whose
// streaming state stays live around it, its loops spilled).
static __device__ __noinline__ void llama_attention(const LlamaStepParams& p, uint32_t l, int pos, uint32_t head,
                                                   float* sm, float* red) {
  const uint32_t hd = p.hd, half = hd / 2, group = p.nq / p.nkv, kvh = head / group;
  float* qs = sm;
  float* kp = qs + hd;
  float* vp = kp + hd;
  float* part = vp + hd;
  float* sc = part + kAttnThreads;
  // two V chunks of kAttnChunk rows after the scores, 16-byte aligned
  uint16_t* vbuf = reinterpret_cast<uint16_t*>(sm + attn_floats(hd, p.max_seq));
  const size_t kvl = static_cast<size_t>(p.nkv) * p.max_seq * hd;
  uint16_t* kc = p.kcache + l * kvl + static_cast<size_t>(kvh) * p.max_seq * hd;
  uint16_t* vc = p.vcache + l * kvl + static_cast<size_t>(kvh) * p.max_seq * hd;
  const uint16_t* cs = p.rope + static_cast<size_t>(pos) * 2 * hd;
  const uint32_t t = threadIdx.x;
  const bool writer = head % group == 0;
  // The cached V rows of the first two chunks start loading now, behind the
  // RoPE, the scores and the softmax.  (Row `pos` is being written by the
  // group's first head meanwhile; its copy is never read: v_pos comes from
  // vp.)
  const int seq = pos + 1;
  const int nch = (seq + kAttnChunk - 1) / kAttnChunk;
  for (int c = 0; c < 2 && c < nch; ++c) {
    const int c0 = c * kAttnChunk;
    attn_copy_rows(vbuf + static_cast<size_t>(c & 1) * kAttnChunk * hd, vc + static_cast<size_t>(c0) * hd,
                   static_cast<uint32_t>(seq - c0 < kAttnChunk ? seq - c0 : kAttnChunk), hd);
  }
  if (t < half) {
    const uint16_t* q = p.qkvb + head * hd;
    const float x1 = bf16_bits_to_f32(__ldcg(q + t)), x2 = bf16_bits_to_f32(__ldcg(q + t + half));
    const float c = bf16_bits_to_f32(cs[t]), s = bf16_bits_to_f32(cs[hd + t]);
    qs[t] = bf16_round(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    qs[t + half] = bf16_round(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
  } else if (t < 2 * half) {
    const uint32_t i = t - half;
    const uint16_t* k = p.qkvb + (p.nq + kvh) * hd;
    const float x1 = bf16_bits_to_f32(__ldcg(k + i)), x2 = bf16_bits_to_f32(__ldcg(k + i + half));
    const float c = bf16_bits_to_f32(cs[i]), s = bf16_bits_to_f32(cs[hd + i]);
    const uint16_t y1 = bf16_bits_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    const uint16_t y2 = bf16_bits_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    kp[i] = bf16_bits_to_f32(y1);
    kp[i + half] = bf16_bits_to_f32(y2);
    if (writer) {
      kc[static_cast<size_t>(pos) * hd + i] = y1;
      kc[static_cast<size_t>(pos) * hd + i + half] = y2;
    }
  } else if (t < 2 * half + hd) {
    const uint32_t d = t - 2 * half;
    const uint16_t v = __ldcg(p.qkvb + (p.nq + p.nkv + kvh) * hd + d);
    vp[d] = bf16_bits_to_f32(v);
    if (writer) vc[static_cast<size_t>(pos) * hd + d] = v;
  }
  attn_sync();
  float mx = -INFINITY;
  for (int j = static_cast<int>(t); j < seq; j += kAttnThreads) {
    float dot = 0.f;
    if (j == pos) {
      for (uint32_t d = 0; d < hd; ++d) dot = fmaf(kp[d], qs[d], dot);
    } else {
      dot = attn_dot(kc + static_cast<size_t>(j) * hd, qs, static_cast<int>(hd));
    }
    const float s = static_cast<float>(static_cast<double>(dot) * p.attn_scale);
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = attn_max(mx, red);
  float sum = 0.f;
  for (int j = static_cast<int>(t); j < seq; j += kAttnThreads) {
    const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(sc[j], mx))));
    sc[j] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = attn_sum(sum, red + 16);
  for (int j = static_cast<int>(t); j < seq; j += kAttnThreads) sc[j] = __fdiv_rn(sc[j], sum);
  attn_sync();
  // out[d] = sum_j p_j v_j[d], thread (g, d) summing j = g, g + G, ... in
  // order (as attention_kernel); the cached rows come through shared memory,
  // double-buffered: chunk c + 2 loads while chunk c + 1 is summed.
  const uint32_t G = kAttnThreads / hd;
  const uint32_t g = t / hd, d = t - g * hd;
  float acc = 0.f;
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    attn_sync();
    const int c0 = c * kAttnChunk;
    const int n = seq - c0 < kAttnChunk ? seq - c0 : kAttnChunk;
    const uint16_t* vsh = vbuf + static_cast<size_t>(c & 1) * kAttnChunk * hd;
    if (g < G)
      for (int j = c0 + static_cast<int>(g); j < c0 + n; j += static_cast<int>(G)) {
        const float v = j == pos ? vp[d] : bf16_bits_to_f32(vsh[static_cast<size_t>(j - c0) * hd + d]);
        acc = fmaf(sc[j], v, acc);
      }
    attn_sync();
    if (c + 2 < nch) {
      const int c2 = (c + 2) * kAttnChunk;
      attn_copy_rows(vbuf + static_cast<size_t>(c & 1) * kAttnChunk * hd, vc + static_cast<size_t>(c2) * hd,
                     static_cast<uint32_t>(seq - c2 < kAttnChunk ? seq - c2 : kAttnChunk), hd);
    }
  }
  if (g < G) part[g * hd + d] = acc;
  attn_sync();
  if (t < hd) {
    float o = 0.f;
    for (uint32_t gg = 0; gg < G; ++gg) o = __fadd_rn(o, part[gg * hd + t]);
    p.attn[head * hd + t] = bf16_bits_rn(o);
  }
}

template <bool FAST>
__global__ void __launch_bounds__(kThreadsPerCta, 1) llama_step_kernel(const __grid_constant__ LlamaStepParams p) {
  constexpr uint32_t NTHR = kConsumerWarps * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ LlamaWork sw[kConsumerWarps];
  __shared__ uint32_t wr[kLlamaMats][kConsumerWarps][4];  // per matrix and warp: unit range [u0, u1)
  __shared__ int pos_s, tok_s, nprompt_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t kt_max = 0;
  for (int k = 0; k < kLlamaMats; ++k) kt_max = p.mat[k].KT > kt_max ? p.mat[k].KT : kt_max;
  const LlamaSmem lay = llama_smem(p.nst, kt_max, p.H, p.hd, p.max_seq, p.mat[3].RT, gridDim.x);
  uint8_t* xs = smem + lay.xs;
  float* xres = reinterpret_cast<float*>(smem + lay.xres);
  float* nw = reinterpret_cast<float*>(smem + lay.nw);  // the current norm weights
  float* red = reinterpret_cast<float*>(smem + lay.red);
  float* asm_ = reinterpret_cast<float*>(smem + lay.attn);  // (shares xs)
  uint2* split = reinterpret_cast<uint2*>(smem + lay.tables);
  uint32_t* span = reinterpret_cast<uint32_t*>(split + p.mat[3].RT);
  uint32_t* cfirst = span + p.mat[3].RT;

  // Each warp starts its weight stream first (its ring, ranges and work list
  // are its own).
  Shape::init_warp_barriers(smem, p.nst, warp);
  if (lane == 0) {
    LlamaWork w{};
    w.layers = p.layers;
    w.lm = p.lm;
    w.L4 = 4 * p.L;
    w.count = 4 * p.L + (p.logits ? 1u : 0u);
    for (int k = 0; k < kLlamaMats; ++k) {
      uint32_t a, b;
      p.pt[k].warp_range(blockIdx.x, warp, a, b);
      wr[k][warp][0] = a;
      wr[k][warp][1] = b;
      w.u0[k] = a;
      w.n[k] = b - a;
      w.KT[k] = p.mat[k].KT;
      w.kt0[k] = a - p.pt[k].kt.div(a) * p.mat[k].KT;
    }
    sw[warp] = w;
  }
  __syncwarp();
  const LlamaWork& me = sw[warp];
  const uint32_t total = p.L * (me.n[0] + me.n[1] + me.n[2] + me.n[3]) + (p.logits ? me.n[4] : 0u);
  ConsumerRing<kUnitsPerStage, LlamaWork> ring;
  ring.setup(smem, p.nst, warp, total, &sw[warp]);
  const unsigned long long bar_base = threadIdx.x == 0 ? grid_base(p.bar, gridDim.x) : 0ull;
  if (threadIdx.x == 0) {
    pos_s = p.state->pos;
    nprompt_s = p.state->n_prompt;
    tok_s = p.tokens[pos_s];
  }
  // Down row tiles -> the CTAs holding them (as the FFN stack's glue reads them).
  const Partition& ptD = p.pt[3];
  for (uint32_t r = threadIdx.x; r < p.mat[3].RT; r += blockDim.x) {
    const uint32_t rb = r * p.mat[3].KT;
    span[r] = ptD.aligned ? 0u : (ptD.cta_of_unit(rb) | (ptD.cta_of_unit(rb + p.mat[3].KT - 1) << 16));
  }
  for (uint32_t c = threadIdx.x; c < gridDim.x; c += blockDim.x) cfirst[c] = ptD.kt.div(ptD.cta_begin(c));
  __syncthreads();
  for (uint32_t r = threadIdx.x; r < p.mat[3].RT; r += blockDim.x) {
    const uint32_t clo = span[r] & 0xFFFFu, chi = span[r] >> 16;
    uint2 o = make_uint2(~0u, ~0u);
    if (chi == clo + 1) {
      o.x = (clo * 2 + (r == cfirst[clo] ? 0 : 1)) * 16;
      o.y = (chi * 2 + (r == cfirst[chi] ? 0 : 1)) * 16;
    } else if (chi > clo + 1) {
      o.x = clo;
    }
    split[r] = o;
  }
  // The act padding (k in [I, 64 KT) of the down matrix) must read as zero.
  if (blockIdx.x == 0) {
    for (uint32_t k = p.I + threadIdx.x; k < p.mat[3].KT * 64; k += blockDim.x)
      *reinterpret_cast<uint16_t*>(p.act + frag_offset(1, 0, k)) = 0;
  }
  __syncthreads();
  const int pos = pos_s;
  const uint32_t H = p.H;
  Fixup fx = p.fx;
  fx.part = reinterpret_cast<float*>(smem + ring_smem_bytes(p.nst));
  Fixup fxd = fx;
  fxd.ws = p.dws;
  const DownIn din{p.down, p.dws, split, cfirst, span, 16u, 0.f};
  uint32_t epoch = 0;
  auto barrier = [&](bool ok) -> bool {
    const bool b = grid_barrier_epoch(p.bar, gridDim.x, bar_base, ++epoch, p.status);
    return b && consumers_and(ok);
  };
  // x += the previous layer's down projection (bf16, as the FFN writes it);
  // a thread's groups of 8 are loaded two at a time before they are added
  // (one pass for hidden <= 8192 with 16 warps).
  auto add_down = [&](uint32_t l) {
    DownIn d = din;
    d.sm = __ldg(&p.layers[l].mul[3]);
    for (uint32_t g0 = threadIdx.x; g0 < H / 8; g0 += 2 * NTHR) {
      float v[2][8];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint32_t g = g0 + q * NTHR;
        if (g < H / 8) d.load8(0, 8 * g, 8 * g, v[q]);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint32_t g = g0 + q * NTHR;
        if (g >= H / 8) continue;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const uint32_t h = 8 * g + t;
          xres[h] = bf16_round(__fadd_rn(xres[h], bf16_round(v[q][t])));
        }
      }
    }
    consumers_sync();
  };

  for (uint32_t l = 0; l < p.L; ++l) {
    const LlamaLayerW* lw = p.layers + l;
    unsigned long long* tr = l == 1 ? p.trace : nullptr;
    trace_mark(tr, 0);
    // ---- residual + attention RMSNorm, then the [q|k|v] projection
    load_norm_w(nw, p.norms + static_cast<size_t>(2 * l) * H, H);
    if (l == 0) {
      const uint16_t* row = p.emb + static_cast<size_t>(tok_s) * H;
      for (uint32_t h = threadIdx.x; h < H; h += NTHR) xres[h] = bf16_round(__half2float(__ushort_as_half(row[h])));
      consumers_sync();
    } else {
      add_down(l - 1);
    }
    llama_norm_frag(xres, H, nw, p.eps, xs, p.mat[0].KT, red);
    trace_mark(tr, 1);
    const uint32_t nqkv = (p.nq + 2 * p.nkv) * p.hd;
    const RowsEpi eq{nullptr, p.qkvb, nqkv, nqkv, __ldg(&lw->mul[0])};
    bool ok = consume_range<1, false, FAST>(ring, p.mat[0], wr[0][warp][0], wr[0][warp][1], xs, fx, 1, eq, p.status);
    trace_mark(tr, 2);
    cta_fixup(p.pt[0], &wr[0][0][0], fx, 1, eq);
    if (!barrier(ok)) break;
    trace_mark(tr, 3);
    // ---- RoPE, KV append, attention (one CTA per query head)
    if (blockIdx.x < p.nq && threadIdx.x < kAttnThreads) llama_attention(p, l, pos, blockIdx.x, asm_, red + 32);
    trace_mark(tr, 4);
    if (!barrier(true)) break;
    trace_mark(tr, 5);
    // ---- O projection
    llama_stage_bf16(p.attn, p.nq * p.hd, xs, p.mat[1].KT);
    trace_mark(tr, 6);
    const RowsEpi eo{nullptr, p.proj, H, H, __ldg(&lw->mul[1])};
    ok = consume_range<1, false, FAST>(ring, p.mat[1], wr[1][warp][0], wr[1][warp][1], xs, fx, 1, eo, p.status);
    trace_mark(tr, 14);
    cta_fixup(p.pt[1], &wr[1][0][0], fx, 1, eo);
    if (tr) {
      consumers_sync();
      trace_mark(tr, 15);
    }
    if (!barrier(ok)) break;
    trace_mark(tr, 7);
    // ---- residual + FFN RMSNorm, gate/up with SwiGLU
    load_norm_w(nw, p.norms + static_cast<size_t>(2 * l + 1) * H, H);
    llama_add_bf16(xres, p.proj, H);
    llama_norm_frag(xres, H, nw, p.eps, xs, p.mat[2].KT, red);
    trace_mark(tr, 8);
    const GateUpEpi eg{p.act, p.I, 1, __ldg(&lw->mul[2]), ALV_ACT_SILU};
    ok = consume_range<1, false, FAST>(ring, p.mat[2], wr[2][warp][0], wr[2][warp][1], xs, fx, 1, eg, p.status);
    trace_mark(tr, 9);
    cta_fixup(p.pt[2], &wr[2][0][0], fx, 1, eg);
    if (!barrier(ok)) break;
    trace_mark(tr, 10);
    // ---- down projection; rows shared between CTAs are summed by the next glue
    stage_from_l2(xs, p.act, static_cast<uint32_t>(frag_bytes(p.mat[3].KT, 1)));
    consumers_sync();
    trace_mark(tr, 11);
    const float dmul = __ldg(&lw->mul[3]);
    const StackEpi ed{true, p.act, p.down, p.I, H, 1, dmul, ALV_ACT_SILU, 1.0f};
    ok = consume_range<1, false, FAST>(ring, p.mat[3], wr[3][warp][0], wr[3][warp][1], xs, fxd, 1, ed, p.status);
    trace_mark(tr, 12);
    cta_fixup<true>(p.pt[3], &wr[3][0][0], fxd, 1, ed);
    if (!barrier(ok)) break;
    trace_mark(tr, 13);
    if (l + 1 < p.L) continue;
    // ---- after the last layer
    if (p.logits) {
      load_norm_w(nw, p.norms + static_cast<size_t>(2 * p.L) * H, H);
      add_down(l);
      llama_norm_frag(xres, H, nw, p.eps, xs, p.mat[4].KT, red);
      const RowsEpi el{nullptr, p.logit16, p.V, p.V, p.lm_mul};
      ok = consume_range<1, false, FAST>(ring, p.mat[4], wr[4][warp][0], wr[4][warp][1], xs, fx, 1, el, p.status);
      cta_fixup(p.pt[4], &wr[4][0][0], fx, 1, el);
      if (!barrier(ok)) break;
      // argmax: the first index of the maximum (np.argmax), per CTA over a
      // slice of the vocabulary, then CTA 0 over the CTAs in order.
      const uint32_t v0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.V / gridDim.x);
      const uint32_t v1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * p.V / gridDim.x);
      float best = -INFINITY;
      int bi = 0x7FFFFFFF;
      for (uint32_t i = v0 + threadIdx.x; i < v1; i += NTHR) {
        const float v = bf16_bits_to_f32(__ldcg(p.logit16 + i));
        if (v > best) {
          best = v;
          bi = static_cast<int>(i);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
          best = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        red[warp] = best;
        reinterpret_cast<int*>(red)[32 + warp] = bi;
      }
      consumers_sync();
      if (threadIdx.x == 0) {
        for (int w = 1; w < kConsumerWarps; ++w) {
          const float rv = red[w];
          const int ri = reinterpret_cast<int*>(red)[32 + w];
          if (rv > best || (rv == best && ri < bi)) {
            best = rv;
            bi = ri;
          }
        }
        p.cand_v[blockIdx.x] = best;
        p.cand_i[blockIdx.x] = bi;
      }
      if (!barrier(true)) break;
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        best = -INFINITY;
        bi = 0x7FFFFFFF;
        for (uint32_t c = 0; c < gridDim.x; ++c) {
          const float rv = __ldcg(p.cand_v + c);
          const int ri = __ldcg(p.cand_i + c);
          if (rv > best || (rv == best && ri < bi)) {
            best = rv;
            bi = ri;
          }
        }
        p.pred[pos + 1] = bi;
        if (pos + 1 >= nprompt_s) p.tokens[pos + 1] = bi;
        p.state->pos = pos + 1;
      }
    } else if (blockIdx.x == 0 && threadIdx.x == 0) {
      p.state->pos = pos + 1;
    }
  }
  ring.drain();  // nothing in flight after a complete step; after a failed wait, let the copies land
}

}  // namespace alv
