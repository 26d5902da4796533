// Device kernels of the Llama decode step around the Q4 matmuls: embedding
// lookup + RMSNorm, RoPE + KV-cache append, GQA attention over the bf16 KV
// cache, residual + RMSNorm, and the greedy argmax that feeds the next step.
// Every rounding point follows the reference's CPU path
// (runtime/py/model.py:531-550, 580-630, 821-864, 919-934): fp32 arithmetic
// with bf16 results where the reference casts to bfloat16; sums are
// reduced in a fixed order (deterministic), which differs from numpy's.
// The position and token of a step live in device memory (DecodeState,
// tokens[]), so a whole step can be captured once in a CUDA graph.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace alv {

struct DecodeState {
  int pos;        // position of the token this step consumes
  int n_prompt;   // tokens[0, n_prompt) came from the prompt
  int pad[2];
};

constexpr int kDecodeThreads = 1024;  // one CTA for the vector kernels

// Sum over the CTA (any multiple of 32 threads <= 1024), identical in every
// thread; `red` holds 32 floats.  Fixed order.
__device__ __forceinline__ float cta_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

__device__ __forceinline__ float cta_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = red[0];
  for (int i = 1; i < nw; ++i) s = fmaxf(s, red[i]);
  return s;
}

// Llama RMSNorm of the H values xv (this thread's share: h = tid + i*1024),
// model.py:531-532: var = mean(x*x) in fp32, inv = 1 / sqrt(var + eps),
// out = bf16((x * inv) * w).
template <int PER>
__device__ __forceinline__ void rmsnorm_store(const float (&xv)[PER], int H, const float* __restrict__ w, float eps,
                                              uint16_t* __restrict__ out, float* red) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int h = threadIdx.x + i * kDecodeThreads;
    if (h < H) ss = __fadd_rn(ss, __fmul_rn(xv[i], xv[i]));
  }
  ss = cta_sum(ss, red);
  const float var = __fdiv_rn(ss, static_cast<float>(H));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int h = threadIdx.x + i * kDecodeThreads;
    if (h < H) out[h] = bf16_bits_rn(__fmul_rn(__fmul_rn(xv[i], inv), w[h]));
  }
}

constexpr int kDecodePer = 8;  // H <= 8192

// x = bf16(token_embd[tokens[pos]]) (f16 -> bf16, model.py:926);
// xn = rmsnorm(x) * attn_norm[0].  One CTA per row: with `st` the decode
// step's position (one row); without it rows b = 0.. of a prefill batch at
// positions pos0 + b (x and xn (rows, H)).
__global__ void __launch_bounds__(kDecodeThreads) embed_norm_kernel(const uint16_t* __restrict__ emb,
                                                                    const DecodeState* st, int pos0, const int* tokens,
                                                                    int H, const float* __restrict__ w, float eps,
                                                                    uint16_t* __restrict__ x,
                                                                    uint16_t* __restrict__ xn) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  x += static_cast<size_t>(blockIdx.x) * H;
  xn += static_cast<size_t>(blockIdx.x) * H;
  const int tok = tokens[st ? st->pos : pos0 + static_cast<int>(blockIdx.x)];
  const uint16_t* row = emb + static_cast<size_t>(tok) * H;
  float xv[kDecodePer];
#pragma unroll
  for (int i = 0; i < kDecodePer; ++i) {
    const int h = threadIdx.x + i * kDecodeThreads;
    xv[i] = 0.f;
    if (h < H) {
      const float v = bf16_round(__half2float(__ushort_as_half(row[h])));
      x[h] = bf16_bits_rn(v);
      xv[i] = v;
    }
  }
  rmsnorm_store(xv, H, w, eps, xn, red);
}

// x = bf16(x + add) (model.py:859, 864); xn = rmsnorm(x) * w.  One CTA per
// row (rows of H values).
__global__ void __launch_bounds__(kDecodeThreads) residual_norm_kernel(uint16_t* __restrict__ x,
                                                                       const uint16_t* __restrict__ add, int H,
                                                                       const float* __restrict__ w, float eps,
                                                                       uint16_t* __restrict__ xn) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  x += static_cast<size_t>(blockIdx.x) * H;
  add += static_cast<size_t>(blockIdx.x) * H;
  xn += static_cast<size_t>(blockIdx.x) * H;
  float xv[kDecodePer];
#pragma unroll
  for (int i = 0; i < kDecodePer; ++i) {
    const int h = threadIdx.x + i * kDecodeThreads;
    xv[i] = 0.f;
    if (h < H) {
      const float v = bf16_round(__fadd_rn(bf16_bits_to_f32(x[h]), bf16_bits_to_f32(add[h])));
      x[h] = bf16_bits_rn(v);
      xv[i] = v;
    }
  }
  rmsnorm_store(xv, H, w, eps, xn, red);
}

// RoPE of q and k and the KV-cache append (model.py:534-550, 838-843):
// per head, with c = cos[i], s = sin[i] of the bf16 table row of `pos`,
//   y[i] = x[i] c - x[i+half] s,   y[i+half] = x[i+half] c + x[i] s
// (products and the sum rounded in fp32, then bf16).  qkv = [q | k | v].
struct RopeParams {
  const uint16_t* qkv;
  const uint16_t* table;   // [max_seq][2*hd]: cos(hd) then sin(hd)
  const DecodeState* st;   // the decode step's position; null: prefill rows at pos0 + blockIdx.x
  int pos0;
  uint16_t* kcache;        // this layer: [nkv][max_seq][hd]
  uint16_t* vcache;
  uint16_t* q_out;         // [nq*hd]
  int nq, nkv, hd, max_seq;
};

__global__ void __launch_bounds__(kDecodeThreads) rope_cache_kernel(RopeParams p) {
  pdl_wait();
  pdl_trigger();
  const int pos = p.st ? p.st->pos : p.pos0 + static_cast<int>(blockIdx.x);
  p.qkv += static_cast<size_t>(blockIdx.x) * (p.nq + 2 * p.nkv) * p.hd;
  p.q_out += static_cast<size_t>(blockIdx.x) * p.nq * p.hd;
  const int half = p.hd / 2;
  const uint16_t* cs = p.table + static_cast<size_t>(pos) * 2 * p.hd;
  const int nq_pairs = p.nq * half, nk_pairs = p.nkv * half;
  for (int e = threadIdx.x; e < nq_pairs + nk_pairs; e += blockDim.x) {
    const bool is_q = e < nq_pairs;
    const int ee = is_q ? e : e - nq_pairs;
    const int h = ee / half, i = ee - h * half;
    const uint16_t* src = p.qkv + (is_q ? 0 : p.nq * p.hd) + h * p.hd;
    const float x1 = bf16_bits_to_f32(src[i]), x2 = bf16_bits_to_f32(src[i + half]);
    const float c = bf16_bits_to_f32(cs[i]), s = bf16_bits_to_f32(cs[p.hd + i]);
    const uint16_t y1 = bf16_bits_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    const uint16_t y2 = bf16_bits_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    if (is_q) {
      p.q_out[h * p.hd + i] = y1;
      p.q_out[h * p.hd + i + half] = y2;
    } else {
      uint16_t* dst = p.kcache + (static_cast<size_t>(h) * p.max_seq + pos) * p.hd;
      dst[i] = y1;
      dst[i + half] = y2;
    }
  }
  const uint16_t* v = p.qkv + (p.nq + p.nkv) * p.hd;
  for (int e = threadIdx.x; e < p.nkv * p.hd; e += blockDim.x) {
    const int h = e / p.hd, d = e - h * p.hd;
    p.vcache[(static_cast<size_t>(h) * p.max_seq + pos) * p.hd + d] = v[e];
  }
}

// k_j . q for one cached key row (hd bf16 values), fmaf in d order.  The
// row's 16-byte loads are issued in batches of 8 before the products, so a
// row costs one memory round trip per 64 values, not one per 8.
__device__ __forceinline__ float attn_dot(const uint16_t* kr, const float* qs, int hd) {
  float dot = 0.f;
  for (int d0 = 0; d0 < hd; d0 += 64) {
    uint4 kw[8];
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (d0 + c * 8 < hd) kw[c] = *reinterpret_cast<const uint4*>(kr + d0 + c * 8);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (d0 + c * 8 >= hd) break;
      const uint32_t ws[4] = {kw[c].x, kw[c].y, kw[c].z, kw[c].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        dot = fmaf(bf16_bits_to_f32(ws[t] & 0xFFFFu), qs[d0 + c * 8 + 2 * t], dot);
        dot = fmaf(bf16_bits_to_f32(ws[t] >> 16), qs[d0 + c * 8 + 2 * t + 1], dot);
      }
    }
  }
  return dot;
}

// sum over j = g, g + G, ... < seq of p_j v_j[d], fmaf in j order; the
// cached values are loaded 8 at a time ahead of the products.  j == own
// (if own >= 0) takes v_own instead of the cache.
__device__ __forceinline__ float attn_pv(const float* sc, const uint16_t* vb, int hd, int d, int g, int G, int seq,
                                         int own, float v_own) {
  float acc = 0.f;
  for (int j0 = g; j0 < seq; j0 += 8 * G) {
    float vv[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int j = j0 + b * G;
      vv[b] = j < seq ? (j == own ? v_own : bf16_bits_to_f32(vb[static_cast<size_t>(j) * hd + d])) : 0.f;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int j = j0 + b * G;
      if (j < seq) acc = fmaf(sc[j], vv[b], acc);
    }
  }
  return acc;
}

// GQA attention of one query head per CTA over positions [0, pos]
// (model.py:580-630): s_j = (k_j . q) * scale (fp32 dot, the scale applied
// in double like numpy's float64 scalar), softmax with exp(s_j - max)
// evaluated correctly rounded, p_j = e_j / sum, out = sum_j p_j v_j -> bf16.
constexpr int kAttnThreads = 256;
struct AttnParams {
  const uint16_t* q;       // [nq*hd] bf16 (after RoPE)
  const uint16_t* kcache;  // this layer
  const uint16_t* vcache;
  const DecodeState* st;   // the decode step's position; null: prefill rows at pos0 + blockIdx.y
  int pos0;
  uint16_t* out;           // [nq*hd] bf16
  int nq, nkv, hd, max_seq;
  double scale;
};

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnParams p) {
  extern __shared__ float sm[];          // [hd] q, [max_seq] scores, [blockDim / hd][hd] partial outputs
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int head = blockIdx.x, kvh = head / (p.nq / p.nkv);
  const int seq = (p.st ? p.st->pos : p.pos0 + static_cast<int>(blockIdx.y)) + 1;  // causal: up to the row's position
  p.q += static_cast<size_t>(blockIdx.y) * p.nq * p.hd;
  p.out += static_cast<size_t>(blockIdx.y) * p.nq * p.hd;
  float* qs = sm;
  float* sc = sm + p.hd;
  float* part = sc + p.max_seq;
  for (int d = threadIdx.x; d < p.hd; d += blockDim.x) qs[d] = bf16_bits_to_f32(p.q[head * p.hd + d]);
  __syncthreads();
  const uint16_t* kb = p.kcache + static_cast<size_t>(kvh) * p.max_seq * p.hd;
  const uint16_t* vb = p.vcache + static_cast<size_t>(kvh) * p.max_seq * p.hd;
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < seq; j += blockDim.x) {
    const float dot = attn_dot(kb + static_cast<size_t>(j) * p.hd, qs, p.hd);
    const float s = static_cast<float>(static_cast<double>(dot) * p.scale);
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = cta_max(mx, red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < seq; j += blockDim.x) {
    const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(sc[j], mx))));
    sc[j] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = cta_sum(sum, red);
  for (int j = threadIdx.x; j < seq; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], sum);
  __syncthreads();
  // out[d] = sum_j p_j v_j[d]: thread (g, d) sums j = g, g+G, ...
  const int G = blockDim.x / p.hd;
  const int g = threadIdx.x / p.hd, d = threadIdx.x - g * p.hd;
  if (g < G) part[g * p.hd + d] = attn_pv(sc, vb, p.hd, d, g, G, seq, -1, 0.f);
  __syncthreads();
  for (int e = threadIdx.x; e < p.hd; e += blockDim.x) {
    float o = 0.f;
    for (int gg = 0; gg < G; ++gg) o = __fadd_rn(o, part[gg * p.hd + e]);
    p.out[head * p.hd + e] = bf16_bits_rn(o);
  }
}

// End of a step: with logits, pred[pos+1] = argmax (the first index of the
// maximum, as np.argmax), which also becomes tokens[pos+1] unless that
// position holds a prompt token (then the prediction is only recorded: a
// teacher-forced run); then pos += 1 (the next step's position).
__global__ void __launch_bounds__(kDecodeThreads) argmax_advance_kernel(const uint16_t* __restrict__ logits, int V,
                                                                        DecodeState* st, int* tokens, int* pred) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  pdl_wait();
  pdl_trigger();
  const int pos = st->pos;
  if (logits) {
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = bf16_bits_to_f32(logits[i]);
      if (v > best) {  // ascending i per thread: keeps the first index of a tie
        best = v;
        bi = i;
      }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
      rv[warp] = best;
      ri[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
        if (rv[w] > best || (rv[w] == best && ri[w] < bi)) {
          best = rv[w];
          bi = ri[w];
        }
      pred[pos + 1] = bi;
      if (pos + 1 >= st->n_prompt) tokens[pos + 1] = bi;
    }
  }
  if (threadIdx.x == 0) st->pos = pos + 1;
}

}  // namespace alv
