// Load-time kernels of the Q4 format: the GPU quantizer, the scale survey,
// the repack from the reference block layout into the unit layout, and the
// dequantizer.  Used by the weight registry in core.cu only.
#pragma once

#include "common.cuh"
#include "stream.cuh"

namespace alv {

// ===========================================================================
// GPU quantizer: restates tools/convert/gemv_q_convert.py:5-85.
// One thread per (row, 32-block); writes one 20-byte reference block.
// ===========================================================================
__global__ void q4_quantize_kernel(const float* __restrict__ W, int N, int K,
                                   uint8_t* __restrict__ out) {
  const int KB = K / 32;
  const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<size_t>(N) * KB) return;
  const size_t row = t / KB, b = t % KB;
  const float* w = W + row * K + b * 32;
  float v[32];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = w[i];
    mx = fmaxf(mx, fabsf(v[i]));
  }
  float s = __fdiv_rn(mx, 7.0f);       // max_vals / 7.0 in float32 (:24-25)
  if (s == 0.0f) s = 1.0f;             // (:27-28)
  // The 20-byte block is 4-byte aligned: write it as five 32-bit words.
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + row * (static_cast<size_t>(KB) * 20) + b * 20);
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = wd * 4 + j;
      int q0 = static_cast<int>(rintf(__fdiv_rn(v[2 * i], s)));      // half-to-even (:34)
      int q1 = static_cast<int>(rintf(__fdiv_rn(v[2 * i + 1], s)));
      q0 = min(max(q0, -8), 7);                                    // (:37)
      q1 = min(max(q1, -8), 7);
      word |= static_cast<uint32_t>((q0 & 0x0F) | ((q1 & 0x0F) << 4)) << (8 * j);  // (:45-48)
    }
    dst[wd] = word;
  }
  // scales.astype(bfloat16) (:51): round-to-nearest-even of a finite float.
  const uint32_t su = __float_as_uint(s);
  dst[4] = (su + 0x7FFFu + ((su >> 16) & 1u)) >> 16;  // bytes 16-17 scale, 18-19 zero
}

// ===========================================================================
// Load-time repack: reference (N, K/32*20) blocks -> unit layout (stream.cuh).
// ===========================================================================
struct RepackSrc {
  const uint8_t* a;      // primary source rows (gemv matrix, FFN gate, FFN down)
  const uint8_t* b;      // FFN up (interleave8) or null
  uint32_t rows;         // valid source rows in the selected slice
  uint32_t row_off;      // first source row (TP slice of gate/up)
  uint64_t row_bytes;    // source row stride in bytes
  uint32_t blk_off;      // first source 32-block (TP slice of down)
  uint32_t K;            // valid columns (multiple of 32)
  uint32_t interleave8;  // tile rows 0-7 from a, 8-15 from b (same source rows)
  uint32_t RT, KT;       // destination tiles

  // Pointer to block 0 of destination row R, or null for padding rows.
  __device__ __forceinline__ const uint8_t* row_ptr(uint32_t R) const {
    uint32_t sr;
    const uint8_t* buf;
    if (interleave8) {
      const uint32_t rr = R & 15;
      sr = (R >> 4) * 8 + (rr & 7);
      buf = rr < 8 ? a : b;
    } else {
      sr = R;
      buf = a;
    }
    if (sr >= rows) return nullptr;
    return buf + (static_cast<uint64_t>(row_off) + sr) * row_bytes + static_cast<uint64_t>(blk_off) * 20;
  }
};

__device__ __forceinline__ bool block_all_zero(const uint8_t* blk) {
  uint32_t acc = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) acc |= blk[i];
  return acc == 0;
}

__device__ __forceinline__ float block_scale(const uint8_t* blk) {
  return bf16_bits_to_f32(static_cast<uint32_t>(blk[16]) | (static_cast<uint32_t>(blk[17]) << 8));
}

// Scale-exponent survey over the blocks that carry a nonzero q: ilogb range
// and a non-finite flag.  info = {emax, emin, nonfinite}.
__global__ void q4_scale_survey_kernel(RepackSrc s, int* info) {
  const uint32_t KB = s.K / 32;
  const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<uint64_t>(s.RT) * 16 * KB) return;
  const uint32_t R = static_cast<uint32_t>(t / KB), B = static_cast<uint32_t>(t % KB);
  const uint8_t* p = s.row_ptr(R);
  if (!p) return;
  const uint8_t* blk = p + static_cast<uint64_t>(B) * 20;
  if (block_all_zero(blk)) return;
  const float sc = block_scale(blk);
  if (sc == 0.f) return;
  if (!isfinite(sc)) {
    atomicOr(&info[2], 1);
    return;
  }
  const int e = ilogbf(sc);
  atomicMax(&info[0], e);
  atomicMin(&info[1], e);
}

// One thread per destination 32-bit word (144 per unit).
__global__ void q4_repack_kernel(RepackSrc s, int fast, int je, uint32_t* __restrict__ out) {
  const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t nunits = static_cast<uint64_t>(s.RT) * s.KT;
  if (t >= nunits * 144) return;
  const uint64_t unit = t / 144;
  const uint32_t wi = static_cast<uint32_t>(t % 144);
  const uint32_t r = static_cast<uint32_t>(unit / s.KT), kt = static_cast<uint32_t>(unit % s.KT);
  uint32_t word = 0;
  if (wi < 128) {
    const uint32_t L = wi >> 2, j = wi & 3, g = L >> 2, t4 = L & 3;
    const uint32_t c = kt * 64 + j * 16 + 2 * t4;
    uint32_t u[2][4];  // [row g / g+8][col c, c+1, c+8, c+9]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint8_t* p = s.row_ptr(r * 16 + g + 8 * h);
      if (p && c < s.K) {
        const uint8_t* blk = p + static_cast<uint64_t>(c / 32) * 20;
        const uint8_t b0 = blk[(c % 32) / 2], b8 = blk[(c % 32) / 2 + 4];
        u[h][0] = (b0 & 15u) ^ 8u;
        u[h][1] = (b0 >> 4) ^ 8u;
        u[h][2] = (b8 & 15u) ^ 8u;
        u[h][3] = (b8 >> 4) ^ 8u;
      } else {
        u[h][0] = u[h][1] = u[h][2] = u[h][3] = 8u;
      }
    }
    word = u[0][0] | (u[1][0] << 4) | (u[0][2] << 8) | (u[1][2] << 12) | (u[0][1] << 16) |
           (u[1][1] << 20) | (u[0][3] << 24) | (u[1][3] << 28);
  } else {
    const uint32_t sw = wi - 128, g = sw >> 1, h = sw & 1;
    const uint8_t* p = s.row_ptr(r * 16 + g + 8 * h);
    uint32_t half[2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const uint32_t B = kt * 2 + b;
      half[b] = 0;
      if (p && B * 32 < s.K) {
        const uint8_t* blk = p + static_cast<uint64_t>(B) * 20;
        const uint32_t bits = static_cast<uint32_t>(blk[16]) | (static_cast<uint32_t>(blk[17]) << 8);
        if (!fast) {
          half[b] = bits;  // generic path: the scale as stored (exact numpy semantics)
        } else if (!block_all_zero(blk) && bf16_bits_to_f32(bits) != 0.f) {
          // s * 2^(133 - je): exact exponent shift of a bf16 value.
          half[b] = __float_as_uint(ldexpf(bf16_bits_to_f32(bits), 133 - je)) >> 16;
        }
      }
    }
    word = half[0] | (half[1] << 16);
  }
  out[t] = word;
}

// Dequantize a unit-layout matrix to bf16 (rows x K row-major).
__global__ void q4_dequant_kernel(Q4Mat m, uint32_t rows, uint32_t K, uint16_t* __restrict__ out) {
  const uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t nunits = static_cast<uint64_t>(m.RT) * m.KT;
  if (t >= nunits * 32) return;
  const uint64_t unit = t >> 5;
  const int lane = static_cast<int>(t & 31), g = lane >> 2, t4 = lane & 3;
  const uint32_t r = static_cast<uint32_t>(unit / m.KT), kt = static_cast<uint32_t>(unit % m.KT);
  const uint8_t* ub = m.units + unit * kUnitBytes;
  const uint4 nib = *reinterpret_cast<const uint4*>(ub + lane * 16);
  const uint2 sc = *reinterpret_cast<const uint2*>(ub + kUnitNibBytes + g * 8);
  const bool fast = m.fast != 0;
  uint32_t S[2][2], C[2][2];
  S[0][0] = (sc.x & 0xFFFF) * 0x10001u;
  S[1][0] = (sc.x >> 16) * 0x10001u;
  S[0][1] = (sc.y & 0xFFFF) * 0x10001u;
  S[1][1] = (sc.y >> 16) * 0x10001u;
  for (int b = 0; b < 2; ++b)
    for (int h = 0; h < 2; ++h) C[b][h] = fast ? bf2_mul(S[b][h], kNeg8Sub) : 0u;
  const uint32_t words[4] = {nib.x, nib.y, nib.z, nib.w};
  for (int j = 0; j < 4; ++j) {
    const int b = j >> 1;
    uint32_t a[4];
    if (fast)
      dequant_word<true>(words[j], S[b][0], C[b][0], S[b][1], C[b][1], bf2_mul(S[b][1], kPow2m4), a);
    else
      dequant_word<false>(words[j], S[b][0], C[b][0], S[b][1], C[b][1], 0u, a);
    const uint32_t c = kt * 64 + j * 16 + 2 * t4;
    const uint32_t rowv[4] = {r * 16 + g, r * 16 + g + 8, r * 16 + g, r * 16 + g + 8};
    const uint32_t colv[4] = {c, c, c + 8, c + 8};
    for (int i = 0; i < 4; ++i) {
      if (rowv[i] >= rows || colv[i] >= K) continue;
      for (int e = 0; e < 2; ++e) {
        const uint32_t bits = e ? (a[i] >> 16) : (a[i] & 0xFFFF);
        const float v = bf16_bits_to_f32(bits) * m.scale_mul;  // exact power-of-two scaling
        out[static_cast<uint64_t>(rowv[i]) * K + colv[i] + e] = bf16_bits_rn(v);
      }
    }
  }
}

}  // namespace alv
