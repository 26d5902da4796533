// Batched prefill gemm_q on the 5th-generation tensor cores (tcgen05, TMEM).
//
//   Y[b, n] = sum_k X[b, k] * W[n, k],   W = bf16_rn(q * scale) (Q4, dequantized
//   in shared memory), X bf16, fp32 accumulation in tensor memory.
//
// Replaces the reference's gemm_q NPU design and kernel
// (kernels/gemm_q/gemm_q.py:28-143, kernels/gemm_q/gemm_q.cc:18-54); its CPU
// check is X_f32 @ dequantize_combined(W).astype(f32).T (gemm_q.py:185-188).
//
// One CTA computes a 128-weight-row x NT-token tile, stepping K by 64:
//   warp 8      copies the stage's eight Q4 units (1-D bulk copies) and the X
//               tile (2-D tensor copy, 128-byte swizzle, no multicast)
//   warps 0-7   dequantize one unit each straight into the A buffer in the
//               K-major 128-byte-swizzle layout the tensor core reads
//   warp 9      one thread issues tcgen05.mma (M=128, N=NT, K=16) x 4 and
//               commits to the stage's `empty` barrier
// then warps 0-7 read the accumulator back with tcgen05.ld (warp w owns TMEM
// lanes 32(w%4)..+31, i.e. weight rows, and half of the token columns) and
// store Y.  Every wait gives up
// after 1 s (status bit; the CTA stops consuming, lets its copies land and
// frees its tensor memory before returning).
#pragma once
#include <cuda.h>

#include "stream.cuh"

namespace alv {

constexpr int kTcM = 128;        // weight rows per tile: 8 unit rows of 16
constexpr int kTcStages = 4;
constexpr int kTcDeqWarps = 8;   // one unit (16 weight rows) each per stage
constexpr int kTcThreads = (kTcDeqWarps + 2) * 32;  // + 1 copy warp + 1 MMA warp

struct GemmParams {
  Q4Mat m;           // weight units; m.RT*16 >= N rows, m.KT*64 >= K
  uint32_t N, B;     // logical rows of W and tokens of X
  float* y32;        // (B, N) row-major outputs (either may be null)
  uint16_t* y16;
  uint32_t* status;
};

// Shared-memory descriptor of a K-major operand in the 128-byte-swizzle
// layout (rows of 128 B, 8-row / 1024-B swizzle atoms): start address, leading
// byte offset 16 (unused for this layout), stride byte offset 1024 between
// 8-row groups, descriptor version 1, swizzle mode 2 (128 B).  Field positions
// per the PTX ISA's tcgen05 shared memory descriptor.
__host__ __device__ constexpr uint64_t umma_desc_sw128(uint32_t saddr) {
  return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) | (static_cast<uint64_t>(16 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B (K-major), fp32
// D, M x N.  Bits: [4,6) D format (1 = f32), [7,10) A format (1 = bf16),
// [10,13) B format (1 = bf16), [15] / [16] A / B major (0 = K), [17,23) N>>3,
// [24,29) M>>4.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(uint32_t M, uint32_t N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Byte offset of element (row, k) (k < 64, bf16) in a 128-byte-swizzle K-major
// tile whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
  return row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + ((k & 7) << 1);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared layout (from a 1024-aligned base): per stage [A 16 KB][X NT*128 B][raw 8 units].
template <int NT>
struct TcLayout {
  static constexpr uint32_t kA = kTcM * 128;           // 16,384
  static constexpr uint32_t kX = NT * 128;             // NT tokens x 64 bf16
  static constexpr uint32_t kRaw = 8 * kUnitBytes;     // 4,608
  static constexpr uint32_t kStage = (kA + kX + kRaw + 1023) / 1024 * 1024;
  static constexpr uint32_t kBytes = kTcStages * kStage + 1024;  // + alignment slack
};

template <int NT, bool FAST>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                 const GemmParams p) {
  using Lay = TcLayout<NT>;
  extern __shared__ uint8_t smem_dyn[];
  __shared__ __align__(8) uint64_t full[kTcStages], deq[kTcStages], empty[kTcStages], accb;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile uint32_t failed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_dyn) + 1023u) & ~1023u;
  const uint32_t rt0 = blockIdx.x * 8;
  const uint32_t nrt = p.m.RT - rt0 < 8 ? p.m.RT - rt0 : 8;
  const uint32_t KC = p.m.KT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], kTcDeqWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accb, 1);
    fence_mbar_init();
    failed = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(static_cast<uint32_t>(NT))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == kTcDeqWarps) {
    // ---- copies ----
    if (lane == 0) {
      uint32_t armed = 0;  // stages armed so far
      for (uint32_t kc = 0; kc < KC && !failed; ++kc) {
        const uint32_t s = kc % kTcStages, ph = (kc / kTcStages) & 1;
        if (kc >= kTcStages && !mbar_wait_bounded(&empty[s], ph ^ 1)) {
          atomicOr(p.status, kStatusMbarTimeout);
          failed = 1;
          break;
        }
        const uint32_t st = base + s * Lay::kStage;
        mbar_arrive_expect_tx(&full[s], nrt * kUnitBytes + Lay::kX);
        for (uint32_t i = 0; i < nrt; ++i)
          bulk_g2s_s(st + Lay::kA + Lay::kX + i * kUnitBytes,
                     p.m.units + (static_cast<size_t>(rt0 + i) * KC + kc) * kUnitBytes, kUnitBytes,
                     smem_u32(&full[s]), l2_policy_evict_first());
        tma_load_2d(st + Lay::kA, &xmap, static_cast<int32_t>(kc * 64), static_cast<int32_t>(blockIdx.y * NT),
                    smem_u32(&full[s]));
        armed = kc + 1;
      }
      // Let every armed stage land before the CTA can exit.
      for (uint32_t kc = armed > kTcStages ? armed - kTcStages : 0; kc < armed; ++kc)
        mbar_wait_bounded(&full[kc % kTcStages], (kc / kTcStages) & 1);
    }
  } else if (warp == kTcDeqWarps + 1) {
    // ---- tensor-core issue ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(kTcM, NT);
      for (uint32_t kc = 0; kc < KC && !failed; ++kc) {
        const uint32_t s = kc % kTcStages, ph = (kc / kTcStages) & 1;
        if (!mbar_wait_bounded(&deq[s], ph)) {
          atomicOr(p.status, kStatusMbarTimeout);
          failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t st = base + s * Lay::kStage;
        const uint64_t ad = umma_desc_sw128(st), bd = umma_desc_sw128(st + Lay::kA);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk)  // K = 16 per instruction: +32 B in the swizzle row
          umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kc | kk) != 0);
        umma_commit(smem_u32(&empty[s]));
      }
      umma_commit(smem_u32(&accb));  // completes once every issued MMA is done
    }
  } else {
    // ---- dequant (warp w: unit w of each stage) ----
    const int g = lane >> 2, t4 = lane & 3;
    for (uint32_t kc = 0; kc < KC && !failed; ++kc) {
      const uint32_t s = kc % kTcStages, ph = (kc / kTcStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], ph))) {
        if (lane == 0) atomicOr(p.status, kStatusMbarTimeout);
        failed = 1;
        break;
      }
      const uint32_t st = base + s * Lay::kStage;
      {
        const uint32_t u = warp;
        uint32_t a[4][4];
        if (u < nrt) {
          const uint32_t ua = st + Lay::kA + Lay::kX + u * kUnitBytes;
          const uint4 nib = lds128_at<0>(ua + lane * 16);
          const uint2 sc = lds64_at<0>(ua + kUnitNibBytes + g * 8);
          uint32_t S[2][2], C[2][2];
          S[0][0] = bf2_bcast(sc.x, 0);
          S[1][0] = bf2_bcast(sc.x, 1);
          S[0][1] = bf2_bcast(sc.y, 0);
          S[1][1] = bf2_bcast(sc.y, 1);
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int r = 0; r < 2; ++r) C[b][r] = FAST ? bf2_mul(S[b][r], kNeg8Sub) : 0u;
          const uint32_t words[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int b = j >> 1;
            dequant_word<FAST>(words[j], S[b][0], C[b][0], S[b][1], C[b][1],
                               FAST ? bf2_mul(S[b][1], kPow2m4) : 0u, a[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) a[j][0] = a[j][1] = a[j][2] = a[j][3] = 0u;
        }
        // a[j][0]: (row g, k 16j+2t4), a[j][1]: (row g+8, same k), a[j][2] / a[j][3]: k + 8
        const uint32_t r0 = 16 * u + g, r1 = r0 + 8;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t k0 = 16 * j + 2 * t4;
          st_shared_u32(st + sw128_offset(r0, k0), a[j][0]);
          st_shared_u32(st + sw128_offset(r1, k0), a[j][1]);
          st_shared_u32(st + sw128_offset(r0, k0 + 8), a[j][2]);
          st_shared_u32(st + sw128_offset(r1, k0 + 8), a[j][3]);
        }
      }
      // generic-proxy writes of A -> visible to the tensor core (async proxy)
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq[s]);
    }
    // ---- epilogue: TMEM -> registers -> Y ----
    const bool acc_ok = mbar_wait_bounded(&accb, 0);
    tc_fence_after();
    if (acc_ok && !failed) {
      const uint32_t quad = warp & 3, half = warp >> 2;
      const uint32_t row = blockIdx.x * kTcM + quad * 32 + lane;
      const float sm = p.m.scale_mul;
#pragma unroll 1
      for (uint32_t c = half * (NT / 2); c < (half + 1) * (NT / 2); c += 16) {
        float v[16];
        tmem_ld16(tmem + ((quad * 32) << 16) + c, v);
        if (row < p.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t b = blockIdx.y * NT + c + i;
            if (b < p.B) {
              const size_t o = static_cast<size_t>(b) * p.N + row;
              const float y = v[i] * sm;
              if (p.y32) p.y32[o] = y;
              if (p.y16) p.y16[o] = bf16_bits_rn(y);
            }
          }
        }
      }
    } else if (!acc_ok && lane == 0) {
      atomicOr(p.status, kStatusMbarTimeout);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(static_cast<uint32_t>(NT))
                 : "memory");
  }
}

}  // namespace alv
