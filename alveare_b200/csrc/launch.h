// Kernel launchers shared between translation units (declared here, defined
// next to their kernels): the decode model (decode.cu) drives the gemv and
// FFN kernels with its own workspace.
#pragma once

#include "internal.h"
#include "kernels.cuh"

namespace alv {

// gemv_kernel with ready parameters (split: fp32 x as hi/lo columns;
// ncols: fragment columns, a power of two; pdl: programmatic dependent
// launch).  Defined in gemv.cu.
int launch_gemv_params(alv_ctx* ctx, const GemvParams& p, bool split, uint32_t ncols, cudaStream_t st,
                       bool pdl = false);

// ffn_kernel with ready parameters (nt: tokens rounded up to a power of
// two).  Defined in ffn.cu.
int launch_ffn_params(alv_ctx* ctx, const FfnParams& p, bool split, uint32_t nt, cudaStream_t st);

// tcgen05 prefill gemm on a repacked matrix: Y[b, n] = sum_k X[b, k] W[n, k],
// X bf16 (B, K) row-major, 16-byte aligned; Y (B, N) fp32 and/or bf16 (either
// may be null).  Defined in gemm.cu.
int launch_gemm_mat(alv_ctx* ctx, const Q4Mat& m, uint32_t N, uint32_t K, int B, const uint16_t* x, float* y32,
                    uint16_t* y16, cudaStream_t st);

// Repack a reference-layout (rows, K/32*20) Q4 matrix already on the device
// into a new unit-layout matrix (its own dequant path).  Defined in core.cu.
int repack_rows(alv_ctx* ctx, const uint8_t* src, uint32_t rows, uint32_t K, Mat* out);

// Repack an FFN's gate/up (interleaved) and down matrices for the I-slice
// [i_begin, i_end) (device sources); both share one dequant path.  Defined
// in core.cu.
int repack_ffn(alv_ctx* ctx, const uint8_t* gate, const uint8_t* up, const uint8_t* down, uint32_t H, uint32_t I,
               uint32_t i_begin, uint32_t i_end, Mat* gu, Mat* dn);

}  // namespace alv
