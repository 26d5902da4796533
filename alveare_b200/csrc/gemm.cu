// Host side of the C ABI, part 5: the batched prefill gemm_q on the tcgen05
// tensor cores (gemm_tc_kernel).
#include <cuda.h>

#include "gemm_tc.cuh"
#include "launch.h"

using namespace alv;

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up once through the runtime.
int tensor_map_encoder(alv_ctx* ctx, EncodeTiledFn* out) {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    ALV_CUDA(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !f)
      return fail(ctx, ALV_ERR_CUDA, "gemm: cuTensorMapEncodeTiled is not available");
    fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  *out = fn;
  return ALV_OK;
}

template <int NT, bool FAST>
int launch_gemm_t(alv_ctx* ctx, const GemmParams& p, const CUtensorMap& map, cudaStream_t st) {
  const size_t smem = TcLayout<NT>::kBytes;
  auto k = gemm_tc_kernel<NT, FAST>;
  int rc = prepare_kernel(ctx, k, smem);
  if (rc) return rc;
  const dim3 grid((p.m.RT + 7) / 8, (p.B + NT - 1) / NT);
  k<<<grid, kTcThreads, smem, st>>>(map, p);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

template <bool FAST>
int launch_gemm_f(alv_ctx* ctx, const GemmParams& p, const CUtensorMap& map, uint32_t nt, cudaStream_t st) {
  switch (nt) {
    case 64: return launch_gemm_t<64, FAST>(ctx, p, map, st);
    case 128: return launch_gemm_t<128, FAST>(ctx, p, map, st);
    case 256: return launch_gemm_t<256, FAST>(ctx, p, map, st);
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "gemm: unsupported token tile");
}

}  // namespace

// The tcgen05 prefill gemm on a repacked matrix: Y[b, n] = sum_k X[b, k] W[n, k]
// for b < B, X bf16 (B, K) row-major and 16-byte aligned, Y (B, N) fp32 and/or bf16.
int alv::launch_gemm_mat(alv_ctx* ctx, const Q4Mat& m, uint32_t N, uint32_t K, int B, const uint16_t* x,
                         float* y32, uint16_t* y16, cudaStream_t st) {
  if (B < 1 || !x || (!y32 && !y16)) return fail(ctx, ALV_ERR_ARG, "gemm: bad argument");
  if (reinterpret_cast<uintptr_t>(x) & 15) return fail(ctx, ALV_ERR_ARG, "gemm: x must be 16-byte aligned");
  EncodeTiledFn enc = nullptr;
  int rc = tensor_map_encoder(ctx, &enc);
  if (rc) return rc;
  const uint32_t nt = B >= 256 ? 256 : (B > 64 ? 128 : 64);
  CUtensorMap map;
  const cuuint64_t dims[2] = {K, static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {64, nt};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(ctx, ALV_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (" + std::to_string(cr) + ")");
  GemmParams p{};
  p.m = m;
  p.N = N;
  p.B = static_cast<uint32_t>(B);
  p.y32 = y32;
  p.y16 = y16;
  p.status = status_ptr(ctx);
  return p.m.fast ? launch_gemm_f<true>(ctx, p, map, nt, st) : launch_gemm_f<false>(ctx, p, map, nt, st);
}

extern "C" int alv_gemm(alv_ctx* ctx, alv_handle h, int B, const uint16_t* x, void* y, int y_dtype, void* stream) {
  if (!ctx || !x || !y || B < 1 || !valid_dtype(y_dtype)) return fail(ctx, ALV_ERR_ARG, "gemm: bad argument");
  Weight* w = get_weight(ctx, h, 1);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "gemm: invalid handle (not a gemv weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  return launch_gemm_mat(ctx, w->a.m, w->a.rows, w->a.cols, B, x, y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr,
                         y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr, static_cast<cudaStream_t>(stream));
}
