// Host side of the C ABI, part 2: the Q4 gemv (decode and decode-batch,
// gemv_kernel) and its allocation-free variant.
#include "launch.h"

namespace alv {
namespace {

// Ring stages a gemv CTA requests before it stages x.  Its x loads queue
// behind every byte already requested from HBM, so for a large matrix all
// stages up front (about the whole matrix for decode shapes) make x arrive
// late and stall the stream: one stage per warp keeps HBM busy while x is
// fetched.  Matrices up to kGemvPrimeAllBytes request every stage up front
// (their whole stream is a few microseconds of HBM time, and a warp's second
// group would otherwise wait a full round trip after x is staged).
constexpr size_t kGemvPrimeAllBytes = size_t{16} << 20;

template <int NCOLS, bool SPLIT, bool FAST>
int launch_gemv_t(alv_ctx* ctx, GemvParams p, cudaStream_t st, bool pdl) {
  const size_t other = part_bytes(p.x.ntok) + frag_bytes(p.m.KT, NCOLS);
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: K too large for the shared-memory fragment stage");
  p.first = static_cast<size_t>(p.m.RT) * p.m.KT * kUnitBytes <= kGemvPrimeAllBytes ? p.nst : 1;
  // Row-aligned unless there are too few row tiles to keep the SMs busy: a
  // row tile split between CTAs costs the finishing CTA a fence, an atomic
  // and a round trip at the end, more than the imbalance of whole rows.
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  if (!Partition::fits(p.m.RT, p.m.KT)) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: matrix too large for one launch");
  p.pt = Partition::make(p.m.RT, p.m.KT, nctas, p.m.RT * 4 >= nctas);
  const size_t smem = ring_smem_bytes(p.nst) + other;
  auto k = gemv_kernel<NCOLS, SPLIT, FAST>;
  // gemv_kernel has no grid barrier (split rows are finished by the last CTA
  // to arrive), so a plain launch is enough; one CTA per SM.
  int rc = prepare_kernel(ctx, k, smem);
  if (rc) return rc;
  return launch_ex(ctx, k, dim3(ctx->num_sms), dim3(kThreadsPerCta), smem, st, pdl, p);
}

template <bool FAST>
int launch_gemv_f(alv_ctx* ctx, const GemvParams& p, bool split, uint32_t ncols, cudaStream_t st, bool pdl) {
  if (split) {
    switch (ncols) {
      case 2: return launch_gemv_t<2, true, FAST>(ctx, p, st, pdl);
      case 4: return launch_gemv_t<4, true, FAST>(ctx, p, st, pdl);
      case 8: return launch_gemv_t<8, true, FAST>(ctx, p, st, pdl);
      case 16: return launch_gemv_t<16, true, FAST>(ctx, p, st, pdl);
    }
  } else {
    switch (ncols) {
      case 1: return launch_gemv_t<1, false, FAST>(ctx, p, st, pdl);
      case 2: return launch_gemv_t<2, false, FAST>(ctx, p, st, pdl);
      case 4: return launch_gemv_t<4, false, FAST>(ctx, p, st, pdl);
      case 8: return launch_gemv_t<8, false, FAST>(ctx, p, st, pdl);
      case 16: return launch_gemv_t<16, false, FAST>(ctx, p, st, pdl);
    }
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "unsupported column count");
}


// Shape and argument checks shared by alv_gemv and alv_gemv_noalloc.
int gemv_args(alv_ctx* ctx, int ntok, const void* x, int x_dtype, const char* who, uint32_t* ncols) {
  const bool split = x_dtype == ALV_F32;
  *ncols = pow2_ceil(static_cast<uint32_t>(split ? 2 * ntok : ntok));
  if (ntok < 1 || *ncols > 16)
    return fail(ctx, ALV_ERR_UNSUPPORTED, std::string(who) + ": ntok must be 1..16 (bf16 x) or 1..8 (fp32 x)");
  if (!x_aligned(x, x_dtype))
    return fail(ctx, ALV_ERR_ARG, std::string(who) + ": x must be " + (split ? "8" : "4") + "-byte aligned");
  return ALV_OK;
}

GemvParams gemv_params(Weight* w, int ntok, const void* x, int x_dtype, void* y, int y_dtype) {
  GemvParams p{};
  p.m = w->a.m;
  p.x = XSrc{x, x_dtype == ALV_BF16, ntok, w->a.cols, w->a.cols};
  p.epi = RowsEpi{y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr,
                  y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr, w->a.rows, w->a.rows,
                  w->a.m.scale_mul};
  return p;
}

}  // namespace

int launch_gemv_params(alv_ctx* ctx, const GemvParams& p, bool split, uint32_t ncols, cudaStream_t st, bool pdl) {
  return p.m.fast ? launch_gemv_f<true>(ctx, p, split, ncols, st, pdl)
                  : launch_gemv_f<false>(ctx, p, split, ncols, st, pdl);
}

int do_gemv(alv_ctx* ctx, Weight* w, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
            cudaStream_t st) {
  uint32_t ncols = 0;
  int rc = gemv_args(ctx, ntok, x, x_dtype, "gemv", &ncols);
  if (rc) return rc;
  if (w->a.m.RT > kMaxCounters) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: too many rows");
  const size_t ws_bytes = align_up(ws_floats(ctx, ntok) * 4, 256);
  rc = ensure_scratch(ctx, ws_bytes);
  if (rc) return rc;
  GemvParams p = gemv_params(w, ntok, x, x_dtype, y, y_dtype);
  p.fx = Fixup{reinterpret_cast<float*>(work_ptr(ctx)), counters_ptr(ctx)};
  p.status = status_ptr(ctx);
  p.trace = ctx->trace;
  // Programmatic dependent launch: the kernel streams its weights while the
  // previous kernel in the stream finishes, and reads x / writes y only after
  // griddepcontrol.wait.
  return launch_gemv_params(ctx, p, x_dtype == ALV_F32, ncols, st, true);
}

}  // namespace alv

using namespace alv;

extern "C" int alv_gemv(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
                        void* stream) {
  if (!ctx || !x || !y || !valid_dtype(x_dtype) || !valid_dtype(y_dtype))
    return fail(ctx, ALV_ERR_ARG, "gemv: bad argument");
  Weight* w = get_weight(ctx, h, 1);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "gemv: invalid handle (not a gemv weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  return do_gemv(ctx, w, ntok, x, x_dtype, y, y_dtype, static_cast<cudaStream_t>(stream));
}

// ===========================================================================
// Allocation-free gemv.
//
// Some callers cannot allocate device memory while they run: a decode loop
// whose GPU memory budget is fixed at start-up (every byte is handed to a
// KV cache or another pool), a host runtime that owns the device allocator
// and forbids others from calling cudaMalloc, or code that must not trigger
// the implicit device synchronization a cudaMalloc/cudaFree can cause.
// alv_gemv may grow the context's scratch arena (cudaMalloc) the first time a
// larger problem arrives; alv_gemv_noalloc never does.  Its split-K workspace
// and arrival counters live in the fixed array below, which every GPU that
// loads this library holds until the process exits.
// ===========================================================================
namespace {
constexpr uint32_t kNoAllocMaxTokens = 4;                 // tokens per call
constexpr uint32_t kNoAllocMaxRowTiles = 16384;           // N <= 262,144 rows
constexpr uint32_t kNoAllocMaxSms = 148;                  // CTAs of one launch (one per SM)
// Split-K workspace: two slots of kNoAllocMaxTokens x 16 floats per CTA.
constexpr size_t kNoAllocWsFloats = static_cast<size_t>(kNoAllocMaxSms) * 2 * kNoAllocMaxTokens * 16;
constexpr size_t kNoAllocCounterBytes = static_cast<size_t>(kNoAllocMaxRowTiles) * 4;
constexpr size_t kNoAllocBytes = kNoAllocCounterBytes + kNoAllocWsFloats * 4;  // 141,312 bytes
static_assert(kNoAllocBytes == 141312, "documented size of the static workspace");
}  // namespace

// [counters: kNoAllocMaxRowTiles x u32][workspace: kNoAllocWsFloats x f32]
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: look up the device address of
// the static array (its host-side name is only a stand-in, not a device
// pointer).  The address is cached per device index for the life of the
// process; a cudaDeviceReset would invalidate it.
int noalloc_scratch(alv_ctx* ctx, uint8_t** out) {
  if (ctx->device < 0 || ctx->device >= 64) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[ctx->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(ctx, ALV_ERR_CUDA, std::string("gemv_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_addr[ctx->device] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_addr[ctx->device]);
  return ALV_OK;
}
}  // namespace

extern "C" int alv_gemv_noalloc(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y,
                                int y_dtype, void* stream) {
  if (!ctx || !x || !y || !valid_dtype(x_dtype) || !valid_dtype(y_dtype))
    return fail(ctx, ALV_ERR_ARG, "gemv_noalloc: bad argument");
  Weight* w = get_weight(ctx, h, 1);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "gemv_noalloc: invalid handle (not a gemv weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  if (ntok < 1 || ntok > static_cast<int>(kNoAllocMaxTokens))
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: ntok must be 1.." + std::to_string(kNoAllocMaxTokens));
  uint32_t ncols = 0;
  if ((rc = gemv_args(ctx, ntok, x, x_dtype, "gemv_noalloc", &ncols))) return rc;
  if (w->a.m.RT > kNoAllocMaxRowTiles)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: N must be <= " + std::to_string(kNoAllocMaxRowTiles * 16));
  if (static_cast<uint32_t>(ctx->num_sms) > kNoAllocMaxSms)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: GPU has more than " + std::to_string(kNoAllocMaxSms) +
                                              " SMs; the static workspace covers one CTA per SM up to that");
  uint8_t* base = nullptr;
  if ((rc = noalloc_scratch(ctx, &base))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the arrival counters this
  // call uses must start at zero.
  ALV_CUDA(ctx, cudaMemsetAsync(base, 0, static_cast<size_t>(w->a.m.RT) * 4, st));
  GemvParams p = gemv_params(w, ntok, x, x_dtype, y, y_dtype);
  p.fx = Fixup{reinterpret_cast<float*>(base + kNoAllocCounterBytes), reinterpret_cast<uint32_t*>(base)};
  p.status = status_ptr(ctx);
  return launch_gemv_params(ctx, p, x_dtype == ALV_F32, ncols, st);
}
