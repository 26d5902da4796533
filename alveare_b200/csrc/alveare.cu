// Host side of the C ABI declared in include/alveare_b200.h: context, scratch
// arena, weight registry (load-time repack), kernel launchers.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "../../include/alveare_b200.h"
#include "gemm_tc.cuh"
#include "kernels.cuh"

using namespace alv;

namespace {

constexpr int kVersion = 100;             // 0.1.0
constexpr uint32_t kMaxCounters = 65536;  // row tiles per matrix (N <= 1,048,576)
constexpr size_t kHeaderBytes = 1024;     // status word + grid barrier
constexpr size_t kMaxSmem = 227 * 1024;

struct Mat {
  uint8_t* dev = nullptr;
  Q4Mat m{};
  uint32_t rows = 0, cols = 0;
  size_t bytes = 0;
};

struct Weight {
  int kind = 0;  // 1 gemv, 2 ffn, 3 ffn stack
  Mat a, b;      // gemv: a; ffn: a = gate/up interleaved, b = down; stack: shapes of every layer
  uint32_t H = 0, I = 0, i_begin = 0, i_end = 0;
  int act = 0;
  // kind 3: the layers (FFN weights), their device descriptors and the
  // stack's own workspace (sync words, split-K partials, down, act)
  std::vector<alv_handle> layers;
  LayerW* layers_dev = nullptr;
  uint8_t* ws = nullptr;
  size_t ws_bytes = 0;
  // kind 3, tensor parallel: this rank's exchange region (cudaMalloc, shared
  // with the peers by CUDA IPC) and every rank's region as mapped here
  int world = 1, rank = 0;
  bool connected = false, broken = false;
  uint8_t* xlocal = nullptr;
  uint32_t xslot = 0, xws_off = 0;
  uint8_t* xr[kMaxRanks] = {};
  unsigned char blob[ALV_IPC_BLOB_BYTES] = {};
};

}  // namespace

struct alv_ctx {
  int device = 0;
  int num_sms = 0;
  std::string err;
  std::vector<std::unique_ptr<Weight>> weights;  // handle = index + 1
  uint8_t* sync = nullptr;                       // [header: status, grid barrier][counters], fixed
  uint8_t* scratch = nullptr;                    // work area (split-K partials, act)
  size_t scratch_bytes = 0;
  std::vector<void*> retired;                    // outgrown buffers, freed with the context
  void* io = nullptr;                            // device staging for host-buffer calls
  size_t io_bytes = 0;
  cudaStream_t stream = nullptr;                 // internal stream (loads, host calls)
  unsigned long long* trace = nullptr;           // optional FFN phase timestamps
};

namespace {

int fail(alv_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return code;
}

#define ALV_CUDA(ctx, call)                                                              \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail((ctx), ALV_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

int set_device(alv_ctx* ctx) {
  ALV_CUDA(ctx, cudaSetDevice(ctx->device));
  return ALV_OK;
}

constexpr size_t kSyncBytes = kHeaderBytes + static_cast<size_t>(kMaxCounters) * 4;
uint32_t* status_ptr(alv_ctx* ctx) { return reinterpret_cast<uint32_t*>(ctx->sync); }
GridBar* bar_ptr(alv_ctx* ctx) { return reinterpret_cast<GridBar*>(ctx->sync + 256); }
uint32_t* counters_ptr(alv_ctx* ctx) { return reinterpret_cast<uint32_t*>(ctx->sync + kHeaderBytes); }
uint8_t* work_ptr(alv_ctx* ctx) { return ctx->scratch; }

// The sync block (status word, grid barrier, arrival counters; counters are
// zero between launches) is allocated once per context.  The work area is
// re-laid out per call and grows on demand; an outgrown area is kept until
// the context is destroyed, so launches captured in a CUDA graph earlier
// still point at live memory.
int ensure_scratch(alv_ctx* ctx, size_t work_bytes) {
  if (!ctx->sync) {
    ALV_CUDA(ctx, cudaMalloc(&ctx->sync, kSyncBytes));
    ALV_CUDA(ctx, cudaMemset(ctx->sync, 0, kSyncBytes));
  }
  if (ctx->scratch && ctx->scratch_bytes >= work_bytes) return ALV_OK;
  ALV_CUDA(ctx, cudaDeviceSynchronize());
  if (ctx->scratch) ctx->retired.push_back(ctx->scratch);
  ctx->scratch = nullptr;
  const size_t bytes = std::max(work_bytes, static_cast<size_t>(8) << 20);
  ALV_CUDA(ctx, cudaMalloc(&ctx->scratch, bytes));
  ALV_CUDA(ctx, cudaMemset(ctx->scratch, 0, bytes));
  ctx->scratch_bytes = bytes;
  return ALV_OK;
}

Weight* get_weight(alv_ctx* ctx, alv_handle h, int kind) {
  if (h == 0 || h > ctx->weights.size()) return nullptr;
  Weight* w = ctx->weights[h - 1].get();
  if (!w || (kind && w->kind != kind)) return nullptr;
  return w;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

uint32_t pow2_ceil(uint32_t v) {
  uint32_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

// Survey the scales of the blocks that will be repacked: the fast dequant
// path needs every nonzero scale finite and the scale exponents within a
// window of 120 binades (je = emax + 6 <= emin + 126).
struct Survey {
  int fast = 0;
  int je = 0;
};

int survey_mat(alv_ctx* ctx, const RepackSrc& s, Survey* out) {
  int* info = nullptr;
  ALV_CUDA(ctx, cudaMalloc(&info, 3 * sizeof(int)));
  const int init[3] = {INT_MIN, INT_MAX, 0};
  ALV_CUDA(ctx, cudaMemcpyAsync(info, init, sizeof(init), cudaMemcpyHostToDevice, ctx->stream));
  const uint64_t nblk = static_cast<uint64_t>(s.RT) * 16 * (s.K / 32);
  if (nblk) {
    q4_scale_survey_kernel<<<static_cast<unsigned>((nblk + 255) / 256), 256, 0, ctx->stream>>>(s, info);
    ALV_CUDA(ctx, cudaGetLastError());
  }
  int h[3];
  ALV_CUDA(ctx, cudaMemcpyAsync(h, info, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
  ALV_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  ALV_CUDA(ctx, cudaFree(info));
  Survey r;
  if (!h[2]) {
    if (h[0] == INT_MIN) {
      r.fast = 1;  // no block with a nonzero q: every stored scale is 0
    } else {
      r.je = h[0] + 6;
      r.fast = (r.je <= h[1] + 126) && r.je >= -126 && r.je <= 127;
      if (!r.fast) r.je = 0;
    }
  }
  *out = r;
  return ALV_OK;
}

// Repack into a new device buffer with the chosen dequant path.
int repack_mat(alv_ctx* ctx, const RepackSrc& s, const Survey& sv, uint32_t rows, uint32_t cols, Mat* out) {
  const uint64_t nunits = static_cast<uint64_t>(s.RT) * s.KT;
  Mat m;
  m.bytes = nunits * kUnitBytes;
  ALV_CUDA(ctx, cudaMalloc(&m.dev, std::max<size_t>(m.bytes, 16)));
  if (nunits) {
    const uint64_t nwords = nunits * 144;
    q4_repack_kernel<<<static_cast<unsigned>((nwords + 255) / 256), 256, 0, ctx->stream>>>(
        s, sv.fast, sv.je, reinterpret_cast<uint32_t*>(m.dev));
    ALV_CUDA(ctx, cudaGetLastError());
  }
  ALV_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  m.m.units = m.dev;
  m.m.RT = s.RT;
  m.m.KT = s.KT;
  m.m.fast = static_cast<uint32_t>(sv.fast);
  m.m.scale_mul = sv.fast ? ldexpf(1.0f, sv.je) : 1.0f;
  m.rows = rows;
  m.cols = cols;
  *out = m;
  return ALV_OK;
}

int build_mat(alv_ctx* ctx, const RepackSrc& s, uint32_t rows, uint32_t cols, Mat* out) {
  Survey sv;
  int rc = survey_mat(ctx, s, &sv);
  if (rc) return rc;
  return repack_mat(ctx, s, sv, rows, cols, out);
}

// Copy a host source buffer to the device (or use the device pointer).
int stage_source(alv_ctx* ctx, const void* src, size_t bytes, int on_device, const uint8_t** dev,
                 uint8_t** owned) {
  *owned = nullptr;
  if (on_device) {
    *dev = static_cast<const uint8_t*>(src);
    return ALV_OK;
  }
  uint8_t* d = nullptr;
  ALV_CUDA(ctx, cudaMalloc(&d, std::max<size_t>(bytes, 16)));
  ALV_CUDA(ctx, cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice));
  *dev = d;
  *owned = d;
  return ALV_OK;
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
// Raise the kernel's dynamic shared-memory limit once per (kernel, device) to
// the maximum, so launches need no per-call attribute changes.
// (The limit covers static + dynamic shared memory; kernels with static
// __shared__ arrays get kMaxSmem minus those bytes.)
template <class K>
int prepare_kernel(alv_ctx* ctx, K kernel, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> max_dyn;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), ctx->device);
  std::lock_guard<std::mutex> lock(mu);
  auto it = max_dyn.find(key);
  if (it == max_dyn.end()) {
    cudaFuncAttributes fa;
    ALV_CUDA(ctx, cudaFuncGetAttributes(&fa, kernel));
    const size_t dyn = fa.sharedSizeBytes < kMaxSmem ? kMaxSmem - fa.sharedSizeBytes : 0;
    ALV_CUDA(ctx, cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn)));
    it = max_dyn.emplace(key, dyn).first;
  }
  if (smem > it->second)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "problem needs " + std::to_string(smem) +
                                              " B of dynamic shared memory (max " + std::to_string(it->second) + ")");
  return ALV_OK;
}

// Ring stages per warp that fit beside `other` bytes of dynamic shared memory
// (at most kMaxStages), leaving room for the kernels' static shared memory
// (per-warp work lists and copy cursors, < kStaticSmemReserve bytes).
constexpr size_t kStaticSmemReserve = 2048;
constexpr uint32_t kMaxStages = 24 / kUnitsPerStage;
uint32_t ring_stages(size_t other) {
  for (uint32_t nst = kMaxStages; nst >= 1; --nst)
    if (ring_smem_bytes(nst) + other + kStaticSmemReserve <= kMaxSmem) return nst;
  return 0;
}

template <int NCOLS, bool SPLIT, bool FAST>
int launch_gemv_t(alv_ctx* ctx, GemvParams p, cudaStream_t st) {
  const size_t other = part_bytes(p.x.ntok) + frag_bytes(p.m.KT, NCOLS);
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: K too large for the shared-memory fragment stage");
  const size_t smem = ring_smem_bytes(p.nst) + other;
  auto k = gemv_kernel<NCOLS, SPLIT, FAST>;
  int rc = prepare_kernel(ctx, k, smem);
  if (rc) return rc;
  k<<<ctx->num_sms, kThreadsPerCta, smem, st>>>(p);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

template <bool FAST>
int launch_gemv_f(alv_ctx* ctx, const GemvParams& p, bool split, uint32_t ncols, cudaStream_t st) {
  if (split) {
    switch (ncols) {
      case 2: return launch_gemv_t<2, true, FAST>(ctx, p, st);
      case 4: return launch_gemv_t<4, true, FAST>(ctx, p, st);
      case 8: return launch_gemv_t<8, true, FAST>(ctx, p, st);
      case 16: return launch_gemv_t<16, true, FAST>(ctx, p, st);
    }
  } else {
    switch (ncols) {
      case 1: return launch_gemv_t<1, false, FAST>(ctx, p, st);
      case 2: return launch_gemv_t<2, false, FAST>(ctx, p, st);
      case 4: return launch_gemv_t<4, false, FAST>(ctx, p, st);
      case 8: return launch_gemv_t<8, false, FAST>(ctx, p, st);
      case 16: return launch_gemv_t<16, false, FAST>(ctx, p, st);
    }
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "unsupported column count");
}

int launch_gemv(alv_ctx* ctx, const GemvParams& p, bool split, uint32_t ncols, cudaStream_t st) {
  return p.m.fast ? launch_gemv_f<true>(ctx, p, split, ncols, st) : launch_gemv_f<false>(ctx, p, split, ncols, st);
}

template <int NT, bool SPLIT, bool FAST>
int launch_ffn_t(alv_ctx* ctx, FfnParams p, cudaStream_t st) {
  constexpr int NCA = SPLIT ? 2 * NT : NT;
  size_t other = part_bytes(p.ntok) + std::max(frag_bytes(p.gu.KT, NCA), frag_bytes(p.dn.KT, NT)) + 32 * sizeof(float);
  if (p.glue) {
    const size_t v = static_cast<size_t>(p.ntok) * p.H;
    other += v * sizeof(float);                                  // tmp
    if (p.glue_tma) other += v * 2 + (p.down_in ? v * 4 : 0);    // raw inputs
  }
  other += 16;                                                   // input mbarrier
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: H or I too large for the shared-memory fragment stage");
  const size_t smem = ring_smem_bytes(p.nst) + other;
  auto k = ffn_kernel<NT, SPLIT, FAST>;
  int rc = prepare_kernel(ctx, k, smem);
  if (rc) return rc;
  k<<<ctx->num_sms, kThreadsPerCta, smem, st>>>(p);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

template <bool FAST>
int launch_ffn_f(alv_ctx* ctx, const FfnParams& p, bool split, uint32_t nt, cudaStream_t st) {
  if (split) {
    switch (nt) {
      case 1: return launch_ffn_t<1, true, FAST>(ctx, p, st);
      case 2: return launch_ffn_t<2, true, FAST>(ctx, p, st);
      case 4: return launch_ffn_t<4, true, FAST>(ctx, p, st);
      case 8: return launch_ffn_t<8, true, FAST>(ctx, p, st);
    }
  } else {
    switch (nt) {
      case 1: return launch_ffn_t<1, false, FAST>(ctx, p, st);
      case 2: return launch_ffn_t<2, false, FAST>(ctx, p, st);
      case 4: return launch_ffn_t<4, false, FAST>(ctx, p, st);
      case 8: return launch_ffn_t<8, false, FAST>(ctx, p, st);
    }
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "unsupported token count");
}

// Both FFN matrices were repacked for the same dequant path.
int launch_ffn(alv_ctx* ctx, const FfnParams& p, bool split, uint32_t nt, cudaStream_t st) {
  return p.gu.fast ? launch_ffn_f<true>(ctx, p, split, nt, st) : launch_ffn_f<false>(ctx, p, split, nt, st);
}

// Split-K CTA partials: two slots of ntok x 16 floats per CTA.
size_t ws_floats(alv_ctx* ctx, const Q4Mat&, int ntok) {
  return static_cast<size_t>(ctx->num_sms) * 2 * ntok * 16;
}

bool valid_dtype(int d) { return d == ALV_F32 || d == ALV_BF16; }

int do_gemv(alv_ctx* ctx, Weight* w, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
            cudaStream_t st) {
  const bool split = x_dtype == ALV_F32;
  const uint32_t ncols = pow2_ceil(static_cast<uint32_t>(split ? 2 * ntok : ntok));
  if (ntok < 1 || ncols > 16)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: ntok must be 1..16 (bf16 x) or 1..8 (fp32 x)");
  if (w->a.m.RT > kMaxCounters) return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv: too many rows");
  const size_t ws_bytes = align_up(ws_floats(ctx, w->a.m, ntok) * 4, 256);
  int rc = ensure_scratch(ctx, ws_bytes);
  if (rc) return rc;
  GemvParams p{};
  p.m = w->a.m;
  p.x = XSrc{x, x_dtype == ALV_BF16, ntok, w->a.cols, w->a.cols};
  p.epi = RowsEpi{y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr,
                  y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr, w->a.rows, w->a.rows,
                  w->a.m.scale_mul};
  p.fx = Fixup{reinterpret_cast<float*>(work_ptr(ctx)), counters_ptr(ctx)};
  p.status = status_ptr(ctx);
  return launch_gemv(ctx, p, split, ncols, st);
}

struct FfnIo {
  const void* x = nullptr;
  int x_dtype = ALV_F32;
  int glue = 0;
  const uint16_t* x_in = nullptr;
  const float* down_in = nullptr;
  uint16_t* x_out = nullptr;
  float* y32 = nullptr;
  uint16_t* y16 = nullptr;
};

int do_ffn(alv_ctx* ctx, Weight* w, int ntok, const FfnIo& io, cudaStream_t st) {
  if (ntok < 1 || ntok > 8) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: ntok must be 1..8");
  if (io.glue && w->H > 32u * kConsumerWarps * kGlueRegs)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_layer: H must be <= " + std::to_string(32u * kConsumerWarps * kGlueRegs));
  const bool split = !io.glue && io.x_dtype == ALV_F32;
  const uint32_t nt = pow2_ceil(static_cast<uint32_t>(ntok));
  if (w->a.m.RT + w->b.m.RT > kMaxCounters) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: too large");
  const size_t wsA = align_up(ws_floats(ctx, w->a.m, ntok) * 4, 256);
  const size_t wsB = align_up(ws_floats(ctx, w->b.m, ntok) * 4, 256);
  const size_t actb = align_up(frag_bytes(w->b.m.KT, static_cast<int>(nt)), 256);
  int rc = ensure_scratch(ctx, wsA + wsB + actb);
  if (rc) return rc;
  uint8_t* wk = work_ptr(ctx);
  FfnParams p{};
  p.gu = w->a.m;
  p.dn = w->b.m;
  p.H = w->H;
  p.I = w->i_end - w->i_begin;
  p.fn = w->act;
  p.ntok = ntok;
  p.x = XSrc{io.x, io.x_dtype == ALV_BF16, ntok, w->H, w->H};
  p.glue = io.glue;
  p.x_in = io.x_in;
  p.down_in = io.down_in;
  p.x_out = io.x_out;
  p.eps = 1e-6f;
  p.out = RowsEpi{io.y32, io.y16, w->H, w->H, w->b.m.scale_mul};
  p.act = wk + wsA + wsB;
  p.fxA = Fixup{reinterpret_cast<float*>(wk), counters_ptr(ctx)};
  p.fxB = Fixup{reinterpret_cast<float*>(wk + wsA), counters_ptr(ctx) + w->a.m.RT};
  p.bar = bar_ptr(ctx);
  p.status = status_ptr(ctx);
  p.trace = ctx->trace;
  auto aligned16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  p.glue_tma = io.glue && aligned16(io.x_in) && (!io.down_in || aligned16(io.down_in));
  return launch_ffn(ctx, p, split, nt, st);
}

int io_buffers(alv_ctx* ctx, size_t bytes) {
  if (ctx->io && ctx->io_bytes >= bytes) return ALV_OK;
  if (ctx->io) ctx->retired.push_back(ctx->io);
  ctx->io = nullptr;
  ALV_CUDA(ctx, cudaMalloc(&ctx->io, bytes));
  ctx->io_bytes = bytes;
  return ALV_OK;
}

// Sync block of an FFN stack's workspace: [status @0][GridBar @256][counters @1024].
size_t stack_sync_bytes(const Weight* w) {
  return kHeaderBytes + static_cast<size_t>(w->a.m.RT + w->b.m.RT) * 4;
}

int check_status(alv_ctx* ctx, cudaStream_t st) {
  ALV_CUDA(ctx, cudaStreamSynchronize(st));
  if (!ctx->sync) return ALV_OK;
  uint32_t s = 0;
  ALV_CUDA(ctx, cudaMemcpy(&s, status_ptr(ctx), sizeof(s), cudaMemcpyDeviceToHost));
  // A kernel that gave up mid-way leaves its status word set: clear that
  // launch's status, barrier and counters.
  if (s) ALV_CUDA(ctx, cudaMemset(ctx->sync, 0, kSyncBytes));
  for (auto& w : ctx->weights) {
    if (!w || w->kind != 3) continue;
    uint32_t t = 0;
    ALV_CUDA(ctx, cudaMemcpy(&t, w->ws, sizeof(t), cudaMemcpyDeviceToHost));
    if (t) ALV_CUDA(ctx, cudaMemset(w->ws, 0, stack_sync_bytes(w.get())));
    // The peer-barrier counters of a tensor-parallel stack are out of step
    // across ranks after a wait gave up: only re-creating it on every rank
    // restores them.
    if (t && w->world > 1) w->broken = true;
    s |= t;
  }
  if (s) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "device-side wait timed out (status 0x%x)", s);
    return fail(ctx, ALV_ERR_TIMEOUT, buf);
  }
  return ALV_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int alv_version(void) { return kVersion; }

int alv_ctx_create(int device, alv_ctx** out) {
  if (!out) return ALV_ERR_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return ALV_ERR_NO_DEVICE;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return ALV_ERR_NO_DEVICE;
  if (prop.major != 10) return ALV_ERR_NO_DEVICE;  // built for sm_100a only
  auto* ctx = new alv_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ctx;
    return ALV_ERR_CUDA;
  }
  if (ensure_scratch(ctx, 0) != ALV_OK) {
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return ALV_ERR_CUDA;
  }
  *out = ctx;
  return ALV_OK;
}

int alv_ctx_destroy(alv_ctx* ctx) {
  if (!ctx) return ALV_ERR_ARG;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  for (auto& w : ctx->weights) {
    if (!w) continue;
    cudaFree(w->a.dev);
    cudaFree(w->b.dev);
    cudaFree(w->layers_dev);
    cudaFree(w->ws);
  }
  cudaFree(ctx->sync);
  cudaFree(ctx->scratch);
  cudaFree(ctx->io);
  for (void* q : ctx->retired) cudaFree(q);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return ALV_OK;
}

const char* alv_last_error(const alv_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int alv_sync_status(alv_ctx* ctx, void* stream) {
  if (!ctx) return ALV_ERR_ARG;
  int rc = set_device(ctx);
  if (rc) return rc;
  return check_status(ctx, static_cast<cudaStream_t>(stream));
}

int alv_q4_quantize(alv_ctx* ctx, const float* w, int N, int K, uint8_t* combined, void* stream) {
  if (!ctx || !w || !combined || N < 0 || K < 0) return fail(ctx, ALV_ERR_ARG, "q4_quantize: bad argument");
  if (K % 32) return fail(ctx, ALV_ERR_SHAPE, "q4_quantize: K must be a multiple of 32");
  int rc = set_device(ctx);
  if (rc) return rc;
  const size_t n = static_cast<size_t>(N) * (K / 32);
  if (n == 0) return ALV_OK;
  q4_quantize_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      w, N, K, combined);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

int alv_gemv_weight_create(alv_ctx* ctx, int N, int K, const void* combined, size_t nbytes,
                           int on_device, alv_handle* out) {
  if (!ctx || !combined || !out || N <= 0 || K <= 0) return fail(ctx, ALV_ERR_ARG, "gemv_weight_create: bad argument");
  if (K % 32) return fail(ctx, ALV_ERR_SHAPE, "gemv_weight_create: K must be a multiple of 32");
  const size_t expect = static_cast<size_t>(N) * (K / 32) * 20;
  if (nbytes != expect)
    return fail(ctx, ALV_ERR_SHAPE, "gemv_weight_create: expected " + std::to_string(expect) + " bytes, got " +
                                        std::to_string(nbytes));
  int rc = set_device(ctx);
  if (rc) return rc;
  const uint8_t* src = nullptr;
  uint8_t* owned = nullptr;
  rc = stage_source(ctx, combined, nbytes, on_device, &src, &owned);
  if (rc) return rc;
  RepackSrc s{};
  s.a = src;
  s.b = nullptr;
  s.rows = static_cast<uint32_t>(N);
  s.row_off = 0;
  s.row_bytes = static_cast<uint64_t>(K / 32) * 20;
  s.blk_off = 0;
  s.K = static_cast<uint32_t>(K);
  s.interleave8 = 0;
  s.RT = static_cast<uint32_t>((N + 15) / 16);
  s.KT = static_cast<uint32_t>((K + 63) / 64);
  auto w = std::make_unique<Weight>();
  w->kind = 1;
  rc = build_mat(ctx, s, static_cast<uint32_t>(N), static_cast<uint32_t>(K), &w->a);
  if (owned) cudaFree(owned);
  if (rc) return rc;
  ctx->weights.push_back(std::move(w));
  *out = static_cast<alv_handle>(ctx->weights.size());
  return ALV_OK;
}

int alv_ffn_weight_create(alv_ctx* ctx, int H, int I, int act, const void* gate, const void* up,
                          const void* down, int on_device, int i_begin, int i_end, alv_handle* out) {
  if (!ctx || !gate || !up || !down || !out || H <= 0 || I <= 0)
    return fail(ctx, ALV_ERR_ARG, "ffn_weight_create: bad argument");
  if (act != ALV_ACT_GELU && act != ALV_ACT_SILU) return fail(ctx, ALV_ERR_ARG, "ffn_weight_create: bad activation");
  if (H % 32 || I % 32) return fail(ctx, ALV_ERR_SHAPE, "ffn_weight_create: H and I must be multiples of 32");
  if (i_begin < 0 || i_end > I || i_begin >= i_end || i_begin % 32 || i_end % 32)
    return fail(ctx, ALV_ERR_SHAPE, "ffn_weight_create: slice must be 32-aligned inside [0, I)");
  int rc = set_device(ctx);
  if (rc) return rc;
  const size_t gu_bytes = static_cast<size_t>(I) * (H / 32) * 20;
  const size_t dn_bytes = static_cast<size_t>(H) * (I / 32) * 20;
  const uint8_t *g = nullptr, *u = nullptr, *d = nullptr;
  uint8_t *og = nullptr, *ou = nullptr, *od = nullptr;
  if ((rc = stage_source(ctx, gate, gu_bytes, on_device, &g, &og)) ||
      (rc = stage_source(ctx, up, gu_bytes, on_device, &u, &ou)) ||
      (rc = stage_source(ctx, down, dn_bytes, on_device, &d, &od))) {
    cudaFree(og);
    cudaFree(ou);
    cudaFree(od);
    return rc;
  }
  const uint32_t Il = static_cast<uint32_t>(i_end - i_begin);
  auto w = std::make_unique<Weight>();
  w->kind = 2;
  w->H = static_cast<uint32_t>(H);
  w->I = static_cast<uint32_t>(I);
  w->i_begin = static_cast<uint32_t>(i_begin);
  w->i_end = static_cast<uint32_t>(i_end);
  w->act = act;
  RepackSrc sa{};
  sa.a = g;
  sa.b = u;
  sa.rows = Il;
  sa.row_off = static_cast<uint32_t>(i_begin);
  sa.row_bytes = static_cast<uint64_t>(H / 32) * 20;
  sa.blk_off = 0;
  sa.K = static_cast<uint32_t>(H);
  sa.interleave8 = 1;
  sa.RT = (Il + 7) / 8;
  sa.KT = static_cast<uint32_t>((H + 63) / 64);
  RepackSrc sb{};
  sb.a = d;
  sb.b = nullptr;
  sb.rows = static_cast<uint32_t>(H);
  sb.row_off = 0;
  sb.row_bytes = static_cast<uint64_t>(I / 32) * 20;
  sb.blk_off = static_cast<uint32_t>(i_begin / 32);
  sb.K = Il;
  sb.interleave8 = 0;
  sb.RT = static_cast<uint32_t>((H + 15) / 16);
  sb.KT = (Il + 63) / 64;
  // One kernel dequantizes both matrices: they share the dequant path.
  Survey sva, svb;
  if (!(rc = survey_mat(ctx, sa, &sva)) && !(rc = survey_mat(ctx, sb, &svb))) {
    if (!(sva.fast && svb.fast)) sva = svb = Survey{};
    rc = repack_mat(ctx, sa, sva, Il, static_cast<uint32_t>(H), &w->a);
    if (!rc) rc = repack_mat(ctx, sb, svb, static_cast<uint32_t>(H), Il, &w->b);
  }
  cudaFree(og);
  cudaFree(ou);
  cudaFree(od);
  if (rc) {
    cudaFree(w->a.dev);
    cudaFree(w->b.dev);
    return rc;
  }
  ctx->weights.push_back(std::move(w));
  *out = static_cast<alv_handle>(ctx->weights.size());
  return ALV_OK;
}

int alv_weight_destroy(alv_ctx* ctx, alv_handle h) {
  if (!ctx) return ALV_ERR_ARG;
  Weight* w = get_weight(ctx, h, 0);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "weight_destroy: invalid handle");
  int rc = set_device(ctx);
  if (rc) return rc;
  for (auto& o : ctx->weights)
    if (o && o->kind == 3 && std::find(o->layers.begin(), o->layers.end(), h) != o->layers.end())
      return fail(ctx, ALV_ERR_ARG, "weight_destroy: the weight is a layer of an FFN stack; destroy the stack first");
  ALV_CUDA(ctx, cudaDeviceSynchronize());
  cudaFree(w->a.dev);
  cudaFree(w->b.dev);
  cudaFree(w->layers_dev);
  cudaFree(w->ws);
  if (w->connected)
    for (int q = 0; q < w->world; ++q)
      if (q != w->rank && w->xr[q]) cudaIpcCloseMemHandle(w->xr[q]);
  cudaFree(w->xlocal);
  ctx->weights[h - 1].reset();
  return ALV_OK;
}

int alv_ffn_set_activation(alv_ctx* ctx, alv_handle h, int act) {
  if (!ctx) return ALV_ERR_ARG;
  if (act != ALV_ACT_GELU && act != ALV_ACT_SILU) return fail(ctx, ALV_ERR_ARG, "ffn_set_activation: bad activation");
  Weight* w = get_weight(ctx, h, 2);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_set_activation: invalid handle (not an ffn weight)");
  w->act = act;
  return ALV_OK;
}

int alv_set_trace(alv_ctx* ctx, uint64_t* trace) {
  if (!ctx) return ALV_ERR_ARG;
  ctx->trace = reinterpret_cast<unsigned long long*>(trace);
  return ALV_OK;
}

int alv_weight_info(alv_ctx* ctx, alv_handle h, int64_t* info) {
  if (!ctx || !info) return ALV_ERR_ARG;
  Weight* w = get_weight(ctx, h, 0);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "weight_info: invalid handle");
  info[0] = w->kind;
  info[1] = w->kind == 1 ? w->a.rows : w->H;
  info[2] = w->kind == 1 ? w->a.cols : (w->i_end - w->i_begin);
  info[3] = w->a.m.fast;
  info[4] = w->kind == 2 ? w->b.m.fast : 0;
  info[5] = static_cast<int64_t>(w->a.bytes + w->b.bytes);
  info[6] = w->i_begin;
  info[7] = w->i_end;
  return ALV_OK;
}

int alv_weight_dequantize(alv_ctx* ctx, alv_handle h, int which, uint16_t* out, void* stream) {
  if (!ctx || !out) return fail(ctx, ALV_ERR_ARG, "weight_dequantize: bad argument");
  Weight* w = get_weight(ctx, h, 0);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "weight_dequantize: invalid handle");
  int rc = set_device(ctx);
  if (rc) return rc;
  const Mat* m = nullptr;
  uint32_t rows = 0, K = 0;
  if (w->kind == 1) {
    if (which != 0) return fail(ctx, ALV_ERR_ARG, "weight_dequantize: gemv weights have one matrix");
    m = &w->a;
    rows = m->rows;
    K = m->cols;
  } else {
    if (which < 0 || which > 2) return fail(ctx, ALV_ERR_ARG, "weight_dequantize: which must be 0..2");
    m = which == 2 ? &w->b : &w->a;
    rows = which == 2 ? w->H : (w->i_end - w->i_begin);
    K = which == 2 ? (w->i_end - w->i_begin) : w->H;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t nthreads = static_cast<uint64_t>(m->m.RT) * m->m.KT * 32;
  if (w->kind == 2 && which < 2) {
    // gate/up live interleaved: dequantize the whole interleaved matrix into a
    // temporary (2*I rows) and gather the requested half.
    const uint32_t rows_all = m->m.RT * 16;
    uint16_t* tmp = nullptr;
    ALV_CUDA(ctx, cudaMalloc(&tmp, static_cast<size_t>(rows_all) * K * 2));
    q4_dequant_kernel<<<static_cast<unsigned>((nthreads + 255) / 256), 256, 0, st>>>(m->m, rows_all, K, tmp);
    ALV_CUDA(ctx, cudaGetLastError());
    for (uint32_t i = 0; i < rows; ++i) {
      const uint32_t src_row = (i / 8) * 16 + (i % 8) + (which == 1 ? 8 : 0);
      ALV_CUDA(ctx, cudaMemcpyAsync(out + static_cast<size_t>(i) * K, tmp + static_cast<size_t>(src_row) * K,
                                    static_cast<size_t>(K) * 2, cudaMemcpyDeviceToDevice, st));
    }
    ALV_CUDA(ctx, cudaStreamSynchronize(st));
    ALV_CUDA(ctx, cudaFree(tmp));
    return ALV_OK;
  }
  if (nthreads) {
    q4_dequant_kernel<<<static_cast<unsigned>((nthreads + 255) / 256), 256, 0, st>>>(m->m, rows, K, out);
    ALV_CUDA(ctx, cudaGetLastError());
  }
  return ALV_OK;
}

int alv_gemv(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
             void* stream) {
  if (!ctx || !x || !y || !valid_dtype(x_dtype) || !valid_dtype(y_dtype))
    return fail(ctx, ALV_ERR_ARG, "gemv: bad argument");
  Weight* w = get_weight(ctx, h, 1);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "gemv: invalid handle (not a gemv weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  return do_gemv(ctx, w, ntok, x, x_dtype, y, y_dtype, static_cast<cudaStream_t>(stream));
}

int alv_ffn(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
            void* stream) {
  if (!ctx || !x || !y || !valid_dtype(x_dtype) || !valid_dtype(y_dtype))
    return fail(ctx, ALV_ERR_ARG, "ffn: bad argument");
  Weight* w = get_weight(ctx, h, 2);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn: invalid handle (not an ffn weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  FfnIo io;
  io.x = x;
  io.x_dtype = x_dtype;
  io.y32 = y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr;
  io.y16 = y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr;
  return do_ffn(ctx, w, ntok, io, static_cast<cudaStream_t>(stream));
}

int alv_ffn_layer(alv_ctx* ctx, alv_handle h, int ntok, const uint16_t* x_in, const float* down_in,
                  uint16_t* x_out, float* down_out, void* stream) {
  if (!ctx || !x_in || !down_out) return fail(ctx, ALV_ERR_ARG, "ffn_layer: bad argument");
  Weight* w = get_weight(ctx, h, 2);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_layer: invalid handle (not an ffn weight)");
  int rc = set_device(ctx);
  if (rc) return rc;
  FfnIo io;
  io.x = x_in;
  io.x_dtype = ALV_BF16;
  io.glue = 1;
  io.x_in = x_in;
  io.down_in = down_in;
  io.x_out = x_out;
  io.y32 = down_out;
  return do_ffn(ctx, w, ntok, io, static_cast<cudaStream_t>(stream));
}

int alv_ffn_stack_finalize(alv_ctx* ctx, int ntok, int H, const uint16_t* x_in, const float* down_in,
                           uint16_t* x_out, void* stream) {
  if (!ctx || !x_in || !down_in || !x_out || ntok < 1 || H <= 0)
    return fail(ctx, ALV_ERR_ARG, "ffn_stack_finalize: bad argument");
  if (static_cast<uint32_t>(H) > 32u * kConsumerWarps * kGlueRegs)
    return fail(ctx, ALV_ERR_UNSUPPORTED,
                "ffn_stack_finalize: H must be <= " + std::to_string(32u * kConsumerWarps * kGlueRegs));
  int rc = set_device(ctx);
  if (rc) return rc;
  ffn_stack_finalize_kernel<<<1, kConsumerWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      ntok, static_cast<uint32_t>(H), x_in, down_in, x_out, 1e-6f);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

static int run_host(alv_ctx* ctx, alv_handle h, int kind, int ntok, const void* x_host, int x_dtype,
                    void* y_host, int y_dtype) {
  if (!ctx || !x_host || !y_host || !valid_dtype(x_dtype) || !valid_dtype(y_dtype) || ntok < 1)
    return fail(ctx, ALV_ERR_ARG, "run: bad argument");
  Weight* w = get_weight(ctx, h, kind);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "run: invalid handle");
  int rc = set_device(ctx);
  if (rc) return rc;
  const size_t K = kind == 1 ? w->a.cols : w->H;
  const size_t N = kind == 1 ? w->a.rows : w->H;
  const size_t xb = static_cast<size_t>(ntok) * K * (x_dtype == ALV_F32 ? 4 : 2);
  const size_t yb = static_cast<size_t>(ntok) * N * (y_dtype == ALV_F32 ? 4 : 2);
  rc = io_buffers(ctx, align_up(xb, 256) + yb);
  if (rc) return rc;
  uint8_t* dx = static_cast<uint8_t*>(ctx->io);
  uint8_t* dy = dx + align_up(xb, 256);
  ALV_CUDA(ctx, cudaMemcpyAsync(dx, x_host, xb, cudaMemcpyHostToDevice, ctx->stream));
  if (kind == 1) {
    rc = do_gemv(ctx, w, ntok, dx, x_dtype, dy, y_dtype, ctx->stream);
  } else {
    FfnIo io;
    io.x = dx;
    io.x_dtype = x_dtype;
    io.y32 = y_dtype == ALV_F32 ? reinterpret_cast<float*>(dy) : nullptr;
    io.y16 = y_dtype == ALV_BF16 ? reinterpret_cast<uint16_t*>(dy) : nullptr;
    rc = do_ffn(ctx, w, ntok, io, ctx->stream);
  }
  if (rc) return rc;
  ALV_CUDA(ctx, cudaMemcpyAsync(y_host, dy, yb, cudaMemcpyDeviceToHost, ctx->stream));
  return check_status(ctx, ctx->stream);
}

int alv_run_gemv(alv_ctx* ctx, alv_handle h, int ntok, const void* x_host, int x_dtype, void* y_host,
                 int y_dtype) {
  return run_host(ctx, h, 1, ntok, x_host, x_dtype, y_host, y_dtype);
}

int alv_run_ffn(alv_ctx* ctx, alv_handle h, int ntok, const void* x_host, int x_dtype, void* y_host,
                int y_dtype) {
  return run_host(ctx, h, 2, ntok, x_host, x_dtype, y_host, y_dtype);
}

}  // extern "C"

// ===========================================================================
// Batched prefill gemm_q on tcgen05 (gemm_tc_kernel).
// ===========================================================================
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

extern "C" int alv_gemm(alv_ctx* ctx, alv_handle h, int B, const uint16_t* x, void* y, int y_dtype, void* stream) {
  if (!ctx || !x || !y || B < 1 || !valid_dtype(y_dtype)) return fail(ctx, ALV_ERR_ARG, "gemm: bad argument");
  Weight* w = get_weight(ctx, h, 1);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "gemm: invalid handle (not a gemv weight)");
  if (reinterpret_cast<uintptr_t>(x) & 15) return fail(ctx, ALV_ERR_ARG, "gemm: x must be 16-byte aligned");
  int rc = set_device(ctx);
  if (rc) return rc;
  EncodeTiledFn enc = nullptr;
  if ((rc = tensor_map_encoder(ctx, &enc))) return rc;
  const uint32_t K = w->a.cols;
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
  p.m = w->a.m;
  p.N = w->a.rows;
  p.B = static_cast<uint32_t>(B);
  p.y32 = y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr;
  p.y16 = y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr;
  p.status = status_ptr(ctx);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return p.m.fast ? launch_gemm_f<true>(ctx, p, map, nt, st) : launch_gemm_f<false>(ctx, p, map, nt, st);
}

// ===========================================================================
// FFN stack: every layer of a decode step in one persistent launch
// (ffn_stack_kernel).  The stack keeps its own workspace, so a launch
// captured in a CUDA graph stays valid whatever else the context runs.
// ===========================================================================
namespace {
constexpr int kStackMaxTokens = 4;

struct StackLayout {
  size_t counters, wsA, wsB, down, act, total;
};

StackLayout stack_layout(alv_ctx* ctx, const Weight* w) {
  StackLayout o;
  o.counters = kHeaderBytes;
  o.wsA = align_up(o.counters + static_cast<size_t>(w->a.m.RT + w->b.m.RT) * 4, 256);
  o.wsB = align_up(o.wsA + ws_floats(ctx, w->a.m, kStackMaxTokens) * 4, 256);
  o.down = align_up(o.wsB + ws_floats(ctx, w->b.m, kStackMaxTokens) * 4, 256);
  o.act = align_up(o.down + static_cast<size_t>(kStackMaxTokens) * w->H * 4, 256);
  o.total = align_up(o.act + frag_bytes(w->b.m.KT, kStackMaxTokens), 256);
  return o;
}

template <int NT, bool FAST, bool TP>
int launch_stack_t(alv_ctx* ctx, StackParams p, cudaStream_t st) {
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  const size_t other = stack_smem_bytes(0, p.gu.KT, p.dn.KT, NT, p.H, p.ntok, p.dn.RT, nctas);
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack: H, I or ntok too large for shared memory");
  const size_t smem = stack_smem_bytes(p.nst, p.gu.KT, p.dn.KT, NT, p.H, p.ntok, p.dn.RT, nctas);
  auto k = ffn_stack_kernel<NT, FAST, TP>;
  int rc = prepare_kernel(ctx, k, smem);
  if (rc) return rc;
  k<<<ctx->num_sms, kThreadsPerCta, smem, st>>>(p);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

template <bool FAST, bool TP>
int launch_stack_f(alv_ctx* ctx, const StackParams& p, uint32_t nt, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_stack_t<1, FAST, TP>(ctx, p, st);
    case 2: return launch_stack_t<2, FAST, TP>(ctx, p, st);
    case 4: return launch_stack_t<4, FAST, TP>(ctx, p, st);
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack: unsupported token count");
}

// Exchange slot of a tensor-parallel stack: [whole rows: kStackMaxTokens x H]
// [CTA partials: #SMs x 2 x kStackMaxTokens x 16], in floats, 64-aligned.
void exchange_shape(alv_ctx* ctx, const Weight* w, uint32_t* xslot, uint32_t* xws_off) {
  const size_t rows = (static_cast<size_t>(kStackMaxTokens) * w->H + 63) / 64 * 64;
  const size_t parts = static_cast<size_t>(ctx->num_sms) * 2 * kStackMaxTokens * 16;
  *xws_off = static_cast<uint32_t>(rows);
  *xslot = static_cast<uint32_t>((rows + parts + 63) / 64 * 64);
}

// Blob layout: [0, 64) cudaIpcMemHandle_t of the exchange region, [64, 80)
// device UUID, [80, 100) u32 world, slot floats, I-slice width, layers, SMs
// (the ranks must agree on all five: each launch passes layers x world x SMs
// peer-barrier arrivals).
constexpr size_t kBlobUuid = 64, kBlobWorld = 80;
static_assert(sizeof(cudaIpcMemHandle_t) <= kBlobUuid, "IPC handle larger than its blob field");
}  // namespace

extern "C" int alv_ffn_stack_create(alv_ctx* ctx, const alv_handle* layers, int n, alv_handle* out) {
  if (!ctx || !layers || !out || n < 1) return fail(ctx, ALV_ERR_ARG, "ffn_stack_create: bad argument");
  const Weight* w0 = get_weight(ctx, layers[0], 2);
  if (!w0) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_create: layer 0 is not an ffn weight");
  if (w0->H > 32u * kConsumerWarps * kGlueRegs)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_create: H must be <= " + std::to_string(32u * kConsumerWarps * kGlueRegs));
  if (w0->a.m.RT + w0->b.m.RT > kMaxCounters) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_create: too large");
  std::vector<LayerW> lw(static_cast<size_t>(n));
  for (int l = 0; l < n; ++l) {
    const Weight* w = get_weight(ctx, layers[l], 2);
    if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_create: layer " + std::to_string(l) + " is not an ffn weight");
    if (w->H != w0->H || w->I != w0->I || w->i_begin != w0->i_begin || w->i_end != w0->i_end ||
        w->a.m.fast != w0->a.m.fast)
      return fail(ctx, ALV_ERR_SHAPE, "ffn_stack_create: layer " + std::to_string(l) +
                                          " differs in shape or dequant path from layer 0");
    lw[l] = LayerW{w->a.m.units, w->b.m.units, w->a.m.scale_mul, w->b.m.scale_mul, {0, 0}};
  }
  int rc = set_device(ctx);
  if (rc) return rc;
  auto s = std::make_unique<Weight>();
  s->kind = 3;
  s->a.m = w0->a.m;
  s->b.m = w0->b.m;
  s->a.rows = w0->a.rows;
  s->a.cols = w0->a.cols;
  s->b.rows = w0->b.rows;
  s->b.cols = w0->b.cols;
  s->H = w0->H;
  s->I = w0->I;
  s->i_begin = w0->i_begin;
  s->i_end = w0->i_end;
  s->act = w0->act;
  s->layers.assign(layers, layers + n);
  const StackLayout lo = stack_layout(ctx, s.get());
  ALV_CUDA(ctx, cudaMalloc(&s->layers_dev, sizeof(LayerW) * lw.size()));
  ALV_CUDA(ctx, cudaMemcpy(s->layers_dev, lw.data(), sizeof(LayerW) * lw.size(), cudaMemcpyHostToDevice));
  ALV_CUDA(ctx, cudaMalloc(&s->ws, lo.total));
  ALV_CUDA(ctx, cudaMemset(s->ws, 0, lo.total));
  s->ws_bytes = lo.total;
  ctx->weights.push_back(std::move(s));
  *out = static_cast<alv_handle>(ctx->weights.size());
  return ALV_OK;
}

extern "C" int alv_ffn_stack_run(alv_ctx* ctx, alv_handle h, int ntok, const uint16_t* x_in, uint16_t* out,
                                 void* stream) {
  if (!ctx || !x_in || !out) return fail(ctx, ALV_ERR_ARG, "ffn_stack_run: bad argument");
  Weight* w = get_weight(ctx, h, 3);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_run: invalid handle (not an ffn stack)");
  if (ntok < 1 || ntok > kStackMaxTokens)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_run: ntok must be 1.." + std::to_string(kStackMaxTokens));
  const Weight* w0 = get_weight(ctx, w->layers[0], 2);
  if (!w0) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_run: a layer was destroyed");
  const bool tp = w->i_begin != 0 || w->i_end != w->I;
  if (tp && !w->connected)
    return fail(ctx, ALV_ERR_ARG, "ffn_stack_run: a stack of I-slices needs alv_ffn_stack_connect first");
  if (w->broken)
    return fail(ctx, ALV_ERR_ARG, "ffn_stack_run: a device wait of this tensor-parallel stack gave up earlier; "
                                  "destroy and re-create it on every rank");
  for (alv_handle lh : w->layers)
    if (!get_weight(ctx, lh, 2) || get_weight(ctx, lh, 2)->act != w0->act)
      return fail(ctx, ALV_ERR_ARG, "ffn_stack_run: layers disagree on the activation");
  int rc = set_device(ctx);
  if (rc) return rc;
  const StackLayout lo = stack_layout(ctx, w);
  StackParams p{};
  p.layers = w->layers_dev;
  p.L = static_cast<uint32_t>(w->layers.size());
  p.gu = w->a.m;
  p.dn = w->b.m;
  p.H = w->H;
  p.I = w->i_end - w->i_begin;
  p.fn = w0->act;
  p.ntok = ntok;
  p.eps = 1e-6f;
  p.x_in = x_in;
  p.out = out;
  p.down = reinterpret_cast<float*>(w->ws + lo.down);
  p.act = w->ws + lo.act;
  uint32_t* cnt = reinterpret_cast<uint32_t*>(w->ws + lo.counters);
  p.fxA = Fixup{reinterpret_cast<float*>(w->ws + lo.wsA), cnt};
  p.fxB = Fixup{reinterpret_cast<float*>(w->ws + lo.wsB), cnt + w->a.m.RT};
  p.bar = reinterpret_cast<GridBar*>(w->ws + 256);
  p.status = reinterpret_cast<uint32_t*>(w->ws);
  p.trace = ctx->trace;
  const uint32_t nt = pow2_ceil(static_cast<uint32_t>(ntok));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tp) {
    p.world = static_cast<uint32_t>(w->world);
    p.rank = static_cast<uint32_t>(w->rank);
    for (int q = 0; q < w->world; ++q) p.xr[q] = w->xr[q];
    p.xslot = w->xslot;
    p.xws_off = w->xws_off;
    return p.gu.fast ? launch_stack_f<true, true>(ctx, p, nt, st) : launch_stack_f<false, true>(ctx, p, nt, st);
  }
  return p.gu.fast ? launch_stack_f<true, false>(ctx, p, nt, st) : launch_stack_f<false, false>(ctx, p, nt, st);
}

extern "C" int alv_activation(alv_ctx* ctx, int act, int n, const uint16_t* gate, const uint16_t* up, uint16_t* out,
                              void* stream) {
  if (!ctx || n < 0 || (n && (!gate || !up || !out)) || (act != ALV_ACT_GELU && act != ALV_ACT_SILU))
    return fail(ctx, ALV_ERR_ARG, "activation: bad argument");
  if (!n) return ALV_OK;
  int rc = set_device(ctx);
  if (rc) return rc;
  const uint32_t threads = 256, blocks = (static_cast<uint32_t>(n) + threads - 1) / threads;
  activation_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(act == ALV_ACT_GELU ? 0 : 1,
                                                                              static_cast<uint32_t>(n), gate, up, out);
  ALV_CUDA(ctx, cudaGetLastError());
  return ALV_OK;
}

extern "C" int alv_ffn_stack_exchange(alv_ctx* ctx, alv_handle h, int world, void* blob) {
  if (!ctx || !blob) return fail(ctx, ALV_ERR_ARG, "ffn_stack_exchange: bad argument");
  Weight* w = get_weight(ctx, h, 3);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_exchange: invalid handle (not an ffn stack)");
  if (world < 2 || world > kMaxRanks)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_exchange: world must be 2.." + std::to_string(kMaxRanks));
  if (w->xlocal) return fail(ctx, ALV_ERR_ARG, "ffn_stack_exchange: already called for this stack");
  int rc = set_device(ctx);
  if (rc) return rc;
  exchange_shape(ctx, w, &w->xslot, &w->xws_off);
  const size_t bytes = kXHeader + static_cast<size_t>(2) * world * w->xslot * 4;
  ALV_CUDA(ctx, cudaMalloc(&w->xlocal, bytes));
  ALV_CUDA(ctx, cudaMemset(w->xlocal, 0, bytes));
  ALV_CUDA(ctx, cudaDeviceSynchronize());
  cudaIpcMemHandle_t ih;
  ALV_CUDA(ctx, cudaIpcGetMemHandle(&ih, w->xlocal));
  cudaDeviceProp prop;
  ALV_CUDA(ctx, cudaGetDeviceProperties(&prop, ctx->device));
  std::memset(w->blob, 0, sizeof(w->blob));
  std::memcpy(w->blob, &ih, sizeof(ih));
  std::memcpy(w->blob + kBlobUuid, &prop.uuid, 16);
  const uint32_t vals[5] = {static_cast<uint32_t>(world), w->xslot, w->i_end - w->i_begin,
                            static_cast<uint32_t>(w->layers.size()), static_cast<uint32_t>(ctx->num_sms)};
  std::memcpy(w->blob + kBlobWorld, vals, sizeof(vals));
  w->world = world;
  std::memcpy(blob, w->blob, ALV_IPC_BLOB_BYTES);
  return ALV_OK;
}

extern "C" int alv_ffn_stack_connect(alv_ctx* ctx, alv_handle h, int rank, int world, const void* blobs) {
  if (!ctx || !blobs) return fail(ctx, ALV_ERR_ARG, "ffn_stack_connect: bad argument");
  Weight* w = get_weight(ctx, h, 3);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_connect: invalid handle (not an ffn stack)");
  if (!w->xlocal || w->connected || world != w->world || rank < 0 || rank >= world)
    return fail(ctx, ALV_ERR_ARG, "ffn_stack_connect: call once, after alv_ffn_stack_exchange with the same world");
  const unsigned char* b = static_cast<const unsigned char*>(blobs);
  auto blob_of = [&](int q) { return b + static_cast<size_t>(q) * ALV_IPC_BLOB_BYTES; };
  if (std::memcmp(blob_of(rank), w->blob, ALV_IPC_BLOB_BYTES) != 0)
    return fail(ctx, ALV_ERR_ARG, "ffn_stack_connect: blobs[rank] is not this stack's blob");
  const uint32_t width = w->i_end - w->i_begin;
  if (static_cast<uint64_t>(width) * world != w->I || w->i_begin != static_cast<uint32_t>(rank) * width)
    return fail(ctx, ALV_ERR_SHAPE, "ffn_stack_connect: the layers are not I-slice `rank` of `world` equal slices");
  for (int q = 0; q < world; ++q) {
    uint32_t vals[5], mine[5];
    std::memcpy(vals, blob_of(q) + kBlobWorld, sizeof(vals));
    std::memcpy(mine, w->blob + kBlobWorld, sizeof(mine));
    if (std::memcmp(vals, mine, sizeof(vals)) != 0)
      return fail(ctx, ALV_ERR_SHAPE, "ffn_stack_connect: rank " + std::to_string(q) +
                                          " differs in world, shape, layer count or SM count");
    for (int o = 0; o < q; ++o)
      if (std::memcmp(blob_of(q) + kBlobUuid, blob_of(o) + kBlobUuid, 16) == 0)
        return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_connect: ranks " + std::to_string(o) + " and " +
                                                  std::to_string(q) + " are on the same GPU");
  }
  int rc = set_device(ctx);
  if (rc) return rc;
  // Peers visible to this process must support native atomics over the link.
  int ndev = 0;
  ALV_CUDA(ctx, cudaGetDeviceCount(&ndev));
  for (int d = 0; d < ndev; ++d) {
    if (d == ctx->device) continue;
    cudaDeviceProp prop;
    ALV_CUDA(ctx, cudaGetDeviceProperties(&prop, d));
    for (int q = 0; q < world; ++q) {
      if (q == rank || std::memcmp(blob_of(q) + kBlobUuid, &prop.uuid, 16) != 0) continue;
      int atomics = 0;
      ALV_CUDA(ctx, cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, ctx->device, d));
      if (!atomics)
        return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack_connect: no native peer atomics to device " + std::to_string(d));
    }
  }
  for (int q = 0; q < world; ++q) {
    if (q == rank) {
      w->xr[q] = w->xlocal;
      continue;
    }
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, blob_of(q), sizeof(ih));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int o = 0; o < q; ++o)
        if (o != rank && w->xr[o]) cudaIpcCloseMemHandle(w->xr[o]);
      std::fill(w->xr, w->xr + kMaxRanks, nullptr);
      return fail(ctx, ALV_ERR_CUDA, std::string("ffn_stack_connect: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    }
    w->xr[q] = static_cast<uint8_t*>(ptr);
  }
  w->rank = rank;
  w->connected = true;
  return ALV_OK;
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
constexpr uint32_t kNoAllocMaxWarps = 2368;               // participating warps covered (>= 148 SMs x 15)
constexpr size_t kNoAllocWsFloats = static_cast<size_t>(kNoAllocMaxWarps) * 2 * kNoAllocMaxTokens * 16;
constexpr size_t kNoAllocCounterBytes = static_cast<size_t>(kNoAllocMaxRowTiles) * 4;
constexpr size_t kNoAllocBytes = kNoAllocCounterBytes + kNoAllocWsFloats * 4;  // 1,277,952 bytes
}  // namespace

// [counters: kNoAllocMaxRowTiles x u32][workspace: kNoAllocWsFloats x f32]
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: look up the device address of
// the static array (its host-side name is only a stand-in, not a device
// pointer).
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
  const bool split = x_dtype == ALV_F32;
  const uint32_t ncols = pow2_ceil(static_cast<uint32_t>(split ? 2 * ntok : ntok));
  if (ntok < 1 || ntok > static_cast<int>(kNoAllocMaxTokens))
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: ntok must be 1.." + std::to_string(kNoAllocMaxTokens));
  if (w->a.m.RT > kNoAllocMaxRowTiles)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: N must be <= " + std::to_string(kNoAllocMaxRowTiles * 16));
  if (static_cast<uint32_t>(ctx->num_sms) * kWarpsPerCta > kNoAllocMaxWarps)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: GPU has more SMs than the static workspace covers");
  if (ws_floats(ctx, w->a.m, ntok) > kNoAllocWsFloats)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "gemv_noalloc: split-K workspace exceeds the static array");
  uint8_t* base = nullptr;
  if ((rc = noalloc_scratch(ctx, &base))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the arrival counters this
  // call uses must start at zero.
  ALV_CUDA(ctx, cudaMemsetAsync(base, 0, static_cast<size_t>(w->a.m.RT) * 4, st));
  GemvParams p{};
  p.m = w->a.m;
  p.x = XSrc{x, x_dtype == ALV_BF16, ntok, w->a.cols, w->a.cols};
  p.epi = RowsEpi{y_dtype == ALV_F32 ? static_cast<float*>(y) : nullptr,
                  y_dtype == ALV_BF16 ? static_cast<uint16_t*>(y) : nullptr, w->a.rows, w->a.rows,
                  w->a.m.scale_mul};
  p.fx = Fixup{reinterpret_cast<float*>(base + kNoAllocCounterBytes), reinterpret_cast<uint32_t*>(base)};
  p.status = status_ptr(ctx);
  return launch_gemv(ctx, p, split, ncols, st);
}
