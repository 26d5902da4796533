// Host-side internals shared by the translation units of the C ABI
// (core.cu, gemv.cu, ffn.cu, stack.cu, gemm.cu, decode.cu): the context, the
// weight registry, status handling and launch helpers.  Not part of the ABI.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/alveare_b200.h"
#include "stream.cuh"

namespace alv {

constexpr int kVersion = 200;             // 0.2.0
constexpr uint32_t kMaxCounters = 65536;  // row tiles per matrix (N <= 1,048,576)
constexpr size_t kHeaderBytes = 1024;     // status word + grid barrier
constexpr size_t kMaxSmem = 227 * 1024;
constexpr int kMaxRanksHost = 8;          // tensor-parallel ranks of one FFN stack

struct Mat {
  uint8_t* dev = nullptr;
  Q4Mat m{};
  uint32_t rows = 0, cols = 0;
  size_t bytes = 0;
};

struct Weight {
  int kind = 0;  // 1 gemv, 2 ffn, 3 ffn stack, 4 decode model
  Mat a, b;      // gemv: a; ffn: a = gate/up interleaved, b = down; stack: shapes of every layer
  uint32_t H = 0, I = 0, i_begin = 0, i_end = 0;
  int act = 0;
  // kind 3: the layers (FFN weights), their device descriptors and the
  // stack's own workspace (sync words, split-K partials, down, act)
  std::vector<alv_handle> layers;
  struct LayerW* layers_dev = nullptr;
  uint8_t* ws = nullptr;     // kinds 3, 4: workspace, starting with the sync block
  size_t ws_bytes = 0;
  size_t sync_bytes = 0;     // kind 4: bytes of the sync block (status, grid barrier, counters)
  // kind 3, tensor parallel: this rank's exchange region (cudaMalloc, shared
  // with the peers by CUDA IPC) and every rank's region as mapped here
  int world = 1, rank = 0;
  bool connected = false, broken = false;
  uint8_t* xlocal = nullptr;
  uint32_t xslot = 0, xws_off = 0;  // exchange slot: LL words per slot, offset of the CTA partials
  uint8_t* xr[kMaxRanksHost] = {};
  unsigned char blob[ALV_IPC_BLOB_BYTES] = {};
  float* probe = nullptr;  // kind 3: optional fp32 copy of the last layer's down projection
  // kind 4: decode model state (owned by decode.cu)
  void* model = nullptr;
  void (*model_free)(void*) = nullptr;
};

}  // namespace alv

struct alv_ctx {
  int device = 0;
  int num_sms = 0;
  std::string err;
  std::vector<std::unique_ptr<alv::Weight>> weights;  // handle = index + 1
  uint8_t* sync = nullptr;                            // [header: status, grid barrier][counters], fixed
  uint8_t* scratch = nullptr;                         // work area (split-K partials, act)
  size_t scratch_bytes = 0;
  std::vector<void*> retired;                         // outgrown buffers, freed with the context
  void* io = nullptr;                                 // device staging for host-buffer calls
  size_t io_bytes = 0;
  cudaStream_t stream = nullptr;                      // internal stream (loads, host calls)
  unsigned long long* trace = nullptr;                // optional FFN phase timestamps
  int64_t allocs = 0;                                 // device allocations made through this context
};

namespace alv {

inline int fail(alv_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return code;
}

#define ALV_CUDA(ctx, call)                                                              \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return ::alv::fail((ctx), ALV_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// Every device allocation of the library goes through here (counted per
// context, reported by alv_ctx_info).
template <class T>
cudaError_t dev_alloc(alv_ctx* ctx, T** p, size_t bytes) {
  ++ctx->allocs;
  return cudaMalloc(reinterpret_cast<void**>(p), bytes);
}

inline int set_device(alv_ctx* ctx) {
  ALV_CUDA(ctx, cudaSetDevice(ctx->device));
  return ALV_OK;
}

constexpr size_t kSyncBytes = kHeaderBytes + static_cast<size_t>(kMaxCounters) * 4;
inline uint32_t* status_ptr(alv_ctx* ctx) { return reinterpret_cast<uint32_t*>(ctx->sync); }
inline uint8_t* bar_bytes(alv_ctx* ctx) { return ctx->sync + 256; }
inline uint32_t* counters_ptr(alv_ctx* ctx) { return reinterpret_cast<uint32_t*>(ctx->sync + kHeaderBytes); }
inline uint8_t* work_ptr(alv_ctx* ctx) { return ctx->scratch; }

// The sync block (status word, grid barrier, arrival counters; counters are
// zero between launches) is allocated once per context.  The work area is
// re-laid out per call and grows on demand; an outgrown area is kept until
// the context is destroyed, so launches captured in a CUDA graph earlier
// still point at live memory.
int ensure_scratch(alv_ctx* ctx, size_t work_bytes);

inline Weight* get_weight(alv_ctx* ctx, alv_handle h, int kind) {
  if (h == 0 || h > ctx->weights.size()) return nullptr;
  Weight* w = ctx->weights[h - 1].get();
  if (!w || (kind && w->kind != kind)) return nullptr;
  return w;
}

inline alv_handle add_weight(alv_ctx* ctx, std::unique_ptr<Weight> w) {
  ctx->weights.push_back(std::move(w));
  return static_cast<alv_handle>(ctx->weights.size());
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline uint32_t pow2_ceil(uint32_t v) {
  uint32_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

inline bool valid_dtype(int d) { return d == ALV_F32 || d == ALV_BF16; }

// Element alignment of an activation buffer: the kernels read fp32 x as
// float2 and bf16 x as 32-bit pairs, so x must be 8- / 4-byte aligned.
inline bool x_aligned(const void* x, int x_dtype) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x);
  return (a & (x_dtype == ALV_F32 ? 7u : 3u)) == 0;
}

// Split-K CTA partials: two slots of ntok x 16 floats per CTA.
inline size_t ws_floats(alv_ctx* ctx, int ntok) { return static_cast<size_t>(ctx->num_sms) * 2 * ntok * 16; }

// Raise the kernel's dynamic shared-memory limit once per (kernel, device) to
// the maximum, so launches need no per-call attribute changes, and check that
// `grid_ctas` CTAs of `smem` bytes can all be resident at once (the
// persistent kernels' grid barriers need every CTA running).  The limit
// covers static + dynamic shared memory; kernels with static __shared__
// arrays get kMaxSmem minus those bytes.
struct KernelLimits {
  size_t max_dyn = 0;
  std::map<size_t, int> resident;  // smem -> CTAs per SM
};
template <class K>
int prepare_kernel(alv_ctx* ctx, K kernel, size_t smem, int threads = 0, int grid_ctas = 0) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, KernelLimits> limits;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), ctx->device);
  std::lock_guard<std::mutex> lock(mu);
  auto it = limits.find(key);
  if (it == limits.end()) {
    cudaFuncAttributes fa;
    ALV_CUDA(ctx, cudaFuncGetAttributes(&fa, kernel));
    KernelLimits kl;
    kl.max_dyn = fa.sharedSizeBytes < kMaxSmem ? kMaxSmem - fa.sharedSizeBytes : 0;
    ALV_CUDA(ctx, cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kl.max_dyn)));
    it = limits.emplace(key, kl).first;
  }
  if (smem > it->second.max_dyn)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "problem needs " + std::to_string(smem) +
                                              " B of dynamic shared memory (max " + std::to_string(it->second.max_dyn) + ")");
  if (grid_ctas > 0) {
    auto r = it->second.resident.find(smem);
    if (r == it->second.resident.end()) {
      int per_sm = 0;
      ALV_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem));
      r = it->second.resident.emplace(smem, per_sm).first;
    }
    if (static_cast<long long>(r->second) * ctx->num_sms < grid_ctas)
      return fail(ctx, ALV_ERR_UNSUPPORTED,
                  "persistent kernel: " + std::to_string(grid_ctas) + " CTAs cannot all be resident (" +
                      std::to_string(r->second) + " per SM on " + std::to_string(ctx->num_sms) + " SMs)");
  }
  return ALV_OK;
}

// Launch a persistent grid-barrier kernel as a cooperative launch: the
// runtime then guarantees that every CTA is resident at once (or refuses
// the launch), instead of the grid barrier assuming it.
template <class P>
int launch_cooperative(alv_ctx* ctx, void (*kernel)(P), const P& p, unsigned grid, unsigned threads, size_t smem,
                       cudaStream_t st, bool pdl = false) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  ALV_CUDA(ctx, cudaLaunchKernelEx(&cfg, kernel, p));
  return ALV_OK;
}

// Launch `kernel`; with `pdl` as a programmatic dependent launch (it may
// start while its predecessor in the stream finishes; the kernel calls
// pdl_wait() before it touches that predecessor's data).
template <class... KArgs, class... Args>
int launch_ex(alv_ctx* ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ALV_CUDA(ctx, cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  return ALV_OK;
}

// Ring stages per warp that fit beside `other` bytes of dynamic shared memory
// (at most kMaxStages), leaving room for the kernels' static shared memory
// (per-warp work lists and copy cursors, < kStaticSmemReserve bytes).
constexpr size_t kStaticSmemReserve = 2048;
uint32_t ring_stages(size_t other);

// Synchronize `st`, read and clear the device status words, report timeouts.
int check_status(alv_ctx* ctx, cudaStream_t st);

// Entry points of one TU used by another.
int do_gemv(alv_ctx* ctx, Weight* w, int ntok, const void* x, int x_dtype, void* y, int y_dtype, cudaStream_t st);

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
int do_ffn(alv_ctx* ctx, Weight* w, int ntok, const FfnIo& io, cudaStream_t st);

// Sync block of an FFN stack's workspace: [status @0][GridBar @256][counters @1024].
inline size_t stack_sync_bytes(const Weight* w) {
  return kHeaderBytes + static_cast<size_t>(w->a.m.RT + w->b.m.RT) * 4;
}

void free_weight_memory(Weight* w);

}  // namespace alv
