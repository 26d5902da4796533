// Host side of the C ABI declared in include/alveare_b200.h, part 1: the
// context, its scratch arena and status words, the weight registry with the
// load-time repack (reference 20-byte blocks -> unit layout), dequantize,
// the activation op, the stack finalize step and the host-buffer calls.
// Kernel families live in gemv.cu, ffn.cu, stack.cu, gemm.cu and decode.cu.
#include "launch.h"
#include "loadtime.cuh"

namespace alv {

// act = bf16(act_fn(gate) * up) elementwise, with the FFN epilogue's own
// functions (the reference's activation step,
// kernels/ffn_fused/ffn_compute_activation.cc:17-64, with model.py's exact
// formulas): gate, up, out bf16 bits.
__global__ void activation_kernel(int fn, uint32_t n, const uint16_t* __restrict__ gate,
                                  const uint16_t* __restrict__ up, uint16_t* __restrict__ out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float g = bf16_bits_to_f32(gate[i]), u = bf16_bits_to_f32(up[i]);
  out[i] = bf16_bits_rn(fn == 0 ? geglu_act(g, u) : swiglu_ref(g, u));
}

// Final residual of an FFN stack: one CTA of the consumer threads (the glue's thread
// layout, so the sums match the in-kernel glue bit for bit).
__global__ void __launch_bounds__(kConsumerWarps * 32, 1)
    ffn_stack_finalize_kernel(int ntok, uint32_t H, const uint16_t* x_in, const float* down_in, uint16_t* x_out,
                              float eps) {
  __shared__ float red[32];
  glue<false, true>(ntok, H, eps, Bf16In{x_in}, F32In{down_in}, Bf16Out{x_out}, XnOut{}, red);
}

int ensure_scratch(alv_ctx* ctx, size_t work_bytes) {
  if (!ctx->sync) {
    ALV_CUDA(ctx, dev_alloc(ctx, &ctx->sync, kSyncBytes));
    ALV_CUDA(ctx, cudaMemset(ctx->sync, 0, kSyncBytes));
  }
  if (ctx->scratch && ctx->scratch_bytes >= work_bytes) return ALV_OK;
  ALV_CUDA(ctx, cudaDeviceSynchronize());
  if (ctx->scratch) ctx->retired.push_back(ctx->scratch);
  ctx->scratch = nullptr;
  const size_t bytes = std::max(work_bytes, static_cast<size_t>(8) << 20);
  ALV_CUDA(ctx, dev_alloc(ctx, &ctx->scratch, bytes));
  ALV_CUDA(ctx, cudaMemset(ctx->scratch, 0, bytes));
  ctx->scratch_bytes = bytes;
  return ALV_OK;
}

uint32_t ring_stages(size_t other) {
  constexpr uint32_t kMaxStages = 24 / kUnitsPerStage;
  for (uint32_t nst = kMaxStages; nst >= 1; --nst)
    if (ring_smem_bytes(nst) + other + kStaticSmemReserve <= kMaxSmem) return nst;
  return 0;
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
    if (!w || (w->kind != 3 && w->kind != 4) || !w->ws) continue;
    uint32_t t = 0;
    ALV_CUDA(ctx, cudaMemcpy(&t, w->ws, sizeof(t), cudaMemcpyDeviceToHost));
    if (t) ALV_CUDA(ctx, cudaMemset(w->ws, 0, w->kind == 3 ? stack_sync_bytes(w.get()) : w->sync_bytes));
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

void free_weight_memory(Weight* w) {
  cudaFree(w->a.dev);
  cudaFree(w->b.dev);
  cudaFree(w->layers_dev);
  cudaFree(w->ws);
  if (w->connected)
    for (int q = 0; q < w->world; ++q)
      if (q != w->rank && w->xr[q]) cudaIpcCloseMemHandle(w->xr[q]);
  cudaFree(w->xlocal);
  if (w->model && w->model_free) w->model_free(w->model);
  w->model = nullptr;
}

namespace {

int io_buffers(alv_ctx* ctx, size_t bytes) {
  if (ctx->io && ctx->io_bytes >= bytes) return ALV_OK;
  if (ctx->io) ctx->retired.push_back(ctx->io);
  ctx->io = nullptr;
  ALV_CUDA(ctx, dev_alloc(ctx, &ctx->io, bytes));
  ctx->io_bytes = bytes;
  return ALV_OK;
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
  ALV_CUDA(ctx, dev_alloc(ctx, &info, 3 * sizeof(int)));
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
  ALV_CUDA(ctx, dev_alloc(ctx, &m.dev, std::max<size_t>(m.bytes, 16)));
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
  ALV_CUDA(ctx, dev_alloc(ctx, &d, std::max<size_t>(bytes, 16)));
  ALV_CUDA(ctx, cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice));
  *dev = d;
  *owned = d;
  return ALV_OK;
}

}  // namespace

int repack_rows(alv_ctx* ctx, const uint8_t* src, uint32_t rows, uint32_t K, Mat* out) {
  RepackSrc s{};
  s.a = src;
  s.b = nullptr;
  s.rows = rows;
  s.row_off = 0;
  s.row_bytes = static_cast<uint64_t>(K / 32) * 20;
  s.blk_off = 0;
  s.K = K;
  s.interleave8 = 0;
  s.RT = (rows + 15) / 16;
  s.KT = (K + 63) / 64;
  return build_mat(ctx, s, rows, K, out);
}

int repack_ffn(alv_ctx* ctx, const uint8_t* g, const uint8_t* u, const uint8_t* d, uint32_t H, uint32_t I,
               uint32_t i_begin, uint32_t i_end, Mat* gu, Mat* dn) {
  const uint32_t Il = i_end - i_begin;
  RepackSrc sa{};
  sa.a = g;
  sa.b = u;
  sa.rows = Il;
  sa.row_off = i_begin;
  sa.row_bytes = static_cast<uint64_t>(H / 32) * 20;
  sa.blk_off = 0;
  sa.K = H;
  sa.interleave8 = 1;
  sa.RT = (Il + 7) / 8;
  sa.KT = (H + 63) / 64;
  RepackSrc sb{};
  sb.a = d;
  sb.b = nullptr;
  sb.rows = H;
  sb.row_off = 0;
  sb.row_bytes = static_cast<uint64_t>(I / 32) * 20;
  sb.blk_off = i_begin / 32;
  sb.K = Il;
  sb.interleave8 = 0;
  sb.RT = (H + 15) / 16;
  sb.KT = (Il + 63) / 64;
  // One kernel dequantizes both matrices: they share the dequant path.
  Survey sva, svb;
  int rc;
  if (!(rc = survey_mat(ctx, sa, &sva)) && !(rc = survey_mat(ctx, sb, &svb))) {
    if (!(sva.fast && svb.fast)) sva = svb = Survey{};
    rc = repack_mat(ctx, sa, sva, Il, H, gu);
    if (!rc) rc = repack_mat(ctx, sb, svb, H, Il, dn);
  }
  if (rc) {
    cudaFree(gu->dev);
    cudaFree(dn->dev);
    gu->dev = dn->dev = nullptr;
  }
  return rc;
}

}  // namespace alv

using namespace alv;

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
  for (auto& w : ctx->weights)
    if (w) free_weight_memory(w.get());
  cudaFree(ctx->sync);
  cudaFree(ctx->scratch);
  cudaFree(ctx->io);
  for (void* q : ctx->retired) cudaFree(q);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return ALV_OK;
}

int alv_ctx_info(alv_ctx* ctx, int64_t* info) {
  if (!ctx || !info) return ALV_ERR_ARG;
  info[0] = ctx->device;
  info[1] = ctx->num_sms;
  info[2] = static_cast<int64_t>(ctx->scratch_bytes);
  info[3] = static_cast<int64_t>(ctx->io_bytes);
  info[4] = ctx->allocs;
  info[5] = static_cast<int64_t>(ctx->weights.size());
  info[6] = info[7] = 0;
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
  auto w = std::make_unique<Weight>();
  w->kind = 2;
  w->H = static_cast<uint32_t>(H);
  w->I = static_cast<uint32_t>(I);
  w->i_begin = static_cast<uint32_t>(i_begin);
  w->i_end = static_cast<uint32_t>(i_end);
  w->act = act;
  rc = repack_ffn(ctx, g, u, d, w->H, w->I, w->i_begin, w->i_end, &w->a, &w->b);
  cudaFree(og);
  cudaFree(ou);
  cudaFree(od);
  if (rc) return rc;
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
  free_weight_memory(w);
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
    ALV_CUDA(ctx, dev_alloc(ctx, &tmp, static_cast<size_t>(rows_all) * K * 2));
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

int alv_activation(alv_ctx* ctx, int act, int n, const uint16_t* gate, const uint16_t* up, uint16_t* out,
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

}  // extern "C"
