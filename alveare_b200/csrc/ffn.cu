// Host side of the C ABI, part 3: the fused FFN (ffn_kernel), plain and with
// the decode layer's norm/residual glue fused in.
#include "launch.h"

namespace alv {
namespace {

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
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  if (!Partition::fits(p.gu.RT, p.gu.KT) || !Partition::fits(p.dn.RT, p.dn.KT))
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: matrix too large for one launch's partition");
  p.ptA = Partition::make(p.gu.RT, p.gu.KT, nctas, true);
  p.ptB = Partition::make(p.dn.RT, p.dn.KT, nctas);
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: H or I too large for the shared-memory fragment stage");
  // As for gemv: small FFNs request every stage at once, large ones one stage
  // per warp before the inputs are staged.
  const size_t wbytes = (static_cast<size_t>(p.gu.RT) * p.gu.KT + static_cast<size_t>(p.dn.RT) * p.dn.KT) * kUnitBytes;
  p.first = wbytes <= (size_t{16} << 20) ? p.nst : 1;
  const size_t smem = ring_smem_bytes(p.nst) + other;
  auto k = ffn_kernel<NT, SPLIT, FAST>;
  // Grid barrier between the phases: every CTA must be resident at once.
  int rc = prepare_kernel(ctx, k, smem, kThreadsPerCta, ctx->num_sms);
  if (rc) return rc;
  // Programmatic dependent launch: the weight stream starts while the
  // previous kernel finishes (the kernel waits before it reads its inputs).
  return launch_cooperative(ctx, k, p, ctx->num_sms, kThreadsPerCta, smem, st, true);
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


}  // namespace

// Both FFN matrices were repacked for the same dequant path.
int launch_ffn_params(alv_ctx* ctx, const FfnParams& p, bool split, uint32_t nt, cudaStream_t st) {
  return p.gu.fast ? launch_ffn_f<true>(ctx, p, split, nt, st) : launch_ffn_f<false>(ctx, p, split, nt, st);
}

int do_ffn(alv_ctx* ctx, Weight* w, int ntok, const FfnIo& io, cudaStream_t st) {
  if (ntok < 1 || ntok > 8) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: ntok must be 1..8");
  if (io.glue && w->H > 32u * kConsumerWarps * kGlueRegs)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_layer: H must be <= " + std::to_string(32u * kConsumerWarps * kGlueRegs));
  const bool split = !io.glue && io.x_dtype == ALV_F32;
  if (!io.glue && !x_aligned(io.x, io.x_dtype))
    return fail(ctx, ALV_ERR_ARG, std::string("ffn: x must be ") + (split ? "8" : "4") + "-byte aligned");
  const uint32_t nt = pow2_ceil(static_cast<uint32_t>(ntok));
  if (w->a.m.RT + w->b.m.RT > kMaxCounters) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn: too large");
  const size_t wsA = align_up(ws_floats(ctx, ntok) * 4, 256);
  const size_t wsB = align_up(ws_floats(ctx, ntok) * 4, 256);
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
  p.bar = reinterpret_cast<GridBar*>(bar_bytes(ctx));
  p.status = status_ptr(ctx);
  p.trace = ctx->trace;
  auto aligned16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  p.glue_tma = io.glue && aligned16(io.x_in) && (!io.down_in || aligned16(io.down_in));
  return launch_ffn_params(ctx, p, split, nt, st);
}

}  // namespace alv

using namespace alv;

extern "C" int alv_ffn(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y, int y_dtype,
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

extern "C" int alv_ffn_layer(alv_ctx* ctx, alv_handle h, int ntok, const uint16_t* x_in, const float* down_in,
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
