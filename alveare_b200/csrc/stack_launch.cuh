// Launch of the one-launch FFN stack kernel (ffn_stack_kernel), one
// explicit instantiation per dequant path and tensor-parallel mode in its own
// translation unit (stack_k_*.cu) so the variants compile in parallel.
#pragma once

#include "internal.h"
#include "kernels.cuh"

namespace alv {

constexpr int kStackMaxTokens = 4;

template <int NT, bool FAST, bool TP>
int launch_stack_t(alv_ctx* ctx, StackParams p, cudaStream_t st) {
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  if (!Partition::fits(p.gu.RT, p.gu.KT) || !Partition::fits(p.dn.RT, p.dn.KT))
    return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack: matrix too large for one launch's partition");
  p.ptA = Partition::make(p.gu.RT, p.gu.KT, nctas, true);
  // Tensor parallelism: whole down rows per CTA, so each rank pushes exactly
  // its H values per token and the gather reads one value per rank (the
  // imbalance of whole rows costs less than the partials' exchange).
  p.ptB = Partition::make(p.dn.RT, p.dn.KT, nctas, TP);
  const size_t other = stack_smem_bytes(0, p.gu.KT, p.dn.KT, NT, p.H, p.ntok, p.dn.RT, nctas);
  p.nst = ring_stages(other);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack: H, I or ntok too large for shared memory");
  const size_t smem = stack_smem_bytes(p.nst, p.gu.KT, p.dn.KT, NT, p.H, p.ntok, p.dn.RT, nctas);
  auto k = ffn_stack_kernel<NT, FAST, TP>;
  // Grid barriers between the phases: every CTA must be resident at once.
  int rc = prepare_kernel(ctx, k, smem, kThreadsPerCta, ctx->num_sms);
  if (rc) return rc;
  return launch_cooperative(ctx, k, p, ctx->num_sms, kThreadsPerCta, smem, st);
}

// Instantiated for each (FAST, TP) in stack_k_*.cu.
template <bool FAST, bool TP>
int launch_stack_f(alv_ctx* ctx, const StackParams& p, uint32_t nt, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_stack_t<1, FAST, TP>(ctx, p, st);
    case 2: return launch_stack_t<2, FAST, TP>(ctx, p, st);
    case 4: return launch_stack_t<4, FAST, TP>(ctx, p, st);
  }
  return fail(ctx, ALV_ERR_UNSUPPORTED, "ffn_stack: unsupported token count");
}

// Compiled only in their own translation units.
extern template int launch_stack_f<true, false>(alv_ctx*, const StackParams&, uint32_t, cudaStream_t);
extern template int launch_stack_f<true, true>(alv_ctx*, const StackParams&, uint32_t, cudaStream_t);
extern template int launch_stack_f<false, false>(alv_ctx*, const StackParams&, uint32_t, cudaStream_t);
extern template int launch_stack_f<false, true>(alv_ctx*, const StackParams&, uint32_t, cudaStream_t);

}  // namespace alv
