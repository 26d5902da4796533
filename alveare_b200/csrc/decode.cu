// Host side of the C ABI, part 6: the Llama greedy decode loop on the GPU.
//
// The reference runs the decode step on the host in numpy (runtime/py/
// model.py:821-934) and sends only the matmuls to the NPU (QKV, O and the
// fused FFN per layer, plus the LM head: runtime/cpp/src/model.cpp:297, 379,
// 404; generator.cpp:28-52).  Here the whole step runs on the device: the
// Q4 matmuls on the streaming gemv / fused-FFN kernels, the glue (embedding,
// RMSNorm, RoPE, KV cache, attention, residuals, argmax) in decode.cuh.
// The step reads its position and token from device memory, so it is
// captured once into a CUDA graph (one with the LM head and argmax, one
// without for prompt tokens) and replayed with no host work per token.
#include "decode.cuh"
#include "launch.h"
#include "llama_step.cuh"

namespace alv {
namespace {

const char* const kProj[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};

struct LlamaModel {
  alv_llama_config cfg{};
  // reference-layout packed sources on the device until the model is built
  std::map<std::string, uint8_t*> raw;
  std::map<std::string, uint32_t> raw_rows;
  bool built = false;
  std::vector<Mat> qkv, o, gu, dn;
  Mat lm;
  uint16_t* emb = nullptr;     // f16 [vocab][H]
  float* norms = nullptr;      // [2L + 1][H]: attn_norm l at 2l, ffn_norm l at 2l+1, output norm at 2L
  uint16_t* rope = nullptr;    // bf16 [max_seq][2 hd]
  uint16_t* kcache = nullptr;  // bf16 [L][nkv][max_seq][hd]
  uint16_t* vcache = nullptr;
  uint16_t* act16 = nullptr;   // activation buffers (bf16)
  uint16_t *x = nullptr, *xn = nullptr, *qkvb = nullptr, *q = nullptr, *attn = nullptr, *proj = nullptr,
           *logits = nullptr;
  DecodeState* state = nullptr;
  // Host copy of state->pos (every step consumes one position), so that no
  // run enqueues a step at a position >= max_seq: the device kernels index
  // the KV cache and the RoPE table with the position unchecked.
  int64_t next_pos = 0;
  int* tokens = nullptr;       // [max_seq + 1] token at each position
  int* pred = nullptr;         // [max_seq + 1] the argmax each logits step predicted for the next position
  // workspace (Weight::ws): [sync block: status, grid barrier, counters][split-K partials][FFN act]
  uint32_t* status = nullptr;
  GridBar* bar = nullptr;
  uint32_t* cnt = nullptr;
  float *ws_gemv = nullptr, *wsA = nullptr, *wsB = nullptr;
  uint8_t* act = nullptr;
  // one-launch step (llama_step_kernel): per-layer weight table, fp32 down
  // rows, CTA partials of shared down rows, argmax candidates
  LlamaLayerW* layers_dev = nullptr;
  float *down32 = nullptr, *dws = nullptr, *cand_v = nullptr;
  int* cand_i = nullptr;
  bool one_launch = false;  // the one-launch step is used (see use_one_launch)
  // batched prefill (allocated on first use): rows of kPrefillRows tokens
  uint16_t *px = nullptr, *pxn = nullptr, *pqkv = nullptr, *pq = nullptr, *pattn = nullptr, *pproj = nullptr,
           *pgu = nullptr, *pact = nullptr;
  std::vector<void*> owned;
  cudaGraphExec_t g_prefill = nullptr, g_decode = nullptr;
  bool loaded_emb = false, loaded_rope = false;
  std::vector<bool> loaded_norm;

  size_t kv_elems() const {
    return static_cast<size_t>(cfg.layers) * cfg.kv_heads * cfg.max_seq * cfg.head_dim;
  }
};

void free_model(void* p) {
  auto* m = static_cast<LlamaModel*>(p);
  if (m->g_prefill) cudaGraphExecDestroy(m->g_prefill);
  if (m->g_decode) cudaGraphExecDestroy(m->g_decode);
  for (auto& kv : m->raw) cudaFree(kv.second);
  for (auto* v : {&m->qkv, &m->o, &m->gu, &m->dn})
    for (auto& mat : *v) cudaFree(mat.dev);
  cudaFree(m->lm.dev);
  for (void* q : m->owned) cudaFree(q);
  delete m;
}

template <class T>
int model_alloc(alv_ctx* ctx, LlamaModel* m, T** p, size_t bytes) {
  ALV_CUDA(ctx, dev_alloc(ctx, p, std::max<size_t>(bytes, 16)));
  m->owned.push_back(*p);
  return ALV_OK;
}

LlamaModel* get_model(alv_ctx* ctx, alv_handle h) {
  Weight* w = get_weight(ctx, h, 4);
  return w ? static_cast<LlamaModel*>(w->model) : nullptr;
}

// Column count of a projection's packed matrix.
uint32_t proj_cols(const alv_llama_config& c, const std::string& proj) {
  if (proj == "ffn_down") return static_cast<uint32_t>(c.intermediate);
  if (proj == "attn_output") return static_cast<uint32_t>(c.heads * c.head_dim);
  return static_cast<uint32_t>(c.hidden);
}
// Rows of a projection the model uses (the on-disk K / V are padded).
uint32_t proj_rows(const alv_llama_config& c, const std::string& proj) {
  if (proj == "attn_q") return static_cast<uint32_t>(c.heads * c.head_dim);
  if (proj == "attn_k" || proj == "attn_v") return static_cast<uint32_t>(c.kv_heads * c.head_dim);
  if (proj == "ffn_gate" || proj == "ffn_up") return static_cast<uint32_t>(c.intermediate);
  return static_cast<uint32_t>(c.hidden);
}

int copy_in(alv_ctx* ctx, void* dst, const void* src, size_t bytes, int on_device) {
  ALV_CUDA(ctx, cudaMemcpy(dst, src, bytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  return ALV_OK;
}

// The one-launch step needs one dequant path for every matrix (its kernel is
// compiled per path), head_dim <= 128 (the attention threads hold q, k, v),
// at most one CTA per query head per SM, and room for its rings.  Otherwise,
// or when the config asks for it, the step runs as separate kernels.
// llama_step_kernel's static shared memory beyond the reserve ring_stages
// keeps (work lists and unit ranges of five matrices per warp).
constexpr size_t kLlamaStaticSmem = 2048;

size_t llama_other_smem(const LlamaModel* m, uint32_t nctas) {
  const alv_llama_config& c = m->cfg;
  const uint32_t kt_max = std::max({m->qkv[0].m.KT, m->o[0].m.KT, m->gu[0].m.KT, m->dn[0].m.KT, m->lm.m.KT});
  return llama_smem(0, kt_max, c.hidden, c.head_dim, c.max_seq, m->dn[0].m.RT, nctas).end;
}

int build_one_launch(alv_ctx* ctx, LlamaModel* m) {
  const alv_llama_config& c = m->cfg;
  m->one_launch = false;
  if (c.per_kernel_step == 1) return ALV_OK;
  const uint32_t fast = m->lm.m.fast;
  for (int l = 0; l < c.layers; ++l)
    for (const Mat* mat : {&m->qkv[l], &m->o[l], &m->gu[l], &m->dn[l]})
      if (mat->m.fast != fast) return ALV_OK;
  if (c.head_dim > 128 || c.heads > ctx->num_sms) return ALV_OK;
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  if (!ring_stages(llama_other_smem(m, nctas) + kLlamaStaticSmem)) return ALV_OK;
  for (const Mat* mat : {&m->qkv[0], &m->o[0], &m->gu[0], &m->dn[0], &m->lm})
    if (!Partition::fits(mat->m.RT, mat->m.KT)) return ALV_OK;
  std::vector<LlamaLayerW> lw(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const Mat* mats[4] = {&m->qkv[l], &m->o[l], &m->gu[l], &m->dn[l]};
    for (int k = 0; k < 4; ++k) {
      lw[l].mat[k] = mats[k]->m.units;
      lw[l].mul[k] = mats[k]->m.scale_mul;
    }
  }
  int rc;
  if ((rc = model_alloc(ctx, m, &m->layers_dev, lw.size() * sizeof(LlamaLayerW))) ||
      (rc = model_alloc(ctx, m, &m->down32, static_cast<size_t>(c.hidden) * 4)) ||
      (rc = model_alloc(ctx, m, &m->dws, ws_floats(ctx, 1) * 4)) ||
      (rc = model_alloc(ctx, m, &m->cand_v, nctas * 4)) || (rc = model_alloc(ctx, m, &m->cand_i, nctas * 4)))
    return rc;
  ALV_CUDA(ctx, cudaMemcpy(m->layers_dev, lw.data(), lw.size() * sizeof(LlamaLayerW), cudaMemcpyHostToDevice));
  m->one_launch = true;
  return ALV_OK;
}

template <bool FAST>
int launch_llama_step_t(alv_ctx* ctx, const LlamaStepParams& p, size_t smem, cudaStream_t st) {
  auto k = llama_step_kernel<FAST>;
  // Grid barriers between the phases: every CTA must be resident at once.
  int rc = prepare_kernel(ctx, k, smem, kThreadsPerCta, ctx->num_sms);
  if (rc) return rc;
  return launch_cooperative(ctx, k, p, ctx->num_sms, kThreadsPerCta, smem, st);
}

// One decode step as one launch of llama_step_kernel.
int launch_llama_step(alv_ctx* ctx, LlamaModel* m, bool logits, cudaStream_t st) {
  const alv_llama_config& c = m->cfg;
  const uint32_t nctas = static_cast<uint32_t>(ctx->num_sms);
  LlamaStepParams p{};
  p.layers = m->layers_dev;
  p.lm = m->lm.m.units;
  p.lm_mul = m->lm.m.scale_mul;
  p.L = static_cast<uint32_t>(c.layers);
  const Mat* mats[kLlamaMats] = {&m->qkv[0], &m->o[0], &m->gu[0], &m->dn[0], &m->lm};
  for (int k = 0; k < kLlamaMats; ++k) {
    const Q4Mat& q = mats[k]->m;
    p.mat[k] = q;
    // the separate-kernel step's partitions: gemv_kernel (row-aligned when
    // RT * 4 >= grid) for qkv, o and the LM head; ffn_kernel's for gate/up
    // (row-aligned) and down
    const bool aligned = k == 2 ? true : (k == 3 ? false : q.RT * 4 >= nctas);
    p.pt[k] = Partition::make(q.RT, q.KT, nctas, aligned);
  }
  p.H = c.hidden;
  p.I = c.intermediate;
  p.nq = c.heads;
  p.nkv = c.kv_heads;
  p.hd = c.head_dim;
  p.max_seq = c.max_seq;
  p.V = c.vocab;
  p.eps = c.rms_eps;
  p.attn_scale = 1.0 / std::sqrt(static_cast<double>(c.head_dim));
  p.logits = logits ? 1 : 0;
  p.emb = m->emb;
  p.norms = m->norms;
  p.rope = m->rope;
  p.kcache = m->kcache;
  p.vcache = m->vcache;
  p.state = m->state;
  p.tokens = m->tokens;
  p.pred = m->pred;
  p.qkvb = m->qkvb;
  p.attn = m->attn;
  p.proj = m->proj;
  p.logit16 = m->logits;
  p.act = m->act;
  p.down = m->down32;
  p.dws = m->dws;
  p.fx = Fixup{m->ws_gemv, m->cnt};
  p.cand_v = m->cand_v;
  p.cand_i = m->cand_i;
  p.bar = m->bar;
  p.status = m->status;
  p.trace = ctx->trace;
  const size_t other = llama_other_smem(m, nctas);
  p.nst = ring_stages(other + kLlamaStaticSmem);
  if (!p.nst) return fail(ctx, ALV_ERR_UNSUPPORTED, "llama: the one-launch step does not fit in shared memory");
  const size_t smem = ring_smem_bytes(p.nst) + other;
  return m->lm.m.fast ? launch_llama_step_t<true>(ctx, p, smem, st) : launch_llama_step_t<false>(ctx, p, smem, st);
}

// Repack every loaded matrix into the unit layout (once, before the first step).
int build_model(alv_ctx* ctx, Weight* w, LlamaModel* m) {
  if (m->built) return ALV_OK;
  const alv_llama_config& c = m->cfg;
  const int L = c.layers;
  if (!m->loaded_emb) return fail(ctx, ALV_ERR_ARG, "llama: token_embd not loaded");
  if (!m->loaded_rope) return fail(ctx, ALV_ERR_ARG, "llama: rope_table not loaded");
  for (int i = 0; i < 2 * L + 1; ++i)
    if (!m->loaded_norm[i]) return fail(ctx, ALV_ERR_ARG, "llama: a norm weight is not loaded (" + std::to_string(i) + ")");
  if (!m->raw.count("lm_head_packed")) return fail(ctx, ALV_ERR_ARG, "llama: lm_head_packed not loaded");
  for (int l = 0; l < L; ++l)
    for (const char* p : kProj)
      if (!m->raw.count("blk." + std::to_string(l) + "." + p + ".weight_packed"))
        return fail(ctx, ALV_ERR_ARG, "llama: blk." + std::to_string(l) + "." + p + ".weight_packed not loaded");
  const uint32_t H = c.hidden, I = c.intermediate;
  const uint32_t nq = c.heads * c.head_dim, nkv = c.kv_heads * c.head_dim;
  const size_t rowb = static_cast<size_t>(H / 32) * 20;
  m->qkv.resize(L);
  m->o.resize(L);
  m->gu.resize(L);
  m->dn.resize(L);
  int rc = ALV_OK;
  uint8_t* cat = nullptr;
  ALV_CUDA(ctx, dev_alloc(ctx, &cat, (nq + 2 * nkv) * rowb));
  for (int l = 0; l < L && !rc; ++l) {
    auto name = [&](const char* p) { return "blk." + std::to_string(l) + "." + p + ".weight_packed"; };
    // [q | k | v] rows in one matrix: one gemv per layer for the three
    // projections (each row is the same dot product as in its own matrix).
    cudaMemcpy(cat, m->raw[name("attn_q")], nq * rowb, cudaMemcpyDeviceToDevice);
    cudaMemcpy(cat + nq * rowb, m->raw[name("attn_k")], nkv * rowb, cudaMemcpyDeviceToDevice);
    cudaMemcpy(cat + (nq + nkv) * rowb, m->raw[name("attn_v")], nkv * rowb, cudaMemcpyDeviceToDevice);
    if ((rc = repack_rows(ctx, cat, nq + 2 * nkv, H, &m->qkv[l]))) break;
    if ((rc = repack_rows(ctx, m->raw[name("attn_output")], H, nq, &m->o[l]))) break;  // (H, heads*head_dim)
    rc = repack_ffn(ctx, m->raw[name("ffn_gate")], m->raw[name("ffn_up")], m->raw[name("ffn_down")], H, I, 0, I,
                    &m->gu[l], &m->dn[l]);
  }
  cudaFree(cat);
  if (!rc) rc = repack_rows(ctx, m->raw["lm_head_packed"], c.vocab, H, &m->lm);
  if (rc) return rc;
  for (auto& kv : m->raw) cudaFree(kv.second);
  m->raw.clear();
  // workspace
  uint32_t rt_max = m->lm.m.RT;
  for (int l = 0; l < L; ++l) {
    rt_max = std::max({rt_max, m->qkv[l].m.RT, m->o[l].m.RT, m->gu[l].m.RT + m->dn[l].m.RT});
  }
  w->sync_bytes = kHeaderBytes + static_cast<size_t>(rt_max) * 4;
  const size_t wsf = ws_floats(ctx, 1) * 4;
  const size_t o_ws = align_up(w->sync_bytes, 256);
  const size_t o_a = o_ws + align_up(wsf, 256), o_b = o_a + align_up(wsf, 256), o_act = o_b + align_up(wsf, 256);
  const size_t total = o_act + align_up(frag_bytes(m->dn[0].m.KT, 1), 256);
  ALV_CUDA(ctx, dev_alloc(ctx, &w->ws, total));  // freed with the weight
  ALV_CUDA(ctx, cudaMemset(w->ws, 0, total));
  w->ws_bytes = total;
  m->status = reinterpret_cast<uint32_t*>(w->ws);
  m->bar = reinterpret_cast<GridBar*>(w->ws + 256);
  m->cnt = reinterpret_cast<uint32_t*>(w->ws + kHeaderBytes);
  m->ws_gemv = reinterpret_cast<float*>(w->ws + o_ws);
  m->wsA = reinterpret_cast<float*>(w->ws + o_a);
  m->wsB = reinterpret_cast<float*>(w->ws + o_b);
  m->act = w->ws + o_act;
  if ((rc = build_one_launch(ctx, m))) return rc;
  m->built = true;
  return ALV_OK;
}

int gemv_into(alv_ctx* ctx, LlamaModel* m, const Mat& mat, const uint16_t* x, uint16_t* y, cudaStream_t st) {
  GemvParams p{};
  p.m = mat.m;
  p.x = XSrc{x, 1, 1, mat.cols, mat.cols};
  p.epi = RowsEpi{nullptr, y, mat.rows, mat.rows, mat.m.scale_mul};
  p.fx = Fixup{m->ws_gemv, m->cnt};
  p.status = m->status;
  return launch_gemv_params(ctx, p, false, 1, st, true);
}

int ffn_into(alv_ctx* ctx, LlamaModel* m, int l, const uint16_t* x, uint16_t* y, cudaStream_t st) {
  FfnParams p{};
  p.gu = m->gu[l].m;
  p.dn = m->dn[l].m;
  p.H = m->cfg.hidden;
  p.I = m->cfg.intermediate;
  p.fn = ALV_ACT_SILU;
  p.ntok = 1;
  p.x = XSrc{x, 1, 1, p.H, p.H};
  p.out = RowsEpi{nullptr, y, p.H, p.H, m->dn[l].m.scale_mul};
  p.act = m->act;
  p.fxA = Fixup{m->wsA, m->cnt};
  p.fxB = Fixup{m->wsB, m->cnt + m->gu[l].m.RT};
  p.bar = m->bar;
  p.status = m->status;
  return launch_ffn_params(ctx, p, false, 1, st);
}

// ---------------------------------------------------------------------------
// Batched prefill (the reference's run_layer_batch, runtime/cpp/src/model.cpp:
// 422-571, there gemma4-only with B = 16 padded rows): prompt positions go
// through each layer kPrefillRows at a time, every projection a tcgen05
// gemm over the whole batch (the fused gate/up matrix in one gemm, SwiGLU on
// its interleaved output, the down projection in one gemm: no K split is
// needed), the glue as the decode step's kernels over rows (one CTA per row;
// causal attention: row b attends to positions <= pos0 + b, its own K/V
// appended first).  The roundings are the decode step's; the gemm sums in
// another order, so the cache and logits agree with the token-by-token path
// to the last few bf16 bits, not bit for bit.
// ---------------------------------------------------------------------------
constexpr int kPrefillRows = 256;

int ensure_prefill(alv_ctx* ctx, LlamaModel* m) {
  if (m->px) return ALV_OK;
  const alv_llama_config& c = m->cfg;
  const size_t R = kPrefillRows, H = c.hidden, nq = static_cast<size_t>(c.heads) * c.head_dim;
  const size_t nqkv = nq + 2 * static_cast<size_t>(c.kv_heads) * c.head_dim;
  const size_t ngu = static_cast<size_t>(m->gu[0].m.RT) * 16;
  int rc;
  if ((rc = model_alloc(ctx, m, &m->px, R * H * 2)) || (rc = model_alloc(ctx, m, &m->pxn, R * H * 2)) ||
      (rc = model_alloc(ctx, m, &m->pqkv, R * nqkv * 2)) || (rc = model_alloc(ctx, m, &m->pq, R * nq * 2)) ||
      (rc = model_alloc(ctx, m, &m->pattn, R * nq * 2)) || (rc = model_alloc(ctx, m, &m->pproj, R * H * 2)) ||
      (rc = model_alloc(ctx, m, &m->pgu, R * ngu * 2)) ||
      (rc = model_alloc(ctx, m, &m->pact, R * static_cast<size_t>(c.intermediate) * 2)))
    return rc;
  return ALV_OK;
}

// Positions [pos0, pos0 + n) of tokens[] (n <= kPrefillRows) through every
// layer: their K/V enter the cache.  No LM head (the last prompt token's
// logits come from the first decode step).
int prefill_rows(alv_ctx* ctx, LlamaModel* m, int pos0, int n, cudaStream_t st) {
  const alv_llama_config& c = m->cfg;
  const int H = c.hidden, L = c.layers, I = c.intermediate;
  const uint32_t nq = c.heads * c.head_dim;
  const float eps = c.rms_eps;
  const size_t kv_layer = static_cast<size_t>(c.kv_heads) * c.max_seq * c.head_dim;
  const size_t attn_smem = static_cast<size_t>(c.head_dim + c.max_seq + kAttnThreads) * sizeof(float);
  int rc = launch_ex(ctx, embed_norm_kernel, dim3(n), dim3(kDecodeThreads), 0, st, false,
                     static_cast<const uint16_t*>(m->emb), static_cast<const DecodeState*>(nullptr), pos0,
                     static_cast<const int*>(m->tokens), H, static_cast<const float*>(m->norms), eps, m->px, m->pxn);
  if (rc) return rc;
  for (int l = 0; l < L; ++l) {
    const Mat& q = m->qkv[l];
    if ((rc = launch_gemm_mat(ctx, q.m, q.rows, q.cols, n, m->pxn, nullptr, m->pqkv, st))) return rc;
    const RopeParams rp{m->pqkv, m->rope, nullptr, pos0, m->kcache + l * kv_layer, m->vcache + l * kv_layer, m->pq,
                        c.heads, c.kv_heads, c.head_dim, c.max_seq};
    if ((rc = launch_ex(ctx, rope_cache_kernel, dim3(n), dim3(kDecodeThreads), 0, st, false, rp))) return rc;
    const AttnParams ap{m->pq, m->kcache + l * kv_layer, m->vcache + l * kv_layer, nullptr, pos0, m->pattn,
                        c.heads, c.kv_heads, c.head_dim, c.max_seq, 1.0 / std::sqrt(static_cast<double>(c.head_dim))};
    if ((rc = launch_ex(ctx, attention_kernel, dim3(c.heads, n), dim3(kAttnThreads), attn_smem, st, false, ap)))
      return rc;
    const Mat& o = m->o[l];
    if ((rc = launch_gemm_mat(ctx, o.m, o.rows, nq, n, m->pattn, nullptr, m->pproj, st))) return rc;
    if ((rc = launch_ex(ctx, residual_norm_kernel, dim3(n), dim3(kDecodeThreads), 0, st, false, m->px,
                        static_cast<const uint16_t*>(m->pproj), H,
                        static_cast<const float*>(m->norms + static_cast<size_t>(2 * l + 1) * H), eps, m->pxn)))
      return rc;
    const Mat& gu = m->gu[l];
    if ((rc = launch_gemm_mat(ctx, gu.m, gu.m.RT * 16, H, n, m->pxn, nullptr, m->pgu, st))) return rc;
    if ((rc = launch_ex(ctx, swiglu_rows_kernel, dim3((I + 255) / 256, n), dim3(256), 0, st, false,
                        static_cast<const uint16_t*>(m->pgu), I, m->pact)))
      return rc;
    const Mat& dn = m->dn[l];
    if ((rc = launch_gemm_mat(ctx, dn.m, H, I, n, m->pact, nullptr, m->pproj, st))) return rc;
    if ((rc = launch_ex(ctx, residual_norm_kernel, dim3(n), dim3(kDecodeThreads), 0, st, false, m->px,
                        static_cast<const uint16_t*>(m->pproj), H,
                        static_cast<const float*>(m->norms + static_cast<size_t>(2 * l + 2) * H), eps, m->pxn)))
      return rc;
  }
  return launch_ex(ctx, set_pos_kernel, dim3(1), dim3(32), 0, st, false, m->state, pos0 + n);
}

// One decode step: the token at state.pos through every layer; with
// `logits`, the LM head and the argmax that writes the next token.
int enqueue_step(alv_ctx* ctx, LlamaModel* m, bool logits, cudaStream_t st) {
  if (m->one_launch) return launch_llama_step(ctx, m, logits, st);
  const alv_llama_config& c = m->cfg;
  const int H = c.hidden, L = c.layers;
  const float eps = c.rms_eps;
  int rc = launch_ex(ctx, embed_norm_kernel, dim3(1), dim3(kDecodeThreads), 0, st, true,
                     static_cast<const uint16_t*>(m->emb), static_cast<const DecodeState*>(m->state), 0,
                     static_cast<const int*>(m->tokens), H, static_cast<const float*>(m->norms), eps, m->x, m->xn);
  if (rc) return rc;
  const size_t kv_layer = static_cast<size_t>(c.kv_heads) * c.max_seq * c.head_dim;
  const size_t attn_smem = static_cast<size_t>(c.head_dim + c.max_seq + kAttnThreads) * sizeof(float);
  for (int l = 0; l < L; ++l) {
    if ((rc = gemv_into(ctx, m, m->qkv[l], m->xn, m->qkvb, st))) return rc;
    const RopeParams rp{m->qkvb, m->rope, m->state, 0, m->kcache + l * kv_layer, m->vcache + l * kv_layer, m->q,
                        c.heads, c.kv_heads, c.head_dim, c.max_seq};
    if ((rc = launch_ex(ctx, rope_cache_kernel, dim3(1), dim3(kDecodeThreads), 0, st, true, rp))) return rc;
    const AttnParams ap{m->q, m->kcache + l * kv_layer, m->vcache + l * kv_layer, m->state, 0, m->attn,
                        c.heads, c.kv_heads, c.head_dim, c.max_seq, 1.0 / std::sqrt(static_cast<double>(c.head_dim))};
    if ((rc = launch_ex(ctx, attention_kernel, dim3(c.heads), dim3(kAttnThreads), attn_smem, st, true, ap))) return rc;
    if ((rc = gemv_into(ctx, m, m->o[l], m->attn, m->proj, st))) return rc;
    if ((rc = launch_ex(ctx, residual_norm_kernel, dim3(1), dim3(kDecodeThreads), 0, st, true, m->x,
                        static_cast<const uint16_t*>(m->proj), H, static_cast<const float*>(m->norms + (2 * l + 1) * H),
                        eps, m->xn)))
      return rc;
    if ((rc = ffn_into(ctx, m, l, m->xn, m->proj, st))) return rc;
    if ((rc = launch_ex(ctx, residual_norm_kernel, dim3(1), dim3(kDecodeThreads), 0, st, true, m->x,
                        static_cast<const uint16_t*>(m->proj), H, static_cast<const float*>(m->norms + (2 * l + 2) * H),
                        eps, m->xn)))
      return rc;
  }
  if (logits && (rc = gemv_into(ctx, m, m->lm, m->xn, m->logits, st))) return rc;
  if ((rc = launch_ex(ctx, argmax_advance_kernel, dim3(1), dim3(kDecodeThreads), 0, st, true,
                      static_cast<const uint16_t*>(logits ? m->logits : nullptr), c.vocab, m->state, m->tokens,
                      m->pred)))
    return rc;
  return ALV_OK;
}

int capture_step(alv_ctx* ctx, LlamaModel* m, bool logits, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  ALV_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_step(ctx, m, logits, ctx->stream);
  const cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(ctx, ALV_ERR_CUDA, std::string("llama: graph capture: ") + cudaGetErrorString(e));
  const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return fail(ctx, ALV_ERR_CUDA, std::string("llama: graph instantiate: ") + cudaGetErrorString(ie));
  return ALV_OK;
}

// Zero the KV cache and set the position to 0 with `prompt` in tokens[].
int start_sequence(alv_ctx* ctx, LlamaModel* m, const int32_t* prompt, int n, cudaStream_t st) {
  ALV_CUDA(ctx, cudaMemsetAsync(m->kcache, 0, m->kv_elems() * 2, st));
  ALV_CUDA(ctx, cudaMemsetAsync(m->vcache, 0, m->kv_elems() * 2, st));
  ALV_CUDA(ctx, cudaMemcpyAsync(m->tokens, prompt, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st));
  const DecodeState s{0, n, {0, 0}};
  ALV_CUDA(ctx, cudaMemcpyAsync(m->state, &s, sizeof(s), cudaMemcpyHostToDevice, st));
  ALV_CUDA(ctx, cudaStreamSynchronize(st));  // the host copies above read stack / caller memory
  m->next_pos = 0;
  return ALV_OK;
}

// Build, warm up (so no kernel attribute or module set-up happens during
// capture) and capture both step graphs.
int prepare_model(alv_ctx* ctx, Weight* w, LlamaModel* m) {
  int rc = build_model(ctx, w, m);
  if (rc) return rc;
  if (m->g_decode) return ALV_OK;
  const int32_t zero = 0;
  if ((rc = start_sequence(ctx, m, &zero, 1, ctx->stream))) return rc;
  if ((rc = enqueue_step(ctx, m, true, ctx->stream))) return rc;
  m->next_pos = 1;
  if ((rc = check_status(ctx, ctx->stream))) return rc;
  if ((rc = capture_step(ctx, m, false, &m->g_prefill))) return rc;
  return capture_step(ctx, m, true, &m->g_decode);
}

}  // namespace
}  // namespace alv

using namespace alv;

extern "C" int alv_llama_create(alv_ctx* ctx, const alv_llama_config* cfg, alv_handle* out) {
  if (!ctx || !cfg || !out) return fail(ctx, ALV_ERR_ARG, "llama_create: bad argument");
  const alv_llama_config& c = *cfg;
  if (c.hidden <= 0 || c.intermediate <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.head_dim <= 0 || c.layers <= 0 ||
      c.vocab <= 0 || c.max_seq <= 1 || !(c.rms_eps > 0.f))
    return fail(ctx, ALV_ERR_ARG, "llama_create: every size must be positive");
  if (c.hidden % 64 || c.intermediate % 64 || c.head_dim % 8 || c.head_dim > 256 || c.heads % c.kv_heads ||
      (c.heads * c.head_dim) % 64)
    return fail(ctx, ALV_ERR_SHAPE, "llama_create: hidden, intermediate and heads*head_dim must be multiples of 64, "
                                    "head_dim a multiple of 8 (<= 256), heads a multiple of kv_heads");
  if (c.hidden > kDecodeThreads * kDecodePer)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "llama_create: hidden must be <= " + std::to_string(kDecodeThreads * kDecodePer));
  if (kAttnThreads % c.head_dim || (c.head_dim + c.max_seq + kAttnThreads) * sizeof(float) > 48 * 1024)
    return fail(ctx, ALV_ERR_UNSUPPORTED, "llama_create: head_dim must divide 256 and max_seq fit the attention stage");
  int rc = set_device(ctx);
  if (rc) return rc;
  auto w = std::make_unique<Weight>();
  w->kind = 4;
  auto* m = new LlamaModel();
  w->model = m;
  w->model_free = free_model;
  m->cfg = c;
  m->loaded_norm.assign(2 * c.layers + 1, false);
  const size_t H = c.hidden;
  const size_t nq = static_cast<size_t>(c.heads) * c.head_dim, nkv = static_cast<size_t>(c.kv_heads) * c.head_dim;
  const size_t acts = 2 * H + (nq + 2 * nkv) + 2 * nq + H + align_up(c.vocab, 8);
  if ((rc = model_alloc(ctx, m, &m->emb, static_cast<size_t>(c.vocab) * H * 2)) ||
      (rc = model_alloc(ctx, m, &m->norms, (2 * c.layers + 1) * H * 4)) ||
      (rc = model_alloc(ctx, m, &m->rope, static_cast<size_t>(c.max_seq) * 2 * c.head_dim * 2)) ||
      (rc = model_alloc(ctx, m, &m->kcache, m->kv_elems() * 2)) ||
      (rc = model_alloc(ctx, m, &m->vcache, m->kv_elems() * 2)) ||
      (rc = model_alloc(ctx, m, &m->act16, align_up(acts, 8) * 2 + 1024)) ||
      (rc = model_alloc(ctx, m, &m->state, sizeof(DecodeState))) ||
      (rc = model_alloc(ctx, m, &m->tokens, (static_cast<size_t>(c.max_seq) + 1) * 4)) ||
      (rc = model_alloc(ctx, m, &m->pred, (static_cast<size_t>(c.max_seq) + 1) * 4))) {
    free_model(m);
    w->model = nullptr;
    return rc;
  }
  // activation buffers, each 16-byte aligned (the attention reads 128-bit rows)
  uint16_t* p = m->act16;
  auto take = [&](size_t n) {
    uint16_t* r = p;
    p += align_up(n, 8);
    return r;
  };
  m->x = take(H);
  m->xn = take(H);
  m->qkvb = take(nq + 2 * nkv);
  m->q = take(nq);
  m->attn = take(nq);
  m->proj = take(H);
  m->logits = take(c.vocab);
  cudaMemset(m->tokens, 0, (static_cast<size_t>(c.max_seq) + 1) * 4);
  cudaMemset(m->pred, 0, (static_cast<size_t>(c.max_seq) + 1) * 4);
  cudaMemset(m->state, 0, sizeof(DecodeState));
  *out = add_weight(ctx, std::move(w));
  return ALV_OK;
}

extern "C" int alv_llama_load(alv_ctx* ctx, alv_handle h, const char* name, const void* data, size_t nbytes,
                              int on_device) {
  if (!ctx || !name || !data) return fail(ctx, ALV_ERR_ARG, "llama_load: bad argument");
  LlamaModel* m = get_model(ctx, h);
  if (!m) return fail(ctx, ALV_ERR_HANDLE, "llama_load: invalid handle (not a llama model)");
  if (m->built) return fail(ctx, ALV_ERR_ARG, "llama_load: the model already ran; create a new one to reload");
  int rc = set_device(ctx);
  if (rc) return rc;
  const alv_llama_config& c = m->cfg;
  const std::string n(name);
  const size_t H = c.hidden;
  auto want = [&](size_t bytes) -> int {
    if (nbytes != bytes)
      return fail(ctx, ALV_ERR_SHAPE, "llama_load: " + n + " has " + std::to_string(nbytes) + " bytes, expected " +
                                          std::to_string(bytes));
    return ALV_OK;
  };
  if (n == "token_embd") {
    if ((rc = want(static_cast<size_t>(c.vocab) * H * 2))) return rc;
    if ((rc = copy_in(ctx, m->emb, data, nbytes, on_device))) return rc;
    m->loaded_emb = true;
    return ALV_OK;
  }
  if (n == "rope_table") {
    if ((rc = want(static_cast<size_t>(c.max_seq) * 2 * c.head_dim * 2))) return rc;
    if ((rc = copy_in(ctx, m->rope, data, nbytes, on_device))) return rc;
    m->loaded_rope = true;
    return ALV_OK;
  }
  int norm_idx = -1;
  if (n == "output_norm.weight") norm_idx = 2 * c.layers;
  int l = -1;
  char proj[32] = {0};
  if (norm_idx < 0 && std::sscanf(name, "blk.%d.%31[a-z_].weight", &l, proj) == 2 && l >= 0 && l < c.layers) {
    const std::string ps(proj);
    if (ps == "attn_norm" && n == "blk." + std::to_string(l) + ".attn_norm.weight") norm_idx = 2 * l;
    if (ps == "ffn_norm" && n == "blk." + std::to_string(l) + ".ffn_norm.weight") norm_idx = 2 * l + 1;
  }
  if (norm_idx >= 0) {
    if ((rc = want(H * 4))) return rc;
    if ((rc = copy_in(ctx, m->norms + norm_idx * H, data, nbytes, on_device))) return rc;
    m->loaded_norm[norm_idx] = true;
    return ALV_OK;
  }
  // packed Q4 matrices: the row count follows from the size (on-disk K / V
  // and the LM head may carry zero padding rows beyond what the model uses)
  uint32_t cols = 0, need = 0;
  if (n == "lm_head_packed") {
    cols = c.hidden;
    need = c.vocab;
  } else if (l >= 0 && n == "blk." + std::to_string(l) + "." + proj + ".weight_packed") {
    const std::string ps(proj);
    if (std::find(std::begin(kProj), std::end(kProj), ps) == std::end(kProj))
      return fail(ctx, ALV_ERR_ARG, "llama_load: unknown tensor " + n);
    cols = proj_cols(c, ps);
    need = proj_rows(c, ps);
  } else {
    return fail(ctx, ALV_ERR_ARG, "llama_load: unknown tensor " + n);
  }
  const size_t rowb = static_cast<size_t>(cols / 32) * 20;
  if (nbytes % rowb || nbytes / rowb < need)
    return fail(ctx, ALV_ERR_SHAPE, "llama_load: " + n + " must hold >= " + std::to_string(need) + " packed rows of " +
                                        std::to_string(rowb) + " bytes");
  auto it = m->raw.find(n);
  if (it != m->raw.end()) {
    cudaFree(it->second);
    m->raw.erase(it);
  }
  uint8_t* d = nullptr;
  ALV_CUDA(ctx, dev_alloc(ctx, &d, nbytes));
  if ((rc = copy_in(ctx, d, data, nbytes, on_device))) {
    cudaFree(d);
    return rc;
  }
  m->raw[n] = d;
  return ALV_OK;
}

extern "C" int alv_llama_start(alv_ctx* ctx, alv_handle h, const int32_t* prompt, int n_prompt, void* stream) {
  if (!ctx || !prompt) return fail(ctx, ALV_ERR_ARG, "llama_start: bad argument");
  Weight* w = get_weight(ctx, h, 4);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "llama_start: invalid handle (not a llama model)");
  auto* m = static_cast<LlamaModel*>(w->model);
  if (n_prompt < 1 || n_prompt > m->cfg.max_seq)
    return fail(ctx, ALV_ERR_ARG, "llama_start: prompt must hold 1..max_seq tokens");
  for (int i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab) return fail(ctx, ALV_ERR_ARG, "llama_start: token id out of range");
  int rc = set_device(ctx);
  if (rc) return rc;
  if ((rc = prepare_model(ctx, w, m))) return rc;
  return start_sequence(ctx, m, prompt, n_prompt, static_cast<cudaStream_t>(stream));
}

extern "C" int alv_llama_run(alv_ctx* ctx, alv_handle h, int n_prompt_steps, int n_decode_steps, void* stream) {
  if (!ctx || n_prompt_steps < 0 || n_decode_steps < 0) return fail(ctx, ALV_ERR_ARG, "llama_run: bad argument");
  Weight* w = get_weight(ctx, h, 4);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "llama_run: invalid handle (not a llama model)");
  auto* m = static_cast<LlamaModel*>(w->model);
  int rc = set_device(ctx);
  if (rc) return rc;
  if ((rc = prepare_model(ctx, w, m))) return rc;
  if (m->next_pos + n_prompt_steps + n_decode_steps > m->cfg.max_seq)
    return fail(ctx, ALV_ERR_ARG, "llama_run: the steps would consume positions beyond max_seq (next position " +
                                      std::to_string(m->next_pos) + ")");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_prompt_steps; ++i, ++m->next_pos) ALV_CUDA(ctx, cudaGraphLaunch(m->g_prefill, st));
  for (int i = 0; i < n_decode_steps; ++i, ++m->next_pos) ALV_CUDA(ctx, cudaGraphLaunch(m->g_decode, st));
  return ALV_OK;
}

namespace {
int copy_ids(alv_ctx* ctx, alv_handle h, bool predicted, int first, int n, int32_t* out_host, void* stream) {
  if (!ctx || !out_host || first < 0 || n < 0) return fail(ctx, ALV_ERR_ARG, "llama_tokens: bad argument");
  LlamaModel* m = get_model(ctx, h);
  if (!m) return fail(ctx, ALV_ERR_HANDLE, "llama_tokens: invalid handle (not a llama model)");
  if (static_cast<int64_t>(first) + n > static_cast<int64_t>(m->cfg.max_seq) + 1)
    return fail(ctx, ALV_ERR_ARG, "llama_tokens: range beyond max_seq");
  int rc = set_device(ctx);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ALV_CUDA(ctx, cudaMemcpyAsync(out_host, (predicted ? m->pred : m->tokens) + first, static_cast<size_t>(n) * 4,
                                cudaMemcpyDeviceToHost, st));
  return check_status(ctx, st);
}
}  // namespace

extern "C" int alv_llama_tokens(alv_ctx* ctx, alv_handle h, int first, int n, int32_t* out_host, void* stream) {
  return copy_ids(ctx, h, false, first, n, out_host, stream);
}

extern "C" int alv_llama_predicted(alv_ctx* ctx, alv_handle h, int first, int n, int32_t* out_host, void* stream) {
  return copy_ids(ctx, h, true, first, n, out_host, stream);
}

extern "C" int alv_llama_generate(alv_ctx* ctx, alv_handle h, const int32_t* prompt, int n_prompt, int steps,
                                  int32_t* out_host, void* stream) {
  if (!ctx || !prompt || !out_host || steps < 0) return fail(ctx, ALV_ERR_ARG, "llama_generate: bad argument");
  LlamaModel* m = get_model(ctx, h);
  if (!m) return fail(ctx, ALV_ERR_HANDLE, "llama_generate: invalid handle (not a llama model)");
  if (n_prompt < 1 || static_cast<int64_t>(n_prompt) + steps > m->cfg.max_seq)
    return fail(ctx, ALV_ERR_ARG, "llama_generate: n_prompt + steps must be <= max_seq (the last step reads position "
                                  "n_prompt + steps - 1)");
  int rc;
  if ((rc = alv_llama_start(ctx, h, prompt, n_prompt, stream))) return rc;
  if ((rc = alv_llama_run(ctx, h, n_prompt - 1, steps, stream))) return rc;
  return alv_llama_tokens(ctx, h, n_prompt, steps, out_host, stream);
}

extern "C" int alv_llama_forward(alv_ctx* ctx, alv_handle h, int token, int pos, uint16_t* logits, void* stream) {
  if (!ctx) return ALV_ERR_ARG;
  Weight* w = get_weight(ctx, h, 4);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "llama_forward: invalid handle (not a llama model)");
  auto* m = static_cast<LlamaModel*>(w->model);
  if (pos < 0 || pos >= m->cfg.max_seq || token < 0 || token >= m->cfg.vocab)
    return fail(ctx, ALV_ERR_ARG, "llama_forward: token or position out of range");
  int rc = set_device(ctx);
  if (rc) return rc;
  if ((rc = prepare_model(ctx, w, m))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DecodeState s{pos, pos + 1, {0, 0}};
  ALV_CUDA(ctx, cudaMemcpyAsync(m->tokens + pos, &token, 4, cudaMemcpyHostToDevice, st));
  ALV_CUDA(ctx, cudaMemcpyAsync(m->state, &s, sizeof(s), cudaMemcpyHostToDevice, st));
  ALV_CUDA(ctx, cudaStreamSynchronize(st));
  if ((rc = enqueue_step(ctx, m, logits != nullptr, st))) return rc;
  m->next_pos = static_cast<int64_t>(pos) + 1;
  if (logits)
    ALV_CUDA(ctx, cudaMemcpyAsync(logits, m->logits, static_cast<size_t>(m->cfg.vocab) * 2, cudaMemcpyDeviceToDevice, st));
  return ALV_OK;
}

extern "C" int alv_llama_prefill(alv_ctx* ctx, alv_handle h, int pos0, int n, void* stream) {
  if (!ctx || pos0 < 0 || n < 0) return fail(ctx, ALV_ERR_ARG, "llama_prefill: bad argument");
  Weight* w = get_weight(ctx, h, 4);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "llama_prefill: invalid handle (not a llama model)");
  auto* m = static_cast<LlamaModel*>(w->model);
  if (static_cast<int64_t>(pos0) + n > m->cfg.max_seq)
    return fail(ctx, ALV_ERR_ARG, "llama_prefill: positions beyond max_seq");
  int rc = set_device(ctx);
  if (rc) return rc;
  if ((rc = prepare_model(ctx, w, m)) || (rc = ensure_prefill(ctx, m))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int p = pos0; p < pos0 + n; p += kPrefillRows)
    if ((rc = prefill_rows(ctx, m, p, std::min(kPrefillRows, pos0 + n - p), st))) return rc;
  m->next_pos = pos0 + n;
  return ALV_OK;
}

extern "C" int alv_llama_info(alv_ctx* ctx, alv_handle h, int64_t* info) {
  if (!ctx || !info) return ALV_ERR_ARG;
  Weight* w = get_weight(ctx, h, 4);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "llama_info: invalid handle (not a llama model)");
  auto* m = static_cast<LlamaModel*>(w->model);
  int rc = set_device(ctx);
  if (rc) return rc;
  if ((rc = build_model(ctx, w, m))) return rc;
  size_t bytes = m->lm.bytes;
  for (int l = 0; l < m->cfg.layers; ++l) bytes += m->qkv[l].bytes + m->o[l].bytes + m->gu[l].bytes + m->dn[l].bytes;
  info[0] = m->one_launch ? 1 : 0;
  info[1] = m->one_launch ? 1 : 7 * static_cast<int64_t>(m->cfg.layers) + 3;
  info[2] = m->cfg.layers;
  info[3] = static_cast<int64_t>(bytes);
  for (int i = 4; i < 8; ++i) info[i] = 0;
  return ALV_OK;
}

extern "C" int alv_llama_reset(alv_ctx* ctx, alv_handle h, void* stream) {
  if (!ctx) return ALV_ERR_ARG;
  LlamaModel* m = get_model(ctx, h);
  if (!m) return fail(ctx, ALV_ERR_HANDLE, "llama_reset: invalid handle (not a llama model)");
  int rc = set_device(ctx);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ALV_CUDA(ctx, cudaMemsetAsync(m->kcache, 0, m->kv_elems() * 2, st));
  ALV_CUDA(ctx, cudaMemsetAsync(m->vcache, 0, m->kv_elems() * 2, st));
  ALV_CUDA(ctx, cudaMemsetAsync(m->state, 0, sizeof(DecodeState), st));
  m->next_pos = 0;
  return ALV_OK;
}
