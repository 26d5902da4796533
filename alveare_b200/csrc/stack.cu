// Host side of the C ABI, part 4: the one-launch FFN stack (ffn_stack_kernel)
// and its tensor-parallel set-up over CUDA IPC.
#include "stack_launch.cuh"

namespace alv {
static_assert(kMaxRanksHost == kMaxRanks, "host and device agree on the rank limit");
}  // namespace alv

using namespace alv;

namespace {

struct StackLayout {
  size_t counters, wsA, wsB, down, act, total;
};

StackLayout stack_layout(alv_ctx* ctx, const Weight* w) {
  StackLayout o;
  o.counters = kHeaderBytes;
  o.wsA = align_up(o.counters + static_cast<size_t>(w->a.m.RT + w->b.m.RT) * 4, 256);
  o.wsB = align_up(o.wsA + ws_floats(ctx, kStackMaxTokens) * 4, 256);
  o.down = align_up(o.wsB + ws_floats(ctx, kStackMaxTokens) * 4, 256);
  o.act = align_up(o.down + static_cast<size_t>(kStackMaxTokens) * w->H * 4, 256);
  o.total = align_up(o.act + frag_bytes(w->b.m.KT, kStackMaxTokens), 256);
  return o;
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
  ALV_CUDA(ctx, dev_alloc(ctx, &s->layers_dev, sizeof(LayerW) * lw.size()));
  ALV_CUDA(ctx, cudaMemcpy(s->layers_dev, lw.data(), sizeof(LayerW) * lw.size(), cudaMemcpyHostToDevice));
  ALV_CUDA(ctx, dev_alloc(ctx, &s->ws, lo.total));
  ALV_CUDA(ctx, cudaMemset(s->ws, 0, lo.total));
  s->ws_bytes = lo.total;
  *out = add_weight(ctx, std::move(s));
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
  p.probe = w->probe;
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
  ALV_CUDA(ctx, dev_alloc(ctx, &w->xlocal, bytes));
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

extern "C" int alv_ffn_stack_set_probe(alv_ctx* ctx, alv_handle h, float* down_last) {
  if (!ctx) return ALV_ERR_ARG;
  Weight* w = get_weight(ctx, h, 3);
  if (!w) return fail(ctx, ALV_ERR_HANDLE, "ffn_stack_set_probe: invalid handle (not an ffn stack)");
  w->probe = down_last;
  return ALV_OK;
}
