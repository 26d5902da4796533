/*
 * alveare_b200 -- C ABI of the B200 (sm_100a) Q4 decode hot path.
 *
 * Drop-in replacement for the NPU boundary of daino-selvatico/alveare:
 *   C++ registry   runtime/cpp/include/alveare/npu.h:44-115 (NpuRegistry)
 *   Python ops     kernels/gemv_q/gemv_q.py:33-43   gemv_q_npu
 *                  kernels/ffn_fused/ffn_fused.py:28-39 ffn_fused_npu
 *                  kernels/gemm_q/gemm_q.py:28-39   gemm_q_npu
 *
 * Conventions
 *  - Plain pointers and sizes only.  `stream` is a cudaStream_t passed as
 *    void* (NULL = legacy default stream).  Device pointers unless a
 *    function says "host".
 *  - Every function returns an alv_status (0 = ok).  No exceptions cross the
 *    ABI; alv_last_error() gives a message for the last failure on a context
 *    (the reference throws std::runtime_error instead, npu.cpp:272-276).
 *  - Weights are given in the reference's packed Q4 layout: (N, K/32*20)
 *    uint8, each 20-byte block = 16 B nibbles (even k low nibble) + bf16
 *    scale (LE) + 2 B pad (tools/convert/gemv_q_convert.py:53-85).  They are
 *    repacked once on the GPU into the library's own layout and referenced
 *    by an opaque handle afterwards (npu.h:28-30, 64-72).
 *  - Activation dtypes: ALV_F32 or ALV_BF16.  fp32 inputs are consumed at
 *    full fp32 precision; outputs are fp32 or bf16 (round-to-nearest-even).
 *  - A context belongs to one device and is thread-compatible, not
 *    thread-safe: calls on one context must be serialized and use one stream
 *    at a time (the reference serializes requests with a mutex,
 *    generator.h:39-42).  Kernel launches are stream-ordered and
 *    asynchronous; alv_sync_status() synchronizes and reports device-side
 *    failures (a bounded wait that timed out).
 */
#ifndef ALVEARE_B200_H
#define ALVEARE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct alv_ctx alv_ctx;
typedef uint32_t alv_handle; /* 0 is never a valid handle */

typedef enum {
  ALV_OK = 0,
  ALV_ERR_ARG = 1,          /* bad pointer, size or enum */
  ALV_ERR_HANDLE = 2,       /* unknown or wrong-kind weight handle */
  ALV_ERR_SHAPE = 3,        /* shape mismatch / unsupported divisibility */
  ALV_ERR_CUDA = 4,         /* CUDA runtime error (message in alv_last_error) */
  ALV_ERR_TIMEOUT = 5,      /* a device-side bounded wait gave up */
  ALV_ERR_UNSUPPORTED = 6,  /* valid request outside this build's limits */
  ALV_ERR_NO_DEVICE = 7     /* no usable sm_100 device */
} alv_status;

enum { ALV_F32 = 0, ALV_BF16 = 1 };
enum { ALV_ACT_GELU = 0, ALV_ACT_SILU = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int alv_version(void);

/* Create / destroy a context on CUDA device `device`.  Replaces the
 * NpuRegistry constructor/destructor (npu.h:48-51). */
int alv_ctx_create(int device, alv_ctx** out);
int alv_ctx_destroy(alv_ctx* ctx);
const char* alv_last_error(const alv_ctx* ctx);

/* info[0..7] = device, SM count, scratch-arena bytes, host-call staging
 * bytes, device allocations the context has made so far (every cudaMalloc of
 * the library on its behalf: sync block, arena growth, weights, staging),
 * registered handles, 0, 0.  Diagnostics; no counterpart in the reference
 * (its registry keeps per-shape buffer objects, npu.cpp:59-72). */
int alv_ctx_info(alv_ctx* ctx, int64_t* info);

/* Synchronize `stream` and report any device-side failure recorded since the
 * last call (ALV_ERR_TIMEOUT).  Clears the recorded status. */
int alv_sync_status(alv_ctx* ctx, void* stream);

/* ---- Q4 format on the GPU ------------------------------------------------ */

/* Quantize a float32 (N, K) row-major device matrix into the reference's
 * packed layout (N, K/32*20) on the device.  GPU restatement of
 * quantize_to_q4_0 + pack_to_combined (tools/convert/gemv_q_convert.py:5-85):
 * per 32-block scale = max|w|/7 (0 -> 1.0), q = clip(rint(w/scale), -8, 7),
 * scale stored as bf16.  K must be a multiple of 32. */
int alv_q4_quantize(alv_ctx* ctx, const float* w, int N, int K, uint8_t* combined, void* stream);

/* ---- weights (NpuRegistry::create_*_weight, npu.h:64-72) ------------------ */

/* Register an (N, K) Q4 matrix for gemv/gemm.  `combined` holds N*(K/32)*20
 * bytes in the reference layout, on the host (on_device = 0) or the device
 * (on_device = 1).  Replaces NpuRegistry::create_gemv_weight (npu.h:68-69). */
int alv_gemv_weight_create(alv_ctx* ctx, int N, int K, const void* combined, size_t nbytes,
                           int on_device, alv_handle* out);

/* Register a fused FFN from its three per-matrix packed buffers:
 * gate, up: (I, H/32*20); down: (H, I/32*20).  [i_begin, i_end) selects the
 * slice of the intermediate dimension this device holds (tensor-parallel
 * split, multiples of 32; pass 0, I for the whole FFN).  act = ALV_ACT_*.
 * Replaces NpuRegistry::create_ffn_fused_weight (npu.h:71-72) together with
 * the load-time repack pack_ffn_fused_weights (runtime/cpp/src/weights.cpp:94-190). */
int alv_ffn_weight_create(alv_ctx* ctx, int H, int I, int act, const void* gate, const void* up,
                          const void* down, int on_device, int i_begin, int i_end,
                          alv_handle* out);

int alv_weight_destroy(alv_ctx* ctx, alv_handle h);

/* Change the activation of a registered FFN (the reference passes it per
 * call: NpuRegistry::run_ffn_fused, npu.h:94-95; ffn_fused_npu(activation=)). */
int alv_ffn_set_activation(alv_ctx* ctx, alv_handle h, int act);

/* info[0..7] = kind (1 gemv, 2 ffn), rows (N or H), cols (K or local I),
 * fast-dequant flag of matrix 0, of matrix 1, device bytes, i_begin, i_end. */
int alv_weight_info(alv_ctx* ctx, alv_handle h, int64_t* info);

/* Dequantize a registered matrix back to bf16 (rows x cols row-major) on the
 * device, with the same arithmetic the kernels use.  which: 0 = gemv matrix
 * or FFN gate, 1 = FFN up, 2 = FFN down.  GPU counterpart of
 * dequantize_combined (tools/ref/gemv_q.py:39-62). */
int alv_weight_dequantize(alv_ctx* ctx, alv_handle h, int which, uint16_t* out, void* stream);

/* ---- compute (device pointers, stream-ordered) ---------------------------- */

/* y[t, n] = sum_k W[n, k] * x[t, k] for t < ntok (1 <= ntok <= 16; fp32 x
 * allows ntok <= 8).  x is (ntok, K), y is (ntok, N), both row-major; x must
 * be 8-byte (fp32) or 4-byte (bf16) aligned, else ALV_ERR_ARG (the kernels
 * read x in element pairs).
 * Replaces NpuRegistry::run_gemv / run_gemm (npu.cpp:269-312) and the
 * gemv_q / gemm_q NPU kernels (kernels/gemv_q/gemv_q.cc:14-73,
 * kernels/gemm_q/gemm_q.cc:18-54). */
int alv_gemv(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y,
             int y_dtype, void* stream);

/* Batched prefill on the tensor cores: Y[b, n] = sum_k X[b, k] * W[n, k] for
 * b < B (any B >= 1), X bf16 (B, K) row-major on the device, 16-byte aligned;
 * Y (B, N) fp32 or bf16; fp32 accumulation.  The Q4 weight is dequantized to
 * bf16 in shared memory tile by tile and multiplied with tcgen05.mma (the
 * accumulator lives in tensor memory).  Replaces NpuRegistry::run_gemm /
 * run_gemm_streamed (npu.cpp:291-338) and the gemm_q NPU design
 * (kernels/gemm_q/gemm_q.py:28-143, gemm_q.cc:18-54). */
int alv_gemm(alv_ctx* ctx, alv_handle h, int B, const uint16_t* x, void* y, int y_dtype, void* stream);

/* Fused FFN on the registered slice: gate = bf16(Wg x), up = bf16(Wu x),
 * act = bf16(act_fn(gate) * up), y = Wd act (fp32 accumulate).  x is
 * (ntok, H), y is (ntok, H); 1 <= ntok <= 8; x aligned as for alv_gemv.  For a tensor-parallel slice y
 * is this device's partial sum (use ALV_F32 and all-reduce).  Replaces
 * NpuRegistry::run_ffn_fused (npu.cpp:340-378) including its host partial
 * sum, and the ffn_fused NPU design (kernels/ffn_fused/ffn_fused.py:28-328). */
int alv_ffn(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y,
            int y_dtype, void* stream);

/* One FFN half-block of a decode layer with the layer glue fused in
 * (runtime/py/model.py:782-806 with unit norm weights):
 *   x      = down_in ? bf16(x_in + bf16(rmsnorm(bf16(down_in)))) : x_in
 *   x_out  = x                         (if x_out != NULL)
 *   down_out = Wd act(Wg, Wu; bf16(rmsnorm(x)))      (fp32, partial for TP)
 * x_in/x_out bf16 (ntok, H); down_in/down_out fp32 (ntok, H); eps 1e-6. */
int alv_ffn_layer(alv_ctx* ctx, alv_handle h, int ntok, const uint16_t* x_in,
                  const float* down_in, uint16_t* x_out, float* down_out, void* stream);

/* Final residual of an FFN stack: x_out = bf16(x_in + bf16(rmsnorm(bf16(down_in)))). */
int alv_ffn_stack_finalize(alv_ctx* ctx, int ntok, int H, const uint16_t* x_in,
                           const float* down_in, uint16_t* x_out, void* stream);

/* Whole FFN stack of a decode step in one launch: the per-layer loop of the
 * decode step (runtime/cpp/src/model.cpp:404 inside the layer loop,
 * runtime/py/model.py:782-806) over n FFN weights, i.e. alv_ffn_layer for
 * layer 0..n-1 followed by alv_ffn_stack_finalize, with identical results.
 * The layers must share H, I, I-slice, activation and dequant path; a stack
 * of I-slices (i_begin, i_end not 0, I) runs only once connected to its
 * tensor-parallel peers (alv_ffn_stack_connect).  The stack references them
 * (destroy the stack with alv_weight_destroy before its layers).  It owns its
 * workspace, so a captured launch stays valid.  No counterpart handle exists
 * in the reference (its registry runs one FFN call per layer). */
int alv_ffn_stack_create(alv_ctx* ctx, const alv_handle* layers, int n, alv_handle* out);

/* out = stack(x_in): x_in, out bf16 (ntok, H) device buffers, 1 <= ntok <= 4
 * (ALV_ERR_UNSUPPORTED when the activations do not fit in shared memory). */
int alv_ffn_stack_run(alv_ctx* ctx, alv_handle stack, int ntok, const uint16_t* x_in, uint16_t* out,
                      void* stream);

/* act = bf16(act_fn(gate) * up) for n bf16 values (device buffers), with
 * the FFN kernels' own epilogue: GeGLU / SwiGLU exactly as
 * runtime/py/model.py:690-693 / :857-859 evaluate them in numpy.  Replaces
 * the reference's activation step kernel
 * (kernels/ffn_fused/ffn_compute_activation.cc:17-64). */
int alv_activation(alv_ctx* ctx, int act, int n, const uint16_t* gate, const uint16_t* up, uint16_t* out,
                   void* stream);

/* Tensor-parallel FFN stack over the GPUs of one node, one process per GPU.
 * The reference splits each FFN's intermediate dimension over compute tiles
 * and sums the partial down projections on the host
 * (kernels/ffn_fused/ffn_fused.py:46-60, runtime/cpp/src/npu.cpp:360-377).
 * Here rank q's stack holds the layers of I-slice q (alv_ffn_create with
 * i_begin / i_end, equal slices), and inside the one stack launch each
 * layer's partial down projection is pushed to every peer GPU over NVLink
 * and summed there in rank order, so no collective library runs between
 * layers and every rank produces the identical `out`.  Setup, on every
 * rank:
 *   alv_ffn_stack_exchange(ctx, stack, world, blob)   (ALV_IPC_BLOB_BYTES)
 *   all-gather the blobs in rank order (any host transport)
 *   alv_ffn_stack_connect(ctx, stack, rank, world, blobs)
 *   a host barrier; then alv_ffn_stack_run on every rank with the same x_in.
 * The ranks' launches wait for one another, so each rank must be on its own
 * GPU (connect checks the device UUIDs).  A rank launched more than a second
 * after the others makes every rank's launch give up (ALV_ERR_TIMEOUT at
 * alv_sync_status); the stack is then unusable (ALV_ERR_ARG) and has to be
 * destroyed and re-created on every rank.  No counterpart in the reference. */
#define ALV_IPC_BLOB_BYTES 128
int alv_ffn_stack_exchange(alv_ctx* ctx, alv_handle stack, int world, void* blob);
int alv_ffn_stack_connect(alv_ctx* ctx, alv_handle stack, int rank, int world, const void* blobs);

/* Test probe: when `down_last` is a device buffer of (ntok, H) fp32, every
 * later alv_ffn_stack_run of this stack also writes the last layer's down
 * projection there, exactly as the final residual step read it (summed over
 * the split-K partials and, for a tensor-parallel stack, over the ranks in
 * rank order), so a layer can be checked against the CPU path before the
 * bf16 rounding of the residual stream.  NULL turns it off.  No counterpart
 * in the reference (its host sum, npu.cpp:360-377, is visible to the caller). */
int alv_ffn_stack_set_probe(alv_ctx* ctx, alv_handle stack, float* down_last);

/* ---- Llama greedy decode on the GPU --------------------------------------
 * The reference's Llama decode step (runtime/py/model.py:821-934 with its
 * NPU matmuls, runtime/cpp/src/model.cpp:297-404 and the greedy loop of
 * runtime/cpp/src/generator.cpp:15-52) with every stage on the device: Q4
 * QKV / O / FFN / LM-head matmuls, RMSNorm, RoPE, a bf16 KV cache, GQA
 * attention, residuals and the argmax.  Rounding points follow the
 * reference's CPU path (bf16 after every projection, norm and residual).  A
 * step reads its position and token from device memory, so the library
 * captures it once into a CUDA graph and replays it per token. */
typedef struct {
  int32_t hidden, intermediate, heads, kv_heads, head_dim, layers, vocab, max_seq;
  float rms_eps;        /* 1e-5 for Llama (model.py:532) */
  /* 0 (default): a step is one launch of a persistent kernel that runs every
   * layer, the LM head and the argmax (grid barriers between the phases);
   * the library falls back to separate kernels when a model does not fit it
   * (head_dim > 128, more query heads than SMs, mixed dequant paths, or too
   * little shared memory).  1: always separate kernels (about seven per
   * layer).  Both give bit-identical logits. */
  int32_t per_kernel_step;
  int32_t reserved[6];
} alv_llama_config;

int alv_llama_create(alv_ctx* ctx, const alv_llama_config* cfg, alv_handle* out);

/* Load one tensor by its name in the reference's quantized-model directory
 * (tools/quantize_model.py:39-125, read by runtime/py/model.py:38-127):
 *   "token_embd"                    float16 (vocab, hidden)
 *   "output_norm.weight", "blk.{l}.attn_norm.weight", "blk.{l}.ffn_norm.weight"
 *                                   float32 (hidden)
 *   "blk.{l}.{attn_q,attn_k,attn_v,attn_output,ffn_gate,ffn_up,ffn_down}.weight_packed",
 *   "lm_head_packed"                Q4 (rows, cols/32*20) uint8; K, V and the
 *                                   LM head may carry zero padding rows
 *   "rope_table"                    bf16 (max_seq, 2*head_dim): cos | sin per
 *                                   position (model.py:230-261)
 * `data` is host memory (on_device = 0) or device memory (1). */
int alv_llama_load(alv_ctx* ctx, alv_handle model, const char* name, const void* data, size_t nbytes,
                   int on_device);

/* Start a sequence: zero the KV cache, put the prompt (host int32 ids) at
 * positions 0..n_prompt-1 and the position at 0.  The first call on a model
 * repacks its weights and captures the step graphs. */
int alv_llama_start(alv_ctx* ctx, alv_handle model, const int32_t* prompt, int n_prompt, void* stream);

/* Enqueue n_prompt_steps steps without logits (prompt tokens), then
 * n_decode_steps steps with logits (LM head + argmax: the argmax becomes the
 * next position's token unless the prompt already holds one there).
 * Each step consumes one position; ALV_ERR_ARG, before any launch, when the
 * steps would reach position max_seq (the library tracks the position that
 * start, prefill, forward, reset and run leave on the host).
 * Asynchronous, stream-ordered. */
int alv_llama_run(alv_ctx* ctx, alv_handle model, int n_prompt_steps, int n_decode_steps, void* stream);

/* Copy token ids [first, first + n) of the sequence to host memory
 * (synchronizes `stream`, reports device-side failures). */
int alv_llama_tokens(alv_ctx* ctx, alv_handle model, int first, int n, int32_t* out_host, void* stream);

/* The argmax each logits step computed for position p (p in [first,
 * first + n)).  Past the prompt it equals the token at p; over a prompt it
 * is a teacher-forced prediction (a prompt of a reference sequence scores
 * every position of it in one run). */
int alv_llama_predicted(alv_ctx* ctx, alv_handle model, int first, int n, int32_t* out_host, void* stream);

/* start + run(n_prompt - 1, steps) + tokens(n_prompt, steps): the greedy loop
 * of tests/test_generation.py:72-99 without an EOS stop.  n_prompt + steps
 * must not exceed max_seq. */
int alv_llama_generate(alv_ctx* ctx, alv_handle model, const int32_t* prompt, int n_prompt, int steps,
                       int32_t* out_host, void* stream);

/* One step at an explicit position, outside any graph: token -> KV cache at
 * `pos`; with `logits` (device, vocab bf16) also the LM head output
 * (model.py:919-934 forward(token, pos)). */
int alv_llama_forward(alv_ctx* ctx, alv_handle model, int token, int pos, uint16_t* logits, void* stream);

/* Batched prefill (Model::run_layer_batch, runtime/cpp/src/model.cpp:422-571):
 * positions [pos0, pos0 + n) of the token list alv_llama_start set go
 * through every layer 256 at a time, each projection one tcgen05 gemm over
 * the batch and causal attention per row; their K/V enter the cache and the
 * position becomes pos0 + n.  No LM head: after a prompt of n_prompt tokens,
 * prefill(0, n_prompt - 1) then run(0, steps) is the greedy loop.  The gemm
 * sums in another order than the decode step's gemv, so the cache agrees
 * with the token-by-token path to the last few bf16 bits. */
int alv_llama_prefill(alv_ctx* ctx, alv_handle model, int pos0, int n, void* stream);

/* Zero the KV cache and the position (runtime/py/model.py reset_caches). */
int alv_llama_reset(alv_ctx* ctx, alv_handle model, void* stream);

/* info[0..7] = 1 if a step is one kernel launch (0: separate kernels, see
 * per_kernel_step), kernel launches per step with the LM head, layers,
 * device bytes of the repacked Q4 weights, 0, 0, 0, 0.  Builds the model
 * (repacks the loaded tensors) if no step has.  Diagnostics; no counterpart
 * in the reference. */
int alv_llama_info(alv_ctx* ctx, alv_handle model, int64_t* info);

/* Allocation-free gemv: same arithmetic and arguments as alv_gemv, for
 * callers that must not allocate device memory while they run (a decode
 * loop with a fixed GPU memory budget, a host runtime that owns the device
 * allocator, code that cannot afford the device synchronization of
 * cudaMalloc/cudaFree).  alv_gemv may grow the context's scratch arena on
 * the first larger call; this entry point never allocates: its split-K
 * workspace and counters live in a static device array of 141,312 bytes
 * that every GPU loading the library holds until process exit.  Limits:
 * ntok <= 4, N <= 262,144 rows, GPUs with <= 148 SMs (one CTA per SM);
 * larger requests return ALV_ERR_UNSUPPORTED.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) and keeps it
 * for the life of the process, so make that first call before any stream
 * capture, and do not call cudaDeviceReset on a device this entry point has
 * used (the kept address would then be stale).  All calls share the one array: calls that overlap on the
 * GPU (different streams, or concurrent host threads) race and must be
 * serialized by the caller.  No counterpart in the reference. */
int alv_gemv_noalloc(alv_ctx* ctx, alv_handle h, int ntok, const void* x, int x_dtype, void* y,
                     int y_dtype, void* stream);

/* Tracing (the reference's per-launch timers, npu.cpp:23-43): when `trace`
 * is a device buffer of (#SMs x 16) uint64, every later alv_ffn / alv_ffn_layer
 * launch writes per-CTA %globaltimer stamps (ns): [0] start, [1] input staged,
 * [2] gate/up phase done, [3] grid barrier passed, [4] act staged, [5] down
 * phase done; with the layer glue also [6] inputs landed, [7] glue done.
 * alv_ffn_stack_run writes the same stamps for its second layer ([0] glue
 * start, [1]-[5] as above, [6] the layer's last barrier passed, [7] / [8]
 * gate/up / down units streamed, before the split-K reduction; inside its
 * glue [9] down loaded, [10] / [11] the norms of down / x reduced, [12] the
 * normalized x written).  Slots [13]-[15] are unused.  alv_gemv launches
 * write [0] start, [1] weights requested, [2] the previous kernel in the
 * stream finished, [3] x staged, [4] warp 0's units consumed, [5] split-K
 * reduction done.  A one-launch Llama step writes, for its second layer,
 * [0] layer start, [1] attention norm staged, [2] qkv units consumed (thread
 * 0's warp), [3] barrier passed, [4] attention done, [5] barrier passed,
 * [6] attention output staged, [14] O units consumed, [15] O reduction done
 * (all warps), [7] O barrier passed, [8] FFN norm staged,
 * [9] gate/up units consumed, [10] barrier passed, [11] act staged, [12]
 * down units consumed, [13] barrier passed.  NULL turns tracing off (the
 * default). */
int alv_set_trace(alv_ctx* ctx, uint64_t* trace);

/* ---- host-buffer convenience (synchronous, like NpuRegistry::run_gemv) ---- */

/* Copy x from host memory, run, copy y back to host memory, synchronize and
 * check status.  Mirrors npu.cpp:269-289 (memcpy to BO, sync, run, wait,
 * sync back). */
int alv_run_gemv(alv_ctx* ctx, alv_handle h, int ntok, const void* x_host, int x_dtype,
                 void* y_host, int y_dtype);
int alv_run_ffn(alv_ctx* ctx, alv_handle h, int ntok, const void* x_host, int x_dtype,
                void* y_host, int y_dtype);

#ifdef __cplusplus
}
#endif

#endif /* ALVEARE_B200_H */
