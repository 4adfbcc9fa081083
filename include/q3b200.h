/*
 * q3b200.h -- C ABI of libq3b200.so, a B200 (sm_100a) implementation of the
 * Qwen3-0.6B Q8_0 decode hot path of abourramouss/qwen3-iree.
 *
 * Conventions
 *   - Every function returns a q3 status (0 = Q3_OK).  On failure
 *     q3_last_error() gives a one-line reason (thread-local).
 *   - "device" pointers are CUDA device pointers owned by the caller unless a
 *     q3_model owns them; "host" pointers are ordinary (or pinned) host memory.
 *   - f16 tensors are IEEE binary16; Q8_0 tensors are the reference's 34-byte
 *     blocks [f16 scale | 32 x int8] in [N, K] row-major block order
 *     (tools/create_q8_irpa.py:103-129, :185-224), rows starting 16-byte aligned.
 *   - `stream` is a cudaStream_t (NULL = the default stream).  Kernel entry
 *     points only enqueue work; they never allocate and never synchronize.
 *   - Shape or alignment violations return Q3_ERR_INVALID before any launch.
 *
 * The reference has no host C API: its path is an IREE module (.vmfb) driven
 * from Python through iree.runtime (scripts/benchmark.py:34-81,
 * scripts/chat.py:84-126), with six hand-written kernels substituted into
 * the executable (compile.sh:34-65).  This header provides both halves:
 *   (1) the six IREE-ABI kernels themselves (same names, same parameters,
 *       same fixed launch grid), plus host launchers for them;
 *   (2) a host API mirroring the module's public functions
 *       (@run, @decode, @generate, @prefill_all, @init_chat, @chat_turn).
 */
#ifndef Q3B200_H
#define Q3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3B200_ABI_VERSION 1

/* ---------------------------------------------------------------- status */
#define Q3_OK 0
#define Q3_ERR_INVALID 1     /* bad argument: shape, alignment, null pointer */
#define Q3_ERR_CUDA 2        /* a CUDA runtime call failed */
#define Q3_ERR_DEVICE 3      /* a kernel raised its error word (wait limit, bad token/position) */
#define Q3_ERR_NOMEM 4       /* device or host allocation failed (model set-up only) */
#define Q3_ERR_STATE 5       /* call out of sequence (e.g. chat turn before init) */
#define Q3_ERR_UNSUPPORTED 6 /* no sm_100 device, or a shape this build does not cover */

const char* q3_strerror(int status);
const char* q3_last_error(void);
int q3_abi_version(void);

/* ------------------------------------------------------ device plumbing
 * For hosts without a CUDA binding (the ctypes twins of scripts/benchmark.py
 * and scripts/chat.py).  Thin wrappers over the CUDA runtime. */
int q3_device_count(int* n);
int q3_set_device(int device);
int q3_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem);
int q3_device_malloc(void** dptr, size_t bytes);
int q3_device_free(void* dptr);
int q3_host_malloc(void** hptr, size_t bytes); /* page-locked */
int q3_host_free(void* hptr);
int q3_memcpy_htod(void* dst, const void* src, size_t bytes, void* stream);
int q3_memcpy_dtoh(void* dst, const void* src, size_t bytes, void* stream);
int q3_memcpy_dtod(void* dst, const void* src, size_t bytes, void* stream);
int q3_memset(void* dst, int value, size_t bytes, void* stream);
int q3_stream_create(void** stream);
int q3_stream_destroy(void* stream);
int q3_stream_synchronize(void* stream);
/* CUDA graphs: capture the calls enqueued on a created stream between begin
 * and end, then replay them (exec is an opaque graph handle). */
int q3_graph_capture_begin(void* stream);
int q3_graph_capture_end(void* stream, void** exec);
int q3_graph_launch(void* exec, void* stream);
int q3_graph_destroy(void* exec);
int q3_event_create(void** event);
int q3_event_destroy(void* event);
int q3_event_record(void* event, void* stream);
int q3_event_synchronize(void* event);
int q3_event_elapsed_ms(void* start, void* end, float* ms);

/* ------------------------------------------------------------ host math
 * RoPE angle tables of rope_decode_q/k (model/qwen3_full.mlir:324-454):
 * cos/sin of f32(pos) * powf(1e6, -(2i/128)), i < 64, for pos < n_pos.
 * cos_out/sin_out: host float[n_pos * 64]. */
int q3_rope_table(int64_t n_pos, float* cos_out, float* sin_out);
/* Q8_0 quantizer of tools/create_q8_irpa.py:103-118 on host memory
 * (n multiple of 32; out: n/32*34 bytes).  Used to build weights. */
int q3_quantize_q8_0(const float* w, int64_t n, uint8_t* out);

/* --------------------------------------------------- stateless kernels */

/* Q8_0 fused dequant + GEMV, y[N] = W[N,K] . x[K] (f32 accumulate, f16 out),
 * in the summation order of the reference's GPU-dialect kernels
 * (kernels/mlir/dispatch_{3,4,12,18,20}_gpu.mlir; per block sum, then scale).
 * Replaces q8_fused_gemv (model/qwen3_full.mlir:536-589).
 * K multiple of 256, K <= 3072; N multiple of 8; w, x 16-byte aligned. */
int q3_gemv_q8(const void* w, const void* x, void* y, int N, int K, void* stream);
/* The same GEMV launched with programmatic dependent launch: its weight rows
 * are copied, and the next launch may begin, while the previous kernel in
 * the stream is still running (x is read and y written only after that
 * kernel has finished).  So w must not be written by the preceding kernel.
 * Back-to-back calls over different weights then stream at HBM rate. */
int q3_gemv_q8_overlapped(const void* w, const void* x, void* y, int N, int K, void* stream);

/* Same, in the CUDA kernels' order (kernels/cuda/dispatch_3.cu:33-47;
 * per element acc += (scale*q)*x). */
int q3_gemv_q8_cuda_order(const void* w, const void* x, void* y, int N, int K, void* stream);

/* L independent GEMVs in one launch: y[l] = W_l . x[l], W_l = w + l*w_stride
 * bytes, x: [L, K] f16, y: [L, N] f16.  The stacked-weights form of
 * model/qwen3_full.mlir:561-566; used to measure streaming bandwidth. L <= 32. */
int q3_gemv_q8_layers(const void* w, int64_t w_stride, const void* x, void* y, int N, int K,
                      int L, void* stream);

/* Fused variants used by the decode step (also exposed for tests):
 *   q3_gemv_q8_norm:   y = W . rmsnorm(x, gamma)        (:779, :620-638)
 *   q3_gemv_q8_resid:  y = r + f16(W . x)               (:739, :801-805 / :852, :858-862)
 *   q3_gemv_q8_swiglu: y[n] = swiglu(gate_n, up_n), gate/up = rows n and
 *                      n + N of W (2N rows), input rmsnorm(x, gamma)  (:807-839)
 * x, r, y are f16; gamma f16[K]. */
int q3_gemv_q8_norm(const void* w, const void* x, const void* gamma, void* y, int N, int K,
                    void* stream);
int q3_gemv_q8_resid(const void* w, const void* x, const void* r, void* y, int N, int K,
                     void* stream);
int q3_gemv_q8_swiglu(const void* w, const void* x, const void* gamma, void* y, int N, int K,
                      void* stream);

/* f16 vocab GEMV fused with the tiled argmax (model/qwen3_full.mlir:1456-1509;
 * kernels/cuda/dispatch_24.cu): logits = W[N,1024] . rmsnorm(x, gamma)
 * (gamma may be NULL: no norm), token = first index of the largest logit
 * (-1 if none is above -inf).  logits (f16[N]) may be NULL.  token is a
 * DEVICE int64.  workspace: q3_vocab_argmax_workspace_bytes() bytes of device
 * memory, zero-filled once before first use (the kernel leaves it re-armed).
 * N multiple of 8, K == 1024. */
size_t q3_vocab_argmax_workspace_bytes(void);
int q3_vocab_argmax(const void* w, const void* x, const void* gamma, void* logits,
                    int64_t* token, void* workspace, int N, int K, void* stream);

/* Decode attention for one layer (model/qwen3_full.mlir:591-748 minus the
 * projections): QK-RMSNorm + RoPE of the raw q/k, K/V written at slot
 * slot0 + pos of the flat caches ([slots, 8, 128] f16), then GQA attention
 * of the 16 q heads over slots slot0 .. slot0 + pos.
 *   qkv:    device f16 [2048 q | 1024 k | 1024 v] (raw projections)
 *   pos:    DEVICE int64 position (pos < S and pos < rope rows)
 *   rope_cos/rope_sin: device f32 [rope_rows, 64] (q3_rope_table)
 *   out:    device f16 [2048]
 *   workspace: q3_attention_workspace_bytes(S) bytes, zero-filled once. */
size_t q3_attention_workspace_bytes(int64_t S);
int q3_decode_attention(const void* qkv, const void* q_norm, const void* k_norm,
                        const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                        void* k_cache, void* v_cache, int64_t slot0, int64_t S,
                        const int64_t* pos, void* out, void* workspace, void* stream);

/* The same decode attention for callers that cannot allocate device memory
 * where they launch (e.g. a kernel substituted into an IREE executable gets
 * only its bindings; code under a fixed memory plan may not cudaMalloc).  No
 * workspace argument and no allocation: the kernel's scratch (softmax
 * partials, arrival counters) lives in a static device array inside the
 * library, sized for S <= 4096 positions (about 1.08 MB per device, held
 * until the process exits); larger S returns Q3_ERR_INVALID.  The first call
 * on each device looks up that array's device address (call it once before
 * any stream capture); the address is kept per device and belongs to the
 * device's primary context, so a caller working in another CUDA context of
 * the device, or after a device reset, must not use this entry point.  All
 * calls share the one array: calls that overlap on
 * the GPU (concurrent streams, several host threads) race and must not be
 * issued.  Each call clears the counters it needs.  Results equal
 * q3_decode_attention bit for bit.  This entry point has no counterpart in
 * the reference. */
int q3_decode_attention_noalloc(const void* qkv, const void* q_norm, const void* k_norm,
                                const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                                void* k_cache, void* v_cache, int64_t slot0, int64_t S,
                                const int64_t* pos, void* out, void* stream);

/* Bounded device waits.  Every wait in these kernels gives up after a spin
 * budget (about 1 s of SM clock), records a code in a device error word and
 * returns.  q3_selftest_bounded_wait launches one such wait on a device flag:
 * it ends when *flag == expect or after limit_cycles (<= 2e9) and then writes
 * 3 (wait expired) into *err if *err was 0.  q3_check_error_word synchronizes
 * `stream` and returns Q3_ERR_DEVICE if the word at err is non-zero. */
int q3_selftest_bounded_wait(const int* flag, int expect, int64_t limit_cycles, int* err,
                             void* stream);
int q3_check_error_word(const int* err, void* stream);

/* ------------------------------------------------- IREE-ABI kernels
 * The six substituted executables of compile.sh:36-42 / :58-65, compiled for
 * sm_100a with the same export names and parameter lists
 * (kernels/cuda/dispatch_{3,4,12,18,20,24}.cu) and the same fixed launch
 * (grid N/8 x 256 threads, cuda/dispatch_N.mlir count()).  Numerics follow
 * the kernels/cuda order, bit for bit.  Declared here for linkers that want
 * the device symbols; the q3_iree_dispatch_* launchers run them on a stream:
 *   q8_stacked / weight  binding 0, b1 binding 1 (input at a fixed offset),
 *   b2 binding 2 (output at a fixed or pushed offset), c* push constants.
 * Replaces: decode_dispatch_3 (attn_q), _4 (attn_k / attn_v), _12 (attn_o),
 * _18 (ffn gate|up), _20 (ffn_down), _24 (vocab, f16 weights). */
int q3_iree_dispatch_3(const void* q8_stacked, const void* b1, void* b2, uint32_t c0,
                       uint32_t c1, void* stream);
int q3_iree_dispatch_4(const void* q8_stacked, const void* b1, void* b2, uint32_t c0,
                       uint32_t c1, uint32_t c2, void* stream);
int q3_iree_dispatch_12(const void* q8_stacked, const void* b1, void* b2, uint32_t c0,
                        uint32_t c1, void* stream);
int q3_iree_dispatch_18(const void* q8_stacked, const void* b1, void* b2, uint32_t c0,
                        uint32_t c1, void* stream);
int q3_iree_dispatch_20(const void* q8_stacked, const void* b1, void* b2, uint32_t c0,
                        uint32_t c1, void* stream);
int q3_iree_dispatch_24(const void* weight, const void* b1, void* b2, uint32_t c0,
                        void* stream);

/* ------------------------------------------------------------- model
 * Weights: device pointers in the reference's parameter layout
 * (tools/create_q8_irpa.py:146-224, model/qwen3_full.mlir:65-79, :772-777).
 * token_embd and output_T may be the same buffer (tied embedding). */
typedef struct q3_weights {
  const void* token_embd;     /* f16 [151936, 1024] */
  const void* output_norm;    /* f16 [1024] */
  const void* output_T;       /* f16 [151936, 1024] */
  const void* attn_norm;      /* f16 [28, 1024]  stacked.attn_norm.weight */
  const void* ffn_norm;       /* f16 [28, 1024]  stacked.ffn_norm.weight */
  const void* attn_q_norm;    /* f16 [28, 128]   stacked.attn_q_norm.weight */
  const void* attn_k_norm;    /* f16 [28, 128]   stacked.attn_k_norm.weight */
  const void* q8_attn_q;      /* Q8_0 [28, 2228224]  stacked.q8.attn_q.weight */
  const void* q8_attn_k;      /* Q8_0 [28, 1114112] */
  const void* q8_attn_v;      /* Q8_0 [28, 1114112] */
  const void* q8_attn_output; /* Q8_0 [28, 2228224] */
  const void* q8_ffn_gate_up; /* Q8_0 [28, 6684672]  gate rows then up rows */
  const void* q8_ffn_down;    /* Q8_0 [28, 3342336] */
} q3_weights;

/* One decoder layer (model/qwen3_full.mlir:751-864) as the fused engine
 * computes it, on caller buffers: x_in f16[1024] -> x_out f16[1024]; the new
 * K/V row is written at slot layer*S + pos of the flat caches and attention
 * runs over slots layer*S + 0..pos.  w: the stacked weights (layer selects
 * the slice); pos: DEVICE int64 (pos < S <= 4096); rope tables f32 [S, 64];
 * workspace: q3_fused_layer_workspace_bytes() bytes.  Three kernels: the
 * attention block, the feed-forward block and the residual rebuild.
 * flags: 0, or Q3_LAYER_OVERLAP -- the first kernel may begin (its weight and
 * K/V copies, its read of pos) while the previous kernel in the stream still
 * runs; then that kernel must not write w, pos or the cached K/V rows. */
#define Q3_LAYER_OVERLAP 1
size_t q3_fused_layer_workspace_bytes(void);
int q3_fused_layer(const q3_weights* w, int layer, const void* x_in, void* x_out, void* k_cache,
                   void* v_cache, int64_t S, const int64_t* pos, const float* rope_cos,
                   const float* rope_sin, void* workspace, int flags, void* stream);

typedef struct q3_model q3_model;

/* Creates a decoder bound to the current device and to `stream` (NULL: the
 * model creates its own).  Owns the KV cache for max_seq_len positions
 * (the flat [28*S, 8, 128] layout of model/qwen3_full.mlir:212-230), the
 * RoPE tables, activations and workspaces; the weights stay caller-owned. */
int q3_model_create(const q3_weights* w, int64_t max_seq_len, void* stream, q3_model** out);
int q3_model_destroy(q3_model* m);
void* q3_model_stream(q3_model* m);

/* @run (model/qwen3_full.mlir:2113-2167): ingest the prompt through the
 * decode path (the @prefill_all route, :1541-1570), take the argmax of its
 * last logits as the first token, then @generate (:1396-1534): tokens in
 * groups of 4, stopping after a group whose last token is eos, or after
 * max_gen tokens.  Like the reference, the first token is fed but not
 * returned.  prompt/out_tokens are HOST int64 buffers (out: max_gen slots);
 * *n_out receives the count.  n_prompt + max_gen + 1 <= max_seq_len. */
int q3_run(q3_model* m, const int64_t* prompt, int64_t n_prompt, int64_t max_gen, int64_t eos,
           int64_t* out_tokens, int64_t* n_out);

/* @decode (model/qwen3_full.mlir:1340-1394): one step for `token` at `pos`
 * (attending to cached positions 0..pos-1), logits f16[151936] written to
 * the DEVICE buffer `logits` (may be NULL), argmax to *next_token (host). */
int q3_decode(q3_model* m, int64_t token, int64_t pos, void* logits, int64_t* next_token);

/* @init_chat / @chat_turn (model/qwen3_full.mlir:2172-2222): a persistent,
 * zero-initialised cache of max_ctx positions; each turn ingests new_tokens
 * at the current position, generates as @run does, and advances the
 * position by n_tokens + n_out + 1, as the reference does. */
int q3_init_chat(q3_model* m, int64_t max_ctx);
int q3_chat_turn(q3_model* m, const int64_t* new_tokens, int64_t n_tokens, int64_t max_gen,
                 int64_t eos, int64_t* out_tokens, int64_t* n_out);

/* Step-level access for harnesses: enqueue `steps` decode steps of the
 * generation graph without synchronising (state must have been set by
 * q3_run or q3_generate_begin).  q3_generate_begin sets up a generation
 * like q3_run but returns after uploading the prompt. */
int q3_generate_begin(q3_model* m, const int64_t* prompt, int64_t n_prompt, int64_t max_gen,
                      int64_t eos);
int q3_generate_steps(q3_model* m, int64_t steps);
int q3_generate_end(q3_model* m, int64_t* out_tokens, int64_t* n_out);

/* Per-kernel device times of a generation step: runs `steps` steps of an
 * instrumented copy of the step graph (a CUDA event recorded between
 * consecutive kernels) and writes, per kernel in launch order, the average
 * time in microseconds and its kind (Q3_KIND_*).  Needs cap >= kernels per
 * step; counts as generation steps of the current generation. */
#define Q3_KIND_QKV 0     /* RMSNorm + Q|K|V projections */
#define Q3_KIND_ATTN 1    /* QK-norm + RoPE + KV write + attention */
#define Q3_KIND_O 2       /* O projection + residual */
#define Q3_KIND_GATE_UP 3 /* RMSNorm + gate|up + SwiGLU */
#define Q3_KIND_DOWN 4    /* down projection + residual */
#define Q3_KIND_VOCAB 5   /* final RMSNorm + vocab GEMV + argmax */
#define Q3_KIND_NORM 6    /* stand-alone RMSNorm (batched decoder only) */
#define Q3_KIND_FUSED_ATTN 7 /* fused engine: RMSNorm + Q|K|V + QK-norm + RoPE + KV write +
                                attention + split O projection */
#define Q3_KIND_FUSED_FFN 8  /* fused engine: O reduction + residual + RMSNorm + gate|up +
                                SwiGLU + split down projection */
int q3_model_profile_steps(q3_model* m, int64_t steps, float* times_us, int32_t* kinds,
                           int64_t cap);

/* Prompt ingestion.  STEPS (default): every prompt token but the last runs
 * one decode step (the reference's @prefill_all route,
 * model/qwen3_full.mlir:1541-1570), so ingestion gives the engine's bits.
 * BATCHED: those positions run as rows of the batched decoder's tensor-core
 * kernels, up to 64 positions per pass (QKV, the new K/V rows, causal
 * attention, O, FFN), writing the same K/V cache rows to within the batched
 * path's tolerance; the last prompt token and generation then run on the
 * model's engine.  Applies to q3_generate_begin, q3_run and q3_chat_turn. */
#define Q3_PREFILL_STEPS 0
#define Q3_PREFILL_BATCHED 1
int q3_model_set_prefill(q3_model* m, int mode);
int q3_model_prefill_mode(q3_model* m, int* mode);
/* Batched prefill of positions pos0 .. pos0+n-1 with tokens[0..n): stores
 * the tokens and writes the K/V rows of every layer (no vocab head).
 * Decoding continues with q3_decode at pos0 + n. */
int q3_model_prefill(q3_model* m, const int64_t* tokens, int64_t pos0, int64_t n);

/* Engines.  FUSED (default where available): two cluster kernels per layer
 * (attention block; feed-forward block) with the O and down projections split
 * along K into 8 slices whose f32 partials are summed in slice order -- 57
 * kernels per step; needs max_seq_len <= 4096.  GRAPH: the reference kernels'
 * per-projection orders, five kernels per layer (141 per step).  Both replay
 * CUDA graphs with programmatic dependent launch.  PERSISTENT: the GRAPH
 * engine's arithmetic inside ONE cooperative kernel with grid barriers
 * between phases.  GRAPH and PERSISTENT give identical bits; FUSED differs
 * from them only by its stated summation orders.  Q3_ENGINE=fused|graph|
 * persistent in the environment selects the engine at creation. */
#define Q3_ENGINE_GRAPH 0
#define Q3_ENGINE_PERSISTENT 1
#define Q3_ENGINE_FUSED 2
int q3_model_set_engine(q3_model* m, int engine);
int q3_model_engine(q3_model* m, int* engine);
/* Kernels this model has launched so far (all engines). */
int q3_model_kernel_launches(q3_model* m, int64_t* n);

/* Phase trace of the PERSISTENT engine: runs `steps` generation steps in one
 * launch and, for step `trace_step`, records per (CTA, phase) four SM clock
 * global-timer stamps in ns (barrier arrival, barrier release, inputs ready,
 * work done) into
 * out[ctas][phases][4] (host; cap entries).  For latency analysis. */
int q3_model_trace_steps(q3_model* m, int64_t steps, int64_t trace_step, long long* out,
                         int64_t cap, int* ctas, int* phases);

/* Phase stamps of the FUSED engine: runs `steps` generation steps from a copy
 * of the step graph whose cluster kernels record, per CTA, the global timer
 * (ns) after each numbered step of the kernel: out[56 launches][128 CTAs]
 * [phases] for the last step.  For latency analysis. */
int q3_model_trace_phases(q3_model* m, int64_t steps, long long* out, int64_t cap,
                          int64_t* n_launches, int* ctas, int* phases);

/* Kernel timeline of the GRAPH engine: runs `steps` decode steps (which
 * advance the sequence) from a copy of the step graph whose kernels record,
 * with the GPU's global timer, their first CTA start, first and last release
 * from the wait on the previous kernel, last CTA end, last CTA start and
 * first CTA end: out[k][6] in ns from the step's first kernel start
 * (averaged over steps),
 * kinds[k] = Q3_KIND_*, *n_kernels = kernels per step.  For latency analysis. */
int q3_model_trace_kernels(q3_model* m, int64_t steps, long long* out, int32_t* kinds,
                           int64_t cap, int64_t* n_kernels);

/* Kernel launches of one generation step of the GRAPH engine. */
int q3_model_launches_per_step(q3_model* m, int64_t* n);
/* Test hook for the device-side checks: writes the decode state on purpose --
 * Q3_POKE_TOKEN: the token table entry at position index; Q3_POKE_POS: the
 * current position -- so that a following step meets an out-of-range token
 * or position.  The kernels then record kErrBadToken / kErrBadPos (4 / 5) in
 * the error word, touch nothing outside their buffers, and the next call
 * returns Q3_ERR_DEVICE; the model stays usable for a new generation. */
#define Q3_POKE_TOKEN 0
#define Q3_POKE_POS 1
int q3_model_poke(q3_model* m, int what, int64_t index, int64_t value);
/* Device error word of the last run (0: none; see q3_strerror(Q3_ERR_DEVICE)). */
int q3_model_device_error(q3_model* m, int* code);

/* ------------------------------------------------------------------ batched decode
 * B independent sequences (1 <= B <= 64) decoded together.  The reference
 * decodes one sequence at a time (model/qwen3_full.mlir:751-864, per-layer
 * dispatch order); these entry points run the same per-sequence arithmetic
 * with each projection as one [B,K]x[K,N] tensor-core contraction (tcgen05,
 * weights dequantised to f16 = f16(scale*q) as model/qwen3_full.mlir:564-579
 * does), so results match the reference within rel-L2 1e-3, not bit for bit.
 * Activations are row-major [B padded to 16][K] f16; rows >= B are ignored. */

/* Batched Q8_0 projection: rows [row0, row0+N) of the Q8_0 matrix `w`
 * (w_rows rows of K, the reference's [N][K/32] x 34-byte layout) times the B
 * activation rows x[b][K] -> y[b][N].
 *   mode 0: y = W x;   mode 1: y = r + W x (r laid out like y);
 *   mode 2: gate rows [row0, row0+N), up rows [row0+N, row0+2N):
 *           y = silu(gate) * up in f16 (model/qwen3_full.mlir:829-839).
 * N % 128 == 0, K % 256 == 0, K <= 3072.  ksplit CTAs (one thread-block
 * cluster) share each 128-row tile, each over K/ksplit; ksplit divides K/256,
 * is at most 8 and leaves at most 2 chunks of 256 per CTA (1 for mode 2);
 * 0 picks one.  No workspace: the split partials are summed in shared memory,
 * in split order. */
int q3_bgemm_q8(const void* w, int64_t w_rows, int64_t row0, const void* x, void* y,
                const void* r, int B, int N, int K, int mode, int ksplit, void* stream);
/* Batched vocab GEMV + argmax (model/qwen3_full.mlir:1456-1509 per row):
 * logits[b][N] (optional, f16) and tokens[b] = first index of the largest f16
 * logit of xn[b] (xn already normalised).  Workspace zero-filled once,
 * 8-byte aligned (16-byte alignment lets the last CTA copy the per-CTA
 * candidates with cp.async; otherwise it loads them directly). */
size_t q3_bvocab_workspace_bytes(void);
int q3_bvocab_argmax(const void* w, int N, const void* xn, int B, void* logits, int64_t* tokens,
                     void* ws, void* stream);

/* Decode attention of one layer for B sequences, the batched decoder's
 * kernel (model/qwen3_full.mlir:591-748 minus the projections, per sequence):
 * QK-RMSNorm + RoPE, the new K/V row written at slot layer*S + pos[b], GQA
 * attention over slots 0..pos[b], streamed by tensor TMA in segments of 512
 * keys.  qkv [B][4096] raw projections; caches [B][28*S][8][128] f16; pos
 * DEVICE int64[B]; out [B][2048].  ws: q3_batch_attention_workspace_bytes(S,
 * B) bytes zero-filled once.  Tolerance-level parity (rel-L2 <= 1e-3). */
size_t q3_batch_attention_workspace_bytes(int64_t S, int B);
int q3_batch_attention(const void* qkv, const void* q_norm, const void* k_norm,
                       const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                       void* k_cache, void* v_cache, int layer, int64_t S, int B,
                       const int64_t* pos, void* out, void* ws, void* stream);

/* Batched decoder: caches of max_batch sequences x max_seq_len positions. */
typedef struct q3_batch q3_batch;
int q3_batch_create(const q3_weights* w, int max_batch, int64_t max_seq_len, void* stream,
                    q3_batch** out);
int q3_batch_destroy(q3_batch* m);
void* q3_batch_stream(q3_batch* m);
/* Sequence b: prompt prompts[b*stride .. + n_prompt[b]), fed one token per
 * step from position 0 (the reference's @prefill_all semantics,
 * model/qwen3_full.mlir:1541-1570); after the prompt each step appends the
 * greedy argmax. */
int q3_batch_begin(q3_batch* m, int B, const int64_t* prompts, int64_t stride,
                   const int64_t* n_prompt);
/* Benchmark set-up: sequence b holds ctx[b] cached positions of seeded
 * pseudo-random K/V and feeds tok[b] at position ctx[b]. */
int q3_batch_begin_random(q3_batch* m, int B, const int64_t* ctx, const int64_t* tok,
                          uint64_t seed);
/* Enqueue `steps` decode steps of all B sequences (asynchronous). */
int q3_batch_steps(q3_batch* m, int64_t steps);
/* Token table [B][max_seq_len+1] and positions [B] to the host (either may
 * be NULL), and the device error word; synchronises. */
int q3_batch_read(q3_batch* m, int64_t* tokens, int64_t* positions, int* device_err);
/* Argmax history [B][max_seq_len+1] to the host: entry p+1 of row b is the
 * greedy token after the step that fed position p, prompt positions included
 * (-1 where no step ran); for teacher-forced checks.  Synchronises. */
int q3_batch_read_argmax(q3_batch* m, int64_t* out);
/* Per-kernel device times of `steps` decode steps (which advance the
 * sequences), averaged per kernel of a step: times_us[i], kinds[i]
 * (Q3_KIND_*) for i < *n_kernels; events between kernels serialise them. */
int q3_batch_profile_steps(q3_batch* m, int64_t steps, float* times_us, int32_t* kinds,
                           int64_t cap, int64_t* n_kernels);
int q3_batch_kernel_launches(q3_batch* m, int64_t* n);
/* Per-CTA phase stamps of the batched projections and attention during the
 * last of `steps` steps: out[launch][512 CTAs][8] global-timer ns (0 where a
 * CTA or stamp did not run), kinds[launch] = Q3_KIND_*; cap >= launches *
 * 4096.  Projections stamp start, release, weights landed, activations
 * landed, accumulators complete, split partials stored, shares arrived, end;
 * attention stamps start, work list ready, release, first q staged, done.
 * For latency analysis. */
int q3_batch_trace_phases(q3_batch* m, int64_t steps, long long* out, int32_t* kinds, int64_t cap,
                          int64_t* n_launches);
/* Kernel timeline of `steps` batched steps, as q3_model_trace_kernels. */
int q3_batch_trace_kernels(q3_batch* m, int64_t steps, long long* out, int32_t* kinds,
                           int64_t cap, int64_t* n_kernels);

#ifdef __cplusplus
}
#endif
#endif /* Q3B200_H */
