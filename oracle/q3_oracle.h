/*
 * q3_oracle.h -- CPU restatement of the Qwen3-0.6B Q8_0 decode hot path of
 * abourramouss/qwen3-iree.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library.
 * It is the checker the CUDA path is compared against, never part of it.
 *
 * Every f16 value is passed as its IEEE binary16 bit pattern (uint16_t).
 * Each function cites the reference file:line whose semantics it restates.
 */
#ifndef Q3_ORACLE_H
#define Q3_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- model constants (model/qwen3_full.mlir:29-64) ---- */
#define Q3O_LAYERS 28
#define Q3O_DIM 1024
#define Q3O_NQ 16
#define Q3O_NKV 8
#define Q3O_HD 128
#define Q3O_FFN 3072
#define Q3O_VOCAB 151936
#define Q3O_QBLK 32
#define Q3O_QBYTES 34

/* attention chunk shared with the CUDA kernel (see q3o_attention) */
#define Q3O_ATT_CHUNK 32
#define Q3O_ATT_GROUP 8  /* chunks folded together before the cross-group fold */

/* numeric primitives */
float q3o_h2f(uint16_t h);
uint16_t q3o_f2h(float f);
float q3o_expf(float x);

/* Q8_0 format: tools/create_q8_irpa.py:103-129 */
void q3o_quantize_q8_0(const float* w, int64_t n, uint8_t* out);
void q3o_dequant_q8_0(const uint8_t* raw, int64_t n, float* out);

/* GEMVs */
void q3o_gemv_q8_mlir(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K);
void q3o_gemv_q8_cuda(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K);
void q3o_gemv_f16(const uint16_t* w, const uint16_t* x, uint16_t* y, int N, int K);
int64_t q3o_argmax_f16(const uint16_t* v, int64_t n);

/* small ops */
void q3o_rmsnorm(const uint16_t* x, const uint16_t* g, uint16_t* y, int n);
void q3o_rope_table(int64_t n_pos, float* cos_t, float* sin_t);
void q3o_qk_norm_rope(const uint16_t* x, const uint16_t* g, int n_heads, int64_t pos,
                      uint16_t* y);
void q3o_swiglu(const uint16_t* gate_up, uint16_t* out, int n);
void q3o_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, int n);
void q3o_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int64_t slot0,
                   int64_t T, uint16_t* out);

/* The fused engine's orders (the CUDA kernels k_fused_attn / k_fused_ffn):
 * a Q8_0 GEMV split along K into nparts slices whose f32 partials are summed
 * in slice order, and the attention folded over a 16-CTA cluster. */
#define Q3O_FUSED_CLUSTER 16
void q3o_gemv_q8_split(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K,
                       int nparts);
void q3o_attention_fused(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                         int64_t slot0, int64_t T, uint16_t* out);

/* model -- weights in the reference's parameter layout (tools/create_q8_irpa.py:146-224) */
typedef struct q3o_weights {
  const uint16_t* token_embd;   /* [151936,1024] f16 */
  const uint16_t* output_norm;  /* [1024] f16 */
  const uint16_t* output_T;     /* [151936,1024] f16 (tied: may equal token_embd) */
  const uint16_t* attn_norm;    /* [28,1024] f16 */
  const uint16_t* ffn_norm;     /* [28,1024] f16 */
  const uint16_t* q_norm;       /* [28,128] f16 */
  const uint16_t* k_norm;       /* [28,128] f16 */
  const uint8_t* q8_q;          /* [28, 2228224] Q8_0 */
  const uint8_t* q8_k;          /* [28, 1114112] */
  const uint8_t* q8_v;          /* [28, 1114112] */
  const uint8_t* q8_o;          /* [28, 2228224] */
  const uint8_t* q8_gate_up;    /* [28, 6684672] */
  const uint8_t* q8_down;       /* [28, 3342336] */
  int n_layers;                 /* <= 28; configs run all 28 */
  int order;                    /* Q3O_ORDER_*: which engine's summation orders */
} q3o_weights;

/* Q3O_ORDER_EXACT: the per-projection orders of the reference kernels (the
 * exact engine).  Q3O_ORDER_FUSED: the O and down projections split along K
 * into 8 slices and the cluster attention fold (the fused engine). */
#define Q3O_ORDER_EXACT 0
#define Q3O_ORDER_FUSED 1

void q3o_layer(const q3o_weights* w, int layer, uint16_t* x, int64_t pos, uint16_t* kc,
               uint16_t* vc, int64_t S);
int64_t q3o_decode_step(const q3o_weights* w, int64_t token, int64_t pos, uint16_t* kc,
                        uint16_t* vc, int64_t S, uint16_t* logits, int want_logits);
int64_t q3o_generate(const q3o_weights* w, const int64_t* prompt, int64_t n_prompt,
                     int64_t max_gen, int64_t eos, uint16_t* kc, uint16_t* vc, int64_t S,
                     int64_t* out_tokens, const int64_t* force_tokens);
int q3o_num_threads(void);
void q3o_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
