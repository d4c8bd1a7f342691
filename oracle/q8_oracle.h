/*
 * q8_oracle.h -- CPU restatement of marian-edge's Q8 greedy translation path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * backend and the timed CPU baseline.  Only tests/, __graft_entry__.smoke()
 * and bench.py (cpu_baseline leg and --impl reference) may load it.  The
 * product library (libmarian_cuda.so) never links or calls it.
 *
 * Every function restates one reference function; the citation is
 * crates/<crate>/src/<file>.rs:<lines> within malusama/marian-edge v0.7.0.
 *
 * Parity pin: the reference's own unit vectors (q8_gemm.rs:609-693,
 * tensor.rs:919-970, position.rs:27-38, shortlist.rs:261-281,
 * legacy_q8.rs:905-952) are checked against this library in
 * tests/test_oracle_golden.py.
 */
#ifndef MARIAN_Q8_ORACLE_H
#define MARIAN_Q8_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OQ_MAX_LAYERS 16
#define OQ_MAXIMUM_POSITION 4096          /* marian-model/src/manifest.rs:13 */
#define OQ_MAXIMUM_SOURCE_TOKENS 256      /* marian-cpu/src/limits.rs:3 */
#define OQ_MAXIMUM_GENERATION_STEPS 256   /* marian-cpu/src/limits.rs:4 */
#define OQ_MAXIMUM_ENGINE_BATCH 256       /* marian-cpu/src/limits.rs:5 */
#define OQ_MAXIMUM_PADDED_CELLS 65536     /* marian-cpu/src/limits.rs:6 */

/* Decoder layer kinds.  SSRU is the reference graph
 * (q8_engine.rs:105-109); SELFATTN is the benchmark-shape extension whose
 * self-attention block reuses the encoder block order (q8_engine.rs:526-557). */
enum { OQ_DECODER_SSRU = 0, OQ_DECODER_SELFATTN = 1 };

/* One Q8 linear: canonical [out, in] int8 weights, static activation alpha
 * and one weight quant_mult (q8_gemm.rs:30-41). */
typedef struct {
    const int8_t *weights;      /* [out_dim, in_dim] */
    float activation_mult;      /* *_QuantMultA */
    float weight_mult;          /* intgemm8 trailing quant_mult */
    const float *bias;          /* [out_dim] or NULL */
    int32_t in_dim;
    int32_t out_dim;
    /* Per-row extension (not in the reference): one weight multiplier per
     * output row, replacing weight_mult for row n; NULL = per tensor. */
    const float *weight_row_mults;
} oq_linear;

typedef struct {
    oq_linear wq, wk, wv, wo;
    const float *ln_scale, *ln_bias;
} oq_attention_block;

typedef struct {
    oq_linear w1, w2;
    const float *ln_scale, *ln_bias;
} oq_ffn_block;

typedef struct {
    oq_linear w, wf;
    const float *ln_scale, *ln_bias;
} oq_ssru_block;

/* A parsed lexical shortlist (marian-model/src/shortlist.rs:56-148): source
 * token t maps to targets[offsets[t] .. offsets[t + 1]); ids below
 * first_num are always candidates.  offsets == NULL means no shortlist file
 * (every id is a candidate, shortlist.rs:66-73). */
typedef struct {
    uint64_t first_num;
    const uint64_t *offsets;   /* [source_vocab + 1] */
    const uint32_t *targets;
} oq_shortlist;

typedef struct {
    int32_t dim, heads, ffn_dim;
    int32_t encoder_layers, decoder_layers, decoder_kind;
    int32_t source_vocab, target_vocab;
    int32_t max_length_factor;
    const int8_t *encoder_embedding; float encoder_embedding_mult;
    const int8_t *decoder_embedding; float decoder_embedding_mult;
    float decoder_output_activation_mult;  /* decoder_Wemb_QuantMultA */
    const float *output_bias;              /* decoder_ff_logit_out_b */
    oq_attention_block encoder_attention[OQ_MAX_LAYERS];
    oq_ffn_block encoder_ffn[OQ_MAX_LAYERS];
    oq_ssru_block decoder_ssru[OQ_MAX_LAYERS];
    oq_attention_block decoder_self[OQ_MAX_LAYERS];
    oq_attention_block decoder_context[OQ_MAX_LAYERS];
    oq_ffn_block decoder_ffn[OQ_MAX_LAYERS];
    oq_shortlist shortlist;  /* per-sentence candidates (q8_engine.rs:576-584) */
} oq_model;

/* Optional capture of intermediate activations for per-layer checks.
 * Buffers are caller-owned; a NULL member is skipped.  Padded [B, Lmax, d]
 * tensors are written in the reference's padded layout. */
typedef struct {
    float *encoder_output;       /* [B*Lmax, d] */
    float *cross_key;            /* [decoder_layers, B*Lmax, d] */
    float *cross_value;          /* [decoder_layers, B*Lmax, d] */
    float *decoder_state_step0;  /* [B, d] final decoder state at step 0 */
    float *top2_gap;             /* [B, 256] top-1 minus top-2 logit per step */
} oq_trace;

/* q8_gemm.rs:569-590.  Returns 0, or -1 - index of the first non-finite
 * value, or -2^31 for an invalid multiplier. */
int64_t oq_quantize_u8(const float *input, size_t n, float mult, uint8_t *out);

/* Exact u8 (zero point 127) x i8 -> i32 GEMM, q8_gemm.rs:539-553.
 * weights are canonical [N, K]. */
void oq_gemm_u8_i8(const uint8_t *a, const int8_t *w, size_t rows, size_t k,
                   size_t n, int32_t *acc);

/* Q8Linear::run_into, q8_gemm.rs:380-448. Returns 0 or a negative error. */
int oq_linear_run(const oq_linear *linear, const float *input, size_t rows,
                  float *output);

/* Generalised epilogue used by the GEMM microbench: y = acc*(rs[m]*cs[n]) +
 * bias[n]; optional ReLU, then optional residual add.  With rs == NULL and
 * cs[n] = 1/(a*w) this is exactly q8_gemm.rs:438-446. */
void oq_epilogue(const int32_t *acc, size_t rows, size_t n, const float *row_scale,
                 const float *col_scale, const float *bias, int relu,
                 const float *residual, float *out);

/* tensor.rs:132-155 + normalize_row tensor.rs:372-385 */
void oq_residual_layer_norm(const float *input, const float *residual,
                            const float *scale, const float *bias, size_t rows,
                            size_t dim, float *out);

/* tensor.rs:184-218 */
void oq_ssru_update_layer_norm(const float *candidate, const float *forget_pre,
                               float *state, const float *residual,
                               const float *scale, const float *bias,
                               size_t rows, size_t dim, float *out);

/* tensor.rs:251-318 (padded batch, key-length mask). */
int oq_attention(const float *q, const float *k, const float *v,
                 const int32_t *lengths, size_t batch, size_t q_len,
                 size_t k_len, size_t dim, size_t heads, float *out);

/* marian-model/src/position.rs:5-21; out is [4096, dim]. */
int oq_sinusoidal_positions(size_t dim, float *out);

/* shortlist.rs:150-198 with no shortlist file: writes candidate ids in
 * ascending order, returns the count. */
size_t oq_full_vocab_candidates(size_t target_vocab, uint32_t *out);

/* shortlist.rs:150-198 LexicalShortlist::candidates for one sentence:
 * writes the ascending candidate ids to out (capacity target_vocab) and
 * returns their count, or -1 for a negative token, -2 for a token beyond
 * the source vocabulary, -3 for no candidates, -4 when EOS (0) is missing. */
int64_t oq_shortlist_candidates(const oq_shortlist *sl, size_t source_vocab, size_t target_vocab,
                                const int32_t *tokens, size_t n, uint32_t *out);

/* q8_engine.rs:749-790 */
int64_t oq_select_token(const float *state, size_t dim, const int8_t *embedding,
                        float embedding_mult, float activation_mult,
                        const float *output_bias, const uint32_t *candidates,
                        size_t n_candidates);

/* Q8CpuEngine::translate_token_ids, q8_engine.rs:353-466.
 *
 * force_len (nullable) is the harness rule the benchmark workloads add: for
 * row b, token 0 is masked while step < force_len[b]-1 and the row's limit
 * is min(max_output_tokens, force_len).  With force_len == NULL the control
 * flow is the reference's unchanged.
 *
 * Outputs: out_offsets [batch+1]; out_tokens up to out_capacity.  Returns
 * 0 on success or a negative code with a message in err. */
int oq_translate(const oq_model *model, const float *positions,
                 const int32_t *tokens, const uint32_t *offsets, size_t batch,
                 const uint32_t *max_output_tokens, const uint32_t *force_len,
                 int32_t *out_tokens, uint32_t *out_offsets, size_t out_capacity,
                 oq_trace *trace, char *err, size_t err_capacity);

#ifdef __cplusplus
}
#endif
#endif
