/*
 * q8_oracle.c -- CPU restatement of marian-edge's Q8 greedy translation path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); see the
 * header.  Floating-point expressions keep the reference's operation order
 * and are compiled with -ffp-contract=off so no multiply-add is fused, as in
 * Rust.  Sums over a row are sequential left folds, as Rust's
 * Iterator::sum is.  exp/sin/cos/log come from the C library, which is what
 * Rust's f32 methods call on Linux.
 */
#include "q8_oracle.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef __AVX2__
#include <immintrin.h>
#endif

#define ACTIVATION_ZERO_POINT 127
#define LAYER_NORM_EPSILON 1.0e-6f

static void set_err(char *err, size_t cap, const char *fmt, ...) {
    if (!err || cap == 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, cap, fmt, ap);
    va_end(ap);
}

/* ---- q8_gemm.rs:569-590 quantize_symmetric_u8_into ---------------------- */
int64_t oq_quantize_u8(const float *input, size_t n, float mult, uint8_t *out) {
    if (!isfinite(mult) || mult <= 0.0f) return INT32_MIN;
    for (size_t i = 0; i < n; ++i) {
        float v = input[i];
        if (!isfinite(v)) return -1 - (int64_t)i;
        float s = rintf(v * mult);          /* round_ties_even (default FE mode) */
        if (s < -127.0f) s = -127.0f;
        if (s > 127.0f) s = 127.0f;
        out[i] = (uint8_t)((int)s + ACTIVATION_ZERO_POINT);
    }
    return 0;
}

/* ---- q8_gemm.rs:539-553 run_scalar_into (exact integer semantics) -------- */
/* Centred activations (q - 127 in [-127, 127]) times int8 weights; rows are
 * blocked by 4 so each weight row is streamed once per block (the integer
 * result is independent of blocking). */
#ifdef __AVX2__
static inline int32_t hsum_epi32(__m256i v) {
    __m128i x = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    x = _mm_add_epi32(x, _mm_shuffle_epi32(x, 0x4E));
    x = _mm_add_epi32(x, _mm_shuffle_epi32(x, 0xB1));
    return _mm_cvtsi128_si32(x);
}
#endif

static int32_t dot_i8(const int16_t *a, const int8_t *w, size_t k) {
    int32_t s = 0;
    size_t i = 0;
#ifdef __AVX2__
    __m256i v = _mm256_setzero_si256();
    for (; i + 16 <= k; i += 16) {
        const __m256i w16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(w + i)));
        v = _mm256_add_epi32(v, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)(a + i)), w16));
    }
    s = hsum_epi32(v);
#endif
    for (; i < k; ++i) s += (int32_t)a[i] * (int32_t)w[i];
    return s;
}

void oq_gemm_u8_i8(const uint8_t *a, const int8_t *w, size_t rows, size_t k,
                   size_t n, int32_t *acc) {
    /* i16 so every u8 (including 255, outside the quantizer's range) is exact */
    int16_t *centred = (int16_t *)malloc(((rows * k) > 0 ? rows * k : 1) * sizeof(int16_t));
    for (size_t i = 0; i < rows * k; ++i) centred[i] = (int16_t)((int)a[i] - ACTIVATION_ZERO_POINT);
    size_t r = 0;
#ifdef __AVX2__
    /* The exact AVX2 widening scheme of q8_avx2.rs:125-229: 16 weights
     * widened to i16, vpmaddwd forms exact i32 pair sums of centred
     * activations times weights (|a| <= 128, |w| <= 127, so no pair sum can
     * saturate), accumulated in i32 lanes.  Integer addition is associative,
     * so the result equals the scalar loop's bit for bit. */
    const size_t k16 = k & ~(size_t)15;
    for (; r + 4 <= rows; r += 4) {
        const int16_t *a0 = centred + r * k, *a1 = a0 + k, *a2 = a1 + k, *a3 = a2 + k;
        for (size_t c = 0; c < n; ++c) {
            const int8_t *wc = w + c * k;
            __m256i v0 = _mm256_setzero_si256(), v1 = v0, v2 = v0, v3 = v0;
            for (size_t i = 0; i < k16; i += 16) {
                const __m256i w16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(wc + i)));
                v0 = _mm256_add_epi32(v0, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)(a0 + i)), w16));
                v1 = _mm256_add_epi32(v1, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)(a1 + i)), w16));
                v2 = _mm256_add_epi32(v2, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)(a2 + i)), w16));
                v3 = _mm256_add_epi32(v3, _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)(a3 + i)), w16));
            }
            int32_t s[4] = {hsum_epi32(v0), hsum_epi32(v1), hsum_epi32(v2), hsum_epi32(v3)};
            for (size_t i = k16; i < k; ++i) {
                const int32_t wv = wc[i];
                s[0] += (int32_t)a0[i] * wv;
                s[1] += (int32_t)a1[i] * wv;
                s[2] += (int32_t)a2[i] * wv;
                s[3] += (int32_t)a3[i] * wv;
            }
            for (int j = 0; j < 4; ++j) acc[(r + j) * n + c] = s[j];
        }
    }
#else
    for (; r + 4 <= rows; r += 4) {
        const int16_t *a0 = centred + r * k, *a1 = a0 + k, *a2 = a1 + k, *a3 = a2 + k;
        for (size_t c = 0; c < n; ++c) {
            const int8_t *wc = w + c * k;
            int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
            for (size_t i = 0; i < k; ++i) {
                int32_t wv = wc[i];
                s0 += (int32_t)a0[i] * wv;
                s1 += (int32_t)a1[i] * wv;
                s2 += (int32_t)a2[i] * wv;
                s3 += (int32_t)a3[i] * wv;
            }
            acc[(r + 0) * n + c] = s0;
            acc[(r + 1) * n + c] = s1;
            acc[(r + 2) * n + c] = s2;
            acc[(r + 3) * n + c] = s3;
        }
    }
#endif
    for (; r < rows; ++r)
        for (size_t c = 0; c < n; ++c) acc[r * n + c] = dot_i8(centred + r * k, w + c * k, k);
    free(centred);
}

/* ---- q8_gemm.rs:380-448 Q8Linear::run_into ------------------------------- */
int oq_linear_run(const oq_linear *L, const float *input, size_t rows, float *output) {
    if (rows == 0) return 0;
    size_t k = (size_t)L->in_dim, n = (size_t)L->out_dim;
    uint8_t *q = (uint8_t *)malloc(rows * k);
    int32_t *acc = (int32_t *)malloc(rows * n * sizeof(int32_t));
    if (!q || !acc) { free(q); free(acc); return -3; }
    if (oq_quantize_u8(input, rows * k, L->activation_mult, q) != 0) {
        free(q); free(acc);
        return -2;
    }
    oq_gemm_u8_i8(q, L->weights, rows, k, n, acc);
    float inverse_scale = 1.0f / (L->activation_mult * L->weight_mult);
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < n; ++c) {
            float bias = L->bias ? L->bias[c] : 0.0f;
            /* per-row extension: the same formula with row c's multiplier */
            float scale = L->weight_row_mults
                              ? 1.0f / (L->activation_mult * L->weight_row_mults[c])
                              : inverse_scale;
            output[r * n + c] = (float)acc[r * n + c] * scale + bias;
        }
    free(q);
    free(acc);
    return 0;
}

void oq_epilogue(const int32_t *acc, size_t rows, size_t n, const float *row_scale,
                 const float *col_scale, const float *bias, int relu,
                 const float *residual, float *out) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < n; ++c) {
            float scale = col_scale[c];
            if (row_scale) scale = row_scale[r] * scale;
            float v = (float)acc[r * n + c] * scale + (bias ? bias[c] : 0.0f);
            if (relu) v = fmaxf(v, 0.0f);
            if (residual) v = v + residual[r * n + c];
            out[r * n + c] = v;
        }
}

/* ---- tensor.rs:372-385 normalize_row ------------------------------------- */
static void normalize_row(float *row, const float *scale, const float *bias, size_t dim) {
    float fdim = (float)dim;
    float sum = 0.0f;
    for (size_t i = 0; i < dim; ++i) sum += row[i];
    float mean = sum / fdim;
    float var = 0.0f;
    for (size_t i = 0; i < dim; ++i) {
        float c = row[i] - mean;
        var += c * c;
    }
    var = var / fdim;
    float inverse_std = 1.0f / sqrtf(var + LAYER_NORM_EPSILON);
    for (size_t i = 0; i < dim; ++i)
        row[i] = (row[i] - mean) * inverse_std * scale[i] + bias[i];
}

/* ---- tensor.rs:132-155 residual_layer_norm_into -------------------------- */
void oq_residual_layer_norm(const float *input, const float *residual,
                            const float *scale, const float *bias, size_t rows,
                            size_t dim, float *out) {
    for (size_t i = 0; i < rows * dim; ++i) out[i] = input[i] + residual[i];
    for (size_t r = 0; r < rows; ++r) normalize_row(out + r * dim, scale, bias, dim);
}

/* ---- tensor.rs:184-218 ssru_update_layer_norm_into ----------------------- */
void oq_ssru_update_layer_norm(const float *candidate, const float *forget_pre,
                               float *state, const float *residual,
                               const float *scale, const float *bias,
                               size_t rows, size_t dim, float *out) {
    size_t n = rows * dim;
    for (size_t i = 0; i < n; ++i) {
        float gate = 1.0f / (1.0f + expf(-forget_pre[i]));
        float next = gate * state[i] + (1.0f - gate) * candidate[i];
        state[i] = next;
    }
    for (size_t i = 0; i < n; ++i) out[i] = fmaxf(state[i], 0.0f) + residual[i];
    for (size_t r = 0; r < rows; ++r) normalize_row(out + r * dim, scale, bias, dim);
}

/* ---- tensor.rs:745-754 softmax_in_place ---------------------------------- */
static void softmax_in_place(float *v, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; ++i) m = fmaxf(m, v[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        v[i] = expf(v[i] - m);
        sum += v[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; ++i) v[i] *= inv;
}

/* ---- tensor.rs:251-318 attention_into ------------------------------------ */
int oq_attention(const float *q, const float *k, const float *v,
                 const int32_t *lengths, size_t batch, size_t q_len,
                 size_t k_len, size_t dim, size_t heads, float *out) {
    if (heads == 0 || dim % heads != 0) return -1;
    for (size_t b = 0; b < batch; ++b)
        if (lengths[b] <= 0 || (size_t)lengths[b] > k_len) return -2;
    size_t hd = dim / heads;
    float attention_scale = 1.0f / sqrtf((float)hd);
    float *scores = (float *)malloc(k_len * sizeof(float));
    memset(out, 0, batch * q_len * dim * sizeof(float));
    for (size_t b = 0; b < batch; ++b) {
        size_t active = (size_t)lengths[b];
        for (size_t qi = 0; qi < q_len; ++qi)
            for (size_t h = 0; h < heads; ++h) {
                const float *qrow = q + (b * q_len + qi) * dim + h * hd;
                for (size_t j = 0; j < active; ++j) {
                    const float *krow = k + (b * k_len + j) * dim + h * hd;
                    float dot = 0.0f;
                    for (size_t i = 0; i < hd; ++i) dot += qrow[i] * krow[i];
                    scores[j] = dot * attention_scale;
                }
                softmax_in_place(scores, active);
                float *o = out + (b * q_len + qi) * dim + h * hd;
                for (size_t j = 0; j < active; ++j) {
                    const float *vrow = v + (b * k_len + j) * dim + h * hd;
                    float w = scores[j];
                    for (size_t i = 0; i < hd; ++i) o[i] += vrow[i] * w;
                }
            }
    }
    free(scores);
    return 0;
}

/* ---- marian-model/src/position.rs:5-21 ----------------------------------- */
int oq_sinusoidal_positions(size_t dim, float *out) {
    if (dim < 4 || dim % 2 != 0) return -1;
    size_t half = dim / 2;
    float ln1e4 = logf(10000.0f);
    for (size_t p = 0; p < OQ_MAXIMUM_POSITION; ++p)
        for (size_t i = 0; i < half; ++i) {
            float frequency = expf(-(float)i * ln1e4 / (float)(half - 1));
            out[p * dim + i] = sinf((float)p * frequency);
            out[p * dim + half + i] = cosf((float)p * frequency);
        }
    return 0;
}

/* ---- marian-model/src/shortlist.rs:150-198 (no shortlist file) ----------- */
size_t oq_full_vocab_candidates(size_t target_vocab, uint32_t *out) {
    unsigned char *present = (unsigned char *)malloc(target_vocab ? target_vocab : 1);
    memset(present, 1, target_vocab);
    if (target_vocab > 1) present[1] = 0;
    if (target_vocab > 7) {
        size_t end = target_vocab < 39 ? target_vocab : 39;
        for (size_t i = 7; i < end; ++i) present[i] = 0;
    }
    size_t count = 0;
    for (size_t i = 0; i < target_vocab; ++i)
        if (present[i]) out[count++] = (uint32_t)i;
    /* Padding to a multiple of 8 with absent ids >= 50: with no shortlist
     * every id >= 50 is present, so nothing is appended. */
    for (size_t i = 50; i < target_vocab; ++i) {
        if (count % 8 == 0) break;
        if (!present[i]) out[count++] = (uint32_t)i;
    }
    free(present);
    return count;  /* already ascending */
}

/* ---- marian-model/src/shortlist.rs:150-198 (with a shortlist file) ------- */
static int cmp_u32(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

int64_t oq_shortlist_candidates(const oq_shortlist *sl, size_t source_vocab, size_t target_vocab,
                                const int32_t *tokens, size_t n, uint32_t *out) {
    unsigned char *present = (unsigned char *)malloc(target_vocab ? target_vocab : 1);
    memset(present, sl->offsets ? 0 : 1, target_vocab);
    if (sl->offsets) {
        for (size_t i = 0; i < sl->first_num && i < target_vocab; ++i) present[i] = 1;
        for (size_t i = 0; i < n; ++i) {
            if (tokens[i] < 0) { free(present); return -1; }
            size_t t = (size_t)tokens[i];
            if (t >= source_vocab) { free(present); return -2; }
            for (uint64_t j = sl->offsets[t]; j < sl->offsets[t + 1]; ++j) present[sl->targets[j]] = 1;
        }
    }
    /* Marian's generation mask: UNK and the byte/control fallbacks */
    if (target_vocab > 1) present[1] = 0;
    if (target_vocab > 7) {
        size_t end = target_vocab < 39 ? target_vocab : 39;
        for (size_t i = 7; i < end; ++i) present[i] = 0;
    }
    size_t count = 0;
    for (size_t i = 0; i < target_vocab; ++i)
        if (present[i]) out[count++] = (uint32_t)i;
    /* pad to a multiple of 8 with the first absent ids from 50 up */
    for (size_t i = 50; i < target_vocab; ++i) {
        if (count % 8 == 0) break;
        if (!present[i]) out[count++] = (uint32_t)i;
    }
    free(present);
    qsort(out, count, sizeof(uint32_t), cmp_u32);
    if (count == 0) return -3;
    if (out[0] != 0) return -4;
    return (int64_t)count;
}

/* ---- q8_engine.rs:749-790 select_token ----------------------------------- */
static int64_t select_token_impl(const float *state, size_t dim, const int8_t *embedding,
                                 float embedding_mult, float activation_mult,
                                 const float *output_bias, const uint32_t *candidates,
                                 size_t n_candidates, int mask_eos, float *top2_gap) {
    if (n_candidates == 0) return -1;
    uint8_t *q = (uint8_t *)malloc(dim);
    if (oq_quantize_u8(state, dim, activation_mult, q) != 0) { free(q); return -2; }
    int16_t *centred = (int16_t *)malloc(dim * sizeof(int16_t));
    for (size_t i = 0; i < dim; ++i) centred[i] = (int16_t)((int)q[i] - ACTIVATION_ZERO_POINT);
    float inverse_scale = 1.0f / (activation_mult * embedding_mult);
    uint32_t best_token = candidates[0];
    float best = -INFINITY, second = -INFINITY;
    for (size_t c = 0; c < n_candidates; ++c) {
        uint32_t token = candidates[c];
        if (mask_eos && token == 0) continue;
        int32_t acc = dot_i8(centred, embedding + (size_t)token * dim, dim);
        float logit = (float)acc * inverse_scale + output_bias[token];
        if (logit > best) {
            second = best;
            best = logit;
            best_token = token;
        } else if (logit > second) {
            second = logit;
        }
    }
    if (top2_gap) *top2_gap = best - second;
    free(q);
    free(centred);
    return (int64_t)best_token;
}

int64_t oq_select_token(const float *state, size_t dim, const int8_t *embedding,
                        float embedding_mult, float activation_mult,
                        const float *output_bias, const uint32_t *candidates,
                        size_t n_candidates) {
    return select_token_impl(state, dim, embedding, embedding_mult, activation_mult,
                             output_bias, candidates, n_candidates, 0, NULL);
}

/* ---- q8_engine.rs:586-603 / :53-74 embedding ----------------------------- */
static float embedding_scale(int dim) {
    /* q8_engine.rs:22 hard-codes 19.595919 = sqrt(384) in f32; sqrtf(dim)
     * reproduces that constant exactly and generalises to other widths. */
    return sqrtf((float)dim);
}

static void embed_row(const int8_t *table, float mult, int32_t token, const float *pos,
                      int dim, float scale, float *dst) {
    const int8_t *row = table + (size_t)token * dim;
    for (int i = 0; i < dim; ++i) {
        float v = (float)row[i] / mult;
        dst[i] = v * scale + pos[i];
    }
}

/* ---- q8_engine.rs:632-651 feed_forward ----------------------------------- */
static int feed_forward(const oq_ffn_block *f, const float *x, size_t rows, int dim,
                        int ffn, float *out) {
    float *hidden = (float *)malloc(rows * ffn * sizeof(float));
    float *proj = (float *)malloc(rows * dim * sizeof(float));
    int rc = oq_linear_run(&f->w1, x, rows, hidden);
    if (rc == 0) {
        for (size_t i = 0; i < rows * (size_t)ffn; ++i) hidden[i] = fmaxf(hidden[i], 0.0f);
        rc = oq_linear_run(&f->w2, hidden, rows, proj);
    }
    if (rc == 0) oq_residual_layer_norm(proj, x, f->ln_scale, f->ln_bias, rows, dim, out);
    free(hidden);
    free(proj);
    return rc;
}

/* Self-attention block in the encoder's order (q8_engine.rs:526-557):
 * Q/K/V projections, masked attention, output projection, residual + LN. */
static int attention_block(const oq_attention_block *a, const float *x_query,
                           const float *key, const float *value,
                           const int32_t *lengths, size_t batch, size_t q_len,
                           size_t k_len, int dim, int heads, float *out) {
    size_t rows = batch * q_len;
    float *q = (float *)malloc(rows * dim * sizeof(float));
    float *att = (float *)malloc(rows * dim * sizeof(float));
    float *proj = (float *)malloc(rows * dim * sizeof(float));
    int rc = oq_linear_run(&a->wq, x_query, rows, q);
    if (rc == 0) rc = oq_attention(q, key, value, lengths, batch, q_len, k_len, dim, heads, att);
    if (rc == 0) rc = oq_linear_run(&a->wo, att, rows, proj);
    if (rc == 0) oq_residual_layer_norm(proj, x_query, a->ln_scale, a->ln_bias, rows, dim, out);
    free(q);
    free(att);
    free(proj);
    return rc;
}

/* ---- q8_engine.rs:353-466 translate_token_ids ---------------------------- */
int oq_translate(const oq_model *m, const float *positions,
                 const int32_t *tokens, const uint32_t *offsets, size_t batch,
                 const uint32_t *max_output_tokens, const uint32_t *force_len,
                 int32_t *out_tokens, uint32_t *out_offsets, size_t out_capacity,
                 oq_trace *trace, char *err, size_t errcap) {
    const int dim = m->dim, heads = m->heads, ffn = m->ffn_dim;
    if (err && errcap) err[0] = 0;
    /* validate_batch, q8_engine.rs:468-509 */
    if (batch == 0 || offsets[0] != 0) { set_err(err, errcap, "invalid packed batch offsets"); return -1; }
    if (batch > OQ_MAXIMUM_ENGINE_BATCH) {
        set_err(err, errcap, "batch contains %zu sentences; maximum is %d", batch, OQ_MAXIMUM_ENGINE_BATCH);
        return -1;
    }
    size_t lmax = 0;
    for (size_t b = 0; b < batch; ++b) {
        if (offsets[b + 1] <= offsets[b]) { set_err(err, errcap, "each input must contain at least one token"); return -1; }
        size_t len = offsets[b + 1] - offsets[b];
        if (len > lmax) lmax = len;
    }
    if (lmax > OQ_MAXIMUM_SOURCE_TOKENS) {
        set_err(err, errcap, "source has %zu tokens; pure Rust Q8 maximum is %d", lmax, OQ_MAXIMUM_SOURCE_TOKENS);
        return -1;
    }
    if (batch * lmax * lmax > OQ_MAXIMUM_PADDED_CELLS) {
        set_err(err, errcap, "padded attention work is %zu cells; pure Rust Q8 maximum is %d",
                batch * lmax * lmax, OQ_MAXIMUM_PADDED_CELLS);
        return -1;
    }
    size_t total = offsets[batch];
    for (size_t i = 0; i < total; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->source_vocab) {
            set_err(err, errcap, "source token %d is outside vocabulary %d", tokens[i], m->source_vocab);
            return -1;
        }

    /* encode, q8_engine.rs:511-574 (padded [B, Lmax]) */
    size_t rows = batch * lmax;
    int32_t *lengths = (int32_t *)malloc(batch * sizeof(int32_t));
    int32_t *padded = (int32_t *)calloc(rows, sizeof(int32_t));
    for (size_t b = 0; b < batch; ++b) {
        lengths[b] = (int32_t)(offsets[b + 1] - offsets[b]);
        memcpy(padded + b * lmax, tokens + offsets[b], lengths[b] * sizeof(int32_t));
    }
    float scale = embedding_scale(dim);
    float *x = (float *)malloc(rows * dim * sizeof(float));
    float *tmp = (float *)malloc(rows * dim * sizeof(float));
    float *kbuf = (float *)malloc(rows * dim * sizeof(float));
    float *vbuf = (float *)malloc(rows * dim * sizeof(float));
    for (size_t t = 0; t < rows; ++t)
        embed_row(m->encoder_embedding, m->encoder_embedding_mult, padded[t],
                  positions + (t % lmax) * dim, dim, scale, x + t * dim);
    int rc = 0;
    for (int l = 0; l < m->encoder_layers && rc == 0; ++l) {
        const oq_attention_block *a = &m->encoder_attention[l];
        rc = oq_linear_run(&a->wk, x, rows, kbuf);
        if (rc == 0) rc = oq_linear_run(&a->wv, x, rows, vbuf);
        if (rc == 0) rc = attention_block(a, x, kbuf, vbuf, lengths, batch, lmax, lmax, dim, heads, tmp);
        if (rc == 0) rc = feed_forward(&m->encoder_ffn[l], tmp, rows, dim, ffn, x);
    }
    if (trace && trace->encoder_output && rc == 0) memcpy(trace->encoder_output, x, rows * dim * sizeof(float));
    int L = m->decoder_layers;
    float *cross_k = (float *)malloc((size_t)L * rows * dim * sizeof(float));
    float *cross_v = (float *)malloc((size_t)L * rows * dim * sizeof(float));
    for (int l = 0; l < L && rc == 0; ++l) {
        rc = oq_linear_run(&m->decoder_context[l].wk, x, rows, cross_k + (size_t)l * rows * dim);
        if (rc == 0) rc = oq_linear_run(&m->decoder_context[l].wv, x, rows, cross_v + (size_t)l * rows * dim);
    }
    if (trace && rc == 0) {
        if (trace->cross_key) memcpy(trace->cross_key, cross_k, (size_t)L * rows * dim * sizeof(float));
        if (trace->cross_value) memcpy(trace->cross_value, cross_v, (size_t)L * rows * dim * sizeof(float));
    }

    /* prepare_candidates, q8_engine.rs:576-584: one list per sentence (the
     * same full-vocabulary list for every row without a shortlist) */
    const size_t tv = (size_t)m->target_vocab;
    uint32_t *cands = (uint32_t *)malloc((m->shortlist.offsets ? batch : 1) * tv * sizeof(uint32_t));
    size_t *n_cands = (size_t *)malloc(batch * sizeof(size_t));
    if (!m->shortlist.offsets) {
        size_t n0 = oq_full_vocab_candidates(tv, cands);
        for (size_t b = 0; b < batch; ++b) n_cands[b] = n0;
    } else {
        for (size_t b = 0; b < batch && rc == 0; ++b) {
            int64_t nc = oq_shortlist_candidates(&m->shortlist, (size_t)m->source_vocab, tv,
                                                 tokens + offsets[b], offsets[b + 1] - offsets[b],
                                                 cands + b * tv);
            if (nc == -3) { set_err(err, errcap, "lexical shortlist produced no candidates"); rc = -1; }
            else if (nc == -4) { set_err(err, errcap, "lexical shortlist does not contain EOS token 0"); rc = -1; }
            else if (nc < 0) { set_err(err, errcap, "invalid source token for the lexical shortlist"); rc = -1; }
            else n_cands[b] = (size_t)nc;
        }
    }

    /* limits, q8_engine.rs:369-379 */
    uint32_t *limits = (uint32_t *)malloc(batch * sizeof(uint32_t));
    uint32_t generation_limit = 0;
    for (size_t b = 0; b < batch; ++b) {
        uint64_t lim = max_output_tokens[b];
        if (force_len && force_len[b] < lim) lim = force_len[b];
        uint64_t by_len = (uint64_t)lengths[b] * (uint64_t)(m->max_length_factor > 1 ? m->max_length_factor : 1);
        if (by_len < lim) lim = by_len;
        if (lim > OQ_MAXIMUM_GENERATION_STEPS) lim = OQ_MAXIMUM_GENERATION_STEPS;
        if (lim > OQ_MAXIMUM_POSITION) lim = OQ_MAXIMUM_POSITION;
        limits[b] = (uint32_t)lim;
        if (limits[b] > generation_limit) generation_limit = limits[b];
    }

    float *states = (float *)calloc((size_t)L * batch * dim, sizeof(float));
    size_t self_cap = OQ_MAXIMUM_GENERATION_STEPS;
    float *self_k = NULL, *self_v = NULL;
    if (m->decoder_kind == OQ_DECODER_SELFATTN) {
        self_k = (float *)calloc((size_t)L * batch * self_cap * dim, sizeof(float));
        self_v = (float *)calloc((size_t)L * batch * self_cap * dim, sizeof(float));
    }
    int32_t *previous = (int32_t *)malloc(batch * sizeof(int32_t));
    unsigned char *finished = (unsigned char *)calloc(batch, 1);
    int32_t *generated = (int32_t *)malloc(batch * OQ_MAXIMUM_GENERATION_STEPS * sizeof(int32_t));
    uint32_t *gen_count = (uint32_t *)calloc(batch, sizeof(uint32_t));
    for (size_t b = 0; b < batch; ++b) previous[b] = -1;
    float *dx = (float *)malloc(batch * dim * sizeof(float));
    float *d1 = (float *)malloc(batch * dim * sizeof(float));
    float *d2 = (float *)malloc(batch * dim * sizeof(float));
    float *dq = (float *)malloc(batch * dim * sizeof(float));
    int32_t *self_len = (int32_t *)malloc(batch * sizeof(int32_t));

    for (uint32_t step = 0; step < generation_limit && rc == 0; ++step) {
        int all = 1;
        for (size_t b = 0; b < batch; ++b) {
            if (!finished[b] && step >= limits[b]) finished[b] = 1;
            all &= finished[b];
        }
        if (all) break;
        /* decoder_input, q8_engine.rs:605-630 */
        const float *pos = positions + (size_t)step * dim;
        for (size_t b = 0; b < batch; ++b) {
            if (previous[b] < 0) memcpy(dx + b * dim, pos, dim * sizeof(float));
            else embed_row(m->decoder_embedding, m->decoder_embedding_mult, previous[b], pos, dim,
                           scale, dx + b * dim);
        }
        for (int l = 0; l < L && rc == 0; ++l) {
            if (m->decoder_kind == OQ_DECODER_SSRU) {
                const oq_ssru_block *s = &m->decoder_ssru[l];
                rc = oq_linear_run(&s->w, dx, batch, d1);
                if (rc == 0) rc = oq_linear_run(&s->wf, dx, batch, d2);
                if (rc == 0) oq_ssru_update_layer_norm(d1, d2, states + (size_t)l * batch * dim, dx,
                                                      s->ln_scale, s->ln_bias, batch, dim, dq);
                if (rc == 0) memcpy(dx, dq, batch * dim * sizeof(float));
            } else {
                const oq_attention_block *a = &m->decoder_self[l];
                float *kc = self_k + (size_t)l * batch * self_cap * dim;
                float *vc = self_v + (size_t)l * batch * self_cap * dim;
                rc = oq_linear_run(&a->wk, dx, batch, d1);
                if (rc == 0) rc = oq_linear_run(&a->wv, dx, batch, d2);
                if (rc == 0) {
                    for (size_t b = 0; b < batch; ++b) {
                        memcpy(kc + (b * self_cap + step) * dim, d1 + b * dim, dim * sizeof(float));
                        memcpy(vc + (b * self_cap + step) * dim, d2 + b * dim, dim * sizeof(float));
                        self_len[b] = (int32_t)step + 1;
                    }
                    rc = attention_block(a, dx, kc, vc, self_len, batch, 1, self_cap, dim, heads, dq);
                }
                if (rc == 0) memcpy(dx, dq, batch * dim * sizeof(float));
            }
            if (rc != 0) break;
            /* cross attention: q8_engine.rs:412-430 */
            rc = attention_block(&m->decoder_context[l], dx, cross_k + (size_t)l * rows * dim,
                                 cross_v + (size_t)l * rows * dim, lengths, batch, 1, lmax, dim,
                                 heads, dq);
            if (rc == 0) rc = feed_forward(&m->decoder_ffn[l], dq, batch, dim, ffn, dx);
        }
        if (rc != 0) break;
        if (trace && trace->decoder_state_step0 && step == 0)
            memcpy(trace->decoder_state_step0, dx, batch * dim * sizeof(float));
        for (size_t b = 0; b < batch; ++b) {
            if (finished[b]) continue;
            int mask_eos = force_len && (uint64_t)step + 1 < (uint64_t)force_len[b];
            float gap = 0.0f;
            int64_t tok = select_token_impl(dx + b * dim, dim, m->decoder_embedding,
                                            m->decoder_embedding_mult,
                                            m->decoder_output_activation_mult, m->output_bias,
                                            cands + (m->shortlist.offsets ? b * tv : 0), n_cands[b],
                                            mask_eos, &gap);
            if (tok < 0) { rc = -2; break; }
            if (trace && trace->top2_gap) trace->top2_gap[b * OQ_MAXIMUM_GENERATION_STEPS + step] = gap;
            previous[b] = (int32_t)tok;
            generated[b * OQ_MAXIMUM_GENERATION_STEPS + gen_count[b]++] = (int32_t)tok;
            if (tok == 0) finished[b] = 1;
        }
    }
    if (rc != 0) {
        if (!err || !errcap || err[0] == 0)
            set_err(err, errcap, "activation contains a non-finite value or the shape is invalid");
    } else {
        size_t pos = 0;
        out_offsets[0] = 0;
        for (size_t b = 0; b < batch && rc == 0; ++b) {
            if (pos + gen_count[b] > out_capacity) {
                set_err(err, errcap, "output capacity %zu is too small", out_capacity);
                rc = -4;
                break;
            }
            memcpy(out_tokens + pos, generated + b * OQ_MAXIMUM_GENERATION_STEPS, gen_count[b] * sizeof(int32_t));
            pos += gen_count[b];
            out_offsets[b + 1] = (uint32_t)pos;
        }
    }
    free(lengths); free(padded); free(x); free(tmp); free(kbuf); free(vbuf);
    free(cross_k); free(cross_v); free(cands); free(n_cands); free(limits); free(states);
    free(self_k); free(self_v); free(previous); free(finished); free(generated);
    free(gen_count); free(dx); free(d1); free(d2); free(dq); free(self_len);
    return rc;
}
