/*
 * marian_cuda.h -- C ABI of libmarian_cuda.so, the B200 (sm_100a) backend for
 * marian-edge's Q8 greedy translation path.
 *
 * The ABI mirrors the engine seam a marian-edge backend calls.  Each entry
 * point names the reference interface it replaces (paths are relative to the
 * marian-edge repository):
 *
 *   mc_create / mc_load_marian_bin   Q8CpuEngine::from_bytes
 *                                    (crates/marian-cpu/src/q8_engine.rs:175-184)
 *                                    + MarianBinaryModel::parse
 *                                    (crates/marian-cpu/src/legacy_q8.rs:179-422)
 *   mc_translate_token_ids           CpuTokenEngine::translate_token_ids
 *                                    (crates/marian-cpu/src/backend.rs:48-57,
 *                                    q8_engine.rs:353-466)
 *   mc_submit / mc_step / mc_poll    the scheduler's worker loop
 *                                    (crates/marian-core/src/scheduler.rs:494-659)
 *                                    as a device-side continuous batcher
 *   mc_is_ready                      TranslationBackend::is_ready
 *                                    (crates/marian-core/src/backend.rs:16-18)
 *   mc_q8_gemm                       Q8Linear::run_into's integer GEMM and
 *                                    epilogue (crates/marian-cpu/src/q8_gemm.rs:380-448)
 *
 * Conventions
 *   - All pointers are plain host pointers unless a parameter says "device".
 *     The caller owns every buffer it passes; the engine owns its device
 *     memory.
 *   - An engine is not thread-safe; like a TranslationBackend it is created,
 *     used and destroyed on one thread (marian-core/src/backend.rs:3-7).
 *   - Every call returns an mc_status.  On failure mc_last_error() holds a
 *     message.  MC_INVALID_INPUT and MC_MODEL leave the engine usable; after
 *     MC_INFERENCE with a device fault, MC_CUDA or MC_DEVICE_TIMEOUT the engine
 *     reports mc_is_ready() == 0 (marian-core/src/scheduler.rs:616-621).
 */
#ifndef MARIAN_CUDA_H
#define MARIAN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MC_OK = 0,
    MC_INVALID_INPUT = 1,   /* BackendError::InvalidInput  (marian-core/src/types.rs:63) */
    MC_MODEL = 2,           /* BackendError::Model         (types.rs:67) */
    MC_INFERENCE = 3,       /* BackendError::Inference     (types.rs:69) */
    MC_DEVICE_TIMEOUT = 4,  /* a bounded device wait gave up */
    MC_CUDA = 5             /* a CUDA runtime call failed */
} mc_status;

typedef struct mc_engine mc_engine;

typedef struct {
    int32_t device;              /* CUDA device ordinal */
    uint32_t max_inflight;       /* decode slots (default 1024) */
    uint32_t max_encode_tokens;  /* packed source tokens per encoder pass (default 65536) */
    uint32_t page_tokens;        /* tokens per KV-cache page: 8, 16 (default) or 32 */
    uint32_t kv_pages;           /* pages per cache pool; 0 = enough for every slot at full length */
    uint32_t max_length_factor;  /* Architecture::max_length_factor, 1..8 (default 3) */
    uint32_t lanes;              /* concurrent decode lanes, 1..8 (default 1; 0 = default):
                                    the active rows are split over this many CUDA streams
                                    whose decode steps overlap on the GPU */
} mc_config;

typedef struct {
    int32_t dim, heads, ffn_dim;
    int32_t encoder_layers, decoder_layers;
    int32_t decoder_kind;        /* 0 = SSRU (reference graph), 1 = self+cross attention */
    int32_t source_vocab, target_vocab;
    uint64_t weight_bytes;       /* int8 + f32 bytes resident on the device */
} mc_model_info;

/* Fills *cfg with the defaults above. */
void mc_config_default(mc_config *cfg);

/* Creates an engine on cfg->device (CUDA context, stream, status word). */
mc_status mc_create(const mc_config *cfg, mc_engine **out);

/* Parses a Marian binary v1 model (legacy_q8.rs:179-422 rules), validates the
 * Q8 tensor schema (q8_engine.rs:1007-1048; SSRU or self-attention decoder)
 * and uploads it.  Sizes the activation buffers and caches. */
mc_status mc_load_marian_bin(mc_engine *e, const uint8_t *bytes, size_t len);

mc_status mc_model_info_get(const mc_engine *e, mc_model_info *info);

/* What mc_inspect_marian_bin found in a model file. */
typedef struct {
    uint64_t tensors;
    uint64_t dense_linears;       /* intgemm8 weights with an activation scale */
    uint64_t embeddings;          /* intgemm8 *_Wemb tables */
    uint64_t activation_scales;   /* *_QuantMultA scalars */
    uint64_t row_scaled_linears;  /* dense weights with *_QuantMultRows (extension below) */
    float decoder_output_alpha;   /* decoder_Wemb_QuantMultA, normalised; 0 if absent */
    int32_t engine_graph;         /* 1: the tensor set is a graph this engine runs */
    int32_t decoder_kind, dim, heads, encoder_layers, decoder_layers;  /* when engine_graph */
} mc_model_report;

/* Host-only check of a Marian binary v1 file, no device or engine needed:
 * MarianBinaryModel::parse and ::validate_q8 (crates/marian-cpu/src/
 * legacy_q8.rs:179-422, 497-542) -- header, names, shapes, 256-byte
 * alignment and zero padding, record lengths, trailing bytes, finite
 * positive multipliers, no -128, every activation scale a positive scalar
 * of an intgemm8 weight, every dense weight with its scale -- then the
 * engine's schema check (q8_engine.rs:1007-1101).  A format or Q8 error
 * returns MC_MODEL with the reason in message; a valid file the engine
 * cannot run returns MC_OK with engine_graph = 0 and the reason.
 *
 * Per-row extension (no counterpart in the reference, whose weights have one
 * multiplier per tensor): a dense weight W may come with a float32 tensor
 * W_QuantMultRows of shape [1, out], one multiplier per output row; the
 * weight's row n is then values[n, :] / W_QuantMultRows[n] and its outputs
 * dequantize with 1 / (alpha * W_QuantMultRows[n]).  mc_load_marian_bin
 * accepts such files. */
mc_status mc_inspect_marian_bin(const uint8_t *bytes, size_t len, mc_model_report *report,
                                char *message, size_t message_capacity);

/* Loads a Marian lexical shortlist (LexicalShortlist::from_bytes and
 * ::candidates, marian-model/src/shortlist.rs:59-198; the engine's
 * prepare_candidates, marian-cpu/src/q8_engine.rs:576-584): each sentence's
 * output token is then the argmax over its own candidates -- ids below
 * firstNum, the shortlist targets of its source tokens, minus UNK and ids
 * 7..38, padded to a multiple of 8 with the first absent ids from 50.
 * bytes == NULL restores the full vocabulary.  Requires a loaded model and
 * no requests in flight.  Malformed files return MC_MODEL; a sentence whose
 * candidates lack EOS (0) is rejected with MC_INFERENCE, as the reference
 * rejects it. */
mc_status mc_load_shortlist(mc_engine *e, const uint8_t *bytes, size_t len);

void mc_destroy(mc_engine *e);

/* Copies the last error message (NUL-terminated, truncated to cap) and
 * returns its full length. */
size_t mc_last_error(const mc_engine *e, char *buf, size_t cap);

/* 1 while the engine can accept work; 0 after a terminal device failure. */
int32_t mc_is_ready(const mc_engine *e);

/* Static batch translation, CpuTokenEngine::translate_token_ids semantics:
 * tokens[n_tokens] packed, offsets[batch+1] (offsets[0] = 0, last =
 * n_tokens, each source non-empty and ending in EOS = 0), max_output_tokens
 * [batch].  force_len (nullable) is the fixed-length harness rule: token 0 is
 * excluded while step < force_len[b] - 1 and the row stops after
 * min(max_output_tokens[b], force_len[b]) tokens.  Output: out_offsets
 * [batch+1] and out_tokens (EOS included when generated), capacity
 * out_capacity tokens. */
mc_status mc_translate_token_ids(mc_engine *e, const int32_t *tokens, size_t n_tokens,
                                 const uint32_t *offsets, uint32_t batch,
                                 const uint32_t *max_output_tokens, const uint32_t *force_len,
                                 int32_t *out_tokens, size_t out_capacity,
                                 uint32_t *out_offsets);

/* Continuous batching.  mc_submit queues one request (tokens end in EOS).
 * mc_step advances every decode lane by one step: it waits for the lane's
 * step in flight (if any) and applies its tokens, admits queued requests
 * into the lane's free slots (one packed encoder pass), and launches the
 * lane's next decode step over its active slots without waiting for it; so
 * a lane's tokens become visible one mc_step call after its step was
 * launched.  active_after counts the active slots of every lane, including
 * those of steps still in flight.  mc_poll returns finished requests:
 * ids[i], lengths[i] and their tokens packed in order into tokens (capacity
 * token_capacity).  Call mc_step until active_after and queued_after are
 * both 0 to drain every request. */
mc_status mc_submit(mc_engine *e, uint64_t request_id, const int32_t *tokens, uint32_t n_tokens,
                    uint32_t max_output_tokens, uint32_t force_len);
mc_status mc_step(mc_engine *e, uint32_t *active_after, uint32_t *queued_after);
mc_status mc_poll(mc_engine *e, uint64_t *ids, uint32_t *lengths, uint32_t max_results,
                  int32_t *tokens, size_t token_capacity, uint32_t *n_results);

/* Per-layer capture for parity tests: runs the encoder and the first decode
 * step of a static batch and copies (host buffers, padded [B, Lmax, dim]
 * layout as the reference uses, nullable): the encoder output, the cross
 * keys/values [decoder_layers, B, Lmax, dim] and the final decoder state of
 * step 0 [B, dim]. */
mc_status mc_trace_first_step(mc_engine *e, const int32_t *tokens, size_t n_tokens,
                              const uint32_t *offsets, uint32_t batch, float *encoder_output,
                              float *cross_key, float *cross_value, float *decoder_state);

/* Encoder pass only (Q8CpuEngine::encode with the cross-cache fill,
 * crates/marian-cpu/src/q8_engine.rs:511-574): one packed varlen encoder
 * pass over a static batch (same input rules as mc_translate_token_ids;
 * at most max_inflight sentences and max_encode_tokens tokens), its cross
 * keys/values written into cache pages, then every slot released.
 * encoder_output (nullable host buffer, packed [n_tokens, dim]) receives
 * the final encoder states in input order. */
mc_status mc_encode_token_ids(mc_engine *e, const int32_t *tokens, size_t n_tokens,
                              const uint32_t *offsets, uint32_t batch, float *encoder_output);

/* Replays an arrival schedule on the calling thread (measurement; the
 * scheduler worker loop's shape, crates/marian-core/src/scheduler.rs:494-659,
 * with the host clock as the arrival process): row b of the packed batch is
 * submitted once arrival_s[b] seconds (ascending) have passed since the
 * call began, steps run while anything is queued or decoding, and
 * latency_s[b] receives the seconds from its arrival to the step that
 * returned its last token.  Generated tokens are dropped.  Requires an idle
 * engine. */
mc_status mc_replay(mc_engine *e, const int32_t *tokens, size_t n_tokens, const uint32_t *offsets,
                    uint32_t batch, const uint32_t *max_output_tokens, const uint32_t *force_len,
                    const double *arrival_s, double *latency_s);

/* The engine's stream (a cudaStream_t), for callers that time or order work. */
void *mc_stream(const mc_engine *e);

/* Kernel classes for the optional per-launch timing of mc_profile.  (The
 * reference measures its hot spots with a CPU microbenchmark instead,
 * crates/marian-cpu/benches/hotspots.rs:45-185.) */
enum {
    MC_K_EMBED = 0,        /* embedding + positions (+ quantized copies) */
    MC_K_GEMM_QKV = 1,     /* Q/K/V, SSRU W/Wf and cross-attention Q projections */
    MC_K_GEMM_OUT = 2,     /* attention output projections */
    MC_K_GEMM_FFN1 = 3,    /* FFN W1 (+ReLU, quantized for W2) */
    MC_K_GEMM_FFN2 = 4,    /* FFN W2 */
    MC_K_GEMM_CROSSKV = 5, /* cross keys/values into the paged cache */
    MC_K_GEMM_VOCAB = 6,   /* tied vocabulary projection + masked argmax */
    MC_K_ATTN_ENC = 7,     /* packed varlen encoder self-attention */
    MC_K_ATTN_SELF = 8,    /* decode self-attention over the paged cache */
    MC_K_ATTN_CROSS = 9,   /* decode cross-attention over the paged cache */
    MC_K_LAYERNORM = 10,   /* residual + LayerNorm (+ quantized copies) */
    MC_K_SSRU = 11,        /* SSRU state update + LayerNorm */
    MC_K_FINALIZE = 12,    /* token selection bookkeeping */
    MC_K_GEMM_LN = 13,     /* output projection or FFN W2 fused with residual + LayerNorm */
    MC_KERNEL_KINDS = 14
};

/* Enables (1) or disables (0) per-launch CUDA-event timing on the engine
 * stream and clears the counters. */
mc_status mc_profile(mc_engine *e, int32_t enable);

/* Reads the counters of one kernel class: launches, total device
 * milliseconds, and the algorithmic flops and bytes of those launches. */
mc_status mc_profile_read(const mc_engine *e, int32_t kind, uint64_t *launches, double *ms,
                          double *flops, double *bytes);

/* Number of kernels the engine has launched since creation. */
uint64_t mc_launch_count(const mc_engine *e);

/* Decode-stream timeline (measurement only; the reference has no
 * counterpart).  mc_timeline(e, 1) clears the counters and records a pair
 * of events around every decode step; mc_timeline_read returns the steps
 * completed since, their summed device duration, and the summed idle time
 * of the decode streams between the end of one step and the start of the
 * next (host round trips, waits for admissions).  Off by default. */
mc_status mc_timeline(mc_engine *e, int32_t enable);
mc_status mc_timeline_read(const mc_engine *e, uint64_t *steps, double *busy_ms, double *idle_ms);

/* Device-level Q8 GEMM (benchmark / operator API), Q8Linear::run_into's
 * integer GEMM and epilogue.  a: device int8 [m, k] (centred activations,
 * i.e. the reference's u8 minus 127), w: device int8 [n, k] (canonical
 * [out, in]).  k must be a multiple of 16 and both bases 16-byte aligned.
 * mode 0 writes the raw int32 accumulators to out [m, n]; mode 1 writes
 * f32 out = acc * (row_scale[m] * col_scale[n]) + bias[n], then ReLU when
 * relu != 0, then + residual[m, n]; row_scale, bias and residual are
 * nullable device pointers.  Runs on stream (a cudaStream_t, 0 = default). */
mc_status mc_q8_gemm(const int8_t *a, const int8_t *w, int32_t m, int32_t n, int32_t k,
                     const float *row_scale, const float *col_scale, const float *bias,
                     const float *residual, int32_t relu, int32_t mode, void *out,
                     void *stream);

/* Device-level Q8 linear, Q8Linear::run_into (q8_gemm.rs:380-448): quantizes
 * the device f32 activations x [m, k] with activation_mult (ties-to-even,
 * clamped to +-127, q8_gemm.rs:569-590) into a stream-ordered scratch buffer
 * (cudaMallocAsync on stream, released after use), runs the int8 GEMM with
 * the device int8 weights w [n, k] (canonical [out, in]) and writes device
 * f32 y [m, n] = acc * (1 / (activation_mult * weight_mult)) + bias[n]
 * (bias nullable).  k must be a multiple of 16.  A non-finite activation
 * sets the non-finite bit read by mc_op_status (the reference returns an
 * error for it). */
mc_status mc_q8_linear(const float *x, int32_t m, int32_t k, const int8_t *w, int32_t n,
                       float activation_mult, float weight_mult, const float *bias, float *y,
                       void *stream);

/* Q8Linear::run_into followed by residual_layer_norm_into
 * (crates/marian-cpu/src/q8_gemm.rs:380-448, tensor.rs:132-155) in one
 * launch, as every Transformer sub-layer of the decoder ends:
 * y = LN(linear(x) + residual) * gamma + beta with eps 1e-6, the linear as
 * in mc_q8_linear (x [m, k] f32 quantized with activation_mult, w [d, k]
 * int8, bias [d] nullable).  residual and y are [m, d] f32; gamma and beta
 * [d].  y_q (nullable) also receives y quantized with y_alpha, centred
 * (the reference's u8 minus 127), as the next linear reads it.  d must be
 * 128, 256, 384 or 512 (else MC_INVALID_INPUT); x, residual, y, gamma and
 * beta 16-byte aligned.  Device pointers, asynchronous on `stream`; status
 * bits as mc_q8_linear (mc_op_status).  Bit-identical to mc_q8_linear
 * followed by the reference's residual LayerNorm. */
mc_status mc_q8_linear_ln(const float *x, int32_t m, int32_t k, const int8_t *w, int32_t d,
                          float activation_mult, float weight_mult, const float *bias,
                          const float *residual, const float *gamma, const float *beta, float *y,
                          int8_t *y_q, float y_alpha, void *stream);

/* Largest m * k accepted by mc_q8_linear_noalloc (bytes of quantized
 * activations in its fixed device scratch). */
#define MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS (8u * 1024u * 1024u)

/* mc_q8_linear without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc -- a host
 * application whose memory manager has reserved the GPU's memory for its own
 * pool, or a latency-critical path that cannot take an allocation's driver
 * call.  Same arguments and results as mc_q8_linear; the quantized
 * activations go to a fixed device array of
 * MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS bytes (plus a status word) that every
 * GPU using the library holds until the process exits.  m * k beyond that
 * size returns MC_INVALID_INPUT without launching anything.  The first call
 * on a device looks up the array's device address (make it before any
 * stream capture) and keeps it for the process: cudaDeviceReset after that
 * call is not supported.  All calls share the array: calls whose kernels
 * overlap on the GPU race.  status_bits (host pointer, nullable): when given, the
 * call synchronizes the stream and returns the status bits recorded since
 * the last report (bit 0: non-finite activation), clearing them; when null
 * the call stays asynchronous and the bits accumulate. */
mc_status mc_q8_linear_noalloc(const float *x, int32_t m, int32_t k, const int8_t *w, int32_t n,
                               float activation_mult, float weight_mult, const float *bias,
                               float *y, void *stream, uint32_t *status_bits);

/* Reads and clears the status word the operator API's kernels write on the
 * current device (non-finite quantizer input, wait timeout); synchronizes. */
mc_status mc_op_status(uint32_t *status_bits);

/* ---- long-text splitting ----------------------------------------------------
 * Replaces marian_core::segment_text (crates/marian-core/src/segmenter.rs:
 * 122-197), which the reference's backends call before tokenizing a request
 * (crates/marian-cpu/src/backend.rs:132-135).  Host-only; no engine needed. */

/* One range of the input: content[start, end) to translate, followed by
 * separator[start, end) to copy to the output verbatim (segmenter.rs:26-46).
 * The ranges of all segments partition the input in order. */
typedef struct {
    uint64_t content_start, content_end;
    uint64_t separator_start, separator_end;
    uint64_t source_pieces;   /* the counter's value for the content */
} mc_text_segment;

/* SegmentError (segmenter.rs:48-72) plus the two failures only a C caller
 * can cause. */
typedef enum {
    MC_SEGMENT_OK = 0,
    MC_SEGMENT_ZERO_PIECE_LIMIT = 1,
    MC_SEGMENT_INPUT_TOO_LARGE = 2,       /* end: input bytes; maximum: 4 MiB */
    MC_SEGMENT_ENCODING = 3,              /* start, end: the range the counter failed on */
    MC_SEGMENT_ENCODING_WORK_LIMIT = 4,   /* maximum: the exceeded limit */
    MC_SEGMENT_TOO_MANY_SEGMENTS = 5,     /* maximum: 4096 */
    MC_SEGMENT_UNSPLITABLE_SCALAR = 6,    /* start, end, pieces, maximum */
    MC_SEGMENT_INVALID_UTF8 = 7,          /* a Rust &str cannot hold such bytes */
    MC_SEGMENT_INVALID_ARGUMENT = 8       /* null pointers, or capacity too small */
} mc_segment_error_kind;

typedef struct {
    int32_t kind;              /* mc_segment_error_kind */
    uint64_t start, end, pieces, maximum;
    char message[256];         /* the reference's Display text (segmenter.rs:74-110) */
} mc_segment_error;

/* The caller's exact source-piece counter for text[0, len) (the closure of
 * segment_text).  Returns 0 and sets *pieces, or non-zero with a message
 * (NUL-terminated, at most message_capacity bytes) on a tokenizer failure. */
typedef int32_t (*mc_piece_count_fn)(void *ctx, const char *text, size_t len, uint64_t *pieces,
                                     char *message, size_t message_capacity);

/* Splits text (UTF-8, len bytes) into segments whose content fits
 * max_pieces.  Writes *n_segments (at most 4096) and, when they fit
 * capacity, the segments.  Every failure returns MC_INVALID_INPUT (the
 * reference backend's BackendError::InvalidInput) and fills *error when
 * given; on success error->kind is MC_SEGMENT_OK. */
mc_status mc_segment_text(const char *text, size_t len, uint64_t max_pieces,
                          mc_piece_count_fn count_pieces, void *ctx, mc_text_segment *segments,
                          size_t capacity, size_t *n_segments, mc_segment_error *error);

#ifdef __cplusplus
}
#endif
#endif
