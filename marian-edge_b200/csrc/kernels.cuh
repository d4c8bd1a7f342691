// kernels.cuh -- launchers for the non-GEMM kernels of the Q8 greedy path.
//
// Floating-point kernels are compiled with --fmad=false so every a*b+c keeps
// two roundings, as the reference's Rust does; reductions whose order the
// reference fixes (LayerNorm sums, attention dot products, softmax sums,
// attention output accumulation) are evaluated in that same sequential order
// by one thread each.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mc {

constexpr int kMaxQuantOut = 8;
constexpr int kMaxPosition = 4096;   // marian-model/src/manifest.rs:13
constexpr int kMaxSeq = 256;         // source tokens and generation steps

// Quantized copies of one f32 activation, one per consuming linear (each
// linear has its own static activation alpha).  Copy i lives at
// base + i * stride (int8, centred).
struct QuantOut {
  int8_t* base;
  long long stride;
  int count;
  float alpha[kMaxQuantOut];
};

// q8_engine.rs:586-603: x = (emb[tok] / qm) * scale + pos[p] for packed tokens.
void launch_embed_encoder(const int32_t* tokens, const int32_t* pos_idx, int n_tokens,
                          const int8_t* emb, float emb_mult, float emb_scale,
                          const float* positions, int d, float* x, const QuantOut& q,
                          uint32_t* status, cudaStream_t s);

// q8_engine.rs:605-630 for one decode step of the active rows.  Also writes
// the per-row EOS mask (harness rule) and the self-attention cache row of
// this step (when self_pages != nullptr).
//
// Decode-step launchers take `rows` (the grid's row capacity) and a nullable
// device row count `rows_dev` that, when given, the kernels read and clamp
// to rows: a CUDA graph captured once for a lane's capacity then serves
// every active-row count.
void launch_embed_decoder(int rows, const int32_t* rows_dev, const int32_t* row_slot,
                          const int32_t* slot_prev,
                          const int32_t* slot_step, const int32_t* slot_force, const int8_t* emb,
                          float emb_mult, float emb_scale, const float* positions, int d, float* x,
                          const QuantOut& q, uint8_t* eos_mask, const int32_t* self_pages,
                          int pages_per_slot, int page_tokens, int32_t* self_row_map,
                          uint32_t* status, cudaStream_t s);

// tensor.rs:132-155: out = LN(a + r) (eps 1e-6) plus quantized copies.
void launch_residual_ln(const float* a, int lda, const float* r, int ldr, const float* gamma,
                        const float* beta, int rows, const int32_t* rows_dev, int d, float* out,
                        const QuantOut& q, uint32_t* status, cudaStream_t s);

// tensor.rs:184-218: SSRU gate/state update, ReLU + residual, LN, quantized
// copies.  cand/fpre are [rows, ld] with the candidate at column 0 and the
// forget pre-activation at column fcol; state is [slots, d] indexed by slot.
void launch_ssru(const float* cf, int ld, int fcol, float* state, const int32_t* row_slot,
                 const float* residual, const float* gamma, const float* beta, int rows,
                 const int32_t* rows_dev, int d, float* out, const QuantOut& q, uint32_t* status,
                 cudaStream_t s);

// tensor.rs:251-318 for packed varlen sequences (no padding): qkv is
// [tokens, 3d] (Q | K | V), cu_seqlens [batch+1]; this launch covers the
// n_seqs sequences listed in seq_ids, none longer than max_len.  Output
// quantized with the output projection's alpha into out_q [tokens, d].
cudaError_t launch_attn_encoder(const float* qkv, const int32_t* cu_seqlens,
                                const int32_t* seq_ids, int n_seqs, int max_len, int d, int heads,
                                int8_t* out_q, float alpha, uint32_t* status, cudaStream_t s);

// A KV pool's tensor maps for the decode attention: boxes of 8, 4, 2 and 1
// cache rows (encode_tmap_kv with group_cols = 4 * d / heads).  Full groups
// of 8 keys use the first; a row's last, partial group uses the smallest
// box that covers it, so at most half a box is read past its last key.
struct alignas(64) KvBoxMaps {
  CUtensorMap box[4];  // box rows 8, 4, 2, 1
};

// tensor.rs:251-318 with one query per row over a paged cache: keys of row r
// are cache rows page_table[slot][j / page_tokens] * page_tokens +
// j % page_tokens for j < slot_len[slot] + len_add, read through the
// pools' tensor maps.  row_order (nullable) lists the rows in the order the
// kernel takes them.  page_tokens is 8, 16 or 32.
cudaError_t launch_attn_decode(const float* q, int ldq, int rows, const int32_t* rows_dev,
                               const int32_t* row_slot, const int32_t* row_order,
                               const int32_t* slot_len, int len_add, const int32_t* page_table,
                               int pages_per_slot, int page_tokens, const KvBoxMaps* k_maps,
                               const KvBoxMaps* v_maps, int d, int heads, int8_t* out_q,
                               float alpha, uint32_t* status, cudaStream_t s);

// Turns the packed per-row maxima into tokens (q8_engine.rs:437-449):
// advances each slot's step/previous token, reports the token and whether
// the row finished (token 0 or its limit), and clears the maxima.
void launch_finalize(int rows, const int32_t* rows_dev, const int32_t* row_slot,
                     unsigned long long* best,
                     int32_t* slot_prev, int32_t* slot_step, const int32_t* slot_limit,
                     int32_t* step_tokens, uint8_t* done, uint32_t* status, cudaStream_t s);

// q8_gemm.rs:569-590: out[i] = clamp(rte(x[i] * alpha), -127, 127) for n
// values (n a multiple of 4), stored centred (the reference's u8 minus 127).
void launch_quantize(const float* x, long long n, float alpha, int8_t* out, uint32_t* status,
                     cudaStream_t s);

// shortlist.rs:150-198 on the device: for admitted request i (slot
// slots[i], source tokens tokens[cu[i] .. cu[i + 1])) writes the candidate
// bitmask masks[slot][(vocab + 31) / 32] of the lexical shortlist
// (offsets[source_vocab + 1], targets, first_num).  vocab <= 393,216.
void launch_shortlist_masks(int n, const int32_t* slots, const int32_t* tokens, const int32_t* cu,
                            const int32_t* offsets, const int32_t* targets, int first_num, int vocab,
                            uint32_t* masks, cudaStream_t s);

// The row table of one decode step, built on the device (one CTA):
// table = [count, 3 unused, row_slot[rmax], order_self[rmax],
// order_cross[rmax]] holds the previous step's rows on entry; rows whose
// `done` flag that step set are dropped (the others keep their order), the
// slots of join = [n, slot...] are appended, and the orders list the rows
// with the most self keys (step + 1) and cross keys (source length) first.
// scratch is [rmax] int32.  A bad slot or join count sets kStatusBadIndex.
void launch_step_rows(int32_t* table, int rmax, const uint8_t* done, const int32_t* join,
                      const int32_t* slot_step, const int32_t* slot_src, int32_t* scratch,
                      uint32_t* status, cudaStream_t s);

// Initializes newly admitted slots: prev = -1, step = 0, limit, force_len,
// source length, SSRU states zeroed (state pools [layers][slots][d]), and
// copies each slot's page-table rows from page_rows ([n][pages_per_slot]
// cross pages, then [n][pages_per_slot] self pages; self_pages nullable).
void launch_init_slots(int n, const int32_t* slots, const int32_t* limits, const int32_t* force,
                       const int32_t* src_len, int32_t* slot_prev, int32_t* slot_step,
                       int32_t* slot_limit, int32_t* slot_force, int32_t* slot_src,
                       float* ssru_state, int layers, int max_slots, int d,
                       const int32_t* page_rows, int32_t* cross_pages, int32_t* self_pages,
                       int pages_per_slot, cudaStream_t s);

}  // namespace mc
