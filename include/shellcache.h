/*
 * shellcache: C ABI of the B200 (sm_100a) rollout-cache path.
 *
 * The path is the decode-time cache work of a hybrid gated-delta-net (GDN) /
 * full-attention decoder, as served by shellsmith's studio_compute sampler:
 *   - the GDN recurrent-state update for one token (and for chunked prefill),
 *   - the append of new keys/values into a paged KV pool,
 *   - split-K decode attention over ragged pages, and its (out, lse) combine.
 *
 * Conventions (every entry point):
 *   - Returns 0 on success, or a positive SC_ERR_* code. No C++ exception
 *     crosses this boundary. sc_last_error() gives the text of the most recent
 *     nonzero status on the calling host thread.
 *   - Every tensor pointer is a device pointer. The caller owns every buffer.
 *     Tensors are dense and row-major in the shape written beside them.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is only
 *     enqueued; nothing synchronises unless the comment says so.
 *   - sc_bf16 is the raw 16-bit pattern of a bfloat16 value.
 *
 * Paged KV pool layout (defined by this library; the reference has no paging):
 *   kv_pool[num_pages][Hkv][2][P][D] bf16, index 0 = keys, 1 = values,
 *   P = page size in tokens. Inside one (page, kv head, K|V) block the row of
 *   token t stores its 16-byte chunk c at chunk position c ^ (t & 7), so one
 *   bulk copy of the block lands in shared memory already bank-swizzled for
 *   ldmatrix. Use sc_kv_gather() to read logical keys/values back.
 *   A slot is page * P + offset; a negative slot means "skip this token".
 */
#ifndef SHELLCACHE_H
#define SHELLCACHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t sc_bf16;

enum {
  SC_OK = 0,
  SC_ERR_INVALID = 1,      /* bad shape, pointer or argument          */
  SC_ERR_UNSUPPORTED = 2,  /* shape outside the compiled kernel set    */
  SC_ERR_CUDA = 3,         /* a CUDA runtime call or launch failed     */
  SC_ERR_DEVICE = 4        /* a kernel reported a device-side fault    */
};

/* Library version (major * 10000 + minor * 100 + patch). */
int sc_version(void);

/* Copies the text of the last nonzero status on this host thread into buf
 * (NUL-terminated, at most n bytes). Returns the last status code. */
int sc_last_error(char* buf, int n);

/* Reads the device-side status word that kernels set when a bounded wait
 * gives up or an index is out of range (0 = clean), then clears it.
 * Synchronises `stream`. Returns SC_OK or SC_ERR_CUDA. */
int sc_device_status(unsigned int* status, void* stream);

/* --------------------------------------------------------------------------
 * (a) GDN single-token recurrent update, state updated IN PLACE.
 *
 * Replaces studio_compute/numerics/gdn_token.py:18-42 `gated_delta_token`
 * (kernel shellsmith_bf16_gdn_token_v1, gdn_token.py:45-79). For each row b,
 * value head h (key head h / (Hv / Hk)) and value row i:
 *   decayed  = g[b,h] * S[i,:]
 *   delta    = beta[b,h] * (v[b,h,i] - decayed . k)
 *   S[i,:]   = decayed + delta * k          (stored back into `state`)
 *   out[b,h,i] = S[i,:] . q
 *
 * q, k   [B, Hk, dk] bf16       (already L2-normalised, as the reference's
 *                                 _normalize_qk leaves them)
 * v      [B, Hv, dv] bf16
 * g      [B, Hv] fp32           multiplicative decay a_t = exp(g_t)
 * beta   [B, Hv] fp32
 * state  [slots, Hv, dv, dk]    fp32 (sc_gdn_decode) or bf16 (_bf16 variant)
 * state_slot [B] int32          state row of batch row b; NULL = identity;
 *                                 a negative entry skips the row; an entry
 *                                 >= num_slots (rows in `state`) is flagged
 *                                 (DEV_BAD_INDEX) and skipped
 * out    [B, Hv, dv] bf16
 * Supported: dk in {32, 64, 128, 256}, Hv % Hk == 0, dv >= 1.
 * The bf16 variant reproduces the reference rounding points: the decayed
 * state is fp32, the updated state is rounded to bf16 and the output is
 * taken from the rounded state (gdn_token.py:60-77).
 * ------------------------------------------------------------------------ */
int sc_gdn_decode(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                  const float* g, const float* beta, float* state,
                  const int32_t* state_slot, sc_bf16* out, int B, int Hk, int Hv,
                  int dk, int dv, int num_slots, void* stream);

int sc_gdn_decode_bf16(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                       const float* g, const float* beta, sc_bf16* state,
                       const int32_t* state_slot, sc_bf16* out, int B, int Hk,
                       int Hv, int dk, int dv, int num_slots, void* stream);

/* sc_gdn_decode for a chain of layers (no reference counterpart: the same
 * math). The caller promises that the kernel queued just before it on the
 * stream writes neither the state rows this call reads nor state_slot (e.g.
 * it is another layer's update, or an attention layer): the state then
 * streams in while that kernel still runs. Consecutive calls on the SAME
 * state rows must use sc_gdn_decode. */
int sc_gdn_decode_chained(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                          const float* g, const float* beta, float* state,
                          const int32_t* state_slot, sc_bf16* out, int B, int Hk,
                          int Hv, int dk, int dv, int num_slots, void* stream);

/* GDN chunked prefill (chunk 64) on tcgen05 tensor cores, state IN PLACE.
 *
 * Replaces studio_compute/numerics/ops.py:151-215 `gated_delta_chunked`
 * (and the fused numerics/gdn_fused.py:86-122 `gated_delta_chunks` once its
 * gates are made): runs every token of each sequence through the recurrence
 * above, starting from its state row and leaving the final state there.
 *
 * Packed token-major layout: token n of sequence b is row
 * cu_seqlens[b] + n (or b * T + n when cu_seqlens is NULL).
 * q, k   [tokens, Hk, 128] bf16 (L2-normalised), 16-byte aligned
 * v      [tokens, Hv, 128] bf16
 * g      [tokens, Hv] fp32 multiplicative decay (clamped to [1e-6, 1] before
 *        its log, as the reference's fp32 chunk path does); beta [tokens, Hv]
 * state  [num_slots, Hv, 128, 128] fp32; state_slot [B] int32 or NULL
 *        (identity); a slot >= num_slots is flagged and its sequence skipped
 * cu_seqlens [B + 1] int32 or NULL (then every sequence has T tokens)
 * out    [tokens, Hv, 128] bf16
 * total_tokens  number of packed tokens when cu_seqlens is given
 * Supported: dk = dv = 128, Hv % Hk == 0. */
int sc_gdn_chunk_prefill(const sc_bf16* q, const sc_bf16* k, const sc_bf16* v,
                         const float* g, const float* beta, float* state,
                         const int32_t* state_slot, const int32_t* cu_seqlens,
                         sc_bf16* out, int B, int T, int total_tokens, int Hk, int Hv,
                         int dk, int dv, int num_slots, void* stream);

/* --------------------------------------------------------------------------
 * (a) GDN layer glue: conv taps, SiLU, q/k norm, gates, gated RMS norm.
 *
 * Replaces the decode-time GDN layer between its projections and out_proj:
 * studio_compute/numerics/bf16.py:44-139 `gdn_inner` (decode_one=True branch)
 * called from `_decode_gdn_token` (bf16.py:191-210), which runs
 * conv1d + SiLU, `_normalize_qk`, the gates of bf16.py:98-102,
 * gated_delta_token and rms_norm(y) * silu(z) as separate MLX ops.
 * Every value is rounded to bf16 where the reference's ops round.
 *
 * Shapes (C = 2*Hk*128 + Hv*128 channels, q | k | v; dk = dv = 128):
 * qkv  [B, C] bf16 (in_proj_qkv output)   z [B, Hv*128] bf16 (in_proj_z)
 * a, b [B, Hv] bf16 (in_proj_a / in_proj_b)
 * conv_w [C, 4] bf16 (the depthwise conv1d weight [C, 4, 1]), 8-byte aligned
 * A_log, dt_bias [Hv] fp32; norm_w [128] bf16; eps of the gated norm
 * taps [num_slots, 4, C] bf16 in/out: a ring of the last inputs; the token at
 *        absolute position t reads rows (t-3..t-1) & 3 and writes row t & 3.
 *        The reference's taps[B, 3, C] are rows (t-3..t-1) & 3 in order; a new
 *        sequence's ring starts at zero.
 * position [B] int32: absolute position t of each row's token (>= 0)
 * state, state_slot, num_slots: as sc_gdn_decode (fp32 state, -1 skips a row)
 * out  [B, Hv*128] bf16: rms_norm(y, norm_w, eps) * silu(z)
 * Launches one 2-CTA cluster per (row, value head). Experimental: on B200 this
 * one-launch form is slower than the three-kernel sc_gdn_decode_glue (0.24
 * against 0.18 ms per config-3 layer: the front and the cluster handshake cut
 * the state bytes each CTA keeps in flight); the engine uses the glue. */
int sc_gdn_decode_fused(const sc_bf16* qkv, const sc_bf16* z, const sc_bf16* a,
                        const sc_bf16* b, const sc_bf16* conv_w, const float* A_log,
                        const float* dt_bias, const sc_bf16* norm_w, float eps,
                        sc_bf16* taps, const int32_t* position, float* state,
                        const int32_t* state_slot, sc_bf16* out, int B, int Hk, int Hv,
                        int num_slots, void* stream);

/* The same layer step as sc_gdn_decode_fused, in three kernels: the front over
 * the rows (which also stores the new tap rows), the bulk-copy state update
 * (launched as a programmatic dependent of the front, so its state loads
 * overlap it) and the gated norm. Same arguments, plus a device workspace of
 * at least sc_gdn_decode_glue_workspace(B, Hk, Hv) bytes, 256-byte aligned,
 * that holds q/k/v/g/beta and the pre-norm output between the kernels. After
 * the call it holds, each part starting on a 256-byte boundary in this order:
 * q, k [B, Hk, 128] bf16, v [B, Hv, 128] bf16, y [B, Hv, 128] bf16 (the
 * recurrence output before the gated norm), g, beta [B, Hv] fp32.
 * Slots must be distinct across rows (state_slot NULL: row b uses slot b). */
size_t sc_gdn_decode_glue_workspace(int B, int Hk, int Hv);
int sc_gdn_decode_glue(const sc_bf16* qkv, const sc_bf16* z, const sc_bf16* a,
                       const sc_bf16* b, const sc_bf16* conv_w, const float* A_log,
                       const float* dt_bias, const sc_bf16* norm_w, float eps,
                       sc_bf16* taps, const int32_t* position, float* state,
                       const int32_t* state_slot, sc_bf16* out, void* workspace,
                       size_t workspace_bytes, int B, int Hk, int Hv, int num_slots,
                       void* stream);

/* The same front for the packed prompt tokens of a prefill (bf16.py:44-102 with
 * L > 1): sequence s is tokens cu_seqlens[s]..cu_seqlens[s+1] of qkv [tokens, C],
 * a, b [tokens, Hv]; it continues from position seq_start[s] of state slot
 * seq_slot[s], reading that slot's tap ring for the first three tokens.
 * Writes the inputs of sc_gdn_chunk_prefill: q, k [tokens, Hk, 128],
 * v [tokens, Hv, 128] bf16, g, beta [tokens, Hv] fp32. With cu_seqlens it does
 * not write taps (sc_gdn_taps_store does, afterwards). cu_seqlens may be NULL
 * when every sequence is one token (nseq == tokens: a decode batch, seq_start =
 * each row's position, distinct slots); then it also stores each row's input
 * into ring row position & 3, completing the step's taps. seq_slot -1 skips. */
int sc_gdn_prefill_front(const sc_bf16* qkv, const sc_bf16* a, const sc_bf16* b,
                         const sc_bf16* conv_w, const float* A_log, const float* dt_bias,
                         sc_bf16* taps, const int32_t* cu_seqlens,
                         const int32_t* seq_slot, const int32_t* seq_start, sc_bf16* q,
                         sc_bf16* k, sc_bf16* v, float* g, float* beta, int nseq,
                         int total_tokens, int Hk, int Hv, int num_slots, void* stream);

/* After a prefill (stream-ordered after sc_gdn_prefill_front): each sequence's
 * last min(3, n) inputs into its tap ring (the new taps of bf16.py:137).
 * cu_seqlens NULL: sequence s is token s; seq_slot -1 skips a sequence. */
int sc_gdn_taps_store(const sc_bf16* qkv, sc_bf16* taps, const int32_t* cu_seqlens,
                      const int32_t* seq_slot, const int32_t* seq_start, int nseq,
                      int channels, int num_slots, void* stream);

/* Gates of the fused chunk path from their logits, for gated_delta_chunks.
 *
 * Replaces the gate math that the reference's fused chunk kernel makes per row
 * (numerics/metal/gdn_chunk_common.metal:61-75 `sampler_gate`, `sampler_beta`,
 * behind numerics/gdn_fused.py:86-122 `gated_delta_chunks`): with each step in
 * fp32 and rounded to bf16,
 *   g    = bf16(exp(bf16(-bf16(exp(bf16(A_log))) * sp))),
 *   sp   = bf16(max(x, 0) + log(1 + exp(-|x|))),  x = bf16(a + bf16(dt_bias)),
 *   beta = bf16(1 / (1 + exp(-b))).
 * a, b [rows, Hv] bf16 logits (-inf marks a padded row: g = 1, beta = 0);
 * A_log, dt_bias [Hv] fp32; g, beta [rows, Hv] fp32 out. g is not clamped:
 * sc_gdn_chunk_prefill clamps it at 1e-6 before its log, as the reference does. */
int sc_gdn_sampler_gates(const sc_bf16* a, const sc_bf16* b, const float* A_log,
                         const float* dt_bias, float* g, float* beta, int64_t rows, int Hv,
                         void* stream);

/* out = rms_norm(y, w, eps) * silu(z) over rows of `width` (a multiple of 128):
 * bf16.py:129-135 for any number of rows (the prefill output). y, z, out
 * [rows, width] bf16, w [width] bf16, all 8-byte aligned. */
int sc_gated_rmsnorm(const sc_bf16* y, const sc_bf16* z, const sc_bf16* w, float eps,
                     sc_bf16* out, long long rows, int width, void* stream);

/* --------------------------------------------------------------------------
 * (b) KV append: scatter new keys/values into the paged pool.
 *
 * Replaces the KV write of mlx-vlm KVCache.update_and_fetch and
 * studio_compute/mlx_request_cache.py:59-63 `OwnedKV.update_and_fetch`
 * (concatenate along L), called from mlx_decode.py:94-100 through
 * _prepare_projected_qkv.
 *
 * k, v          [ntok, Hkv, D] bf16
 * slot_mapping  [ntok] int64, slot = page * P + offset, < 0 = skip
 * kv_pool       [num_pages, Hkv, 2, P, D] bf16 (layout above)
 * Supported: D in {64, 128, 256}, P in {8, 16, 32}.
 * ------------------------------------------------------------------------ */
int sc_kv_append(const sc_bf16* k, const sc_bf16* v, sc_bf16* kv_pool,
                 const int64_t* slot_mapping, int ntok, int Hkv, int D, int P,
                 int64_t num_pages, void* stream);

/* Reads logical keys/values back out of the pool: for each token i,
 * k_out[i] / v_out[i] ([Hkv, D]) = the entries at slot_mapping[i]
 * (zeros where the slot is negative). The inverse of sc_kv_append. */
int sc_kv_gather(const sc_bf16* kv_pool, const int64_t* slot_mapping,
                 sc_bf16* k_out, sc_bf16* v_out, int ntok, int Hkv, int D, int P,
                 int64_t num_pages, void* stream);

/* Copies whole pages inside a pool: page dst[i] <- page src[i], all heads.
 * The copy-on-write step of a forked prefix (replaces the private copies of
 * studio_compute/mlx_request_cache.py:15-39 `fork_cache`). */
int sc_kv_copy_pages(sc_bf16* kv_pool, const int32_t* src, const int32_t* dst,
                     int npages, int Hkv, int D, int P, int64_t num_pages,
                     void* stream);

/* --------------------------------------------------------------------------
 * (b') 8-bit KV pages (cache_precision = "8bit").
 *
 * Replaces the 8-bit cache of studio_compute/inference.py:87-94 (each layer's
 * cache made an mlx-vlm QuantizedKVCache: 8 bits, groups of 64 along D, a
 * scale and bias per group, attention on the dequantised rows). Rule of this
 * build (the library's own rounding is not in the reference tree):
 *   scale = bf16((max - min) / 255), bias = bf16(min),
 *   code = clamp(rint((w - bias) / scale), 0, 255), 0 when scale == 0.
 * Pool: uint8 [num_pages][Hkv][34 * D] (sc_kv_q8_block_bytes(D) per page and
 * kv head: K codes, V^T codes in the tensor-core fragment order, then K/V
 * scale and bias [16][D/64] bf16). D in {128, 256}, P = 16. */
int sc_kv_q8_block_bytes(int D);
int sc_kv_append_q8(const sc_bf16* k, const sc_bf16* v, uint8_t* kv_pool,
                    const int64_t* slot_mapping, int ntok, int Hkv, int D, int P,
                    int64_t num_pages, void* stream);
/* codes [ntok][Hkv][2][D] uint8 (K, V), scale_bias [ntok][Hkv][2][D/64][2] bf16. */
int sc_kv_gather_q8(const uint8_t* kv_pool, const int64_t* slot_mapping, int ntok, int Hkv,
                    int D, int P, int64_t num_pages, uint8_t* codes, sc_bf16* scale_bias,
                    void* stream);
int sc_kv_copy_pages_q8(uint8_t* kv_pool, const int32_t* src, const int32_t* dst, int npages,
                        int Hkv, int D, int P, int64_t num_pages, void* stream);
/* sc_paged_decode_attention over an 8-bit pool (same split plan, partials and
 * combine); kv_pool 16-byte aligned. */
int sc_paged_decode_attention_q8(const sc_bf16* q, const uint8_t* kv_pool, int64_t num_pages,
                                 const int32_t* block_table, const int32_t* ctx_len,
                                 const int32_t* seq_order, int B,
                                 int Hq, int Hkv, int D, int P, int max_pages,
                                 int pages_per_split, int num_splits, float scale,
                                 float* part_out, float* part_lse, sc_bf16* out, float* lse_out,
                                 void* stream);

/* --------------------------------------------------------------------------
 * (c) Split-K paged decode attention (one query token per sequence).
 *
 * Replaces the per-request decode SDPA of studio_compute/mlx_decode.py:80-106
 * `_attention_rows` (mlx-vlm scaled_dot_product_attention over the cache).
 * The math is scripts/mlx_attention_qualify.py:234-275 `numpy_attention`
 * with one query at offset ctx_len - 1 (attends to every cached token):
 *   out[b,h] = softmax(scale * q[b,h] . K_b[j]^T) V_b[j],  j < ctx_len[b],
 *   kv head of h = h / (Hq / Hkv).
 *
 * q            [B, Hq, D] bf16
 * kv_pool      [num_pages, Hkv, 2, P, D] bf16
 * block_table  [B, max_pages] int32 (row stride max_pages); an entry outside
 *              [0, num_pages) sets the device status word (DEV_BAD_INDEX)
 * ctx_len      [B] int32, tokens to attend (includes the appended token)
 * seq_order    [B] int32 or NULL: a permutation of 0..B-1, the order in which
 *              the sequences' CTAs launch (longest first keeps the last wave
 *              short on ragged batches); NULL launches in row order
 * pages_per_split  pages one CTA reduces; the sequence is cut into
 *                  ceil(ceil(ctx_len / P) / pages_per_split) splits
 * num_splits   grid bound: >= the largest split count in the batch
 * part_out     [B, Hq, num_splits, D] fp32 scratch (normalised partials)
 * part_lse     [B, Hq, num_splits] fp32 scratch (natural-log partial lse)
 * out          [B, Hq, D] bf16
 * lse_out      [B, Hq] fp32 or NULL: natural-log logsumexp of the scaled
 *              scores (what a cross-device combine needs)
 * When num_splits == 1 the scratch may be NULL and no combine launches.
 * A sequence with ctx_len == 0 gets a zero output and lse = -inf.
 * Supported: D in {64, 128, 256}, P == 16, Hq % Hkv == 0.
 * ------------------------------------------------------------------------ */
int sc_paged_decode_attention(const sc_bf16* q, const sc_bf16* kv_pool,
                              int64_t num_pages, const int32_t* block_table,
                              const int32_t* ctx_len, const int32_t* seq_order, int B,
                              int Hq, int Hkv, int D,
                              int P, int max_pages, int pages_per_split,
                              int num_splits, float scale,
                              float* part_out, float* part_lse, sc_bf16* out,
                              float* lse_out, void* stream);

/* The same attention, writing each row's normalised fp32 output and its lse
 * packed as packed[B * Hq][D + 1] (lse at index D): the per-device partial of
 * a sequence whose KV pages are split across GPUs. Gather the parts of every
 * device into [nparts][rows][D + 1] and merge them with
 * sc_attention_combine_packed. No reference counterpart (the reference runs
 * one device). */
int sc_paged_decode_attention_packed(const sc_bf16* q, const sc_bf16* kv_pool,
                                     int64_t num_pages, const int32_t* block_table,
                                     const int32_t* ctx_len, int B, int Hq, int Hkv,
                                     int D, int P, int max_pages, int pages_per_split,
                                     int num_splits, float scale, float* part_out,
                                     float* part_lse, float* packed, void* stream);

/* Merges gathered packed parts [nparts][rows][D + 1] (as written by
 * sc_paged_decode_attention_packed on each device) into out [rows, D] bf16
 * and lse_out [rows] fp32 (or NULL). Parts with lse = -inf are ignored.
 * D <= 512. */
int sc_attention_combine_packed(const float* gathered, int nparts, int rows, int D,
                                sc_bf16* out, float* lse_out, void* stream);

/* --------------------------------------------------------------------------
 * (e) Peer exchange of the packed partials over NVLink (replaces the NCCL
 * all-gather of step 3 of the KV-sharded sequence; no reference counterpart).
 *
 * sc_exchange_put: one CTA per rank p copies `bytes` (a multiple of 16) from
 * src to peer_dst[p] (this rank's slot in rank p's receive buffer, mapped
 * with CUDA IPC), then release-stores *epoch_base + epoch_add into
 * *peer_flag[p] (rank p's flag for this rank). peer_dst and peer_flag are
 * device arrays of `world` device addresses.
 * sc_exchange_wait: waits (bounded; a timeout sets the device status word)
 * until flags[r] >= *epoch_base + epoch_add for every rank r < world. Kernels
 * after it on the stream see every rank's block. Plain stores and loads over
 * NVLink only (no multicast). */
int sc_exchange_put(const void* src, long long bytes, void* const* peer_dst,
                    unsigned int* const* peer_flag, const unsigned int* epoch_base,
                    unsigned int epoch_add, int world, void* stream);
int sc_exchange_wait(const unsigned int* flags, int world, const unsigned int* epoch_base,
                     unsigned int epoch_add, void* stream);
/* sc_exchange_wait with the number of polls of one flag before it gives up
 * (sc_exchange_wait: 2^24, seconds with its 64 ns back-off): a caller's own
 * time-out, or a test that a wait nobody answers ends with the status bit. */
int sc_exchange_wait_limited(const unsigned int* flags, int world,
                             const unsigned int* epoch_base, unsigned int epoch_add,
                             unsigned int max_polls, void* stream);

/* The same exchange folded into the attention kernels (two launches fewer per
 * layer):
 * sc_paged_decode_attention_exchange: sc_paged_decode_attention_packed whose
 * split merge writes the packed rows [B * Hq][D + 1] into `packed` (16-byte
 * aligned; B*Hq*(D+1)*4 a multiple of 16); the merge CTA that finishes last
 * copies the block to peer_dst[p] for every rank p (float* device addresses)
 * and release-stores *epoch_base + epoch_add into *peer_flag[p]. `counter` is
 * a device word that is zero before the first call (the kernel leaves it
 * zero). Needs num_splits > 1.
 * sc_attention_combine_exchange: sc_attention_combine_packed that first waits
 * (bounded, as sc_exchange_wait) for flags[r] to reach the epoch for every
 * r < nparts; after a timeout it writes nothing and sets the status word. */
int sc_paged_decode_attention_exchange(const sc_bf16* q, const sc_bf16* kv_pool,
                                       int64_t num_pages, const int32_t* block_table,
                                       const int32_t* ctx_len, int B, int Hq, int Hkv, int D,
                                       int P, int max_pages, int pages_per_split,
                                       int num_splits, float scale, float* part_out,
                                       float* part_lse, float* packed, float* const* peer_dst,
                                       unsigned int* const* peer_flag, unsigned int* counter,
                                       const unsigned int* epoch_base, unsigned int epoch_add,
                                       int world, void* stream);
int sc_attention_combine_exchange(const float* gathered, const unsigned int* flags,
                                  const unsigned int* epoch_base, unsigned int epoch_add,
                                  int nparts, int rows, int D, sc_bf16* out, float* lse_out,
                                  void* stream);

/* One attention layer of a decode step: the KV append of the step's new token
 * (sc_kv_append) folded into split-K decode attention
 * (sc_paged_decode_attention), one launch plus the split merge. The merge is
 * the separate kernel of sc_paged_decode_attention when a sequence needs more
 * than one split, or, with in_kernel_merge != 0 and num_splits <= 16, done by
 * the last split of each sequence to finish (no merge launch).
 *
 * Replaces, as one kernel, the KV write of mlx_request_cache.py:59-63
 * (`OwnedKV.update_and_fetch`) and the per-request SDPA of mlx_decode.py:80-106
 * (`_attention_rows`); math of scripts/mlx_attention_qualify.py:234-275.
 *
 * k_new, v_new [B, Hkv, D] bf16 (16-byte aligned) are each row's new token;
 * slot_mapping [B] int64 its slot (page * 16 + offset, < 0: nothing appended).
 * ctx_len counts the new token. The rows are written to the pool once, and a
 * CTA whose pages include the slot's page takes the rows from k_new / v_new, so
 * the result equals sc_kv_append followed by sc_paged_decode_attention; the
 * slot's page must not be shared with another row of the launch (copy-on-write
 * of a partial page guarantees that). Other arguments as in
 * sc_paged_decode_attention, with exactly one of out (bf16 rows, lse_out
 * optional) or packed ([B * Hq][D + 1] fp32, lse at index D, as
 * sc_paged_decode_attention_packed); out 8-byte aligned. num_splits > 1 needs
 * part_out and part_lse, and the in-kernel merge also `counters`:
 * B * Hkv * ceil(Hq / Hkv / 8) uint32, zero before the first call; each launch
 * leaves them zero (after a DeviceFault, zero them again).
 * Launches that share counters or scratch must not overlap on the GPU. */
int sc_paged_decode_attention_fused(const sc_bf16* q, const sc_bf16* k_new,
                                    const sc_bf16* v_new, const int64_t* slot_mapping,
                                    sc_bf16* kv_pool, int64_t num_pages,
                                    const int32_t* block_table, const int32_t* ctx_len,
                                    const int32_t* seq_order, int B, int Hq, int Hkv, int D,
                                    int P, int max_pages, int pages_per_split, int num_splits,
                                    float scale, float* part_out, float* part_lse,
                                    unsigned int* counters, sc_bf16* out, float* lse_out,
                                    float* packed, int in_kernel_merge, void* stream);

/* Split-K decode attention that allocates nothing and takes no scratch.
 *
 * No counterpart in the reference: it exists for callers of this library
 * that cannot allocate device memory at call time -- a plain C / FFI host
 * that embeds the library without a device allocator of its own, a process
 * whose device memory belongs to another framework's caching allocator (a
 * raw cudaMalloc beside it escapes that pool's accounting), or a decode loop
 * that must neither synchronise the device (cudaFree does) nor risk running
 * out of memory in the middle of a step.
 *
 * Same arguments and results as sc_paged_decode_attention without
 * part_out / part_lse: the split partials go to a fixed array inside the
 * library of SC_NOALLOC_SCRATCH_FLOATS floats (32 MiB), which every GPU that
 * loads the library holds until the process exits. A call needs
 * B * Hq * num_splits * (D + 1) floats when num_splits > 1 and returns
 * SC_ERR_INVALID (nothing launched) when that exceeds the array.
 * The first call on a device that needs the array (num_splits > 1) looks up
 * its device address (a one-time set-up per device) and caches it for the
 * life of the process; make that first call before any stream capture. The
 * cached address belongs to the device's primary context: after
 * cudaDeviceReset (or anything else that destroys that context) this entry
 * point must not be called again in the same process.
 * All calls share the one array and it keeps the last call's contents;
 * nothing in it needs to start at zero, because every partial a call reads
 * is written earlier in the same call. Calls that overlap on the GPU (other
 * streams, other host threads) race on the array: serialise them.
 * It calls no cudaMalloc, cudaFree or other allocating routine. */
#define SC_NOALLOC_SCRATCH_FLOATS 8388608
int sc_paged_decode_attention_noalloc(const sc_bf16* q, const sc_bf16* kv_pool,
                                      int64_t num_pages, const int32_t* block_table,
                                      const int32_t* ctx_len, int B, int Hq, int Hkv,
                                      int D, int P, int max_pages,
                                      int pages_per_split, int num_splits,
                                      float scale, sc_bf16* out, float* lse_out,
                                      void* stream);

/* Merges per-part normalised outputs with their lse:
 *   out[r] = sum_s exp(lse[r,s] - M) o[r,s] / sum_s exp(lse[r,s] - M)
 * over s < nparts (rows r = 0..rows-1, parts with lse = -inf ignored).
 * part_out [rows, nparts, D] fp32, part_lse [rows, nparts] fp32,
 * out [rows, D] bf16, lse_out [rows] fp32 or NULL.
 * This is the cross-GPU combine of a KV-sharded long sequence. D <= 512. */
int sc_attention_combine(const float* part_out, const float* part_lse,
                         int rows, int nparts, int D, sc_bf16* out,
                         float* lse_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SHELLCACHE_H */
