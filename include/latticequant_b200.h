/*
 * latticequant_b200.h -- C ABI of the B200 (sm_100a) LatticeQuant KV-cache
 * codec library (latticequant_b200/liblq_b200.so).
 *
 * Every entry point is asynchronous on the CUDA stream it is given
 * (cudaStream_t passed as void*, NULL = legacy default stream), takes device
 * pointers and plain sizes, allocates nothing, and returns an LQ_* status for
 * argument / launch errors.  Data-dependent failures (alphabet larger than L,
 * corrupt bitstream, ...) are raised by the kernels as LQ_EF_* bits OR-ed
 * into a caller-provided device word `err`, readable after the stream
 * synchronises.  No kernel traps or asserts.
 *
 * Data layout (one "chunk" = one tensor handed to
 * CompressedKVCache._compress_tensor, reference llm/compressed_kv_cache.py:176):
 *   x        [n_chunks][n_heads][bph][8] elements, bph = seq*head_dim/8
 *   block    one 8-element E8 vector; N = n_heads*bph blocks per chunk
 *   tile     TB consecutive blocks of a chunk (TB multiple of 32); the last
 *            tile of a chunk may be short
 *   stream s 8*coset + coord (coord 7 carries coord8_half)
 *   lane     (chunk, tile, s): the symbols of stream s whose blocks lie in
 *            the tile, rANS-coded with the chunk's table for s; each lane is
 *            one reference-format stream (core/gpu_ans.py:105-139)
 *   words    all lanes of all chunks back to back, lane l at
 *            [lane_off[l], lane_off[l+1]), ceil(n_bits/32) words each
 */
#ifndef LATTICEQUANT_B200_H
#define LATTICEQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define LQ_OK 0
#define LQ_ERR_INVALID (-1)  /* bad argument: null pointer, size, dtype, alignment */
#define LQ_ERR_ALPHABET (-2) /* a stream alphabet exceeds L = 1024 symbols */
#define LQ_ERR_CAPACITY (-3) /* an output buffer is too small */
#define LQ_ERR_CUDA (-4)     /* CUDA launch / runtime error */
#define LQ_ERR_STREAM (-5)   /* corrupt bitstream / metadata */

/* ---- device error flags (OR-ed into *err by kernels) ---- */
#define LQ_EF_ALPHABET 0x1u   /* table build: alphabet > L (reference hangs here) */
#define LQ_EF_SYMRANGE 0x2u   /* a lattice coordinate outside [-LQ_SYM_LIMIT, LQ_SYM_LIMIT) */
#define LQ_EF_CAPACITY 0x4u   /* compressed output larger than the given capacity */
#define LQ_EF_BITSTREAM 0x8u  /* lane metadata points outside the word buffer */
#define LQ_EF_NONFINITE 0x10u /* non-finite input or scaled input */
#define LQ_EF_NOCONVERGE 0x20u /* table normalisation did not converge */
#define LQ_EF_TIMEOUT 0x40u    /* a bulk copy into shared memory did not complete within a second */

/* ---- dtypes ---- */
#define LQ_F32 0
#define LQ_F16 1
#define LQ_BF16 2

#define LQ_L 1024          /* rANS table size, core/gpu_ans.py:44-45 */
#define LQ_SYM_LIMIT 512   /* lattice coordinates must lie in [-512, 512) */
#define LQ_HIST_BINS 1024  /* per-stream histogram bins, value v -> bin v + 512 */
#define LQ_NSTREAMS 16

/* Library version (major*10000 + minor*100 + patch). */
int lq_version(void);

/* Human-readable text for an LQ_* status. */
const char *lq_strerror(int status);

/* ------------------------------------------------------------------------
 * Per-head variance and scale.
 * Replaces llm/compressed_kv_cache.py:183-196 (sigma2 = mean(t^2) per head,
 * scale = sqrt(2*pi*e*sigma2*4^-b), 1.0 where sigma2 < 1e-12, fp16 copy) and
 * core/e8_quantizer.py:137-148 (compute_scale).  The sum of squares follows
 * torch's CPU reduction tree bit for bit; sqrt is IEEE.
 *   x            [n_heads_total][elems_per_head], dtype LQ_F32/F16/BF16
 *   vol_mult     fp32(4 ** -bits)
 *   sigma2, scale_f32, scale_f16 [n_heads_total] (each may be NULL)
 *   workspace    lq_head_scales_workspace() bytes (may be NULL when that is 0)
 * ---------------------------------------------------------------------- */
size_t lq_head_scales_workspace(int64_t n_heads_total, int64_t elems_per_head);
int lq_head_scales(const void *x, int dtype, int64_t n_heads_total, int64_t elems_per_head, float vol_mult,
                   float *sigma2, float *scale_f32, uint16_t *scale_f16, void *workspace, size_t workspace_bytes,
                   void *stream);

/* ------------------------------------------------------------------------
 * lq_head_scales without a workspace argument.  It has no counterpart in
 * the reference, which computes the scales with torch on whatever device the
 * tensor lives on.  It is for callers that cannot allocate device memory: a
 * host that owns all GPU memory and hands out no allocator (a serving engine
 * with a pre-reserved pool, a foreign-language plugin without torch), or a
 * latency-critical decode step that must not pay the device-wide
 * synchronisation a cudaMalloc/cudaFree can cause.  Results are identical to
 * lq_head_scales.
 *   limit     the partial sums use a scratch array inside the library of
 *             LQ_HEAD_SCALES_STATIC_FLOATS floats (4 MiB) that every GPU which
 *             loads the library holds until the process exits; a problem with
 *             lq_head_scales_workspace(n, e) > 4 MiB returns LQ_ERR_CAPACITY
 *             before anything is launched (e.g. heads of 2^20 elements: at
 *             most 254 heads per call)
 *   set-up    the first call on a device (with that device current) looks up
 *             the array's device address; make that first call before any
 *             CUDA stream capture.  The address is cached per device and
 *             context: after cudaDeviceReset (or in a context created by the
 *             caller) the next call looks it up again, so that call, too,
 *             belongs outside a capture
 *   sharing   all calls use the same array, which keeps the last call's
 *             contents (nothing needs to start at zero); calls that can
 *             overlap on the GPU -- different streams without ordering, or
 *             several host threads -- race on it and must be serialised
 * ---------------------------------------------------------------------- */
#define LQ_HEAD_SCALES_STATIC_FLOATS (1 << 20)
int lq_head_scales_static(const void *x, int dtype, int64_t n_heads_total, int64_t elems_per_head, float vol_mult,
                          float *sigma2, float *scale_f32, uint16_t *scale_f16, void *stream);

/* ------------------------------------------------------------------------
 * E8 quantisation + parity-aware symbolisation + coset packing + histograms.
 * Replaces the E8 / symbol part of _compress_tensor
 * (llm/compressed_kv_cache.py:198-228): x / scale -> encode_e8
 * (core/e8_quantizer.py:61-83) -> e8_to_symbols (core/entropy_coder.py:46-68)
 * -> pack_coset_bits (llm/compressed_kv_cache.py:46-54), plus the per-stream
 * counts that feed build_rans_table (:236-253).
 *   scale_f32    [n_chunks][n_heads]
 *   sym_cols     lq_sym_cols_bytes() bytes, 16-byte aligned: per tile and
 *                coordinate an int8 column ([n_chunks][n_tiles][8][TB])
 *                holding the coset-0 blocks' symbols in block order from the
 *                front and the coset-1 blocks' from the back; a symbol
 *                outside [-127, 127] is written as -128 there and in full to
 *                the same index of the int16 plane that follows, and its
 *                tile's u32 flag (after that plane) is set
 *   coset_words  [n_chunks][ceil(N/32)] u32, bit i of word w = block 32w+i
 *   tile_n0      [n_chunks][n_tiles] number of coset-0 blocks per tile
 *   hist         [n_chunks][16][LQ_HIST_BINS] u32, zeroed by this call
 *   deq          optional [n_chunks][N][8] in deq_dtype: q * scale_f32 (the
 *                buffer update() returns, :204); NULL to skip
 *   q_out        optional [n_chunks][N][8] fp32 lattice points; NULL to skip
 * ---------------------------------------------------------------------- */
size_t lq_sym_cols_bytes(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks);
int lq_e8_quantize(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph, const float *scale_f32,
                   int64_t tile_blocks, void *sym_cols, uint32_t *coset_words, uint32_t *tile_n0, uint32_t *hist,
                   void *deq, int deq_dtype, float *q_out, uint32_t *err, void *stream);

/* lq_e8_quantize with the outlier side channel (no counterpart in the
 * reference, whose table build never ends for alphabets over L): a token of
 * blocks_per_token consecutive blocks (a power of two <= 32 dividing bph and
 * tile_blocks) holding any symbol outside [-limit, limit] is written to
 * outlier_rec as blocks_per_token records (block index in the chunk, coset,
 * 8 symbols; int32 x 10 each) and coded as zero blocks, so every stream's
 * alphabet stays within 2*limit+5 values.  deq / q_out keep the true points.
 *   outlier_words  optional [n_chunks][ceil(N/32)] bitmap of extracted blocks
 *   outlier_rec    [n_chunks][outlier_cap][10]; outlier_count [n_chunks]
 *                  (zeroed by this call); a full list raises LQ_EF_CAPACITY */
int lq_e8_quantize_outliers(const void *x, int dtype, int64_t n_chunks, int64_t n_heads, int64_t bph,
                            const float *scale_f32, int64_t tile_blocks, void *sym_cols, uint32_t *coset_words,
                            uint32_t *tile_n0, uint32_t *hist, void *deq, int deq_dtype, float *q_out, int limit,
                            int blocks_per_token, uint32_t *outlier_words, int32_t *outlier_rec,
                            uint32_t *outlier_count, int64_t outlier_cap, uint32_t *err, void *stream);

/* Put the extracted blocks back into a decoded chunk batch: point * fp16
 * head scale into out (out_dtype), symbols into sym_out (either may be NULL). */
int lq_patch_outliers(const int32_t *outlier_rec, const uint32_t *outlier_count, int64_t n_chunks,
                      int64_t outlier_cap, int64_t n_heads, int64_t bph, const uint16_t *scale_f16, void *out,
                      int out_dtype, int32_t *sym_out, uint32_t *err, void *stream);

/* Plain encode_e8 (core/e8_quantizer.py:61-83) / encode_d8 (:20-58) on (n,8) fp32. */
int lq_encode_e8(const float *x, int64_t n, float *out, int d8_only, void *stream);

/* ------------------------------------------------------------------------
 * rANS tables from histograms.
 * Replaces build_rans_table (core/gpu_ans.py:62-98) with the alphabet rule
 * of llm/compressed_kv_cache.py:246-250 ([min-2, max+2]).  Ties in the
 * normalisation are broken by ascending symbol index.
 *   hist         [n_tables][LQ_HIST_BINS]
 *   tab_lo       [n_tables] first alphabet value
 *   tab_nsym     [n_tables] alphabet size (0 = empty stream)
 *   tab_freq     [n_tables][LQ_L] u16 normalised frequencies
 * lq_expand_tables turns frequencies into the packed coder tables used by
 * lq_rans_encode (enc_tab) and lq_rans_decode (dec_tab), [n_tables][LQ_L]
 * u32 each; either may be NULL.
 * ---------------------------------------------------------------------- */
int lq_build_tables(const uint32_t *hist, int64_t n_tables, int32_t *tab_lo, int32_t *tab_nsym, uint16_t *tab_freq,
                    uint32_t *err, void *stream);
int lq_expand_tables(const int32_t *tab_nsym, const uint16_t *tab_freq, int64_t n_tables, uint32_t *enc_tab,
                     uint32_t *dec_tab, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Lane encode.  Replaces rans_encode (core/gpu_ans.py:105-139) run over
 * the 16 streams of each chunk (llm/compressed_kv_cache.py:236-268).
 *   words        [words_cap] output, lanes back to back
 *   lane_off     [n_chunks*n_tiles*16 + 1] u32 word offsets (last = total)
 *   lane_nbits   [n_lanes] u32, lane_state [n_lanes] u32 (final state = the
 *                decoder's initial state)
 *   workspace    lq_rans_encode_workspace() bytes
 * ---------------------------------------------------------------------- */
size_t lq_rans_encode_workspace(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks);
int lq_rans_encode(const void *sym_cols, const uint32_t *tile_n0, int64_t n_chunks, int64_t n_vectors,
                   int64_t tile_blocks, const int32_t *tab_lo, const int32_t *tab_nsym, const uint32_t *enc_tab,
                   uint32_t *words, int64_t words_cap, uint32_t *lane_off, uint32_t *lane_nbits,
                   uint32_t *lane_state, void *workspace, size_t workspace_bytes, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Lane decode + dequantisation.  Replaces _decompress_chunk
 * (llm/compressed_kv_cache.py:289-332): gpu_rans_decode of every stream,
 * unpack_coset_bits, symbols_to_e8 (core/entropy_coder.py:71-89) and
 * multiplication by the fp16 per-head scale, output in out_dtype.
 *   dec_tab      [n_chunks*16][LQ_L] from lq_expand_tables
 *   out          [n_chunks][N][8] in out_dtype (NULL to skip)
 *   sym_out      optional [n_chunks][N][8] int32 decoded symbols
 *   workspace    lq_rans_decode_workspace() bytes
 * ---------------------------------------------------------------------- */
size_t lq_rans_decode_workspace(int64_t n_chunks, int64_t n_vectors, int64_t tile_blocks);
int lq_rans_decode(const uint32_t *words, int64_t n_words, const uint32_t *lane_off, const uint32_t *lane_nbits,
                   const uint32_t *lane_state, const uint32_t *coset_words, const uint32_t *tile_n0,
                   int64_t n_chunks, int64_t n_heads, int64_t bph, int64_t tile_blocks, const int32_t *tab_lo,
                   const int32_t *tab_nsym, const uint16_t *tab_freq, const uint32_t *dec_tab,
                   const uint16_t *scale_f16, void *out, int out_dtype, int32_t *sym_out, void *workspace,
                   size_t workspace_bytes, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Fused dequant + decode attention over one compressed K chunk and one V
 * chunk of the same geometry (a (B, Hkv, S, D) cache tensor each, as
 * CompressedKVCache._compress_tensor stores them,
 * llm/compressed_kv_cache.py:176-287).  Replaces _decompress_chunk (:289-332)
 * + the concatenated bf16 buffer update() returns (:385-395) + transformers'
 * SDPA with repeat_kv: for every batch b and query head h,
 *   o[b][h] = softmax(q[b][h] . K[b][h/G]^T * sm_scale) V[b][h/G]
 * with K, V = symbols_to_e8 * fp16 head scale, never materialised.
 *   geometry   batch B, n_kv_heads Hkv, seq_len S tokens, head_dim 64/128;
 *              scale_per_token = 0: the chunks hold B*Hkv heads of S*head_dim/8
 *              blocks with one scale per head (a prefill chunk);
 *              scale_per_token = 1: they hold B*Hkv*S heads of head_dim/8
 *              blocks, one scale per token (decode appends encoded together,
 *              each token keeping the scale the reference gives it alone)
 *   q          [B][Hkv*group][head_dim] in q_dtype (16-byte aligned)
 *   out        [B][Hkv*group][head_dim] in out_dtype
 *   lse        optional [B][Hkv*group] fp32 ln(sum_t exp(s_t)), the form
 *              lq_attn_merge combines across key sets (sequence shards)
 *   tok_mask   optional [B*Hkv][ceil(S/32)] u32 bitmap of tokens to leave
 *              out (e.g. the chunks' outlier tokens, attended separately)
 *   workspace  lq_attn_decode_workspace() bytes (per-CTA partials)
 * Needs head_dim 64 or 128, group 1..8, tile_blocks dividing S*head_dim/8.
 * ---------------------------------------------------------------------- */
typedef struct lq_chunk_view {
    const uint32_t *words;
    int64_t n_words;
    const uint32_t *lane_off, *lane_nbits, *lane_state;
    const uint32_t *coset_words, *tile_n0;
    const int32_t *tab_lo, *tab_nsym;
    const uint16_t *tab_freq;
    const uint32_t *dec_tab;
    const uint16_t *scale_f16;
    int64_t n_heads, bph, tile_blocks;
    /* optional (may be NULL): the chunk's 16 decode tables in the kernels'
     * shared-memory form, from lq_stage_tables, 16-byte aligned; with it each
     * CTA fills its table region with one bulk copy (cp.async.bulk) instead of
     * loading and converting the tables thread by thread */
    const uint32_t *staged_tab;
} lq_chunk_view;

/* The decode tables of n_tables streams (lq_expand_tables' dec_tab, with the
 * streams' tab_lo) in the shared-memory form lq_attn_decode copies in bulk:
 *   staged [n_tables][LQ_L] u32 (a chunk's 16 tables are 64 KB)
 * No reference counterpart (the reference keeps numpy tables on the host). */
int lq_stage_tables(const uint32_t *dec_tab, const int32_t *tab_lo, int64_t n_tables, uint32_t *staged, void *stream);

size_t lq_attn_decode_workspace(int64_t n_heads, int64_t bph, int64_t tile_blocks, int group, int head_dim);
int lq_attn_decode(const lq_chunk_view *k, const lq_chunk_view *v, const void *q, int q_dtype, int64_t batch,
                   int64_t n_kv_heads, int64_t seq_len, int scale_per_token, int group, int head_dim, float sm_scale,
                   void *out, int out_dtype, float *lse, const uint32_t *tok_mask, void *workspace,
                   size_t workspace_bytes, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Decode attention over the compact fixed-rate layout.  Replaces the
 * reference's merge of the compact chunk into an fp16 buffer
 * (llm/fused_triton_merge.py:33-177, fused_decompress_chunk) followed by
 * SDPA with repeat_kv: the kernel reads each block from the packed codes or
 * the fp16 fallback rows and attends in registers.
 *   packed      [n_repr][bits] bytes, the representable blocks in block
 *               order, big-endian [coset | u0..u6 (bits) | u7 >> 1 (bits-1)]
 *               (core/compact_storage.py:87-222); 16-byte aligned
 *   fallback    [n_fallback][8] fp16, the other blocks' values (scaled),
 *               16-byte aligned
 *   mask_words  [ceil(n_heads*bph/32)] u32: bit i of word w set when block
 *               32w+i is representable
 *   word_rank   [same] int32: representable blocks before word w
 *   scales      [n_heads] fp32 head scales of the representable blocks
 * Blocks are (B*Hkv, seq*head_dim/8) in head-major order; seq*head_dim/8
 * must be a multiple of 32.  Results as lq_attn_decode (o, optional lse). */
typedef struct lq_compact_view {
    const uint8_t *packed;
    int64_t n_repr;
    const uint16_t *fallback;
    int64_t n_fallback;
    const uint32_t *mask_words;
    const int32_t *word_rank;
    const float *scales;
    int64_t n_heads, bph;
    int bits;
} lq_compact_view;

size_t lq_attn_compact_workspace(int64_t n_heads, int64_t seq_len, int group, int head_dim);
int lq_attn_decode_compact(const lq_compact_view *k, const lq_compact_view *v, const void *q, int q_dtype,
                           int64_t batch, int64_t n_kv_heads, int64_t seq_len, int group, int head_dim,
                           float sm_scale, void *out, int out_dtype, float *lse, void *workspace,
                           size_t workspace_bytes, uint32_t *err, void *stream);

/* Merge attention parts over disjoint key sets (the all-gathered sequence
 * shards, or several chunks of one layer): o = sum_i o_i exp(lse_i - lse),
 * lse = ln sum_i exp(lse_i).
 *   o_parts [n_parts][rows][head_dim] fp32, lse_parts [n_parts][rows] fp32
 *   out     [rows][head_dim] in out_dtype; lse optional [rows] */
int lq_attn_merge(const float *o_parts, const float *lse_parts, int64_t n_parts, int64_t rows, int head_dim,
                  void *out, int out_dtype, float *lse, void *stream);

/* lq_attn_merge over parts packed one after another, each [rows][head_dim]
 * o values followed by its [rows] lse values -- the layout one all-gather of
 * every rank's (o, lse) buffer produces, so a sequence-sharded decode step
 * needs one collective.  No reference counterpart (the reference attends on
 * one GPU).
 *   parts   [n_parts][rows * head_dim + rows] fp32 */
int lq_attn_merge_packed(const float *parts, int64_t n_parts, int64_t rows, int head_dim, void *out, int out_dtype,
                         float *lse, void *stream);

/* One decode step's attention over the dense end of a layer's cache, merged
 * with the finished attention of its compressed parts, in one launch.
 * Replaces, for a cache whose older tokens are compressed, the reference's
 * SDPA over the whole dequantised buffer that update() returns
 * (llm/compressed_kv_cache.py:342-395, read with repeat_kv): the parts come
 * from lq_attn_decode / lq_attn_decode_compact, the dense tokens (the open
 * tail, tails kept dequantised) are attended here.
 *   q        [batch * n_kv_heads * group][head_dim] in q_dtype (query head
 *            kvh * group + g reads kv head kvh); out the same shape and dtype
 *   segment s < n_seg (host arrays): k_seg[s], v_seg[s] [batch * n_kv_heads]
 *            [cap_seg[s]][head_dim] in kv_dtype, 16-byte aligned, of which
 *            the first len_seg[s] tokens count -- or, where last_seg is not
 *            NULL and last_seg[s] is, last_seg[s][0] + 1 tokens (a device slot
 *            index, so a captured CUDA graph replays with a moving length)
 *   o_parts  [n_parts][rows][head_dim] fp32 normalised, lse_parts
 *            [n_parts][rows] natural log (rows = batch * n_kv_heads * group)
 *   lse      optional [rows]: the merged log-sum-exp.  No keys at all gives
 *            o = 0, lse = -inf.  head_dim 64 or 128, group 1..8. */
#define LQ_DENSE_MAX_SEGMENTS 8
int lq_attn_dense_merge(const void *q, int q_dtype, int n_seg, const void *const *k_seg, const void *const *v_seg,
                        const int64_t *cap_seg, const int64_t *len_seg, const int64_t *const *last_seg, int kv_dtype,
                        const float *o_parts, const float *lse_parts, int64_t n_parts, int64_t batch,
                        int64_t n_kv_heads, int group, int head_dim, float sm_scale, void *out, float *lse,
                        void *stream);

/* Fused merge of the compact layout with an fp16 fallback
 * (llm/fused_triton_merge.py:33-177): for each of n_heads*bph blocks,
 * repr_mask[k] != 0 -> decode code repr_rank[k] of `packed` (bits bytes per
 * code) times scales[k / bph] to fp16; else copy fallback row fb_rank[k].
 * repr_rank / fb_rank are the exclusive prefix counts of the mask and of its
 * complement.  coord7's parity uses the non-negative remainder (the
 * reference kernel's signed remainder decodes odd negative sums wrongly).
 *   out  [n_heads*bph][8] fp16, 16-byte aligned; fallback 16-byte aligned */
int lq_compact_merge(const uint8_t *packed, int64_t n_repr, int bits, const uint8_t *repr_mask,
                     const int32_t *repr_rank, const int32_t *fb_rank, const uint16_t *fallback, int64_t n_fallback,
                     const float *scales, int64_t n_heads, int64_t bph, uint16_t *out, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Randomized Hadamard transform (core/pipeline.py:33-122) on fp32 vectors
 * of length d (a power of two, 2..4096):
 *   out = (FWHT(x * pre_signs) / sqrt(d)) * post_signs
 * with either sign vector NULL: pre_signs for RHT.forward, post_signs for
 * RHT.inverse, neither for fast_hadamard_transform.  Bit-exact with torch.
 * ---------------------------------------------------------------------- */
int lq_fwht(const float *x, int64_t n_vec, int d, const float *pre_signs, const float *post_signs, float *out,
            void *stream);

/* ------------------------------------------------------------------------
 * Reference-stream decode: the argument meaning of _rans_decode_kernel
 * (core/gpu_ans.py:175-235) as prepared by prepare_gpu_decode (:274-342):
 * bit offsets, n_bits, initial states, symbol counts, per-table lookup /
 * freqs / cumfreqs / alphabet padded to max_sym, table id per stream, int64
 * output at out_offsets.  One thread per stream.
 * ---------------------------------------------------------------------- */
int lq_rans_decode_streams(const uint32_t *bitstream, int64_t n_words, const int64_t *bit_offsets,
                           const int64_t *n_bits, const int64_t *init_states, const int64_t *n_decode,
                           const int32_t *lookup, const int32_t *freqs, const int32_t *cumfreqs,
                           const int32_t *alphabet, const int32_t *table_id, int64_t max_sym, int64_t n_streams,
                           int64_t *out, const int64_t *out_offsets, uint32_t *err, void *stream);

/* ------------------------------------------------------------------------
 * Compact fixed-rate layout (core/compact_storage.py:87-222).
 * lq_pack_e8: q (n,8) fp32 valid in-range E8 points -> (n,b) bytes; counts
 * of invalid / out-of-range rows go to n_bad[0] / n_bad[1] (u32, zeroed by
 * the call) so the host can raise the reference's ValueError.
 * lq_unpack_e8: (n,b) bytes -> q (n,8) fp32, or, with scales != NULL,
 * (q * scales[head_idx[i]]) rounded to fp16 -- triton_unpack_e8_4bit
 * (core/triton_dequant.py:139-177) for b = 4.
 * ---------------------------------------------------------------------- */
int lq_pack_e8(const float *q, int64_t n, int bits, uint8_t *out, uint32_t *n_bad, void *stream);
int lq_unpack_e8(const uint8_t *packed, int64_t n, int bits, const float *scales, const int32_t *head_idx,
                 float *q_out, uint16_t *f16_out, void *stream);

/* ------------------------------------------------------------------------
 * Element-wise entry points of the reference's core modules.
 *   lq_quantize_e8     quantize_e8 (core/e8_quantizer.py:90-110): n blocks of x
 *                      (fp32) -> q = encode_e8(x / scale), xhat = q * scale
 *   lq_e8_to_symbols   e8_to_symbols (core/entropy_coder.py:46-68): coset[n],
 *                      sym[n][8] (coords 0..6, coord8_half)
 *   lq_symbols_to_e8   symbols_to_e8 (core/entropy_coder.py:71-89)
 *   lq_check_e8        validate_e8 (core/compact_storage.py:39-80) and, for
 *                      bits > 0, check_representable (:235-249); each output
 *                      may be NULL
 *   lq_pack_bits / lq_unpack_bits
 *                      pack_coset_bits / unpack_coset_bits
 *                      (llm/compressed_kv_cache.py:46-63): bit i <-> byte i/8, bit i%8
 *   lq_map_symbols     symbol values -> table indices, nearest alphabet entry
 *                      and first index on ties (core/gpu_ans.py:115-119)
 *   lq_rans_encode_streams / lq_rans_finish_streams
 *                      rans_encode (core/gpu_ans.py:105-139) of independent
 *                      streams: symbol indices, one thread per stream, into
 *                      slots [slot_off[i], slot_off[i+1]) of at least
 *                      ceil(10*n/32) words; then reference words
 *                      (ceil(n_bits/32) + 1, the last one zero) at dst_off[i]
 * ---------------------------------------------------------------------- */
int lq_quantize_e8(const float *x, int64_t n, float scale, float *q_out, float *xhat, void *stream);
int lq_e8_to_symbols(const float *q, int64_t n, int32_t *coset, int32_t *sym, void *stream);
int lq_symbols_to_e8(const int32_t *coset, const int32_t *sym, int64_t n, float *q, void *stream);
int lq_check_e8(const float *q, int64_t n, float atol, int bits, uint8_t *valid, uint8_t *coset, uint8_t *in_range,
                void *stream);
int lq_pack_bits(const uint8_t *in, int64_t n, uint8_t *out, void *stream);
int lq_unpack_bits(const uint8_t *in, int64_t n, uint8_t *out, void *stream);
int lq_map_symbols(const int64_t *sym, int64_t n, const int64_t *alphabet, int32_t n_alpha, int contiguous,
                   int32_t *out, void *stream);
int lq_rans_encode_streams(const int32_t *sym_idx, const int64_t *sym_off, const int64_t *n_sym,
                           const int32_t *table_id, const int32_t *tab_nsym, const uint32_t *enc_tab,
                           int64_t n_streams, const int64_t *slot_off, uint32_t *slots, int64_t *nbits,
                           uint32_t *state, uint32_t *err, void *stream);
int lq_rans_finish_streams(const uint32_t *slots, const int64_t *slot_off, const int64_t *nbits, int64_t n_streams,
                           const int64_t *dst_off, uint32_t *dst, void *stream);

/* ------------------------------------------------------------------------
 * Diagnostics for tests: run one internal device helper over arrays.
 *   LQ_SELFTEST_DIV      out[i] = a[i] / b[i] (fp32) through the quantiser's
 *                        division (reciprocal + FMA correction); must equal IEEE
 *   LQ_SELFTEST_FASTDIV  out[i] = a[i] / d (u32, a[i] < 2^31, 1 <= d < 2^31)
 *                        through the invariant-divisor multiply-shift
 * ---------------------------------------------------------------------- */
#define LQ_SELFTEST_DIV 1
#define LQ_SELFTEST_FASTDIV 2
int lq_selftest(int which, const void *a, const void *b, int64_t n, uint32_t d, void *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LATTICEQUANT_B200_H */
