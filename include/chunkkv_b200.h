/*
 * chunkkv_b200 — C ABI of the B200 (sm_100a) blend-prefill kernels.
 *
 * The reference (sarvanithin/chunkkv) is pure Python: its blend prefill is
 * TorchEngine.prefill (src/chunkkv/engine/torch_engine.py:80-178) over torch
 * library calls, and it has no FFI of its own.  Every entry point below
 * replaces one step of that method (or of the re-RoPE helpers / the store
 * insert); the reference line range each one stands in for is given beside it.
 *
 * Conventions shared by every entry point:
 *   - all pointers are DEVICE pointers unless named *_host; bf16 tensors are
 *     passed as uint16_t* (raw bf16 bit patterns), row-major, contiguous
 *     unless a stride argument says otherwise;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     asynchronous on that stream and never synchronises the device;
 *   - no entry point allocates device memory: callers pass every buffer;
 *   - the return value is a ckv_status; on failure ckv_last_error() gives a
 *     one-line message (thread-local) and nothing was launched.
 * Faults detected on the device (a bounded wait that ran out, an index the
 * kernel refused) are recorded in a device error word that
 * ckv_get_device_error() reads and clears after a synchronisation.
 */
#ifndef CHUNKKV_B200_H
#define CHUNKKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CKV_API __attribute__((visibility("default")))
#else
#define CKV_API
#endif

typedef void* ckv_stream_t; /* cudaStream_t */

typedef enum {
  CKV_OK = 0,
  CKV_ERR_ARG = 1,         /* bad shape / pointer / alignment (python: ValueError) */
  CKV_ERR_CUDA = 2,        /* launch or runtime failure (python: RuntimeError) */
  CKV_ERR_DEVICE = 3,      /* device-side error word set (python: RuntimeError) */
  CKV_ERR_UNSUPPORTED = 4  /* shape the kernels do not cover (python: NotImplementedError) */
} ckv_status;

/* Device-side error bits reported by ckv_get_device_error(). */
#define CKV_DEV_ERR_WAIT_TIMEOUT   0x1u  /* a bounded wait (mbarrier or peer counter) ran out */
#define CKV_DEV_ERR_PAGE_RANGE     0x2u  /* a page id outside [0, n_pages) was skipped */
#define CKV_DEV_ERR_SELECT_UNCOMPUTED 0x4u /* selection kept a position never computed
                                              (torch_engine.py:151 assert) */
#define CKV_DEV_ERR_POSITION_RANGE 0x8u  /* a position outside [0, n_ctx) was skipped */

/* ---- library -------------------------------------------------------------- */
CKV_API const char* ckv_version(void);
CKV_API const char* ckv_last_error(void);
/* Reads and clears the device error word of the current device (synchronises
 * the device first).  *code receives the OR of CKV_DEV_ERR_* bits. */
CKV_API int ckv_get_device_error(uint32_t* code);

/* ---- re-RoPE (scheduler/rerope.py:16-61; torch_engine.py:33,46-59) -------- */

/* table[p][j] = (cos, sin)(fp32(p) * inv_freq[j]) for p < max_pos, j < half_dim.
 * Angles exactly as torch_engine.py:54 forms them (fp32 product, fp32 cos/sin). */
CKV_API int ckv_rope_table(const float* inv_freq, int half_dim, int max_pos, float* table,
                   ckv_stream_t stream);

/* Re-RoPE of post-RoPE keys by a whole-tensor shift `delta`
 * (TorchEngine.shift_keys, torch_engine.py:56-59; rerope.shift_keys, rerope.py:56-61).
 * src/dst: [rows][head_dim] bf16 (any (B,H,L) flattening); rotary pairs are
 * (j, j + rot_dims/2) for j < rot_dims/2; dims >= rot_dims are copied.
 * delta == 0 copies.  src == dst is allowed. */
CKV_API int ckv_shift_keys(const uint16_t* src, uint16_t* dst, int64_t rows, int head_dim,
                   int rot_dims, int delta, const float* inv_freq, ckv_stream_t stream);

/* RoPE at explicit positions (rerope.apply_rope, rerope.py:50-53;
 * TorchEngine._rope, torch_engine.py:53-54).  src/dst: [batch_heads][seq][head_dim];
 * positions: [seq] int32. */
CKV_API int ckv_apply_rope(const uint16_t* src, uint16_t* dst, int64_t batch_heads, int seq,
                   int head_dim, int rot_dims, const int32_t* positions,
                   const float* inv_freq, ckv_stream_t stream);

/* fp32 forms of the two above, for fp32 keys: the reference rotates in fp32 and
 * returns the input dtype (torch_engine.py:46-51, 56-59; rerope.py:36-61), so fp32
 * keys stay fp32.  src/dst: fp32 rows, 16-byte aligned; same layout and pairs. */
CKV_API int ckv_shift_keys_f32(const float* src, float* dst, int64_t rows, int head_dim, int rot_dims,
                               int delta, const float* inv_freq, ckv_stream_t stream);
CKV_API int ckv_apply_rope_f32(const float* src, float* dst, int64_t batch_heads, int seq, int head_dim,
                               int rot_dims, const int32_t* positions, const float* inv_freq,
                               ckv_stream_t stream);

/* ---- gather of moved chunks into the blended cache -------------------------
 * Replaces base_kv (torch_engine.py:96-103) for ALL layers in one launch:
 * for every chunk c and layer l in [max(layer_lo, meta.layer_begin), min(layer_hi, meta.layer_end)),
 *   k_out[l - layer_lo][h][dst_start + t][:] = shift(K_c[l][h][src_off + t][:], delta)
 *   v_out[l - layer_lo][h][dst_start + t][:] = V_c[l][h][src_off + t][:]
 * k_out/v_out: [layer_hi - layer_lo][n_kv_heads][n_ctx][head_dim].
 * chunk_meta: [n_chunks][CKV_META_STRIDE] int32 (CKV_META_* fields below).
 *
 * Paged source: page pool [n_pages][n_layers][2 (K,V)][n_kv_heads][CKV_PAGE_TOKENS][head_dim],
 * the chunk's pages listed at page_table[meta.table_offset ...]. */
#define CKV_PAGE_TOKENS 16
#define CKV_META_STRIDE 8
#define CKV_META_TABLE_OFFSET 0 /* first page-table slot (paged) / first pointer slot (dense) */
#define CKV_META_LENGTH 1       /* tokens to copy */
#define CKV_META_DST_START 2    /* destination position (Placement.start) */
#define CKV_META_DELTA 3        /* Placement.start - ChunkKV.start */
#define CKV_META_LAYER_BEGIN 4  /* first layer to copy (1 skips a layer 0 that is recomputed) */
#define CKV_META_LAYER_END 5    /* one past the last layer to copy */
#define CKV_META_SRC_OFFSET 6   /* first token of the chunk to copy */
#define CKV_META_HEAD_STRIDE 7  /* dense source only: elements between heads */

CKV_API int ckv_blend_gather_paged(const uint16_t* pool, int64_t n_pages, const int32_t* page_table,
                           const int32_t* chunk_meta, int n_chunks, const float* inv_freq,
                           int rot_dims, uint16_t* k_out, uint16_t* v_out, int layer_lo,
                           int layer_hi, int n_layers, int n_kv_heads, int head_dim, int n_ctx,
                           ckv_stream_t stream);

/* Dense source: k_ptrs/v_ptrs are device arrays of device addresses,
 * [n_chunks * n_layers] (slot meta.table_offset + l), each pointing at a
 * (H, len, D) tensor with head stride meta.head_stride and token stride head_dim
 * (what ChunkKV.keys[l] holds, torch_engine.py:101-102). */
CKV_API int ckv_blend_gather_dense(const uint64_t* k_ptrs, const uint64_t* v_ptrs,
                           const int32_t* chunk_meta, int n_chunks, const float* inv_freq,
                           int rot_dims, uint16_t* k_out, uint16_t* v_out, int layer_lo,
                           int layer_hi, int n_kv_heads, int head_dim, int n_ctx,
                           ckv_stream_t stream);

/* ---- store insert (PrefillResult.chunk base.py:55-60 + KVStore.put kvstore.py:47-58) --
 * Writes `length` tokens of every layer into pages page_ids[0 .. ceil(length/16)).
 * k_ptrs/v_ptrs: device arrays [n_layers] of device addresses of (H, >=length, D)
 * sources with head stride head_stride (elements) and token stride head_dim. */
CKV_API int ckv_pages_write(uint16_t* pool, int64_t n_pages, const int32_t* page_ids, int length,
                    const uint64_t* k_ptrs, const uint64_t* v_ptrs, int64_t head_stride,
                    int n_layers, int n_kv_heads, int head_dim, ckv_stream_t stream);

/* ---- layer-1 deviation + pooled top-k (torch_engine.py:117-153) ------------
 * Fused: per active token diff = sum (bf16(k - K))^2 + sum (bf16(v - V))^2,
 * norm = sum k^2 + sum v^2 (fp32), then in the last CTA to finish: per-chunk
 * rel = sum diff / sum norm, escalation, budget capped at the eligible count,
 * top-`budget` by diff (ties: lower position first), compaction.
 *   k_fresh/v_fresh: [n_act][n_kv_heads*head_dim] rows at stride fresh_row_stride
 *   k_base/v_base  : [n_kv_heads][n_ctx][head_dim] (layer-1 blended cache before the write)
 *   active         : [n_act] ascending positions computed at layer 1
 *   pos_flags      : [n_ctx] bit0 cached, bit1 sink, bit2 exact
 *   sel_meta       : [n_chunks][4] start, length, budget (-1: ratio <= 0, not pooled), exact
 * Outputs: diff/norm [n_ctx] (positions not in `active` untouched), rel [n_chunks],
 *   keep_abs [n_ctx] ascending kept positions, sel [n_ctx] their index in `active`,
 *   counts [8]: n_sel, selected_cached, budget_final, n_eligible, escalated_mask_lo,
 *   status (0 ok), n_keep_fresh, reserved.
 * The threshold is compared in double, as the reference compares the Python float
 * rel (torch_engine.py:132-134).
 * Scratch: CKV_SELECT_SCRATCH_BYTES(n_ctx) bytes, 16-byte aligned (a score key and
 * a flag byte per position; the selection uses it only when n_ctx is larger than
 * what it keeps in shared memory, 43008 positions).  control: CKV_SELECT_CONTROL_BYTES
 * bytes, 16-byte aligned (the last-CTA ticket and the first radix level's histogram,
 * which every CTA adds its rows to); it must be zero before the first call and every
 * call leaves it zero (zero it again after a device error).  Calls that share a
 * control block or scratch must not overlap on the GPU. */
#define CKV_SEL_META_STRIDE 4
#define CKV_SELECT_SCRATCH_BYTES(n_ctx) (5 * (((size_t)(n_ctx) + 15) / 16 * 16))
#define CKV_SELECT_CONTROL_BYTES 8448
CKV_API int ckv_deviation_select(const uint16_t* k_fresh, const uint16_t* v_fresh,
                         int64_t fresh_row_stride, const uint16_t* k_base,
                         const uint16_t* v_base, const int32_t* active, int n_act,
                         const uint8_t* pos_flags, int n_ctx, const int32_t* sel_meta,
                         int n_chunks, int has_threshold, double escalate_threshold,
                         int n_kv_heads, int head_dim, float* diff, float* norm, float* rel,
                         int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* scratch,
                         void* control, ckv_stream_t stream);

/* Allocation-free variant of ckv_deviation_select — no counterpart in the
 * reference.  For callers that can pass their inputs and outputs but cannot
 * provide (allocate) the selection's scratch: its per-position keys and flags and
 * its control block live in a static device array inside the library, held by every GPU that
 * loads it until process exit (CKV_SELECT_CONTROL_BYTES + 5 * CKV_NOALLOC_MAX_CTX
 * bytes, 328 KiB).  Same arguments and results as ckv_deviation_select without
 * `scratch` and `control`; n_ctx must be at most
 * CKV_NOALLOC_MAX_CTX (else CKV_ERR_ARG).  The first call on a device looks up
 * the array's device address; make that first call before any stream capture.
 * Calls share the array: calls that overlap on the GPU race. */
#define CKV_NOALLOC_MAX_CTX 65536
CKV_API int ckv_deviation_select_noalloc(const uint16_t* k_fresh, const uint16_t* v_fresh,
                                         int64_t fresh_row_stride, const uint16_t* k_base,
                                         const uint16_t* v_base, const int32_t* active, int n_act,
                                         const uint8_t* pos_flags, int n_ctx,
                                         const int32_t* sel_meta, int n_chunks, int has_threshold,
                                         double escalate_threshold, int n_kv_heads, int head_dim,
                                         float* diff, float* norm, float* rel, int32_t* keep_abs,
                                         int32_t* sel, int32_t* counts, ckv_stream_t stream);

/* Deviation scores only (torch_engine.py:118-124), the first phase of
 * ckv_deviation_select: diff/norm [n_ctx] at the positions in `active`, summed
 * over the n_kv_heads heads given.  A tensor-parallel rank scores its own KV
 * heads; the sum of the ranks' scores (an all-reduce) then feeds
 * ckv_select_from_scores on every rank. */
CKV_API int ckv_deviation_scores(const uint16_t* k_fresh, const uint16_t* v_fresh,
                                 int64_t fresh_row_stride, const uint16_t* k_base,
                                 const uint16_t* v_base, const int32_t* active, int n_act,
                                 const uint8_t* pos_flags, int n_ctx, int n_kv_heads, int head_dim,
                                 float* diff, float* norm, ckv_stream_t stream);

/* Selection only, from given fp32 scores (torch_engine.py:125-153): the same
 * device code as the second phase of ckv_deviation_select, one CTA.  `active`
 * is implied: every non-exact position, ascending.  scratch: as for
 * ckv_deviation_select, CKV_SELECT_SCRATCH_BYTES(n_ctx) bytes. */
CKV_API int ckv_select_from_scores(const float* diff, const float* norm, const uint8_t* pos_flags,
                           int n_ctx, const int32_t* sel_meta, int n_chunks,
                           int has_threshold, double escalate_threshold, float* rel,
                           int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* scratch,
                           ckv_stream_t stream);

/* Shrink to the selection (torch_engine.py:152-156): for i < counts[0]
 *   h_out[i] = h_in[sel[i]], x_out[i] = x_in[sel[i]]  (rows of `hidden`)
 *   k_cache[h][keep_abs[i]] = k_fresh[sel[i]][h], same for v.
 * Rows at or beyond counts[0] (up to max_rows) are left untouched. */
CKV_API int ckv_apply_selection(const int32_t* sel, const int32_t* keep_abs, const int32_t* counts,
                        int max_rows, const uint16_t* h_in, uint16_t* h_out,
                        const uint16_t* x_in, uint16_t* x_out, int hidden,
                        const uint16_t* k_fresh, const uint16_t* v_fresh,
                        int64_t fresh_row_stride, uint16_t* k_cache, uint16_t* v_cache,
                        int n_kv_heads, int head_dim, int n_ctx, ckv_stream_t stream);

/* ---- decoder pieces of the recompute (torch_engine.py:61-76, 105-107, 112-165) -- */

/* out[i] = table[tokens[rows[i]]] (embed_tokens, torch_engine.py:105-107). */
CKV_API int ckv_embed(const uint16_t* table, int vocab, int hidden, const int32_t* tokens,
              const int32_t* rows, int n_rows, uint16_t* out, ckv_stream_t stream);

/* Qwen2RMSNorm: y = w * bf16(x * rsqrt(mean(x^2) + eps)) (fp32 inside). */
CKV_API int ckv_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int hidden,
                float eps, ckv_stream_t stream);

/* ---- decode projections, m <= 8 rows (greedy decode, torch_engine.py:180-198) ------
 * One warp per weight row (row pair for RoPE), the weight streamed once; same epilogues
 * and rounding points as ckv_linear_residual / ckv_linear_swiglu / ckv_qkv_rope:
 *   ckv_gemv_residual   h[m][n] = bf16(h + bf16(x W^T))
 *   ckv_gemv_swiglu     out[m][j] = bf16(bf16(silu(bf16(g))) * bf16(u)), gate/up rows
 *                       interleaved in 128-row blocks as for ckv_linear_swiglu
 *   ckv_gemv_qkv_rope   all q, k, v columns of w_qkv (rows q | k | v) with bias; RoPE at
 *                       positions[m] from rope_table [rope_max_pos][head_dim/2] (cos, sin);
 *                       q -> q_out [m][Hq*D], k / v -> caches [Hk][n_ctx][D] at the row's
 *                       position (an out-of-range position is skipped and recorded). */
CKV_API int ckv_gemv_residual(const uint16_t* x, const uint16_t* w, uint16_t* h, int m, int n, int k,
                              ckv_stream_t stream);
CKV_API int ckv_gemv_swiglu(const uint16_t* x, const uint16_t* w_gate_up, uint16_t* out, int m,
                            int inter, int k, ckv_stream_t stream);
CKV_API int ckv_gemv_qkv_rope(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* b_qkv, int m,
                              int k, int n_q_heads, int n_kv_heads, int head_dim,
                              const int32_t* positions, const float* rope_table, int rope_max_pos,
                              uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, int n_ctx,
                              ckv_stream_t stream);
/* The same two projections of x = RMSNorm(h) with norm_w (the rounding of ckv_rmsnorm,
 * Qwen2RMSNorm before the attention and before the MLP): each CTA normalises the rows
 * itself, saving the separate RMSNorm launch of a decode step.  m <= 4, k <= 5120. */
CKV_API int ckv_gemv_swiglu_rmsnorm(const uint16_t* h, const uint16_t* norm_w, float eps,
                                    const uint16_t* w_gate_up, uint16_t* out, int m, int inter, int k,
                                    ckv_stream_t stream);
CKV_API int ckv_gemv_qkv_rope_rmsnorm(const uint16_t* h, const uint16_t* norm_w, float eps,
                                      const uint16_t* w_qkv, const uint16_t* b_qkv, int m, int k,
                                      int n_q_heads, int n_kv_heads, int head_dim,
                                      const int32_t* positions, const float* rope_table,
                                      int rope_max_pos, uint16_t* q_out, uint16_t* k_cache,
                                      uint16_t* v_cache, int n_ctx, ckv_stream_t stream);

/* ---- tensor parallel over NVLink peer memory (no collective library) ------------
 * The o_proj / down_proj row-parallel GEMM and the following all-reduce + residual add
 * (torch_engine.py:70-76), split over `ranks` GPUs (one process each):
 *   ckv_linear_partial    out = x W^T, this rank's bf16 partial rows [m][n] in its own
 *                         buffer; its last CTA then adds 1 to flags[q][rank] on every
 *                         rank q.
 *   ckv_reduce_add_gather on each rank, for the 128-row blocks it owns (block b -> rank
 *                         b % ranks): waits until its partial counters reach `epoch`, reads
 *                         every rank's partial rows (part_peer[q]) over NVLink, sums them in
 *                         rank order in fp32, h = bf16(h + bf16(sum)), and writes the row
 *                         into every rank's h (h_peer[q]); its last CTA adds 1 to
 *                         gather_peer[q][rank] on every rank and waits until its own gather
 *                         counters reach `epoch`.  The next RMSNorm then runs locally.
 * part_peer / flags / h_peer / gather_peer are device arrays of `ranks` device addresses
 * (this rank's own at index rank), mapped with ckv_ipc_open.  Counters start at 0 and
 * `epoch` counts the exchanges made so far, this one included.  Two partial buffers must
 * alternate between consecutive exchanges.  Waits are bounded (2 s,
 * CKV_DEV_ERR_WAIT_TIMEOUT).  No multicast objects are used. */
#define CKV_MAX_RANKS 8
CKV_API int ckv_linear_partial(const uint16_t* x, const uint16_t* w, uint16_t* out, int m, int n,
                               int k, const uint64_t* flags, uint32_t* ticket, int rank, int ranks,
                               ckv_stream_t stream);
CKV_API int ckv_reduce_add_gather(const uint64_t* part_peer, int rank, int ranks, int m, int hidden,
                                  const uint16_t* h, const uint64_t* h_peer, const uint32_t* part_cnt,
                                  uint32_t* gather_cnt, const uint64_t* gather_peer, uint32_t* ticket,
                                  uint32_t epoch, ckv_stream_t stream);
/* Device memory that other processes can map (CUDA IPC, plain peer mappings): allocate
 * (zeroed) and get its 64-byte handle; open a peer's handle; close / free. */
CKV_API int ckv_ipc_alloc(int64_t bytes, void** ptr, void* handle64);
CKV_API int ckv_ipc_open(const void* handle64, void** ptr);
CKV_API int ckv_ipc_close(void* ptr);
CKV_API int ckv_ipc_free(void* ptr);

/* Residual add then RMSNorm, for a row-parallel projection whose partial sums
 * were all-reduced (tensor parallel; torch_engine.py:70-76 residual adds):
 *   h = bf16(h + delta); y = w * bf16(h * rsqrt(mean(h^2) + eps)).
 * h is updated in place; y must not alias h or delta.  hidden <= 5120. */
CKV_API int ckv_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, uint16_t* y,
                            int rows, int hidden, float eps, ckv_stream_t stream);

/* out = bf16(x @ w^T (+ bias)); x [m][k], w [n][k] (nn.Linear), out [m][n].
 * tcgen05/TMEM GEMM; k % 8 == 0, n % 16 == 0, 16-byte aligned rows. */
CKV_API int ckv_linear(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* out,
               int m, int n, int k, ckv_stream_t stream);

/* h = bf16(h + bf16(x @ w^T)) in place (o_proj / down_proj + residual,
 * torch_engine.py:72-73). */
CKV_API int ckv_linear_residual(const uint16_t* x, const uint16_t* w, uint16_t* h, int m, int n, int k,
                        ckv_stream_t stream);

/* out = bf16(silu(bf16(x@Wg^T)) * bf16(x@Wu^T)) (Qwen2MLP gate/up).  w_gate_up
 * interleaves the two weights in blocks of 128 rows: rows [256b, 256b+128) are
 * gate rows [128b, 128b+128), rows [256b+128, 256b+256) the matching up rows.
 * out [m][inter]; inter % 128 == 0. */
CKV_API int ckv_linear_swiglu(const uint16_t* x, const uint16_t* w_gate_up, uint16_t* out, int m,
                      int inter, int k, ckv_stream_t stream);

/* QKV projection + bias + RoPE at `positions` (TorchEngine._qkv, torch_engine.py:61-66)
 * for output columns [col_begin, col_end) of w_qkv ([Hq*D + 2*H*D][k], q|k|v rows).
 * q heads -> q_out [m][Hq*D]; k/v heads -> scattered into k_cache/v_cache
 * [H][n_ctx][D] at positions[i] (torch_engine.py:155-156) when those are non-NULL,
 * else into k_compact/v_compact [m][H*D].  rope_table from ckv_rope_table with
 * rope_max_pos > every position. */
CKV_API int ckv_qkv_rope(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* b_qkv, int m, int k,
                 int col_begin, int col_end, int n_q_heads, int n_kv_heads, int head_dim,
                 const int32_t* positions, const float* rope_table, int rope_max_pos,
                 uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, int n_ctx,
                 uint16_t* k_compact, uint16_t* v_compact, ckv_stream_t stream);

/* Attention of m query tokens over the blended cache with the reference's
 * position mask key j visible iff j <= positions[i] (torch_engine.py:68-70,157),
 * GQA n_q_heads / n_kv_heads (at most 128 query heads per KV head).
 * q/out [m][Hq][D]; caches [H][n_ctx][D]; head_dim 64 or 128.  tcgen05/TMEM kernel.
 * The kernel is persistent (one CTA per SM) and takes its work items from two
 * scheduler words at the start of `workspace` (16-byte aligned): zero them once when
 * the buffer is allocated; every call leaves them at zero again, so calls may reuse the
 * buffer in stream order but must not overlap on the GPU.  Past those 256 bytes the
 * workspace holds the partials that let long rows be split along the keys when whole
 * rows would leave SMs idle.  ckv_attention_workspace_size() gives the bytes for both
 * (at least 256).  With a smaller workspace the keys are not split; with NULL the
 * items are assigned statically (CTA c takes items c, c + grid, ...).  Every schedule
 * gives the same result up to the key split's rounding.  One query token (m == 1) with
 * 1, 2, 4, 5, 6, 7, 8 or 16 query heads per KV head and a workspace of the size given
 * for m == 1 takes a split-KV path on CUDA cores instead (decode); it reads the
 * position on the device, so a captured launch serves every later position. */
CKV_API int64_t ckv_attention_workspace_size(int m, int n_q_heads, int n_kv_heads, int head_dim,
                                             int n_ctx);
/* Kernels one ckv_attention call launches at this shape and workspace size: 1, or 2 when
 * a merge kernel follows (key splits, or the decode path); 0 for a shape ckv_attention
 * refuses. */
CKV_API int ckv_attention_launches(int m, int n_q_heads, int n_kv_heads, int head_dim, int n_ctx,
                                   int64_t workspace_bytes);
CKV_API int ckv_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          const int32_t* positions, uint16_t* out, int m, int n_q_heads,
                          int n_kv_heads, int head_dim, int n_ctx, float scale, void* workspace,
                          int64_t workspace_bytes, ckv_stream_t stream);

/* Small-m projection (lm_head on the logit rows, torch_engine.py:75-76,165):
 * out [m][n] = bf16(x [m][k] @ w[n][k]^T), m <= 8. */
CKV_API int ckv_gemv(const uint16_t* x, const uint16_t* w, uint16_t* out, int m, int n, int k,
             ckv_stream_t stream);

/* Greedy next token of the decode loop (TorchEngine.generate, torch_engine.py:185,196-197):
 * token[0] = argmax of one bf16 logits row (NaN first, then the largest value, ties to the
 * lower index, as torch.argmax), and, when position is not NULL, position[0] += 1. */
CKV_API int ckv_greedy_next(const uint16_t* logits, int n, int32_t* token, int32_t* position,
                            ckv_stream_t stream);

/* log_softmax of one bf16 row into fp32 (TorchEngine.last_logprobs, torch_engine.py:200-201). */
CKV_API int ckv_log_softmax(const uint16_t* logits, int n, float* out, ckv_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* CHUNKKV_B200_H */
