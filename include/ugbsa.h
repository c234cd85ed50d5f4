/*
 * ugbsa.h -- C ABI of libugbsa, the B200 (sm_100a) block-sparse attention
 * prefill path with the uncertainty-gated (sigma router) block selector.
 *
 * The reference project is pure Python; its hot path is two functions behind
 * the Hugging Face AttentionInterface hook ("block_sparse",
 * src/sparse_attention.py:751-806):
 *   _block_select_kv_idx_v2(query, key_states, scaling)   src/sparse_attention.py:588-748
 *   block_sparse_attn_v2(q, k, v, kv_idx, scale)          src/triton_block_attn.py:267-298
 * Each entry point below names the part of that path it replaces.  A Python
 * caller binds them with ctypes, as the package ugbsa.sparse_attention does
 * (its ugbsa/_lib.py lists every signature).
 *
 * Conventions
 *  - Every function returns an int status: 0 (UGBSA_OK) or a UGBSA_ERR_* code.
 *    ugbsa_status_string() describes a code.
 *  - All tensor pointers are DEVICE pointers owned by the caller.  Q/K/V are
 *    addressed as [B, H, S, D] with element strides given in ugbsa_strides
 *    (the innermost, d, stride must be 1; the others multiples of 8 elements
 *    for bf16/fp16 so that TMA can address them).
 *  - Every launch goes to the given cudaStream_t and is asynchronous; no entry
 *    point synchronises the host except ugbsa_read_device_error().
 *  - The library allocates nothing: scratch memory is a caller-supplied
 *    workspace whose size ugbsa_select_workspace_bytes_ex() reports.
 *  - Block size is fixed at 64 tokens (BLOCK / BLOCK_M / BLOCK_N of the
 *    reference, src/sparse_attention.py:51, triton_block_attn.py:267).
 */
#ifndef UGBSA_H
#define UGBSA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in cuda_runtime.h */
typedef struct CUstream_st *ugbsa_stream_t;

enum {
    UGBSA_OK = 0,
    UGBSA_ERR_ARG = 1,          /* null pointer, negative size, bad enum            */
    UGBSA_ERR_SHAPE = 2,        /* Hq % Hkv != 0, S out of range, kmax mismatch      */
    UGBSA_ERR_DTYPE = 3,        /* unsupported dtype for this entry point            */
    UGBSA_ERR_ALIGN = 4,        /* pointer / stride not 16-byte addressable         */
    UGBSA_ERR_UNSUPPORTED = 5,  /* head_dim not in {64, 128, 256}                    */
    UGBSA_ERR_WORKSPACE = 6,    /* workspace missing or too small                    */
    UGBSA_ERR_LAUNCH = 7,       /* CUDA launch / attribute error                     */
    UGBSA_ERR_DEVICE = 8,       /* a kernel recorded a device-side error (timeout)   */
    UGBSA_ERR_NO_DEVICE = 9,    /* no sm_100 device / driver entry point missing     */
    UGBSA_ERR_TOO_LARGE = 10    /* problem exceeds ugbsa_select_noalloc's fixed scratch */
};

enum { UGBSA_F32 = 0, UGBSA_BF16 = 1, UGBSA_F16 = 2 };

/* Selector.mode (src/sparse_attention.py:58), restricted to the v2 modes (:776) */
enum { UGBSA_MODE_TOPK = 0, UGBSA_MODE_QUEST = 1, UGBSA_MODE_ROUTER = 2 };
/* Selector.router_score (:90) */
enum { UGBSA_SCORE_MEAN = 0, UGBSA_SCORE_QUEST = 1 };
/* Selector.router_mode (:80) */
enum { UGBSA_ROUTER_ABS = 0, UGBSA_ROUTER_QUANTILE = 1 };
/* Selector.router_grain (:81) */
enum { UGBSA_GRAIN_CELL = 0, UGBSA_GRAIN_ROW = 1 };

/* Element strides of a [B, H, S, D] view. */
typedef struct {
    int64_t b, h, s, d;
} ugbsa_strides;

/* The Selector knobs the v2 path reads (src/sparse_attention.py:58-97). */
typedef struct {
    int mode;               /* UGBSA_MODE_*                          */
    int router_score;       /* UGBSA_SCORE_* (router mode only)      */
    int router_mode;        /* UGBSA_ROUTER_*                        */
    int router_grain;       /* UGBSA_GRAIN_*                         */
    double router_quantile; /* q of the bottom-q trigger             */
    double router_tau;      /* abs-mode threshold (compared as fp32) */
    int budget_blocks;      /* per-row budget, clamped to [k_min, k_max] then doubled (:688-689) */
    int k_min, k_max;
} ugbsa_selector_config;

/* Library version (major*10000 + minor*100 + patch). */
int ugbsa_version(void);

/* Human-readable text for a status code (static storage). */
const char *ugbsa_status_string(int status);

/* Budget arithmetic of src/sparse_attention.py:688-695 for a sequence of
 * S tokens: k_base (per-tile slots) and kmax (slots of kv_idx, 2*k_base for
 * the router, capped at the block count). */
int ugbsa_select_budget(const ugbsa_selector_config *cfg, int S, int *k_base, int *kmax);

/* Bytes of scratch memory ugbsa_select needs for this problem: exactly what it
 * lays out for this dtype, head_dim D and KV head count (ugbsa_select returns
 * UGBSA_ERR_WORKSPACE when given less). */
size_t ugbsa_select_workspace_bytes_ex(const ugbsa_selector_config *cfg, int dtype, int B, int Hq, int Hkv, int S,
                                       int D);

/* A bound of ugbsa_select_workspace_bytes_ex over every dtype, head_dim
 * (<= 256) and KV head count (<= Hq), for callers that size the workspace
 * before they know those: at least as large as the exact size, often larger. */
size_t ugbsa_select_workspace_bytes(const ugbsa_selector_config *cfg, int B, int Hq, int S);

/*
 * Block summaries of K, one per 64-token block and KV head
 * (replaces src/sparse_attention.py:617-646: F.pad + view + mean / amin / amax).
 *   quest = 0: out_a = K-mean   [B, Hkv, NB, D] fp32
 *   quest = 1: out_a = K-min, out_b = K-max  [B, Hkv, NB, D] fp32
 * Rows past S count as the reference's zero padding.
 * Optional out_norm [B, Hkv, NB] fp32 receives the Euclidean norm of the
 * mean (quest = 0) or of max(|K-min|, |K-max|) (quest = 1); pass NULL to skip.
 */
int ugbsa_block_summary(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                        float *out_a, float *out_b, float *out_norm, ugbsa_stream_t stream);

/*
 * Tile scoring, top-kmax, sigma router and kv_idx emission
 * (replaces src/sparse_attention.py:638-748 after the summaries).
 *   Q        [B, Hq, S, D] (dtype)
 *   summ_a/b summaries from ugbsa_block_summary of the matching KV heads
 *            (Q head h reads KV head h / (Hq/Hkv), the reference's repeat_kv, :761)
 *   kv_idx   [B, Hq, Qt, kmax] int32 out, contiguous.  Slots in descending
 *            tile score (ties -> lower block id); slots >= k_base of tiles the
 *            router did not trigger hold NB (the sentinel, :720-725).
 *   sigma    optional [B, Hq, Qt] fp32 out: per-tile margin after the grain
 *            step (NaN where undefined); NULL to skip.
 *   trigger  optional [B, Hq, Qt] uint8 out: 1 where the tile kept 2*k_base; NULL to skip.
 *   workspace >= ugbsa_select_workspace_bytes_ex(cfg, dtype, B, Hq, Hkv, S, D)
 *            bytes of device memory.
 */
int ugbsa_select(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B, int Hq,
                 int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax,
                 float *sigma, uint8_t *trigger, void *workspace, size_t workspace_bytes, ugbsa_stream_t stream);

/*
 * ugbsa_select without a workspace argument, for callers that cannot allocate
 * device memory (a serving runtime whose memory planner already owns the whole
 * device, a binding that only holds the tensors it was handed).  No
 * counterpart in the reference, which allocates freely through PyTorch.
 * The scratch comes from a fixed 1 MiB array inside the library (held by every
 * GPU that loads it until exit); problems whose
 * ugbsa_select_workspace_bytes_ex(cfg, dtype, B, Hq, Hkv, S, D) exceeds it
 * return UGBSA_ERR_TOO_LARGE.  With bf16 Q and head_dim 64 / 128 / 256 that
 * size grows with S^2 (the exact tile scores, 4*B*Hq*ceil(S/64)^2 bytes): 28
 * query / 4 KV heads at head_dim 128 fit up to about 5K tokens, one head up to
 * about 28K; other dtypes and head dims fit any S the selector accepts at 28
 * heads.  The array is shared by all calls on
 * a device: calls whose kernels overlap on the GPU race.  The first call on a
 * device looks the array's address up (cudaGetSymbolAddress) and should come
 * before any stream capture.  Same arguments and results as ugbsa_select.
 */
int ugbsa_select_noalloc(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                         int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg,
                         int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger, ugbsa_stream_t stream);

/*
 * ugbsa_select in two halves, for heads sharded across GPUs (the reference is
 * single-device; its row-grain head mean, src/sparse_attention.py:708-710, is
 * the one step that couples heads).  ugbsa_select == tiles + finish on one GPU.
 *
 * ugbsa_select_tiles: scoring, top-kmax and the per-tile margin for this
 *   shard's Hq heads (reading Hkv KV heads' summaries).  Writes kv_idx with all
 *   kmax slots filled (no sentinel yet), sigma_cells [B, Hq, Qt] fp32 and, if
 *   sigma_rowsum is not NULL, its per-tile sum over these heads [B, Qt] fp32
 *   (head order; exact, since the margins are subnormal).  workspace: scratch
 *   of at least ugbsa_select_workspace_bytes_ex(cfg, dtype, B, Hq, Hkv, S, D)
 *   bytes (or the looser ugbsa_select_workspace_bytes(cfg, B, Hq, S)).
 * Between the halves the caller combines shards: row grain -> SUM all-reduce of
 *   sigma_rowsum over ranks; cell grain -> all-gather of sigma_cells.
 * ugbsa_select_finish: quantile over all Hq_total heads and sentinel fill of
 *   this shard's kv_idx.  sigma_all is the combined array ([B, Qt] sums over
 *   all heads for row grain, [B, Hq_total, Qt] cells for cell grain).
 */
int ugbsa_select_tiles(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                       int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx,
                       int kmax, float *sigma_cells, float *sigma_rowsum, void *workspace, size_t workspace_bytes,
                       ugbsa_stream_t stream);

size_t ugbsa_select_finish_workspace_bytes(int B, int S);

int ugbsa_select_finish(const float *sigma_cells, const float *sigma_all, int B, int Hq, int Hq_total, int S,
                        const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger,
                        void *workspace, size_t workspace_bytes, ugbsa_stream_t stream);

/*
 * Query-row slices, for a sequence split across GPUs: a call holds all heads
 * but only some query rows of the S-token sequence (keys, values and block
 * summaries cover all S tokens).  The reference has no such split; each slice
 * computes exactly what the unsplit call computes for its tiles, bit for bit.
 *
 * Which rows: local query tile t (rows 64t .. 64t + 63 of Q) is sequence tile
 *   row_base / 64 + t + 2 * (t / 2) * (pair_stride - 1),
 * i.e. pairs of consecutive tiles dealt with stride pair_stride starting at
 * row_base.  pair_stride 1: the contiguous rows row_base .. row_base + Sq - 1;
 * pair_stride m > 1 with row_base = 128 r: the pairs r, r + m, r + 2m, ... (rank
 * r of m dealing tile pairs round-robin, which balances the causal cost).  Sq is
 * the number of rows Q holds: every tile 64 rows except the sequence's last.
 *
 * ugbsa_select_tiles_rows: Q [B, Hq, Sq, D]; row_base a multiple of 128.
 *   kv_idx [B, Hq, ceil(Sq/64), kmax], sigma_cells [B, Hq, ceil(Sq/64)],
 *   sigma_rowsum [B, ceil(Sq/64)] are the slice's tiles.  Bf16 Q with head_dim
 *   64, 128 or 256 (the tensor-core scorer) unless the slice is the whole sequence;
 *   otherwise UGBSA_ERR_UNSUPPORTED.  The workspace bound is the unsplit one,
 *   ugbsa_select_workspace_bytes_ex(cfg, dtype, B, Hq, Hkv, S, D).
 * Between the halves the ranks gather the slices' margins into sigma_all
 *   (row grain: [B, ceil(S/64)] head sums in sequence-tile order; cell grain:
 *   all B * Hq * ceil(S/64) cells in any order, the quantile ignores positions).
 * ugbsa_select_finish_rows: the quantile over sigma_all and the sentinel fill
 *   of the slice's kv_idx; row_base a multiple of 64 (of 128 when dealt).
 * ugbsa_attn_rows: Q [B, Hq, Sq, D], kv_idx the slice's tiles, keys 0 .. Sk-1.
 *   pair_stride 1: out [B, Hq, Sq, D] holds the slice's rows (row_base a
 *   multiple of 64, row_base + Sq <= Sk); pair_stride > 1: out [B, Hq, Sk, D]
 *   is indexed by sequence row and only the slice's rows are written.
 * The unsuffixed entry points are these with row_base 0, pair_stride 1, Sq = S.
 */
int ugbsa_select_tiles_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                            int B, int Hq, int Hkv, int S, int D, int row_base, int pair_stride, int Sq, float scale,
                            const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma_cells,
                            float *sigma_rowsum, void *workspace, size_t workspace_bytes, ugbsa_stream_t stream);

int ugbsa_select_finish_rows(const float *sigma_cells, const float *sigma_all, int B, int Hq, int Hq_total, int S,
                             int row_base, int pair_stride, int Sq, const ugbsa_selector_config *cfg,
                             int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger, void *workspace,
                             size_t workspace_bytes, ugbsa_stream_t stream);

int ugbsa_attn_rows(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                    ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                    int row_base, int pair_stride, float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream);

/*
 * Block-sparse causal attention over per-tile kv_idx lists
 * (replaces src/triton_block_attn.py:184-298, _fwd_kernel_v2 + block_sparse_attn_v2).
 *   Q [B, Hq, Sq, D], K/V [B, Hkv, Sk, D] (bf16 or fp16 on the tensor cores;
 *   fp32 on CUDA cores with fp32 products and sums, no output peers), GQA
 *   resolved inside (no repeat_kv copy).  kv_idx [B, Hq, ceil(Sq/64), kmax] int32,
 *   contiguous; entries >= NB (= ceil(Sk/64)) and blocks starting after the
 *   tile's last row are skipped (triton_block_attn.py:231-233).
 *   out [B, Hq, Sq, D] in the input dtype, written through its own strides
 *   (so the caller can write straight into a [B, S, H, D] buffer).
 */
int ugbsa_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
               ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
               float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream);

/*
 * Attention whose output also lands in other GPUs' buffers (sharded layers:
 * the output all-gather done by the attention kernel itself over NVLink).
 * peer_out[i] points at the same [B, Hq, Sq, D] view as out, inside a buffer
 * of another GPU mapped into this process (ugbsa_peer_buffer_open), with the
 * strides os; npeers <= UGBSA_MAX_PEERS.  Each output tile is written to out
 * and to every peer view.  The peers may read their copies once this launch
 * has completed (e.g. after a collective ordered behind it on the stream);
 * they must not be reading the previous contents while it runs.
 */
#define UGBSA_MAX_PEERS 7

int ugbsa_attn_rows_peers(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs,
                          ugbsa_strides ks, ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq,
                          int Hkv, int Sq, int Sk, int D, int row_base, int pair_stride, float scale, void *out,
                          ugbsa_strides os, void *const *peer_out, int npeers, ugbsa_stream_t stream);

/*
 * Device buffers that other processes (other GPUs of the node) can map:
 * ugbsa_peer_buffer_alloc allocates on the current device and returns an
 * opaque handle to pass to the other ranks; ugbsa_peer_buffer_open maps a
 * handle from another rank into this process (peer access enabled);
 * ugbsa_peer_buffer_close unmaps it; ugbsa_peer_buffer_free releases the
 * owner's allocation after every peer has closed it.
 */
typedef struct {
    unsigned char bytes[64];
} ugbsa_ipc_handle;

int ugbsa_peer_buffer_alloc(size_t bytes, void **ptr, ugbsa_ipc_handle *handle);
int ugbsa_peer_buffer_open(const ugbsa_ipc_handle *handle, void **ptr);
int ugbsa_peer_buffer_close(void *ptr);
int ugbsa_peer_buffer_free(void *ptr);

/*
 * Block-sparse decode: one query row per head against a KV cache of S keys.
 * The reference decodes densely (src/sparse_attention.py:756-770, SDPA over the
 * whole cache for Q == 1); this applies the v2 block policy to the decode row,
 * reusing the cache's block summaries:
 *
 * ugbsa_block_summary_update: (re)computes the summaries of blocks
 *   first_block .. ceil(S/64)-1 of K [B, Hkv, S, D] into summary arrays of
 *   capacity nb_capacity blocks ([B, Hkv, nb_capacity, D] fp32, the layout of
 *   ugbsa_block_summary with NB = nb_capacity), e.g. only the last, growing
 *   block after each decode step.
 * ugbsa_decode_select: q [B, Hq, 1, D] (strides qs); scores every block
 *   (exact fp32, the selection's canonical order) for the row at position S-1,
 *   forces the sink and the row's own (last) block, keeps the top kmax
 *   (descending score, ties to the lower id; kmax from ugbsa_select_budget at
 *   S), and applies the router over the B x Hq cells (one tile per cell):
 *   kv_idx [B, Hq, kmax] with sentinel NB in the untriggered cells' slots
 *   >= k_base; sigma / trigger [B, Hq] optional.  S <= 524288 (8192 blocks),
 *   D in {64, 128, 256}, at most 16 Q heads per KV head.
 * ugbsa_decode_attn: out [B, Hq, 1, D] = softmax over the keys (< S) of the
 *   kept blocks, fp32 accumulation, split over the kept blocks; kmax <= 1024.
 * Both take a workspace of ugbsa_decode_workspace_bytes(B, Hq, S, D, kmax)
 * bytes (one buffer serves both calls in turn, and ugbsa_decode_step).
 */
int ugbsa_block_summary_update(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                               int first_block, int nb_capacity, float *out_a, float *out_b, ugbsa_stream_t stream);

size_t ugbsa_decode_workspace_bytes(int B, int Hq, int S, int D, int kmax);

int ugbsa_decode_select(const void *q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                        int nb_capacity, int B, int Hq, int Hkv, int S, int D, float scale,
                        const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger,
                        void *workspace, size_t workspace_bytes, ugbsa_stream_t stream);

int ugbsa_decode_attn(const void *q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                      ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int S, int D,
                      float scale, void *out, ugbsa_strides os, void *workspace, size_t workspace_bytes,
                      ugbsa_stream_t stream);

/*
 * ugbsa_decode_step: a whole decode step -- the same results as
 * ugbsa_block_summary_update(first_block = ceil(S/64) - 1) + ugbsa_decode_select
 * + ugbsa_decode_attn (kv_idx, sigma, trigger bit-identical; out identical) in
 * three launches instead of five when B * Hq <= 256: the refresh of the cache's
 * last block (forced in this step, so never scored) runs inside the selection
 * after the scoring, and the router's threshold / trigger / sentinel fill run
 * inside the attention.  summ_a / summ_b: the cache summaries (capacity
 * nb_capacity blocks), updated in place; kv_idx [B, Hq, kmax] is written (sigma,
 * trigger optional).  bf16 / fp16, D in {64, 128, 256}; workspace of
 * ugbsa_decode_workspace_bytes(B, Hq, S, D, kmax) bytes.
 */
int ugbsa_decode_step(const void *q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                      ugbsa_strides vs, float *summ_a, float *summ_b, int nb_capacity, int B, int Hq, int Hkv, int S,
                      int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma,
                      uint8_t *trigger, void *out, ugbsa_strides os, void *workspace, size_t workspace_bytes,
                      ugbsa_stream_t stream);

/*
 * Fused per-head RMSNorm + rotary embedding + K block summary: the caller side
 * of the hook for models that normalise Q and K per head and then rotate them
 * (transformers' Qwen3 / Qwen3.5-MoE attention: q_norm / k_norm, then
 * apply_rotary_pos_emb, which the reference imports at
 * src/sparse_attention.py:47-48).  One pass over a projection's heads:
 *   X [B, H, S, D] (any strides, unit innermost; e.g. the [B, S, H*D] projection
 *   output viewed as [B, S, H, D] and transposed), bf16 or fp16;
 *   weight [D] (X's dtype); eps;
 *   cos, sin [B, S, rot_dim] (X's dtype; element strides cs_b, cs_s, cs_b = 0
 *   broadcasts one batch); the first rot_dim columns are rotated (rot_dim a
 *   power of two, 16 <= rot_dim <= D), the rest pass through;
 *   Y [B, H, S, D] (may be X itself: each row is read before it is written).
 * norm_mode UGBSA_NORM_SCALE: y = T(w * T(x * r)) (Qwen3RMSNorm);
 * UGBSA_NORM_NONE: y = x, no per-head norm (Qwen2 / Llama attention: rotary
 * only; weight may be NULL);
 * UGBSA_NORM_OFFSET: y = T((x * r) * (1 + w)) (Qwen3.5-MoE / Qwen3-Next), with
 * r = 1 / sqrt(mean(fp32(x^2)) + eps); then out = T(T(y * cos) +
 * T(rotate_half(y) * sin)) on the rotated columns.  summary (for K):
 * UGBSA_SUMMARY_MEAN / _QUEST also writes the block summaries of Y exactly as
 * ugbsa_block_summary would (summ_a mean or Kmin, summ_b Kmax, [B, H, NB, D]
 * fp32), so the selection needs no separate pass over K.  D in {64, 128, 256}.
 */
enum {
    UGBSA_NORM_SCALE = 0,
    UGBSA_NORM_OFFSET = 1,
    UGBSA_NORM_NONE = 2,
    UGBSA_SUMMARY_NONE = 0,
    UGBSA_SUMMARY_MEAN = 1,
    UGBSA_SUMMARY_QUEST = 2
};

int ugbsa_qk_norm_rope(const void *X, int dtype, ugbsa_strides xs, const void *weight, int norm_mode, float eps,
                       const void *cos, const void *sin, int64_t cs_b, int64_t cs_s, int rot_dim, int B, int H,
                       int S, int D, void *Y, ugbsa_strides ys, int summary, float *summ_a, float *summ_b,
                       ugbsa_stream_t stream);

/*
 * Block-score diagnostic (replaces the per-call recording of
 * src/dump_block_scores.py:100-181, which wraps the selector without changing
 * its result).  For every (b, h, tile) of a prefill, over the tile's UNFORCED
 * tile scores (causally invisible blocks -inf, no sink / self forcing), sorted
 * descending as s:
 *   k_b = min(2 * budget_blocks, NB)   (no k_min / k_max clamp)
 *   rho_k = min(2 * k_b, NB)           (must satisfy k_b < rho_k < NB)
 *   g = s[k_b-1] - s[k_b],  r = max(s[0] - s[k_b], 1e-9),
 *   sigma = clamp(g / r, 0, 2),  g_rho = s[rho_k-1] - s[rho_k]
 * written to g, r, sigma, g_rho [B, Hq, ceil(S/64)] fp32 (IEEE inf / NaN as
 * they fall; NaN passes the clamps).  If tau_hat is not NULL, also the
 * noise-scale estimate tau_hat [B, Hq] = sqrt(max(0, mean((bs[i+1] - bs[i])^2)
 * / 2)) over n = min(1024, S-1) query rows i spaced max(1, (S-1)/n) apart
 * (clamped to S-2) and all NB blocks, bs the unmasked per-row block scores;
 * it needs ugbsa_block_order_stats_workspace_bytes(B, Hq, S) of workspace.
 * Scores are exact fp32 (same canonical order as ugbsa_select's).  Returns
 * UGBSA_ERR_SHAPE when rho_k <= k_b or rho_k >= NB (the reference records
 * nothing there).  Diagnostics only: CUDA-core scoring of every visible block.
 */
size_t ugbsa_block_order_stats_workspace_bytes(int B, int Hq, int S);

int ugbsa_block_order_stats(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                            int B, int Hq, int Hkv, int S, int D, float scale, int quest, int budget_blocks,
                            float *g, float *r, float *sigma, float *g_rho, float *tau_hat, void *workspace,
                            size_t workspace_bytes, ugbsa_stream_t stream);

/*
 * The v1 per-row selector and its attention (the reference's _block_select_mask,
 * src/sparse_attention.py:208-382, modes topk / quest / router, and its v1
 * kernel block_sparse_attn with the per-row inner mask,
 * src/triton_block_attn.py:39-181).  Every query row ranks, by its own fp32
 * score (the canonical order of ugbsa_select), the blocks that start at or
 * before it and keeps the top k_bud = clamp(budget_blocks, k_min, k_max)
 * (ties to the lower block id), plus the sink and its own block.  Router: the
 * row's margin on its raw scores at k_eff = clamp(budget_blocks, 1, NB-1),
 * rows with more than k_eff visible blocks eligible, row grain = head mean,
 * quantile over the eligible cells (ineligible and NaN as +inf, k =
 * int(q * eligible count), the row-grain count being of rows) or abs
 * threshold; a triggered (head, row) keeps every visible block.
 *
 * ugbsa_select_rows: Q [B, Hq, S, D]; summaries as for ugbsa_select;
 *   keep_bits [B, Hq, S, ceil(NB/32)] uint32 out (bit j of a row: block j kept);
 *   kv_idx (optional) [B, Hq, ceil(S/64), NB] int32 out: per tile the union of
 *   its rows' blocks, ascending, then the sentinel NB;  sigma (optional)
 *   [B, Hq, S] fp32: the margin after the grain step that the threshold is
 *   compared with (+inf for ineligible rows; NaN without the router);
 *   trigger (optional) [B, Hq, S] uint8.  NB <= 6144.  Workspace:
 *   ugbsa_select_rows_workspace_bytes (the per-row scores, 4*B*Hq*S*NB bytes,
 *   as the reference materialises them).
 * ugbsa_keep_to_tiles: a caller's keep mask keep [B, H, S, NB] uint8 (or NULL
 *   when keep_bits already holds the bits) -> keep_bits, and kv_idx as above
 *   (NULL to skip).
 * ugbsa_attn_rowmask: attention over kv_idx (kmax slots, NB for the lists
 *   above) where row m uses a listed block only if its bit in keep_bits
 *   [B, Hq, S, ceil(NB/32)] is set; bf16 / fp16, head_dim 64 / 128 / 256, the
 *   whole sequence (Sq = Sk = S).
 */
size_t ugbsa_select_rows_workspace_bytes(const ugbsa_selector_config *cfg, int B, int Hq, int S);

int ugbsa_select_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                      int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg,
                      uint32_t *keep_bits, int32_t *kv_idx, float *sigma, uint8_t *trigger, void *workspace,
                      size_t workspace_bytes, ugbsa_stream_t stream);

int ugbsa_keep_to_tiles(const uint8_t *keep, uint32_t *keep_bits, int B, int H, int S, int32_t *kv_idx,
                        ugbsa_stream_t stream);

int ugbsa_attn_rowmask(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                       ugbsa_strides vs, const int32_t *kv_idx, int kmax, const uint32_t *keep_bits, int B, int Hq,
                       int Hkv, int S, int D, float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream);

/*
 * Reads and clears the library's device-side error word (a host sync on the
 * given stream).  Returns UGBSA_OK, or UGBSA_ERR_DEVICE if a kernel gave up on
 * a bounded wait since the last call; *bits (optional) receives the raw bits.
 */
int ugbsa_read_device_error(ugbsa_stream_t stream, int *bits);

/*
 * Check of the kernels' failure path: launches one CTA that waits on a
 * barrier nothing arrives at, with the bounded wait every kernel uses (a
 * 2-second limit).  It gives up, records the timeout bit and returns; the next
 * ugbsa_read_device_error then reports UGBSA_ERR_DEVICE with bit 1 and the
 * context stays usable.  A test aid; the reference has nothing like it.
 */
int ugbsa_check_wait_limit(ugbsa_stream_t stream);

/*
 * Check of the exact scorer's arithmetic: for i < n, mixed[2i] / mixed[2i+1] =
 * the mixed-precision fma (bf16 x bf16 + fp32, one rounding) the exact chains
 * use on the low / high bf16 halves of a[i], b[i] with addend c[2i] / c[2i+1],
 * and ref[...] = __fmaf_rn of the same values converted to fp32.  The two must
 * agree bit for bit (NaN with NaN).  Device pointers.  A test aid.
 */
int ugbsa_check_bf16_fma(const uint32_t *a, const uint32_t *b, const float *c, float *mixed, float *ref, int n,
                         ugbsa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* UGBSA_H */
