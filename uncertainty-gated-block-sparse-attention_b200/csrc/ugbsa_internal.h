// ugbsa_internal.h -- declarations shared by the .cu files of libugbsa (not installed).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ugbsa.h"

namespace ugbsa {

// cuTensorMapEncodeTiled through the driver entry point (no -lcuda link).
int encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, unsigned rank, void *addr,
                      const cuuint64_t *dims, const cuuint64_t *strides_bytes, const cuuint32_t *box,
                      const cuuint32_t *elem_strides);

int launch_block_summary(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                         float *out_a, float *out_b, float *out_norm, cudaStream_t stream);
// blocks nb0 .. ceil(S/64)-1 only, into [B, Hkv, NBo, D] outputs (a growing cache's summaries)
int launch_block_summary_range(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                               int nb0, int NBo, float *out_a, float *out_b, float *out_norm, cudaStream_t stream);

// bound over dtype, head dim and KV heads (the legacy size query)
size_t select_workspace_bytes(int B, int Hq, int S);
// what launch_select lays out (ugbsa_select checks against this)
size_t select_workspace_bytes_exact(int dtype, int B, int Hq, int Hkv, int S, int D);
size_t select_finish_workspace_bytes(int B, int S);
// Qt: the tiles the call scores (all ceil(S/64) unless the query rows are a slice)
size_t select_tiles_scratch_bytes(int dtype, int B, int Hq, int Hkv, int S, int D, int Qt);

// tensor-core scoring path (select_tc.cu): bf16 Q, head_dim 64 or 128
bool tc_select_supported(int dtype, int D);
size_t tc_scratch_bytes(int B, int Hq, int Hkv, int S, int D, int Qt);
// Q holds Sq query rows: local tile t is sequence tile seq_tile(t, t_base, pair_stride)
// (t_base even); the summaries cover all S keys; outputs are indexed by local tile
int launch_select_tiles_tc(const void *Q, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B, int Hq,
                           int Hkv, int S, int D, int t_base, int pair_stride, int Sq, float scale, bool quest,
                           int k_base, int kmax, bool router, int32_t *kv_idx, float *sigma_cell, void *scratch,
                           cudaStream_t stream);

int launch_select_tiles(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                        int Hq, int Hkv, int S, int D, int t_base, int pair_stride, int Sq, float scale,
                        const ugbsa_selector_config *cfg, int k_base, int kmax, int32_t *kv_idx, float *sigma_cell,
                        float *sigma_rowsum, void *scratch, cudaStream_t stream);

// sigma_all covers every tile of the sequence; sigma_cell / kv_idx / outputs the
// Qt local tiles, local tile t being sequence tile seq_tile(t, t_base, pair_stride)
int launch_select_finish(const float *sigma_cell, const float *sigma_all, int B, int Hq, int H_total, int S,
                         int t_base, int pair_stride, int Qt, const ugbsa_selector_config *cfg, int k_base, int kmax,
                         int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace,
                         cudaStream_t stream);

int launch_select(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                  int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int k_base, int kmax,
                  int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace, cudaStream_t stream);

// fused per-head RMSNorm + rotary embedding (+ K block summary) (rope.cu)
// norm_mode: 0 scale, 1 offset, 2 none (weight unused)
int launch_qk_norm_rope(const void *X, int dtype, ugbsa_strides xs, const void *weight, int norm_mode, float eps,
                        const void *cos, const void *sin, int64_t cs_b, int64_t cs_s, int rot_dim, int B, int H,
                        int S, int D, void *Y, ugbsa_strides ys, int summary, float *summ_a, float *summ_b,
                        cudaStream_t stream);

// the finish with the quantile over Qt_all tiles per (b, head) (a decode step: 1)
int launch_select_finish_q(const float *sigma_cell, const float *sigma_all, int B, int Hq, int H_total, int S,
                           int Qt_all, int t_base, int pair_stride, int Qt_local, const ugbsa_selector_config *cfg,
                           int k_base, int kmax, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out,
                           void *workspace, cudaStream_t stream);
int launch_sigma_rowsum(const float *sigma_cell, int B, int Hq, int Qt, float *rowsum, cudaStream_t stream);

// decode (decode.cu): one query row per head over a cache of S keys.
// launch_decode_select: scores + top-kmax + sigma per (b, q-head) (a cluster of CTAs per cell);
// launch_decode_finish: the router over the B x Hq cells (B * Hq <= 1024, else UNSUPPORTED)
// refresh_K (optional, the fused step): the cluster's last CTA also recomputes the summary of
// the cache's last block from these K rows once the scoring has read the summaries
int launch_decode_select(const void *Q, int dtype, int64_t qb, int64_t qh, const float *summ_a, const float *summ_b,
                         int NBs, int B, int Hq, int Hkv, int S, int D, float scale, bool quest, int k_base, int kmax,
                         bool router, int32_t *kv_idx, float *sigma_cell, cudaStream_t stream,
                         const void *refresh_K = nullptr, ugbsa_strides refresh_ks = ugbsa_strides{0, 0, 0, 0});
int launch_decode_finish(const float *sigma_cell, int B, int Hq, int S, const ugbsa_selector_config *cfg, int k_base,
                         int kmax, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, cudaStream_t stream);
int launch_check_bf16_fma(const uint32_t *a, const uint32_t *b, const float *c, float *mixed, float *ref, int n,
                          cudaStream_t stream);
int decode_nsplit(int B, int Hq, int kmax);
size_t decode_attn_workspace_bytes(int B, int Hq, int D, int kmax);
// the selection's router taken inside the attention (the fused step; B * Hq <= 256):
// kv_idx as the selection left it (the attention finalises it), the cells' margins
struct DecodeRouter {
    const ugbsa_selector_config *cfg;
    int k_base;
    const float *sigma_cell;
    int32_t *kv_idx;
    float *sigma_out;
    uint8_t *trigger_out;
};
int launch_decode_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                       ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int S, int D,
                       float scale, void *out, ugbsa_strides os, void *workspace, cudaStream_t stream,
                       const DecodeRouter *router = nullptr);

// block-score diagnostic (select.cu): order statistics of the unforced tile scores
// at ranks k_b, rho_k (rho_k < NB) and, if tau_hat, the noise scale (workspace:
// block_order_stats_workspace_bytes)
size_t block_order_stats_workspace_bytes(int B, int Hq, int S);
int launch_block_order_stats(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                             int B, int Hq, int Hkv, int S, int D, float scale, bool quest, int k_b, int rho_k,
                             float *g, float *r, float *sigma, float *g_rho, float *tau_hat, void *workspace,
                             cudaStream_t stream);

// Q holds Sq query rows, local tile t being sequence tile seq_tile(t, t_base, pair_stride)
// (keys 0 .. Sk - 1).  pair_stride 1: out holds the same rows as Q; otherwise out holds
// every sequence row.  peers[0 .. npeers-1] (npeers < 8): the same output view in other
// GPUs' buffers.
int launch_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                int t_base, int pair_stride, float scale, void *out, ugbsa_strides os, void *const *peers,
                int npeers, cudaStream_t stream, int *err);
// v1 per-row selector (select_rows.cu); row scores by select_tile_kernel<..., ROWS> (select.cu)
int launch_row_scores(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                      int Hq, int Hkv, int S, int D, float scale, bool quest, float *row_scores, cudaStream_t stream);
size_t select_rows_workspace_bytes(int B, int Hq, int S);
void rows_budget(const ugbsa_selector_config *cfg, int NB, int *k_bud, int *k_eff);
int launch_select_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                       int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg,
                       uint32_t *keep_bits, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace,
                       cudaStream_t stream);
int launch_rows_to_tiles(const uint32_t *keep_bits, int B, int H, int S, int32_t *kv_idx, cudaStream_t stream);
int launch_keep_pack(const uint8_t *keep, int B, int H, int S, int NB, uint32_t *bits, cudaStream_t stream);
// attention with a per-row keep mask [B, Hq, Sq, ceil(NB/32)] (launch_attn's kernels, whole sequence)
int launch_attn_rowmask(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                        ugbsa_strides vs, const int32_t *kv_idx, int kmax, const uint32_t *rowmask, int B, int Hq,
                        int Hkv, int Sq, int Sk, int D, float scale, void *out, ugbsa_strides os, cudaStream_t stream,
                        int *err);
// fp32 Q/K/V (CUDA cores, attn_f32.cu); same row mapping as launch_attn, no peers
int launch_attn_f32(const float *Q, const float *K, const float *V, ugbsa_strides qs, ugbsa_strides ks,
                    ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                    int t_base, int pair_stride, float scale, float *out, ugbsa_strides os, cudaStream_t stream);
// two-tile (M=128) variant for D = 64 / 128; UGBSA_ERR_UNSUPPORTED when its
// shared memory does not fit (the caller then uses launch_attn's single-tile kernel)
int launch_attn_pair(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                     ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                     float scale, void *out, ugbsa_strides os, cudaStream_t stream, int *err);

// Device error word of the current device (sticky until ugbsa_read_device_error).
int *device_error_word();

}  // namespace ugbsa
