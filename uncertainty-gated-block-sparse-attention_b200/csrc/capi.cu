// capi.cu -- the extern "C" entry points of libugbsa (declared in include/ugbsa.h).
//
// Host-side validation, budget arithmetic (src/sparse_attention.py:688-695),
// the driver entry point for TMA tensor maps, and the device error word.
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "ugbsa_internal.h"

// One sticky error word per device: kernels OR timeout bits into it;
// ugbsa_read_device_error() reads and clears it.
static __device__ int g_ugbsa_device_error;

namespace ugbsa {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, unsigned rank, void *addr,
                      const cuuint64_t *dims, const cuuint64_t *strides_bytes, const cuuint32_t *box,
                      const cuuint32_t *elem_strides) {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return UGBSA_ERR_NO_DEVICE;
    const CUresult r = g_encode(map, dtype, rank, addr, dims, strides_bytes, box, elem_strides,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? UGBSA_OK : UGBSA_ERR_ALIGN;
}

int *device_error_word() {
    static int *ptrs[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_ugbsa_device_error) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<int *>(p);
    }
    return ptrs[dev];
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int elt_size(int dtype) { return dtype == UGBSA_F32 ? 4 : 2; }

// Q/K/V views: d contiguous, the other strides 16-byte multiples, base aligned.
static int check_view(const void *p, int dtype, ugbsa_strides st) {
    if (!p) return UGBSA_ERR_ARG;
    if (st.d != 1) return UGBSA_ERR_ALIGN;
    const int e = elt_size(dtype);
    if (!aligned16(p)) return UGBSA_ERR_ALIGN;
    if ((st.s * e) % 16 || (st.h * e) % 16 || (st.b * e) % 16) return UGBSA_ERR_ALIGN;
    if (st.s < 0 || st.h < 0 || st.b < 0) return UGBSA_ERR_ALIGN;
    return UGBSA_OK;
}

static void budget(const ugbsa_selector_config *c, int NB, int *kb, int *km) {
    // k_bud_row = max(min(k_max, budget_blocks), k_min); k_base = min(2*k_bud_row, NB)
    int row = c->budget_blocks < c->k_max ? c->budget_blocks : c->k_max;
    row = row > c->k_min ? row : c->k_min;
    const long long base = 2LL * row < NB ? 2LL * row : NB;
    long long mx = base;
    if (c->mode == UGBSA_MODE_ROUTER) mx = 2 * base < NB ? 2 * base : NB;
    *kb = (int)base;
    *km = (int)mx;
}

static bool cfg_is_quest(const ugbsa_selector_config *c) {
    return c->mode == UGBSA_MODE_QUEST || (c->mode == UGBSA_MODE_ROUTER && c->router_score == UGBSA_SCORE_QUEST);
}

static int check_cfg(const ugbsa_selector_config *c) {
    if (!c) return UGBSA_ERR_ARG;
    if (c->mode < 0 || c->mode > 2) return UGBSA_ERR_ARG;
    if (c->router_score < 0 || c->router_score > 1) return UGBSA_ERR_ARG;
    if (c->router_mode < 0 || c->router_mode > 1) return UGBSA_ERR_ARG;
    if (c->router_grain < 0 || c->router_grain > 1) return UGBSA_ERR_ARG;
    if (c->budget_blocks < 1 && c->k_min < 1) return UGBSA_ERR_ARG;
    return UGBSA_OK;
}

}  // namespace ugbsa

using namespace ugbsa;

extern "C" {

int ugbsa_version(void) { return 100; }

const char *ugbsa_status_string(int s) {
    switch (s) {
        case UGBSA_OK: return "ok";
        case UGBSA_ERR_ARG: return "invalid argument";
        case UGBSA_ERR_SHAPE: return "unsupported or inconsistent shape";
        case UGBSA_ERR_DTYPE: return "unsupported dtype";
        case UGBSA_ERR_ALIGN: return "pointer or stride not 16-byte addressable (innermost stride must be 1)";
        case UGBSA_ERR_UNSUPPORTED: return "unsupported head_dim (64, 128 or 256 for attention; <= 256 and a multiple of 8 otherwise)";
        case UGBSA_ERR_WORKSPACE: return "workspace missing or too small";
        case UGBSA_ERR_LAUNCH: return "CUDA launch failed";
        case UGBSA_ERR_DEVICE: return "a kernel gave up on a bounded device-side wait";
        case UGBSA_ERR_NO_DEVICE: return "no usable sm_100 device or driver entry point";
        case UGBSA_ERR_TOO_LARGE: return "problem too large for the 1 MiB fixed scratch of ugbsa_select_noalloc";
    }
    return "unknown status";
}

int ugbsa_select_budget(const ugbsa_selector_config *cfg, int S, int *k_base, int *kmax) {
    if (check_cfg(cfg) != UGBSA_OK || S <= 0 || !k_base || !kmax) return UGBSA_ERR_ARG;
    budget(cfg, (S + 63) / 64, k_base, kmax);
    return UGBSA_OK;
}

size_t ugbsa_select_workspace_bytes(const ugbsa_selector_config *cfg, int B, int Hq, int S) {
    (void)cfg;
    if (B <= 0 || Hq <= 0 || S <= 0) return 0;
    return select_workspace_bytes(B, Hq, S);
}

size_t ugbsa_select_workspace_bytes_ex(const ugbsa_selector_config *cfg, int dtype, int B, int Hq, int Hkv, int S,
                                       int D) {
    (void)cfg;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return 0;
    return select_workspace_bytes_exact(dtype, B, Hq, Hkv, S, D);
}

int ugbsa_block_summary(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                        float *out_a, float *out_b, float *out_norm, ugbsa_stream_t stream) {
    if (B <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return UGBSA_ERR_SHAPE;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    int rc = check_view(K, dtype, ks);
    if (rc) return rc;
    if (!out_a || (quest && !out_b)) return UGBSA_ERR_ARG;
    if (!aligned16(out_a) || (quest && !aligned16(out_b))) return UGBSA_ERR_ALIGN;
    return launch_block_summary(K, dtype, ks, B, Hkv, S, D, quest ? 1 : 0, out_a, out_b, out_norm,
                                reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_select(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B, int Hq,
                 int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax,
                 float *sigma, uint8_t *trigger, void *workspace, size_t workspace_bytes, ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return UGBSA_ERR_SHAPE;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    if ((rc = check_view(Q, dtype, qs))) return rc;
    const bool quest = (cfg->mode == UGBSA_MODE_QUEST) ||
                       (cfg->mode == UGBSA_MODE_ROUTER && cfg->router_score == UGBSA_SCORE_QUEST);
    if (!summ_a || (quest && !summ_b) || !kv_idx) return UGBSA_ERR_ARG;
    if (!aligned16(summ_a) || (quest && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    const int NB = (S + 63) / 64;
    if (NB > 8192) return UGBSA_ERR_SHAPE;  // sort keys live in shared memory
    int kb, km;
    budget(cfg, NB, &kb, &km);
    if (km != kmax) return UGBSA_ERR_SHAPE;
    if (!workspace || workspace_bytes < select_workspace_bytes_exact(dtype, B, Hq, Hkv, S, D))
        return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    return launch_select(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, scale, cfg, kb, km, kv_idx, sigma,
                         trigger, workspace, reinterpret_cast<cudaStream_t>(stream));
}

// The Sq query rows of a call: local tile t = 0 .. ceil(Sq/64) - 1 is sequence tile
// seq_tile(t, row_base / 64, pair_stride) and holds min(64, S - 64 * tile) rows.
static int check_tiles(int S, int row_base, int pair_stride, int Sq, int align) {
    if (row_base < 0 || row_base % align || pair_stride < 1 || Sq <= 0) return UGBSA_ERR_SHAPE;
    const int t_base = row_base / 64;
    if (pair_stride > 1 && (t_base & 1)) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64, nt = (Sq + 63) / 64;
    int64_t rows = 0;
    for (int t = 0; t < nt; ++t) {
        const int g = seq_tile(t, t_base, pair_stride);
        if (g >= NB) return UGBSA_ERR_SHAPE;
        rows += (S - 64 * g < 64) ? S - 64 * g : 64;
    }
    return rows == Sq ? UGBSA_OK : UGBSA_ERR_SHAPE;
}

int ugbsa_select_tiles_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                            int B, int Hq, int Hkv, int S, int D, int row_base, int pair_stride, int Sq, float scale,
                            const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma_cells,
                            float *sigma_rowsum, void *workspace, size_t workspace_bytes, ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64;
    if (NB > 8192) return UGBSA_ERR_SHAPE;
    // a slice starts on a tile pair (128 rows) and covers whole tiles up to the sequence end
    if ((rc = check_tiles(S, row_base, pair_stride, Sq, 128))) return rc;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    if ((rc = check_view(Q, dtype, qs))) return rc;
    if (!summ_a || (cfg_is_quest(cfg) && !summ_b) || !kv_idx || !sigma_cells) return UGBSA_ERR_ARG;
    if (!aligned16(summ_a) || (cfg_is_quest(cfg) && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    int kb, km;
    budget(cfg, NB, &kb, &km);
    if (km != kmax) return UGBSA_ERR_SHAPE;
    const int Qt = (Sq + 63) / 64;
    const size_t need = select_tiles_scratch_bytes(dtype, B, Hq, Hkv, S, D, Qt);
    if (need && (!workspace || workspace_bytes < need)) return UGBSA_ERR_WORKSPACE;
    if (need && !aligned16(workspace)) return UGBSA_ERR_ALIGN;
    return launch_select_tiles(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, row_base / 64, pair_stride, Sq, scale,
                               cfg, kb, km, kv_idx, sigma_cells, sigma_rowsum, workspace,
                               reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_select_tiles(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                       int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx,
                       int kmax, float *sigma_cells, float *sigma_rowsum, void *workspace, size_t workspace_bytes,
                       ugbsa_stream_t stream) {
    return ugbsa_select_tiles_rows(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, 0, 1, S, scale, cfg, kv_idx,
                                   kmax, sigma_cells, sigma_rowsum, workspace, workspace_bytes, stream);
}

size_t ugbsa_select_finish_workspace_bytes(int B, int S) {
    if (B <= 0 || S <= 0) return 0;
    return select_finish_workspace_bytes(B, S);
}

int ugbsa_select_finish_rows(const float *sigma_cells, const float *sigma_all, int B, int Hq, int Hq_total, int S,
                             int row_base, int pair_stride, int Sq, const ugbsa_selector_config *cfg,
                             int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger, void *workspace,
                             size_t workspace_bytes, ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hq_total < Hq || S <= 0) return UGBSA_ERR_SHAPE;
    if ((rc = check_tiles(S, row_base, pair_stride, Sq, 64))) return rc;
    if (!sigma_cells || !sigma_all || !kv_idx) return UGBSA_ERR_ARG;
    int kb, km;
    budget(cfg, (S + 63) / 64, &kb, &km);
    if (km != kmax) return UGBSA_ERR_SHAPE;
    if (!workspace || workspace_bytes < select_finish_workspace_bytes(B, S)) return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    return launch_select_finish(sigma_cells, sigma_all, B, Hq, Hq_total, S, row_base / 64, pair_stride,
                                (Sq + 63) / 64, cfg, kb, km, kv_idx, sigma, trigger, workspace,
                                reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_select_finish(const float *sigma_cells, const float *sigma_all, int B, int Hq, int Hq_total, int S,
                        const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger,
                        void *workspace, size_t workspace_bytes, ugbsa_stream_t stream) {
    return ugbsa_select_finish_rows(sigma_cells, sigma_all, B, Hq, Hq_total, S, 0, 1, S, cfg, kv_idx, kmax, sigma,
                                    trigger, workspace, workspace_bytes, stream);
}

static int attn_checked(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                        ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk,
                        int D, int row_base, int pair_stride, float scale, void *out, ugbsa_strides os,
                        void *const *peers, int npeers, ugbsa_stream_t stream) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || Hq % Hkv || kmax <= 0) return UGBSA_ERR_SHAPE;
    int rc;
    if ((row_base != 0 || pair_stride != 1) && (rc = check_tiles(Sk, row_base, pair_stride, Sq, 64))) return rc;
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype != UGBSA_BF16 && dtype != UGBSA_F16 && dtype != UGBSA_F32) return UGBSA_ERR_DTYPE;
    if ((rc = check_view(Q, dtype, qs)) || (rc = check_view(K, dtype, ks)) || (rc = check_view(V, dtype, vs)) ||
        (rc = check_view(out, dtype, os)))
        return rc;
    if (!kv_idx) return UGBSA_ERR_ARG;
    if (npeers < 0 || npeers > UGBSA_MAX_PEERS || (npeers > 0 && !peers)) return UGBSA_ERR_ARG;
    if (dtype == UGBSA_F32) {   // CUDA-core kernel; output peers are a bf16 / fp16 feature
        if (npeers > 0) return UGBSA_ERR_DTYPE;
        if (kmax > 8192) return UGBSA_ERR_SHAPE;
        return launch_attn_f32(static_cast<const float *>(Q), static_cast<const float *>(K),
                               static_cast<const float *>(V), qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D,
                               row_base / 64, pair_stride, scale, static_cast<float *>(out), os,
                               reinterpret_cast<cudaStream_t>(stream));
    }
    for (int i = 0; i < npeers; ++i)
        if ((rc = check_view(peers[i], dtype, os))) return rc;
    if (kmax > 8192) return UGBSA_ERR_SHAPE;
    int *err = device_error_word();
    if (!err) return UGBSA_ERR_NO_DEVICE;
    return launch_attn(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D, row_base / 64, pair_stride,
                       scale, out, os, peers, npeers, reinterpret_cast<cudaStream_t>(stream), err);
}

int ugbsa_attn_rows(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                    ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                    int row_base, int pair_stride, float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream) {
    return attn_checked(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D, row_base, pair_stride, scale,
                        out, os, nullptr, 0, stream);
}

int ugbsa_attn_rows_peers(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs,
                          ugbsa_strides ks, ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq,
                          int Hkv, int Sq, int Sk, int D, int row_base, int pair_stride, float scale, void *out,
                          ugbsa_strides os, void *const *peer_out, int npeers, ugbsa_stream_t stream) {
    return attn_checked(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D, row_base, pair_stride, scale,
                        out, os, peer_out, npeers, stream);
}

// ------------------------------------------------------------ decode
int ugbsa_block_summary_update(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                               int first_block, int nb_capacity, float *out_a, float *out_b, ugbsa_stream_t stream) {
    if (B <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64;
    if (first_block < 0 || first_block >= NB || nb_capacity < NB) return UGBSA_ERR_SHAPE;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    int rc = check_view(K, dtype, ks);
    if (rc) return rc;
    if (!out_a || (quest && !out_b)) return UGBSA_ERR_ARG;
    if (!aligned16(out_a) || (quest && !aligned16(out_b))) return UGBSA_ERR_ALIGN;
    return launch_block_summary_range(K, dtype, ks, B, Hkv, S, D, quest ? 1 : 0, first_block, nb_capacity, out_a,
                                      out_b, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

static size_t al256s(size_t x) { return (x + 255) / 256 * 256; }

size_t ugbsa_decode_workspace_bytes(int B, int Hq, int S, int D, int kmax) {
    if (B <= 0 || Hq <= 0 || S <= 0 || D <= 0 || kmax <= 0) return 0;
    const size_t sel = al256s((size_t)B * Hq * 4) + al256s((size_t)B * 4) + al256s(select_finish_workspace_bytes(B, S));
    const size_t att = decode_attn_workspace_bytes(B, Hq, D, kmax);
    return sel + al256s(att);   // the fused step holds the cells' margins while the attention runs
}

int ugbsa_decode_select(const void *q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                        int nb_capacity, int B, int Hq, int Hkv, int S, int D, float scale,
                        const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma, uint8_t *trigger,
                        void *workspace, size_t workspace_bytes, ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64;
    if (NB > 8192 || nb_capacity < NB) return UGBSA_ERR_SHAPE;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    if (!q || !kv_idx || !summ_a || (cfg_is_quest(cfg) && !summ_b)) return UGBSA_ERR_ARG;
    if (qs.d != 1) return UGBSA_ERR_ALIGN;
    if (!aligned16(summ_a) || (cfg_is_quest(cfg) && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    int kb, km;
    budget(cfg, NB, &kb, &km);
    if (km != kmax) return UGBSA_ERR_SHAPE;
    if (!workspace || workspace_bytes < ugbsa_decode_workspace_bytes(B, Hq, S, D, kmax)) return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (kb < km);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *cells = reinterpret_cast<float *>(ws);
    float *rowsum = reinterpret_cast<float *>(ws + al256s((size_t)B * Hq * 4));
    void *fin_ws = ws + al256s((size_t)B * Hq * 4) + al256s((size_t)B * 4);
    if ((rc = launch_decode_select(q, dtype, qs.b, qs.h, summ_a, summ_b, nb_capacity, B, Hq, Hkv, S, D, scale,
                                   cfg_is_quest(cfg), kb, km, router, kv_idx, cells, st)))
        return rc;
    if ((int64_t)B * Hq <= 1024) return launch_decode_finish(cells, B, Hq, S, cfg, kb, km, kv_idx, sigma, trigger, st);
    // many cells: the prefill finish (row sums, radix quantile, finalize) on one-tile rows
    const bool row = cfg->router_grain == UGBSA_GRAIN_ROW;
    if (router && row && (rc = launch_sigma_rowsum(cells, B, Hq, 1, rowsum, st))) return rc;
    return launch_select_finish_q(cells, (router && row) ? rowsum : cells, B, Hq, Hq, S, 1, 0, 1, 1, cfg, kb, km,
                                  kv_idx, sigma, trigger, fin_ws, st);
}

int ugbsa_decode_attn(const void *q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                      ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int S, int D,
                      float scale, void *out, ugbsa_strides os, void *workspace, size_t workspace_bytes,
                      ugbsa_stream_t stream) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || Hq % Hkv || kmax <= 0) return UGBSA_ERR_SHAPE;
    if (kmax > 1024) return UGBSA_ERR_SHAPE;   // kept blocks staged in shared memory
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype != UGBSA_BF16 && dtype != UGBSA_F16) return UGBSA_ERR_DTYPE;
    int rc;
    if ((rc = check_view(q, dtype, qs)) || (rc = check_view(K, dtype, ks)) || (rc = check_view(V, dtype, vs)) ||
        (rc = check_view(out, dtype, os)))
        return rc;
    if (!kv_idx) return UGBSA_ERR_ARG;
    if (!workspace || workspace_bytes < decode_attn_workspace_bytes(B, Hq, D, kmax)) return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    return launch_decode_attn(q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, S, D, scale, out, os, workspace,
                              reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_decode_step(const void *q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                      ugbsa_strides vs, float *summ_a, float *summ_b, int nb_capacity, int B, int Hq, int Hkv, int S,
                      int D, float scale, const ugbsa_selector_config *cfg, int32_t *kv_idx, int kmax, float *sigma,
                      uint8_t *trigger, void *out, ugbsa_strides os, void *workspace, size_t workspace_bytes,
                      ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv || kmax <= 0) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64;
    if (NB > 8192 || nb_capacity < NB || kmax > 1024) return UGBSA_ERR_SHAPE;
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype != UGBSA_BF16 && dtype != UGBSA_F16) return UGBSA_ERR_DTYPE;
    if ((rc = check_view(q, dtype, qs)) || (rc = check_view(K, dtype, ks)) || (rc = check_view(V, dtype, vs)) ||
        (rc = check_view(out, dtype, os)))
        return rc;
    const bool quest = cfg_is_quest(cfg);
    if (!kv_idx || !summ_a || (quest && !summ_b)) return UGBSA_ERR_ARG;
    if (!aligned16(summ_a) || (quest && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    int kb, km;
    budget(cfg, NB, &kb, &km);
    if (km != kmax) return UGBSA_ERR_SHAPE;
    if (!workspace || workspace_bytes < ugbsa_decode_workspace_bytes(B, Hq, S, D, kmax)) return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (kb < km);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *cells = reinterpret_cast<float *>(ws);
    const size_t sel = al256s((size_t)B * Hq * 4) + al256s((size_t)B * 4) + al256s(select_finish_workspace_bytes(B, S));
    void *att_ws = ws + sel;
    if ((int64_t)B * Hq <= 256) {
        // three launches: selection (+ the last block's summary), attention (+ the router), merge
        if ((rc = launch_decode_select(q, dtype, qs.b, qs.h, summ_a, summ_b, nb_capacity, B, Hq, Hkv, S, D, scale,
                                       quest, kb, km, router, kv_idx, cells, st, K, ks)))
            return rc;
        DecodeRouter r{cfg, kb, cells, kv_idx, sigma, trigger};
        return launch_decode_attn(q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, S, D, scale, out, os, att_ws,
                                  st, &r);
    }
    // many cells: the separate calls
    if ((rc = ugbsa_block_summary_update(K, dtype, ks, B, Hkv, S, D, quest ? 1 : 0, NB - 1, nb_capacity, summ_a,
                                         summ_b, stream)))
        return rc;
    if ((rc = ugbsa_decode_select(q, dtype, qs, summ_a, summ_b, nb_capacity, B, Hq, Hkv, S, D, scale, cfg, kv_idx,
                                  kmax, sigma, trigger, workspace, workspace_bytes, stream)))
        return rc;
    return launch_decode_attn(q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, S, D, scale, out, os, att_ws, st);
}

// ------------------------------------------------------------ norm + rotary producer
int ugbsa_qk_norm_rope(const void *X, int dtype, ugbsa_strides xs, const void *weight, int norm_mode, float eps,
                       const void *cos, const void *sin, int64_t cs_b, int64_t cs_s, int rot_dim, int B, int H,
                       int S, int D, void *Y, ugbsa_strides ys, int summary, float *summ_a, float *summ_b,
                       ugbsa_stream_t stream) {
    if (B <= 0 || H <= 0 || S <= 0) return UGBSA_ERR_SHAPE;
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    if (rot_dim < 16 || rot_dim > D || (rot_dim & (rot_dim - 1))) return UGBSA_ERR_UNSUPPORTED;
    if (dtype != UGBSA_BF16 && dtype != UGBSA_F16) return UGBSA_ERR_DTYPE;
    if (norm_mode != UGBSA_NORM_SCALE && norm_mode != UGBSA_NORM_OFFSET && norm_mode != UGBSA_NORM_NONE)
        return UGBSA_ERR_ARG;
    if (summary < UGBSA_SUMMARY_NONE || summary > UGBSA_SUMMARY_QUEST) return UGBSA_ERR_ARG;
    if (!(eps >= 0.f)) return UGBSA_ERR_ARG;
    int rc;
    if ((rc = check_view(X, dtype, xs)) || (rc = check_view(Y, dtype, ys))) return rc;
    const bool has_w = norm_mode != UGBSA_NORM_NONE;
    if ((has_w && !weight) || !cos || !sin) return UGBSA_ERR_ARG;
    if ((has_w && !aligned16(weight)) || !aligned16(cos) || !aligned16(sin)) return UGBSA_ERR_ALIGN;
    if (cs_b < 0 || cs_s < rot_dim || (cs_b * 2) % 16 || (cs_s * 2) % 16) return UGBSA_ERR_ALIGN;
    if (summary && (!summ_a || (summary == UGBSA_SUMMARY_QUEST && !summ_b))) return UGBSA_ERR_ARG;
    if (summary && (!aligned16(summ_a) || (summary == UGBSA_SUMMARY_QUEST && !aligned16(summ_b))))
        return UGBSA_ERR_ALIGN;
    return launch_qk_norm_rope(X, dtype, xs, weight, norm_mode == UGBSA_NORM_NONE ? 2 : (norm_mode == UGBSA_NORM_OFFSET ? 1 : 0), eps, cos, sin, cs_b,
                               cs_s, rot_dim, B, H, S, D, Y, ys, summary, summ_a, summ_b,
                               reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------ block-score diagnostic
size_t ugbsa_block_order_stats_workspace_bytes(int B, int Hq, int S) {
    if (B <= 0 || Hq <= 0 || S <= 1) return 0;
    return block_order_stats_workspace_bytes(B, Hq, S);
}

int ugbsa_block_order_stats(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                            int B, int Hq, int Hkv, int S, int D, float scale, int quest, int budget_blocks,
                            float *g, float *r, float *sigma, float *g_rho, float *tau_hat, void *workspace,
                            size_t workspace_bytes, ugbsa_stream_t stream) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 1 || D <= 0 || Hq % Hkv || budget_blocks <= 0) return UGBSA_ERR_SHAPE;
    const int NB = (S + 63) / 64;
    if (NB > 8192) return UGBSA_ERR_SHAPE;
    const int k_b = 2 * budget_blocks < NB ? 2 * budget_blocks : NB;
    const int rho_k = 2 * k_b < NB ? 2 * k_b : NB;
    if (rho_k <= k_b || rho_k >= NB) return UGBSA_ERR_SHAPE;   // no rank rho_k in the tile's sort
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    int rc;
    if ((rc = check_view(Q, dtype, qs))) return rc;
    if (!summ_a || (quest && !summ_b) || !g || !r || !sigma || !g_rho) return UGBSA_ERR_ARG;
    if (!aligned16(summ_a) || (quest && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    if (tau_hat) {
        if (!workspace || workspace_bytes < block_order_stats_workspace_bytes(B, Hq, S)) return UGBSA_ERR_WORKSPACE;
        if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    }
    return launch_block_order_stats(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, scale, quest != 0, k_b, rho_k,
                                    g, r, sigma, g_rho, tau_hat, workspace, reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------ peer buffers (CUDA IPC)
int ugbsa_peer_buffer_alloc(size_t bytes, void **ptr, ugbsa_ipc_handle *handle) {
    if (!ptr || !handle || bytes == 0) return UGBSA_ERR_ARG;
    *ptr = nullptr;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return UGBSA_ERR_LAUNCH;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(ugbsa_ipc_handle), "IPC handle size");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return UGBSA_ERR_LAUNCH;
    }
    memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    return UGBSA_OK;
}

int ugbsa_peer_buffer_open(const ugbsa_ipc_handle *handle, void **ptr) {
    if (!ptr || !handle) return UGBSA_ERR_ARG;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->bytes, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return UGBSA_ERR_LAUNCH;
    }
    *ptr = p;
    return UGBSA_OK;
}

int ugbsa_peer_buffer_close(void *ptr) {
    if (!ptr) return UGBSA_ERR_ARG;
    if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
        cudaGetLastError();
        return UGBSA_ERR_LAUNCH;
    }
    return UGBSA_OK;
}

int ugbsa_peer_buffer_free(void *ptr) {
    if (!ptr) return UGBSA_ERR_ARG;
    if (cudaFree(ptr) != cudaSuccess) {
        cudaGetLastError();
        return UGBSA_ERR_LAUNCH;
    }
    return UGBSA_OK;
}

int ugbsa_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
               ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
               float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream) {
    return ugbsa_attn_rows(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D, 0, 1, scale, out, os,
                           stream);
}

// One CTA waits on a shared-memory barrier that nothing arrives at, through the
// same bounded wait the kernels use: it must give up after the wait limit, record
// the timeout bit in the device error word and return.
__global__ void __launch_bounds__(32) wait_limit_check_kernel(int *err) {
    __shared__ uint64_t bar;
    __shared__ int s_abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    const WaitCtx wc{err, &s_abort};
    (void)mbar_wait(&bar, 0, wc);
}

int ugbsa_check_wait_limit(ugbsa_stream_t stream) {
    int *err = device_error_word();
    if (!err) return UGBSA_ERR_NO_DEVICE;
    wait_limit_check_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(err);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int ugbsa_check_bf16_fma(const uint32_t *a, const uint32_t *b, const float *c, float *mixed, float *ref, int n,
                         ugbsa_stream_t stream) {
    if (n < 0 || (n > 0 && (!a || !b || !c || !mixed || !ref))) return UGBSA_ERR_ARG;
    if (!device_error_word()) return UGBSA_ERR_NO_DEVICE;
    return launch_check_bf16_fma(a, b, c, mixed, ref, n, reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_read_device_error(ugbsa_stream_t stream, int *bits) {
    int *err = device_error_word();
    if (!err) return UGBSA_ERR_NO_DEVICE;
    int h = 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return UGBSA_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return UGBSA_ERR_LAUNCH;
    if (h) {
        const int zero = 0;
        if (cudaMemcpyAsync(err, &zero, sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess) return UGBSA_ERR_LAUNCH;
        cudaStreamSynchronize(s);
    }
    if (bits) *bits = h;
    return h ? UGBSA_ERR_DEVICE : UGBSA_OK;
}

}  // extern "C"

// ------------------------------------------------------------ v1 per-row selection
size_t ugbsa_select_rows_workspace_bytes(const ugbsa_selector_config *cfg, int B, int Hq, int S) {
    (void)cfg;
    if (B <= 0 || Hq <= 0 || S <= 0) return 0;
    return select_rows_workspace_bytes(B, Hq, S);
}

int ugbsa_select_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                      int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg,
                      uint32_t *keep_bits, int32_t *kv_idx, float *sigma, uint8_t *trigger, void *workspace,
                      size_t workspace_bytes, ugbsa_stream_t stream) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return UGBSA_ERR_SHAPE;
    if (D % 8 || D > 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype < UGBSA_F32 || dtype > UGBSA_F16) return UGBSA_ERR_DTYPE;
    if ((rc = check_view(Q, dtype, qs))) return rc;
    if (!summ_a || (cfg_is_quest(cfg) && !summ_b) || !keep_bits) return UGBSA_ERR_ARG;
    if (!aligned16(summ_a) || (cfg_is_quest(cfg) && !aligned16(summ_b))) return UGBSA_ERR_ALIGN;
    const int NB = (S + 63) / 64;
    if (NB > 6144) return UGBSA_ERR_SHAPE;   // a row's block keys are ranked in shared memory
    if (!workspace || workspace_bytes < select_rows_workspace_bytes(B, Hq, S)) return UGBSA_ERR_WORKSPACE;
    if (!aligned16(workspace)) return UGBSA_ERR_ALIGN;
    return launch_select_rows(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, scale, cfg, keep_bits, kv_idx, sigma,
                              trigger, workspace, reinterpret_cast<cudaStream_t>(stream));
}

int ugbsa_keep_to_tiles(const uint8_t *keep, uint32_t *keep_bits, int B, int H, int S, int32_t *kv_idx,
                        ugbsa_stream_t stream) {
    if (B <= 0 || H <= 0 || S <= 0) return UGBSA_ERR_SHAPE;
    if (!keep_bits) return UGBSA_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int rc;
    if (keep && (rc = launch_keep_pack(keep, B, H, S, (S + 63) / 64, keep_bits, st))) return rc;
    if (kv_idx) return launch_rows_to_tiles(keep_bits, B, H, S, kv_idx, st);
    return UGBSA_OK;
}

int ugbsa_attn_rowmask(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                       ugbsa_strides vs, const int32_t *kv_idx, int kmax, const uint32_t *keep_bits, int B, int Hq,
                       int Hkv, int S, int D, float scale, void *out, ugbsa_strides os, ugbsa_stream_t stream) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || Hq % Hkv || kmax <= 0) return UGBSA_ERR_SHAPE;
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    if (dtype != UGBSA_BF16 && dtype != UGBSA_F16) return UGBSA_ERR_DTYPE;
    int rc;
    if ((rc = check_view(Q, dtype, qs)) || (rc = check_view(K, dtype, ks)) || (rc = check_view(V, dtype, vs)) ||
        (rc = check_view(out, dtype, os)))
        return rc;
    if (!kv_idx || !keep_bits) return UGBSA_ERR_ARG;
    if (kmax > 8192) return UGBSA_ERR_SHAPE;
    int *err = device_error_word();
    if (!err) return UGBSA_ERR_NO_DEVICE;
    return launch_attn_rowmask(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, keep_bits, B, Hq, Hkv, S, S, D, scale, out,
                               os, reinterpret_cast<cudaStream_t>(stream), err);
}
