// select_rows.cu -- the v1 per-row selector and its tile lists (sm_100a).
//
// Replaces the reference's per-row policy _block_select_mask (src/sparse_attention.py:
// 208-382, modes topk / quest / router) and the kv_idx construction of its v1
// kernel (_compute_kv_idx, src/triton_block_attn.py:125-147):
//
//  0. select_tile_kernel<..., ROWS> (select.cu): every query row's fp32 score
//     of every block up to its tile's last one (the canonical fmaf chains of
//     the v2 path), into a [B, H, S, NB] workspace.
//  1. row_rank_kernel, one warp per (b, head, row): the row ranks the blocks
//     that start at or before it (:240-244) and keeps the top k_bud =
//     clamp(budget, k_min, k_max) (:266-279; ties to the lower block id),
//     then the sink and its own block (:281-283), as a bit mask
//     [B, H, S, ceil(NB/32)]; router: the row's margin on the RAW scores at
//     k_eff = clamp(budget, 1, NB-1) (:303-316) by radix selection of the
//     k_eff-th and (k_eff+1)-th largest values.
//  2. rows_quantile_kernel, one CTA (router only): row grain -> head sum in
//     head order / H (:322); ineligible rows (at most k_eff visible blocks)
//     and NaN as +inf; quantile -> the k-th smallest of those values
//     (kthvalue, k = int(q * eligible count), :325-337).
//  3. rows_finalize_kernel, one warp per (b, head, row): triggered cells keep
//     every visible block (:345-347); optional margin / trigger outputs.
//  4. rows_to_tiles_kernel, one warp per (b, head, tile): the union of the
//     tile's 64 rows' masks as ascending block ids, sentinel NB after them
//     (kv_idx [B, H, Qt, NB]); the attention kernel masks each row to its own
//     blocks (triton_block_attn.py:87-104).
// keep_pack_kernel turns a caller's uint8 [B, H, S, NB] keep mask into the bits.
#include <cfloat>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

namespace {

struct RowRankParams {
    int B, H, S, NB, NBW;
    int k_bud, k_eff, router;
    const float *rs;      // [B,H,S,NB]
    uint32_t *keep;       // [B,H,S,NBW]
    float *sigma;         // [B,H,S]
};

// k-th largest (1-based) of the n ordered keys in keys[] by a byte-wise radix
// selection with a per-warp histogram; returns the key
__device__ uint32_t warp_kth_largest(const uint32_t *keys, int n, int k, uint32_t *hist) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        for (int j = lane; j < n; j += 32) {
            const uint32_t u = keys[j];
            if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
        }
        __syncwarp();
        // from the top bin down: the bin holding the k-th largest
        uint32_t c[8], sum = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            c[e] = hist[255 - (8 * lane + e)];
            sum += c[e];
        }
        uint32_t incl = sum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        const uint32_t excl = incl - sum;
        int bin = -1, knew = 0;
        if (excl < (uint32_t)k && (uint32_t)k <= incl) {
            uint32_t run = excl;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                if (bin < 0 && run + c[e] >= (uint32_t)k) {
                    bin = 255 - (8 * lane + e);
                    knew = k - (int)run;
                }
                run += c[e];
            }
        }
        const unsigned who = __ballot_sync(0xffffffffu, bin >= 0);
        const int src = __ffs(who) - 1;
        bin = __shfl_sync(0xffffffffu, bin, src);
        k = __shfl_sync(0xffffffffu, knew, src);
        prefix |= (uint32_t)bin << shift;
        mask |= 255u << shift;
        __syncwarp();
    }
    return prefix;
}

__global__ void __launch_bounds__(256) row_rank_kernel(const RowRankParams p) {
    extern __shared__ uint32_t smem_u32[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t cell = (int64_t)blockIdx.x * 8 + warp;
    if (cell >= (int64_t)p.B * p.H * p.S) return;   // warp-uniform
    uint32_t *keys = smem_u32 + warp * (p.NB + 256);
    uint32_t *hist = keys + p.NB;
    const int r = (int)(cell % p.S);
    const int own = r / 64;
    const int nvis = own + 1;                       // blocks that start at or before row r
    const float *row = p.rs + cell * p.NB;
    for (int j = lane; j < nvis; j += 32) keys[j] = ordered_key(row[j]);
    __syncwarp();
    // top k_bud: every key above the k_bud-th largest, then the equal ones in block order
    uint32_t theta = 0;
    int need_eq = 0;
    const bool all = nvis <= p.k_bud;
    if (!all) {
        theta = warp_kth_largest(keys, nvis, p.k_bud, hist);
        int gt = 0;
        for (int j = lane; j < nvis; j += 32) gt += keys[j] > theta;
        for (int off = 16; off > 0; off >>= 1) gt += __shfl_xor_sync(0xffffffffu, gt, off);
        need_eq = p.k_bud - gt;
    }
    uint32_t *out = p.keep + cell * p.NBW;
    int eq_seen = 0;
    for (int w0 = 0; w0 < p.NBW; w0 += 32) {
        // lane l assembles word w0 + l from 32 ballots (one per bit position)
        uint32_t mine = 0;
        for (int bit = 0; bit < 32; ++bit) {
            const int jb = (w0 + bit) * 32;   // first block of word w0 + bit
            const int j = jb + lane;
            bool kept = false, eq = false;
            if (j < nvis) {
                const uint32_t u = keys[j];
                eq = !all && u == theta;
                kept = all || u > theta;
            }
            const unsigned eqm = __ballot_sync(0xffffffffu, eq);
            if (eq && eq_seen + __popc(eqm & ((1u << lane) - 1u)) < need_eq) kept = true;
            eq_seen += __popc(eqm);
            if (j == 0 || j == own) kept = true;
            const unsigned km = __ballot_sync(0xffffffffu, kept);
            if (lane == bit) mine = km;
        }
        if (w0 + lane < p.NBW) out[w0 + lane] = mine;
    }
    if (p.router && nvis <= p.k_eff && lane == 0) p.sigma[cell] = __int_as_float(0x7fc00000);   // ineligible
    if (p.router && nvis > p.k_eff) {
        uint32_t top = 0;
        for (int j = lane; j < nvis; j += 32) top = max(top, keys[j]);
        for (int off = 16; off > 0; off >>= 1) top = max(top, __shfl_xor_sync(0xffffffffu, top, off));
        const uint32_t u1 = warp_kth_largest(keys, nvis, p.k_eff, hist);       // s[k_eff - 1]
        const uint32_t u2 = warp_kth_largest(keys, nvis, p.k_eff + 1, hist);   // s[k_eff]
        if (lane == 0) {
            const float s_top = key_value(top), s_km1 = key_value(u1), s_k = key_value(u2);
            float spread = __fsub_rn(s_top, s_k);
            if (spread < 1e-6f) spread = 1e-6f;   // clamp(min=1e-6); NaN passes through
            p.sigma[cell] = __fdiv_rn(__fsub_rn(s_km1, s_k), spread);
        }
    }
}

struct RowQuantParams {
    int B, H, S, row_grain, mode_quantile, k_eff;
    int64_t kq;           // 0: no threshold (no eligible cell)
    float tau;
    const float *sigma;   // [B,H,S]
    float *m_safe;        // [B*S] (row grain) or [B*H*S]
    float *thresh;
};

__device__ __forceinline__ uint32_t asc_key_rows(float v) {
    if (v != v) return 0xffffffffu;
    v = __fadd_rn(v, 0.0f);
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(1024) rows_quantile_kernel(const RowQuantParams p) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int64_t s_k;
    const int tid = threadIdx.x;
    const int64_t n = p.row_grain ? (int64_t)p.B * p.S : (int64_t)p.B * p.H * p.S;
    for (int64_t i = tid; i < n; i += blockDim.x) {
        const int r = (int)(i % p.S);
        float m;
        if (p.row_grain) {
            const int64_t b = i / p.S;
            float acc = 0.f;
            for (int h = 0; h < p.H; ++h) acc = __fadd_rn(acc, p.sigma[(b * p.H + h) * p.S + r]);
            m = __fdiv_rn(acc, (float)p.H);
        } else {
            m = p.sigma[i];
        }
        const bool elig = (r / 64 + 1) > p.k_eff;
        p.m_safe[i] = (elig && m == m) ? m : INFINITY;
    }
    __syncthreads();
    if (!p.mode_quantile) {
        if (tid == 0) p.thresh[0] = p.tau;
        return;
    }
    if (p.kq <= 0) {
        if (tid == 0) p.thresh[0] = __int_as_float(0x7fc00000);
        return;
    }
    if (tid == 0) {
        s_k = p.kq;
        s_prefix = 0;
        s_mask = 0;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int64_t i = tid; i < n; i += blockDim.x) {
            const uint32_t u = asc_key_rows(p.m_safe[i]);
            if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int64_t k = s_k;
            uint32_t bin = 0;
            for (; bin < 256; ++bin) {
                if ((int64_t)hist[bin] >= k) break;
                k -= hist[bin];
            }
            if (bin > 255) bin = 255;
            s_k = k;
            s_prefix = prefix | (bin << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    if (tid == 0) {
        const uint32_t u = s_prefix;
        p.thresh[0] = (u == 0xffffffffu) ? __int_as_float(0x7fc00000)
                                         : __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
    }
}

struct RowFinParams {
    int B, H, S, NBW, row_grain, mode_quantile, router;
    const float *m_safe, *thresh, *sigma_cells;
    uint32_t *keep;
    float *sigma_out;       // margin after the grain step (NaN for ineligible rows' raw values as computed)
    uint8_t *trigger_out;
};

__global__ void __launch_bounds__(256) rows_finalize_kernel(const RowFinParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t cell = (int64_t)blockIdx.x * 8 + warp;
    if (cell >= (int64_t)p.B * p.H * p.S) return;
    const int r = (int)(cell % p.S);
    bool unc = false;
    float eff = __int_as_float(0x7fc00000);
    if (p.router) {
        const int64_t i = p.row_grain ? (cell / ((int64_t)p.H * p.S)) * p.S + r : cell;
        const float m = p.m_safe[i];
        const float th = p.thresh[0];
        unc = p.mode_quantile ? (m <= th) : (m < th);   // ineligible cells hold +inf
        eff = m;
        if (unc) {   // every visible block
            const int own = r / 64;
            uint32_t *out = p.keep + cell * p.NBW;
            for (int w = lane; w < p.NBW; w += 32) {
                const int lo = 32 * w;
                uint32_t v = 0;
                if (own >= lo + 31) v = 0xffffffffu;
                else if (own >= lo) v = (uint32_t)((2ull << (own - lo)) - 1ull);
                out[w] = v;
            }
        }
    }
    if (lane == 0) {
        if (p.sigma_out) p.sigma_out[cell] = eff;
        if (p.trigger_out) p.trigger_out[cell] = unc ? 1 : 0;
    }
}

struct RowTileParams {
    int B, H, S, NB, NBW, Qt;
    const uint32_t *keep;   // [B,H,S,NBW]
    int32_t *kv_idx;        // [B,H,Qt,NB]
};

__global__ void __launch_bounds__(256) rows_to_tiles_kernel(const RowTileParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tcell = (int64_t)blockIdx.x * 8 + warp;
    if (tcell >= (int64_t)p.B * p.H * p.Qt) return;
    const int t = (int)(tcell % p.Qt);
    const int64_t bh = tcell / p.Qt;
    const uint32_t *rows = p.keep + (bh * p.S + (int64_t)t * 64) * p.NBW;
    const int nrows = min(64, p.S - t * 64);
    int32_t *out = p.kv_idx + tcell * p.NB;
    int n = 0;
    for (int w0 = 0; w0 < p.NBW; w0 += 32) {
        const int w = w0 + lane;
        uint32_t u = 0;
        if (w < p.NBW)
            for (int rr = 0; rr < nrows; ++rr) u |= __ldg(rows + (int64_t)rr * p.NBW + w);
        const int c = __popc(u);
        int incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        int pos = n + incl - c;
        while (u) {
            const int bit = __ffs(u) - 1;
            u &= u - 1u;
            out[pos++] = 32 * w + bit;
        }
        n += __shfl_sync(0xffffffffu, incl, 31);
    }
    for (int j = n + lane; j < p.NB; j += 32) out[j] = p.NB;
}

__global__ void __launch_bounds__(256) keep_pack_kernel(const uint8_t *__restrict__ keep, int64_t nrows, int NB,
                                                        int NBW, uint32_t *__restrict__ bits) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nrows * NBW) return;
    const int64_t row = i / NBW;
    const int w = (int)(i % NBW);
    const uint8_t *k = keep + row * NB;
    uint32_t v = 0;
    for (int b = 0; b < 32; ++b) {
        const int j = 32 * w + b;
        if (j < NB && k[j]) v |= 1u << b;
    }
    bits[i] = v;
}

}  // namespace

// ---------------------------------------------------------------- host
static int64_t al256r(int64_t x) { return (x + 255) / 256 * 256; }

// workspace: [row scores B*H*S*NB fp32][sigma cells B*H*S][m_safe B*H*S][thresh]
size_t select_rows_workspace_bytes(int B, int Hq, int S) {
    const int64_t NB = (S + 63) / 64;
    const int64_t cells = (int64_t)B * Hq * S;
    return (size_t)(al256r(cells * NB * 4) + 2 * al256r(cells * 4) + 256);
}

void rows_budget(const ugbsa_selector_config *cfg, int NB, int *k_bud, int *k_eff) {
    int kb = cfg->budget_blocks < cfg->k_max ? cfg->budget_blocks : cfg->k_max;
    kb = kb > cfg->k_min ? kb : cfg->k_min;
    *k_bud = kb < NB ? kb : NB;
    int ke = cfg->budget_blocks < NB - 1 ? cfg->budget_blocks : NB - 1;
    *k_eff = ke < 1 ? 1 : ke;
}

int launch_select_rows(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                       int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg,
                       uint32_t *keep_bits, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace,
                       cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    const int NBW = (NB + 31) / 32;
    const int64_t cells = (int64_t)B * Hq * S;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *rs = reinterpret_cast<float *>(ws);
    float *sig = reinterpret_cast<float *>(ws + al256r(cells * NB * 4));
    float *msafe = reinterpret_cast<float *>(ws + al256r(cells * NB * 4) + al256r(cells * 4));
    float *thresh = reinterpret_cast<float *>(ws + al256r(cells * NB * 4) + 2 * al256r(cells * 4));
    const bool quest = (cfg->mode == UGBSA_MODE_QUEST) ||
                       (cfg->mode == UGBSA_MODE_ROUTER && cfg->router_score == UGBSA_SCORE_QUEST);
    const bool router = cfg->mode == UGBSA_MODE_ROUTER;
    int rc = launch_row_scores(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, scale, quest, rs, stream);
    if (rc != UGBSA_OK) return rc;
    int k_bud, k_eff;
    rows_budget(cfg, NB, &k_bud, &k_eff);
    RowRankParams rp;
    rp.B = B; rp.H = Hq; rp.S = S; rp.NB = NB; rp.NBW = NBW;
    rp.k_bud = k_bud; rp.k_eff = k_eff; rp.router = router ? 1 : 0;
    rp.rs = rs; rp.keep = keep_bits; rp.sigma = sig;
    const size_t smem = (size_t)8 * (NB + 256) * 4;
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    if (cudaFuncSetAttribute(row_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    const int64_t grid = (cells + 7) / 8;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    row_rank_kernel<<<(unsigned)grid, 256, smem, stream>>>(rp);
    if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    const bool row_grain = cfg->router_grain == UGBSA_GRAIN_ROW;
    const bool mode_q = cfg->router_mode == UGBSA_ROUTER_QUANTILE;
    if (router) {
        RowQuantParams qp;
        qp.B = B; qp.H = Hq; qp.S = S; qp.row_grain = row_grain ? 1 : 0; qp.mode_quantile = mode_q ? 1 : 0;
        qp.k_eff = k_eff;
        // eligible rows: more than k_eff visible blocks, i.e. r >= 64 * k_eff; the row-grain
        // count is of rows (the reference sums a [1, 1, S] mask, :331-335)
        const int64_t elig_rows = S > 64 * (int64_t)k_eff ? S - 64 * (int64_t)k_eff : 0;
        const int64_t n_elig = row_grain ? elig_rows : (int64_t)B * Hq * elig_rows;
        int64_t kq = n_elig > 0 ? (int64_t)(cfg->router_quantile * (double)n_elig) : 0;
        if (n_elig > 0 && kq < 1) kq = 1;
        qp.kq = kq;
        qp.tau = (float)cfg->router_tau;
        qp.sigma = sig; qp.m_safe = msafe; qp.thresh = thresh;
        rows_quantile_kernel<<<1, 1024, 0, stream>>>(qp);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    if (router || sigma_out || trigger_out) {
        RowFinParams fp;
        fp.B = B; fp.H = Hq; fp.S = S; fp.NBW = NBW;
        fp.row_grain = row_grain ? 1 : 0; fp.mode_quantile = mode_q ? 1 : 0; fp.router = router ? 1 : 0;
        fp.m_safe = msafe; fp.thresh = thresh; fp.sigma_cells = sig;
        fp.keep = keep_bits; fp.sigma_out = sigma_out; fp.trigger_out = trigger_out;
        rows_finalize_kernel<<<(unsigned)grid, 256, 0, stream>>>(fp);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    if (kv_idx) return launch_rows_to_tiles(keep_bits, B, Hq, S, kv_idx, stream);
    return UGBSA_OK;
}

int launch_rows_to_tiles(const uint32_t *keep_bits, int B, int H, int S, int32_t *kv_idx, cudaStream_t stream) {
    RowTileParams tp;
    tp.B = B; tp.H = H; tp.S = S; tp.NB = (S + 63) / 64; tp.NBW = (tp.NB + 31) / 32; tp.Qt = tp.NB;
    tp.keep = keep_bits; tp.kv_idx = kv_idx;
    const int64_t tiles = (int64_t)B * H * tp.Qt;
    rows_to_tiles_kernel<<<(unsigned)((tiles + 7) / 8), 256, 0, stream>>>(tp);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_keep_pack(const uint8_t *keep, int B, int H, int S, int NB, uint32_t *bits, cudaStream_t stream) {
    const int NBW = (NB + 31) / 32;
    const int64_t n = (int64_t)B * H * S * NBW;
    if (n <= 0) return UGBSA_OK;
    keep_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(keep, (int64_t)B * H * S, NB, NBW, bits);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

}  // namespace ugbsa
