/*
 * ugbsa_oracle.c -- CPU restatement of the uncertainty-gated block-sparse
 * attention prefill path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the CUDA library and
 * the Python host package) links, loads or calls this file.  It is the checker
 * used by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg.
 *
 * It restates, in plain C, the reference's v2 selector
 *   src/sparse_attention.py:588-748  (_block_select_kv_idx_v2)
 * and its block-sparse attention semantics
 *   src/triton_block_attn.py:184-264 (_fwd_kernel_v2)
 *   src/triton_block_attn.py:301-312 (reference_attn, masked SDPA).
 *
 * Canonical arithmetic order (the reference's torch reductions have no fixed
 * order; this file fixes one, and the CUDA kernels follow the same one so the
 * GPU can be compared bit for bit):
 *   block mean   m[d]  = (((0 + k0[d]) + k1[d]) + ... + k63[d]) / 64     (rows past
 *                        S are the reference's zero padding, :617-625)
 *   Quest env    min/max over the 64 rows, zero padding rows included    (:636-637)
 *   mean score   s     = fl(dot * scale), dot = fmaf chain over d = 0..D-1 (:647-648)
 *   Quest score  s     = fl(fl(dp + dn) * scale), dp = fmaf chain of
 *                        max(q,0)*Kmax, dn = fmaf chain of min(q,0)*Kmin   (:638-642)
 *   tile score   max over the 64 rows of the tile; padded query rows score 0 (:655-656)
 *   ranking      descending value, ties broken by lower block index (a stable
 *                descending sort; torch.topk's tie order is unspecified)  (:697-698)
 *   sigma        fl(fl(s[kb-1]-s[kb]) / clamp(fl(s[0]-s[kb]), 1e-6f))      (:700-707)
 *   row grain    fl(sum over heads in order h = 0..H-1) / H                (:708-710)
 *   quantile     k-th smallest of the expanded [B,H,Qt] array, NaN last    (:711-718)
 * IEEE division and subnormals are kept (sigma is subnormal by construction).
 */
#include <float.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BLK 64

static inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

/* Threads of the oracle's parallel regions (a process launched under torchrun
 * inherits OMP_NUM_THREADS=1; the CPU baseline asks for every host core). */
void oracle_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int oracle_get_threads(void) { return omp_get_max_threads(); }

/* -------------------------------------------------------------------------- */
/* Block summaries: sparse_attention.py:617-646                                */
/* K is addressed as K[b*sb + h*sh + s*ss + d*sd] (element strides).          */
/* mean mode: out_a = mean [B,Hkv,NB,D]; quest mode: out_a = min, out_b = max */
/* -------------------------------------------------------------------------- */
int oracle_block_summary(const float *K, int64_t sb, int64_t sh, int64_t ss, int64_t sd,
                         int B, int Hkv, int S, int D, int quest,
                         float *out_a, float *out_b) {
    if (B <= 0 || Hkv <= 0 || S <= 0 || D <= 0) return 1;
    const int NB = (int)cdiv64(S, BLK);
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < Hkv; ++h)
            for (int nb = 0; nb < NB; ++nb) {
                float *oa = out_a + (((int64_t)b * Hkv + h) * NB + nb) * D;
                float *ob = quest ? out_b + (((int64_t)b * Hkv + h) * NB + nb) * D : NULL;
                for (int d = 0; d < D; ++d) {
                    float acc = 0.0f, mn = 0.0f, mx = 0.0f;
                    for (int r = 0; r < BLK; ++r) {
                        const int s = nb * BLK + r;
                        const float x = (s < S) ? K[b * sb + h * sh + (int64_t)s * ss + d * sd] : 0.0f;
                        if (quest) {
                            if (r == 0) { mn = x; mx = x; }
                            else { mn = (x < mn) ? x : mn; mx = (x > mx) ? x : mx; }
                        } else {
                            acc = acc + x;
                        }
                    }
                    if (quest) { oa[d] = mn; ob[d] = mx; }
                    else oa[d] = acc / 64.0f;
                }
            }
    return 0;
}

/* -------------------------------------------------------------------------- */
/* Tile scores: sparse_attention.py:638-666.                                   */
/* ts[B,Hq,Qt,NB]: max over the tile's rows of the per-row block score for the */
/* causally visible blocks (64*blk <= min(64t+63, S-1)); -inf elsewhere.      */
/* GQA: Q head h reads summaries of KV head h / (Hq/Hkv) (repeat_kv, :761).    */
/* -------------------------------------------------------------------------- */
int oracle_tile_scores_range(const float *Q, int64_t sb, int64_t sh, int64_t ss, int64_t sd,
                             const float *summ_a, const float *summ_b,
                             int B, int Hq, int Hkv, int S, int D, float scale, int quest,
                             int t_begin, int t_end, float *ts) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return 1;
    const int NB = (int)cdiv64(S, BLK);
    const int Qt = NB;
    if (t_begin < 0) t_begin = 0;
    if (t_end > Qt) t_end = Qt;
    const int G = Hq / Hkv;
    /* per (b, h): transposed summaries sT[d][blk] so the inner loop runs over
     * blocks, then the tiles in parallel (each (row, block) chain is the same
     * sequence of fmaf whichever thread runs it) */
    float *sa = (float *)malloc(sizeof(float) * (size_t)D * NB);
    float *sbT = quest ? (float *)malloc(sizeof(float) * (size_t)D * NB) : NULL;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < Hq; ++h) {
            const int kvh = h / G;
            const float *A = summ_a + ((int64_t)b * Hkv + kvh) * NB * D;
            const float *Bm = quest ? summ_b + ((int64_t)b * Hkv + kvh) * NB * D : NULL;
#pragma omp parallel for schedule(static)
            for (int nb = 0; nb < NB; ++nb)
                for (int d = 0; d < D; ++d) {
                    sa[(size_t)d * NB + nb] = A[(int64_t)nb * D + d];
                    if (quest) sbT[(size_t)d * NB + nb] = Bm[(int64_t)nb * D + d];
                }
#pragma omp parallel
            {
                float *acc = (float *)malloc(sizeof(float) * NB);
                float *acc2 = (float *)malloc(sizeof(float) * NB);
                float *qp = (float *)malloc(sizeof(float) * D);
                float *qn = (float *)malloc(sizeof(float) * D);
#pragma omp for schedule(dynamic)
                for (int t = t_begin; t < t_end; ++t) {
                    float *row = ts + (((int64_t)b * Hq + h) * Qt + t) * NB;
                    int last = t * BLK + BLK - 1;
                    if (last > S - 1) last = S - 1;
                    const int nvis = last / BLK + 1;
                    for (int j = 0; j < NB; ++j) row[j] = -INFINITY;
                    for (int r = t * BLK; r < t * BLK + BLK; ++r) {
                        if (r >= S) {
                            /* zero-padded query row scores exactly 0 (F.pad, :623-625) */
                            for (int j = 0; j < nvis; ++j) row[j] = (0.0f > row[j]) ? 0.0f : row[j];
                            continue;
                        }
                        const float *q = Q + b * sb + h * sh + (int64_t)r * ss;
                        for (int d = 0; d < D; ++d) {
                            float x = q[d * sd];
                            qp[d] = x > 0.0f ? x : 0.0f;
                            qn[d] = x < 0.0f ? x : 0.0f;
                        }
                        for (int j = 0; j < nvis; ++j) { acc[j] = 0.0f; acc2[j] = 0.0f; }
                        if (!quest) {
                            for (int d = 0; d < D; ++d) {
                                const float qd = q[d * sd];
                                const float *col = sa + (size_t)d * NB;
                                for (int j = 0; j < nvis; ++j) acc[j] = fmaf(qd, col[j], acc[j]);
                            }
                            for (int j = 0; j < nvis; ++j) {
                                float s = acc[j] * scale;
                                row[j] = (s > row[j]) ? s : row[j];
                            }
                        } else {
                            /* summ_a = Kmin, summ_b = Kmax */
                            for (int d = 0; d < D; ++d) {
                                const float *cmin = sa + (size_t)d * NB;
                                const float *cmax = sbT + (size_t)d * NB;
                                const float p = qp[d], n = qn[d];
                                for (int j = 0; j < nvis; ++j) {
                                    acc[j] = fmaf(p, cmax[j], acc[j]);
                                    acc2[j] = fmaf(n, cmin[j], acc2[j]);
                                }
                            }
                            for (int j = 0; j < nvis; ++j) {
                                float s = (acc[j] + acc2[j]) * scale;
                                row[j] = (s > row[j]) ? s : row[j];
                            }
                        }
                    }
                }
                free(acc); free(acc2); free(qp); free(qn);
            }
        }
    free(sa); free(sbT);
    return 0;
}

int oracle_tile_scores(const float *Q, int64_t sb, int64_t sh, int64_t ss, int64_t sd,
                       const float *summ_a, const float *summ_b,
                       int B, int Hq, int Hkv, int S, int D, float scale, int quest,
                       float *ts) {
    return oracle_tile_scores_range(Q, sb, sh, ss, sd, summ_a, summ_b, B, Hq, Hkv, S, D, scale, quest,
                                    0, (int)cdiv64(S, BLK), ts);
}

/* -------------------------------------------------------------------------- */
/* Selection from tile scores: sparse_attention.py:660-725                     */
/* -------------------------------------------------------------------------- */
typedef struct {
    int mode;          /* 0 topk, 1 quest, 2 router      (Selector.mode, :58)            */
    int router_mode;   /* 0 abs, 1 quantile              (Selector.router_mode, :80)     */
    int router_grain;  /* 0 cell, 1 row                  (Selector.router_grain, :81)    */
    double router_quantile; /*                           (Selector.router_quantile, :83) */
    double router_tau;      /*                           (Selector.router_tau, :82)      */
    int budget_blocks, k_min, k_max; /*                  (:59, :61)                      */
} oracle_cfg;

/* budget arithmetic, sparse_attention.py:688-695 */
void oracle_budget(const oracle_cfg *c, int NB, int *k_base, int *kmax) {
    int kb_row = c->budget_blocks < c->k_max ? c->budget_blocks : c->k_max;
    kb_row = kb_row > c->k_min ? kb_row : c->k_min;
    int kb = 2 * kb_row < NB ? 2 * kb_row : NB;
    int km = kb;
    if (c->mode == 2) km = 2 * kb < NB ? 2 * kb : NB;
    *k_base = kb;
    *kmax = km;
}

typedef struct { float v; int i; } vi_t;

/* descending by value, NaN first (torch sorts NaN as the largest), ties -> lower index */
static int cmp_desc(const void *a, const void *b) {
    const vi_t *x = (const vi_t *)a, *y = (const vi_t *)b;
    const int xn = isnan(x->v), yn = isnan(y->v);
    if (xn != yn) return xn ? -1 : 1;
    if (!xn) {
        if (x->v > y->v) return -1;
        if (x->v < y->v) return 1;
    }
    return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* ascending, NaN last (torch.kthvalue), ties arbitrary (values equal) */
static int cmp_asc_nanlast(const void *a, const void *b) {
    const float x = *(const float *)a, y = *(const float *)b;
    const int xn = isnan(x), yn = isnan(y);
    if (xn != yn) return xn ? 1 : -1;
    if (xn) return 0;
    return (x < y) ? -1 : (x > y);
}

/*
 * ts          [B,H,Qt,NB] raw tile scores (only the visible entries are read).
 * kv_idx      [B,H,Qt,kmax] int32 out.
 * sigma       [B,H,Qt] out (per-cell margin; NaN when not computed) -- may be NULL.
 * sigma_eff   [B,H,Qt] out (margin after the grain step) -- may be NULL.
 * trig        [B,H,Qt] out (1 = tile got the doubled budget) -- may be NULL.
 * thresh_out  scalar out (quantile threshold, or fp32(tau) in abs mode) -- may be NULL.
 * Returns 0, or 1 on bad arguments.
 */
int oracle_select_from_scores(const float *ts, int B, int H, int S, const oracle_cfg *c,
                              int32_t *kv_idx, float *sigma, float *sigma_eff,
                              uint8_t *trig, float *thresh_out) {
    if (B <= 0 || H <= 0 || S <= 0) return 1;
    const int NB = (int)cdiv64(S, BLK);
    const int Qt = NB;
    int kb, km;
    oracle_budget(c, NB, &kb, &km);
    const int router = (c->mode == 2) && (kb < km);
    const int64_t ncell = (int64_t)B * H * Qt;
    float *sig = (float *)malloc(sizeof(float) * (size_t)ncell);
    int32_t *idx_all = (int32_t *)malloc(sizeof(int32_t) * (size_t)ncell * km);

#pragma omp parallel for schedule(dynamic)
    for (int64_t cell = 0; cell < ncell; ++cell) {
        const int t = (int)(cell % Qt);
        const float *row = ts + cell * NB;
        vi_t *a = (vi_t *)malloc(sizeof(vi_t) * NB);
        int last = t * BLK + BLK - 1;
        if (last > S - 1) last = S - 1;
        const int self_blk = last / BLK;
        for (int j = 0; j < NB; ++j) {
            float v = (j * BLK <= last) ? row[j] : -INFINITY;  /* :660-666 */
            v = v + 0.0f;                                      /* -0 -> +0 */
            a[j].v = v;
            a[j].i = j;
        }
        a[0].v = FLT_MAX;          /* :679 */
        a[self_blk].v = FLT_MAX;   /* :680-684 */
        qsort(a, NB, sizeof(vi_t), cmp_desc);
        for (int j = 0; j < km; ++j) idx_all[cell * km + j] = a[j].i;
        float s = NAN;
        if (router) {
            const float s_top = a[0].v, s_km1 = a[kb - 1].v, s_k = a[kb].v;
            float spread = s_top - s_k;
            if (spread < 1e-6f) spread = 1e-6f;   /* clamp(min=1e-6); NaN passes through */
            s = (s_km1 - s_k) / spread;
        }
        sig[cell] = s;
        free(a);
    }

    float thresh = NAN;
    uint8_t *unc = (uint8_t *)calloc((size_t)ncell, 1);
    float *eff = (float *)malloc(sizeof(float) * (size_t)ncell);
    if (router) {
        if (c->router_grain == 1) {
            for (int b = 0; b < B; ++b)
                for (int t = 0; t < Qt; ++t) {
                    float acc = 0.0f;
                    for (int h = 0; h < H; ++h) acc = acc + sig[((int64_t)b * H + h) * Qt + t];
                    const float m = acc / (float)H;
                    for (int h = 0; h < H; ++h) eff[((int64_t)b * H + h) * Qt + t] = m;
                }
        } else {
            memcpy(eff, sig, sizeof(float) * (size_t)ncell);
        }
        if (c->router_mode == 1) {
            int64_t kq = (int64_t)(c->router_quantile * (double)ncell);
            if (kq < 1) kq = 1;
            if (c->router_grain == 1) {
                /* each row value appears H times in the expanded array */
                const int64_t n = (int64_t)B * Qt;
                float *v = (float *)malloc(sizeof(float) * (size_t)n);
                for (int b = 0; b < B; ++b)
                    for (int t = 0; t < Qt; ++t) v[(int64_t)b * Qt + t] = eff[((int64_t)b * H) * Qt + t];
                qsort(v, n, sizeof(float), cmp_asc_nanlast);
                thresh = v[(kq - 1) / H];
                free(v);
            } else {
                float *v = (float *)malloc(sizeof(float) * (size_t)ncell);
                memcpy(v, eff, sizeof(float) * (size_t)ncell);
                qsort(v, ncell, sizeof(float), cmp_asc_nanlast);
                thresh = v[kq - 1];
                free(v);
            }
            for (int64_t i = 0; i < ncell; ++i) unc[i] = (eff[i] <= thresh);
        } else {
            thresh = (float)c->router_tau;
            for (int64_t i = 0; i < ncell; ++i) unc[i] = (eff[i] < thresh);
        }
    } else {
        for (int64_t i = 0; i < ncell; ++i) eff[i] = NAN;
    }

    for (int64_t cell = 0; cell < ncell; ++cell)
        for (int j = 0; j < km; ++j) {
            int32_t v = idx_all[cell * km + j];
            if (router && j >= kb && !unc[cell]) v = NB;  /* :720-725 */
            kv_idx[cell * km + j] = v;
        }
    if (sigma) memcpy(sigma, sig, sizeof(float) * (size_t)ncell);
    if (sigma_eff) memcpy(sigma_eff, eff, sizeof(float) * (size_t)ncell);
    if (trig) memcpy(trig, unc, (size_t)ncell);
    if (thresh_out) *thresh_out = thresh;
    free(sig); free(idx_all); free(unc); free(eff);
    return 0;
}

/* Per-tile ranking and sigma for tiles [t_begin, t_end) of every (b, h): the
 * per-tile part of oracle_select_from_scores (used to time a bounded sample). */
int oracle_rank_tiles_range(const float *ts, int B, int H, int S, const oracle_cfg *c, int t_begin, int t_end,
                            int32_t *kv_idx, float *sigma) {
    const int NB = (int)cdiv64(S, BLK);
    const int Qt = NB;
    int kb, km;
    oracle_budget(c, NB, &kb, &km);
    const int router = (c->mode == 2) && (kb < km);
    if (t_begin < 0) t_begin = 0;
    if (t_end > Qt) t_end = Qt;
    const int nt = t_end - t_begin;
    if (nt <= 0) return 0;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int bh = 0; bh < B * H; ++bh)
        for (int tt = 0; tt < nt; ++tt) {
            const int t = t_begin + tt;
            const int64_t cell = (int64_t)bh * Qt + t;
            const float *row = ts + cell * NB;
            vi_t *a = (vi_t *)malloc(sizeof(vi_t) * NB);
            int last = t * BLK + BLK - 1;
            if (last > S - 1) last = S - 1;
            const int self_blk = last / BLK;
            for (int j = 0; j < NB; ++j) {
                a[j].v = ((j * BLK <= last) ? row[j] : -INFINITY) + 0.0f;
                a[j].i = j;
            }
            a[0].v = FLT_MAX;
            a[self_blk].v = FLT_MAX;
            qsort(a, NB, sizeof(vi_t), cmp_desc);
            for (int j = 0; j < km; ++j) kv_idx[cell * km + j] = a[j].i;
            float sg = NAN;
            if (router) {
                float spread = a[0].v - a[kb].v;
                if (spread < 1e-6f) spread = 1e-6f;
                sg = (a[kb - 1].v - a[kb].v) / spread;
            }
            sigma[cell] = sg;
            free(a);
        }
    return 0;
}

/* -------------------------------------------------------------------------- */
/* Block-sparse attention: semantics of triton_block_attn.py:184-264.          */
/* Every slot of kv_idx[b,h,t,:] is visited in order; a slot is skipped when it */
/* holds the sentinel (>= NB) or its block starts after the tile's last row    */
/* (:231-233).  Inside a block, key n is used by row m iff n <= m and n < Sk    */
/* (:243-246).  Accumulation is in double; rows with no usable key give 0      */
/* (:261).  Q [B,Hq,Sq,D], K/V [B,Hkv,Sk,D] (strided), out [B,Hq,Sq,D] dense.  */
/* -------------------------------------------------------------------------- */
int oracle_attn_range(const float *Q, int64_t qb, int64_t qh, int64_t qs, int64_t qd,
                      const float *K, int64_t kb_, int64_t kh, int64_t ks, int64_t kd,
                      const float *V, int64_t vb, int64_t vh, int64_t vs, int64_t vd,
                      const int32_t *kv_idx, int kmax,
                      int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale,
                      int t_begin, int t_end, float *out) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || D <= 0 || Hq % Hkv || kmax <= 0) return 1;
    const int NB = (int)cdiv64(Sk, BLK);
    const int Qt = (int)cdiv64(Sq, BLK);
    const int G = Hq / Hkv;
    if (t_begin < 0) t_begin = 0;
    if (t_end > Qt) t_end = Qt;
    const int nt = t_end - t_begin;
    if (nt <= 0) return 0;
    /* one query row per iteration: (b, h, tile, row within the tile) */
    const int64_t nrows = (int64_t)B * Hq * nt * BLK;
#pragma omp parallel
    {
        double *logit = (double *)malloc(sizeof(double) * (size_t)kmax * BLK);
        int *keyn = (int *)malloc(sizeof(int) * (size_t)kmax * BLK);
        double *acc = (double *)malloc(sizeof(double) * D);
#pragma omp for schedule(dynamic, 16)
        for (int64_t it = 0; it < nrows; ++it) {
            const int rr = (int)(it % BLK);
            const int t = t_begin + (int)((it / BLK) % nt);
            const int h = (int)((it / ((int64_t)BLK * nt)) % Hq);
            const int b = (int)(it / ((int64_t)BLK * nt * Hq));
            const int m = t * BLK + rr;
            if (m >= Sq) continue;
            const int kvh = h / G;
            const int32_t *slots = kv_idx + (((int64_t)b * Hq + h) * Qt + t) * kmax;
            const int tile_last = t * BLK + BLK - 1;
            const float *q = Q + b * qb + h * qh + (int64_t)m * qs;
            int n_used = 0;
            double mx = -INFINITY;
            for (int j = 0; j < kmax; ++j) {
                const int blk = slots[j];
                if (blk < 0 || blk >= NB) continue;
                if (blk * BLK > tile_last) continue;
                for (int c = 0; c < BLK; ++c) {
                    const int n = blk * BLK + c;
                    if (n >= Sk || n > m) continue;
                    const float *k = K + b * kb_ + kvh * kh + (int64_t)n * ks;
                    double dot = 0.0;
                    for (int d = 0; d < D; ++d) dot += (double)q[d * qd] * (double)k[d * kd];
                    dot *= (double)scale;
                    logit[n_used] = dot;
                    keyn[n_used] = n;
                    ++n_used;
                    if (dot > mx) mx = dot;
                }
            }
            float *o = out + (((int64_t)b * Hq + h) * Sq + m) * D;
            if (n_used == 0) {
                for (int d = 0; d < D; ++d) o[d] = 0.0f;
                continue;
            }
            double l = 0.0;
            for (int d = 0; d < D; ++d) acc[d] = 0.0;
            for (int u = 0; u < n_used; ++u) {
                const double p = exp(logit[u] - mx);
                l += p;
                const float *v = V + b * vb + kvh * vh + (int64_t)keyn[u] * vs;
                for (int d = 0; d < D; ++d) acc[d] += p * (double)v[d * vd];
            }
            for (int d = 0; d < D; ++d) o[d] = (float)(acc[d] / l);
        }
        free(logit); free(keyn); free(acc);
    }
    return 0;
}

int oracle_attn(const float *Q, int64_t qb, int64_t qh, int64_t qs, int64_t qd,
                const float *K, int64_t kb_, int64_t kh, int64_t ks, int64_t kd,
                const float *V, int64_t vb, int64_t vh, int64_t vs, int64_t vd,
                const int32_t *kv_idx, int kmax,
                int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale,
                float *out) {
    return oracle_attn_range(Q, qb, qh, qs, qd, K, kb_, kh, ks, kd, V, vb, vh, vs, vd, kv_idx, kmax,
                             B, Hq, Hkv, Sq, Sk, D, scale, 0, (int)cdiv64(Sq, BLK), out);
}

/*
 * Decode scores: the exact fp32 score of one query row per (b, head) against
 * every block summary, in the canonical order above (the row sits at position
 * S-1, so every block is visible; no tile max, no padded rows).  q [B, Hq, D]
 * with element strides (qb, qh, qd); summaries [B, Hkv, nb_stride, D];
 * out [B, Hq, NB].  This path has no counterpart in the reference, which
 * decodes densely (src/sparse_attention.py:756-770).
 */
int oracle_decode_scores(const float *Q, int64_t qb, int64_t qh, int64_t qd, const float *summ_a,
                         const float *summ_b, int nb_stride, int B, int Hq, int Hkv, int S, int D, float scale,
                         int quest, float *out) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return 1;
    const int NB = (int)cdiv64(S, BLK);
    if (nb_stride < NB) return 1;
    const int G = Hq / Hkv;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < Hq; ++h) {
            const float *q = Q + b * qb + h * qh;
            const float *A = summ_a + ((int64_t)b * Hkv + h / G) * nb_stride * D;
            const float *Bm = quest ? summ_b + ((int64_t)b * Hkv + h / G) * nb_stride * D : NULL;
            for (int j = 0; j < NB; ++j) {
                float acc = 0.0f, acc2 = 0.0f;
                for (int d = 0; d < D; ++d) {
                    const float x = q[d * qd];
                    if (quest) {
                        acc = fmaf(x > 0.0f ? x : 0.0f, Bm[(int64_t)j * D + d], acc);
                        acc2 = fmaf(x < 0.0f ? x : 0.0f, A[(int64_t)j * D + d], acc2);
                    } else {
                        acc = fmaf(x, A[(int64_t)j * D + d], acc);
                    }
                }
                out[((int64_t)b * Hq + h) * NB + j] = quest ? (acc + acc2) * scale : acc * scale;
            }
        }
    return 0;
}

/* -------------------------------------------------------------------------- */
/* v1 per-row selection: sparse_attention.py:208-382 (_block_select_mask),    */
/* modes topk / quest / router, and the per-row keep mask of its kernel        */
/* (triton_block_attn.py:39-122).  Every query row r (Q == K, prefill) ranks   */
/* the blocks that start at or before r by its own fp32 score (the canonical   */
/* chains above, :221-239), keeps the top k_bud = clamp(budget, k_min, k_max)  */
/* (ties to the lower block id), then the sink and its own block (:281-283).   */
/* Router (:295-352): per-(head, row) margin of the RAW scores at             */
/* k_eff = clamp(budget, 1, NB-1); rows with more than k_eff visible blocks    */
/* are eligible; row grain averages over heads; quantile over the eligible    */
/* cells (ineligible and NaN as +inf, k = int(q * eligible count) where the    */
/* row-grain count is of rows, not batch x rows, :331-335); triggered cells    */
/* keep every visible block.                                                   */
/* -------------------------------------------------------------------------- */

/* rs [B,H,S,NB]: row r's score of block j, -inf where block j starts after r */
int oracle_row_scores(const float *Q, int64_t sb, int64_t sh, int64_t ss, int64_t sd,
                      const float *summ_a, const float *summ_b,
                      int B, int Hq, int Hkv, int S, int D, float scale, int quest, float *rs) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || D <= 0 || Hq % Hkv) return 1;
    const int NB = (int)cdiv64(S, BLK);
    const int G = Hq / Hkv;
#pragma omp parallel for collapse(3) schedule(dynamic, 64)
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < Hq; ++h)
            for (int r = 0; r < S; ++r) {
                const int kvh = h / G;
                const float *A = summ_a + ((int64_t)b * Hkv + kvh) * NB * D;
                const float *Bm = quest ? summ_b + ((int64_t)b * Hkv + kvh) * NB * D : NULL;
                const float *q = Q + b * sb + h * sh + (int64_t)r * ss;
                float *row = rs + (((int64_t)b * Hq + h) * S + r) * NB;
                const int nvis = r / BLK + 1;
                for (int j = 0; j < NB; ++j) {
                    if (j >= nvis) { row[j] = -INFINITY; continue; }
                    if (!quest) {
                        float acc = 0.0f;
                        for (int d = 0; d < D; ++d) acc = fmaf(q[d * sd], A[(int64_t)j * D + d], acc);
                        row[j] = acc * scale;
                    } else {
                        float ap = 0.0f, an = 0.0f;
                        for (int d = 0; d < D; ++d) {
                            const float x = q[d * sd];
                            ap = fmaf(x > 0.0f ? x : 0.0f, Bm[(int64_t)j * D + d], ap);
                            an = fmaf(x < 0.0f ? x : 0.0f, A[(int64_t)j * D + d], an);
                        }
                        row[j] = (ap + an) * scale;
                    }
                }
            }
    return 0;
}

/* keep [B,H,S,NB] uint8 out; sigma / eff [B,H,S] (NaN unless router); trig [B,H,S];
 * thresh_out: the quantile threshold (NaN when none), fp32(tau) in abs mode. */
int oracle_select_rows_from_scores(const float *rs, int B, int H, int S, const oracle_cfg *c, uint8_t *keep,
                                   float *sigma, float *eff_out, uint8_t *trig, float *thresh_out) {
    if (B <= 0 || H <= 0 || S <= 0) return 1;
    const int NB = (int)cdiv64(S, BLK);
    int kb = c->budget_blocks < c->k_max ? c->budget_blocks : c->k_max;   /* :268 */
    kb = kb > c->k_min ? kb : c->k_min;
    if (kb > NB) kb = NB;
    const int router = c->mode == 2;
    int keff = c->budget_blocks < NB - 1 ? c->budget_blocks : NB - 1;       /* :303-304 */
    if (keff < 1) keff = 1;
    const int64_t ncell = (int64_t)B * H * S;
    float *sig = (float *)malloc(sizeof(float) * (size_t)ncell);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t cell = 0; cell < ncell; ++cell) {
        const int r = (int)(cell % S);
        const float *row = rs + cell * NB;
        uint8_t *kp = keep + cell * NB;
        vi_t *a = (vi_t *)malloc(sizeof(vi_t) * NB);
        for (int j = 0; j < NB; ++j) { a[j].v = row[j] + 0.0f; a[j].i = j; }
        qsort(a, NB, sizeof(vi_t), cmp_desc);
        memset(kp, 0, (size_t)NB);
        for (int j = 0; j < kb; ++j) kp[a[j].i] = 1;
        kp[0] = 1;                 /* :282 */
        kp[r / BLK] = 1;           /* :283 */
        float s = NAN;
        if (router) {
            const float s_top = a[0].v, s_km1 = a[keff - 1].v, s_k = a[keff].v;
            float spread = s_top - s_k;
            if (spread < 1e-6f) spread = 1e-6f;
            s = (s_km1 - s_k) / spread;
        }
        sig[cell] = s;
        free(a);
    }
    float thresh = NAN;
    float *eff = (float *)malloc(sizeof(float) * (size_t)ncell);
    uint8_t *unc = (uint8_t *)calloc((size_t)ncell, 1);
    if (router) {
        const int row_grain = c->router_grain == 1;
        /* eligibility is per row: more than k_eff visible blocks */
        int64_t n_elig_rows = 0;
        for (int r = 0; r < S; ++r) n_elig_rows += (r / BLK + 1) > keff;
        for (int b = 0; b < B; ++b)
            for (int r = 0; r < S; ++r) {
                if (row_grain) {
                    float acc = 0.0f;
                    for (int h = 0; h < H; ++h) acc = acc + sig[((int64_t)b * H + h) * S + r];
                    const float m = acc / (float)H;
                    for (int h = 0; h < H; ++h) eff[((int64_t)b * H + h) * S + r] = m;
                } else {
                    for (int h = 0; h < H; ++h) eff[((int64_t)b * H + h) * S + r] = sig[((int64_t)b * H + h) * S + r];
                }
            }
        if (c->router_mode == 1) {
            /* the scored cells: [B,1,S] for row grain, [B,H,S] for cell grain */
            const int64_t n = row_grain ? (int64_t)B * S : ncell;
            const int64_t n_elig = row_grain ? n_elig_rows : (int64_t)B * H * n_elig_rows;
            float *v = (float *)malloc(sizeof(float) * (size_t)n);
            for (int64_t i = 0; i < n; ++i) {
                const int64_t src = row_grain ? ((i / S) * H) * S + (i % S) : i;
                const int r = (int)(i % S);
                const float m = eff[src];
                v[i] = ((r / BLK + 1) > keff && !isnan(m)) ? m : INFINITY;
            }
            int64_t kq = n_elig > 0 ? (int64_t)(c->router_quantile * (double)n_elig) : 0;
            if (n_elig > 0 && kq < 1) kq = 1;
            if (kq > 0) {
                float *sorted = (float *)malloc(sizeof(float) * (size_t)n);
                memcpy(sorted, v, sizeof(float) * (size_t)n);
                qsort(sorted, n, sizeof(float), cmp_asc_nanlast);
                thresh = sorted[kq - 1];
                free(sorted);
                for (int64_t cell = 0; cell < ncell; ++cell) {
                    const int r = (int)(cell % S);
                    const int64_t i = row_grain ? (cell / ((int64_t)H * S)) * S + r : cell;
                    unc[cell] = (r / BLK + 1) > keff && v[i] <= thresh;
                }
            }
            free(v);
        } else {
            thresh = (float)c->router_tau;
            for (int64_t cell = 0; cell < ncell; ++cell) {
                const int r = (int)(cell % S);
                unc[cell] = (r / BLK + 1) > keff && eff[cell] < thresh;
            }
        }
        for (int64_t cell = 0; cell < ncell; ++cell)
            if (unc[cell]) {   /* dense row: every visible block (:345-347) */
                const int r = (int)(cell % S);
                uint8_t *kp = keep + cell * NB;
                for (int j = 0; j < NB; ++j) kp[j] = (j * BLK <= r);
            }
    } else {
        for (int64_t i = 0; i < ncell; ++i) eff[i] = NAN;
    }
    if (sigma) memcpy(sigma, sig, sizeof(float) * (size_t)ncell);
    if (eff_out) memcpy(eff_out, eff, sizeof(float) * (size_t)ncell);
    if (trig) memcpy(trig, unc, (size_t)ncell);
    if (thresh_out) *thresh_out = thresh;
    free(sig); free(eff); free(unc);
    return 0;
}

/* Attention with a per-row keep mask (triton_block_attn.py:39-122): row m uses
 * key n iff keep[b,h,m,n/64], n <= m and n < Sk; float64 accumulation; rows with
 * no usable key give 0.  keep [B,Hq,Sq,NB] uint8; out [B,Hq,Sq,D] dense. */
int oracle_attn_keep(const float *Q, int64_t qb, int64_t qh, int64_t qs, int64_t qd,
                     const float *K, int64_t kb_, int64_t kh, int64_t ks, int64_t kd,
                     const float *V, int64_t vb, int64_t vh, int64_t vs, int64_t vd,
                     const uint8_t *keep, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, float *out) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || D <= 0 || Hq % Hkv) return 1;
    const int NB = (int)cdiv64(Sk, BLK);
    const int G = Hq / Hkv;
    const int64_t nrows = (int64_t)B * Hq * Sq;
#pragma omp parallel
    {
        double *logit = (double *)malloc(sizeof(double) * (size_t)Sk);
        double *acc = (double *)malloc(sizeof(double) * D);
#pragma omp for schedule(dynamic, 16)
        for (int64_t it = 0; it < nrows; ++it) {
            const int m = (int)(it % Sq);
            const int h = (int)((it / Sq) % Hq);
            const int b = (int)(it / ((int64_t)Sq * Hq));
            const int kvh = h / G;
            const uint8_t *kp = keep + it * NB;
            const float *q = Q + b * qb + h * qh + (int64_t)m * qs;
            double mx = -INFINITY;
            int n_used = 0;
            for (int n = 0; n <= m && n < Sk; ++n) {
                if (!kp[n / BLK]) { logit[n] = NAN; continue; }
                const float *k = K + b * kb_ + kvh * kh + (int64_t)n * ks;
                double dot = 0.0;
                for (int d = 0; d < D; ++d) dot += (double)q[d * qd] * (double)k[d * kd];
                dot *= (double)scale;
                logit[n] = dot;
                if (dot > mx) mx = dot;
                ++n_used;
            }
            float *o = out + it * D;
            if (n_used == 0) {
                for (int d = 0; d < D; ++d) o[d] = 0.0f;
                continue;
            }
            double l = 0.0;
            for (int d = 0; d < D; ++d) acc[d] = 0.0;
            for (int n = 0; n <= m && n < Sk; ++n) {
                if (!kp[n / BLK]) continue;
                const double p = exp(logit[n] - mx);
                l += p;
                const float *v = V + b * vb + kvh * vh + (int64_t)n * vs;
                for (int d = 0; d < D; ++d) acc[d] += p * (double)v[d * vd];
            }
            for (int d = 0; d < D; ++d) o[d] = (float)(acc[d] / l);
        }
        free(logit); free(acc);
    }
    return 0;
}
