// select.cu -- tile scoring, top-kmax, sigma router and kv_idx emission (sm_100a).
//
// Replaces src/sparse_attention.py:638-748 (everything after the block
// summaries in _block_select_kv_idx_v2) with three launches:
//
//  1. select_tile_kernel, one CTA per (b, q-head, 64-row tile):
//       per-row block scores in fp32 (fmaf chain over d, then * scale;
//       Quest: two chains max(q,0)*Kmax and min(q,0)*Kmin, added, then scaled),
//       max over the tile's rows (:655-656), causal visibility (:660-666),
//       sink and self block forced to FLT_MAX (:675-684), a full descending
//       sort of (score, lower-index-first) keys, the top kmax ids written to
//       kv_idx and the per-tile margin
//       sigma = (s[kb-1]-s[kb]) / max(s[0]-s[kb], 1e-6)  (:700-707)
//       written to the workspace.
//  2. select_quantile_kernel, one CTA: row-grain head mean of sigma
//     (sum over heads in order, then / H, :708-710) and the k-th smallest
//     margin of the expanded [B,H,Qt] array by radix selection, NaN last
//     (kthvalue, :711-716).
//  3. select_finalize_kernel: tiles that did not trigger get the sentinel NB
//     in slots >= k_base (:720-725); optional sigma / trigger outputs.
//
// Scores are computed exactly in the canonical order shared with
// oracle/ugbsa_oracle.c, so kv_idx, sigma and the trigger decisions match the
// CPU restatement bit for bit.  IEEE division, no flush-to-zero: sigma is a
// subnormal number (s[0] is the forced FLT_MAX).
#include <cfloat>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

constexpr int kSelThreads = 256;

struct SelParams {
    int B, Hq, Hkv, S, D, NB, Qt, NBpad;
    float scale;
    int k_base, kmax, router;
    int32_t *kv_idx;
    float *sigma_cell;  // workspace [B*Hq*Qt]
    // order statistics (the STATS variant): ranks k_b and rho_k of the unforced sort
    int k_b, rho_k;
    float *st_g, *st_r, *st_sigma, *st_grho;   // [B*Hq*Qt] each
    // per-row scores (the ROWS variant, the v1 selector): [B,Hq,S,NB], blocks < the tile's nvis
    float *row_scores;
};

__device__ __forceinline__ void load8f(const float *p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void load8f(const __nv_bfloat16 *p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void load8f(const __half *p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

// Shared-memory layout of select_tile_kernel (floats unless noted):
//   sQ  [D][QSTR]          query tile, transposed (row index fastest), rows >= S zero
//   sA  [D][KSTR]          summary chunk (mean or Kmin), transposed (block fastest)
//   sB  [D][KSTR]          Kmax chunk (Quest only)
//   red [8][NBC]           cross-warp max scratch
//   ts  [NBpad]            tile scores
//   keys[NBpad] (uint64)   sort keys
template <int NBC>
struct SelLayout {
    static constexpr int QSTR = 64 + 4;
    static constexpr int KSTR = NBC + 4;
};

// STATS: instead of kv_idx / sigma, the order statistics of the block-score
// diagnostic over the unforced, causally masked tile scores (p.st_*).
// ROWS: every row's score of every block up to the tile's last visible one goes
// to p.row_scores (the v1 selector ranks blocks per row); no tile max, no ranking.
template <typename T, bool QUEST, int NBC, int TB, bool STATS = false, bool ROWS = false>
__global__ void __launch_bounds__(kSelThreads) select_tile_kernel(const T *__restrict__ Q, int64_t qb, int64_t qh,
                                                                   int64_t qs, const float *__restrict__ summ_a,
                                                                   const float *__restrict__ summ_b,
                                                                   const SelParams p) {
    using L = SelLayout<NBC>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int D = p.D;
    float *sQ = reinterpret_cast<float *>(smem_raw);
    float *sA = sQ + D * L::QSTR;
    float *sB = sA + D * L::KSTR;
    float *red = sB + (QUEST ? D * L::KSTR : 0);
    float *ts = red + 8 * NBC;
    uint64_t *keys = reinterpret_cast<uint64_t *>(ts + p.NBpad);

    const int tid = threadIdx.x;
    const int item = blockIdx.x;
    const int t = p.Qt - 1 - (item % p.Qt);
    const int bh = item / p.Qt;
    const int h = bh % p.Hq;
    const int b = bh / p.Hq;
    const int kvh = h / (p.Hq / p.Hkv);
    int last = t * 64 + 63;
    if (last > p.S - 1) last = p.S - 1;
    const int self_blk = last / 64;
    const int nvis = self_blk + 1;

    // ---- query tile -> sQ (transposed); rows past S are the zero padding
    {
        const T *qbase = Q + (int64_t)b * qb + (int64_t)h * qh;
        const int ngroups = D / 8;
        for (int i = tid; i < 64 * ngroups; i += kSelThreads) {
            const int r = i & 63, g = i >> 6;
            const int row = t * 64 + r;
            float x[8];
            if (row < p.S) load8f(qbase + (int64_t)row * qs + g * 8, x);
            else {
#pragma unroll
                for (int j = 0; j < 8; ++j) x[j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) sQ[(g * 8 + j) * L::QSTR + r] = x[j];
        }
    }

    const int ty = tid >> 4;   // rows 4*ty .. 4*ty+3
    const int tx = tid & 15;   // blocks TB*tx .. TB*tx+TB-1 of the chunk
    const float *A = summ_a + ((int64_t)b * p.Hkv + kvh) * p.NB * D;
    const float *Bm = QUEST ? summ_b + ((int64_t)b * p.Hkv + kvh) * p.NB * D : nullptr;

    for (int c0 = 0; c0 < nvis; c0 += NBC) {
        __syncthreads();  // previous chunk fully consumed (and sQ written)
        const int nq = D / 4;
        for (int i = tid; i < NBC * nq; i += kSelThreads) {
            const int blk = i % NBC, g = i / NBC;
            const int gb = c0 + blk;
            float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
            if (gb < p.NB) {
                va = __ldg(reinterpret_cast<const float4 *>(A + (int64_t)gb * D + g * 4));
                if (QUEST) vb = __ldg(reinterpret_cast<const float4 *>(Bm + (int64_t)gb * D + g * 4));
            }
            sA[(g * 4 + 0) * L::KSTR + blk] = va.x;
            sA[(g * 4 + 1) * L::KSTR + blk] = va.y;
            sA[(g * 4 + 2) * L::KSTR + blk] = va.z;
            sA[(g * 4 + 3) * L::KSTR + blk] = va.w;
            if (QUEST) {
                sB[(g * 4 + 0) * L::KSTR + blk] = vb.x;
                sB[(g * 4 + 1) * L::KSTR + blk] = vb.y;
                sB[(g * 4 + 2) * L::KSTR + blk] = vb.z;
                sB[(g * 4 + 3) * L::KSTR + blk] = vb.w;
            }
        }
        __syncthreads();

        float acc[4][TB], acc2[4][TB];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < TB; ++j) { acc[i][j] = 0.f; acc2[i][j] = 0.f; }

#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            const float4 q4 = *reinterpret_cast<const float4 *>(sQ + d * L::QSTR + 4 * ty);
            const float q[4] = {q4.x, q4.y, q4.z, q4.w};
            float ka[TB], kb[TB];
            if constexpr (TB == 4) {
                const float4 a4 = *reinterpret_cast<const float4 *>(sA + d * L::KSTR + 4 * tx);
                ka[0] = a4.x; ka[1] = a4.y; ka[2] = a4.z; ka[3] = a4.w;
                if constexpr (QUEST) {
                    const float4 b4 = *reinterpret_cast<const float4 *>(sB + d * L::KSTR + 4 * tx);
                    kb[0] = b4.x; kb[1] = b4.y; kb[2] = b4.z; kb[3] = b4.w;
                }
            } else {
                const float2 a2 = *reinterpret_cast<const float2 *>(sA + d * L::KSTR + 2 * tx);
                ka[0] = a2.x; ka[1] = a2.y;
                if constexpr (QUEST) {
                    const float2 b2 = *reinterpret_cast<const float2 *>(sB + d * L::KSTR + 2 * tx);
                    kb[0] = b2.x; kb[1] = b2.y;
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (QUEST) {
                    const float qp = q[i] > 0.f ? q[i] : 0.f;
                    const float qn = q[i] < 0.f ? q[i] : 0.f;
#pragma unroll
                    for (int j = 0; j < TB; ++j) {
                        acc[i][j] = __fmaf_rn(qp, kb[j], acc[i][j]);   // max(q,0) * Kmax
                        acc2[i][j] = __fmaf_rn(qn, ka[j], acc2[i][j]); // min(q,0) * Kmin
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < TB; ++j) acc[i][j] = __fmaf_rn(q[i], ka[j], acc[i][j]);
                }
            }
        }
        if constexpr (ROWS) {
            float *rs = p.row_scores + (((int64_t)b * p.Hq + h) * p.S) * p.NB;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = t * 64 + 4 * ty + i;
                if (row >= p.S) continue;
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    const int blk = c0 + TB * tx + j;
                    if (blk >= nvis) continue;
                    rs[(int64_t)row * p.NB + blk] = QUEST ? __fmul_rn(__fadd_rn(acc[i][j], acc2[i][j]), p.scale)
                                                          : __fmul_rn(acc[i][j], p.scale);
                }
            }
            continue;
        }
        // scores -> max over this thread's 4 rows
        float m[TB];
#pragma unroll
        for (int j = 0; j < TB; ++j) {
            m[j] = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float s = QUEST ? __fmul_rn(__fadd_rn(acc[i][j], acc2[i][j]), p.scale)
                                      : __fmul_rn(acc[i][j], p.scale);
                m[j] = (s > m[j]) ? s : m[j];
            }
            const float o = __shfl_xor_sync(0xffffffffu, m[j], 16);
            m[j] = (o > m[j]) ? o : m[j];
        }
        const int warp = tid >> 5;
        if ((tid & 16) == 0) {
#pragma unroll
            for (int j = 0; j < TB; ++j) red[warp * NBC + TB * tx + j] = m[j];
        }
        __syncthreads();
        if (tid < NBC) {
            float v = red[tid];
#pragma unroll
            for (int w = 1; w < 8; ++w) {
                const float o = red[w * NBC + tid];
                v = (o > v) ? o : v;
            }
            if (c0 + tid < nvis) ts[c0 + tid] = v;
        }
    }
    if constexpr (ROWS) return;
    __syncthreads();

    // ---- ranking keys: descending score, ties -> lower block id
    for (int j = tid; j < p.NBpad; j += kSelThreads) {
        uint64_t key = 0;  // padding past NB: below everything
        if (j < p.NB) {
            float v = (j < nvis) ? ts[j] : -INFINITY;
            if (!STATS && (j == 0 || j == self_blk)) v = FLT_MAX;
            key = ((uint64_t)ordered_key(v) << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
        }
        keys[j] = key;
    }
    __syncthreads();
    // bitonic sort, descending
    for (int k = 2; k <= p.NBpad; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < p.NBpad; i += kSelThreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = keys[i], c = keys[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < c) : (a > c)) {
                        keys[i] = c;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    const int64_t cell = ((int64_t)b * p.Hq + h) * p.Qt + t;
    if constexpr (STATS) {
        if (tid == 0) {
            // IEEE float32 throughout, inf / NaN as they fall (torch semantics:
            // clamp passes NaN through)
            const float s0 = key_value((uint32_t)(keys[0] >> 32));
            const float skm1 = key_value((uint32_t)(keys[p.k_b - 1] >> 32));
            const float sk = key_value((uint32_t)(keys[p.k_b] >> 32));
            const float srm1 = key_value((uint32_t)(keys[p.rho_k - 1] >> 32));
            const float sr = key_value((uint32_t)(keys[p.rho_k] >> 32));
            const float g = __fsub_rn(skm1, sk);
            float r = __fsub_rn(s0, sk);
            if (r < 1e-9f) r = 1e-9f;
            float sg = __fdiv_rn(g, r);
            if (sg < 0.f) sg = 0.f;
            if (sg > 2.f) sg = 2.f;
            p.st_g[cell] = g;
            p.st_r[cell] = r;
            p.st_sigma[cell] = sg;
            p.st_grho[cell] = __fsub_rn(srm1, sr);
        }
        return;
    }
    int32_t *out = p.kv_idx + cell * p.kmax;
    for (int j = tid; j < p.kmax; j += kSelThreads) out[j] = (int32_t)(0xffffffffu - (uint32_t)(keys[j] & 0xffffffffu));
    if (tid == 0) {
        float sig = __int_as_float(0x7fc00000);
        if (p.router) {
            const float s_top = key_value((uint32_t)(keys[0] >> 32));
            const float s_km1 = key_value((uint32_t)(keys[p.k_base - 1] >> 32));
            const float s_k = key_value((uint32_t)(keys[p.k_base] >> 32));
            float spread = __fsub_rn(s_top, s_k);
            if (spread < 1e-6f) spread = 1e-6f;  // clamp(min=1e-6); NaN passes through
            sig = __fdiv_rn(__fsub_rn(s_km1, s_k), spread);
        }
        p.sigma_cell[cell] = sig;
    }
}

// ---------------------------------------------------------------- noise scale
// Block-score diagnostic, noise-scale estimate: one CTA per (b, h, sampled row
// pair (i, i+1)) sums, over all NB blocks (no causal mask), the squared
// difference of the two rows' block scores (Quest: the two envelope sums, then
// added and scaled; mean: one sum, scaled).  Lanes split the head dimension.
template <typename T, bool QUEST>
__global__ void __launch_bounds__(128) pair_diff_kernel(const T *__restrict__ Q, int64_t qb, int64_t qh, int64_t qs,
                                                        const float *__restrict__ summ_a,
                                                        const float *__restrict__ summ_b, int Hq, int Hkv, int S,
                                                        int D, int NB, float scale, int n_pairs, int stride,
                                                        float *__restrict__ partial) {
    __shared__ float sq[2][256];
    __shared__ float red[4];
    const int pr = blockIdx.x % n_pairs;
    const int bh = blockIdx.x / n_pairs;
    const int h = bh % Hq, b = bh / Hq;
    const int kvh = h / (Hq / Hkv);
    int i = pr * stride;
    if (i > S - 2) i = S - 2;
    const T *qbase = Q + (int64_t)b * qb + (int64_t)h * qh;
    for (int e = threadIdx.x; e < 2 * D; e += 128) {
        const int rr = e / D, d = e % D;
        float x[8];
        load8f(qbase + (int64_t)(i + rr) * qs + (d & ~7), x);
        sq[rr][d] = x[d & 7];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *A = summ_a + ((int64_t)b * Hkv + kvh) * NB * D;
    const float *Bm = QUEST ? summ_b + ((int64_t)b * Hkv + kvh) * NB * D : nullptr;
    float acc = 0.f;
    for (int j = warp; j < NB; j += 4) {
        float p0 = 0.f, n0 = 0.f, p1 = 0.f, n1 = 0.f;
        for (int d = lane; d < D; d += 32) {
            const float x0 = sq[0][d], x1 = sq[1][d];
            const float ka = __ldg(A + (int64_t)j * D + d);
            if (QUEST) {
                const float kb = __ldg(Bm + (int64_t)j * D + d);
                p0 = __fmaf_rn(x0 > 0.f ? x0 : 0.f, kb, p0);
                n0 = __fmaf_rn(x0 < 0.f ? x0 : 0.f, ka, n0);
                p1 = __fmaf_rn(x1 > 0.f ? x1 : 0.f, kb, p1);
                n1 = __fmaf_rn(x1 < 0.f ? x1 : 0.f, ka, n1);
            } else {
                p0 = __fmaf_rn(x0, ka, p0);
                p1 = __fmaf_rn(x1, ka, p1);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            p0 += __shfl_xor_sync(0xffffffffu, p0, o);
            p1 += __shfl_xor_sync(0xffffffffu, p1, o);
            if (QUEST) {
                n0 += __shfl_xor_sync(0xffffffffu, n0, o);
                n1 += __shfl_xor_sync(0xffffffffu, n1, o);
            }
        }
        const float s0 = (QUEST ? p0 + n0 : p0) * scale;
        const float s1 = (QUEST ? p1 + n1 : p1) * scale;
        const float df = s1 - s0;
        acc = __fmaf_rn(df, df, acc);
    }
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) partial[(int64_t)bh * n_pairs + pr] = (red[0] + red[1]) + (red[2] + red[3]);
}

// tau_hat[bh] = sqrt(max(0, sum(partial) / (n_pairs * NB) / 2)), the sum in fp64, pair order
__global__ void pair_diff_finish_kernel(const float *__restrict__ partial, int nbh, int n_pairs, int NB,
                                        float *__restrict__ tau_hat) {
    const int bh = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (bh >= nbh) return;
    double acc = 0.0;
    for (int k = lane; k < n_pairs; k += 32) acc += (double)partial[(int64_t)bh * n_pairs + k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        const double tau = 0.5 * acc / ((double)n_pairs * (double)NB);
        tau_hat[bh] = (float)sqrt(tau > 0.0 ? tau : 0.0);
    }
}

// ---------------------------------------------------------------- row sums
// sum over this shard's heads, in head order, of the per-tile margins
// (the numerator of the reference's row-grain head mean, :708-710)
__global__ void __launch_bounds__(256) sigma_rowsum_kernel(const float *__restrict__ sigma_cell, int B, int Hq,
                                                           int Qt, float *__restrict__ rowsum) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * Qt) return;
    const int bb = (int)(i / Qt), tt = (int)(i % Qt);
    float acc = 0.f;
    for (int hh = 0; hh < Hq; ++hh) acc = __fadd_rn(acc, sigma_cell[((int64_t)bb * Hq + hh) * Qt + tt]);
    rowsum[i] = acc;
}

// ---------------------------------------------------------------- quantile
struct QuantParams {
    int B, Qt, H_total;
    int grain_row;      // 1: margins averaged over heads
    int mode_quantile;  // 1: bottom-q quantile; 0: abs threshold
    int64_t kq;         // 1-based rank in the expanded [B, H_total, Qt] array
    float tau;          // fp32(tau), abs mode
    const float *rowsum;     // row grain: [B*Qt] sums over all H_total heads
    const float *cells_all;  // cell grain: [B*H_total*Qt] margins of all heads
    float *eff_row;     // [B*Qt] out (row grain)
    float *thresh;      // [1] out
};

__device__ __forceinline__ uint32_t asc_key(float v) {
    if (v != v) return 0xffffffffu;  // NaN sorts last (kthvalue)
    v = __fadd_rn(v, 0.0f);
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(1024) select_quantile_kernel(const QuantParams p) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int64_t s_k;
    const int tid = threadIdx.x;
    const int64_t nrow = (int64_t)p.B * p.Qt;
    if (p.grain_row) {
        for (int64_t i = tid; i < nrow; i += blockDim.x) p.eff_row[i] = __fdiv_rn(p.rowsum[i], (float)p.H_total);
        __syncthreads();
    }
    if (!p.mode_quantile) {
        if (tid == 0) p.thresh[0] = p.tau;
        return;
    }
    const float *vals = p.grain_row ? p.eff_row : p.cells_all;
    const int64_t n = p.grain_row ? nrow : nrow * p.H_total;
    // each row value appears H_total times in the expanded array
    const int64_t kk = p.grain_row ? (p.kq - 1) / p.H_total + 1 : p.kq;
    if (n <= (int64_t)blockDim.x) {
        // few values (a decode step): the k-th smallest by counting, one pass -- value i
        // has rank #(v < v_i) + #(v == v_i, j < i) in the ascending order of the keys
        if (tid < n) {
            const uint32_t ui = asc_key(vals[tid]);
            int64_t rank = 0;
            for (int64_t j = 0; j < n; ++j) {
                const uint32_t uj = asc_key(vals[j]);
                rank += (uj < ui || (uj == ui && j < tid)) ? 1 : 0;
            }
            if (rank == kk - 1) {
                float v;
                if (ui == 0xffffffffu) v = __int_as_float(0x7fc00000);
                else {
                    const uint32_t bb = (ui & 0x80000000u) ? (ui & 0x7fffffffu) : ~ui;
                    v = __uint_as_float(bb);
                }
                p.thresh[0] = v;
            }
        }
        return;
    }
    if (tid == 0) {
        s_k = kk;
        s_prefix = 0;
        s_mask = 0;
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int64_t i = tid; i < n; i += blockDim.x) {
            const uint32_t u = asc_key(vals[i]);
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
        float v;
        if (u == 0xffffffffu) v = __int_as_float(0x7fc00000);
        else {
            const uint32_t bb = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
            v = __uint_as_float(bb);
        }
        p.thresh[0] = v;
    }
}

struct FinParams {
    int B, Hq, Qt, NB, k_base, kmax, router, grain_row, mode_quantile;
    int Qt_all;                // row means cover all Qt_all tiles of the sequence
    int t_base, pair_stride;   // local cell tile t is sequence tile seq_tile(t, t_base, pair_stride)
    const float *sigma_cell, *eff_row, *thresh;
    int32_t *kv_idx;
    float *sigma_out;
    uint8_t *trigger_out;
};

__global__ void __launch_bounds__(256) select_finalize_kernel(const FinParams p) {
    const int64_t ncell = (int64_t)p.B * p.Hq * p.Qt;
    const int64_t cell = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (cell >= ncell) return;
    float eff = __int_as_float(0x7fc00000);
    bool unc = false;
    if (p.router) {
        const int tt = (int)(cell % p.Qt);
        const int bb = (int)(cell / ((int64_t)p.Hq * p.Qt));
        eff = p.grain_row ? p.eff_row[(int64_t)bb * p.Qt_all + seq_tile(tt, p.t_base, p.pair_stride)]
                          : p.sigma_cell[cell];
        const float th = p.thresh[0];
        unc = p.mode_quantile ? (eff <= th) : (eff < th);
        if (!unc) {
            int32_t *row = p.kv_idx + cell * p.kmax;
            for (int j = p.k_base + lane; j < p.kmax; j += 32) row[j] = p.NB;
        }
    }
    if (lane == 0) {
        if (p.sigma_out) p.sigma_out[cell] = eff;
        if (p.trigger_out) p.trigger_out[cell] = unc ? 1 : 0;
    }
}

// ---------------------------------------------------------------- host side
// workspace: [sigma cells B*Hq*Qt][row sums B*Qt][row means B*Qt][thresh]
static int64_t al256(int64_t x) { return (x + 255) / 256 * 256; }

// workspace: [tensor-core scoring scratch][sigma cells][row sums][row means][thresh]
static size_t select_tail_bytes(int B, int Hq, int S) {
    const int64_t Qt = (S + 63) / 64;
    const int64_t cells = (int64_t)B * Hq * Qt;
    const int64_t rows = (int64_t)B * Qt;
    return (size_t)(al256(cells * 4) + 2 * al256(rows * 4) + 256);
}

// Bound over every dtype, head dim (<= 256) and KV head count (<= Hq): the
// tensor-core scratch is largest at D = 256 with Hkv = Hq.
size_t select_workspace_bytes(int B, int Hq, int S) {
    const int Qt = (S + 63) / 64;
    return al256((int64_t)tc_scratch_bytes(B, Hq, Hq, S, 256, Qt)) + select_tail_bytes(B, Hq, S);
}

// what the tiles stage reads from the front of the workspace
size_t select_tiles_scratch_bytes(int dtype, int B, int Hq, int Hkv, int S, int D, int Qt) {
    return tc_select_supported(dtype, D) ? al256((int64_t)tc_scratch_bytes(B, Hq, Hkv, S, D, Qt)) : 0;
}

// exactly what launch_select lays out for this problem
size_t select_workspace_bytes_exact(int dtype, int B, int Hq, int Hkv, int S, int D) {
    const int Qt = (S + 63) / 64;
    return select_tiles_scratch_bytes(dtype, B, Hq, Hkv, S, D, Qt) + select_tail_bytes(B, Hq, S);
}

size_t select_finish_workspace_bytes(int B, int S) {
    const int64_t rows = (int64_t)B * ((S + 63) / 64);
    return (size_t)(al256(rows * 4) + 256);
}

static int next_pow2(int x) {
    int p = 64;
    while (p < x) p <<= 1;
    return p;
}

template <typename T, bool QUEST, int NBC, int TB, bool STATS = false, bool ROWS = false>
static int launch_tile_t(const T *Q, ugbsa_strides qs, const float *sa, const float *sb, const SelParams &sp,
                         cudaStream_t stream) {
    using L = SelLayout<NBC>;
    const size_t smem = (size_t)sp.D * L::QSTR * 4 + (size_t)sp.D * L::KSTR * 4 * (QUEST ? 2 : 1) +
                        (ROWS ? (size_t)16 : (size_t)8 * NBC * 4 + (size_t)sp.NBpad * 4 + (size_t)sp.NBpad * 8 + 16);
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    auto kern = select_tile_kernel<T, QUEST, NBC, TB, STATS, ROWS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    const int64_t grid = (int64_t)sp.B * sp.Hq * sp.Qt;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    kern<<<(unsigned)grid, kSelThreads, smem, stream>>>(Q, qs.b, qs.h, qs.s, sa, sb, sp);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

template <typename T, bool STATS = false, bool ROWS = false>
static int launch_tile_d(const T *Q, ugbsa_strides qs, const float *sa, const float *sb, bool quest,
                         const SelParams &sp, cudaStream_t stream) {
    if (sp.D <= 128) {
        return quest ? launch_tile_t<T, true, 64, 4, STATS, ROWS>(Q, qs, sa, sb, sp, stream)
                     : launch_tile_t<T, false, 64, 4, STATS, ROWS>(Q, qs, sa, sb, sp, stream);
    }
    return quest ? launch_tile_t<T, true, 32, 2, STATS, ROWS>(Q, qs, sa, sb, sp, stream)
                 : launch_tile_t<T, false, 32, 2, STATS, ROWS>(Q, qs, sa, sb, sp, stream);
}

// per-row scores [B,Hq,S,NB] of every (row, block up to the row's tile) -- the v1 selector's input
int launch_row_scores(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                      int Hq, int Hkv, int S, int D, float scale, bool quest, float *row_scores,
                      cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    SelParams sp{};
    sp.B = B; sp.Hq = Hq; sp.Hkv = Hkv; sp.S = S; sp.D = D; sp.NB = NB; sp.Qt = NB;
    sp.NBpad = next_pow2(NB);
    sp.scale = scale;
    sp.row_scores = row_scores;
    switch (dtype) {
        case UGBSA_F32: return launch_tile_d<float, false, true>((const float *)Q, qs, summ_a, summ_b, quest, sp, stream);
        case UGBSA_BF16:
            return launch_tile_d<__nv_bfloat16, false, true>((const __nv_bfloat16 *)Q, qs, summ_a, summ_b, quest, sp,
                                                             stream);
        case UGBSA_F16: return launch_tile_d<__half, false, true>((const __half *)Q, qs, summ_a, summ_b, quest, sp, stream);
    }
    return UGBSA_ERR_DTYPE;
}

static bool cfg_quest(const ugbsa_selector_config *cfg) {
    return (cfg->mode == UGBSA_MODE_QUEST) || (cfg->mode == UGBSA_MODE_ROUTER && cfg->router_score == UGBSA_SCORE_QUEST);
}

int launch_select_tiles(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                        int Hq, int Hkv, int S, int D, int t_base, int pair_stride, int Sq, float scale,
                        const ugbsa_selector_config *cfg, int k_base, int kmax, int32_t *kv_idx, float *sigma_cell,
                        float *sigma_rowsum, void *scratch, cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    const int Qt = (Sq + 63) / 64;
    if (tc_select_supported(dtype, D)) {
        const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (k_base < kmax);
        int rc = launch_select_tiles_tc(Q, qs, summ_a, summ_b, B, Hq, Hkv, S, D, t_base, pair_stride, Sq, scale,
                                        cfg_quest(cfg), k_base, kmax, router, kv_idx, sigma_cell, scratch, stream);
        if (rc != UGBSA_OK) return rc;
        if (sigma_rowsum) {
            const int64_t rows = (int64_t)B * Qt;
            sigma_rowsum_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(sigma_cell, B, Hq, Qt,
                                                                                    sigma_rowsum);
            if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
        }
        return UGBSA_OK;
    }
    // a slice of the query rows needs the tensor-core path
    if (t_base != 0 || pair_stride != 1 || Sq != S) return UGBSA_ERR_UNSUPPORTED;
    SelParams sp;
    sp.B = B; sp.Hq = Hq; sp.Hkv = Hkv; sp.S = S; sp.D = D; sp.NB = NB; sp.Qt = NB;
    sp.NBpad = next_pow2(NB);
    sp.scale = scale;
    sp.k_base = k_base; sp.kmax = kmax;
    sp.router = (cfg->mode == UGBSA_MODE_ROUTER) && (k_base < kmax) ? 1 : 0;
    sp.kv_idx = kv_idx;
    sp.sigma_cell = sigma_cell;
    const bool quest = cfg_quest(cfg);
    int rc;
    switch (dtype) {
        case UGBSA_F32: rc = launch_tile_d((const float *)Q, qs, summ_a, summ_b, quest, sp, stream); break;
        case UGBSA_BF16: rc = launch_tile_d((const __nv_bfloat16 *)Q, qs, summ_a, summ_b, quest, sp, stream); break;
        case UGBSA_F16: rc = launch_tile_d((const __half *)Q, qs, summ_a, summ_b, quest, sp, stream); break;
        default: return UGBSA_ERR_DTYPE;
    }
    if (rc != UGBSA_OK) return rc;
    if (sigma_rowsum) {
        const int64_t rows = (int64_t)B * NB;
        sigma_rowsum_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(sigma_cell, B, Hq, NB, sigma_rowsum);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    return UGBSA_OK;
}

int launch_select_finish_q(const float *sigma_cell, const float *sigma_all, int B, int Hq, int H_total, int S,
                           int Qt_all, int t_base, int pair_stride, int Qt_local, const ugbsa_selector_config *cfg,
                           int k_base, int kmax, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out,
                           void *workspace, cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    const int Qt = Qt_all;   // the quantile runs over every tile of the call (the sequence's, or a decode step's one)
    const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (k_base < kmax);
    const bool grain_row = cfg->router_grain == UGBSA_GRAIN_ROW;
    const bool mode_q = cfg->router_mode == UGBSA_ROUTER_QUANTILE;
    const int64_t rows = (int64_t)B * Qt;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *eff_row = reinterpret_cast<float *>(ws);
    float *thresh = reinterpret_cast<float *>(ws + al256(rows * 4));
    if (router) {
        QuantParams qp;
        qp.B = B; qp.Qt = Qt; qp.H_total = H_total;
        qp.grain_row = grain_row ? 1 : 0;
        qp.mode_quantile = mode_q ? 1 : 0;
        const int64_t numel = (int64_t)B * H_total * Qt;
        int64_t kq = (int64_t)(cfg->router_quantile * (double)numel);  // int(q * numel), :713-714
        if (kq < 1) kq = 1;
        if (kq > numel) kq = numel;
        qp.kq = kq;
        qp.tau = (float)cfg->router_tau;
        qp.rowsum = grain_row ? sigma_all : nullptr;
        qp.cells_all = grain_row ? nullptr : sigma_all;
        qp.eff_row = eff_row;
        qp.thresh = thresh;
        select_quantile_kernel<<<1, 1024, 0, stream>>>(qp);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    if (router || sigma_out || trigger_out) {
        FinParams fp;
        fp.B = B; fp.Hq = Hq; fp.Qt = Qt_local; fp.Qt_all = Qt; fp.t_base = t_base; fp.pair_stride = pair_stride;
        fp.NB = NB; fp.k_base = k_base; fp.kmax = kmax;
        fp.router = router ? 1 : 0;
        fp.grain_row = grain_row ? 1 : 0;
        fp.mode_quantile = mode_q ? 1 : 0;
        fp.sigma_cell = sigma_cell; fp.eff_row = eff_row; fp.thresh = thresh;
        fp.kv_idx = kv_idx; fp.sigma_out = sigma_out; fp.trigger_out = trigger_out;
        const int64_t grid = ((int64_t)B * Hq * Qt_local + 7) / 8;
        select_finalize_kernel<<<(unsigned)grid, 256, 0, stream>>>(fp);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    return UGBSA_OK;
}

int launch_sigma_rowsum(const float *sigma_cell, int B, int Hq, int Qt, float *rowsum, cudaStream_t stream) {
    const int64_t rows = (int64_t)B * Qt;
    sigma_rowsum_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(sigma_cell, B, Hq, Qt, rowsum);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

size_t block_order_stats_workspace_bytes(int B, int Hq, int S) {
    const int64_t n_pairs = S > 1 ? (S - 1 < 1024 ? S - 1 : 1024) : 0;
    return (size_t)al256((int64_t)B * Hq * n_pairs * 4);
}

int launch_block_order_stats(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b,
                             int B, int Hq, int Hkv, int S, int D, float scale, bool quest, int k_b, int rho_k,
                             float *g, float *r, float *sigma, float *g_rho, float *tau_hat, void *workspace,
                             cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    SelParams sp{};
    sp.B = B; sp.Hq = Hq; sp.Hkv = Hkv; sp.S = S; sp.D = D; sp.NB = NB; sp.Qt = NB;
    sp.NBpad = next_pow2(NB);
    sp.scale = scale;
    sp.k_b = k_b; sp.rho_k = rho_k;
    sp.st_g = g; sp.st_r = r; sp.st_sigma = sigma; sp.st_grho = g_rho;
    int rc;
    switch (dtype) {
        case UGBSA_F32: rc = launch_tile_d<float, true>((const float *)Q, qs, summ_a, summ_b, quest, sp, stream); break;
        case UGBSA_BF16:
            rc = launch_tile_d<__nv_bfloat16, true>((const __nv_bfloat16 *)Q, qs, summ_a, summ_b, quest, sp, stream);
            break;
        case UGBSA_F16: rc = launch_tile_d<__half, true>((const __half *)Q, qs, summ_a, summ_b, quest, sp, stream); break;
        default: return UGBSA_ERR_DTYPE;
    }
    if (rc != UGBSA_OK || !tau_hat) return rc;
    const int n_pairs = S - 1 < 1024 ? S - 1 : 1024;
    const int stride = (S - 1) / n_pairs > 1 ? (S - 1) / n_pairs : 1;
    float *partial = static_cast<float *>(workspace);
    const int64_t grid = (int64_t)B * Hq * n_pairs;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
#define UGBSA_PAIR_DIFF(TT)                                                                                        \
    (quest ? pair_diff_kernel<TT, true><<<(unsigned)grid, 128, 0, stream>>>(                                       \
                 (const TT *)Q, qs.b, qs.h, qs.s, summ_a, summ_b, Hq, Hkv, S, D, NB, scale, n_pairs, stride, partial) \
           : pair_diff_kernel<TT, false><<<(unsigned)grid, 128, 0, stream>>>(                                      \
                 (const TT *)Q, qs.b, qs.h, qs.s, summ_a, summ_b, Hq, Hkv, S, D, NB, scale, n_pairs, stride, partial))
    switch (dtype) {
        case UGBSA_F32: UGBSA_PAIR_DIFF(float); break;
        case UGBSA_BF16: UGBSA_PAIR_DIFF(__nv_bfloat16); break;
        default: UGBSA_PAIR_DIFF(__half); break;
    }
#undef UGBSA_PAIR_DIFF
    if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    const int nbh = B * Hq;
    pair_diff_finish_kernel<<<(unsigned)((nbh + 7) / 8), 256, 0, stream>>>(partial, nbh, n_pairs, NB, tau_hat);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_select_finish(const float *sigma_cell, const float *sigma_all, int B, int Hq, int H_total, int S,
                         int t_base, int pair_stride, int Qt_local, const ugbsa_selector_config *cfg, int k_base,
                         int kmax, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace,
                         cudaStream_t stream) {
    return launch_select_finish_q(sigma_cell, sigma_all, B, Hq, H_total, S, (S + 63) / 64, t_base, pair_stride,
                                  Qt_local, cfg, k_base, kmax, kv_idx, sigma_out, trigger_out, workspace, stream);
}

int launch_select(const void *Q, int dtype, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B,
                  int Hq, int Hkv, int S, int D, float scale, const ugbsa_selector_config *cfg, int k_base, int kmax,
                  int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, void *workspace, cudaStream_t stream) {
    const int64_t Qt = (S + 63) / 64;
    const int64_t cells = (int64_t)B * Hq * Qt;
    const int64_t rows = (int64_t)B * Qt;
    uint8_t *scratch = static_cast<uint8_t *>(workspace);
    uint8_t *ws = scratch + select_tiles_scratch_bytes(dtype, B, Hq, Hkv, S, D, (int)Qt);
    float *sigma_cell = reinterpret_cast<float *>(ws);
    float *rowsum = reinterpret_cast<float *>(ws + al256(cells * 4));
    void *fin_ws = ws + al256(cells * 4) + al256(rows * 4);
    const bool row = cfg->router_grain == UGBSA_GRAIN_ROW;
    const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (k_base < kmax);
    int rc = launch_select_tiles(Q, dtype, qs, summ_a, summ_b, B, Hq, Hkv, S, D, 0, 1, S, scale, cfg, k_base,
                                 kmax, kv_idx, sigma_cell, (router && row) ? rowsum : nullptr, scratch, stream);
    if (rc != UGBSA_OK) return rc;
    return launch_select_finish(sigma_cell, row ? rowsum : sigma_cell, B, Hq, Hq, S, 0, 1, (int)Qt, cfg, k_base, kmax,
                                kv_idx, sigma_out, trigger_out, fin_ws, stream);
}

}  // namespace ugbsa
