// select_tc.cu -- tensor-core-guided exact tile scoring (sm_100a, bf16 Q).
//
// Same contract and bit-identical results as select_tile_kernel (select.cu),
// which evaluates every per-row block score on fp32 CUDA cores
// (src/sparse_attention.py:638-707).  The exact tile score of a block is the
// maximum over the tile's 64 rows of the canonical fp32 score; finding that
// row is what the tensor core does here, so only one row per block needs the
// exact fp32 evaluation:
//
//  A. score_exact_kernel, one CTA per (b, q-head, pair of tiles); with two
//     passes when its per-tile arrays fit (see the kernel).
//     tcgen05 GEMM: A operand = 128 block summaries in bf16 (M=128), B operand
//     = the two tiles' 128 query rows (N=128), accumulated in TMEM over d:
//       Quest:  Kmax.Q+ + Kmin.Q-   (bf16 envelopes; Q+ = max(q,0), Q- = min(q,0))
//       mean:   Khi.Q  + Klo.Q      (fp32 mean split into two bf16 parts)
//     Epilogue (thread = block, one warp group per tile): approximate row
//     scores s~_r, their max T~, and every row with s~_r >= T~ - 2 eps (nearly
//     always the argmax alone) is re-evaluated in the canonical fp32 order
//     (the oracle's fmaf chains); the maximum of those is the exact tile score,
//     written to the workspace.
//  B. rank_kernel, one CTA per (b, q-head, tile): sink/self forcing, the
//     kmax-th largest exact score by radix selection, a sort of the blocks at
//     or above it (descending, ties -> lower id), kv_idx and sigma.
//
// Error bound per (row r, block b), unscaled:
//   |s~ - canonical| <= |q_r| (2^-14 |k_b| + |res_b|) =: eps
// |q_r| is the row's Euclidean norm (rounded up), |k_b| the norm of the bf16
// operand magnitude (Quest: max(|Kmin|,|Kmax|) per d), |res_b| the norm of what
// the bf16 operands miss of the fp32 summary; sum |q_d k_d| <= |q||k|.  The
// canonical fmaf chain over D <= 128 terms is within D*2^-24 <= 2^-17 of the
// exact dot relative to sum |q_d k_d|; the tensor core multiplies bf16 exactly
// and accumulates in fp32, taken as within 2^-15 (4x the bound of a truncating
// fp32 accumulator).  tests/test_gpu_parity.py measures the tensor core's
// actual error against it.  The exact maximum's row r* satisfies
// s~_r* >= T~ - 2 eps, so it is always among the re-evaluated rows.
// Non-finite values re-evaluate all 64 rows.
#include <cfloat>
#include <cstdlib>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

constexpr float kTcRelErr = 6.103515625e-05f;  // 2^-14
constexpr float kNormPad = 1.00390625f;        // 1 + 2^-8, rounds norms up

// ---------------------------------------------------------------- operands
// fp32 summaries -> bf16 MMA operands + (|k|, |res|) per block.
//   quest: op0 = bf16(Kmax), op1 = bf16(Kmin)   (exact for bf16 K)
//   mean : op0 = bf16(m),    op1 = bf16(m - op0)
template <bool QUEST>
__global__ void __launch_bounds__(256) summary_operands_kernel(const float *__restrict__ sa, const float *__restrict__ sb,
                                                               int64_t nrows, int D, __nv_bfloat16 *__restrict__ op0,
                                                               __nv_bfloat16 *__restrict__ op1,
                                                               float2 *__restrict__ norms) {
    const int tpr = D / 8;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / tpr) + threadIdx.x / tpr;
    const int part = threadIdx.x % tpr;
    const bool active = row < nrows;
    float kk = 0.f, rr = 0.f;
    if (active) {
        const int64_t o = row * D + part * 8;
        float a[8], b[8];
        const float4 *pa = reinterpret_cast<const float4 *>(sa + o);
        float4 a0 = pa[0], a1 = pa[1];
        a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
        if (QUEST) {
            const float4 *pb = reinterpret_cast<const float4 *>(sb + o);
            float4 b0 = pb[0], b1 = pb[1];
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
        }
        __align__(16) __nv_bfloat16 h0[8], h1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (QUEST) {
                // a = Kmin, b = Kmax
                h0[i] = __float2bfloat16_rn(b[i]);
                h1[i] = __float2bfloat16_rn(a[i]);
                const float rmax = fabsf(b[i] - __bfloat162float(h0[i]));
                const float rmin = fabsf(a[i] - __bfloat162float(h1[i]));
                const float m = fmaxf(fabsf(__bfloat162float(h0[i])), fabsf(__bfloat162float(h1[i])));
                const float r = fmaxf(rmax, rmin);
                kk = fmaf(m, m, kk);
                rr = fmaf(r, r, rr);
            } else {
                h0[i] = __float2bfloat16_rn(a[i]);
                const float rest = a[i] - __bfloat162float(h0[i]);   // exact
                h1[i] = __float2bfloat16_rn(rest);
                const float r = fabsf(rest - __bfloat162float(h1[i]));
                const float m = fabsf(__bfloat162float(h0[i])) + fabsf(__bfloat162float(h1[i]));
                kk = fmaf(m, m, kk);
                rr = fmaf(r, r, rr);
            }
        }
        *reinterpret_cast<uint4 *>(op0 + o) = *reinterpret_cast<const uint4 *>(h0);
        *reinterpret_cast<uint4 *>(op1 + o) = *reinterpret_cast<const uint4 *>(h1);
    }
    for (int off = tpr >> 1; off > 0; off >>= 1) {
        kk += __shfl_xor_sync(0xffffffffu, kk, off);
        rr += __shfl_xor_sync(0xffffffffu, rr, off);
    }
    if (active && part == 0) norms[row] = make_float2(sqrtf(kk) * kNormPad, sqrtf(rr) * kNormPad);
}

// ---------------------------------------------------------------- kernel A
template <int D, bool QUEST>
struct TcLayout {
    static constexpr int DH = D / 64;
    static constexpr int Q_BYTES = DH * 128 * 128;      // [dh][128 rows][128 B]
    // [dh][128 blocks][128 B], one operand; D = 256: a stage holds one 64-column slab
    // of both operands (a chunk passes through DH stages), so Q and the stages fit
    static constexpr int K_BYTES = (D > 128 ? 1 : DH) * 128 * 128;
    static constexpr int STAGES = 2;
    static constexpr int OFF_Q0 = 0;                              // Q+ (Quest) or Q (mean)
    static constexpr int OFF_Q1 = OFF_Q0 + Q_BYTES;               // Q- (Quest only)
    static constexpr int OFF_K = OFF_Q1 + (QUEST ? Q_BYTES : 0);  // [stage][op][...]
    static constexpr int SMEM = OFF_K + STAGES * 2 * K_BYTES;
};

constexpr int kScoreThreads = 320;   // warps 0-7 epilogue, 8 producer, 9 MMA

struct TcParams {
    int B, Hq, Hkv, S, NB, Qt, npairs, kmax;
    int t_base, pair_stride;   // local tile t is sequence tile seq_tile(t, t_base, pair_stride)
    float scale;
    float *escore;        // [B,Hq,Qt,NB] exact scaled tile scores (visible blocks), local tiles
    const float2 *norms;  // [B,Hkv,NB] (|k|, |res|)
    const float *summ_a, *summ_b;   // fp32 summaries (mean | Kmin, Kmax)
    const __nv_bfloat16 *op0, *op1; // bf16 operand copies (Quest: Kmax, Kmin)
    int *err;
};

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// offset of the 16-byte chunk `ch` (8 elements) of row `r` in a [dh][rows][128 B] swizzled slab set
__device__ __forceinline__ uint32_t sw_off(int dh, int r, int ch) {
    return (uint32_t)(dh * 16384 + r * 128 + ((ch ^ (r & 7)) << 4));
}

// fp32 fma of the low (high) bf16 halves of two packed words into c: a product
// of two bf16 values is exact in fp32, so this is __fmaf_rn of their fp32
// values (one rounding) without unpacking them first
__device__ __forceinline__ float fma_bf16_lo(uint32_t a, uint32_t b, float c) {
    float d;
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %3;\n\t}"
        : "=f"(d) : "r"(a), "r"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float fma_bf16_hi(uint32_t a, uint32_t b, float c) {
    float d;
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, ah, bh, %3;\n\t}"
        : "=f"(d) : "r"(a), "r"(b), "f"(c));
    return d;
}

// canonical Quest score, query row R of the Q+/Q- buffers, block row lb of the
// staged bf16 envelopes (exact copies of the fp32 summary)
template <int D>
__device__ __forceinline__ float exact_quest_smem(const uint8_t *qp, const uint8_t *qn, const uint8_t *kmax,
                                                  const uint8_t *kmin, int R, int lb, float scale) {
    float ap = 0.f, an = 0.f;
#pragma unroll
    for (int dh = 0; dh < D / 64; ++dh) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 a = *reinterpret_cast<const uint4 *>(qp + sw_off(dh, R, ch));
            const uint4 c = *reinterpret_cast<const uint4 *>(qn + sw_off(dh, R, ch));
            const uint4 x = *reinterpret_cast<const uint4 *>(kmax + sw_off(dh, lb, ch));
            const uint4 y = *reinterpret_cast<const uint4 *>(kmin + sw_off(dh, lb, ch));
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
            const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ap = fma_bf16_lo(aw[e], xw[e], ap);
                an = fma_bf16_lo(cw[e], yw[e], an);
                ap = fma_bf16_hi(aw[e], xw[e], ap);
                an = fma_bf16_hi(cw[e], yw[e], an);
            }
        }
    }
    return __fmul_rn(__fadd_rn(ap, an), scale);
}

// canonical Quest score with the fp32 envelopes from global memory
template <int D>
__device__ __forceinline__ float exact_quest_global(const uint8_t *qp, const uint8_t *qn, const float *kmax,
                                                    const float *kmin, int R, float scale) {
    float ap = 0.f, an = 0.f;
#pragma unroll 1
    for (int dh = 0; dh < D / 64; ++dh) {
#pragma unroll 2
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 a = *reinterpret_cast<const uint4 *>(qp + sw_off(dh, R, ch));
            const uint4 c = *reinterpret_cast<const uint4 *>(qn + sw_off(dh, R, ch));
            const int d0 = dh * 64 + ch * 8;
            const float4 x0 = __ldg(reinterpret_cast<const float4 *>(kmax + d0));
            const float4 x1 = __ldg(reinterpret_cast<const float4 *>(kmax + d0 + 4));
            const float4 y0 = __ldg(reinterpret_cast<const float4 *>(kmin + d0));
            const float4 y1 = __ldg(reinterpret_cast<const float4 *>(kmin + d0 + 4));
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const float ys[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ap = __fmaf_rn(bf_lo(aw[e]), xs[2 * e], ap);
                an = __fmaf_rn(bf_lo(cw[e]), ys[2 * e], an);
                ap = __fmaf_rn(bf_hi(aw[e]), xs[2 * e + 1], ap);
                an = __fmaf_rn(bf_hi(cw[e]), ys[2 * e + 1], an);
            }
        }
    }
    return __fmul_rn(__fadd_rn(ap, an), scale);
}

// canonical Quest score with the bf16 envelope copies read from L2: every load
// is issued before the chains start
template <int D>
__device__ __forceinline__ float exact_quest_l2(const uint8_t *qp, const uint8_t *qn, const __nv_bfloat16 *kmax,
                                                const __nv_bfloat16 *kmin, int R, float scale) {
    const uint4 *px = reinterpret_cast<const uint4 *>(kmax);
    const uint4 *py = reinterpret_cast<const uint4 *>(kmin);
    uint4 x[D / 8], y[D / 8];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        x[i] = __ldg(px + i);
        y[i] = __ldg(py + i);
    }
    float ap = 0.f, an = 0.f;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        const int dh = i >> 3, ch = i & 7;
        const uint4 a = *reinterpret_cast<const uint4 *>(qp + sw_off(dh, R, ch));
        const uint4 c = *reinterpret_cast<const uint4 *>(qn + sw_off(dh, R, ch));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
        const uint32_t xw[4] = {x[i].x, x[i].y, x[i].z, x[i].w}, yw[4] = {y[i].x, y[i].y, y[i].z, y[i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            ap = fma_bf16_lo(aw[e], xw[e], ap);
            an = fma_bf16_lo(cw[e], yw[e], an);
            ap = fma_bf16_hi(aw[e], xw[e], ap);
            an = fma_bf16_hi(cw[e], yw[e], an);
        }
    }
    return __fmul_rn(__fadd_rn(ap, an), scale);
}

// canonical Quest score with the bf16 envelope copies read from L2 one 64-column
// slab at a time (head dim 256: the whole rows would take 256 registers)
template <int D>
__device__ __forceinline__ float exact_quest_l2c(const uint8_t *qp, const uint8_t *qn, const __nv_bfloat16 *kmax,
                                                 const __nv_bfloat16 *kmin, int R, float scale) {
    const uint4 *px = reinterpret_cast<const uint4 *>(kmax);
    const uint4 *py = reinterpret_cast<const uint4 *>(kmin);
    float ap = 0.f, an = 0.f;
#pragma unroll 1
    for (int dh = 0; dh < D / 64; ++dh) {
        uint4 x[8], y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x[i] = __ldg(px + dh * 8 + i);
            y[i] = __ldg(py + dh * 8 + i);
        }
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 a = *reinterpret_cast<const uint4 *>(qp + sw_off(dh, R, ch));
            const uint4 c = *reinterpret_cast<const uint4 *>(qn + sw_off(dh, R, ch));
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
            const uint32_t xw[4] = {x[ch].x, x[ch].y, x[ch].z, x[ch].w};
            const uint32_t yw[4] = {y[ch].x, y[ch].y, y[ch].z, y[ch].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ap = fma_bf16_lo(aw[e], xw[e], ap);
                an = fma_bf16_lo(cw[e], yw[e], an);
                ap = fma_bf16_hi(aw[e], xw[e], ap);
                an = fma_bf16_hi(cw[e], yw[e], an);
            }
        }
    }
    return __fmul_rn(__fadd_rn(ap, an), scale);
}

// canonical mean score with the fp32 mean read from L2, one 64-element half's
// loads issued before its chain
template <int D>
__device__ __forceinline__ float exact_mean_l2(const uint8_t *q, const float *km, int R, float scale) {
    const float4 *pk = reinterpret_cast<const float4 *>(km);
    float acc = 0.f;
#pragma unroll 1
    for (int dh = 0; dh < D / 64; ++dh) {
        float4 x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = __ldg(pk + dh * 16 + i);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 a = *reinterpret_cast<const uint4 *>(q + sw_off(dh, R, ch));
            const float xs[8] = {x[2 * ch].x, x[2 * ch].y, x[2 * ch].z, x[2 * ch].w,
                                 x[2 * ch + 1].x, x[2 * ch + 1].y, x[2 * ch + 1].z, x[2 * ch + 1].w};
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc = __fmaf_rn(bf_lo(aw[e]), xs[2 * e], acc);
                acc = __fmaf_rn(bf_hi(aw[e]), xs[2 * e + 1], acc);
            }
        }
    }
    return __fmul_rn(acc, scale);
}

// canonical mean score, query row R of the Q buffer, fp32 mean from global memory
template <int D>
__device__ __forceinline__ float exact_mean_global(const uint8_t *q, const float *km, int R, float scale) {
    float acc = 0.f;
#pragma unroll 1
    for (int dh = 0; dh < D / 64; ++dh) {
#pragma unroll 2
        for (int ch = 0; ch < 8; ++ch) {
            const uint4 a = *reinterpret_cast<const uint4 *>(q + sw_off(dh, R, ch));
            const int d0 = dh * 64 + ch * 8;
            const float4 x0 = __ldg(reinterpret_cast<const float4 *>(km + d0));
            const float4 x1 = __ldg(reinterpret_cast<const float4 *>(km + d0 + 4));
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc = __fmaf_rn(bf_lo(aw[e]), xs[2 * e], acc);
                acc = __fmaf_rn(bf_hi(aw[e]), xs[2 * e + 1], acc);
            }
        }
    }
    return __fmul_rn(acc, scale);
}

__device__ __forceinline__ uint32_t ord_key(float v) {
    v = __fadd_rn(v, 0.0f);
    if (v != v) return 0xffffffffu;
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_val(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// TWO_PASS (when the per-tile arrays fit in shared memory): pass 1 runs the
// tensor-core GEMM over the summary chunks and keeps, per (tile, block), a
// rigorous interval [lo, hi] of the exact tile score and the row(s) that may
// hold it; each tile takes theta = a lower bound of the kmax-th largest lo
// among its visible blocks (radix selection); pass 2 evaluates the exact fp32
// score only for blocks with hi >= theta -- the others cannot be in the
// tile's top kmax and get -inf.  Pass 2 runs per warp with no synchronisation:
// the summary rows of 16 candidates at a time are copied from L2 into the
// freed envelope stages (cp.async, coalesced) while the previous 16 are
// evaluated.  Without TWO_PASS every visible block is evaluated in the GEMM's
// epilogue from the staged envelopes.
template <int D, bool QUEST, bool TWO_PASS>
__global__ void __launch_bounds__(kScoreThreads, 1)
    score_exact_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK0,
                       const __grid_constant__ CUtensorMap mapK1, const TcParams p) {
    using L = TcLayout<D, QUEST>;
    constexpr int DH = L::DH;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ0 = smem + L::OFF_Q0;
    uint8_t *sQ1 = smem + L::OFF_Q1;
    uint8_t *sK = smem + L::OFF_K;
    // TWO_PASS per (tile, block): lower-bound key, width of the bound interval, row code
    uint32_t *sL = reinterpret_cast<uint32_t *>(smem + L::SMEM);                   // [2][NB]
    __half *sW = reinterpret_cast<__half *>(sL + (TWO_PASS ? 2 * p.NB : 0));       // [2][NB]
    uint8_t *sC = reinterpret_cast<uint8_t *>(sW + (TWO_PASS ? 2 * p.NB : 0));     // [2][NB]

    __shared__ uint64_t bar_q, bar_kfull[2], bar_kempty[2], bar_afull[2], bar_aempty[2], bar_prep, bar_done,
        bar_grp[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ float s_sq[128];
    __shared__ float s_qn[128];
    __shared__ uint32_t s_prefix[2], s_mask[2];
    __shared__ int s_k[2];
    __shared__ uint32_t s_kmn[8], s_kmx[8];      // per-warp key range
    __shared__ uint32_t s_other[8][32];          // per warp: blocks with several rows / fp32 envelopes

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x;
    const int pr = p.npairs - 1 - (item % p.npairs);   // heavy pairs first
    const int bh = item / p.npairs;
    const int h = bh % p.Hq, b = bh / p.Hq;
    const int kvh = h / (p.Hq / p.Hkv);
    const int t0 = 2 * pr;   // local tile (row coordinate in Q)
    const int ntiles = (t0 + 1 < p.Qt) ? 2 : 1;
    const int t_last = seq_tile(t0, p.t_base, p.pair_stride) + ntiles - 1;
    const int self_last = min(t_last * 64 + 63, p.S - 1) / 64;
    const int nchunks = (self_last + 1 + 127) / 128;

    if (threadIdx.x == 0) {
        mbar_init(&bar_q, 1);
        mbar_init(&bar_prep, 8);
        mbar_init(&bar_done, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar_kfull[i], 1);
            // the MMA commit, or the 8 epilogue warps (D = 256 reads no stage in the epilogue)
            mbar_init(&bar_kempty[i], (TWO_PASS || D > 128) ? 1 : 8);
            mbar_init(&bar_afull[i], 1);
            mbar_init(&bar_aempty[i], 8);
            mbar_init(&bar_grp[i], 4);
        }
        fence_barrier_init();
        s_abort = 0;
    }
    if (warp == 9) {
        tmem_alloc(&s_tmem, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const WaitCtx wc{p.err, &s_abort};

    if (warp == 8) {
        if (lane == 0) {
            // ---- producer: the two query tiles, then the summary chunks
            mbar_arrive_expect_tx(&bar_q, 2 * 64 * D * 2);
            for (int j = 0; j < 2; ++j)
                for (int dh = 0; dh < DH; ++dh)
                    tma_load_4d(sQ0 + dh * 16384 + j * 8192, &mapQ, &bar_q, 64 * dh, (t0 + j) * 64, h, b);
            bool ok = true;
            int issued = -1;
            if constexpr (D > 128) {
                // one 64-column slab of both operands per stage: stage use g = chunk * DH + dh
                for (int g = 0; g < nchunks * DH && ok; ++g) {
                    const int s = g & 1, c = g / DH, dh = g % DH;
                    ok = mbar_wait(&bar_kempty[s], ((g >> 1) & 1) ^ 1, wc);
                    if (!ok) break;
                    uint8_t *dst = sK + s * 2 * L::K_BYTES;
                    mbar_arrive_expect_tx(&bar_kfull[s], 2 * 128 * 64 * 2);
                    tma_load_4d(dst, &mapK0, &bar_kfull[s], 64 * dh, c * 128, kvh, b);
                    tma_load_4d(dst + L::K_BYTES, &mapK1, &bar_kfull[s], 64 * dh, c * 128, kvh, b);
                    issued = g;
                }
            } else {
                for (int g = 0; g < nchunks && ok; ++g) {
                    const int s = g & 1, c = g;
                    ok = mbar_wait(&bar_kempty[s], ((g >> 1) & 1) ^ 1, wc);
                    if (!ok) break;
                    uint8_t *dst = sK + s * 2 * L::K_BYTES;
                    mbar_arrive_expect_tx(&bar_kfull[s], 2 * 128 * D * 2);
                    for (int dh = 0; dh < DH; ++dh) {
                        tma_load_4d(dst + dh * 16384, &mapK0, &bar_kfull[s], 64 * dh, c * 128, kvh, b);
                        tma_load_4d(dst + L::K_BYTES + dh * 16384, &mapK1, &bar_kfull[s], 64 * dh, c * 128, kvh,
                                    b);
                    }
                    issued = g;
                }
            }
            if (!ok) {
                mbar_wait_drain(&bar_q, 0, p.err);
                if (issued >= 0) mbar_wait_drain(&bar_kfull[issued & 1], (issued >> 1) & 1, p.err);
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            // ---- MMA issuer (pass 1)
            constexpr uint32_t idesc = idesc_f16(128, 128, 1, 0, 0);
            const uint32_t aQ0 = smem_u32(sQ0), aQ1 = smem_u32(QUEST ? sQ1 : sQ0), aK = smem_u32(sK);
            bool ok = mbar_wait(&bar_prep, 0, wc);   // Q+/Q- written by the epilogue warps
            if constexpr (D > 128) {
                // a chunk accumulates over DH slab stages, each freed once its MMAs have read it
                for (int c = 0; c < nchunks && ok; ++c) {
                    const int a = c & 1;
                    ok = mbar_wait(&bar_aempty[a], ((c >> 1) & 1) ^ 1, wc);
                    if (!ok) break;
                    const uint32_t acc = tmem + a * 128;
                    for (int dh = 0; dh < DH && ok; ++dh) {
                        const int g = c * DH + dh, s = g & 1;
                        ok = mbar_wait(&bar_kfull[s], (g >> 1) & 1, wc);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t k0 = aK + s * 2 * L::K_BYTES, k1 = k0 + L::K_BYTES;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_f16_ss(acc, smem_desc_sw128(k0 + kk * 32, 16, 1024),
                                        smem_desc_sw128(aQ0 + dh * 16384 + kk * 32, 16, 1024), idesc,
                                        (dh > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_f16_ss(acc, smem_desc_sw128(k1 + kk * 32, 16, 1024),
                                        smem_desc_sw128(aQ1 + dh * 16384 + kk * 32, 16, 1024), idesc, 1u);
                        umma_commit(&bar_kempty[s]);
                    }
                    if (ok) umma_commit(&bar_afull[a]);
                }
            }
            for (int c = 0; c < nchunks && ok && D <= 128; ++c) {
                const int s = c & 1, a = c & 1;
                ok = mbar_wait(&bar_kfull[s], (c >> 1) & 1, wc);
                if (!ok) break;
                ok = mbar_wait(&bar_aempty[a], ((c >> 1) & 1) ^ 1, wc);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc = tmem + a * 128;
                const uint32_t k0 = aK + s * 2 * L::K_BYTES, k1 = k0 + L::K_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4 * DH; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_f16_ss(acc, smem_desc_sw128(k0 + off, 16, 1024), smem_desc_sw128(aQ0 + off, 16, 1024), idesc,
                                kk > 0 ? 1u : 0u);
                }
#pragma unroll
                for (int kk = 0; kk < 4 * DH; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_f16_ss(acc, smem_desc_sw128(k1 + off, 16, 1024), smem_desc_sw128(aQ1 + off, 16, 1024), idesc,
                                1u);
                }
                umma_commit(&bar_afull[a]);                 // the epilogue frees the accumulator
                if (TWO_PASS) umma_commit(&bar_kempty[s]);  // stage free once the MMAs have read it
            }
            umma_commit(&bar_done);
            mbar_wait_drain(&bar_done, 0, p.err);
        }
    } else {
        // ---- epilogue warps 0-7.  Prepare Q+/Q- and the row norms first:
        // 16-byte chunk idx = k * 256 + tid is chunk idx & 7 of row (idx >> 3) & 127
        // in half idx >> 10: a warp reads and writes 512 contiguous bytes (no bank
        // conflicts; a thread per row would put all 32 lanes on the same banks),
        // and the 8 chunks of a row in each half fall to one group of 8 lanes,
        // which sum the row's squares (the norm only feeds a padded error bound,
        // so its summation order is free).
        bool ok = __all_sync(0xffffffffu, mbar_wait(&bar_q, 0, wc));
        const int tid = threadIdx.x;
        {
            float sq[4] = {0.f, 0.f, 0.f, 0.f};   // rows (k * 32 + tid / 8) & 127, k = 0..3
            if (ok) {
#pragma unroll
                for (int k = 0; k < 4 * DH; ++k) {
                    const int idx = k * 256 + tid;
                    const int ch = idx & 7, row = (idx >> 3) & 127, dh = idx >> 10;
                    uint8_t *base0 = sQ0 + dh * 16384 + row * 128 + ch * 16;   // swizzle: elementwise, ignore
                    uint8_t *base1 = sQ1 + dh * 16384 + row * 128 + ch * 16;
                    const uint4 v = *reinterpret_cast<uint4 *>(base0);
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                    uint32_t pos[4], neg[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = bf_lo(w[e]), hi = bf_hi(w[e]);
                        sq[k & 3] = fmaf(lo, lo, sq[k & 3]);
                        sq[k & 3] = fmaf(hi, hi, sq[k & 3]);
                        const uint32_t plo = (w[e] & 0x8000u) ? 0u : (w[e] & 0xffffu);
                        const uint32_t phi = (w[e] & 0x80000000u) ? 0u : (w[e] & 0xffff0000u);
                        const uint32_t nlo = (w[e] & 0x8000u) ? (w[e] & 0xffffu) : 0u;
                        const uint32_t nhi = (w[e] & 0x80000000u) ? (w[e] & 0xffff0000u) : 0u;
                        pos[e] = plo | phi;
                        neg[e] = nlo | nhi;
                    }
                    if (QUEST) {
                        *reinterpret_cast<uint4 *>(base0) = make_uint4(pos[0], pos[1], pos[2], pos[3]);
                        *reinterpret_cast<uint4 *>(base1) = make_uint4(neg[0], neg[1], neg[2], neg[3]);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) sq[k] += __shfl_xor_sync(0xffffffffu, sq[k], off);
                if ((tid & 7) == 0) s_sq[(k * 32 + (tid >> 3)) & 127] = sq[k];
            }
        }
        if (QUEST) fence_proxy_async_smem();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (tid < 128) s_qn[tid] = sqrtf(s_sq[tid]) * kNormPad;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (lane == 0) mbar_arrive(&bar_prep);

        const int grp = warp >> 2;                 // warp group: tile grp of the pair
        const int sp = warp & 3;                   // TMEM subpartition
        const int lb = sp * 32 + lane;             // block row of the chunk
        const int gtid = sp * 32 + lane;           // thread index within the group
        const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
        // largest row norm of this group's tile (NaN norms dropped, as fmaxf does)
        float qm;
        {
            const float a = s_qn[grp * 64 + lane], c = s_qn[grp * 64 + 32 + lane];
            const float m = fmaxf(fmaxf(a, c), 0.f);
            qm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
        }
        const int t = t0 + grp;   // local tile
        const bool have_tile = grp < ntiles;
        const int self_t = have_tile ? min(seq_tile(t, p.t_base, p.pair_stride) * 64 + 63, p.S - 1) / 64 : -1;
        const int nvis = self_t + 1;
        const float2 *nrm = p.norms + ((int64_t)b * p.Hkv + kvh) * p.NB;
        const float *A = p.summ_a + ((int64_t)b * p.Hkv + kvh) * p.NB * D;
        const float *Bm = QUEST ? p.summ_b + ((int64_t)b * p.Hkv + kvh) * p.NB * D : nullptr;
        float *out = p.escore + (((int64_t)b * p.Hq + h) * p.Qt + t) * p.NB;
        uint32_t *tL = sL + grp * p.NB;
        __half *tW = sW + grp * p.NB;
        uint8_t *tC = sC + grp * p.NB;
        uint32_t key_min = 0xffffffffu, key_max = 0u;   // over this thread's non-forced blocks

        // exact tile score of block blk from the staged envelopes (stage base),
        // evaluating the rows in mask cm
        auto exact_tile = [&](const uint8_t *stage, int blk, uint64_t cm, bool exact_ops) -> float {
            float best = -INFINITY;
            while (cm) {
                const int r = __ffsll((long long)cm) - 1;
                cm &= cm - 1;
                const int R = grp * 64 + r;
                float s;
                if (QUEST) {
                    s = exact_ops ? exact_quest_smem<D>(sQ0, sQ1, stage, stage + L::K_BYTES, R, lb, p.scale)
                                  : exact_quest_global<D>(sQ0, sQ1, Bm + (int64_t)blk * D, A + (int64_t)blk * D, R,
                                                          p.scale);
                } else {
                    s = exact_mean_global<D>(sQ0, A + (int64_t)blk * D, R, p.scale);
                }
                best = (s > best) ? s : best;
            }
            return best;
        };

        // ---- pass 1 (and the only pass without TWO_PASS)
        for (int c = 0; c < nchunks && ok; ++c) {
            const int a = c & 1;
            const int blk = c * 128 + lb;
            const float2 kn = (have_tile && blk <= self_t) ? __ldg(nrm + blk) : make_float2(0.f, 0.f);
            ok = __all_sync(0xffffffffu, mbar_wait(&bar_afull[a], (c >> 1) & 1, wc));
            if (!ok) break;
            tc_fence_after();
            if (have_tile) {
                uint32_t v[64];
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    tmem_ld16(tmem + a * 128 + grp * 64 + q4 * 16 + lane_base,
                              *reinterpret_cast<uint32_t(*)[16]>(&v[q4 * 16]));
                tmem_wait_ld();
                reg_fence(v);
                if (blk <= self_t) {
                    // approximate tile max (NaN dropped; all-NaN gives NaN = non-finite),
                    // three-input maxima: 32 instructions for the 64 rows
                    float m22[22], m8[8];
#pragma unroll
                    for (int r = 0; r < 21; ++r)
                        m22[r] = fmax3f(__uint_as_float(v[3 * r]), __uint_as_float(v[3 * r + 1]),
                                        __uint_as_float(v[3 * r + 2]));
                    m22[21] = __uint_as_float(v[63]);
#pragma unroll
                    for (int r = 0; r < 7; ++r) m8[r] = fmax3f(m22[3 * r], m22[3 * r + 1], m22[3 * r + 2]);
                    m8[7] = m22[21];
                    const float T = fmax3f(fmax3f(m8[0], m8[1], m8[2]), fmax3f(m8[3], m8[4], m8[5]),
                                           fmaxf(m8[6], m8[7]));
                    // D = 256: the tensor core sums twice the terms, twice the allowance
                    const float eps = qm * fmaf(kTcRelErr * (D > 128 ? 2.f : 1.f), kn.x, kn.y) * kNormPad;
                    const float thr = __fsub_rd(T, 2.f * eps);
                    const bool finite = isfinite(T) && isfinite(eps);
                    // rows that may hold the exact maximum (the approximate argmax among them)
                    uint32_t m_lo = 0u, m_hi = 0u;
#pragma unroll
                    for (int r = 0; r < 32; ++r) {
                        m_lo |= (__uint_as_float(v[r]) >= thr) ? (1u << r) : 0u;
                        m_hi |= (__uint_as_float(v[r + 32]) >= thr) ? (1u << r) : 0u;
                    }
                    uint64_t cm = finite ? (((uint64_t)m_hi << 32) | m_lo) : ~0ull;
                    if (TWO_PASS) {
                        // exact tile score in [lo, hi]; key 0 (below every finite key) marks a
                        // non-finite block, always a candidate.  The width is rounded up, so
                        // lo + width (rounded up) >= hi.
                        const float lo = __fmul_rd(__fsub_rd(T, eps), p.scale);
                        const float hi = __fmul_ru(__fadd_ru(T, eps), p.scale);
                        const uint32_t key = finite ? ord_key(lo) : 0u;
                        tL[blk] = key;
                        tW[blk] = __float2half_ru(__fsub_ru(hi, lo));
                        // code: bit 7 several rows, bit 6 fp32 Quest envelopes needed, bits 0-5 the row
                        const uint8_t f32 = (QUEST && kn.y != 0.f) ? 64 : 0;
                        tC[blk] = (__popcll(cm) == 1) ? (uint8_t)((__ffsll((long long)cm) - 1) | f32)
                                                      : (uint8_t)(128 | f32);
                        if (blk != 0 && blk != self_t) {
                            key_min = min(key_min, key);
                            key_max = max(key_max, key);
                        }
                    } else {
                        // envelopes exact in bf16 and staged whole (D = 256 stages one slab at a
                        // time: its chains read the fp32 summaries)
                        const bool exact_ops = D <= 128 && QUEST && kn.y == 0.f;
                        out[blk] = exact_tile(sK + a * 2 * L::K_BYTES, blk, cm, exact_ops);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bar_aempty[a]);                  // accumulator
                // envelope stage (freed by the MMA in TWO_PASS and at D = 256)
                if (!TWO_PASS && D <= 128) mbar_arrive(&bar_kempty[a]);
            }
        }
        // bounded barrier over the 4 warps of this group
        uint32_t gphase = 0;
        auto group_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_grp[grp]);
            const bool r = __all_sync(0xffffffffu, mbar_wait(&bar_grp[grp], gphase, wc));
            gphase ^= 1u;
            return r;
        };
        if (TWO_PASS && ok) {
            // ---- theta: a lower bound of the kmax-th largest lower bound among
            // the tile's visible blocks (the two forced blocks take their slots
            // first).  Radix selection over the ordered keys, starting at the
            // first bit where the group's smallest and largest key differ and
            // stopping once the bin holding theta has at most 16 keys: the
            // bin's lower edge is then theta, a few extra candidates at most.
            key_min = __reduce_min_sync(0xffffffffu, key_min);
            key_max = __reduce_max_sync(0xffffffffu, key_max);
            if (lane == 0) {
                s_kmn[warp] = key_min;
                s_kmx[warp] = key_max;
            }
            ok = group_sync();
            uint32_t theta = 0u;   // 0: every visible block is a candidate
            if (ok && have_tile && nvis > p.kmax) {
                uint32_t kmn = 0xffffffffu, kmx = 0u;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    kmn = min(kmn, s_kmn[grp * 4 + w]);
                    kmx = max(kmx, s_kmx[grp * 4 + w]);
                }
                const int nforced = (self_t == 0) ? 1 : 2;
                int k = p.kmax - nforced;   // rank among the non-forced blocks
                if (k <= 0) {
                    theta = 0xffffffffu;
                } else if (kmn == kmx) {
                    theta = kmn;
                } else {
                    int lowbit = 32 - __clz(kmn ^ kmx);   // bits below are not yet fixed
                    uint32_t prefix = (uint32_t)((unsigned long long)kmx & (~0ull << lowbit));
                    // a histogram per warp, in the warp's own pass-2 staging area of the
                    // envelope stages (every MMA and copy has completed; no other warp
                    // uses that area): no cross-warp atomics, no barrier to clear it
                    uint32_t *whist = reinterpret_cast<uint32_t *>(
                        sK + (D <= 128 ? warp * 2 * (16 * 4 * D) : warp * 1024));
                    while (ok) {
                        const int shift = max(lowbit - 8, 0);
                        const uint32_t nb = 1u << (lowbit - shift);
                        const uint32_t himask = (uint32_t)(~0ull << lowbit);
                        for (int i = lane; i < 256; i += 32) whist[i] = 0u;
                        __syncwarp();
                        for (int j = gtid; j < nvis; j += 128) {
                            const uint32_t u = tL[j];
                            if (j != 0 && j != self_t && (u & himask) == prefix)
                                atomicAdd(&whist[(nb - 1u) - ((u >> shift) & (nb - 1u))], 1u);
                        }
                        ok = group_sync();
                        if (!ok) break;
                        if (gtid < 32) {
                            const uint32_t *h0 = reinterpret_cast<const uint32_t *>(
                                sK + (D <= 128 ? (grp * 4) * 2 * (16 * 4 * D) : (grp * 4) * 1024));
                            const int wstride = D <= 128 ? 2 * (16 * 4 * D) / 4 : 256;   // words between warps
                            uint32_t cc[8], sum = 0;
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                uint32_t c = 0u;
#pragma unroll
                                for (int w = 0; w < 4; ++w) c += h0[w * wstride + 8 * gtid + e];
                                cc[e] = c;
                                sum += c;
                            }
                            uint32_t incl = sum;
#pragma unroll
                            for (int off = 1; off < 32; off <<= 1) {
                                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
                                if (gtid >= off) incl += y;
                            }
                            const uint32_t excl = incl - sum;
                            if (excl < (uint32_t)k && (uint32_t)k <= incl) {
                                uint32_t run = excl, selc = 0;
                                int bin = 8 * gtid + 7;
#pragma unroll
                                for (int e = 0; e < 8; ++e) {
                                    if (run + cc[e] >= (uint32_t)k) {
                                        bin = 8 * gtid + e;
                                        selc = cc[e];
                                        break;
                                    }
                                    run += cc[e];
                                }
                                s_k[grp] = (int)((uint32_t)k - run);
                                s_prefix[grp] = prefix | (((nb - 1u) - (uint32_t)bin) << shift);
                                s_mask[grp] = selc;
                            }
                        }
                        ok = group_sync();
                        if (!ok) break;
                        prefix = s_prefix[grp];
                        k = s_k[grp];
                        lowbit = shift;
                        if (s_mask[grp] <= 16u || shift == 0) break;
                    }
                    theta = prefix;
                }
            }
            // ---- pass 2, per warp over its own blocks (those of lane 0..31 in
            // each 128-block step), no synchronisation with the other warps.
            // Every MMA has completed (each accumulator was consumed) and no
            // copy is in flight, so the envelope stages become two staging
            // buffers per warp.  Candidates with one possible row and
            // bf16-exact envelopes (or a mean summary) are gathered 16 at a
            // time; the next batch's summary rows are copied from L2 with
            // coalesced 16-byte cp.async while the current batch is evaluated
            // from shared memory (Quest: lane pairs run the Q+ and Q- chains).
            // Blocks with several possible rows or fp32 Quest envelopes are
            // evaluated by the whole warp as they are met.
            // 16-byte chunks per candidate, candidates per copy (two-pass runs at D <= 128)
            constexpr int CPC = D / 4, CPI = CPC <= 32 ? 32 / CPC : 1;
            constexpr int kBatch = 16;
            constexpr int kBuf = kBatch * 4 * D;         // bytes per staging buffer
            static_assert(!TWO_PASS || D > 128 || 8 * 2 * kBuf <= L::STAGES * 2 * L::K_BYTES,
                          "staging exceeds the envelope stages");
            uint8_t *stg = sK + warp * 2 * kBuf;
            const uint32_t lt_mask = (1u << lane) - 1u;
            const __nv_bfloat16 *O0 = p.op0 + ((int64_t)b * p.Hkv + kvh) * p.NB * D;
            const __nv_bfloat16 *O1 = p.op1 + ((int64_t)b * p.Hkv + kvh) * p.NB * D;
            auto exact_at = [&](int R, int bk, bool f32) -> float {
                if (QUEST) {
                    if (!f32 && D > 128)
                        return exact_quest_l2c<D>(sQ0, sQ1, O0 + (int64_t)bk * D, O1 + (int64_t)bk * D, R, p.scale);
                    if (!f32)
                        return exact_quest_l2<D>(sQ0, sQ1, O0 + (int64_t)bk * D, O1 + (int64_t)bk * D, R, p.scale);
                    return exact_quest_global<D>(sQ0, sQ1, Bm + (int64_t)bk * D, A + (int64_t)bk * D, R, p.scale);
                }
                return exact_mean_l2<D>(sQ0, A + (int64_t)bk * D, R, p.scale);
            };
            // the whole warp evaluates block bk over the rows in mask (lo, hi) and
            // keeps the oracle's running max over rows in order: NaN never
            // replaces, and of equal values (only +-0 differ in bits) the lowest row's
            auto warp_exact = [&](int bk, uint64_t rows, bool f32) {
                unsigned long long key = (unsigned long long)ord_key(-INFINITY) << 32;
#pragma unroll 1
                for (int r = lane; r < 64; r += 32) {
                    if (!((rows >> r) & 1ull)) continue;
                    const float sc = exact_at(grp * 64 + r, bk, f32);
                    if (sc == sc) {
                        const unsigned long long kk = ((unsigned long long)ord_key(sc) << 32) |
                                                      ((uint32_t)(63 - r) << 1) | (__float_as_uint(sc) >> 31);
                        key = kk > key ? kk : key;
                    }
                }
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) {
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
                    key = o > key ? o : key;
                }
                if (lane == 0) {
                    float r = ord_val((uint32_t)(key >> 32));
                    if (r == 0.f && (key & 1ull)) r = -0.f;
                    out[bk] = r;
                }
            };
            // scan, per warp, all of its steps (32 blocks each) in one unrolled
            // pass: forced and provably-out blocks get their outputs, the rare
            // blocks with several rows or fp32 envelopes are evaluated by the
            // warp, and the fast candidates (block << 6 | row) are listed in the
            // warp's own slots of the lower-bound array, which theta no longer
            // needs: entry k goes to the slot of step k / 32, lane k % 32, a step
            // this warp has already read.
            const int nsteps = have_tile ? (nvis + 127) / 128 : 0;
            auto slot = [&](int k) -> int { return (k >> 5) * 128 + sp * 32 + (k & 31); };
            int nf = 0;   // fast candidates listed
            int no = 0;   // rare blocks listed in s_other[warp]
            for (int s0 = 0; s0 < nsteps; s0 += 4) {
                uint32_t fm[4], om[4], oc[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = (s0 + u) * 128 + sp * 32 + lane;
                    bool fast = false, other = false;
                    uint32_t code = 0u;
                    if (j < nvis) {
                        if (j == 0 || j == self_t) {
                            out[j] = FLT_MAX;
                        } else {
                            const uint32_t lk = tL[j];
                            // upper bound of the exact score (NaN when lo = -inf: a candidate)
                            const bool cand =
                                lk == 0u || ord_key(__fadd_ru(ord_val(lk), __half2float(tW[j]))) >= theta;
                            if (!cand) {
                                out[j] = -INFINITY;   // provably outside the tile's top kmax
                            } else {
                                code = tC[j];
                                fast = code < 64u;
                                other = !fast;
                            }
                        }
                    }
                    oc[u] = code;
                    fm[u] = __ballot_sync(0xffffffffu, fast);
                    om[u] = __ballot_sync(0xffffffffu, other);
                }
                __syncwarp();   // the four steps' slots are read before any is overwritten
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if ((fm[u] >> lane) & 1u) {
                        const int j = (s0 + u) * 128 + sp * 32 + lane;
                        tL[slot(nf + __popc(fm[u] & lt_mask))] = ((uint32_t)j << 6) | oc[u];
                    }
                    nf += __popc(fm[u]);
                    // the rare blocks are listed and evaluated after the fast batches
                    // (evaluated right here only when the short list is full)
                    if (no + __popc(om[u]) <= 32) {
                        if ((om[u] >> lane) & 1u)
                            s_other[warp][no + __popc(om[u] & lt_mask)] =
                                ((uint32_t)((s0 + u) * 128 + sp * 32 + lane) << 8) | oc[u];
                        no += __popc(om[u]);
                    } else {
                        uint32_t oth = om[u];
                        while (oth) {
                            const int src = __ffs(oth) - 1;
                            oth &= oth - 1u;
                            const uint32_t c2 = __shfl_sync(0xffffffffu, oc[u], src);
                            const uint64_t rows = (c2 & 128u) ? ~0ull : (1ull << (c2 & 63u));
                            warp_exact((s0 + u) * 128 + sp * 32 + src, rows, (c2 & 64u) != 0u);
                        }
                    }
                }
            }
            __syncwarp();
            if constexpr (D <= 128) {
                // batch k0 .. k0 + 15 of the list: lane c < n holds entry c
                auto entry = [&](int k0, int n) -> uint32_t { return lane < n ? tL[slot(k0 + lane)] : 0u; };
                // copies the summary rows of a batch into staging buffer buf
                auto stage = [&](int buf, uint32_t ent, int n) {
                    uint8_t *sb = stg + buf * kBuf;
    #pragma unroll
                    for (int i = 0; i < kBatch / CPI; ++i) {
                        const int c = i * CPI + lane / CPC, x = lane % CPC;
                        const int bk = (int)(__shfl_sync(0xffffffffu, ent, c) >> 6);
                        if (c < n) {
                            const void *src;
                            if (QUEST) src = ((x < D / 8) ? O0 : O1) + (int64_t)bk * D + (x % (D / 8)) * 8;
                            else src = A + (int64_t)bk * D + x * 4;
                            cp_async16(sb + c * 4 * D + ((x ^ (c & 7)) << 4), src);
                        }
                    }
                    cp_async_commit();
                };
                // evaluates a batch from staging buffer buf
                auto evaluate = [&](int buf, uint32_t ent, int n) {
                    const uint8_t *sb = stg + buf * kBuf;
                    if (QUEST) {
                        const int c = lane >> 1, half = lane & 1;
                        const uint32_t e = __shfl_sync(0xffffffffu, ent, c);
                        float acc = 0.f;
                        if (c < n) {
                            const int R = grp * 64 + (int)(e & 63u);
                            const uint8_t *qs = half ? sQ1 : sQ0;
                            const uint8_t *ks = sb + c * 4 * D;
    #pragma unroll
                            for (int i = 0; i < D / 8; ++i) {
                                const uint4 a = *reinterpret_cast<const uint4 *>(qs + sw_off(i >> 3, R, i & 7));
                                const uint4 xv =
                                    *reinterpret_cast<const uint4 *>(ks + (((half * (D / 8) + i) ^ (c & 7)) << 4));
                                const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
    #pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    acc = fma_bf16_lo(aw[q], xw[q], acc);
                                    acc = fma_bf16_hi(aw[q], xw[q], acc);
                                }
                            }
                        }
                        const float an = __shfl_xor_sync(0xffffffffu, acc, 1);
                        if (c < n && half == 0) out[e >> 6] = __fmul_rn(__fadd_rn(acc, an), p.scale);
                    } else if (lane < n) {
                        const int c = lane;
                        const uint32_t e = ent;
                        const int R = grp * 64 + (int)(e & 63u);
                        const uint8_t *ks = sb + c * 4 * D;
                        float acc = 0.f;
    #pragma unroll
                        for (int i = 0; i < D / 8; ++i) {
                            const uint4 a = *reinterpret_cast<const uint4 *>(sQ0 + sw_off(i >> 3, R, i & 7));
                            const float4 x0 = *reinterpret_cast<const float4 *>(ks + (((2 * i) ^ (c & 7)) << 4));
                            const float4 x1 = *reinterpret_cast<const float4 *>(ks + (((2 * i + 1) ^ (c & 7)) << 4));
                            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                            const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    #pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                acc = __fmaf_rn(bf_lo(aw[q]), xs[2 * q], acc);
                                acc = __fmaf_rn(bf_hi(aw[q]), xs[2 * q + 1], acc);
                            }
                        }
                        out[e >> 6] = __fmul_rn(acc, p.scale);
                    }
                };
                int cur = 0;
                int n_cur = min(kBatch, nf);
                uint32_t e_cur = entry(0, n_cur);
                stage(0, e_cur, n_cur);
                for (int k0 = 0; k0 < nf; k0 += kBatch) {
                    const int n_next = min(kBatch, nf - (k0 + kBatch));
                    const uint32_t e_next = entry(k0 + kBatch, n_next);
                    stage(cur ^ 1, e_next, n_next);
                    cp_async_wait_group1();   // the current batch has landed
                    __syncwarp();
                    evaluate(cur, e_cur, n_cur);
                    __syncwarp();             // this buffer is refilled next
                    cur ^= 1;
                    n_cur = n_next;
                    e_cur = e_next;
                }
                cp_async_wait_all();
            } else {
                // head dim 256: a lane per candidate, 32 at a time, the candidate's summary
                // row read from L2 in slabs (its staging would not fit the envelope stages)
                for (int k0 = 0; k0 < nf; k0 += 32) {
                    if (k0 + lane < nf) {
                        const uint32_t e = tL[slot(k0 + lane)];
                        out[e >> 6] = exact_at(grp * 64 + (int)(e & 63u), (int)(e >> 6), false);
                    }
                }
                __syncwarp();
            }
            for (int k = 0; k < no; ++k) {
                const uint32_t e = s_other[warp][k], c2 = e & 255u;
                const uint64_t rows = (c2 & 128u) ? ~0ull : (1ull << (c2 & 63u));
                warp_exact((int)(e >> 8), rows, (c2 & 64u) != 0u);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ---------------------------------------------------------------- kernel B
struct RankParams {
    int B, Hq, S, NB, Qt, NBpad;
    int t_base, pair_stride;   // local tile t is sequence tile seq_tile(t, t_base, pair_stride)
    int k_base, kmax, router;
    const float *escore;
    int32_t *kv_idx;
    float *sigma_cell;
};

// smem: key32 [NBpad] u32 (value keys), sort keys [NBpad] u64
// Descending bitonic sort of keys[0 .. P) (P a power of two >= 64) by the 256
// threads of the CTA: compare-exchange distances of 32 and more go through
// shared memory, one CTA barrier each; the shorter ones run in registers with
// warp shuffles (the partner of index i is in the same warp), one barrier for
// the whole run.
__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
    return ((uint64_t)hi << 32) | lo;
}

__device__ void bitonic_desc_256(uint64_t *keys, int P) {
    const int tid = threadIdx.x;
    for (int k = 2; k <= P; k <<= 1) {
        int j = k >> 1;
        for (; j >= 32; j >>= 1) {
            for (int i = tid; i < P; i += 256) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = keys[i], y = keys[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        keys[i] = y;
                        keys[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
        for (int i0 = tid & ~31; i0 < P; i0 += 256) {   // warp-uniform loop
            const int i = i0 + (tid & 31);
            const bool has = i < P;
            uint64_t x = has ? keys[i] : 0ull;
            const bool desc = (i & k) == 0;
            for (int jj = j; jj > 0; jj >>= 1) {
                const uint64_t y = shfl_xor_u64(x, jj);
                const bool lower = (i & jj) == 0;
                x = (lower == desc) ? (x > y ? x : y) : (x < y ? x : y);
            }
            if (has) keys[i] = x;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(256) rank_kernel(const RankParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint64_t *keys = reinterpret_cast<uint64_t *>(smem_raw);
    uint32_t *key32 = reinterpret_cast<uint32_t *>(keys + (p.NBpad > 1024 ? p.NBpad : 1024));
    __shared__ uint32_t hist[256];
    // per-warp histograms of the radix passes, over the sort keys (written only after the passes)
    uint32_t(*whist)[256] = reinterpret_cast<uint32_t(*)[256]>(keys);
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k, s_n;

    const int tid = threadIdx.x;
    const int item = blockIdx.x;
    const int t = p.Qt - 1 - (item % p.Qt);
    const int bh = item / p.Qt;
    const int h = bh % p.Hq, b = bh / p.Hq;
    const int last = min(seq_tile(t, p.t_base, p.pair_stride) * 64 + 63, p.S - 1);
    const int self_blk = last / 64;
    const int nvis = self_blk + 1;
    const int64_t cell = ((int64_t)b * p.Hq + h) * p.Qt + t;
    const float *es = p.escore + cell * p.NB;

    // the visible blocks' keys: eight loads per thread issued together (the score
    // array is read once, from memory)
    for (int j0 = 0; j0 < nvis; j0 += 8 * 256) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * 256 + tid;
            v[u] = (j < nvis) ? __ldcs(es + j) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * 256 + tid;
            if (j < nvis) key32[j] = (j == 0 || j == self_blk) ? ord_key(FLT_MAX) : ord_key(v[u]);
        }
    }
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_k = p.kmax;
        s_n = 0;
    }
    __syncthreads();
    // V = kmax-th largest value key (descending radix select); all visible when nvis <= kmax
    uint32_t V = 0u;
    if (nvis > p.kmax) {
        const int lane = tid & 31, warp = tid >> 5;
        for (int shift = 24; shift >= 0; shift -= 8) {
            // a histogram per warp: no cross-warp atomics (the keys cluster in few bins)
            for (int i = lane; i < 256; i += 32) whist[warp][i] = 0u;
            __syncwarp();
            const uint32_t prefix = s_prefix, mask = s_mask;
            for (int j = tid; j < nvis; j += 256) {
                const uint32_t u = key32[j];
                if ((u & mask) == prefix) atomicAdd(&whist[warp][255u - ((u >> shift) & 255u)], 1u);
            }
            __syncthreads();
            {
                uint32_t c = 0u;
#pragma unroll
                for (int w = 0; w < 8; ++w) c += whist[w][tid];
                hist[tid] = c;
            }
            __syncthreads();
            if (tid < 32) {
                uint32_t c[8], sum = 0;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    c[e] = hist[8 * tid + e];
                    sum += c[e];
                }
                uint32_t incl = sum;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
                    if (tid >= off) incl += y;
                }
                const uint32_t excl = incl - sum;
                const uint32_t k = (uint32_t)s_k;
                if (excl < k && k <= incl) {
                    uint32_t run = excl;
                    int bin = 8 * tid + 7;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        if (run + c[e] >= k) {
                            bin = 8 * tid + e;
                            break;
                        }
                        run += c[e];
                    }
                    s_k = (int)(k - run);
                    s_prefix = prefix | ((255u - (uint32_t)bin) << shift);
                    s_mask = mask | (255u << shift);
                }
            }
            __syncthreads();
        }
        V = s_prefix;
    }
    // blocks at or above V (ties at V included), keyed for the final order (one
    // counter update per warp; the positions' order does not matter before the sort)
    {
        const int lane = tid & 31;
        for (int j0 = tid - lane; j0 < nvis; j0 += 256) {
            const int j = j0 + lane;
            const uint32_t u = (j < nvis) ? key32[j] : 0u;
            const bool in = (j < nvis) && (u >= V);
            const unsigned m = __ballot_sync(0xffffffffu, in);
            int base = 0;
            if (lane == 0 && m) base = atomicAdd(&s_n, __popc(m));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (in) keys[base + __popc(m & ((1u << lane) - 1u))] = ((uint64_t)u << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
        }
    }
    __syncthreads();
    const int n = s_n;
    int P = 64;
    while (P < n) P <<= 1;
    for (int i = n + tid; i < P; i += 256) keys[i] = 0ull;
    __syncthreads();
    bitonic_desc_256(keys, P);
    int32_t *out = p.kv_idx + cell * p.kmax;
    // slots past the visible blocks (nvis < kmax) hold the invisible ids in order
    for (int i = tid; i < p.kmax; i += 256)
        out[i] = (i < n) ? (int32_t)(0xffffffffu - (uint32_t)(keys[i] & 0xffffffffu)) : i;
    if (tid == 0) {
        float sig = __int_as_float(0x7fc00000);
        if (p.router) {
            auto val = [&](int pos) { return pos < n ? ord_val((uint32_t)(keys[pos] >> 32)) : -INFINITY; };
            const float s_top = val(0), s_km1 = val(p.k_base - 1), s_k = val(p.k_base);
            float spread = __fsub_rn(s_top, s_k);
            if (spread < 1e-6f) spread = 1e-6f;
            sig = __fdiv_rn(__fsub_rn(s_km1, s_k), spread);
        }
        p.sigma_cell[cell] = sig;
    }
}

// Diagnostic: the mixed-precision bf16 fma of the exact chains against
// __fmaf_rn of the fp32 values, for the low and high halves of n word pairs.
__global__ void bf16_fma_check_kernel(const uint32_t *a, const uint32_t *b, const float *c, float *mixed,
                                      float *ref, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t x = a[i], y = b[i];
    mixed[2 * i] = fma_bf16_lo(x, y, c[2 * i]);
    mixed[2 * i + 1] = fma_bf16_hi(x, y, c[2 * i + 1]);
    ref[2 * i] = __fmaf_rn(bf_lo(x), bf_lo(y), c[2 * i]);
    ref[2 * i + 1] = __fmaf_rn(bf_hi(x), bf_hi(y), c[2 * i + 1]);
}

int launch_check_bf16_fma(const uint32_t *a, const uint32_t *b, const float *c, float *mixed, float *ref, int n,
                          cudaStream_t stream) {
    if (n <= 0) return UGBSA_OK;
    bf16_fma_check_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a, b, c, mixed, ref, n);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

// ---------------------------------------------------------------- host
bool tc_select_supported(int dtype, int D) { return dtype == UGBSA_BF16 && (D == 64 || D == 128 || D == 256); }

static int64_t al256(int64_t x) { return (x + 255) / 256 * 256; }

size_t tc_scratch_bytes(int B, int Hq, int Hkv, int S, int D, int Qt) {
    const int64_t NB = (S + 63) / 64;
    const int64_t cells = (int64_t)B * Hq * Qt;
    return (size_t)(al256(cells * NB * 4) + 2 * al256((int64_t)B * Hkv * NB * D * 2) +
                    al256((int64_t)B * Hkv * NB * 8));
}

static int map_rows(CUtensorMap *m, const void *ptr, int D, int64_t rows_dim, int H, int B, int64_t s_stride,
                    int64_t h_stride, int64_t b_stride, int box_rows) {
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)rows_dim, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)s_stride * 2, (cuuint64_t)h_stride * 2, (cuuint64_t)b_stride * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, es);
}

template <int D, bool QUEST>
static int launch_score(const CUtensorMap &mQ, const CUtensorMap &mK0, const CUtensorMap &mK1, const TcParams &tp,
                        cudaStream_t stream) {
    using L = TcLayout<D, QUEST>;
    const size_t base = L::SMEM + 1024;
    if constexpr (D > 128) {
        // two passes when the per-tile arrays fit next to the slab stages (pass 2 reads
        // the candidates' summary rows from L2, a lane per candidate); one pass otherwise
        const size_t two = base + (size_t)2 * tp.NB * 7 + 16;
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, score_exact_kernel<D, QUEST, true>) != cudaSuccess) return UGBSA_ERR_LAUNCH;
        bool use_two = two + fa.sharedSizeBytes <= 227 * 1024;
        if (const char *e = getenv("UGBSA_SCORE_ONE_PASS")) use_two = use_two && e[0] != '1';
        const size_t smem = use_two ? two : base;
        auto kern = use_two ? score_exact_kernel<D, QUEST, true> : score_exact_kernel<D, QUEST, false>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return UGBSA_ERR_LAUNCH;
        const int64_t grid = (int64_t)tp.B * tp.Hq * tp.npairs;
        kern<<<(unsigned)grid, kScoreThreads, smem, stream>>>(mQ, mK0, mK1, tp);
        return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
    } else {
        // two passes when the per-tile arrays (2 tiles x NB x (float + byte)) fit next to the pipeline
        const size_t two = base + (size_t)2 * tp.NB * 7 + 16;
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, score_exact_kernel<D, QUEST, true>) != cudaSuccess) return UGBSA_ERR_LAUNCH;
        bool use_two = two + fa.sharedSizeBytes <= 227 * 1024;
        // UGBSA_SCORE_ONE_PASS=1 selects the single-pass variant where both fit (parity tests cover both)
        if (const char *e = getenv("UGBSA_SCORE_ONE_PASS")) use_two = use_two && e[0] != '1';
        const size_t smem = use_two ? two : base;
        auto kern = use_two ? score_exact_kernel<D, QUEST, true> : score_exact_kernel<D, QUEST, false>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return UGBSA_ERR_LAUNCH;
        const int64_t grid = (int64_t)tp.B * tp.Hq * tp.npairs;
        kern<<<(unsigned)grid, kScoreThreads, smem, stream>>>(mQ, mK0, mK1, tp);
        return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
    }
}

int launch_select_tiles_tc(const void *Q, ugbsa_strides qs, const float *summ_a, const float *summ_b, int B, int Hq,
                           int Hkv, int S, int D, int t_base, int pair_stride, int Sq, float scale, bool quest,
                           int k_base, int kmax, bool router, int32_t *kv_idx, float *sigma_cell, void *scratch,
                           cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    const int Qt = (Sq + 63) / 64;
    const int64_t cells = (int64_t)B * Hq * Qt;
    uint8_t *ws = static_cast<uint8_t *>(scratch);
    float *escore = reinterpret_cast<float *>(ws);
    ws += al256(cells * NB * 4);
    __nv_bfloat16 *op0 = reinterpret_cast<__nv_bfloat16 *>(ws);
    ws += al256((int64_t)B * Hkv * NB * D * 2);
    __nv_bfloat16 *op1 = reinterpret_cast<__nv_bfloat16 *>(ws);
    ws += al256((int64_t)B * Hkv * NB * D * 2);
    float2 *norms = reinterpret_cast<float2 *>(ws);

    int *err = device_error_word();
    if (!err) return UGBSA_ERR_NO_DEVICE;
    // 1. operands
    {
        const int64_t nrows = (int64_t)B * Hkv * NB;
        const int rows_per = 256 / (D / 8);
        const int64_t grid = (nrows + rows_per - 1) / rows_per;
        if (quest)
            summary_operands_kernel<true><<<(unsigned)grid, 256, 0, stream>>>(summ_a, summ_b, nrows, D, op0, op1, norms);
        else
            summary_operands_kernel<false><<<(unsigned)grid, 256, 0, stream>>>(summ_a, nullptr, nrows, D, op0, op1, norms);
        if (cudaGetLastError() != cudaSuccess) return UGBSA_ERR_LAUNCH;
    }
    // 2. tensor-core-guided exact tile scores
    CUtensorMap mQ, mK0, mK1;
    int rc;
    if ((rc = map_rows(&mQ, Q, D, Sq, Hq, B, qs.s, qs.h, qs.b, 64)) != UGBSA_OK) return rc;
    const int64_t kh = (int64_t)NB * D, kb = (int64_t)Hkv * NB * D;
    if ((rc = map_rows(&mK0, op0, D, NB, Hkv, B, D, kh, kb, 128)) != UGBSA_OK) return rc;
    if ((rc = map_rows(&mK1, op1, D, NB, Hkv, B, D, kh, kb, 128)) != UGBSA_OK) return rc;
    TcParams tp;
    tp.B = B; tp.Hq = Hq; tp.Hkv = Hkv; tp.S = S; tp.NB = NB; tp.Qt = Qt; tp.npairs = (Qt + 1) / 2;
    tp.t_base = t_base; tp.pair_stride = pair_stride;
    tp.kmax = kmax;
    tp.scale = scale; tp.escore = escore; tp.norms = norms; tp.summ_a = summ_a; tp.summ_b = summ_b; tp.err = err;
    tp.op0 = op0; tp.op1 = op1;
    if (D == 64) rc = quest ? launch_score<64, true>(mQ, mK0, mK1, tp, stream) : launch_score<64, false>(mQ, mK0, mK1, tp, stream);
    else if (D == 128) rc = quest ? launch_score<128, true>(mQ, mK0, mK1, tp, stream) : launch_score<128, false>(mQ, mK0, mK1, tp, stream);
    else rc = quest ? launch_score<256, true>(mQ, mK0, mK1, tp, stream) : launch_score<256, false>(mQ, mK0, mK1, tp, stream);
    if (rc != UGBSA_OK) return rc;
    // 3. ranking
    RankParams rp;
    rp.B = B; rp.Hq = Hq; rp.S = S; rp.NB = NB; rp.Qt = Qt;
    rp.t_base = t_base; rp.pair_stride = pair_stride;
    int P = 64;
    while (P < NB) P <<= 1;
    rp.NBpad = P;
    rp.k_base = k_base; rp.kmax = kmax; rp.router = router ? 1 : 0;
    rp.escore = escore; rp.kv_idx = kv_idx; rp.sigma_cell = sigma_cell;
    const size_t smem = (size_t)(P > 1024 ? P : 1024) * 8 + (size_t)P * 4 + 16;   // sort keys (>= the 8 KB of histograms) + value keys
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    if (cudaFuncSetAttribute(rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    rank_kernel<<<(unsigned)cells, 256, smem, stream>>>(rp);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

}  // namespace ugbsa
