// rope.cu -- fused per-head RMSNorm + rotary embedding + K block summary (sm_100a).
//
// The caller side of the hook for models that normalise Q and K per head and
// then rotate them (Qwen3 / Qwen3.5-MoE-style attention: q_norm / k_norm, then
// apply_rotary_pos_emb, which the reference imports from transformers at
// src/sparse_attention.py:47-48).  One pass over the projection output writes
// the rotated heads and, for K, the 64-row block summaries the selector needs,
// so the selector's own summary pass over K is not needed.
//
// Arithmetic (element d of one head row x, input dtype T = bf16 / fp16, as the
// transformers modules compute it):
//   v    = sum_d fp32(x_d^2) / D in fp32, r = 1 / sqrt(v + eps)
//   mode SCALE  (Qwen3 / Llama RMSNorm):  y = T(w * T(x * r))
//   mode OFFSET (Qwen3.5 / Qwen3-Next):   y = T((x * r) * (1 + w))
//   mode NONE   (Qwen2 / Llama: rotary without a per-head norm):  y = x
//   rotary dims d < R (R = cos / sin width):
//     out_d = T(T(y_d * cos_d) + T(rot_d * sin_d)),  rot_d = -y_{d+R/2} (d < R/2), y_{d-R/2} (else)
//   d >= R: out_d = y_d
// The fp32 sum of squares runs in a different order than torch's reduction, and
// 1/sqrt is correctly rounded here; the two can differ in the last bit of r,
// which moves a rounded element by one unit in its last place on rare inputs.
// The K summaries use the selector's canonical order (block_summary_kernel):
//   mean = sequential fp32 sum of the block's 64 output rows * 2^-6, Quest min /
//   max; rows past S count as 0.
//
// One CTA per (b, 64-row block, group of heads), 256 threads: D/8
// threads per row, each owning 8 consecutive columns (16-byte loads and
// stores); the rotary partner columns come from lane ^ (R/16) of the same row
// group.  HBM-bound: X read once, Y written once, cos / sin read once per block.
#include <type_traits>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

namespace {

template <typename T>
__device__ __forceinline__ void ld8(const T *p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
}

template <typename T2>
__device__ __forceinline__ T2 to_pair(float a, float b) {
    if constexpr (std::is_same<T2, __nv_bfloat162>::value) return __floats2bfloat162_rn(a, b);
    else return __floats2half2_rn(a, b);
}

}  // namespace

struct RopeParams {
    int B, H, S, D, NB, R;
    int norm_mode;     // 0: y = w T(x r), 1: y = (x r)(1 + w), 2: y = x (no norm, W unused)
    float eps;
    int64_t xb, xh, xs, yb, yh, ys, cb, cs;
    int summary;       // 0 none, 1 mean, 2 Quest
    float *summ_a, *summ_b;
    int hpc, ngroups;  // heads per CTA, head groups
};

// One CTA per (b, 64-row block, group of heads), looping over its heads:
// the block's cos / sin rows are staged in shared memory once for the group; each thread loads
// all its rows of a head (NP independent 16-byte loads in flight) before it
// computes them, and issues the next head's loads before storing this one's.
// At D <= 128 the register cap (64) lets four CTAs share an SM: more loads in
// flight per SM.  The fp32 element work runs on packed pairs (mul / add .f32x2).
template <typename T, int D>
__global__ void __launch_bounds__(256, (D <= 128) ? 4 : 2)
    qk_norm_rope_kernel(const T *__restrict__ X, const T *__restrict__ W, const T *__restrict__ Cs,
                        const T *__restrict__ Sn, T *Y, const RopeParams p) {
    constexpr int TPR = D / 8;          // threads per row
    constexpr int RPP = 256 / TPR;      // rows per pass
    constexpr int NP = 64 / RPP;        // passes per 64-row block
    extern __shared__ __align__(16) uint8_t smem[];
    T *s_cos = reinterpret_cast<T *>(smem);              // [64][R]
    T *s_sin = s_cos + 64 * p.R;                         // [64][R]
    float *s_tile = reinterpret_cast<float *>(s_sin + 64 * p.R);   // [64][D] (summary only)

    const int hg = blockIdx.x % p.ngroups;
    const int blk = (blockIdx.x / p.ngroups) % p.NB;
    const int b = blockIdx.x / (p.ngroups * p.NB);
    const int h_begin = hg * p.hpc;
    const int h_end = min(p.H, h_begin + p.hpc);
    const int part = threadIdx.x % TPR;
    const int rsub = threadIdx.x / TPR;
    const int d0 = part * 8;
    const int half = p.R / 2;
    const int xr = p.R / 16;   // lane distance of the rotary partner
    const int row0 = blk * 64;

    // cos / sin rows of the block -> shared memory (rows past S: zero)
    {
        const int cpr = p.R / 8;   // 16-byte chunks per row
        for (int i = threadIdx.x; i < 64 * cpr; i += 256) {
            const int r = i / cpr, c = (i % cpr) * 8;
            uint4 vc = make_uint4(0u, 0u, 0u, 0u), vs = vc;
            if (row0 + r < p.S) {
                const int64_t o = (int64_t)b * p.cb + (int64_t)(row0 + r) * p.cs + c;
                vc = __ldg(reinterpret_cast<const uint4 *>(Cs + o));
                vs = __ldg(reinterpret_cast<const uint4 *>(Sn + o));
            }
            *reinterpret_cast<uint4 *>(s_cos + r * p.R + c) = vc;
            *reinterpret_cast<uint4 *>(s_sin + r * p.R + c) = vs;
        }
    }
    using T2 = typename std::conditional<std::is_same<T, __nv_bfloat16>::value, __nv_bfloat162, __half2>::type;
    float w[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 wraw = make_uint4(0u, 0u, 0u, 0u);
    if (p.norm_mode != 2) {
        ld8(W + d0, w);
        wraw = __ldg(reinterpret_cast<const uint4 *>(W + d0));
    }
    const T2 *w2 = reinterpret_cast<const T2 *>(&wraw);
    float w1[8];   // 1 + w (offset mode), fp32 as the reference's weight.float()
#pragma unroll
    for (int i = 0; i < 8; ++i) w1[i] = __fadd_rn(1.0f, w[i]);
    __syncthreads();

    auto load_head = [&](int h, uint4 (&x)[NP]) {
        const T *xbase = X + (int64_t)b * p.xb + (int64_t)h * p.xh + d0;
#pragma unroll
        for (int ps = 0; ps < NP; ++ps) {
            const int row = row0 + ps * RPP + rsub;
            x[ps] = (row < p.S) ? __ldg(reinterpret_cast<const uint4 *>(xbase + (int64_t)row * p.xs))
                                : make_uint4(0u, 0u, 0u, 0u);
        }
    };

    // Element ops on pairs (bf16x2 / f16x2, one rounding each): a product or a
    // sum of two values of T is exact in fp32 up to the final rounding, so the
    // paired instructions give what the reference's fp32-then-round ops give.
    uint4 xa[NP], xn[NP];
    load_head(h_begin, xa);
    for (int h = h_begin; h < h_end; ++h) {
        if (h + 1 < h_end) load_head(h + 1, xn);
        T *ybase = Y + (int64_t)b * p.yb + (int64_t)h * p.yh + d0;
#pragma unroll
        for (int ps = 0; ps < NP; ++ps) {
            const int r = ps * RPP + rsub;
            const int row = row0 + r;
            const bool valid = row < p.S;
            float x[8];
            {
                const uint32_t u[4] = {xa[ps].x, xa[ps].y, xa[ps].z, xa[ps].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = (std::is_same<T, __nv_bfloat16>::value)
                                         ? make_float2(__uint_as_float(u[i] << 16), __uint_as_float(u[i] & 0xffff0000u))
                                         : __half22float2(*reinterpret_cast<const __half2 *>(&u[i]));
                    x[2 * i] = f.x;
                    x[2 * i + 1] = f.y;
                }
            }
            uint32_t yv[4];
            if (p.norm_mode == 2) {   // no norm: the input pairs as they are
                yv[0] = xa[ps].x; yv[1] = xa[ps].y; yv[2] = xa[ps].z; yv[3] = xa[ps].w;
            } else {
                // x^2 rounded (as pow(2)), then summed: packed fp32 pairs, the even and the
                // odd columns in the two halves, joined at the end
                uint64_t sq = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint64_t v = f32x2(x[2 * i], x[2 * i + 1]);
                    sq = (i == 0) ? fmul_x2(v, v) : fadd_x2(sq, fmul_x2(v, v));
                }
                float se, so;
                f32x2_split(sq, se, so);
                float ss = __fadd_rn(se, so);
#pragma unroll
                for (int off = TPR >> 1; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
                // D is a power of two: the mean's division is an exact scaling; 1 / sqrt as
                // two correctly rounded steps
                const float rs = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / (float)D), p.eps)));
                const uint64_t rs2 = f32x2(rs, rs);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float n0, n1;
                    f32x2_split(fmul_x2(f32x2(x[2 * i], x[2 * i + 1]), rs2), n0, n1);
                    T2 v;
                    if (p.norm_mode == 1) {
                        float a0, a1;
                        f32x2_split(fmul_x2(f32x2(n0, n1), f32x2(w1[2 * i], w1[2 * i + 1])), a0, a1);
                        v = to_pair<T2>(a0, a1);
                    } else {
                        v = __hmul2_rn(w2[i], to_pair<T2>(n0, n1));
                    }
                    yv[i] = *reinterpret_cast<uint32_t *>(&v);
                }
            }
            uint32_t yp[4];   // the rotary partner columns
#pragma unroll
            for (int i = 0; i < 4; ++i) yp[i] = __shfl_xor_sync(0xffffffffu, yv[i], xr);
            uint4 o;
            uint32_t *ov = reinterpret_cast<uint32_t *>(&o);
            if (d0 < p.R) {
                const uint4 craw = *reinterpret_cast<const uint4 *>(s_cos + r * p.R + d0);
                const uint4 sraw = *reinterpret_cast<const uint4 *>(s_sin + r * p.R + d0);
                const T2 *c2 = reinterpret_cast<const T2 *>(&craw);
                const T2 *s2 = reinterpret_cast<const T2 *>(&sraw);
                const bool lo = d0 < half;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const T2 y2 = *reinterpret_cast<const T2 *>(&yv[i]);
                    T2 rot = *reinterpret_cast<const T2 *>(&yp[i]);
                    if (lo) rot = __hneg2(rot);
                    const T2 v = __hadd2_rn(__hmul2_rn(y2, c2[i]), __hmul2_rn(rot, s2[i]));   // no mul-add contraction
                    ov[i] = *reinterpret_cast<const uint32_t *>(&v);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) ov[i] = yv[i];
            }
            if (valid) *reinterpret_cast<uint4 *>(ybase + (int64_t)row * p.ys) = o;
            if (p.summary) {
                float of[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = (std::is_same<T, __nv_bfloat16>::value)
                                         ? make_float2(__uint_as_float(ov[i] << 16), __uint_as_float(ov[i] & 0xffff0000u))
                                         : __half22float2(*reinterpret_cast<const __half2 *>(&ov[i]));
                    of[2 * i] = valid ? f.x : 0.f;
                    of[2 * i + 1] = valid ? f.y : 0.f;
                }
                *reinterpret_cast<float4 *>(s_tile + r * D + d0) = make_float4(of[0], of[1], of[2], of[3]);
                *reinterpret_cast<float4 *>(s_tile + r * D + d0 + 4) = make_float4(of[4], of[5], of[6], of[7]);
            }
        }
        if (p.summary) {
            __syncthreads();
            const int64_t orow = ((int64_t)b * p.H + h) * p.NB + blk;
            for (int d = threadIdx.x; d < D; d += 256) {
                if (p.summary == 2) {
                    float mn = s_tile[d], mx = s_tile[d];
                    for (int rr = 1; rr < 64; ++rr) {
                        const float v = s_tile[rr * D + d];
                        mn = (v < mn) ? v : mn;
                        mx = (v > mx) ? v : mx;
                    }
                    p.summ_a[orow * D + d] = mn;
                    p.summ_b[orow * D + d] = mx;
                } else {
                    float acc = 0.f;
                    for (int rr = 0; rr < 64; ++rr) acc = __fadd_rn(acc, s_tile[rr * D + d]);
                    p.summ_a[orow * D + d] = __fmul_rn(acc, 0.015625f);
                }
            }
            __syncthreads();   // the tile is rewritten by the next head
        }
#pragma unroll
        for (int ps = 0; ps < NP; ++ps) xa[ps] = xn[ps];
    }
}

template <typename T, int D>
static int launch_rope_t(const void *X, const void *weight, const void *cos, const void *sin, void *Y,
                         const RopeParams &p, cudaStream_t stream) {
    const size_t smem = (size_t)2 * 64 * p.R * sizeof(T) + (p.summary ? (size_t)64 * D * 4 : 0);
    auto k = qk_norm_rope_kernel<T, D>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    const int64_t grid = (int64_t)p.B * p.NB * p.ngroups;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    k<<<(unsigned)grid, 256, smem, stream>>>((const T *)X, (const T *)weight, (const T *)cos, (const T *)sin,
                                             (T *)Y, p);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_qk_norm_rope(const void *X, int dtype, ugbsa_strides xs, const void *weight, int norm_mode, float eps,
                        const void *cos, const void *sin, int64_t cs_b, int64_t cs_s, int rot_dim, int B, int H,
                        int S, int D, void *Y, ugbsa_strides ys, int summary, float *summ_a, float *summ_b,
                        cudaStream_t stream) {
    RopeParams p;
    p.B = B; p.H = H; p.S = S; p.D = D; p.NB = (S + 63) / 64; p.R = rot_dim;
    p.norm_mode = norm_mode;
    p.eps = eps;
    p.xb = xs.b; p.xh = xs.h; p.xs = xs.s;
    p.yb = ys.b; p.yh = ys.h; p.ys = ys.s;
    p.cb = cs_b; p.cs = cs_s;
    p.summary = summary;
    p.summ_a = summ_a; p.summ_b = summ_b;
    // heads per CTA: all of them (the staged cos / sin serve every head) unless
    // that leaves fewer than about four waves of CTAs (148 SMs, ~3 CTAs each)
    {
        const int64_t blocks = (int64_t)B * p.NB;
        int64_t ng = (1800 + blocks - 1) / blocks;
        if (ng > H) ng = H;
        if (ng < 1) ng = 1;
        p.hpc = (int)((H + ng - 1) / ng);
        p.ngroups = (H + p.hpc - 1) / p.hpc;
    }
    const bool bf = dtype == UGBSA_BF16;
#define UGBSA_ROPE_CASE(DD)                                                                                        \
    if (D == DD)                                                                                                   \
        return bf ? launch_rope_t<__nv_bfloat16, DD>(X, weight, cos, sin, Y, p, stream)                            \
                  : launch_rope_t<__half, DD>(X, weight, cos, sin, Y, p, stream);
    UGBSA_ROPE_CASE(64)
    UGBSA_ROPE_CASE(128)
    UGBSA_ROPE_CASE(256)
#undef UGBSA_ROPE_CASE
    return UGBSA_ERR_UNSUPPORTED;
}

}  // namespace ugbsa
