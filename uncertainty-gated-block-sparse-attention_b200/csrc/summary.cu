// summary.cu -- per-block K summaries (sm_100a).
//
// Replaces the reference's block summary (src/sparse_attention.py:617-646):
// F.pad of K to a multiple of 64 rows, then mean (K-mean / router scoring) or
// amin + amax (Quest envelope) over each 64-row block, per KV head.  The
// reference computes this after repeat_kv; the values are identical for every
// Q head of a group, so it is done once per KV head here.
//
// Arithmetic order (the canonical one shared with oracle/ugbsa_oracle.c):
//   mean[d] = (((0 + k0[d]) + k1[d]) + ... + k63[d]) * 2^-6, rows >= S add 0;
//   min/max over the 64 rows, rows >= S count as 0 (the zero padding).
//
// Bandwidth-bound: each thread owns 8 consecutive columns of one block and
// streams the block's 64 rows with 16-byte loads (two for fp32 input), several
// rows in flight held as raw words, so a thread stays within 64 registers and
// the whole grid is resident at once (4 CTAs of 256 threads per SM: 592 slots
// for the 512 CTAs of a 128K x 4-head K).  The Quest envelope of 16-bit K stays
// in its own format (min / max are exact there): packed two-lane min / max on
// the raw words, 8 rows in flight, widened to fp32 once.  Measured at 128K, 4
// KV heads, bf16 (CUDA-graph replays): 24.6 us for the mean (86% of HBM),
// 27.2 us for Quest (81%; 34 us with the envelope in fp32 registers).  K is read
// exactly once.
#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

// raw 16-byte words of 8 consecutive elements (fp32: two words)
template <typename T> struct Raw8 { uint4 w; };
template <> struct Raw8<float> { uint4 w[2]; };
__device__ __forceinline__ void load_raw(const __nv_bfloat16 *p, Raw8<__nv_bfloat16> &r) {
    r.w = __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ void load_raw(const __half *p, Raw8<__half> &r) {
    r.w = __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ void load_raw(const float *p, Raw8<float> &r) {
    r.w[0] = __ldg(reinterpret_cast<const uint4 *>(p));
    r.w[1] = __ldg(reinterpret_cast<const uint4 *>(p) + 1);
}
__device__ __forceinline__ void zero_raw(Raw8<__nv_bfloat16> &r) { r.w = make_uint4(0u, 0u, 0u, 0u); }
__device__ __forceinline__ void zero_raw(Raw8<__half> &r) { r.w = make_uint4(0u, 0u, 0u, 0u); }
__device__ __forceinline__ void zero_raw(Raw8<float> &r) { r.w[0] = r.w[1] = make_uint4(0u, 0u, 0u, 0u); }
__device__ __forceinline__ void to_f32(const Raw8<__nv_bfloat16> &r, float (&x)[8]) {
    const uint32_t w[4] = {r.w.x, r.w.y, r.w.z, r.w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void to_f32(const Raw8<__half> &r, float (&x)[8]) {
    const uint32_t w[4] = {r.w.x, r.w.y, r.w.z, r.w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void to_f32(const Raw8<float> &r, float (&x)[8]) {
    x[0] = __uint_as_float(r.w[0].x); x[1] = __uint_as_float(r.w[0].y);
    x[2] = __uint_as_float(r.w[0].z); x[3] = __uint_as_float(r.w[0].w);
    x[4] = __uint_as_float(r.w[1].x); x[5] = __uint_as_float(r.w[1].y);
    x[6] = __uint_as_float(r.w[1].z); x[7] = __uint_as_float(r.w[1].w);
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

__device__ __forceinline__ void load8(const float *p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void load8(const __half *p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h2 = *reinterpret_cast<const __half2 *>(&w[i]);
        const float2 f = __half22float2(h2);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

// Packed min / max of two 16-bit lanes (min.bf16x2 / min.f16x2): exact, so the
// Quest envelope of 16-bit K is kept in its own format (4 words per 8 columns)
// and widened once at the end.  A NaN in a later row is ignored, as by the
// ordered compare of the oracle.
__device__ __forceinline__ uint32_t pmin(uint32_t a, uint32_t b, __nv_bfloat16) {
    const __nv_bfloat162 r = __hmin2(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                                     *reinterpret_cast<const __nv_bfloat162 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t pmax(uint32_t a, uint32_t b, __nv_bfloat16) {
    const __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                                     *reinterpret_cast<const __nv_bfloat162 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t pmin(uint32_t a, uint32_t b, __half) {
    const __half2 r = __hmin2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t pmax(uint32_t a, uint32_t b, __half) {
    const __half2 r = __hmax2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
}

// Quest envelope of 16-bit K: 8 rows in flight (4 registers each), the running
// min / max in 8 packed registers.
template <typename T>
__global__ void __launch_bounds__(256, 4) quest_summary16_kernel(const T *__restrict__ K, int64_t sb, int64_t sh,
                                                              int64_t ss, int B, int Hkv, int S, int D, int NB,
                                                              int nb0, int NBo, float *__restrict__ out_a,
                                                              float *__restrict__ out_b, float *__restrict__ out_norm) {
    const int tpr = D / 8;
    const int rows_per_cta = blockDim.x / tpr;
    const int64_t row_id = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / tpr;
    const int part = threadIdx.x % tpr;
    const int nbl = NB - nb0;
    const int64_t nrows = (int64_t)B * Hkv * nbl;
    const bool active = row_id < nrows;
    const int nb = active ? nb0 + (int)(row_id % nbl) : 0;
    const int h = active ? (int)((row_id / nbl) % Hkv) : 0;
    const int b = active ? (int)(row_id / ((int64_t)nbl * Hkv)) : 0;
    const int64_t out_row = ((int64_t)b * Hkv + h) * NBo + nb;
    const int d0 = part * 8;

    uint32_t mn[4] = {0u, 0u, 0u, 0u}, mx[4] = {0u, 0u, 0u, 0u};
    if (active) {
        const T *base = K + (int64_t)b * sb + (int64_t)h * sh + (int64_t)nb * 64 * ss + d0;
        const int r_end = min(64, S - nb * 64);   // valid rows of this block (>= 1)
        const uint4 w0 = __ldg(reinterpret_cast<const uint4 *>(base));
        mn[0] = mx[0] = w0.x; mn[1] = mx[1] = w0.y; mn[2] = mx[2] = w0.z; mn[3] = mx[3] = w0.w;
        constexpr int RIF = 8;
#pragma unroll 1
        for (int r0 = 0; r0 < 64; r0 += RIF) {
            uint4 w[RIF];
#pragma unroll
            for (int u = 0; u < RIF; ++u) {
                const int r = r0 + u;
                w[u] = (r < r_end) ? __ldg(reinterpret_cast<const uint4 *>(base + (int64_t)r * ss))
                                   : make_uint4(0u, 0u, 0u, 0u);   // zero padding rows
            }
#pragma unroll
            for (int u = 0; u < RIF; ++u) {
                const uint32_t x[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    mn[i] = pmin(x[i], mn[i], T());
                    mx[i] = pmax(x[i], mx[i], T());
                }
            }
        }
    }
    float fmn[8], fmx[8];
    Raw8<T> rn, rx;
    rn.w = make_uint4(mn[0], mn[1], mn[2], mn[3]);
    rx.w = make_uint4(mx[0], mx[1], mx[2], mx[3]);
    to_f32(rn, fmn);
    to_f32(rx, fmx);
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float m = fmaxf(fabsf(fmn[i]), fabsf(fmx[i]));
        sq = fmaf(m, m, sq);
    }
    for (int off = tpr >> 1; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (!active) return;
    const int64_t o = out_row * D + d0;
    reinterpret_cast<float4 *>(out_a + o)[0] = make_float4(fmn[0], fmn[1], fmn[2], fmn[3]);
    reinterpret_cast<float4 *>(out_a + o)[1] = make_float4(fmn[4], fmn[5], fmn[6], fmn[7]);
    reinterpret_cast<float4 *>(out_b + o)[0] = make_float4(fmx[0], fmx[1], fmx[2], fmx[3]);
    reinterpret_cast<float4 *>(out_b + o)[1] = make_float4(fmx[4], fmx[5], fmx[6], fmx[7]);
    if (out_norm && part == 0) out_norm[out_row] = sqrtf(sq);
}

template <typename T, bool QUEST>
__global__ void __launch_bounds__(256, 4) block_summary_kernel(const T *__restrict__ K, int64_t sb, int64_t sh,
                                                            int64_t ss, int B, int Hkv, int S, int D, int NB,
                                                            int nb0, int NBo, float *__restrict__ out_a,
                                                            float *__restrict__ out_b, float *__restrict__ out_norm) {
    const int tpr = D / 8;                       // threads per block row (<= 32)
    const int rows_per_cta = blockDim.x / tpr;
    const int64_t row_id = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / tpr;
    const int part = threadIdx.x % tpr;
    // blocks nb0 .. NB-1 of every (b, head); outputs are [B, Hkv, NBo, D]
    const int nbl = NB - nb0;
    const int64_t nrows = (int64_t)B * Hkv * nbl;
    const bool active = row_id < nrows;
    const int nb = active ? nb0 + (int)(row_id % nbl) : 0;
    const int h = active ? (int)((row_id / nbl) % Hkv) : 0;
    const int b = active ? (int)(row_id / ((int64_t)nbl * Hkv)) : 0;
    const int64_t out_row = ((int64_t)b * Hkv + h) * NBo + nb;
    const int d0 = part * 8;

    float acc[8], mn[8], mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { acc[i] = 0.f; mn[i] = 0.f; mx[i] = 0.f; }
    if (active) {
        const T *base = K + (int64_t)b * sb + (int64_t)h * sh + d0;
        const int r_end = min(64, S - nb * 64);   // valid rows of this block (>= 1)
        constexpr int RIF = (QUEST && sizeof(T) == 4) ? 2 : 4;   // rows in flight (fp32 envelope: 2, within 64 registers)
#pragma unroll 1
        for (int r0 = 0; r0 < 64; r0 += RIF) {
            Raw8<T> raw[RIF];
#pragma unroll
            for (int u = 0; u < RIF; ++u) {
                const int r = r0 + u;
                if (r < r_end) load_raw(base + (int64_t)(nb * 64 + r) * ss, raw[u]);
                else zero_raw(raw[u]);
            }
#pragma unroll
            for (int u = 0; u < RIF; ++u) {
                const int r = r0 + u;
                float xu[8];
                to_f32(raw[u], xu);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (QUEST) {
                        if (r == 0) { mn[i] = xu[i]; mx[i] = xu[i]; }
                        else {
                            mn[i] = (xu[i] < mn[i]) ? xu[i] : mn[i];
                            mx[i] = (xu[i] > mx[i]) ? xu[i] : mx[i];
                        }
                    } else {
                        acc[i] = __fadd_rn(acc[i], xu[i]);
                    }
                }
            }
        }
    }
    float sq = 0.f;
    float o0[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (QUEST) {
            const float m = fmaxf(fabsf(mn[i]), fabsf(mx[i]));
            sq = fmaf(m, m, sq);
        } else {
            o0[i] = __fmul_rn(acc[i], 0.015625f);
            sq = fmaf(o0[i], o0[i], sq);
        }
    }
    // norm over the row's tpr threads (consecutive lanes, tpr divides 32)
    for (int off = tpr >> 1; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (!active) return;
    const int64_t o = out_row * D + d0;
    if (QUEST) {
        reinterpret_cast<float4 *>(out_a + o)[0] = make_float4(mn[0], mn[1], mn[2], mn[3]);
        reinterpret_cast<float4 *>(out_a + o)[1] = make_float4(mn[4], mn[5], mn[6], mn[7]);
        reinterpret_cast<float4 *>(out_b + o)[0] = make_float4(mx[0], mx[1], mx[2], mx[3]);
        reinterpret_cast<float4 *>(out_b + o)[1] = make_float4(mx[4], mx[5], mx[6], mx[7]);
    } else {
        reinterpret_cast<float4 *>(out_a + o)[0] = make_float4(o0[0], o0[1], o0[2], o0[3]);
        reinterpret_cast<float4 *>(out_a + o)[1] = make_float4(o0[4], o0[5], o0[6], o0[7]);
    }
    if (out_norm && part == 0) out_norm[out_row] = sqrtf(sq);
}

// A few blocks (a decode step's growing last block): one CTA per block stages
// its 64 rows in shared memory with every load in flight at once, then thread d
// runs column d's sum / min / max down the rows in the canonical order.
template <typename T, bool QUEST, int D>
__global__ void __launch_bounds__(256) block_summary_few_kernel(const T *__restrict__ K, int64_t sb, int64_t sh,
                                                                int64_t ss, int Hkv, int S, int nb0, int nbl, int NBo,
                                                                float *__restrict__ out_a, float *__restrict__ out_b) {
    constexpr int CH = D * (int)sizeof(T) / 16;   // 16-byte chunks per row
    __shared__ __align__(16) T rows[64 * D];
    grid_dep_launch();   // a decode step's selection may become resident meanwhile
    const int row_id = blockIdx.x;
    const int nb = nb0 + row_id % nbl;
    const int h = (row_id / nbl) % Hkv;
    const int b = row_id / (nbl * Hkv);
    const int r_end = min(64, S - nb * 64);
    const T *base = K + (int64_t)b * sb + (int64_t)h * sh + (int64_t)nb * 64 * ss;
    for (int i = threadIdx.x; i < 64 * CH; i += 256) {
        const int r = i / CH, c = i % CH;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);   // rows >= S: the zero padding
        if (r < r_end) v = __ldg(reinterpret_cast<const uint4 *>(base + (int64_t)r * ss) + c);
        reinterpret_cast<uint4 *>(rows + r * D)[c] = v;
    }
    __syncthreads();
    const int d = threadIdx.x;
    if (d >= D) return;
    const int64_t o = (((int64_t)b * Hkv + h) * NBo + nb) * D + d;
    if (QUEST) {
        float mn = to_f(rows[d]), mx = mn;
        for (int r = 1; r < 64; ++r) {
            const float x = to_f(rows[r * D + d]);
            mn = (x < mn) ? x : mn;
            mx = (x > mx) ? x : mx;
        }
        out_a[o] = mn;
        out_b[o] = mx;
    } else {
        float acc = 0.f;
        for (int r = 0; r < 64; ++r) acc = __fadd_rn(acc, to_f(rows[r * D + d]));
        out_a[o] = __fmul_rn(acc, 0.015625f);
    }
}

template <typename T>
static int launch_summary_t(const T *K, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest, int nb0, int NBo,
                            float *out_a, float *out_b, float *out_norm, cudaStream_t stream) {
    const int NB = (S + 63) / 64;
    const int tpr = D / 8;
    const int rows_per_cta = 256 / tpr;
    const int64_t nrows = (int64_t)B * Hkv * (NB - nb0);
    const int64_t grid = (nrows + rows_per_cta - 1) / rows_per_cta;
    if (grid <= 0) return UGBSA_OK;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    // a few blocks and no norms (a decode refresh): one CTA per block, its rows staged at once
    if (nrows <= 148 && !out_norm && 64 * D * (int)sizeof(T) <= 32768) {
        const int nbl = NB - nb0;
#define UGBSA_FEW(DD)                                                                                              \
        if constexpr (64 * DD * sizeof(T) <= 32768)                                                                \
        if (D == DD) {                                                                                             \
            if (quest)                                                                                             \
                block_summary_few_kernel<T, true, DD><<<(unsigned)nrows, 256, 0, stream>>>(                       \
                    K, ks.b, ks.h, ks.s, Hkv, S, nb0, nbl, NBo, out_a, out_b);                                     \
            else                                                                                                   \
                block_summary_few_kernel<T, false, DD><<<(unsigned)nrows, 256, 0, stream>>>(                      \
                    K, ks.b, ks.h, ks.s, Hkv, S, nb0, nbl, NBo, out_a, out_b);                                     \
            return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;                                \
        }
        UGBSA_FEW(64)
        UGBSA_FEW(128)
        UGBSA_FEW(256)
#undef UGBSA_FEW
    }
    if (quest) {
        if constexpr (sizeof(T) == 2)
            quest_summary16_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(K, ks.b, ks.h, ks.s, B, Hkv, S, D, NB, nb0,
                                                                          NBo, out_a, out_b, out_norm);
        else
            block_summary_kernel<T, true><<<(unsigned)grid, 256, 0, stream>>>(K, ks.b, ks.h, ks.s, B, Hkv, S, D, NB,
                                                                              nb0, NBo, out_a, out_b, out_norm);
    }
    else
        block_summary_kernel<T, false><<<(unsigned)grid, 256, 0, stream>>>(K, ks.b, ks.h, ks.s, B, Hkv, S, D, NB,
                                                                           nb0, NBo, out_a, out_b, out_norm);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_block_summary_range(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                               int nb0, int NBo, float *out_a, float *out_b, float *out_norm, cudaStream_t stream) {
    switch (dtype) {
        case UGBSA_F32:
            return launch_summary_t((const float *)K, ks, B, Hkv, S, D, quest, nb0, NBo, out_a, out_b, out_norm,
                                    stream);
        case UGBSA_BF16:
            return launch_summary_t((const __nv_bfloat16 *)K, ks, B, Hkv, S, D, quest, nb0, NBo, out_a, out_b,
                                    out_norm, stream);
        case UGBSA_F16:
            return launch_summary_t((const __half *)K, ks, B, Hkv, S, D, quest, nb0, NBo, out_a, out_b, out_norm,
                                    stream);
    }
    return UGBSA_ERR_DTYPE;
}

int launch_block_summary(const void *K, int dtype, ugbsa_strides ks, int B, int Hkv, int S, int D, int quest,
                         float *out_a, float *out_b, float *out_norm, cudaStream_t stream) {
    return launch_block_summary_range(K, dtype, ks, B, Hkv, S, D, quest, 0, (S + 63) / 64, out_a, out_b, out_norm,
                                      stream);
}

}  // namespace ugbsa
