// attn_f32.cu -- block-sparse causal attention for fp32 Q/K/V on CUDA cores.
//
// The reference's kernel takes fp32 inputs as well (src/triton_block_attn.py:
// 267-298; its tl.dot runs them at TF32 precision) and BASELINE config 1 is an
// fp32 layer.  The tensor-core kernel (attn.cu) reads bf16 / fp16 tiles only, so
// fp32 layers come here: the same slot semantics (skip the sentinel and blocks
// that start after the tile's last row, causal mask inside a block, online
// softmax in fp32, out = acc / l with the l > 0 guard), with every product and
// sum in fp32 -- more precise than TF32, and the same work per (tile, slot).
//
// One CTA of 256 threads per (b, q-head, 64-row tile).  Warp w owns rows
// 8w .. 8w + 7 of the tile.  Per kept block:
//   scores  lane j computes keys j and j + 32 for its warp's 8 rows from the
//           K block in shared memory (row stride D + 1: conflict-free column
//           reads) and the Q tile (broadcast float4 reads);
//   softmax row max / sum over the 64 keys by warp shuffles; P to shared memory;
//   P.V     lane j owns output columns j, j + 32, ... for its 8 rows (V rows
//           read contiguously, P broadcast).
// K and V blocks are loaded with 16-byte loads by all threads; the next block's
// loads are issued into registers before the current block is consumed.
// Shared memory: Q 64 x D, K 64 x (D + 1), V 64 x D, P 64 x 65 floats (D = 256:
// 209 KB, one CTA per SM; D = 128: 105 KB, two).
#include <cfloat>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

namespace {

constexpr int kF32Threads = 256;

struct AttnF32Params {
    const float *Q, *K, *V;
    int64_t qb, qh, qs, kb, kh, ks, vb, vh, vs;
    const int32_t *kv_idx;
    int kmax;
    int B, Hq, Hkv, Sq, Sk, Qt, NB;
    int t_base, pair_stride;   // local tile t is sequence tile seq_tile(t, t_base, pair_stride)
    int out_row0, row_limit;   // sequence row g goes to out row g - out_row0 when g < row_limit
    float scale;
    float *out;
    int64_t ob, oh, os;
};

template <int D>
struct F32Smem {
    static constexpr int KSTR = D + 1;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + 64 * D * 4;
    static constexpr int OFF_V = OFF_K + 64 * KSTR * 4;
    static constexpr int OFF_P = OFF_V + 64 * D * 4;
    static constexpr int OFF_LIST = OFF_P + 64 * 65 * 4;
};

// all 256 threads: rows [0, 64) x D floats of a block starting at key row k0
// (rows at or past nrows read as zero) into registers, 16 bytes at a time
template <int D>
struct BlockRegs {
    static constexpr int N = 64 * D / 4 / kF32Threads;   // float4 per thread
    float4 v[N];
    __device__ __forceinline__ void load(const float *base, int64_t rstride, int k0, int nrows) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int idx = i * kF32Threads + threadIdx.x;
            const int r = idx / (D / 4), c = idx % (D / 4);
            v[i] = (k0 + r < nrows) ? __ldg(reinterpret_cast<const float4 *>(base + (int64_t)(k0 + r) * rstride) + c)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __device__ __forceinline__ void store(float *dst, int stride) const {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int idx = i * kF32Threads + threadIdx.x;
            const int r = idx / (D / 4), c = idx % (D / 4);
            float *d = dst + r * stride + c * 4;
            if (stride % 4 == 0) {
                *reinterpret_cast<float4 *>(d) = v[i];
            } else {
                d[0] = v[i].x; d[1] = v[i].y; d[2] = v[i].z; d[3] = v[i].w;
            }
        }
    }
};

template <int D>
__global__ void __launch_bounds__(kF32Threads, 1) attn_f32_kernel(const AttnF32Params p) {
    using L = F32Smem<D>;
    extern __shared__ __align__(16) uint8_t smem[];
    float *sQ = reinterpret_cast<float *>(smem + L::OFF_Q);
    float *sK = reinterpret_cast<float *>(smem + L::OFF_K);
    float *sV = reinterpret_cast<float *>(smem + L::OFF_V);
    float *sP = reinterpret_cast<float *>(smem + L::OFF_P);
    int *sList = reinterpret_cast<int *>(smem + L::OFF_LIST);
    __shared__ int s_n;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x;
    const int t = p.Qt - 1 - (item % p.Qt);   // heavy tiles first
    const int bh = item / p.Qt;
    const int h = bh % p.Hq, b = bh / p.Hq;
    const int kvh = h / (p.Hq / p.Hkv);
    const int tile_row = t * 64;                                       // first row of the tile in Q
    const int tile_first = 64 * seq_tile(t, p.t_base, p.pair_stride);  // its sequence position
    const int tile_last = tile_first + 63;
    const int q_rows = min(64, p.Sq - tile_row);

    // usable slots in slot order (the sentinel and blocks after the tile dropped)
    if (warp == 0) {
        const int32_t *row = p.kv_idx + ((int64_t)(b * p.Hq + h) * p.Qt + t) * p.kmax;
        int n = 0;
        for (int base = 0; base < p.kmax; base += 32) {
            const int j = base + lane;
            const int blk = (j < p.kmax) ? __ldg(row + j) : -1;
            const bool ok = blk >= 0 && blk < p.NB && blk * 64 <= tile_last;
            const unsigned m = __ballot_sync(0xffffffffu, ok);
            if (ok) sList[n + __popc(m & ((1u << lane) - 1u))] = blk;
            n += __popc(m);
        }
        if (lane == 0) s_n = n;
    }
    {
        BlockRegs<D> q;
        q.load(p.Q + (int64_t)b * p.qb + (int64_t)h * p.qh, p.qs, tile_row, p.Sq);
        q.store(sQ, D);
    }
    __syncthreads();
    const int n = s_n;
    const float *Kh = p.K + (int64_t)b * p.kb + (int64_t)kvh * p.kh;
    const float *Vh = p.V + (int64_t)b * p.vb + (int64_t)kvh * p.vh;

    constexpr int CPL = D / 32;   // output columns per lane
    float acc[8][CPL];
    float m_i[8], l_i[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        m_i[r] = -1.0e30f;
        l_i[r] = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc[r][c] = 0.f;
    }

    // D <= 128: the next block's K / V loads are in flight while this block is
    // consumed; D = 256 would need 128 more registers for that and loads in place
    constexpr bool kPrefetch = D <= 128;
    BlockRegs<D> kr, vr;
    if (kPrefetch && n > 0) {
        kr.load(Kh, p.ks, sList[0] * 64, p.Sk);
        vr.load(Vh, p.vs, sList[0] * 64, p.Sk);
    }
    for (int i = 0; i < n; ++i) {
        const int blk = sList[i];
        __syncthreads();   // the previous block's K, V and P are no longer read
        if (!kPrefetch) {
            kr.load(Kh, p.ks, blk * 64, p.Sk);
            vr.load(Vh, p.vs, blk * 64, p.Sk);
        }
        kr.store(sK, L::KSTR);
        vr.store(sV, D);
        __syncthreads();
        if (kPrefetch && i + 1 < n) {   // next block's loads overlap this block's math
            kr.load(Kh, p.ks, sList[i + 1] * 64, p.Sk);
            vr.load(Vh, p.vs, sList[i + 1] * 64, p.Sk);
        }
        // scores for rows 8w .. 8w + 7, keys lane and lane + 32
        float s0[8], s1[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) s0[r] = s1[r] = 0.f;
        const float *k0 = sK + lane * L::KSTR, *k1 = sK + (lane + 32) * L::KSTR;
        const float *qrow = sQ + (warp * 8) * D;
#pragma unroll 2
        for (int d = 0; d < D; d += 4) {
            const float a0 = k0[d], a1 = k0[d + 1], a2 = k0[d + 2], a3 = k0[d + 3];
            const float c0 = k1[d], c1 = k1[d + 1], c2 = k1[d + 2], c3 = k1[d + 3];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float4 qv = *reinterpret_cast<const float4 *>(qrow + r * D + d);
                s0[r] = fmaf(qv.x, a0, s0[r]); s0[r] = fmaf(qv.y, a1, s0[r]);
                s0[r] = fmaf(qv.z, a2, s0[r]); s0[r] = fmaf(qv.w, a3, s0[r]);
                s1[r] = fmaf(qv.x, c0, s1[r]); s1[r] = fmaf(qv.y, c1, s1[r]);
                s1[r] = fmaf(qv.z, c2, s1[r]); s1[r] = fmaf(qv.w, c3, s1[r]);
            }
        }
        const int key0 = blk * 64 + lane, key1 = key0 + 32;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int lr = warp * 8 + r;           // row within the tile
            const int g = tile_first + lr;         // its sequence position
            const bool row_ok = lr < q_rows;
            float x0 = (row_ok && key0 <= g && key0 < p.Sk) ? s0[r] * p.scale : -1.0e30f;
            float x1 = (row_ok && key1 <= g && key1 < p.Sk) ? s1[r] * p.scale : -1.0e30f;
            float mx = fmaxf(x0, x1);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_i[r], mx);
            const float alpha = expf(m_i[r] - m_new);
            const float p0 = expf(x0 - m_new), p1 = expf(x1 - m_new);
            float sum = p0 + p1;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l_i[r] = fmaf(l_i[r], alpha, sum);
            m_i[r] = m_new;
#pragma unroll
            for (int c = 0; c < CPL; ++c) acc[r][c] *= alpha;
            sP[lr * 65 + lane] = p0;
            sP[lr * 65 + lane + 32] = p1;
        }
        __syncwarp();
        // P.V for the warp's rows (its own P rows only: no CTA barrier needed)
#pragma unroll 4
        for (int j = 0; j < 64; ++j) {
            float vv[CPL];
#pragma unroll
            for (int c = 0; c < CPL; ++c) vv[c] = sV[j * D + lane + 32 * c];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float pr = sP[(warp * 8 + r) * 65 + j];
#pragma unroll
                for (int c = 0; c < CPL; ++c) acc[r][c] = fmaf(pr, vv[c], acc[r][c]);
            }
        }
    }
    // out = acc / l (l > 0 guard), rows of this tile that exist
    float *ob = p.out + (int64_t)b * p.ob + (int64_t)h * p.oh;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int lr = warp * 8 + r;
        const int g = tile_first + lr;
        if (lr >= q_rows || g >= p.row_limit) continue;
        const float inv_l = l_i[r] > 0.f ? 1.f / l_i[r] : 1.f;
        float *o = ob + (int64_t)(g - p.out_row0) * p.os;
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[lane + 32 * c] = acc[r][c] * inv_l;
    }
}

template <int D>
int launch_f32_t(const AttnF32Params &p, cudaStream_t stream) {
    using L = F32Smem<D>;
    const size_t smem = (size_t)L::OFF_LIST + (size_t)p.kmax * 4;
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    if (cudaFuncSetAttribute(attn_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    const int64_t grid = (int64_t)p.B * p.Hq * p.Qt;
    if (grid <= 0) return UGBSA_OK;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    attn_f32_kernel<D><<<(unsigned)grid, kF32Threads, smem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

}  // namespace

int launch_attn_f32(const float *Q, const float *K, const float *V, ugbsa_strides qs, ugbsa_strides ks,
                    ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                    int t_base, int pair_stride, float scale, float *out, ugbsa_strides os, cudaStream_t stream) {
    if (t_base < 0 || pair_stride < 1 || (pair_stride > 1 && (t_base & 1))) return UGBSA_ERR_SHAPE;
    AttnF32Params p;
    p.Q = Q; p.K = K; p.V = V;
    p.qb = qs.b; p.qh = qs.h; p.qs = qs.s;
    p.kb = ks.b; p.kh = ks.h; p.ks = ks.s;
    p.vb = vs.b; p.vh = vs.h; p.vs = vs.s;
    p.kv_idx = kv_idx;
    p.kmax = kmax;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Sq = Sq; p.Sk = Sk;
    p.Qt = (Sq + 63) / 64;
    p.NB = (Sk + 63) / 64;
    p.t_base = t_base; p.pair_stride = pair_stride;
    if (pair_stride == 1) {
        p.out_row0 = 64 * t_base;
        p.row_limit = 64 * t_base + Sq;
    } else {
        p.out_row0 = 0;
        p.row_limit = Sk;
    }
    p.scale = scale;
    p.out = out;
    p.ob = os.b; p.oh = os.h; p.os = os.s;
    switch (D) {
        case 64: return launch_f32_t<64>(p, stream);
        case 128: return launch_f32_t<128>(p, stream);
        case 256: return launch_f32_t<256>(p, stream);
    }
    return UGBSA_ERR_UNSUPPORTED;
}

}  // namespace ugbsa
