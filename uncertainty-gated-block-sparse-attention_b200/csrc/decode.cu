// decode.cu -- block-sparse decode (one query row per head) over a KV cache (sm_100a).
//
// The reference decodes densely (src/sparse_attention.py:756-770: Q == 1 goes
// to SDPA over the whole cache).  This path applies the v2 block policy to the
// decode row instead, reusing the block summaries the prefill computed (and
// refreshing only the cache's last, growing block):
//
//   score(block j) = the row's exact fp32 score against the block summary, in
//     the selection's canonical order (one fma chain over d; Quest: two chains
//     max(q,0)*Kmax and min(q,0)*Kmin, added, then scaled);
//   every block is visible (the row sits at position S-1); the sink (block 0)
//     and the row's own block (the last) are forced to the top; top-kmax in
//     descending score, ties to the lower block id; sigma margin and router as
//     in the prefill selection over the B x Hq decode cells (one tile each);
//   attention: softmax over the keys of the kept blocks (keys < S), repeated
//     ids counted again.
//
// Kernels (ugbsa_decode_select / _attn: the summary refresh, the selection, the
// router finish, the attention and the merge; ugbsa_decode_step folds the refresh
// into the selection and the finish into the attention, three launches):
//
//  decode_select_kernel -- a thread-block cluster of CL CTAs per (b, kv head):
//    CTA c stages its rows of the group's block summaries in shared memory
//    (coalesced cp.async, rounds of 64 rows, a swizzled layout), and its warps
//    run the canonical fp32 chains of every Q head of the group over them (a
//    lane per row, a warp per (tile, chain) with an accumulator per head), so
//    each summary element is read from memory and from shared memory once for
//    the whole group.  The order keys go to the CTA that ranks the head (head g:
//    CTA g % CL); after the cluster barrier each CTA finds its heads' kmax-th
//    largest key by a radix selection, gathers the blocks at or above it and
//    ranks them by counting (rank = number of candidates before it in (score
//    desc, id asc) order), writing kv_idx[rank] and sigma.  No global handshake:
//    two cluster barriers are the only waits.  In the fused step the cluster's
//    last CTA then recomputes the summary of the cache's last block (forced in
//    this step, never scored) for the steps that follow.
//  decode_finish_kernel -- one CTA: row-grain head mean, the quantile over the
//    B x Hq cells by counting, the sentinel fill of the untriggered cells.
//  decode_group_attn_kernel -- one CTA per (b, kv head, split): the union of
//    the group's G lists (a bitmap per head; the entries are the union's block
//    ids, each block's heads read from the bitmaps when it is used), so each
//    kept K/V block is read once for the whole group rather than once per Q
//    head.  The block's K and V tiles arrive by TMA (128-byte swizzle, two or
//    three blocks in flight, bounded mbarrier waits); the G query rows (padded
//    to 16) form the A operand of mma.sync m16n8k16 (16-bit inputs, fp32
//    accumulation): warp w takes keys 16w..16w+15 of the block, S = Q.K^T,
//    masked to the heads of the entry, per-warp online softmax, O += P.V with P
//    as 16-bit.  A list that repeats a block (never the selection's own lists)
//    is processed slot by slot instead, one head per entry.  In the fused step
//    each CTA also derives its heads' router triggers (the finish's rules) and
//    drops the untriggered heads' slots >= k_base.  decode_combine_kernel
//    merges the splits' partial (o, m, l).
#include <cooperative_groups.h>

#include <cfloat>
#include <cstdlib>
#include <type_traits>
#include <utility>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace cg = cooperative_groups;

namespace ugbsa {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

// ascending order key of the quantile (NaN last; -0 folded into +0)
__device__ __forceinline__ uint32_t asc_key_dec(float v) {
    if (v != v) return 0xffffffffu;
    v = __fadd_rn(v, 0.0f);
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace

// host: launch with the programmatic stream-serialization attribute (the kernel may
// become resident while its predecessor in the stream finishes; it calls
// grid_dep_wait() before reading that predecessor's output)
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args &&...args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...) == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

// ------------------------------------------------------------------ selection
constexpr int kDecMaxGroup = 16;
constexpr int kDecSelThreads = 512;
constexpr int kDecMaxCluster = 16;   // 16 needs the non-portable cluster size; 8 otherwise

struct DecSelParams {
    int B, Hq, Hkv, G, S, NB, NBs, CL, chunk, hpc;   // hpc: heads ranked per CTA (head g by CTA g % CL)
    int nbuf;                                        // staged rounds in flight (1 .. kDecSelMaxBufs)
    int64_t qb, qh;
    float scale;
    int k_base, kmax, router;
    const float *summ_a, *summ_b;
    int32_t *kv_idx;    // [B*Hq, kmax]
    float *sigma_cell;  // [B*Hq]
    // optional refresh of the cache's last block summary (ugbsa_decode_step): K rows
    // (K's dtype is Q's), written into summ_a / summ_b row NB - 1 after the scoring
    const void *rK;
    int64_t rkb, rkh, rks;
};

// Summary of block nb of K [b, kvh] (rows >= S count as 0) by the CTA's first D
// threads from rows staged in shared memory: the canonical order of the block
// summary kernels (mean: ((0 + k0) + k1) + ... then * 2^-6; Quest: min / max from
// row 0 on), written to row nb of the [B, Hkv, NBs, D] summaries.
template <typename T, bool QUEST, int D>
__device__ void refresh_block_summary(const T *__restrict__ K, int64_t kb, int64_t kh, int64_t ks, int b, int kvh,
                                      int Hkv, int S, int nb, int NBs, float *sa, float *sb, T *rows, int nthreads) {
    constexpr int CH = D * (int)sizeof(T) / 16;
    const int r_end = min(64, S - nb * 64);
    const T *base = K + (int64_t)b * kb + (int64_t)kvh * kh + (int64_t)nb * 64 * ks;
    for (int i = threadIdx.x; i < 64 * CH; i += nthreads) {
        const int r = i / CH, c = i % CH;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < r_end) v = __ldg(reinterpret_cast<const uint4 *>(base + (int64_t)r * ks) + c);
        reinterpret_cast<uint4 *>(rows + r * D)[c] = v;
    }
    __syncthreads();
    const int d = threadIdx.x;
    if (d < D) {
        const int64_t o = (((int64_t)b * Hkv + kvh) * NBs + nb) * D + d;
        if (QUEST) {
            float mn = to_f<T>(rows[d]), mx = mn;
            for (int r = 1; r < 64; ++r) {
                const float x = to_f<T>(rows[r * D + d]);
                mn = (x < mn) ? x : mn;
                mx = (x > mx) ? x : mx;
            }
            sa[o] = mn;
            sb[o] = mx;
        } else {
            float acc = 0.f;
            for (int r = 0; r < 64; ++r) acc = __fadd_rn(acc, to_f<T>(rows[r * D + d]));
            sa[o] = __fmul_rn(acc, 0.015625f);
        }
    }
}

template <int D> struct DecSelCfg {
    static constexpr int TR = 32;                       // summary rows per staged tile (a lane per row)
    static constexpr int TILE_BYTES = 2 * TR * D * 4;   // both operands (Quest), fp32
};
constexpr int kDecSelMaxBufs = 2;   // staged rounds in flight (a CTA's rows stream from L2 / HBM), as shared memory allows

__device__ __forceinline__ void cp_async_wait_upto(int n) {   // wait until at most n groups are pending
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}

// 16-byte chunk c of row r in a staged [rows][D] fp32 operand: chunk c & 7 of each
// 128-byte segment at (c & 7) ^ (r & 7), so a warp's lanes (32 rows) reading the
// same chunk hit distinct banks
__device__ __forceinline__ int sel_swz(int r, int c) { return (c & ~7) | ((c & 7) ^ (r & 7)); }

// shared memory: rounds [BUFS][2 tiles][2 ops][TR][D] f32 (then the candidates [NB] u64) |
// q [2][G][D] f32 | keys [hpc][NB] u32 | partial chains [32 combos][2 TR] f32
template <typename T, bool QUEST, int D, int GM>
__global__ void __launch_bounds__(kDecSelThreads, 1) decode_select_kernel(const T *__restrict__ Q,
                                                                          const DecSelParams p) {
    using C = DecSelCfg<D>;
    constexpr int NW = kDecSelThreads / 32;
    constexpr int NCH = QUEST ? 2 : 1;                   // chains per head
    constexpr int CH4 = D / 4;                           // 16-byte chunks per row
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int grp = blockIdx.x / p.CL;                   // b * Hkv + kv head
    const int kvh = grp % p.Hkv, b = grp / p.Hkv;
    const int G = p.G, NB = p.NB;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    extern __shared__ __align__(16) uint8_t smem[];
    float *tiles = reinterpret_cast<float *>(smem);
    uint64_t *cand = reinterpret_cast<uint64_t *>(smem);   // after the scoring, over the tiles
    const int BUFS = p.nbuf;
    // the candidates [NB] u64 reuse the tile buffers; the query rows after them stay 16-byte aligned
    const size_t cand_bytes = (size_t)((NB + 1) & ~1) * 8;
    const size_t tiles_bytes = (size_t)BUFS * 2 * C::TILE_BYTES > cand_bytes ? (size_t)BUFS * 2 * C::TILE_BYTES
                                                                             : cand_bytes;
    float *sq = reinterpret_cast<float *>(smem + tiles_bytes);   // [NCH][G][D]
    uint32_t *keys = reinterpret_cast<uint32_t *>(sq + NCH * G * D);
    float *part = reinterpret_cast<float *>(keys + p.hpc * ((NB + 3) & ~3));   // [32 combos][2 TR rows]
    __shared__ uint32_t whist[NW][256];
    __shared__ uint32_t tot[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k, s_n;
    __shared__ float s_val[3];
    grid_dep_launch();
    grid_dep_wait();   // the summaries (a refresh just before) are complete

    // the rows of this CTA: [r0, r1), staged by cp.async in rounds of two TR-row tiles
    const int r0 = crank * p.chunk, r1 = min(NB, r0 + p.chunk);
    constexpr int RR = 2 * C::TR;                           // rows per round (a lane runs two chains)
    const int nrounds = r1 > r0 ? (r1 - r0 + RR - 1) / RR : 0;
    const float *opA = p.summ_a + ((int64_t)b * p.Hkv + kvh) * p.NBs * D;   // Quest: Kmin; mean: the mean
    const float *opB = QUEST ? p.summ_b + ((int64_t)b * p.Hkv + kvh) * p.NBs * D : opA;   // Quest: Kmax
    // round buffer: [2 tiles][NCH ops][TR rows][D]
    auto stage = [&](int rd) {
        float *dst = tiles + (size_t)(rd % BUFS) * (2 * C::TILE_BYTES / 4);
        const int rb = r0 + rd * RR;
        for (int i = tid; i < 2 * NCH * C::TR * CH4; i += kDecSelThreads) {
            const int tt = i / (NCH * C::TR * CH4), op = (i / (C::TR * CH4)) % NCH, r = (i / CH4) % C::TR,
                      c = i % CH4;
            const int row = rb + tt * C::TR + r;
            if (row < r1) {
                const float *src = (op == 0 ? opB : opA) + (int64_t)row * D + c * 4;
                cp_async16(dst + (((size_t)tt * 2 + op) * C::TR + r) * D + sel_swz(r, c) * 4, src);
            }
        }
        cp_async_commit();
    };
    // BUFS - 1 rounds ahead; one commit group per round slot (empty past the end), so
    // waiting for all but the newest BUFS - 1 groups completes the current round
    for (int rd = 0; rd < BUFS - 1; ++rd) {
        if (rd < nrounds) stage(rd);
        else cp_async_commit();
    }
    // the group's query rows (while the first rows are in flight): Quest max(q,0) and
    // min(q,0); mean q
    for (int i = tid; i < G * D; i += kDecSelThreads) {
        const int g = i / D, d = i % D;
        const float x = to_f<T>(Q[(int64_t)b * p.qb + (int64_t)(kvh * G + g) * p.qh + d]);
        if (QUEST) {
            sq[i] = x > 0.f ? x : 0.f;
            sq[G * D + i] = x < 0.f ? x : 0.f;
        } else {
            sq[i] = x;
        }
    }

    // chains: warp w < 2 * NCH takes tile w / NCH of the round and chain w % NCH for
    // every head of the group (up to GM fma chains per lane, one row per lane): each
    // staged element is read from shared memory once for all the heads
    for (int rd = 0; rd < nrounds; ++rd) {
        if (rd + BUFS - 1 < nrounds) stage(rd + BUFS - 1);
        else cp_async_commit();
        cp_async_wait_upto(BUFS - 1);
        __syncthreads();
        const float *tb = tiles + (size_t)(rd % BUFS) * (2 * C::TILE_BYTES / 4);
        if (warp < 2 * NCH) {
            const int tt = warp / NCH, ch = warp % NCH;
            const float4 *row = reinterpret_cast<const float4 *>(tb + ((size_t)(tt * 2 + ch) * C::TR + lane) * D);
            const float4 *q4 = reinterpret_cast<const float4 *>(sq + (size_t)ch * G * D);
            float acc[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) acc[g] = 0.f;
#pragma unroll 4
            for (int c = 0; c < CH4; ++c) {
                const float4 kv = row[sel_swz(lane, c)];
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g < G) {
                        const float4 qv = q4[g * CH4 + c];
                        acc[g] = __fmaf_rn(qv.x, kv.x, acc[g]);
                        acc[g] = __fmaf_rn(qv.y, kv.y, acc[g]);
                        acc[g] = __fmaf_rn(qv.z, kv.z, acc[g]);
                        acc[g] = __fmaf_rn(qv.w, kv.w, acc[g]);
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < GM; ++g)
                if (g < G) part[(g * NCH + ch) * RR + tt * C::TR + lane] = acc[g];
        }
        __syncthreads();
        // every CTA of the cluster is running before any writes another's shared memory
        // (taken once per thread: here in the first staged round, or below by a CTA without rows)
        if (rd == 0) cluster.sync();
        // score -> order key, into the owner CTA of the head (sink and own block forced)
        const int rb = r0 + rd * RR;
        for (int i = tid; i < G * RR; i += kDecSelThreads) {
            const int g = i / RR, r = i % RR;
            const int j = rb + r;
            if (j >= r1) continue;
            uint32_t u;
            if (j == 0 || j == NB - 1) {
                u = ordered_key(FLT_MAX);
            } else {
                // Quest: (max(q,0).Kmax + min(q,0).Kmin) * scale; mean: (q.mean) * scale
                const float v = QUEST ? __fmul_rn(__fadd_rn(part[(g * 2) * RR + r], part[(g * 2 + 1) * RR + r]),
                                                  p.scale)
                                      : __fmul_rn(part[g * RR + r], p.scale);
                u = ordered_key(v);
            }
            uint32_t *dk = cluster.map_shared_rank(keys, g % p.CL);
            dk[(size_t)(g / p.CL) * ((NB + 3) & ~3) + j] = u;
        }
    }
    if (nrounds == 0) cluster.sync();   // the first barrier, for a CTA without rows
    cp_async_wait_all();
    cluster.sync();   // every key is with its head's CTA

    // each CTA ranks the heads it owns
    for (int gl = 0; gl < p.hpc; ++gl) {
        const int g = crank + gl * p.CL;
        if (g >= G) break;
        const int cell = b * p.Hq + kvh * G + g;
        const uint32_t *hk = keys + (size_t)gl * ((NB + 3) & ~3);
        if (tid == 0) {
            s_n = 0;
            s_prefix = 0u;
            s_mask = 0u;
            s_k = p.kmax;
            s_val[0] = s_val[1] = s_val[2] = -INFINITY;
        }
        __syncthreads();
        // V: a key at or below the kmax-th largest (every candidate of the top kmax has
        // a key >= V; a few extra candidates only cost the counting rank below).
        // The forced sink / own blocks take their slots first: V is the (kmax - 2)-th
        // largest of the other keys, by a descending radix selection that starts at the
        // first bit where their smallest and largest key differ and stops once the bin
        // holding V has at most 16 keys (its lower edge is then V).  Keys at or above
        // the forced value (FLT_MAX, infinite or NaN scores) can push a forced block out
        // of the top kmax; then the selection runs over all keys instead.
        uint32_t V = 0u;
        if (NB > p.kmax) {
            const uint32_t kforced = ordered_key(FLT_MAX);
            uint32_t kmn = 0xffffffffu, kmx = 0u;
            for (int j = tid; j < NB; j += kDecSelThreads) {
                if (j == 0 || j == NB - 1) continue;
                const uint32_t u = hk[j];
                kmn = min(kmn, u);
                kmx = max(kmx, u);
            }
            kmn = __reduce_min_sync(0xffffffffu, kmn);
            kmx = __reduce_max_sync(0xffffffffu, kmx);
            if (lane == 0) {
                whist[warp][0] = kmn;
                whist[warp][1] = kmx;
            }
            __syncthreads();
            kmn = 0xffffffffu;
            kmx = 0u;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                kmn = min(kmn, whist[w][0]);
                kmx = max(kmx, whist[w][1]);
            }
            __syncthreads();
            const bool excl_forced = kmx < kforced;   // no other key ties with or passes the forced ones
            const int nforced = NB >= 2 ? 2 : 1;
            int k = excl_forced ? p.kmax - nforced : p.kmax;
            if (!excl_forced) {
                kmn = 0u;
                kmx = 0xffffffffu;
            }
            if (k <= 0) {
                V = kforced;
            } else if (kmn == kmx) {
                V = kmn;
            } else {
                int lowbit = 32 - __clz(kmn ^ kmx);   // bits below are not yet fixed
                uint32_t prefix = (uint32_t)((unsigned long long)kmx & (~0ull << lowbit));
                for (;;) {
                    const int shift = max(lowbit - 8, 0);
                    const uint32_t nbins = 1u << (lowbit - shift);
                    const uint32_t himask = (uint32_t)(~0ull << lowbit);
                    for (int i = lane; i < 256; i += 32) whist[warp][i] = 0u;
                    __syncwarp();
                    for (int j = tid; j < NB; j += kDecSelThreads) {
                        if (excl_forced && (j == 0 || j == NB - 1)) continue;
                        const uint32_t u = hk[j];
                        if ((u & himask) == prefix)
                            atomicAdd(&whist[warp][(nbins - 1u) - ((u >> shift) & (nbins - 1u))], 1u);
                    }
                    __syncthreads();
                    if (tid < 256) {
                        uint32_t c = 0u;
#pragma unroll
                        for (int w = 0; w < NW; ++w) c += whist[w][tid];
                        tot[tid] = c;
                    }
                    __syncthreads();
                    if (warp == 0) {
                        uint32_t cnt[8], sum = 0u;
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            cnt[e] = tot[8 * lane + e];
                            sum += cnt[e];
                        }
                        uint32_t incl = sum;
#pragma unroll
                        for (int off = 1; off < 32; off <<= 1) {
                            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
                            if (lane >= off) incl += y;
                        }
                        const uint32_t excl = incl - sum;
                        if (excl < (uint32_t)k && (uint32_t)k <= incl) {
                            uint32_t run = excl, selc = 0u;
                            int bin = 8 * lane + 7;
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                if (run + cnt[e] >= (uint32_t)k) {
                                    bin = 8 * lane + e;
                                    selc = cnt[e];
                                    break;
                                }
                                run += cnt[e];
                            }
                            s_k = (int)((uint32_t)k - run);
                            s_prefix = prefix | (((nbins - 1u) - (uint32_t)bin) << shift);
                            s_mask = selc;
                        }
                    }
                    __syncthreads();
                    prefix = s_prefix;
                    k = s_k;
                    lowbit = shift;
                    const uint32_t selc = s_mask;
                    __syncthreads();   // s_prefix / s_k / s_mask are rewritten by the next pass
                    if (selc <= 16u || shift == 0) break;
                }
                V = prefix;
            }
        }
        // candidates: key >= V (every block when NB <= kmax)
        for (int jb = tid - lane; jb < NB; jb += kDecSelThreads) {
            const int j = jb + lane;
            const uint32_t u = (j < NB) ? hk[j] : 0u;
            const bool in = (j < NB) && (u >= V);
            const unsigned m = __ballot_sync(0xffffffffu, in);
            int base = 0;
            if (lane == 0 && m) base = atomicAdd(&s_n, __popc(m));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (in)
                cand[base + __popc(m & ((1u << lane) - 1u))] =
                    ((uint64_t)u << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
        }
        __syncthreads();
        // rank by counting: the number of candidates before this one in (score desc,
        // id asc); four threads per candidate, each counting a quarter of the list
        const int n = s_n;
        const int64_t out0 = (int64_t)cell * p.kmax;
        const int quarter = tid & 3;
        for (int ib = 0; ib < n; ib += kDecSelThreads / 4) {
            const int i = ib + (tid >> 2);
            const uint64_t ki = (i < n) ? cand[i] : 0ull;
            int r = 0;
            if (i < n)
                for (int j = quarter; j < n; j += 4) r += (cand[j] > ki) ? 1 : 0;
            r += __shfl_xor_sync(0xffffffffu, r, 1);
            r += __shfl_xor_sync(0xffffffffu, r, 2);
            if (i < n && quarter == 0) {
                if (r < p.kmax) p.kv_idx[out0 + r] = (int32_t)(0xffffffffu - (uint32_t)(ki & 0xffffffffu));
                const float val = key_value((uint32_t)(ki >> 32));
                if (r == 0) s_val[0] = val;
                if (r == p.k_base - 1) s_val[1] = val;
                if (r == p.k_base) s_val[2] = val;
            }
        }
        // slots past the visible blocks (NB < kmax) hold the invisible ids in order
        for (int i = n + tid; i < p.kmax; i += kDecSelThreads) p.kv_idx[out0 + i] = i;
        __syncthreads();
        if (tid == 0) {
            float sig = __int_as_float(0x7fc00000);
            if (p.router) {
                const float s_top = s_val[0], s_km1 = s_val[1], s_kb = s_val[2];
                float spread = __fsub_rn(s_top, s_kb);
                if (spread < 1e-6f) spread = 1e-6f;
                sig = __fdiv_rn(__fsub_rn(s_km1, s_kb), spread);
            }
            p.sigma_cell[cell] = sig;
        }
        __syncthreads();
    }
    // the cache's last block (forced in this step, never scored): its summary for the
    // next steps, by the cluster's last CTA once every staged row has been read
    if (p.rK && crank == p.CL - 1) {
        __syncthreads();
        refresh_block_summary<T, QUEST, D>(reinterpret_cast<const T *>(p.rK), p.rkb, p.rkh, p.rks, b, kvh, p.Hkv,
                                           p.S, NB - 1, p.NBs, const_cast<float *>(p.summ_a),
                                           const_cast<float *>(p.summ_b), reinterpret_cast<T *>(smem),
                                           kDecSelThreads);
    }
}

// One CTA over the B x Hq decode cells (B * Hq <= 1024): the router's
// threshold and trigger (prefill rules on one-tile rows) and the sentinel fill.
struct DecFinParams {
    int B, Hq, NB, k_base, kmax, router, grain_row, mode_quantile;
    int64_t kq;   // 1-based rank in the expanded [B, Hq] array
    float tau;
    const float *sigma_cell;
    int32_t *kv_idx;
    float *sigma_out;
    uint8_t *trigger_out;
};

__global__ void __launch_bounds__(1024) decode_finish_kernel(const DecFinParams p) {
    __shared__ float s_cell[1024];
    __shared__ float s_row[1024];
    __shared__ float s_th;
    const int tid = threadIdx.x;
    const int ncell = p.B * p.Hq;
    grid_dep_launch();
    grid_dep_wait();   // the selection's margins and lists are complete
    if (tid < ncell) s_cell[tid] = p.sigma_cell[tid];   // one load per thread, all in flight
    __syncthreads();
    if (p.router) {
        if (p.grain_row && tid < p.B) {
            float acc = 0.f;
            for (int hh = 0; hh < p.Hq; ++hh) acc = __fadd_rn(acc, s_cell[tid * p.Hq + hh]);
            s_row[tid] = __fdiv_rn(acc, (float)p.Hq);
        }
        if (tid == 0) s_th = p.tau;
        __syncthreads();
        if (p.mode_quantile) {
            const float *vals = p.grain_row ? s_row : s_cell;
            const int n = p.grain_row ? p.B : ncell;
            const int64_t kk = p.grain_row ? (p.kq - 1) / p.Hq + 1 : p.kq;
            if (tid < n) {
                const uint32_t ui = asc_key_dec(vals[tid]);
                int64_t rank = 0;
                for (int j = 0; j < n; ++j) {
                    const uint32_t uj = asc_key_dec(vals[j]);
                    rank += (uj < ui || (uj == ui && j < tid)) ? 1 : 0;
                }
                if (rank == kk - 1) {
                    float v;
                    if (ui == 0xffffffffu) v = __int_as_float(0x7fc00000);
                    else v = __uint_as_float((ui & 0x80000000u) ? (ui & 0x7fffffffu) : ~ui);
                    s_th = v;
                }
            }
        }
        __syncthreads();
    }
    const float th = s_th;
    for (int c = tid; c < ncell; c += blockDim.x) {
        float eff = __int_as_float(0x7fc00000);
        bool unc = false;
        if (p.router) {
            eff = p.grain_row ? s_row[c / p.Hq] : s_cell[c];
            unc = p.mode_quantile ? (eff <= th) : (eff < th);
        }
        if (p.sigma_out) p.sigma_out[c] = eff;
        if (p.trigger_out) p.trigger_out[c] = unc ? 1 : 0;
    }
    if (p.router && p.kmax > p.k_base) {
        const int w = p.kmax - p.k_base;
        for (int64_t i = tid; i < (int64_t)ncell * w; i += blockDim.x) {
            const int c = (int)(i / w);
            const float eff = p.grain_row ? s_row[c / p.Hq] : s_cell[c];
            const bool unc = p.mode_quantile ? (eff <= th) : (eff < th);
            if (!unc) p.kv_idx[(int64_t)c * p.kmax + p.k_base + (int)(i % w)] = p.NB;
        }
    }
}

int launch_decode_select(const void *Q, int dtype, int64_t qb, int64_t qh, const float *summ_a, const float *summ_b,
                         int NBs, int B, int Hq, int Hkv, int S, int D, float scale, bool quest, int k_base, int kmax,
                         bool router, int32_t *kv_idx, float *sigma_cell, cudaStream_t stream, const void *refresh_K,
                         ugbsa_strides refresh_ks) {
    if (Hq / Hkv > kDecMaxGroup) return UGBSA_ERR_UNSUPPORTED;
    if (D != 64 && D != 128 && D != 256) return UGBSA_ERR_UNSUPPORTED;
    DecSelParams p = {};
    p.rK = refresh_K;
    p.rkb = refresh_ks.b; p.rkh = refresh_ks.h; p.rks = refresh_ks.s;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = Hq / Hkv; p.S = S; p.NB = (S + 63) / 64; p.NBs = NBs;
    // a cluster per (b, kv head): enough CTAs for the group's heads or 128 summary rows
    // each, up to 16 when the device schedules clusters of 16 (else 8)
    int cl = (p.NB + 127) / 128;
    if (cl < p.G) cl = p.G;
    if (cl > 8) cl = kDecMaxCluster;
    // many groups (a batch of sequences): clusters of 8, half the CTAs (one CTA holds an SM)
    if ((int64_t)B * Hkv * cl > 148 && cl > 8) cl = 8;
    p.qb = qb; p.qh = qh; p.scale = scale;
    p.k_base = k_base; p.kmax = kmax; p.router = router ? 1 : 0;
    p.summ_a = summ_a; p.summ_b = summ_b; p.kv_idx = kv_idx; p.sigma_cell = sigma_cell;
    const int nch = quest ? 2 : 1;
    // the kernel for this shape (GM accumulators per lane: the group size rounded up to 4, 8 or 16)
    const int gm = p.G <= 4 ? 4 : (p.G <= 8 ? 8 : 16);
    void (*kern)(const void *, DecSelParams) = nullptr;
#define UGBSA_DEC_SEL_G(TT, DD, GG)                                                                                \
    if (gm == GG)                                                                                                  \
        kern = reinterpret_cast<void (*)(const void *, DecSelParams)>(                                             \
            quest ? decode_select_kernel<TT, true, DD, GG> : decode_select_kernel<TT, false, DD, GG>);
#define UGBSA_DEC_SEL(TT, DD)                                                                                      \
    if (D == DD) {                                                                                                 \
        UGBSA_DEC_SEL_G(TT, DD, 4) else UGBSA_DEC_SEL_G(TT, DD, 8) else UGBSA_DEC_SEL_G(TT, DD, 16)                \
    }
#define UGBSA_DEC_SEL_T(TT) UGBSA_DEC_SEL(TT, 64) else UGBSA_DEC_SEL(TT, 128) else UGBSA_DEC_SEL(TT, 256)
    switch (dtype) {
        case UGBSA_F32: UGBSA_DEC_SEL_T(float); break;
        case UGBSA_BF16: UGBSA_DEC_SEL_T(__nv_bfloat16); break;
        case UGBSA_F16: UGBSA_DEC_SEL_T(__half); break;
        default: return UGBSA_ERR_DTYPE;
    }
#undef UGBSA_DEC_SEL_T
#undef UGBSA_DEC_SEL
#undef UGBSA_DEC_SEL_G
    if (!kern) return UGBSA_ERR_UNSUPPORTED;
    if (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        cl = 8;
    // as many staged rounds (two 32-row tiles of both operands) in flight as the shared
    // memory allows (up to two); the cluster shrinks to 8 if the device cannot place 16
    const size_t tile = (size_t)2 * 2 * 32 * D * 4;
    const size_t budget_bytes = 200 * 1024;
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute at[2];
    size_t smem = 0;
    for (int attempt = 0; attempt < 2; ++attempt) {
        p.CL = cl;
        p.chunk = (p.NB + p.CL - 1) / p.CL;
        p.hpc = (p.G + p.CL - 1) / p.CL;
        const size_t rest = (size_t)nch * p.G * D * 4 + (size_t)p.hpc * ((p.NB + 3) & ~3) * 4 + (size_t)32 * 64 * 4;
        int nbuf = kDecSelMaxBufs;
        while (nbuf > 1 && (size_t)nbuf * tile + rest > budget_bytes) --nbuf;
        p.nbuf = nbuf;
        const size_t cand = (size_t)((p.NB + 1) & ~1) * 8;   // as the kernel lays it out
        const size_t tiles = (size_t)nbuf * tile > cand ? (size_t)nbuf * tile : cand;
        smem = tiles + rest;
        if (smem > budget_bytes) return UGBSA_ERR_SHAPE;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return UGBSA_ERR_LAUNCH;
        lc = cudaLaunchConfig_t{};
        lc.gridDim = dim3((unsigned)(B * Hkv * p.CL));
        lc.blockDim = dim3(kDecSelThreads);
        lc.dynamicSmemBytes = smem;
        lc.stream = stream;
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)p.CL;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // may overlap the refresh's tail
        at[1].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = at;
        lc.numAttrs = 2;
        if (cl <= 8) break;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &lc) == cudaSuccess && nclusters > 0) break;
        cudaGetLastError();
        cl = 8;
    }
    const cudaError_t e = cudaLaunchKernelEx(&lc, kern, Q, p);
    return e == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_decode_finish(const float *sigma_cell, int B, int Hq, int S, const ugbsa_selector_config *cfg, int k_base,
                         int kmax, int32_t *kv_idx, float *sigma_out, uint8_t *trigger_out, cudaStream_t stream) {
    if ((int64_t)B * Hq > 1024) return UGBSA_ERR_UNSUPPORTED;
    const bool router = (cfg->mode == UGBSA_MODE_ROUTER) && (k_base < kmax);
    if (!router && !sigma_out && !trigger_out) return UGBSA_OK;
    DecFinParams p;
    p.B = B; p.Hq = Hq; p.NB = (S + 63) / 64; p.k_base = k_base; p.kmax = kmax;
    p.router = router ? 1 : 0;
    p.grain_row = cfg->router_grain == UGBSA_GRAIN_ROW ? 1 : 0;
    p.mode_quantile = cfg->router_mode == UGBSA_ROUTER_QUANTILE ? 1 : 0;
    const int64_t numel = (int64_t)B * Hq;
    int64_t kq = (int64_t)(cfg->router_quantile * (double)numel);  // int(q * numel), :713-714
    if (kq < 1) kq = 1;
    if (kq > numel) kq = numel;
    p.kq = kq;
    p.tau = (float)cfg->router_tau;
    p.sigma_cell = sigma_cell; p.kv_idx = kv_idx; p.sigma_out = sigma_out; p.trigger_out = trigger_out;
    return launch_pdl(decode_finish_kernel, dim3(1), dim3(1024), 0, stream, p);
}

// ------------------------------------------------------------------ attention
struct DecAttnParams {
    int B, Hq, Hkv, G, S, NB, NBW, kmax, nsplit;
    int64_t qb, qh, ob, oh;
    float scale_log2, inv_kmax;
    const int32_t *kv_idx;
    float *part;   // [B*Hq, nsplit, D + 2]: o (unnormalised), m, l
    int *err;      // device error word (a wait that ran out)
    // the router of the selection's finish, taken here (ugbsa_decode_step; B * Hq <= 256):
    // each CTA derives its heads' triggers from the cells' margins; untriggered heads
    // keep slots < k_base only; split 0 writes sigma / trigger and the sentinel fill
    const float *sigma_cell;   // null: kv_idx is final
    int router, k_base, grain_row, mode_quantile;
    int64_t kq;
    float tau;
    int32_t *kv_idx_w;
    float *sigma_out;
    uint8_t *trigger_out;
};

// The finish's router for the G heads of group (b, kvh): bit g of the result set
// when head g is not triggered (its slots >= k_base are dropped).  One warp, on
// the cells' margins staged in shared memory (sig [B*Hq]; row [B] is scratch);
// the same arithmetic as decode_finish_kernel (row-grain head mean in head order,
// the quantile's k-th smallest by counting, NaN last).
__device__ uint32_t fused_router_untriggered(const DecAttnParams &p, int b, int kvh, int G, const float *sig,
                                             float *row, float *eff_out) {
    const int lane = threadIdx.x & 31;
    const int ncell = p.B * p.Hq;
    if (!p.router) {   // top-k / Quest modes: no margins, nothing dropped
        if (eff_out)
            for (int g = 0; g < G; ++g) eff_out[g] = __int_as_float(0x7fc00000);
        return 0u;
    }
    if (p.grain_row) {   // the head mean of each row, once
        for (int bb = lane; bb < p.B; bb += 32) {
            float acc = 0.f;
            for (int hh = 0; hh < p.Hq; ++hh) acc = __fadd_rn(acc, sig[bb * p.Hq + hh]);
            row[bb] = __fdiv_rn(acc, (float)p.Hq);
        }
        __syncwarp();
    }
    const float *vals = p.grain_row ? row : sig;
    float th = p.tau;
    if (p.mode_quantile) {
        const int n = p.grain_row ? p.B : ncell;
        const int64_t kk = p.grain_row ? (p.kq - 1) / p.Hq + 1 : p.kq;
        float found = 0.f;
        bool got = false;
        for (int i = lane; i < n; i += 32) {
            const uint32_t ui = asc_key_dec(vals[i]);
            int64_t rank = 0;
            for (int j = 0; j < n; ++j) {
                const uint32_t uj = asc_key_dec(vals[j]);
                rank += (uj < ui || (uj == ui && j < i)) ? 1 : 0;
            }
            if (rank == kk - 1) {
                found = (ui == 0xffffffffu) ? __int_as_float(0x7fc00000)
                                            : __uint_as_float((ui & 0x80000000u) ? (ui & 0x7fffffffu) : ~ui);
                got = true;
            }
        }
        const unsigned who = __ballot_sync(0xffffffffu, got);
        th = __shfl_sync(0xffffffffu, found, who ? __ffs(who) - 1 : 0);
    }
    uint32_t untrig = 0u;
    for (int g = 0; g < G; ++g) {
        const int cell = b * p.Hq + kvh * G + g;
        const float eff = p.grain_row ? row[b] : sig[cell];
        const bool unc = p.mode_quantile ? (eff <= th) : (eff < th);
        if (!unc) untrig |= 1u << g;
        if (eff_out) eff_out[g] = eff;
    }
    return untrig;
}

template <typename T> struct MmaOps;
template <> struct MmaOps<__nv_bfloat16> {
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
};
template <> struct MmaOps<__half> {
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        const __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// byte offset of 16-byte chunk c of row r in a swizzled [rows][D] 16-bit tile
// (the query rows, written by the threads)
template <int D>
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

// byte offset of chunk c of row r in a 64-row K / V tile as TMA writes it with
// the 128-byte swizzle: [D / 64 column slabs][64 rows][128 B], chunk c & 7 of a
// row stored at (c & 7) ^ (r & 7)
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
    return (uint32_t)((c >> 3) * (64 * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

constexpr int kDecAttnThreads = 128;

// shared memory: Q [16][D] | stages [2][K, V][64][D] | head bitmaps [G][NBW] | entries [cap]
template <int D> struct DecAttnCfg {
    static constexpr int STAGES = D <= 128 ? 3 : 2;   // K/V blocks in flight per CTA (two CTAs per SM at D <= 128)
};

template <typename T, int D>
__global__ void __launch_bounds__(kDecAttnThreads) decode_group_attn_kernel(const T *__restrict__ Q,
                                                                            const __grid_constant__ CUtensorMap mapK,
                                                                            const __grid_constant__ CUtensorMap mapV,
                                                                            const DecAttnParams p) {
    constexpr int CH = D / 8;             // 16-byte chunks per row
    constexpr int TILE = 64 * D * 2;      // bytes of one 64-row K or V tile
    constexpr int NT = D / 8;             // n-tiles of the output
    constexpr int STAGES = DecAttnCfg<D>::STAGES;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // stages first, 1024-byte aligned (the 128-byte swizzle's period)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sStage = smem;
    uint8_t *sQ = smem + STAGES * 2 * TILE;
    uint32_t *bm = reinterpret_cast<uint32_t *>(sQ + 16 * D * 2);
    uint32_t *entries = bm + p.G * p.NBW;
    __shared__ int s_dup, s_nent, s_abort;
    __shared__ uint32_t s_untrig;
    __shared__ float s_sig[256], s_row[256];
    __shared__ int s_wsum[kDecAttnThreads / 32];
    __shared__ __align__(8) uint64_t bar_full[STAGES];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    grid_dep_launch();
    grid_dep_wait();   // kv_idx (the selection's finish just before) is complete
    const int grp = blockIdx.x / p.nsplit, split = blockIdx.x % p.nsplit;
    const int kvh = grp % p.Hkv, b = grp / p.Hkv;
    const int G = p.G;
    const int cell0 = b * p.Hq + kvh * G;
    const bool use_bitmap = p.NBW > 0;

    // the first batch of the group's list ids (consecutive rows of kv_idx) and the
    // query rows are loaded together, before the bitmaps are cleared
    constexpr int IDB = 16;   // ids per thread per batch
    const int32_t *lists = p.kv_idx + (int64_t)cell0 * p.kmax;
    const int total = G * p.kmax;
    int ids[IDB];
#pragma unroll
    for (int u = 0; u < IDB; ++u) {
        const int i = u * kDecAttnThreads + tid;
        ids[u] = (use_bitmap && i < total) ? __ldg(lists + i) : -1;
    }
    // query rows (G of 16; the rest zero), swizzled for ldmatrix
    for (int i = tid; i < 16 * CH; i += kDecAttnThreads) {
        const int r = i / CH, c = i % CH;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < G) v = *reinterpret_cast<const uint4 *>(Q + (int64_t)b * p.qb + (int64_t)(kvh * G + r) * p.qh + c * 8);
        *reinterpret_cast<uint4 *>(sQ + tile_off<D>(r, c)) = v;
    }
    if (tid == 0) {
        s_dup = use_bitmap ? 0 : 1;
        s_abort = 0;
        for (int i = 0; i < STAGES; ++i) mbar_init(&bar_full[i], 1);
        fence_barrier_init();
    }
    if (p.sigma_cell) {   // the cells' margins (B * Hq <= 256), for the router below
        for (int i = tid; i < p.B * p.Hq; i += kDecAttnThreads) s_sig[i] = p.sigma_cell[i];
        __syncthreads();
    }
    if (warp == 0) {
        // the router (fused step): heads whose slots >= k_base are dropped
        uint32_t untrig = 0u;
        if (p.sigma_cell) {
            float eff[kDecMaxGroup];
            untrig = fused_router_untriggered(p, b, kvh, G, s_sig, s_row, eff);
            if (split == 0 && lane == 0)
                for (int g = 0; g < G; ++g) {
                    const int cell = cell0 + g;
                    if (p.sigma_out) p.sigma_out[cell] = eff[g];
                    // triggered: a router cell that kept its slots >= k_base (never without a router)
                    if (p.trigger_out) p.trigger_out[cell] = (p.router && !((untrig >> g) & 1u)) ? 1 : 0;
                }
        }
        if (lane == 0) s_untrig = untrig;
    }
    if (use_bitmap)
        for (int i = tid; i < G * p.NBW; i += kDecAttnThreads) bm[i] = 0u;
    __syncthreads();
    const uint32_t untrig_all = s_untrig;
    // the union of the group's lists: a bit per (head, block); a repeat marks the group.
    // The head of flat slot i is i / kmax, taken as (i + 0.5) * (1 / kmax) rounded down:
    // exact, since (i + 0.5) / kmax is at least 0.5 / kmax from an integer.
    if (use_bitmap) {
        for (int i0 = 0; i0 < total; i0 += IDB * kDecAttnThreads) {
            if (i0 > 0) {
#pragma unroll
                for (int u = 0; u < IDB; ++u) {
                    const int i = i0 + u * kDecAttnThreads + tid;
                    ids[u] = (i < total) ? __ldg(lists + i) : -1;
                }
            }
#pragma unroll
            for (int u = 0; u < IDB; ++u) {
                const int i = i0 + u * kDecAttnThreads + tid;
                const int blk = ids[u];
                if (i < total && blk >= 0 && blk < p.NB) {
                    const int g = (int)(((float)i + 0.5f) * p.inv_kmax);
                    if (((untrig_all >> g) & 1u) && i - g * p.kmax >= p.k_base) continue;   // dropped slot
                    const uint32_t bit = 1u << (blk & 31);
                    const uint32_t old = atomicOr(&bm[g * p.NBW + (blk >> 5)], bit);
                    if (old & bit) s_dup = 1;
                }
            }
        }
        __syncthreads();
    }
    int nent;
    if (!s_dup) {
        // entries = the union's block ids in order (the heads that keep one are read
        // from the bitmaps when it is used)
        const int per_t = (p.NBW + kDecAttnThreads - 1) / kDecAttnThreads;
        const int w0 = tid * per_t, w1 = min(p.NBW, w0 + per_t);
        int cnt = 0;
        for (int w = w0; w < w1; ++w) {
            uint32_t u = 0u;
#pragma unroll
            for (int g = 0; g < kDecMaxGroup; ++g)
                if (g < G) u |= bm[g * p.NBW + w];
            cnt += __popc(u);
        }
        // exclusive scan of the per-thread counts
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        if (lane == 31) s_wsum[warp] = incl;
        __syncthreads();
        int base = incl - cnt;
        for (int w = 0; w < warp; ++w) base += s_wsum[w];
        if (tid == kDecAttnThreads - 1) s_nent = base + cnt;
        for (int w = w0; w < w1; ++w) {
            uint32_t u = 0u;
#pragma unroll
            for (int g = 0; g < kDecMaxGroup; ++g)
                if (g < G) u |= bm[g * p.NBW + w];
            while (u) {
                const int bit = __ffs(u) - 1;
                u &= u - 1u;
                entries[base++] = (uint32_t)(w * 32 + bit);
            }
        }
        __syncthreads();
        nent = s_nent;
    } else {
        nent = G * p.kmax;   // slot by slot: entry e = head e / kmax, slot e % kmax
    }
    auto entry = [&](int e, int &blk, uint32_t &mask) {
        if (!s_dup) {
            blk = (int)entries[e];
            const int w = blk >> 5, bit = blk & 31;
            mask = 0u;
#pragma unroll
            for (int g = 0; g < kDecMaxGroup; ++g)
                if (g < G) mask |= ((bm[g * p.NBW + w] >> bit) & 1u) << g;
        } else {
            const int g = e / p.kmax, slot = e % p.kmax;
            blk = __ldg(p.kv_idx + (int64_t)(cell0 + g) * p.kmax + slot);
            const bool dropped = ((untrig_all >> g) & 1u) && slot >= p.k_base;
            mask = (!dropped && blk >= 0 && blk < p.NB) ? (1u << g) : 0u;
        }
    };
    const int per = (nent + p.nsplit - 1) / p.nsplit;
    const int e0 = split * per, e1 = min(nent, e0 + per);
    // the finish's sentinel fill of the untriggered heads' slots >= k_base (split 0,
    // after its own reads; the other splits drop those slots whatever they read)
    if (p.sigma_cell && split == 0 && untrig_all && p.kmax > p.k_base) {
        const int w = p.kmax - p.k_base;
        for (int i = tid; i < G * w; i += kDecAttnThreads) {
            const int g = i / w;
            if ((untrig_all >> g) & 1u) p.kv_idx_w[(int64_t)(cell0 + g) * p.kmax + p.k_base + i % w] = p.NB;
        }
    }

    // one thread issues a block's K and V tiles by TMA (rows past S arrive as zeros);
    // every thread waits on the stage's barrier, with a time limit
    const WaitCtx wc{p.err, &s_abort};
    auto issue = [&](int e, int stage) {
        int blk;
        uint32_t mask;
        entry(e, blk, mask);
        if (!mask) {
            mbar_arrive(&bar_full[stage]);   // nothing to load: complete the phase
            return;
        }
        uint8_t *sk = sStage + stage * 2 * TILE, *sv = sk + TILE;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bar_full[stage], 2 * TILE);
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
            tma_load_4d(sk + h * 64 * 128, &mapK, &bar_full[stage], h * 64, blk * 64, kvh, b);
            tma_load_4d(sv + h * 64 * 128, &mapV, &bar_full[stage], h * 64, blk * 64, kvh, b);
        }
    };

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;   // rows lane/4 and lane/4 + 8
    const int r_lo = lane >> 2, r_hi = r_lo + 8;
    const int mi = lane >> 3, rr = lane & 7;
    // the query rows' A fragments, loaded once
    uint32_t qa[D / 16][4];
    {
        const uint32_t aQ = smem_u32(sQ);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) ldsm_x4(aQ + tile_off<D>((mi & 1) * 8 + rr, 2 * ks + (mi >> 1)), qa[ks]);
    }

    // STAGES - 1 entries ahead of the one being computed
    int issued = e0;   // entries issued so far (thread 0's count; the others follow the same rule)
    if (tid == 0)
        for (; issued < min(e1, e0 + STAGES - 1); ++issued) issue(issued, (issued - e0) % STAGES);
    bool ok = true;
    for (int e = e0; e < e1; ++e) {
        const int st = (e - e0) % STAGES;
        if (tid == 0 && e + STAGES - 1 < e1) {
            issue(e + STAGES - 1, (e - e0 + STAGES - 1) % STAGES);
            issued = e + STAGES;
        }
        ok = mbar_wait(&bar_full[st], (uint32_t)(((e - e0) / STAGES) & 1), wc);
        if (__syncthreads_or(!ok)) {   // a wait ran out: drain this thread's issued loads below
            ok = false;
            if (tid == 0)
                for (int q = e; q < issued; ++q)
                    mbar_wait_drain(&bar_full[(q - e0) % STAGES], (uint32_t)(((q - e0) / STAGES) & 1), p.err);
            break;
        }
        int blk;
        uint32_t mask;
        entry(e, blk, mask);
        if (mask) {
            const uint32_t sk = smem_u32(sStage + st * 2 * TILE), sv = sk + TILE;
            // S = Q . K^T for keys 16w .. 16w+15 (two n-tiles)
            float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t bk[4];
                ldsm_x4(sk + kv_off(16 * warp + (mi >> 1) * 8 + rr, 2 * ks + (mi & 1)), bk);
                MmaOps<T>::mma(s0, qa[ks], bk[0], bk[1]);
                MmaOps<T>::mma(s1, qa[ks], bk[2], bk[3]);
            }
            // mask (heads of the entry, keys < S), scale to log2 units, online softmax per row
            const bool on_lo = (mask >> r_lo) & 1u, on_hi = (mask >> r_hi) & 1u;
            const int kc = blk * 64 + 16 * warp + (lane & 3) * 2;   // key of s0[0]; s0[1] +1; s1 +8
            float x[8] = {s0[0], s0[1], s1[0], s1[1], s0[2], s0[3], s1[2], s1[3]};
            const int kofs[4] = {0, 1, 8, 9};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const bool kin = kc + kofs[i] < p.S;
                x[i] = (on_lo && kin) ? x[i] * p.scale_log2 : -INFINITY;
                x[4 + i] = (on_hi && kin) ? x[4 + i] * p.scale_log2 : -INFINITY;
            }
            float mx_lo = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
            float mx_hi = fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7]));
            mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
            mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
            const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
            const float al_lo = (mn_lo == -INFINITY) ? 1.f : exp2f(m_lo - mn_lo);
            const float al_hi = (mn_hi == -INFINITY) ? 1.f : exp2f(m_hi - mn_hi);
            float pr[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pr[i] = (x[i] == -INFINITY) ? 0.f : exp2f(x[i] - mn_lo);
                pr[4 + i] = (x[4 + i] == -INFINITY) ? 0.f : exp2f(x[4 + i] - mn_hi);
            }
            float ps_lo = pr[0] + pr[1] + pr[2] + pr[3], ps_hi = pr[4] + pr[5] + pr[6] + pr[7];
            ps_lo += __shfl_xor_sync(0xffffffffu, ps_lo, 1);
            ps_lo += __shfl_xor_sync(0xffffffffu, ps_lo, 2);
            ps_hi += __shfl_xor_sync(0xffffffffu, ps_hi, 1);
            ps_hi += __shfl_xor_sync(0xffffffffu, ps_hi, 2);
            l_lo = l_lo * al_lo + ps_lo;
            l_hi = l_hi * al_hi + ps_hi;
            m_lo = mn_lo;
            m_hi = mn_hi;
            if (__any_sync(0xffffffffu, al_lo != 1.f || al_hi != 1.f)) {   // a row's maximum moved
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    o[j][0] *= al_lo;
                    o[j][1] *= al_lo;
                    o[j][2] *= al_hi;
                    o[j][3] *= al_hi;
                }
            }
            // O += P . V: P (16 heads x 16 keys) from the S fragments, V by transposed ldmatrix
            uint32_t pa[4];
            pa[0] = MmaOps<T>::pack(pr[0], pr[1]);   // row lo, keys 0-1 (+2*(lane&3))
            pa[1] = MmaOps<T>::pack(pr[4], pr[5]);   // row hi
            pa[2] = MmaOps<T>::pack(pr[2], pr[3]);   // row lo, keys 8-9
            pa[3] = MmaOps<T>::pack(pr[6], pr[7]);   // row hi, keys 8-9
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                uint32_t bv[4];
                ldsm_x4_t(sv + kv_off(16 * warp + (mi & 1) * 8 + rr, j + (mi >> 1)), bv);
                MmaOps<T>::mma(o[j], pa, bv[0], bv[1]);
                MmaOps<T>::mma(o[j + 1], pa, bv[2], bv[3]);
            }
        }
        __syncthreads();   // the stage is read; the next issue may overwrite it
    }

    if (!ok) {   // the step's result is void (the device error word says why): no contribution
        m_lo = m_hi = -INFINITY;
        l_lo = l_hi = 0.f;
    }
    // merge the four warps (their key quarters) through shared memory, then one partial per head
    constexpr int OS = D + 8;                             // padded row: float2 stores in two wavefronts
    float *sm = reinterpret_cast<float *>(sStage);        // [4 warps][16 rows] m, l
    float *sl = sm + 4 * 16;
    float *so = sl + 4 * 16;                              // [4 warps][16 rows][OS]
    if ((lane & 3) == 0) {
        sm[warp * 16 + r_lo] = m_lo;
        sm[warp * 16 + r_hi] = m_hi;
        sl[warp * 16 + r_lo] = l_lo;
        sl[warp * 16 + r_hi] = l_hi;
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int col = 8 * j + (lane & 3) * 2;
        *reinterpret_cast<float2 *>(so + (warp * 16 + r_lo) * OS + col) = make_float2(o[j][0], o[j][1]);
        *reinterpret_cast<float2 *>(so + (warp * 16 + r_hi) * OS + col) = make_float2(o[j][2], o[j][3]);
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kDecAttnThreads) {
        const int r = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + r]);
        float acc = 0.f, L = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float mw = sm[w * 16 + r];
                if (mw == -INFINITY) continue;
                const float f = exp2f(mw - M);
                acc += so[(w * 16 + r) * OS + d] * f;
                L += sl[w * 16 + r] * f;
            }
        }
        float *dst = p.part + ((int64_t)(cell0 + r) * p.nsplit + split) * (D + 2);
        dst[d] = acc;
        if (d == 0) {
            dst[D] = M;
            dst[D + 1] = L;
        }
    }
}

// one CTA per (b, q-head): the cell's partials [nsplit][D + 2] are brought into
// shared memory with every copy in flight at once, then merged there
template <typename T, int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(const DecAttnParams p, T *__restrict__ out) {
    extern __shared__ __align__(16) float s_part[];   // [nsplit][D + 2], then the factors [nsplit]
    __shared__ float s_M, s_L;
    const int cell = blockIdx.x;
    const int h = cell % p.Hq, b = cell / p.Hq;
    const int d = threadIdx.x;
    grid_dep_wait();   // every split's partials are written
    const int nfl = p.nsplit * (D + 2);
    const float *base = p.part + (int64_t)cell * nfl;
    float *s_f = s_part + ((nfl + 3) & ~3);
    if ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) {   // nsplit even: every cell's partials 16-byte aligned
        const int n16 = nfl / 4;
        for (int i = d; i < n16; i += D) cp_async16(s_part + 4 * i, base + 4 * i);
        cp_async_commit();
        for (int i = 4 * n16 + d; i < nfl; i += D) s_part[i] = base[i];
        cp_async_wait_all();
    } else {
        for (int i = d; i < nfl; i += D) s_part[i] = base[i];
    }
    __syncthreads();
    if (d < 32) {
        float M = -INFINITY;
        for (int s = d; s < p.nsplit; s += 32) M = fmaxf(M, s_part[s * (D + 2) + D]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int s = d; s < p.nsplit; s += 32) {
            const float ms = s_part[s * (D + 2) + D];
            const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
            L += s_part[s * (D + 2) + D + 1] * f;
            s_f[s] = f;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        if (d == 0) {
            s_M = M;
            s_L = L;
        }
    }
    __syncthreads();
    float o = 0.f;
    if (s_M != -INFINITY)
        for (int s = 0; s < p.nsplit; ++s) o += s_part[s * (D + 2) + d] * s_f[s];
    const float L = s_L;
    const float r = (L > 0.f) ? o / L : 0.f;
    T *dst = out + (int64_t)b * p.ob + (int64_t)h * p.oh + d;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) *dst = __float2bfloat16_rn(r);
    else *dst = __float2half_rn(r);
}

// splits per KV group, at most: a CTA per block of a list (the union of the group's
// lists is longer), bounded so that all cells x splits stay within ~4800 partials
// (the workspace is sized by this bound)
int decode_nsplit(int B, int Hq, int kmax) {
    int ns = kmax;
    int cap = (int)((4800 + (int64_t)B * Hq - 1) / ((int64_t)B * Hq));
    if (cap > 512) cap = 512;
    if (ns > cap) ns = cap;
    return ns < 1 ? 1 : ns;
}

// the splits used: about two CTAs per SM over all (b, kv head) groups, an even
// count where the bound allows (each cell's partials then start 16-byte aligned)
// (UGBSA_DECODE_CTAS_PER_SM overrides the two, for tuning)
static int decode_nsplit_used(int B, int Hq, int Hkv, int kmax) {
    const int ns = decode_nsplit(B, Hq, kmax);
    int per_sm = 2;
    if (const char *e = getenv("UGBSA_DECODE_CTAS_PER_SM")) per_sm = atoi(e) > 0 ? atoi(e) : 2;
    int64_t want = ((int64_t)per_sm * 148 + (int64_t)B * Hkv - 1) / ((int64_t)B * Hkv);
    want += want & 1;
    return (int)(want < ns ? want : ns);
}

size_t decode_attn_workspace_bytes(int B, int Hq, int D, int kmax) {
    return (size_t)B * Hq * decode_nsplit(B, Hq, kmax) * (D + 2) * 4;
}

int launch_decode_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                       ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int S, int D,
                       float scale, void *out, ugbsa_strides os, void *workspace, cudaStream_t stream,
                       const DecodeRouter *router) {
    DecAttnParams p = {};
    if (router) {
        if ((int64_t)B * Hq > 256) return UGBSA_ERR_UNSUPPORTED;
        const ugbsa_selector_config *cfg = router->cfg;
        p.sigma_cell = router->sigma_cell;
        p.router = (cfg->mode == UGBSA_MODE_ROUTER) && (router->k_base < kmax) ? 1 : 0;
        p.k_base = router->k_base;
        p.grain_row = cfg->router_grain == UGBSA_GRAIN_ROW ? 1 : 0;
        p.mode_quantile = cfg->router_mode == UGBSA_ROUTER_QUANTILE ? 1 : 0;
        const int64_t numel = (int64_t)B * Hq;
        int64_t kq = (int64_t)(cfg->router_quantile * (double)numel);  // int(q * numel), :713-714
        if (kq < 1) kq = 1;
        if (kq > numel) kq = numel;
        p.kq = kq;
        p.tau = (float)cfg->router_tau;
        p.kv_idx_w = router->kv_idx;
        p.sigma_out = router->sigma_out;
        p.trigger_out = router->trigger_out;
    }
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = Hq / Hkv; p.S = S; p.NB = (S + 63) / 64; p.kmax = kmax;
    if (p.G > kDecMaxGroup) return UGBSA_ERR_UNSUPPORTED;
    // the union is built in shared memory when its bitmaps and list fit (NB <= 8192); else slot by slot
    p.NBW = (p.NB <= 8192) ? (p.NB + 31) / 32 : 0;
    p.nsplit = decode_nsplit_used(B, Hq, Hkv, kmax);
    p.qb = qs.b; p.qh = qs.h;
    p.ob = os.b; p.oh = os.h;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.inv_kmax = (float)(1.0 / (double)kmax);
    p.kv_idx = kv_idx;
    p.part = static_cast<float *>(workspace);
    p.err = device_error_word();
    if (!p.err) return UGBSA_ERR_NO_DEVICE;
    // K / V as [B, Hkv, S, D] tensors, 64-column x 64-row boxes with the 128-byte swizzle;
    // rows at or past S (the cache's unused capacity) read as zeros
    CUtensorMap mapK, mapV;
    {
        const CUtensorMapDataType dt =
            dtype == UGBSA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)Hkv, (cuuint64_t)B};
        cuuint32_t box[4] = {64, 64, 1, 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        cuuint64_t kst[3] = {(cuuint64_t)ks.s * 2, (cuuint64_t)ks.h * 2, (cuuint64_t)ks.b * 2};
        cuuint64_t vst[3] = {(cuuint64_t)vs.s * 2, (cuuint64_t)vs.h * 2, (cuuint64_t)vs.b * 2};
        int rc = encode_tensor_map(&mapK, dt, 4, const_cast<void *>(K), dims, kst, box, es);
        if (rc == UGBSA_OK) rc = encode_tensor_map(&mapV, dt, 4, const_cast<void *>(V), dims, vst, box, es);
        if (rc != UGBSA_OK) return rc;
    }
    int cap = p.G * kmax;
    if (cap > p.NB) cap = p.NB;
    const int stages = D <= 128 ? DecAttnCfg<128>::STAGES : DecAttnCfg<256>::STAGES;
    const size_t stage = (size_t)stages * 2 * 64 * D * 2;
    const size_t merge = (size_t)4 * 16 * (2 + D + 8) * 4;   // reuses the stages
    const size_t smem = 1024 + (stage > merge ? stage : merge) + (size_t)16 * D * 2 +
                        (p.NBW ? (size_t)p.G * p.NBW * 4 + (size_t)cap * 4 : 0);
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    // the combine holds one cell's partials and their factors
    const int nfl = p.nsplit * (D + 2);
    const size_t csmem = (size_t)((nfl + 3) & ~3) * 4 + (size_t)p.nsplit * 4;
    if (csmem > 227 * 1024) return UGBSA_ERR_SHAPE;
    const dim3 grid((unsigned)(B * Hkv * p.nsplit));
#define UGBSA_DEC_ATTN(TT, DD)                                                                                     \
    if (D == DD) {                                                                                                 \
        auto k = decode_group_attn_kernel<TT, DD>;                                                                 \
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)        \
            return UGBSA_ERR_LAUNCH;                                                                               \
        int rc_ = launch_pdl(k, grid, dim3(kDecAttnThreads), smem, stream, (const TT *)Q, mapK, mapV, p);          \
        if (rc_ != UGBSA_OK) return rc_;                                                                           \
        auto kc = decode_combine_kernel<TT, DD>;                                                                   \
        if (cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem) != cudaSuccess)      \
            return UGBSA_ERR_LAUNCH;                                                                               \
        return launch_pdl(kc, dim3((unsigned)(B * Hq)), dim3(DD), csmem, stream, p, (TT *)out);                    \
    }
    if (dtype == UGBSA_BF16) {
        UGBSA_DEC_ATTN(__nv_bfloat16, 64)
        UGBSA_DEC_ATTN(__nv_bfloat16, 128)
        UGBSA_DEC_ATTN(__nv_bfloat16, 256)
    } else {
        UGBSA_DEC_ATTN(__half, 64)
        UGBSA_DEC_ATTN(__half, 128)
        UGBSA_DEC_ATTN(__half, 256)
    }
#undef UGBSA_DEC_ATTN
    return UGBSA_ERR_UNSUPPORTED;
}

}  // namespace ugbsa
