// attn.cu -- block-sparse causal attention over per-tile kv_idx lists (sm_100a).
//
// Replaces the reference's Triton kernel _fwd_kernel_v2 / block_sparse_attn_v2
// (src/triton_block_attn.py:184-298) with the same semantics:
//   for each (b, q-head h, 64-row tile t), visit the slots of kv_idx[b,h,t,:] in
//   order; skip the sentinel (>= NB) and blocks that start after the tile's last
//   row (:231-233); S = Q K^T * scale with the causal (key <= row) and bounds
//   (key < Sk) masks (:243-246); online softmax in fp32; O += P(bf16) V; O / l
//   with an l > 0 guard (:261); output in the input dtype.
// GQA is resolved by reading KV head h / (Hq/Hkv) directly (no repeat_kv copy).
//
// B200 design.  One CTA per (b, h, t); 7 warps:
//   warps 0-3  softmax: S from TMEM (tcgen05.ld 16x256b), fp32 online softmax
//              with a lazy rescale (the running max only moves when a row's max
//              grows by more than 2^8, so O is rarely touched), P -> bf16 ->
//              TMEM (tcgen05.st 16x128b: the key pairs a thread holds are the
//              P columns it stores), epilogue O / l.
//   warp 4     K producer: compacts the tile's kv_idx to the usable blocks,
//              TMA-loads Q once and two K blocks per step.
//   warp 5     MMA issuer (one thread): tcgen05.mma kind::f16, M=64 (the tile's
//              64 query rows), N=128 (two key blocks per step), fp32 in TMEM;
//              P.V takes its A operand (P) from TMEM.
//   warp 6     V producer: two V blocks per step.
// TMEM (256 columns for D <= 128, 2 CTAs per SM): an M=64 accumulator or A
// operand takes 16 lanes of each 32-lane subpartition.  S is double-buffered
// in lanes 16-31 (columns [0,128) even steps, [128,256) odd steps); O takes
// lanes 0-15 of columns [0,D) and P lanes 0-15 of columns [D, D+64): an A
// operand in TMEM must sit in the same lanes as the accumulator it feeds.
// P never goes through shared memory, which leaves the K / V copies and the
// Q, K and V operand reads as the shared-memory traffic of a step.  The MMA
// thread issues QK^T(i+2) right after PV(i), so the tensor core computes the
// next scores while the softmax warps work on the current ones.
// Every mbarrier wait is time-bounded (common.cuh); on expiry the kernel
// records an error bit, drains its in-flight copies and MMAs, frees TMEM and
// returns.
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "ugbsa_internal.h"

namespace ugbsa {

template <int D, int VST = 1>   // VST: V stages (two at head dim 256, where one CTA holds an SM)
struct AttnSmem {
    static constexpr int DH = D / 64;                  // 64-column (128 B) slabs of a row
    static constexpr int Q_BYTES = DH * 64 * 128;      // [dh][64 rows][128 B]
    static constexpr int K_BYTES = DH * 128 * 128;     // [dh][128 keys][128 B]
    static constexpr int V_BYTES = DH * 128 * 128;     // [dh][128 keys][128 B]
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + K_BYTES;
    static constexpr int OFF_LIST = OFF_V + VST * V_BYTES;   // int32[kmax]
    // lanes 16-31: two S buffers of 128 columns; lanes 0-15: O (D columns) + P (64)
    static constexpr int TMEM_COLS = (D + 64) <= 256 ? 256 : 512;
    static_assert(2 * 128 <= TMEM_COLS && D + 64 <= TMEM_COLS, "S, O and P must fit the TMEM allocation");
};

constexpr int kAttnThreads = 224;
constexpr int kMaxDest = 8;
constexpr float kRescaleThreshold = 8.0f;  // log2 domain
constexpr uint32_t kLane16 = 16u << 16;    // TMEM address of lane 16

struct AttnParams {
    const int32_t *kv_idx;
    int kmax;
    int B, Hq, Hkv, Sq, Sk, Qt, NB;
    int t_base, pair_stride;   // local tile t (Q rows 64t ..) is sequence tile seq_tile(t, t_base, pair_stride)
    int out_row0, row_limit;   // sequence row g goes to out row g - out_row0 when g < row_limit
    float scale_log2;
    void *out;
    int64_t os_b, os_h, os_s;
    int *err;
    // output copies: dest[0] = out, dest[1 .. ndest-1] = the same view in peer
    // GPUs' buffers (NVLink stores; identical strides)
    void *dest[kMaxDest];
    int ndest;
    // optional per-row keep mask [B, Hq, Sq, nbw] (the v1 per-row selector): a row
    // uses a listed block only if its bit is set (triton_block_attn.py:87-104)
    const uint32_t *rowmask;
    int nbw;
};

__device__ __forceinline__ void tmem_ld16x256_x16(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// 16 lanes x 64 columns: thread t gives lane t/4 (register 2j) and lane t/4 + 8
// (register 2j+1) of column 4j + t%4, j = 0..15
__device__ __forceinline__ void tmem_st16x128_x16(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x128b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// tcgen05.mma kind::f16 with the A operand in TMEM (K-major; its lanes those of d_tmem)
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st16x256_x4(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

template <int D, bool BF16, int VST = 1>
__global__ void __launch_bounds__(kAttnThreads, (D <= 128) ? 2 : 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                    const __grid_constant__ CUtensorMap mapV, const AttnParams p) {
    using L = AttnSmem<D, VST>;
    constexpr int DH = L::DH;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem + L::OFF_Q;
    uint8_t *sK = smem + L::OFF_K;
    uint8_t *sV = smem + L::OFF_V;
    int32_t *sList = reinterpret_cast<int32_t *>(smem + L::OFF_LIST);

    __shared__ uint64_t bar_q_full, bar_k_full, bar_k_empty, bar_v_full[2], bar_v_empty[2], bar_s_full[2],
        bar_p_full, bar_p_free, bar_o_done;
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_nvalid;
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // work item: heads-major, tiles heavy-first within a head (keeps one KV
    // head's blocks hot in L2 while its Q heads sweep their tiles)
    const int item = blockIdx.x;
    const int t = p.Qt - 1 - (item % p.Qt);
    const int bh = item / p.Qt;
    const int h = bh % p.Hq;
    const int b = bh / p.Hq;
    const int kvh = h / (p.Hq / p.Hkv);
    const int tile_row = t * 64;                                       // first row of the tile in Q
    const int tile_first = 64 * seq_tile(t, p.t_base, p.pair_stride);  // its sequence position
    const int tile_last = tile_first + 63;

    if (threadIdx.x == 0) {
        mbar_init(&bar_q_full, 1);
        mbar_init(&bar_k_full, 1);
        mbar_init(&bar_k_empty, 1);
        mbar_init(&bar_v_full[0], 1);
        mbar_init(&bar_v_empty[0], 1);
        mbar_init(&bar_v_full[1], 1);
        mbar_init(&bar_v_empty[1], 1);
        mbar_init(&bar_s_full[0], 1);
        mbar_init(&bar_s_full[1], 1);
        mbar_init(&bar_p_full, 4);
        mbar_init(&bar_p_free, 1);
        mbar_init(&bar_o_done, 1);
        fence_barrier_init();
        s_abort = 0;
    }
    if (warp == 5) {
        tmem_alloc(&s_tmem_base, L::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 4) {
        // compact the usable slots, keeping slot order
        const int32_t *row = p.kv_idx + ((int64_t)(b * p.Hq + h) * p.Qt + t) * p.kmax;
        int n = 0;
        for (int base = 0; base < p.kmax; base += 32) {
            const int j = base + lane;
            int blk = (j < p.kmax) ? __ldg(row + j) : -1;
            const bool ok = (blk >= 0) && (blk < p.NB) && (blk * 64 <= tile_last);
            const unsigned m = __ballot_sync(0xffffffffu, ok);
            if (ok) sList[n + __popc(m & ((1u << lane) - 1u))] = blk;
            n += __popc(m);
        }
        if (lane == 0) {
            s_nvalid = n;
            tma_prefetch_desc(&mapQ);
            tma_prefetch_desc(&mapK);
            tma_prefetch_desc(&mapV);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem_base;
    const uint32_t tS = tmem + kLane16;  // lanes 16-31: columns [0,128) even steps, [128,256) odd steps
    const uint32_t tO = tmem;            // lanes 0-15, columns [0, D)
    const uint32_t tP = tmem + D;        // lanes 0-15, columns [D, D+64): P as bf16 / fp16 pairs
    const int nvalid = s_nvalid;
    const int nsteps = (nvalid + 1) >> 1;
    const WaitCtx wc{p.err, &s_abort};

    if (warp == 4) {
        if (lane == 0) {
            // ---------------- K producer (and Q)
            bool ok = true;
            mbar_arrive_expect_tx(&bar_q_full, 64 * D * 2);
            for (int dh = 0; dh < DH; ++dh) tma_load_4d(sQ + dh * 8192, &mapQ, &bar_q_full, 64 * dh, tile_row, h, b);
            int issued = -1;
            for (int i = 0; i < nsteps && ok; ++i) {
                const int nb = min(2, nvalid - 2 * i);
                ok = mbar_wait(&bar_k_empty, (i & 1) ^ 1, wc);
                if (!ok) break;
                mbar_arrive_expect_tx(&bar_k_full, nb * 64 * D * 2);
                for (int j = 0; j < nb; ++j) {
                    const int blk = sList[2 * i + j];
                    for (int dh = 0; dh < DH; ++dh)
                        tma_load_4d(sK + dh * 16384 + j * 8192, &mapK, &bar_k_full, 64 * dh, blk * 64, kvh, b);
                }
                issued = i;
            }
            if (!ok) {
                mbar_wait_drain(&bar_q_full, 0, p.err);
                if (issued >= 0) mbar_wait_drain(&bar_k_full, issued & 1, p.err);
            }
        }
    } else if (warp == 6) {
        if (lane == 0) {
            // ---------------- V producer
            bool ok = true;
            int issued = -1;
            for (int i = 0; i < nsteps && ok; ++i) {
                const int nb = min(2, nvalid - 2 * i);
                const int vs = i % VST;                            // the step's V stage and its use count
                const uint32_t vph = (uint32_t)((i / VST) & 1);
                ok = mbar_wait(&bar_v_empty[vs], vph ^ 1, wc);
                if (!ok) break;
                mbar_arrive_expect_tx(&bar_v_full[vs], nb * 64 * D * 2);
                for (int j = 0; j < nb; ++j) {
                    const int blk = sList[2 * i + j];
                    for (int dh = 0; dh < DH; ++dh)
                        tma_load_4d(sV + vs * L::V_BYTES + dh * 16384 + j * 8192, &mapV, &bar_v_full[vs], 64 * dh,
                                    blk * 64, kvh, b);
                }
                issued = i;
            }
            if (!ok)   // the copies of the last VST issued steps may still be in flight
                for (int q = max(0, issued - VST + 1); q <= issued; ++q)
                    mbar_wait_drain(&bar_v_full[q % VST], (uint32_t)((q / VST) & 1), p.err);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            // ---------------- MMA issuer: QK(0), QK(1), then PV(i), QK(i+2)
            constexpr uint32_t idesc_qk2 = idesc_f16(64, 128, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t idesc_qk1 = idesc_f16(64, 64, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t idesc_pv = idesc_f16(64, D, BF16 ? 1 : 0, 0, 1);
            const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
            auto issue_qk = [&](int j) -> bool {
                if (!mbar_wait(&bar_k_full, j & 1, wc)) return false;
                tc_fence_after();
                const int nb = min(2, nvalid - 2 * j);
                const uint32_t idqk = (nb == 2) ? idesc_qk2 : idesc_qk1;
                const uint32_t dS = tS + ((j & 1) ? 128u : 0u);
#pragma unroll
                for (int s = 0; s < 4 * DH; ++s) {
                    const uint64_t da = smem_desc_sw128(aQ + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024);
                    const uint64_t db = smem_desc_sw128(aK + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
                    umma_f16_ss(dS, da, db, idqk, s > 0 ? 1u : 0u);
                }
                umma_commit(&bar_k_empty);
                umma_commit(&bar_s_full[j & 1]);
                return true;
            };
            bool ok = mbar_wait(&bar_q_full, 0, wc);
            for (int j = 0; j < 2 && j < nsteps && ok; ++j) ok = issue_qk(j);
            for (int i = 0; i < nsteps && ok; ++i) {
                const int nb = min(2, nvalid - 2 * i);
                ok = mbar_wait(&bar_p_full, i & 1, wc);
                if (!ok) break;
                ok = mbar_wait(&bar_v_full[i % VST], (uint32_t)((i / VST) & 1), wc);
                if (!ok) break;
                tc_fence_after();
                const uint32_t aVs = aV + (uint32_t)((i % VST) * L::V_BYTES);
                for (int s = 0; s < 4 * nb; ++s) {
                    // keys 16s .. 16s+15: P columns 8s .. 8s+7
                    const uint64_t db = smem_desc_sw128(aVs + s * 2048, 16384, 1024);
                    umma_f16_ts(tO, tP + 8 * s, db, idesc_pv, (i > 0 || s > 0) ? 1u : 0u);
                }
                umma_commit(&bar_v_empty[i % VST]);
                umma_commit(&bar_p_free);
                if (i + 2 < nsteps) ok = issue_qk(i + 2);
            }
            // completion of everything issued (also the drain on the error path)
            umma_commit(&bar_o_done);
            if (!ok) mbar_wait_drain(&bar_o_done, 0, p.err);
        }
    } else {
        // ---------------- softmax warps 0-3 (rows 16w .. 16w+15 of the tile)
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const int r0 = warp * 16 + (lane >> 2);   // tile-local rows r0, r0 + 8
        const int g0 = tile_first + r0, g1 = g0 + 8;
        const int cq = 2 * (lane & 3);            // column offset inside each 8-column chunk
        const float sl2 = p.scale_log2;
        float m0 = -INFINITY, m1 = -INFINITY;     // running max of raw scores (reference point)
        float l0 = 0.f, l1 = 0.f;                 // per-thread partial row sums
        bool ok = true;
        for (int i = 0; i < nsteps; ++i) {
            const int nb = min(2, nvalid - 2 * i);
            ok = __all_sync(0xffffffffu, mbar_wait(&bar_s_full[i & 1], (i >> 1) & 1, wc));
            if (!ok) break;
            tc_fence_after();
            uint32_t sr[64];
            tmem_ld16x256_x16(tS + lane_base + ((i & 1) ? 128u : 0u), sr);
            tmem_wait_ld();
            reg_fence(sr);
            // keys of this step: block j covers columns [64j, 64j+64)
            const int blk0 = sList[2 * i];
            const int blk1 = (nb == 2) ? sList[2 * i + 1] : -1;
            const bool mask0 = (blk0 * 64 + 63 > tile_first) || (blk0 * 64 + 63 >= p.Sk);
            const bool mask1 = (nb == 2) && ((blk1 * 64 + 63 > tile_first) || (blk1 * 64 + 63 >= p.Sk));
            float x[64];
#pragma unroll
            for (int e = 0; e < 64; ++e) x[e] = __uint_as_float(sr[e]);
            if (nb == 1) {
#pragma unroll
                for (int e = 32; e < 64; ++e) x[e] = -INFINITY;
            }
            if (p.rowmask) {
                // rows of the tile that did not select a listed block: -inf there
                const int64_t rbase = ((int64_t)b * p.Hq + h) * p.Sq + tile_row;
                const int lr0 = r0, lr1 = r0 + 8;
                const bool in0 = tile_row + lr0 < p.Sq, in1 = tile_row + lr1 < p.Sq;
                const uint32_t *m0p = p.rowmask + (rbase + (in0 ? lr0 : 0)) * p.nbw;
                const uint32_t *m1p = p.rowmask + (rbase + (in1 ? lr1 : 0)) * p.nbw;
                const bool k00 = !in0 || ((__ldg(m0p + (blk0 >> 5)) >> (blk0 & 31)) & 1u);
                const bool k10 = !in1 || ((__ldg(m1p + (blk0 >> 5)) >> (blk0 & 31)) & 1u);
                const bool k01 = nb < 2 || !in0 || ((__ldg(m0p + (blk1 >> 5)) >> (blk1 & 31)) & 1u);
                const bool k11 = nb < 2 || !in1 || ((__ldg(m1p + (blk1 >> 5)) >> (blk1 & 31)) & 1u);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const bool keep0 = (c < 8) ? k00 : k01, keep1 = (c < 8) ? k10 : k11;
                    if (!keep0) { x[4 * c] = -INFINITY; x[4 * c + 1] = -INFINITY; }
                    if (!keep1) { x[4 * c + 2] = -INFINITY; x[4 * c + 3] = -INFINITY; }
                }
            }
            if (mask0 || mask1) {
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int j = c >> 3;
                    if ((j == 0 && !mask0) || (j == 1 && !mask1)) continue;
                    const int key = (j == 0 ? blk0 : blk1) * 64 + (c & 7) * 8 + cq;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int kk = key + e;
                        if (kk > g0 || kk >= p.Sk) x[4 * c + e] = -INFINITY;
                        if (kk > g1 || kk >= p.Sk) x[4 * c + 2 + e] = -INFINITY;
                    }
                }
            }
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                mx0 = fmax3f(mx0, x[4 * c], x[4 * c + 1]);
                mx1 = fmax3f(mx1, x[4 * c + 2], x[4 * c + 3]);
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            // lazy rescale: move the reference max only when it grows by > 2^8 (log2 units)
            float alpha0 = 1.f, alpha1 = 1.f;
            const bool up0 = (mx0 - m0) * sl2 > kRescaleThreshold;
            const bool up1 = (mx1 - m1) * sl2 > kRescaleThreshold;
            if (up0) { alpha0 = (m0 == -INFINITY) ? 0.f : fast_exp2((m0 - mx0) * sl2); m0 = mx0; l0 *= alpha0; }
            if (up1) { alpha1 = (m1 == -INFINITY) ? 0.f : fast_exp2((m1 - mx1) * sl2); m1 = mx1; l1 *= alpha1; }
            const float nb0 = (m0 == -INFINITY) ? 0.f : -m0 * sl2;
            const float nb1 = (m1 == -INFINITY) ? 0.f : -m1 * sl2;
            // P = exp2(s * scale*log2e - m * scale*log2e), packed to 16-bit pairs
            // exponent arguments and row sums on fp32 pairs (one instruction per two values)
            uint32_t pk[32];
            const uint64_t sl2x2 = f32x2(sl2, sl2), nb0x2 = f32x2(nb0, nb0), nb1x2 = f32x2(nb1, nb1);
            uint64_t ps0 = f32x2(0.f, 0.f), ps1 = ps0;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                float a00, a01, a10, a11;
                f32x2_split(ffma_x2(f32x2(x[4 * c + 0], x[4 * c + 1]), sl2x2, nb0x2), a00, a01);
                f32x2_split(ffma_x2(f32x2(x[4 * c + 2], x[4 * c + 3]), sl2x2, nb1x2), a10, a11);
                const float p00 = fast_exp2(a00), p01 = fast_exp2(a01);
                const float p10 = fast_exp2(a10), p11 = fast_exp2(a11);
                ps0 = fadd_x2(ps0, f32x2(p00, p01));
                ps1 = fadd_x2(ps1, f32x2(p10, p11));
                pk[2 * c] = BF16 ? pack_bf16x2(p00, p01) : pack_f16x2(p00, p01);
                pk[2 * c + 1] = BF16 ? pack_bf16x2(p10, p11) : pack_f16x2(p10, p11);
            }
            {
                float s0a, s0b, s1a, s1b;
                f32x2_split(ps0, s0a, s0b);
                f32x2_split(ps1, s1a, s1b);
                l0 += s0a + s0b;
                l1 += s1a + s1b;
            }
            // P(i-1) consumed and O up to date once PV(i-1) has completed
            if (i > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(&bar_p_free, (i - 1) & 1, wc));
                if (!ok) break;
                tc_fence_after();
                if (__any_sync(0xffffffffu, up0 || up1)) {
#pragma unroll
                    for (int cc = 0; cc < D / 32; ++cc) {
                        uint32_t o[16];
                        tmem_ld16x256_x4(tO + lane_base + cc * 32, o);
                        tmem_wait_ld();
                        reg_fence(o);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            o[4 * q4 + 0] = __float_as_uint(__uint_as_float(o[4 * q4 + 0]) * alpha0);
                            o[4 * q4 + 1] = __float_as_uint(__uint_as_float(o[4 * q4 + 1]) * alpha0);
                            o[4 * q4 + 2] = __float_as_uint(__uint_as_float(o[4 * q4 + 2]) * alpha1);
                            o[4 * q4 + 3] = __float_as_uint(__uint_as_float(o[4 * q4 + 3]) * alpha1);
                        }
                        tmem_st16x256_x4(tO + lane_base + cc * 32, o);
                    }
                    tmem_wait_st();
                }
            }
            // P -> TMEM: pk[2c] / pk[2c+1] hold keys 8c + cq, +1 of rows r0 / r0 + 8,
            // i.e. P column 4c + (lane & 3): the 16x128b store's layout
            tmem_st16x128_x16(tP + lane_base, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_p_full);
        }
        // ---------------- epilogue
        if (ok && nsteps > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bar_o_done, 0, wc));
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        const float inv0 = (l0 > 0.f) ? 1.f / l0 : 0.f;
        const float inv1 = (l1 > 0.f) ? 1.f / l1 : 0.f;
        bool direct = true;   // registers -> global (D = 256)
        if constexpr (D <= 128) {
            {
                direct = false;
                // Stage the tile in the K stage (free once O is done), 16-byte chunks
                // XOR-swizzled by row, then every thread stores whole 16-byte chunks, a
                // warp covering contiguous rows: full-line writes to this GPU's output
                // and to each peer's copy (NVLink).  About 1.5% faster than 4-byte stores
                // from the accumulator registers even for one destination.
                constexpr int RB = D * 2;    // bytes per staged row
                if (ok) {
                    tc_fence_after();
#pragma unroll
                    for (int cc = 0; cc < D / 32; ++cc) {
                        uint32_t o[16];
                        if (nsteps > 0) {
                            tmem_ld16x256_x4(tO + lane_base + cc * 32, o);
                            tmem_wait_ld();
                            reg_fence(o);
                        } else {
#pragma unroll
                            for (int e = 0; e < 16; ++e) o[e] = 0u;
                        }
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            const int ch = cc * 4 + q4;
                            const uint32_t wa = BF16 ? pack_bf16x2(__uint_as_float(o[4 * q4 + 0]) * inv0,
                                                                   __uint_as_float(o[4 * q4 + 1]) * inv0)
                                                     : pack_f16x2(__uint_as_float(o[4 * q4 + 0]) * inv0,
                                                                  __uint_as_float(o[4 * q4 + 1]) * inv0);
                            const uint32_t wb = BF16 ? pack_bf16x2(__uint_as_float(o[4 * q4 + 2]) * inv1,
                                                                   __uint_as_float(o[4 * q4 + 3]) * inv1)
                                                     : pack_f16x2(__uint_as_float(o[4 * q4 + 2]) * inv1,
                                                                  __uint_as_float(o[4 * q4 + 3]) * inv1);
                            const int off = ((ch ^ (r0 & 7)) << 4) + cq * 2;
                            *reinterpret_cast<uint32_t *>(sK + r0 * RB + off) = wa;
                            *reinterpret_cast<uint32_t *>(sK + (r0 + 8) * RB + off) = wb;
                        }
                    }
                }
                named_bar_sync(1, 128);
                if (ok && *(volatile int *)&s_abort == 0) {
                    constexpr int CPR = D / 8;              // 16-byte chunks per row
                    constexpr int NCH = 64 * CPR / 128;     // chunks per thread
                    const int tid = threadIdx.x;            // softmax warps are threads 0..127
                    uint4 v[NCH];
#pragma unroll
                    for (int k = 0; k < NCH; ++k) {
                        const int idx = tid + k * 128, r = idx / CPR, c = idx % CPR;
                        v[k] = *reinterpret_cast<const uint4 *>(sK + r * RB + ((c ^ (r & 7)) << 4));
                    }
                    typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
                    for (int d = 0; d < p.ndest; ++d) {
                        T *out = reinterpret_cast<T *>(p.dest[d]) + (int64_t)b * p.os_b + (int64_t)h * p.os_h;
#pragma unroll
                        for (int k = 0; k < NCH; ++k) {
                            const int idx = tid + k * 128, r = idx / CPR, c = idx % CPR;
                            const int g = tile_first + r;
                            if (g < p.row_limit)
                                *reinterpret_cast<uint4 *>(out + (int64_t)(g - p.out_row0) * p.os_s + c * 8) = v[k];
                        }
                    }
                }
            }
        }
        if (ok && direct) {
            tc_fence_after();
            typedef typename std::conditional<BF16, __nv_bfloat16, __half>::type T;
            T *out = reinterpret_cast<T *>(p.out) + (int64_t)b * p.os_b + (int64_t)h * p.os_h;
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc) {
                uint32_t o[16];
                if (nsteps > 0) {
                    tmem_ld16x256_x4(tO + lane_base + cc * 32, o);
                    tmem_wait_ld();
                    reg_fence(o);
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = 0u;
                }
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const int col = cc * 32 + q4 * 8 + cq;
                    const float a0 = __uint_as_float(o[4 * q4 + 0]) * inv0;
                    const float a1 = __uint_as_float(o[4 * q4 + 1]) * inv0;
                    const float b0 = __uint_as_float(o[4 * q4 + 2]) * inv1;
                    const float b1 = __uint_as_float(o[4 * q4 + 3]) * inv1;
                    const uint32_t wa = BF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
                    const uint32_t wb = BF16 ? pack_bf16x2(b0, b1) : pack_f16x2(b0, b1);
                    const int64_t o0 = (int64_t)(g0 - p.out_row0) * p.os_s + col;
                    const int64_t o1 = (int64_t)(g1 - p.out_row0) * p.os_s + col;
                    if (g0 < p.row_limit) *reinterpret_cast<uint32_t *>(out + o0) = wa;
                    if (g1 < p.row_limit) *reinterpret_cast<uint32_t *>(out + o1) = wb;
                    for (int d = 1; d < p.ndest; ++d) {   // peer copies (D = 256 only; D <= 128 stages)
                        T *po = reinterpret_cast<T *>(p.dest[d]) + (int64_t)b * p.os_b + (int64_t)h * p.os_h;
                        if (g0 < p.row_limit) *reinterpret_cast<uint32_t *>(po + o0) = wa;
                        if (g1 < p.row_limit) *reinterpret_cast<uint32_t *>(po + o1) = wb;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

static int make_map_4d(CUtensorMap *m, const void *ptr, bool bf16, int D, int S, int H, int B, ugbsa_strides st) {
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)st.s * 2, (cuuint64_t)st.h * 2, (cuuint64_t)st.b * 2};
    cuuint32_t box[4] = {64, 64, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return encode_tensor_map(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                             const_cast<void *>(ptr), dims, strides, box, es);
}

template <int D, bool BF16>
static int launch_attn_t(const void *Q, const void *K, const void *V, ugbsa_strides qs, ugbsa_strides ks,
                         ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk,
                         int t_base, int pair_stride, float scale, void *out, ugbsa_strides os, void *const *peers,
                         int npeers, cudaStream_t stream, int *err, const uint32_t *rowmask = nullptr) {
    using L = AttnSmem<D>;
    CUtensorMap mQ, mK, mV;
    int rc;
    if ((rc = make_map_4d(&mQ, Q, BF16, D, Sq, Hq, B, qs)) != UGBSA_OK) return rc;
    if ((rc = make_map_4d(&mK, K, BF16, D, Sk, Hkv, B, ks)) != UGBSA_OK) return rc;
    if ((rc = make_map_4d(&mV, V, BF16, D, Sk, Hkv, B, vs)) != UGBSA_OK) return rc;
    AttnParams p;
    p.kv_idx = kv_idx;
    p.kmax = kmax;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Sq = Sq; p.Sk = Sk;
    p.Qt = (Sq + 63) / 64;
    p.t_base = t_base;
    p.pair_stride = pair_stride;
    if (pair_stride == 1) {   // out holds the call's rows
        p.out_row0 = 64 * t_base;
        p.row_limit = 64 * t_base + Sq;
    } else {                  // out holds every row of the sequence
        p.out_row0 = 0;
        p.row_limit = Sk;
    }
    p.NB = (Sk + 63) / 64;
    p.rowmask = rowmask;
    p.nbw = (p.NB + 31) / 32;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.os_b = os.b; p.os_h = os.h; p.os_s = os.s;
    p.err = err;
    if (npeers < 0 || npeers >= kMaxDest) return UGBSA_ERR_ARG;
    p.ndest = 1 + npeers;
    p.dest[0] = out;
    for (int i = 0; i < kMaxDest - 1; ++i) p.dest[i + 1] = (i < npeers) ? peers[i] : nullptr;
    // head dim 256 (one CTA per SM): a second V stage when it fits, so that the next
    // step's V blocks land while P.V runs
    const size_t smem2 = (size_t)AttnSmem<D, 2>::OFF_LIST + (size_t)kmax * 4 + 1024;
    const bool two_v = D > 128 && smem2 <= 227 * 1024 - 512;
    const size_t smem = two_v ? smem2 : (size_t)L::OFF_LIST + (size_t)kmax * 4 + 1024;
    if (smem > 227 * 1024) return UGBSA_ERR_SHAPE;
    auto kern = two_v ? attn_fwd_kernel<D, BF16, 2> : attn_fwd_kernel<D, BF16, 1>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return UGBSA_ERR_LAUNCH;
    const int64_t grid = (int64_t)B * Hq * p.Qt;
    if (grid <= 0) return UGBSA_OK;
    if (grid > 0x7fffffff) return UGBSA_ERR_SHAPE;
    kern<<<(unsigned)grid, kAttnThreads, smem, stream>>>(mQ, mK, mV, p);
    return cudaGetLastError() == cudaSuccess ? UGBSA_OK : UGBSA_ERR_LAUNCH;
}

int launch_attn(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                ugbsa_strides vs, const int32_t *kv_idx, int kmax, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                int t_base, int pair_stride, float scale, void *out, ugbsa_strides os, void *const *peers,
                int npeers, cudaStream_t stream, int *err) {
    const bool bf = (dtype == UGBSA_BF16);
    if (t_base < 0 || pair_stride < 1 || (pair_stride > 1 && (t_base & 1))) return UGBSA_ERR_SHAPE;
    // D = 64 / 128 with UGBSA_ATTN_PAIR=1: the two-tile M=128 variant (attn_pair.cu),
    // when its shared memory fits.  Its tensor-core rate is twice this kernel's but
    // its exp2 and K-stage budget are not yet balanced, so it is opt-in; the parity
    // tests cover both.
    const char *pair = getenv("UGBSA_ATTN_PAIR");
    if ((D == 64 || D == 128) && t_base == 0 && pair_stride == 1 && npeers == 0 && pair && pair[0] == '1') {
        const int rc = launch_attn_pair(Q, K, V, dtype, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, D, scale, out,
                                        os, stream, err);
        if (rc != UGBSA_ERR_UNSUPPORTED) return rc;
    }
#define UGBSA_ATTN_CASE(DD)                                                                                        \
    if (D == DD)                                                                                                   \
        return bf ? launch_attn_t<DD, true>(Q, K, V, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, t_base,        \
                                            pair_stride, scale, out, os, peers, npeers, stream, err)               \
                  : launch_attn_t<DD, false>(Q, K, V, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, t_base,       \
                                             pair_stride, scale, out, os, peers, npeers, stream, err);
    UGBSA_ATTN_CASE(64)
    UGBSA_ATTN_CASE(128)
    UGBSA_ATTN_CASE(256)
#undef UGBSA_ATTN_CASE
    return UGBSA_ERR_UNSUPPORTED;
}

int launch_attn_rowmask(const void *Q, const void *K, const void *V, int dtype, ugbsa_strides qs, ugbsa_strides ks,
                        ugbsa_strides vs, const int32_t *kv_idx, int kmax, const uint32_t *rowmask, int B, int Hq,
                        int Hkv, int Sq, int Sk, int D, float scale, void *out, ugbsa_strides os, cudaStream_t stream,
                        int *err) {
    const bool bf = (dtype == UGBSA_BF16);
#define UGBSA_ATTN_CASE(DD)                                                                                        \
    if (D == DD)                                                                                                   \
        return bf ? launch_attn_t<DD, true>(Q, K, V, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, 0, 1, scale,   \
                                            out, os, nullptr, 0, stream, err, rowmask)                            \
                  : launch_attn_t<DD, false>(Q, K, V, qs, ks, vs, kv_idx, kmax, B, Hq, Hkv, Sq, Sk, 0, 1, scale,  \
                                             out, os, nullptr, 0, stream, err, rowmask);
    UGBSA_ATTN_CASE(64)
    UGBSA_ATTN_CASE(128)
    UGBSA_ATTN_CASE(256)
#undef UGBSA_ATTN_CASE
    return UGBSA_ERR_UNSUPPORTED;
}

}  // namespace ugbsa
