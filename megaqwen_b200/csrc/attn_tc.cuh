// Causal GQA flash attention for prefill on the 5th-generation tensor cores
// (tcgen05, accumulators in TMEM).
//
// Persistent: one CTA per SM walks a list of work items, an item being (block
// of 128 query rows, q head, sequence).  Items are ordered heaviest (latest
// query block) first and dealt to the CTAs in a snake order (round r gives
// item r * G + c to CTA c, or r * G + G - 1 - c on odd rounds), so the loads
// balance like longest-processing-time-first.  TMEM, barriers and tensor maps
// are set up once per CTA; the rings, S/P buffers and barrier phases run on
// per-CTA tile counters g across items.  (One CTA per item cost 3.4 us of
// set-up, Q load and pipeline fill per item plus a 1.4 us gap before the next
// CTA started on the SM, against 1.23 us per 128-key tile.)
// 448 threads:
//   warp 0      TMA producers: lane 0 loads each item's Q into buffer it & 1
//               (once item it - 2 has no S MMA left to run; the next item's
//               Q and first K tile are prefetched into L2 when an item
//               starts), then K tiles of 128 keys into a 2-stage ring (a
//               stage is freed as soon as S_g is done); lane 1 loads the V^T
//               tiles into a 2-stage ring;
//   warp 1      TMEM owner; one thread issues the MMAs:
//                 S_g = Q K_g^T  (M=128 queries, N=128 keys, K=128 dims) into
//                                 one of two S buffers,
//                 O += P_g V_g   (M=128 queries, N=128 dims, K=128 keys),
//                                 accumulated in TMEM across the item's tiles;
//               S_{g+1} is issued before PV_g, across items too, so the
//               tensor core works while the softmax warps are busy; an item's first PV waits until
//               the output warps have read the previous item's O;
//   warps 2-9   softmax: warp w owns query rows 32 (w % 4) .. (its TMEM lane
//               quadrant) and column half (w - 2) / 4 of S; row maxima are
//               exchanged with the partner warp through shared memory.  exp2
//               of S_g in registers, P_g stored as bf16 into one of two TMEM
//               buffers, from which the P V MMA reads its A operand.  P is
//               taken relative to the row maximum in use; O in TMEM is
//               rescaled (tcgen05.ld / st) only when a row maximum grows by
//               more than 2^8, so P stays below 256 and most tiles touch O not
//               at all.  Each half keeps its own row sum, handed to the output
//               warps through shared memory at the end of the item;
//   warps 10-13 output: one per TMEM lane quadrant, a thread per query row;
//               after the item's last PV they read O, scale by 1 / row sum
//               and store bf16, while the softmax warps are already on the
//               next item's first tile.
// All operands are K-major: Q [q][d], K [key][d], P [q][key] (TMEM) and V^T [d][key]
// (the QKV GEMM epilogue writes V transposed per sequence and kv head).
// Scores are in the log2 domain: the QKV epilogue stores q pre-multiplied by
// the attention scale x log2 e.  Every wait is bounded and sets an error code.
#pragma once

#include <cuda_bf16.h>

#include "mq_tc.cuh"

namespace mq {
namespace fa {

constexpr int BQ = 128;                     // query rows per CTA
constexpr int BK = 128;                     // keys per tile
constexpr int HD = 128;                     // head dim
constexpr int ATOM = 128 * 128;             // bytes of a 128-row x 64-element swizzled atom (16 KB)
constexpr int TILE = 2 * ATOM;              // a 128 x 128 bf16 operand (32 KB)
constexpr int SM_Q = 0;                     // [2] Q buffers (item it uses it & 1)
constexpr int KST = 2, VST = 2;             // K and V^T ring depths (separate rings: K is freed after S_g)
constexpr int SM_K = SM_Q + 2 * TILE;       // [KST] stages
constexpr int SM_V = SM_K + KST * TILE;     // [VST] stages (V^T)
constexpr int SM_BAR = SM_V + VST * TILE;
constexpr int SM_RED = SM_BAR + 256;        // fp32 [2 tiles][2 halves][128 rows] row maxima
constexpr int SM_SUM = SM_RED + 2 * 2 * 128 * 4;   // fp32 [2 items][2 halves][128 rows] row sums
constexpr int SMEM = SM_SUM + 2 * 2 * 128 * 4 + 1024;   // + alignment slack
constexpr int SOFT_WARPS = 8;               // two warps per TMEM lane quadrant, one per column half
constexpr int EPI_WARP0 = 2 + SOFT_WARPS;   // four output warps, one per TMEM lane quadrant
constexpr int THREADS = 64 + 32 * SOFT_WARPS + 128;
// TMEM columns: S_j buffers at 0 / 128 (fp32), O at 256 (fp32), P_j buffers at
// 384 / 448 (bf16 packed two per column: 128 keys = 64 columns)
constexpr uint32_t TM_O = 256, TM_P = 384;

struct Args {
    __nv_bfloat16* O;       // [M, 2048] bf16, row m = b * S + s
    int S;                  // sequence length
    int B;                  // sequences
    // K is read straight from the layer's K cache (rows of 128): key s of kv head
    // h of sequence b is row k_row0 + b * k_seq_rows + h * k_head_rows + s
    long long k_row0, k_seq_rows, k_head_rows;
    int* err;
    long long timeout_cycles;
    unsigned long long* trace;   // optional: %globaltimer stamps of block (0,0,0), softmax warp 2, tiles < 32
};

__device__ __forceinline__ void fa_stamp(const Args& a, int j, int k) {
    if (a.trace && j < 32 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 64) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[j * 8 + k] = t;
    }
}

// 2^x on the special-function unit (ex2.approx.ftz: 2^-inf = 0)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ bool fa_wait(uint64_t* bar, uint32_t parity, long long limit) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

// Work item `it` of CTA c among G: (q head, sequence, query block), or false
// past the end.  Linear item k: heads fastest, then sequences, then query
// blocks from the last (heaviest) to the first.
struct Item {
    int h, b, qb;
};
__device__ __forceinline__ bool item_of(int it, int c, int G, int B, int nqb, Item& I) {
    const int k = it * G + ((it & 1) ? (G - 1 - c) : c);
    if (k >= 16 * B * nqb) return false;
    I.h = k & 15;
    I.b = (k >> 4) % B;
    I.qb = nqb - 1 - (k >> 4) / B;
    return true;
}

// tmQ: Qb [M, 2048]; tmK: the K cache as rows of 128 (see Args); tmV: V^T [B * 8 * 128, ldv]
// (rows = (b * 8 + kvh) * 128 + d).  Key rows past S (the last tile) hold other
// cache rows or TMA zero fill; the softmax masks them.
__global__ void __launch_bounds__(THREADS, 1)
fa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
             const __grid_constant__ CUtensorMap tmV, const Args args) {
    extern __shared__ uint8_t fa_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
    uint64_t* q_full = bars + 0;      // [2]
    uint64_t* k_full = bars + 2;      // [KST]
    uint64_t* k_empty = bars + 4;     // [KST]
    uint64_t* v_full = bars + 7;      // [VST]
    uint64_t* v_empty = bars + 9;     // [VST]
    uint64_t* s_full = bars + 11;     // [2]
    uint64_t* s_free = bars + 13;     // [2]
    uint64_t* p_full = bars + 15;     // [2] P_g stored on p_full[g & 1] (one barrier per P buffer)
    uint64_t* o_full = bars + 17;     // [2] PV_g completion on o_full[g & 1]
    uint64_t* q_empty = bars + 19;    // [2] every S MMA of the item using that Q buffer has completed
    uint64_t* l_full = bars + 21;     // the item's row sums are in SM_SUM[it & 1]
    uint64_t* o_empty = bars + 22;    // the output warps have read the item's O
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 23);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int S = args.S, B = args.B;
    const int nqb = (S + BQ - 1) / BQ;
    const int c = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long lim = args.timeout_cycles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        mbar_init(l_full, SOFT_WARPS);
        mbar_init(o_empty, 4);
        for (int i = 0; i < KST; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], SOFT_WARPS);
        }
        mbar_init(&p_full[0], SOFT_WARPS);
        mbar_init(&p_full[1], SOFT_WARPS);
        mbar_init(&o_full[0], 1);
        mbar_init(&o_full[1], 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // Programmatic dependent launch: the set-up above overlapped the previous
    // kernel's tail; nothing it wrote is read before pdl_wait.
    pdl_trigger();
    pdl_wait();

    // Tile counters run across the CTA's items: tile g of the CTA uses K stage
    // g % KST, V stage / S buffer / P buffer g & 1, with phases from g.
    if (warp == 0) {
        if (lane == 0) {
            int g = 0;
            Item I;
            for (int it = 0; item_of(it, c, G, B, nqb, I); ++it) {
                // Q buffer it & 1 is the A operand of every S MMA of item it - 2
                const int qs = it & 1;
                if (it >= 2 && !fa_wait(&q_empty[qs], ((it >> 1) - 1) & 1, lim)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 45);
                    break;
                }
                if (*abort_flag) break;
                const int kvh = I.h >> 1, nt = I.qb + 1;
                uint8_t* qd = smem + SM_Q + qs * TILE;
                mbar_arrive_expect_tx(&q_full[qs], TILE);
                tma_load_2d(qd, &tmQ, I.h * HD, I.b * S + I.qb * BQ, &q_full[qs]);
                tma_load_2d(qd + ATOM, &tmQ, I.h * HD + 64, I.b * S + I.qb * BQ, &q_full[qs]);
                // the next item's Q and first K tile into L2 (loaded a few tiles before this
                // item ends)
                Item N;
                if (item_of(it + 1, c, G, B, nqb, N)) {
                    tma_prefetch_2d(&tmQ, N.h * HD, N.b * S + N.qb * BQ);
                    tma_prefetch_2d(&tmQ, N.h * HD + 64, N.b * S + N.qb * BQ);
                    const int nrow = (int)(args.k_row0 + N.b * args.k_seq_rows + (N.h >> 1) * args.k_head_rows);
                    tma_prefetch_2d(&tmK, 0, nrow);
                    tma_prefetch_2d(&tmK, 64, nrow);
                }
                bool ok = true;
                for (int j = 0; j < nt; ++j, ++g) {
                    const int st = g % KST, u = g / KST;
                    if (u >= 1 && !fa_wait(&k_empty[st], (u - 1) & 1, lim)) {
                        *abort_flag = 1;
                        atomicExch(args.err, 41);
                        ok = false;
                        break;
                    }
                    if (*abort_flag) {
                        ok = false;
                        break;
                    }
                    uint8_t* kd = smem + SM_K + st * TILE;
                    mbar_arrive_expect_tx(&k_full[st], TILE);
                    const int krow =
                        (int)(args.k_row0 + I.b * args.k_seq_rows + kvh * args.k_head_rows) + j * BK;
                    tma_load_2d(kd, &tmK, 0, krow, &k_full[st]);
                    tma_load_2d(kd + ATOM, &tmK, 64, krow, &k_full[st]);
                }
                if (!ok) break;
            }
        } else if (lane == 1) {
            int g = 0;
            Item I;
            bool ok = true;
            for (int it = 0; ok && item_of(it, c, G, B, nqb, I); ++it) {
                const int vrow = (I.b * 8 + (I.h >> 1)) * HD, nt = I.qb + 1;
                for (int j = 0; j < nt; ++j, ++g) {
                    const int st = g & 1, u = g >> 1;
                    if (u >= 1 && !fa_wait(&v_empty[st], (u - 1) & 1, lim)) {
                        *abort_flag = 1;
                        atomicExch(args.err, 44);
                        ok = false;
                        break;
                    }
                    if (*abort_flag) {
                        ok = false;
                        break;
                    }
                    uint8_t* vd = smem + SM_V + st * TILE;
                    mbar_arrive_expect_tx(&v_full[st], TILE);
                    tma_load_2d(vd, &tmV, j * BK, vrow, &v_full[st]);
                    tma_load_2d(vd + ATOM, &tmV, j * BK + 64, vrow, &v_full[st]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(BQ, BK);
            // O (+)= P_g V_g; `first` starts item it's accumulator, once the output
            // warps have read the O of item it - 1
            auto pv = [&](int g, bool first, int it) -> bool {
                if (first && it >= 1 && !fa_wait(o_empty, (it - 1) & 1, lim)) return false;
                // P_g stored in TMEM and O rescaled (if the row maxima moved) by the softmax warps
                if (!fa_wait(&p_full[g & 1], (g >> 1) & 1, lim)) return false;
                if (!fa_wait(&v_full[g & 1], (g >> 1) & 1, lim)) return false;
                tc_fence_after();
                const uint32_t sv = smem_u32(smem + SM_V + (g & 1) * TILE);
                const uint32_t pa = tmem + TM_P + (g & 1) * 64;
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
                    tc_mma_f16_ts(tmem + TM_O, pa + k * 8, sw128_kmajor_desc(sv + off), idesc, !first || k != 0);
                }
                tc_commit(&o_full[g & 1]);
                tc_commit(&v_empty[g & 1]);
                return true;
            };
            // PV_{g-1} is issued after S_g, across item boundaries too: the next item's first
            // S MMAs (its Q is double-buffered) run while the softmax finishes the last tile.
            bool ok = true;
            int g = 0;
            int pg = -1, pit = 0;   // the tile whose PV is pending, its item
            bool pfirst = false;
            Item I;
            for (int it = 0; ok && item_of(it, c, G, B, nqb, I); ++it) {
                const int nt = I.qb + 1, qs = it & 1;
                if (!fa_wait(&q_full[qs], (it >> 1) & 1, lim)) {
                    ok = false;
                    break;
                }
                const uint32_t sq = smem_u32(smem + SM_Q + qs * TILE);
                for (int j = 0; j < nt; ++j, ++g) {
                    const int st = g & 1, u = g >> 1, kst = g % KST;
                    if (!fa_wait(&k_full[kst], (g / KST) & 1, lim) ||
                        (u >= 1 && !fa_wait(&s_free[st], (u - 1) & 1, lim)) || *abort_flag) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sk = smem_u32(smem + SM_K + kst * TILE);
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k) {
                        const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
                        tc_mma_f16(tmem + st * BK, sw128_kmajor_desc(sq + off), sw128_kmajor_desc(sk + off), idesc,
                                   k != 0);
                    }
                    tc_commit(&s_full[st]);
                    tc_commit(&k_empty[kst]);   // K_g read: its stage can take K_{g+KST}
                    if (j == nt - 1) tc_commit(&q_empty[qs]);   // the item's last S: its Q buffer is free
                    // S_g is issued before PV_{g-1} so the tensor core works while the softmax runs
                    if (pg >= 0 && !pv(pg, pfirst, pit)) {
                        ok = false;
                        break;
                    }
                    pg = g;
                    pfirst = j == 0;
                    pit = it;
                }
            }
            if (ok && pg >= 0 && !pv(pg, pfirst, pit)) ok = false;
            if (!ok) {
                *abort_flag = 1;
                atomicExch(args.err, 42);
            }
        }
    } else if (warp < EPI_WARP0) {
        // softmax: thread = (query row r, column half hh)
        const int quad = warp & 3, hh = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t oa = tmem + lane_off + TM_O + hh * 64;   // this thread's half of its O row
        float* red = reinterpret_cast<float*>(smem + SM_RED);     // [2][2][128]
        float* rsum = reinterpret_cast<float*>(smem + SM_SUM);    // [2 items][2][128]
        constexpr float RESCALE_LOG2 = 8.f;
        // after a failed wait the loops still run to the end (without waiting) so that the
        // partner warp's named barriers are always matched
        bool ok = true;
        int g = 0;
        Item I;
        for (int it = 0; item_of(it, c, G, B, nqb, I); ++it) {
            const int qb = I.qb, nt = qb + 1;
            const int qrow = qb * BQ + r;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < nt; ++j, ++g) {
                const int st = g & 1, u = g >> 1;
                fa_stamp(args, g, 0);
                if (ok && (!fa_wait(&s_full[st], u & 1, lim) || *abort_flag)) ok = false;
                fa_stamp(args, g, 1);
                tc_fence_after();
                const int k0 = j * BK + hh * 64;
                float sv[64];
                tmem_ld32(tmem + lane_off + st * BK + hh * 64, sv);
                tmem_ld32(tmem + lane_off + st * BK + hh * 64 + 32, sv + 32);
                // S buffer consumed: the MMA may compute S_{g+2} into it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[st]);
                fa_stamp(args, g, 2);
                // scores are already in the log2 domain (q is stored pre-scaled); only the diagonal
                // tile and a tile past the sequence end need the causal / length mask
                float tmax = -INFINITY;
                if (j == qb || (j + 1) * BK > S) {
                    // keys k0 + i are visible for i <= last (causal and length limits in one compare)
                    const int last = min(qrow, S - 1) - k0;
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        sv[i] = i > last ? -INFINITY : sv[i];
                        tmax = fmaxf(tmax, sv[i]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i) tmax = fmaxf(tmax, sv[i]);
                }
                // row maximum over both halves (partner warp w +- 4 shares the lane quadrant)
                red[(st * 2 + hh) * 128 + r] = tmax;
                fa_stamp(args, g, 3);
                named_bar_sync(1 + quad, 64);
                tmax = fmaxf(tmax, red[(st * 2 + (hh ^ 1)) * 128 + r]);
                fa_stamp(args, g, 4);
                // move the row to a new maximum only when it grew by more than 2^8
                float corr = 1.f;
                if (tmax > m + RESCALE_LOG2) {
                    corr = ex2_approx(m - tmax);   // 0 on the first tile (m = -inf)
                    m = tmax;
                }
                l *= corr;
                if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
                    // O rescale: PV_{g-1} must have completed
                    if (ok && !fa_wait(&o_full[(g - 1) & 1], ((g - 1) >> 1) & 1, lim)) ok = false;
                    tc_fence_after();
#pragma unroll 1
                    for (int cc = 0; cc < 64; cc += 16) {
                        float v[16];
                        tmem_ld16(oa + cc, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] *= corr;
                        tmem_st16(oa + cc, v);
                    }
                }
                // P_g goes to TMEM buffer g & 1, last read by PV_{g-2}
                if (g >= 2 && ok && !fa_wait(&o_full[st], (u - 1) & 1, lim)) ok = false;
                // P = exp2(s - m) (at most 2^8), bf16 packed in pairs: keys 64 hh .. + 63 = columns 32 hh .. + 31
                // (two stores of 16 columns keep fewer packed words live)
                float psum = 0.f;
#pragma unroll
                for (int hq = 0; hq < 2; ++hq) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int e = 32 * hq + 2 * i;
                        const float p0 = ex2_approx(sv[e] - m), p1 = ex2_approx(sv[e + 1] - m);
                        psum += p0 + p1;
                        __nv_bfloat162 t = __floats2bfloat162_rn(p0, p1);
                        pk[i] = *reinterpret_cast<uint32_t*>(&t);
                    }
                    tmem_st16_nowait(tmem + lane_off + TM_P + st * 64 + hh * 32 + 16 * hq, pk);
                }
                fa_stamp(args, g, 5);
                tmem_st_wait();
                fa_stamp(args, g, 6);
                l += psum;
                // P stored and O rescale done: PV_g may start
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[st]);
            }
            // this half's row sum for the output warps (the row maximum is shared).  The
            // output warps must be past item it - 1 first: after a one-tile item nothing
            // else keeps l_full from completing two phases ahead of their wait.
            if (it >= 1 && ok && !fa_wait(o_empty, (it - 1) & 1, lim)) ok = false;
            rsum[((it & 1) * 2 + hh) * 128 + r] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(l_full);
        }
    } else {
        // output: thread = query row r of its TMEM lane quadrant, all 128 dims of O.
        // Item it's O is complete when its last PV (tile g - 1) has; read, scale
        // by 1 / row sum, store bf16, then release O to the next item's first PV.
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t oa = tmem + ((uint32_t)(quad * 32) << 16) + TM_O;
        const float* rsum = reinterpret_cast<const float*>(smem + SM_SUM);
        bool ok = true;
        int g = 0;
        Item I;
        for (int it = 0; item_of(it, c, G, B, nqb, I); ++it) {
            g += I.qb + 1;
            const int qrow = I.qb * BQ + r;
            if (ok && (!fa_wait(l_full, it & 1, lim) || !fa_wait(&o_full[(g - 1) & 1], ((g - 1) >> 1) & 1, lim) ||
                       *abort_flag))
                ok = false;
            if (!ok) {
                if (lane == 0) atomicExch(args.err, 43);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const float inv = 1.f / (rsum[((it & 1) * 2) * 128 + r] + rsum[((it & 1) * 2 + 1) * 128 + r]);
            __nv_bfloat16* out = args.O + ((size_t)I.b * S + qrow) * 2048 + I.h * HD;
#pragma unroll
            for (int cc = 0; cc < HD; cc += 32) {
                float v[32];
                tmem_ld32(oa + cc, v);
                if (cc == HD - 32) {
                    // every O column read: the next item's first PV may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(o_empty);
                }
                if (qrow < S) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 pk;
                        __nv_bfloat162 b0 = __floats2bfloat162_rn(v[i] * inv, v[i + 1] * inv);
                        __nv_bfloat162 b1 = __floats2bfloat162_rn(v[i + 2] * inv, v[i + 3] * inv);
                        __nv_bfloat162 b2 = __floats2bfloat162_rn(v[i + 4] * inv, v[i + 5] * inv);
                        __nv_bfloat162 b3 = __floats2bfloat162_rn(v[i + 6] * inv, v[i + 7] * inv);
                        pk.x = *reinterpret_cast<uint32_t*>(&b0);
                        pk.y = *reinterpret_cast<uint32_t*>(&b1);
                        pk.z = *reinterpret_cast<uint32_t*>(&b2);
                        pk.w = *reinterpret_cast<uint32_t*>(&b3);
                        *reinterpret_cast<uint4*>(out + cc + i) = pk;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace fa
}  // namespace mq
