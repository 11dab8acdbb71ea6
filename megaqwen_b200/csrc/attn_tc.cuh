// Causal GQA flash attention for prefill on the 5th-generation tensor cores
// (tcgen05, accumulators in TMEM).
//
// One CTA = (block of 128 query rows, q head, sequence); 320 threads:
//   warp 0      TMA producers: lane 0 loads Q once, then K tiles of 128 keys
//               into a 3-stage ring (a stage is freed as soon as S_j is
//               done); lane 1 loads the V^T tiles into a 2-stage ring;
//   warp 1      TMEM owner; one thread issues the MMAs:
//                 S_j = Q K_j^T  (M=128 queries, N=128 keys, K=128 dims) into
//                                 one of two S buffers,
//                 O += P_j V_j   (M=128 queries, N=128 dims, K=128 keys),
//                                 accumulated in TMEM across the key tiles;
//               S_{j+1} is issued before O_j so the tensor core works while
//               the softmax warps are busy;
//   warps 2-9   softmax and output: warp w owns query rows 32 (w % 4) ..
//               (its TMEM lane quadrant) and column half (w - 2) / 4 of S
//               and O; row maxima are exchanged with the partner warp through
//               shared memory.  exp2 of S_j in registers, P_j stored as bf16
//               into one of two TMEM buffers, from which the P V MMA reads
//               its A operand.  P is taken relative to the row maximum in use; O
//               in TMEM is rescaled (tcgen05.ld / st) only when a row maximum
//               grows by more than 2^8, so P stays below 256 and most tiles
//               touch O not at all.  Each half keeps its own row sum, added at
//               the end.
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
constexpr int SM_Q = 0;
constexpr int KST = 3, VST = 2;             // K and V^T ring depths (separate rings: K is freed after S_j)
constexpr int SM_K = SM_Q + TILE;           // [KST] stages
constexpr int SM_V = SM_K + KST * TILE;     // [VST] stages (V^T)
constexpr int SM_BAR = SM_V + VST * TILE;
constexpr int SM_RED = SM_BAR + 256;        // fp32 [2 tiles][2 halves][128 rows] row maxima
constexpr int SMEM = SM_RED + 2 * 2 * 128 * 4 + 1024;   // + barriers, row-max exchange, alignment slack
constexpr int SOFT_WARPS = 8;               // two warps per TMEM lane quadrant, one per column half
constexpr int THREADS = 64 + 32 * SOFT_WARPS;
// TMEM columns: S_j buffers at 0 / 128 (fp32), O at 256 (fp32), P_j buffers at
// 384 / 448 (bf16 packed two per column: 128 keys = 64 columns)
constexpr uint32_t TM_O = 256, TM_P = 384;

struct Args {
    __nv_bfloat16* O;       // [M, 2048] bf16, row m = b * S + s
    int S;                  // sequence length
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

// tmQ: Qb [M, 2048]; tmK: the K cache as rows of 128 (see Args); tmV: V^T [B * 8 * 128, ldv]
// (rows = (b * 8 + kvh) * 128 + d).  Key rows past S (the last tile) hold other
// cache rows or TMA zero fill; the softmax masks them.
__global__ void __launch_bounds__(THREADS, 1)
fa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
             const __grid_constant__ CUtensorMap tmV, const Args args) {
    extern __shared__ uint8_t fa_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;      // [KST]
    uint64_t* k_empty = bars + 4;     // [KST]
    uint64_t* v_full = bars + 7;      // [VST]
    uint64_t* v_empty = bars + 9;     // [VST]
    uint64_t* s_full = bars + 11;     // [2]
    uint64_t* s_free = bars + 13;     // [2]
    uint64_t* p_full = bars + 15;     // [2] P_j stored on p_full[j & 1] (one barrier per P buffer)
    uint64_t* o_full = bars + 17;     // [2] PV_j completion on o_full[j & 1]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 19);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int S = args.S;
    const int nqb = (S + BQ - 1) / BQ;
    // grid (heads, batch, query blocks): CTAs are dispatched in linear block
    // order, so every (head, sequence) pair's heaviest (latest) query block
    // starts before any lighter one (longest-processing-time-first).
    const int qb = nqb - 1 - (int)blockIdx.z;
    const int h = blockIdx.x, b = blockIdx.y, kvh = h >> 1;
    const int q0 = qb * BQ;
    const int nt = qb + 1;                      // key tiles 0..qb (causal)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long lim = args.timeout_cycles;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
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

    if (warp == 0) {
        const int row0 = b * S;
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, TILE);
            tma_load_2d(smem + SM_Q, &tmQ, h * HD, row0 + q0, q_full);
            tma_load_2d(smem + SM_Q + ATOM, &tmQ, h * HD + 64, row0 + q0, q_full);
            for (int j = 0; j < nt; ++j) {
                const int st = j % KST, u = j / KST;
                if (u >= 1 && !fa_wait(&k_empty[st], (u - 1) & 1, lim)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 41);
                    break;
                }
                if (*abort_flag) break;
                uint8_t* kd = smem + SM_K + st * TILE;
                mbar_arrive_expect_tx(&k_full[st], TILE);
                const int krow = (int)(args.k_row0 + b * args.k_seq_rows + kvh * args.k_head_rows) + j * BK;
                tma_load_2d(kd, &tmK, 0, krow, &k_full[st]);
                tma_load_2d(kd + ATOM, &tmK, 64, krow, &k_full[st]);
            }
        } else if (lane == 1) {
            const int vrow = (b * 8 + kvh) * HD;
            for (int j = 0; j < nt; ++j) {
                const int st = j & 1, u = j >> 1;
                if (u >= 1 && !fa_wait(&v_empty[st], (u - 1) & 1, lim)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 44);
                    break;
                }
                if (*abort_flag) break;
                uint8_t* vd = smem + SM_V + st * TILE;
                mbar_arrive_expect_tx(&v_full[st], TILE);
                tma_load_2d(vd, &tmV, j * BK, vrow, &v_full[st]);
                tma_load_2d(vd + ATOM, &tmV, j * BK + 64, vrow, &v_full[st]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(BQ, BK);
            const uint32_t sq = smem_u32(smem + SM_Q);
            bool ok = fa_wait(q_full, 0, lim);
            // O_j = P_j V_j into the O buffer
            auto pv = [&](int j) -> bool {
                // P_j stored in TMEM and O rescaled (if the row maxima moved) by the softmax warps
                if (!fa_wait(&p_full[j & 1], (j >> 1) & 1, lim)) return false;
                if (!fa_wait(&v_full[j & 1], (j >> 1) & 1, lim)) return false;
                tc_fence_after();
                const uint32_t sv = smem_u32(smem + SM_V + (j & 1) * TILE);
                const uint32_t pa = tmem + TM_P + (j & 1) * 64;
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
                    tc_mma_f16_ts(tmem + TM_O, pa + k * 8, sw128_kmajor_desc(sv + off), idesc, (j | k) != 0);
                }
                tc_commit(&o_full[j & 1]);
                tc_commit(&v_empty[j & 1]);
                return true;
            };
            for (int j = 0; ok && j < nt; ++j) {
                const int st = j & 1, u = j >> 1, kst = j % KST;
                if (!fa_wait(&k_full[kst], (j / KST) & 1, lim) ||
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
                tc_commit(&k_empty[kst]);   // K_j read: its stage can take K_{j+KST}
                if (j >= 1 && !pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && !pv(nt - 1)) ok = false;
            if (!ok) {
                *abort_flag = 1;
                atomicExch(args.err, 42);
            }
        }
    } else {
        // softmax / output: thread = (query row r, column half hh)
        const int quad = warp & 3, hh = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int qrow = q0 + r;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t oa = tmem + lane_off + TM_O + hh * 64;   // this thread's half of its O row
        float* red = reinterpret_cast<float*>(smem + SM_RED);     // [2][2][128]
        constexpr float RESCALE_LOG2 = 8.f;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int st = j & 1, u = j >> 1;
            // after a failed wait the loop still runs to the end (without waiting) so that the
            // partner warp's named barriers are always matched
            fa_stamp(args, j, 0);
            if (ok && (!fa_wait(&s_full[st], u & 1, lim) || *abort_flag)) ok = false;
            fa_stamp(args, j, 1);
            tc_fence_after();
            const int k0 = j * BK + hh * 64;
            float sv[64];
            tmem_ld32(tmem + lane_off + st * BK + hh * 64, sv);
            tmem_ld32(tmem + lane_off + st * BK + hh * 64 + 32, sv + 32);
            // S buffer consumed: the MMA may compute S_{j+2} into it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[st]);
            fa_stamp(args, j, 2);
            // scores are already in the log2 domain (q is stored pre-scaled); only the diagonal
            // tile and a tile past the sequence end need the causal / length mask
            float tmax = -INFINITY;
            if (j == qb || (j + 1) * BK > S) {
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const int key = k0 + i;
                    sv[i] = (key > qrow || key >= S) ? -INFINITY : sv[i];
                    tmax = fmaxf(tmax, sv[i]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i) tmax = fmaxf(tmax, sv[i]);
            }
            // row maximum over both halves (partner warp w +- 4 shares the lane quadrant)
            red[(st * 2 + hh) * 128 + r] = tmax;
            fa_stamp(args, j, 3);
            named_bar_sync(1 + quad, 64);
            tmax = fmaxf(tmax, red[(st * 2 + (hh ^ 1)) * 128 + r]);
            fa_stamp(args, j, 4);
            // move the row to a new maximum only when it grew by more than 2^8
            float corr = 1.f;
            if (tmax > m + RESCALE_LOG2) {
                corr = ex2_approx(m - tmax);   // 0 on the first tile (m = -inf)
                m = tmax;
            }
            l *= corr;
            if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
                // O rescale: PV_{j-1} must have completed
                if (ok && !fa_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, lim)) ok = false;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 64; c += 32) {
                    float v[32];
                    tmem_ld32(oa + c, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] *= corr;
                    tmem_st32(oa + c, v);
                }
            }
            // P_j goes to TMEM buffer j & 1, last read by PV_{j-2}
            if (j >= 2 && ok && !fa_wait(&o_full[st], (u - 1) & 1, lim)) ok = false;
            // P = exp2(s - m) (at most 2^8), bf16 packed in pairs: keys 64 hh .. + 63 = columns 32 hh .. + 31
            float psum = 0.f;
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float p0 = ex2_approx(sv[2 * i] - m), p1 = ex2_approx(sv[2 * i + 1] - m);
                psum += p0 + p1;
                __nv_bfloat162 t = __floats2bfloat162_rn(p0, p1);
                pk[i] = *reinterpret_cast<uint32_t*>(&t);
            }
            fa_stamp(args, j, 5);
            tmem_st32_u(tmem + lane_off + TM_P + st * 64 + hh * 32, pk);
            fa_stamp(args, j, 6);
            l += psum;
            // P stored and O rescale done: PV_j may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[st]);
        }
        // both halves' row sums (same row maximum)
        named_bar_sync(1 + quad, 64);
        red[hh * 128 + r] = l;
        named_bar_sync(1 + quad, 64);
        const float ltot = l + red[(hh ^ 1) * 128 + r];
        if (ok && fa_wait(&o_full[(nt - 1) & 1], ((nt - 1) >> 1) & 1, lim)) {
            tc_fence_after();
            const float inv = 1.f / ltot;
            __nv_bfloat16* out = args.O + ((size_t)b * S + qrow) * 2048 + h * HD + hh * 64;
#pragma unroll
            for (int c = 0; c < 64; c += 32) {
                float v[32];
                tmem_ld32(oa + c, v);
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
                        *reinterpret_cast<uint4*>(out + c + i) = pk;
                    }
                }
            }
        } else {
            if (lane == 0) atomicExch(args.err, 43);
            *abort_flag = 1;
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
