// Persistent tcgen05 GEMM for prefill: C[M, N] = A[M, K] . B[N, K]^T, bf16
// operands (both K-major), fp32 accumulation in TMEM, fused epilogues.
//
// One CTA per SM walks the 128 x BN output tiles t = blockIdx.x, + gridDim.x ..
// (BN = 256 where every B map allows it: half the A re-reads per FLOP)
// Warp 0 (one thread) streams A/B K-slices of 64 through an mbarrier ring with
// TMA; warp 1 owns TMEM and one of its threads issues the MMAs; warps 2-9 run
// the epilogue (two per TMEM lane quadrant, one per column half).  The accumulator is double-buffered in TMEM, so the epilogue
// of tile i overlaps the MMAs of tile i + 1 and the loads run ahead across
// tile boundaries.  Every wait is bounded and sets an error code.
//
// B may be up to three matrices side by side (q | k | v): tile columns
// [0, nb0) read map 0, [nb0, nb0 + nb1) map 1, the rest map 2.  EPI_SILU_MUL
// reads gate (map 0) and up (map 1) for the same tile into two accumulators.
//
// EPI_QKV (prefill QKV projection): each 128 columns of a tile are one head.  q and k
// heads get RMSNorm over the head (x norm weight) and rotate-half RoPE at the
// row's position, in the thread that owns the row (no cross-thread traffic);
// q goes to Qb, k and v to the sequence's K/V cache (bf16), v also transposed.
#pragma once

#include <cuda_bf16.h>

#include "gemm_tc.cuh"

namespace mq {

constexpr int EPI_QKV = 4;

constexpr int P_EPI_WARPS = 8;                           // two per TMEM lane quadrant
constexpr int P_THREADS = 64 + 32 * P_EPI_WARPS;

template <int EPI, int BN>
struct PCfg {
    static constexpr int NB = (EPI == EPI_SILU_MUL) ? 2 : 1;          // B tiles per stage
    static constexpr int B_BYTES = BN * GEMM_BK * 2;                  // one B tile (BN rows x 64)
    static constexpr int STAGE = GEMM_TILE_BYTES + NB * B_BYTES;      // A tile (128 rows) + B tiles
    // EPI_QKV stages the cos / sin rows of a tile's 128 positions (64 KB) and
    // keeps one ring stage fewer for them
    static constexpr int ROPE_BYTES = EPI == 4 ? 2 * GEMM_BM * 128 * 2 : 0;
    static constexpr int NSTAGES = EPI == 4 ? 3 : ((6 * STAGE <= 200 * 1024) ? 6 : 4);
    static constexpr int ACC_COLS = BN * NB;                          // one accumulator buffer
    static constexpr int TMEM_COLS = 2 * ACC_COLS;                    // double-buffered
    static constexpr int SMEM = NSTAGES * STAGE + 1024 + 256 + ROPE_BYTES;
    static_assert(TMEM_COLS <= 512, "two accumulator buffers fit in TMEM");
    static_assert(BN * NB <= 256, "one MMA covers the stacked B tiles (N <= 256)");
};

struct QkvPrefillEpi {
    const __nv_bfloat16* q_norm;
    const __nv_bfloat16* k_norm;
    const __nv_bfloat16* cos_table;   // [max_seq, 128]
    const __nv_bfloat16* sin_table;
    __nv_bfloat16* Qb;                // [M, 2048]
    __nv_bfloat16* k_cache;           // layer base of sequence 0: [8, max_seq, 128]
    __nv_bfloat16* v_cache;
    long long cache_seq_stride;       // elements between sequences' caches
    int S, start_pos, max_seq;
    __nv_bfloat16* Vt;                // optional: V transposed per (sequence, kv head): [B * 8 * 128, ldvt]
    int ldvt;
    float q_scale;                    // q is stored pre-multiplied (attention scale x log2 e)
};

struct PArgs {
    void* C;             // output (fp32 or bf16, see epilogue)
    int ldc;             // elements
    int M, K;
    int tiles_m, tiles_n;
    int nb0, nb1;        // tile columns of B maps 0 and 1
    QkvPrefillEpi qkv;
    int* err;
    long long timeout_cycles;
};

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
    uint4 pk;
    __nv_bfloat162 b0 = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 b2 = __floats2bfloat162_rn(v[4], v[5]);
    __nv_bfloat162 b3 = __floats2bfloat162_rn(v[6], v[7]);
    pk.x = *reinterpret_cast<uint32_t*>(&b0);
    pk.y = *reinterpret_cast<uint32_t*>(&b1);
    pk.z = *reinterpret_cast<uint32_t*>(&b2);
    pk.w = *reinterpret_cast<uint32_t*>(&b3);
    return pk;
}

// QK-norm + RoPE (q, k heads) or plain rounding (v heads) of one row of one
// head from the accumulator, written as bf16 to the operand buffer and, for k
// and v, to the cache.  map: 0 q, 1 k, 2 v; head within the map.  Every lane
// of the warp calls it (the TMEM loads are warp-collective); lanes whose row
// is past M store nothing.
// cs / sn: this row's cos / sin table rows, staged in shared memory with the
// 16-byte chunk c of the row stored at chunk c ^ sw (sw = row & 15), so that
// the 8 lanes of a quarter warp (8 consecutive rows) read 8 different banks.
__device__ __forceinline__ void qkv_row_epilogue(const PArgs& a, uint32_t acc, int map, int head, int row_in,
                                                 const __nv_bfloat16* cs, const __nv_bfloat16* sn, int sw) {
    const QkvPrefillEpi& e = a.qkv;
    const bool valid = row_in < a.M;
    const int row = valid ? row_in : 0;
    const int b = row / e.S, p = e.start_pos + (row - b * e.S);
    // q goes to Qb; k and v only to the cache (the attention reads K from the
    // cache and V from V^T)
    __nv_bfloat16* dst = map == 0 ? e.Qb + (size_t)row * 2048 + head * 128 : nullptr;
    __nv_bfloat16* cache = map == 0 ? nullptr
                                    : (map == 1 ? e.k_cache : e.v_cache) + b * e.cache_seq_stride +
                                          ((size_t)head * e.max_seq + p) * 128;
    if (map == 2) {
        // V^T row d of (sequence b, kv head): lanes hold consecutive positions, so each
        // scalar store of the warp covers 64 contiguous bytes
        __nv_bfloat16* vt = e.Vt ? e.Vt + ((size_t)(b * 8 + head) * 128) * e.ldvt + (row - b * e.S) : nullptr;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
            float v[32];
            tmem_ld32(acc + c, v);
            if (valid) {
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    const uint4 pk = pack8_bf16(v + i);
                    *reinterpret_cast<uint4*>(cache + c + i) = pk;
                }
                if (vt) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) vt[(size_t)(c + i) * e.ldvt] = __float2bfloat16(v[i]);
                }
            }
        }
        return;
    }
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
        float v[32];
        tmem_ld32(acc + c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
    }
    const float r = rsqrtf(ss / 128.f + 1e-6f);
    const __nv_bfloat16* nw = map == 0 ? e.q_norm : e.k_norm;
    const float osc = map == 0 ? e.q_scale : 1.f;
    // rotate-half pairs (d, d + 64): chunk c with chunk c + 64; weights, cos and
    // sin rows are read 8 bf16 at a time
#pragma unroll
    for (int c = 0; c < 64; c += 32) {
        float x1[32], x2[32];
        tmem_ld32(acc + c, x1);
        tmem_ld32(acc + c + 64, x2);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
            const int d = c + i;
            const uint4 w1 = *reinterpret_cast<const uint4*>(nw + d), w2 = *reinterpret_cast<const uint4*>(nw + d + 64);
            const int k1 = ((d >> 3) ^ sw) << 3, k2 = (((d + 64) >> 3) ^ sw) << 3;
            const uint4 c1 = *reinterpret_cast<const uint4*>(cs + k1), c2 = *reinterpret_cast<const uint4*>(cs + k2);
            const uint4 s1 = *reinterpret_cast<const uint4*>(sn + k1), s2 = *reinterpret_cast<const uint4*>(sn + k2);
            const uint32_t w1v[4] = {w1.x, w1.y, w1.z, w1.w}, w2v[4] = {w2.x, w2.y, w2.z, w2.w};
            const uint32_t c1v[4] = {c1.x, c1.y, c1.z, c1.w}, c2v[4] = {c2.x, c2.y, c2.z, c2.w};
            const uint32_t s1v[4] = {s1.x, s1.y, s1.z, s1.w}, s2v[4] = {s2.x, s2.y, s2.z, s2.w};
            float o1[8], o2[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int h = j >> 1;
                const float nw1 = (j & 1) ? bf16hi(w1v[h]) : bf16lo(w1v[h]);
                const float nw2 = (j & 1) ? bf16hi(w2v[h]) : bf16lo(w2v[h]);
                const float cc1 = (j & 1) ? bf16hi(c1v[h]) : bf16lo(c1v[h]);
                const float cc2 = (j & 1) ? bf16hi(c2v[h]) : bf16lo(c2v[h]);
                const float ss1 = (j & 1) ? bf16hi(s1v[h]) : bf16lo(s1v[h]);
                const float ss2 = (j & 1) ? bf16hi(s2v[h]) : bf16lo(s2v[h]);
                const float a1 = x1[i + j] * r * nw1;
                const float a2 = x2[i + j] * r * nw2;
                o1[j] = (a1 * cc1 - a2 * ss1) * osc;
                o2[j] = (a2 * cc2 + a1 * ss2) * osc;
            }
            if (valid) {
                const uint4 p1 = pack8_bf16(o1), p2 = pack8_bf16(o2);
                __nv_bfloat16* out = map == 0 ? dst : cache;
                *reinterpret_cast<uint4*>(out + d) = p1;
                *reinterpret_cast<uint4*>(out + d + 64) = p2;
            }
        }
    }
}

template <int EPI, int BN>
__global__ void __launch_bounds__(P_THREADS, 1)
gemm_persist_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                    const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                    const PArgs args) {
    using Cfg = PCfg<EPI, BN>;
    extern __shared__ uint8_t persist_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(persist_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::NSTAGES * Cfg::STAGE);
    uint64_t* empty = full + Cfg::NSTAGES;
    uint64_t* accf = empty + Cfg::NSTAGES;      // [2] MMA -> epilogue
    uint64_t* acce = accf + 2;                  // [2] epilogue -> MMA
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    // EPI_QKV: cos / sin rows of the tile's positions, [2 (cos, sin)][128 rows][128]
    __nv_bfloat16* rope = reinterpret_cast<__nv_bfloat16*>(smem + Cfg::NSTAGES * Cfg::STAGE + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = args.tiles_m * args.tiles_n;
    const int nk = args.K / GEMM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::NSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], P_EPI_WARPS);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB0);
        prefetch_tmap(&tmB1);
        prefetch_tmap(&tmB2);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
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

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;   // k-blocks issued so far (ring position)
            for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
                const int m0 = (t / args.tiles_n) * GEMM_BM;
                int nt = t % args.tiles_n;
                const CUtensorMap* tb = &tmB0;
                if (EPI != EPI_SILU_MUL && nt >= args.nb0) {
                    nt -= args.nb0;
                    tb = &tmB1;
                    if (nt >= args.nb1) {
                        nt -= args.nb1;
                        tb = &tmB2;
                    }
                }
                const int n0 = nt * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % Cfg::NSTAGES;
                    if (g >= (uint32_t)Cfg::NSTAGES &&
                        !bounded_wait(&empty[s], ((g / Cfg::NSTAGES) & 1) ^ 1, args.timeout_cycles)) {
                        *abort_flag = 1;
                        atomicExch(args.err, 31);
                        break;
                    }
                    uint8_t* st = smem + s * Cfg::STAGE;
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
                    tma_load_2d(st, &tmA, kb * GEMM_BK, m0, &full[s]);
                    tma_load_2d(st + GEMM_TILE_BYTES, tb, kb * GEMM_BK, n0, &full[s]);
                    if (Cfg::NB == 2)
                        tma_load_2d(st + GEMM_TILE_BYTES + Cfg::B_BYTES, &tmB1, kb * GEMM_BK, n0, &full[s]);
                }
            }
            // on an abort every copy still in flight lands before the CTA may exit
            if (*abort_flag)
                for (uint32_t q = g > (uint32_t)Cfg::NSTAGES ? g - Cfg::NSTAGES : 0; q < g; ++q)
                    bounded_wait(&full[q % Cfg::NSTAGES], (q / Cfg::NSTAGES) & 1, args.timeout_cycles);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // gate/up: the two B tiles are stacked in shared memory (gate rows, then up rows), so one
            // MMA with N = 2 BN fills both accumulators (gate at columns 0.., up at BN..)
            constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, BN * Cfg::NB);
            uint32_t g = 0;
            int i = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x, ++i) {
                const int b = i & 1, u = i >> 1;
                if (u >= 1 && !bounded_wait(&acce[b], (u - 1) & 1, args.timeout_cycles)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 32);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * Cfg::ACC_COLS);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % Cfg::NSTAGES;
                    if (!bounded_wait(&full[s], (g / Cfg::NSTAGES) & 1, args.timeout_cycles) || *abort_flag) {
                        *abort_flag = 1;
                        atomicExch(args.err, 33);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * Cfg::STAGE);
#pragma unroll
                    for (int k = 0; k < GEMM_BK / 16; ++k) {
                        const uint64_t ad = sw128_kmajor_desc(sa + k * 32);
                        tc_mma_f16(acc, ad, sw128_kmajor_desc(sa + GEMM_TILE_BYTES + k * 32), idesc, (kb | k) != 0);
                    }
                    tc_commit(&empty[s]);
                }
                tc_commit(&accf[b]);   // also after an abort: arrives once the issued MMAs are done
            }
        }
    } else {
        // epilogue: warp w covers TMEM lanes 32 * (w % 4) .. + 31 (row of the tile) and
        // column half (w - 2) / 4 of the tile
        const int quad = warp & 3, half = (warp - 2) >> 2;
        constexpr int HB = BN / 2;   // columns per epilogue warp
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            const int b = i & 1, u = i >> 1;
            if (EPI == EPI_ADD_F32) {
                // the residual rows this lane adds to: pull them into L2 while the MMAs run
                const int prow = (t / args.tiles_n) * GEMM_BM + quad * 32 + lane;
                if (prow < args.M) {
                    const float* pp = reinterpret_cast<const float*>(args.C) + (size_t)prow * args.ldc +
                                      (t % args.tiles_n) * BN + half * HB;
#pragma unroll
                    for (int q = 0; q < HB * 4; q += 128)
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(pp) + q));
                }
            }
            if (EPI == EPI_QKV) {
                // Stage the cos / sin rows of this quadrant's 32 positions while the
                // MMAs run (warp half 0: cos, 1: sin; one 256-byte row per 16 lanes):
                // one round of coalesced loads instead of dependent per-row loads in
                // the epilogue.  The partner warp of the quadrant is done with the
                // previous tile's rows at the first barrier.
                // All 16 loads of a lane are issued before the barrier and stored after it, so
                // the tile pays one load latency, overlapped with the wait for the partner warp
                // (with four loads in flight at a time, four loaded-L2 round trips per tile sat
                // on the epilogue's path).
                const int mt = (t / args.tiles_n) * GEMM_BM;
                const bool is_v = (t % args.tiles_n) >= args.nb0 + args.nb1;
                uint4 rows[16];
                if (!is_v) {
                    const __nv_bfloat16* tab = half ? args.qkv.sin_table : args.qkv.cos_table;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int i = lane + 32 * k, r = i >> 4, ch = i & 15;
                        const int grow = mt + quad * 32 + r;
                        const int gr = grow < args.M ? grow : 0;
                        const int pp = args.qkv.start_pos + gr % args.qkv.S;
                        rows[k] = *reinterpret_cast<const uint4*>(tab + (size_t)pp * 128 + ch * 8);
                    }
                }
                named_bar_sync(1 + quad, 64);
                if (!is_v) {
                    __nv_bfloat16* dst = rope + (size_t)(half * GEMM_BM + quad * 32) * 128;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int i = lane + 32 * k, r = i >> 4, ch = i & 15;
                        *reinterpret_cast<uint4*>(dst + r * 128 + ((ch ^ (r & 15)) * 8)) = rows[k];
                    }
                }
            }
            bool acc_ok = bounded_wait(&accf[b], u & 1, args.timeout_cycles) && !*abort_flag;
            // EPI_QKV: the quadrant's two warps decide together (the barrier also publishes the staged rows)
            if (EPI == EPI_QKV) acc_ok = !named_bar_or(1 + quad, 64, !acc_ok);
            if (!acc_ok) {
                if (lane == 0) atomicExch(args.err, 34);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int m0 = (t / args.tiles_n) * GEMM_BM;
            const int nt_all = t % args.tiles_n;
            const int row = m0 + quad * 32 + lane;
            const uint32_t acc = tmem + (uint32_t)(b * Cfg::ACC_COLS) + ((uint32_t)(quad * 32) << 16);
            if (EPI == EPI_QKV) {
                int map = 0, head = nt_all;
                if (head >= args.nb0) {
                    head -= args.nb0;
                    map = 1;
                    if (head >= args.nb1) {
                        head -= args.nb1;
                        map = 2;
                    }
                }
                // one head per epilogue warp (BN = 256), or the two halves of one head
                const __nv_bfloat16* cs = rope + (size_t)(quad * 32 + lane) * 128;
                const __nv_bfloat16* sn = rope + (size_t)(GEMM_BM + quad * 32 + lane) * 128;
                if (BN == 256) {
                    qkv_row_epilogue(args, acc + half * 128, map, head * 2 + half, row, cs, sn, lane & 15);
                } else {
                    // BN = 128: the partner warp stays idle for this tile
                    if (half == 0) qkv_row_epilogue(args, acc, map, head, row, cs, sn, lane & 15);
                }
            } else {
                const int n0 = nt_all * BN + half * HB;
                for (int c0 = 0; c0 < HB; c0 += 32) {
                    const int c = half * HB + c0;
                    float v[32];
                    tmem_ld32(acc + c, v);
                    if (EPI == EPI_SILU_MUL) {
                        float up[32];
                        tmem_ld32(acc + BN + c, up);
#pragma unroll
                        for (int q = 0; q < 32; ++q) v[q] = v[q] / (1.0f + expf(-v[q])) * up[q];
                    }
                    if (row < args.M) {
                        if (EPI == EPI_STORE_F32 || EPI == EPI_ADD_F32) {
                            float* out = reinterpret_cast<float*>(args.C) + (size_t)row * args.ldc + n0 + c0;
#pragma unroll
                            for (int q = 0; q < 32; q += 4) {
                                float4 o = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                                if (EPI == EPI_ADD_F32) {
                                    const float4 p = *reinterpret_cast<const float4*>(out + q);
                                    o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
                                }
                                *reinterpret_cast<float4*>(out + q) = o;
                            }
                        } else {
                            __nv_bfloat16* out =
                                reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + n0 + c0;
#pragma unroll
                            for (int q = 0; q < 32; q += 8) *reinterpret_cast<uint4*>(out + q) = pack8_bf16(v + q);
                        }
                    }
                }
            }
            // this warp's lanes have read the buffer: hand it back to the MMA thread
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

}  // namespace mq
