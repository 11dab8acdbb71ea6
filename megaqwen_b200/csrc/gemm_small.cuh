// Small-batch weight-streaming GEMM for batched decode (sm_100a tcgen05).
//
//   out[b, n] = epilogue( sum_k X[b, k] W[n, k] )   for b < Bv tokens, all n
//
// Operands are swapped relative to the prefill GEMM: the MMA's M side is 128
// weight rows (A = W tile, K-major), its N side the NP padded tokens (B = X,
// K-major), so one tcgen05.mma.kind::f16 (M=128, N=NP, K=16) covers the batch.
//
// Grid (tiles, 1, S) in clusters of (1, 1, S), S <= 16: the S CTAs of a cluster split
// the K dimension of one 128-row tile.  Each CTA stages its fp32 partial tile
// [NP][128] in its own shared memory, and after a cluster barrier CTA r sums
// the rows (tokens) of slice r across the S partials through distributed
// shared memory, in rank order (deterministic, no atomics), and applies the
// epilogue:
//   SM_STORE   out_f32[b, col + n] = acc            (q | k | v side by side)
//   SM_RESID   out_f32[b, n] += acc                 (residual stream)
//   SM_SILU    act_bf16[b, n] = silu(acc_gate) * acc_up
//              (gate and up tiles t in the same CTA: two TMEM accumulators)
//   SM_QKV     q|k|v heads: QK-RMSNorm + RoPE, q to fp32, k/v rows into the cache
//   SM_ARGMAX  (S == 1) optional logits store, and per token the largest
//              value of the tile with its lowest index, merged into a 64-bit
//              key per token with atomicMax (the LM head's fused argmax)
//
// Warp 0 (one thread) streams the K slices with TMA through an mbarrier ring;
// the whole slice of a CTA fits in the ring, so every weight byte of the GEMM
// is in flight at once.  The kernel is a programmatic dependent launch: the
// weight tiles are requested before pdl_wait (they do not depend on the
// previous kernel), the token tiles after it.  Warp 1 owns TMEM and issues the
// MMAs; warps 2-5 (one TMEM lane quadrant each, thread = weight row n) run the
// epilogue.  Every mbarrier wait is bounded and sets an error code.
#pragma once

#include <cuda_bf16.h>

#include "gemm_tc.cuh"
#include "megaqwen_b200.h"

namespace mq {

enum SmallMode { SM_STORE = 0, SM_RESID = 1, SM_SILU = 2, SM_ARGMAX = 3, SM_QKV = 4 };

// SM_QKV epilogue operands: the q/k/v projections of one layer, one head per
// 128-row tile.  q and k heads get RMSNorm over the head (x norm weight) and
// rotate-half RoPE at the sequence's position; q goes to Qf (fp32), k and v
// rows (bf16) into the sequence's cache at that position.
struct QkvEpi {
    const __nv_bfloat16* q_norm;
    const __nv_bfloat16* k_norm;
    const __nv_bfloat16* cos_table;   // [max_seq, 128]
    const __nv_bfloat16* sin_table;
    const int* pos;                   // [Bv]
    float* Qf;                        // [Bv, 2048]
    __nv_bfloat16* k_cache;           // layer base of sequence 0: [8, max_seq, 128]
    __nv_bfloat16* v_cache;
    long long seq_stride;             // elements between sequences' caches
    int max_seq;
};

template <int NP, int MODE>
struct Small2Cfg {
    static constexpr int NW = (MODE == SM_SILU) ? 2 : 1;                // weight tiles per stage
    static constexpr int W_BYTES = GEMM_BM * GEMM_BK * 2;               // 16 KB
    static constexpr int X_BYTES = NP * GEMM_BK * 2;
    static constexpr int STAGE = NW * W_BYTES + X_BYTES;
    static constexpr int MAX_STAGES = 8;
    static constexpr int ACC_COLS = NW * NP;
    static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : 256;
    static constexpr int RED_LD = (MODE == SM_ARGMAX) ? 129 : 128;     // floats per staged token row
    static constexpr int RED_BYTES = NW * NP * RED_LD * 4;
    __host__ __device__ static constexpr int ring_bytes(int stages) { return stages * STAGE; }
    __host__ __device__ static constexpr int smem_bytes(int stages) {
        return (ring_bytes(stages) > RED_BYTES ? ring_bytes(stages) : RED_BYTES) + 1024 + 256;
    }
};

struct Small2Args {
    float* out;              // SM_STORE / SM_RESID: fp32 [Bv, ldo]; SM_ARGMAX: optional logits [Bv, ldo]
    __nv_bfloat16* act;      // SM_SILU: bf16 [Bv, ldo]
    unsigned long long* best;  // SM_ARGMAX: [Bv] keys
    int ldo;
    int tiles0, tiles1;      // SM_STORE: tiles of maps 0 and 1 (the rest belong to map 2)
    int col1, col2;          // SM_STORE: output column offsets of maps 1 and 2
    int Bv;
    int K;
    int kpb;                 // K blocks (of 64) per split
    int stages;              // ring depth; smem launched as smem_bytes(stages)
    int* err;
    long long timeout_cycles;
    QkvEpi qkv;              // SM_QKV
    // RMSNorm folded into the GEMMs: a consumer (SM_QKV, SM_SILU, SM_ARGMAX) scales
    // row b by 1/rms from ss_in; a producer (SM_RESID) also writes xw_out =
    // bf16(x * w_next) (the next operand) and ss_out (per-tile sums of squares).
    const float* ss_in;      // [Bv, 8] or null
    float* ss_out;           // [Bv, 8]
    const __nv_bfloat16* w_next;
    __nv_bfloat16* xw_out;   // [NP, 1024] or null
    unsigned long long* trace;   // optional: 8 %globaltimer stamps per CTA (phase timing)
};

__device__ __forceinline__ void trace_stamp(const Small2Args& a, int k) {
    if (a.trace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        const int cta = blockIdx.x + gridDim.x * blockIdx.z;
        a.trace[cta * 8 + k] = t;
    }
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f32x4(const float* local, uint32_t rank) {
    uint32_t remote;
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}
// order-preserving map of a float to an unsigned key (larger float -> larger key)
__device__ __forceinline__ uint32_t f32_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 1 / rms of token row b of the residual stream from its per-128-column
// partial sums of squares (the producer's epilogue wrote them), 1 if absent.
__device__ __forceinline__ float row_rstd(const float* ss, int b) {
    if (!ss) return 1.f;
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < MQ_HIDDEN_SIZE / 128; ++i) t += ss[b * (MQ_HIDDEN_SIZE / 128) + i];
    return rsqrtf(t / (float)MQ_HIDDEN_SIZE + 1e-6f);
}

// Epilogue operands that do not depend on the split-K sum (fetched early).
struct EpiPre {
    float4 x;       // SM_RESID: residual stream value
    uint2 w;        // SM_RESID: next RMSNorm weight; SM_QKV: q/k norm weight
    uint2 cs, sn;   // SM_QKV: RoPE cos / sin at the row's position
    float rs;       // row rstd (SM_QKV, SM_SILU)
    int p;          // SM_QKV: position
};

template <int MODE>
__device__ __forceinline__ EpiPre epi_prefetch(const Small2Args& a, int map, int b, int c4, int n0) {
    EpiPre e;
    if (MODE == SM_RESID) {
        e.x = *reinterpret_cast<const float4*>(a.out + (size_t)b * a.ldo + n0 + c4);
        if (a.w_next) e.w = *reinterpret_cast<const uint2*>(a.w_next + n0 + c4);
    }
    if (MODE == SM_QKV || MODE == SM_SILU) e.rs = row_rstd(a.ss_in, b);
    if (MODE == SM_QKV) {
        e.p = a.qkv.pos[b];
        if (map < 2) {
            e.w = *reinterpret_cast<const uint2*>((map == 0 ? a.qkv.q_norm : a.qkv.k_norm) + c4);
            e.cs = *reinterpret_cast<const uint2*>(a.qkv.cos_table + (size_t)e.p * GEMM_BM + c4);
            e.sn = *reinterpret_cast<const uint2*>(a.qkv.sin_table + (size_t)e.p * GEMM_BM + c4);
        }
    }
    return e;
}

__device__ __forceinline__ float4 bf16x4(uint2 v) {
    return make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y));
}
__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    return pk;
}

// The epilogue of one (token row b, columns c4..c4+3) item; one warp holds one
// full 128-column row of the tile (lane = c4 / 4).
template <int MODE>
__device__ __forceinline__ void epi_finish(const Small2Args& a, int map, int tile, int col_off, int n0, int b, int c4,
                                           float4 acc, float4 acc2, const EpiPre& e) {
    if (MODE == SM_QKV) {
        const QkvEpi& q = a.qkv;
        float4 x = make_float4(acc.x * e.rs, acc.y * e.rs, acc.z * e.rs, acc.w * e.rs);
        if (map < 2) {
            const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
            const float rh = rsqrtf(ss / (float)GEMM_BM + 1e-6f);
            const float4 nw = bf16x4(e.w);
            x.x *= rh * nw.x; x.y *= rh * nw.y; x.z *= rh * nw.z; x.w *= rh * nw.w;
            // rotate-half partner dims (c4 +- 64) live in lane ^ 16
            const float y0 = __shfl_xor_sync(0xffffffffu, x.x, 16), y1 = __shfl_xor_sync(0xffffffffu, x.y, 16);
            const float y2 = __shfl_xor_sync(0xffffffffu, x.z, 16), y3 = __shfl_xor_sync(0xffffffffu, x.w, 16);
            const float4 cs = bf16x4(e.cs), sn = bf16x4(e.sn);
            const float sg = c4 < 64 ? -1.f : 1.f;
            x.x = x.x * cs.x + sg * y0 * sn.x;
            x.y = x.y * cs.y + sg * y1 * sn.y;
            x.z = x.z * cs.z + sg * y2 * sn.z;
            x.w = x.w * cs.w + sg * y3 * sn.w;
        }
        if (map == 0) {
            *reinterpret_cast<float4*>(q.Qf + (size_t)b * 2048 + n0 + c4) = x;
        } else {
            __nv_bfloat16* row = (map == 1 ? q.k_cache : q.v_cache) + b * q.seq_stride +
                                 ((size_t)tile * q.max_seq + e.p) * GEMM_BM + c4;
            *reinterpret_cast<uint2*>(row) = pack_bf16x4(x.x, x.y, x.z, x.w);
        }
    } else if (MODE == SM_STORE) {
        *reinterpret_cast<float4*>(a.out + (size_t)b * a.ldo + col_off + n0 + c4) = acc;
    } else if (MODE == SM_RESID) {
        float4 x = e.x;
        x.x += acc.x; x.y += acc.y; x.z += acc.z; x.w += acc.w;
        *reinterpret_cast<float4*>(a.out + (size_t)b * a.ldo + n0 + c4) = x;
        if (a.xw_out) {
            // next GEMM operand bf16(x * w_next) and this tile's sum of squares of the row
            const float4 w = bf16x4(e.w);
            *reinterpret_cast<uint2*>(a.xw_out + (size_t)b * MQ_HIDDEN_SIZE + n0 + c4) =
                pack_bf16x4(x.x * w.x, x.y * w.y, x.z * w.z, x.w * w.w);
            const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
            if ((threadIdx.x & 31) == 0) a.ss_out[b * (MQ_HIDDEN_SIZE / 128) + n0 / 128] = ss;
        }
    } else if (MODE == SM_SILU) {
        const float g0 = acc.x * e.rs, g1 = acc.y * e.rs, g2 = acc.z * e.rs, g3 = acc.w * e.rs;
        *reinterpret_cast<uint2*>(a.act + (size_t)b * a.ldo + n0 + c4) =
            pack_bf16x4(g0 / (1.0f + expf(-g0)) * (acc2.x * e.rs), g1 / (1.0f + expf(-g1)) * (acc2.y * e.rs),
                        g2 / (1.0f + expf(-g2)) * (acc2.z * e.rs), g3 / (1.0f + expf(-g3)) * (acc2.w * e.rs));
    }
}

template <int NP, int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                  const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmX,
                  const Small2Args args) {
    using Cfg = Small2Cfg<NP, MODE>;
    extern __shared__ uint8_t small2_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(small2_smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = args.stages;
    const int region = Cfg::ring_bytes(S) > Cfg::RED_BYTES ? Cfg::ring_bytes(S) : Cfg::RED_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + region);
    uint64_t* empty = full + Cfg::MAX_STAGES;
    uint64_t* accf = empty + Cfg::MAX_STAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accf + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* red = reinterpret_cast<float*>(smem);   // reuses the ring once all MMAs have completed

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int tile = blockIdx.x, col_off = 0, map = 0;
    const CUtensorMap* tmA = &tmW0;
    if ((MODE == SM_STORE || MODE == SM_QKV) && tile >= args.tiles0) {
        tile -= args.tiles0;
        tmA = &tmW1;
        col_off = args.col1;
        map = 1;
        if (tile >= args.tiles1) {
            tile -= args.tiles1;
            tmA = &tmW2;
            col_off = args.col2;
            map = 2;
        }
    }
    const int n0 = tile * GEMM_BM;
    const int ksplits = gridDim.z;
    const int kb0 = blockIdx.z * args.kpb;
    const int nk = max(0, min(args.kpb, args.K / GEMM_BK - kb0));

    const int pre = min(nk, S);
    if (threadIdx.x == 0) {
        trace_stamp(args, 0);
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        *abort_flag = 0;
        fence_mbar_init();
        // the weight slices do not depend on the previous kernel: request them first
        for (int i = 0; i < pre; ++i) {
            uint8_t* st = smem + i * Cfg::STAGE;
            mbar_arrive_expect_tx(&full[i], Cfg::STAGE);
            tma_load_2d(st, tmA, (kb0 + i) * GEMM_BK, n0, &full[i]);
            if (Cfg::NW == 2) tma_load_2d(st + Cfg::W_BYTES, &tmW1, (kb0 + i) * GEMM_BK, n0, &full[i]);
        }
        prefetch_tmap(&tmX);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_trigger();
    const uint32_t tmem = *tmem_holder;
    // everything but the producer waits for the predecessor grid here
    if (threadIdx.x != 0) pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            trace_stamp(args, 1);
            pdl_wait();
            asm volatile("fence.proxy.async.global;" ::: "memory");
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + i * Cfg::STAGE + Cfg::NW * Cfg::W_BYTES, &tmX, (kb0 + i) * GEMM_BK, 0, &full[i]);
            int issued = pre;
            for (int i = pre; i < nk; ++i) {
                const int s = i % S;
                if (!bounded_wait(&empty[s], ((i / S) & 1) ^ 1, args.timeout_cycles)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 21);
                    break;
                }
                if (*abort_flag) break;
                uint8_t* st = smem + s * Cfg::STAGE;
                mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
                tma_load_2d(st, tmA, (kb0 + i) * GEMM_BK, n0, &full[s]);
                if (MODE == SM_SILU) tma_load_2d(st + Cfg::W_BYTES, &tmW1, (kb0 + i) * GEMM_BK, n0, &full[s]);
                tma_load_2d(st + Cfg::NW * Cfg::W_BYTES, &tmX, (kb0 + i) * GEMM_BK, 0, &full[s]);
                ++issued;
            }
            for (int i = issued > S ? issued - S : 0; i < issued; ++i)
                bounded_wait(&full[i % S], (i / S) & 1, args.timeout_cycles);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, NP);
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (!bounded_wait(&full[s], (i / S) & 1, args.timeout_cycles) || *abort_flag) {
                    *abort_flag = 1;
                    atomicExch(args.err, 22);
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(smem + s * Cfg::STAGE);
                const uint32_t xb = a + Cfg::NW * Cfg::W_BYTES;
#pragma unroll
                for (int k = 0; k < GEMM_BK / 16; ++k) {
                    tc_mma_f16(tmem, sw128_kmajor_desc(a + k * 32), sw128_kmajor_desc(xb + k * 32), idesc,
                               (i | k) != 0);
                    if (MODE == SM_SILU)
                        tc_mma_f16(tmem + NP, sw128_kmajor_desc(a + Cfg::W_BYTES + k * 32),
                                   sw128_kmajor_desc(xb + k * 32), idesc, (i | k) != 0);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accf);
        }
    }
    // ---- partial tile -> shared memory (red[acc][b][n]) ----
    const int quad = warp & 3;
    const int n = quad * 32 + lane;   // weight row within the tile (= TMEM lane) for warps 2-5
    if (warp >= 2) {
        const bool got = nk > 0 && bounded_wait(accf, 0, args.timeout_cycles) && !*abort_flag;
        if (threadIdx.x == 64) trace_stamp(args, 2);
        if (nk > 0 && !got) {
            if (lane == 0) atomicExch(args.err, 23);
            *abort_flag = 1;
        }
        tc_fence_after();
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll
        for (int a = 0; a < Cfg::NW; ++a) {
#pragma unroll
            for (int c = 0; c < NP; c += 32) {
                float v[32];
                if (got) {
                    tmem_ld32(lane_base + a * NP + c, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c + j < NP) red[(a * NP + c + j) * Cfg::RED_LD + n] = v[j];
            }
        }
    }
    tc_fence_before();
    if (MODE == SM_ARGMAX) {
        __shared__ float s_rstd[NP];
        for (int b = threadIdx.x; b < args.Bv; b += blockDim.x) s_rstd[b] = row_rstd(args.ss_in, b);
        __syncthreads();
        // logits store (coalesced along n) and per-token tile maximum
        if (warp >= 2) {
            if (args.out) {
                for (int b = 0; b < args.Bv; ++b)
                    args.out[(size_t)b * args.ldo + n0 + n] = red[b * Cfg::RED_LD + n] * s_rstd[b];
            }
        }
        for (int b = threadIdx.x; b < args.Bv; b += blockDim.x) {
            const float* row = red + b * Cfg::RED_LD;
            const float rs = s_rstd[b];
            float bv = row[0] * rs;
            int bi = 0;
            for (int j = 1; j < GEMM_BM; ++j) {
                const float x = row[j] * rs;
                if (x > bv) { bv = x; bi = j; }
            }
            const unsigned long long key =
                ((unsigned long long)f32_key(bv) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)(n0 + bi));
            atomicMax(args.best + b, key);
        }
    } else {
        // rows (tokens) of this CTA's slice, summed over the cluster's partials in rank order;
        // thread -> (row, 4 consecutive n), one warp per row.  Operands of the epilogue that do
        // not depend on the sum are fetched before the cluster barrier.
        const int per = (args.Bv + ksplits - 1) / ksplits;
        const int r = (int)cluster_rank();
        const int b_lo = r * per, b_hi = min(args.Bv, b_lo + per);
        const int nitems = max(0, b_hi - b_lo) * 32;
        constexpr int PF = 4;
        EpiPre pf[PF];
#pragma unroll
        for (int k = 0; k < PF; ++k) {
            const int item = threadIdx.x + k * blockDim.x;
            if (item < nitems) pf[k] = epi_prefetch<MODE>(args, map, b_lo + (item >> 5), (item & 31) * 4, n0);
        }
        if (threadIdx.x == 64) trace_stamp(args, 3);
        cluster_sync_all();
        if (threadIdx.x == 64) trace_stamp(args, 4);
        auto reduce = [&](int b, int c4, float4* acc) {
#pragma unroll
            for (int a = 0; a < Cfg::NW; ++a) {
                const float* loc = red + (a * NP + b) * Cfg::RED_LD + c4;
                float4 v[16];
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    if (q < ksplits) v[q] = ld_dsmem_f32x4(loc, (uint32_t)q);
                float4 sum = v[0];
#pragma unroll
                for (int q = 1; q < 16; ++q)
                    if (q < ksplits) {
                        sum.x += v[q].x; sum.y += v[q].y; sum.z += v[q].z; sum.w += v[q].w;
                    }
                acc[a] = sum;
            }
        };
#pragma unroll
        for (int k = 0; k < PF; ++k) {
            const int item = threadIdx.x + k * blockDim.x;
            if (item < nitems) {
                const int b = b_lo + (item >> 5), c4 = (item & 31) * 4;
                float4 acc[Cfg::NW];
                reduce(b, c4, acc);
                epi_finish<MODE>(args, map, tile, col_off, n0, b, c4, acc[0], acc[Cfg::NW - 1], pf[k]);
            }
        }
        for (int item = threadIdx.x + PF * blockDim.x; item < nitems; item += blockDim.x) {
            const int b = b_lo + (item >> 5), c4 = (item & 31) * 4;
            const EpiPre q = epi_prefetch<MODE>(args, map, b, c4, n0);
            float4 acc[Cfg::NW];
            reduce(b, c4, acc);
            epi_finish<MODE>(args, map, tile, col_off, n0, b, c4, acc[0], acc[Cfg::NW - 1], q);
        }
        if (threadIdx.x == 64) trace_stamp(args, 5);
        cluster_sync_all();   // peers read this CTA's partials until here
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
    if (threadIdx.x == 64) trace_stamp(args, 6);
}

}  // namespace mq
