// tcgen05 GEMM for prefill: C[M, N] = A[M, K] . B[N, K]^T, bf16 operands in
// global memory (both K-major, i.e. row-major activations and row-major
// nn.Linear weights), fp32 accumulation in TMEM, fused epilogues.
//
// One CTA computes one 128 x 128 output tile.  Warp 0 (one thread) streams
// A/B K-slices of 64 elements through an mbarrier ring with TMA (128-byte
// swizzle); warp 1 allocates TMEM and one of its threads issues the
// tcgen05.mma instructions (M=128, N=128, K=16 each) and commits each stage
// back to the producer; warps 2-5 (one TMEM lane quadrant each) read the
// accumulator with tcgen05.ld and apply the epilogue.  Every wait is bounded.
#pragma once

#include <cuda_bf16.h>

#include "mq_tc.cuh"

namespace mq {

enum GemmEpi {
    EPI_STORE_F32 = 0,   // C_f32[m, n] = acc
    EPI_ADD_F32 = 1,     // C_f32[m, n] += acc        (residual stream)
    EPI_SILU_MUL = 2,    // C_bf16[m, n] = silu(acc_gate) * acc_up  (two B operands)
    EPI_STORE_BF16 = 3,  // C_bf16[m, n] = acc
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;
constexpr int GEMM_TILE_BYTES = GEMM_BM * GEMM_BK * 2;   // 16 KB per operand tile

template <int EPI>
struct GemmCfg {
    static constexpr int NB = (EPI == EPI_SILU_MUL) ? 2 : 1;                 // B operands
    static constexpr int STAGE = GEMM_TILE_BYTES * (1 + NB);
    static constexpr int NSTAGES = (EPI == EPI_SILU_MUL) ? 4 : 6;
    static constexpr int SMEM = NSTAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int TMEM_COLS = GEMM_BN * NB;
};

struct GemmArgs {
    void* C;             // output (fp32 or bf16, see epilogue)
    int ldc;             // elements
    int M, N, K;
    int* err;            // set to a non-zero code when a wait times out
    long long timeout_cycles;
};

__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, long long limit) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

template <int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmB2, const GemmArgs args) {
    using Cfg = GemmCfg<EPI>;
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::NSTAGES * Cfg::STAGE);
    uint64_t* empty = full + Cfg::NSTAGES;
    uint64_t* accf = empty + Cfg::NSTAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accf + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * GEMM_BN, m0 = blockIdx.y * GEMM_BM;
    const int nk = args.K / GEMM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::NSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (Cfg::NB == 2) prefetch_tmap(&tmB2);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % Cfg::NSTAGES;
                if (kb >= Cfg::NSTAGES &&
                    !bounded_wait(&empty[s], ((kb / Cfg::NSTAGES) & 1) ^ 1, args.timeout_cycles)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 1);
                    break;
                }
                if (*abort_flag) break;
                uint8_t* st = smem + s * Cfg::STAGE;
                mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
                tma_load_2d(st, &tmA, kb * GEMM_BK, m0, &full[s]);
                tma_load_2d(st + GEMM_TILE_BYTES, &tmB, kb * GEMM_BK, n0, &full[s]);
                if (Cfg::NB == 2) tma_load_2d(st + 2 * GEMM_TILE_BYTES, &tmB2, kb * GEMM_BK, n0, &full[s]);
                ++issued;
            }
            // every issued copy lands before the CTA may exit
            for (int kb = issued > Cfg::NSTAGES ? issued - Cfg::NSTAGES : 0; kb < issued; ++kb)
                bounded_wait(&full[kb % Cfg::NSTAGES], (kb / Cfg::NSTAGES) & 1, args.timeout_cycles);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, GEMM_BN);
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % Cfg::NSTAGES;
                if (!bounded_wait(&full[s], (kb / Cfg::NSTAGES) & 1, args.timeout_cycles) || *abort_flag) {
                    *abort_flag = 1;
                    atomicExch(args.err, 2);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(smem + s * Cfg::STAGE);
#pragma unroll
                for (int k = 0; k < GEMM_BK / 16; ++k) {
                    const uint64_t ad = sw128_kmajor_desc(a + k * 32);
                    const uint64_t bd = sw128_kmajor_desc(a + GEMM_TILE_BYTES + k * 32);
                    tc_mma_f16(tmem, ad, bd, idesc, (kb | k) != 0);
                    if (Cfg::NB == 2) {
                        const uint64_t bd2 = sw128_kmajor_desc(a + 2 * GEMM_TILE_BYTES + k * 32);
                        tc_mma_f16(tmem + GEMM_BN, ad, bd2, idesc, (kb | k) != 0);
                    }
                }
                tc_commit(&empty[s]);
            }
            (void)ok;
            tc_commit(accf);  // also on failure: arrives once the issued MMAs are done
        }
    } else {
        // epilogue: warp w covers TMEM lanes 32 * (w % 4) .. + 31
        const int quad = warp & 3;
        const int row = m0 + quad * 32 + lane;
        const bool got = bounded_wait(accf, 0, args.timeout_cycles) && !*abort_flag;
        if (!got) {
            if (lane == 0) atomicExch(args.err, 3);
            *abort_flag = 1;
        } else {
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
            for (int c = 0; c < GEMM_BN; c += 32) {
                float v[32];
                tmem_ld32(lane_base + c, v);
                if (EPI == EPI_SILU_MUL) {
                    float u[32];
                    tmem_ld32(lane_base + GEMM_BN + c, u);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = v[i] / (1.0f + expf(-v[i])) * u[i];
                }
                if (row < args.M) {
                    if (EPI == EPI_STORE_F32 || EPI == EPI_ADD_F32) {
                        float* out = reinterpret_cast<float*>(args.C) + (size_t)row * args.ldc + n0 + c;
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                            if (EPI == EPI_ADD_F32) {
                                const float4 p = *reinterpret_cast<const float4*>(out + i);
                                o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
                            }
                            *reinterpret_cast<float4*>(out + i) = o;
                        }
                    } else {
                        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + n0 + c;
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            uint4 pk;
                            __nv_bfloat162 b0 = __floats2bfloat162_rn(v[i], v[i + 1]);
                            __nv_bfloat162 b1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
                            __nv_bfloat162 b3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
                            pk.x = *reinterpret_cast<uint32_t*>(&b0);
                            pk.y = *reinterpret_cast<uint32_t*>(&b1);
                            pk.z = *reinterpret_cast<uint32_t*>(&b2);
                            pk.w = *reinterpret_cast<uint32_t*>(&b3);
                            *reinterpret_cast<uint4*>(out + i) = pk;
                        }
                    }
                }
            }
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

namespace mq {

}  // namespace mq
