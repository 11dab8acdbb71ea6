// Two-SM (CTA pair) tcgen05 GEMM for the large prefill GEMMs: the residual-add
// projection (C_f32 += A . B^T; the routing in prefill.cu uses it there) and
// gate/up with SiLU*mul (supported, measured slower than the one-CTA kernel,
// not routed).
//
// A thread-block cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): CTA r of the pair holds rows
// [128 r, 128 r + 128) of the A tile and its half of the 256 B rows (for
// gate/up: CTA 0 the 128 gate rows, CTA 1 the 128 up rows) in its own shared
// memory, and its own 128 output rows x 256 columns in its own TMEM.  Per
// 64-wide K slice a CTA therefore loads 16 KB of A and 16 KB of B for 128 x 256
// outputs, against 16 + 32 KB in the one-CTA 128 x 256 tile: a third less
// L2-to-SM traffic per FLOP (measured gain on the residual-add GEMMs at
// B = 8 x 2048: 104.5 -> 101.7 us per launch).
//
// Roles (both CTAs unless stated): warp 0 lane 0 issues the TMA loads of the
// CTA's slices; the loads complete on the leader CTA's `full` barrier
// (.cta_group::2 form, no multicast: every load reads only this GPU's memory
// into the issuing CTA's shared memory).  Warp 1 allocates TMEM for the pair
// (cta_group::2); in the leader one thread issues the MMAs and commits to the
// `empty` / `accf` barriers of both CTAs (tcgen05.commit multicast).  Warps 2-9
// run the epilogue on their CTA's rows and arrive on the leader's `acce`
// barrier when a TMEM buffer is drained.  Double-buffered accumulators (2 x 256
// columns).  Every wait is bounded and sets an error code; every thread reaches
// the final cluster barrier, so no CTA leaves while its peer may still signal
// it.
#pragma once

#include <cuda_bf16.h>

#include "gemm_persist.cuh"

namespace mq {

constexpr int PAIR_STAGE = 2 * GEMM_TILE_BYTES;              // A slice + B slice (16 KB each)
constexpr int PAIR_NSTAGES = 6;
constexpr int PAIR_TMEM_COLS = 512;                          // two 256-column accumulators
constexpr int PAIR_SMEM = PAIR_NSTAGES * PAIR_STAGE + 1024 + 256;

__device__ __forceinline__ uint32_t pair_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t pair_mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void pair_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory, completion counted on an mbarrier of
// either CTA of the pair (bar: shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the barrier at this shared-memory offset in both CTAs of the pair
// once every previously issued MMA of this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((unsigned short)3)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// EPI_ADD_F32: 256 x 256 pair tiles of C (N % 256 == 0), CTA r reads B rows
//   [n0 + 128 r, +128) of map 0.
// EPI_SILU_MUL: 256 x 128 pair tiles of act (N % 128 == 0), CTA 0 reads gate
//   rows [n0, +128) (map 0), CTA 1 up rows (map 1); TMEM columns 0..127 hold
//   gate, 128..255 up, in both CTAs.
template <int EPI>
__global__ void __launch_bounds__(P_THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                 const __grid_constant__ CUtensorMap tmB1, const PArgs args) {
    static_assert(EPI == EPI_ADD_F32 || EPI == EPI_SILU_MUL, "pair GEMM epilogues");
    constexpr int TN = EPI == EPI_SILU_MUL ? 128 : 256;   // output columns per pair tile
    extern __shared__ uint8_t pair_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pair_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + PAIR_NSTAGES * PAIR_STAGE);
    uint64_t* empty = full + PAIR_NSTAGES;
    uint64_t* accf = empty + PAIR_NSTAGES;      // [2] MMA -> epilogue (both CTAs)
    uint64_t* acce = accf + 2;                  // [2] epilogues of both CTAs -> MMA (leader)
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = pair_rank();
    const bool leader = rank == 0;
    const int npairs = gridDim.x / 2, pair = blockIdx.x / 2;
    const int tiles_n = args.tiles_n;               // pair tiles per 256-row block
    const int ntiles = args.tiles_m * tiles_n;      // pair tiles (tiles_m counts 256-row blocks)
    const int nk = args.K / GEMM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PAIR_NSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 2 * P_EPI_WARPS);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB0);
        prefetch_tmap(&tmB1);
    }
    pair_sync();   // both CTAs' barriers exist before any load or commit targets them
    if (warp == 1) {
        tmem_alloc_pair(tmem_holder, PAIR_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    pair_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // Programmatic dependent launch: the set-up above overlapped the previous
    // kernel's tail; nothing it wrote is read before pdl_wait.
    pdl_trigger();
    pdl_wait();
    const uint32_t full_leader = pair_mapa(smem_u32(full), 0);
    const uint32_t acce_leader = pair_mapa(smem_u32(acce), 0);

    if (warp == 0) {
        if (lane == 0) {
            const CUtensorMap* tb = (EPI == EPI_SILU_MUL && rank == 1) ? &tmB1 : &tmB0;
            uint32_t g = 0;
            for (int t = pair; t < ntiles && !*abort_flag; t += npairs) {
                const int m0 = (t / tiles_n) * 256 + (int)rank * 128;
                const int n0 = (t % tiles_n) * TN + (EPI == EPI_ADD_F32 ? (int)rank * 128 : 0);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % PAIR_NSTAGES;
                    if (g >= (uint32_t)PAIR_NSTAGES &&
                        !bounded_wait(&empty[s], ((g / PAIR_NSTAGES) & 1) ^ 1, args.timeout_cycles)) {
                        *abort_flag = 1;
                        atomicExch(args.err, 51);
                        break;
                    }
                    uint8_t* st = smem + s * PAIR_STAGE;
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * PAIR_STAGE);   // both CTAs' slices
                    const uint32_t fb = full_leader + s * 8;
                    tma_load_2d_pair(st, &tmA, kb * GEMM_BK, m0, fb);
                    tma_load_2d_pair(st + GEMM_TILE_BYTES, tb, kb * GEMM_BK, n0, fb);
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(256, 256);
            uint32_t g = 0;
            int i = 0;
            for (int t = pair; t < ntiles && !*abort_flag; t += npairs, ++i) {
                const int b = i & 1, u = i >> 1;
                if (u >= 1 && !bounded_wait(&acce[b], (u - 1) & 1, args.timeout_cycles)) {
                    *abort_flag = 1;
                    atomicExch(args.err, 52);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * 256);
                bool good = true;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const uint32_t s = g % PAIR_NSTAGES;
                    if (!bounded_wait(&full[s], (g / PAIR_NSTAGES) & 1, args.timeout_cycles) || *abort_flag) {
                        *abort_flag = 1;
                        atomicExch(args.err, 53);
                        good = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * PAIR_STAGE);
#pragma unroll
                    for (int k = 0; k < GEMM_BK / 16; ++k)
                        tc_mma_f16_pair(acc, sw128_kmajor_desc(sa + k * 32),
                                        sw128_kmajor_desc(sa + GEMM_TILE_BYTES + k * 32), idesc, (kb | k) != 0);
                    tc_commit_pair(&empty[s]);
                }
                tc_commit_pair(&accf[b]);   // also after an abort: arrives once the issued MMAs are done
                if (!good) break;
            }
        }
    } else {
        // epilogue: warp w covers TMEM lanes 32 (w % 4) .. (rows of this CTA) and
        // column half (w - 2) / 4 of the 256 accumulator columns
        const int quad = warp & 3, half = (warp - 2) >> 2;
        int i = 0;
        for (int t = pair; t < ntiles; t += npairs, ++i) {
            const int b = i & 1, u = i >> 1;
            const int row = (t / tiles_n) * 256 + (int)rank * 128 + quad * 32 + lane;
            if (EPI == EPI_ADD_F32 && row < args.M) {
                // the residual row segment this lane adds to: into L2 while the MMAs run
                const float* pp = reinterpret_cast<const float*>(args.C) + (size_t)row * args.ldc +
                                  (t % tiles_n) * 256 + half * 128;
#pragma unroll
                for (int q = 0; q < 128 * 4; q += 128)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(pp) + q));
            }
            if (!bounded_wait(&accf[b], u & 1, args.timeout_cycles) || *abort_flag) {
                if (lane == 0) atomicExch(args.err, 54);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(b * 256) + ((uint32_t)(quad * 32) << 16);
            if (EPI == EPI_SILU_MUL) {
                // half h: output columns 64 h .. 64 h + 63 of the tile (gate at c, up at 128 + c)
                for (int c0 = 0; c0 < 64; c0 += 32) {
                    const int c = half * 64 + c0;
                    float v[32], up[32];
                    tmem_ld32(acc + c, v);
                    tmem_ld32(acc + 128 + c, up);
#pragma unroll
                    for (int q = 0; q < 32; ++q) v[q] = v[q] / (1.0f + expf(-v[q])) * up[q];
                    if (row < args.M) {
                        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc +
                                             (t % tiles_n) * TN + c;
#pragma unroll
                        for (int q = 0; q < 32; q += 8) *reinterpret_cast<uint4*>(out + q) = pack8_bf16(v + q);
                    }
                }
            } else {
                for (int c0 = 0; c0 < 128; c0 += 32) {
                    const int c = half * 128 + c0;
                    float v[32];
                    tmem_ld32(acc + c, v);
                    if (row < args.M) {
                        float* out = reinterpret_cast<float*>(args.C) + (size_t)row * args.ldc + (t % tiles_n) * 256 + c;
#pragma unroll
                        for (int q = 0; q < 32; q += 4) {
                            const float4 p = *reinterpret_cast<const float4*>(out + q);
                            *reinterpret_cast<float4*>(out + q) =
                                make_float4(v[q] + p.x, v[q + 1] + p.y, v[q + 2] + p.z, v[q + 3] + p.w);
                        }
                    }
                }
            }
            // this warp has read the buffer: tell the leader's MMA thread
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) mbar_arrive(&acce[b]);
                else mbar_arrive_remote(acce_leader + b * 8);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // no CTA leaves (or frees TMEM) while its peer may still commit to or arrive on it
    pair_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, PAIR_TMEM_COLS);
    }
}

}  // namespace mq
