// Causal GQA flash attention for prefill on the tensor cores (mma.sync
// m16n8k16, bf16 inputs, fp32 accumulation), online softmax in registers.
//
// Q [M, 16*128], K/V [M, 8*128] bf16 rows m = b*S + s; O [M, 16*128] bf16.
// One CTA = (query block of 64, q head, sequence), 4 warps x 16 query rows.
// Key/value blocks of 64 rows are staged in shared memory with rows padded to
// 272 bytes so ldmatrix reads are bank-conflict free; they are double-buffered
// with cp.async so block kb + 1 loads while block kb is computed.  Scores are scaled in
// the log2 domain (exp2).  Heavier (later) query blocks are scheduled first.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "mq_ptx.cuh"

namespace mq {
namespace pf {

constexpr int FA_B = 64;          // query rows per CTA and keys per block
constexpr int FA_LD = 136;        // padded row (elements)
constexpr int FA_SMEM = 5 * FA_B * FA_LD * 2;   // Q tile + double-buffered K, V tiles (dynamic shared memory)

__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&t);
}

// Asynchronously copy rows [r0, r0+64) of a [.., ld]-strided bf16 matrix (128
// columns starting at col0) into padded shared memory (cp.async, 16 bytes per
// copy); rows >= rmax are zero-filled.
__device__ __forceinline__ void fa_load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int ld, int col0, int r0,
                                             int rmax) {
    for (int i = threadIdx.x; i < FA_B * 16; i += blockDim.x) {
        const int r = i >> 4, c = (i & 15) * 8;
        const bool ok = r0 + r < rmax;
        const __nv_bfloat16* g = ok ? src + (size_t)(r0 + r) * ld + col0 + c : src;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + r * FA_LD + c)), "l"(g),
                     "r"(ok ? 16u : 0u)
                     : "memory");
    }
}
__device__ __forceinline__ void fa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

static __global__ void __launch_bounds__(128) flash_attn_causal_kernel(const __nv_bfloat16* __restrict__ Q,
                                                                const __nv_bfloat16* __restrict__ K,
                                                                const __nv_bfloat16* __restrict__ V,
                                                                __nv_bfloat16* __restrict__ O, int S,
                                                                float scale_log2) {
    extern __shared__ __align__(16) __nv_bfloat16 fa_smem[];
    __nv_bfloat16* sQ = fa_smem;
    __nv_bfloat16* sK0 = sQ + FA_B * FA_LD;       // K tiles [2], then V tiles [2]
    __nv_bfloat16* sV0 = sK0 + 2 * FA_B * FA_LD;
    const int nqb = (S + FA_B - 1) / FA_B;
    const int qb = nqb - 1 - (int)blockIdx.x;
    const int h = blockIdx.y, b = blockIdx.z, kvh = h / (NQ / NKV);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int q0 = qb * FA_B;
    const size_t base = (size_t)b * S;
    const __nv_bfloat16* Kg = K + base * (NKV * D);
    const __nv_bfloat16* Vg = V + base * (NKV * D);

    // Q and the first K/V tile in flight together; tile kb + 1 loads while kb computes
    fa_load_tile(sQ, Q + base * (NQ * D), NQ * D, h * D, q0, S);
    fa_load_tile(sK0, Kg, NKV * D, kvh * D, 0, S);
    fa_load_tile(sV0, Vg, NKV * D, kvh * D, 0, S);
    fa_commit();
    uint32_t qf[8][4];
    float oacc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const int qrow[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};

    for (int kb = 0; kb <= qb; ++kb) {
        const int k0 = kb * FA_B;
        if (kb + 1 <= qb) {
            const int nb = (kb + 1) & 1;
            fa_load_tile(sK0 + nb * FA_B * FA_LD, Kg, NKV * D, kvh * D, k0 + FA_B, S);
            fa_load_tile(sV0 + nb * FA_B * FA_LD, Vg, NKV * D, kvh * D, k0 + FA_B, S);
            fa_commit();
            fa_wait<1>();
        } else {
            fa_wait<0>();
        }
        __syncthreads();
        if (kb == 0) {
#pragma unroll
            for (int s = 0; s < 8; ++s)
                ldm_x4(smem_u32(sQ + (warp * 16 + (lane & 15)) * FA_LD + s * 16 + (lane >> 4) * 8), qf[s][0], qf[s][1],
                       qf[s][2], qf[s][3]);
        }
        const __nv_bfloat16* sK = sK0 + (kb & 1) * FA_B * FA_LD;
        const __nv_bfloat16* sV = sV0 + (kb & 1) * FA_B * FA_LD;
        float sacc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                uint32_t b0, b1, b2, b3;
                const int i = lane >> 3;
                ldm_x4(smem_u32(sK + (8 * j + (i >> 1) * 8 + (lane & 7)) * FA_LD + s * 16 + (i & 1) * 8), b0, b1, b2,
                       b3);
                mma_bf16(sacc[j], qf[s], b0, b1);
                mma_bf16(sacc[j + 1], qf[s], b2, b3);
            }
        }
        // scale (log2 domain), causal + length mask, online softmax
        float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = k0 + 8 * j + 2 * t + (e & 1);
                const int r = e >> 1;
                float v = sacc[j][e] * scale_log2;
                if (key > qrow[r] || key >= S) v = -INFINITY;
                sacc[j][e] = v;
                mx[r] = fmaxf(mx[r], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            corr[r] = exp2f(mrow[r] - mx[r]);
            mrow[r] = mx[r];
            lrow[r] *= corr[r];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            oacc[j][0] *= corr[0]; oacc[j][1] *= corr[0];
            oacc[j][2] *= corr[1]; oacc[j][3] *= corr[1];
        }
        uint32_t pa[4][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = exp2f(sacc[j][0] - mrow[0]), p1 = exp2f(sacc[j][1] - mrow[0]);
            const float p2 = exp2f(sacc[j][2] - mrow[1]), p3 = exp2f(sacc[j][3] - mrow[1]);
            lrow[0] += p0 + p1;
            lrow[1] += p2 + p3;
            const int kt = j >> 1, hi = j & 1;
            pa[kt][hi * 2 + 0] = pack_bf16(p0, p1);
            pa[kt][hi * 2 + 1] = pack_bf16(p2, p3);
        }
        // O += P V  (V^T fragments through ldmatrix.trans)
#pragma unroll
        for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                uint32_t b0, b1, b2, b3;
                const int i = lane >> 3;
                ldm_x4_t(smem_u32(sV + (16 * kt + (i & 1) * 8 + (lane & 7)) * FA_LD + 16 * jj + (i >> 1) * 8), b0,
                         b1, b2, b3);
                mma_bf16(oacc[2 * jj], pa[kt], b0, b1);
                mma_bf16(oacc[2 * jj + 1], pa[kt], b2, b3);
            }
        }
        __syncthreads();   // every warp is done with this buffer before it is refilled
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (qrow[r] >= S) continue;
        const float inv = 1.f / lrow[r];
        __nv_bfloat16* o = O + (base + qrow[r]) * (NQ * D) + h * D;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<uint32_t*>(o + 8 * j + 2 * t) = pack_bf16(oacc[j][2 * r] * inv, oacc[j][2 * r + 1] * inv);
    }
}

}  // namespace pf
}  // namespace mq
