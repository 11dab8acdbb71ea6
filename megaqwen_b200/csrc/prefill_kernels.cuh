// Prefill kernels around the tcgen05 GEMMs and attention: embedding gather,
// RMSNorm to bf16 and argmax.
//
// The kernels begin with pdl_wait/pdl_trigger so that the batched decode can
// launch them as programmatic dependents (no-ops in an ordinary launch).
//
// Activation layout: rows m = b * S + s (sequence b, position s), row-major.
// Residual stream X fp32 [M, 1024]; GEMM operands bf16.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "megaqwen_b200.h"
#include "mq_ptx.cuh"

namespace mq {
namespace pf {

typedef __nv_bfloat16 bf16;
constexpr int H = MQ_HIDDEN_SIZE;
constexpr int D = MQ_HEAD_DIM;
constexpr int NQ = MQ_NUM_Q_HEADS;
constexpr int NKV = MQ_NUM_KV_HEADS;

// X[m, :] = embed[ids[m], :] (fp32).  One warp per row.
static __global__ void embed_kernel(const int* __restrict__ ids, const bf16* __restrict__ embed, float* __restrict__ X,
                             int M) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    const bf16* row = embed + (size_t)ids[m] * H;
    float* out = X + (size_t)m * H;
#pragma unroll
    for (int i = 0; i < H / 256; ++i) {
        const int c = (lane + 32 * i) * 8;
        const uint4 w = *reinterpret_cast<const uint4*>(row + c);
        *reinterpret_cast<float4*>(out + c) = make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
        *reinterpret_cast<float4*>(out + c + 4) = make_float4(bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w));
    }
}

// out[r, :] = bf16(x * rsqrt(mean(x^2) + eps) * w) with x = X[r * in_stride + in_offset, :].
// One warp per output row (demo_e2e.py:37-53 math, fp32).
static __global__ void rmsnorm_bf16_kernel(const float* __restrict__ X, const bf16* __restrict__ w, bf16* __restrict__ out,
                                    int rows, int in_stride, int in_offset) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float* x = X + ((size_t)r * in_stride + in_offset) * H;
    float v[32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = (lane + 32 * i) * 8;
        const float4 a = *reinterpret_cast<const float4*>(x + c);
        const float4 b = *reinterpret_cast<const float4*>(x + c + 4);
        v[8 * i + 0] = a.x; v[8 * i + 1] = a.y; v[8 * i + 2] = a.z; v[8 * i + 3] = a.w;
        v[8 * i + 4] = b.x; v[8 * i + 5] = b.y; v[8 * i + 6] = b.z; v[8 * i + 7] = b.w;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[8 * i + e] * v[8 * i + e];
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / (float)H + 1e-6f);
    bf16* o = out + (size_t)r * H;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = (lane + 32 * i) * 8;
        const uint4 wq = *reinterpret_cast<const uint4*>(w + c);
        const float wf[8] = {bf16lo(wq.x), bf16hi(wq.x), bf16lo(wq.y), bf16hi(wq.y),
                             bf16lo(wq.z), bf16hi(wq.z), bf16lo(wq.w), bf16hi(wq.w)};
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 t = __floats2bfloat162_rn(v[8 * i + 2 * e] * rstd * wf[2 * e],
                                                     v[8 * i + 2 * e + 1] * rstd * wf[2 * e + 1]);
            pk[e] = *reinterpret_cast<uint32_t*>(&t);
        }
        *reinterpret_cast<uint4*>(o + c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

// Greedy argmax of each sequence's logits row in two launches (one block per
// sequence over 151,936 logits took ~74 us): argmax_part_kernel, grid
// (sequences, ARGMAX_SPLIT), leaves each chunk's (value, index) best in
// `part`; argmax_final_kernel, one block per sequence, reduces them.  The
// order is (larger value, then lower index) in both stages, so the result is
// the first index of the row maximum, as a one-pass scan gives; NaN never wins.
constexpr int ARGMAX_SPLIT = 64;

__device__ __forceinline__ void argmax_take(float& best, int& bi, float v, int i) {
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
}

__device__ __forceinline__ void argmax_block(float& best, int& bi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_take(best, bi, ov, oi);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) argmax_take(best, bi, sv[w], si[w]);
}

static __global__ void __launch_bounds__(256) argmax_part_kernel(const float* __restrict__ logits, int V,
                                                                 int logits_ld, float2* __restrict__ part) {
    pdl_wait();
    pdl_trigger();
    const float* x = logits + (size_t)blockIdx.x * logits_ld;
    const int a = (int)(((long long)blockIdx.y * V) / ARGMAX_SPLIT);
    const int e = (int)(((long long)(blockIdx.y + 1) * V) / ARGMAX_SPLIT);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = a + threadIdx.x; i < e; i += blockDim.x) argmax_take(best, bi, x[i], i);
    argmax_block(best, bi);
    if (threadIdx.x == 0) part[blockIdx.x * ARGMAX_SPLIT + blockIdx.y] = make_float2(best, __int_as_float(bi));
}

static __global__ void __launch_bounds__(ARGMAX_SPLIT) argmax_final_kernel(const float2* __restrict__ part,
                                                                           int* __restrict__ tokens) {
    pdl_wait();
    pdl_trigger();
    const float2 p = part[blockIdx.x * ARGMAX_SPLIT + threadIdx.x];
    float best = p.x;
    int bi = __float_as_int(p.y);
    argmax_block(best, bi);
    if (threadIdx.x == 0) tokens[blockIdx.x] = bi;
}

}  // namespace pf
}  // namespace mq
