// Prefill kernels around the tcgen05 GEMM: embedding gather, RMSNorm to bf16,
// QK-norm + RoPE + K/V cache write, causal GQA flash attention on the tensor
// cores (mma.sync m16n8k16 bf16 -> fp32), and argmax.
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

// Per token: q/k heads RMSNorm (head_dim) x norm weight, rotate-half RoPE at
// position start_pos + s; Q, K, V to bf16 operands; K, V rows into the bf16
// cache [L, 8, max_seq, 128] of sequence b (layer offset folded into the
// pointers).  One block of 32 warps per token: warps 0-15 q heads, 16-23 k
// heads, 24-31 v heads; lane owns dims lane + 32j (rotate-half pairs in-lane).
struct QkvArgs {
    const float* qkv;        // [M, 4096] fp32: q | k | v
    const bf16* q_norm;
    const bf16* k_norm;
    const bf16* cos_table;   // [max_seq, 128]
    const bf16* sin_table;
    bf16* Qb;                // [M, 2048]
    bf16* Kb;                // [M, 1024]
    bf16* Vb;                // [M, 1024]
    bf16* k_cache;           // layer base of sequence 0
    bf16* v_cache;
    long long cache_seq_stride;  // elements between sequences' caches
    int S, start_pos, max_seq_len;
    const int* pos_dev;      // optional: position of sequence b is pos_dev[b] (batched decode, S == 1)
    float* Qf;               // optional: fp32 q [M, 2048] instead of bf16 Qb
};

static __global__ void __launch_bounds__(1024) qknorm_rope_kernel(const QkvArgs a) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = m / a.S, p = a.pos_dev ? a.pos_dev[b] : a.start_pos + (m - b * a.S);
    const float* row = a.qkv + (size_t)m * 4096;
    float e[4];
    if (warp < NQ + NKV) {
        const bool isq = warp < NQ;
        const float* x = row + (isq ? warp * D : 2048 + (warp - NQ) * D);
        const bf16* nw = isq ? a.q_norm : a.k_norm;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) { e[j] = x[lane + 32 * j]; ss += e[j] * e[j]; }
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / (float)D + 1e-6f);
#pragma unroll
        for (int j = 0; j < 4; ++j) e[j] = e[j] * r * __bfloat162float(nw[lane + 32 * j]);
        const bf16* cs = a.cos_table + (size_t)p * D;
        const bf16* sn = a.sin_table + (size_t)p * D;
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = lane + 32 * j;
            const float c = __bfloat162float(cs[i]), s = __bfloat162float(sn[i]);
            o[j] = (j < 2) ? (e[j] * c - e[j + 2] * s) : (e[j] * c + e[j - 2] * s);
        }
        if (isq && a.Qf) {
#pragma unroll
            for (int j = 0; j < 4; ++j) a.Qf[(size_t)m * 2048 + warp * D + lane + 32 * j] = o[j];
        } else if (isq) {
#pragma unroll
            for (int j = 0; j < 4; ++j) a.Qb[(size_t)m * 2048 + warp * D + lane + 32 * j] = __float2bfloat16(o[j]);
        } else {
            const int kh = warp - NQ;
            bf16* kc = a.k_cache + b * a.cache_seq_stride + ((size_t)kh * a.max_seq_len + p) * D;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bf16 v = __float2bfloat16(o[j]);
                a.Kb[(size_t)m * 1024 + kh * D + lane + 32 * j] = v;
                kc[lane + 32 * j] = v;
            }
        }
    } else {
        const int vh = warp - NQ - NKV;
        const float* x = row + 3072 + vh * D;
        bf16* vc = a.v_cache + b * a.cache_seq_stride + ((size_t)vh * a.max_seq_len + p) * D;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const bf16 v = __float2bfloat16(x[lane + 32 * j]);
            a.Vb[(size_t)m * 1024 + vh * D + lane + 32 * j] = v;
            vc[lane + 32 * j] = v;
        }
    }
}

// tokens[r] = lowest index of the maximum of logits[r, :V]; logits_ld elements per row.
static __global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int V, int logits_ld,
                                                      int* __restrict__ tokens) {
    pdl_wait();
    pdl_trigger();
    const float* x = logits + (size_t)blockIdx.x * logits_ld;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = x[i];
        if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
        tokens[blockIdx.x] = bi;
    }
}

}  // namespace pf
}  // namespace mq
