// Batched decode (B independent sequences, one token each per step) for
// sm_100a: the weights are streamed once per step for all B tokens through
// the small-batch tcgen05 GEMM (gemm_tc_small_kernel: weights on the MMA's
// 128-row side, tokens on its N side, split-K with fp32 red.add); attention is
// split-K over each sequence's own cache length; norms, RoPE, SiLU and argmax
// are the prefill kernels.  No host synchronisation inside a step.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "gemm_small.cuh"
#include "megaqwen_b200.h"
#include "prefill_kernels.cuh"
#include "attn_fa.cuh"

namespace mq {

bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows);
int note_cuda(cudaError_t e, const char* what);

namespace db {

typedef __nv_bfloat16 bf16;
constexpr int D = MQ_HEAD_DIM;
constexpr int ATT_CHUNK_MIN = 256;   // cache positions per attention work unit: 256, 512 or 1024 per step
constexpr int PART = 132;            // floats per (unit, head): m, l, pad, pad, acc[128]

__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

// Output dimension held by accumulator row g of 8x8 block (u, r) after the
// in-register transpose of a 16-byte-per-lane row load (lane t loads dims
// 32u + 8t .. 32u + 8t + 7, register r holds the pair 32u + 8t + 2r).
__device__ __forceinline__ int vdim(int u, int r, int g) { return 32 * u + 8 * (g >> 1) + 2 * r + (g & 1); }

// One unit = (chunk c, kv head h, sequence b), 4 warps: both q heads of kv
// head h against cache positions [c*chunk, min(L, c*chunk+chunk)), L = pos[b] + 1
// (the row at pos[b] was written by this step's QK-norm/RoPE kernel).  Warp w
// takes the 16-position groups w, w+4, .. of the chunk.
//
// No shared-memory staging: each lane loads 16-byte pieces of K and V rows
// straight into registers.  S^T = K Q^T runs on mma.sync m16n8k16 with 16
// positions as the M side and the q heads as N (heads 0/1 real, the others
// zero); the summation order over head dims is permuted consistently in Q and
// K so the 16-byte pieces are the A fragments as loaded.  O^T = V^T P^T takes
// V^T and P^T from movmatrix transposes of the loaded V rows and of the
// exponentiated scores.  Online softmax in the log2 domain (q pre-scaled by
// scale * log2 e); the four warps merge through shared memory and the unit
// writes its (max, sum, unnormalised acc) per q head.
__global__ void __launch_bounds__(128, 4) attn_unit_kernel(const float* __restrict__ Qf, const bf16* __restrict__ kc,
                                                        const bf16* __restrict__ vc, const int* __restrict__ pos,
                                                        long long seq_stride, int max_seq, int C, float scale_log2,
                                                        int chunk, float* __restrict__ part,
                                                        int* __restrict__ counters, bf16* __restrict__ out) {
    __shared__ float sm_ml[4][4];
    __shared__ float sm_acc[4][2][D];
    __shared__ int s_last;
    pdl_wait();
    pdl_trigger();
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int L = pos[b] + 1, p0 = c * chunk;
    float* pp = part + (((size_t)b * 8 + h) * C + c) * 2 * PART;
    if (p0 >= L) {
        if (threadIdx.x < 2) {
            pp[threadIdx.x * PART] = -INFINITY;
            pp[threadIdx.x * PART + 1] = 0.f;
        }
        return;
    }
    const int n = min(chunk, L - p0);
    const int ngroups = (n + 15) >> 4;
    const bf16* kb = kc + b * seq_stride + ((size_t)h * max_seq + p0) * D;
    const bf16* vb = vc + b * seq_stride + ((size_t)h * max_seq + p0) * D;

    // B fragments of Q^T: lane (g, t), g < 2 = q head 2h+g; k-step (u, half)
    uint32_t qb[4][2][2];
    {
        const float* q = Qf + (size_t)b * 2048 + (2 * h + (g & 1)) * D;
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int d0 = 32 * u + 8 * t + 4 * hf;
                if (g < 2) {
                    qb[u][hf][0] = pf::pack_bf16(q[d0] * scale_log2, q[d0 + 1] * scale_log2);
                    qb[u][hf][1] = pf::pack_bf16(q[d0 + 2] * scale_log2, q[d0 + 3] * scale_log2);
                } else {
                    qb[u][hf][0] = qb[u][hf][1] = 0u;
                }
            }
    }
    float oacc[4][2][4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) oacc[u][qq][0] = oacc[u][qq][1] = oacc[u][qq][2] = oacc[u][qq][3] = 0.f;
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};

    uint4 kr[2][4], vr[2][4];
    auto load = [&](int grp, uint4 (&k)[2][4], uint4 (&v)[2][4]) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int row = 16 * grp + 8 * hr + g;
            const bool ok = row < n;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const size_t off = (size_t)row * D + 32 * u + 8 * t;
                k[hr][u] = ok ? *reinterpret_cast<const uint4*>(kb + off) : make_uint4(0, 0, 0, 0);
                v[hr][u] = ok ? *reinterpret_cast<const uint4*>(vb + off) : make_uint4(0, 0, 0, 0);
            }
        }
    };
    // Each warp loads one 16-position group at a time straight into registers;
    // the latency is covered by the other resident warps (4+ CTAs per SM at
    // <= 128 registers) rather than by a second register buffer.
    // L2 prefetch of this warp's K/V rows two groups ahead (one bulk prefetch per
    // matrix and group, issued by lane 0), so the register loads hit L2
    auto prefetch = [&](int grp) {
        if (lane == 0 && grp < ngroups) {
            const int r0 = 16 * grp, rows = min(16, n - r0);
            bulk_prefetch_l2(kb + (size_t)r0 * D, (uint32_t)(rows * D * 2));
            bulk_prefetch_l2(vb + (size_t)r0 * D, (uint32_t)(rows * D * 2));
        }
    };
    prefetch(warp);
    prefetch(warp + 4);
    for (int grp = warp; grp < ngroups; grp += 4) {
        prefetch(grp + 8);
        load(grp, kr, vr);
        // S^T[16 positions][8 heads]
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t r0[4] = {kr[0][u].x, kr[0][u].y, kr[0][u].z, kr[0][u].w};
            const uint32_t r1[4] = {kr[1][u].x, kr[1][u].y, kr[1][u].z, kr[1][u].w};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const uint32_t a[4] = {r0[2 * hf], r1[2 * hf], r0[2 * hf + 1], r1[2 * hf + 1]};
                pf::mma_bf16(s, a, qb[u][hf][0], qb[u][hf][1]);
            }
        }
        // s[0], s[1]: position g, heads 2t, 2t+1; s[2], s[3]: position g + 8
        const int pa = 16 * grp + g, pb = pa + 8;
        if (pa >= n) s[0] = s[1] = -INFINITY;
        if (pb >= n) s[2] = s[3] = -INFINITY;
        float mx[2] = {fmaxf(s[0], s[2]), fmaxf(s[1], s[3])};
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o));
            mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o));
        }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float mn = fmaxf(mrun[r], mx[r]);
            corr[r] = exp2f(mrun[r] - mn);
            mrun[r] = mn;
            lrun[r] *= corr[r];
        }
        const float e0 = exp2f(s[0] - mrun[0]), e1 = exp2f(s[1] - mrun[1]);
        const float e2 = exp2f(s[2] - mrun[0]), e3 = exp2f(s[3] - mrun[1]);
        lrun[0] += e0 + e2;
        lrun[1] += e1 + e3;
        // P^T as the B operand (k = position, n = head): transposes of the score blocks
        const uint32_t pb0 = movm_t(pf::pack_bf16(e0, e1));
        const uint32_t pb1 = movm_t(pf::pack_bf16(e2, e3));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t r0[4] = {vr[0][u].x, vr[0][u].y, vr[0][u].z, vr[0][u].w};
            const uint32_t r1[4] = {vr[1][u].x, vr[1][u].y, vr[1][u].z, vr[1][u].w};
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                float* o = oacc[u][qq];
                o[0] *= corr[0]; o[1] *= corr[1]; o[2] *= corr[0]; o[3] *= corr[1];
                const uint32_t a[4] = {movm_t(r0[qq]), movm_t(r0[qq + 2]), movm_t(r1[qq]), movm_t(r1[qq + 2])};
                pf::mma_bf16(o, a, pb0, pb1);
            }
        }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        lrun[0] += __shfl_xor_sync(0xffffffffu, lrun[0], o);
        lrun[1] += __shfl_xor_sync(0xffffffffu, lrun[1], o);
    }
    // lanes with t == 0 hold heads 0/1: c0/c1 at dim row g, c2/c3 at dim row g + 8
    if (t == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const int d0 = vdim(u, qq, g), d1 = vdim(u, qq + 2, g);
                sm_acc[warp][0][d0] = oacc[u][qq][0];
                sm_acc[warp][1][d0] = oacc[u][qq][1];
                sm_acc[warp][0][d1] = oacc[u][qq][2];
                sm_acc[warp][1][d1] = oacc[u][qq][3];
            }
        if (lane == 0) {
            sm_ml[warp][0] = mrun[0];
            sm_ml[warp][1] = mrun[1];
            sm_ml[warp][2] = lrun[0];
            sm_ml[warp][3] = lrun[1];
        }
    }
    __syncthreads();
    const int d = threadIdx.x;
    const int nact = (L + chunk - 1) / chunk;   // chunks holding positions of this sequence
    bf16* o = out + (size_t)b * 2048 + (2 * h) * D + d;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w][r]);
        float A = 0.f, Ls = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (sm_ml[w][r] == -INFINITY) continue;   // warp saw no positions
            const float e = exp2f(sm_ml[w][r] - M);
            A += sm_acc[w][r][d] * e;
            Ls += sm_ml[w][2 + r] * e;
        }
        if (nact == 1) {
            o[r * D] = __float2bfloat16(A / Ls);
        } else {
            pp[r * PART + 4 + d] = A;
            if (d == 0) {
                pp[r * PART] = M;
                pp[r * PART + 1] = Ls;
            }
        }
    }
    if (nact == 1) return;
    // the last unit of (sequence, kv head) to finish merges all chunks
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(counters + b * 8 + h, 1) == nact - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) counters[b * 8 + h] = 0;   // ready for the next layer
    const float* base = part + (((size_t)b * 8 + h) * C) * 2 * PART;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float M = -INFINITY;
        for (int cc = 0; cc < nact; ++cc) M = fmaxf(M, __ldcg(base + (size_t)cc * 2 * PART + r * PART));
        float A = 0.f, Ls = 0.f;
        for (int cc = 0; cc < nact; ++cc) {
            const float* q = base + (size_t)cc * 2 * PART + r * PART;
            const float e = exp2f(__ldcg(q) - M);
            Ls += __ldcg(q + 1) * e;
            A += __ldcg(q + 4 + d) * e;
        }
        o[r * D] = __float2bfloat16(A / Ls);
    }
}

// X[b] = embed[tokens[b]] (fp32), the first GEMM operand Xw[b] = bf16(X[b] * w)
// (w = layer 0's input RMSNorm weight; the 1/rms scale is applied in the GEMM
// epilogue) and the per-128-column sums of squares of X[b]; clears the LM
// head's argmax keys and the attention merge counters of this step.
__global__ void embed_step_kernel(const int* __restrict__ tokens, const bf16* __restrict__ embed,
                                  const bf16* __restrict__ w, float* __restrict__ X, bf16* __restrict__ Xw,
                                  float* __restrict__ ss, unsigned long long* __restrict__ best,
                                  int* __restrict__ counters, int B) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    if (lane == 0) best[b] = 0ull;
    if (lane < 8) counters[b * 8 + lane] = 0;
    const bf16* row = embed + (size_t)tokens[b] * MQ_HIDDEN_SIZE;
    float* out = X + (size_t)b * MQ_HIDDEN_SIZE;
    bf16* xw = Xw + (size_t)b * MQ_HIDDEN_SIZE;
#pragma unroll
    for (int i = 0; i < MQ_HIDDEN_SIZE / 256; ++i) {
        const int c = (lane + 32 * i) * 8;   // lanes 0-15 cover tile 2i, lanes 16-31 tile 2i+1
        const uint4 e = *reinterpret_cast<const uint4*>(row + c);
        const uint4 wq = *reinterpret_cast<const uint4*>(w + c);
        const float v[8] = {bf16lo(e.x), bf16hi(e.x), bf16lo(e.y), bf16hi(e.y),
                            bf16lo(e.z), bf16hi(e.z), bf16lo(e.w), bf16hi(e.w)};
        const float wf[8] = {bf16lo(wq.x), bf16hi(wq.x), bf16lo(wq.y), bf16hi(wq.y),
                             bf16lo(wq.z), bf16hi(wq.z), bf16lo(wq.w), bf16hi(wq.w)};
        *reinterpret_cast<float4*>(out + c) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(out + c + 4) = make_float4(v[4], v[5], v[6], v[7]);
        uint32_t pk[4];
        float sq = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * k] * wf[2 * k], v[2 * k + 1] * wf[2 * k + 1]);
            pk[k] = *reinterpret_cast<uint32_t*>(&t);
            sq += v[2 * k] * v[2 * k] + v[2 * k + 1] * v[2 * k + 1];
        }
        *reinterpret_cast<uint4*>(xw + c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if ((lane & 15) == 0) ss[b * 8 + 2 * i + (lane >> 4)] = sq;
    }
}

// tokens[b] = argmax from the LM head's 64-bit keys (value key << 32 | ~index); positions[b] += 1.
__global__ void finish_step_kernel(const unsigned long long* __restrict__ best, int* __restrict__ tokens,
                                   int* __restrict__ pos, int B) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    tokens[b] = (int)(0xffffffffu - (uint32_t)(best[b] & 0xffffffffull));
    pos[b] += 1;
}

// Every kernel of a step is launched as a programmatic dependent of the
// previous one; each begins with pdl_wait, so stream order still holds.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ((KArgs)args)...);
}

struct Layout {
    size_t X, Xw, ss, Qf, part, cnt, attn, act, best, total;
};

int np_of(int B) { return B <= 16 ? 16 : B <= 32 ? 32 : B <= 64 ? 64 : 128; }

Layout layout(int B, int max_seq) {
    const size_t NP = (size_t)np_of(B);
    const int C = (max_seq + ATT_CHUNK_MIN - 1) / ATT_CHUNK_MIN;
    Layout L;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o += (bytes + 1023) & ~size_t(1023); return r; };
    L.X = take((size_t)B * 1024 * 4);
    L.Xw = take(NP * 1024 * 2);
    L.ss = take((size_t)B * 8 * 4);
    L.Qf = take((size_t)B * 2048 * 4);
    L.part = take((size_t)B * 8 * C * 2 * PART * 4);
    L.cnt = take((size_t)B * 8 * 4);
    L.attn = take(NP * 2048 * 2);
    L.act = take(NP * 3072 * 2);
    L.best = take((size_t)B * 8);
    L.total = o;
    return L;
}

unsigned long long* g_trace = nullptr;
int g_launches = 0;   // small GEMM launches so far (all modes), for MQ_SMALL_TRACE

// Deepest ring that fits the 227 KB shared-memory limit of a CTA.
template <typename Cfg>
constexpr int fit_stages() {
    int s = Cfg::MAX_STAGES;
    while (s > 1 && Cfg::smem_bytes(s) > 232448) --s;
    return s;
}

// One small-batch GEMM launch (gemm_small_kernel): up to three weight maps of
// Nmap[i] rows x K (SM_STORE side by side; SM_SILU: gate, up).  The K split S
// (the cluster size, <= 8) targets about one CTA per SM.
// Cluster size (K split) and ring depth per GEMM shape, chosen once per
// device from the occupancy calculator: the largest split whose clusters all
// fit in one wave, up to about two CTAs per SM.
struct SplitChoice {
    int dev, mode, np, total, kblocks;
    int S, kpb, stages;
};
std::mutex g_split_mu;
std::vector<SplitChoice> g_splits;

template <int NPV, int MODE>
int launch_small(int total, int kblocks, Small2Args a, const CUtensorMap* tw, const CUtensorMap& tx, cudaStream_t st) {
    using Cfg = Small2Cfg<NPV, MODE>;
    auto kernel = gemm_small_kernel<NPV, MODE>;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = MODE == SM_ARGMAX ? 1 : 2;

    SplitChoice ch = {dev, MODE, NPV, total, kblocks, 1, kblocks, std::min(kblocks, 4)};
    bool found = false;
    {
        std::lock_guard<std::mutex> lk(g_split_mu);
        for (const SplitChoice& c : g_splits)
            if (c.dev == dev && c.mode == MODE && c.np == NPV && c.total == total && c.kblocks == kblocks) {
                ch = c;
                found = true;
                break;
            }
    }
    if (!found) {
        cudaError_t ea = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              Cfg::smem_bytes(fit_stages<Cfg>()));
        if (ea != cudaSuccess) return note_cuda(ea, "small gemm smem attribute");
        if (MODE != SM_ARGMAX) {
            ea = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            const int cands[] = {16, 12, 8, 6, 4, 3, 2, 1};
            for (int S : cands) {
                if (S > kblocks || (ea != cudaSuccess && S > 8)) continue;
                const int kpb = (kblocks + S - 1) / S;
                if ((kblocks + kpb - 1) / kpb != S || total * S > 320) continue;
                const int stages = std::min(kpb, fit_stages<Cfg>());
                cfg.gridDim = dim3(total, 1, S);
                cfg.dynamicSmemBytes = (size_t)Cfg::smem_bytes(stages);
                attr[1].val.clusterDim.z = S;
                int nclusters = 0;
                if (cudaOccupancyMaxActiveClusters(&nclusters, kernel, &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    continue;
                }
#if MQ_PROFILE_HOOKS
                if (getenv("MQ_SPLIT_VERBOSE"))
                    fprintf(stderr, "  mode %d NP %d tiles %d: S %d smem %d -> %d clusters\n", MODE, NPV, total, S,
                            (int)cfg.dynamicSmemBytes, nclusters);
#endif
                if (nclusters >= total || S == 1) {
                    ch.S = S;
                    ch.kpb = kpb;
                    ch.stages = stages;
                    break;
                }
            }
        }
#if MQ_PROFILE_HOOKS
        if (getenv("MQ_SPLIT_VERBOSE"))
            fprintf(stderr, "small gemm mode %d NP %d tiles %d kblocks %d -> S %d kpb %d stages %d\n", MODE, NPV,
                    total, kblocks, ch.S, ch.kpb, ch.stages);
#endif
        std::lock_guard<std::mutex> lk(g_split_mu);
        g_splits.push_back(ch);
    }
    a.kpb = ch.kpb;
    a.stages = ch.stages;
    cfg.gridDim = dim3(total, 1, ch.S);
    cfg.dynamicSmemBytes = (size_t)Cfg::smem_bytes(ch.stages);
    attr[1].val.clusterDim.z = ch.S;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tw[0], tw[1], tw[2], tx, a);
    return e == cudaSuccess ? MQ_OK : note_cuda(e, "small gemm launch");
}

// One small-batch GEMM (gemm_small_kernel): up to three weight maps of
// Nmap[i] rows x K (side by side for SM_QKV / SM_STORE; gate, up for SM_SILU).
template <int MODE>
int small_gemm(const void* const* W, const int* Nmap, int nmaps, int K, const void* X, int NP, const Small2Args& base,
               cudaStream_t st) {
    CUtensorMap tw[3], tx;
    int tiles[3] = {0, 0, 0}, cols[3] = {0, 0, 0}, total = 0;
    for (int i = 0; i < 3; ++i) {
        const int m = i < nmaps ? i : nmaps - 1;
        if (!make_tmap(&tw[i], W[m], (uint64_t)Nmap[m], (uint64_t)K, (uint64_t)K, GEMM_BM)) return MQ_ERR_CUDA;
        if (i < nmaps) {
            tiles[i] = Nmap[i] / GEMM_BM;
            cols[i] = total * GEMM_BM;
            total += tiles[i];
        }
    }
    if (MODE == SM_SILU) total = tiles[0];   // gate tile t and up tile t share a CTA
    if (!make_tmap(&tx, X, (uint64_t)NP, (uint64_t)K, (uint64_t)K, (uint32_t)NP)) return MQ_ERR_CUDA;
    Small2Args a = base;
    a.tiles0 = tiles[0];
    a.tiles1 = tiles[1];
    a.col1 = cols[1];
    a.col2 = cols[2];
    a.K = K;
    a.timeout_cycles = 4000000000ll;
    a.trace = nullptr;
#if MQ_PROFILE_HOOKS
    {
        // phase-timing hook: MQ_SMALL_TRACE=<n> stamps the n-th small GEMM launch of the process
        static const int trace_at = [] { const char* e = getenv("MQ_SMALL_TRACE"); return e ? atoi(e) : -1; }();
        if (trace_at >= 0 && g_launches++ == trace_at) {
            if (!g_trace) cudaMalloc(&g_trace, 8 * 4096 * sizeof(unsigned long long));
            cudaMemsetAsync(g_trace, 0, 8 * 4096 * sizeof(unsigned long long), st);
            a.trace = g_trace;
        }
    }
#endif
    const int kblocks = K / GEMM_BK;
    switch (NP) {
        case 16: return launch_small<16, MODE>(total, kblocks, a, tw, tx, st);
        case 32: return launch_small<32, MODE>(total, kblocks, a, tw, tx, st);
        case 64: return launch_small<64, MODE>(total, kblocks, a, tw, tx, st);
        case 128: return launch_small<128, MODE>(total, kblocks, a, tw, tx, st);
        default: return MQ_ERR_INVALID_ARGUMENT;
    }
}

}  // namespace db

int decode_batch(const mq_decode_batch_params* p, cudaStream_t st) {
    using namespace db;
    if (!p || !p->tokens || !p->positions || !p->embed || !p->layers_host || !p->final_norm || !p->lm_head ||
        !p->cos_table || !p->sin_table || !p->k_cache || !p->v_cache || !p->workspace || !p->err_flag)
        return MQ_ERR_INVALID_ARGUMENT;
    const int B = p->batch;
    if (B < 1 || B > 128 || p->num_layers < 1 || p->num_layers > MQ_MAX_LAYERS || p->max_seq_len < 1)
        return MQ_ERR_INVALID_ARGUMENT;
    const Layout L = layout(B, p->max_seq_len);
    if (p->workspace_bytes < L.total) return MQ_ERR_WORKSPACE;
    uint8_t* ws = (uint8_t*)p->workspace;
    float* X = (float*)(ws + L.X);
    bf16* Xw = (bf16*)(ws + L.Xw);
    float* ss = (float*)(ws + L.ss);
    float* Qf = (float*)(ws + L.Qf);
    float* part = (float*)(ws + L.part);
    bf16* attn = (bf16*)(ws + L.attn);
    bf16* act = (bf16*)(ws + L.act);
    unsigned long long* best = (unsigned long long*)(ws + L.best);
    const int NP = np_of(B);
    // the largest unit (256 / 512 / 1024 positions) that still gives >= 512 units over the
    // (bucketed, up to 2x) context: long units amortise a unit's start-up and merge,
    // enough of them keep every SM busy
    int chunk = 1024;
    while (chunk > ATT_CHUNK_MIN && (long long)B * 8 * ((p->max_context + chunk - 1) / chunk) < 512) chunk >>= 1;
    const int C = (p->max_context + chunk - 1) / chunk;
    if (C < 1 || p->max_context > p->max_seq_len) return MQ_ERR_INVALID_ARGUMENT;
    const int norm_blocks = (B + 7) / 8;
    cudaError_t e = cudaSuccess;
    auto ok = [&](cudaError_t r) { if (r != cudaSuccess && e == cudaSuccess) e = r; };
    Small2Args ga = {};
    ga.Bv = B;
    ga.err = p->err_flag;

    int* counters = (int*)(ws + L.cnt);
    ok(launch(embed_step_kernel, dim3(norm_blocks), dim3(256), 0, st, (const int*)p->tokens, (const bf16*)p->embed,
              (const bf16*)p->layers_host[0].input_layernorm_weight, X, Xw, ss, best, counters, B));
    for (int l = 0; l < p->num_layers; ++l) {
        const LDGLayerWeights& W = p->layers_host[l];
        const void* wqkv[3] = {W.q_proj_weight, W.k_proj_weight, W.v_proj_weight};
        const int nqkv[3] = {2048, 1024, 1024};
        Small2Args a = ga;
        a.ss_in = ss;
        const size_t layer_off = (size_t)l * MQ_NUM_KV_HEADS * p->max_seq_len * D;
        bf16* kc_l = (bf16*)p->k_cache + layer_off;
        bf16* vc_l = (bf16*)p->v_cache + layer_off;
        a.qkv.q_norm = (const bf16*)W.q_norm_weight;
        a.qkv.k_norm = (const bf16*)W.k_norm_weight;
        a.qkv.cos_table = (const bf16*)p->cos_table;
        a.qkv.sin_table = (const bf16*)p->sin_table;
        a.qkv.pos = p->positions;
        a.qkv.Qf = Qf;
        a.qkv.k_cache = kc_l;
        a.qkv.v_cache = vc_l;
        a.qkv.seq_stride = p->cache_seq_stride;
        a.qkv.max_seq = p->max_seq_len;
        int rc = small_gemm<SM_QKV>(wqkv, nqkv, 3, 1024, Xw, NP, a, st);
        if (rc) return rc;
        ok(launch(attn_unit_kernel, dim3(C, 8, B), dim3(128), 0, st, (const float*)Qf, (const bf16*)kc_l,
                  (const bf16*)vc_l, (const int*)p->positions, p->cache_seq_stride, p->max_seq_len, C,
                  p->attn_scale * 1.4426950408889634f, chunk, part, counters, attn));
        const void* wo[1] = {W.o_proj_weight};
        const int no[1] = {1024};
        a = ga;
        a.out = X;
        a.ldo = 1024;
        a.w_next = (const bf16*)W.post_attn_layernorm_weight;
        a.xw_out = Xw;
        a.ss_out = ss;
        rc = small_gemm<SM_RESID>(wo, no, 1, 2048, attn, NP, a, st);
        if (rc) return rc;
        const void* wgu[2] = {W.gate_proj_weight, W.up_proj_weight};
        const int ngu[2] = {3072, 3072};
        a = ga;
        a.act = act;
        a.ldo = 3072;
        a.ss_in = ss;
        rc = small_gemm<SM_SILU>(wgu, ngu, 2, 1024, Xw, NP, a, st);
        if (rc) return rc;
        const void* wd[1] = {W.down_proj_weight};
        const int nd[1] = {1024};
        a = ga;
        a.out = X;
        a.ldo = 1024;
        a.w_next = (const bf16*)(l + 1 < p->num_layers ? p->layers_host[l + 1].input_layernorm_weight : p->final_norm);
        a.xw_out = Xw;
        a.ss_out = ss;
        rc = small_gemm<SM_RESID>(wd, nd, 1, 3072, act, NP, a, st);
        if (rc) return rc;
    }
    const void* wl[1] = {p->lm_head};
    const int nl[1] = {MQ_VOCAB_SIZE};
    Small2Args a = ga;
    a.out = p->logits;
    a.ldo = MQ_VOCAB_SIZE;
    a.best = best;
    a.ss_in = ss;
    int rc = small_gemm<SM_ARGMAX>(wl, nl, 1, 1024, Xw, NP, a, st);
    if (rc) return rc;
    ok(launch(finish_step_kernel, dim3((B + 127) / 128), dim3(128), 0, st, (const unsigned long long*)best, p->tokens,
              p->positions, B));
    if (e != cudaSuccess) return note_cuda(e, "batch decode launch");
    e = cudaGetLastError();
    return e == cudaSuccess ? MQ_OK : note_cuda(e, "batch decode");
}

size_t decode_batch_workspace_bytes(int batch, int max_seq_len) { return db::layout(batch, max_seq_len).total; }

namespace db {
// tokens[b] from the LM head's 64-bit keys (value key << 32 | ~index).
__global__ void tokens_from_keys_kernel(const unsigned long long* __restrict__ best, int* __restrict__ tokens, int B) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) tokens[b] = (int)(0xffffffffu - (uint32_t)(best[b] & 0xffffffffull));
}
}  // namespace db

// Tied LM head and greedy argmax of B <= 128 already-normalized rows (the
// prefill's last positions): x is bf16 [lm_head_rows(B), 1024], rows past B
// allocated but unused; logits (fp32 [B, vocab]) are written only if non-null;
// best is B 64-bit words of scratch.  The small-batch GEMM streams the
// embedding once with the (value, lowest index) maximum fused into its epilogue.
int lm_head_rows(int B) { return db::np_of(B); }
int lm_head_argmax(const void* lm_head, const void* x, int B, float* logits, unsigned long long* best, int* tokens,
                   int* err, cudaStream_t st) {
    using namespace db;
    if (B < 1 || B > 128) return MQ_ERR_INVALID_ARGUMENT;
    if (cudaMemsetAsync(best, 0, (size_t)B * sizeof(unsigned long long), st) != cudaSuccess) return MQ_ERR_CUDA;
    const void* wl[1] = {lm_head};
    const int nl[1] = {MQ_VOCAB_SIZE};
    Small2Args a = {};
    a.Bv = B;
    a.err = err;
    a.out = logits;
    a.ldo = MQ_VOCAB_SIZE;
    a.best = best;
    a.ss_in = nullptr;
    const int rc = small_gemm<SM_ARGMAX>(wl, nl, 1, 1024, x, np_of(B), a, st);
    if (rc) return rc;
    const cudaError_t e = launch(tokens_from_keys_kernel, dim3(1), dim3(128), 0, st, (const unsigned long long*)best,
                                 tokens, B);
    return e == cudaSuccess ? MQ_OK : note_cuda(e, "lm head argmax");
}

}  // namespace mq

extern "C" {

size_t mq_decode_batch_workspace_bytes(int batch, int max_seq_len) {
    return mq::decode_batch_workspace_bytes(batch, max_seq_len);
}

#if MQ_PROFILE_HOOKS
// Copies the phase stamps of the traced small GEMM launch (MQ_SMALL_TRACE) to host.
int mq_debug_small_trace(unsigned long long* host, int n) {
    if (!mq::db::g_trace) return 0;
    cudaMemcpy(host, mq::db::g_trace, (size_t)n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    return n;
}
#endif

int mq_decode_batch(const mq_decode_batch_params* params, cudaStream_t stream) {
    return mq::decode_batch(params, stream);
}

}  // extern "C"
