// Prefill building blocks for sm_100a: the tcgen05 GEMM (gemm_tc.cuh) and its
// host-side launch (TMA tensor maps), plus the C-ABI entry mq_gemm_bf16.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "gemm_tc.cuh"
#include "gemm_persist.cuh"
#include "gemm_pair.cuh"
#include "megaqwen_b200.h"

namespace mq {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// K-major bf16 matrix [rows, cols] with row stride ld (elements); box 64 x 128,
// 128-byte swizzle (matches sw128_kmajor_desc).
}  // namespace

bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {GEMM_BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

int num_sms() {
    static int sms[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 148;
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    return sms[dev] > 0 ? sms[dev] : 148;
}

// Launch as a programmatic dependent of the previous kernel in the stream (the
// GEMMs and the attention call pdl_wait after their set-up: barrier init, TMEM
// allocation, tensor-map prefetch), so that set-up overlaps the previous tail.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// One persistent GEMM launch: A [M, K] against up to three B maps side by side
// (Nmap[i] rows each; EPI_SILU_MUL: gate, up), one CTA per SM, BN-wide tiles.
template <int EPI, int BN>
int launch_persist_bn(const void* A, int lda, const void* const* Bm, const int* Nmap, int nmaps, int ldb, void* C,
                      int ldc, int M, int K, const QkvPrefillEpi* qkv, int* err, cudaStream_t stream) {
    using Cfg = PCfg<EPI, BN>;
    static bool configured[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MQ_ERR_CUDA;
    if (dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(gemm_persist_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cfg::SMEM) != cudaSuccess)
            return MQ_ERR_CUDA;
        configured[dev] = true;
    }
    CUtensorMap ta, tb[3];
    if (!make_tmap(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, GEMM_BM)) return MQ_ERR_CUDA;
    for (int i = 0; i < 3; ++i) {
        const int m = i < nmaps ? i : nmaps - 1;
        if (!make_tmap(&tb[i], Bm[m], (uint64_t)Nmap[m], (uint64_t)K, (uint64_t)ldb, BN)) return MQ_ERR_CUDA;
    }
    PArgs a = {};
    a.C = C;
    a.ldc = ldc;
    a.M = M;
    a.K = K;
    a.tiles_m = (M + GEMM_BM - 1) / GEMM_BM;
    a.nb0 = Nmap[0] / BN;
    a.nb1 = nmaps > 1 ? Nmap[1] / BN : 0;
    a.tiles_n = EPI == EPI_SILU_MUL ? a.nb0 : a.nb0 + a.nb1 + (nmaps > 2 ? Nmap[2] / BN : 0);
    if (qkv) a.qkv = *qkv;
    a.err = err;
    a.timeout_cycles = 4000000000ll;  // ~2 s at 1.9 GHz
    const int ntiles = a.tiles_m * a.tiles_n;
    const int grid = ntiles < num_sms() ? ntiles : num_sms();
    const cudaError_t e = launch_pdl(gemm_persist_kernel<EPI, BN>, dim3(grid), dim3(P_THREADS), (size_t)Cfg::SMEM,
                                     stream, ta, tb[0], tb[1], tb[2], a);
    return e == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
}

// 256-wide tiles where every B map's rows allow them (gate/up keep 128: two accumulators)
template <int EPI>
int launch_persist(const void* A, int lda, const void* const* Bm, const int* Nmap, int nmaps, int ldb, void* C, int ldc,
                   int M, int K, const QkvPrefillEpi* qkv, int* err, cudaStream_t stream) {
    bool wide = EPI != EPI_SILU_MUL;
    int ncols = 0;
    for (int i = 0; i < nmaps; ++i) {
        wide = wide && Nmap[i] % 256 == 0;
        ncols += Nmap[i];
    }
    // only when the wide tiles still fill every SM at least once
    wide = wide && (long long)((M + GEMM_BM - 1) / GEMM_BM) * (ncols / 256) >= num_sms();
    if (EPI != EPI_SILU_MUL && wide)
        return launch_persist_bn<EPI, (EPI == EPI_SILU_MUL ? 128 : 256)>(A, lda, Bm, Nmap, nmaps, ldb, C, ldc, M, K,
                                                                         qkv, err, stream);
    return launch_persist_bn<EPI, 128>(A, lda, Bm, Nmap, nmaps, ldb, C, ldc, M, K, qkv, err, stream);
}

// The CTA-pair GEMM (gemm_pair.cuh) for EPI_ADD_F32 / EPI_SILU_MUL: 256-row
// pair tiles, launched as clusters of two, one pair per two SMs.
template <int EPI>
int launch_pair(const void* A, int lda, const void* B, const void* B2, int ldb, void* C, int ldc, int M, int N, int K,
                int* err, cudaStream_t stream) {
    static bool configured[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MQ_ERR_CUDA;
    if (dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM) !=
            cudaSuccess)
            return MQ_ERR_CUDA;
        configured[dev] = true;
    }
    CUtensorMap ta, tb0, tb1;
    if (!make_tmap(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, GEMM_BM) ||
        !make_tmap(&tb0, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 128) ||
        !make_tmap(&tb1, B2 ? B2 : B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 128))
        return MQ_ERR_CUDA;
    PArgs a = {};
    a.C = C;
    a.ldc = ldc;
    a.M = M;
    a.K = K;
    a.tiles_m = (M + 255) / 256;
    a.tiles_n = EPI == EPI_SILU_MUL ? N / 128 : N / 256;
    a.err = err;
    a.timeout_cycles = 4000000000ll;
    const int ntiles = a.tiles_m * a.tiles_n;
    const int pairs = std::min(ntiles, num_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = PAIR_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI>, ta, tb0, tb1, a);
    return e == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
}

// The pair GEMM serves the residual-add GEMMs once their 256 x 256 pair tiles
// fill every SM pair twice (B = 8 x 2048 prompts): 101.7 against 104.5 us per
// launch.  Gate/up stays on the one-CTA kernel, where the pair version measured
// 177 against 173 us (B = 8) and 33.5 against 32 us (B = 1).
bool use_pair(int epi, int M, int N) {
    if (epi == EPI_ADD_F32 && N % 256 == 0) return (long long)((M + 255) / 256) * (N / 256) >= num_sms();
    return false;
}

template <int EPI>
int launch_gemm(const void* A, int lda, const void* B, int ldb, const void* B2, void* C, int ldc, int M, int N,
                int K, int* err, cudaStream_t stream) {
    if ((EPI == EPI_ADD_F32 || EPI == EPI_SILU_MUL) && use_pair(EPI, M, N))
        return launch_pair<EPI == EPI_SILU_MUL ? EPI_SILU_MUL : EPI_ADD_F32>(A, lda, B, B2, ldb, C, ldc, M, N, K, err,
                                                                          stream);
    const void* Bm[2] = {B, B2 ? B2 : B};
    const int Nm[2] = {N, N};
    return launch_persist<EPI>(A, lda, Bm, Nm, EPI == EPI_SILU_MUL ? 2 : 1, ldb, C, ldc, M, K, nullptr, err, stream);
}

}  // namespace

int gemm_bf16(const void* A, int lda, const void* B, int ldb, const void* B2, void* C, int ldc, int M, int N, int K,
              int epi, int* err, cudaStream_t stream) {
    if (!A || !B || !C || !err || M < 1 || N < 1 || K < 1) return MQ_ERR_INVALID_ARGUMENT;
    if (N % GEMM_BN || K % GEMM_BK || lda % 8 || ldb % 8 || ldc % 8) return MQ_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & 15) return MQ_ERR_INVALID_ARGUMENT;
    switch (epi) {
        case EPI_STORE_F32: return launch_gemm<EPI_STORE_F32>(A, lda, B, ldb, B2, C, ldc, M, N, K, err, stream);
        case EPI_ADD_F32: return launch_gemm<EPI_ADD_F32>(A, lda, B, ldb, B2, C, ldc, M, N, K, err, stream);
        case EPI_SILU_MUL:
            if (!B2 || ((uintptr_t)B2 & 15)) return MQ_ERR_INVALID_ARGUMENT;
            return launch_gemm<EPI_SILU_MUL>(A, lda, B, ldb, B2, C, ldc, M, N, K, err, stream);
        case EPI_STORE_BF16: return launch_gemm<EPI_STORE_BF16>(A, lda, B, ldb, B2, C, ldc, M, N, K, err, stream);
        default: return MQ_ERR_INVALID_ARGUMENT;
    }
}

}  // namespace mq

extern "C" int mq_gemm_bf16(const void* A, int lda, const void* B, int ldb, const void* B2, void* C, int ldc, int M,
                            int N, int K, int epilogue, int* err_flag, cudaStream_t stream) {
    return mq::gemm_bf16(A, lda, B, ldb, B2, C, ldc, M, N, K, epilogue, err_flag, stream);
}

// =============================================================================
// Prefill forward (batched): the reference's launch_prefill_float
// (csrc/megakernel/fused_prefill.cu:601-867) on tcgen05 GEMMs.
// =============================================================================
#include "prefill_kernels.cuh"
#include "attn_fa.cuh"
#include "attn_tc.cuh"

namespace mq {
// LM head + argmax of the last positions (small-batch GEMM, decode_batch.cu)
int lm_head_rows(int B);
int lm_head_argmax(const void* lm_head, const void* x, int B, float* logits, unsigned long long* best, int* tokens,
                   int* err, cudaStream_t st);

namespace {

// An RMSNorm launch, as a programmatic dependent or plain.
template <typename... Args>
cudaError_t launch_norm(bool pdl, dim3 grid, cudaStream_t st, Args... args) {
    if (pdl) return launch_pdl(pf::rmsnorm_bf16_kernel, grid, dim3(256), 0, st, args...);
    pf::rmsnorm_bf16_kernel<<<grid, 256, 0, st>>>(args...);
    return cudaGetLastError();
}

unsigned long long* g_fa_trace = nullptr;

struct PrefillLayout {
    size_t X, Xn, Qb, Vt, Ob, act, lastn, logits, part, err, total;
};

PrefillLayout prefill_layout(int B, int S) {
    const size_t M = (size_t)B * S;
    PrefillLayout L;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o += (bytes + 255) & ~size_t(255); return r; };
    L.X = take(M * 1024 * 4);
    L.Xn = take(M * 1024 * 2);
    L.Qb = take(M * 2048 * 2);
    L.Vt = take((size_t)B * 8 * 128 * ((S + 7) / 8 * 8) * 2);   // V^T per (sequence, kv head), rows padded to 8
    L.Ob = take(M * 2048 * 2);
    L.act = take(M * 3072 * 2);
    L.lastn = take((size_t)(B > 128 ? B : lm_head_rows(B)) * 1024 * 2);   // LM-head operand rows (padded)
    L.logits = take((size_t)B * MQ_VOCAB_SIZE * 4);
    L.part = take((size_t)B * pf::ARGMAX_SPLIT * 8);
    L.err = take(256);
    L.total = o;
    return L;
}

#define MQ_TRY(x)                       \
    do {                                \
        int rc_ = (x);                  \
        if (rc_ != MQ_OK) return rc_;   \
    } while (0)

}  // namespace

int prefill_forward(const mq_prefill_params* p, cudaStream_t st) {
    if (!p || !p->ids || !p->embed || !p->layers_host || !p->final_norm || !p->lm_head || !p->cos_table ||
        !p->sin_table || !p->k_cache || !p->v_cache || !p->out_tokens || !p->workspace)
        return MQ_ERR_INVALID_ARGUMENT;
    const int B = p->batch, S = p->seq_len;
    if (B < 1 || S < 1 || p->num_layers < 1 || p->num_layers > MQ_MAX_LAYERS) return MQ_ERR_INVALID_ARGUMENT;
    if (p->start_pos != 0 || S > p->max_seq_len) return MQ_ERR_INVALID_ARGUMENT;
    const PrefillLayout L = prefill_layout(B, S);
    if (p->workspace_bytes < L.total) return MQ_ERR_WORKSPACE;
    uint8_t* ws = (uint8_t*)p->workspace;
    float* X = (float*)(ws + L.X);
    pf::bf16* Xn = (pf::bf16*)(ws + L.Xn);
    pf::bf16* Qb = (pf::bf16*)(ws + L.Qb);
    pf::bf16* Ob = (pf::bf16*)(ws + L.Ob);
    pf::bf16* act = (pf::bf16*)(ws + L.act);
    pf::bf16* lastn = (pf::bf16*)(ws + L.lastn);
    float* logits = p->logits ? p->logits : (float*)(ws + L.logits);
    int* err = p->err_flag ? p->err_flag : (int*)(ws + L.err);
    const int M = B * S;
    const float scale_log2 = p->attn_scale * 1.4426950408889634f;

    {
        static bool fa_configured[64] = {false};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return MQ_ERR_CUDA;
        if (!fa_configured[dev]) {
            if (cudaFuncSetAttribute(fa::fa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::SMEM) !=
                cudaSuccess)
                return MQ_ERR_CUDA;
            fa_configured[dev] = true;
        }
    }
    // attention operands: Q [M, 2048], K straight from the K cache (rows of 128 over all
    // sequences and layers) and V^T [B * 8 * 128, ldvt] (zero padding past S)
    pf::bf16* Vt = (pf::bf16*)(ws + L.Vt);
    const int ldvt = (S + 7) / 8 * 8;
    if (p->cache_seq_stride % MQ_HEAD_DIM != 0) return MQ_ERR_INVALID_ARGUMENT;
    const long long seq_rows = p->cache_seq_stride / MQ_HEAD_DIM;
    const long long head_rows = p->max_seq_len;
    const long long cache_rows = (long long)(B - 1) * seq_rows + (long long)p->num_layers * MQ_NUM_KV_HEADS * head_rows;
    CUtensorMap tmQ, tmK, tmV;
    if (!make_tmap(&tmQ, Qb, (uint64_t)M, 2048, 2048, fa::BQ) ||
        !make_tmap(&tmK, p->k_cache, (uint64_t)cache_rows, MQ_HEAD_DIM, MQ_HEAD_DIM, fa::BK) ||
        !make_tmap(&tmV, Vt, (uint64_t)B * 8 * 128, (uint64_t)ldvt, (uint64_t)ldvt, 128))
        return MQ_ERR_CUDA;
    if (ldvt != S && cudaMemsetAsync(Vt, 0, (size_t)B * 8 * 128 * ldvt * 2, st) != cudaSuccess) return MQ_ERR_CUDA;
    const bool norm_pdl = M <= 4096;   // B = 1 x 2048: 3.95 -> 3.93 ms as dependents
    pf::embed_kernel<<<(M + 7) / 8, 256, 0, st>>>(p->ids, (const pf::bf16*)p->embed, X, M);
    for (int l = 0; l < p->num_layers; ++l) {
        const LDGLayerWeights& W = p->layers_host[l];
        // the norms are programmatic dependents only for short prompts: for M = 16384
        // their blocks sat resident through the preceding GEMM and B = 8 was 3 % slower
        if (launch_norm(norm_pdl, dim3((M + 7) / 8), st, X, (const pf::bf16*)W.input_layernorm_weight, Xn, M, 1, 0) !=
            cudaSuccess)
            return MQ_ERR_CUDA;
        {
            // q | k | v projections with QK-norm, RoPE and the K/V cache write in the epilogue
            QkvPrefillEpi e;
            e.q_norm = (const pf::bf16*)W.q_norm_weight;
            e.k_norm = (const pf::bf16*)W.k_norm_weight;
            e.cos_table = (const pf::bf16*)p->cos_table;
            e.sin_table = (const pf::bf16*)p->sin_table;
            e.Qb = Qb;
            const size_t layer_off = (size_t)l * MQ_NUM_KV_HEADS * p->max_seq_len * MQ_HEAD_DIM;
            e.k_cache = (pf::bf16*)p->k_cache + layer_off;
            e.v_cache = (pf::bf16*)p->v_cache + layer_off;
            e.cache_seq_stride = p->cache_seq_stride;
            e.S = S;
            e.start_pos = 0;
            e.max_seq = p->max_seq_len;
            e.Vt = Vt;
            e.ldvt = ldvt;
            e.q_scale = scale_log2;
            const void* Bm[3] = {W.q_proj_weight, W.k_proj_weight, W.v_proj_weight};
            const int Nm[3] = {2048, 1024, 1024};
            MQ_TRY(launch_persist<EPI_QKV>(Xn, 1024, Bm, Nm, 3, 1024, nullptr, 0, M, 1024, &e, err, st));
        }
        {
            fa::Args fa_args;
            fa_args.O = Ob;
            fa_args.S = S;
            fa_args.B = B;
            fa_args.k_row0 = (long long)l * MQ_NUM_KV_HEADS * head_rows;
            fa_args.k_seq_rows = seq_rows;
            fa_args.k_head_rows = head_rows;
            fa_args.err = err;
            fa_args.timeout_cycles = 4000000000ll;
            fa_args.trace = nullptr;
#if MQ_PROFILE_HOOKS
            {
                // profiling hook: MQ_FA_TRACE=<layer> stamps one attention block of that layer
                static const int at = [] { const char* e = getenv("MQ_FA_TRACE"); return e ? atoi(e) : -1; }();
                if (at == l) {
                    if (!g_fa_trace) cudaMalloc(&g_fa_trace, 32 * 8 * sizeof(unsigned long long));
                    cudaMemsetAsync(g_fa_trace, 0, 32 * 8 * sizeof(unsigned long long), st);
                    fa_args.trace = g_fa_trace;
                }
            }
#endif
            // persistent: one CTA per SM over (q head, sequence, query block) items
            const int items = MQ_NUM_Q_HEADS * B * ((S + fa::BQ - 1) / fa::BQ);
            const int fgrid = items < num_sms() ? items : num_sms();
            if (launch_pdl(fa::fa_tc_kernel, dim3(fgrid), dim3(fa::THREADS), (size_t)fa::SMEM, st, tmQ, tmK, tmV,
                           fa_args) != cudaSuccess)
                return MQ_ERR_CUDA;
        }
        MQ_TRY(gemm_bf16(Ob, 2048, W.o_proj_weight, 2048, nullptr, X, 1024, M, 1024, 2048, EPI_ADD_F32, err, st));
        if (launch_norm(norm_pdl, dim3((M + 7) / 8), st, X, (const pf::bf16*)W.post_attn_layernorm_weight, Xn, M, 1,
                        0) != cudaSuccess)
            return MQ_ERR_CUDA;
        MQ_TRY(gemm_bf16(Xn, 1024, W.gate_proj_weight, 1024, W.up_proj_weight, act, 3072, M, 3072, 1024, EPI_SILU_MUL,
                         err, st));
        MQ_TRY(gemm_bf16(act, 3072, W.down_proj_weight, 3072, nullptr, X, 1024, M, 1024, 3072, EPI_ADD_F32, err, st));
    }
    // last position of each sequence: final norm, tied LM head, argmax
    if (launch_norm(norm_pdl, dim3((B + 7) / 8), st, X, (const pf::bf16*)p->final_norm, lastn, B, S, S - 1) !=
        cudaSuccess)
        return MQ_ERR_CUDA;
    if (B <= 128) {
        // small-batch GEMM with the argmax fused (streams the embedding at close to the HBM rate)
        MQ_TRY(lm_head_argmax(p->lm_head, lastn, B, p->logits, (unsigned long long*)(ws + L.part), p->out_tokens,
                              err, st));
        return cudaGetLastError() == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
    }
    MQ_TRY(gemm_bf16(lastn, 1024, p->lm_head, 1024, nullptr, logits, MQ_VOCAB_SIZE, B, MQ_VOCAB_SIZE, 1024,
                     EPI_STORE_F32, err, st));
    pf::argmax_part_kernel<<<dim3(B, pf::ARGMAX_SPLIT), 256, 0, st>>>(logits, MQ_VOCAB_SIZE, MQ_VOCAB_SIZE,
                                                                       (float2*)(ws + L.part));
    pf::argmax_final_kernel<<<B, pf::ARGMAX_SPLIT, 0, st>>>((const float2*)(ws + L.part), p->out_tokens);
    return cudaGetLastError() == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
}

size_t prefill_workspace_bytes(int batch, int seq_len) { return prefill_layout(batch, seq_len).total; }

}  // namespace mq

namespace {
std::mutex g_pf_mutex;
struct PfWs {
    void* ptr = nullptr;
    size_t bytes = 0;
};
PfWs g_pf_ws[64];
thread_local int g_pf_last_error = 0;
}  // namespace

extern "C" {

size_t mq_prefill_workspace_bytes(int batch, int seq_len) { return mq::prefill_workspace_bytes(batch, seq_len); }

int mq_prefill(const mq_prefill_params* params, cudaStream_t stream) { return mq::prefill_forward(params, stream); }

void launch_prefill_float(const int* input_token_ids, int* output_token_id, int seq_len, const void* embed_weight,
                          const PrefillLayerWeights* layer_weights, const void* final_norm_weight,
                          const void* lm_head_weight, const void* cos_table, const void* sin_table, void* k_cache,
                          void* v_cache, void* /*hidden_bf16*/, void* /*residual*/, void* /*normalized*/,
                          void* /*q_proj*/, void* /*k_proj*/, void* /*v_proj*/, void* /*attn_out*/,
                          void* /*o_proj_out*/, void* /*mlp_norm*/, void* /*gate_out*/, void* /*up_out*/,
                          void* /*mlp_intermediate*/, void* /*down_out*/, void* /*final_hidden*/,
                          void* /*block_max_vals*/, void* /*block_max_idxs*/, void* /*hidden_bf16_out*/,
                          int num_layers, int max_seq_len, float attn_scale, void* /*cublas_handle*/,
                          cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) { g_pf_last_error = MQ_ERR_CUDA; return; }
    const size_t need = mq::prefill_workspace_bytes(1, seq_len);
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_pf_mutex);
        if (g_pf_ws[dev].bytes < need) {
            if (g_pf_ws[dev].ptr) {
                cudaStreamSynchronize(stream);
                cudaFree(g_pf_ws[dev].ptr);
            }
            g_pf_ws[dev].ptr = nullptr;
            g_pf_ws[dev].bytes = 0;
            if (cudaMalloc(&g_pf_ws[dev].ptr, need) != cudaSuccess) { g_pf_last_error = MQ_ERR_CUDA; return; }
            g_pf_ws[dev].bytes = need;
        }
        ws = g_pf_ws[dev].ptr;
    }
    mq_prefill_params p = {};
    p.ids = input_token_ids;
    p.batch = 1;
    p.seq_len = seq_len;
    p.embed = embed_weight;
    p.layers_host = layer_weights;
    p.final_norm = final_norm_weight;
    p.lm_head = lm_head_weight;
    p.cos_table = cos_table;
    p.sin_table = sin_table;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.num_layers = num_layers;
    p.max_seq_len = max_seq_len;
    p.attn_scale = attn_scale;
    p.out_tokens = output_token_id;
    p.workspace = ws;
    p.workspace_bytes = need;
    g_pf_last_error = mq::prefill_forward(&p, stream);
}

void launch_prefill_megakernel(const int* token_ids, int* output_token_id, int seq_len, const void* embed_weight,
                               const PrefillLayerWeights* layer_weights, const void* final_norm_weight,
                               const void* lm_head_weight, const void* cos_table, const void* sin_table,
                               void* k_cache, void* v_cache, void* /*hidden*/, void* /*residual*/,
                               void* /*normalized*/, void* /*q_proj*/, void* /*k_proj*/, void* /*v_proj*/,
                               void* /*attn_out*/, void* /*mlp_intermediate*/, void* /*final_hidden*/,
                               void* /*hidden_bf16_out*/, void* /*block_max_vals*/, void* /*block_max_idxs*/,
                               int num_layers, int max_seq_len, float attn_scale, cudaStream_t stream) {
    // The reference passes a DEVICE array of layer pointers here (unlike
    // launch_prefill_float); the engine reads the pointers on the host.
    if (num_layers < 1 || num_layers > MQ_MAX_LAYERS || !layer_weights) { g_pf_last_error = MQ_ERR_INVALID_ARGUMENT; return; }
    PrefillLayerWeights host[MQ_MAX_LAYERS];
    if (cudaMemcpyAsync(host, layer_weights, sizeof(PrefillLayerWeights) * num_layers, cudaMemcpyDeviceToHost,
                        stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess) {
        g_pf_last_error = MQ_ERR_CUDA;
        return;
    }
    launch_prefill_float(token_ids, output_token_id, seq_len, embed_weight, host, final_norm_weight, lm_head_weight,
                         cos_table, sin_table, k_cache, v_cache, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                         nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                         nullptr, num_layers, max_seq_len, attn_scale, nullptr, stream);
}

int mq_prefill_get_last_error(void) { return g_pf_last_error; }

#if MQ_PROFILE_HOOKS
// Copies the attention trace stamps of the last MQ_FA_TRACE prefill (profiling).
int mq_debug_fa_trace(unsigned long long* host, int n) {
    if (!mq::g_fa_trace) return 0;
    cudaMemcpy(host, mq::g_fa_trace, (size_t)n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    return n;
}
#endif

}  // extern "C"
