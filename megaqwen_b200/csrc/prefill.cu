// Prefill building blocks for sm_100a: the tcgen05 GEMM (gemm_tc.cuh) and its
// host-side launch (TMA tensor maps), plus the C-ABI entry mq_gemm_bf16.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gemm_tc.cuh"
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
bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {GEMM_BK, GEMM_BM};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
int launch_gemm(const void* A, int lda, const void* B, int ldb, const void* B2, void* C, int ldc, int M, int N,
                int K, int* err, cudaStream_t stream) {
    using Cfg = GemmCfg<EPI>;
    static bool configured[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MQ_ERR_CUDA;
    if (dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(gemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
            cudaSuccess)
            return MQ_ERR_CUDA;
        configured[dev] = true;
    }
    CUtensorMap ta, tb, tb2;
    if (!make_tmap(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda)) return MQ_ERR_CUDA;
    if (!make_tmap(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb)) return MQ_ERR_CUDA;
    tb2 = tb;
    if (EPI == EPI_SILU_MUL && !make_tmap(&tb2, B2, (uint64_t)N, (uint64_t)K, (uint64_t)ldb)) return MQ_ERR_CUDA;
    GemmArgs a;
    a.C = C;
    a.ldc = ldc;
    a.M = M;
    a.N = N;
    a.K = K;
    a.err = err;
    a.timeout_cycles = 4000000000ll;  // ~2 s at 1.9 GHz
    dim3 grid(N / GEMM_BN, (M + GEMM_BM - 1) / GEMM_BM);
    gemm_tc_kernel<EPI><<<grid, GEMM_THREADS, Cfg::SMEM, stream>>>(ta, tb, tb2, a);
    return cudaGetLastError() == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
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
