// Shared definitions of the tcgen05 GEMMs (gemm_persist.cuh for prefill,
// gemm_small.cuh for batched decode): tile sizes, epilogue codes and the
// bounded mbarrier wait.  Operands are bf16 in global memory, both K-major
// (row-major activations and row-major nn.Linear weights), loaded by TMA with
// the 128-byte swizzle; accumulation is fp32 in TMEM.
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

}  // namespace mq
