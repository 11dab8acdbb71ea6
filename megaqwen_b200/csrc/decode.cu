// Persistent batch-1 decode step for Qwen3-0.6B on B200 (sm_100a).
//
// One cooperative launch, one CTA per SM, runs a whole decode step: embedding,
// 28 x [RMSNorm, QKV, QK-norm, RoPE, KV write, GQA attention, O + residual,
// RMSNorm, gate/up + SiLU*mul, down + residual], final norm, tied LM head and
// argmax.  Replaces the reference's cooperative kernel + two LM-head kernels
// (csrc/megakernel/fused_decode_ldg.cu:617-723, :771-887).
//
// Structure (B200-first, not the reference's):
//  * Every CTA owns a fixed slice of every weight matrix (contiguous rows) and
//    streams it with bulk async copies (cp.async.bulk, TMA engine) into a ring
//    of shared-memory stages guarded by mbarriers.  A dedicated producer warp
//    runs ahead through the CTA's whole per-token tile list (all layers, then
//    the LM head), so HBM keeps streaming while consumers wait on data.
//  * There is no grid-wide barrier.  Each phase's outputs are published as
//    64-bit words {tag, fp32 value} with single relaxed stores; consumers poll
//    exactly the words they need until the tag matches (flag-in-word
//    handoff), so a handoff costs one store-to-L2 plus one poll.
//  * RMSNorms are recomputed redundantly by every CTA from the polled vector.
//  * Attention is split-K flash decoding: 8 kv heads x C position chunks, one
//    work unit per CTA, each unit serving both q heads of its kv head (every
//    K/V byte read once).  Units of up to 128 positions use fp32 dot products
//    spread over all 15 warps; longer units the tensor cores (mma.sync).
//    With C > 1, unit 0 of each kv head combines the partial (max, sum, acc)
//    triples.
//  * The LM head is fused: each CTA takes a slice of vocabulary rows, keeps a
//    running (value, index) best, publishes it with one 64-bit atomicMax, and
//    the last CTA to arrive writes the token.
//  * Every wait is bounded by %globaltimer; on expiry the CTA records an error
//    in the workspace and all CTAs leave after their in-flight copies land.
//
// Numerics follow the reference PyTorch forward on fp32 weights (demo_e2e.py
// Backend.TORCH): fp32 activations and residual stream, bf16 K/V cache (the
// current position's K/V are rounded to bf16 before use, demo_e2e.py:298-300),
// bf16 RoPE tables, fp32 softmax.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "megaqwen_b200.h"
#include "mq_ptx.cuh"

namespace mq {

typedef __nv_bfloat16 bf16;

constexpr int H = MQ_HIDDEN_SIZE;          // 1024
constexpr int I = MQ_INTERMEDIATE_SIZE;    // 3072
constexpr int NQ = MQ_NUM_Q_HEADS;         // 16
constexpr int NKV = MQ_NUM_KV_HEADS;       // 8
constexpr int D = MQ_HEAD_DIM;             // 128
constexpr int QS = NQ * D;                 // 2048
constexpr int KVS = NKV * D;               // 1024
constexpr int QKV = QS + 2 * KVS;          // 4096
constexpr int V = MQ_VOCAB_SIZE;           // 151936

constexpr int NCW = 15;                    // consumer warps (16 warps in all: 128 registers per thread)
constexpr int NCT = NCW * 32;              // consumer threads
constexpr int NTHREADS = NCT + 32;         // + one producer warp
constexpr int STAGE_BYTES = 32768;
constexpr int NSTAGES = 5;
constexpr int MAX_CTAS = 256;
constexpr int MAX_TP = MQ_MAX_TP;          // largest tensor-parallel group
constexpr int CMAX = MAX_CTAS / NKV;       // max position chunks per kv head
static_assert(CMAX <= 32, "the split-K combine holds one unit per lane");
constexpr int PART_STRIDE = 132;           // tagged words per (unit, head): acc[128], m, l, pad, pad

constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int QKV_TILE = cmin(NCW, STAGE_BYTES / (H * 2));      // 15 rows
constexpr int O_TILE = cmin(NCW, STAGE_BYTES / (QS * 2));       // 8 rows (T = 1; rows per stage are TP_(o_tile, O_TILE))
constexpr int GU_TILE = cmin(NCW, STAGE_BYTES / (2 * H * 2));   // 8 gate+up row pairs
constexpr int DOWN_TILE = cmin(NCW, STAGE_BYTES / (I * 2));     // 5 rows (T = 1; rows per stage are TP_(dn_tile, DOWN_TILE))
constexpr int LM_TILE = cmin(NCW, STAGE_BYTES / (H * 2));       // 15 rows
constexpr int HPT = (H + NCT - 1) / NCT;             // hidden elements per consumer thread (3)
constexpr int MV_GROUP = 3;                          // ring stages consumed together by a matvec phase
constexpr int MV_Q = 3;                              // rows per warp in a group
static_assert(MV_GROUP * QKV_TILE <= MV_Q * NCW && MV_GROUP * LM_TILE <= MV_Q * NCW &&
              MV_GROUP * GU_TILE <= MV_Q * NCW && MV_GROUP * NCW <= MV_Q * NCW,
              "a group's rows fit MV_Q rows per warp (O and down stages hold at most NCW rows)");
static_assert(MV_GROUP < NSTAGES, "the producer can fill a whole group");
constexpr int KV_TILE = STAGE_BYTES / (2 * D * 2);   // 64 positions (K and V)
// Units of up to two 64-position tiles (every unit up to p = 2303) run the
// fp32 attention path; longer ones the tensor-core path (measured: fp32 for
// all units was 2 % faster at p = 2048 but 1.4 % slower at 8192 and 5 % at
// 32768).
constexpr int ATTN_FP32_MAX_TILES = 2;
static_assert(KV_TILE == 64 && 4 * MV_GROUP <= NCW, "attention: 4 groups of 16 positions per tile, one warp each");
static_assert(QKV_TILE <= NCW && O_TILE <= NCW && GU_TILE <= NCW && DOWN_TILE <= NCW && LM_TILE <= NCW,
              "one consumer warp per row of a tile");

constexpr int BAR_CONSUMERS = 1;
// In-phase trace stamps (phase, tile, attention and clock64 micro stamps) are
// compiled only with -DMQ_DECODE_TRACE=1: their code, even when not executed,
// spreads the hot loop over more instruction-cache lines and costs ~10 % of
// the step.  The per-kernel start/end stamps are always available.
#ifndef MQ_DECODE_TRACE
#define MQ_DECODE_TRACE 0
#endif
constexpr bool kGT = MQ_DECODE_TRACE;
constexpr int TRACE_STRIDE = 2048;        // trace slots per CTA: phases [0,512), tiles [512, 2012)           // named barrier id for the consumer warps

// ---- workspace layout (bytes) ------------------------------------------------
struct Control {
    uint32_t epoch;               // bumped by the last CTA of every successful step
    uint32_t error;               // first error code (0 = none)
    uint32_t info;                // where the first error happened (phase<<8 | layer)
    uint32_t lm_count;            // arrivals at the LM-head argmax
    unsigned long long lm_best;   // packed (ordered value, ~index) running max
    int32_t last_token;
    int32_t last_position;
    uint32_t pad[56];
};
static_assert(sizeof(Control) == 256, "control block is 256 bytes");

constexpr size_t OFF_CTRL = 0;
constexpr size_t OFF_QKV = 256;
constexpr size_t OFF_ATTN = OFF_QKV + 2ull * QKV * 8;
// O-projection and down-projection outputs are per-rank partials
// [parity][rank][1024] (one rank: the whole vector); every rank stores its
// partial into every rank's workspace and the consumer adds them in rank order.
constexpr size_t OFF_HMID = OFF_ATTN + 2ull * QS * 8;
constexpr size_t OFF_ACT = OFF_HMID + 2ull * MAX_TP * H * 8;
constexpr size_t OFF_HOUT = OFF_ACT + 2ull * I * 8;
constexpr size_t OFF_PART = OFF_HOUT + 2ull * MAX_TP * H * 8;
constexpr size_t OFF_LMX = OFF_PART + (size_t)NKV * CMAX * 2 * PART_STRIDE * 8;   // [MAX_TP] {key, tag}
constexpr size_t WS_BYTES = OFF_LMX + (size_t)MAX_TP * 16;

// ---- shared memory layout (bytes, dynamic) -------------------------------------
constexpr int SM_STAGES = 0;
constexpr int SM_X = SM_STAGES + NSTAGES * STAGE_BYTES;  // fp32 [3072], planar (see store_x)
constexpr int SM_H2 = SM_X + I * 4;                       // fp32 [1024] post-attention residual
constexpr int SM_ACC = SM_X;                              // attention combine acc [16][2][128] aliases X,H2
constexpr int SM_H = SM_H2 + H * 4;                       // fp32 [1024] layer-input residual
constexpr int SM_QKVRAW = SM_H + H * 4;                   // fp32 [512]  raw q(256) k(128) v(128)
constexpr int SM_QN = SM_QKVRAW + 512 * 4;                // fp32 [256]  normed+roped q of 2 heads
constexpr int SM_KP = SM_QN + 256 * 4;                    // fp32 [128]  bf16-rounded k of position p
constexpr int SM_VP = SM_KP + 128 * 4;                    // fp32 [128]  bf16-rounded v of position p
constexpr int SM_ML = SM_VP + 128 * 4;                    // fp32 [16][2][2] per-warp (m, l) + current position
constexpr int SM_RED = SM_ML + (NCW + 1) * 4 * 4;         // fp32 [2][16]
constexpr int SM_BEST = SM_RED + 2 * NCW * 4;             // fp32 [16] + int [16]
constexpr int SM_FLAGS = SM_BEST + 2 * NCW * 4;           // int [4]
constexpr int SM_BARS = SM_FLAGS + 16;                    // uint64 full[NSTAGES], empty[NSTAGES]
constexpr int SM_LAYERS = SM_BARS + 2 * NSTAGES * 8;      // LDGLayerWeights [num_layers] copy
constexpr int SM_SCHED = SM_LAYERS + MQ_MAX_LAYERS * (int)sizeof(LDGLayerWeights);  // Sched
constexpr int SM_PARAMS = SM_SCHED + 256;                 // KParams copy (see decode_step_kernel)
constexpr int SMEM_BYTES = SM_PARAMS + 512;
static_assert(SM_ACC + (NCW + 1) * 2 * D * 4 <= SM_H, "attention combine scratch fits in X+H2");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(SM_BARS % 8 == 0, "mbarrier alignment");

enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

struct KParams {
    int input_token;
    const int* input_token_ptr;
    int* output_token;
    float* logits;
    const bf16* embed;
    const LDGLayerWeights* layers;
    const bf16* final_norm;
    const bf16* lm_head;
    const bf16* cos_table;
    const bf16* sin_table;
    bf16* k_cache;
    bf16* v_cache;
    bf16* hidden_out;
    float* norm_out;
    uint8_t* ws;
    int num_layers;
    int position;
    int* position_ptr;
    int max_seq_len;
    float attn_scale;
    int attn_chunk;
    long long timeout_ns;
    int inject_skip_cta;
    unsigned long long* trace;
    mq_host_result* host_result;   // mapped host memory (device-visible address) or null
    uint32_t host_seq;
    int rank, tp;                  // tensor-parallel rank and group size (1: single GPU)
    uint8_t* peer_ws[MAX_TP];      // every rank's workspace; [rank] == ws
};
static_assert(sizeof(KParams) <= 512 && sizeof(KParams) % 4 == 0, "KParams copy fits its slot");

// Per-CTA slice of every phase (identical on the producer and consumer side).
struct Sched {
    int G, c;
    int pos, L;                       // position and cache length (pos + 1)
    int tag_base;                     // (epoch + 1) << 6
    int qkv_a, qkv_b, o_a, o_b, gu_a, gu_b, dn_a, dn_b, lm_a, lm_b;
    int has_unit, ug, uj, C, kv_s, kv_e, last;
    // tensor parallel: rank, group size, this rank's q/k rows per matrix
    // (QS/T, KVS/T), first q/k row, O input columns (QS/T from column q0),
    // act columns [ia_a, ia_a + ia) of the down projection, rows per O and
    // down stage
    int rank, tp, qt, kt, q0, k0, ia_a, ia, o_tile, dn_tile;
};

static_assert(sizeof(Sched) <= 256, "Sched fits its shared-memory slot");

// Tensor-parallel geometry in code templated on MT (multi-GPU): the
// single-GPU instantiation (MT == false) sees compile-time constants, so its
// code is that of a kernel without tensor parallelism.
#define TP_(field, single) (MT ? S.field : (single))

// Dynamic shared memory of the decode kernel.  Everything a CTA keeps on chip
// is addressed from this base with the SM_* offsets above, so no pointer to it
// occupies a register.
extern __shared__ __align__(1024) uint8_t g_smem[];
template <typename T>
__device__ __forceinline__ T* sm(int off) { return reinterpret_cast<T*>(g_smem + off); }

__device__ __forceinline__ int split_at(int n, int G, int c) { return (int)(((long long)c * n) / G); }

__device__ __forceinline__ uint32_t tag_of(const Sched& S, int layer) { return (uint32_t)S.tag_base | (uint32_t)layer; }

__device__ __forceinline__ uint64_t ll_word(float v, uint32_t tag) {
    return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
}

__device__ __forceinline__ Control* ctrl_of(const KParams& P) { return reinterpret_cast<Control*>(P.ws + OFF_CTRL); }
__device__ __forceinline__ uint64_t* ll_qkv(const KParams& P, int l) {
    return reinterpret_cast<uint64_t*>(P.ws + OFF_QKV) + (size_t)(l & 1) * QKV;
}
__device__ __forceinline__ uint64_t* ll_attn(const KParams& P, int l) {
    return reinterpret_cast<uint64_t*>(P.ws + OFF_ATTN) + (size_t)(l & 1) * QS;
}
// Partials of rank 0; rank r's follow at + r * H.
__device__ __forceinline__ size_t off_hmid(int l) { return OFF_HMID + (size_t)(l & 1) * MAX_TP * H * 8; }
__device__ __forceinline__ size_t off_hout(int l) { return OFF_HOUT + (size_t)(l & 1) * MAX_TP * H * 8; }
__device__ __forceinline__ uint64_t* ll_hmid(const KParams& P, int l) {
    return reinterpret_cast<uint64_t*>(P.ws + off_hmid(l));
}
__device__ __forceinline__ uint64_t* ll_act(const KParams& P, int l) {
    return reinterpret_cast<uint64_t*>(P.ws + OFF_ACT) + (size_t)(l & 1) * I;
}
__device__ __forceinline__ uint64_t* ll_hout(const KParams& P, int l) {
    return reinterpret_cast<uint64_t*>(P.ws + off_hout(l));
}
__device__ __forceinline__ uint64_t* lmx_of(uint8_t* ws, int r) {
    return reinterpret_cast<uint64_t*>(ws + OFF_LMX) + 2 * r;
}
// Tagged words that other GPUs write or read are accessed at system scope.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Split-K partial of unit j, head h of kv head g as tagged words: acc[128]
// (unnormalised), max (log2 domain) at 128, sum at 129.
__device__ __forceinline__ uint64_t* part_of(const KParams& P, int g, int j, int h) {
    return reinterpret_cast<uint64_t*>(P.ws + OFF_PART) + ((size_t)(g * CMAX + j) * 2 + h) * PART_STRIDE;
}

__device__ __forceinline__ void record_error(const KParams& P, uint32_t code, uint32_t info) {
    Control* C = ctrl_of(P);
    if (atomicCAS(&C->error, 0u, code) == 0u) atomicExch(&C->info, info);
}

__device__ __forceinline__ bool global_error(const KParams& P) { return ld_relaxed_u32(&ctrl_of(P)->error) != 0u; }

// Planar storage of an fp32 vector of length K (multiple of 8): element i of
// 8-group c lives at c*4 + (i&3) in plane (i>>2)&1, planes K/2 floats apart.
// A lane reading 8-groups l, l+32, ... then issues conflict-free 16-byte loads.
__device__ __forceinline__ int planar_index(int i, int K) { return ((i >> 2) & 1) * (K >> 1) + (i >> 3) * 4 + (i & 3); }

// Two-lane fp32 accumulator for the matvecs: acc += (w pairs) * (x pairs) with
// the packed fp32x2 FMA of sm_100 (two independent chains, half the FMAs).
__device__ __forceinline__ unsigned long long f2pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float f2sum(unsigned long long v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return a + b;
}
__device__ __forceinline__ void dot8x2(unsigned long long& acc, uint4 w, float4 lo, float4 hi) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(f2pack(bf16lo(w.x), bf16hi(w.x))), "l"(f2pack(lo.x, lo.y)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(f2pack(bf16lo(w.y), bf16hi(w.y))), "l"(f2pack(lo.z, lo.w)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(f2pack(bf16lo(w.z), bf16hi(w.z))), "l"(f2pack(hi.x, hi.y)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(f2pack(bf16lo(w.w), bf16hi(w.w))), "l"(f2pack(hi.z, hi.w)));
}

__device__ __forceinline__ float dot8(uint4 w, float4 lo, float4 hi) {
    float s = bf16lo(w.x) * lo.x;
    s = fmaf(bf16hi(w.x), lo.y, s);
    s = fmaf(bf16lo(w.y), lo.z, s);
    s = fmaf(bf16hi(w.y), lo.w, s);
    s = fmaf(bf16lo(w.z), hi.x, s);
    s = fmaf(bf16hi(w.z), hi.y, s);
    s = fmaf(bf16lo(w.w), hi.z, s);
    s = fmaf(bf16hi(w.w), hi.w, s);
    return s;
}

__device__ __forceinline__ const char* qkv_row(const LDGLayerWeights& W, int r) {
    if (r < QS) return (const char*)W.q_proj_weight + (size_t)r * H * 2;
    if (r < QS + KVS) return (const char*)W.k_proj_weight + (size_t)(r - QS) * H * 2;
    return (const char*)W.v_proj_weight + (size_t)(r - QS - KVS) * H * 2;
}

// Row j of this rank's [q; k; v] rows -> its row in the concatenated
// [q (2048); k (1024); v (1024)] space (one rank: the identity).
template <bool MT>
__device__ __forceinline__ int qkv_global(const Sched& S, int j) {
    if (j < TP_(qt, QS)) return TP_(q0, 0) + j;
    if (j < TP_(qt, QS) + TP_(kt, KVS)) return QS + TP_(k0, 0) + (j - TP_(qt, QS));
    return QS + KVS + TP_(k0, 0) + (j - TP_(qt, QS) - TP_(kt, KVS));
}

// ---- the per-CTA tile lists, shared by producer and consumers ------------------
// for_tiles calls f(first_row, rows, src1, bytes1, src2, bytes2, stride) for
// every stage-sized tile this CTA owns in one phase of one layer, in ring
// order.  stride == 0: one or two contiguous copies placed back to back;
// stride > 0: `rows` rows of bytes1 bytes, stride bytes apart in global
// memory, packed in the stage.
template <bool MT, class F>
__device__ __forceinline__ void for_tiles(const KParams& P, const Sched& S, int phase, int l, F&& f) {
    if (phase == PH_LM) {
        for (int r = S.lm_a; r < S.lm_b;) {
            int n = min(S.lm_b - r, LM_TILE);
            f(r, n, (const char*)P.lm_head + (size_t)r * H * 2, n * H * 2, (const char*)nullptr, 0, 0);
            r += n;
        }
        return;
    }
    const LDGLayerWeights& W = sm<LDGLayerWeights>(SM_LAYERS)[l];
    if (phase == PH_QKV) {
        // This rank's rows of [q; k; v] in tiles of QKV_TILE; a tile that
        // crosses a matrix boundary is two bulk copies into one stage.
        const int b1 = TP_(qt, QS), b2 = TP_(qt, QS) + TP_(kt, KVS);
        for (int r = S.qkv_a; r < S.qkv_b; r += QKV_TILE) {
            const int e = min(S.qkv_b, r + QKV_TILE);
            const int cut = (r < b1 && e > b1) ? b1 : ((r < b2 && e > b2) ? b2 : e);
            f(r, e - r, qkv_row(W, qkv_global<MT>(S, r)), (cut - r) * H * 2,
              cut < e ? qkv_row(W, qkv_global<MT>(S, cut)) : (const char*)nullptr, (e - cut) * H * 2, 0);
        }
    } else if (phase == PH_ATTN) {
        for (int t = S.kv_s; t < S.kv_e; t += KV_TILE) {
            int n = min(S.kv_e - t, KV_TILE);
            size_t off = (((size_t)l * NKV + S.ug) * P.max_seq_len + t) * D * 2;
            f(t, n, (const char*)P.k_cache + off, n * D * 2, (const char*)P.v_cache + off, n * D * 2, 0);
        }
    } else if (phase == PH_O) {
        // rows [o_a, o_b) x this rank's attention columns [q0, q0 + qt)
        for (int r = S.o_a; r < S.o_b;) {
            int n = min(S.o_b - r, TP_(o_tile, O_TILE));
            const char* src = (const char*)W.o_proj_weight + ((size_t)r * QS + TP_(q0, 0)) * 2;
            if (TP_(tp, 1) == 1) f(r, n, src, n * QS * 2, (const char*)nullptr, 0, 0);
            else f(r, n, src, TP_(qt, QS) * 2, (const char*)nullptr, 0, QS * 2);
            r += n;
        }
    } else if (phase == PH_GU) {
        for (int r = S.gu_a; r < S.gu_b;) {
            int n = min(S.gu_b - r, GU_TILE);
            f(r, n, (const char*)W.gate_proj_weight + (size_t)r * H * 2, n * H * 2,
              (const char*)W.up_proj_weight + (size_t)r * H * 2, n * H * 2, 0);
            r += n;
        }
    } else {
        // rows [dn_a, dn_b) x this rank's act columns [ia_a, ia_a + ia)
        for (int r = S.dn_a; r < S.dn_b;) {
            int n = min(S.dn_b - r, TP_(dn_tile, DOWN_TILE));
            const char* src = (const char*)W.down_proj_weight + ((size_t)r * I + TP_(ia_a, 0)) * 2;
            if (TP_(tp, 1) == 1) f(r, n, src, n * I * 2, (const char*)nullptr, 0, 0);
            else f(r, n, src, TP_(ia, I) * 2, (const char*)nullptr, 0, I * 2);
            r += n;
        }
    }
}

// The per-token phase sequence of one CTA.
template <class Vis>
__device__ __forceinline__ void walk(const KParams& P, const Sched& S, Vis& v) {
    for (int l = 0; l < P.num_layers; ++l) {
        if (!v.run(PH_QKV, l)) return;
        if (S.has_unit && !v.run(PH_ATTN, l)) return;
        if (!v.run(PH_O, l)) return;
        if (!v.run(PH_GU, l)) return;
        if (!v.run(PH_DOWN, l)) return;
    }
    v.run(PH_LM, P.num_layers);
}

// ---- producer: one thread issuing bulk copies into the stage ring ---------------
template <bool MT>
struct Producer {
    const KParams& P;
    uint8_t* smem;
    uint64_t* full;
    uint64_t* empty;
    volatile int* flags;
    uint32_t n = 0;          // tiles issued
    bool ok = true;
    uint64_t policy;

    __device__ Producer(const KParams& p, uint8_t* s) : P(p), smem(s) {
        full = reinterpret_cast<uint64_t*>(s + SM_BARS);
        empty = full + NSTAGES;
        flags = reinterpret_cast<volatile int*>(s + SM_FLAGS);
        policy = policy_evict_first();
    }
    __device__ __forceinline__ bool run(int phase, int l) {
        for_tiles<MT>(P, *sm<Sched>(SM_SCHED), phase, l,
                  [&](int, int rows, const char* s1, int b1, const char* s2, int b2, int stride) {
                      tile(phase, l, s1, b1, s2, b2, stride, rows);
                  });
        return ok;
    }

    // Out of line: one copy of the issue code serves all six tile loops (a
    // smaller producer leaves more of the instruction cache to the consumers).
    __device__ __noinline__ void tile(int phase, int layer, const char* src1, int b1, const char* src2, int b2,
                                      int stride, int rows) {
        if (!ok) return;
        const uint32_t s = n % NSTAGES;
        if (n >= (uint32_t)NSTAGES) {
            const uint32_t par = ((n / NSTAGES) & 1u) ^ 1u;
            uint64_t t0 = 0;
            uint32_t spins = 0;
            while (!mbar_try_wait(&empty[s], par)) {
                if ((++spins & 63u) == 0) {
                    uint64_t now = globaltimer_ns();
                    if (t0 == 0) t0 = now;
                    if (flags[0] != 0 || global_error(P) || (long long)(now - t0) > P.timeout_ns) {
                        if (flags[0] == 0 && !global_error(P))
                            record_error(P, MQ_ERR_PIPE_TIMEOUT, 0x100u | ((uint32_t)phase << 8) | layer);
                        ok = false;
                        return;
                    }
                }
            }
        }
        uint8_t* dst = smem + SM_STAGES + s * STAGE_BYTES;
        if (kGT && P.trace && n < 320) P.trace[(size_t)blockIdx.x * TRACE_STRIDE + 512 + 4 * n] = globaltimer_ns();
        if (stride) {
            // strided rows (tensor-parallel column slices): one copy per row
            mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * b1));
            for (int i = 0; i < rows; ++i)
                bulk_g2s(dst + (size_t)i * b1, src1 + (size_t)i * stride, (uint32_t)b1, &full[s], policy);
        } else {
            mbar_arrive_expect_tx(&full[s], (uint32_t)(b1 + b2));
            bulk_g2s(dst, src1, (uint32_t)b1, &full[s], policy);
            if (b2) bulk_g2s(dst + b1, src2, (uint32_t)b2, &full[s], policy);
        }
        ++n;
    }

    // Wait (bounded) for every issued copy to land before the CTA may exit.
    __device__ __forceinline__ void drain() {
        uint32_t first = n > (uint32_t)NSTAGES ? n - NSTAGES : 0;
        for (uint32_t k = first; k < n; ++k) {
            const uint32_t s = k % NSTAGES, par = (k / NSTAGES) & 1u;
            uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[s], par)) {
                if ((long long)(globaltimer_ns() - t0) > P.timeout_ns) break;
            }
        }
    }
};

// Online-softmax state of one warp of an attention work unit (two q heads of
// one kv head), in mma.sync fragment form.  Scores are in the log2 domain.
//   S^T = K Q^T on m16n8k16: 16 positions on M, N columns 0/1 = q heads 0/1
//   rounded to bf16 and columns 2/3 = their bf16 remainders (hi + lo carries
//   the fp32 q), so one MMA gives near-fp32 scores.  P^T is split the same way
//   (columns 0/1 = bf16(p), 2/3 = remainder) for O^T = V^T P^T.
//   Accumulator lane (g, t): t == 0 holds the hi columns of heads 0/1, t == 1
//   the lo columns; the two are summed at the end of the phase.
// The B fragments of Q^T live in shared memory (SM_QKVRAW, free once q is
// normed): uint2 [k-step u*2+half][lane].
struct AttnState {
    float o[4][2][4];       // O^T accumulators per (u, q) block
    float m[2], l[2];       // running max / sum of the lane's two columns
};

__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
    __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&t);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }
// Head dim held by accumulator row g of block (u, r): lane t loads dims
// 32u + 8t .. +7 of a row as 16 bytes, register r holds the pair 32u + 8t + 2r.
__device__ __forceinline__ int attn_vdim(int u, int r, int g) { return 32 * u + 8 * (g >> 1) + 2 * r + (g & 1); }

// Running LM-head argmax of one warp (value, then lowest index on ties).
struct LmBest {
    float v;
    int i;
};

// ---- consumers: 16 warps computing on staged tiles -------------------------------
template <bool MT>
struct Consumer {
    const KParams& P;
    const Sched& S;
    int ct, warp, lane;
    uint32_t n = 0;          // tiles consumed
    bool ok = true;          // this thread's view; made collective at begin()
    int red_par = 0;
    float nrm = 1.f;   // rstd of the phase's RMSNorm (norm phases scale their dot products by it)

    __device__ static float* sx() { return sm<float>(SM_X); }
    __device__ static float* sh() { return sm<float>(SM_H); }
    __device__ static float* sh2() { return sm<float>(SM_H2); }
    __device__ static float* sred() { return sm<float>(SM_RED); }
    __device__ static uint64_t* full() { return sm<uint64_t>(SM_BARS); }
    __device__ static uint64_t* empty() { return sm<uint64_t>(SM_BARS) + NSTAGES; }
    __device__ static volatile int* flags() { return sm<volatile int>(SM_FLAGS); }

    __device__ Consumer(const KParams& p, const Sched& s) : P(p), S(s) {
        ct = threadIdx.x - 32;
        warp = ct >> 5;
        lane = ct & 31;
    }

    __device__ __forceinline__ void fail(uint32_t code, uint32_t info) {
        if (ok) {
            if (!global_error(P)) record_error(P, code, info);
            flags()[0] = 1;
        }
        ok = false;
    }

    // Poll `count` tagged words into registers: thread ct owns words ct + k*NCT
    // (k < NK <= 8, all loads in flight at once) and receives their values in
    // vals.  Bounded; callers synchronise X themselves.
    template <int NK>
    __device__ __forceinline__ int poll(const uint64_t* src, int count, uint32_t tag, float* vals, uint32_t info) {
        int cnt = 0;
        uint32_t pending = 0;
#pragma unroll
        for (int k = 0; k < NK; ++k)
            if (ct + k * NCT < count) { pending |= 1u << k; cnt = k + 1; }
        if (!ok) return cnt;
        uint64_t t0 = 0;
        uint32_t spins = 0;
        while (pending) {
            uint64_t w[NK];
#pragma unroll
            for (int k = 0; k < NK; ++k)
                if (pending & (1u << k)) w[k] = ld_relaxed_u64(src + ct + k * NCT);
#pragma unroll
            for (int k = 0; k < NK; ++k)
                if ((pending & (1u << k)) && (uint32_t)(w[k] >> 32) == tag) {
                    vals[k] = __uint_as_float((uint32_t)w[k]);
                    pending &= ~(1u << k);
                }
            if (pending && ((++spins & 31u) == 0)) {
                uint64_t now = globaltimer_ns();
                if (t0 == 0) t0 = now;
                if (flags()[0] != 0 || global_error(P)) { ok = false; break; }
                if ((long long)(now - t0) > P.timeout_ns) { fail(MQ_ERR_WAIT_TIMEOUT, info); break; }
            }
        }
        return cnt;
    }

    __device__ __forceinline__ void ll_store(uint64_t* p, uint64_t w) {
        st_relaxed_u64(p, w);
    }

    // Store one tagged word at byte offset `off` of every rank's workspace
    // (one rank: its own, gpu scope; several: system scope over NVLink).
    __device__ __forceinline__ void publish_all(size_t off, uint64_t w) {
        if (TP_(tp, 1) == 1) {
            st_relaxed_u64(reinterpret_cast<uint64_t*>(P.ws + off), w);
            return;
        }
        for (int r = 0; r < TP_(tp, 1); ++r) st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(P.peer_ws[r] + off), w);
    }

    // vals[k] = base[i] + the ranks' partials of element i = ct + k*NCT
    // (src0: rank 0's tagged words, rank r's at + r*H), added in rank order
    // so that every CTA of every rank gets bit-identical sums.  Ranks are
    // polled four at a time, all their words in flight together.
    template <int NK>
    __device__ __forceinline__ void poll_sum(const uint64_t* src0, uint32_t tag, const float* base, float* vals,
                                             uint32_t info) {
        if (!MT) {
            float part[NK];
            poll<NK>(src0, H, tag, part, info);
#pragma unroll
            for (int k = 0; k < NK; ++k) vals[k] = (ct + k * NCT < H) ? base[ct + k * NCT] + part[k] : 0.f;
            return;
        }
#pragma unroll
        for (int k = 0; k < NK; ++k) vals[k] = (ct + k * NCT < H) ? base[ct + k * NCT] : 0.f;
        const bool sys = TP_(tp, 1) > 1;
        for (int r0 = 0; r0 < TP_(tp, 1); r0 += 4) {
            const int nr = min(4, TP_(tp, 1) - r0);
            float part[NK * 4];
            uint32_t pending = 0;
#pragma unroll
            for (int k = 0; k < NK; ++k)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    part[k * 4 + q] = 0.f;
                    if (q < nr && ct + k * NCT < H) pending |= 1u << (k * 4 + q);
                }
            uint64_t t0 = 0;
            uint32_t spins = 0;
            while (ok && pending) {
                uint64_t w[NK * 4];
#pragma unroll
                for (int j = 0; j < NK * 4; ++j)
                    if (pending & (1u << j)) {
                        const uint64_t* a = src0 + (size_t)(r0 + (j & 3)) * H + ct + (j >> 2) * NCT;
                        w[j] = sys ? ld_relaxed_sys_u64(a) : ld_relaxed_u64(a);
                    }
#pragma unroll
                for (int j = 0; j < NK * 4; ++j)
                    if ((pending & (1u << j)) && (uint32_t)(w[j] >> 32) == tag) {
                        part[j] = __uint_as_float((uint32_t)w[j]);
                        pending &= ~(1u << j);
                    }
                if (pending && ((++spins & 31u) == 0)) {
                    uint64_t now = globaltimer_ns();
                    if (t0 == 0) t0 = now;
                    if (flags()[0] != 0 || global_error(P)) { ok = false; break; }
                    if ((long long)(now - t0) > P.timeout_ns) { fail(MQ_ERR_WAIT_TIMEOUT, info); break; }
                }
            }
#pragma unroll
            for (int k = 0; k < NK; ++k)
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (q < nr) vals[k] += part[k * 4 + q];
        }
    }

    // Collective: all consumer threads agree on failure.
    __device__ __forceinline__ bool agree() {
        bool bad = named_bar_or(BAR_CONSUMERS, NCT, !ok);
        if (bad) ok = false;
        return !bad;
    }

    __device__ __forceinline__ float block_sum(float v) {
        // caller guarantees a barrier separates consecutive uses of one parity
        float* r = sred() + red_par * NCW;
        red_par ^= 1;
        v = warp_sum(v);
        if (lane == 0) r[warp] = v;
        return 0.f;  // the total is read after the next barrier via read_sum()
    }
    __device__ __forceinline__ float read_sum() {
        const float* r = sred() + (red_par ^ 1) * NCW;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NCW; ++i) s += r[i];
        return s;
    }

    // Optional per-phase timestamps (profiling): slot (l*6+phase)*2 on entry,
    // +1 once the phase's input vector has arrived.
    template <int KIND>
    __device__ __forceinline__ bool begin(int phase, int l) {
        const bool tr = P.trace != nullptr && ct == 0;
        if (kGT && tr) P.trace[(size_t)S.c * TRACE_STRIDE + (l * 6 + phase) * 2] = globaltimer_ns();
        micro(l, phase, 0);
        bool r = begin_impl<KIND>(phase, l);
        micro(l, phase, 3);
        if (kGT && tr) P.trace[(size_t)S.c * TRACE_STRIDE + (l * 6 + phase) * 2 + 1] = globaltimer_ns();
        return r;
    }

    __device__ __forceinline__ const LDGLayerWeights& layer(int l) const {
        return reinterpret_cast<const LDGLayerWeights*>(g_smem + SM_LAYERS)[l];
    }

    // Every load that does not depend on the polled vector (norm weights, RoPE
    // rows) is issued before the poll so its latency overlaps the wait.
    template <int KIND>
    __device__ __forceinline__ bool begin_impl(int phase, int l) {
        float v[8];
        if (KIND == 0 || KIND == 2) {
            const bf16* w = (phase == PH_LM)  ? P.final_norm
                            : (phase == PH_GU) ? (const bf16*)layer(l).post_attn_layernorm_weight
                                               : (const bf16*)layer(l).input_layernorm_weight;
            float wv[HPT];
#pragma unroll
            for (int k = 0; k < HPT; ++k) {
                v[k] = 0.f;
                wv[k] = (ct + k * NCT < H) ? __bfloat162float(w[ct + k * NCT]) : 0.f;
            }
            named_bar_sync(BAR_CONSUMERS, NCT);   // the previous phase is done with X
            // QKV/LM: layer input h (embedding row at layer 0, else the previous
            // layer's output); GU: the post-attention residual.
            if (phase != PH_GU && l == 0) {
                const bf16* row = P.embed + (size_t)flags()[1] * H;
#pragma unroll
                for (int k = 0; k < HPT; ++k)
                    if (ct + k * NCT < H) v[k] = __bfloat162float(row[ct + k * NCT]);
            } else {
                // one call site: the poll loop is inlined once per phase kind.
                // GU: h + the ranks' O partials; QKV / LM: the post-attention
                // residual + the ranks' down partials of the previous layer.
                const bool gu = phase == PH_GU;
                poll_sum<HPT>(gu ? ll_hmid(P, l) : ll_hout(P, l - 1), tag_of(S, gu ? l : l - 1), gu ? sh() : sh2(), v,
                              ((uint32_t)phase << 8) | l);
            }
            micro(l, phase, 1);
            float* res = (phase == PH_GU) ? sh2() : sh();
            // RMSNorm folded into the matvec: X holds x * w (no barrier for the
            // sum of squares first); the phase scales each dot product by rstd.
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < HPT; ++k) {
                const int i = ct + k * NCT;
                if (i < H) {
                    if (ok) res[i] = v[k];
                    ss += v[k] * v[k];
                    sx()[planar_index(i, H)] = v[k] * wv[k];
                }
            }
            block_sum(ss);
            if (!agree()) return false;   // publishes X and the per-warp sums
            micro(l, phase, 2);
            const float rstd = rsqrtf(read_sum() / (float)H + 1e-6f);
            nrm = rstd;
            if (KIND == 2 && S.c == 0) {
#pragma unroll
                for (int k = 0; k < HPT; ++k) {
                    const int i = ct + k * NCT;
                    if (i >= H) continue;
                    if (P.hidden_out) P.hidden_out[i] = __float2bfloat16(v[k]);
                    if (P.norm_out) P.norm_out[i] = v[k] * rstd * wv[k];
                }
            }
            return true;
        }
        if (KIND == 3) {
            const int K = (phase == PH_O) ? TP_(qt, QS) : TP_(ia, I);     // this rank's attention / act slice
            const uint64_t* src = (phase == PH_O) ? ll_attn(P, l) + TP_(q0, 0) : ll_act(P, l) + TP_(ia_a, 0);
            named_bar_sync(BAR_CONSUMERS, NCT);   // the previous phase is done with X
            int cnt = poll<(I + NCT - 1) / NCT>(src, K, tag_of(S, l), v, ((uint32_t)phase << 8) | l);
            micro(l, phase, 1);
#pragma unroll
            for (int k = 0; k < (I + NCT - 1) / NCT; ++k) {
                int i = ct + k * NCT;
                if (k < cnt && i < K) sx()[planar_index(i, K)] = v[k];
            }
            if (!agree()) return false;   // publishes X
            micro(l, phase, 2);
            return true;
        }
        // PH_ATTN: raw q (2 heads), k, v of kv head g -> smem, then QK-norm + RoPE.
        {
            const int g = S.ug;
            const uint64_t* src = ll_qkv(P, l);
            float* raw = reinterpret_cast<float*>(g_smem + SM_QKVRAW);
            const LDGLayerWeights& W = layer(l);
            // warps 0,1: q heads 2g, 2g+1; warp 2: k head g.  Lane owns elements
            // lane + 32m (m = 0..3); rotate-half pairs (m, m+2) stay in the lane.
            float nwv[4], csv[4], snv[4];
            if (warp < 3) {
                const bf16* nw = (const bf16*)(warp < 2 ? W.q_norm_weight : W.k_norm_weight);
                const bf16* cs = P.cos_table + (size_t)S.pos * D;
                const bf16* sn = P.sin_table + (size_t)S.pos * D;
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    nwv[m] = __bfloat162float(nw[lane + 32 * m]);
                    csv[m] = __bfloat162float(cs[lane + 32 * m]);
                    snv[m] = __bfloat162float(sn[lane + 32 * m]);
                }
            }
            // 512 words: q rows [256g, 256g+256), k rows [2048+128g, +128), v rows [3072+128g, +128);
            // thread ct polls words j = ct and j = ct + NCT (j < 512).
            float val[2] = {0.f, 0.f};
            if (ok) {
                uint64_t t0 = 0;
                uint32_t spins = 0;
                const uint32_t tag = tag_of(S, l);
                uint32_t pending = 1u | ((ct + NCT < 512) ? 2u : 0u);
                int idx[2];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int j = ct + k * NCT;
                    idx[k] = j < 256 ? 256 * g + j : (j < 384 ? QS + 128 * g + (j - 256) : QS + KVS + 128 * g + (j - 384));
                }
                while (pending) {
                    uint64_t w[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k)
                        if (pending & (1u << k)) w[k] = ld_relaxed_u64(src + idx[k]);
#pragma unroll
                    for (int k = 0; k < 2; ++k)
                        if ((pending & (1u << k)) && (uint32_t)(w[k] >> 32) == tag) {
                            val[k] = __uint_as_float((uint32_t)w[k]);
                            pending &= ~(1u << k);
                        }
                    if (pending && (++spins & 31u) == 0) {
                        uint64_t now = globaltimer_ns();
                        if (t0 == 0) t0 = now;
                        if (flags()[0] != 0 || global_error(P)) { ok = false; break; }
                        if ((long long)(now - t0) > P.timeout_ns) { fail(MQ_ERR_WAIT_TIMEOUT, (1u << 8) | l); break; }
                    }
                }
            }
            if (!agree()) return false;
            raw[ct] = val[0];
            if (ct + NCT < 512) raw[ct + NCT] = val[1];
            named_bar_sync(BAR_CONSUMERS, NCT);
            float* qn = reinterpret_cast<float*>(g_smem + SM_QN);
            float* kp = reinterpret_cast<float*>(g_smem + SM_KP);
            float* vp = reinterpret_cast<float*>(g_smem + SM_VP);
            if (warp < 3) {
                const float* x = raw + (warp < 2 ? warp * D : 256);
                float e[4];
                float ss = 0.f;
#pragma unroll
                for (int m = 0; m < 4; ++m) { e[m] = x[lane + 32 * m]; ss += e[m] * e[m]; }
                ss = warp_sum(ss);
                float r = rsqrtf(ss / (float)D + 1e-6f);
#pragma unroll
                for (int m = 0; m < 4; ++m) e[m] = e[m] * r * nwv[m];
                float o[4];
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    float c = csv[m], s = snv[m];
                    o[m] = (m < 2) ? (e[m] * c - e[m + 2] * s) : (e[m] * c + e[m - 2] * s);
                }
                if (warp < 2) {
#pragma unroll
                    for (int m = 0; m < 4; ++m) qn[warp * D + lane + 32 * m] = o[m];
                } else {
                    bf16* kc = P.k_cache + (((size_t)l * NKV + g) * P.max_seq_len + S.pos) * D;
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        bf16 b = __float2bfloat16(o[m]);
                        kp[lane + 32 * m] = __bfloat162float(b);
                        if (S.last) kc[lane + 32 * m] = b;
                    }
                }
            } else if (warp == 3) {
                const float* x = raw + 384;
                bf16* vc = P.v_cache + (((size_t)l * NKV + g) * P.max_seq_len + S.pos) * D;
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    bf16 b = __float2bfloat16(x[lane + 32 * m]);
                    vp[lane + 32 * m] = __bfloat162float(b);
                    if (S.last) vc[lane + 32 * m] = b;
                }
            }
            named_bar_sync(BAR_CONSUMERS, NCT);
            return true;
        }
    }

    // Warp-uniform bounded wait for stage s to fill (all lanes iterate together).
    __device__ __forceinline__ bool wait_full(uint32_t s, uint32_t par, int phase, int l) {
        if (!ok) return false;
        uint64_t t0 = 0;
        uint32_t spins = 0;
        // one lane per warp polls: 480 threads polling one mbarrier serialise
        // at the barrier (~300 cycles per poll even when the phase is done)
        while (!__shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_try_wait(&full()[s], par) : 0, 0)) {
            if ((++spins & 63u) == 0) {
                int verdict = 0;
                if (lane == 0) {
                    uint64_t now = globaltimer_ns();
                    if (t0 == 0) t0 = now;
                    if (flags()[0] != 0 || global_error(P)) verdict = 1;
                    else if ((long long)(now - t0) > P.timeout_ns) verdict = 2;
                }
                verdict = __shfl_sync(0xffffffffu, verdict, 0);
                if (verdict == 1) { ok = false; return false; }
                if (verdict == 2) {
                    if (lane == 0) fail(MQ_ERR_PIPE_TIMEOUT, 0x200u | ((uint32_t)phase << 8) | l);
                    ok = false;
                    return false;
                }
            }
        }
        __syncwarp();   // lane 0's acquire of the stage orders the other lanes' reads after it
        return true;
    }

    // One phase of one layer: wait for its input vector, then consume this
    // CTA's tiles.  Phase-local state (attention accumulators, LM best) lives
    // only inside this call.
    template <int KIND>
    __device__ __forceinline__ bool run(int phase, int l) {
        if (!begin<KIND>(phase, l)) return false;
        if (KIND == 1) {
            if (S.kv_e - S.kv_s <= ATTN_FP32_MAX_TILES * KV_TILE) attn_fp32(l);
            else attn_long(l);
            attn_stamp(l, 2);
            finish_attn(l);
            attn_stamp(l, 4);
            return true;
        }
        float xr[32];  // K=1024 phases: this lane's input chunks lane + 32u, read once per phase
        if (KIND == 0 || KIND == 2) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = lane + 32 * u;
                const float4 lo = *reinterpret_cast<const float4*>(sx() + c * 4);
                const float4 hi = *reinterpret_cast<const float4*>(sx() + H / 2 + c * 4);
                xr[8 * u + 0] = lo.x; xr[8 * u + 1] = lo.y; xr[8 * u + 2] = lo.z; xr[8 * u + 3] = lo.w;
                xr[8 * u + 4] = hi.x; xr[8 * u + 5] = hi.y; xr[8 * u + 6] = hi.z; xr[8 * u + 7] = hi.w;
            }
        }
        micro(l, phase, 4);
        if (KIND == 2) {
            LmBest best{-INFINITY, 0x7fffffff};
            mv_phase<2, PH_LM>(l, xr, &best);
            end_lm(best);
            return true;
        }
        if (KIND == 0) {
            if (phase == PH_QKV) mv_phase<0, PH_QKV>(l, xr, nullptr);
            else mv_phase<0, PH_GU>(l, xr, nullptr);
        } else {
            if (phase == PH_O) mv_phase<3, PH_O>(l, xr, nullptr);
            else mv_phase<3, PH_DOWN>(l, xr, nullptr);
        }
        return true;
    }

    // Matrix-vector products of one phase.  The phase's tiles are consumed in
    // groups of up to MV_GROUP ring stages; the group's rows are spread over
    // the 15 warps (row j -> warp j mod 15), so each warp runs up to three
    // independent dot-product chains at once instead of one chain per tile.
    // One warp per row: 16-byte chunks strided over the lanes, one shuffle
    // reduction per row.  K = 1024 inputs come from registers (xr), K = 2048 /
    // 3072 from the planar X vector.  The tiling matches for_tiles exactly.
    template <int KIND, int phase>
    __device__ __forceinline__ void mv_phase(int l, const float* xr, LmBest* bst) {
        int a, b;
        const int T = phase == PH_QKV ? QKV_TILE : phase == PH_GU ? GU_TILE : phase == PH_O ? TP_(o_tile, O_TILE)
                      : phase == PH_DOWN ? TP_(dn_tile, DOWN_TILE) : LM_TILE;
        if (phase == PH_QKV) { a = S.qkv_a; b = S.qkv_b; }
        else if (phase == PH_GU) { a = S.gu_a; b = S.gu_b; }
        else if (phase == PH_O) { a = S.o_a; b = S.o_b; }
        else if (phase == PH_DOWN) { a = S.dn_a; b = S.dn_b; }
        else { a = S.lm_a; b = S.lm_b; }
        const int K = (phase == PH_O) ? TP_(qt, QS) : (phase == PH_DOWN ? TP_(ia, I) : H);
        const int R = b - a;
        const int ntiles = (R + T - 1) / T;
        const uint32_t tag = tag_of(S, l);
        for (int g0 = 0; g0 < ntiles; g0 += MV_GROUP) {
            const int g1 = min(ntiles, g0 + MV_GROUP);
            const bool tr = P.trace && ct == 0 && n < 320;
            if (kGT && tr) P.trace[(size_t)S.c * TRACE_STRIDE + 513 + 4 * n] = globaltimer_ns();
            bool got = true;
            for (int i = g0; i < g1; ++i) {
                const uint32_t t = n + (uint32_t)(i - g0);
                got = wait_full(t % NSTAGES, (t / NSTAGES) & 1u, phase, l) && got;
            }
            if (kGT && tr) P.trace[(size_t)S.c * TRACE_STRIDE + 514 + 4 * n] = globaltimer_ns();
            if (g0 == 0) micro(l, phase, 5);
            const int j0 = g0 * T, j1 = min(g1 * T, R);
            if (got) {
                float acc[MV_Q], up[MV_Q];
#pragma unroll
                for (int q = 0; q < MV_Q; ++q) {
                    acc[q] = 0.f;
                    up[q] = 0.f;
                    const int j = j0 + warp + NCW * q;
                    unsigned long long a2 = 0ull, u2 = 0ull;   // fp32x2 partial sums (two chains)
                    if (j < j1) {
                        const int ti = j / T, lr = j - ti * T;
                        const uint8_t* st = g_smem + SM_STAGES + ((n + (uint32_t)(ti - g0)) % NSTAGES) * STAGE_BYTES;
                        if (KIND == 0 || KIND == 2) {
                            const uint4* w = reinterpret_cast<const uint4*>(st + lr * H * 2);
                            const uint4* wu = reinterpret_cast<const uint4*>(st + (min(T, R - ti * T) + lr) * H * 2);
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int c = lane + 32 * u;
                                const float4 lo = make_float4(xr[8 * u + 0], xr[8 * u + 1], xr[8 * u + 2], xr[8 * u + 3]);
                                const float4 hi = make_float4(xr[8 * u + 4], xr[8 * u + 5], xr[8 * u + 6], xr[8 * u + 7]);
                                dot8x2(a2, w[c], lo, hi);
                                if (KIND == 0 && phase == PH_GU) dot8x2(u2, wu[c], lo, hi);
                            }
                        } else {
                            const uint4* w = reinterpret_cast<const uint4*>(st + (size_t)lr * K * 2);
                            const int chunks = K >> 3;
#pragma unroll 2
                            for (int c = lane; c < chunks; c += 32)
                                dot8x2(a2, w[c], *reinterpret_cast<const float4*>(sx() + c * 4),
                                       *reinterpret_cast<const float4*>(sx() + K / 2 + c * 4));
                        }
                        acc[q] = f2sum(a2);
                        if (KIND == 0 && phase == PH_GU) up[q] = f2sum(u2);
                    }
                }
                if (g0 == 0) micro(l, phase, 6);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                    for (int q = 0; q < MV_Q; ++q) {
                        acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], o);
                        if (KIND == 0 && phase == PH_GU) up[q] += __shfl_xor_sync(0xffffffffu, up[q], o);
                    }
                }
                if (g0 == 0) micro(l, phase, 7);
                if (lane == 0) {
#pragma unroll
                    for (int q = 0; q < MV_Q; ++q) {
                        const int j = j0 + warp + NCW * q;
                        if (j >= j1) continue;
                        const int r = a + j;
                        const float v = (KIND == 0 || KIND == 2) ? acc[q] * nrm : acc[q];
                        if (KIND == 2) {
                            if (P.logits) P.logits[r] = v;
                            if (v > bst->v || (v == bst->v && r < bst->i)) { bst->v = v; bst->i = r; }
                        } else if (phase == PH_GU) {
                            ll_store(ll_act(P, l) + r, ll_word(v / (1.0f + expf(-v)) * (up[q] * nrm), tag));
                        } else if (phase == PH_QKV) {
                            if (!((S.c == P.inject_skip_cta - 1) && l == 0))
                                ll_store(ll_qkv(P, l) + qkv_global<MT>(S, r), ll_word(v, tag));
                        } else if (phase == PH_O) {
                            publish_all(off_hmid(l) + ((size_t)TP_(rank, 0) * H + r) * 8, ll_word(v, tag));
                        } else {
                            publish_all(off_hout(l) + ((size_t)TP_(rank, 0) * H + r) * 8, ll_word(v, tag));
                        }
                    }
                }
                if (g0 == 0) micro(l, phase, 8);
                if (kGT && tr) P.trace[(size_t)S.c * TRACE_STRIDE + 515 + 4 * n] = globaltimer_ns();
                for (int i = g0; i < g1; ++i) release((n + (uint32_t)(i - g0)) % NSTAGES);
                if (g0 == 0) micro(l, phase, 9);
            }
            n += (uint32_t)(g1 - g0);
        }
    }

    // 16 cached positions (rows 16 grp .. +15 of a staged K/V tile, n valid) into
    // this warp's attention state.  K rows are the A fragments of S^T as
    // loaded (16 bytes per lane; the head-dim order is permuted identically in
    // Q), V^T and P^T come from movmatrix transposes.
    __device__ __forceinline__ void attn_group(AttnState& a, const uint8_t* kb, const uint8_t* vb, int grp, int n) {
        const int g = lane >> 2, t = lane & 3;
        const int ra = 16 * grp + g, rb = ra + 8;
        const bool va = ra < n, vbk = rb < n;
        const uint2* qbs = sm<uint2>(SM_QKVRAW);
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint4 k0 = va ? *reinterpret_cast<const uint4*>(kb + ra * (D * 2) + 64 * u + 16 * t) : make_uint4(0, 0, 0, 0);
            const uint4 k1 = vbk ? *reinterpret_cast<const uint4*>(kb + rb * (D * 2) + 64 * u + 16 * t) : make_uint4(0, 0, 0, 0);
            const uint32_t a0[4] = {k0.x, k1.x, k0.y, k1.y};
            const uint32_t a1[4] = {k0.z, k1.z, k0.w, k1.w};
            const uint2 q0 = qbs[(u * 2 + 0) * 32 + lane], q1 = qbs[(u * 2 + 1) * 32 + lane];
            mma16816(sc, a0, q0.x, q0.y);
            mma16816(sc, a1, q1.x, q1.y);
        }
        // hi + lo columns: lanes t = 0 and t = 1 both get the full scores of heads 0/1
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 1);
        if (!va) sc[0] = sc[1] = -INFINITY;
        if (!vbk) sc[2] = sc[3] = -INFINITY;
        float mx[2] = {fmaxf(sc[0], sc[2]), fmaxf(sc[1], sc[3])};
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o));
            mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o));
        }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float mn = fmaxf(a.m[r], mx[r]);
            corr[r] = exp2f(a.m[r] - mn);
            a.m[r] = mn;
            a.l[r] *= corr[r];
        }
        const float e0 = exp2f(sc[0] - a.m[0]), e1 = exp2f(sc[1] - a.m[1]);
        const float e2 = exp2f(sc[2] - a.m[0]), e3 = exp2f(sc[3] - a.m[1]);
        a.l[0] += e0 + e2;
        a.l[1] += e1 + e3;
        // P^T columns: t == 0 -> bf16(p), t == 1 -> remainder, t >= 2 -> 0
        uint32_t pa, pb;
        if (t == 0) {
            pa = pack2_bf16(e0, e1);
            pb = pack2_bf16(e2, e3);
        } else if (t == 1) {
            pa = pack2_bf16(e0 - bf16_round(e0), e1 - bf16_round(e1));
            pb = pack2_bf16(e2 - bf16_round(e2), e3 - bf16_round(e3));
        } else {
            pa = pb = 0u;
        }
        const uint32_t pb0 = movm_t(pa), pb1 = movm_t(pb);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint4 v0 = va ? *reinterpret_cast<const uint4*>(vb + ra * (D * 2) + 64 * u + 16 * t) : make_uint4(0, 0, 0, 0);
            const uint4 v1 = vbk ? *reinterpret_cast<const uint4*>(vb + rb * (D * 2) + 64 * u + 16 * t) : make_uint4(0, 0, 0, 0);
            const uint32_t r0[4] = {v0.x, v0.y, v0.z, v0.w};
            const uint32_t r1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                float* o = a.o[u][qq];
                o[0] *= corr[0]; o[1] *= corr[1]; o[2] *= corr[0]; o[3] *= corr[1];
                const uint32_t av[4] = {movm_t(r0[qq]), movm_t(r0[qq + 2]), movm_t(r1[qq]), movm_t(r1[qq + 2])};
                mma16816(o, av, pb0, pb1);
            }
        }
    }

    // The attention unit's cached positions: K/V tiles of KV_TILE positions (the
    // tiling of for_tiles), consumed MV_GROUP stages at a time so that 12 of
    // the 15 warps work at once: warp w takes 16-position group w % 4 of tile
    // w / 4 of the batch.
    __device__ __forceinline__ void attn_phase(AttnState& a, int l) {
        const int ntiles = (S.kv_e - S.kv_s + KV_TILE - 1) / KV_TILE;
        for (int g0 = 0; g0 < ntiles; g0 += MV_GROUP) {
            const int g1 = min(ntiles, g0 + MV_GROUP);
            bool got = true;
            for (int i = g0; i < g1; ++i) {
                const uint32_t t = n + (uint32_t)(i - g0);
                got = wait_full(t % NSTAGES, (t / NSTAGES) & 1u, PH_ATTN, l) && got;
            }
            if (got) {
                const int ti = g0 + (warp >> 2), grp = warp & 3;
                if (ti < g1) {
                    const int nrows = min(S.kv_e - (S.kv_s + ti * KV_TILE), KV_TILE);
                    if (grp * 16 < nrows) {
                        const uint8_t* st = g_smem + SM_STAGES + ((n + (uint32_t)(ti - g0)) % NSTAGES) * STAGE_BYTES;
                        attn_group(a, st, st + nrows * D * 2, grp, nrows);
                    }
                }
                for (int i = g0; i < g1; ++i) release((n + (uint32_t)(i - g0)) % NSTAGES);
            }
            n += (uint32_t)(g1 - g0);
        }
    }

    __device__ __forceinline__ void release(uint32_t s) {
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_relaxed(&empty()[s]);
        }
    }

    // Trace slots 340 + 5 l + k of the attention phase (k: 0 q fragments built,
    // 1 start of tiles, 2 tiles done, 3 local merge done, 4 phase done),
    // consumer thread 0.
    // clock64 micro-stamps inside the phases of layer 14 (slots 1792 + phase*24 + k)
    __device__ __forceinline__ void micro(int l, int phase, int k) {
        if (kGT && P.trace && l == 14 && ct == 0) P.trace[(size_t)S.c * TRACE_STRIDE + 1792 + phase * 24 + k] = clock64();
    }
    __device__ __forceinline__ void attn_stamp(int l, int k) {
        if (kGT && P.trace && ct == 0) P.trace[(size_t)S.c * TRACE_STRIDE + 340 + 5 * l + k] = globaltimer_ns();
    }

    __device__ __forceinline__ void end_attn(AttnState& a, int l) {
        float* acc = reinterpret_cast<float*>(g_smem + SM_ACC);   // [16][2][128]
        float* ml = reinterpret_cast<float*>(g_smem + SM_ML);     // [16][2][2]
        const int g = lane >> 2, t = lane & 3;
        // this warp: row-group sums, then hi + lo accumulator columns
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            a.l[0] += __shfl_xor_sync(0xffffffffu, a.l[0], o);
            a.l[1] += __shfl_xor_sync(0xffffffffu, a.l[1], o);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int qq = 0; qq < 2; ++qq)
#pragma unroll
                for (int i = 0; i < 4; ++i) a.o[u][qq][i] += __shfl_xor_sync(0xffffffffu, a.o[u][qq][i], 1);
        if (t == 0) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const int d0 = attn_vdim(u, qq, g), d1 = attn_vdim(u, qq + 2, g);
                    acc[(warp * 2 + 0) * D + d0] = a.o[u][qq][0];
                    acc[(warp * 2 + 1) * D + d0] = a.o[u][qq][1];
                    acc[(warp * 2 + 0) * D + d1] = a.o[u][qq][2];
                    acc[(warp * 2 + 1) * D + d1] = a.o[u][qq][3];
                }
        }
        if (lane == 0) {
            ml[warp * 4 + 0] = a.m[0]; ml[warp * 4 + 1] = a.l[0];
            ml[warp * 4 + 2] = a.m[1]; ml[warp * 4 + 3] = a.l[1];
        }
    }

    // A unit of more than KV_TILE cached positions: the tensor-core path
    // (mma.sync m16n8k16 over 16-position groups, q and p as bf16 hi + lo).
    __device__ __forceinline__ void attn_long(int l) {
        AttnState a;
        const float* qn = sm<float>(SM_QN);
        const float sc = P.attn_scale * 1.4426950408889634f;   // log2 domain
        uint32_t* qbs = sm<uint32_t>(SM_QKVRAW);
        // word w = (k-step * 32 + lane') * 2 + j of the B fragments, one or two per thread;
        // column g' = lane' / 4: head g' & 1, hi (g' < 2) or remainder (g' < 4), else 0
        for (int w = ct; w < 512; w += NCT) {
            const int jj = w & 1, lw = (w >> 1) & 31, ks = w >> 6;
            const int gw = lw >> 2, tw = lw & 3;
            const int d0 = 32 * (ks >> 1) + 8 * tw + 4 * (ks & 1) + 2 * jj;
            const float* q = qn + (gw & 1) * D;
            const float x0 = q[d0] * sc, x1 = q[d0 + 1] * sc;
            const float h0 = bf16_round(x0), h1 = bf16_round(x1);
            qbs[w] = gw < 2 ? pack2_bf16(h0, h1) : gw < 4 ? pack2_bf16(x0 - h0, x1 - h1) : 0u;
        }
        attn_stamp(l, 0);
        named_bar_sync(BAR_CONSUMERS, NCT);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) a.o[u][qq][0] = a.o[u][qq][1] = a.o[u][qq][2] = a.o[u][qq][3] = 0.f;
        a.m[0] = a.m[1] = -INFINITY;
        a.l[0] = a.l[1] = 0.f;
        attn_stamp(l, 1);
        attn_phase(a, l);
        end_attn(a, l);
    }

    // Attention of one unit in plain fp32, for units of up to
    // ATTN_FP32_MAX_TILES staged tiles: warp w takes positions w, w + 15, ..
    // of each 64-position tile, so all 15 warps work and no q fragments,
    // transposes or fragment reductions are needed.  Lane owns head dims
    // 4 lane .. 4 lane + 3 of both q heads; scores are in the log2 domain like
    // the tensor-core path's, and a warp's (max, sum, acc) is carried across
    // tiles with the usual online-softmax rescale.  The warp's state goes to
    // its entry slot for finish_attn.
    __device__ __forceinline__ void attn_fp32(int l) {
        constexpr int RPW = (KV_TILE + NCW - 1) / NCW;   // positions per warp and tile (5)
        float* acc = reinterpret_cast<float*>(g_smem + SM_ACC);
        float* ml = reinterpret_cast<float*>(g_smem + SM_ML);
        const float sc = P.attn_scale * 1.4426950408889634f;
        const float4 qa = *reinterpret_cast<const float4*>(sm<float>(SM_QN) + 4 * lane);
        const float4 qb = *reinterpret_cast<const float4*>(sm<float>(SM_QN) + D + 4 * lane);
        const int total = S.kv_e - S.kv_s;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int t0 = 0; t0 < total; t0 += KV_TILE) {
            const int nrows = min(total - t0, KV_TILE);
            const bool got = wait_full(n % NSTAGES, (n / NSTAGES) & 1u, PH_ATTN, l);
            if (got && warp < nrows) {
                const uint8_t* kb = g_smem + SM_STAGES + (n % NSTAGES) * STAGE_BYTES;
                const uint8_t* vb = kb + nrows * D * 2;
                float s0[RPW], s1[RPW];
#pragma unroll
                for (int i = 0; i < RPW; ++i) {
                    const int r = warp + NCW * i;
                    s0[i] = s1[i] = 0.f;
                    if (r < nrows) {
                        const uint2 kw = *reinterpret_cast<const uint2*>(kb + r * (D * 2) + 8 * lane);
                        const float k0 = bf16lo(kw.x), k1 = bf16hi(kw.x), k2 = bf16lo(kw.y), k3 = bf16hi(kw.y);
                        s0[i] = qa.x * k0 + qa.y * k1 + qa.z * k2 + qa.w * k3;
                        s1[i] = qb.x * k0 + qb.y * k1 + qb.z * k2 + qb.w * k3;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int i = 0; i < RPW; ++i) {
                        s0[i] += __shfl_xor_sync(0xffffffffu, s0[i], o);
                        s1[i] += __shfl_xor_sync(0xffffffffu, s1[i], o);
                    }
                float t0m = m0, t1m = m1;
#pragma unroll
                for (int i = 0; i < RPW; ++i) {
                    if (warp + NCW * i < nrows) {
                        s0[i] *= sc;
                        s1[i] *= sc;
                        t0m = fmaxf(t0m, s0[i]);
                        t1m = fmaxf(t1m, s1[i]);
                    }
                }
                const float c0 = exp2f(m0 - t0m), c1 = exp2f(m1 - t1m);   // 0 on the first tile
                m0 = t0m;
                m1 = t1m;
                l0 *= c0;
                l1 *= c1;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    a0[j] *= c0;
                    a1[j] *= c1;
                }
#pragma unroll
                for (int i = 0; i < RPW; ++i) {
                    const int r = warp + NCW * i;
                    if (r < nrows) {
                        const float e0 = exp2f(s0[i] - m0), e1 = exp2f(s1[i] - m1);
                        l0 += e0;
                        l1 += e1;
                        const uint2 vw = *reinterpret_cast<const uint2*>(vb + r * (D * 2) + 8 * lane);
                        const float v[4] = {bf16lo(vw.x), bf16hi(vw.x), bf16lo(vw.y), bf16hi(vw.y)};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            a0[j] = fmaf(e0, v[j], a0[j]);
                            a1[j] = fmaf(e1, v[j], a1[j]);
                        }
                    }
                }
            }
            release(n % NSTAGES);
            n += 1;
        }
        *reinterpret_cast<float4*>(acc + (warp * 2 + 0) * D + 4 * lane) = make_float4(a0[0], a0[1], a0[2], a0[3]);
        *reinterpret_cast<float4*>(acc + (warp * 2 + 1) * D + 4 * lane) = make_float4(a1[0], a1[1], a1[2], a1[3]);
        if (lane == 0) {
            ml[warp * 4 + 0] = m0; ml[warp * 4 + 1] = l0;
            ml[warp * 4 + 2] = m1; ml[warp * 4 + 3] = l1;
        }
    }

    // Merge of the unit's warp entries (+ the current position), then the
    // split-K publish / combine (both attention paths).
    __device__ __forceinline__ void finish_attn(int l) {
        float* acc = reinterpret_cast<float*>(g_smem + SM_ACC);   // [16][2][128]
        float* ml = reinterpret_cast<float*>(g_smem + SM_ML);     // [16][2][2]
        if (warp == NCW - 1) {
            // entry NCW: the current position (last unit only), fp32 q.k of the
            // bf16-rounded k/v held in shared memory
            const bool cur = ok && S.last;
            const float* qn = sm<float>(SM_QN);
            const float* kp = reinterpret_cast<const float*>(g_smem + SM_KP);
            const float* vp = reinterpret_cast<const float*>(g_smem + SM_VP);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                s0 += qn[4 * lane + i] * kp[4 * lane + i];
                s1 += qn[D + 4 * lane + i] * kp[4 * lane + i];
            }
            s0 = warp_sum(s0) * (P.attn_scale * 1.4426950408889634f);
            s1 = warp_sum(s1) * (P.attn_scale * 1.4426950408889634f);
            if (lane == 0) {
                ml[NCW * 4 + 0] = cur ? s0 : -INFINITY; ml[NCW * 4 + 1] = cur ? 1.f : 0.f;
                ml[NCW * 4 + 2] = cur ? s1 : -INFINITY; ml[NCW * 4 + 3] = cur ? 1.f : 0.f;
            }
            const float4 v4 = cur ? *reinterpret_cast<const float4*>(vp + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(acc + (NCW * 2 + 0) * D + 4 * lane) = v4;
            *reinterpret_cast<float4*>(acc + (NCW * 2 + 1) * D + 4 * lane) = v4;
        }
        named_bar_sync(BAR_CONSUMERS, NCT);
        const int h = warp;  // warps 0 and 1 combine heads 0 and 1
        const uint32_t tag = tag_of(S, l);
        // Pass 0 merges this unit's warps (+ the current position).  With C > 1
        // the units j >= 1 publish that partial as tagged words and leave; unit
        // 0 (the kv head's combiner) polls them into the same entry slots and
        // pass 1 merges them with its own partial.
        for (int pass = 0;; ++pass) {
            float M = -INFINITY, Ls = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
            if (warp < 2) {
                // lane w <= NCW holds entry w's (max, sum); the weights are shuffled to all lanes
                const float mw = lane <= NCW ? ml[lane * 4 + 2 * h] : -INFINITY;
                M = mw;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
                const float ew = mw == -INFINITY ? 0.f : exp2f(mw - M);   // entries without positions weigh 0
                Ls = warp_sum(lane <= NCW ? ml[lane * 4 + 2 * h + 1] * ew : 0.f);
#pragma unroll
                for (int w = 0; w <= NCW; ++w) {
                    const float e = __shfl_sync(0xffffffffu, ew, w);
                    const float4 av = *reinterpret_cast<const float4*>(acc + (w * 2 + h) * D + 4 * lane);
                    A[0] += av.x * e; A[1] += av.y * e; A[2] += av.z * e; A[3] += av.w * e;
                }
            }
            if (S.C == 1 || pass == 1) {
                if (warp < 2 && ok) {
                    uint64_t* out = ll_attn(P, l) + 256 * S.ug;
                    const float inv = 1.0f / Ls;
#pragma unroll
                    for (int i = 0; i < 4; ++i) ll_store(out + h * D + 4 * lane + i, ll_word(A[i] * inv, tag));
                }
                return;
            }
            if (S.uj != 0) {
                if (warp < 2 && ok) {
                    uint64_t* pw = part_of(P, S.ug, S.uj, h);
#pragma unroll
                    for (int i = 0; i < 4; ++i) ll_store(pw + 4 * lane + i, ll_word(A[i], tag));
                    if (lane == 0) {
                        ll_store(pw + 128, ll_word(M, tag));
                        ll_store(pw + 129, ll_word(Ls, tag));
                    }
                }
                return;
            }
            attn_stamp(l, 3);
            named_bar_sync(BAR_CONSUMERS, NCT);   // pass 0 is done reading the entry slots
            if (warp < 2) {
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[(NCW * 2 + h) * D + 4 * lane + i] = A[i];
                if (lane == 0) { ml[NCW * 4 + 2 * h] = M; ml[NCW * 4 + 2 * h + 1] = Ls; }
            }
            gather_partials(l, tag, acc, ml);
            named_bar_sync(BAR_CONSUMERS, NCT);
        }
    }

    // Combiner (unit 0 of a kv head, C > 1): warp w polls the tagged partials of
    // units 1 + w, 1 + w + NCW, .. (all words of a unit in flight at once),
    // merges them and stores the result in entry slot w (max -inf: empty).
    __device__ __forceinline__ void gather_partials(int l, uint32_t tag, float* acc, float* ml) {
        float mm[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f}, am[2][4] = {};
        for (int r = 0; r < (CMAX - 1 + NCW - 1) / NCW; ++r) {
            const int j = 1 + warp + r * NCW;
            if (j >= S.C) break;   // warp-uniform
            const uint64_t* p0 = part_of(P, S.ug, j, 0);
            const uint64_t* p1 = part_of(P, S.ug, j, 1);
            uint64_t w[9];
            uint32_t pending = lane < 4 ? 0x1ffu : 0xffu;
            uint64_t t0 = 0;
            uint32_t spins = 0;
            while (ok && pending) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (pending & (1u << i)) w[i] = ld_relaxed_u64(p0 + 4 * lane + i);
                    if (pending & (1u << (4 + i))) w[4 + i] = ld_relaxed_u64(p1 + 4 * lane + i);
                }
                if (pending & 0x100u) w[8] = ld_relaxed_u64((lane < 2 ? p0 : p1) + 128 + (lane & 1));
#pragma unroll
                for (int i = 0; i < 9; ++i)
                    if ((pending & (1u << i)) && (uint32_t)(w[i] >> 32) == tag) pending &= ~(1u << i);
                if (pending && ((++spins & 31u) == 0)) {
                    uint64_t now = globaltimer_ns();
                    if (t0 == 0) t0 = now;
                    if (flags()[0] != 0 || global_error(P)) { ok = false; break; }
                    if ((long long)(now - t0) > P.timeout_ns) { fail(MQ_ERR_WAIT_TIMEOUT, ((uint32_t)PH_ATTN << 8) | l); break; }
                }
            }
            const float mlv = __uint_as_float((uint32_t)w[8]);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const float mj = __shfl_sync(0xffffffffu, mlv, 2 * hh), lj = __shfl_sync(0xffffffffu, mlv, 2 * hh + 1);
                const float nm = fmaxf(mm[hh], mj);
                const float c0 = mm[hh] == -INFINITY ? 0.f : exp2f(mm[hh] - nm), c1 = exp2f(mj - nm);
#pragma unroll
                for (int i = 0; i < 4; ++i) am[hh][i] = am[hh][i] * c0 + __uint_as_float((uint32_t)w[4 * hh + i]) * c1;
                lsum[hh] = lsum[hh] * c0 + lj * c1;
                mm[hh] = nm;
            }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[(warp * 2 + hh) * D + 4 * lane + i] = am[hh][i];
            if (lane == 0) { ml[warp * 4 + 2 * hh] = mm[hh]; ml[warp * 4 + 2 * hh + 1] = lsum[hh]; }
        }
    }

    __device__ __forceinline__ void end_lm(const LmBest& best) {
        float* bv = reinterpret_cast<float*>(g_smem + SM_BEST);
        int* bi = reinterpret_cast<int*>(g_smem + SM_BEST) + NCW;
        float v = best.v;
        int i = best.i;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, v, o);
            int oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        if (lane == 0) { bv[warp] = v; bi[warp] = i; }
        if (!agree()) return;
        if (ct == 0) {
            float v = bv[0];
            int i = bi[0];
            for (int w = 1; w < NCW; ++w)
                if (bv[w] > v || (bv[w] == v && bi[w] < i)) { v = bv[w]; i = bi[w]; }
            uint32_t u = __float_as_uint(v);
            uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            unsigned long long key = ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
            Control* C = ctrl_of(P);
            atomicMax(&C->lm_best, key);
            __threadfence();
            uint32_t old = atomicAdd(&C->lm_count, 1u);
            if (old == (uint32_t)(S.G - 1)) {
                __threadfence();
                unsigned long long best = atomicExch(&C->lm_best, 0ull);
                atomicExch(&C->lm_count, 0u);
                if (TP_(tp, 1) > 1) {
                    // the ranks' best keys: {key, tag} into every rank's slot,
                    // then the maximum over all slots (bounded waits)
                    const uint64_t stag = (uint64_t)(uint32_t)S.tag_base;
                    for (int r = 0; r < TP_(tp, 1); ++r) {
                        uint64_t* slot = lmx_of(P.peer_ws[r], TP_(rank, 0));
                        st_relaxed_sys_u64(slot, best);
                        st_release_sys_u64(slot + 1, stag);
                    }
                    const uint64_t t0 = globaltimer_ns();
                    for (int r = 0; r < TP_(tp, 1); ++r) {
                        const uint64_t* slot = lmx_of(P.ws, r);
                        uint32_t spins = 0;
                        while (ld_acquire_sys_u64(slot + 1) != stag) {
                            if ((++spins & 31u) == 0 &&
                                (global_error(P) || (long long)(globaltimer_ns() - t0) > P.timeout_ns)) {
                                if (!global_error(P)) record_error(P, MQ_ERR_WAIT_TIMEOUT, ((uint32_t)PH_LM << 8) | 0x80u);
                                return;
                            }
                        }
                        const unsigned long long k2 = ld_relaxed_sys_u64(slot);
                        if (k2 > best) best = k2;
                    }
                }
                int tok = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
                if (P.output_token) *P.output_token = tok;
                if (P.host_result) {
                    // token, error, info first, then the sequence word the host waits on
                    volatile mq_host_result* hr = P.host_result;
                    hr->token = tok;
                    hr->error = ld_relaxed_u32(&C->error);
                    hr->info = C->info;
                    __threadfence_system();
                    hr->seq = P.host_seq;
                    __threadfence_system();
                }
                C->last_token = tok;
                C->last_position = S.pos;
                if (P.position_ptr) *P.position_ptr = S.pos + 1;
                // The tags of this step's words are (epoch + 1) << 6 | layer, so the
                // counter wraps after 2^25 steps (the tag stays within 32 bits).  A
                // wrap is harmless: a handoff slot read in a step is written in that
                // step, and the word it held before came from the previous step (a
                // different epoch) or, for attention partials of a chunk index the
                // previous step did not use, from an older step, which would have to be
                // exactly 2^25 steps old to match.  A failed step leaves the epoch as
                // it is and the host zeroes the whole workspace before the next one.
                C->epoch = (C->epoch + 1u) & ((1u << 25) - 1u);
                __threadfence();
            }
        }
    }
};

// Consumer progress between phase calls: tiles consumed (bits 0-23), block-sum
// parity (bit 24), this thread failed (bit 25), stop the walk (bit 26).
template <int KIND, bool MT>
__device__ __noinline__ uint32_t consumer_phase(const KParams* P, int phase, int l, uint32_t st) {
    Consumer<MT> c(*P, *sm<Sched>(SM_SCHED));
    c.n = st & 0xffffffu;
    c.red_par = (st >> 24) & 1u;
    c.ok = ((st >> 25) & 1u) == 0;
    const bool go = c.template run<KIND>(phase, l);
    return (c.n & 0xffffffu) | ((uint32_t)c.red_par << 24) | (c.ok ? 0u : (1u << 25)) | (go ? 0u : (1u << 26));
}

// Walk visitor for the consumer warps: each phase kind is its own function so
// the register allocator sees one phase at a time (no spills).
template <bool MT>
struct ConsumerWalk {
    const KParams* P;
    uint32_t st = 0;
    __device__ bool run(int phase, int l) {
        if (phase == PH_ATTN) st = consumer_phase<1, MT>(P, phase, l, st);
        else if (phase == PH_LM) st = consumer_phase<2, MT>(P, phase, l, st);
        else if (phase == PH_O || phase == PH_DOWN) st = consumer_phase<3, MT>(P, phase, l, st);
        else st = consumer_phase<0, MT>(P, phase, l, st);
        return (st & (1u << 26)) == 0;
    }
};

// MT: the tensor-parallel instantiation (tp_size > 1); the single-GPU one is
// compiled with the partition sizes as constants.
template <bool MT>
__global__ void __launch_bounds__(NTHREADS, 1) decode_step_kernel(const __grid_constant__ KParams P) {
    Control* C = ctrl_of(P);
    volatile int* flags = sm<volatile int>(SM_FLAGS);
    const int pos = P.position_ptr ? *P.position_ptr : P.position;
    const int tok = P.input_token_ptr ? *P.input_token_ptr : P.input_token;
    if (pos < 0 || pos >= P.max_seq_len) {
        if (blockIdx.x == 0 && threadIdx.x == 0) record_error(P, MQ_ERR_BAD_POSITION, (uint32_t)pos);
        return;
    }
    if (tok < 0 || tok >= V) {
        if (blockIdx.x == 0 && threadIdx.x == 0) record_error(P, MQ_ERR_BAD_TOKEN, (uint32_t)tok);
        return;
    }

    // The CTA's slice of every phase lives in shared memory (not registers).
    Sched& S = *sm<Sched>(SM_SCHED);
    if (threadIdx.x == 0) {
        S.G = gridDim.x;
        S.c = blockIdx.x;
        S.pos = pos;
        S.L = pos + 1;
        S.tag_base = (int)((C->epoch + 1u) << 6);
        // tensor parallel (T ranks, this one `rank`): q/k/v rows and the
        // attention of kv heads [8 rank / T, 8 (rank + 1) / T); O and down
        // rows over this rank's input slice (row-parallel partials); gate/up
        // rows and LM rows of this rank's slice.  T = 1: the whole model.
        const int T = P.tp, rk = P.rank;
        S.tp = T;
        S.rank = rk;
        S.qt = QS / T;  S.kt = KVS / T;
        S.q0 = S.qt * rk; S.k0 = S.kt * rk;
        S.ia = I / T;   S.ia_a = S.ia * rk;
        S.o_tile = min(NCW, STAGE_BYTES / (S.qt * 2));
        S.dn_tile = min(NCW, STAGE_BYTES / (S.ia * 2));
        const int nq = S.qt + 2 * S.kt;
        S.qkv_a = split_at(nq, S.G, S.c);  S.qkv_b = split_at(nq, S.G, S.c + 1);
        S.o_a = split_at(H, S.G, S.c);     S.o_b = split_at(H, S.G, S.c + 1);
        S.gu_a = S.ia_a + split_at(S.ia, S.G, S.c);
        S.gu_b = S.ia_a + split_at(S.ia, S.G, S.c + 1);
        S.dn_a = S.o_a;                    S.dn_b = S.o_b;
        const int va = (int)((long long)V * rk / T), vb = (int)((long long)V * (rk + 1) / T);
        S.lm_a = va + split_at(vb - va, S.G, S.c);
        S.lm_b = va + split_at(vb - va, S.G, S.c + 1);
        const int chunk = P.attn_chunk > 0 ? P.attn_chunk : 64;
        int C_ = (S.L + chunk - 1) / chunk;
        const int NH = NKV / T;   // kv heads of this rank
        C_ = min(C_, S.G / NH);
        C_ = min(C_, CMAX);
        C_ = max(C_, 1);
        S.C = C_;
        const int U = NH * C_;
        const int u = (int)(((long long)S.c * U + S.G - 1) / S.G);
        S.has_unit = (u < U) && (int)(((long long)u * S.G) / U) == S.c;
        S.ug = NH * rk + u / C_;
        S.uj = u % C_;
        const int ps = split_at(S.L, C_, S.uj), pe = split_at(S.L, C_, S.uj + 1);
        S.last = (S.uj == C_ - 1);
        S.kv_s = ps;
        S.kv_e = S.last ? pe - 1 : pe;   // the current position comes from registers, not the cache

        uint64_t* full = sm<uint64_t>(SM_BARS);
        uint64_t* empty = full + NSTAGES;
        for (int s = 0; s < NSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        fence_mbar_init();
        flags[0] = 0;
        flags[1] = tok;
        flags[2] = 0;
    }
    {
        // per-layer pointer table -> shared memory (read at every phase start)
        const uint64_t* src = reinterpret_cast<const uint64_t*>(P.layers);
        uint64_t* dst = sm<uint64_t>(SM_LAYERS);
        const int words = P.num_layers * (int)(sizeof(LDGLayerWeights) / 8);
        for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    }
    {
        // The phases read their parameters from a shared-memory copy: kernel
        // parameters live in the constant bank, whose cache shares the SM's
        // instruction/constant cache with this kernel's large code and misses
        // (an L2 round trip per parameter read) between phases.
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&P);
        uint32_t* dst = sm<uint32_t>(SM_PARAMS);
        for (int i = threadIdx.x; i < (int)(sizeof(KParams) / 4); i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    const KParams& Ps = *sm<KParams>(SM_PARAMS);

    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) {
            Producer<MT> pr(Ps, g_smem);
            walk(Ps, S, pr);
            if (P.trace) P.trace[(size_t)blockIdx.x * TRACE_STRIDE + 502] = globaltimer_ns();
            pr.drain();
        }
        return;
    }
    ConsumerWalk<MT> cs{&Ps};
    if (P.trace && threadIdx.x == 32) P.trace[(size_t)blockIdx.x * TRACE_STRIDE + 500] = globaltimer_ns();
    walk(Ps, S, cs);
    if (P.trace && threadIdx.x == 32) P.trace[(size_t)blockIdx.x * TRACE_STRIDE + 501] = globaltimer_ns();
}

#undef TP_

}  // namespace mq

// =============================================================================
// Host side: C ABI
// =============================================================================

namespace {

thread_local int g_last_error = MQ_OK;
thread_local char g_detail[256] = "";

// Record which CUDA call failed and why; returns MQ_ERR_CUDA.
int cuda_fail(cudaError_t e, const char* what) {
    snprintf(g_detail, sizeof(g_detail), "%s: %s", what, cudaGetErrorString(e));
    return MQ_ERR_CUDA;
}

int note(int code, const char* what) {
    snprintf(g_detail, sizeof(g_detail), "%s", what);
    return code;
}

struct DeviceWorkspace {
    void* ptr = nullptr;
};
std::mutex g_ws_mutex;
std::vector<DeviceWorkspace> g_ws;  // one default workspace per device

int set_err(int e) {
    g_last_error = e;
    return e;
}

bool kernel_configured[64] = {false};

int configure_kernel(int dev) {
    if (dev >= 0 && dev < 64 && kernel_configured[dev]) return MQ_OK;
    for (auto kern : {mq::decode_step_kernel<false>, mq::decode_step_kernel<true>}) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, mq::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic shared memory)");
    }
    if (dev >= 0 && dev < 64) kernel_configured[dev] = true;
    return MQ_OK;
}

int default_ctas(int dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    int n = sms < mq::MAX_CTAS ? sms : mq::MAX_CTAS;
    return n;
}

void* default_workspace(int dev, cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_ws_mutex);
    if ((int)g_ws.size() <= dev) g_ws.resize(dev + 1);
    if (!g_ws[dev].ptr) {
        void* p = nullptr;
        if (cudaMalloc(&p, mq::WS_BYTES) != cudaSuccess) return nullptr;
        if (cudaMemsetAsync(p, 0, mq::WS_BYTES, stream) != cudaSuccess) return nullptr;
        g_ws[dev].ptr = p;
    }
    return g_ws[dev].ptr;
}

int launch(const mq_decode_params* p, cudaStream_t stream) {
    if (!p || !p->embed || !p->layers || !p->final_norm || !p->lm_head || !p->cos_table || !p->sin_table ||
        !p->k_cache || !p->v_cache)
        return MQ_ERR_INVALID_ARGUMENT;
    if (!p->workspace || p->workspace_bytes < mq::WS_BYTES) return MQ_ERR_WORKSPACE;
    if (p->num_layers < 1 || p->num_layers > MQ_MAX_LAYERS || p->max_seq_len < 1) return MQ_ERR_INVALID_ARGUMENT;
    if (!p->position_ptr && (p->position < 0 || p->position >= p->max_seq_len)) return MQ_ERR_INVALID_ARGUMENT;
    if (!p->input_token_ptr && (p->input_token < 0 || p->input_token >= MQ_VOCAB_SIZE))
        return MQ_ERR_INVALID_ARGUMENT;
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
    // Per-device set-up (kernel attribute, SM count, occupancy check), once.
    static int dev_ctas[64] = {0};
    if (dev < 0 || dev >= 64) return note(MQ_ERR_INVALID_ARGUMENT, "device index above 63");
    if (!dev_ctas[dev]) {
        int rc = configure_kernel(dev);
        if (rc) return rc;
        int maxb = 0;
        ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&maxb, mq::decode_step_kernel<true>, mq::NTHREADS, mq::SMEM_BYTES);
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (maxb < 1) return note(MQ_ERR_CUDA, "decode kernel does not fit on one SM (occupancy 0)");
        dev_ctas[dev] = default_ctas(dev);
    }
    int G = p->num_ctas > 0 ? p->num_ctas : dev_ctas[dev];
    if (G < mq::NKV || G > mq::MAX_CTAS) return MQ_ERR_INVALID_ARGUMENT;
    const int T = p->tp_size > 0 ? p->tp_size : 1;
    if (T != 1 && T != 2 && T != 4 && T != 8) return note(MQ_ERR_INVALID_ARGUMENT, "tp_size must be 1, 2, 4 or 8");
    if (p->tp_rank < 0 || p->tp_rank >= T) return note(MQ_ERR_INVALID_ARGUMENT, "tp_rank out of range");
    if (T > 1 && !p->peer_workspaces) return note(MQ_ERR_INVALID_ARGUMENT, "tp_size > 1 needs peer_workspaces");
    mq::KParams k;
    std::memset(&k, 0, sizeof(k));
    k.tp = T;
    k.rank = p->tp_rank;
    for (int r = 0; r < T; ++r) {
        k.peer_ws[r] = T == 1 ? (uint8_t*)p->workspace : (uint8_t*)p->peer_workspaces[r];
        if (!k.peer_ws[r]) return note(MQ_ERR_INVALID_ARGUMENT, "peer_workspaces holds a null pointer");
    }
    if (k.peer_ws[p->tp_rank] != (uint8_t*)p->workspace)
        return note(MQ_ERR_INVALID_ARGUMENT, "peer_workspaces[tp_rank] must be this rank's workspace");
    k.input_token = p->input_token;
    k.input_token_ptr = p->input_token_ptr;
    k.output_token = p->output_token;
    k.logits = p->logits;
    k.embed = (const mq::bf16*)p->embed;
    k.layers = p->layers;
    k.final_norm = (const mq::bf16*)p->final_norm;
    k.lm_head = (const mq::bf16*)p->lm_head;
    k.cos_table = (const mq::bf16*)p->cos_table;
    k.sin_table = (const mq::bf16*)p->sin_table;
    k.k_cache = (mq::bf16*)p->k_cache;
    k.v_cache = (mq::bf16*)p->v_cache;
    k.hidden_out = (mq::bf16*)p->hidden_out;
    k.norm_out = p->normalized_out;
    k.ws = (uint8_t*)p->workspace;
    k.num_layers = p->num_layers;
    k.position = p->position;
    k.position_ptr = p->position_ptr;
    k.max_seq_len = p->max_seq_len;
    k.attn_scale = p->attn_scale;
    k.attn_chunk = p->attn_chunk;
    k.timeout_ns = p->timeout_ns > 0 ? p->timeout_ns : 2000000000ll;
    k.inject_skip_cta = p->inject_skip_cta;
    k.trace = p->trace;
    k.host_result = p->host_result;
    k.host_seq = p->host_seq;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(mq::NTHREADS);
    cfg.dynamicSmemBytes = mq::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;   // always cooperative: the CTAs wait on each other, so all must be resident
    cudaError_t e = T > 1 ? cudaLaunchKernelEx(&cfg, mq::decode_step_kernel<true>, k)
                          : cudaLaunchKernelEx(&cfg, mq::decode_step_kernel<false>, k);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(decode_step_kernel, cooperative)");
    return MQ_OK;
}

void launch_ref_abi(int input_token_id, int* output_token_id, float* logits, const void* embed_weight,
                    const LDGLayerWeights* layer_weights, const void* final_norm_weight, const void* lm_head_weight,
                    const void* cos_table, const void* sin_table, void* k_cache, void* v_cache, void* hidden_buffer,
                    void* g_normalized, int num_layers, int position, int cache_len, int max_seq_len, float attn_scale,
                    cudaStream_t stream) {
    if (cache_len != position + 1) { set_err(MQ_ERR_INVALID_ARGUMENT); return; }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_err(MQ_ERR_CUDA); return; }
    void* ws = default_workspace(dev, stream);
    if (!ws) { set_err(MQ_ERR_CUDA); return; }
    mq_decode_params p = {};
    p.input_token = input_token_id;
    p.output_token = output_token_id;
    p.logits = logits;
    p.embed = embed_weight;
    p.layers = layer_weights;
    p.final_norm = final_norm_weight;
    p.lm_head = lm_head_weight;
    p.cos_table = cos_table;
    p.sin_table = sin_table;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.hidden_out = hidden_buffer;
    p.normalized_out = (float*)g_normalized;
    p.workspace = ws;
    p.workspace_bytes = mq::WS_BYTES;
    p.num_layers = num_layers;
    p.position = position;
    p.max_seq_len = max_seq_len;
    p.attn_scale = attn_scale;
    set_err(launch(&p, stream));
}

}  // namespace

extern "C" {

void launch_ldg_decode(int input_token_id, int* output_token_id, const void* embed_weight,
                       const LDGLayerWeights* layer_weights, const void* final_norm_weight,
                       const void* lm_head_weight, const void* cos_table, const void* sin_table, void* k_cache,
                       void* v_cache, void* hidden_buffer, void* /*g_activations*/, void* /*g_residual*/,
                       void* /*g_q*/, void* /*g_k*/, void* /*g_v*/, void* /*g_attn_out*/,
                       void* /*g_mlp_intermediate*/, void* g_normalized, void* /*block_max_vals*/,
                       void* /*block_max_idxs*/, int num_layers, int position, int cache_len, int max_seq_len,
                       float attn_scale, cudaStream_t stream) {
    launch_ref_abi(input_token_id, output_token_id, nullptr, embed_weight, layer_weights, final_norm_weight,
                   lm_head_weight, cos_table, sin_table, k_cache, v_cache, hidden_buffer, g_normalized, num_layers,
                   position, cache_len, max_seq_len, attn_scale, stream);
}

void launch_ldg_decode_with_logits(int input_token_id, int* output_token_id, float* logits_output,
                                   const void* embed_weight, const LDGLayerWeights* layer_weights,
                                   const void* final_norm_weight, const void* lm_head_weight, const void* cos_table,
                                   const void* sin_table, void* k_cache, void* v_cache, void* hidden_buffer,
                                   void* /*g_activations*/, void* /*g_residual*/, void* /*g_q*/, void* /*g_k*/,
                                   void* /*g_v*/, void* /*g_attn_out*/, void* /*g_mlp_intermediate*/,
                                   void* g_normalized, void* /*block_max_vals*/, void* /*block_max_idxs*/,
                                   int num_layers, int position, int cache_len, int max_seq_len, float attn_scale,
                                   cudaStream_t stream) {
    launch_ref_abi(input_token_id, output_token_id, logits_output, embed_weight, layer_weights, final_norm_weight,
                   lm_head_weight, cos_table, sin_table, k_cache, v_cache, hidden_buffer, g_normalized, num_layers,
                   position, cache_len, max_seq_len, attn_scale, stream);
}

size_t mq_decode_workspace_bytes(void) { return mq::WS_BYTES; }

int mq_decode_workspace_init(void* workspace, size_t bytes, cudaStream_t stream) {
    if (!workspace || bytes < mq::WS_BYTES) return MQ_ERR_WORKSPACE;
    return cudaMemsetAsync(workspace, 0, mq::WS_BYTES, stream) == cudaSuccess ? MQ_OK : MQ_ERR_CUDA;
}

int mq_decode(const mq_decode_params* params, cudaStream_t stream) { return launch(params, stream); }

namespace {
__global__ void set_epoch_kernel(mq::Control* c, uint32_t e) { c->epoch = e; }
}  // namespace

int mq_decode_workspace_set_epoch(void* workspace, uint32_t epoch, cudaStream_t stream) {
    if (!workspace) return MQ_ERR_WORKSPACE;
    if (epoch >= (1u << 25)) return MQ_ERR_INVALID_ARGUMENT;
    set_epoch_kernel<<<1, 1, 0, stream>>>(reinterpret_cast<mq::Control*>(workspace), epoch);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MQ_OK : cuda_fail(e, "set_epoch_kernel");
}

}  // extern "C"

// ---- decode without any allocation -------------------------------------------
// Scratch for mq_decode_noalloc: one workspace's worth (MQ_NOALLOC_SCRATCH_BYTES)
// in a file-scope device array.  Every GPU that loads this library holds it
// until the process exits.  In host code the symbol is only a stand-in; the
// device address comes from cudaGetSymbolAddress, taken once per device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[mq::WS_BYTES];
static_assert(mq::WS_BYTES == MQ_NOALLOC_SCRATCH_BYTES, "header states the static scratch size");

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {nullptr};
}  // namespace

extern "C" {

int mq_decode_noalloc(const mq_decode_params* params, cudaStream_t stream) {
    if (!params) return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc: params is NULL");
    if (params->num_ctas > mq::MAX_CTAS)
        return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc: num_ctas exceeds the 256 CTAs the static scratch holds");
    if (params->num_layers > MQ_MAX_LAYERS)
        return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc: num_layers exceeds the 63 layers the static scratch holds");
    if (params->tp_size > 1)
        return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc: tensor-parallel steps need caller workspaces (mq_decode)");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc: device index above 63");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mutex);
        if (!g_noalloc_ptr[dev]) {
            // First call on this device (device current): resolve the array's
            // device address and clear it.  No allocation happens.
            void* ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
            e = cudaMemsetAsync(ptr, 0, mq::WS_BYTES, stream);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static scratch)");
            g_noalloc_ptr[dev] = ptr;
        }
        scratch = g_noalloc_ptr[dev];
    }
    mq_decode_params p = *params;
    p.workspace = scratch;
    p.workspace_bytes = mq::WS_BYTES;
    return launch(&p, stream);
}

// The static scratch of this device, or null before the first
// mq_decode_noalloc call on it.
static void* noalloc_scratch_of_current_device(int* rc) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { *rc = cuda_fail(e, "cudaGetDevice"); return nullptr; }
    if (dev < 0 || dev >= 64) { *rc = note(MQ_ERR_INVALID_ARGUMENT, "device index above 63"); return nullptr; }
    std::lock_guard<std::mutex> lk(g_noalloc_mutex);
    *rc = MQ_OK;
    return g_noalloc_ptr[dev];
}

int mq_decode_noalloc_reset(cudaStream_t stream) {
    int rc = MQ_OK;
    void* ptr = noalloc_scratch_of_current_device(&rc);
    if (rc) return rc;
    if (!ptr) return MQ_OK;   // never used on this device: nothing to clear
    const cudaError_t e = cudaMemsetAsync(ptr, 0, mq::WS_BYTES, stream);
    return e == cudaSuccess ? MQ_OK : cuda_fail(e, "cudaMemsetAsync(static scratch)");
}

int mq_decode_noalloc_fetch(int* token, uint32_t* error, uint32_t* info, cudaStream_t stream) {
    int rc = MQ_OK;
    void* ptr = noalloc_scratch_of_current_device(&rc);
    if (rc) return rc;
    if (!ptr) return note(MQ_ERR_INVALID_ARGUMENT, "mq_decode_noalloc_fetch: no mq_decode_noalloc call on this device yet");
    mq::Control c;   // host stack: pageable copy, no pinned allocation
    cudaError_t e = cudaMemcpyAsync(&c, ptr, 32, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(static scratch result)");
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    if (token) *token = c.last_token;
    if (error) *error = c.error;
    if (info) *info = c.info;
    return MQ_OK;
}

int mq_decode_read_error(const void* workspace, uint32_t* error, uint32_t* info, cudaStream_t stream) {
    if (!workspace) return MQ_ERR_WORKSPACE;
    uint32_t h[3] = {0, 0, 0};
    if (cudaMemcpyAsync(h, workspace, sizeof(h), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return MQ_ERR_CUDA;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return MQ_ERR_CUDA;
    if (error) *error = h[1];
    if (info) *info = h[2];
    return MQ_OK;
}

int mq_decode_fetch(const void* workspace, int* token, uint32_t* error, uint32_t* info, cudaStream_t stream) {
    if (!workspace) return MQ_ERR_WORKSPACE;
    static thread_local uint32_t* pinned = nullptr;
    if (!pinned && cudaHostAlloc((void**)&pinned, 64, cudaHostAllocDefault) != cudaSuccess) return MQ_ERR_CUDA;
    cudaError_t e = cudaMemcpyAsync(pinned, workspace, 32, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(result)");
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    const mq::Control* c = reinterpret_cast<const mq::Control*>(pinned);
    if (token) *token = c->last_token;
    if (error) *error = c->error;
    if (info) *info = c->info;
    return MQ_OK;
}

int mq_decode_default_ctas(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    return default_ctas(dev);
}

int mq_get_last_error(void) { return g_last_error; }

const char* mq_last_error_detail(void) { return g_detail; }

const char* mq_error_string(int code) {
    switch (code) {
        case MQ_OK: return "ok";
        case MQ_ERR_INVALID_ARGUMENT: return "invalid argument";
        case MQ_ERR_WAIT_TIMEOUT: return "inter-CTA handoff wait timed out";
        case MQ_ERR_PIPE_TIMEOUT: return "shared-memory pipeline wait timed out";
        case MQ_ERR_BAD_TOKEN: return "input token out of range";
        case MQ_ERR_BAD_POSITION: return "position out of range";
        case MQ_ERR_CUDA: return "CUDA runtime error";
        case MQ_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown error";
    }
}

const char* mq_version(void) { return "megaqwen_b200 0.1"; }

}  // extern "C"

namespace mq {
// Records the failing CUDA call for mq_last_error_detail (used by the other
// translation units of the library); returns MQ_ERR_CUDA.
int note_cuda(cudaError_t e, const char* what) { return cuda_fail(e, what); }
}  // namespace mq
