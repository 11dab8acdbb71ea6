/*
 * megaqwen_b200.h -- C ABI of the B200 (sm_100a) Qwen3-0.6B decode engine.
 *
 * Drop-in for the extern "C" launchers of Infatoshi/MegaQwen's torch
 * extension.  Every pointer argument is a plain device pointer unless stated;
 * no torch types cross this boundary.  Tensors use the reference layouts:
 *   weights     bf16, row-major [out_features, in_features] (HF nn.Linear)
 *   embed/lm    bf16 [151936, 1024] (lm_head may alias embed: tied)
 *   cos/sin     bf16 [max_seq_len, 128] (halves duplicated)
 *   k/v cache   bf16 [num_layers, 8, max_seq_len, 128] contiguous
 *
 * Reference interfaces replaced (file:line inside the MegaQwen tree):
 *   LDGLayerWeights               csrc/megakernel/fused_decode_ldg.cu:24-36
 *   launch_ldg_decode             csrc/megakernel/fused_decode_ldg.cu:893-969
 *   launch_ldg_decode_with_logits csrc/megakernel/fused_decode_ldg.cu:972-1057
 *   launch_prefill_float          csrc/megakernel/fused_prefill.cu:601-867
 *   launch_prefill_megakernel     csrc/megakernel/fused_prefill_megakernel.cu:938-1020
 */
#ifndef MEGAQWEN_B200_H
#define MEGAQWEN_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Model constants (Qwen3-0.6B; csrc/megakernel/config.cuh:33-40). */
#define MQ_HIDDEN_SIZE 1024
#define MQ_INTERMEDIATE_SIZE 3072
#define MQ_NUM_Q_HEADS 16
#define MQ_NUM_KV_HEADS 8
#define MQ_HEAD_DIM 128
#define MQ_VOCAB_SIZE 151936
#define MQ_MAX_LAYERS 63
#define MQ_MAX_TP 8          /* largest tensor-parallel group of mq_decode */

/* Per-layer weight pointers, same field order and size as the reference's
 * LDGLayerWeights (fused_decode_ldg.cu:24-36) and PrefillLayerWeights
 * (fused_prefill.cu:28-40). */
typedef struct LDGLayerWeights {
    const void* input_layernorm_weight;
    const void* q_proj_weight;
    const void* k_proj_weight;
    const void* v_proj_weight;
    const void* q_norm_weight;
    const void* k_norm_weight;
    const void* o_proj_weight;
    const void* post_attn_layernorm_weight;
    const void* gate_proj_weight;
    const void* up_proj_weight;
    const void* down_proj_weight;
} LDGLayerWeights;

typedef LDGLayerWeights PrefillLayerWeights;

/* Status codes (0 = success). */
enum {
    MQ_OK = 0,
    MQ_ERR_INVALID_ARGUMENT = 1,   /* bad size, position, token, null pointer */
    MQ_ERR_WAIT_TIMEOUT = 2,       /* an inter-CTA handoff wait ran out of time */
    MQ_ERR_PIPE_TIMEOUT = 3,       /* a shared-memory pipeline wait ran out of time */
    MQ_ERR_BAD_TOKEN = 4,          /* input token outside [0, vocab) (device check) */
    MQ_ERR_BAD_POSITION = 5,       /* position outside [0, max_seq_len) (device check) */
    MQ_ERR_CUDA = 6,               /* a CUDA runtime call failed */
    MQ_ERR_WORKSPACE = 7           /* workspace missing or too small */
};

/* ---- reference ABI -------------------------------------------------------
 * launch_ldg_decode: one batch-1 decode step; replaces fused_decode_ldg.cu:893.
 * Same 27 arguments.  layer_weights is a DEVICE array of num_layers structs.
 * Writes the greedy next token to output_token_id (device int32), the K/V rows
 * of `position` into the caches, the final bf16 hidden state (before the final
 * norm) into hidden_buffer and the final-normed fp32 hidden into g_normalized.
 * g_activations, g_residual, g_q, g_k, g_v, g_attn_out, g_mlp_intermediate,
 * block_max_vals and block_max_idxs are accepted and not used: the engine
 * keeps its inter-CTA state in a per-device workspace allocated on the first
 * call on each device.  cache_len must equal position + 1.  Returns nothing,
 * like the reference; mq_get_last_error() reports the launch status.        */
void launch_ldg_decode(int input_token_id, int* output_token_id, const void* embed_weight,
                       const LDGLayerWeights* layer_weights, const void* final_norm_weight,
                       const void* lm_head_weight, const void* cos_table, const void* sin_table, void* k_cache,
                       void* v_cache, void* hidden_buffer, void* g_activations, void* g_residual, void* g_q,
                       void* g_k, void* g_v, void* g_attn_out, void* g_mlp_intermediate, void* g_normalized,
                       void* block_max_vals, void* block_max_idxs, int num_layers, int position, int cache_len,
                       int max_seq_len, float attn_scale, cudaStream_t stream);

/* launch_ldg_decode_with_logits: as above, plus the full fp32 logits
 * [151936] into logits_output; replaces fused_decode_ldg.cu:972-1057.       */
void launch_ldg_decode_with_logits(int input_token_id, int* output_token_id, float* logits_output,
                                   const void* embed_weight, const LDGLayerWeights* layer_weights,
                                   const void* final_norm_weight, const void* lm_head_weight, const void* cos_table,
                                   const void* sin_table, void* k_cache, void* v_cache, void* hidden_buffer,
                                   void* g_activations, void* g_residual, void* g_q, void* g_k, void* g_v,
                                   void* g_attn_out, void* g_mlp_intermediate, void* g_normalized,
                                   void* block_max_vals, void* block_max_idxs, int num_layers, int position,
                                   int cache_len, int max_seq_len, float attn_scale, cudaStream_t stream);

/* Result of a decode step written straight to host memory (see
 * mq_decode_params.host_result).  seq is written last. */
typedef struct mq_host_result {
    volatile unsigned int seq;
    int token;
    unsigned int error;
    unsigned int info;
} mq_host_result;

/* ---- native API ------------------------------------------------------------
 * The decode step with an explicit, caller-owned workspace and an explicit
 * status.  Extends launch_ldg_decode (fused_decode_ldg.cu:893-921) with:
 *   - input token from device memory (input_token_ptr; greedy feedback when it
 *     equals output_token) and, optionally, position from device memory
 *     (position_ptr, advanced by one on success) so steps can be replayed
 *     without host round trips;
 *   - an error word in the workspace written by bounded device-side waits.  */
typedef struct mq_decode_params {
    int input_token;               /* used when input_token_ptr is NULL */
    const int* input_token_ptr;    /* device int32, optional */
    int* output_token;             /* device int32, optional */
    float* logits;                 /* device fp32 [151936], optional */
    const void* embed;
    const LDGLayerWeights* layers; /* device array [num_layers] */
    const void* final_norm;
    const void* lm_head;
    const void* cos_table;
    const void* sin_table;
    void* k_cache;
    void* v_cache;
    void* hidden_out;              /* device bf16 [1024], optional */
    float* normalized_out;         /* device fp32 [1024], optional */
    void* workspace;               /* device, mq_decode_workspace_bytes() bytes, zeroed once */
    size_t workspace_bytes;
    int num_layers;
    int position;                  /* used when position_ptr is NULL */
    int* position_ptr;             /* device int32, optional; incremented on success */
    int max_seq_len;
    float attn_scale;
    int num_ctas;                  /* 0: one CTA per SM */
    int attn_chunk;                /* target KV positions per attention work unit; 0: default */
    long long timeout_ns;          /* bound on every device wait; 0: default (2 s) */
    int inject_skip_cta;           /* test hook: CTA (value - 1) withholds its layer-0 QKV handoff
                                      stores, so the others' waits run out; 0: off */
    unsigned long long* trace;     /* optional device buffer [num_ctas * 2048] of %globaltimer
                                      stamps per CTA, phase and tile (profiling); NULL: off.
                                      Only kernel start/end are stamped unless the library was
                                      built with MQ_DECODE_TRACE=1 (see megaqwen_b200/build.py) */
    mq_host_result* host_result;   /* optional: device-visible address of mapped pinned host memory
                                      (cudaHostAllocMapped + cudaHostGetDevicePointer).  The step's
                                      last CTA writes token, error and info there, then seq =
                                      host_seq, so a host thread can wait for the token without a
                                      device-to-host copy and a stream synchronise.  Nothing is
                                      written when the step fails before its argmax: wait with a
                                      bound and fall back to mq_decode_fetch.  NULL: off */
    unsigned int host_seq;
    /* KV-head tensor parallel decode, one rank per GPU (no counterpart in the
       reference, which runs on one GPU).  tp_size 0 or 1: single GPU.  tp_size
       T in {2, 4, 8}: rank r = tp_rank computes the q/k/v rows and attention of
       kv heads [8r/T, 8(r+1)/T), the O and down projections over its own
       attention / act columns (row-parallel partials), gate/up rows
       [3072r/T, 3072(r+1)/T) and vocabulary rows [151936r/T, 151936(r+1)/T); it
       reads only those parts of the full-size weight tensors and writes only
       its heads' cache rows.  The kernel stores the per-layer O and down
       partials and the argmax keys into every rank's workspace itself (peer
       stores over NVLink), and every rank adds the partials in rank order.
       peer_workspaces: HOST array of T device addresses, valid in this
       process (CUDA IPC or peer access), of every rank's workspace, entry
       tp_rank being `workspace`.  The ranks launch the same steps (same token
       and position) and zero their workspaces together. */
    int tp_rank;
    int tp_size;
    void* const* peer_workspaces;
} mq_decode_params;

size_t mq_decode_workspace_bytes(void);
/* Zero a workspace (stream-ordered).  Needed once before first use and after
 * any call that returned an error. */
int mq_decode_workspace_init(void* workspace, size_t bytes, cudaStream_t stream);
/* Set the step counter kept in a workspace (stream-ordered).  Every step tags
 * its inter-CTA handoff words with this counter, which wraps to 0 after
 * 2^25 - 1; this entry point lets tests and diagnostics run steps across the
 * wrap.  epoch must be below 2^25. */
int mq_decode_workspace_set_epoch(void* workspace, uint32_t epoch, cudaStream_t stream);
/* Launch one decode step.  Host-side argument checks return an error code
 * without launching; device-side failures land in the workspace error word. */
int mq_decode(const mq_decode_params* params, cudaStream_t stream);

/* mq_decode_noalloc: the same decode step for callers that must not allocate
 * device memory -- for example code running under an allocator or memory
 * pool that owns all device memory, or a runtime whose own workspace budget is
 * fixed up front and cannot grant the few hundred KB mq_decode needs.  It has
 * no counterpart in the reference.  The inter-CTA scratch lives in a static
 * device array of MQ_NOALLOC_SCRATCH_BYTES bytes (held on every GPU that loads
 * this library, until the process exits); params->workspace and
 * workspace_bytes are ignored.  The caller still passes every input and output
 * buffer.  The first call on a device resolves the array's address and clears
 * it, so make that first call before any stream capture.  Every call on a
 * device shares the array, so calls that overlap on the GPU (different
 * streams, or other threads) race.  num_ctas above 256 or num_layers above 63
 * are rejected with MQ_ERR_INVALID_ARGUMENT.  Any device-side failure of a
 * step -- a wait that ran out, or an input token or position (read from
 * input_token_ptr / position_ptr) out of range -- leaves the output token
 * unwritten and an error word in the scratch, after which every later step on
 * that device fails too until mq_decode_noalloc_reset() clears the scratch.
 * Learn a step's status from host_result (written by the step) or from
 * mq_decode_noalloc_fetch().  The device address of the array is cached per
 * device index for the life of the process: after cudaDeviceReset() (or any
 * new primary context) this entry point must not be used again.  Calls no
 * cudaMalloc, cudaFree or other allocating routine. */
#define MQ_NOALLOC_SCRATCH_BYTES 950656
int mq_decode_noalloc(const mq_decode_params* params, cudaStream_t stream);
/* Clear the static scratch of the current device (stream-ordered, no
 * allocation), e.g. after a step reported an error.  No-op before the first
 * mq_decode_noalloc call on the device. */
int mq_decode_noalloc_reset(cudaStream_t stream);
/* Status of the last mq_decode_noalloc step on the current device: the greedy
 * token of the last successful step, the error word and the info word.
 * Copies 32 bytes into host stack memory and synchronises `stream`; allocates
 * nothing. */
int mq_decode_noalloc_fetch(int* token, uint32_t* error, uint32_t* info, cudaStream_t stream);
/* Copy the workspace error word (and the auxiliary info word) to the host;
 * synchronises `stream`. */
int mq_decode_read_error(const void* workspace, uint32_t* error, uint32_t* info, cudaStream_t stream);
/* Copy the step result from the workspace to the host and synchronise
 * `stream`: the greedy token of the last successful step, the error word and
 * the auxiliary info word.  One 32-byte device-to-host copy. */
int mq_decode_fetch(const void* workspace, int* token, uint32_t* error, uint32_t* info, cudaStream_t stream);
/* Number of CTAs the decode kernel would use on the current device. */
int mq_decode_default_ctas(void);

/* ---- prefill building block --------------------------------------------------
 * mq_gemm_bf16: C[M, N] = A[M, K] . B[N, K]^T on the sm_100a tensor cores
 * (tcgen05, fp32 accumulation in TMEM), A and B bf16 row-major (K contiguous,
 * leading dimensions lda/ldb in elements).  Replaces the cublasGemmEx calls of
 * the reference prefill (csrc/megakernel/fused_prefill.cu:674-824).
 * epilogue: 0 store fp32, 1 add into fp32 C (residual), 2 C_bf16 =
 * silu(A.B^T) * (A.B2^T) (gate/up), 3 store bf16.  N % 128 == 0, K % 64 == 0.
 * err_flag: device int set non-zero if a bounded device wait ran out. */
int mq_gemm_bf16(const void* A, int lda, const void* B, int ldb, const void* B2, void* C, int ldc, int M, int N,
                 int K, int epilogue, int* err_flag, cudaStream_t stream);

/* ---- prefill ------------------------------------------------------------------
 * mq_prefill: prompts of `batch` sequences x `seq_len` tokens, positions
 * 0..seq_len-1, through all layers on the tensor cores (tcgen05 GEMMs, flash
 * attention), writing each sequence's K/V cache rows and its greedy next token.
 * Replaces launch_prefill_float (csrc/megakernel/fused_prefill.cu:601-867) and
 * extends it to batches.  Sequence b's caches start at k_cache/v_cache +
 * b * cache_seq_stride elements, each [num_layers, 8, max_seq_len, 128]. */
typedef struct mq_prefill_params {
    const int* ids;                        /* device int32 [batch * seq_len] */
    int batch;
    int seq_len;
    int start_pos;                         /* must be 0 */
    const void* embed;
    const LDGLayerWeights* layers_host;    /* HOST array [num_layers] (as the reference passes) */
    const void* final_norm;
    const void* lm_head;
    const void* cos_table;
    const void* sin_table;
    void* k_cache;
    void* v_cache;
    long long cache_seq_stride;            /* elements between sequences' caches */
    int num_layers;
    int max_seq_len;
    float attn_scale;
    int* out_tokens;                       /* device int32 [batch] */
    float* logits;                         /* device fp32 [batch, 151936], optional */
    void* hidden_out;                      /* unused, reserved */
    void* workspace;                       /* device, mq_prefill_workspace_bytes(batch, seq_len) */
    size_t workspace_bytes;
    int* err_flag;                         /* optional device int: set when a device wait ran out */
} mq_prefill_params;

size_t mq_prefill_workspace_bytes(int batch, int seq_len);
int mq_prefill(const mq_prefill_params* params, cudaStream_t stream);

/* launch_prefill_float: the reference prefill launcher, same arguments
 * (fused_prefill.cu:601-636).  layer_weights is a HOST array as in the
 * reference; the bf16 scratch buffers and the cuBLAS handle are accepted and
 * not used (the engine keeps a per-device workspace, allocated on first use). */
void launch_prefill_float(const int* input_token_ids, int* output_token_id, int seq_len, const void* embed_weight,
                          const PrefillLayerWeights* layer_weights, const void* final_norm_weight,
                          const void* lm_head_weight, const void* cos_table, const void* sin_table, void* k_cache,
                          void* v_cache, void* hidden_bf16, void* residual, void* normalized, void* q_proj,
                          void* k_proj, void* v_proj, void* attn_out, void* o_proj_out, void* mlp_norm,
                          void* gate_out, void* up_out, void* mlp_intermediate, void* down_out, void* final_hidden,
                          void* block_max_vals, void* block_max_idxs, void* hidden_bf16_out, int num_layers,
                          int max_seq_len, float attn_scale, void* cublas_handle, cudaStream_t stream);
/* launch_prefill_megakernel: the reference's short-prompt prefill launcher,
 * same arguments (fused_prefill_megakernel.cu:938-966).  layer_weights is a
 * DEVICE array there (megakernel_decode.py:911-916); it is read back to the
 * host and the prompt runs through the tensor-core prefill.  The fp32 scratch
 * buffers are accepted and not used.  Status: mq_prefill_get_last_error(). */
void launch_prefill_megakernel(const int* token_ids, int* output_token_id, int seq_len, const void* embed_weight,
                               const PrefillLayerWeights* layer_weights, const void* final_norm_weight,
                               const void* lm_head_weight, const void* cos_table, const void* sin_table,
                               void* k_cache, void* v_cache, void* hidden, void* residual, void* normalized,
                               void* q_proj, void* k_proj, void* v_proj, void* attn_out, void* mlp_intermediate,
                               void* final_hidden, void* hidden_bf16_out, void* block_max_vals,
                               void* block_max_idxs, int num_layers, int max_seq_len, float attn_scale,
                               cudaStream_t stream);
int mq_prefill_get_last_error(void);

/* ---- batched decode -----------------------------------------------------------
 * mq_decode_batch: one greedy decode step for `batch` (1..128) independent
 * sequences.  Sequence b consumes tokens[b] at position positions[b], appends
 * its K/V rows there, and on return (stream order) tokens[b] holds its next
 * token and positions[b] has advanced by one.  The weights are read once per
 * step for all sequences (small-batch tcgen05 GEMMs, split-K).  This is the
 * batch >= 16 serving path the reference drives through its per-sequence
 * decoder (csrc/megakernel/ldg_decode.cu launch_ldg_decode called once per
 * sequence); numerics follow the single-sequence decode with bf16 GEMM
 * operands.  max_context >= max_b(positions[b] + 1) bounds the attention grid
 * (host-known, so a step needs no device->host read).  Caches as in
 * mq_prefill_params. */
typedef struct mq_decode_batch_params {
    int* tokens;                           /* device int32 [batch], in/out */
    int* positions;                        /* device int32 [batch], in/out */
    int batch;
    int max_context;
    const void* embed;
    const LDGLayerWeights* layers_host;    /* HOST array [num_layers] */
    const void* final_norm;
    const void* lm_head;
    const void* cos_table;
    const void* sin_table;
    void* k_cache;
    void* v_cache;
    long long cache_seq_stride;
    int num_layers;
    int max_seq_len;
    float attn_scale;
    float* logits;                         /* device fp32 [batch, 151936], optional */
    void* workspace;                       /* device, mq_decode_batch_workspace_bytes(batch, max_seq_len) */
    size_t workspace_bytes;
    int* err_flag;                         /* device int: set when a device wait ran out (required) */
} mq_decode_batch_params;

size_t mq_decode_batch_workspace_bytes(int batch, int max_seq_len);
int mq_decode_batch(const mq_decode_batch_params* params, cudaStream_t stream);

/* Last status recorded by the reference-ABI launchers on this host thread. */
int mq_get_last_error(void);
const char* mq_error_string(int code);
/* Text of the last failing CUDA runtime call on this host thread ("" if none). */
const char* mq_last_error_detail(void);
/* Library version string. */
const char* mq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MEGAQWEN_B200_H */
