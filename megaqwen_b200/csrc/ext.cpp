// Torch extension: the reference's Python-facing classes and module functions,
// implemented over the C ABI in include/megaqwen_b200.h.
//
// Mirrors, by name, arguments and error behaviour:
//   MegakernelDecoder             csrc/megakernel/megakernel_decode.py:90-242
//   MegakernelPrefillDecoder      csrc/megakernel/megakernel_decode.py:375-660
//   MegakernelFusedPrefillDecoder csrc/megakernel/megakernel_decode.py:788-1053
//   init_ldg_layer_weights / init_ldg_embed_weight / decode_ldg /
//   decode_ldg_with_logits        chat.py:147-323
// Differences, all additive: decode steps and prefill check position <
// max_seq_len and raise RuntimeError; device-side wait failures raise
// RuntimeError with the engine's error text.

#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "megaqwen_b200.h"

namespace {

constexpr int kHidden = MQ_HIDDEN_SIZE;
constexpr int kInter = MQ_INTERMEDIATE_SIZE;
constexpr int kQ = MQ_NUM_Q_HEADS * MQ_HEAD_DIM;
constexpr int kKV = MQ_NUM_KV_HEADS * MQ_HEAD_DIM;
constexpr int kVocab = MQ_VOCAB_SIZE;

void check_bf16(const torch::Tensor& t, const char* name, std::vector<int64_t> shape) {
    if (!t.is_cuda()) throw std::runtime_error(std::string(name) + " must be a CUDA tensor");
    if (t.scalar_type() != torch::kBFloat16) throw std::runtime_error(std::string(name) + " must be bfloat16");
    if (!t.is_contiguous()) throw std::runtime_error(std::string(name) + " must be contiguous");
    if (t.sizes().vec() != shape) throw std::runtime_error(std::string(name) + " has the wrong shape");
}

std::vector<int64_t> layer_shape(int k) {
    switch (k) {
        case 0: return {kHidden};
        case 1: return {kQ, kHidden};
        case 2: return {kKV, kHidden};
        case 3: return {kKV, kHidden};
        case 4: return {MQ_HEAD_DIM};
        case 5: return {MQ_HEAD_DIM};
        case 6: return {kHidden, kQ};
        case 7: return {kHidden};
        case 8: return {kInter, kHidden};
        case 9: return {kInter, kHidden};
        default: return {kHidden, kInter};
    }
}

const char* kLayerNames[11] = {"input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm",
                               "o_proj", "post_attention_layernorm", "gate_proj", "up_proj", "down_proj"};

LDGLayerWeights make_layer(const std::vector<torch::Tensor>& t, size_t base) {
    LDGLayerWeights w;
    w.input_layernorm_weight = t[base + 0].data_ptr();
    w.q_proj_weight = t[base + 1].data_ptr();
    w.k_proj_weight = t[base + 2].data_ptr();
    w.v_proj_weight = t[base + 3].data_ptr();
    w.q_norm_weight = t[base + 4].data_ptr();
    w.k_norm_weight = t[base + 5].data_ptr();
    w.o_proj_weight = t[base + 6].data_ptr();
    w.post_attn_layernorm_weight = t[base + 7].data_ptr();
    w.gate_proj_weight = t[base + 8].data_ptr();
    w.up_proj_weight = t[base + 9].data_ptr();
    w.down_proj_weight = t[base + 10].data_ptr();
    return w;
}

torch::Tensor layer_table(const std::vector<LDGLayerWeights>& host, const torch::Device& dev) {
    auto cpu = torch::empty({(int64_t)(host.size() * sizeof(LDGLayerWeights))}, torch::kUInt8);
    std::memcpy(cpu.data_ptr(), host.data(), host.size() * sizeof(LDGLayerWeights));
    return cpu.to(dev);
}

[[noreturn]] void raise_engine(int code, uint32_t info, const char* where) {
    throw std::runtime_error(std::string(where) + ": " + mq_error_string(code) + " (code " + std::to_string(code) +
                             ", info 0x" + [&] {
                                 char b[16];
                                 snprintf(b, sizeof(b), "%x", info);
                                 return std::string(b);
                             }() + ")" + (code == MQ_ERR_CUDA ? std::string(" ") + mq_last_error_detail() : ""));
}

// ---------------------------------------------------------------------------
class MegakernelDecoder {
public:
    MegakernelDecoder(torch::Tensor embed_weight, std::vector<torch::Tensor> layer_weights_flat,
                      torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
                      torch::Tensor sin_table, int num_layers, int max_seq_len)
        : num_layers_(num_layers), max_seq_len_(max_seq_len) {
        if (num_layers < 1 || num_layers > MQ_MAX_LAYERS) throw std::runtime_error("num_layers out of range");
        if (max_seq_len < 1) throw std::runtime_error("max_seq_len must be positive");
        if ((int)layer_weights_flat.size() != num_layers * 11)
            throw std::runtime_error("layer_weights_flat must hold num_layers * 11 tensors");
        check_bf16(embed_weight, "embed_weight", {kVocab, kHidden});
        check_bf16(final_norm_weight, "final_norm_weight", {kHidden});
        check_bf16(lm_head_weight, "lm_head_weight", {kVocab, kHidden});
        if (!cos_table.is_cuda() || cos_table.scalar_type() != torch::kBFloat16 || !cos_table.is_contiguous() ||
            cos_table.dim() != 2 || cos_table.size(1) != MQ_HEAD_DIM || cos_table.size(0) < max_seq_len)
            throw std::runtime_error("cos_table must be contiguous bf16 [>=max_seq_len, 128] on the GPU");
        if (!sin_table.is_cuda() || sin_table.scalar_type() != torch::kBFloat16 || !sin_table.is_contiguous() ||
            sin_table.sizes() != cos_table.sizes())
            throw std::runtime_error("sin_table must match cos_table");
        for (int i = 0; i < num_layers * 11; ++i)
            check_bf16(layer_weights_flat[i], kLayerNames[i % 11], layer_shape(i % 11));
        device_ = embed_weight.device();
        c10::cuda::CUDAGuard guard(device_);
        embed_ = embed_weight;
        final_norm_ = final_norm_weight;
        lm_head_ = lm_head_weight;
        cos_ = cos_table;
        sin_ = sin_table;
        layer_tensors_ = layer_weights_flat;
        std::vector<LDGLayerWeights> host(num_layers);
        for (int i = 0; i < num_layers; ++i) host[i] = make_layer(layer_weights_flat, (size_t)i * 11);
        d_layers_ = layer_table(host, device_);
        layers_host_ = host;
        auto bf = torch::dtype(torch::kBFloat16).device(device_);
        auto f32 = torch::dtype(torch::kFloat32).device(device_);
        auto i32 = torch::dtype(torch::kInt32).device(device_);
        k_cache_ = torch::zeros({num_layers, MQ_NUM_KV_HEADS, max_seq_len, MQ_HEAD_DIM}, bf);
        v_cache_ = torch::zeros({num_layers, MQ_NUM_KV_HEADS, max_seq_len, MQ_HEAD_DIM}, bf);
        hidden_buffer_ = torch::zeros({kHidden}, bf);
        g_normalized_ = torch::zeros({kHidden}, f32);
        output_token_ = torch::zeros({1}, i32);
        dev_position_ = torch::zeros({1}, i32);
        workspace_ = torch::zeros({(int64_t)mq_decode_workspace_bytes()}, torch::dtype(torch::kUInt8).device(device_));
        position_ = 0;
        attn_scale_ = 1.0f / sqrtf(128.0f);
    }

    virtual ~MegakernelDecoder() {
        if (hres_) cudaFreeHost(hres_);   // errors at interpreter exit are ignored
    }

    int decode_step(int input_token_id) {
        step(input_token_id, nullptr, nullptr);
        return last_token_;
    }

    std::tuple<int, torch::Tensor> decode_step_with_logits(int input_token_id) {
        auto logits = torch::empty({kVocab}, torch::dtype(torch::kFloat32).device(device_));
        step(input_token_id, nullptr, logits.data_ptr<float>());
        return std::make_tuple(last_token_, logits);
    }

    // Greedy decode of `steps` tokens starting from `first_token` with the token
    // fed back on the device: no host round trip between steps.  Returns the
    // generated tokens (device int32 [steps]).
    torch::Tensor generate_greedy(int first_token, int steps) {
        if (steps < 0) throw std::runtime_error("steps must be non-negative");
        if (position_ + steps > max_seq_len_) throw std::runtime_error("generation would exceed max_seq_len");
        if (first_token < 0 || first_token >= kVocab) throw std::runtime_error("token out of range");
        c10::cuda::CUDAGuard guard(device_);
        auto out = torch::empty({steps + 1}, torch::dtype(torch::kInt32).device(device_));
        out.narrow(0, 0, 1).fill_(first_token);
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        for (int i = 0; i < steps; ++i) {
            mq_decode_params p = params(0, nullptr);
            p.input_token_ptr = out.data_ptr<int>() + i;
            p.output_token = out.data_ptr<int>() + i + 1;
            p.position = position_ + i;
            int rc = mq_decode(&p, stream);
            if (rc) raise_engine(rc, 0, "generate_greedy");
        }
        check_device("generate_greedy", stream);
        position_ += steps;
        return out.narrow(0, 1, steps);
    }

    void reset() {
        position_ = 0;
        k_cache_.zero_();
        v_cache_.zero_();
    }

    int position() const { return position_; }
    void set_position(int p) {
        if (p < 0 || p > max_seq_len_) throw std::runtime_error("position out of range");
        position_ = p;
    }
    torch::Tensor get_k_cache() const { return k_cache_; }
    torch::Tensor get_v_cache() const { return v_cache_; }
    torch::Tensor get_hidden_buffer() const { return hidden_buffer_; }
    torch::Tensor get_normalized() const { return g_normalized_; }
    int last_token() const { return last_token_; }

    // Tuning / test hooks
    void set_num_ctas(int n) { num_ctas_ = n; }
    void set_attn_chunk(int n) { attn_chunk_ = n; }
    void set_timeout_ns(long long t) { timeout_ns_ = t; }
    void set_inject_skip_cta(int c) { inject_skip_cta_ = c; }
    // Step counter of the handoff tags (wraps at 2^25): lets tests run across the wrap.
    void set_step_epoch(int64_t e) {
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        int rc = mq_decode_workspace_set_epoch(workspace_.data_ptr(), (uint32_t)e, stream);
        if (rc) raise_engine(rc, 0, "set_step_epoch");
    }
    // Profiling: device int64 buffer of num_ctas * 512 timestamps, or 0 to disable.
    void set_trace(int64_t ptr) { trace_ = reinterpret_cast<unsigned long long*>(ptr); }
    int num_ctas() const { return num_ctas_ > 0 ? num_ctas_ : mq_decode_default_ctas(); }

    // Raw decode step for benchmarks: token from a device pointer (feedback),
    // no host synchronisation.  Advances the host position.
    void decode_step_async(int64_t input_token_ptr, int64_t output_token_ptr) {
        if (position_ >= max_seq_len_) throw std::runtime_error("position exceeds max_seq_len");
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        mq_decode_params p = params(0, nullptr);
        p.input_token_ptr = reinterpret_cast<const int*>(input_token_ptr);
        p.output_token = reinterpret_cast<int*>(output_token_ptr);
        int rc = mq_decode(&p, stream);
        if (rc) raise_engine(rc, 0, "decode_step_async");
        position_ += 1;
    }

    // Reads and clears the device error word; raises if it was set.
    void check() {
        c10::cuda::CUDAGuard guard(device_);
        check_device("check", c10::cuda::getCurrentCUDAStream(device_.index()).stream());
    }

protected:
    mq_decode_params params(int token, float* logits) {
        mq_decode_params p = {};
        p.input_token = token;
        p.output_token = output_token_.data_ptr<int>();
        p.logits = logits;
        p.embed = embed_.data_ptr();
        p.layers = reinterpret_cast<const LDGLayerWeights*>(d_layers_.data_ptr());
        p.final_norm = final_norm_.data_ptr();
        p.lm_head = lm_head_.data_ptr();
        p.cos_table = cos_.data_ptr();
        p.sin_table = sin_.data_ptr();
        p.k_cache = k_cache_.data_ptr();
        p.v_cache = v_cache_.data_ptr();
        p.hidden_out = hidden_buffer_.data_ptr();
        p.normalized_out = g_normalized_.data_ptr<float>();
        p.workspace = workspace_.data_ptr();
        p.workspace_bytes = (size_t)workspace_.numel();
        p.num_layers = num_layers_;
        p.position = position_;
        p.max_seq_len = max_seq_len_;
        p.attn_scale = attn_scale_;
        p.num_ctas = num_ctas_;
        p.attn_chunk = attn_chunk_;
        p.timeout_ns = timeout_ns_;
        p.inject_skip_cta = inject_skip_cta_;
        p.trace = trace_;
        if (tp_size_ > 1) {
            for (void* q : peer_ws_)
                if (!q) throw std::runtime_error("tensor-parallel decoder is not connected to every rank (connect)");
            p.tp_rank = tp_rank_;
            p.tp_size = tp_size_;
            p.peer_workspaces = peer_ws_.data();
        }
        return p;
    }

    void check_device(const char* where, cudaStream_t stream) {
        int tok = 0;
        uint32_t err = 0, info = 0;
        int rc = mq_decode_fetch(workspace_.data_ptr(), &tok, &err, &info, stream);
        if (rc) raise_engine(rc, 0, where);
        if (err) {
            mq_decode_workspace_init(workspace_.data_ptr(), (size_t)workspace_.numel(), stream);
            raise_engine((int)err, info, where);
        }
        last_token_ = tok;
    }

    void step(int input_token_id, const int* token_ptr, float* logits) {
        if (position_ >= max_seq_len_) throw std::runtime_error("position exceeds max_seq_len");
        if (!token_ptr && (input_token_id < 0 || input_token_id >= kVocab))
            throw std::runtime_error("input token out of range");
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        mq_decode_params p = params(input_token_id, logits);
        p.input_token_ptr = token_ptr;
        const bool fast = ensure_host_result();
        if (fast) {
            if (++hseq_ == 0) ++hseq_;
            p.host_result = hres_dev_;
            p.host_seq = hseq_;
        }
        int rc = mq_decode(&p, stream);
        if (rc) raise_engine(rc, 0, "decode_step");
        // The mapped-result path reads no stream status; a sticky CUDA error
        // raised after the kernel wrote its result is caught here on the host
        // (no device round trip) and reported through the checked path.
        // step() waits for its result on the host, so it must not be called
        // while the current stream is being captured into a CUDA graph.
        if (fast && wait_host_result(hseq_, stream) && cudaPeekAtLastError() == cudaSuccess)
            last_token_ = hres_->token;
        else
            check_device("decode_step", stream);
        position_ += 1;
    }

    // Mapped pinned host memory the kernel writes its result to (one per
    // decoder).  Without it every step would pay a device-to-host copy and a
    // stream synchronise.
    bool ensure_host_result() {
        if (hres_) return true;
        if (hres_failed_) return false;
        void* h = nullptr;
        void* d = nullptr;
        if (cudaHostAlloc(&h, sizeof(mq_host_result), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
            cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
            if (h) cudaFreeHost(h);
            cudaGetLastError();
            hres_failed_ = true;
            return false;
        }
        std::memset(h, 0, sizeof(mq_host_result));
        hres_ = static_cast<mq_host_result*>(h);
        hres_dev_ = static_cast<mq_host_result*>(d);
        return true;
    }

    // Spin until the step's sequence word arrives.  Returns false (the caller
    // then takes the copy-and-synchronise path, which reports errors) when the
    // step recorded an error or the stream finished without writing it.
    bool wait_host_result(unsigned int want, cudaStream_t stream) {
        for (unsigned int i = 1;; ++i) {
            if (hres_->seq == want) {
                std::atomic_thread_fence(std::memory_order_acquire);
                return hres_->error == 0;
            }
            if ((i & 1023u) == 0) {
                const cudaError_t q = cudaStreamQuery(stream);
                if (q != cudaErrorNotReady) {
                    if (hres_->seq == want) {
                        std::atomic_thread_fence(std::memory_order_acquire);
                        return hres_->error == 0;
                    }
                    return false;
                }
            }
        }
    }

    int num_layers_;
    int max_seq_len_;
    int position_;
    float attn_scale_;
    int last_token_ = -1;
    int num_ctas_ = 0;
    int attn_chunk_ = 0;
    long long timeout_ns_ = 0;
    int inject_skip_cta_ = 0;
    unsigned long long* trace_ = nullptr;
    int tp_rank_ = 0, tp_size_ = 1;         // tensor parallel (MegakernelTPDecoder)
    std::vector<void*> peer_ws_;            // every rank's workspace, device addresses valid here
    mq_host_result* hres_ = nullptr;       // host address of the mapped result
    mq_host_result* hres_dev_ = nullptr;   // its device-visible address
    bool hres_failed_ = false;
    unsigned int hseq_ = 0;
    torch::Device device_{torch::kCUDA, 0};
    torch::Tensor embed_, final_norm_, lm_head_, cos_, sin_, d_layers_;
    std::vector<torch::Tensor> layer_tensors_;
    std::vector<LDGLayerWeights> layers_host_;
    torch::Tensor k_cache_, v_cache_, hidden_buffer_, g_normalized_, output_token_, dev_position_, workspace_;
};

// Prefill + decode.  prefill_step runs the prompt through the tensor-core
// prefill (mq_prefill: tcgen05 GEMMs, flash attention) and writes the K/V
// cache rows 0..S-1, like the reference's cuBLAS prefill (fused_prefill.cu:
// 601-867); decode_step then continues at position S.
// ---------------------------------------------------------------------------
// KV-head tensor-parallel batch-1 decoder: one instance per rank (one GPU per
// process), all ranks stepping together.  Same weights and call surface as
// MegakernelDecoder; the kernel computes this rank's heads, row-parallel
// partials and vocabulary slice and exchanges partials with the other ranks
// over NVLink by itself.  The workspace is a plain cudaMalloc allocation so
// that its CUDA IPC handle (ipc_handle) can be opened by the other ranks
// (connect).  No counterpart in the reference, which runs on one GPU.
class MegakernelTPDecoder : public MegakernelDecoder {
public:
    MegakernelTPDecoder(torch::Tensor embed_weight, std::vector<torch::Tensor> layer_weights_flat,
                        torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
                        torch::Tensor sin_table, int num_layers, int max_seq_len, int tp_rank, int tp_size)
        : MegakernelDecoder(embed_weight, layer_weights_flat, final_norm_weight, lm_head_weight, cos_table, sin_table,
                            num_layers, max_seq_len) {
        if (tp_size != 1 && tp_size != 2 && tp_size != 4 && tp_size != 8)
            throw std::runtime_error("tp_size must be 1, 2, 4 or 8");
        if (tp_rank < 0 || tp_rank >= tp_size) throw std::runtime_error("tp_rank out of range");
        c10::cuda::CUDAGuard guard(device_);
        const size_t bytes = mq_decode_workspace_bytes();
        void* ws = nullptr;
        if (cudaMalloc(&ws, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc(tensor-parallel workspace) failed");
        if (cudaMemset(ws, 0, bytes) != cudaSuccess) throw std::runtime_error("cudaMemset(workspace) failed");
        own_ws_ = ws;
        workspace_ = torch::from_blob(ws, {(int64_t)bytes}, torch::dtype(torch::kUInt8).device(device_));
        tp_rank_ = tp_rank;
        tp_size_ = tp_size;
        peer_ws_.assign(tp_size, nullptr);
        peer_ws_[tp_rank] = ws;
        opened_.assign(tp_size, false);
    }
    ~MegakernelTPDecoder() override {
        for (int r = 0; r < tp_size_; ++r)
            if (opened_[r] && peer_ws_[r]) cudaIpcCloseMemHandle(peer_ws_[r]);
        workspace_ = torch::Tensor();
        if (own_ws_) cudaFree(own_ws_);
    }

    // CUDA IPC handle of this rank's workspace (64 bytes), for the other ranks.
    py::bytes ipc_handle() {
        c10::cuda::CUDAGuard guard(device_);
        cudaIpcMemHandle_t h;
        if (cudaIpcGetMemHandle(&h, own_ws_) != cudaSuccess) throw std::runtime_error("cudaIpcGetMemHandle failed");
        return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
    }

    // Open every other rank's workspace from its IPC handle (handles[r] for
    // rank r; this rank's own entry is ignored).
    void connect(std::vector<std::string> handles) {
        if ((int)handles.size() != tp_size_) throw std::runtime_error("connect needs one handle per rank");
        c10::cuda::CUDAGuard guard(device_);
        for (int r = 0; r < tp_size_; ++r) {
            if (r == tp_rank_ || opened_[r]) continue;
            if (handles[r].size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
            cudaIpcMemHandle_t h;
            std::memcpy(&h, handles[r].data(), sizeof(h));
            void* p = nullptr;
            const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess)
                throw std::runtime_error(std::string("cudaIpcOpenMemHandle failed: ") + cudaGetErrorString(e));
            peer_ws_[r] = p;
            opened_[r] = true;
        }
        connected_ = true;
    }

    // Zero this rank's workspace (all ranks together, between steps, e.g.
    // after a step failed on any rank).
    void zero_workspace() {
        c10::cuda::CUDAGuard guard(device_);
        mq_decode_workspace_init(own_ws_, mq_decode_workspace_bytes(),
                                 c10::cuda::getCurrentCUDAStream(device_.index()).stream());
        cudaStreamSynchronize(c10::cuda::getCurrentCUDAStream(device_.index()).stream());
    }

    int tp_rank() const { return tp_rank_; }
    int tp_size() const { return tp_size_; }
    bool connected() const { return connected_ || tp_size_ == 1; }

private:
    void* own_ws_ = nullptr;
    std::vector<bool> opened_;
    bool connected_ = false;
};

class MegakernelPrefillDecoder : public MegakernelDecoder {
public:
    MegakernelPrefillDecoder(torch::Tensor embed_weight, std::vector<torch::Tensor> layer_weights_flat,
                             torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
                             torch::Tensor sin_table, int num_layers, int max_seq_len, int max_prefill_len)
        : MegakernelDecoder(embed_weight, layer_weights_flat, final_norm_weight, lm_head_weight, cos_table,
                            sin_table, num_layers, max_seq_len),
          max_prefill_len_(max_prefill_len) {
        c10::cuda::CUDAGuard guard(device_);
        input_tokens_ = torch::zeros({std::max(1, max_prefill_len)}, torch::dtype(torch::kInt32).device(device_));
        err_ = torch::zeros({1}, torch::dtype(torch::kInt32).device(device_));
    }

    int prefill_step(torch::Tensor input_token_ids) {
        const int seq_len = check_prompt(input_token_ids);
        c10::cuda::CUDAGuard guard(device_);
        input_tokens_.narrow(0, 0, seq_len).copy_(input_token_ids.to(torch::kInt32).to(device_));
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        const size_t need = mq_prefill_workspace_bytes(1, seq_len);
        if (!pf_ws_.defined() || (size_t)pf_ws_.numel() < need)
            pf_ws_ = torch::empty({(int64_t)need}, torch::dtype(torch::kUInt8).device(device_));
        mq_prefill_params p = {};
        p.ids = input_tokens_.data_ptr<int>();
        p.batch = 1;
        p.seq_len = seq_len;
        p.embed = embed_.data_ptr();
        p.layers_host = layers_host_.data();
        p.final_norm = final_norm_.data_ptr();
        p.lm_head = lm_head_.data_ptr();
        p.cos_table = cos_.data_ptr();
        p.sin_table = sin_.data_ptr();
        p.k_cache = k_cache_.data_ptr();
        p.v_cache = v_cache_.data_ptr();
        p.cache_seq_stride = 0;
        p.num_layers = num_layers_;
        p.max_seq_len = max_seq_len_;
        p.attn_scale = attn_scale_;
        p.out_tokens = output_token_.data_ptr<int>();
        p.logits = last_logits_requested_ ? ensure_logits() : nullptr;
        p.workspace = pf_ws_.data_ptr();
        p.workspace_bytes = (size_t)pf_ws_.numel();
        p.err_flag = err_.data_ptr<int>();
        int rc = mq_prefill(&p, stream);
        if (rc) raise_engine(rc, 0, "prefill_step");
        const int tok = output_token_.item<int>();
        if (err_.item<int>() != 0) {
            err_.zero_();
            raise_engine(MQ_ERR_PIPE_TIMEOUT, 0, "prefill_step");
        }
        position_ = seq_len;
        last_token_ = tok;
        return tok;
    }

    // prefill_step that also returns the fp32 logits of the last position.
    std::tuple<int, torch::Tensor> prefill_step_with_logits(torch::Tensor input_token_ids) {
        last_logits_requested_ = true;
        int tok;
        try {
            tok = prefill_step(input_token_ids);
        } catch (...) {
            last_logits_requested_ = false;
            throw;
        }
        last_logits_requested_ = false;
        return std::make_tuple(tok, logits_.clone());
    }

    // The prompt through the decode kernel one position at a time (device-side
    // token feed, one host synchronisation): the reference decode-only
    // generators' way of consuming a prompt (megakernel_decode.py:1166-1167).
    int prefill_step_sequential(torch::Tensor input_token_ids) {
        const int seq_len = check_prompt(input_token_ids);
        c10::cuda::CUDAGuard guard(device_);
        input_tokens_.narrow(0, 0, seq_len).copy_(input_token_ids.to(torch::kInt32).to(device_));
        cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        for (int i = 0; i < seq_len; ++i) {
            mq_decode_params p = params(0, nullptr);
            p.input_token_ptr = input_tokens_.data_ptr<int>() + i;
            p.position = i;
            int rc = mq_decode(&p, stream);
            if (rc) raise_engine(rc, 0, "prefill_step");
        }
        check_device("prefill_step", stream);
        position_ = seq_len;
        return last_token_;
    }

    int max_prefill_len() const { return max_prefill_len_; }

protected:
    // megakernel_decode.py:496-504 checks, plus token range and max_seq_len.
    int check_prompt(const torch::Tensor& ids) {
        if (ids.dim() != 1) throw std::runtime_error("input_token_ids must be 1-D");
        const int seq_len = (int)ids.size(0);
        if (seq_len > max_prefill_len_) throw std::runtime_error("Prefill sequence length exceeds maximum");
        if (seq_len == 0) throw std::runtime_error("Empty input sequence");
        if (seq_len > max_seq_len_) throw std::runtime_error("Prefill sequence length exceeds max_seq_len");
        auto cpu_ids = ids.to(torch::kCPU).to(torch::kInt64);
        auto acc = cpu_ids.accessor<int64_t, 1>();
        for (int i = 0; i < seq_len; ++i)
            if (acc[i] < 0 || acc[i] >= kVocab) throw std::runtime_error("input token out of range");
        return seq_len;
    }
    float* ensure_logits() {
        if (!logits_.defined()) logits_ = torch::empty({kVocab}, torch::dtype(torch::kFloat32).device(device_));
        return logits_.data_ptr<float>();
    }

    int max_prefill_len_;
    bool last_logits_requested_ = false;
    torch::Tensor input_tokens_, pf_ws_, err_, logits_;
};

// Batched prefill: ids int32 [B, S] on the GPU, caches
// [B, L, 8, max_seq_len, 128] bf16; returns the greedy next token of each
// sequence (device int32 [B]) and optionally writes logits [B, 151936].
torch::Tensor prefill_batch(torch::Tensor embed, std::vector<torch::Tensor> layer_weights_flat, torch::Tensor final_norm,
                            torch::Tensor lm_head, torch::Tensor cos, torch::Tensor sin, torch::Tensor ids,
                            torch::Tensor k_cache, torch::Tensor v_cache, c10::optional<torch::Tensor> logits,
                            c10::optional<torch::Tensor> workspace) {
    if (ids.dim() != 2 || ids.scalar_type() != torch::kInt32 || !ids.is_cuda() || !ids.is_contiguous())
        throw std::runtime_error("ids must be a contiguous int32 [B, S] CUDA tensor");
    const int B = (int)ids.size(0), S = (int)ids.size(1);
    const int L = (int)layer_weights_flat.size() / 11;
    if (L < 1 || (int)layer_weights_flat.size() != L * 11) throw std::runtime_error("layer_weights_flat must hold L * 11 tensors");
    if (k_cache.dim() != 5 || k_cache.size(0) != B || k_cache.size(1) != L || k_cache.size(2) != MQ_NUM_KV_HEADS ||
        k_cache.size(4) != MQ_HEAD_DIM || k_cache.scalar_type() != torch::kBFloat16 || !k_cache.is_contiguous() ||
        v_cache.sizes() != k_cache.sizes() || !v_cache.is_contiguous())
        throw std::runtime_error("caches must be contiguous bf16 [B, L, 8, max_seq_len, 128]");
    const int max_seq = (int)k_cache.size(3);
    if (S > max_seq || S < 1) throw std::runtime_error("sequence length exceeds max_seq_len");
    c10::cuda::CUDAGuard guard(ids.device());
    std::vector<LDGLayerWeights> host(L);
    for (int i = 0; i < L; ++i) host[i] = make_layer(layer_weights_flat, (size_t)i * 11);
    const size_t need = mq_prefill_workspace_bytes(B, S);
    torch::Tensor ws = (workspace.has_value() && (size_t)workspace->numel() >= need)
                           ? *workspace
                           : torch::empty({(int64_t)need}, torch::dtype(torch::kUInt8).device(ids.device()));
    auto out = torch::empty({B}, torch::dtype(torch::kInt32).device(ids.device()));
    auto err = torch::zeros({1}, torch::dtype(torch::kInt32).device(ids.device()));
    mq_prefill_params p = {};
    p.ids = ids.data_ptr<int>();
    p.batch = B;
    p.seq_len = S;
    p.embed = embed.data_ptr();
    p.layers_host = host.data();
    p.final_norm = final_norm.data_ptr();
    p.lm_head = lm_head.data_ptr();
    p.cos_table = cos.data_ptr();
    p.sin_table = sin.data_ptr();
    p.k_cache = k_cache.data_ptr();
    p.v_cache = v_cache.data_ptr();
    p.cache_seq_stride = (long long)L * MQ_NUM_KV_HEADS * max_seq * MQ_HEAD_DIM;
    p.num_layers = L;
    p.max_seq_len = max_seq;
    p.attn_scale = 1.0f / sqrtf(128.0f);
    p.out_tokens = out.data_ptr<int>();
    p.logits = logits.has_value() ? logits->data_ptr<float>() : nullptr;
    p.workspace = ws.data_ptr();
    p.workspace_bytes = (size_t)ws.numel();
    p.err_flag = err.data_ptr<int>();
    int rc = mq_prefill(&p, c10::cuda::getCurrentCUDAStream(ids.device().index()).stream());
    if (rc) raise_engine(rc, 0, "prefill_batch");
    return out;
}

// The reference's GEMV-megakernel prefill class for short prompts
// (megakernel_decode.py:788-1053): same interface, max_prefill_len 64 by default.
class MegakernelFusedPrefillDecoder : public MegakernelPrefillDecoder {
public:
    using MegakernelPrefillDecoder::MegakernelPrefillDecoder;
};

// ---------------------------------------------------------------------------
// chat.py module-function ABI (chat.py:147-323): weights registered in
// module-level state, caller-owned caches and scratch, reference launchers.
std::vector<LDGLayerWeights> g_layer_weights;
torch::Tensor g_d_layer_weights;
torch::Tensor g_embed_weight;
std::vector<std::vector<torch::Tensor>> g_keepalive;

void init_ldg_layer_weights(std::vector<torch::Tensor> input_layernorm_weights, std::vector<torch::Tensor> q_proj_weights,
                            std::vector<torch::Tensor> k_proj_weights, std::vector<torch::Tensor> v_proj_weights,
                            std::vector<torch::Tensor> q_norm_weights, std::vector<torch::Tensor> k_norm_weights,
                            std::vector<torch::Tensor> o_proj_weights,
                            std::vector<torch::Tensor> post_attn_layernorm_weights,
                            std::vector<torch::Tensor> gate_proj_weights, std::vector<torch::Tensor> up_proj_weights,
                            std::vector<torch::Tensor> down_proj_weights) {
    std::vector<std::vector<torch::Tensor>*> lists = {
        &input_layernorm_weights, &q_proj_weights, &k_proj_weights, &v_proj_weights,
        &q_norm_weights, &k_norm_weights, &o_proj_weights, &post_attn_layernorm_weights,
        &gate_proj_weights, &up_proj_weights, &down_proj_weights};
    size_t L = input_layernorm_weights.size();
    if (L < 1 || L > MQ_MAX_LAYERS) throw std::runtime_error("number of layers out of range");
    std::vector<torch::Tensor> flat;
    for (size_t i = 0; i < L; ++i)
        for (int k = 0; k < 11; ++k) {
            if (lists[k]->size() != L) throw std::runtime_error("all eleven weight lists must have the same length");
            check_bf16((*lists[k])[i], kLayerNames[k], layer_shape(k));
            flat.push_back((*lists[k])[i]);
        }
    g_layer_weights.resize(L);
    for (size_t i = 0; i < L; ++i) g_layer_weights[i] = make_layer(flat, i * 11);
    c10::cuda::CUDAGuard guard(flat[0].device());
    g_d_layer_weights = layer_table(g_layer_weights, flat[0].device());
    g_keepalive.assign(1, flat);
}

void init_ldg_embed_weight(torch::Tensor embed_weight) {
    check_bf16(embed_weight, "embed_weight", {kVocab, kHidden});
    g_embed_weight = embed_weight;
}

int decode_ldg_impl(int input_token_id, float* logits, torch::Tensor final_norm_weight, torch::Tensor lm_head_weight,
                    torch::Tensor cos_table, torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
                    torch::Tensor hidden_buffer, torch::Tensor g_activations, torch::Tensor g_residual,
                    torch::Tensor g_q, torch::Tensor g_k, torch::Tensor g_v, torch::Tensor g_attn_out,
                    torch::Tensor g_mlp_intermediate, torch::Tensor g_normalized, torch::Tensor block_max_vals,
                    torch::Tensor block_max_idxs, int num_layers, int position, int cache_len, int max_seq_len) {
    if (!g_d_layer_weights.defined() || !g_embed_weight.defined())
        throw std::runtime_error("call init_ldg_layer_weights and init_ldg_embed_weight first");
    if (num_layers != (int)g_layer_weights.size()) throw std::runtime_error("num_layers does not match the weights");
    if (position < 0 || position >= max_seq_len) throw std::runtime_error("position exceeds max_seq_len");
    if (input_token_id < 0 || input_token_id >= kVocab) throw std::runtime_error("input token out of range");
    check_bf16(k_cache, "k_cache", {num_layers, MQ_NUM_KV_HEADS, max_seq_len, MQ_HEAD_DIM});
    check_bf16(v_cache, "v_cache", {num_layers, MQ_NUM_KV_HEADS, max_seq_len, MQ_HEAD_DIM});
    c10::cuda::CUDAGuard guard(k_cache.device());
    float attn_scale = 1.0f / sqrtf(128.0f);
    auto output_token = torch::empty({1}, torch::dtype(torch::kInt32).device(k_cache.device()));
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(k_cache.device().index()).stream();
    auto ptr = [](torch::Tensor& t) -> void* { return t.defined() && t.numel() ? t.data_ptr() : nullptr; };
    if (logits) {
        launch_ldg_decode_with_logits(input_token_id, output_token.data_ptr<int>(), logits, g_embed_weight.data_ptr(),
                                      reinterpret_cast<const LDGLayerWeights*>(g_d_layer_weights.data_ptr()),
                                      final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
                                      sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                      ptr(hidden_buffer), ptr(g_activations), ptr(g_residual), ptr(g_q), ptr(g_k),
                                      ptr(g_v), ptr(g_attn_out), ptr(g_mlp_intermediate), ptr(g_normalized),
                                      ptr(block_max_vals), ptr(block_max_idxs), num_layers, position, cache_len,
                                      max_seq_len, attn_scale, stream);
    } else {
        launch_ldg_decode(input_token_id, output_token.data_ptr<int>(), g_embed_weight.data_ptr(),
                          reinterpret_cast<const LDGLayerWeights*>(g_d_layer_weights.data_ptr()),
                          final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
                          sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), ptr(hidden_buffer),
                          ptr(g_activations), ptr(g_residual), ptr(g_q), ptr(g_k), ptr(g_v), ptr(g_attn_out),
                          ptr(g_mlp_intermediate), ptr(g_normalized), ptr(block_max_vals), ptr(block_max_idxs),
                          num_layers, position, cache_len, max_seq_len, attn_scale, stream);
    }
    int rc = mq_get_last_error();
    if (rc) raise_engine(rc, 0, "decode_ldg");
    return output_token.item<int>();
}

int decode_ldg(int input_token_id, torch::Tensor final_norm_weight, torch::Tensor lm_head_weight,
               torch::Tensor cos_table, torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
               torch::Tensor hidden_buffer, torch::Tensor g_activations, torch::Tensor g_residual, torch::Tensor g_q,
               torch::Tensor g_k, torch::Tensor g_v, torch::Tensor g_attn_out, torch::Tensor g_mlp_intermediate,
               torch::Tensor g_normalized, torch::Tensor block_max_vals, torch::Tensor block_max_idxs, int num_layers,
               int position, int cache_len, int max_seq_len) {
    return decode_ldg_impl(input_token_id, nullptr, final_norm_weight, lm_head_weight, cos_table, sin_table, k_cache,
                           v_cache, hidden_buffer, g_activations, g_residual, g_q, g_k, g_v, g_attn_out,
                           g_mlp_intermediate, g_normalized, block_max_vals, block_max_idxs, num_layers, position,
                           cache_len, max_seq_len);
}

std::tuple<int, torch::Tensor> decode_ldg_with_logits(
    int input_token_id, torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
    torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor hidden_buffer,
    torch::Tensor g_activations, torch::Tensor g_residual, torch::Tensor g_q, torch::Tensor g_k, torch::Tensor g_v,
    torch::Tensor g_attn_out, torch::Tensor g_mlp_intermediate, torch::Tensor g_normalized,
    torch::Tensor block_max_vals, torch::Tensor block_max_idxs, int num_layers, int position, int cache_len,
    int max_seq_len) {
    auto logits = torch::empty({kVocab}, torch::dtype(torch::kFloat32).device(k_cache.device()));
    int tok = decode_ldg_impl(input_token_id, logits.data_ptr<float>(), final_norm_weight, lm_head_weight, cos_table,
                              sin_table, k_cache, v_cache, hidden_buffer, g_activations, g_residual, g_q, g_k, g_v,
                              g_attn_out, g_mlp_intermediate, g_normalized, block_max_vals, block_max_idxs,
                              num_layers, position, cache_len, max_seq_len);
    return std::make_tuple(tok, logits);
}

}  // namespace


// ---------------------------------------------------------------------------
// Batched greedy decode (config 5 serving path): `batch` independent
// sequences, each with its own cache [L, 8, max_seq_len, 128] and position.
// step() launches one decode step for all of them without a host sync; with
// use_graph the step is captured once per attention-context bucket (chunks of
// 256 positions, doubled) and replayed.
class MegakernelBatchDecoder {
public:
    MegakernelBatchDecoder(torch::Tensor embed_weight, std::vector<torch::Tensor> layer_weights_flat,
                           torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
                           torch::Tensor sin_table, int num_layers, int max_seq_len, int batch, bool use_graph)
        : num_layers_(num_layers), max_seq_len_(max_seq_len), batch_(batch), use_graph_(use_graph) {
        if (num_layers < 1 || num_layers > MQ_MAX_LAYERS) throw std::runtime_error("num_layers out of range");
        if (batch < 1 || batch > 128) throw std::runtime_error("batch must be in [1, 128]");
        if ((int)layer_weights_flat.size() != num_layers * 11)
            throw std::runtime_error("layer_weights_flat must hold num_layers * 11 tensors");
        check_bf16(embed_weight, "embed_weight", {kVocab, kHidden});
        check_bf16(final_norm_weight, "final_norm_weight", {kHidden});
        check_bf16(lm_head_weight, "lm_head_weight", {kVocab, kHidden});
        for (int i = 0; i < num_layers * 11; ++i)
            check_bf16(layer_weights_flat[i], kLayerNames[i % 11], layer_shape(i % 11));
        if (cos_table.dim() != 2 || cos_table.size(0) < max_seq_len || sin_table.sizes() != cos_table.sizes())
            throw std::runtime_error("cos/sin tables must be [>=max_seq_len, 128]");
        device_ = embed_weight.device();
        c10::cuda::CUDAGuard guard(device_);
        keep_ = layer_weights_flat;
        keep_.push_back(embed_weight);
        keep_.push_back(final_norm_weight);
        keep_.push_back(lm_head_weight);
        keep_.push_back(cos_table);
        keep_.push_back(sin_table);
        host_.resize(num_layers);
        for (int i = 0; i < num_layers; ++i) host_[i] = make_layer(layer_weights_flat, (size_t)i * 11);
        auto bf = torch::dtype(torch::kBFloat16).device(device_);
        auto i32 = torch::dtype(torch::kInt32).device(device_);
        k_cache_ = torch::zeros({batch, num_layers, MQ_NUM_KV_HEADS, max_seq_len, MQ_HEAD_DIM}, bf);
        v_cache_ = torch::zeros_like(k_cache_);
        tokens_ = torch::zeros({batch}, i32);
        positions_ = torch::zeros({batch}, i32);
        err_ = torch::zeros({1}, i32);
        logits_ = torch::empty({batch, kVocab}, torch::dtype(torch::kFloat32).device(device_));
        ws_ = torch::empty({(int64_t)mq_decode_batch_workspace_bytes(batch, max_seq_len)},
                           torch::dtype(torch::kUInt8).device(device_));
        p_ = {};
        p_.tokens = tokens_.data_ptr<int>();
        p_.positions = positions_.data_ptr<int>();
        p_.batch = batch;
        p_.embed = embed_weight.data_ptr();
        p_.layers_host = host_.data();
        p_.final_norm = final_norm_weight.data_ptr();
        p_.lm_head = lm_head_weight.data_ptr();
        p_.cos_table = cos_table.data_ptr();
        p_.sin_table = sin_table.data_ptr();
        p_.k_cache = k_cache_.data_ptr();
        p_.v_cache = v_cache_.data_ptr();
        p_.cache_seq_stride = (long long)num_layers * MQ_NUM_KV_HEADS * max_seq_len * MQ_HEAD_DIM;
        p_.num_layers = num_layers;
        p_.max_seq_len = max_seq_len;
        p_.attn_scale = 1.0f / sqrtf(128.0f);
        p_.workspace = ws_.data_ptr();
        p_.workspace_bytes = (size_t)ws_.numel();
        p_.err_flag = err_.data_ptr<int>();
    }
    ~MegakernelBatchDecoder() {
        drop_graph();
        if (cap_stream_) cudaStreamDestroy(cap_stream_);
    }

    // tokens / positions: int [batch] (any device); position b must be < max_seq_len.
    void set_state(torch::Tensor tokens, torch::Tensor positions) {
        auto t = tokens.to(torch::kInt32).cpu().contiguous();
        auto q = positions.to(torch::kInt32).cpu().contiguous();
        if (t.numel() != batch_ || q.numel() != batch_) throw std::runtime_error("tokens/positions must have batch entries");
        int mx = 0;
        for (int b = 0; b < batch_; ++b) {
            const int tk = t.data_ptr<int>()[b], ps = q.data_ptr<int>()[b];
            if (tk < 0 || tk >= kVocab) throw std::runtime_error("token out of range");
            if (ps < 0 || ps >= max_seq_len_) throw std::runtime_error("position out of range");
            mx = std::max(mx, ps);
        }
        c10::cuda::CUDAGuard guard(device_);
        tokens_.copy_(t);
        positions_.copy_(q);
        max_pos_ = mx;
    }

    // One step for all sequences; returns the device token tensor (updated in place).
    torch::Tensor step(bool with_logits) {
        if (max_pos_ >= max_seq_len_) throw std::runtime_error("position exceeds max_seq_len");
        c10::cuda::CUDAGuard guard(device_);
        cudaStream_t st = c10::cuda::getCurrentCUDAStream(device_.index()).stream();
        const int chunks = (max_pos_ + 1 + 255) / 256;
        int bucket = 1;
        while (bucket < chunks) bucket *= 2;
        const int ctx = std::min(bucket * 256, max_seq_len_);
        p_.max_context = ctx;
        p_.logits = with_logits ? logits_.data_ptr<float>() : nullptr;
        if (!use_graph_ || with_logits) {
            const int rc = mq_decode_batch(&p_, st);
            if (rc) raise_engine(rc, 0, "batch step");
        } else {
            if (!graph_exec_ || graph_ctx_ != ctx || graph_stream_ != st) {
                drop_graph();
                // one eager step before capture configures the kernels (attributes are not graph nodes)
                if (!warmed_) {
                    const int rc = mq_decode_batch(&p_, st);
                    if (rc) raise_engine(rc, 0, "batch step");
                    warmed_ = true;
                    ++max_pos_;
                    return tokens_;
                }
                // captured on a private stream (the legacy default stream cannot be captured)
                if (!cap_stream_ && cudaStreamCreateWithFlags(&cap_stream_, cudaStreamNonBlocking) != cudaSuccess)
                    throw std::runtime_error("cudaStreamCreateWithFlags failed");
                cudaGraph_t g = nullptr;
                if (cudaStreamBeginCapture(cap_stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
                    throw std::runtime_error("cudaStreamBeginCapture failed");
                const int rc = mq_decode_batch(&p_, cap_stream_);
                const cudaError_t ce = cudaStreamEndCapture(cap_stream_, &g);
                if (rc || ce != cudaSuccess) {
                    if (g) cudaGraphDestroy(g);
                    raise_engine(rc ? rc : MQ_ERR_CUDA, 0, "batch step capture");
                }
                if (cudaGraphInstantiate(&graph_exec_, g, 0) != cudaSuccess) {
                    cudaGraphDestroy(g);
                    graph_exec_ = nullptr;
                    throw std::runtime_error("cudaGraphInstantiate failed");
                }
                cudaGraphDestroy(g);
                graph_ctx_ = ctx;
                graph_stream_ = st;
            }
            if (cudaGraphLaunch(graph_exec_, st) != cudaSuccess) throw std::runtime_error("cudaGraphLaunch failed");
        }
        ++max_pos_;
        return tokens_;
    }

    // The additive batch entrypoint: consumes tokens[b] (int [batch]) at each
    // sequence's current position and returns the greedy next tokens (device
    // int32 [batch]); positions advance by one.
    torch::Tensor decode_step_batched(torch::Tensor tokens) {
        if (tokens.numel() != batch_) throw std::runtime_error("tokens must have batch entries");
        c10::cuda::CUDAGuard guard(device_);
        tokens_.copy_(tokens.to(torch::kInt32).view({batch_}), true);
        return step(false).clone();
    }

    // Runs n steps and returns the generated tokens [n, batch] (device).
    torch::Tensor generate(int n) {
        c10::cuda::CUDAGuard guard(device_);
        auto out = torch::empty({n, batch_}, tokens_.options());
        for (int i = 0; i < n; ++i) out[i].copy_(step(false), true);
        return out;
    }

    // Raises if a device wait ran out (synchronises).
    void check() {
        c10::cuda::CUDAGuard guard(device_);
        const int e = err_.cpu().item<int>();
        if (e) raise_engine(MQ_ERR_PIPE_TIMEOUT, (uint32_t)e, "batch decode");
    }

    torch::Tensor tokens() { return tokens_; }
    torch::Tensor positions() { return positions_; }
    torch::Tensor logits() { return logits_; }
    torch::Tensor get_k_cache() { return k_cache_; }
    torch::Tensor get_v_cache() { return v_cache_; }
    int batch() const { return batch_; }
    int64_t workspace_bytes() const { return ws_.numel(); }

private:
    void drop_graph() {
        if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
        graph_exec_ = nullptr;
    }
    int num_layers_, max_seq_len_, batch_;
    bool use_graph_, warmed_ = false;
    int max_pos_ = 0, graph_ctx_ = 0;
    cudaStream_t graph_stream_ = nullptr, cap_stream_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
    torch::Device device_{torch::kCPU};
    std::vector<torch::Tensor> keep_;
    std::vector<LDGLayerWeights> host_;
    torch::Tensor k_cache_, v_cache_, tokens_, positions_, err_, logits_, ws_;
    mq_decode_batch_params p_;
};

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "B200 (sm_100a) Qwen3-0.6B decode engine: reference-compatible torch extension";
    py::class_<MegakernelDecoder>(m, "MegakernelDecoder")
        .def(py::init<torch::Tensor, std::vector<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor,
                      torch::Tensor, int, int>(),
             py::arg("embed_weight"), py::arg("layer_weights_flat"), py::arg("final_norm_weight"),
             py::arg("lm_head_weight"), py::arg("cos_table"), py::arg("sin_table"), py::arg("num_layers"),
             py::arg("max_seq_len"))
        .def("decode_step", &MegakernelDecoder::decode_step)
        .def("decode_step_with_logits", &MegakernelDecoder::decode_step_with_logits)
        .def("generate_greedy", &MegakernelDecoder::generate_greedy)
        .def("decode_step_async", &MegakernelDecoder::decode_step_async)
        .def("check", &MegakernelDecoder::check)
        .def("reset", &MegakernelDecoder::reset)
        .def("position", &MegakernelDecoder::position)
        .def("set_position", &MegakernelDecoder::set_position)
        .def("get_k_cache", &MegakernelDecoder::get_k_cache)
        .def("get_v_cache", &MegakernelDecoder::get_v_cache)
        .def("get_hidden_buffer", &MegakernelDecoder::get_hidden_buffer)
        .def("get_normalized", &MegakernelDecoder::get_normalized)
        .def("last_token", &MegakernelDecoder::last_token)
        .def("set_num_ctas", &MegakernelDecoder::set_num_ctas)
        .def("num_ctas", &MegakernelDecoder::num_ctas)
        .def("set_attn_chunk", &MegakernelDecoder::set_attn_chunk)
        .def("set_timeout_ns", &MegakernelDecoder::set_timeout_ns)
        .def("set_inject_skip_cta", &MegakernelDecoder::set_inject_skip_cta)
        .def("set_trace", &MegakernelDecoder::set_trace)
        .def("set_step_epoch", &MegakernelDecoder::set_step_epoch);
    py::class_<MegakernelTPDecoder, MegakernelDecoder>(m, "MegakernelTPDecoder")
        .def(py::init<torch::Tensor, std::vector<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor,
                      torch::Tensor, int, int, int, int>(),
             py::arg("embed_weight"), py::arg("layer_weights"), py::arg("final_norm_weight"),
             py::arg("lm_head_weight"), py::arg("cos_table"), py::arg("sin_table"), py::arg("num_layers"),
             py::arg("max_seq_len"), py::arg("tp_rank"), py::arg("tp_size"))
        .def("ipc_handle", &MegakernelTPDecoder::ipc_handle)
        .def("connect", &MegakernelTPDecoder::connect)
        .def("zero_workspace", &MegakernelTPDecoder::zero_workspace)
        .def("tp_rank", &MegakernelTPDecoder::tp_rank)
        .def("tp_size", &MegakernelTPDecoder::tp_size)
        .def("connected", &MegakernelTPDecoder::connected);
    py::class_<MegakernelPrefillDecoder, MegakernelDecoder>(m, "MegakernelPrefillDecoder")
        .def(py::init<torch::Tensor, std::vector<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor,
                      torch::Tensor, int, int, int>(),
             py::arg("embed_weight"), py::arg("layer_weights_flat"), py::arg("final_norm_weight"),
             py::arg("lm_head_weight"), py::arg("cos_table"), py::arg("sin_table"), py::arg("num_layers"),
             py::arg("max_seq_len"), py::arg("max_prefill_len") = 512)
        .def("prefill_step", &MegakernelPrefillDecoder::prefill_step)
        .def("prefill_step_with_logits", &MegakernelPrefillDecoder::prefill_step_with_logits)
        .def("prefill_step_sequential", &MegakernelPrefillDecoder::prefill_step_sequential)
        .def("max_prefill_len", &MegakernelPrefillDecoder::max_prefill_len);
    py::class_<MegakernelFusedPrefillDecoder, MegakernelPrefillDecoder>(m, "MegakernelFusedPrefillDecoder")
        .def(py::init<torch::Tensor, std::vector<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor,
                      torch::Tensor, int, int, int>(),
             py::arg("embed_weight"), py::arg("layer_weights_flat"), py::arg("final_norm_weight"),
             py::arg("lm_head_weight"), py::arg("cos_table"), py::arg("sin_table"), py::arg("num_layers"),
             py::arg("max_seq_len"), py::arg("max_prefill_len") = 64);
    py::class_<MegakernelBatchDecoder>(m, "MegakernelBatchDecoder")
        .def(py::init<torch::Tensor, std::vector<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor,
                      torch::Tensor, int, int, int, bool>(),
             py::arg("embed_weight"), py::arg("layer_weights_flat"), py::arg("final_norm_weight"),
             py::arg("lm_head_weight"), py::arg("cos_table"), py::arg("sin_table"), py::arg("num_layers"),
             py::arg("max_seq_len"), py::arg("batch"), py::arg("use_graph") = true)
        .def("set_state", &MegakernelBatchDecoder::set_state)
        .def("step", &MegakernelBatchDecoder::step, py::arg("with_logits") = false)
        .def("generate", &MegakernelBatchDecoder::generate)
        .def("decode_step_batched", &MegakernelBatchDecoder::decode_step_batched)
        .def("check", &MegakernelBatchDecoder::check)
        .def("tokens", &MegakernelBatchDecoder::tokens)
        .def("positions", &MegakernelBatchDecoder::positions)
        .def("logits", &MegakernelBatchDecoder::logits)
        .def("get_k_cache", &MegakernelBatchDecoder::get_k_cache)
        .def("get_v_cache", &MegakernelBatchDecoder::get_v_cache)
        .def("batch", &MegakernelBatchDecoder::batch)
        .def("workspace_bytes", &MegakernelBatchDecoder::workspace_bytes);
    m.def("init_ldg_layer_weights", &init_ldg_layer_weights);
    m.def("init_ldg_embed_weight", &init_ldg_embed_weight);
    m.def("decode_ldg", &decode_ldg);
    m.def("decode_ldg_with_logits", &decode_ldg_with_logits);
    m.def("workspace_bytes", []() { return (int64_t)mq_decode_workspace_bytes(); });
    m.def("default_ctas", []() { return mq_decode_default_ctas(); });
    m.def("prefill_batch", &prefill_batch, py::arg("embed"), py::arg("layer_weights_flat"), py::arg("final_norm"),
          py::arg("lm_head"), py::arg("cos"), py::arg("sin"), py::arg("ids"), py::arg("k_cache"), py::arg("v_cache"),
          py::arg("logits") = py::none(), py::arg("workspace") = py::none());
    m.def("prefill_workspace_bytes", [](int b, int s) { return (int64_t)mq_prefill_workspace_bytes(b, s); });
    m.def("version", []() { return std::string(mq_version()); });
}
