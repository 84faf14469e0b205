// CUDA host runtime of the Qwen3 token loop: the reference's host object model
// (Config / RunState / BaseLayer subclasses / BaseModel, include/minfer/base/*.hpp,
// include/minfer/models/qwen3/module.hpp) rebuilt over the libmfcuda C ABI.
// Each layer class has a `cuda_forward` that issues the fused device ops;
// BaseModel::forward becomes one frame (a captured CUDA graph per frame kind).
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf.hpp"
#include "minfer_cuda.h"
#include "sampler.hpp"

namespace minfer {

constexpr int kPrefillChunk = 4096;  // prompt tokens per batched-prefill pass
constexpr int kTopkMax = 64;         // largest top_k sampled from device candidates (mf_topk)
// step-record bytes read back after a host-driven frame: token, pos, next_token,
// chain, frame, the exchange status (MF_STEP_STATUS) and the decode-kernel
// status (MF_STEP_DSTATUS)
constexpr size_t kStepReadback = 28;

// A bounded wait on the device gave up (a tensor-parallel exchange whose peer
// did not arrive, or a prefill kernel's pipeline wait): the results of that
// work are invalid. The C ABI reports it as MF_E_TIMEOUT.
struct WaitTimeout : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// include/minfer/base/config.hpp:22 plus the CUDA device this runtime adds
enum class DeviceType : int { CPU = 0, METAL = 1, CUDA = 2 };

// include/minfer/base/config.hpp:37-51 (RunParams)
struct RunParams {
    size_t num_iters = 0;
    size_t max_seq_len = 0;
    size_t top_k = 1;
    float temp = 0.0f;
    float top_p = 1.0f;
    float min_p = 0.0f;
    float penalty_pres = 0.0f;
    int seed = 0;
};

// include/minfer/base/config.hpp:53-75 (Config), filled from GGUF metadata as
// src/base/config.cpp:277-337 does.
struct Config {
    size_t vocab_size = 0, model_max_seq_len = 0;
    int d_model = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, d_head = 0, d_rotary = 0, d_ff = 0;
    int n_active_experts = 0, n_experts = 0;
    float rms_norm_eps = 1e-6f, freq_base = 1e6f;
    uint32_t eos_token_id = 0, padding_token_id = 0;
    size_t user_max_seq_len = 0, top_k = 1, num_iters = 0;
    int seed = 0;
    float temp = 0.f, top_p = 1.f, min_p = 0.f, penalty_pres = 0.f;
    DataType weight_dtype = DataType::INVALID;  // projection weights
    DataType head_dtype = DataType::INVALID;    // lm_head weight
    bool untied_head = false;
    // tensor parallelism: this process holds rank tp_rank of tp_size
    int tp_rank = 0, tp_size = 1;

    // Dense models split attention and FFN (tensor parallelism). MoE models
    // do the same when the KV heads divide over the ranks (every expert's FFN
    // rows split like a dense FFN: moe_tp), else they split their experts over
    // the ranks and replicate attention (expert parallelism).
    bool moe_tp = false;
    bool ep() const { return tp_size > 1 && n_experts > 0 && !moe_tp; }
    bool attn_split() const { return tp_size > 1 && (n_experts == 0 || moe_tp); }
    int heads_local() const { return attn_split() ? n_heads / tp_size : n_heads; }
    int kv_heads_local() const { return attn_split() ? n_kv_heads / tp_size : n_kv_heads; }
    int ff_local() const { return attn_split() ? d_ff / tp_size : d_ff; }
    int experts_local() const { return ep() ? n_experts / tp_size : n_experts; }
    int expert_lo() const { return ep() ? tp_rank * experts_local() : 0; }
    // vocabulary rows [vocab_offset(), vocab_offset() + vocab_local()) of the lm_head
    size_t vocab_local() const { return vocab_size / tp_size + ((size_t)tp_rank < vocab_size % tp_size ? 1 : 0); }
    size_t vocab_offset() const {
        return (size_t)tp_rank * (vocab_size / tp_size) + std::min<size_t>(tp_rank, vocab_size % tp_size);
    }

    static Config from_gguf(const GGUFFile& f, const RunParams& rp);
};

// include/minfer/base/stats.hpp:3-15
struct GenStats {
    int num_tokens_gen = 0;
    float ttft = 0.f;
    float throughput = 0.f;
    float prefill_time = 0.f;
    float bandwidth = 0.f;
    double decode_seconds = 0.0;
    double bytes_read = 0.0;
};

// Device-resident run state (include/minfer/base/config.hpp:77-102). The KV
// cache layout is [layer][kv_head][position][d_head], fp32 as the reference
// keeps it, or bf16 when the model was set to a bf16 cache.
struct RunState {
    int rank = 0;
    void* stream = nullptr;
    mf_buf *x = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    mf_buf *scores = nullptr, *expert_ids = nullptr, *expert_w = nullptr;
    mf_buf *k_cache = nullptr, *v_cache = nullptr, *rope = nullptr;
    mf_buf *attn_ws = nullptr, *lmh_ws = nullptr;
    int32_t* h_step = nullptr;  // pinned {token, pos, next_token, chain}
    void* d_step = nullptr;
    float* h_logits = nullptr;  // pinned copy of the last logits (host-logit frames)
    // sampling from device top-k candidates: k > 0 while a frame reads back k
    // (id, logit) pairs instead of the whole vocabulary
    int topk_k = 0;
    mf_buf *topk_ids = nullptr, *topk_vals = nullptr, *topk_ws = nullptr;
    size_t topk_ws_bytes = 0;
    void* h_topk = nullptr;  // pinned: kTopkMax ids, then kTopkMax logits
    // sampling on the device (chained sampled frames): the draws of the run
    // [max_seq + 1], the sampled ids [max_seq + 1], flags (mf_sample_step)
    bool device_sample = false;
    float smp_temp = 0.f, smp_top_p = 1.f, smp_min_p = 0.f;
    int smp_top_k = 0, smp_n_draws = 0;
    mf_buf *smp_draws = nullptr, *smp_ids = nullptr, *smp_flags = nullptr;
    int attn_split = 1;
    int cur_pos = 0;
    uint32_t token_id = 0;
    bool compute_logits = false;
    bool host_logits = false;
    size_t kv_bytes_per_pos = 0;
    size_t kv_layer_elems = 0;  // this rank's n_kv_heads * max_seq * d_head
    int kv_dtype = MF_F32;      // MF_F32 or MF_BF16
    size_t kv_elem = 4;         // bytes per cache element
    void* kv_layer(const mf_buf* cache, int layer) const {
        return (char*)mf_ptr(cache) + (size_t)layer * kv_layer_elems * kv_elem;
    }
    // tensor parallelism: exchange state and the two residual buffers the
    // all-reduces alternate between (x aliases xb[0])
    mf_comm* comm = nullptr;
    mf_buf* xb[2] = {nullptr, nullptr};
    // batched prefill (allocated on first use): residual rows, bf16 hi/lo
    // GEMM operands (two pairs: a GEMM's input and its SwiGLU output), the
    // fused QKV rows, normalised/rotated queries, token ids
    int pf_cap = 0;  // rows per chunk
    mf_buf *pf_x = nullptr, *pf_hi = nullptr, *pf_lo = nullptr, *pf_hhi = nullptr, *pf_hlo = nullptr;
    mf_buf *pf_qkv = nullptr, *pf_q = nullptr, *pf_tok = nullptr;
    mf_buf* pf_gu = nullptr;  // fp32-weight models: gate/up rows before the SwiGLU [rows][2 d_ff]
    // MoE layers: normalised rows [rows][d] (fp32, the router's input), per
    // layer the prompt's expert ids / weights [L][rows][k], the grouping
    // (expert row and tile offsets [E + 1], grouped row of each (token, slot)
    // [rows * k]), the grouped operands [rows * k][d] (bf16 hi/lo), the
    // grouped SwiGLU outputs [rows * k][d_ff] (bf16 hi/lo) and down outputs
    // [rows * k][d] (fp32)
    mf_buf *pf_xn = nullptr, *pf_ids = nullptr, *pf_wts = nullptr, *pf_grows = nullptr, *pf_gtiles = nullptr;
    mf_buf *pf_pos = nullptr, *pf_ghi = nullptr, *pf_glo = nullptr, *pf_mhi = nullptr, *pf_mlo = nullptr;
    mf_buf* pf_y = nullptr;
    mf_buf* pf_att = nullptr;  // tensor-core attention operands (bf16 hi/lo Q, K, V^T)
    size_t pf_att_bytes = 0;
    bool pf_simt_attn = false;  // MF_PREFILL_SIMT_ATTN=1: the SIMT attention kernel instead
    // tensor parallelism: prompt rows one bulk exchange slot holds, exchanges so far, a zero partial
    int pf_bulk_rows = 0;
    unsigned long long pf_epoch = 0;
    mf_buf* zero_d = nullptr;
};

class BaseLayer {
public:
    virtual ~BaseLayer();
    virtual void cuda_forward(RunState& rs) = 0;
    // Batched prefill of rows [0, n) of the prefill buffers at positions pos0.. (tcgen05 GEMMs).
    virtual void prefill_forward(RunState& rs, int n, int pos0);
    // fp32-weight layers make the bf16 hi/lo weight copies the prefill GEMMs take.
    virtual void split_for_prefill(int rank) {}
    virtual void upload(const GGUFFile& f, int rank) = 0;
    size_t read_bytes() const { return read_bytes_; }

protected:
    void own(mf_buf* b) { bufs_.push_back(b); }
    size_t read_bytes_ = 0;
    std::vector<mf_buf*> bufs_;
};

class Qwen3Model {
public:
    Qwen3Model(const std::string& path, const RunParams& rp, int rank = 0, int tp_rank = 0, int tp_size = 1);
    ~Qwen3Model();

    void set_device(DeviceType d);  // CUDA: upload weights, allocate the run state
    // KV cache element type (MF_F32, the reference's, or MF_BF16); set before
    // set_device(CUDA). A bf16 cache rounds every appended row to nearest even.
    void set_kv_dtype(int dtype);
    int kv_dtype() const { return kv_dtype_; }
    DeviceType device() const { return device_; }
    const Config& config() const { return cfg_; }

    // One token step (BaseModel::forward, src/base/model.cpp:36-59) as one frame.
    void forward(uint32_t token, int pos, bool compute_logits, bool host_logits);
    const float* host_logits() const { return rs_.h_logits; }
    uint32_t device_argmax() const { return (uint32_t)rs_.h_step[2]; }
    // Bytes the reference counts per forward (src/base/module.cpp read bytes).
    size_t read_bytes(bool with_logits) const;
    // Batched prefill of `n` prompt tokens at positions [pos0, pos0 + n) in
    // chunks (the reference's token-by-token prefill, src/base/model.cpp:120-129,
    // as tensor-core GEMMs); leaves the last token's logits / greedy id like
    // forward(). False when the model is not eligible (see prefill_supported).
    bool prefill(const uint32_t* tokens, int n, int pos0, bool compute_logits, bool host_logits);
    bool prefill_supported() const;

    struct GenOptions {
        bool stop_at_eos = false;
        const uint32_t* forced = nullptr;  // teacher forcing: feed forced[i] after step i
        bool trace = false;                // host logits every step (margins, callbacks)
        bool batched_prefill = true;       // tensor-core prefill when supported (else token by token)
        std::function<void(size_t step, const float* logits, uint32_t picked)> on_step;
    };
    // BaseModel::generate without the tokenizer (src/base/model.cpp:99-186).
    std::vector<uint32_t> generate(const std::vector<uint32_t>& prompt, size_t n_gen, const GenOptions& opt,
                                   GenStats* stats, std::vector<float>* margins);
    // BaseModel::benchmark (src/base/model.cpp:188-236): 512 random prompt ids
    // (std::mt19937(seed), uniform over the vocabulary) prefilled with logits
    // on the last only ("pp512"), then 128 forwards of fresh random ids at
    // positions 0..127 with logits ("tg128"); the same byte count and
    // bandwidth formula. batched_prefill runs the 512 ids through the
    // tensor-core prefill instead of 512 decode frames (when supported).
    GenStats benchmark(bool batched_prefill);
    // Greedy decode with the device feeding itself: frame i embeds the argmax
    // of frame i-1 (chained step record), frames are queued back to back with
    // no host round trip. Returns the last greedy id; the caller times it.
    uint32_t decode_chained(uint32_t token, int start_pos, int n);
    // Sampled decode with the device feeding itself: frame i forwards the id
    // frame i-1 sampled on the device (mf_sample_step with draws[i]), no host
    // round trip. Returns the n sampled ids; *tie is set when equal logits
    // among a step's candidates made the order of equal values decide.
    std::vector<uint32_t> decode_sampled_chained(uint32_t token, int start_pos, int n, const std::vector<float>& draws,
                                                 bool* tie);

    // Tensor parallelism: after set_device(CUDA), every rank exports its
    // handle, and connects with all ranks' handles ordered by tp_rank.
    void comm_handle(void* out, size_t n) const;
    void comm_connect(const void* handles, size_t n);
    int comm_status(int* status);

    // Test access
    int read_experts(int layer, int* ids, float* w) const;
    // the expert ids / weights the last batched prefill chose for its first
    // n tokens at `layer` ([n][k] each)
    int read_prefill_experts(int layer, int* ids, float* w, int n) const;
    int read_kv(int layer, float* k, float* v, int n_pos) const;
    int read_x(float* x) const;
    void reset_sampler();

private:
    void build_layers();
    void alloc_state();
    void alloc_prefill(int rows);
    void issue_frame(bool readback);
    void read_back_logits();  // logits, or their top-k candidates, to pinned host memory
    void read_full_logits();  // the last frame's logits to pinned host memory, synchronously
    // throws WaitTimeout when the step record read back last carries exchange
    // or decode-kernel status bits
    void check_exchange_status() const;

    std::string path_;
    GGUFFile file_;
    Config cfg_;
    RunParams rp_;
    int rank_ = 0;
    int frame_base_ = 0;  // this model's frame ids: frame_base_ + kind
    // Sequence number of this model's frames, written to the step record's
    // frame field (tensor-parallel exchange tags derive from it). Kept per
    // model: the step record is shared by every model on the device, and all
    // ranks of a sharded model must count only that model's frames.
    int32_t frame_seq_ = 0;
    int32_t next_frame() { return ++frame_seq_; }
    DeviceType device_ = DeviceType::CPU;
    int kv_dtype_ = MF_F32;
    std::vector<std::unique_ptr<BaseLayer>> layers_;
    RunState rs_;
    std::unique_ptr<Sampler> sampler_;
    std::vector<mf_buf*> state_bufs_;
};

}  // namespace minfer
