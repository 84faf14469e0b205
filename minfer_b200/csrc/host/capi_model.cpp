// extern "C" surface of the host runtime (include/minfer_model.h).
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>
#include <stdexcept>

#include "minfer_model.h"
#include "model.hpp"
#include "tokenizer.hpp"

struct mf_model {
    std::unique_ptr<minfer::Qwen3Model> m;
};
struct mf_tokenizer {
    std::unique_ptr<minfer::Qwen3Tokenizer> t;
};

namespace {
thread_local char g_host_err[512] = "";
int herr(int code, const char* msg) {
    std::snprintf(g_host_err, sizeof(g_host_err), "%s", msg);
    return code;
}
}  // namespace

#define MF_TRY(body)                                   \
    try {                                              \
        body;                                          \
    } catch (const minfer::WaitTimeout& e) {       \
        return herr(MF_E_TIMEOUT, e.what());           \
    } catch (const std::bad_alloc&) {                  \
        return herr(MF_E_OOM, "host allocation failed"); \
    } catch (const std::invalid_argument& e) {         \
        return herr(MF_E_INVALID, e.what());           \
    } catch (const std::exception& e) {                \
        return herr(MF_E_STATE, e.what());             \
    }

extern "C" {

// Host-runtime failures are reported through this function; libmfcuda's own
// message is used when the host layer has none.
int mf_host_last_error(char* buf, size_t n) {
    if (!buf || n == 0) return MF_E_INVALID;
    if (g_host_err[0]) {
        std::snprintf(buf, n, "%s", g_host_err);
        return MF_OK;
    }
    return mf_last_error(buf, n);
}

int mf_model_load(const char* gguf_path, const mf_run_params* rp, int rank, mf_model** out) {
    return mf_model_load_tp(gguf_path, rp, rank, 0, 1, out);
}

int mf_model_load_tp(const char* gguf_path, const mf_run_params* rp, int rank, int tp_rank, int tp_size,
                     mf_model** out) {
    if (!gguf_path || !rp || !out) return herr(MF_E_INVALID, "null argument");
    g_host_err[0] = 0;
    minfer::RunParams p;
    p.num_iters = rp->num_iters;
    p.max_seq_len = rp->max_seq_len;
    p.top_k = rp->top_k;
    p.temp = rp->temp;
    p.top_p = rp->top_p;
    p.min_p = rp->min_p;
    p.penalty_pres = rp->penalty_pres;
    p.seed = rp->seed;
    MF_TRY({
        auto* h = new mf_model;
        try {
            h->m = std::make_unique<minfer::Qwen3Model>(gguf_path, p, rank, tp_rank, tp_size);
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
    return MF_OK;
}

int mf_model_set_kv_dtype(mf_model* m, int dtype) {
    if (!m) return herr(MF_E_INVALID, "null model");
    g_host_err[0] = 0;
    MF_TRY(m->m->set_kv_dtype(dtype));
    return MF_OK;
}

int mf_model_to_cuda(mf_model* m) {
    if (!m) return herr(MF_E_INVALID, "null model");
    g_host_err[0] = 0;
    MF_TRY(m->m->set_device(minfer::DeviceType::CUDA));
    return MF_OK;
}

int mf_model_comm_handle(const mf_model* m, void* out, size_t n) {
    if (!m || !out) return herr(MF_E_INVALID, "null argument");
    g_host_err[0] = 0;
    MF_TRY(m->m->comm_handle(out, n));
    return MF_OK;
}

int mf_model_comm_connect(mf_model* m, const void* handles, size_t n) {
    if (!m || !handles) return herr(MF_E_INVALID, "null argument");
    g_host_err[0] = 0;
    MF_TRY(m->m->comm_connect(handles, n));
    return MF_OK;
}

int mf_model_comm_status(mf_model* m, int* status) {
    if (!m || !status) return herr(MF_E_INVALID, "null argument");
    const int rc = m->m->comm_status(status);
    return rc ? herr(rc, "exchange status read failed") : MF_OK;
}

int mf_model_info_get(const mf_model* m, mf_model_info* out) {
    if (!m || !out) return herr(MF_E_INVALID, "null argument");
    const minfer::Config& c = m->m->config();
    std::memset(out, 0, sizeof(*out));
    out->vocab_size = c.vocab_size;
    out->max_seq_len = c.user_max_seq_len;
    out->d_model = c.d_model;
    out->n_layers = c.n_layers;
    out->n_heads = c.n_heads;
    out->n_kv_heads = c.n_kv_heads;
    out->d_head = c.d_head;
    out->d_ff = c.d_ff;
    out->n_experts = c.n_experts;
    out->n_active_experts = c.n_active_experts;
    out->weight_dtype = (int)c.weight_dtype;
    out->untied_head = c.untied_head ? 1 : 0;
    out->eos_token_id = c.eos_token_id;
    out->rms_norm_eps = c.rms_norm_eps;
    out->freq_base = c.freq_base;
    if (m->m->device() == minfer::DeviceType::CUDA) {
        out->read_bytes_logits = m->m->read_bytes(true);
        out->read_bytes_no_logits = m->m->read_bytes(false);
    }
    out->kv_bytes_per_pos = 2ull * c.n_layers * c.kv_heads_local() * c.d_head * (m->m->kv_dtype() == MF_BF16 ? 2 : 4);
    out->tp_rank = c.tp_rank;
    out->tp_size = c.tp_size;
    out->expert_parallel = c.ep() ? 1 : 0;
    return MF_OK;
}

void mf_model_free(mf_model* m) { delete m; }

int mf_model_forward(mf_model* m, uint32_t token, int pos, int compute_logits, int host_logits) {
    if (!m) return herr(MF_E_INVALID, "null model");
    g_host_err[0] = 0;
    MF_TRY(m->m->forward(token, pos, compute_logits != 0, host_logits != 0));
    return MF_OK;
}

int mf_model_logits(const mf_model* m, float* out, size_t n) {
    if (!m || !out) return herr(MF_E_INVALID, "null argument");
    const size_t V = m->m->config().vocab_size;
    if (n > V) return herr(MF_E_INVALID, "more logits requested than the vocabulary holds");
    if (!m->m->host_logits()) return herr(MF_E_STATE, "model is not on CUDA");
    std::memcpy(out, m->m->host_logits(), n * sizeof(float));
    return MF_OK;
}

int mf_model_argmax(const mf_model* m, uint32_t* out) {
    if (!m || !out) return herr(MF_E_INVALID, "null argument");
    *out = m->m->device_argmax();
    return MF_OK;
}

int mf_model_generate(mf_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_gen, int flags,
                      const uint32_t* forced, uint32_t* out_ids, size_t* n_out, float* margins,
                      mf_gen_stats* stats) {
    return mf_model_generate_logits(m, prompt, n_prompt, n_gen, flags, forced, out_ids, n_out, margins, stats,
                                    nullptr, 0, nullptr);
}

int mf_model_generate_logits(mf_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_gen, int flags,
                             const uint32_t* forced, uint32_t* out_ids, size_t* n_out, float* margins,
                             mf_gen_stats* stats, const size_t* steps, size_t n_steps, float* logits_out) {
    if (!m || !prompt || !out_ids || !n_out) return herr(MF_E_INVALID, "null argument");
    if (n_steps && (!steps || !logits_out)) return herr(MF_E_INVALID, "steps and logits_out are required");
    g_host_err[0] = 0;
    MF_TRY({
        minfer::Qwen3Model::GenOptions o;
        o.stop_at_eos = (flags & MF_GEN_STOP_AT_EOS) != 0;
        o.batched_prefill = (flags & MF_GEN_TOKEN_PREFILL) == 0;
        o.trace = (flags & MF_GEN_MARGINS) != 0 || n_steps > 0;
        o.forced = forced;
        if (n_steps) {
            const size_t V = m->m->config().vocab_size;
            o.on_step = [=](size_t step, const float* lg, uint32_t) {
                for (size_t i = 0; i < n_steps; ++i)
                    if (steps[i] == step && lg) std::memcpy(logits_out + i * V, lg, V * sizeof(float));
            };
        }
        std::vector<uint32_t> pr(prompt, prompt + n_prompt);
        minfer::GenStats st;
        std::vector<float> mg;
        std::vector<uint32_t> ids = m->m->generate(pr, n_gen, o, &st, o.trace ? &mg : nullptr);
        std::memcpy(out_ids, ids.data(), ids.size() * sizeof(uint32_t));
        *n_out = ids.size();
        if (margins && o.trace) std::memcpy(margins, mg.data(), mg.size() * sizeof(float));
        if (stats) {
            stats->num_tokens_gen = st.num_tokens_gen;
            stats->ttft = st.ttft;
            stats->throughput = st.throughput;
            stats->prefill_time = st.prefill_time;
            stats->bandwidth = st.bandwidth;
            stats->decode_seconds = st.decode_seconds;
            stats->bytes_read = st.bytes_read;
        }
    });
    return MF_OK;
}

int mf_model_benchmark(mf_model* m, int flags, mf_gen_stats* stats) {
    if (!m || !stats) return herr(MF_E_INVALID, "null argument");
    g_host_err[0] = 0;
    MF_TRY({
        const minfer::GenStats st = m->m->benchmark((flags & MF_GEN_TOKEN_PREFILL) == 0);
        stats->num_tokens_gen = st.num_tokens_gen;
        stats->ttft = st.ttft;
        stats->throughput = st.throughput;
        stats->prefill_time = st.prefill_time;
        stats->bandwidth = st.bandwidth;
        stats->decode_seconds = st.decode_seconds;
        stats->bytes_read = st.bytes_read;
    });
    return MF_OK;
}

int mf_model_prefill(mf_model* m, const uint32_t* tokens, size_t n, int pos0, int compute_logits, int host_logits) {
    if (!m || !tokens || n == 0) return herr(MF_E_INVALID, "bad arguments");
    g_host_err[0] = 0;
    bool ok = false;
    MF_TRY(ok = m->m->prefill(tokens, (int)n, pos0, compute_logits != 0, host_logits != 0));
    return ok ? MF_OK : herr(MF_E_UNSUPPORTED, "batched prefill needs a dense model with bf16 or fp32 weights");
}

int mf_model_decode_chained(mf_model* m, uint32_t token, int start_pos, int n, uint32_t* last_id) {
    if (!m) return herr(MF_E_INVALID, "null model");
    g_host_err[0] = 0;
    MF_TRY({
        const uint32_t id = m->m->decode_chained(token, start_pos, n);
        if (last_id) *last_id = id;
    });
    return MF_OK;
}

int mf_model_reset_sampler(mf_model* m) {
    if (!m) return herr(MF_E_INVALID, "null model");
    MF_TRY(m->m->reset_sampler());
    return MF_OK;
}

int mf_model_experts(const mf_model* m, int layer, int* ids, float* weights) {
    if (!m || !ids) return herr(MF_E_INVALID, "null argument");
    const int rc = m->m->read_experts(layer, ids, weights);
    return rc ? herr(rc, "no experts at this layer") : MF_OK;
}

int mf_model_prefill_experts(const mf_model* m, int layer, int* ids, float* weights, int n_tokens) {
    if (!m) return herr(MF_E_INVALID, "null model");
    const int rc = m->m->read_prefill_experts(layer, ids, weights, n_tokens);
    return rc ? herr(rc, "no prefill routing at this layer") : MF_OK;
}

int mf_model_kv(const mf_model* m, int layer, float* k, float* v, int n_pos) {
    if (!m) return herr(MF_E_INVALID, "null model");
    const int rc = m->m->read_kv(layer, k, v, n_pos);
    return rc ? herr(rc, "kv read failed") : MF_OK;
}

int mf_model_x(const mf_model* m, float* x) {
    if (!m || !x) return herr(MF_E_INVALID, "null argument");
    return m->m->read_x(x);
}

int mf_sample(const float* logits, size_t vocab, const mf_run_params* rp, const uint32_t* seen, size_t n_seen,
              size_t n_draws, uint32_t* out) {
    if (!logits || !rp || !out || vocab == 0 || (n_seen && !seen)) return herr(MF_E_INVALID, "bad arguments");
    MF_TRY({
        minfer::SamplerParams sp;
        sp.vocab_size = vocab;
        sp.top_k = rp->top_k;
        sp.temp = rp->temp;
        sp.top_p = rp->top_p;
        sp.min_p = rp->min_p;
        sp.penalty_pres = rp->penalty_pres;
        sp.seed = rp->seed;
        minfer::Sampler smp(sp);
        for (size_t i = 0; i < n_seen; ++i) smp.add_token(seen[i]);
        for (size_t i = 0; i < n_draws; ++i) out[i] = smp.sample(logits);
    });
    return MF_OK;
}

int mf_sample_candidates(const float* logits, size_t vocab, const mf_run_params* rp, size_t n_draws, uint32_t* out) {
    if (!logits || !rp || !out || vocab == 0) return herr(MF_E_INVALID, "bad arguments");
    if (rp->penalty_pres != 0.0f || rp->top_k + 1 > vocab) return herr(MF_E_INVALID, "needs top_k < vocab, no penalty");
    MF_TRY({
        minfer::SamplerParams sp;
        sp.vocab_size = vocab;
        sp.top_k = rp->top_k;
        sp.temp = rp->temp;
        sp.top_p = rp->top_p;
        sp.min_p = rp->min_p;
        sp.seed = rp->seed;
        minfer::Sampler smp(sp);
        // the device's list: value descending, equal values lower index first
        const size_t n = rp->top_k + 1;
        std::vector<uint32_t> idx(vocab);
        for (size_t i = 0; i < vocab; ++i) idx[i] = (uint32_t)i;
        std::partial_sort(idx.begin(), idx.begin() + n, idx.end(), [&](uint32_t a, uint32_t b) {
            return logits[a] > logits[b] || (logits[a] == logits[b] && a < b);
        });
        std::vector<float> vals(n);
        for (size_t i = 0; i < n; ++i) vals[i] = logits[idx[i]];
        const bool decisive = minfer::Sampler::candidates_decisive(vals.data(), n);
        for (size_t i = 0; i < n_draws; ++i)
            out[i] = decisive ? smp.sample_candidates(idx.data(), vals.data(), rp->top_k) : smp.sample(logits);
    });
    return MF_OK;
}

int mf_random_prompt(int seed, uint32_t vocab, size_t n, uint32_t* out) {
    if (!out || vocab == 0) return herr(MF_E_INVALID, "bad arguments");
    std::mt19937 gen(seed);
    std::uniform_int_distribution<> distrib(0, (int)vocab - 1);
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)distrib(gen);
    return MF_OK;
}

// ---- tokenizer

#define TOK_TRY(...)                                    \
    try {                                               \
        g_host_err[0] = 0;                              \
        __VA_ARGS__;                                    \
    } catch (const std::domain_error& e) {              \
        return herr(MF_E_UNSUPPORTED, e.what());        \
    } catch (const std::invalid_argument& e) {          \
        return herr(MF_E_INVALID, e.what());            \
    } catch (const std::out_of_range& e) {              \
        return herr(MF_E_INVALID, e.what());            \
    } catch (const std::bad_alloc&) {                   \
        return herr(MF_E_OOM, "host allocation failed"); \
    } catch (const std::exception& e) {                 \
        return herr(MF_E_STATE, e.what());              \
    }

namespace {
size_t put_bytes(const std::string& s, char* out, size_t cap) {
    if (out) std::memcpy(out, s.data(), std::min(s.size(), cap));
    return s.size();
}
}  // namespace

int mf_tokenizer_load(const char* gguf_path, mf_tokenizer** out) {
    if (!gguf_path || !out) return herr(MF_E_INVALID, "null argument");
    TOK_TRY({
        minfer::GGUFFile f;
        if (f.open(gguf_path) != 0) return herr(MF_E_INVALID, f.error().c_str());
        auto t = std::make_unique<mf_tokenizer>();
        t->t = minfer::Qwen3Tokenizer::from_gguf(f);
        *out = t.release();
    });
    return MF_OK;
}

int mf_tokenizer_create(const char* const* tokens, const size_t* token_lens, const uint32_t* token_types,
                        size_t n_tokens, const char* const* merges, const size_t* merge_lens, size_t n_merges,
                        const char* chat_template, uint32_t eos_id, uint32_t pad_id, mf_tokenizer** out) {
    if (!out || (n_tokens && (!tokens || !token_lens || !token_types)) || (n_merges && (!merges || !merge_lens)))
        return herr(MF_E_INVALID, "null argument");
    TOK_TRY({
        std::vector<std::string> tk(n_tokens), mg(n_merges);
        for (size_t i = 0; i < n_tokens; ++i) tk[i].assign(tokens[i], token_lens[i]);
        for (size_t i = 0; i < n_merges; ++i) mg[i].assign(merges[i], merge_lens[i]);
        std::vector<uint32_t> ty(token_types, token_types + n_tokens);
        auto t = std::make_unique<mf_tokenizer>();
        t->t = std::make_unique<minfer::Qwen3Tokenizer>(tk, mg, ty, chat_template ? chat_template : "", eos_id, pad_id);
        *out = t.release();
    });
    return MF_OK;
}

void mf_tokenizer_free(mf_tokenizer* t) { delete t; }

int mf_tokenizer_info(const mf_tokenizer* t, size_t* vocab_size, uint32_t* eos_id, uint32_t* pad_id) {
    if (!t) return herr(MF_E_INVALID, "null tokenizer");
    if (vocab_size) *vocab_size = t->t->vocab_size();
    if (eos_id) *eos_id = t->t->eos_id();
    if (pad_id) *pad_id = t->t->pad_id();
    return MF_OK;
}

int mf_tokenizer_encode(const mf_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap, size_t* n) {
    if (!t || !n || (len && !text) || (cap && !ids)) return herr(MF_E_INVALID, "null argument");
    TOK_TRY({
        std::vector<uint32_t> v;
        try {
            v = t->t->encode(std::string(text ? text : "", len));
        } catch (const std::runtime_error& e) {  // a byte or merged string missing from the vocabulary
            return herr(MF_E_INVALID, e.what());
        }
        std::copy(v.begin(), v.begin() + (long)std::min(v.size(), cap), ids);
        *n = v.size();
    });
    return MF_OK;
}

int mf_tokenizer_decode(const mf_tokenizer* t, const uint32_t* ids, size_t n_ids, char* out, size_t cap, size_t* n) {
    if (!t || !n || (n_ids && !ids) || (cap && !out)) return herr(MF_E_INVALID, "null argument");
    TOK_TRY({ *n = put_bytes(t->t->decode(std::vector<uint32_t>(ids, ids + n_ids)), out, cap); });
    return MF_OK;
}

int mf_tokenizer_pre_split(const mf_tokenizer* t, const char* text, size_t len, size_t* ends, size_t cap, size_t* n) {
    if (!t || !n || (len && !text) || (cap && !ends)) return herr(MF_E_INVALID, "null argument");
    TOK_TRY({
        const auto v = t->t->pre_split(std::string(text ? text : "", len));
        for (size_t i = 0; i < v.size() && i < cap; ++i) ends[i] = v[i].second;
        *n = v.size();
    });
    return MF_OK;
}

int mf_tokenizer_apply_chat_template(const mf_tokenizer* t, const char* messages_json, const char* tools_json,
                                     int add_generation_prompt, char* out, size_t cap, size_t* n) {
    if (!t || !messages_json || !n || (cap && !out)) return herr(MF_E_INVALID, "null argument");
    TOK_TRY({
        *n = put_bytes(t->t->apply_chat_template_json(messages_json, tools_json ? tools_json : "",
                                                      add_generation_prompt != 0),
                       out, cap);
    });
    return MF_OK;
}

}  // extern "C"
