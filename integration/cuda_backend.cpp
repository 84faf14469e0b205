/*
 * minfer_cuda_app: minfer's own host loop on the B200 runtime.
 *
 * The reference's BaseModel (include/minfer/base/model.hpp:17-41,
 * src/base/model.cpp), Config/RunState, Sampler, GGUF reader and stats are
 * compiled unchanged from the reference's sources. This file adds what a
 * `-d cuda` build of minfer adds: a BaseModel subclass whose forward()
 * (virtual, src/base/model.cpp:36-59) runs one token through the CUDA
 * runtime's C ABI (include/minfer_model.h: mf_model_forward, mf_model_logits)
 * and hands the logits back in the reference's RunState, so the reference's
 * own loops drive the GPU:
 *
 *   minfer_cuda_app bench MODEL [--seed S] [--max-seq N]
 *       BaseModel::benchmark (src/base/model.cpp:188-236) as shipped: pp512
 *       + tg128 of random ids; prints its stats as one JSON line.
 *   minfer_cuda_app generate MODEL --prompt-file F --gen G [--temp T --top-k K
 *       --top-p P --min-p M --pres X --seed S]
 *       BaseModel::generate's loop (src/base/model.cpp:119-173) on token ids
 *       (the tokenizer is not part of this path): prompt forwards, then the
 *       reference's Sampler::sample on each step's logits, EOS ignored;
 *       prints the ids as one JSON line.
 *   minfer_cuda_app text MODEL --prompt TEXT --gen G [--max-seq N ...]
 *       BaseModel::generate(std::string&) (src/base/model.cpp:99-186) as
 *       shipped, text in: the model's BaseTokenizer is CudaTokenizer below, the
 *       reference's tokenizer interface (include/minfer/base/tokenizer.hpp)
 *       over this runtime's tokenizer (mf_tokenizer_*), in place of the
 *       PCRE2/minja Qwen3Tokenizer; the loop prints what the reference prints.
 *   minfer_cuda_app tokenize MODEL --prompt TEXT
 *       CudaTokenizer alone (no GPU): the chat-template prompt of one user
 *       message and its ids, as one JSON line.
 *
 * The layers are assembled as src/models/qwen3/model.cpp:9-86 does (views of
 * the mapped file, never run here) so BaseModel::get_read_bytes reports the
 * reference's byte counts; an untied `output.weight` is used when present.
 */
#include "minfer/base/config.hpp"
#include "minfer/base/model.hpp"
#include "minfer/base/module.hpp"
#include "minfer/base/sampler.hpp"
#include "minfer/base/stats.hpp"
#include "minfer/base/tensor.hpp"
#include "minfer/base/tokenizer.hpp"
#include "minfer/models/qwen3/module.hpp"
#include "minfer_model.h"
#include "nlohmann/json.hpp"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void ck(int rc, const char* what) {
    if (rc != MF_OK) {
        char msg[512];
        mf_host_last_error(msg, sizeof(msg));
        throw std::runtime_error(std::string(what) + ": " + msg);
    }
}

// BaseTokenizer over mf_tokenizer_*: what the reference's generate(std::string&)
// calls (apply_chat_template, encode, decode_token, get_eos_id).
class CudaTokenizer : public BaseTokenizer {
public:
    CudaTokenizer(const std::string& gguf_path, uint32_t eos, uint32_t pad) : BaseTokenizer(eos, pad) {
        ck(mf_tokenizer_load(gguf_path.c_str(), &t_), "mf_tokenizer_load");
    }
    ~CudaTokenizer() override { mf_tokenizer_free(t_); }

    std::vector<uint32_t> encode(const std::string& text) override {
        std::vector<uint32_t> ids(text.size() + 1);  // (every id covers at least one byte)
        size_t n = 0;
        ck(mf_tokenizer_encode(t_, text.data(), text.size(), ids.data(), ids.size(), &n), "mf_tokenizer_encode");
        ids.resize(n);
        return ids;
    }
    std::string decode(const std::vector<uint32_t>& ids) override { return bytes(ids.data(), ids.size()); }
    std::string decode_token(uint32_t id) override { return bytes(&id, 1); }
    std::string apply_chat_template(const std::vector<Message>& messages, const std::vector<Tool>& tools,
                                    bool add_generation_prompt) override {
        // the JSON the reference's Qwen3Tokenizer builds from these structs
        nlohmann::ordered_json msgs = nlohmann::ordered_json::array(), tl = nlohmann::ordered_json::array();
        for (const auto& m : messages) {
            nlohmann::ordered_json j;
            j["role"] = m.role;
            j["content"] = m.content;
            if (!m.reasoning_content.empty()) j["reasoning_content"] = m.reasoning_content;
            if (!m.tool_calls.empty()) {
                j["tool_calls"] = nlohmann::ordered_json::array();
                for (const auto& tc : m.tool_calls)
                    j["tool_calls"].push_back({{"name", tc.first}, {"arguments", nlohmann::ordered_json::parse(tc.second)}});
            }
            msgs.push_back(j);
        }
        for (const auto& t : tools)
            tl.push_back({{"name", t.name}, {"description", t.description},
                          {"parameters", nlohmann::ordered_json::parse(t.parameters)}});
        const std::string mj = msgs.dump(), tj = tl.dump();
        std::string out(4096, '\0');
        size_t n = 0;
        for (int pass = 0; pass < 2; ++pass) {
            ck(mf_tokenizer_apply_chat_template(t_, mj.c_str(), tj.c_str(), add_generation_prompt, &out[0], out.size(),
                                                &n),
               "mf_tokenizer_apply_chat_template");
            if (n <= out.size()) break;
            out.resize(n);
        }
        out.resize(n);
        return out;
    }

private:
    std::string bytes(const uint32_t* ids, size_t k) {
        std::string out(16 * k + 16, '\0');
        size_t n = 0;
        for (int pass = 0; pass < 2; ++pass) {
            ck(mf_tokenizer_decode(t_, ids, k, &out[0], out.size(), &n), "mf_tokenizer_decode");
            if (n <= out.size()) break;
            out.resize(n);
        }
        out.resize(n);
        return out;
    }
    mf_tokenizer* t_ = nullptr;
};

class CudaQwen3 : public BaseModel {
public:
    CudaQwen3(const std::string& path, const RunParams& rp, const mf_run_params& mp) : BaseModel(path, rp) {
        auto& T = model_data->tensors;
        append_layer(std::make_unique<Qwen3Embed>(config->vocab_size, config->d_model, T.at("token_embd.weight")));
        for (int i = 0; i < config->n_layers; ++i) {
            const std::string p = "blk." + std::to_string(i) + ".";
            append_layer(std::make_unique<Qwen3GQA>(
                i, config->d_model, config->n_heads, config->n_kv_heads, config->d_head, config->d_rotary,
                (int)config->user_max_seq_len, config->rms_norm_eps, config->freq_base, T.at(p + "attn_q.weight"),
                T.at(p + "attn_k.weight"), T.at(p + "attn_v.weight"), T.at(p + "attn_output.weight"),
                T.at(p + "attn_q_norm.weight"), T.at(p + "attn_k_norm.weight"), T.at(p + "attn_norm.weight")));
            const bool moe = config->n_experts > 0;
            append_layer(std::make_unique<Qwen3MoE>(
                config->d_model, config->d_ff, config->n_experts, config->n_active_experts, config->rms_norm_eps,
                T.at(p + "ffn_norm.weight"), moe ? T.at(p + "ffn_gate_inp.weight") : nullptr,
                T.at(p + (moe ? "ffn_gate_exps.weight" : "ffn_gate.weight")),
                T.at(p + (moe ? "ffn_down_exps.weight" : "ffn_down.weight")),
                T.at(p + (moe ? "ffn_up_exps.weight" : "ffn_up.weight"))));
        }
        append_layer(std::make_unique<Qwen3FinalRMSNorm>(config->d_model, config->rms_norm_eps,
                                                         T.at("output_norm.weight")));
        const bool untied = T.count("output.weight") != 0;
        append_layer(std::make_unique<Qwen3LMHead>(config->d_model, (int)config->vocab_size,
                                                   T.at(untied ? "output.weight" : "token_embd.weight"), nullptr));
        const int dev = 0;
        ck(mf_init(1, &dev), "mf_init");
        ck(mf_model_load(path.c_str(), &mp, 0, &m_), "mf_model_load");
        ck(mf_model_to_cuda(m_), "mf_model_to_cuda");
        tokenizer = std::make_unique<CudaTokenizer>(path, config->eos_token_id, config->padding_token_id);
    }
    ~CudaQwen3() override {
        if (m_) mf_model_free(m_);
    }

    // BaseModel::forward on the CUDA runtime: one frame per token, the logits
    // copied into the reference's RunState when it asks for them
    void forward(std::shared_ptr<RunState> rs) override {
        ck(mf_model_forward(m_, rs->token_id, rs->cur_pos, rs->compute_logits ? 1 : 0, rs->compute_logits ? 1 : 0),
           "mf_model_forward");
        if (rs->compute_logits) ck(mf_model_logits(m_, std::get<float*>(rs->logits), config->vocab_size), "logits");
    }

    // BaseModel::generate's loop (src/base/model.cpp:119-173) on token ids, EOS ignored
    std::vector<uint32_t> generate_ids(const std::vector<uint32_t>& prompt, size_t n_gen) {
        for (size_t i = 0; i < prompt.size(); ++i) {
            run_state->cur_pos = (int)i;
            run_state->token_id = prompt[i];
            run_state->compute_logits = (i + 1 == prompt.size());
            forward(run_state);
        }
        for (uint32_t t : prompt) sampler->add_token(t);
        std::vector<uint32_t> tokens = prompt, out;
        const size_t num_iters = std::min(n_gen, config->user_max_seq_len - tokens.size());
        for (size_t g = 0; g < num_iters; ++g) {
            const uint32_t next = sampler->sample(std::get<float*>(run_state->logits));
            sampler->add_token(next);
            tokens.push_back(next);
            out.push_back(next);
            run_state->cur_pos = (int)tokens.size() - 1;
            run_state->token_id = next;
            run_state->compute_logits = true;
            forward(run_state);
        }
        return out;
    }

    const GenStats& gen_stats() const { return *stats; }

private:
    mf_model* m_ = nullptr;
};

int usage() {
    std::fprintf(stderr,
                 "usage: minfer_cuda_app bench MODEL [--seed S] [--max-seq N]\n"
                 "       minfer_cuda_app generate MODEL --prompt-file F --gen G [--max-seq N]\n"
                 "           [--temp T --top-k K --top-p P --min-p M --pres X --seed S]\n"
                 "       minfer_cuda_app text MODEL --prompt TEXT --gen G [--max-seq N] [sampler flags]\n"
                 "       minfer_cuda_app tokenize MODEL --prompt TEXT\n");
    return 2;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) return usage();
    const std::string mode = argv[1], model = argv[2];
    std::string prompt_file, prompt_text;
    size_t gen = 16, max_seq = 0, top_k = 1;
    float temp = 0.f, top_p = 1.f, min_p = 0.f, pres = 0.f;
    int seed = 0;
    for (int i = 3; i < argc; ++i) {
        const std::string a = argv[i];
        if (i + 1 >= argc) return usage();
        const std::string v = argv[++i];
        if (a == "--prompt-file") prompt_file = v;
        else if (a == "--prompt") prompt_text = v;
        else if (a == "--gen") gen = std::stoul(v);
        else if (a == "--max-seq") max_seq = std::stoul(v);
        else if (a == "--temp") temp = std::stof(v);
        else if (a == "--top-k") top_k = std::stoul(v);
        else if (a == "--top-p") top_p = std::stof(v);
        else if (a == "--min-p") min_p = std::stof(v);
        else if (a == "--pres") pres = std::stof(v);
        else if (a == "--seed") seed = std::stoi(v);
        else return usage();
    }
    try {
        if (mode == "tokenize") {  // the BaseTokenizer adapter alone, on the host
            mf_tokenizer* probe = nullptr;
            ck(mf_tokenizer_load(model.c_str(), &probe), "mf_tokenizer_load");
            uint32_t eos = 0, pad = 0;
            ck(mf_tokenizer_info(probe, nullptr, &eos, &pad), "mf_tokenizer_info");
            mf_tokenizer_free(probe);
            CudaTokenizer tok(model, eos, pad);
            std::vector<BaseTokenizer::Message> msgs;
            msgs.emplace_back("user", prompt_text);
            const std::string formatted = tok.apply_chat_template(msgs, {}, true);
            const std::vector<uint32_t> ids = tok.encode(formatted);
            nlohmann::ordered_json j;
            j["mode"] = "tokenize";
            j["formatted"] = formatted;
            j["ids"] = ids;
            j["round_trip"] = tok.decode(ids) == formatted;
            j["eos"] = tok.get_eos_id();
            std::printf("%s\n", j.dump().c_str());
            return 0;
        }
        std::vector<uint32_t> prompt;
        if (mode == "generate") {
            std::ifstream f(prompt_file, std::ios::binary);
            if (!f) throw std::runtime_error("cannot read the prompt file");
            uint32_t t;
            while (f.read(reinterpret_cast<char*>(&t), sizeof(t))) prompt.push_back(t);
            if (prompt.empty()) throw std::runtime_error("empty prompt");
            if (max_seq == 0) max_seq = prompt.size() + gen + 1;
        } else if (mode == "bench") {
            if (max_seq == 0) max_seq = 4096;
        } else if (mode == "text") {
            if (max_seq == 0) max_seq = 1024;
        } else {
            return usage();
        }
        const RunParams rp(gen, max_seq, top_k, temp, top_p, min_p, pres, seed);
        const mf_run_params mp = {gen, max_seq, top_k, temp, top_p, min_p, pres, seed};
        CudaQwen3 m(model, rp, mp);
        if (mode == "bench") {
            m.benchmark();  // the reference's loop, unchanged (it prints its own stats too)
            const GenStats& st = m.gen_stats();
            std::printf("{\"mode\":\"bench\",\"num_tokens_gen\":%d,\"prefill_time\":%.6f,\"ttft\":%.6f,"
                        "\"throughput\":%.3f,\"bandwidth\":%.3f}\n",
                        st.num_tokens_gen, st.prefill_time, st.ttft, st.throughput, st.bandwidth);
            return 0;
        }
        if (mode == "text") {
            m.generate(prompt_text);  // the reference's text loop, unchanged (it prints its own output)
            const GenStats& st = m.gen_stats();
            std::printf("{\"mode\":\"text\",\"num_tokens_gen\":%d,\"throughput\":%.3f}\n", st.num_tokens_gen,
                        st.throughput);
            return 0;
        }
        const std::vector<uint32_t> ids = m.generate_ids(prompt, gen);
        std::printf("{\"mode\":\"generate\",\"ids\":[");
        for (size_t i = 0; i < ids.size(); ++i) std::printf("%s%u", i ? "," : "", ids[i]);
        std::printf("]}\n");
    } catch (const std::exception& e) {
        std::fprintf(stderr, "minfer_cuda_app: %s\n", e.what());
        return 1;
    }
    return 0;
}
