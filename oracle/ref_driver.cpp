/*
 * minfer_ref_run: drives the reference's own CPU token loop on a GGUF file
 * and dumps what the parity tests compare against. Test infrastructure only.
 *
 * It links the reference's unmodified sources (BaseModel, Config, RunState,
 * Sampler, the Qwen3* layers, the CPU ops). What it adds:
 *  - layer assembly as in src/models/qwen3/model.cpp:9-86, without the
 *    tokenizer (the workloads are token ids). One deliberate deviation: when
 *    the file holds `output.weight` (an untied lm_head) it is used for the
 *    logits; src/models/qwen3/model.cpp:79-85 always uses token_embd.weight.
 *  - the prompt -> sample -> forward loop of BaseModel::generate
 *    (src/base/model.cpp:119-173) with the chat template/encode/decode steps
 *    removed and an option to ignore EOS so the decode length is fixed;
 *  - random prompt ids drawn exactly as BaseModel::benchmark does
 *    (src/base/model.cpp:189-193: std::mt19937(seed) +
 *    uniform_int_distribution<>(0, V-1));
 *  - a decode-timing mode: a fixed number of forwards at a chosen context
 *    (the tg loop of src/base/model.cpp:216-224, started at `--bench-context`
 *    instead of 0);
 *  - dumps: sampled ids, top-2 logit margin per step, chosen logit rows,
 *    MoE expert ids/weights per layer per forward (read from RunState after
 *    each Qwen3MoE::forward, src/models/qwen3/module.cpp:440-476).
 */
#include "minfer/base/model.hpp"
#include "minfer/base/module.hpp"
#include "minfer/base/config.hpp"
#include "minfer/base/sampler.hpp"
#include "minfer/base/stats.hpp"
#include "minfer/base/tensor.hpp"
#include "minfer/models/qwen3/module.hpp"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <random>
#include <sstream>
#include <string>
#include <vector>

namespace {

struct Options {
    std::string model;
    std::string prompt_file;
    std::string out = "ref_out";
    size_t random_prompt = 0;
    int prompt_seed = 0;
    size_t gen = 16;
    size_t max_seq = 0;
    float temp = 0.0f, top_p = 1.0f, min_p = 0.0f, pres = 0.0f;
    size_t top_k = 1;
    int seed = 0;
    bool ignore_eos = true;
    bool tied_head = false;
    std::vector<long> dump_steps;  // decode steps whose full logits are written; -1 = all
    long bench_context = -1;
    int bench_steps = 0, bench_warmup = 0;
    bool llama_bench = false;  // run BaseModel::benchmark (pp512 + tg128) as it is
};

std::vector<long> parse_list(const std::string& s) {
    std::vector<long> out;
    std::stringstream ss(s);
    std::string item;
    while (std::getline(ss, item, ',')) {
        if (!item.empty()) out.push_back(std::stol(item));
    }
    return out;
}

class RefQwen3 : public BaseModel {
public:
    RefQwen3(const std::string& path, const RunParams& rp, bool tied_head) : BaseModel(path, rp) {
        auto& T = model_data->tensors;
        auto add = [&](std::unique_ptr<BaseLayer> layer, bool is_moe) {
            order_.push_back(layer.get());
            moe_.push_back(is_moe);
            append_layer(std::move(layer));
        };
        add(std::make_unique<Qwen3Embed>(config->vocab_size, config->d_model, T.at("token_embd.weight")), false);
        for (int i = 0; i < config->n_layers; ++i) {
            const std::string p = "blk." + std::to_string(i) + ".";
            add(std::make_unique<Qwen3GQA>(
                    i, config->d_model, config->n_heads, config->n_kv_heads, config->d_head, config->d_rotary,
                    (int)config->user_max_seq_len, config->rms_norm_eps, config->freq_base,
                    T.at(p + "attn_q.weight"), T.at(p + "attn_k.weight"), T.at(p + "attn_v.weight"),
                    T.at(p + "attn_output.weight"), T.at(p + "attn_q_norm.weight"), T.at(p + "attn_k_norm.weight"),
                    T.at(p + "attn_norm.weight")),
                false);
            const bool moe = config->n_experts > 0;
            add(std::make_unique<Qwen3MoE>(
                    config->d_model, config->d_ff, config->n_experts, config->n_active_experts, config->rms_norm_eps,
                    T.at(p + "ffn_norm.weight"), moe ? T.at(p + "ffn_gate_inp.weight") : nullptr,
                    T.at(p + (moe ? "ffn_gate_exps.weight" : "ffn_gate.weight")),
                    T.at(p + (moe ? "ffn_down_exps.weight" : "ffn_down.weight")),
                    T.at(p + (moe ? "ffn_up_exps.weight" : "ffn_up.weight"))),
                true);
        }
        add(std::make_unique<Qwen3FinalRMSNorm>(config->d_model, config->rms_norm_eps, T.at("output_norm.weight")),
            false);
        const bool untied = !tied_head && T.count("output.weight");
        add(std::make_unique<Qwen3LMHead>(config->d_model, (int)config->vocab_size,
                                          T.at(untied ? "output.weight" : "token_embd.weight"), nullptr),
            false);
        untied_ = untied;
    }

    void forward(std::shared_ptr<RunState> rs) override {
        for (size_t i = 0; i < order_.size(); ++i) {
            order_[i]->forward(rs);
            if (moe_[i] && record_experts_ && config->n_experts > 0) {
                const int k = config->n_active_experts;
                const int* ids = std::get<int*>(rs->active_experts);
                const float* w = std::get<float*>(rs->active_experts_weights);
                expert_ids_.insert(expert_ids_.end(), ids, ids + k);
                expert_w_.insert(expert_w_.end(), w, w + k);
            }
        }
    }

    void step(uint32_t token, int pos, bool logits) {
        run_state->cur_pos = pos;
        run_state->token_id = token;
        run_state->compute_logits = logits;
        forward(run_state);
    }

    const float* logits() const { return std::get<float*>(run_state->logits); }
    Config& cfg() { return *config; }
    Sampler& sampler_ref() { return *sampler; }
    RunState& state() { return *run_state; }
    const GenStats& gen_stats() const { return *stats; }
    bool untied() const { return untied_; }

    bool record_experts_ = true;
    std::vector<int> expert_ids_;
    std::vector<float> expert_w_;

private:
    std::vector<BaseLayer*> order_;
    std::vector<bool> moe_;
    bool untied_ = false;
};

double now_s() {
    using namespace std::chrono;
    return duration_cast<duration<double>>(steady_clock::now().time_since_epoch()).count();
}

void top2(const float* l, size_t n, size_t& i1, float& v1, float& v2) {
    i1 = 0;
    v1 = l[0];
    v2 = -INFINITY;
    for (size_t i = 1; i < n; ++i) {
        if (l[i] > v1) {
            v2 = v1;
            v1 = l[i];
            i1 = i;
        } else if (l[i] > v2) {
            v2 = l[i];
        }
    }
}

template <typename T>
void write_json_array(std::ostream& os, const std::vector<T>& v) {
    os << "[";
    for (size_t i = 0; i < v.size(); ++i) {
        if (i) os << ",";
        os << v[i];
    }
    os << "]";
}

int usage() {
    std::fprintf(stderr,
                 "usage: minfer_ref_run <model.gguf> [--prompt-file F | --random-prompt P --prompt-seed S]\n"
                 "  [--gen G] [--max-seq N] [--temp T --top-k K --top-p P --min-p M --pres X --seed S]\n"
                 "  [--stop-at-eos] [--tied-head] [--dump-logits a,b,...|-1] [--out PREFIX]\n"
                 "  [--bench-context C --bench-steps K --bench-warmup W] [--llama-bench]\n");
    return 2;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return usage();
    Options o;
    o.model = argv[1];
    for (int i = 2; i < argc; ++i) {
        std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) {
                std::fprintf(stderr, "%s needs a value\n", a.c_str());
                std::exit(2);
            }
            return argv[++i];
        };
        if (a == "--prompt-file") o.prompt_file = next();
        else if (a == "--random-prompt") o.random_prompt = std::stoul(next());
        else if (a == "--prompt-seed") o.prompt_seed = std::stoi(next());
        else if (a == "--gen") o.gen = std::stoul(next());
        else if (a == "--max-seq") o.max_seq = std::stoul(next());
        else if (a == "--temp") o.temp = std::stof(next());
        else if (a == "--top-k") o.top_k = std::stoul(next());
        else if (a == "--top-p") o.top_p = std::stof(next());
        else if (a == "--min-p") o.min_p = std::stof(next());
        else if (a == "--pres") o.pres = std::stof(next());
        else if (a == "--seed") o.seed = std::stoi(next());
        else if (a == "--stop-at-eos") o.ignore_eos = false;
        else if (a == "--tied-head") o.tied_head = true;
        else if (a == "--dump-logits") o.dump_steps = parse_list(next());
        else if (a == "--out") o.out = next();
        else if (a == "--bench-context") o.bench_context = std::stol(next());
        else if (a == "--bench-steps") o.bench_steps = std::stoi(next());
        else if (a == "--bench-warmup") o.bench_warmup = std::stoi(next());
        else if (a == "--llama-bench") o.llama_bench = true;
        else return usage();
    }

    std::vector<uint32_t> prompt;
    if (!o.prompt_file.empty()) {
        std::ifstream f(o.prompt_file, std::ios::binary);
        uint32_t t;
        while (f.read(reinterpret_cast<char*>(&t), sizeof(t))) prompt.push_back(t);
    }

    size_t max_seq = o.max_seq;
    const bool bench = o.bench_context >= 0;
    if (o.llama_bench && max_seq < 512) max_seq = 512;  // benchmark() prefills positions 0..511
    if (max_seq == 0) {
        max_seq = bench ? (size_t)o.bench_context + o.bench_steps + o.bench_warmup
                        : (o.random_prompt ? o.random_prompt : prompt.size()) + o.gen + 1;
    }

    const double t_load0 = now_s();
    RunParams rp(o.gen, max_seq, o.top_k, o.temp, o.top_p, o.min_p, o.pres, o.seed);
    RefQwen3 m(o.model, rp, o.tied_head);
    const double t_load = now_s() - t_load0;
    Config& c = m.cfg();
    const size_t V = c.vocab_size;

    if (o.random_prompt) {
        std::mt19937 gen(o.prompt_seed);
        std::uniform_int_distribution<> distrib(0, (int)V - 1);
        prompt.clear();
        for (size_t i = 0; i < o.random_prompt; ++i) prompt.push_back((uint32_t)distrib(gen));
    }

    std::ofstream js(o.out + ".json");
    js.precision(9);

    if (o.llama_bench) {
        // the reference's own benchmark loop (src/base/model.cpp:188-236),
        // unchanged; its stats are read back from the protected GenStats
        m.record_experts_ = false;
        m.benchmark();
        const GenStats& st = m.gen_stats();
        js << "{\"mode\":\"llama_bench\",\"num_tokens_gen\":" << st.num_tokens_gen << ",\"prefill_time\":"
           << st.prefill_time << ",\"ttft\":" << st.ttft << ",\"throughput\":" << st.throughput
           << ",\"bandwidth\":" << st.bandwidth << ",\"load_seconds\":" << t_load << "}\n";
        return 0;
    }

    if (bench) {
        // decode forwards at positions [C, C+W+K): the KV rows below C are
        // zero-filled so every step reads a full context of C+1 rows.
        RunState& rs = m.state();
        const size_t kv_elems = (size_t)c.n_layers * c.n_kv_heads * max_seq * c.d_head;
        std::memset(std::get<float*>(rs.k_cache), 0, kv_elems * sizeof(float));
        std::memset(std::get<float*>(rs.v_cache), 0, kv_elems * sizeof(float));
        m.record_experts_ = false;
        std::mt19937 gen(o.prompt_seed);
        std::uniform_int_distribution<> distrib(0, (int)V - 1);
        std::vector<double> dt;
        for (int s = 0; s < o.bench_warmup + o.bench_steps; ++s) {
            const double t0 = now_s();
            m.step((uint32_t)distrib(gen), (int)o.bench_context + s, true);
            const double t1 = now_s();
            if (s >= o.bench_warmup) dt.push_back(t1 - t0);
        }
        double tot = 0;
        for (double d : dt) tot += d;
        js << "{\"mode\":\"bench\",\"context\":" << o.bench_context << ",\"steps\":" << o.bench_steps
           << ",\"seconds\":" << tot << ",\"tok_per_s\":" << (dt.empty() ? 0.0 : dt.size() / tot)
           << ",\"step_seconds\":";
        write_json_array(js, dt);
        js << ",\"read_bytes_per_token\":" << m.get_read_bytes() << ",\"kv_bytes_per_pos\":" << rs.kv_bytes_per_pos
           << ",\"load_seconds\":" << t_load << "}\n";
        return 0;
    }

    // --- BaseModel::generate loop without the tokenizer (src/base/model.cpp:119-173)
    const double t0 = now_s();
    for (size_t i = 0; i < prompt.size(); ++i) {
        m.step(prompt[i], (int)i, i + 1 == prompt.size());
    }
    const double t_prefill = now_s() - t0;
    const size_t n_prompt_forwards = prompt.size();
    Sampler& smp = m.sampler_ref();
    for (uint32_t t : prompt) smp.add_token(t);

    std::vector<uint32_t> tokens = prompt;
    std::vector<uint32_t> out_ids;
    std::vector<float> margins, top1v;
    std::vector<long> dumped;
    std::ofstream lf(o.out + ".logits.f32", std::ios::binary);
    const size_t num_iters = std::min(c.num_iters, c.user_max_seq_len - tokens.size());
    size_t generated = 0;
    const double t1 = now_s();
    while (generated < num_iters) {
        const float* lg = m.logits();
        size_t i1;
        float v1, v2;
        top2(lg, V, i1, v1, v2);
        margins.push_back(v1 - v2);
        top1v.push_back(v1);
        const bool dump_all = !o.dump_steps.empty() && o.dump_steps[0] == -1;
        if (dump_all || std::find(o.dump_steps.begin(), o.dump_steps.end(), (long)generated) != o.dump_steps.end()) {
            lf.write(reinterpret_cast<const char*>(lg), V * sizeof(float));
            dumped.push_back((long)generated);
        }
        const uint32_t next = smp.sample(lg);
        smp.add_token(next);
        tokens.push_back(next);
        out_ids.push_back(next);
        generated++;
        if (!o.ignore_eos && next == c.eos_token_id) break;
        m.step(next, (int)tokens.size() - 1, true);
    }
    const double t_decode = now_s() - t1;

    std::ofstream ef(o.out + ".experts.bin", std::ios::binary);
    if (!m.expert_ids_.empty()) {
        ef.write(reinterpret_cast<const char*>(m.expert_ids_.data()), m.expert_ids_.size() * sizeof(int));
        ef.write(reinterpret_cast<const char*>(m.expert_w_.data()), m.expert_w_.size() * sizeof(float));
    }

    js << "{\"mode\":\"generate\",\"vocab\":" << V << ",\"n_layers\":" << c.n_layers
       << ",\"n_experts\":" << c.n_experts << ",\"k\":" << c.n_active_experts
       << ",\"untied_head\":" << (m.untied() ? "true" : "false") << ",\"prompt\":";
    write_json_array(js, prompt);
    js << ",\"ids\":";
    write_json_array(js, out_ids);
    js << ",\"margins\":";
    write_json_array(js, margins);
    js << ",\"top1\":";
    write_json_array(js, top1v);
    js << ",\"dumped_steps\":";
    write_json_array(js, dumped);
    js << ",\"n_forwards\":" << (n_prompt_forwards + generated) << ",\"prefill_seconds\":" << t_prefill
       << ",\"decode_seconds\":" << t_decode << ",\"load_seconds\":" << t_load << "}\n";
    return 0;
}
