// ctypes driver around the reference's own Qwen3Tokenizer
// (src/models/qwen3/tokenizer.cpp, compiled unmodified from the reference
// tree with its vendored minja/nlohmann headers and the system PCRE2 runtime).
// Test infrastructure: it produces the tokenizer golden vectors and checks the
// product tokenizer against the reference; nothing in the product links it.
//
// The pieces of regex_split are read through the class's private member
// (access opened for this translation unit only).
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <chrono>

#include "extern/minja/chat-template.hpp"
#include "extern/nlohmann/json.hpp"
#define private public
#include "minfer/models/qwen3/tokenizer.hpp"
#undef private

namespace {
thread_local std::string g_err;

int fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}

// blob: u64 n_tokens, then per token u64 length + bytes + u32 type; u64
// n_merges, per merge u64 length + bytes; u64 template length + bytes; u32
// eos, u32 pad.
struct Reader {
    const char* p;
    const char* end;
    uint64_t u64() {
        uint64_t v;
        std::memcpy(&v, p, 8);
        p += 8;
        return v;
    }
    uint32_t u32() {
        uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }
    std::string str() {
        const uint64_t n = u64();
        std::string s(p, n);
        p += n;
        return s;
    }
};

size_t put(const std::string& s, char* out, size_t cap) {
    std::memcpy(out, s.data(), s.size() < cap ? s.size() : cap);
    return s.size();
}
}  // namespace

extern "C" {

const char* tref_error() { return g_err.c_str(); }

void* tref_create(const char* blob, size_t n) {
    try {
        Reader r{blob, blob + n};
        std::vector<std::string> tokens, merges;
        std::vector<uint32_t> types;
        const uint64_t nt = r.u64();
        for (uint64_t i = 0; i < nt; ++i) {
            tokens.push_back(r.str());
            types.push_back(r.u32());
        }
        const uint64_t nm = r.u64();
        for (uint64_t i = 0; i < nm; ++i) merges.push_back(r.str());
        const std::string tmpl = r.str();
        const uint32_t eos = r.u32(), pad = r.u32();
        return new Qwen3Tokenizer(tokens, merges, types, tmpl, eos, pad);
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void tref_free(void* t) { delete static_cast<Qwen3Tokenizer*>(t); }

int tref_encode(void* t, const char* text, size_t n, uint32_t* ids, size_t cap, size_t* n_ids) {
    try {
        const auto v = static_cast<Qwen3Tokenizer*>(t)->encode(std::string(text, n));
        for (size_t i = 0; i < v.size() && i < cap; ++i) ids[i] = v[i];
        *n_ids = v.size();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// piece lengths of regex_split
int tref_split(void* t, const char* text, size_t n, uint64_t* lens, size_t cap, size_t* n_pieces) {
    try {
        const auto v = static_cast<Qwen3Tokenizer*>(t)->regex_split(std::string(text, n));
        for (size_t i = 0; i < v.size() && i < cap; ++i) lens[i] = v[i].size();
        *n_pieces = v.size();
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int tref_decode(void* t, const uint32_t* ids, size_t n, char* out, size_t cap, size_t* n_bytes) {
    try {
        *n_bytes = put(static_cast<Qwen3Tokenizer*>(t)->decode(std::vector<uint32_t>(ids, ids + n)), out, cap);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// messages: [{"role", "content", "reasoning_content"?, "tool_calls"?: [[name, arguments-json-text]]}]
// tools: [{"name", "description", "parameters": json-text}]
int tref_chat(void* t, const char* messages_json, const char* tools_json, int add_generation_prompt, char* out,
              size_t cap, size_t* n_bytes) {
    try {
        using nlohmann::json;
        std::vector<BaseTokenizer::Message> msgs;
        for (const auto& m : json::parse(messages_json)) {
            BaseTokenizer::Message msg(m.at("role").get<std::string>(), m.at("content").get<std::string>());
            if (m.contains("reasoning_content")) msg.reasoning_content = m.at("reasoning_content").get<std::string>();
            if (m.contains("tool_calls"))
                for (const auto& tc : m.at("tool_calls"))
                    msg.tool_calls.emplace_back(tc.at(0).get<std::string>(), tc.at(1).get<std::string>());
            msgs.push_back(msg);
        }
        std::vector<BaseTokenizer::Tool> tools;
        for (const auto& x : json::parse(tools_json))
            tools.push_back({x.at("name").get<std::string>(), x.at("description").get<std::string>(),
                             x.at("parameters").get<std::string>()});
        *n_bytes = put(static_cast<Qwen3Tokenizer*>(t)->apply_chat_template(msgs, tools, add_generation_prompt != 0),
                       out, cap);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// The chat-template engine the tokenizer holds, given any JSON messages and
// tools (tools_json NULL: no tools value, as the probes render), the way
// apply_chat_template calls it (tokenizer.cpp:328-334).
int tref_chat_json(void* t, const char* messages_json, const char* tools_json, int add_generation_prompt, char* out,
                   size_t cap, size_t* n_bytes) {
    try {
        using nlohmann::ordered_json;
        minja::chat_template_inputs inputs;
        inputs.messages = ordered_json::parse(messages_json);
        inputs.tools = tools_json ? ordered_json::parse(tools_json) : ordered_json();
        inputs.add_generation_prompt = add_generation_prompt != 0;
        inputs.extra_context = ordered_json{};
        inputs.now = std::chrono::system_clock::now();
        *n_bytes = put(static_cast<Qwen3Tokenizer*>(t)->_chat_template->apply(inputs, {}), out, cap);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}
}
