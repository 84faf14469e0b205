// Chat templates: a Jinja-subset renderer with the semantics of the template
// engine the reference renders `tokenizer.chat_template` with (minja, vendored
// as include/extern/minja; call site src/models/qwen3/tokenizer.cpp:291-335),
// and the JSON values it renders from.
//
// Built: text with {{ }}, {% %} and {# #} tags and their '-' trim markers,
// trim_blocks + lstrip_blocks + no trailing newline (the options the
// reference's chat_template parses with); if/elif/else, for (tuple targets,
// inline `if` filter, else, loop.*), set (names, tuples, namespace attributes,
// block set), macros (parameters with defaults), filter blocks,
// break/continue, generation blocks; the expression grammar with
// minja's precedence, its value semantics (byte strings, integer division of
// integers, objects always true, ...) and its filters/methods; the capability
// probes and every polyfill of its chat_template (system role, typed content,
// tools with an inferred tool-call example, tool calls, tool responses,
// object arguments). Not built (rendering raises std::domain_error): call
// blocks (the reference's engine has none either) and recursive loops.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace minfer {

class Value;
struct CallArgs {
    std::vector<Value> pos;
    std::vector<std::pair<std::string, Value>> kw;
};

class Value {
public:
    enum Kind { NUL, BOOL, INT, FLOAT, STR, ARR, OBJ };  // (a callable is an OBJ with a function)
    using Arr = std::vector<Value>;
    using Obj = std::vector<std::pair<std::string, Value>>;  // insertion order
    using Fn = std::function<Value(CallArgs&)>;

    Value() = default;
    explicit Value(bool b) : k_(BOOL), b_(b) {}
    explicit Value(int64_t i) : k_(INT), i_(i) {}
    explicit Value(int i) : k_(INT), i_(i) {}
    explicit Value(double f) : k_(FLOAT), f_(f) {}
    explicit Value(std::string s) : k_(STR), s_(std::move(s)) {}
    explicit Value(const char* s) : k_(STR), s_(s) {}
    static Value array(Arr a = {});
    static Value object();
    static Value function(Fn f);

    Kind kind() const { return k_; }
    bool is_null() const { return k_ == NUL; }
    bool is_string() const { return k_ == STR; }
    bool is_array() const { return k_ == ARR; }
    bool is_object() const { return k_ == OBJ; }
    bool is_number() const { return k_ == INT || k_ == FLOAT; }
    bool is_callable() const { return fn_ != nullptr; }

    bool b() const { return b_; }
    int64_t i() const;  // integers; floats truncate; anything else throws
    double f() const;   // numbers; anything else throws
    const std::string& str() const;  // strings; anything else throws
    Arr& arr() const;
    Obj& obj() const;
    Value call(CallArgs& a) const;

    // containers (shared: copies of a Value alias one array/object)
    void push(Value v);
    void set(const std::string& key, Value v);
    const Value* find(const std::string& key) const;
    void erase(const std::string& key);
    size_t size() const;

    bool truthy() const;
    std::string to_str() const;                   // minja to_str: strings raw, floats %f, None/True/False
    std::string dump(int indent = -1, bool json = false) const;  // Python repr, or JSON with json=true
    // plain JSON text: compact without spaces (indent < 0), or pretty with
    // `indent` spaces per level and empty containers as [] / {}
    std::string json_text(int indent = -1) const;
    bool equals(const Value& o) const;

private:
    void dump_to(std::string& out, int indent, int level, bool json) const;
    Kind k_ = NUL;
    bool b_ = false;
    int64_t i_ = 0;
    double f_ = 0;
    std::string s_;
    std::shared_ptr<Arr> a_;
    std::shared_ptr<Obj> o_;
    std::shared_ptr<Fn> fn_;
};

// Parses JSON text (objects keep their key order; integers stay integers).
// Throws std::invalid_argument on malformed input.
Value parse_json(const std::string& text);

struct TemplateNode;

class ChatTemplate {
public:
    // Parses the template and runs the capability probes. A template that
    // does not parse leaves the object usable: render then throws the error.
    explicit ChatTemplate(const std::string& source, std::string bos_token = "<|im_start|>",
                          std::string eos_token = "<|im_end|>");
    ~ChatTemplate();
    // messages / tools: JSON arrays as the reference's apply_chat_template
    // builds them (tools null: no `tools` variable). Throws
    // std::runtime_error from the template (raise_exception, type errors) and
    // std::domain_error for constructs that are not built.
    std::string render(const Value& messages, const Value& tools, bool add_generation_prompt) const;

    struct Caps {
        bool supports_system_role = false, supports_tools = false, supports_tool_calls = false,
             supports_tool_responses = false, requires_object_arguments = false,
             requires_non_null_content = false, requires_typed_content = false;
    };
    const Caps& caps() const { return caps_; }

private:
    std::string raw_render(const Value& messages, const Value* tools, bool add_generation_prompt) const;
    std::string try_raw_render(const Value& messages, const Value* tools) const;
    void check_parsed() const;  // throws the parse error, if any
    bool parse_unsupported_ = false;
    std::shared_ptr<TemplateNode> root_;
    std::string parse_error_;
    std::string bos_, eos_;
    Caps caps_;
    std::string tool_call_example_;
};

}  // namespace minfer
