// Qwen3 tokenizer: special-token split, pattern pre-split, rank-ordered BPE.
#include "tokenizer.hpp"

#include <algorithm>
#include <climits>
#include <cstring>
#include <stdexcept>

#include "chat_template.hpp"
#include "gguf.hpp"

namespace minfer {

namespace {

struct CodeRange {
    uint32_t lo, hi;
};
#include "unicode_tables.inc"

template <size_t N>
bool in_ranges(const CodeRange (&r)[N], uint32_t cp) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp > r[mid].hi)
            lo = mid + 1;
        else if (cp < r[mid].lo)
            hi = mid;
        else
            return true;
    }
    return false;
}

bool is_letter(uint32_t cp) {
    if (cp < 0x80) return (cp | 0x20) >= 'a' && (cp | 0x20) <= 'z';
    return in_ranges(kLetterRanges, cp);
}
bool is_number(uint32_t cp) {
    if (cp < 0x80) return cp >= '0' && cp <= '9';
    return in_ranges(kNumberRanges, cp);
}
// \s under PCRE2_UCP: \p{Z} (Zs Zl Zp), horizontal space \h and vertical space \v
bool is_space(uint32_t cp) {
    if (cp < 0x80) return cp == ' ' || (cp >= 0x09 && cp <= 0x0D);
    switch (cp) {
        case 0x85: case 0xA0: case 0x1680: case 0x180E: case 0x2028: case 0x2029: case 0x202F: case 0x205F:
        case 0x3000:
            return true;
        default:
            return cp >= 0x2000 && cp <= 0x200A;
    }
}

// Strict UTF-8 (RFC 3629: no overlong forms, no surrogates, at most
// U+10FFFF), the validity PCRE2 requires of a UTF subject. Returns the
// sequence length at p (p < end), or 0 if no valid character starts there.
int utf8_len(const uint8_t* p, const uint8_t* end, uint32_t* cp) {
    const uint8_t c = p[0];
    if (c < 0x80) {
        *cp = c;
        return 1;
    }
    int n;
    uint32_t v, lo = 0x80, hi = 0xBF;  // bounds of the second byte
    if (c >= 0xC2 && c <= 0xDF) {
        n = 2;
        v = c & 0x1F;
    } else if (c >= 0xE0 && c <= 0xEF) {
        n = 3;
        v = c & 0x0F;
        if (c == 0xE0) lo = 0xA0;
        if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
        n = 4;
        v = c & 0x07;
        if (c == 0xF0) lo = 0x90;
        if (c == 0xF4) hi = 0x8F;
    } else {
        return 0;
    }
    if (end - p < n) return 0;
    for (int i = 1; i < n; ++i) {
        const uint8_t b = p[i];
        if (i == 1 ? (b < lo || b > hi) : (b & 0xC0) != 0x80) return 0;
        v = (v << 6) | (b & 0x3F);
    }
    *cp = v;
    return n;
}

// First offset in [from, end) at which decoding from `from` fails, or end.
size_t first_invalid(const uint8_t* s, size_t from, size_t end) {
    uint32_t cp;
    while (from < end) {
        const int n = utf8_len(s + from, s + end, &cp);
        if (!n) return from;
        from += n;
    }
    return end;
}

// The match at `pos` of the reference's pre-split pattern
//   '(?i:[sdmt]|ll|ve|re) | [^\r\n\p{L}\p{N}]?+\p{L}++ | \p{N}{1,3}+
//   | ?[^\s\p{L}\p{N}]++[\r\n]*+ | \s++$ | \s*[\r\n] | \s+(?!\S) | \s
// over the subject [.., end), whose bytes from pos are valid UTF-8. Every
// character starts a match of some alternative, so the unanchored search the
// reference runs always matches at pos itself. Returns the match's end.
size_t pattern_match(const uint8_t* s, size_t pos, size_t end) {
    uint32_t c0, c1;
    const int n0 = utf8_len(s + pos, s + end, &c0);
    // 1. contractions, caseless (s also matches U+017F LATIN SMALL LETTER LONG S)
    if (c0 == '\'' && pos + 1 < end) {
        const size_t p = pos + 1;
        const int n1 = utf8_len(s + p, s + end, &c1);
        const uint32_t l1 = c1 < 0x80 ? (c1 | 0x20) : c1;
        if (l1 == 's' || l1 == 'd' || l1 == 'm' || l1 == 't' || c1 == 0x17F) return p + n1;
        if (p + 1 < end) {
            const uint32_t l2 = s[p + 1] | 0x20;
            if ((l1 == 'l' && l2 == 'l') || (l1 == 'v' && l2 == 'e') || (l1 == 'r' && l2 == 'e')) return p + 2;
        }
    }
    // 2. an optional non-letter, non-number (not CR/LF) then letters; both possessive
    {
        size_t p = pos;
        if (!is_letter(c0) && !is_number(c0) && c0 != '\r' && c0 != '\n') p += n0;
        size_t q = p;
        while (q < end) {
            const int n = utf8_len(s + q, s + end, &c1);
            if (!is_letter(c1)) break;
            q += n;
        }
        if (q > p) return q;
    }
    // 3. one to three numbers
    if (is_number(c0)) {
        size_t q = pos;
        for (int i = 0; i < 3 && q < end; ++i) {
            const int n = utf8_len(s + q, s + end, &c1);
            if (!is_number(c1)) break;
            q += n;
        }
        return q;
    }
    // 4. an optional space, then a run of characters that are none of
    //    space/letter/number, then CR/LF
    {
        size_t p = pos + (c0 == ' ' ? 1 : 0);
        size_t q = p;
        while (q < end) {
            const int n = utf8_len(s + q, s + end, &c1);
            if (is_space(c1) || is_letter(c1) || is_number(c1)) break;
            q += n;
        }
        if (q > p) {
            while (q < end && (s[q] == '\r' || s[q] == '\n')) ++q;
            return q;
        }
    }
    // c0 is white space from here on: the run of white space from pos
    size_t r = pos, last_start = pos, last_nl = SIZE_MAX;
    int run = 0;
    while (r < end) {
        const int n = utf8_len(s + r, s + end, &c1);
        if (!is_space(c1)) break;
        if (c1 == '\r' || c1 == '\n') last_nl = r;
        last_start = r;
        r += n;
        ++run;
    }
    if (r == end) return end;                   // 5. white space up to the end of the subject
    if (last_nl != SIZE_MAX) return last_nl + 1;  // 6. white space through the last CR/LF
    if (run >= 2) return last_start;            // 7. white space not followed by a non-space
    return pos + n0;                            // 8. one white space character
}

uint64_t pair_key(int32_t a, int32_t b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }

}  // namespace

Qwen3Tokenizer::Qwen3Tokenizer(const std::vector<std::string>& tokens, const std::vector<std::string>& merges,
                               const std::vector<uint32_t>& token_types, const std::string& chat_template,
                               uint32_t eos_id, uint32_t pad_id)
    : vocab_(tokens), types_(token_types), eos_id_(eos_id), pad_id_(pad_id) {
    if (tokens.size() != token_types.size())
        throw std::invalid_argument("Token and token_type arrays must have same size");
    vocab_to_id_.reserve(vocab_.size());
    for (size_t i = 0; i < vocab_.size(); ++i) vocab_to_id_[vocab_[i]] = (uint32_t)i;  // a repeated string: last id
    for (size_t i = 0; i < vocab_.size(); ++i) {
        const uint32_t t = types_[i];
        // an empty special would match everywhere without advancing: never a special
        if ((t == CONTROL_TOKEN || t == USER_DEFINED_TOKEN) && !vocab_[i].empty()) {
            const uint32_t id = vocab_to_id_.at(vocab_[i]);
            auto& b = specials_[(uint8_t)vocab_[i][0]];
            if (std::find(b.begin(), b.end(), id) == b.end()) b.push_back(id);
        }
    }
    for (auto& b : specials_)
        std::stable_sort(b.begin(), b.end(),
                         [&](uint32_t a, uint32_t c) { return vocab_[a].size() > vocab_[c].size(); });
    // symbols 0..255 are the single bytes
    for (int b = 0; b < 256; ++b) intern(std::string(1, (char)b));
    rules_.reserve(merges.size());
    for (const std::string& m : merges) {
        const size_t sp = m.find(' ');  // the first space splits left from right
        if (sp == std::string::npos) throw std::invalid_argument("Invalid merge rule format: " + m);
        const std::string l = m.substr(0, sp), r = m.substr(sp + 1);
        Rule rule;
        rule.left = intern(l);
        rule.right = intern(r);
        rule.merged = intern(l + r);
        pair_ranks_[pair_key(rule.left, rule.right)].push_back((int32_t)rules_.size());
        rules_.push_back(rule);
    }
    sym_vocab_.assign(syms_.size(), -1);
    for (size_t i = 0; i < syms_.size(); ++i) {
        auto it = vocab_to_id_.find(syms_[i]);
        if (it != vocab_to_id_.end()) sym_vocab_[i] = it->second;
    }
    chat_ = std::make_unique<ChatTemplate>(chat_template);
}

Qwen3Tokenizer::~Qwen3Tokenizer() = default;

std::unique_ptr<Qwen3Tokenizer> Qwen3Tokenizer::from_gguf(const GGUFFile& f) {
    auto strs = [&](const char* key) -> const std::vector<std::string>& {
        const MetaValue* v = f.get(key);
        if (!v || v->kind != MetaValue::ARRAY_STR) throw std::invalid_argument(std::string("missing ") + key);
        return v->strs;
    };
    const MetaValue* tt = f.get("tokenizer.ggml.token_type");
    if (!tt || tt->kind != MetaValue::ARRAY_NUM) throw std::invalid_argument("missing tokenizer.ggml.token_type");
    std::vector<uint32_t> types(tt->nums.size());
    for (size_t i = 0; i < types.size(); ++i) types[i] = (uint32_t)tt->nums[i];
    return std::make_unique<Qwen3Tokenizer>(strs("tokenizer.ggml.tokens"), strs("tokenizer.ggml.merges"), types,
                                            f.get_string("tokenizer.chat_template"),
                                            (uint32_t)f.get_uint("tokenizer.ggml.eos_token_id"),
                                            (uint32_t)f.get_uint("tokenizer.ggml.padding_token_id"));
}

int32_t Qwen3Tokenizer::intern(const std::string& s) {
    auto it = sym_id_.find(s);
    if (it != sym_id_.end()) return it->second;
    const int32_t id = (int32_t)syms_.size();
    sym_id_.emplace(s, id);
    syms_.push_back(s);
    return id;
}

std::pair<size_t, size_t> Qwen3Tokenizer::next_special(const std::string& text, size_t from) const {
    const size_t n = text.size();
    for (size_t i = from; i < n; ++i) {
        for (uint32_t id : specials_[(uint8_t)text[i]]) {
            const std::string& sp = vocab_[id];
            if (sp.size() <= n - i && std::memcmp(text.data() + i, sp.data(), sp.size()) == 0) return {i, sp.size()};
        }
    }
    return {n, 0};
}

std::vector<std::pair<size_t, size_t>> Qwen3Tokenizer::pre_split(const std::string& text) const {
    std::vector<std::pair<size_t, size_t>> out;
    const uint8_t* s = (const uint8_t*)text.data();
    const size_t n = text.size();
    size_t pos = 0;
    std::pair<size_t, size_t> sp = next_special(text, 0);
    // bytes [pos, valid_end) decode as valid UTF-8 from pos up to seg_end
    size_t valid_from = SIZE_MAX, bad = 0;
    while (pos < n) {
        if (sp.first < pos) sp = next_special(text, pos);
        if (sp.first == pos) {
            out.push_back({pos, pos + sp.second});
            pos += sp.second;
            valid_from = SIZE_MAX;
            sp = next_special(text, pos);
            continue;
        }
        const size_t seg_end = sp.first;
        if (valid_from == SIZE_MAX) {
            valid_from = pos;
            bad = first_invalid(s, pos, seg_end);
        }
        if (bad < seg_end) {
            // the subject fails PCRE2's UTF check: one byte per piece up to
            // and including the invalid byte, then check again after it
            for (; pos <= bad; ++pos) out.push_back({pos, pos + 1});
            valid_from = SIZE_MAX;
            continue;
        }
        const size_t e = pattern_match(s, pos, seg_end);
        out.push_back({pos, e});
        pos = e;
        if (pos == seg_end) valid_from = SIZE_MAX;
    }
    return out;
}

std::vector<uint32_t> Qwen3Tokenizer::bpe(const char* p, size_t n) const {
    // The reference walks the rules in rank order and applies each to the
    // whole word once, left to right (tokenizer.cpp:251-275). The rules that
    // change anything are, in turn, the lowest-ranked rule above the last one
    // applied whose pair occurs in the word; a pass never creates a pair of its
    // own rule. So: the word as a linked list, a min-heap of (rank, position)
    // holding for every adjacent pair its lowest rank above the last applied
    // rule, and one pass per popped rank, left to right over that rank's
    // positions. O(n log n) in the piece's bytes.
    struct Node {
        int32_t sym, prev, next;
    };
    std::vector<Node> w(n);
    for (size_t i = 0; i < n; ++i) w[i] = {(uint8_t)p[i], (int32_t)i - 1, i + 1 < n ? (int32_t)(i + 1) : -1};
    using Entry = std::pair<int32_t, int32_t>;  // (rank, position of the pair's left symbol)
    std::vector<Entry> heap;
    auto push = [&](int32_t i, int64_t after) {
        if (i < 0 || w[i].next < 0) return;
        auto it = pair_ranks_.find(pair_key(w[i].sym, w[w[i].next].sym));
        if (it == pair_ranks_.end()) return;
        auto r = std::upper_bound(it->second.begin(), it->second.end(), after);
        if (r == it->second.end()) return;
        heap.emplace_back(*r, i);
        std::push_heap(heap.begin(), heap.end(), std::greater<Entry>());
    };
    for (size_t i = 0; i + 1 < n; ++i) push((int32_t)i, -1);
    std::vector<int32_t> at, merged;
    while (!heap.empty()) {
        const int32_t rank = heap.front().first;
        at.clear();
        while (!heap.empty() && heap.front().first == rank) {  // the pass's positions, left to right
            at.push_back(heap.front().second);
            std::pop_heap(heap.begin(), heap.end(), std::greater<Entry>());
            heap.pop_back();
        }
        std::sort(at.begin(), at.end());
        const Rule& rule = rules_[(size_t)rank];
        merged.clear();
        for (int32_t i : at) {
            // stale entries (a symbol merged since, or a repeated entry) no
            // longer show the rule's pair
            const int32_t j = w[i].next;
            if (j < 0 || w[i].sym != rule.left || w[j].sym != rule.right) continue;
            w[i].sym = rule.merged;
            w[i].next = w[j].next;
            if (w[j].next >= 0) w[w[j].next].prev = i;
            w[j].sym = -1;  // (removed)
            merged.push_back(i);
        }
        // the pairs the merges made, at their lowest rank above this one
        for (int32_t i : merged) {
            push(w[i].prev, rank);
            push(i, rank);
        }
    }
    std::vector<uint32_t> ids;
    for (int32_t i = n ? 0 : -1; i >= 0; i = w[i].next) {
        const int64_t id = sym_vocab_[(size_t)w[i].sym];
        if (id < 0)
            throw std::runtime_error(std::string(n <= 1 ? "Byte" : "BPE") + " token '" + syms_[(size_t)w[i].sym] +
                                     "' not found in vocab to id map");
        ids.push_back((uint32_t)id);
    }
    return ids;
}

std::vector<uint32_t> Qwen3Tokenizer::encode(const std::string& text) const {
    std::vector<uint32_t> ids;
    if (text.empty()) return ids;
    for (const auto& piece : pre_split(text)) {
        const size_t len = piece.second - piece.first;
        const char* p = text.data() + piece.first;
        const uint8_t b0 = (uint8_t)*p;
        bool special = false;
        for (uint32_t id : specials_[b0]) {
            if (vocab_[id].size() == len && std::memcmp(vocab_[id].data(), p, len) == 0) {
                ids.push_back(id);
                special = true;
                break;
            }
        }
        if (special) continue;
        std::string key(p, len);
        {
            std::lock_guard<std::mutex> g(cache_mu_);
            auto it = cache_.find(key);
            if (it != cache_.end()) {
                ids.insert(ids.end(), it->second.begin(), it->second.end());
                continue;
            }
        }
        std::vector<uint32_t> t = bpe(p, len);
        ids.insert(ids.end(), t.begin(), t.end());
        std::lock_guard<std::mutex> g(cache_mu_);
        if (cache_.size() >= (1u << 16)) cache_.clear();
        cache_.emplace(std::move(key), std::move(t));
    }
    return ids;
}

std::string Qwen3Tokenizer::decode_token(uint32_t id) const {
    if (id >= vocab_.size()) throw std::out_of_range("Token ID exceeds vocab size");
    if (types_[id] == UNUSED_TOKEN) return "<UNK>";
    return vocab_[id];
}

std::string Qwen3Tokenizer::decode(const std::vector<uint32_t>& ids) const {
    std::string out;
    out.reserve(ids.size() * 4);
    for (uint32_t id : ids) out += decode_token(id);
    return out;
}

std::string Qwen3Tokenizer::apply_chat_template(const std::vector<Message>& messages, const std::vector<Tool>& tools,
                                                bool add_generation_prompt) const {
    // the JSON shape the reference builds (tokenizer.cpp:296-326)
    Value msgs = Value::array();
    for (const Message& m : messages) {
        Value o = Value::object();
        o.set("role", Value(m.role));
        o.set("content", Value(m.content));
        if (!m.reasoning_content.empty()) o.set("reasoning_content", Value(m.reasoning_content));
        if (!m.tool_calls.empty()) {
            Value calls = Value::array();
            for (const auto& tc : m.tool_calls) {
                Value c = Value::object();
                c.set("name", Value(tc.first));
                c.set("arguments", parse_json(tc.second));
                calls.push(std::move(c));
            }
            o.set("tool_calls", std::move(calls));
        }
        msgs.push(std::move(o));
    }
    Value tl = Value::array();
    for (const Tool& t : tools) {
        Value o = Value::object();
        o.set("name", Value(t.name));
        o.set("description", Value(t.description));
        o.set("parameters", parse_json(t.parameters));
        tl.push(std::move(o));
    }
    return chat_->render(msgs, tl, add_generation_prompt);
}

std::string Qwen3Tokenizer::apply_chat_template_json(const std::string& messages_json, const std::string& tools_json,
                                                     bool add_generation_prompt) const {
    Value msgs = parse_json(messages_json);
    Value tl = tools_json.empty() ? Value::array() : parse_json(tools_json);
    if (!msgs.is_array() || !tl.is_array()) throw std::invalid_argument("messages and tools must be JSON arrays");
    return chat_->render(msgs, tl, add_generation_prompt);
}

}  // namespace minfer
