"""The host tokenizer (no GPU) against the reference's own tokenizer.

Golden vectors (tests/golden/tokenizer_cases.json, made by
tests/golden/make_tokenizer_golden.py from the reference's tokenizer.cpp
compiled with its vendored chat-template engine): for every text the pieces of
the pre-split and the ids; for every chat case the rendered prompt. Where the
reference build is present (oracle/_ref/libtokenizer_ref.so) seeded random
texts are compared live as well. The reference's own test is the
encode -> decode round trip (tests/src/qwen3/tokenizer/tokenizer.cpp:45-67),
run here over every text.
"""
import json
import random
from pathlib import Path

import pytest

from oracle import tokenizer_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def vocab():
    return json.loads((GOLDEN / "tokenizer_vocab.json").read_text())


@pytest.fixture(scope="module")
def cases():
    return json.loads((GOLDEN / "tokenizer_cases.json").read_text())


def _args(v):
    return ([bytes.fromhex(t) for t in v["tokens"]], [bytes.fromhex(m) for m in v["merges"]], v["types"])


@pytest.fixture(scope="module")
def toks(vocab):
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    return {name: Qwen3Tokenizer.from_vocab(tokens, merges, types, tmpl, vocab["eos"], vocab["pad"])
            for name, tmpl in vocab["templates"].items()}


def _chat_inputs(c):
    # the JSON the reference builds from its Message/Tool structs
    msgs = []
    for m in c["messages"]:
        d = {k: v for k, v in m.items() if k != "tool_calls"}
        if "tool_calls" in m:
            d["tool_calls"] = [{"name": n, "arguments": json.loads(a)} for n, a in m["tool_calls"]]
        msgs.append(d)
    tools = [dict(t, parameters=json.loads(t["parameters"])) for t in c["tools"]]
    return msgs, tools


def test_golden_pieces_and_ids(toks, cases):
    t = toks["chatml_min"]
    for c in cases["texts"]:
        b = bytes.fromhex(c["text"])
        assert [len(p) for p in t.pre_split(b)] == c["pieces"], b
        assert t.encode(b) == c["ids"], b


def test_round_trip(toks, cases):
    t = toks["chatml_min"]
    for c in cases["texts"]:
        b = bytes.fromhex(c["text"])
        assert t.decode(t.encode(b)) == b
    assert t.encode("") == [] and t.decode([]) == b""


def test_golden_chat_templates(toks, cases):
    for c in cases["chats"]:
        msgs, tools = _chat_inputs(c)
        assert toks[c["template"]].apply_chat_template(msgs, tools, c["add_generation_prompt"]) == c["expected"], c


def test_message_structs(toks, cases):
    """The Message/Tool mirror builds the same JSON as the reference."""
    from minfer_b200.tokenizer import Message, Tool

    c = next(c for c in cases["chats"] if c["template"] == "chatml_tools" and c["tools"] and
             any("tool_calls" in m for m in c["messages"]))
    msgs = [Message(m["role"], m["content"], m.get("reasoning_content", ""), [tuple(x) for x in m.get("tool_calls", [])])
            for m in c["messages"]]
    tools = [Tool(t["name"], t["description"], t["parameters"]) for t in c["tools"]]
    assert toks["chatml_tools"].apply_chat_template(msgs, tools, c["add_generation_prompt"]) == c["expected"]


def _random_texts(seed, n):
    rng = random.Random(seed)
    blocks = [(0x20, 0x7E), (0xA0, 0x24F), (0x370, 0x3FF), (0x400, 0x4FF), (0x600, 0x6FF), (0x900, 0x97F),
              (0x3040, 0x30FF), (0x4E00, 0x4FFF), (0xAC00, 0xAD00), (0x2000, 0x206F), (0x1F300, 0x1F64F),
              (0xFF00, 0xFFEF), (0x660, 0x669), (0x2160, 0x2188)]
    specials = ["<|im_start|>", "<|im_end|>", "<think>", "</tool_call>", "<|unused_1|>"]
    out = []
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(1, 30)):
            r = rng.random()
            if r < 0.35:
                parts.append(rng.choice(" \t\n\r  \n\n'sSdllve"))
            elif r < 0.4:
                parts.append(rng.choice(specials))
            else:
                lo, hi = rng.choice(blocks)
                parts.append(chr(rng.randint(lo, hi)))
        b = "".join(parts).encode("utf-8", "surrogatepass")
        if rng.random() < 0.1:
            i = rng.randint(0, len(b))
            b = b[:i] + bytes([rng.choice([0x80, 0xBF, 0xC2, 0xE0, 0xED, 0xF0, 0xF5, 0xFF])]) + b[i:]
        out.append(b)
    return out


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_live_reference_random_texts(vocab, toks):
    tokens, merges, types = _args(vocab)
    ref = tokenizer_ref.RefTokenizer(tokens, types, merges, vocab["templates"]["chatml_min"], vocab["eos"],
                                     vocab["pad"])
    t = toks["chatml_min"]
    for b in _random_texts(2024, 600):
        assert [len(p) for p in t.pre_split(b)] == ref.split(b), b
        assert t.encode(b) == ref.encode(b), b


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_live_reference_random_chats(vocab, toks):
    from minfer_b200._lib import MinferError

    tokens, merges, types = _args(vocab)
    rng = random.Random(5)
    words = ["hi", "Oslo", "2+2", "it's", "世界", "", " ", "\n", "<b>&'\"", "x" * 30]
    for name in ("chatml_min", "chatml_tools", "exprs"):
        ref = tokenizer_ref.RefTokenizer(tokens, types, merges, vocab["templates"][name], vocab["eos"], vocab["pad"])
        for _ in range(25):
            msgs = []
            for _ in range(rng.randint(1, 5)):
                role = rng.choice(["system", "user", "assistant", "user"])
                m = {"role": role, "content": " ".join(rng.choice(words) for _ in range(rng.randint(0, 4)))}
                if role == "assistant" and rng.random() < 0.4:
                    m["reasoning_content"] = rng.choice(words) + "\n"
                msgs.append(m)
            gen = rng.random() < 0.5
            try:
                expected = ref.chat(msgs, [], gen)
            except RuntimeError:  # the template fails on these messages (an empty content's [-3:]): so does ours
                with pytest.raises(MinferError):
                    toks[name].apply_chat_template(msgs, [], gen)
                continue
            assert toks[name].apply_chat_template(msgs, [], gen) == expected, (name, msgs)


def test_reference_error_behaviour(vocab):
    from minfer_b200._lib import MF_E_INVALID, MinferError
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    with pytest.raises(MinferError) as e:  # token and type arrays of different lengths
        Qwen3Tokenizer.from_vocab(tokens, merges, types[:-1])
    assert e.value.code == MF_E_INVALID
    with pytest.raises(MinferError):  # a merge rule without a space
        Qwen3Tokenizer.from_vocab(tokens, merges + [b"ab"], types)
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, "", vocab["eos"], vocab["pad"])
    with pytest.raises(MinferError):  # an id past the vocabulary
        t.decode([len(tokens)])
    unused = types.index(5)
    assert t.decode_token(unused) == b"<UNK>"
    assert t.decode_token(vocab["eos"]) == b"<|im_end|>"
    assert (t.get_eos_id(), t.get_pad_id()) == (vocab["eos"], vocab["pad"])
    # a vocabulary without the byte the text needs: the reference throws
    no_z = Qwen3Tokenizer.from_vocab([b"a", b"b"], [], [1, 1])
    assert no_z.encode("abba") == [0, 1, 1, 0]
    with pytest.raises(MinferError) as e:
        no_z.encode("abz")
    assert e.value.code == MF_E_INVALID


def test_template_errors(vocab):
    from minfer_b200._lib import MF_E_STATE, MF_E_UNSUPPORTED, MinferError
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    raising = "{{ raise_exception('too many messages') if messages | length > 2 else 'ok' }}"
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, raising)
    assert t.apply_chat_template([{"role": "user", "content": "x"}]) == "ok"
    with pytest.raises(MinferError) as e:
        t.apply_chat_template([{"role": "user", "content": "x"}] * 3)
    assert e.value.code == MF_E_STATE and "too many messages" in str(e.value)
    macro = "{% macro f(x, y='!') %}<{{ x }}{{ y }}>{% endmacro %}{{ f(1) }}{{ f('a', y='?') }}"
    assert Qwen3Tokenizer.from_vocab(tokens, merges, types, macro).apply_chat_template(
        [{"role": "user", "content": "x"}]) == "<1!><a?>"
    call = "{% call f() %}x{% endcall %}"  # (call blocks: the reference's engine has none either)
    with pytest.raises(MinferError) as e:
        Qwen3Tokenizer.from_vocab(tokens, merges, types, call).apply_chat_template([{"role": "user", "content": "x"}])
    assert e.value.code == MF_E_UNSUPPORTED
    # a template that cannot show tools gets them in a system message (the tools polyfill)
    plain = "{% for m in messages %}{{ m.role }}: {{ m.content }}\n{% endfor %}"
    out = Qwen3Tokenizer.from_vocab(tokens, merges, types, plain).apply_chat_template(
        [{"role": "user", "content": "x"}], [{"name": "f", "description": "d", "parameters": {}}])
    assert out.startswith("system: You can call any of the following tools to satisfy the user's requests: [")


def test_load_from_gguf_model():
    """mf_tokenizer_load reads the tokenizer keys of a model file (the tiny
    synthetic models carry a printable-ASCII vocabulary whose other bytes are
    spelled <0xNN>, so text with those bytes cannot be encoded, by the
    reference either)."""
    from conftest import TINY, tiny_model
    from minfer_b200._lib import MinferError
    from minfer_b200.gguf_synth import synth_vocab
    from minfer_b200.tokenizer import Qwen3Tokenizer

    cfg = TINY["tiny-bf16"]
    t = Qwen3Tokenizer.from_gguf(tiny_model("tiny-bf16"))
    toks, types, merges, eos, pad = synth_vocab(cfg.vocab, cfg.seed)
    assert (t.vocab_size, t.eos_id, t.pad_id) == (cfg.vocab, eos, pad)
    ids = t.encode("Hello!")
    assert t.decode(ids) == b"Hello!"
    with pytest.raises(MinferError):
        t.encode("two words")
    if tokenizer_ref.available():
        ref = tokenizer_ref.RefTokenizer(toks, types, merges, "", eos, pad)
        for s in [b"Hello!", b"a1b2c3", b"<|special_0|>xyz", b"(((!!!)))"]:
            assert t.encode(s) == ref.encode(s)


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_qwen3_sized_vocabulary_vs_reference():
    """A vocabulary of Qwen3's size (151936 entries, ~149k merge rules, the
    byte-level synthetic one the text models use): ids identical to the
    reference's, whose encode walks every rule for every piece (about 2.4 s
    for these 6 KB; ours well under a millisecond)."""
    from minfer_b200.gguf_synth import synth_byte_vocab
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, types, merges, eos, pad = synth_byte_vocab(151936, 3)
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, "", eos, pad)
    ref = tokenizer_ref.RefTokenizer(tokens, types, merges, "", eos, pad)
    rng = random.Random(1)
    words = ["the", "kernel", "streams", "every", "weight", "row", "once", "Token", "2048", "it's", "大模型",
             "テスト", "x8SIIc", "Erx", "<|im_end|>", "\n\n", "  "]
    text = " ".join(rng.choice(words) for _ in range(1000)).encode()
    ids = t.encode(text)
    assert ids == ref.encode(text) and t.decode(ids) == text
    for b in _random_texts(99, 20):
        assert t.encode(b) == ref.encode(b), b


POLYFILL_TEMPLATES = {
    # shows roles and contents only: tools, tool calls and tool responses need polyfills
    "plain": "{% for m in messages %}{{ m.role }}: {{ m.content }}\n{% endfor %}"
             "{% if add_generation_prompt %}assistant: {% endif %}",
    # refuses system messages: they are merged into the next user message
    "no_system": "{% for m in messages %}{% if m.role == 'system' %}{{ raise_exception('no system role') }}{% endif %}"
                 "<{{ m.role }}>{{ m.content }}</{{ m.role }}>{% endfor %}",
    # reads content as a list of typed parts
    "typed": "{% for m in messages %}{{ m.role }}:{% for p in m.content %}{{ p.text }}{% endfor %}\n{% endfor %}",
    # renders tools and calls, but call arguments only as a mapping
    "object_args": "{% if tools %}{% for t in tools %}{{ t | tojson }}\n{% endfor %}{% endif %}"
                   "{% for m in messages %}[{{ m.role }}] {{ m.content if m.content is string else '' }}"
                   "{% if m.tool_calls %}{% for tc in m.tool_calls %}<call {{ tc.function.name }}>"
                   "{% for k, v in tc.function.arguments | items %}<parameter={{ k }}>{{ v }}{% endfor %}"
                   "</call>{% endfor %}{% endif %}\n{% endfor %}",
}


def _openai_messages():
    call = {"id": "call_7", "type": "function",
            "function": {"name": "get_weather", "arguments": "{\"city\": \"Oslo\", \"days\": 2}"}}
    call_obj = {"id": "call_8", "type": "function", "function": {"name": "calc", "arguments": {"expr": "2+2"}}}
    return [
        [{"role": "user", "content": "hi"}],
        [{"role": "system", "content": "Be terse."}, {"role": "system", "content": "Use metric."},
         {"role": "user", "content": "weather?"}, {"role": "assistant", "content": "Sunny."},
         {"role": "user", "content": ""}],
        [{"role": "system", "content": "sys"}, {"role": "user", "content": "weather in Oslo?"},
         {"role": "assistant", "content": None, "tool_calls": [call]},
         {"role": "tool", "name": "get_weather", "content": "{\"temp\": -3}", "tool_call_id": "call_7"},
         {"role": "assistant", "content": "", "tool_calls": [call_obj, {"type": "other", "x": 1}]},
         {"role": "tool", "content": "4"}, {"role": "assistant", "content": "Cold."}],
    ]


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_polyfills_vs_reference(vocab):
    """Templates that cannot render system messages, tools, tool calls, tool
    responses or string contents themselves: the reference's chat-template
    engine rewrites the conversation first (and infers a tool-call example
    from the template); the renders must be identical, or both must fail."""
    from minfer_b200._lib import MinferError
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    tools = [{"type": "function", "function": {"name": "get_weather", "description": "Weather <now>.",
                                               "parameters": {"type": "object",
                                                              "properties": {"city": {"type": "string"}},
                                                              "required": ["city"]}}}]
    templates = dict(POLYFILL_TEMPLATES, chatml_tools=vocab["templates"]["chatml_tools"],
                     chatml_min=vocab["templates"]["chatml_min"], exprs=vocab["templates"]["exprs"])
    n_ok = n_err = 0
    for name, tmpl in templates.items():
        t = Qwen3Tokenizer.from_vocab(tokens, merges, types, tmpl, vocab["eos"], vocab["pad"])
        ref = tokenizer_ref.RefTokenizer(tokens, types, merges, tmpl, vocab["eos"], vocab["pad"])
        for msgs in _openai_messages():
            for tl in ([], tools):
                for gen in (True, False):
                    try:
                        expected = ref.chat_json(msgs, tl, gen)
                    except RuntimeError:
                        with pytest.raises(MinferError):
                            t.apply_chat_template(msgs, tl, gen)
                        n_err += 1
                        continue
                    assert t.apply_chat_template(msgs, tl, gen) == expected, (name, msgs, tl, gen)
                    n_ok += 1
    assert n_ok > 3 * n_err


_TESTS = ["defined", "none", "string", "number", "integer", "float", "mapping", "iterable", "sequence", "boolean",
          "true", "false"]
_SUBSCRIPTS = ["0", "1", "-1", ":2", "1:", "::-1", "::2", "'k'", "-2:", "1:3"]


def _random_expression(rng, d=0):
    """A random expression over literals, the render's variables, operators,
    filters, methods, subscripts, slices, tests and conditionals."""
    atoms = ["1", "2", "0", "-3", "2.5", "0.1", "'ab'", "'a b c'", "''", "\"x'y\"", "true", "false", "none",
             "[1, 2, 3]", "[]", "['x', 'y']", "{'k': 1, 'j': 'v'}", "{}", "messages", "messages[0]",
             "messages[0].content", "messages[-1].role", "add_generation_prompt", "bos_token", "undefined_thing",
             "(1, 'a')", "[none, 0, '']", "'  pad\\n'", "'A-b-C'", "10", "7", "3.0", "'l1\\nl2\\n\\nl4'",
             "'\\n'", "range(3)", "range(1, 7, 2)", "range(5, 0, -2)", "namespace(a=1).a", "namespace(a=1, b='x')",
             "(messages | selectattr('role', 'equalto', 'user') | list)",
             "(messages | map(attribute='content') | join(' '))", "(['b', 'a'] | map('upper') | list)",
             "({'b': 1, 'a': 2} | dictsort)", "joiner(',')()", "(messages | rejectattr('role') | list)",
             "([1, 2, 1] | select('equalto', 1) | list)", "({'a': 1}.items() | list)", "[3, 1].pop(0)",
             "range(end=3)", "(messages | map(attribute='nope', default='d') | list)", "range", "namespace",
             "joiner(',')", "length", "(range == range)", "(range is defined)"]
    if d > 3 or rng.random() < 0.3:
        return rng.choice(atoms)
    r = rng.random()
    a = _random_expression(rng, d + 1)
    if r < 0.3:
        op = rng.choice(["+", "-", "*", "**", "~", "==", "!=", "<", ">", "<=", ">=", "and", "or", "in", "not in"])
        return f"({a} {op} {_random_expression(rng, d + 1)})"
    if r < 0.45:
        f = rng.choice(["length", "trim", "tojson", "upper", "lower", "list", "unique", "last", "count", "string", "int",
                        "items", "dictsort", "safe", "escape", "join(',')", "default('dflt')", "default('d', true)",
                        "map(attribute='role')", "selectattr('role')", "select('equalto', 1)", "reject('equalto', 1)",
                        "tojson(indent=2)", "join", "first", "indent(2)", "indent(3, true)", "indent(first=true)",
                        "length(1)", "tojson(bogus=1)", "trim('x')", "string", "join(*['-'])", "tojson(**{'indent': 1})",
                        "default(*[1, 2])"])
        return f"({a} | {f})"
    if r < 0.6:
        m = rng.choice(["strip()", "strip('a')", "lstrip()", "rstrip('\\n')", "split(' ')", "split('-')", "upper()",
                        "lower()", "title()", "capitalize()", "startswith('a')", "endswith('c')",
                        "replace('a', 'Z')", "replace('a', 'Z', 1)", "items()", "keys()", "get('k')", "get('q', 5)",
                        "append(4)", "pop()"])
        return f"{a}.{m}"
    if r < 0.7:
        return f"{a}[{rng.choice(_SUBSCRIPTS)}]"
    if r < 0.8:
        return f"({a} is {rng.choice(_TESTS)})"
    if r < 0.87:
        return f"(not {a})"
    if r < 0.94:
        return f"({a} if {_random_expression(rng, d + 1)} else {_random_expression(rng, d + 1)})"
    return f"(-{a})"


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_random_expressions_vs_reference(vocab):
    """Seeded random expressions (literals, operators, filters, methods,
    subscripts, slices, tests, conditionals) as one-tag templates: the render
    is the reference engine's, or both fail. (Integer division and modulo are
    left out: the reference divides integers unchecked, and a zero divisor
    kills its process with SIGFPE; ours raises an error.)"""
    from minfer_b200._lib import MinferError
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    msgs = [{"role": "user", "content": "Hello world"}, {"role": "assistant", "content": "a-b-c"}]
    rng = random.Random(11)
    ok = 0
    for _ in range(500):
        tmpl = "{{ " + _random_expression(rng) + " }}"
        ours = Qwen3Tokenizer.from_vocab(tokens, merges, types, tmpl)
        try:  # (a template the reference cannot parse fails its constructor; ours fails at render)
            ref = tokenizer_ref.RefTokenizer(tokens, types, merges, tmpl, vocab["eos"], vocab["pad"])
            expected = ref.chat_json(msgs, [], True)
        except RuntimeError:
            with pytest.raises(MinferError):
                ours.apply_chat_template(msgs, [], True)
            continue
        assert ours.apply_chat_template(msgs, [], True) == expected, tmpl
        ok += 1
    assert ok > 150



# random templates: text with spaces/newlines around nested for/if/set blocks,
# filter blocks and macros, loop variables, namespaces, break/continue and
# '-' trim markers
_WS = ["", " ", "  ", "\n", "\n  ", "  \n", "\t", "\n\n", " x ", "text\n", "\n    "]
_EXPRS = ["m.role", "m.content", "loop.index", "loop.first", "loop.last", "loop.length", "loop.revindex",
          "ns.n", "x", "messages | length", "m.content[:3]", "bos_token", "loop.index0 ~ '/' ~ loop.length",
          "loop.previtem.role if loop.previtem else 'none'", "loop.cycle('a', 'b')", "y"]
_CONDS = ["loop.first", "m.role == 'user'", "not loop.last", "x", "ns.n > 1", "m.content", "add_generation_prompt",
          "'o' in m.content", "y is defined"]
_OUTER_EXPRS = ["x", "ns.n", "messages | length", "bos_token", "y", "add_generation_prompt"]
_OUTER_CONDS = ["x", "ns.n > 1", "add_generation_prompt", "y is defined"]
_SETS = ["set x = x ~ 'a'", "set ns.n = ns.n + 1", "set y = 3", "set x, y = ['p', 'q']"]


def _tag(rng, body, kind="%"):
    left = "-" if rng.random() < 0.3 else ""
    right = "-" if rng.random() < 0.3 else ""
    open_, close = {"%": ("{%", "%}"), "{": ("{{", "}}"), "#": ("{#", "#}")}[kind]
    return f"{open_}{left} {body} {right}{close}"


def _body(rng, depth, in_loop):
    parts = []
    for _ in range(rng.randint(1, 4)):
        r = rng.random()
        parts.append(rng.choice(_WS))
        if r < 0.3 or depth > 2:
            parts.append(_tag(rng, rng.choice(_EXPRS if in_loop else _OUTER_EXPRS), "{"))
        elif r < 0.5:
            cond = " if m.role != 'system'" if rng.random() < 0.3 else ""
            parts.append(_tag(rng, "for m in messages" + cond))
            parts.append(_body(rng, depth + 1, True))
            if rng.random() < 0.2:
                parts.append(_tag(rng, "else"))
                parts.append(_body(rng, depth + 1, False))
            parts.append(_tag(rng, "endfor"))
        elif r < 0.7:
            parts.append(_tag(rng, "if " + rng.choice(_CONDS if in_loop else _OUTER_CONDS)))
            parts.append(_body(rng, depth + 1, in_loop))
            if rng.random() < 0.4:
                parts.append(_tag(rng, "elif " + rng.choice(["x", "true", "false"])))
                parts.append(_body(rng, depth + 1, in_loop))
            if rng.random() < 0.4:
                parts.append(_tag(rng, "else"))
                parts.append(_body(rng, depth + 1, in_loop))
            parts.append(_tag(rng, "endif"))
        elif r < 0.8:
            parts.append(_tag(rng, rng.choice(_SETS)))
        elif r < 0.86:
            parts.append(_tag(rng, "set z"))
            parts.append(_body(rng, depth + 1, in_loop))
            parts.append(_tag(rng, "endset"))
            parts.append(_tag(rng, "z", "{"))
        elif r < 0.88:
            parts.append(_tag(rng, rng.choice(["filter upper", "filter trim", "filter lower", "filter indent"])))
            parts.append(_body(rng, depth + 1, in_loop))
            parts.append(_tag(rng, "endfilter"))
        elif r < 0.9:
            parts.append(_tag(rng, "macro mk(who, sep='-')"))
            parts.append(rng.choice(_WS) + _tag(rng, "who ~ sep ~ x", "{") + rng.choice(_WS))
            if rng.random() < 0.5:
                parts.append(_tag(rng, "set x = x ~ '!'"))
            parts.append(_tag(rng, "endmacro"))
            parts.append(_tag(rng, rng.choice(["mk('a')", "mk('b', sep='+')", "mk(who='c')", "mk(1, 2)", "mk()"]), "{"))
        elif r < 0.92 and in_loop:
            parts.append(_tag(rng, rng.choice(["break", "continue"])))
        else:
            parts.append(_tag(rng, "comment", "#"))
        parts.append(rng.choice(_WS))
    return "".join(parts)


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_random_templates_vs_reference(vocab):
    """Seeded random templates exercise the whitespace rules (trim_blocks,
    lstrip_blocks, '-' markers, trailing newline), scoping and loop state:
    every render identical to the reference engine's."""
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    msgs = [{"role": "system", "content": "sys"}, {"role": "user", "content": "Hello world"},
            {"role": "assistant", "content": "a-b-c"}, {"role": "user", "content": "foo"}]
    rng = random.Random(3)
    for _ in range(300):
        tmpl = _tag(rng, "set ns = namespace(n=0)") + _tag(rng, "set x = 'v'") + _body(rng, 0, False)
        ref = tokenizer_ref.RefTokenizer(tokens, types, merges, tmpl, vocab["eos"], vocab["pad"])
        ours = Qwen3Tokenizer.from_vocab(tokens, merges, types, tmpl)
        assert ours.apply_chat_template(msgs, [], True) == ref.chat_json(msgs, [], True), tmpl


@pytest.mark.skipif(not tokenizer_ref.available(), reason="the reference tokenizer build (oracle/_ref) is absent")
def test_long_pieces_vs_reference(vocab):
    """Single pieces of up to 20000 letters (one pre-split match each): the
    heap-driven merges give the reference's ids."""
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, "", vocab["eos"], vocab["pad"])
    ref = tokenizer_ref.RefTokenizer(tokens, types, merges, "", vocab["eos"], vocab["pad"])
    rng = random.Random(4)
    for n in (2, 3, 17, 200, 3000, 20000):
        for alphabet in ("aaab", "etaoinshrdlu", "ab"):
            s = "".join(rng.choice(alphabet) for _ in range(n)).encode()
            assert len(t.pre_split(s)) == 1
            assert t.encode(s) == ref.encode(s), (n, alphabet)


def test_integration_adapter_vs_reference():
    """minfer's BaseTokenizer interface over this tokenizer (CudaTokenizer in
    integration/cuda_backend.cpp, run here without a GPU) gives the
    reference tokenizer's prompt and ids for a model file's vocabulary and
    chat template."""
    import subprocess

    from conftest import TEXT_MODEL, text_model
    from minfer_b200.gguf_synth import CHAT_TEMPLATE, synth_vocab

    app = Path(__file__).resolve().parent.parent / "integration" / "_build" / "minfer_cuda_app"
    if not app.exists() or not tokenizer_ref.available():
        pytest.skip("the integration app or the reference tokenizer is not built (both need the reference sources)")
    path = text_model()
    text = "Hello, world! It's 2 + 2 = 4; 世界\n  tabs\there"
    r = subprocess.run([str(app), "tokenize", path, "--prompt", text], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    tokens, types, merges, eos, pad = synth_vocab(TEXT_MODEL.vocab, TEXT_MODEL.seed, TEXT_MODEL.byte_vocab)
    ref = tokenizer_ref.RefTokenizer(tokens, types, merges, CHAT_TEMPLATE, eos, pad)
    expected = ref.chat([{"role": "user", "content": text}], [], True)
    assert out["formatted"] == expected
    assert out["ids"] == ref.encode(expected.encode())
    assert out["round_trip"] and out["eos"] == eos


def test_c_abi_short_buffers(vocab):
    """The C entry points write at most `cap` items and report the full count,
    so a caller can size its buffer and call again."""
    import ctypes as C

    from minfer_b200._lib import MF_OK, host_lib
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, merges, types = _args(vocab)
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, vocab["templates"]["chatml_min"], vocab["eos"], vocab["pad"])
    lib = host_lib()
    text = b"The quick brown fox jumps over the lazy dog."
    full = t.encode(text)
    ids = (C.c_uint32 * 3)(7, 7, 7)
    n = C.c_size_t()
    assert lib.mf_tokenizer_encode(t._h, text, len(text), ids, 2, C.byref(n)) == MF_OK
    assert n.value == len(full) and list(ids) == full[:2] + [7]
    arr = (C.c_uint32 * len(full))(*full)
    out = C.create_string_buffer(b"#" * 8, 8)
    assert lib.mf_tokenizer_decode(t._h, arr, len(full), out, 5, C.byref(n)) == MF_OK
    assert n.value == len(text) and out.raw[:5] == text[:5] and out.raw[5:8] == b"###"
    out = C.create_string_buffer(4)
    mj = b'[{"role": "user", "content": "hi"}]'
    assert lib.mf_tokenizer_apply_chat_template(t._h, mj, None, 1, out, 4, C.byref(n)) == MF_OK
    assert n.value == len(t.apply_chat_template([{"role": "user", "content": "hi"}]).encode())
    ends = (C.c_size_t * 1)()
    assert lib.mf_tokenizer_pre_split(t._h, text, len(text), ends, 1, C.byref(n)) == MF_OK
    assert n.value == len(t.pre_split(text)) and ends[0] == len(t.pre_split(text)[0])


def test_byte_vocabulary_generator():
    """The synthetic models' byte-level vocabulary (gguf_synth.synth_byte_vocab,
    used by the text tests): every single byte, every merge's result an entry,
    the chat specials typed as control tokens, and any byte string encodes and
    decodes back unchanged."""
    from minfer_b200.gguf_synth import CHAT_TEMPLATE, synth_byte_vocab
    from minfer_b200.tokenizer import Qwen3Tokenizer

    tokens, types, merges, eos, pad = synth_byte_vocab(1024, 107)
    assert len(tokens) == len(types) == 1024 and len(set(tokens[:256])) == 256
    vocab = set(tokens)
    for m in merges:  # "left right", where either part may hold spaces: some split gives an entry
        assert any(m[k:k + 1] == b" " and m[:k] + m[k + 1:] in vocab for k in range(1, len(m) - 1)), m
    assert tokens[eos] == b"<|im_end|>" and tokens[pad] == b"<|endoftext|>"
    assert types[tokens.index(b"<|im_start|>")] == 3 and types[-1] == 5
    t = Qwen3Tokenizer.from_vocab(tokens, merges, types, CHAT_TEMPLATE, eos, pad)
    rng = random.Random(8)
    for _ in range(200):
        b = bytes(rng.randrange(256) for _ in range(rng.randint(0, 64)))
        assert t.decode(t.encode(b)) == b


def test_json_output_needs_utf8():
    """Strings written as JSON (tojson, printed lists and objects) must be
    UTF-8; printed directly they pass through as bytes."""
    import ctypes as C

    from minfer_b200._lib import MF_E_STATE, MF_OK
    from minfer_b200.tokenizer import Qwen3Tokenizer

    t = Qwen3Tokenizer.from_vocab([bytes([i]) for i in range(256)], [], [1] * 256,
                                  "{{ messages[0].content }}{% if messages[0].role == 'json' %}"
                                  "|{{ messages[0].content | tojson }}{% endif %}")
    out = C.create_string_buffer(256)
    n = C.c_size_t()

    def render(role, content):
        mj = b'[{"role": "' + role + b'", "content": "' + content + b'"}]'
        return t._lib.mf_tokenizer_apply_chat_template(t._h, mj, None, 1, out, 256, C.byref(n))

    assert render(b"user", b"bad \xff") == MF_OK and out.raw[:n.value] == b"bad \xff"
    assert render(b"json", b"ok \xc3\xa9") == MF_OK and out.raw[:n.value] == b'ok \xc3\xa9|"ok \xc3\xa9"'
    assert render(b"json", b"bad \xff") == MF_E_STATE
