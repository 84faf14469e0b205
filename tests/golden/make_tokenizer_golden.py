"""Writes the tokenizer fixtures of tests/golden/:

* tokenizer_vocab.json: a byte-level BPE vocabulary (the 256 single bytes,
  merged strings, special and unused tokens, merge rules as "left right" byte
  strings, the byte form the reference's GGUF converter writes) trained here
  on seeded synthetic text, plus chat templates written for the tests;
* tokenizer_cases.json: for every test text, the pieces and ids of the
  reference's own tokenizer (oracle/_ref/libtokenizer_ref.so, built from
  src/models/qwen3/tokenizer.cpp), and for every chat case the rendered
  prompt of its chat template path (minja).

Run from the repository root in the development container, after
`make -C oracle REF=<reference checkout> tokenizer`:
    python tests/golden/make_tokenizer_golden.py
"""
import json
import random
import sys
from collections import Counter
from pathlib import Path

import regex

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import tokenizer_ref  # noqa: E402

# training split only (the product and the reference use their own split)
TRAIN_SPLIT = regex.compile(r"""'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}++|\p{N}{1,3}+| ?[^\s\p{L}\p{N}]++[\r\n]*+|\s++$|\s*[\r\n]|\s+(?!\S)|\s""")

SPECIALS = [("<|endoftext|>", 3), ("<|im_start|>", 3), ("<|im_end|>", 3), ("<think>", 4), ("</think>", 4),
            ("<tool_call>", 4), ("</tool_call>", 4)]
N_UNUSED = 3
N_MERGES = 700

SYLL = ["ka", "to", "ren", "mi", "sol", "ve", "tha", "in", "er", "on", "an", "qu", "ix", "el", "or", "us", "st",
        "pre", "ing", "ed", "ly", "the", "and", "com", "pu", "ter", "gra", "ph", "ic", "al"]
PROSE = (
    "The kernel streams every weight row once per token, so the decode step is bound by memory bandwidth. "
    "Each layer normalises its input, projects queries, keys and values, rotates them, and attends over the cache. "
    "A router picks eight experts for every token; their outputs are weighted and summed. "
    "Numbers like 3.14159, 2048 and 151936 appear in configs, and so do paths such as /tmp/model.gguf. "
    "It's what they'd said: we're done, you'll see, I'm sure, it's fine. "
    "def forward(x):\n    return x * 2  # doubled\n\tindent\r\nwindows line\n\n\nend "
)


def corpus(rng: random.Random) -> str:
    parts = [PROSE] * 4
    for _ in range(4000):
        w = "".join(rng.choice(SYLL) for _ in range(rng.randint(1, 3)))
        if rng.random() < 0.15:
            w = w.capitalize()
        parts.append(w + rng.choice([" ", " ", " ", ", ", ". ", "\n", "  "]))
    for _ in range(300):
        parts.append(" " + str(rng.randint(0, 10 ** rng.randint(1, 7))))
        parts.append(" " + "".join(chr(rng.randint(0x4E00, 0x4E00 + 400)) for _ in range(rng.randint(1, 4))))
        parts.append(" " + "".join(chr(rng.randint(0x430, 0x44F)) for _ in range(rng.randint(2, 6))))
    return "".join(parts)


def train(text: str) -> list[tuple[bytes, bytes]]:
    words = Counter(m.encode() for m in TRAIN_SPLIT.findall(text))
    seqs = {w: [bytes([b]) for b in w] for w in words}
    merges = []
    for _ in range(N_MERGES):
        pairs = Counter()
        for w, c in words.items():
            s = seqs[w]
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append((a, b))
        for w in words:
            s = seqs[w]
            i, out = 0, []
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    return merges


def build_vocab():
    rng = random.Random(1234)
    merges = train(corpus(rng))
    tokens = [bytes([b]) for b in range(256)]
    seen = set(tokens)
    for a, b in merges:
        if a + b not in seen:
            tokens.append(a + b)
            seen.add(a + b)
    types = [1] * len(tokens)
    for s, t in SPECIALS:
        tokens.append(s.encode())
        types.append(t)
    for i in range(N_UNUSED):
        tokens.append(b"<|unused_%d|>" % i)
        types.append(5)
    eos = tokens.index(b"<|im_end|>")
    pad = tokens.index(b"<|endoftext|>")
    return tokens, types, [a + b" " + b for a, b in merges], eos, pad


TEMPLATES = {
    # the synthetic GGUF models' template (minfer_b200/gguf_synth.py)
    "chatml_min": (
        "{%- for message in messages %}{{- '<|im_start|>' + message.role + '\\n' + message.content + "
        "'<|im_end|>' + '\\n' }}{%- endfor %}{%- if add_generation_prompt %}{{- '<|im_start|>assistant\\n' }}"
        "{%- endif %}"),
    # system prompt, tools, reasoning, tool calls and tool responses; block
    # tags on their own lines exercise trim_blocks / lstrip_blocks
    "chatml_tools": """{%- set ns = namespace(last_user=-1, n_tools=0) %}
{%- for m in messages %}
    {%- if m.role == 'user' %}{% set ns.last_user = loop.index0 %}{% endif %}
{%- endfor %}
{%- if tools %}
{{- bos_token }}system
{%- if messages[0].role == 'system' %}
{{ messages[0].content | trim }}

{% endif %}
# Tools ({{ tools | length }})
{% for tool in tools %}
{{- tool | tojson }}
{% set ns.n_tools = ns.n_tools + 1 %}
{% endfor %}
Call at most {{ ns.n_tools }} tool{{ 's' if ns.n_tools != 1 else '' }}.{{ eos_token }}
{% elif messages[0].role == 'system' %}
{{- bos_token + 'system\\n' + messages[0].content + eos_token + '\\n' }}
{%- endif %}
{%- for m in messages %}
    {%- if m.role == 'system' %}
    {%- elif m.role == 'user' or (m.role == 'assistant' and m.tool_calls is not defined) %}
        {%- set text = m.content if m.content is string else '' %}
        {%- if m.role == 'assistant' and m.reasoning_content is defined and loop.index0 > ns.last_user %}
{{- bos_token + m.role + '\\n<think>\\n' + m.reasoning_content.strip('\\n') + '\\n</think>\\n\\n' + text.lstrip('\\n') + eos_token + '\\n' }}
        {%- else %}
{{- bos_token ~ m.role ~ '\\n' ~ text ~ eos_token ~ '\\n' }}
        {%- endif %}
    {%- elif m.role == 'assistant' %}
{{- bos_token + 'assistant' }}
        {%- if m.content %}{{ '\\n' + m.content }}{% endif %}
        {%- for tc in m.tool_calls %}
            {%- set f = tc.function if tc.function is defined else tc %}
{{- '\\n<tool_call>\\n{"name": "' + f.name + '", "arguments": ' }}
            {%- if f.arguments is string %}{{ f.arguments }}{% else %}{{ f.arguments | tojson }}{% endif %}
{{- '}\\n</tool_call>' }}
        {%- endfor %}
{{- eos_token + '\\n' }}
    {%- elif m.role == 'tool' %}
        {%- if loop.first or messages[loop.index0 - 1].role != 'tool' %}{{ bos_token + 'user' }}{% endif %}
{{- '\\n<tool_response>\\n' + m.content + '\\n</tool_response>' }}
        {%- if loop.last or messages[loop.index0 + 1].role != 'tool' %}{{ eos_token + '\\n' }}{% endif %}
    {%- endif %}
{%- endfor %}
{%- if add_generation_prompt %}
{{- bos_token + 'assistant\\n' }}
{%- endif %}
""",
    # expressions and filters: arithmetic, comparisons, membership, slices,
    # string methods, list and dict literals, for/else, loop variables
    "exprs": """{% set words = messages | map(attribute='content') | list %}
{% for m in messages %}
{{ loop.index }}/{{ loop.length }} {{ m.role | upper }}{% if loop.first %} (first){% endif %}{% if loop.last %} (last){% endif %}: {{ m.content[:12] }}|{{ m.content[-3:] }}|{{ m.content | length }}
{% if 'e' in m.content %}has e{% else %}no e{% endif %} {{ m.content.split(' ') | length }} words
{% endfor %}
{% for x in [] %}never{% else %}empty loop{% endfor %}
{{ (7 // 2) }} {{ 7 % 3 }} {{ 2 ** 5 }} {{ -3 + 10 * 2 }} {{ 1.5 * 2 }} {{ 10 / 4 }}
{{ [1, 2, 3][::-1] | join(',') }} {{ 'abc'[::-1] }} {{ {'a': 1, 'b': [2, 3]} | tojson }}
{{ 'x' ~ 1 ~ true ~ none }} {{ none is none }} {{ 3 is number }} {{ 'q' is string }} {{ [1] is iterable }}
{{ not true or false and true }} {{ 1 < 2 }} {{ 2 >= 3 }} {{ 'b' not in 'abc' }} {{ messages | length > 1 }}
{{ '  pad  ' | trim }}|{{ 'A-B-C'.replace('-', '+') }}|{{ 'Mixed Case'.lower() }}|{{ 'title me'.title() }}|{{ 'cap'.capitalize() }}|{{ 'ab' | upper | lower }}
{{ undefined_var | default('dflt') }} {{ messages[0].role }} {{ (messages | last).role }} {{ range(3) | list | join('-') }} {{ [3, 1, 3] | unique | list | length }} {{ add_generation_prompt }}
{%- if add_generation_prompt %}

<|im_start|>assistant
{% endif %}""",
}

TEXTS = [
    "", "Hello, world!", "The quick brown fox jumps over the lazy dog.", "This is a simple test.",
    "<|im_start|>", "<|im_end|>", "<|endoftext|>", "<|im_start|>user\nHello<|im_end|>",
    "<|im_start|>system\nBe brief.<|im_end|>\n<|im_start|>user\nHi there<|im_end|>\n<|im_start|>assistant\n",
    "<think>\nreasoning here\n</think>\n\nanswer", "<tool_call>\n{\"name\": \"f\"}\n</tool_call>",
    "Hello, \u4e16\u754c!", "Caf\u00e9 na\u00efve r\u00e9sum\u00e9", "\U0001F680 \U0001F31F \u2728",
    "\u041f\u0440\u0438\u0432\u0435\u0442 \u043c\u0438\u0440", "\u0645\u0631\u062d\u0628\u0627 \u0628\u0627\u0644\u0639\u0627\u0644\u0645",
    "1234567890", "!@#$%^&*()", "3.14159", "user@example.com", "https://example.com/a/b?c=d&e=f",
    "Hello 123 world! \U0001F30D", "Code: `print('hello')`", "Math: 2 + 2 = 4", "Line1\nLine2\tTabbed",
    "it's we're they'd I'll you've she'S IT'LL WE'RE o'Ma 'x '\u017f", "  leading and trailing  ",
    "a\n\nb\r\n\r\nc \n d  \n  e", "tabs\t\tand\t spaces \t", "trailing newline\n", "   ", "\n", "\r\n\r\n",
    "ideographic\u3000space and nbsp\u00a0here\u2028line sep", "x\u2003\u2003y", "digits \u0661\u0662\u0663\u0664 \u00b2\u00b3 \u2167",
    "mixed123abc456", "....!!!???\n\nword", " ...leading space punct", "a<|im_end|>b<|im_start|>c",
    "<|im_end|><|im_end|>", "<|im_start", "unused <|unused_0|> text", "x" * 300 + " " + "ab" * 200,
    "word " * 50 + "\n" * 3,
]
INVALID = [b"bad \xff byte", b"\xc3\xa9\xff\xc3\xa9 after", b"trunc \xe4\xb8", b"\xed\xa0\x80 surrogate",
           b"overlong \xc0\xaf", b"ok <|im_end|>\xfe\xfe<|im_start|> ok", b"\x80\x80 lead", b"tail \xf4\x90\x80\x80"]


def fuzz_texts(rng: random.Random, n: int) -> list[bytes]:
    pool = (list(" \t\n\r\n") + list("abcXYZ'sSdmtlvre019.,!?-_/") + ["\u00e9", "\u4e2d", "\u0416", "\U0001F600",
            "\u3000", "\u00a0", "\u0663", "\u017f", "\u2028", "<|im_end|>", "<think>", "  ", "\n\n"])
    out = []
    for _ in range(n):
        s = "".join(rng.choice(pool) for _ in range(rng.randint(1, 40)))
        b = s.encode()
        if rng.random() < 0.15:  # an invalid byte somewhere
            i = rng.randint(0, len(b))
            b = b[:i] + bytes([rng.choice([0xff, 0x80, 0xc3, 0xe4])]) + b[i:]
        out.append(b)
    return out


def chat_cases():
    tool = {"name": "get_weather", "description": "Weather for a city.",
            "parameters": json.dumps({"type": "object", "properties": {"city": {"type": "string"}},
                                      "required": ["city"]})}
    calc = {"name": "calc", "description": "Evaluate <expr> & return.", "parameters": "{\"expr\": \"string\"}"}
    sys_user = [{"role": "system", "content": "You are terse."}, {"role": "user", "content": "What is 2+2?"}]
    convo = sys_user + [
        {"role": "assistant", "content": "4", "reasoning_content": "\nadd them\n"},
        {"role": "user", "content": "And the weather in Oslo?"},
        {"role": "assistant", "content": "", "tool_calls": [["get_weather", "{\"city\": \"Oslo\", \"units\": [1, 2.5, true, null]}"]]},
        {"role": "tool", "content": "{\"temp\": -3}"},
        {"role": "tool", "content": "second result"},
        {"role": "assistant", "content": "Cold: -3.", "reasoning_content": "read the tool"},
    ]
    plain = [{"role": "user", "content": "Hi \u4e16\u754c, it's me!"}, {"role": "assistant", "content": "Hello o/"},
             {"role": "user", "content": "one two three four"}]
    cases = []
    for name, msgs, tools in [("chatml_min", plain, []), ("chatml_min", sys_user, []),
                              ("chatml_tools", sys_user, []), ("chatml_tools", plain, []),
                              ("chatml_tools", convo, [tool, calc]), ("chatml_tools", convo, []),
                              ("chatml_tools", sys_user, [calc]), ("exprs", plain, []), ("exprs", sys_user, [])]:
        for gen in (True, False):
            cases.append({"template": name, "messages": msgs, "tools": tools, "add_generation_prompt": gen})
    return cases


def main():
    if not tokenizer_ref.available():
        sys.exit("oracle/_ref/libtokenizer_ref.so is not built (make -C oracle REF=<reference checkout> tokenizer)")
    tokens, types, merges, eos, pad = build_vocab()
    vocab = {"tokens": [t.hex() for t in tokens], "types": types, "merges": [m.hex() for m in merges],
             "eos": eos, "pad": pad, "templates": TEMPLATES}
    (HERE / "tokenizer_vocab.json").write_text(json.dumps(vocab, indent=0) + "\n")

    cases = {"texts": [], "chats": []}
    refs = {name: tokenizer_ref.RefTokenizer(tokens, types, merges, tmpl, eos, pad) for name, tmpl in TEMPLATES.items()}
    ref = refs["chatml_min"]
    texts = [t.encode() for t in TEXTS] + INVALID + fuzz_texts(random.Random(77), 150)
    for b in texts:
        ids = ref.encode(b)
        assert ref.decode(ids) == b, b  # the reference's round trip
        cases["texts"].append({"text": b.hex(), "pieces": ref.split(b), "ids": ids})
    for c in chat_cases():
        c = dict(c, expected=refs[c["template"]].chat(c["messages"], c["tools"], c["add_generation_prompt"]))
        cases["chats"].append(c)
    (HERE / "tokenizer_cases.json").write_text(json.dumps(cases, indent=0, ensure_ascii=False) + "\n")
    print(f"{len(tokens)} tokens, {len(merges)} merges, {len(cases['texts'])} texts, {len(cases['chats'])} chats")


if __name__ == "__main__":
    main()
