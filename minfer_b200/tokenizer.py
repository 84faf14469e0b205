"""Qwen3 tokenizer (host side, no GPU): the reference's Qwen3Tokenizer
interface (include/minfer/models/qwen3/tokenizer.hpp: encode, decode,
decode_token, apply_chat_template) over the C++ implementation in
libminfer_host.so (csrc/host/tokenizer.cpp, csrc/host/chat_template.cpp).

Text is bytes or str (str is encoded as UTF-8); decode returns bytes, since
a token's string is raw bytes and a prefix of a sequence may end inside a
UTF-8 character."""
import ctypes as C
import json
from dataclasses import dataclass, field

from ._lib import MF_E_INVALID, MinferError, check, host_lib


@dataclass
class Message:
    """BaseTokenizer::Message (include/minfer/base/tokenizer.hpp:13-20)."""
    role: str
    content: str
    reasoning_content: str = ""
    tool_calls: list[tuple[str, str]] = field(default_factory=list)  # (name, arguments as JSON text)

    def to_json(self) -> dict:
        d = {"role": self.role, "content": self.content}
        if self.reasoning_content:
            d["reasoning_content"] = self.reasoning_content
        if self.tool_calls:
            # the reference parses each arguments text into a JSON value
            d["tool_calls"] = [{"name": n, "arguments": json.loads(a)} for n, a in self.tool_calls]
        return d


@dataclass
class Tool:
    """BaseTokenizer::Tool (include/minfer/base/tokenizer.hpp:22-26)."""
    name: str
    description: str
    parameters: str  # JSON text

    def to_json(self) -> dict:
        return {"name": self.name, "description": self.description, "parameters": json.loads(self.parameters)}


def _b(text) -> bytes:
    return text.encode() if isinstance(text, str) else bytes(text)


class Qwen3Tokenizer:
    def __init__(self, handle: C.c_void_p):
        self._lib = host_lib()
        self._h = handle
        vs, eos, pad = C.c_size_t(), C.c_uint32(), C.c_uint32()
        check(self._lib.mf_tokenizer_info(self._h, C.byref(vs), C.byref(eos), C.byref(pad)))
        self.vocab_size, self.eos_id, self.pad_id = vs.value, eos.value, pad.value

    @classmethod
    def from_gguf(cls, path: str) -> "Qwen3Tokenizer":
        h = C.c_void_p()
        check(host_lib().mf_tokenizer_load(str(path).encode(), C.byref(h)))
        return cls(h)

    @classmethod
    def from_vocab(cls, tokens: list[bytes], merges: list[bytes], token_types: list[int], chat_template: str = "",
                   eos_id: int = 0, pad_id: int = 0) -> "Qwen3Tokenizer":
        """Qwen3Tokenizer(tokens, merges, token_types, chat_template, eos_id, pad_id)."""
        if len(token_types) != len(tokens):  # (the C entry point takes one count for both arrays)
            raise MinferError(MF_E_INVALID, "Token and token_type arrays must have same size")
        tk = [_b(t) for t in tokens]
        mg = [_b(m) for m in merges]
        tp = (C.c_char_p * max(1, len(tk)))(*tk)
        tl = (C.c_size_t * max(1, len(tk)))(*[len(t) for t in tk])
        ty = (C.c_uint32 * max(1, len(token_types)))(*token_types)
        mp = (C.c_char_p * max(1, len(mg)))(*mg)
        ml = (C.c_size_t * max(1, len(mg)))(*[len(m) for m in mg])
        h = C.c_void_p()
        check(host_lib().mf_tokenizer_create(tp, tl, ty, len(tk), mp, ml, len(mg), chat_template.encode(), eos_id,
                                             pad_id, C.byref(h)))
        return cls(h)

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.mf_tokenizer_free(self._h)
            self._h = None

    def encode(self, text) -> list[int]:
        b = _b(text)
        cap = len(b) + 16
        while True:
            buf = (C.c_uint32 * cap)()
            n = C.c_size_t()
            check(self._lib.mf_tokenizer_encode(self._h, b, len(b), buf, cap, C.byref(n)))
            if n.value <= cap:
                return list(buf[: n.value])
            cap = n.value

    def decode(self, ids) -> bytes:
        ids = list(ids)
        arr = (C.c_uint32 * max(1, len(ids)))(*ids)
        cap = 16 * len(ids) + 16
        while True:
            out = C.create_string_buffer(cap)
            n = C.c_size_t()
            check(self._lib.mf_tokenizer_decode(self._h, arr, len(ids), out, cap, C.byref(n)))
            if n.value <= cap:
                return out.raw[: n.value]
            cap = n.value

    def decode_token(self, token_id: int) -> bytes:
        return self.decode([token_id])

    # BaseTokenizer::get_eos_id / get_pad_id (include/minfer/base/tokenizer.hpp:41-42)
    def get_eos_id(self) -> int:
        return self.eos_id

    def get_pad_id(self) -> int:
        return self.pad_id

    def pre_split(self, text) -> list[bytes]:
        """The pieces encode turns into ids (the reference's regex_split)."""
        b = _b(text)
        cap = len(b) + 1
        ends = (C.c_size_t * cap)()
        n = C.c_size_t()
        check(self._lib.mf_tokenizer_pre_split(self._h, b, len(b), ends, cap, C.byref(n)))
        out, start = [], 0
        for e in ends[: n.value]:
            out.append(b[start:e])
            start = e
        return out

    def apply_chat_template(self, messages, tools=(), add_generation_prompt: bool = True) -> str:
        """messages: Message objects or dicts of the JSON shape the reference
        builds from them; tools likewise. The prompt's bytes are returned as
        str (a template that slices strings works on bytes, so bytes that are
        not UTF-8 come back as surrogate escapes)."""
        msgs = [m.to_json() if isinstance(m, Message) else m for m in messages]
        tls = [t.to_json() if isinstance(t, Tool) else t for t in tools]
        mj, tj = json.dumps(msgs).encode(), json.dumps(tls).encode()
        cap = 4096
        while True:
            out = C.create_string_buffer(cap)
            n = C.c_size_t()
            check(self._lib.mf_tokenizer_apply_chat_template(self._h, mj, tj, int(add_generation_prompt), out, cap,
                                                             C.byref(n)))
            if n.value <= cap:
                return out.raw[: n.value].decode(errors="surrogateescape")
            cap = n.value


__all__ = ["Qwen3Tokenizer", "Message", "Tool", "MinferError"]
