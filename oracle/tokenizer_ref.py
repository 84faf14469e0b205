"""ctypes access to the reference's own tokenizer (oracle/_ref/libtokenizer_ref.so,
built by `make -C oracle REF=<reference checkout> tokenizer` from src/models/qwen3/tokenizer.cpp and the
vendored minja/nlohmann headers, against the system PCRE2 runtime).

Test infrastructure: the tokenizer golden vectors come from here, and the
tokenizer tests compare the product with it where the library is built.
"""
import ctypes as C
import json
import struct
from pathlib import Path

LIB = Path(__file__).resolve().parent / "_ref" / "libtokenizer_ref.so"


def available() -> bool:
    return LIB.exists()


def _blob(tokens: list[bytes], types: list[int], merges: list[bytes], template: str, eos: int, pad: int) -> bytes:
    out = [struct.pack("<Q", len(tokens))]
    for t, ty in zip(tokens, types):
        out += [struct.pack("<Q", len(t)), t, struct.pack("<I", ty)]
    out.append(struct.pack("<Q", len(merges)))
    for m in merges:
        out += [struct.pack("<Q", len(m)), m]
    tb = template.encode()
    out += [struct.pack("<Q", len(tb)), tb, struct.pack("<II", eos, pad)]
    return b"".join(out)


class RefTokenizer:
    def __init__(self, tokens, types, merges, template, eos, pad):
        lib = C.CDLL(str(LIB))
        lib.tref_create.restype = C.c_void_p
        lib.tref_create.argtypes = [C.c_char_p, C.c_size_t]
        lib.tref_free.argtypes = [C.c_void_p]
        lib.tref_error.restype = C.c_char_p
        lib.tref_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_uint32), C.c_size_t,
                                    C.POINTER(C.c_size_t)]
        lib.tref_split.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_uint64), C.c_size_t,
                                   C.POINTER(C.c_size_t)]
        lib.tref_decode.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.c_size_t, C.c_char_p, C.c_size_t,
                                    C.POINTER(C.c_size_t)]
        lib.tref_chat.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int, C.c_char_p, C.c_size_t,
                                  C.POINTER(C.c_size_t)]
        lib.tref_chat_json.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int, C.c_char_p, C.c_size_t,
                                       C.POINTER(C.c_size_t)]
        self.lib = lib
        blob = _blob(tokens, types, merges, template, eos, pad)
        self.h = lib.tref_create(blob, len(blob))
        if not self.h:
            raise RuntimeError(lib.tref_error().decode(errors="replace"))

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.tref_free(self.h)

    def _err(self):
        return RuntimeError(self.lib.tref_error().decode(errors="replace"))

    def encode(self, text: bytes) -> list[int]:
        cap = 4 * len(text) + 16
        buf = (C.c_uint32 * cap)()
        n = C.c_size_t()
        if self.lib.tref_encode(self.h, text, len(text), buf, cap, C.byref(n)):
            raise self._err()
        return list(buf[: n.value])

    def split(self, text: bytes) -> list[int]:
        cap = len(text) + 16
        buf = (C.c_uint64 * cap)()
        n = C.c_size_t()
        if self.lib.tref_split(self.h, text, len(text), buf, cap, C.byref(n)):
            raise self._err()
        return list(buf[: n.value])

    def decode(self, ids: list[int]) -> bytes:
        arr = (C.c_uint32 * max(1, len(ids)))(*ids)
        cap = 64 * len(ids) + 64
        out = C.create_string_buffer(cap)
        n = C.c_size_t()
        if self.lib.tref_decode(self.h, arr, len(ids), out, cap, C.byref(n)):
            raise self._err()
        return out.raw[: n.value]

    def chat(self, messages: list[dict], tools: list[dict], add_generation_prompt: bool) -> str:
        """messages: {role, content, reasoning_content?, tool_calls?: [[name, arguments JSON text]]};
        tools: {name, description, parameters: JSON text} (the reference's Message/Tool)."""
        cap = 1 << 20
        out = C.create_string_buffer(cap)
        n = C.c_size_t()
        if self.lib.tref_chat(self.h, json.dumps(messages).encode(), json.dumps(tools).encode(),
                              int(add_generation_prompt), out, cap, C.byref(n)):
            raise self._err()
        return out.raw[: n.value].decode(errors="surrogateescape")

    def chat_json(self, messages, tools, add_generation_prompt: bool) -> str:
        """The chat-template engine on any JSON messages/tools (tools None: unset)."""
        cap = 1 << 20
        out = C.create_string_buffer(cap)
        n = C.c_size_t()
        tj = None if tools is None else json.dumps(tools).encode()
        if self.lib.tref_chat_json(self.h, json.dumps(messages).encode(), tj, int(add_generation_prompt), out, cap,
                                   C.byref(n)):
            raise self._err()
        return out.raw[: n.value].decode(errors="surrogateescape")
