"""Byte-level BPE tokenizer with the reference's Python API
(src/rust_tokenizer.py: ``RustTokenizer``, ``get_rust_tokenizer``) over this
build's C++ library ``libmi_bpe.so`` (mamba_integer_b200/tokenizer/bpe.cpp,
C ABI in include/mi_bpe.h, the same entry-point names as the reference's Rust
cdylib, src/rust_tokenizer/src/lib.rs).

Host code only; the model consumes the ids.  Decoding follows the reference:
the byte string of every id is built from the merges in id order and the
concatenation is decoded as UTF-8 with replacement.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmi_bpe.so")


class RustTokenizer:
    def __init__(self, lib_path: Optional[str] = None, merges_path: Optional[str] = None):
        path = lib_path or LIB_PATH
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing; build it with `python -m mamba_integer_b200.build`")
        self.lib = ctypes.CDLL(path)
        self.lib.tokenizer_new.restype = ctypes.c_void_p
        self.lib.tokenizer_free.argtypes = [ctypes.c_void_p]
        self.lib.tokenizer_train.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_uint]
        self.lib.tokenizer_train.restype = ctypes.c_int
        self.lib.tokenizer_encode.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t)]
        self.lib.tokenizer_encode.restype = ctypes.POINTER(ctypes.c_uint)
        self.lib.tokenizer_free_ids.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_size_t]
        self.lib.tokenizer_save.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        self.lib.tokenizer_save.restype = ctypes.c_int
        self.lib.tokenizer_load.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        self.lib.tokenizer_load.restype = ctypes.c_int
        self.lib.mi_bpe_pretokenize.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t), ctypes.c_size_t,
                                                ctypes.POINTER(ctypes.c_size_t)]
        self.lib.mi_bpe_pretokenize.restype = ctypes.c_int
        self.tokenizer_ptr = self.lib.tokenizer_new()
        if not self.tokenizer_ptr:
            raise MemoryError("tokenizer_new failed")
        self.id_to_bytes: Dict[int, bytes] = {i: bytes([i]) for i in range(256)}
        if merges_path and os.path.exists(merges_path):
            self.load(merges_path)

    def __del__(self):
        if getattr(self, "lib", None) is not None and getattr(self, "tokenizer_ptr", None):
            self.lib.tokenizer_free(self.tokenizer_ptr)
            self.tokenizer_ptr = None

    def train(self, input_path: str, vocab_size: int) -> None:
        if self.lib.tokenizer_train(self.tokenizer_ptr, input_path.encode("utf-8"), vocab_size) != 0:
            raise Exception("Tokenizer training failed")

    def load(self, path: str) -> None:
        if self.lib.tokenizer_load(self.tokenizer_ptr, path.encode("utf-8")) != 0:
            raise Exception("Tokenizer load failed")
        self.id_to_bytes = {i: bytes([i]) for i in range(256)}
        merges = []
        with open(path, "r") as f:
            for line in f:
                parts = line.strip().split()
                if len(parts) != 2:
                    continue
                a, b = map(int, parts[0].split(","))
                merges.append((int(parts[1]), a, b))
        for idx, a, b in sorted(merges):
            self.id_to_bytes[idx] = self.id_to_bytes.get(a, b"") + self.id_to_bytes.get(b, b"")

    def encode(self, text: str) -> List[int]:
        n = ctypes.c_size_t(0)
        ptr = self.lib.tokenizer_encode(self.tokenizer_ptr, text.encode("utf-8"), ctypes.byref(n))
        if not ptr:
            return []
        ids = [ptr[i] for i in range(n.value)]
        self.lib.tokenizer_free_ids(ptr, n)
        return ids

    def save(self, output_path: str) -> None:
        if self.lib.tokenizer_save(self.tokenizer_ptr, output_path.encode("utf-8")) != 0:
            raise Exception("Tokenizer save failed")

    def decode(self, ids) -> str:
        return b"".join(self.id_to_bytes.get(int(i), b"") for i in ids).decode("utf-8", errors="replace")

    def pretokenize(self, text: str) -> List[str]:
        """The pieces the split pattern cuts text into (before any merge)."""
        raw = text.encode("utf-8")
        n = ctypes.c_size_t(0)
        cap = len(raw) + 1
        ends = (ctypes.c_size_t * cap)()
        rc = self.lib.mi_bpe_pretokenize(raw, ends, cap, ctypes.byref(n))
        if rc != 0:
            raise ValueError(f"mi_bpe_pretokenize failed ({rc})")
        out, start = [], 0
        for i in range(n.value):
            out.append(raw[start:ends[i]].decode("utf-8"))
            start = ends[i]
        return out


def get_rust_tokenizer(merges_path: Optional[str] = None) -> RustTokenizer:
    """The tokenizer over this build's library (the reference searches for its
    Rust librustbpe.so, src/rust_tokenizer.py:86-114)."""
    return RustTokenizer(LIB_PATH, merges_path)
