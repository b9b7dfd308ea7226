"""Oracle of the BPE tokenizer (TEST INFRASTRUCTURE ONLY, see oracle/__init__).

A restatement of the reference's Rust tokenizer (src/rust_tokenizer/src/lib.rs)
in Python: the split pattern (lib.rs:8-9) run by the `regex` module (a
backtracking engine with Unicode classes, possessive quantifiers and
lookahead, as the reference's fancy-regex 0.11 is), the greedy merge loop of
tokenizer_encode (lib.rs:84-93) and the training loop of tokenizer_train
(lib.rs:26-71) with ties broken towards the smallest pair (the reference's
hash-map order is arbitrary).  The reference tokenizer itself is a Rust crate
and cannot be built here (no cargo), so parity with it is pinned only through
this restatement and the pattern's own engine.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import regex

PATTERN = (r"'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
           r"\s*[\r\n]|\s+(?!\S)|\s+")
_RX = regex.compile(PATTERN)


def pretokenize(text: str) -> List[str]:
    return [m.group(0) for m in _RX.finditer(text)]


def load_merges(path: str) -> Dict[Tuple[int, int], int]:
    merges = {}
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) != 2:
                continue
            a, b = map(int, parts[0].split(","))
            merges[(a, b)] = int(parts[1])
    return merges


def encode(text: str, merges: Dict[Tuple[int, int], int]) -> List[int]:
    out: List[int] = []
    for piece in pretokenize(text):
        ids = list(piece.encode("utf-8"))
        while len(ids) >= 2:
            best = None
            for i in range(len(ids) - 1):
                m = merges.get((ids[i], ids[i + 1]))
                if m is not None and (best is None or m < best[1]):
                    best = (i, m)
            if best is None:
                break
            i, m = best
            ids[i:i + 2] = [m]
        out.extend(ids)
    return out


def train(lines: List[str], vocab_size: int) -> Dict[Tuple[int, int], int]:
    counts: Dict[tuple, int] = {}
    for line in lines:
        for piece in pretokenize(line):
            k = tuple(piece.encode("utf-8"))
            counts[k] = counts.get(k, 0) + 1
    merges: Dict[Tuple[int, int], int] = {}
    for i in range(max(0, vocab_size - 256)):
        pc: Dict[Tuple[int, int], int] = {}
        for ids, c in counts.items():
            for a, b in zip(ids, ids[1:]):
                pc[(a, b)] = pc.get((a, b), 0) + c
        if not pc:
            break
        top = max(pc.values())
        pair = min(p for p, c in pc.items() if c == top)
        new_id = 256 + i
        merges[pair] = new_id
        nxt: Dict[tuple, int] = {}
        for ids, c in counts.items():
            out, j = [], 0
            while j < len(ids):
                if j + 1 < len(ids) and (ids[j], ids[j + 1]) == pair:
                    out.append(new_id)
                    j += 2
                else:
                    out.append(ids[j])
                    j += 1
            nxt[tuple(out)] = nxt.get(tuple(out), 0) + c
        counts = nxt
    return merges
