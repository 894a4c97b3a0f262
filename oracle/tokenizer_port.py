"""Pure-Python restatement of the reference tokenizer and random stream (TEST INFRASTRUCTURE ONLY:
the checker for the library's tokenizer.c and sampler.c; nothing in the product imports it).

Follows the reference step by step, including its quirks:

* ``load``: tokenizer.bin = int32 vocab_size, max_token_length, bos_id, eos_id, then per piece
  float32 score, int32 length, bytes (src/tokenizer.c:11-48).
* ``encode`` (src/tokenizer.c:93-209): BOS id 1 if asked; the " " piece when the text is not
  empty; code points of a leading byte plus at most three continuation bytes, looked up whole or
  spelled as byte tokens (byte + 3); then, while some adjacent pair concatenates to a piece whose
  score is above -1e10, merge the best-scoring pair, the first (leftmost) one on ties -- a full
  rescan per merge, exactly as the reference does; EOS id 2 if asked.
* ``decode`` (src/tokenizer.c:60-71): one leading space dropped after token 1; a piece that the
  C format "<0x%02hhX>" matches becomes that byte.
* ``random_u32`` / ``random_f32``: the xorshift* stream of src/sampler.c:96-106.

Pinned against the compiled reference (oracle/_ref) in tests/test_host_api.py.
"""
from __future__ import annotations

import struct

import numpy as np

MASK64 = (1 << 64) - 1


def load(path: str):
    with open(path, "rb") as f:
        data = f.read()
    vocab_size, max_len, bos, eos = struct.unpack_from("<iiii", data, 0)
    off = 16
    pieces, scores = [], []
    for _ in range(vocab_size):
        score, n = struct.unpack_from("<fi", data, off)
        off += 8
        pieces.append(data[off:off + n])
        off += n
        scores.append(np.float32(score))
    return pieces, scores, max_len, bos, eos


def encode(pieces, scores, text: bytes, bos: bool, eos: bool) -> list[int]:
    # str_lookup on NUL-terminated strings: a piece is found by its bytes up to the first NUL
    lookup = {}
    for i, p in enumerate(pieces):
        key = p.split(b"\0", 1)[0]
        # bsearch over the sorted table may return any of equal keys; test vocabularies have none
        lookup.setdefault(key, i)
    toks = []
    if bos:
        toks.append(1)
    if text:
        toks.append(lookup[b" "])
    i = 0
    while i < len(text):
        j = i + 1
        while j < len(text) and j - i < 4 and (text[j] & 0xC0) == 0x80:
            j += 1
        cp = text[i:j]
        if cp in lookup:
            toks.append(lookup[cp])
        else:
            toks.extend(b + 3 for b in cp)
        i = j
    while True:
        best, best_id, best_idx = np.float32(-1e10), -1, -1
        for k in range(len(toks) - 1):
            cand = pieces[toks[k]].split(b"\0", 1)[0] + pieces[toks[k + 1]].split(b"\0", 1)[0]
            tid = lookup.get(cand, -1)
            if tid != -1 and scores[tid] > best:
                best, best_id, best_idx = scores[tid], tid, k
        if best_idx == -1:
            break
        toks[best_idx] = best_id
        del toks[best_idx + 1]
    if eos:
        toks.append(2)
    return toks


def _scan_byte(piece: bytes):
    """sscanf(piece, "<0x%02hhX>", &b) == 1 for the pieces tokenizers hold: "<0x" then one or two
    hex digits."""
    if not piece.startswith(b"<0x"):
        return None
    digits = b""
    for c in piece[3:5]:
        if chr(c) in "0123456789abcdefABCDEF":
            digits += bytes([c])
        else:
            break
    return int(digits, 16) if digits else None


def decode(pieces, prev: int, token: int) -> bytes:
    p = pieces[token].split(b"\0", 1)[0]
    if prev == 1 and p[:1] == b" ":
        p = p[1:]
    b = _scan_byte(p)
    return bytes([b]) if b is not None else p


def random_u32(state: int) -> tuple[int, int]:
    state ^= state >> 12
    state ^= (state << 25) & MASK64
    state ^= state >> 27
    return ((state * 0x2545F4914F6CDD1D) & MASK64) >> 32, state


def random_f32(state: int) -> tuple[float, int]:
    u, state = random_u32(state)
    return float(np.float32(u >> 8) / np.float32(16777216.0)), state
