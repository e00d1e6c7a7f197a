"""CPU restatement of the reference's byte-level BPE tokenizer
(src/LLM.Core/Tokenizer/BpeTokenizer.cs) -- test infrastructure only.

The library's native tokenizer (forge-lm_b200/csrc/tokenizer.hpp) is checked
against this file.  Training restates TrainDocuments (BpeTokenizer.cs:90-236)
as a recount-every-merge loop with the same selection rule (highest count,
ties to the lowest pair key (left << 32) | right, at least 2 occurrences,
no pair across a document boundary); encoding is the rule Encode
is defined by (rank-greedy merging, BpeTokenizer.cs:259-318), written as the
plain repeated search for the lowest-rank pair, not as the reference's queues.
"""
from __future__ import annotations

import json


def pair_key(left: int, right: int) -> int:
    return (left << 32) | (right & 0xFFFFFFFF)


def train_documents(documents: list[bytes], num_merges: int) -> list[tuple[int, int, int]]:
    """Merges (left, right, new_id) in rank order."""
    seq: list[int] = []
    for d, doc in enumerate(documents):
        if d:
            seq.append(-1)  # boundary sentinel: never part of a pair
        seq.extend(doc)
    merges: list[tuple[int, int, int]] = []
    next_id = 256
    for _ in range(num_merges):
        if len(seq) < 2:
            break
        counts: dict[int, int] = {}
        for a, b in zip(seq, seq[1:]):
            if a >= 0 and b >= 0:
                k = pair_key(a, b)
                counts[k] = counts.get(k, 0) + 1
        if not counts:
            break
        best = min(counts, key=lambda k: (-counts[k], k))
        if counts[best] < 2:
            break
        left, right = best >> 32, best & 0xFFFFFFFF
        merges.append((left, right, next_id))
        out, i = [], 0
        while i < len(seq):
            if i + 1 < len(seq) and seq[i] == left and seq[i + 1] == right:
                out.append(next_id)
                i += 2
            else:
                out.append(seq[i])
                i += 1
        seq = out
        next_id += 1
    return merges


def encode(data: bytes, merges: list[tuple[int, int, int]]) -> list[int]:
    """Encode's defining rule (the class remarks of BpeTokenizer.cs, restated
    here rather than its algorithm at BpeTokenizer.cs:273-318): start from
    the byte ids; while some adjacent pair is a learned merge, take the pair
    of lowest rank and merge its leftmost occurrence; repeat.

    One pass per chosen rank merges every occurrence of that pair left to
    right, skipping overlaps: that is the same sequence of leftmost merges,
    because merging a pair of rank r only creates pairs that contain the new
    id 256 + r, and every such pair has a rank above r."""
    rank = {pair_key(l, r): k for k, (l, r, _) in enumerate(merges)}
    seq = list(data)
    while len(seq) > 1:
        best = min((rank[k] for k in (pair_key(a, b) for a, b in zip(seq, seq[1:])) if k in rank), default=None)
        if best is None:
            break
        left, right, new_id = merges[best]
        out, i = [], 0
        while i < len(seq):
            if i + 1 < len(seq) and seq[i] == left and seq[i + 1] == right:
                out.append(new_id)
                i += 2
            else:
                out.append(seq[i])
                i += 1
        seq = out
    return seq


def vocab_bytes(merges: list[tuple[int, int, int]]) -> list[bytes]:
    vocab = [bytes([i]) for i in range(256)]
    for l, r, _ in merges:
        vocab.append(vocab[l] + vocab[r])
    vocab.append(b"")  # EOS
    return vocab


def decode(ids: list[int], merges: list[tuple[int, int, int]]) -> bytes:
    vocab = vocab_bytes(merges)
    return b"".join(vocab[i] for i in ids)


def save(path, merges: list[tuple[int, int, int]]) -> None:
    """BpeTokenizer.Save's JSON (BpeTokenizer.cs:341-351; EOS = 256 + merges)."""
    with open(path, "w", encoding="utf-8") as f:
        json.dump({"Version": 2, "Merges": [list(m) for m in merges], "EosTokenId": 256 + len(merges)}, f, indent=2)
