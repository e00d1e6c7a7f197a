"""CPU restatement of the reference's byte-level BPE tokenizer
(src/LLM.Core/Tokenizer/BpeTokenizer.cs) -- test infrastructure only.

The library's native tokenizer (forge-lm_b200/csrc/tokenizer.hpp) is checked
against this file.  Training restates TrainDocuments (BpeTokenizer.cs:90-236)
as a recount-every-merge loop with the same selection rule (highest count,
ties to the lowest pair key (left << 32) | right, at least 2 occurrences,
no pair across a document boundary); encoding restates Encode
(BpeTokenizer.cs:259-318) with its per-rank position queues.
"""
from __future__ import annotations

import json
from collections import deque


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
    n = len(data)
    if n == 0:
        return []
    rank = {pair_key(l, r): k for k, (l, r, _) in enumerate(merges)}
    seq = list(data)
    nxt = [i + 1 if i + 1 < n else -1 for i in range(n)]
    prv = [i - 1 for i in range(n)]
    queues: list[deque | None] = [None] * len(merges)

    def push(r, i):
        if queues[r] is None:
            queues[r] = deque()
        queues[r].append(i)

    for i in range(n - 1):
        r = rank.get(pair_key(seq[i], seq[i + 1]))
        if r is not None:
            push(r, i)
    for r in range(len(merges)):
        q = queues[r]
        if q is None:
            continue
        new_id = merges[r][2]
        while q:
            i = q.popleft()
            j = nxt[i]
            if j < 0 or rank.get(pair_key(seq[i], seq[j])) != r:
                continue
            seq[i] = new_id
            nj = nxt[j]
            nxt[i] = nj
            nxt[j] = -1
            prv[j] = -1
            if nj >= 0:
                prv[nj] = i
                r2 = rank.get(pair_key(new_id, seq[nj]))
                if r2 is not None:
                    push(r2, i)
            p = prv[i]
            if p >= 0:
                r3 = rank.get(pair_key(seq[p], new_id))
                if r3 is not None:
                    push(r3, p)
    out, i = [], 0
    while i >= 0:
        out.append(seq[i])
        i = nxt[i]
    return out


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
