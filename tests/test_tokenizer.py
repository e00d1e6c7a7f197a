"""The library's byte-level BPE tokenizer against the oracle restatement
(oracle/tokenizer.py) of src/LLM.Core/Tokenizer/BpeTokenizer.cs, following
the reference's tokenizer tests (tests/LLM.Core.Tests/BpeTokenizerTests.cs:
round trips, unseen and unicode text, untrained identity, EncodeDocument,
save/load, rejected files) on this file's own seeded corpora."""
import json

import numpy as np
import pytest

from oracle import tokenizer as OT


def corpus(seed: int, n_words: int) -> bytes:
    """Seeded English-ish text: words over a small alphabet, punctuation and
    newlines, with a few accented and emoji words."""
    rng = np.random.default_rng(seed)
    syll = ["th", "e", "an", "qu", "ick", "o", "re", "st", "ing", "al", "ou", "er", "s", "t", "ly", "ça", "ñ", "🌧"]
    words = []
    for k in range(n_words):
        w = "".join(syll[i] for i in rng.integers(0, len(syll), rng.integers(1, 4)))
        words.append(w + (", " if k % 7 == 3 else ".\n" if k % 11 == 10 else " "))
    return "".join(words).encode("utf-8")


@pytest.fixture(scope="module")
def trained(pkg, tmp_path_factory):
    c = corpus(11, 1500)
    merges = OT.train_documents([c], 200)
    path = tmp_path_factory.mktemp("tok") / "tok.json"
    OT.save(path, merges)
    return pkg.BpeTokenizer(path), merges, c


SAMPLES = ["a sentence the trainer never saw, with digits 0123456789",
           "accents: façade, niño, crème brûlée — and 🌧 🌍",
           "tabs\tand\nnewlines\r\nmixed", "", "x", "🦊🐕🌍", "the the the the the"]


def test_encode_matches_oracle_and_round_trips(trained):
    tok, merges, c = trained
    assert tok.vocab_size == 256 + len(merges) + 1 and tok.eos_token_id == 256 + len(merges)
    for s in SAMPLES + [c.decode("utf-8")]:
        ids = tok.encode(s)
        assert ids == OT.encode(s.encode("utf-8"), merges), s[:30]
        assert tok.decode(ids) == s
    rep = "the quick string, the quick string. " * 20
    ids = tok.encode(rep)
    assert len(ids) < len(rep.encode("utf-8"))  # merges compress repetitive text


def test_untrained_is_identity_over_bytes(pkg, tmp_path):
    p = tmp_path / "empty.json"
    OT.save(p, [])
    tok = pkg.BpeTokenizer(p)
    assert tok.vocab_size == 257 and tok.eos_token_id == 256
    data = np.random.default_rng(7).integers(0, 256, 1000, dtype=np.uint8).tobytes()
    assert tok.encode(data) == list(data)
    s = "untrained héllo 🌍"
    assert tok.decode(tok.encode(s)) == s


def test_encode_document_appends_eos(trained):
    tok, _, _ = trained
    doc = "One complete document.\n"
    plain, framed = tok.encode(doc), tok.encode_document(doc)
    assert framed[:-1] == plain and framed[-1] == tok.eos_token_id
    assert tok.decode(framed) == doc  # EOS decodes to no text


def test_stream_decoder_holds_partial_utf8(trained):
    tok, _, _ = trained
    s = "🌍 x"
    ids = tok.encode(s)
    byte_ids = [b for b in s.encode("utf-8")]  # one id per byte: splits the emoji
    dec = tok.stream_decoder()
    out = "".join(dec.decode_token(i) for i in byte_ids) + dec.flush()
    assert out == s and tok.decode(ids) == s


def test_decode_rejects_unknown_ids(pkg, trained):
    tok, _, _ = trained
    with pytest.raises(pkg.ArgumentError):
        tok.decode([tok.vocab_size])
    with pytest.raises(pkg.ArgumentError):
        tok.decode([-1])


@pytest.mark.parametrize("case", ["version", "short_merge", "unknown_ids", "wrong_new_id", "wrong_eos", "garbage"])
def test_load_rejections(pkg, tmp_path, case):
    """BpeTokenizer.Load (BpeTokenizer.cs:353-389) throws InvalidDataException."""
    good = {"Version": 2, "Merges": [[97, 98, 256], [256, 99, 257]], "EosTokenId": 258}
    bad = json.loads(json.dumps(good))
    if case == "version":
        bad["Version"] = 1
    elif case == "short_merge":
        bad["Merges"][1] = [256, 99]
    elif case == "unknown_ids":
        bad["Merges"][1] = [300, 99, 257]
    elif case == "wrong_new_id":
        bad["Merges"][1] = [256, 99, 260]
    elif case == "wrong_eos":
        bad["EosTokenId"] = 300
    p = tmp_path / "bad.json"
    p.write_text("{not json" if case == "garbage" else json.dumps(bad))
    with pytest.raises(pkg.InvalidDataError):
        pkg.BpeTokenizer(p)
    q = tmp_path / "good.json"
    q.write_text(json.dumps(good, indent=2))
    assert pkg.BpeTokenizer(q).encode("abc") == [257]


def test_training_oracle_properties():
    """The restated trainer: the dominant pair first, no merge across document
    boundaries (BpeTokenizer.cs:100-112), vocabulary grows with merges."""
    ab = b"ab" * 100
    assert OT.train_documents([ab], 1) == [(97, 98, 256)]
    assert len(OT.train_documents([ab], 5)) == 5
    assert OT.train_documents([b"a", b"b", b"a", b"b"], 10) == []


def test_encode_random_tables_against_definition(pkg, tmp_path):
    """Random merge tables (each merge joins earlier ids, as Load requires)
    over a three-letter alphabet, so runs like "aaaa" overlap and merges nest:
    the library's encoder against the rank-greedy definition."""
    rng = np.random.default_rng(23)
    for t in range(6):
        merges, pairs = [], set()
        ids = [97, 98, 99]
        while len(merges) < 40:
            a, b = int(rng.choice(ids)), int(rng.choice(ids))
            if (a, b) in pairs:
                continue
            pairs.add((a, b))
            merges.append((a, b, 256 + len(merges)))
            ids.append(256 + len(merges) - 1)
        path = tmp_path / f"rand{t}.json"
        OT.save(path, merges)
        tok = pkg.BpeTokenizer(path)
        for n in (1, 2, 3, 7, 64, 1000):
            data = bytes(rng.choice([97, 98, 99], n).tolist())
            assert tok.encode(data) == OT.encode(data, merges), (t, n)
            assert tok.decode_bytes(tok.encode(data)) == data
        assert tok.encode(b"a" * 257) == OT.encode(b"a" * 257, merges)
