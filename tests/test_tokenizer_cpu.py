"""WordPiece tokenizer (host): bbh_tokenize against transformers' BertTokenizer on the same
vocab.txt -- the tokenizer the reference's scripts use (scripts/dump_corpus.py:34-38,
BERT uncased, truncation to max_length, [CLS] ... [SEP]). The vocabulary is generated here
from the test corpus (the MiniLM vocab is not in this container); texts mix English,
punctuation, accented Latin, combining marks, Greek, Cyrillic, CJK, Hangul, emoji,
full-width forms, control and zero-width characters, odd whitespace and over-long words."""
import unicodedata as ud

import numpy as np
import pytest

WORDS = ("the cat sat on mat running jumped quickly unaffable hello world model embedding sentence "
         "naïve café résumé Über straße İstanbul ÆSIR øre Ελληνικά καλημέρα Москва привет ёлка "
         "日本語 中文 한국어 안녕하세요 ｆｕｌｌｗｉｄｔｈ １２３ émoji 🙂 x² ½ ﬁne Ǆemal étude").split()
PUNCT = list(".,;:!?\"'()[]{}-—–…«»¿¡@#$%^&*_+=<>/\\|~`") + ["。", "、", "！", "？", "·"]
SPACES = [" ", "  ", "\t", "\n", " ", "　", " ", "\r\n"]
NOISE = ["\u0007", "​", "﻿", "­", "�", "\u0000"[:0]]


def make_texts(seed, n):
    rng = np.random.default_rng(seed)
    out = ["", " ", "A", "hello, world!", "unaffable", "x" * 150, "ab" * 60 + " end"]
    for _ in range(n):
        parts = []
        for _ in range(int(rng.integers(1, 40))):
            r = rng.random()
            if r < 0.6:
                w = WORDS[int(rng.integers(len(WORDS)))]
                if rng.random() < 0.3:
                    w = w.upper() if rng.random() < 0.5 else w.capitalize()
                parts.append(w)
            elif r < 0.8:
                parts.append(PUNCT[int(rng.integers(len(PUNCT)))])
            elif r < 0.9:
                parts.append(NOISE[int(rng.integers(len(NOISE)))])
            else:
                parts.append(str(int(rng.integers(0, 10 ** 6))))
            parts.append(SPACES[int(rng.integers(len(SPACES)))] if rng.random() < 0.8 else "")
        out.append("".join(parts))
    return out


def norm(s):
    return "".join(c for c in ud.normalize("NFD", s.lower()) if ud.category(c) != "Mn")


def write_vocab(path, texts, lowercase):
    toks = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]
    seen = set(toks)
    chars = sorted({c for t in texts for c in (norm(t) if lowercase else t) if not c.isspace()})
    chars = [c for i, c in enumerate(chars) if i % 10 != 3]  # some characters stay unknown -> [UNK]
    words = sorted({(norm(w) if lowercase else w) for w in WORDS})
    for tok in chars + ["##" + c for c in chars] + words + ["##ing", "##ed", "##s", "un", "##aff", "##able", "run"]:
        if tok not in seen:
            seen.add(tok)
            toks.append(tok)
    with open(path, "w", encoding="utf-8") as f:
        f.write("\n".join(toks) + "\n")


@pytest.mark.parametrize("lowercase", [True, False])
@pytest.mark.parametrize("max_len", [128, 16])
def test_matches_bert_tokenizer(tmp_path, lowercase, max_len):
    import bbh
    from transformers import BertTokenizer

    texts = make_texts(7, 400)
    vocab = str(tmp_path / "vocab.txt")
    write_vocab(vocab, make_texts(7, 400)[:300], lowercase)  # some characters stay unknown
    ref = BertTokenizer(vocab, do_lower_case=lowercase)(texts, truncation=True, max_length=max_len)["input_ids"]
    v = bbh.Vocab(vocab, lowercase)
    ids, cu = v.tokenize(texts, max_len)
    got = [ids[cu[i]:cu[i + 1]].tolist() for i in range(len(texts))]
    bad = [i for i in range(len(texts)) if got[i] != ref[i]]
    assert not bad, f"{len(bad)} texts differ, first {texts[bad[0]]!r}: {got[bad[0]]} vs {ref[bad[0]]}"


def test_capacity_and_errors(tmp_path):
    import bbh

    vocab = str(tmp_path / "vocab.txt")
    write_vocab(vocab, ["hello world"], True)
    v = bbh.Vocab(vocab)
    ids, cu = v.tokenize(["hello world"] * 3 + [""], 8)
    assert cu.tolist() == [0, 4, 8, 12, 14] and ids[:4].tolist() == [2, ids[1], ids[2], 3]
    bad = tmp_path / "bad.txt"
    bad.write_text("hello\nworld\n")
    with pytest.raises(bbh.BBHError) as e:
        bbh.Vocab(str(bad))
    assert e.value.code == -4
