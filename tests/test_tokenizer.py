"""Native tokenizer / schema formatter (NativeTokenizer.swift:55-264) on CPU.

The checkpoint's tokenizer.json is not available, so the Unigram restatement is pinned to
the tokenizers library (the format's own implementation) on seeded synthetic
vocabularies with the DeBERTa-v3 normalizer / pre-tokenizer chain; the schema formatter is
checked for the reference's layout rules."""
from __future__ import annotations

import json

import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")

SPECIALS = ["[PAD]", "[CLS]", "[SEP]", "[UNK]", "[MASK]", "[P]", "[L]", "[SEP_STRUCT]", "[SEP_TEXT]",
            "[DESCRIPTION]", "[E]", "[C]", "[R]"]
ALPHA = "abcdefghijklmnopqrstuvwxyz0123456789().,:-'"


def _synthetic(seed=0, n_pieces=600, lowercase=False):
    """A Unigram tokenizer.json like DeBERTa-v3's: Strip, NFKC, collapse spaces; Metaspace."""
    from tokenizers import Regex, Tokenizer, models, normalizers, pre_tokenizers
    rng = np.random.default_rng(seed)
    pieces = {}
    for ch in ALPHA:
        pieces[ch] = None
        pieces["▁" + ch] = None
    pieces["▁"] = None
    while len(pieces) < n_pieces:
        k = int(rng.integers(2, 7))
        s = "".join(rng.choice(list(ALPHA[:26]), k))
        pieces[("▁" + s) if rng.random() < 0.5 else s] = None
    vocab = [(t, 0.0) for t in ["[PAD]", "[CLS]", "[SEP]", "[UNK]"]]
    scores = -np.sort(rng.uniform(2.0, 14.0, len(pieces)))[::-1]
    rng.shuffle(scores)
    vocab += [(p, float(s)) for p, s in zip(pieces, scores)]
    tok = Tokenizer(models.Unigram(vocab, unk_id=3, byte_fallback=False))
    norms = [normalizers.Strip(), normalizers.NFKC(), normalizers.Replace(Regex(" {2,}"), " ")]
    if lowercase:
        norms.insert(0, normalizers.Lowercase())
    tok.normalizer = normalizers.Sequence(norms)
    tok.pre_tokenizer = pre_tokenizers.Metaspace(replacement="▁", prepend_scheme="always")
    tok.add_special_tokens(SPECIALS)
    return tok


@pytest.fixture(scope="module")
def tok_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("tok")
    tok = _synthetic()
    tok.save(str(d / "tokenizer.json"))
    (d / "tokenizer_config.json").write_text(json.dumps({"tokenizer_class": "DebertaV2Tokenizer"}))
    return d, tok


def _random_text(rng, n):
    chars = ALPHA + "  éèüßﬁ½ΩЖ中!?"
    return "".join(rng.choice(list(chars), n))


def test_unigram_matches_tokenizers_library(tok_dir):
    from gliner_decide_metal_b200.tokenizer import UnigramTokenizer
    d, tok = tok_dir
    mine = UnigramTokenizer.from_file(d / "tokenizer.json")
    rng = np.random.default_rng(1)
    texts = ["the quick brown fox.", "  spaced   out  ", "ﬁne café", "", "x", "中文 mixed ½ text"]
    texts += [_random_text(rng, int(rng.integers(1, 40))) for _ in range(400)]
    for t in texts:
        enc = tok.encode(t, add_special_tokens=False)
        assert mine.encode(t) == enc.ids, (t, mine.tokenize(t), enc.tokens)
        assert mine.tokenize(t) == enc.tokens, t


@pytest.mark.parametrize("seed", [2, 3])
def test_unigram_matches_on_other_vocabularies(tmp_path, seed):
    from gliner_decide_metal_b200.tokenizer import UnigramTokenizer
    tok = _synthetic(seed=seed, n_pieces=300 + 200 * seed, lowercase=True)
    tok.save(str(tmp_path / "tokenizer.json"))
    mine = UnigramTokenizer.from_file(tmp_path / "tokenizer.json")
    rng = np.random.default_rng(seed)
    for _ in range(300):
        t = _random_text(rng, int(rng.integers(1, 30))).upper()
        assert mine.encode(t) == tok.encode(t, add_special_tokens=False).ids, t


def test_split_words_rules():
    from gliner_decide_metal_b200.tokenizer import split_words
    assert split_words("") == ["."]
    assert split_words("Hello World") == ["hello", "world", "."]
    assert split_words("Really?") == ["really", "?"]
    assert split_words("Mail a.b@c.io or @user, see https://x.y/z now!") == \
        ["mail", "a.b@c.io", "or", "@user", ",", "see", "https://x.y/z", "now", "!"]
    assert split_words("state-of-the-art snake_case 3.5") == ["state-of-the-art", "snake_case", "3", ".", "5", "."]


@pytest.mark.parametrize("text,words", [
    # combining marks are ICU word characters (\p{Mark}): decomposed accents stay in the word
    ("cafe\u0301 nai\u0308ve", ["cafe\u0301", "nai\u0308ve", "."]),
    # only decimal digits are ICU word characters: superscripts and fractions split off
    ("x\u00b2 \u00bd", ["x", "\u00b2", "\u00bd", "."]),
    # Other_Alphabetic symbols (circled letters) are word characters; lower-cased like Swift
    ("\u24b6\u24b7", ["\u24d0\u24d1", "."]),
    # ZWJ / ZWNJ and connector punctuation other than "_" join words
    ("co\u200dop a\u200cb x\u203fy", ["co\u200dop", "a\u200cb", "x\u203fy", "."]),
    # \v, U+001C-U+001F and U+0085 are not ICU white space: each is a token of its own
    ("a\x0bb\x1cc\x85d", ["a", "\x0b", "b", "\x1c", "c", "\x85", "d", "."]),
    # \p{Z} separators are white space (no-break space, ideographic space, line separator)
    ("a\u00a0b\u3000c\u2028d", ["a", "b", "c", "d", "."]),
    # case-insensitive ASCII classes: the Kelvin sign folds to k, long s to s
    # (the URL runs to the next white space, so it takes the appended sentence end too)
    ("\u212aelvin@x.io HTTP\u017f://A.b", ["kelvin@x.io", "http\u017f://a.b."]),
    # CJK and Hangul are alphabetic; full-width punctuation is not
    ("\u65e5\u672c\u8a9e\uff0c\ud55c\uad6d\uc5b4", ["\u65e5\u672c\u8a9e", "\uff0c", "\ud55c\uad6d\uc5b4", "."]),
])
def test_split_words_follows_icu_classes(text, words):
    """NSRegularExpression is ICU: \\w = [\\p{Alphabetic}\\p{Mark}\\p{Nd}\\p{Pc}\\u200c\\u200d] and
    \\s = [\\t\\n\\f\\r\\p{Z}] (ICU regular-expression documentation), which differ from
    Python re's classes on each case here (NativeTokenizer.swift:67-71,198-212)."""
    from gliner_decide_metal_b200.tokenizer import split_words
    assert split_words(text) == words


def test_schema_layout(tok_dir):
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200.tokenizer import NativeDecisionTokenizer, schema_entries
    d, tok = tok_dir
    nt = NativeDecisionTokenizer(d)
    tasks = [g.DecisionTask("sentiment", ("positive", "negative", "neutral")),
             g.DecisionTask("topic", ("sports", "politics"), True, prompt="what is it about",
                            label_descriptions={"sports": "games and teams"})]
    ents = [e.text for e in schema_entries("Great game last night", tasks)]
    assert ents[:4] == ["(", "[P]", "sentiment", "("]
    assert ents[4:10] == ["[L]", "positive", "[L]", "negative", "[L]", "neutral"]
    assert ents[10:13] == [")", ")", "[SEP_STRUCT]"]
    assert ents[15] == "topic: what is it about [DESCRIPTION] sports: games and teams"
    assert ents[-6:] == ["[SEP_TEXT]", "great", "game", "last", "night", "."]
    ids, markers = nt.encode_schema("Great game last night", tasks)
    L_id = tok.token_to_id("[L]")
    assert [len(m) for m in markers] == [3, 2]
    assert all(ids[p] == L_id for m in markers for p in m)
    assert ids.count(L_id) == 5 and ids[1] == tok.token_to_id("[P]")
    assert ids.count(tok.token_to_id("[SEP_STRUCT]")) == 1 and ids.count(tok.token_to_id("[SEP_TEXT]")) == 1
    # the entries between special tokens are tokenised on their own
    assert ids[2:2 + len(tok.encode("sentiment", add_special_tokens=False).ids)] == \
        tok.encode("sentiment", add_special_tokens=False).ids
    inp = nt.make_input("Great game last night", tasks)
    B, L, hm, o = inp.shape
    assert (B, hm, o) == (1, 2, 3)
    assert L == min(b for b in g.DEFAULT_BUCKETS if b >= len(ids))  # smallest bucket that holds the ids
    assert list(inp.input_ids[0, :len(ids)]) == ids
    assert (inp.input_ids[0, len(ids):] == tok.token_to_id("[PAD]")).all()
    assert inp.attention_mask[0].astype(np.float32).sum() == len(ids)
    assert list(inp.marker_indices[0, 0]) == markers[0] and list(inp.marker_indices[0, 1, :2]) == markers[1]
    assert list(inp.marker_mask[0, 1]) == [1.0, 1.0, 0.0]


def test_special_tokens_inside_text_and_errors(tok_dir):
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200.tokenizer import NativeDecisionTokenizer, TokenizerFilesError
    d, tok = tok_dir
    nt = NativeDecisionTokenizer(d)
    # earliest match first, the longer one on a tie ([SEP_TEXT] vs [SEP])
    got = nt.token_ids("ab[SEP_TEXT]cd[SEP]")
    want = (tok.encode("ab", add_special_tokens=False).ids + [tok.token_to_id("[SEP_TEXT]")] +
            tok.encode("cd", add_special_tokens=False).ids + [tok.token_to_id("[SEP]")])
    assert got == want
    with pytest.raises(g.NoTaskLabelsError):
        nt.make_input("text", [])
    with pytest.raises(g.NoTaskLabelsError):
        nt.make_input("text", [g.DecisionTask("t", ())])
    with pytest.raises(g.InputDoesNotFitError):
        nt.make_input("word " * 200, [g.DecisionTask("t", ("a", "b"))], buckets=[32, 64])
    with pytest.raises(TokenizerFilesError):
        NativeDecisionTokenizer(d / "missing")


def test_raw_jsonl_parsing_and_layout(tok_dir, tmp_path):
    """RawExample lines (RawCLI.swift:11-15) through the tokenizer into rows of one group."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import serve
    from gliner_decide_metal_b200.tokenizer import NativeDecisionTokenizer
    d, _ = tok_dir
    lines = [{"id": "a", "text": "Loved it", "tasks": [{"name": "sentiment", "labels": ["pos", "neg"]}]},
             {"id": "b", "text": "Terrible service!", "tasks": [
                 {"name": "sentiment", "labels": ["pos", "neg"], "multiLabel": True, "prompt": "tone",
                  "labelDescriptions": {"pos": "good"}}]}]
    p = tmp_path / "raw.jsonl"
    p.write_text("\n".join(json.dumps(x) for x in lines) + "\n")
    ex = serve.load_raw_jsonl(p)
    assert [e.id for e in ex] == ["a", "b"]
    assert ex[1].tasks[0] == g.DecisionTask("sentiment", ("pos", "neg"), True, "tone", {"pos": "good"})
    nt = NativeDecisionTokenizer(d)
    rows = [nt.make_input(e.text, e.tasks) for e in ex]
    assert all(r.shape[2:] == (1, 2) for r in rows)


def _spm_tokenizer(tmp_path, seed=0):
    """A DeBERTa-v3-style tokenizer.json from a SentencePiece unigram model with the nmt_nfkc
    normalization rule, trained here: the model's pieces and scores, its precompiled
    character map as a Precompiled normalizer (Strip, Precompiled, collapse spaces as the
    DeBERTa-v2 conversion writes), Metaspace pre-tokenizer."""
    spm = pytest.importorskip("sentencepiece")
    from sentencepiece import sentencepiece_model_pb2 as pb
    from tokenizers import Regex, Tokenizer, models, normalizers, pre_tokenizers
    rng = np.random.default_rng(seed)
    syll = ["ka", "to", "ri", "mu", "sen", "ver", "al", "on", "de", "ba", "qu", "ix", "ph", "str", "ing", "ed",
            "ly", "tion", "ﬁ", "é", "ü", "ß", "Ω", "½", "①", "ｶ", "中", "文", "é", "Å", "™", "…"]
    lines = [" ".join("".join(rng.choice(syll, int(rng.integers(1, 4)))) for _ in range(int(rng.integers(5, 20))))
             for _ in range(3000)]
    corpus = tmp_path / "corpus.txt"
    corpus.write_text("\n".join(lines), encoding="utf-8")
    spm.SentencePieceTrainer.train(input=str(corpus), model_prefix=str(tmp_path / "m"), vocab_size=400,
                                   model_type="unigram", normalization_rule_name="nmt_nfkc", pad_id=0, unk_id=1,
                                   bos_id=2, eos_id=3, pad_piece="[PAD]", unk_piece="[UNK]", bos_piece="[CLS]",
                                   eos_piece="[SEP]", num_threads=1, minloglevel=2)
    m = pb.ModelProto()
    m.ParseFromString((tmp_path / "m.model").read_bytes())
    tok = Tokenizer(models.Unigram([(p.piece, p.score) for p in m.pieces], unk_id=1, byte_fallback=False))
    tok.normalizer = normalizers.Sequence([normalizers.Strip(),
                                           normalizers.Precompiled(m.normalizer_spec.precompiled_charsmap),
                                           normalizers.Replace(Regex(" {2,}"), " ")])
    tok.pre_tokenizer = pre_tokenizers.Metaspace(replacement="▁", prepend_scheme="always")
    tok.add_special_tokens(SPECIALS[4:])
    return tok


def test_precompiled_nmt_nfkc_matches_tokenizers_library(tmp_path):
    """The Precompiled (SentencePiece nmt_nfkc) normalizer and the whole Unigram pipeline
    against the tokenizers library, on text with ligatures, full-width and circled forms,
    combining marks, emoji and other non-ASCII."""
    from gliner_decide_metal_b200.tokenizer import UnigramTokenizer
    tok = _spm_tokenizer(tmp_path)
    tok.save(str(tmp_path / "tokenizer.json"))
    mine = UnigramTokenizer.from_file(tmp_path / "tokenizer.json")
    rng = np.random.default_rng(7)
    alphabet = list("abcdefghijklmnopqrstuvwxyzABC  .,") + ["ﬁ", "ﬂ", "é", "é", "Å", "Å", "ü", "ß", "Ω", "Ω",
                                                           "½", "①", "⑳", "ｶ", "ﾀ", "ｱ", "ｄ", "中", "文", "™", "…",
                                                           "　", " ", "👍", "👍🏽", "🇩🇪", "​", "ℌ"]
    texts = ["ﬁne Café ①② ｶﾀｶﾅ  double  space", "été Ångström", "👍🏽 ok 🇩🇪", "½ ™ …"]
    texts += ["".join(rng.choice(alphabet, int(rng.integers(1, 30)))) for _ in range(400)]
    for t in texts:
        assert mine.normalize(t) == tok.normalizer.normalize_str(t), t
        enc = tok.encode(t, add_special_tokens=False)
        assert mine.encode(t) == enc.ids, (t, mine.tokenize(t), enc.tokens)


def test_raw_stream_pipeline_matches_shape_grouping(tok_dir):
    """Raw-text rows through the pipelined stream path (tokenising the next chunk while the
    current one is classified) give the same predictions as RawCLI's shape grouping."""
    import gliner_decide_metal_b200 as g
    from gliner_decide_metal_b200 import serve
    from gliner_decide_metal_b200.tokenizer import NativeDecisionTokenizer
    from test_serve import _FakeModel
    d, _ = tok_dir
    nt = NativeDecisionTokenizer(d)
    rng = np.random.default_rng(2)
    words = ["good", "bad", "match", "team", "vote", "price", "rain", "sun"]
    ex = []
    for i in range(37):
        tasks = [g.DecisionTask("s", ("pos", "neg", "neu")), g.DecisionTask("t", ("a", "b", "c", "d", "e"), True)]
        ex.append(serve.RawExample(f"r{i}", " ".join(rng.choice(words, int(rng.integers(1, 60)))), tasks[: 1 + i % 2]))
    a = serve.run_raw_examples(_FakeModel(), nt, ex, batch_size=8, group_by="shape")
    m = _FakeModel()
    b = serve.run_raw_examples(m, nt, ex, batch_size=8, group_by="stream")
    assert [x.id for x in b] == [e.id for e in ex]
    assert len(m.batches) == 5 and len({(hm, o) for _, _, hm, o in m.batches}) == 1
    for x, y in zip(a, b):
        assert [(p.task, p.labels, p.probabilities) for p in x.predictions] == \
            [(p.task, p.labels, p.probabilities) for p in y.predictions]


@pytest.mark.parametrize("variant", ["lower_punct", "prepend_never", "whitespace", "nfd"])
def test_pipeline_variants_match_tokenizers_library(tmp_path, variant):
    """Other normalizer / pre-tokenizer chains a tokenizer.json may carry (Lowercase,
    Punctuation, WhitespaceSplit, NFD, Metaspace prepend schemes) against the library."""
    from tokenizers import Regex, normalizers, pre_tokenizers
    from gliner_decide_metal_b200.tokenizer import UnigramTokenizer
    tok = _synthetic(seed=5, n_pieces=500)
    if variant == "lower_punct":
        tok.normalizer = normalizers.Sequence([normalizers.Lowercase(), normalizers.Strip()])
        tok.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.Punctuation(behavior="isolated"),
                                                     pre_tokenizers.Metaspace(replacement="▁", prepend_scheme="always")])
    elif variant == "prepend_never":
        tok.pre_tokenizer = pre_tokenizers.Metaspace(replacement="▁", prepend_scheme="never")
    elif variant == "whitespace":
        tok.normalizer = normalizers.Replace(Regex("[0-9]"), "")
        tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    elif variant == "nfd":
        tok.normalizer = normalizers.NFD()
    tok.save(str(tmp_path / "tokenizer.json"))
    mine = UnigramTokenizer.from_file(tmp_path / "tokenizer.json")
    rng = np.random.default_rng(11)
    texts = ["Hello, World!", "x", "a.b,c", "  spaced   out  ", "Café über"]
    texts += [_random_text(rng, int(rng.integers(1, 30))) for _ in range(200)]
    for t in texts:
        assert mine.encode(t) == tok.encode(t, add_special_tokens=False).ids, (variant, t)
