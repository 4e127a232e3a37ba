"""The prompt layer on CPU: the text tokenizer's pre-split, byte-pair merges, validation and
specials (protocol.mm:428-592, tokenization_yue2.py:8-31), and the prompt layout and
request validation (protocol.py:73-148). tiktoken and the real ``qwen.tiktoken`` are not on
this machine, so the expected values below are derived by hand from the published rules
(the pattern's alternatives in order; merge the lowest-ranked adjacent pair, leftmost on
ties) on a synthetic vocabulary of the reference's size."""
import base64
import os

import pytest

from tests.conftest import ROOT, _load


@pytest.fixture(scope="module")
def proto():
    return _load("yue2_mlx_b200_protocol", os.path.join(ROOT, "yue2-mlx_b200", "protocol.py"))


MERGES = [b"ll", b"he", b"hell", b"aa", b"aaa", b"Th", b"The", b" w", b" wo", b" wor", b" worl", b" world"]


def _vocab_file(path, merges=MERGES, count=151643, extra=()):
    """Every byte at rank = its value, then `merges` in order, then filler tokens (4-byte
    strings starting 0xFF, which UTF-8 text never contains) up to `count`."""
    toks = [bytes([b]) for b in range(256)] + list(merges)
    i = 0
    while len(toks) < count:
        toks.append(b"\xff" + i.to_bytes(3, "big"))
        i += 1
    lines = [base64.b64encode(t) + b" " + str(r).encode() for r, t in enumerate(toks[:count])]
    lines += list(extra)
    with open(path, "wb") as f:
        f.write(b"\n".join(lines) + b"\n")
    return path


@pytest.fixture(scope="module")
def tok(proto, tmp_path_factory):
    return proto.TextTokenizer(_vocab_file(str(tmp_path_factory.mktemp("tok") / "qwen.tiktoken")))


def test_pre_tokenizer_pieces(tok):
    text = "Hello world's 123!\n\nOK  it's\tdone \n"
    pieces = [m.group() for m in tok._split.finditer(text)]
    # " " before a digit: no alternative with a letter or punctuation fits, and "\s+(?!\S)"
    # fails before "1", so the last one takes it alone; digits one by one; "!" takes the
    # newlines after it; the tab is the letter run's optional leading non-letter.
    assert pieces == ["Hello", " world", "'s", " ", "1", "2", "3", "!\n\n", "OK", " ", " it", "'s", "\tdone",
                      " \n"]
    assert "".join(pieces) == text


def test_merges_take_the_lowest_rank_first(tok):
    r = tok.ranks
    # h e l l o: "ll" (256) before "he" (257), then "hell" (258); "hello" is no token.
    assert tok.encode("hello") == [r[b"hell"], ord("o")]
    # a a a a: three "aa" pairs of equal rank, the leftmost first; then "aa"+"aa" is no
    # token, and "aaa" (260) never forms although it is one: (aa, a) lost to (a, a).
    assert tok.encode("aaaa") == [r[b"aa"], r[b"aa"]]
    # A piece that is itself a token is one id; " world" is also reached by merges.
    assert tok.encode("The world") == [r[b"The"], r[b" world"]]
    # Bytes outside the merges stay single bytes (UTF-8 of e-acute: 0xC3 0xA9).
    assert tok.encode("\u00e9") == [0xC3, 0xA9]


def test_nfc_normalization_and_round_trip(tok):
    assert tok.encode("e\u0301") == tok.encode("\u00e9") == [0xC3, 0xA9]  # decomposed -> composed
    text = "The world, hello! 42 \u00e9t\u00e9\n"
    assert tok.decode(tok.encode(text)) == text


def test_specials_follow_the_ordinary_tokens(proto, tok):
    assert tok.n_vocab == proto.EOD + 208
    assert tok.decode([proto.EOD]) == "<|endoftext|>"
    assert tok.decode([proto.ABC_START, proto.ABC_END]) == "<abc></abc>"
    assert tok.decode([proto.EOD + 8]) == "<extra_0>" and tok.decode([proto.EOD + 207]) == "<extra_199>"
    assert tok.decode([-1, proto.EOD + 208, ord("x")]) == "x"  # out of range: skipped
    assert tok.encode("<|endoftext|>")[0] == ord("<")  # special text is ordinary text


@pytest.mark.parametrize("mutate,needle", [
    (lambda p: _vocab_file(p, count=1000), "151643 ordinary tokens"),
    (lambda p: _vocab_file(p, extra=[base64.b64encode(b"zz") + b" 151643"]), "Invalid"),
    (lambda p: _vocab_file(p, extra=[b"!!notbase64!! 5"]), "base64"),
    (lambda p: _vocab_file(p, extra=[base64.b64encode(b"zz") + b" 5 7"]), "Invalid"),
    (lambda p: _vocab_file(p, extra=[base64.b64encode(b"zz") + b" 5"]), "151643 ordinary tokens"),  # rank reused
])
def test_vocabulary_validation(proto, tmp_path, mutate, needle):
    path = mutate(str(tmp_path / "qwen.tiktoken"))
    with pytest.raises(ValueError, match=needle):
        proto.TextTokenizer(path)


def test_missing_byte_token_is_an_error(proto, tmp_path):
    # Rank 0 holds a 2-byte token instead of the byte 0x00, so b"\x00" cannot be encoded.
    path = str(tmp_path / "qwen.tiktoken")
    toks = [b"\x00\x01"] + [bytes([b]) for b in range(1, 256)]
    i = 0
    while len(toks) < 151643:
        toks.append(b"\xff" + i.to_bytes(3, "big"))
        i += 1
    with open(path, "wb") as f:
        f.write(b"\n".join(base64.b64encode(t) + b" " + str(r).encode() for r, t in enumerate(toks)) + b"\n")
    with pytest.raises(ValueError, match="missing a byte token"):
        proto.TextTokenizer(path).encode("a\x00")


def test_prompt_layout(proto, tok):
    P = proto
    full = P.SongRequest(style="pop", lyrics="la la", cot="full")
    text = tok.encode(full.text())
    assert full.text() == P.INSTRUCTIONS["full"] + "\n[Tags]\npop\n[Lyrics]\nla la\n"
    assert P.token_prefixes(full, tok) == [P.EOD] + text + [P.ABC_START]
    assert P.token_prefixes(full, tok, abc_ids=[5, 6]) == [P.EOD] + text + [P.ABC_START, 5, 6, P.ABC_END,
                                                                           P.MUSIC_START]
    ext = P.SongRequest(style="pop", lyrics="la la", cot="melody", abc="X:1")
    assert P.token_prefixes(ext, tok) == ([P.EOD] + tok.encode(ext.text()) + [P.ABC_START] + tok.encode("X:1")
                                          + [P.ABC_END, P.MUSIC_START])
    off = P.SongRequest(style="pop", lyrics="la la", cot="off")
    assert P.token_prefixes(off, tok)[-3:] == [P.ABC_START, P.ABC_END, P.MUSIC_START]
    assert P.negative_prefix(off, tok) == [P.EOD] + tok.encode(P.INSTRUCTIONS["off"]) + [P.MUSIC_START]
    assert P.negative_prefix(full, tok, abc_ids=[7]) == ([P.EOD] + tok.encode(P.INSTRUCTIONS["full"])
                                                         + [P.ABC_START, 7, P.ABC_END, P.MUSIC_START])
    assert off.guidance == 1.01 and full.guidance == 1.0
    assert P.SongRequest(style="a", lyrics="b", cfg_scale=1.5).guidance == 1.5
    with pytest.raises(ValueError, match="positive-branch"):
        P.negative_prefix(full, tok)
    with pytest.raises(ValueError, match="ordinary text vocabulary"):
        P.token_prefixes(full, tok, abc_ids=[P.EOD])


@pytest.mark.parametrize("kw,needle", [
    (dict(cot="maybe"), "cot must be"),
    (dict(seed=-1), "seed"),
    (dict(id="../x"), "filename-safe"),
    (dict(cot="off", abc="X:1"), "External ABC"),
    (dict(abc="   "), "External ABC"),
    (dict(cfg_scale=21.0), "cfg_scale"),
    (dict(cfg_scale=float("nan")), "cfg_scale"),
])
def test_request_validation(proto, kw, needle):
    with pytest.raises(ValueError, match=needle):
        proto.SongRequest(style="s", lyrics="l", **kw)


def test_chunk_ranges(proto):
    assert proto.chunk_ranges(10, 100, context=130) == [(0, 10)]
    assert proto.chunk_ranges(30, 100, context=123) == [(0, 10), (10, 20), (20, 30)]
    with pytest.raises(ValueError, match="no acoustic context"):
        proto.chunk_ranges(5, 127, context=130)
