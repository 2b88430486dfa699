"""The Linux tokenizer (include/plamo_tokenizer.h), host only.

Pinned by the reference's own tokenizer tests (tests/{utf8,string,score,json,
vocab,vocab_load,trie,unigram,encode,boundary,preprocess,decode,tokenizer}.c),
compiled unchanged where they lie and linked against the product library.
Then known answers worked out by hand on a synthetic vocabulary: the
Unigram choice (global cost, longer piece on ties), special-token and
repeated-run segment boundaries, UTF-8 byte fallback, decoding and the
translation prompt.
"""
import ctypes
import os
import subprocess

import pytest

from conftest import REF, load_package

REFERENCE_TESTS = ["utf8", "string", "score", "json", "vocab", "vocab_load", "trie", "unigram", "encode",
                   "boundary", "preprocess", "decode", "tokenizer"]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "tests")),
                    reason="reference checkout not mounted on this machine")
@pytest.mark.parametrize("name", REFERENCE_TESTS)
def test_reference_tokenizer_tests_pass_against_library(tmp_path, name):
    pkg = load_package()
    libdir = os.path.dirname(pkg.LIB_PATH)
    exe = tmp_path / f"test-{name}"
    subprocess.run(["gcc", "-O2", "-w", os.path.join(REF, "tests", f"{name}.c"), "-L", libdir, "-lplamo_cuda",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, r.stdout + r.stderr
    # vocab_load needs the official vocabulary file, absent here
    assert "PASS" in r.stdout or (name == "vocab_load" and "SKIP" in r.stdout), r.stdout


# Synthetic vocabulary: row 0 unused, rows 1..256 the byte pieces, then these
# pieces (score = log-probability), then filler up to 107520 rows.
PIECES = [("日本", "-1.0"), ("日", "-2.0"), ("本語", "-1.5"), ("語", "-3.0"), ("<|plamo:bos|>", "0.0", "CONTROL"),
          ("a", "-1.0"), ("aa", "-2.0"), ("ba", "-0.5"), ("b", "-1.0")]
ID = {p[0]: 257 + i for i, p in enumerate(PIECES)}


def byte_id(b):
    return 1 + b


@pytest.fixture(scope="module")
def tokenizer(tmp_path_factory):
    pkg = load_package()
    lib = pkg.load()
    path = tmp_path_factory.mktemp("vocab") / "tokenizer.jsonl"
    rows = ['["unused", 0, "NORMAL"]']
    rows += [f'["<0x{b:02X}>", 0, "BYTE"]' for b in range(256)]
    for p in PIECES:
        rows.append(f'["{p[0]}", {p[1]}, "{p[2] if len(p) > 2 else "NORMAL"}"]')
    rows += ['["x", -1, "NORMAL"]'] * (107520 - len(rows))
    path.write_text("\n".join(rows) + "\n", encoding="utf-8")
    err = ctypes.create_string_buffer(256)
    t = lib.plamo_tokenizer_open(str(path).encode(), err, 256)
    assert t, err.value
    yield lib, t
    lib.plamo_tokenizer_close(t)


def encode(tok, text, direction=0):
    lib, t = tok
    ids = ctypes.POINTER(ctypes.c_uint32)()
    err = ctypes.create_string_buffer(256)
    n = lib.plamo_tokenizer_encode(t, text.encode() if isinstance(text, str) else text, direction,
                                   ctypes.byref(ids), err, 256)
    if n == 2**64 - 1:
        return None, err.value.decode()
    return [ids[i] for i in range(n)], None


def test_global_cost_beats_greedy_prefix(tokenizer):
    # 日本+語 costs 1.0 + 3.0; 日+本語 costs 2.0 + 1.5
    assert encode(tokenizer, "日本語")[0] == [ID["日"], ID["本語"]]


def test_equal_cost_prefers_the_longer_piece(tokenizer):
    # a+a and aa both cost 2.0
    assert encode(tokenizer, "aa")[0] == [ID["aa"]]


def test_special_tokens_are_their_own_segments(tokenizer):
    assert encode(tokenizer, "a<|plamo:bos|>a")[0] == [ID["a"], ID["<|plamo:bos|>"], ID["a"]]


def test_runs_of_four_are_their_own_segment(tokenizer):
    # Without the boundary, ba + aa + a (0.5 + 2.0 + 1.0) would beat b + aa + aa (1.0 + 4.0).
    assert encode(tokenizer, "baaaa")[0] == [ID["b"], ID["aa"], ID["aa"]]
    assert encode(tokenizer, "baaa")[0] == [ID["ba"], ID["aa"]]


def test_uncovered_scalars_fall_back_to_utf8_bytes(tokenizer):
    want = [ID["語"]] + [byte_id(b) for b in "😀".encode()]
    assert encode(tokenizer, "語😀")[0] == want


def test_decode_round_trips_the_text(tokenizer):
    lib, t = tokenizer
    text = "b日本語aa😀 <|plamo:bos|>"
    ids, _ = encode(tokenizer, text)
    out = b""
    for i in ids:
        p = ctypes.c_char_p()
        n = lib.plamo_tokenizer_decode(t, i, ctypes.byref(p))
        assert n != 2**64 - 1
        out += ctypes.string_at(p, n)
    assert out.decode() == text
    assert lib.plamo_tokenizer_decode(t, 107520, ctypes.byref(ctypes.c_char_p())) == 2**64 - 1


def test_translation_directions_wrap_the_prompt_template(tokenizer):
    lib, t = tokenizer
    buf = ctypes.create_string_buffer(4096)
    for direction, src, dst in ((1, b"en", b"ja"), (2, b"ja", b"en")):
        n = lib.plamo_translation_prompt("日本語".encode(), src, dst, buf, 4096)
        assert n != 2**64 - 1
        assert encode(tokenizer, "日本語", direction)[0] == encode(tokenizer, buf.value)[0]
    ids = ctypes.POINTER(ctypes.c_uint32)()
    err = ctypes.create_string_buffer(256)
    for direction, src in ((0, b"en"), (1, b"ja")):
        n = lib.plamo_tokenizer_prefix(t, direction, ctypes.byref(ids), err, 256)
        assert lib.plamo_translation_prefix(src, buf, 4096) != 2**64 - 1
        assert [ids[i] for i in range(n)] == encode(tokenizer, buf.value)[0]
    assert lib.plamo_tokenizer_prefix(t, 2, ctypes.byref(ids), err, 256) == 2**64 - 1


def test_invalid_requests_fail_with_a_reason(tokenizer):
    assert encode(tokenizer, "a", 3)[1] == "tokenizer: translation direction must be 0, 1 or 2"
    assert "UTF-8" in encode(tokenizer, b"\xff")[1]
    assert "4096" in encode(tokenizer, "a" * 4097)[1]
    assert encode(tokenizer, "")[0] == []


def test_python_tokenizer_class(tokenizer, tmp_path):
    pkg = load_package()
    lib, t = tokenizer
    # the module fixture's vocabulary, reopened through the package class
    rows = ['["unused", 0, "NORMAL"]'] + [f'["<0x{b:02X}>", 0, "BYTE"]' for b in range(256)]
    rows += [f'["{p[0]}", {p[1]}, "{p[2] if len(p) > 2 else "NORMAL"}"]' for p in PIECES]
    rows += ['["x", -1, "NORMAL"]'] * (107520 - len(rows))
    path = tmp_path / "v.jsonl"
    path.write_text("\n".join(rows) + "\n", encoding="utf-8")
    with pkg.Tokenizer(path) as tok:
        ids = tok.encode("日本語😀")
        assert ids.tolist() == encode(tokenizer, "日本語😀")[0]
        assert tok.decode(ids).decode() == "日本語😀"
        assert tok.encode("日本語", 1).tolist() == encode(tokenizer, "日本語", 1)[0]
        assert tok.prefix(0).size > 0
        with pytest.raises(ValueError, match="direction"):
            tok.encode("a", 3)
        with pytest.raises(ValueError):
            tok.decode([107520])
    with pytest.raises(ValueError, match="missing"):
        pkg.Tokenizer(tmp_path / "absent.jsonl")
