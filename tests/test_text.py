"""Byte-level BPE tokenizer, chat templates and the JSON DOM (C++).

Fixture and expectations follow crates/spark-text/tests/tokenizer.rs and
chat_template.rs of the reference."""
import json

import pytest

from sparkpipe_rs_b200.core import core, StatusError

A, B, C, AB, ABC, UNK, STOP, SPACE, X, Y, Z, XY, XYZ = range(13)


def fixture_json():
    return json.dumps({
        "model": {
            "type": "BPE", "unk_token": "<unk>", "byte_fallback": False,
            "vocab": {"a": A, "b": B, "c": C, "ab": AB, "abc": ABC, "<unk>": UNK, "<|stop|>": STOP,
                      "Ġ": SPACE, "x": X, "y": Y, "z": Z, "xy": XY, "xyz": XYZ},
            "merges": ["a b", "ab c", "x y", "xy z"],
        },
        "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False},
        "added_tokens": [{"id": STOP, "content": "<|stop|>", "special": True}],
    })


def tok():
    return core().Tokenizer.from_hf_json(fixture_json())


def test_encodes_byte_bpe_and_special_tokens():
    t = tok()
    assert t.encode("abc") == [ABC]
    assert t.encode("a<|stop|>bc") == [A, STOP, B, C]
    assert t.encode("a<|stop|>bc", allow_special=False)[0] == A
    assert t.encode("xyz abc") == [XYZ, SPACE, A, B, C] or t.encode("xyz abc")[0] == XYZ
    assert t.decode([ABC, STOP, XY]) == "abc<|stop|>xy"
    assert t.decode([ABC, STOP, XY], skip_special=True) == "abcxy"
    assert t.is_special(STOP) and not t.is_special(ABC)
    assert t.token_bytes(SPACE) == b" "


def test_unknown_bytes_map_to_unk():
    t = tok()
    assert t.encode("q") == [UNK]


def test_compiled_roundtrip_and_piece_cache():
    t = tok()
    t2 = core().Tokenizer.from_compiled(t.to_compiled())
    for s in ["abc", "xyzabc<|stop|>", "abab c"]:
        assert t2.encode(s) == t.encode(s)
    t.encode("abc abc abc")
    assert t.cache_hits > 0
    with pytest.raises(StatusError):
        core().Tokenizer.from_compiled(b"nope")


def test_piece_boundaries_gpt2_byte_classes():
    sp = core().Tokenizer.split_pieces
    text = b"Hello world's 123  x!?"
    pieces = [text[a:a + n] for a, n in sp(text)]
    assert pieces == [b"Hello", b" world", b"'s", b" 123", b"  ", b"x", b"!?"]
    t2 = b"we're ok"
    assert [t2[a:a + n] for a, n in sp(t2)] == [b"we", b"'re", b" ok"]


def test_batch_encode_matches_sequential():
    t = tok()
    texts = ["abc xyz", "xyzxyz", "a b c", "<|stop|>abc"] * 8
    assert t.encode_batch(texts, workers=4) == [t.encode(s) for s in texts]


def test_large_merge_table_and_fuzz_roundtrip():
    merges = ["a b"] + [f"unused_left_{i:06d} unused_right_{i:06d}" for i in range(1, 4000)]
    spec = {"model": {"type": "BPE", "unk_token": "<unk>", "vocab": {"a": 0, "b": 1, "ab": 2, "<unk>": 3},
                      "merges": merges}}
    t = core().Tokenizer.from_hf_json(json.dumps(spec))
    assert t.encode("ab") == [2]
    # a byte-complete vocabulary round-trips arbitrary bytes
    import random

    alphabet = [chr(c) for c in range(33, 127)]
    vocab = {ch: i for i, ch in enumerate(alphabet)}
    vocab["Ġ"] = len(vocab)
    full = core().Tokenizer.from_hf_json(json.dumps({"model": {"type": "BPE", "vocab": vocab, "merges": []}}))
    rng = random.Random(0)
    for _ in range(50):
        s = "".join(rng.choice(alphabet + [" "]) for _ in range(rng.randint(0, 40)))
        assert full.decode(full.encode(s)) == s


def test_glm_chat_template():
    C = core()
    out = C.render_chat([("system", "be brief"), ("user", "hi"), ("assistant", "yo"), ("tool", "42")], "glm",
                        C.CHAT_ADD_GENERATION_PROMPT | C.CHAT_ENABLE_THINKING, "high")
    assert out == ("[gMASK]<sop><|system|>Reasoning Effort: High<|system|>be brief<|user|>hi"
                   "<|assistant|><think></think>yo<|observation|><tool_response>42</tool_response>"
                   "<|assistant|><think>")
    assert C.render_chat([("user", "q")], "glm", 0, "", 64) == "[gMASK]<sop><|user|>q"
    with pytest.raises(StatusError):
        C.render_chat([("user", "q" * 100)], "glm", 0, "", 32)
    with pytest.raises(StatusError):
        C.render_chat([("user", "q")], "glm", 8, "", 64)
    ds = C.render_chat([("user", "hi")], "deepseek", C.CHAT_ADD_GENERATION_PROMPT, "", 1024)
    assert ds.startswith("<｜begin▁of▁sentence｜><｜User｜>hi") and ds.endswith("<｜Assistant｜>")


def test_json_dom_roundtrip():
    C = core()
    src = '{"a": [1, 2.5, "x\\u00e9\\ud83d\\ude00", true, null], "b": {"c": -3}}'
    assert json.loads(C.json_normalize(src)) == json.loads(src)
    for bad in ["{", "[1,]", '{"a" 1}', "tru"]:
        with pytest.raises(StatusError):
            C.json_normalize(bad)
